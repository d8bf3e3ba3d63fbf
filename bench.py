#!/usr/bin/env python3
"""Decode throughput of the LLaMA-3-8B-shape Q4_K continuous-batching step.

Workload: 32 layers, d_model 4096, 32 query / 8 KV heads,
head_dim 128, SwiGLU FFN 14336, vocab 128256, RoPE theta 5e5; Q4_K linear
weights from N(0, 0.02), f32 embedding and LM head; 256 active sequences per
GPU with ragged contexts.  A step = one continuous-batching decode step of all
256 sequences through the engine's C ABI (slate_llama_batch_step_device, one
CUDA graph); `value` = tokens/s over all ranks with inputs already in HBM,
`e2e` = the same through slate_llama_batch_step with host buffers.

Contexts: prompt U[128, 4096] plus a uniform offset of U[0, 256) already-decoded
tokens (the steady state of 256-token budgets under continuous refill), seeded
on the device as synthetic K/V.  The timed window is shorter than a budget, so
no sequence finishes inside it.  The KV cache is f32 by default, the
reference's own dtype (llama_infer.c:225-226); the same measurement with an f16
cache is reported as the labelled extra `variant_kv_f16`.  The KV read per step
(~150 GB f32, ~75 GB f16) exceeds the 126 MB L2, so no flush is needed between
steps.

Multi-GPU: sequences are independent, so each rank is a replica running its own
256 sequences (weak scaling, no collective on the data path); torch.distributed
(nccl) only provides the barrier and the max-over-ranks timing.

--impl reference: the reference's own CPU path (oracle/_ref, the unmodified
slate sources) on this host's cores: one slate_llama_decode_step session per
thread, each holding a seeded history of the benchmark's own context
distribution; a step = every session decodes one greedy token.  The process
maps only oracle/ libraries (the workload file is written by the CPU-only
writer in oracle/build).
"""
from __future__ import annotations

import argparse
import json
import os
import select
import shutil
import statistics
import subprocess
import sys
import threading
import time

import numpy as np

ROOT = os.path.dirname(os.path.abspath(__file__))
sys.path.insert(0, ROOT)

CFG3 = dict(n_layers=32, d_model=4096, ffn_hidden=14336, n_heads=32, n_kv_heads=8, vocab=128256,
            max_seq=4352, theta_base=500000.0, rms_eps=1e-5)
METRIC = "decode tok/s (box), LLaMA-3-8B-shape Q4_K, 256 ragged seqs; p50 step latency"
# 70B shape, tensor parallel; prompts U[256, 2048] + 256 tokens
CFG5 = dict(n_layers=80, d_model=8192, ffn_hidden=28672, n_heads=64, n_kv_heads=8, vocab=128256,
            max_seq=2368, theta_base=500000.0, rms_eps=1e-5)
METRIC70 = "decode tok/s (box), LLaMA-3-70B-shape Q4_K tensor-parallel, 512 ragged seqs per TP group"
# ~1B, 64 requests, prompts lognormal (median 256, clipped to
# 2048), 128 greedy tokens, Poisson arrivals at 20 req/s.  BASELINE.json gives no
# sigma for the lognormal; 0.75 is used (mean prompt ~339 tokens) and recorded.
CFG2 = dict(n_layers=16, d_model=2048, ffn_hidden=8192, n_heads=32, n_kv_heads=8, vocab=32000,
            max_seq=2304, theta_base=10000.0, rms_eps=1e-5)
METRIC1B = "decode tok/s (box), ~1B-shape Q4_K, 64 ragged seqs; p50 step latency"
# Mistral-7B shape, 32 sequences, prompts U[8192, 32768],
# 128 greedy tokens, f16 KV cache in 16-token pages
CFG4 = dict(n_layers=32, d_model=4096, ffn_hidden=14336, n_heads=32, n_kv_heads=8, vocab=32000,
            max_seq=32896, theta_base=1000000.0, rms_eps=1e-5)
METRIC_MISTRAL = "decode tok/s (box), Mistral-7B-shape Q4_K long context, 32 ragged seqs; p50 step latency"
MODELS = {"8b": dict(cfg=CFG3, metric=METRIC, batch=256, prompt=(128, 4096), budget=256, period=0,
                     kv="f32", file_gb=9,
                     workload="llama3-8b-shape q4k continuous-batching decode (BASELINE config 3)"),
          "1b": dict(cfg=CFG2, metric=METRIC1B, batch=64, prompt=("lognormal", 256, 0.75, 2048),
                     budget=128, period=0, kv="f32", file_gb=2,
                     workload="~1b-shape q4k continuous-batching decode (BASELINE config 2)"),
          "mistral": dict(cfg=CFG4, metric=METRIC_MISTRAL, batch=32, prompt=(8192, 32768), budget=128,
                          period=0, kv="f16", file_gb=6,
                          workload="mistral-7b-shape q4k long-context decode (BASELINE config 4)"),
          "70b": dict(cfg=CFG5, metric=METRIC70, batch=512, prompt=(256, 2048), budget=256, period=8,
                      kv="f32", file_gb=60,
                      workload="llama3-70b-shape q4k tensor-parallel decode (BASELINE config 5)")}
# DRAM bytes (read + write) per algorithmic byte of one attention launch, from ncu
# captures of 32 rows at the 8B shape with 1024-token chunks (dram__bytes_read.sum +
# dram__bytes_write.sum over K/V + q + output bytes).  f16 KV (attn_chunk_mma):
# 300.39 MB read + 5.20 MB written for 300.74 MB.  Traffic scales with the K/V
# tokens read, so a full launch's traffic is the ratio times its algorithmic bytes.
# f32 KV (attn_chunk, 256 rows, contexts capped at 1024, mean 956): 2040.80 MB read
# + 11.49 MB written for 2019.67 MB.
ATTN_TRAFFIC_RATIO = {"f16": 1.0161, "f32": 1.0161}


def parse():
    ap = argparse.ArgumentParser()
    ap.add_argument("--gpus", type=int, default=1)
    ap.add_argument("--steps", type=int, default=20)
    ap.add_argument("--warmup", type=int, default=3)
    ap.add_argument("--impl", default="ours", choices=["ours", "reference"])
    ap.add_argument("--kv", default=None, choices=["f16", "f32"],
                    help="KV cache dtype of the headline (default: f32, the reference's; f16 for "
                         "the Mistral config, which mandates it, and for 70b below 4-way TP)")
    ap.add_argument("--variant-kv", default="auto", choices=["auto", "none", "f16", "f32"],
                    help="also time the other KV dtype and report it as variant_kv_<dtype> "
                         "(auto: f16 when the headline is f32)")
    ap.add_argument("--model", default="8b", choices=list(MODELS),
                    help="8b: the headline (config 3, replicas); 70b: config 5 with --tp")
    ap.add_argument("--tp", type=int, default=1,
                    help="tensor-parallel ranks per model replica (70b: 2, 4 or 8)")
    ap.add_argument("--batch", type=int, default=0, help="sequences per replica (0: the config's)")
    ap.add_argument("--seed", type=int, default=1234)
    ap.add_argument("--layers", type=int, default=0,
                    help="reduce only for debugging; 0 = the config's (32 for 8b, 80 for 70b)")
    ap.add_argument("--prefill-tokens", type=int, default=4000,
                    help="after the decode timing, time one prompt of this many tokens (0: skip)")
    ap.add_argument("--lanes", type=int, default=1, choices=[1, 2],
                    help="2: the batch's halves as two lanes on two streams (see slate_cuda_opts_t)")
    ap.add_argument("--gemm-path", type=int, default=0,
                    help="0 auto (tcgen05 3-pass hi/lo split; stream-K kernel from 128 rows), 1 CUDA "
                         "cores, 2 tcgen05 single f16 pass, 3 3-pass tile-per-CTA kernel only, 4 "
                         "exact-weight stream-K kernel, 5 3-pass stream-K kernel from 16 rows, 6 "
                         "exact-weight kernel with x rounded once to f16")
    ap.add_argument("--attn-path", type=int, default=0,
                    help="0: tensor-core attention for f16 KV (mma.sync), 1: CUDA-core kernel")
    ap.add_argument("--max-ctx", type=int, default=0,
                    help="cap every context (profiling captures of the GEMMs on a small device "
                         "footprint; 0 = the config's distribution)")
    ap.add_argument("--e2e-steps", type=int, default=-1,
                    help="host-API steps for the e2e figure (default: --steps)")
    ap.add_argument("--no-cpu-baseline", action="store_true")
    ap.add_argument("--cpu-steps", type=int, default=4,
                    help="decode steps of the reference sessions for cpu_baseline (after 1 warm-up)")
    ap.add_argument("--cpu-threads", type=int, default=0, help="reference sessions (0: all cores)")
    ap.add_argument("--refill-steps", type=int, default=-1,
                    help="steps of the continuous-refill replay after the decode timing (finished "
                         "sequences replaced by prefilled new requests; default --steps, 0: skip)")
    ap.add_argument("--trace", default="auto", choices=["auto", "none", "poisson"],
                    help="poisson: replay BASELINE config 2's Poisson arrivals (20 req/s) through the "
                         "host API after the decode timing (auto: for --model 1b)")
    return ap.parse_args()


def model_path(args, cfg) -> str:
    tag = f"slate_b200_{args.model}_L{cfg['n_layers']}_s{args.seed}.gguf"
    need = MODELS[args.model]["file_gb"] << 30
    for d in (os.environ.get("SLATE_BENCH_DIR"), "/dev/shm", "/tmp"):
        if d and os.path.isdir(d) and shutil.disk_usage(d).free > need:
            return os.path.join(d, tag)
    return os.path.join("/tmp", tag)


def ensure_model(args, cfg, barrier, writer) -> str:
    """The benchmark's GGUF, written once per host by `writer` (the product's
    slate_b200.synth_gguf, or oracle.synth_gguf -- the same bytes -- in the
    reference arm, which must not map the product library)."""
    path = model_path(args, cfg)
    if int(os.environ.get("LOCAL_RANK", "0")) == 0 and not os.path.exists(path):
        tmp = path + f".{os.getpid()}.tmp"
        # the 70B file repeats a period of 8 distinct random layers (written in
        # about a minute instead of ten); the engine still holds every layer
        writer(tmp, q4k=True, seed=args.seed, layer_period=MODELS[args.model]["period"], **cfg)
        os.rename(tmp, path)
    barrier()
    return path


def tp_group_id(dist, world, tp, rank, make_id):
    """The NCCL id of this rank's tensor-parallel group (ranks [g*tp, g*tp+tp)):
    made by the group's first rank, shared with an all-gather over all ranks."""
    mine = make_id() if rank % tp == 0 else None
    ids = [None] * world
    dist.all_gather_object(ids, mine)
    return ids[(rank // tp) * tp]


def prompt_lengths(spec, rng, n):
    """Prompt lengths of the config: U[lo, hi], or a clipped lognormal."""
    pr = spec["prompt"]
    if pr[0] == "lognormal":
        _, median, sigma, clip = pr
        return np.clip(np.round(rng.lognormal(np.log(median), sigma, n)), 1, clip).astype(np.int64)
    return rng.integers(pr[0], pr[1] + 1, n)


def contexts(args, cfg, n, replica, steps, with_done=False):
    """Prompt lengths of the config plus U[0, budget) already-decoded tokens per
    sequence (the steady state of fixed budgets under continuous refill)."""
    spec = MODELS[args.model]
    rng = np.random.default_rng(args.seed * 1000 + replica)
    prompt = prompt_lengths(spec, rng, n)
    done = rng.integers(0, spec["budget"], n)
    cap = cfg["max_seq"] - steps - 1
    if args.max_ctx:
        cap = min(cap, args.max_ctx)
    ctx = np.minimum(prompt + done, cap).astype(np.int64)
    return (ctx, done) if with_done else ctx


class ClockSampler:
    """nvidia-smi clocks / throttle reasons sampled during the timed region."""
    Q = ("index,clocks.sm,clocks.max.sm,power.draw,clocks_event_reasons.active,"
         "clocks_event_reasons.hw_slowdown,clocks_event_reasons.hw_thermal_slowdown,"
         "clocks_event_reasons.sw_thermal_slowdown,clocks_event_reasons.sw_power_cap")

    def __init__(self, gpus):
        self.gpus = set(gpus)
        self.p = None
        self.out = ""

    def __enter__(self):
        if shutil.which("nvidia-smi"):
            self.p = subprocess.Popen(["nvidia-smi", f"--query-gpu={self.Q}", "--format=csv,noheader,nounits",
                                       "-lms", "100"], stdout=subprocess.PIPE, stderr=subprocess.DEVNULL,
                                      text=True)
            # nvidia-smi takes a moment to start: wait (at most 5 s) for its first
            # sample, taken before the timed region and left out of the summary,
            # so that a short timed region is still sampled from its start
            if select.select([self.p.stdout], [], [], 5.0)[0]:
                self.p.stdout.readline()
        return self

    def __exit__(self, *a):
        if self.p:
            self.p.terminate()
            try:
                self.out, _ = self.p.communicate(timeout=5)
            except subprocess.TimeoutExpired:
                self.p.kill()

    def summary(self):
        sm, mx, pw, reasons = [], [], [], set()
        names = ["hw_slowdown", "hw_thermal_slowdown", "sw_thermal_slowdown", "sw_power_cap"]
        for line in self.out.splitlines():
            f = [x.strip() for x in line.split(",")]
            if len(f) < 9 or not f[0].isdigit() or int(f[0]) not in self.gpus:
                continue
            try:
                sm.append(float(f[1]))
                mx.append(float(f[2]))
            except ValueError:
                continue
            try:
                pw.append(float(f[3]))
            except ValueError:
                pass
            for n, v in zip(names, f[5:9]):
                if v.lower() == "active":
                    reasons.add(n)
        if not sm:
            return None
        return {"sm_mhz": statistics.median(sm), "sm_max_mhz": max(mx), "reasons": sorted(reasons),
                "power_w": statistics.median(pw) if pw else None, "samples": len(sm)}


def kv_dtype_name(args) -> str:
    """The headline KV dtype: --kv, else the config's: f32 (the reference's),
    f16 for the Mistral config (BASELINE config 4 mandates it; its f32 cache
    would need ~172 GB) and for the 70B shape below 4-way tensor parallelism
    (~214 GB of f32 cache per GPU at 2-way)."""
    if args.kv:
        return args.kv
    if args.model == "70b" and args.tp < 4:
        return "f16"
    return MODELS[args.model]["kv"]


# ---------------------------------------------------------------------------
# reference CPU path (oracle/_ref: the reference's own sources)
# ---------------------------------------------------------------------------
def reference_cpu(path, ctx, seeds, warmup, steps, threads=0):
    """Greedy decode through the reference's slate_llama_decode_step
    (src/loader/llama_infer.c:274-279), one session per host thread.

    The reference's LLaMA path is single-threaded and unbatched
    (util/quant.c:306-313, backend/backend_cpu.c:33-36), so one session per
    core is its best host throughput.  Session i holds a seeded history of
    ctx[i] tokens (slate_ref_session_seed_context: the values the CUDA engine
    seeds for the same seed) and decodes warmup + steps tokens, each fed its
    previous greedy token; a step ends when every session has its token.  The
    session count is capped by host memory (each session callocs a dense f32
    KV cache of 2 * layers * max_seq * kv_dim floats, llama_infer.c:225-226)."""
    import oracle as O
    ref = O.Reference()
    g, m = ref.open(path)
    c = ref.config(m)
    V = c["vocab"]
    sess_bytes = 2 * c["n_layers"] * c["max_seq"] * c["n_kv_heads"] * c["head_dim"] * 4
    n = threads or os.cpu_count() or 1
    try:
        avail = os.sysconf("SC_AVPHYS_PAGES") * os.sysconf("SC_PAGE_SIZE")
        n = max(1, min(n, int(0.6 * avail // sess_bytes)))
    except (ValueError, OSError):
        pass
    n = min(n, len(ctx))
    sess = [None] * n
    out = [np.zeros(V, np.float32) for _ in range(n)]
    tok = [int(t) for t in np.random.default_rng(int(seeds[0])).integers(0, V, n)]
    rcs = [0] * n
    t_seed = time.time()

    def make(i):
        sess[i] = ref.session(m, int(ctx[i]), int(seeds[i]))

    th = [threading.Thread(target=make, args=(i,)) for i in range(n)]
    for t in th:
        t.start()
    for t in th:
        t.join()
    t_seed = time.time() - t_seed
    gate = threading.Barrier(n + 1)
    stop = []

    def worker(i):
        while True:
            gate.wait()
            if stop:
                return
            rcs[i] = ref.decode(sess[i], tok[i], out[i])
            tok[i] = int(np.argmax(out[i]))
            gate.wait()

    th = [threading.Thread(target=worker, args=(i,)) for i in range(n)]
    for t in th:
        t.start()
    step_s = []
    for k in range(warmup + steps):
        t0 = time.perf_counter()
        gate.wait()
        gate.wait()
        if k >= warmup:
            step_s.append(time.perf_counter() - t0)
        if any(rcs):
            break
    stop.append(True)
    gate.wait()
    for t in th:
        t.join()
    for s in sess:
        ref.lib.slate_llama_session_free(s)
    ref.close(g, m)
    if any(rcs) or len(step_s) < steps:
        raise RuntimeError(f"reference decode failed: rc {sorted(set(rcs))}")
    tot = sum(step_s)
    used = np.asarray(ctx[:n], np.float64)
    return {"value": n * steps / tot, "unit": "tok/s", "cores": n, "kind": "reference",
            "ms_per_step": 1000.0 * tot / steps, "p50_step_ms": 1000.0 * float(np.median(step_s)),
            "steps": steps, "warmup": warmup, "sessions": n, "mean_ctx": float(used.mean()),
            "sample": (f"{n} reference sessions in parallel (one per host thread, the unbatched "
                       f"slate_llama_decode_step), histories of {int(used.min())}-{int(used.max())} "
                       f"tokens (mean {used.mean():.0f}) seeded from the benchmark's context "
                       f"distribution, {warmup} warm-up + {steps} timed greedy tokens each"),
            "seed_s": round(t_seed, 1)}


# ---------------------------------------------------------------------------
# one measurement of the CUDA engine
# ---------------------------------------------------------------------------
def measure(args, cfg, path, kv_name, env, full=True):
    """Warm-up + timed decode steps of one engine with a KV cache of `kv_name`;
    with `full`, also the e2e figure, per-kernel times and the prompt prefill."""
    import torch
    import slate_b200 as sb
    dist, barrier, world, local, tp, tp_rank, replica, tp_id = (
        env[k] for k in ("dist", "barrier", "world", "local", "tp", "tp_rank", "replica", "tp_id"))
    kv = sb.KV_F16 if kv_name == "f16" else sb.KV_F32
    esz = 2 if kv == sb.KV_F16 else 4
    n = args.batch
    total_steps = args.warmup + args.steps
    e2e_steps = (args.e2e_steps if args.e2e_steps >= 0 else args.steps) if full else 0
    ctx, done = contexts(args, cfg, n, replica, 3 * total_steps + 4, with_done=True)
    D, L, V = cfg["d_model"], cfg["n_layers"], cfg["vocab"]
    hd = D // cfg["n_heads"]
    nq, nkv, F = cfg["n_heads"] // tp, cfg["n_kv_heads"] // tp, cfg["ffn_hidden"] // tp
    # pool: every sequence's pages through the last step, the two prefill prompts
    pf = args.prefill_tokens if full and 0 < args.prefill_tokens < cfg["max_seq"] else 0
    refill = args.refill_steps if full and tp == 1 and args.trace != "poisson" else 0
    trace = full and tp == 1 and args.trace == "poisson"
    pages = int(sum((int(c) + total_steps + e2e_steps + 2) // 16 + 1 for c in ctx)) + 2 * (pf // 16 + 2) + 64
    if refill:
        # admitted prompts reuse released sequences' pages; this covers the
        # difference between their lengths (about 3 sigma over ~20 admissions)
        pages += 1024
    if trace:
        pages = max(pages, int(MODELS[args.model]["batch"]) * (cfg["max_seq"] // 16 + 1))
    # prompts run in chunks of max_batch rows: engines that prefill get a box of
    # at least 256 rows (the decode graph of n rows is the same whatever the box)
    box = max(n, 256) if (pf or refill or trace) else n
    eng = sb.LlamaBatch(path, device=local, max_batch=box, max_slots=n, kv_dtype=kv,
                        max_seq=cfg["max_seq"], kv_pages=pages, gemm_path=args.gemm_path,
                        attn_path=args.attn_path, tp_size=tp, tp_rank=tp_rank, tp_id=tp_id,
                        lanes=args.lanes)
    slots = np.array([eng.open() for _ in range(n)], np.int32)
    assert (slots >= 0).all(), sb.last_error()
    for s, c in zip(slots, ctx):
        rc = eng.seed_context(int(s), int(c), args.seed + int(s))
        assert rc == 0, (rc, sb.last_error())
    stream = torch.cuda.ExternalStream(eng.stream(), device=torch.device("cuda", local))
    d_slots = torch.tensor(slots, device="cuda")
    rng = np.random.default_rng(args.seed + replica)     # one token stream per TP group
    d_tok = [torch.tensor(rng.integers(0, V, n).astype(np.int32), device="cuda"),
             torch.zeros(n, dtype=torch.int32, device="cuda")]

    def dstep(i):
        rc = eng.step_device(d_slots.data_ptr(), n, d_tok[i & 1].data_ptr(), d_tok[(i + 1) & 1].data_ptr())
        assert rc == 0, sb.last_error()

    for i in range(args.warmup):
        dstep(i)
    assert eng.sync() == 0, "device rejected a warm-up step"
    torch.cuda.synchronize()
    barrier()
    ev = [torch.cuda.Event(enable_timing=True) for _ in range(args.steps + 1)]
    with ClockSampler([local] if world == 1 else range(world)) as clk:
        torch.cuda.synchronize()
        barrier()
        with torch.cuda.stream(stream):
            ev[0].record(stream)
            for i in range(args.steps):
                dstep(args.warmup + i)
                ev[i + 1].record(stream)
        torch.cuda.synchronize()
        barrier()
    assert eng.sync() == 0, "device rejected a timed step"
    step_ms = [ev[i].elapsed_time(ev[i + 1]) for i in range(args.steps)]
    tot_ms = ev[0].elapsed_time(ev[-1])
    if dist:
        t = torch.tensor([tot_ms], device="cuda")
        dist.all_reduce(t, op=dist.ReduceOp.MAX)
        tot_ms = float(t.item())
    replicas = world // tp
    res = {"kv": kv_name, "value": n * replicas * args.steps / (tot_ms / 1000.0), "tot_ms": tot_ms,
           "step_ms": step_ms, "ctx": ctx, "replicas": replicas, "clocks": clk.summary(),
           "launches": eng.launches_per_step(n) * args.steps}

    # end to end through the host-buffer API: H2D slots+tokens, D2H greedy tokens;
    # right after the timed region, so that both run in the same power state
    if e2e_steps:
        host_tok = d_tok[args.steps & 1 ^ (args.warmup & 1)].cpu().numpy()
        torch.cuda.synchronize()
        barrier()
        t0 = time.perf_counter()
        for _ in range(e2e_steps):
            rc, host_tok, _ = eng.step(slots, host_tok)
            assert rc == 0, sb.last_error()
        e2e_s = time.perf_counter() - t0
        if dist:
            t = torch.tensor([e2e_s], device="cuda", dtype=torch.float64)
            dist.all_reduce(t, op=dist.ReduceOp.MAX)
            e2e_s = float(t.item())
        res["e2e"] = {"value": n * replicas * e2e_steps / e2e_s, "unit": "tok/s",
                      "h2d_bytes_per_step": n * 8, "d2h_bytes_per_step": n * 4}

    # per-kernel timing of the dominant kernels on the same state and stream
    layer = cfg["n_layers"] // 2
    groups = [("attention", sb.PROF_ATTENTION)]
    if full:
        groups += [("qkv", sb.PROF_QKV), ("wo", sb.PROF_WO), ("gate_up", sb.PROF_GATE_UP),
                   ("down", sb.PROF_DOWN), ("lm_head", sb.PROF_LM_HEAD)]
        if tp > 1:                       # two per layer, after Wo and after down
            groups += [("allreduce", sb.PROF_ALLREDUCE)]
    kt = {name: eng.profile(k, n, layer, iters=10) for name, k in groups}
    res["kernel_ms"] = kt
    ctx_now = ctx + total_steps + e2e_steps            # contexts seen by the profiled launch
    res["attn_bytes"] = float(ctx_now.sum()) * 2 * nkv * hd * esz + n * nq * hd * 4 * 3
    q4k = 144 / 256
    w_layer = (D * (nq + 2 * nkv) * hd + nq * hd * D + 3 * D * F) * q4k
    head = V // tp * D * 4
    kv_read_step = float((ctx + total_steps - args.steps // 2).sum()) * 2 * nkv * hd * esz * L
    res["step_bytes"] = w_layer * L + head + kv_read_step + n * 2 * nkv * hd * esz * L

    # prompt prefill through slate_llama_batch_prefill (chunks of max_batch
    # prompt rows with the causal prefill attention): one sequence's slot is
    # released and a fresh prompt of --prefill-tokens tokens admitted into it
    res["prefill"] = None
    if pf and n >= 2:
        for s in slots[:2]:
            assert eng.release(int(s)) == 0, sb.last_error()
        warm, ps = eng.open(), eng.open()
        prng = np.random.default_rng(args.seed)
        prompts = [prng.integers(0, V, pf).astype(np.int32) for _ in range(2)]
        rc, _ = eng.prefill(warm, prompts[0], want_logits=False)   # captures the chunk graphs
        assert rc == 0, sb.last_error()
        torch.cuda.synchronize()
        t0 = time.perf_counter()
        rc, _ = eng.prefill(ps, prompts[1], want_logits=False)
        pf_s = time.perf_counter() - t0
        assert rc == 0, sb.last_error()
        res["prefill"] = {"tokens": pf, "ms": pf_s * 1e3, "tok_s": pf / pf_s, "rows_per_step": box,
                          "note": "one prompt into a released slot through the host API (wall "
                                  "clock, chunk graphs already captured by a first prompt)"}
        slots[0], slots[1] = warm, ps
        done[0] = done[1] = 0
    res["refill"] = None
    if refill:
        # remaining budgets of a steady state: the seeded decoded counts advanced
        # by the steps run so far, wrapped at the budget (a sequence past its
        # budget stands for its successor), so admissions arrive at the steady
        # rate of rows / budget per step rather than in one burst
        budget = MODELS[args.model]["budget"]
        left = budget - (done + total_steps + e2e_steps) % budget
        res["refill"] = refill_trace(eng, args, MODELS[args.model], slots, left, V, args.seed)
    res["trace"] = None
    if trace:
        for s in slots:
            assert eng.release(int(s)) == 0, sb.last_error()
        res["trace"] = poisson_trace(eng, args, MODELS[args.model], V, args.seed)
    eng.close()
    return res


def refill_trace(eng, args, spec, slots, left, V, seed):
    """Continuous refill ("a continuous refill so that 256
    sequences stay active") through the host API.  Every sequence has a budget
    of spec['budget'] output tokens (`left` of them remain); a finished one is
    released and a new request admitted into a fresh slot: its prompt, drawn
    from the config's prompt distribution, runs through
    slate_llama_batch_prefill and its first output token is the prompt's greedy
    token.  Each step then decodes every row with slate_llama_batch_step.
    Served tok/s = output tokens (decode rows plus first tokens) / wall time,
    prefill included."""
    import slate_b200 as sb
    rng = np.random.default_rng(seed + 77)
    n = len(slots)
    slots, left = slots.copy(), left.copy()
    toks = rng.integers(0, V, n).astype(np.int32)
    out_tok = prompt_tok = admitted = 0
    pf_s, step_s, stopped = 0.0, [], None
    t0 = time.perf_counter()
    for _ in range(args.refill_steps):
        for r in np.nonzero(left <= 0)[0]:
            assert eng.release(int(slots[r])) == 0, sb.last_error()
            s_new = eng.open()
            assert s_new >= 0, sb.last_error()
            prompt = rng.integers(0, V, int(prompt_lengths(spec, rng, 1)[0])).astype(np.int32)
            tp = time.perf_counter()
            rc, lg = eng.prefill(s_new, prompt, want_logits=True)
            pf_s += time.perf_counter() - tp
            if rc == -2:
                stopped = "KV pool full"
                break
            assert rc == 0, sb.last_error()
            slots[r], toks[r], left[r] = s_new, int(np.argmax(lg)), spec["budget"] - 1
            out_tok += 1
            prompt_tok += len(prompt)
            admitted += 1
        if stopped:
            break
        ts = time.perf_counter()
        rc, toks, _ = eng.step(slots, toks)
        assert rc == 0, sb.last_error()
        step_s.append(time.perf_counter() - ts)
        out_tok += n
        left -= 1
    wall = time.perf_counter() - t0
    return {"value": out_tok / wall, "unit": "tok/s", "steps": len(step_s), "admitted": admitted,
            "prompt_tokens": prompt_tok, "prefill_s": round(pf_s, 3), "wall_s": round(wall, 3),
            "decode_step_p50_ms": 1e3 * float(np.median(step_s)) if step_s else None,
            "stopped": stopped,
            "note": "continuous refill through the host API (slate_llama_batch_step + "
                    "slate_llama_batch_prefill for each admitted prompt), wall clock, prefill "
                    "included; output tokens = decode rows + each prompt's first token"}


def poisson_trace(eng, args, spec, V, seed, n_req=64, rate=20.0, max_tokens=128):
    """BASELINE config 2's request trace through the host API: n_req requests
    with Poisson arrivals at `rate` per second, prompts from the config's
    distribution (seeded tokens), max_tokens greedy tokens each.  A request is
    admitted (slate_llama_batch_prefill; its first token is the prompt's greedy
    token) once it has arrived and a row is free, then decodes in the batch
    steps until done.  Reports served tok/s over the makespan (first arrival to
    last completion), time to first token and time per output token."""
    import slate_b200 as sb
    rng = np.random.default_rng(seed + 99)
    arrivals = np.cumsum(rng.exponential(1.0 / rate, n_req))
    arrivals -= arrivals[0]
    plens = prompt_lengths(spec, rng, n_req)
    prompts = [rng.integers(0, V, int(x)).astype(np.int32) for x in plens]
    w = eng.open()                              # warm-up: chunk graphs for prompts
    assert w >= 0, sb.last_error()
    rc, _ = eng.prefill(w, prompts[0][: min(len(prompts[0]), 64)], want_logits=False)
    assert rc == 0 and eng.release(w) == 0, sb.last_error()
    pending, active = list(range(n_req)), {}
    ttft, t_first, t_done, step_s = {}, {}, {}, []
    t0 = time.perf_counter()
    while pending or active:
        while pending and arrivals[pending[0]] <= time.perf_counter() - t0 and len(active) < eng.max_batch:
            r = pending.pop(0)
            s = eng.open()
            assert s >= 0, sb.last_error()
            rc, lg = eng.prefill(s, prompts[r], want_logits=True)
            assert rc == 0, sb.last_error()
            now = time.perf_counter() - t0
            active[s] = [r, int(np.argmax(lg)), 1]
            ttft[r], t_first[r] = now - arrivals[r], now
        if not active:
            time.sleep(max(0.0, arrivals[pending[0]] - (time.perf_counter() - t0)))
            continue
        sl = list(active)
        ts = time.perf_counter()
        rc, out, _ = eng.step(sl, [active[s][1] for s in sl])
        assert rc == 0, sb.last_error()
        step_s.append(time.perf_counter() - ts)
        now = time.perf_counter() - t0
        for i, s in enumerate(sl):
            a = active[s]
            a[1], a[2] = int(out[i]), a[2] + 1
            if a[2] >= max_tokens:
                assert eng.release(s) == 0, sb.last_error()
                t_done[a[0]] = now
                del active[s]
    makespan = max(t_done.values())
    tpot = [(t_done[r] - t_first[r]) / (max_tokens - 1) for r in range(n_req)]
    return {"value": n_req * max_tokens / makespan, "unit": "tok/s", "requests": n_req,
            "rate_req_s": rate, "max_tokens": max_tokens, "makespan_s": round(makespan, 3),
            "ttft_p50_ms": 1e3 * float(np.median(list(ttft.values()))),
            "ttft_p95_ms": 1e3 * float(np.percentile(list(ttft.values()), 95)),
            "tpot_p50_ms": 1e3 * float(np.median(tpot)),
            "decode_step_p50_ms": 1e3 * float(np.median(step_s)), "steps": len(step_s),
            "prompt_mean": float(plens.mean()),
            "note": "Poisson arrivals replayed on the wall clock through the host API "
                    "(slate_llama_batch_prefill per admitted prompt, slate_llama_batch_step for "
                    "the running batch); served tok/s = all output tokens / makespan"}


def attn_kernel_name(kv_name, args):
    return ("attn_chunk_mma+attn_combine" if kv_name == "f16" and args.attn_path == 0
            else "attn_chunk+attn_combine") + " (paged GQA attention, one layer)"


def main():
    args = parse()
    rank = int(os.environ.get("RANK", "0"))
    world = int(os.environ.get("WORLD_SIZE", "1"))
    local = int(os.environ.get("LOCAL_RANK", "0"))
    spec = MODELS[args.model]
    cfg = dict(spec["cfg"])
    if args.layers:
        cfg["n_layers"] = args.layers
    if not args.batch:
        args.batch = spec["batch"]
    tp = max(1, args.tp)
    if world % tp:
        raise SystemExit(f"--tp {tp} must divide the {world} ranks")
    replica, tp_rank = rank // tp, rank % tp
    kv_name = kv_dtype_name(args)
    if args.refill_steps < 0:
        args.refill_steps = args.steps
    if args.trace == "auto":
        args.trace = "poisson" if args.model == "1b" else "none"

    if args.impl == "reference":
        if rank != 0:
            return 0
        if args.model != "8b":
            print(json.dumps({"impl": "reference", "unavailable":
                              "the reference CPU arm is timed on the 8b headline config only"}))
            return 0
        import oracle as O
        if not O.Reference.available():
            print(json.dumps({"impl": "reference", "unavailable":
                              "oracle/_ref/libslate_ref.so was not built (reference sources absent at build time)"}))
            return 0
        t0 = time.time()
        path = ensure_model(args, cfg, lambda: None, O.synth_gguf)
        ctx = contexts(args, cfg, args.batch, 0, 3 * (args.warmup + args.steps) + 4)
        cpu = reference_cpu(path, ctx, [args.seed + i for i in range(len(ctx))], args.warmup,
                            args.steps, args.cpu_threads)
        line = {"metric": METRIC, "value": cpu["value"], "unit": "tok/s", "n_gpus": args.gpus,
                "steps": args.steps, "warmup": args.warmup, "ms_per_step": cpu["ms_per_step"],
                "p50_step_ms": cpu["p50_step_ms"], "higher_is_better": True, "scaling": "weak",
                "vs_baseline": None, "dtype": "f32", "data": "synthetic", "impl": "reference",
                "config": {"workload": "llama3-8b-shape q4k greedy decode, reference CPU sessions "
                                       "(BASELINE config 3 contexts)",
                           "seqs": cpu["sessions"], "kv_dtype": "f32", "mean_ctx": cpu["mean_ctx"],
                           "step": "every session decodes one token"},
                "cpu_baseline": {k: cpu[k] for k in ("value", "unit", "cores", "kind", "sample")},
                "e2e": {"value": cpu["value"], "unit": "tok/s", "h2d_bytes_per_step": 0,
                        "d2h_bytes_per_step": 0},
                "wall_s": round(time.time() - t0, 1)}
        print(json.dumps(line))
        return 0

    import torch
    import slate_b200 as sb
    torch.cuda.set_device(local)
    if world > 1:
        import datetime
        import torch.distributed as dist
        dist.init_process_group("nccl", timeout=datetime.timedelta(seconds=600),
                                device_id=torch.device("cuda", local))

        def barrier():
            dist.barrier()
    else:
        dist = None

        def barrier():
            pass

    path = ensure_model(args, cfg, barrier, sb.synth_gguf)
    tp_id = tp_group_id(dist, world, tp, rank, sb.tp_unique_id) if tp > 1 else b""
    env = dict(dist=dist, barrier=barrier, world=world, local=local, tp=tp, tp_rank=tp_rank,
               replica=replica, tp_id=tp_id)
    main_res = measure(args, cfg, path, kv_name, env, full=True)
    variant = args.variant_kv
    if variant == "auto":
        variant = "f16" if kv_name == "f32" and args.model == "8b" else "none"
    var_res = None
    if variant != "none" and variant != kv_name:
        if tp > 1:                      # a fresh NCCL group for the second engine
            env["tp_id"] = tp_group_id(dist, world, tp, rank, sb.tp_unique_id)
        var_res = measure(args, cfg, path, variant, env, full=False)

    cpu = None
    if rank == 0 and world == 1 and args.model == "8b" and not args.no_cpu_baseline:
        import oracle as O
        if O.Reference.available():
            ctx = main_res["ctx"]
            cpu = reference_cpu(path, ctx, [args.seed + i for i in range(len(ctx))], 1,
                                args.cpu_steps, args.cpu_threads)
    if dist:
        barrier()
        dist.destroy_process_group()
    if rank != 0:
        return 0
    peaks = {}
    try:
        peaks = json.load(open(os.path.join(ROOT, "MEASURED_PEAKS.json")))
        peak, peak_src = float(peaks["hbm_gbs"]), "measured"
    except Exception:
        peak, peak_src = 6650.0, "fallback"

    def step_roofline(r):
        step_s = r["tot_ms"] / 1000.0 / args.steps
        return {"bytes_per_step": r["step_bytes"], "achieved_GBps": r["step_bytes"] / step_s / 1e9,
                "frac_of_measured": r["step_bytes"] / step_s / 1e9 / peak,
                "frac_of_8TBps": r["step_bytes"] / step_s / 8e12}

    def attn_roofline(r):
        ms = r["kernel_ms"]["attention"]
        achieved = r["attn_bytes"] / (ms / 1000.0) / 1e9
        ratio = ATTN_TRAFFIC_RATIO.get(r["kv"]) if args.attn_path == 0 or r["kv"] == "f32" else None
        return {"bound": "hbm", "kernel": attn_kernel_name(r["kv"], args), "achieved": achieved,
                "peak": peak, "peak_source": peak_src, "unit": "GB/s", "frac": achieved / peak,
                "traffic": None if ratio is None else ratio * r["attn_bytes"],
                "algorithmic_bytes_per_launch": r["attn_bytes"], "launch_ms": ms}

    r = main_res
    replicas = r["replicas"]
    n = args.batch
    line = {
        "metric": spec["metric"], "value": r["value"], "unit": "tok/s", "n_gpus": world, "steps": args.steps,
        "warmup": args.warmup, "ms_per_step": r["tot_ms"] / args.steps,
        "p50_step_ms": float(np.median(r["step_ms"])), "higher_is_better": True, "scaling": "weak",
        "vs_baseline": None,
        "dtype": "f32" if kv_name == "f32" else "f32 (KV cache stored as f16)", "data": "synthetic",
        "config": {"workload": spec["workload"],
                   "model": f"llama3-{args.model}-shape random N(0,0.02) Q4_K", "layers": cfg["n_layers"],
                   "global_batch": n * replicas, "seqs_per_replica": n, "kv_dtype": kv_name,
                   "mean_ctx": float(r["ctx"].mean()),
                   "parallelism": f"replicas x{replicas}" + (f", tensor parallel {tp}" if tp > 1 else ""),
                   "gemm_path": {0: "tcgen05 3-pass hi/lo, stream-K (weights in TMEM) from 128 rows",
                                 1: "cuda-core f32", 2: "tcgen05 1-pass f16",
                                 3: "tcgen05 3-pass hi/lo, tile per CTA",
                                 4: "tcgen05 exact f16 weights, 2-pass x, stream-K",
                                 5: "tcgen05 3-pass hi/lo, weights in TMEM, stream-K",
                                 6: "tcgen05 exact f16 weights, 1-pass f16 x, stream-K"}[args.gemm_path],
                   "attn_path": ("mma.sync f16 hi/lo" if args.attn_path == 0 and kv_name == "f16"
                                 else "cuda-core"),
                   "lanes": args.lanes,
                   "l2": "inputs larger than L2 (KV read per step >> 126 MB)"},
        "roofline": attn_roofline(r),
        "step_roofline": step_roofline(r),
        "kernel_ms": r["kernel_ms"],
        "e2e": r.get("e2e"),
        "gpu_launches": r["launches"],
        "prefill": r["prefill"],
        "refill": r["refill"],
        "clocks": r["clocks"],
        "cpu_baseline": None if cpu is None else {k: cpu[k] for k in ("value", "unit", "cores", "kind", "sample")},
    }
    if r.get("trace"):
        line["trace_poisson"] = r["trace"]
    if var_res is not None:
        v = var_res
        line[f"variant_kv_{v['kv']}"] = {
            "value": v["value"], "unit": "tok/s", "ms_per_step": v["tot_ms"] / args.steps,
            "p50_step_ms": float(np.median(v["step_ms"])), "kv_dtype": v["kv"],
            "note": "same workload, seeds and steps with the KV cache in " + v["kv"],
            "roofline": attn_roofline(v), "step_roofline": step_roofline(v), "clocks": v["clocks"],
            "gpu_launches": v["launches"]}
    print(json.dumps(line))
    return 0


if __name__ == "__main__":
    sys.exit(main())
