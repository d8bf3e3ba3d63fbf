"""Batch-engine parity through the C ABI (slate_llama_batch_*) against the
oracle's independent per-sequence sessions (src/loader/llama_infer.c
semantics), on the reference's golden models and on synthetic models.

Tolerances (written here, applied to every logit of every step):
  * f32 KV cache: max |engine - oracle| <= 1e-4 * max |oracle logits|
  * f16 KV cache: <= 2e-3 * max |oracle logits|
Greedy ids must equal the oracle's argmax; the only accepted difference is a
near-tie, where the oracle's own top-2 gap is within that tolerance -- those
are counted and reported, and every sequence is teacher-forced with the
engine's token so a tie never cascades.
"""
import os
import threading

import numpy as np
import pytest

from conftest import golden
from gpu_util import greedy_agrees, scale_err, seeded_kv
from test_golden import TINY, read_ref_logits

pytestmark = pytest.mark.gpu


def make_engine(sb, path, **kw):
    return sb.LlamaBatch(path, **kw)


@pytest.mark.parametrize("gguf,ref", TINY)
def test_engine_prefill_matches_reference_fixture(sb, oracle, gguf, ref):
    """test_llama_infer{,_gqa,_q4k}.c on the GPU engine: Linf < 1e-3 vs numpy."""
    prompt, want = read_ref_logits(ref)
    eng = make_engine(sb, golden(gguf), max_batch=4)
    s = eng.open()
    rc, lg = eng.prefill(s, prompt)
    assert rc == 0 and eng.position(s) == len(prompt)
    assert np.max(np.abs(lg - want)) < 1e-3
    m = oracle.open(golden(gguf))
    o, _ = m.decode_many(prompt[None, :])
    assert scale_err(lg, o[0, -1]) < 1e-4
    eng.close()


def run_continuous(eng, requests, max_batch, rng):
    """Continuous batching: requests (prompt, n_new) join when a batch row is
    free and leave when done.  Returns per-request token streams and logits."""
    waiting = list(range(len(requests)))
    active = {}                                # req -> dict(slot, fed, stream, logits)
    done = {}
    while waiting or active:
        while waiting and len(active) < max_batch:
            r = waiting.pop(0)
            slot = eng.open()
            assert slot >= 0
            active[r] = dict(slot=slot, fed=0, stream=[], logits=[])
        reqs = list(active)
        rng.shuffle(reqs)                       # row order must not matter
        slots, toks = [], []
        for r in reqs:
            a, (prompt, _) = active[r], requests[r]
            tok = prompt[a["fed"]] if a["fed"] < len(prompt) else a["stream"][-1]
            slots.append(a["slot"])
            toks.append(tok)
        rc, out, lg = eng.step(slots, toks, want_logits=True)
        assert rc == 0, rc
        for i, r in enumerate(reqs):
            a, (prompt, n_new) = active[r], requests[r]
            a["fed"] += 1
            if a["fed"] >= len(prompt):
                a["stream"].append(int(out[i]))
                a["logits"].append(lg[i])
            if len(a["stream"]) >= n_new:
                assert eng.release(a["slot"]) == 0
                done[r] = a
                del active[r]
    return done


def check_against_oracle(oracle, path, requests, done, tol):
    """Teacher-forced oracle sessions fed prompt + the engine's own tokens."""
    m = oracle.open(path)
    n_tie = 0
    worst = 0.0
    for r, (prompt, n_new) in enumerate(requests):
        stream = done[r]["stream"]
        feed = np.array(list(prompt) + stream[:-1], np.int32)
        lg, _ = m.decode_many(feed[None, :])
        ref = lg[0, len(prompt) - 1:]
        got = np.stack(done[r]["logits"])
        assert ref.shape == got.shape
        scale = max(np.abs(ref).max(), 1e-30)
        err = np.max(np.abs(got - ref)) / scale
        worst = max(worst, err)
        assert err <= tol, (r, err)
        for t, tok in enumerate(stream):
            ok, tie = greedy_agrees(tok, ref[t], tol * scale)
            assert ok, (r, t, tok, int(np.argmax(ref[t])))
            n_tie += tie
    m.close()
    return n_tie, worst


def test_config1_continuous_batching(sb, oracle, workdir):
    """tiny all-f32 GQA decoder, 16 requests, prompts
    U{4..32}, 32 greedy tokens each, joining and leaving a batch of 8."""
    path = os.path.join(str(workdir), "cfg1.gguf")
    sb.synth_gguf(path, n_layers=2, d_model=64, ffn_hidden=172, n_heads=4, n_kv_heads=2,
                  vocab=256, max_seq=128, q4k=False, seed=0)
    rng = np.random.default_rng(0)
    reqs = [(rng.integers(0, 256, rng.integers(4, 33)).astype(np.int32), 32) for _ in range(16)]
    eng = make_engine(sb, path, max_batch=8, max_slots=8)
    done = run_continuous(eng, reqs, 8, rng)
    eng.close()
    n_tie, worst = check_against_oracle(oracle, path, reqs, done, 1e-4)
    print(f"config1: worst logit err {worst:.2e} of scale, near-ties {n_tie}")


@pytest.mark.parametrize("kv_dtype,tol", [(0, 1e-4), (1, 2e-3)])
@pytest.mark.parametrize("max_batch", [4, 24, 70])
def test_gqa_q4k_continuous_batching(sb, oracle, workdir, kv_dtype, tol, max_batch):
    """Q4_K GQA model through GEMV (<=8 rows), BN-64 and BN-128 tiled GEMMs."""
    path = os.path.join(str(workdir), "gqa_q4k.gguf")
    if not os.path.exists(path):
        sb.synth_gguf(path, n_layers=2, d_model=512, ffn_hidden=1024, n_heads=8, n_kv_heads=2,
                      vocab=512, max_seq=512, q4k=True, seed=7)
    rng = np.random.default_rng(max_batch + kv_dtype)
    n_req = max_batch + 6
    reqs = [(rng.integers(0, 512, rng.integers(1, 40)).astype(np.int32), int(rng.integers(3, 12)))
            for _ in range(n_req)]
    eng = make_engine(sb, path, max_batch=max_batch, kv_dtype=kv_dtype)
    done = run_continuous(eng, reqs, max_batch, rng)
    eng.close()
    check_against_oracle(oracle, path, reqs, done, tol)


def test_graphs_and_eager_agree(sb, workdir):
    path = os.path.join(str(workdir), "gqa_q4k.gguf")
    if not os.path.exists(path):
        sb.synth_gguf(path, n_layers=2, d_model=512, ffn_hidden=1024, n_heads=8, n_kv_heads=2,
                      vocab=512, max_seq=512, q4k=True, seed=7)
    outs = []
    for graphs in (True, False):
        eng = make_engine(sb, path, max_batch=8, use_graphs=graphs)
        slots = [eng.open() for _ in range(5)]
        toks = np.array([1, 2, 3, 4, 5], np.int32)
        res = []
        for _ in range(6):
            rc, out, lg = eng.step(slots, toks, want_logits=True)
            assert rc == 0, sb.last_error()
            res.append(lg)
            toks = out
        outs.append(np.stack(res))
        eng.close()
    assert np.array_equal(outs[0], outs[1])


def test_error_codes_leave_state_unchanged(sb, workdir):
    path = os.path.join(str(workdir), "err.gguf")
    sb.synth_gguf(path, n_layers=1, d_model=256, ffn_hidden=256, n_heads=4, n_kv_heads=2,
                  vocab=300, max_seq=20, q4k=True, seed=3)
    eng = make_engine(sb, path, max_batch=2, max_slots=2)
    a, b = eng.open(), eng.open()
    assert eng.open() == -2                                  # no free slot
    assert eng.step([a], [300])[0] == -3                     # token == vocab
    assert eng.step([a], [-1])[0] == -3
    assert eng.step([a, a], [1, 2])[0] == -1                 # same slot twice
    assert eng.step([5], [1])[0] == -1                       # slot never opened
    assert eng.position(a) == 0
    for i in range(20):
        assert eng.step([a, b], [i, i])[0] == 0
    assert eng.step([a], [1])[0] == -2                       # cache full (max_seq 20)
    assert eng.position(a) == 20
    assert eng.release(b) == 0 and eng.open() == b and eng.position(b) == 0
    assert eng.step([b], [7])[0] == 0 and eng.position(b) == 1
    eng.close()


def test_page_pool_exhaustion(sb, workdir):
    path = os.path.join(str(workdir), "err.gguf")
    if not os.path.exists(path):
        sb.synth_gguf(path, n_layers=1, d_model=256, ffn_hidden=256, n_heads=4, n_kv_heads=2,
                      vocab=300, max_seq=20, q4k=True, seed=3)
    eng = make_engine(sb, path, max_batch=4, max_slots=4, kv_pages=2)
    a, b, c = eng.open(), eng.open(), eng.open()
    assert eng.step([a, b], [1, 2])[0] == 0                  # two pages in use
    assert eng.step([c], [3])[0] == -2                       # third page unavailable
    assert eng.step([a, b], [4, 5])[0] == 0                  # existing pages keep working
    assert eng.release(a) == 0
    assert eng.step([c], [3])[0] == 0                        # page came back
    eng.close()


@pytest.mark.parametrize("kv_dtype", [0, 1])
def test_seeded_context_is_the_documented_generator(sb, workdir, kv_dtype):
    """seed_context writes the generator the reference-side timing reproduces
    (tests/gpu_util.seeded_kv, oracle/ref_session.c): exactly in an f32 cache,
    its f16 rounding in an f16 cache."""
    path = os.path.join(str(workdir), "gqa_q4k.gguf")
    if not os.path.exists(path):
        sb.synth_gguf(path, n_layers=2, d_model=512, ffn_hidden=1024, n_heads=8, n_kv_heads=2,
                      vocab=512, max_seq=512, q4k=True, seed=7)
    eng = make_engine(sb, path, max_batch=4, max_seq=1024, kv_dtype=kv_dtype)
    s = eng.open()
    assert eng.seed_context(s, 333, seed=987654321) == 0
    rc, K, V = eng.read_kv(s, 333, 2, 128)
    assert rc == 0, sb.last_error()
    Kw, Vw = seeded_kv(987654321, 333, 2, 128)
    if kv_dtype == 1:
        Kw, Vw = Kw.astype(np.float16).astype(np.float32), Vw.astype(np.float16).astype(np.float32)
    assert np.array_equal(K, Kw) and np.array_equal(V, Vw)
    eng.close()


def test_seeded_context_matches_oracle(sb, oracle, workdir):
    """Long contexts: seed 40..700-token histories, read them back, seed the
    oracle sessions with the same K/V, then decode 3 tokens in one batch."""
    path = os.path.join(str(workdir), "gqa_q4k.gguf")
    if not os.path.exists(path):
        sb.synth_gguf(path, n_layers=2, d_model=512, ffn_hidden=1024, n_heads=8, n_kv_heads=2,
                      vocab=512, max_seq=512, q4k=True, seed=7)
    eng = make_engine(sb, path, max_batch=8, max_seq=1024)
    m = oracle.open(path)
    ctxs = [40, 255, 256, 257, 511, 700]
    slots = [eng.open() for _ in ctxs]
    sess = []
    for s, c in zip(slots, ctxs):
        assert eng.seed_context(s, c, seed=1000 + c) == 0 and eng.position(s) == c
        rc, K, V = eng.read_kv(s, c, 2, 128)
        assert rc == 0 and np.abs(K).max() < 1 and np.abs(K).max() > 0.5
        o = m.session(max_seq=1024)
        assert o.seed_kv(K, V) == 0
        sess.append(o)
    toks = np.array([3, 1, 4, 1, 5, 9], np.int32)
    for _ in range(3):
        rc, out, lg = eng.step(slots, toks, want_logits=True)
        assert rc == 0, sb.last_error()
        for i, o in enumerate(sess):
            rc, ref = o.decode(int(toks[i]))
            assert rc == 0, sb.last_error()
            assert scale_err(lg[i], ref) < 1e-4
            assert greedy_agrees(int(out[i]), ref, 1e-4 * np.abs(ref).max())[0]
        toks = out
    m.close()
    eng.close()


def test_device_step_matches_host_step(sb, workdir):
    import torch
    path = os.path.join(str(workdir), "gqa_q4k.gguf")
    if not os.path.exists(path):
        sb.synth_gguf(path, n_layers=2, d_model=512, ffn_hidden=1024, n_heads=8, n_kv_heads=2,
                      vocab=512, max_seq=512, q4k=True, seed=7)
    res = []
    for dev_api in (False, True):
        eng = make_engine(sb, path, max_batch=16)
        slots = np.array([eng.open() for _ in range(12)], np.int32)
        toks = np.arange(12, dtype=np.int32) * 7
        seq = []
        if dev_api:
            d_s = torch.tensor(slots, device="cuda")
            d_t = torch.tensor(toks, device="cuda")
            d_o = torch.zeros(12, dtype=torch.int32, device="cuda")
            for _ in range(5):
                assert eng.step_device(d_s.data_ptr(), 12, d_t.data_ptr(), d_o.data_ptr()) == 0
                assert eng.sync() == 0
                seq.append(d_o.cpu().numpy().copy())
                d_t.copy_(d_o)
            assert eng.position(int(slots[0])) == 5
        else:
            for _ in range(5):
                rc, out, _ = eng.step(slots, toks)
                assert rc == 0, sb.last_error()
                seq.append(out.copy())
                toks = out
        res.append(np.stack(seq))
        eng.close()
    assert np.array_equal(res[0], res[1])


@pytest.mark.parametrize("kv_dtype,tol", [(0, 1e-4), (1, 2e-3)])
def test_two_lanes_match_oracle(sb, oracle, workdir, kv_dtype, tol):
    """With lanes=2 a decode step of more than max_batch / 2 rows runs as two
    lanes (the halves of the batch on two streams, each with its own GEMM
    operands and stream-K workspace, their attentions taking turns); with
    lanes=1 the same steps run as one chain.  Both match the oracle's
    per-sequence sessions, rows in a rotating order."""
    path = os.path.join(str(workdir), "paths_q4k.gguf")
    if not os.path.exists(path):
        sb.synth_gguf(path, n_layers=2, d_model=1024, ffn_hidden=2816, n_heads=16, n_kv_heads=4,
                      vocab=2000, max_seq=64, q4k=True, seed=11)
    n, T = 90, 4
    rng = np.random.default_rng(90 + kv_dtype)
    feed = rng.integers(0, 2000, (n, T)).astype(np.int32)
    m = oracle.open(path)
    ref, _ = m.decode_many(feed)
    m.close()
    scale = np.abs(ref).max()
    for lanes in (2, 1):
        eng = make_engine(sb, path, max_batch=96, kv_dtype=kv_dtype, lanes=lanes)
        slots = np.array([eng.open() for _ in range(n)], np.int32)
        for t in range(T):
            order = np.roll(np.arange(n), 7 * t)
            rc, out, lg = eng.step(slots[order], feed[order, t], want_logits=True)
            assert rc == 0, (lanes, t, sb.last_error())
            got = lg[np.argsort(order)]
            err = np.max(np.abs(got - ref[:, t])) / scale
            assert err < tol, (lanes, t, err)
        eng.close()


def test_device_step_rejects_repeated_slot(sb, workdir):
    """slate_llama_batch_step_device validates on the device: a slot that
    occurs twice in one step is a bad slot (-1, as slate_llama_batch_step),
    and the step leaves positions unchanged."""
    import torch
    path = os.path.join(str(workdir), "gqa_q4k.gguf")
    if not os.path.exists(path):
        sb.synth_gguf(path, n_layers=2, d_model=512, ffn_hidden=1024, n_heads=8, n_kv_heads=2,
                      vocab=512, max_seq=512, q4k=True, seed=7)
    eng = make_engine(sb, path, max_batch=64)
    slots = [eng.open() for _ in range(40)]
    slots[39] = slots[3]
    d_s = torch.tensor(np.array(slots, np.int32), device="cuda")
    d_t = torch.zeros(40, dtype=torch.int32, device="cuda")
    d_o = torch.zeros(40, dtype=torch.int32, device="cuda")
    assert eng.step_device(d_s.data_ptr(), 40, d_t.data_ptr(), d_o.data_ptr()) == 0
    assert eng.sync() == -1
    assert eng.position(slots[3]) == 0
    eng.close()


def test_scheduler_batches_concurrent_callers(sb, oracle, workdir):
    path = os.path.join(str(workdir), "gqa_q4k.gguf")
    if not os.path.exists(path):
        sb.synth_gguf(path, n_layers=2, d_model=512, ffn_hidden=1024, n_heads=8, n_kv_heads=2,
                      vocab=512, max_seq=512, q4k=True, seed=7)
    eng = make_engine(sb, path, max_batch=8)
    sched = sb.Scheduler(eng, 8)
    n_workers, n_tok = 6, 10
    streams = {}

    def worker(w):
        slot = eng.open()
        tok, out = 11 * w + 1, []
        for _ in range(n_tok):
            rc, nxt, _ = sched.decode(slot, tok)
            assert rc == 0, sb.last_error()
            out.append(nxt)
            tok = nxt
        streams[w] = out

    th = [threading.Thread(target=worker, args=(w,)) for w in range(n_workers)]
    for t in th:
        t.start()
    for t in th:
        t.join()
    _, batches, avg = sched.stats()
    sched.close()
    eng.close()
    assert batches >= n_tok and avg >= 1.0
    m = oracle.open(path)
    for w, out in streams.items():
        feed = np.array([11 * w + 1] + out[:-1], np.int32)
        lg, ids = m.decode_many(feed[None, :])
        for t in range(n_tok):
            assert greedy_agrees(out[t], lg[0, t], 1e-4 * np.abs(lg[0, t]).max())[0]
    m.close()


@pytest.mark.parametrize("n_rows", [1, 2, 3, 40, 150])
def test_gemm_paths_agree_with_oracle(sb, oracle, workdir, n_rows):
    """The GEMM paths of the engine -- the default (0: the 3-pass split, on the
    stream-K kernel from 128 rows), the tile-per-CTA 3-pass kernel (3), the
    exact-weight stream-K kernel (4) and its one-pass mode (6), the 3-pass
    stream-K kernel (5; the stream-K kernels with their STORE / residual ADD /
    fused SiLU*up epilogues) and CUDA cores (1) -- each match the oracle on a
    2-layer Q4_K model at batch sizes with a partial second row tile."""
    path = os.path.join(str(workdir), "paths_q4k.gguf")
    if not os.path.exists(path):
        sb.synth_gguf(path, n_layers=2, d_model=1024, ffn_hidden=2816, n_heads=16, n_kv_heads=4,
                      vocab=2000, max_seq=64, q4k=True, seed=11)
    rng = np.random.default_rng(n_rows)
    T = 3
    feed = rng.integers(0, 2000, (n_rows, T)).astype(np.int32)
    m = oracle.open(path)
    ref, _ = m.decode_many(feed)
    m.close()
    scale = np.abs(ref).max()
    # (path, bound): x rounded once to f16 (path 6) carries ~2^-12 per element
    for gp, tol in ((0, 1e-4), (3, 1e-4), (4, 1e-4), (5, 1e-4), (1, 1e-4), (6, 3e-3)):
        eng = make_engine(sb, path, max_batch=n_rows, gemm_path=gp)
        slots = [eng.open() for _ in range(n_rows)]
        for t in range(T):
            rc, out, lg = eng.step(slots, feed[:, t], want_logits=True)
            assert rc == 0, (gp, rc, sb.last_error())
            err = np.max(np.abs(lg - ref[:, t])) / scale
            assert err < tol, (gp, t, err)
        eng.close()


@pytest.mark.parametrize("kv_dtype,tol", [(1, 2e-3), (0, 1e-4)])
@pytest.mark.parametrize("max_batch", [64, 256])
def test_prefill_attention_long_prompt(sb, oracle, workdir, max_batch, kv_dtype, tol):
    """The causal prefill attention (head_dim 128, four query heads per kv
    head -- the 8B head geometry) on prompts that cross the 1024-token context
    chunks and 16-token pages inside a step, two sequences prefilled one after
    the other: the f16 cache through the tensor-core prefill kernel, the f32
    cache through the four-row tiles of the CUDA-core kernel.  The last prompt
    logits and three decoded steps against the oracle's token-by-token
    sessions (2e-3 of scale for f16 KV, 1e-4 for f32)."""
    path = os.path.join(str(workdir), "prefill_hd128.gguf")
    if not os.path.exists(path):
        sb.synth_gguf(path, n_layers=2, d_model=1024, ffn_hidden=2048, n_heads=8, n_kv_heads=2,
                      vocab=1000, max_seq=2048, theta_base=500000.0, q4k=True, seed=23)
    rng = np.random.default_rng(max_batch)
    lens = [1300, 1037]
    prompts = [rng.integers(0, 1000, L).astype(np.int32) for L in lens]
    eng = make_engine(sb, path, max_batch=max_batch, max_slots=2, kv_dtype=kv_dtype)
    slots = [eng.open() for _ in lens]
    last = []
    for s, p in zip(slots, prompts):
        rc, lg = eng.prefill(s, p)
        assert rc == 0, sb.last_error()
        last.append(lg)
    toks = np.array([int(np.argmax(l)) for l in last], np.int32)
    streams = [[t] for t in toks]
    dec = []
    for _ in range(3):
        rc, out, lg = eng.step(np.array(slots, np.int32), toks, want_logits=True)
        assert rc == 0, sb.last_error()
        dec.append(lg)
        toks = out
        for i, t in enumerate(out):
            streams[i].append(int(t))
    eng.close()
    m = oracle.open(path)
    for i, p in enumerate(prompts):
        feed = np.array(list(p) + streams[i][:-1], np.int32)
        ref, _ = m.decode_many(feed[None, :])
        ref = ref[0]
        scale = np.abs(ref).max()
        assert np.max(np.abs(last[i] - ref[len(p) - 1])) / scale <= tol, (i, "prefill")
        for t in range(3):
            assert np.max(np.abs(dec[t][i] - ref[len(p) + t])) / scale <= tol, (i, t)
    m.close()


@pytest.mark.parametrize("kv_dtype,tol", [(0, 1e-4), (1, 2e-3)])
@pytest.mark.parametrize("max_batch", [16, 64])
def test_batched_prefill_matches_oracle(sb, oracle, workdir, kv_dtype, tol, max_batch):
    """Prefill in chunks of max_batch prompt tokens (rows of one slot at
    consecutive positions, crossing 16-token pages inside a chunk), then greedy
    decode of all sequences together; every logit against the oracle's
    token-by-token sessions (llama_infer.c:262-272 semantics)."""
    path = os.path.join(str(workdir), "prefill_q4k.gguf")
    if not os.path.exists(path):
        sb.synth_gguf(path, n_layers=2, d_model=512, ffn_hidden=1024, n_heads=8, n_kv_heads=2,
                      vocab=800, max_seq=512, q4k=True, seed=17)
    rng = np.random.default_rng(max_batch + kv_dtype)
    lens = [1, 15, 17, 100, 333]
    prompts = [rng.integers(0, 800, L).astype(np.int32) for L in lens]
    eng = make_engine(sb, path, max_batch=max_batch, max_slots=len(lens), kv_dtype=kv_dtype)
    slots = [eng.open() for _ in lens]
    last = []
    for s, p in zip(slots, prompts):
        rc, lg = eng.prefill(s, p)
        assert rc == 0, sb.last_error()
        assert eng.position(s) == len(p)
        last.append(lg)
    m = oracle.open(path)
    n_new = 6
    toks = np.array([int(np.argmax(l)) for l in last], np.int32)
    streams = [[t] for t in toks]
    dec = []
    for _ in range(n_new - 1):
        rc, out, lg = eng.step(slots, toks, want_logits=True)
        assert rc == 0, sb.last_error()
        dec.append(lg)
        toks = out
        for i, t in enumerate(out):
            streams[i].append(int(t))
    for i, p in enumerate(prompts):
        feed = np.array(list(p) + streams[i][:-1], np.int32)
        ref, _ = m.decode_many(feed[None, :])
        ref = ref[0]
        scale = np.abs(ref).max()
        assert np.max(np.abs(last[i] - ref[len(p) - 1])) / scale <= tol, (i, "prefill")
        for t in range(n_new - 1):
            err = np.max(np.abs(dec[t][i] - ref[len(p) + t])) / scale
            assert err <= tol, (i, t, err)
    m.close()
    eng.close()


@pytest.mark.parametrize("n_rows", [5, 40])
def test_llama_cpp_order_and_f16_embeddings(sb, oracle, workdir, n_rows):
    """A file in llama.cpp's Q4_K nibble order loaded with q4k_order=1, and a file
    with an f16 embedding table, give logits bitwise equal to the Slate-order /
    f32-table engine (GEMV rows and tensor-core rows); that engine matches the
    oracle."""
    cfg = dict(n_layers=2, d_model=512, ffn_hidden=1024, n_heads=8, n_kv_heads=2, vocab=700,
               max_seq=64, q4k=True, seed=23)
    paths = {}
    for name, kw in (("slate", {"embd_f16": 2}), ("ggml", {"embd_f16": 2, "q4k_order": 1}),
                     ("f16", {"embd_f16": 1})):
        paths[name] = os.path.join(str(workdir), f"fmt_{name}.gguf")
        if not os.path.exists(paths[name]):
            sb.synth_gguf(paths[name], **cfg, **kw)
    rng = np.random.default_rng(n_rows)
    T = 3
    feed = rng.integers(0, 700, (n_rows, T)).astype(np.int32)
    outs = {}
    for name, q4k_order in (("slate", 0), ("ggml", 1), ("f16", 0)):
        eng = make_engine(sb, paths[name], max_batch=n_rows, q4k_order=q4k_order)
        slots = [eng.open() for _ in range(n_rows)]
        lgs = []
        for t in range(T):
            rc, _, lg = eng.step(slots, feed[:, t], want_logits=True)
            assert rc == 0, (name, sb.last_error())
            lgs.append(lg)
        outs[name] = np.stack(lgs, 1)
        eng.close()
    assert np.array_equal(outs["ggml"], outs["slate"])
    assert np.array_equal(outs["f16"], outs["slate"])
    m = oracle.open(paths["slate"])
    ref, _ = m.decode_many(feed)
    m.close()
    assert np.max(np.abs(outs["slate"] - ref)) / np.abs(ref).max() <= 1e-4
