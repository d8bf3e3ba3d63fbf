"""slate_b200 -- ctypes binding of libslate_cuda.so, the sm_100a backend for
eating-and-drinking/slate's LLaMA Q4_K continuous-batching decode.

The library's C ABI is declared in include/slate_cuda.h; this module mirrors
it for Python callers (tests, bench.py).  There is no CPU fallback: importing
works without a GPU (the library only needs the CUDA driver when a device
call is made), but a missing or unloadable library raises immediately.
"""
from __future__ import annotations

import ctypes as C
import os

import numpy as np

HERE = os.path.dirname(os.path.abspath(__file__))
LIB_PATH = os.path.join(HERE, "libslate_cuda.so")

KV_F32 = 0
KV_F16 = 1
PROF_ATTENTION, PROF_QKV, PROF_WO, PROF_GATE_UP, PROF_DOWN, PROF_LM_HEAD, PROF_STEP, PROF_ALLREDUCE = \
    range(8)

if not os.path.exists(LIB_PATH):
    raise ImportError(
        f"{LIB_PATH} is missing: build it with `python -c 'import __graft_entry__ as g; g.build()'` "
        "(or `make -C slate_b200/csrc`)")
lib = C.CDLL(LIB_PATH)

c_int, c_int64, c_float, c_size, c_u64 = C.c_int, C.c_int64, C.c_float, C.c_size_t, C.c_uint64
P = C.c_void_p
Pi32 = C.POINTER(C.c_int32)
Pf32 = C.POINTER(C.c_float)


class LayerDesc(C.Structure):
    """slate_llama_layer_desc_t (member-for-member slate_llama_layer_t)."""
    _fields_ = [(n, P) for n in ("attn_norm", "attn_q", "attn_k", "attn_v", "attn_output",
                                 "ffn_norm", "ffn_gate", "ffn_up", "ffn_down")] + \
               [(n, c_int) for n in ("attn_q_dtype", "attn_k_dtype", "attn_v_dtype",
                                     "attn_output_dtype", "ffn_gate_dtype", "ffn_up_dtype",
                                     "ffn_down_dtype")]


class LlamaDesc(C.Structure):
    _fields_ = [(n, c_int) for n in ("n_layers", "d_model", "ffn_hidden", "n_heads", "n_kv_heads",
                                     "head_dim", "max_seq", "vocab")] + [
        ("theta_base", c_float), ("rms_eps", c_float), ("tied_output", c_int),
        ("token_embd", P), ("token_embd_dtype", c_int), ("output_norm", P),
        ("output", P), ("output_dtype", c_int), ("layers", C.POINTER(C.POINTER(LayerDesc)))]


class CudaOpts(C.Structure):
    _fields_ = [("device", c_int), ("max_batch", c_int), ("max_slots", c_int),
                ("kv_dtype", c_int), ("max_seq", c_int), ("kv_pages", c_int64),
                ("kv_bytes", c_size), ("use_graphs", c_int), ("gemm_path", c_int),
                ("attn_path", c_int), ("tp_size", c_int), ("tp_rank", c_int),
                ("tp_id", C.c_ubyte * 128), ("q4k_order", c_int), ("lanes", c_int)]


class SamplerConfig(C.Structure):
    """slate_sampler_config_t (include/slate/sampling.h:15-20)."""
    _fields_ = [("temperature", c_float), ("top_k", c_int), ("top_p", c_float), ("seed", c_u64)]


def sampler_configs(n, temperature=1.0, top_k=0, top_p=0.0):
    """An array of n SamplerConfig; each argument a scalar or a length-n sequence."""
    arr = (SamplerConfig * n)()
    t, k, p = (np.broadcast_to(np.asarray(v), (n,)) for v in (temperature, top_k, top_p))
    for i in range(n):
        arr[i] = SamplerConfig(float(t[i]), int(k[i]), float(p[i]), 0)
    return arr


class SynthConfig(C.Structure):
    _fields_ = [(n, c_int) for n in ("n_layers", "d_model", "ffn_hidden", "n_heads", "n_kv_heads",
                                     "vocab", "max_seq")] + [
        ("theta_base", c_float), ("rms_eps", c_float), ("q4k", c_int), ("tied_output", c_int),
        ("seed", c_u64), ("n_threads", c_int), ("layer_period", c_int), ("q4k_order", c_int),
        ("embd_f16", c_int)]


class BackendBase(C.Structure):
    _fields_ = [("name", C.c_char_p)] + [(n, P) for n in (
        "alloc", "release", "copy_h2d", "copy_d2h", "matvec", "linear_batch", "matvec_q4k",
        "rmsnorm_row", "silu_mul", "add_inplace", "embed_lookup", "attention_step", "sync")]


class BackendCuda(C.Structure):
    _fields_ = [("base", BackendBase), ("abi_version", c_int), ("device", c_int)] + [
        (n, P) for n in ("matmul_q4k_batch", "matmul_f32_batch", "rmsnorm_rows", "argmax_rows",
                         "rope_kv_append_paged", "attention_paged_gqa", "matmul_q4k_batch_tc")]


def _proto(name, res, *args):
    f = getattr(lib, name)
    f.restype = res
    f.argtypes = list(args)
    return f


# -- exported C ABI (every symbol declared in include/slate_cuda.h) ---------
EXPORTS = {
    "slate_backend_cuda": (P,),
    "slate_backend_cuda_create": (C.POINTER(BackendCuda), c_int),
    "slate_backend_cuda_host_coherent": (P, c_int),
    "slate_cuda_pageable_memory_access": (c_int, c_int),
    "slate_cuda_last_error": (C.c_char_p,),
    "slate_cuda_tp_unique_id": (c_int, P, c_size),
    "slate_cuda_sample_rows": (c_int, Pi32, P, c_int, c_int, c_int, P, C.POINTER(c_u64)),
    "slate_cuda_attention_paged_gqa_noalloc": (c_int, P, P, P, P, P, c_int, P, c_int64, c_int, c_int,
                                               c_int, c_int, c_int, c_int, P),
    "slate_llama_batch_new_desc": (P, C.POINTER(LlamaDesc), C.POINTER(CudaOpts)),
    "slate_llama_batch_new_gguf": (P, C.c_char_p, C.POINTER(CudaOpts)),
    "slate_llama_batch_free": (None, P),
    "slate_llama_batch_vocab": (c_int, P),
    "slate_llama_batch_max_batch": (c_int, P),
    "slate_llama_batch_max_seq": (c_int, P),
    "slate_llama_batch_free_pages": (c_int64, P),
    "slate_llama_batch_open": (c_int, P),
    "slate_llama_batch_close": (c_int, P, c_int),
    "slate_llama_batch_position": (c_int, P, c_int),
    "slate_llama_batch_step": (c_int, P, Pi32, c_int, Pi32, Pi32, Pf32),
    "slate_llama_batch_step_sample": (c_int, P, Pi32, c_int, Pi32, P, C.POINTER(c_u64), Pi32, Pf32),
    "slate_llama_batch_step_device": (c_int, P, P, c_int, P, P, P, P),
    "slate_llama_batch_sync": (c_int, P),
    "slate_llama_batch_prefill": (c_int, P, c_int, Pi32, c_int, Pf32),
    "slate_llama_batch_seed_context": (c_int, P, c_int, c_int, c_u64),
    "slate_llama_batch_read_kv": (c_int, P, c_int, c_int, Pf32, Pf32),
    "slate_llama_batch_stream": (P, P),
    "slate_llama_batch_launches_per_step": (c_int, P, c_int),
    "slate_llama_batch_profile": (c_int, P, c_int, c_int, c_int, c_int, Pf32),
    "slate_llama_scheduler_new": (P, P, c_int),
    "slate_llama_scheduler_free": (None, P),
    "slate_llama_scheduler_decode": (c_int, P, c_int, C.c_int32, Pi32, Pf32),
    "slate_llama_scheduler_pending": (c_int, P),
    "slate_llama_scheduler_total_batches": (C.c_uint64, P),
    "slate_llama_scheduler_avg_batch_size": (C.c_double, P),
    "slate_gguf_model_open": (P, C.c_char_p, C.POINTER(LlamaDesc)),
    "slate_gguf_model_close": (None, P),
    "slate_q4k_quantize_rows": (c_int, P, Pf32, c_int64, c_int),
    "slate_synth_llama_gguf": (c_int, C.c_char_p, C.POINTER(SynthConfig)),
}
F = {name: _proto(name, *sig) for name, sig in EXPORTS.items()}


def last_error() -> str:
    return F["slate_cuda_last_error"]().decode()


def _ptr(a, t=C.c_float):
    return a.ctypes.data_as(C.POINTER(t))


def quantize_q4k(w: np.ndarray) -> np.ndarray:
    """Rows of f32 (K % 256 == 0) -> Slate-layout Q4_K bytes [rows, K/256*144]."""
    w = np.ascontiguousarray(w, dtype=np.float32)
    rows, K = w.shape
    out = np.zeros((rows, K // 256 * 144), dtype=np.uint8)
    rc = F["slate_q4k_quantize_rows"](out.ctypes.data, _ptr(w), rows, K)
    if rc:
        raise ValueError(f"slate_q4k_quantize_rows rc={rc}")
    return out


def synth_gguf(path: str, *, n_layers, d_model, ffn_hidden, n_heads, n_kv_heads, vocab, max_seq,
               theta_base=10000.0, rms_eps=1e-5, q4k=True, tied_output=False, seed=0,
               n_threads=0, layer_period=0, q4k_order=0, embd_f16=0) -> None:
    """Writes a synthetic LLaMA GGUF (N(0,0.02) weights; Q4_K in Slate's nibble
    order, or llama.cpp's with q4k_order=1; embd_f16: 1 f16 embedding/output
    tables, 2 f32 tables holding f16-rounded values)."""
    cfg = SynthConfig(n_layers, d_model, ffn_hidden, n_heads, n_kv_heads, vocab, max_seq,
                      theta_base, rms_eps, int(q4k), int(tied_output), seed, n_threads,
                      layer_period, q4k_order, embd_f16)
    rc = F["slate_synth_llama_gguf"](path.encode(), C.byref(cfg))
    if rc:
        raise OSError(f"slate_synth_llama_gguf({path}) rc={rc}")


def sample_rows(d_logits, ld, B, V, cfg, rng):
    """slate_cuda_sample_rows: device logits pointer, host configs and uint64
    RNG states (updated in place).  Returns (rc, tokens[B])."""
    assert rng.dtype == np.uint64 and rng.flags.c_contiguous and len(rng) == B
    out = np.zeros(B, dtype=np.int32)
    rc = F["slate_cuda_sample_rows"](_ptr(out, C.c_int32), d_logits, ld, B, V, C.byref(cfg),
                                     rng.ctypes.data_as(C.POINTER(c_u64)))
    return rc, out


def tp_unique_id() -> bytes:
    """128-byte id for a tensor-parallel group (slate_cuda_tp_unique_id)."""
    buf = C.create_string_buffer(128)
    rc = F["slate_cuda_tp_unique_id"](buf, 128)
    if rc:
        raise RuntimeError(f"slate_cuda_tp_unique_id rc={rc}: {last_error()}")
    return buf.raw


class LlamaBatch:
    """Device-resident batch engine (slate_llama_batch_*) over one GGUF."""

    def __init__(self, gguf_path: str, *, device=0, max_batch=16, max_slots=0, kv_dtype=KV_F32,
                 max_seq=0, kv_pages=0, kv_bytes=0, use_graphs=True, gemm_path=0, attn_path=0,
                 tp_size=0, tp_rank=0, tp_id=b"", q4k_order=0, lanes=0):
        self.opts = CudaOpts(device, max_batch, max_slots, kv_dtype, max_seq, kv_pages, kv_bytes,
                             int(use_graphs), gemm_path, attn_path, tp_size, tp_rank)
        self.opts.q4k_order = q4k_order
        self.opts.lanes = lanes
        if tp_id:
            C.memmove(self.opts.tp_id, bytes(tp_id), min(len(tp_id), 128))
        self.h = F["slate_llama_batch_new_gguf"](gguf_path.encode(), C.byref(self.opts))
        if not self.h:
            raise RuntimeError(f"slate_llama_batch_new_gguf failed: {last_error()}")
        self.vocab = F["slate_llama_batch_vocab"](self.h)
        self.max_batch = F["slate_llama_batch_max_batch"](self.h)
        self.max_seq = F["slate_llama_batch_max_seq"](self.h)

    def close(self):
        if self.h:
            F["slate_llama_batch_free"](self.h)
            self.h = None

    def __del__(self):
        try:
            self.close()
        except Exception:
            pass

    def open(self) -> int:
        return F["slate_llama_batch_open"](self.h)

    def release(self, slot: int) -> int:
        return F["slate_llama_batch_close"](self.h, slot)

    def position(self, slot: int) -> int:
        return F["slate_llama_batch_position"](self.h, slot)

    def free_pages(self) -> int:
        return F["slate_llama_batch_free_pages"](self.h)

    def step(self, slots, tokens, want_logits=False):
        """Returns (rc, out_tokens[n], logits[n, V] or None)."""
        slots = np.ascontiguousarray(slots, dtype=np.int32)
        tokens = np.ascontiguousarray(tokens, dtype=np.int32)
        n = len(slots)
        out = np.zeros(n, dtype=np.int32)
        lg = np.zeros((n, self.vocab), dtype=np.float32) if want_logits else None
        rc = F["slate_llama_batch_step"](self.h, _ptr(slots, C.c_int32), n, _ptr(tokens, C.c_int32),
                                         _ptr(out, C.c_int32),
                                         _ptr(lg) if lg is not None else None)
        return rc, out, lg

    def step_sample(self, slots, tokens, cfg, rng, want_logits=False):
        """Sampling step: cfg from sampler_configs(n, ...), rng uint64[n] (updated
        in place).  Returns (rc, out_tokens[n], logits[n, V] or None)."""
        slots = np.ascontiguousarray(slots, dtype=np.int32)
        tokens = np.ascontiguousarray(tokens, dtype=np.int32)
        n = len(slots)
        assert rng.dtype == np.uint64 and rng.flags.c_contiguous and len(rng) == n
        out = np.zeros(n, dtype=np.int32)
        lg = np.zeros((n, self.vocab), dtype=np.float32) if want_logits else None
        rc = F["slate_llama_batch_step_sample"](self.h, _ptr(slots, C.c_int32), n,
                                                _ptr(tokens, C.c_int32), C.byref(cfg),
                                                rng.ctypes.data_as(C.POINTER(c_u64)),
                                                _ptr(out, C.c_int32),
                                                _ptr(lg) if lg is not None else None)
        return rc, out, lg

    def step_device(self, d_slots, n, d_tokens, d_out_tokens, d_out_logits=None, stream=None):
        return F["slate_llama_batch_step_device"](self.h, d_slots, n, d_tokens, d_out_tokens,
                                                  d_out_logits, stream)

    def sync(self) -> int:
        return F["slate_llama_batch_sync"](self.h)

    def prefill(self, slot, tokens, want_logits=True):
        tokens = np.ascontiguousarray(tokens, dtype=np.int32)
        lg = np.zeros(self.vocab, dtype=np.float32) if want_logits else None
        rc = F["slate_llama_batch_prefill"](self.h, slot, _ptr(tokens, C.c_int32), len(tokens),
                                            _ptr(lg) if lg is not None else None)
        return rc, lg

    def seed_context(self, slot, n_tokens, seed) -> int:
        return F["slate_llama_batch_seed_context"](self.h, slot, n_tokens, seed)

    def read_kv(self, slot, n, n_layers, kv_dim):
        K = np.zeros((n_layers, n, kv_dim), dtype=np.float32)
        V = np.zeros_like(K)
        rc = F["slate_llama_batch_read_kv"](self.h, slot, n, _ptr(K), _ptr(V))
        return rc, K, V

    def stream(self):
        return F["slate_llama_batch_stream"](self.h)

    def launches_per_step(self, n) -> int:
        return F["slate_llama_batch_launches_per_step"](self.h, n)

    def profile(self, kernel, n, layer=0, iters=10) -> float:
        """Mean ms per launch of one kernel group (PROF_*) for the last step's rows."""
        ms = C.c_float(0)
        rc = F["slate_llama_batch_profile"](self.h, kernel, n, layer, iters, C.byref(ms))
        if rc:
            raise RuntimeError(f"profile rc={rc}: {last_error()}")
        return ms.value


class Scheduler:
    """slate_llama_scheduler_*: one decoder thread micro-batching decode calls."""

    def __init__(self, batch: LlamaBatch, max_batch: int):
        self.batch = batch
        self.h = F["slate_llama_scheduler_new"](batch.h, max_batch)
        if not self.h:
            raise RuntimeError("slate_llama_scheduler_new failed")

    def decode(self, slot, token, want_logits=False):
        out = np.zeros(1, dtype=np.int32)
        lg = np.zeros(self.batch.vocab, dtype=np.float32) if want_logits else None
        rc = F["slate_llama_scheduler_decode"](self.h, slot, token, _ptr(out, C.c_int32),
                                               _ptr(lg) if lg is not None else None)
        return rc, int(out[0]), lg

    def stats(self):
        return (F["slate_llama_scheduler_pending"](self.h),
                F["slate_llama_scheduler_total_batches"](self.h),
                F["slate_llama_scheduler_avg_batch_size"](self.h))

    def close(self):
        if self.h:
            F["slate_llama_scheduler_free"](self.h)
            self.h = None
