"""oracle -- TEST INFRASTRUCTURE: CPU checkers for the CUDA decode path.

Two checkers and one workload writer, all loaded with ctypes:
  * `Oracle`    -- build/liboracle.so, the C restatement in slate_oracle.c of
                   the reference's LLaMA Q4_K decode (each function cites the
                   reference file:line it follows);
  * `Reference` -- _ref/libslate_ref.so, the reference's own sources
                   (eating-and-drinking/slate) compiled unmodified by
                   oracle/Makefile; absent where the reference tree was never
                   available to build it.
  * `synth_gguf` -- build/libslate_synth.so, the synthetic-model writer of
                   slate_b200/csrc/synth.c compiled alone (no CUDA), so a
                   process that times the reference on the CPU writes the same
                   workload file without mapping the product library.

Only tests/, __graft_entry__.smoke() and bench.py's CPU-baseline leg use this
package; the product library never links or calls it.
"""
from __future__ import annotations

import ctypes as C
import os
import subprocess

import numpy as np

HERE = os.path.dirname(os.path.abspath(__file__))
ORACLE_SO = os.path.join(HERE, "build", "liboracle.so")
SYNTH_SO = os.path.join(HERE, "build", "libslate_synth.so")
REF_SO = os.path.join(HERE, "_ref", "libslate_ref.so")

Pf = C.POINTER(C.c_float)
Pi = C.POINTER(C.c_int32)


def build(ref_root: str | None = None) -> None:
    """Builds the restatement and, when the reference tree exists, _ref."""
    args = ["make", "-C", HERE, "-j8"]
    if ref_root:
        args.append(f"REF={ref_root}")
    subprocess.run(args, check=True, stdout=subprocess.DEVNULL)


class SynthConfig(C.Structure):
    """slate_synth_config_t (include/slate_cuda.h)."""
    _fields_ = [(n, C.c_int) for n in ("n_layers", "d_model", "ffn_hidden", "n_heads", "n_kv_heads",
                                       "vocab", "max_seq")] + [
        ("theta_base", C.c_float), ("rms_eps", C.c_float), ("q4k", C.c_int), ("tied_output", C.c_int),
        ("seed", C.c_uint64), ("n_threads", C.c_int), ("layer_period", C.c_int), ("q4k_order", C.c_int),
        ("embd_f16", C.c_int)]


def synth_gguf(path: str, *, n_layers, d_model, ffn_hidden, n_heads, n_kv_heads, vocab, max_seq,
               theta_base=10000.0, rms_eps=1e-5, q4k=True, tied_output=False, seed=0,
               n_threads=0, layer_period=0, q4k_order=0, embd_f16=0) -> None:
    """slate_synth_llama_gguf from build/libslate_synth.so: the same bytes as
    slate_b200.synth_gguf for the same arguments."""
    if not os.path.exists(SYNTH_SO):
        build()
    lib = C.CDLL(SYNTH_SO)
    lib.slate_synth_llama_gguf.restype = C.c_int
    lib.slate_synth_llama_gguf.argtypes = [C.c_char_p, C.POINTER(SynthConfig)]
    cfg = SynthConfig(n_layers, d_model, ffn_hidden, n_heads, n_kv_heads, vocab, max_seq,
                      theta_base, rms_eps, int(q4k), int(tied_output), seed, n_threads,
                      layer_period, q4k_order, embd_f16)
    rc = lib.slate_synth_llama_gguf(path.encode(), C.byref(cfg))
    if rc:
        raise OSError(f"slate_synth_llama_gguf({path}) rc={rc}")


def _f(a):
    return np.ascontiguousarray(a, dtype=np.float32)


class OrcConfig(C.Structure):
    _fields_ = [(n, C.c_int) for n in ("n_layers", "d_model", "ffn_hidden", "n_heads",
                                       "n_kv_heads", "head_dim", "max_seq", "vocab")] + [
        ("theta_base", C.c_float), ("rms_eps", C.c_float), ("tied_output", C.c_int)]


class Oracle:
    """The C restatement (slate_oracle.c)."""

    def __init__(self):
        if not os.path.exists(ORACLE_SO):
            build()
        L = self.lib = C.CDLL(ORACLE_SO)
        for name, res, args in [
            ("orc_f16_to_f32", C.c_float, [C.c_uint16]),
            ("orc_dequant_q4k", None, [Pf, C.c_void_p, C.c_int64]),
            ("orc_dot_q4k", C.c_float, [C.c_void_p, Pf, C.c_int64]),
            ("orc_q4k_matvec", None, [Pf, C.c_void_p, Pf, C.c_int, C.c_int]),
            ("orc_matvec_f32", None, [Pf, Pf, Pf, C.c_int, C.c_int]),
            ("orc_linear_batch", None, [Pf, Pf, Pf, C.c_int, C.c_int, C.c_int]),
            ("orc_rmsnorm_row", None, [Pf, Pf, Pf, C.c_int, C.c_float]),
            ("orc_silu_mul", None, [Pf, Pf, Pf, C.c_int]),
            ("orc_rope_row", None, [Pf, C.c_int, C.c_int, C.c_int, C.c_float]),
            ("orc_rope_tables", None, [Pf, Pf, C.c_int, C.c_int, C.c_float]),
            ("orc_attention_gqa", None, [Pf, Pf, Pf, Pf, Pf, C.c_int, C.c_int, C.c_int, C.c_int]),
            ("orc_attention_step", None, [Pf, Pf, Pf, Pf, Pf, C.c_int, C.c_int]),
            ("orc_argmax", C.c_int, [Pf, C.c_int]),
            ("orc_model_open", C.c_void_p, [C.c_char_p]),
            ("orc_model_close", None, [C.c_void_p]),
            ("orc_model_config", C.POINTER(OrcConfig), [C.c_void_p]),
            ("orc_model_tensor", C.c_void_p, [C.c_void_p, C.c_char_p, Pi]),
            ("orc_session_new", C.c_void_p, [C.c_void_p, C.c_int]),
            ("orc_session_free", None, [C.c_void_p]),
            ("orc_session_position", C.c_int, [C.c_void_p]),
            ("orc_decode_step", C.c_int, [C.c_void_p, C.c_int32, Pf]),
            ("orc_session_seed_kv", C.c_int, [C.c_void_p, C.c_int, Pf, Pf]),
            ("orc_decode_many", C.c_int, [C.c_void_p, C.c_int, C.c_int, Pi, Pf, Pi, C.c_int]),
        ]:
            fn = getattr(L, name)
            fn.restype = res
            fn.argtypes = args

    # numerics primitives
    def dequant_q4k(self, blocks: np.ndarray, n: int) -> np.ndarray:
        out = np.zeros(n, dtype=np.float32)
        self.lib.orc_dequant_q4k(out.ctypes.data_as(Pf), blocks.ctypes.data, n)
        return out

    def dot_q4k(self, blocks, y) -> float:
        y = _f(y)
        return self.lib.orc_dot_q4k(blocks.ctypes.data, y.ctypes.data_as(Pf), y.size)

    def q4k_matvec(self, A, x, M, K):
        x = _f(x)
        y = np.zeros(M, dtype=np.float32)
        self.lib.orc_q4k_matvec(y.ctypes.data_as(Pf), A.ctypes.data, x.ctypes.data_as(Pf), M, K)
        return y

    def matvec_f32(self, A, x):
        A, x = _f(A), _f(x)
        y = np.zeros(A.shape[0], dtype=np.float32)
        self.lib.orc_matvec_f32(y.ctypes.data_as(Pf), A.ctypes.data_as(Pf), x.ctypes.data_as(Pf),
                                A.shape[0], A.shape[1])
        return y

    def rmsnorm(self, x, w, eps):
        x, w = _f(x), _f(w)
        y = np.zeros_like(x)
        self.lib.orc_rmsnorm_row(y.ctypes.data_as(Pf), x.ctypes.data_as(Pf), w.ctypes.data_as(Pf),
                                 x.size, eps)
        return y

    def silu_mul(self, g, u):
        g, u = _f(g), _f(u)
        y = np.zeros_like(g)
        self.lib.orc_silu_mul(y.ctypes.data_as(Pf), g.ctypes.data_as(Pf), u.ctypes.data_as(Pf), g.size)
        return y

    def rope(self, row, n_heads, hd, pos, theta):
        r = _f(row).copy()
        self.lib.orc_rope_row(r.ctypes.data_as(Pf), n_heads, hd, pos, theta)
        return r

    def rope_tables(self, max_seq, hd, theta):
        c = np.zeros((max_seq, hd // 2), np.float32)
        s = np.zeros_like(c)
        self.lib.orc_rope_tables(c.ctypes.data_as(Pf), s.ctypes.data_as(Pf), max_seq, hd, theta)
        return c, s

    def attention_gqa(self, q, K, V, nq, nkv, hd):
        q, K, V = _f(q), _f(K), _f(V)
        L = K.shape[0]
        out = np.zeros(nq * hd, dtype=np.float32)
        sc = np.zeros(L, dtype=np.float32)
        self.lib.orc_attention_gqa(out.ctypes.data_as(Pf), q.ctypes.data_as(Pf), K.ctypes.data_as(Pf),
                                   V.ctypes.data_as(Pf), sc.ctypes.data_as(Pf), L, nq, nkv, hd)
        return out

    def argmax(self, p) -> int:
        p = _f(p)
        return self.lib.orc_argmax(p.ctypes.data_as(Pf), p.size)

    # model
    def open(self, path: str) -> "OracleModel":
        return OracleModel(self, path)


class OracleModel:
    def __init__(self, o: Oracle, path: str):
        self.o = o
        self.h = o.lib.orc_model_open(path.encode())
        if not self.h:
            raise RuntimeError(f"oracle could not open {path}")
        c = o.lib.orc_model_config(self.h).contents
        self.cfg = {f: getattr(c, f) for f, _ in OrcConfig._fields_}

    def close(self):
        if self.h:
            self.o.lib.orc_model_close(self.h)
            self.h = None

    def tensor(self, name):
        dt = C.c_int32(0)
        p = self.o.lib.orc_model_tensor(self.h, name.encode(), C.byref(dt))
        return p, dt.value

    def session(self, max_seq=0):
        return OracleSession(self, max_seq)

    def decode_many(self, tokens: np.ndarray, want_logits=True, n_threads=0):
        """tokens [n_seq, n_steps] (teacher forced) -> (logits or None, greedy ids)."""
        tokens = np.ascontiguousarray(tokens, dtype=np.int32)
        n, t = tokens.shape
        V = self.cfg["vocab"]
        lg = np.zeros((n, t, V), dtype=np.float32) if want_logits else None
        ids = np.zeros((n, t), dtype=np.int32)
        nt = n_threads or os.cpu_count() or 1
        rc = self.o.lib.orc_decode_many(self.h, n, t, tokens.ctypes.data_as(Pi),
                                        lg.ctypes.data_as(Pf) if lg is not None else None,
                                        ids.ctypes.data_as(Pi), nt)
        if rc:
            raise RuntimeError(f"orc_decode_many rc={rc}")
        return lg, ids


class OracleSession:
    def __init__(self, m: OracleModel, max_seq=0):
        self.m = m
        self.h = m.o.lib.orc_session_new(m.h, max_seq)

    def decode(self, token):
        lg = np.zeros(self.m.cfg["vocab"], dtype=np.float32)
        rc = self.m.o.lib.orc_decode_step(self.h, int(token), lg.ctypes.data_as(Pf))
        return rc, lg

    def seed_kv(self, K, V):
        K, V = _f(K), _f(V)
        return self.m.o.lib.orc_session_seed_kv(self.h, K.shape[1], K.ctypes.data_as(Pf),
                                                V.ctypes.data_as(Pf))

    def position(self):
        return self.m.o.lib.orc_session_position(self.h)

    def close(self):
        if self.h:
            self.m.o.lib.orc_session_free(self.h)
            self.h = None

    def __del__(self):
        self.close()


class RefLlamaConfig(C.Structure):
    """slate_llama_config_t (include/slate/llama.h:53-65)."""
    _fields_ = [(n, C.c_int) for n in ("n_layers", "d_model", "ffn_hidden", "n_heads",
                                       "n_kv_heads", "head_dim", "max_seq", "vocab")] + [
        ("theta_base", C.c_float), ("rms_eps", C.c_float), ("tied_output", C.c_int)]


class RefSamplerConfig(C.Structure):
    """slate_sampler_config_t as include/slate/sampling.h:15-20 declares it."""
    _fields_ = [("temperature", C.c_float), ("top_k", C.c_int), ("top_p", C.c_float),
                ("seed", C.c_uint64)]


class Reference:
    """The reference library itself (unmodified sources, oracle/_ref)."""

    @staticmethod
    def available() -> bool:
        return os.path.exists(REF_SO)

    def __init__(self):
        if not self.available():
            raise FileNotFoundError(REF_SO)
        L = self.lib = C.CDLL(REF_SO)
        for name, res, args in [
            ("slate_gguf_open", C.c_void_p, [C.c_char_p]),
            ("slate_gguf_close", None, [C.c_void_p]),
            ("slate_llama_open", C.c_void_p, [C.c_void_p]),
            ("slate_llama_free", None, [C.c_void_p]),
            ("slate_llama_config", C.POINTER(RefLlamaConfig), [C.c_void_p]),
            ("slate_llama_session_new", C.c_void_p, [C.c_void_p]),
            ("slate_llama_session_free", None, [C.c_void_p]),
            ("slate_llama_session_position", C.c_int, [C.c_void_p]),
            ("slate_llama_prefill", C.c_int, [C.c_void_p, Pi, C.c_int, Pf]),
            ("slate_llama_decode_step", C.c_int, [C.c_void_p, C.c_int32, Pf]),
            ("slate_ref_session_set_position", C.c_int, [C.c_void_p, C.c_int]),
            ("slate_ref_session_seed_context", C.c_int, [C.c_void_p, C.c_int, C.c_uint64]),
            ("slate_dequant_q4_k", None, [Pf, C.c_void_p, C.c_int64]),
            ("slate_dot_q4_k_f32", C.c_float, [C.c_void_p, Pf, C.c_int64]),
            ("slate_q4_k_matvec", None, [Pf, C.c_void_p, Pf, C.c_int, C.c_int]),
            ("slate_backend_cpu", C.c_void_p, []),
            ("slate_backend_cuda", C.c_void_p, []),
            ("slate_backend_default", C.c_void_p, []),
            ("slate_sample_token", C.c_int,
             [Pf, C.c_int, C.POINTER(RefSamplerConfig), C.POINTER(C.c_uint64)]),
        ]:
            fn = getattr(L, name)
            fn.restype = res
            fn.argtypes = args

    def sample_token(self, logits, temperature, top_k, top_p, rng):
        """slate_sample_token (util/sampling.c:43-83) -> (token, next rng state)."""
        lg = np.ascontiguousarray(logits, dtype=np.float32)
        cfg = RefSamplerConfig(float(temperature), int(top_k), float(top_p), 0)
        st = C.c_uint64(int(rng))
        tok = self.lib.slate_sample_token(lg.ctypes.data_as(Pf), len(lg), C.byref(cfg), C.byref(st))
        return int(tok), int(st.value)

    def open(self, path: str):
        g = self.lib.slate_gguf_open(path.encode())
        if not g:
            raise RuntimeError(f"slate_gguf_open({path}) failed")
        m = self.lib.slate_llama_open(g)
        if not m:
            self.lib.slate_gguf_close(g)
            raise RuntimeError(f"slate_llama_open({path}) failed")
        return g, m

    def config(self, m) -> dict:
        c = self.lib.slate_llama_config(m).contents
        return {f: getattr(c, f) for f, _ in RefLlamaConfig._fields_}

    def close(self, g, m):
        self.lib.slate_llama_free(m)
        self.lib.slate_gguf_close(g)

    def session(self, m, context=0, seed=0):
        """A reference session (slate_llama_session_new) with a seeded
        `context`-token history (slate_ref_session_seed_context: the values the
        CUDA engine's seed_context writes for the same seed)."""
        s = self.lib.slate_llama_session_new(m)
        if not s:
            raise MemoryError("slate_llama_session_new failed")
        if context and self.lib.slate_ref_session_seed_context(s, int(context), int(seed)) != 0:
            self.lib.slate_llama_session_free(s)
            raise ValueError(f"context {context} does not fit the session")
        return s

    def decode(self, s, token, out):
        """slate_llama_decode_step into the f32 array `out` (vocab long)."""
        return self.lib.slate_llama_decode_step(s, int(token), out.ctypes.data_as(Pf))
