"""Pins the checkers and the Q4_K quantiser to the reference's golden vectors.

Fixtures in tests/golden/ were written by the reference's own generators
(tools/make_*.py, via tests/golden/make_golden.py).  The assertions restate
the reference's C tests:
  tests/test_q4k.c:28-77, tests/test_gguf_q4k.c:21-96, tests/test_rope.c:17-93,
  tests/test_llama_infer.c / _gqa.c / _q4k.c (Linf < 1e-3 vs numpy logits).
"""
import struct

import numpy as np
import pytest

from conftest import golden
from gguf_util import read_gguf


def lcg_floats(seed, n, shift, mask_bits, scale_fn):
    s = seed
    out = np.zeros(n, dtype=np.float32)
    for i in range(n):
        s = (s * 6364136223846793005 + 1442695040888963407) & (2**64 - 1)
        out[i] = scale_fn((s >> shift) & ((1 << mask_bits) - 1))
    return out


def load_q4k_block():
    raw = open(golden("slate_q4k_test.bin"), "rb").read()
    block = np.frombuffer(raw[:144], np.uint8).copy()
    orig = np.frombuffer(raw[144:144 + 1024], np.float32)
    recon = np.frombuffer(raw[1168:2192], np.float32)
    return block, orig, recon


def test_q4k_block_dequant_bit_exact(oracle):
    """test_q4k.c [1]-[3]."""
    block, orig, recon = load_q4k_block()
    out = oracle.dequant_q4k(block, 256)
    assert np.array_equal(out, recon)                        # spec conformance, exact
    assert np.abs(out - orig).mean() < 0.05                  # quantisation budget
    y = lcg_floats(0xBEEF, 256, 11, 24, lambda v: (np.float32(v) / np.float32(1 << 24) - np.float32(0.5)) * np.float32(2))
    ref = float(np.dot(out.astype(np.float64), y.astype(np.float64)))
    assert abs(oracle.dot_q4k(block, y) - ref) / (abs(ref) + 1e-9) < 1e-5


def test_q4k_gguf_dequant_and_matvec(oracle):
    """test_gguf_q4k.c: GGUF tensor -> dequant (0 diff), dot, 16x256 matvec."""
    kv, t = read_gguf(golden("slate_q4k.gguf"))
    ty, dims, data = t["weight"]
    assert ty == 12 and dims == [256, 16]
    expected = np.fromfile(golden("slate_q4k_expected.f32"), np.float32)
    deq = oracle.dequant_q4k(data, 16 * 256)
    assert np.array_equal(deq, expected)
    y = lcg_floats(0xC0FFEE, 4096, 24, 16, lambda v: np.float32(v) / np.float32(65536) - np.float32(0.5))
    ref = float(np.dot(deq.astype(np.float64), y.astype(np.float64)))
    assert abs(oracle.dot_q4k(data, y) - ref) / (abs(ref) + 1e-9) < 1e-5
    x = lcg_floats(0xABCD, 256, 24, 16, lambda v: np.float32(v) / np.float32(65536) - np.float32(0.5))
    yv = oracle.q4k_matvec(data, x, 16, 256)
    yr = deq.reshape(16, 256).astype(np.float64) @ x.astype(np.float64)
    assert np.max(np.abs(yv - yr) / (np.abs(yr) + 1e-9)) < 1e-4


def test_rope_golden(oracle):
    """test_rope.c: GGML non-interleaved rotation at positions 7..11."""
    raw = open(golden("slate_rope_ref.bin"), "rb").read()
    B, T, H, hd = struct.unpack_from("<iiii", raw, 0)
    theta = struct.unpack_from("<f", raw, 16)[0]
    n = B * T * H * hd
    x = np.frombuffer(raw, np.float32, n, 20).reshape(B, T, H * hd)
    pos = np.frombuffer(raw, np.int32, T, 20 + 4 * n)
    y = np.frombuffer(raw, np.float32, n, 20 + 4 * n + 4 * T).reshape(B, T, H * hd)
    for b in range(B):
        for t in range(T):
            got = oracle.rope(x[b, t], H, hd, int(pos[t]), theta)
            assert np.max(np.abs(got - y[b, t])) < 1e-5


def read_ref_logits(name):
    raw = open(golden(name), "rb").read()
    n = struct.unpack_from("<i", raw, 0)[0]
    prompt = np.frombuffer(raw, np.int32, n, 4)
    V = struct.unpack_from("<i", raw, 4 + 4 * n)[0]
    logits = np.frombuffer(raw, np.float32, V, 8 + 4 * n)
    return prompt, logits


TINY = [("slate_tiny_llama.gguf", "slate_llama_ref.bin"),
        ("slate_tiny_llama_gqa.gguf", "slate_tiny_llama_gqa_ref.bin"),
        ("slate_tiny_llama_q4k.gguf", "slate_tiny_llama_q4k_ref.bin")]


@pytest.mark.parametrize("gguf,ref", TINY)
def test_oracle_prefill_matches_numpy_reference(oracle, gguf, ref):
    """test_llama_infer{,_gqa,_q4k}.c: last-position logits Linf < 1e-3."""
    prompt, want = read_ref_logits(ref)
    m = oracle.open(golden(gguf))
    s = m.session()
    for tok in prompt:
        rc, lg = s.decode(tok)
        assert rc == 0
    assert np.max(np.abs(lg - want)) < 1e-3
    s.close()
    m.close()


@pytest.mark.parametrize("gguf,ref", TINY)
def test_reference_prefill_matches_numpy_reference(reference, gguf, ref):
    """The reference library itself reproduces its own fixture (sanity of _ref)."""
    import ctypes as C
    prompt, want = read_ref_logits(ref)
    g, m = reference.open(golden(gguf))
    s = reference.lib.slate_llama_session_new(m)
    out = np.zeros(len(want), np.float32)
    p = np.ascontiguousarray(prompt)
    rc = reference.lib.slate_llama_prefill(s, p.ctypes.data_as(C.POINTER(C.c_int32)), len(p),
                                           out.ctypes.data_as(C.POINTER(C.c_float)))
    assert rc == 0
    assert np.max(np.abs(out - want)) < 1e-3
    reference.lib.slate_llama_session_free(s)
    reference.close(g, m)


# ---- the product quantiser reproduces the reference generators' bytes ----------

def test_quantizer_reproduces_single_block(sb):
    block, orig, _ = load_q4k_block()
    assert np.array_equal(sb.quantize_q4k(orig.reshape(1, 256)).reshape(-1), block)


def test_quantizer_reproduces_gguf_tensor(sb):
    """tools/make_q4k_gguf.py: np.random.seed(42); normal(0, 0.5, (16, 256))."""
    np.random.seed(42)
    w = np.random.normal(0, 0.5, (16, 256)).astype(np.float32)
    _, t = read_gguf(golden("slate_q4k.gguf"))
    assert np.array_equal(sb.quantize_q4k(w).reshape(-1), t["weight"][2])


def test_quantizer_reproduces_tiny_llama_q4k(sb):
    """tools/make_tiny_llama_q4k_gguf.py:104-130 weight stream, every Q4_K tensor."""
    rng = np.random.default_rng(0xCAFE)
    D, H, FFN, V, L = 256, 4, 512, 64, 2

    def w(shape):
        return rng.normal(0, 0.02, shape).astype(np.float32)

    w((V, D)); w((V, D))                      # token_embd, output (f32)
    _, t = read_gguf(golden("slate_tiny_llama_q4k.gguf"))
    for i in range(L):
        for name, shape in [("attn_q", (D, D)), ("attn_k", (D, D)), ("attn_v", (D, D)),
                            ("attn_output", (D, D)), ("ffn_gate", (FFN, D)), ("ffn_up", (FFN, D)),
                            ("ffn_down", (D, FFN))]:
            q = sb.quantize_q4k(w(shape))
            ty, _, data = t[f"blk.{i}.{name}.weight"]
            assert ty == 12 and np.array_equal(q.reshape(-1), data), (i, name)
