"""Stochastic sampling with the reference sampler's semantics
(src/util/sampling.c:9-83): the device sampler (slate_cuda_sample_rows and the
engine's sampling step) against the reference library's slate_sample_token on
the same logits and RNG states -- tokens and next states must be identical."""
import ctypes as C

import numpy as np
import pytest

from gpu_util import Backend


def test_reference_sampler_own_test(reference):
    """tests/test_sampling.c on the checker: greedy and top_k=1 always take the
    dominant token; T=1 draws follow the softmax (token 1 most frequent)."""
    logits = np.array([0.1, 2.5, 0.2, -1.0], np.float32)
    rng = 0xC0FFEE
    for _ in range(10):
        t, rng = reference.sample_token(logits, 0.0, 0, 0.0, rng)
        assert t == 1
    counts = np.zeros(4, int)
    for _ in range(10000):
        t, rng = reference.sample_token(logits, 1.0, 0, 0.0, rng)
        counts[t] += 1
    assert counts[1] == counts.max()
    p = np.exp(logits - logits.max())
    p /= p.sum()
    assert np.allclose(counts / 10000, p, atol=0.02)
    for _ in range(100):
        t, rng = reference.sample_token(logits, 1.0, 1, 0.0, rng)
        assert t == 1


CASES = [  # (temperature, top_k, top_p)
    (0.0, 0, 0.0), (1.0, 0, 0.0), (0.7, 0, 0.9), (1.0, 40, 0.0), (0.8, 40, 0.95),
    (1.5, 1, 0.0), (1.0, 7, 0.5), (2.0, 1000, 0.9), (1.0, 2048, 0.0), (1.0, 10 ** 6, 0.0),
    (0.3, 5, 1.0),
]


def make_logits(rng, B, V, kind):
    if kind == "normal":
        return rng.normal(0, 3, (B, V)).astype(np.float32)
    if kind == "peaked":
        L = rng.normal(0, 1, (B, V)).astype(np.float32)
        L[np.arange(B), rng.integers(0, V, B)] += 12
        return L
    # ties: values on a coarse grid, many equal probabilities
    return (rng.integers(-4, 5, (B, V)) * 0.5).astype(np.float32)


@pytest.mark.gpu
@pytest.mark.parametrize("V", [5000, 128256])
@pytest.mark.parametrize("kind", ["normal", "peaked", "ties"])
def test_device_sampler_matches_reference(sb, reference, V, kind):
    be = Backend(sb)
    rng = np.random.default_rng(V + len(kind))
    B = len(CASES) * 3
    L = make_logits(rng, B, V, kind)
    d = be.dev(L)
    cfg = sb.sampler_configs(B, [c[0] for c in CASES] * 3, [c[1] for c in CASES] * 3,
                             [c[2] for c in CASES] * 3)
    state = rng.integers(1, 2 ** 63, B, dtype=np.uint64)
    for rnd in range(3):                      # states carry over between rounds
        want, want_state = [], []
        for r in range(B):
            c = cfg[r]
            t, s2 = reference.sample_token(L[r], c.temperature, c.top_k, c.top_p, int(state[r]))
            want.append(t)
            want_state.append(s2)
        rc, got = sb.sample_rows(d, V, B, V, cfg, state)
        assert rc == 0, sb.last_error()
        assert list(got) == want, (rnd, [(r, CASES[r % len(CASES)], got[r], want[r])
                                         for r in range(B) if got[r] != want[r]][:5])
        assert [int(x) for x in state] == want_state
    be.free_all()


@pytest.mark.gpu
def test_engine_sampling_step(sb, reference, workdir):
    """The engine's sampling step draws what the reference sampler draws from
    the same step's logits; temperature-0 rows equal the greedy step."""
    import os
    path = os.path.join(str(workdir), "sample_q4k.gguf")
    if not os.path.exists(path):
        sb.synth_gguf(path, n_layers=2, d_model=512, ffn_hidden=1024, n_heads=8, n_kv_heads=4,
                      vocab=3000, max_seq=64, q4k=True, seed=13)
    rng = np.random.default_rng(3)
    n = 24
    a = sb.LlamaBatch(path, max_batch=n)
    g = sb.LlamaBatch(path, max_batch=n)
    sa = [a.open() for _ in range(n)]
    sg = [g.open() for _ in range(n)]
    temps = np.where(np.arange(n) % 4 == 0, 0.0, 0.9)
    cfg = sb.sampler_configs(n, temps, np.where(np.arange(n) % 3 == 0, 0, 50), 0.9)
    state = rng.integers(1, 2 ** 63, n, dtype=np.uint64)
    toks = rng.integers(0, 3000, n).astype(np.int32)
    for t in range(5):
        before = state.copy()
        rc, out, lg = a.step_sample(sa, toks, cfg, state, want_logits=True)
        assert rc == 0, sb.last_error()
        rcg, outg, _ = g.step(sg, toks)
        assert rcg == 0
        for r in range(n):
            c = cfg[r]
            want, s2 = reference.sample_token(lg[r], c.temperature, c.top_k, c.top_p, int(before[r]))
            assert out[r] == want, (t, r)
            assert int(state[r]) == s2
            if temps[r] == 0:
                assert out[r] == outg[r]
        toks = out.copy()
        # keep the greedy engine on the same sequence
        toks_g = out.copy()
        assert np.array_equal(toks, toks_g)
    a.close()
    g.close()
