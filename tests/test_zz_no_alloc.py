"""slate_cuda_attention_paged_gqa_noalloc: the attention entry point whose
scratch is a fixed device array instead of cudaMallocAsync.  Its output must
match the vtable's attention_paged_gqa on the same inputs (1e-5 of scale, the
attention tolerance of test_gpu_kernels), on two calls in a row that share
the array, for the tensor-core (f16) and CUDA-core (f32) kernels.  Collected
last so it also runs after every other test in one process."""
import ctypes as C

import numpy as np
import pytest

from gpu_util import Backend, scale_err


def paged_case(rng, ctxs, nkv, hd, kv_dtype, layers=2, layer=1):
    max_pages = max((c + 15) // 16 for c in ctxs) + 1
    n_pages = sum((c + 15) // 16 for c in ctxs) + 4
    perm = rng.permutation(n_pages)
    table = -np.ones((len(ctxs), max_pages), np.int32)
    k = 0
    for r, c in enumerate(ctxs):
        for pg in range((c + 15) // 16):
            table[r, pg] = perm[k]
            k += 1
    et = np.float16 if kv_dtype == 1 else np.float32
    pool = rng.uniform(-1, 1, (layers, n_pages, 2, nkv, 16, hd)).astype(et)
    pos = np.array([c - 1 for c in ctxs], np.int32)
    return pool, table, pos, max_pages, n_pages, layer


@pytest.fixture(scope="module")
def be(sb):
    b = Backend(sb)
    yield b
    b.free_all()


@pytest.mark.gpu
@pytest.mark.parametrize("kv_dtype", [1, 0])
def test_noalloc_matches_vtable_on_two_calls(sb, be, kv_dtype):
    nq, nkv, hd = 32, 8, 128
    noalloc = sb.F["slate_cuda_attention_paged_gqa_noalloc"]
    rng = np.random.default_rng(5 + kv_dtype)
    # the second call is smaller than the first: nothing of the first call's
    # partials may leak into it
    for call, ctxs in enumerate(([1, 17, 600, 2100, 4000], [3, 513])):
        pool, table, pos, max_pages, n_pages, layer = paged_case(rng, ctxs, nkv, hd, kv_dtype)
        B = len(ctxs)
        q = rng.normal(0, 1, (B, nq * hd)).astype(np.float32)
        d_q, d_pos, d_pool, d_table = be.dev(q), be.dev(pos), be.dev(pool), be.dev(table)
        d_slots = be.dev(np.arange(B, dtype=np.int32))
        want_d = be.empty(B * nq * hd * 4)
        rc = be.attention_paged_gqa(want_d, d_q, d_pos, d_slots, d_table, max_pages, d_pool, n_pages,
                                    layer, B, nq, nkv, hd, kv_dtype)
        assert rc == 0, sb.last_error()
        want = be.host(want_d, (B, nq * hd))
        got_d = be.empty(B * nq * hd * 4)
        be.fn["sync"]()                      # inputs were uploaded on the vtable's stream
        rc = noalloc(got_d, d_q, d_pos, d_slots, d_table, max_pages, d_pool, n_pages, layer, B, nq,
                     nkv, hd, kv_dtype, None)
        assert rc == 0, sb.last_error()
        got = be.host(got_d, (B, nq * hd))
        assert np.isfinite(got).all()
        err = scale_err(got, want)
        assert err < 1e-5, (call, err)


def test_noalloc_rejects_oversized_request(sb):
    """Beyond the fixed scratch the call fails with -1 and says why, before any
    device work (so this runs without a GPU)."""
    noalloc = sb.F["slate_cuda_attention_paged_gqa_noalloc"]
    dummy = C.c_void_p(256)             # never dereferenced: the size check comes first
    # 1024 rows x 32 heads x 5 chunks of 1024 tokens (4352-token cap) x 130 floats > 2^21
    rc = noalloc(dummy, dummy, dummy, dummy, dummy, 272, dummy, 1000, 0, 1024, 32, 8, 128, 1, None)
    assert rc == -1
    assert "limit" in sb.last_error()
