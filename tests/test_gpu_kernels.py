"""Kernel conformance through the C-ABI vtable (slate_backend_cuda_create):
the reference's own backend contract (tests/test_backend.c:31-187, same inputs
and tolerances) plus the appended batched Q4_K / paged-attention entries,
each against the oracle."""
import numpy as np
import pytest

from conftest import golden
from gguf_util import read_gguf
from gpu_util import Backend, scale_err

pytestmark = pytest.mark.gpu


@pytest.fixture(scope="module")
def be(sb):
    b = Backend(sb)
    yield b
    b.free_all()


def test_backend_identity(be):
    assert be.name == "cuda"


def test_backend_c_contract(be, oracle):
    """tests/test_backend.c, case by case, with its tolerances."""
    # mem round trip (odd size)
    src = (np.arange(137, dtype=np.float32) * 0.5 - 12.0)
    assert np.array_equal(be.host(be.dev(src), 137), src)
    # matvec M=7 K=11, tol 1e-4
    A = np.array([((i * 13 + 5) % 17) * 0.05 - 0.4 for i in range(77)], np.float32).reshape(7, 11)
    x = np.array([k * 0.1 - 0.5 for k in range(11)], np.float32)
    y = be.empty(7 * 4)
    be.matvec(y, be.dev(A), be.dev(x), 7, 11)
    assert np.max(np.abs(be.host(y, 7) - A.astype(np.float64) @ x)) < 1e-4
    # linear_batch B=4 K=8 N=6, tol 1e-4
    X = np.array([((i * 7) % 13) * 0.1 - 0.6 for i in range(32)], np.float32).reshape(4, 8)
    W = np.array([((i * 5) % 11) * 0.08 - 0.4 for i in range(48)], np.float32).reshape(8, 6)
    Cd = be.empty(24 * 4)
    be.linear_batch(Cd, be.dev(X), be.dev(W), 4, 8, 6)
    assert np.max(np.abs(be.host(Cd, (4, 6)) - X.astype(np.float64) @ W)) < 1e-4
    # rmsnorm D=16, tol 1e-5
    x = np.array([(i - 8) * 0.3 for i in range(16)], np.float32)
    w = np.array([0.5 + i * 0.05 for i in range(16)], np.float32)
    yd = be.empty(64)
    be.rmsnorm_row(yd, be.dev(x), be.dev(w), 16, 1e-5)
    assert np.max(np.abs(be.host(yd, 16) - oracle.rmsnorm(x, w, 1e-5))) < 1e-5
    # silu_mul H=24, tol 1e-5
    g = np.array([(i - 12) * 0.4 for i in range(24)], np.float32)
    u = np.array([(i + 1) * 0.1 for i in range(24)], np.float32)
    yd = be.empty(96)
    be.silu_mul(yd, be.dev(g), be.dev(u), 24)
    assert np.max(np.abs(be.host(yd, 24) - oracle.silu_mul(g, u))) < 1e-5
    # add_inplace D=32, exact
    y0 = np.arange(32, dtype=np.float32) * 0.1
    xa = (np.arange(32, dtype=np.float32) - 16) * 0.2
    yd = be.dev(y0)
    be.add_inplace(yd, be.dev(xa), 32)
    assert np.array_equal(be.host(yd, 32), y0 + xa)
    # embed_lookup V=5 D=8 token 3, exact
    Wt = np.arange(40, dtype=np.float32)
    yd = be.empty(32)
    be.embed_lookup(yd, be.dev(Wt), 3, 8)
    assert np.array_equal(be.host(yd, 8), Wt[24:32])
    # attention_step L=5 D=16, tol 1e-5
    q = np.array([(i - 8) * 0.1 for i in range(16)], np.float32)
    K = np.array([((i * 7) % 13) * 0.05 for i in range(80)], np.float32).reshape(5, 16)
    V = np.array([((i * 5) % 11) * 0.07 for i in range(80)], np.float32).reshape(5, 16)
    od = be.empty(64)
    be.attention_step(od, be.dev(q), be.dev(K), be.dev(V), be.empty(20), 5, 16)
    s = (K.astype(np.float64) @ q) / 4.0
    p = np.exp(s - s.max()); p /= p.sum()
    assert np.max(np.abs(be.host(od, 16) - p @ V)) < 1e-5
    be.sync()


def test_matvec_q4k_golden(be, oracle):
    _, t = read_gguf(golden("slate_q4k.gguf"))
    data = t["weight"][2]
    x = np.random.default_rng(0).uniform(-0.5, 0.5, 256).astype(np.float32)
    yd = be.empty(64)
    be.matvec_q4k(yd, be.dev(data), be.dev(x), 16, 256)
    assert scale_err(be.host(yd, 16), oracle.q4k_matvec(data, x, 16, 256)) < 1e-5


@pytest.mark.parametrize("B,M,K", [(1, 256, 256), (3, 384, 512), (8, 1000, 1024), (9, 1024, 2048),
                                   (64, 768, 1024), (65, 640, 512), (200, 1280, 4096)])
def test_matmul_q4k_batch(be, oracle, sb, B, M, K):
    """GEMV (B <= 8) and tiled (BN 64 / 128) paths, ragged M, vs the oracle."""
    rng = np.random.default_rng(B * 1000 + M)
    q = sb.quantize_q4k(rng.normal(0, 0.02, (M, K)).astype(np.float32))
    X = rng.normal(0, 1, (B, K)).astype(np.float32)
    Y = be.empty(B * M * 4)
    assert be.matmul_q4k_batch(Y, be.dev(q), be.dev(X), B, M, K) == 0
    got = be.host(Y, (B, M))
    want = np.stack([oracle.q4k_matvec(q, X[b], M, K) for b in range(B)])
    assert scale_err(got, want) < 1e-5


@pytest.mark.parametrize("B,M,K", [(1, 300, 256), (5, 130, 384), (40, 256, 512), (2, 33, 100)])
def test_matmul_f32_batch(be, B, M, K):
    rng = np.random.default_rng(K)
    A = rng.normal(0, 0.02, (M, K)).astype(np.float32)
    X = rng.normal(0, 1, (B, K)).astype(np.float32)
    Y = be.empty(B * M * 4)
    assert be.matmul_f32_batch(Y, be.dev(A), be.dev(X), B, M, K) == 0
    assert scale_err(be.host(Y, (B, M)), X.astype(np.float64) @ A.T.astype(np.float64)) < 1e-5


def test_rmsnorm_rows(be, oracle):
    rng = np.random.default_rng(5)
    X = rng.normal(0, 2, (7, 4096)).astype(np.float32)
    w = rng.uniform(0.5, 1.5, 4096).astype(np.float32)
    Y = be.empty(X.nbytes)
    assert be.rmsnorm_rows(Y, be.dev(X), be.dev(w), 7, 4096, 1e-5) == 0
    got = be.host(Y, X.shape)
    for b in range(7):
        assert scale_err(got[b], oracle.rmsnorm(X[b], w, 1e-5)) < 1e-6


def test_argmax_rows_first_max(be, oracle):
    """util/sampling.c:14-18: the first index of the maximum wins ties."""
    rng = np.random.default_rng(9)
    L = rng.normal(0, 1, (6, 128256)).astype(np.float32)
    L[1, 77] = L[1, 99999] = 50.0          # tie: lowest index
    L[2, :] = 1.0                           # all equal -> 0
    L[3, -1] = 9.0                          # last element
    L[4, 0] = 9.0
    L[5, 1000:1003] = 7.0
    out = be.empty(6 * 4)
    assert be.argmax_rows(out, be.dev(L), 6, L.shape[1]) == 0
    got = be.host(out, 6, np.int32)
    assert list(got) == [oracle.argmax(r) for r in L]
    assert got[1] == 77 and got[2] == 0


def build_paged(rng, ctxs, L_layers, nkv, hd, n_pages, kv_dtype, layer):
    """Random K/V history in a shuffled page pool; returns pool array, page table
    and the dense per-row [ctx, nkv*hd] K/V that the oracle reads."""
    max_pages = max((c + 15) // 16 for c in ctxs) + 1
    perm = rng.permutation(n_pages)
    table = -np.ones((len(ctxs), max_pages), np.int32)
    k = 0
    for r, c in enumerate(ctxs):
        for pg in range((c + 15) // 16):
            table[r, pg] = perm[k]
            k += 1
    et = np.float16 if kv_dtype == 1 else np.float32
    pool = rng.uniform(-1, 1, (L_layers, n_pages, 2, nkv, 16, hd)).astype(et)
    dense = []
    for r, c in enumerate(ctxs):
        Kd = np.zeros((c, nkv * hd), np.float32)
        Vd = np.zeros((c, nkv * hd), np.float32)
        for t in range(c):
            pg, o = table[r, t // 16], t % 16
            Kd[t] = pool[layer, pg, 0, :, o, :].astype(np.float32).reshape(-1)
            Vd[t] = pool[layer, pg, 1, :, o, :].astype(np.float32).reshape(-1)
        dense.append((Kd, Vd))
    return pool, table, dense, max_pages


@pytest.mark.parametrize("nq,nkv,hd", [(8, 2, 64), (32, 8, 128), (4, 2, 16), (8, 8, 32), (64, 8, 128), (8, 2, 8)])
@pytest.mark.parametrize("kv_dtype", [0, 1])
def test_rope_append_and_paged_attention(be, oracle, nq, nkv, hd, kv_dtype):
    rng = np.random.default_rng(nq * 7 + hd + kv_dtype)
    ctxs = [1, 15, 16, 17, 300, 600]       # positions = ctx - 1 (token appended at pos)
    B, layers, layer, n_pages, theta = len(ctxs), 3, 1, 128, 500000.0
    pool, table, dense, max_pages = build_paged(rng, ctxs, layers, nkv, hd, n_pages, kv_dtype, layer)
    pos = np.array([c - 1 for c in ctxs], np.int32)
    slots = np.arange(B, dtype=np.int32)
    q = rng.normal(0, 1, (B, nq * hd)).astype(np.float32)
    kk = rng.normal(0, 1, (B, nkv * hd)).astype(np.float32)
    vv = rng.normal(0, 1, (B, nkv * hd)).astype(np.float32)
    cs, sn = oracle.rope_tables(1024, hd, theta)      # the engine builds the same tables
    d_pool, d_table = be.dev(pool), be.dev(table)
    d_q, d_k = be.dev(q), be.dev(kk)
    d_pos, d_slots = be.dev(pos), be.dev(slots)
    rc = be.rope_kv_append_paged(d_q, d_k, be.dev(vv), d_pos, d_slots, d_table, max_pages, d_pool,
                                 n_pages, layer, B, nq, nkv, hd, kv_dtype, be.dev(cs), be.dev(sn))
    assert rc == 0
    q_rot = be.host(d_q, q.shape)
    pool_after = be.host(d_pool, pool.shape, pool.dtype)
    out = be.empty(B * nq * hd * 4)
    rc = be.attention_paged_gqa(out, d_q, d_pos, d_slots, d_table, max_pages, d_pool, n_pages, layer,
                                B, nq, nkv, hd, kv_dtype)
    assert rc == 0
    got = be.host(out, (B, nq * hd))
    for r, c in enumerate(ctxs):
        want_q = oracle.rope(q[r], nq, hd, int(pos[r]), theta)
        assert scale_err(q_rot[r], want_q) < 1e-5
        want_k = oracle.rope(kk[r], nkv, hd, int(pos[r]), theta)
        pg, o = table[r, pos[r] // 16], pos[r] % 16
        app_k = pool_after[layer, pg, 0, :, o, :].astype(np.float32).reshape(-1)
        app_v = pool_after[layer, pg, 1, :, o, :].astype(np.float32).reshape(-1)
        et = np.float16 if kv_dtype else np.float32
        # f16 cache: one rounding of the rotated value (<= 2^-11 relative)
        assert scale_err(app_k, want_k) < (6e-4 if kv_dtype else 1e-5)
        assert np.array_equal(app_v, vv[r].astype(et).astype(np.float32))
        Kd, Vd = dense[r]
        Kd[c - 1], Vd[c - 1] = app_k, app_v
        want = oracle.attention_gqa(q_rot[r], Kd, Vd, nq, nkv, hd)
        assert scale_err(got[r], want) < 1e-5, (r, c)
    # other layers untouched
    other = [l for l in range(layers) if l != layer]
    assert np.array_equal(pool_after[other], pool[other])


@pytest.mark.parametrize("passes,tol", [(3, 1e-5), (1, 3e-3)])
@pytest.mark.parametrize("B,M,K", [(16, 128, 256), (40, 384, 1024), (256, 1024, 4096),
                                   (100, 256, 14336), (300, 256, 512)])
def test_matmul_q4k_tensor_cores(be, oracle, sb, B, M, K, passes, tol):
    """tcgen05 path: 3-pass hi/lo split reproduces f32 products; the single
    f16 pass stays within f16 operand rounding.  Reference = the oracle's exact
    Q4_K dequantisation, products in float64."""
    rng = np.random.default_rng(B + M + K + passes)
    q = sb.quantize_q4k(rng.normal(0, 0.02, (M, K)).astype(np.float32))
    X = rng.normal(0, 1, (B, K)).astype(np.float32)
    Y = be.empty(B * M * 4)
    rc = be.matmul_q4k_batch_tc(Y, be.dev(q), be.dev(X), B, M, K, passes)
    assert rc == 0, be.sb.last_error()
    got = be.host(Y, (B, M))
    Wd = oracle.dequant_q4k(q, M * K).reshape(M, K).astype(np.float64)
    want = X.astype(np.float64) @ Wd.T
    assert scale_err(got, want) < tol


@pytest.mark.parametrize("B,M,K", [(1, 128, 256), (5, 256, 1024), (16, 128, 256), (130, 384, 4096),
                                   (256, 1024, 4096), (256, 6144, 4096), (100, 256, 14336),
                                   (300, 256, 512), (513, 512, 2048)])
@pytest.mark.parametrize("one_sm", ["0", "1"])
def test_matmul_q4k_exact_weights(be, oracle, sb, monkeypatch, B, M, K, one_sm):
    """passes=2: f16(sc*q) weights are exact, x enters as f16 hi + lo, the
    d / dmin block scales are applied per super-block in f32 -- f32-level
    products like the 3-pass split, over a stream-K schedule whose shared tiles
    are summed by the last CTA to finish (shapes with 1..5 tiles per SM and
    partial row tiles).  Weights with M % 256 == 0 run on CTA pairs unless
    SLATE_Q4_ONE_SM=1 keeps them on single CTAs."""
    monkeypatch.setenv("SLATE_Q4_ONE_SM", one_sm)
    rng = np.random.default_rng(B * 7 + M + K)
    q = sb.quantize_q4k(rng.normal(0, 0.02, (M, K)).astype(np.float32))
    X = rng.normal(0, 1, (B, K)).astype(np.float32)
    Y = be.empty(B * M * 4)
    for rep in range(2):                      # counters must be left at zero
        rc = be.matmul_q4k_batch_tc(Y, be.dev(q), be.dev(X), B, M, K, 2)
        assert rc == 0, be.sb.last_error()
        got = be.host(Y, (B, M))
        Wd = oracle.dequant_q4k(q, M * K).reshape(M, K).astype(np.float64)
        want = X.astype(np.float64) @ Wd.T
        assert scale_err(got, want) < 1e-5, rep


@pytest.mark.parametrize("B,M,K", [(16, 128, 256), (40, 384, 1024), (130, 384, 4096),
                                   (256, 1024, 4096), (256, 6144, 4096), (100, 256, 14336),
                                   (300, 256, 512), (513, 512, 2048)])
def test_matmul_q4k_streamk(be, oracle, sb, monkeypatch, B, M, K):
    """passes=3 on the stream-K kernel (SLATE_TC_SK=1): Q4_K dequantised into
    tensor memory as f16 hi + lo, x as f16 hi + lo, three MMA passes; the
    (tile, K step) space split evenly over one CTA per SM, shared tiles summed
    by the last CTA to finish (shapes with fewer units than SMs, 1..5 tiles per
    SM, and partial row tiles).  Two calls: the tile counters must be left at
    zero."""
    monkeypatch.setenv("SLATE_TC_SK", "1")
    rng = np.random.default_rng(B * 11 + M + K)
    q = sb.quantize_q4k(rng.normal(0, 0.02, (M, K)).astype(np.float32))
    X = rng.normal(0, 1, (B, K)).astype(np.float32)
    Y = be.empty(B * M * 4)
    Wd = oracle.dequant_q4k(q, M * K).reshape(M, K).astype(np.float64)
    want = X.astype(np.float64) @ Wd.T
    for rep in range(2):
        rc = be.matmul_q4k_batch_tc(Y, be.dev(q), be.dev(X), B, M, K, 3)
        assert rc == 0, be.sb.last_error()
        got = be.host(Y, (B, M))
        assert scale_err(got, want) < 1e-5, rep


@pytest.mark.parametrize("B", [1, 3, 8, 9, 16])
@pytest.mark.parametrize("M,K", [(128, 256), (384, 1024), (6144, 4096), (4096, 4096),
                                 (256, 14336), (28672, 4096)])
def test_matmul_q4k_small_batch(be, oracle, sb, B, M, K):
    """passes=4, the small-batch kernel: the quants q enter the mma.sync
    tensor cores exactly, x as f16 hi + lo after a power-of-two scale per row
    and K chunk, and each sub-block's sum(q*x) is scaled by d*sc with
    dmin*m*sum(x) subtracted in f32.  Shapes with one K chunk and with up to 16
    chunks summed by the last CTA of a row block; two calls (the row-block
    counters must be left at zero)."""
    rng = np.random.default_rng(B * 13 + M + K)
    q = sb.quantize_q4k(rng.normal(0, 0.02, (M, K)).astype(np.float32))
    X = rng.normal(0, 1, (B, K)).astype(np.float32)
    Y = be.empty(B * M * 4)
    Wd = oracle.dequant_q4k(q, M * K).reshape(M, K).astype(np.float64)
    want = X.astype(np.float64) @ Wd.T
    for rep in range(2):
        rc = be.matmul_q4k_batch_tc(Y, be.dev(q), be.dev(X), B, M, K, 4)
        assert rc == 0, be.sb.last_error()
        got = be.host(Y, (B, M))
        assert scale_err(got, want) < 1e-5, rep


def test_matmul_q4k_small_batch_magnitudes(be, oracle, sb):
    """Rows of very different size (1e-4 .. 1e4, one all-zero row) keep f32-level
    accuracy each: the hi/lo split happens after each row's own power-of-two
    scale, so small activations do not fall into f16 subnormals."""
    M, K, B = 512, 2048, 6
    rng = np.random.default_rng(77)
    q = sb.quantize_q4k(rng.normal(0, 0.02, (M, K)).astype(np.float32))
    X = rng.normal(0, 1, (B, K)).astype(np.float32)
    X *= np.array([1e-4, 1e-2, 1.0, 1e2, 1e4, 0.0], np.float32)[:, None]
    Y = be.empty(B * M * 4)
    rc = be.matmul_q4k_batch_tc(Y, be.dev(q), be.dev(X), B, M, K, 4)
    assert rc == 0, be.sb.last_error()
    got = be.host(Y, (B, M))
    Wd = oracle.dequant_q4k(q, M * K).reshape(M, K).astype(np.float64)
    want = X.astype(np.float64) @ Wd.T
    for r in range(B - 1):
        assert scale_err(got[r], want[r]) < 1e-5, r
    assert not got[B - 1].any()


def run_attention(be, monkeypatch, path, q, pool, table, pos, nq, nkv, hd, kv_dtype, layer, n_pages):
    """attention_paged_gqa with the kernel picked by SLATE_CUDA_ATTN_PATH
    ("0": tensor cores where the f16 shape allows, "1": CUDA cores)."""
    monkeypatch.setenv("SLATE_CUDA_ATTN_PATH", path)
    B = q.shape[0]
    out = be.empty(B * nq * hd * 4)
    rc = be.attention_paged_gqa(out, be.dev(q), be.dev(pos), be.dev(np.arange(B, dtype=np.int32)),
                                be.dev(table), table.shape[1], be.dev(pool), n_pages, layer, B, nq,
                                nkv, hd, kv_dtype)
    assert rc == 0, be.sb.last_error()
    return be.host(out, (B, nq * hd))


@pytest.mark.parametrize("nq,nkv,hd", [(32, 8, 128), (8, 2, 64), (8, 8, 64), (16, 2, 128), (64, 8, 128)])
@pytest.mark.parametrize("kv_dtype", [0, 1])
@pytest.mark.parametrize("path", ["0", "1"])
def test_paged_attention_ignores_rows_past_context(be, oracle, monkeypatch, nq, nkv, hd, kv_dtype, path):
    """Rows of a sequence's last page beyond its position hold stale bits in a
    live pool; here they are NaN and must not reach the output (0 * NaN)."""
    rng = np.random.default_rng(hd + nq + kv_dtype)
    ctxs = [1, 7, 16, 33, 513, 1030]
    layers, layer, n_pages = 2, 1, 160
    pool, table, dense, _ = build_paged(rng, ctxs, layers, nkv, hd, n_pages, kv_dtype, layer)
    for r, c in enumerate(ctxs):
        if c % 16:
            pool[:, table[r, c // 16], :, :, c % 16:, :] = np.nan
    pos = np.array([c - 1 for c in ctxs], np.int32)
    q = rng.normal(0, 1, (len(ctxs), nq * hd)).astype(np.float32)
    got = run_attention(be, monkeypatch, path, q, pool, table, pos, nq, nkv, hd, kv_dtype, layer, n_pages)
    assert np.isfinite(got).all()
    for r in range(len(ctxs)):
        Kd, Vd = dense[r]
        want = oracle.attention_gqa(q[r], Kd, Vd, nq, nkv, hd)
        assert scale_err(got[r], want) < 1e-5, (r, ctxs[r])


@pytest.mark.parametrize("nq,nkv,hd", [(32, 8, 128), (32, 4, 64)])
def test_paged_attention_kernels_agree_long_context(be, oracle, monkeypatch, nq, nkv, hd):
    """f16 pool, contexts across several 512-token chunks: the tensor-core and
    CUDA-core kernels both match the oracle on large-magnitude q (peaked
    softmax) and small-magnitude q (flat softmax)."""
    rng = np.random.default_rng(nq + hd)
    ctxs = [2047, 2048, 3001, 4097]
    layers, layer = 1, 0
    n_pages = sum((c + 15) // 16 for c in ctxs) + 3
    pool, table, dense, _ = build_paged(rng, ctxs, layers, nkv, hd, n_pages, 1, layer)
    pos = np.array([c - 1 for c in ctxs], np.int32)
    for sigma in (4.0, 1e-3):
        q = rng.normal(0, sigma, (len(ctxs), nq * hd)).astype(np.float32)
        outs = [run_attention(be, monkeypatch, p, q, pool, table, pos, nq, nkv, hd, 1, layer, n_pages)
                for p in ("0", "1")]
        for r in range(len(ctxs)):
            Kd, Vd = dense[r]
            want = oracle.attention_gqa(q[r], Kd, Vd, nq, nkv, hd)
            for got in outs:
                assert scale_err(got[r], want) < 1e-5, (sigma, r)
