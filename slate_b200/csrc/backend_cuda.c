/*
 * backend_cuda.c -- the CUDA implementation of Slate's compute-backend vtable
 * (include/slate/backend.h:41-99), replacing src/backend/backend_cuda_stub.c.
 *
 * The reference vtable is a process-wide singleton of plain function pointers
 * with no context argument and void returns, so this backend keeps one bound
 * device and one stream; every entry enqueues on that stream and returns at
 * once, and sync() waits (cudaStreamSynchronize).  copy_h2d / copy_d2h are
 * synchronous like the CPU backend's memcpy.  Errors of the void entries are
 * recorded for slate_cuda_last_error(); the appended entries return them.
 */
#define _GNU_SOURCE
#include "sb_internal.h"
#include "sb_kernels.h"
#include "sb_tc.h"

#include <pthread.h>
#include <stdlib.h>
#include <string.h>

static slate_backend_cuda_t g_be;
static cudaStream_t g_stream;
static int g_device = -1;
static pthread_mutex_t g_init = PTHREAD_MUTEX_INITIALIZER;

static void note(int rc, const char* what) {
    if (rc == 0) rc = sb_cuda_check(cudaGetLastError(), what);
    else if (rc == -1) sb_set_error("%s: unsupported arguments", what);
}

static void* be_alloc(size_t bytes) {
    if (bytes == 0) return NULL;   /* backend_cpu.c:23 returns NULL for 0 bytes */
    void* p = NULL;
    if (sb_cuda_check(cudaMalloc(&p, bytes), "alloc")) return NULL;
    return p;
}
static void be_release(void* p) {
    if (!p) return;
    cudaStreamSynchronize(g_stream);
    cudaFree(p);
}
static void be_h2d(void* dst, const void* src, size_t bytes) {
    sb_cuda_check(cudaMemcpyAsync(dst, src, bytes, cudaMemcpyHostToDevice, g_stream), "copy_h2d");
    sb_cuda_check(cudaStreamSynchronize(g_stream), "copy_h2d");
}
static void be_d2h(void* dst, const void* src, size_t bytes) {
    sb_cuda_check(cudaMemcpyAsync(dst, src, bytes, cudaMemcpyDeviceToHost, g_stream), "copy_d2h");
    sb_cuda_check(cudaStreamSynchronize(g_stream), "copy_d2h");
}

static int aligned16(const void* p) { return ((uintptr_t)p & 15u) == 0; }

/* y[M] = A[M,K]·x  (backend_cpu.c:33-36) */
static void be_matvec(float* y, const float* A, const float* x, int M, int K) {
    int rc;
    if (K % 128 == 0 && aligned16(A) && aligned16(x)) {
        sb_matrix W = {SB_WT_F32, A, M, M, K, K, 0};
        rc = sb_gemm(&W, x, K, 1, y, M, SB_EPI_STORE, 0, g_stream);
    } else {
        rc = sb_matvec_f32_generic(y, A, x, M, K, g_stream);
    }
    note(rc, "matvec");
}
/* C[B,N] = X[B,K]·W[K,N]  (backend_cpu.c:38-42) */
static void be_linear_batch(float* C, const float* X, const float* W, int B, int K, int N) {
    note(sb_linear_batch_generic(C, X, W, B, K, N, g_stream), "linear_batch");
}
/* y[M] = Q4K(A)[M,K]·x  (backend_cpu.c:44-46) */
static void be_matvec_q4k(float* y, const void* A, const float* x, int M, int K) {
    note(sb_q4k_matmul_generic(y, A, x, 1, M, K, g_stream), "matvec_q4k");
}
static void be_rmsnorm_row(float* y, const float* x, const float* w, int D, float eps) {
    note(sb_rmsnorm_rows(y, D, x, D, w, 1, D, eps, g_stream), "rmsnorm_row");
}
static void be_silu_mul(float* y, const float* g, const float* u, int H) {
    note(sb_silu_mul(y, g, u, H, g_stream), "silu_mul");
}
static void be_add(float* y, const float* x, int D) {
    note(sb_add_inplace(y, x, D, g_stream), "add_inplace");
}
static void be_embed(float* y, const float* W, int token, int D) {
    note(sb_embed_lookup(y, W, token, D, g_stream), "embed_lookup");
}
static void be_attention_step(float* out, const float* q, const float* K, const float* V,
                              float* scores, int L, int D) {
    (void)scores;  /* the device kernel keeps scores in shared memory */
    note(sb_attention_step(out, q, K, V, L, D, g_stream), "attention_step");
}
static void be_sync(void) { sb_cuda_check(cudaStreamSynchronize(g_stream), "sync"); }

/* ---- appended, status-returning entries -------------------------------- */
static int fin(int rc, const char* what) {
    if (rc == -1) { sb_set_error("%s: unsupported arguments", what); return -1; }
    return rc ? rc : sb_cuda_check(cudaGetLastError(), what);
}
static int be_matmul_q4k(float* Y, const void* A, const float* X, int B, int M, int K) {
    return fin(sb_q4k_matmul_generic(Y, A, X, B, M, K, g_stream), "matmul_q4k_batch");
}
static int be_matmul_f32(float* Y, const float* A, const float* X, int B, int M, int K) {
    if (K % 128 == 0 && aligned16(A) && aligned16(X)) {
        sb_matrix W = {SB_WT_F32, A, M, M, K, K, 0};
        return fin(sb_gemm(&W, X, K, B, Y, M, SB_EPI_STORE, 0, g_stream), "matmul_f32_batch");
    }
    int rc = 0;
    for (int b = 0; b < B && !rc; ++b)
        rc = sb_matvec_f32_generic(Y + (size_t)b * M, A, X + (size_t)b * K, M, K, g_stream);
    return fin(rc, "matmul_f32_batch");
}
static int be_rmsnorm_rows(float* Y, const float* X, const float* w, int B, int D, float eps) {
    return fin(sb_rmsnorm_rows(Y, D, X, D, w, B, D, eps, g_stream), "rmsnorm_rows");
}
static int be_argmax_rows(int32_t* out, const float* logits, int B, int V) {
    return fin(sb_argmax_rows(out, logits, V, B, V, g_stream), "argmax_rows");
}
static int be_rope_kv(float* q, float* k, const float* v, const int32_t* pos,
                      const int32_t* row_slot, const int32_t* page_table, int max_pages,
                      void* pool, int64_t n_pages, int layer, int B, int nq, int nkv, int hd,
                      int kv_dtype, const float* rc, const float* rs) {
    /* the kernel takes one [q | k | v] row per batch entry; these entries may
     * live in separate buffers, so gather them into a scratch row block */
    const int qd = nq * hd, kd = nkv * hd, ld = qd + 2 * kd;
    float* tmp = NULL;
    int rcode = sb_cuda_check(cudaMallocAsync((void**)&tmp, (size_t)B * ld * 4, g_stream), "scratch");
    if (rcode) return rcode;
    rcode = sb_cuda_check(cudaMemcpy2DAsync(tmp, (size_t)ld * 4, q, (size_t)qd * 4, (size_t)qd * 4, B,
                                            cudaMemcpyDeviceToDevice, g_stream), "gather q");
    if (!rcode) rcode = sb_cuda_check(cudaMemcpy2DAsync(tmp + qd, (size_t)ld * 4, k, (size_t)kd * 4,
                                                        (size_t)kd * 4, B, cudaMemcpyDeviceToDevice,
                                                        g_stream), "gather k");
    if (!rcode) rcode = sb_cuda_check(cudaMemcpy2DAsync(tmp + qd + kd, (size_t)ld * 4, v,
                                                        (size_t)kd * 4, (size_t)kd * 4, B,
                                                        cudaMemcpyDeviceToDevice, g_stream), "gather v");
    if (!rcode) rcode = fin(sb_rope_append(tmp, ld, B, nq, nkv, hd, pos, row_slot, page_table,
                                           max_pages, pool, n_pages, layer, kv_dtype, rc, rs,
                                           g_stream), "rope_kv_append_paged");
    if (!rcode) rcode = sb_cuda_check(cudaMemcpy2DAsync(q, (size_t)qd * 4, tmp, (size_t)ld * 4,
                                                        (size_t)qd * 4, B, cudaMemcpyDeviceToDevice,
                                                        g_stream), "scatter q");
    if (!rcode) rcode = sb_cuda_check(cudaMemcpy2DAsync(k, (size_t)kd * 4, tmp + qd, (size_t)ld * 4,
                                                        (size_t)kd * 4, B, cudaMemcpyDeviceToDevice,
                                                        g_stream), "scatter k");
    cudaFreeAsync(tmp, g_stream);
    return rcode;
}
static int be_attention_paged(float* out, const float* q, const int32_t* pos,
                              const int32_t* row_slot, const int32_t* page_table, int max_pages,
                              const void* pool, int64_t n_pages, int layer, int B, int nq, int nkv,
                              int hd, int kv_dtype) {
    int max_seq = max_pages * SB_PAGE_TOKENS;
    size_t nf = sb_attention_scratch_floats(B, nq, hd, max_seq);
    float* scr = NULL;
    int* err = NULL;
    int e = 0;
    int rc = sb_cuda_check(cudaMallocAsync((void**)&scr, nf * 4 + 16, g_stream), "scratch");
    if (rc) return rc;
    err = (int*)(scr + nf);
    rc = sb_cuda_check(cudaMemsetAsync(err, 0, 4, g_stream), "memset");
    if (!rc && sb_attention_prepare(nq, nkv, hd, kv_dtype)) rc = -1;
    /* f16 pools of supported shapes run the tensor-core kernel; its map spans
     * layers [0, layer] of the pool */
    unsigned char map[SB_KVMAP_BYTES];
    const void* mapp = NULL;
    const char* path = getenv("SLATE_CUDA_ATTN_PATH");     /* "1": CUDA-core kernel only */
    if (!rc && sb_attention_mma_supported(nq, nkv, hd, kv_dtype) && !(path && path[0] == '1')) {
        if (sb_attention_make_map(map, (void*)pool, n_pages, layer + 1, nkv, hd)) rc = -1;
        else mapp = map;
    }
    if (!rc)
        rc = fin(sb_attention_paged(out, nq * hd, q, nq * hd, B, nq, nkv, hd, pos, row_slot,
                                    page_table, max_pages, pool, mapp, n_pages, layer, kv_dtype,
                                    max_seq, 0, scr, err, g_stream),
                 "attention_paged_gqa");
    if (!rc) rc = sb_cuda_check(cudaMemcpyAsync(&e, err, 4, cudaMemcpyDeviceToHost, g_stream), "err");
    if (!rc) rc = sb_cuda_check(cudaStreamSynchronize(g_stream), "attention_paged_gqa");
    if (!rc && e) {
        sb_set_error("attention pipeline reported %d", e);
        rc = -5;
    }
    cudaFreeAsync(scr, g_stream);
    return rc;
}

/* passes 2: the exact-weight kernel (gemm_q4k.cu), any B >= 1 */
static int be_matmul_q4k_exact(float* Y, const void* A, const float* X, int B, int M, int K) {
    sb_matrix W = {SB_WT_Q4K, A, M, M, K, 0, 0};
    sb_q4_prepare();
    const int r_pad = (B + 127) / 128 * 128;
    const size_t xs_bytes = (size_t)((K / 256 + 1) & ~1) * r_pad * 8 * 2;
    const int tiles = sb_q4_tiles(M, B);
    void *hi = NULL, *lo = NULL, *xh = NULL, *xl = NULL, *ws = NULL, *cnt = NULL;
    int rc = sb_cuda_check(cudaMallocAsync(&hi, (size_t)B * K * 2, g_stream), "alloc");
    if (!rc) rc = sb_cuda_check(cudaMallocAsync(&lo, (size_t)B * K * 2, g_stream), "alloc");
    if (!rc) rc = sb_cuda_check(cudaMallocAsync(&xh, xs_bytes, g_stream), "alloc");
    if (!rc) rc = sb_cuda_check(cudaMallocAsync(&xl, xs_bytes, g_stream), "alloc");
    if (!rc) rc = sb_cuda_check(cudaMallocAsync(&ws, sb_q4_ws_floats() * 4, g_stream), "alloc");
    if (!rc) rc = sb_cuda_check(cudaMallocAsync(&cnt, (size_t)tiles * 4 + 16, g_stream), "alloc");
    if (!rc) rc = sb_cuda_check(cudaMemsetAsync(cnt, 0, (size_t)tiles * 4 + 16, g_stream), "memset");
    if (!rc) rc = sb_cuda_check(cudaMemsetAsync(xh, 0, xs_bytes, g_stream), "memset");
    if (!rc) rc = sb_cuda_check(cudaMemsetAsync(xl, 0, xs_bytes, g_stream), "memset");
    if (!rc) rc = sb_cuda_check(cudaStreamSynchronize(g_stream), "alloc sync");
    int* err = (int*)cnt + tiles;
    sb_q4_operand op;
    if (!rc && sb_q4_make_operand(&op, hi, lo, xh, xl, B, r_pad, K, K)) rc = -1;
    if (!rc) rc = fin(sb_q4_split(X, K, B, &op, g_stream), "q4 split");
    if (!rc) rc = fin(sb_q4_gemm(&W, &op, B, Y, M, SB_EPI_STORE, (float*)ws, (int*)cnt, err, g_stream),
                      "matmul_q4k_batch_tc");
    int e = 0;
    if (!rc) rc = sb_cuda_check(cudaMemcpyAsync(&e, err, 4, cudaMemcpyDeviceToHost, g_stream), "err");
    if (!rc) rc = sb_cuda_check(cudaStreamSynchronize(g_stream), "matmul_q4k_batch_tc");
    if (!rc && e) {
        sb_set_error("tensor-core pipeline wait timed out (stage %d)", e);
        rc = -5;
    }
    void* bufs[6] = {hi, lo, xh, xl, ws, cnt};
    for (int i = 0; i < 6; ++i)
        if (bufs[i]) cudaFreeAsync(bufs[i], g_stream);
    return rc;
}

/* passes 3 on the stream-K kernel (gemm_sk.cu) */
static int be_matmul_q4k_sk(float* Y, const void* A, const float* X, int B, int M, int K) {
    sb_matrix W = {SB_WT_Q4K, A, M, M, K, 0, 0};
    sb_sk_prepare();
    void *hi = NULL, *lo = NULL, *ws = NULL, *err = NULL;
    int rc = sb_cuda_check(cudaMallocAsync(&hi, (size_t)B * K * 2, g_stream), "alloc");
    if (!rc) rc = sb_cuda_check(cudaMallocAsync(&lo, (size_t)B * K * 2, g_stream), "alloc");
    if (!rc) rc = sb_cuda_check(cudaMallocAsync(&ws, sb_sk_ws_floats(0) * 4, g_stream), "alloc");
    if (!rc) rc = sb_cuda_check(cudaMallocAsync(&err, 16, g_stream), "alloc");
    if (!rc) rc = sb_cuda_check(cudaMemsetAsync(err, 0, 16, g_stream), "memset");
    if (!rc) rc = sb_cuda_check(cudaStreamSynchronize(g_stream), "alloc sync");
    sb_tc_operand op;
    if (!rc && sb_tc_make_operand(&op, hi, lo, B, K, K)) rc = -1;
    if (!rc) rc = fin(sb_tc_split(X, K, B, &op, g_stream), "tc split");
    if (!rc) rc = fin(sb_sk_gemm(&W, &op, B, (float*)ws, Y, M, SB_EPI_STORE, NULL, NULL, 0, NULL, (int*)err,
                                 g_stream),
                      "matmul_q4k_batch_tc");
    int e = 0;
    if (!rc) rc = sb_cuda_check(cudaMemcpyAsync(&e, err, 4, cudaMemcpyDeviceToHost, g_stream), "err");
    if (!rc) rc = sb_cuda_check(cudaStreamSynchronize(g_stream), "matmul_q4k_batch_tc");
    if (!rc && e) {
        sb_set_error("tensor-core pipeline wait timed out (stage %d)", e);
        rc = -5;
    }
    void* bufs[4] = {hi, lo, ws, err};
    for (int i = 0; i < 4; ++i)
        if (bufs[i]) cudaFreeAsync(bufs[i], g_stream);
    return rc;
}

/* passes 4: the small-batch kernel (gemm_mv.cu), 1 <= B <= 16 */
static int be_matmul_q4k_mv(float* Y, const void* A, const float* X, int B, int M, int K) {
    sb_matrix W = {SB_WT_Q4K, A, M, M, K, 0, 0};
    const size_t wsf = sb_mv_ws_floats(M, K);
    void *ws = NULL, *cnt = NULL;
    int rc = sb_cuda_check(cudaMallocAsync(&ws, wsf * 4 + 16, g_stream), "alloc");
    if (!rc) rc = sb_cuda_check(cudaMallocAsync(&cnt, (size_t)M / 128 * 4, g_stream), "alloc");
    if (!rc) rc = sb_cuda_check(cudaMemsetAsync(cnt, 0, (size_t)M / 128 * 4, g_stream), "memset");
    if (!rc) rc = fin(sb_mv_gemm(&W, X, K, B, Y, M, SB_EPI_STORE, (float*)ws, (int*)cnt, g_stream),
                      "matmul_q4k_batch_tc");
    if (!rc) rc = sb_cuda_check(cudaStreamSynchronize(g_stream), "matmul_q4k_batch_tc");
    if (ws) cudaFreeAsync(ws, g_stream);
    if (cnt) cudaFreeAsync(cnt, g_stream);
    return rc;
}

static int be_matmul_q4k_tc(float* Y, const void* A, const float* X, int B, int M, int K,
                            int passes) {
    if (passes == 4) {
        if (M % 128 || K % 256 || B < 1 || B > SB_MV_MAX_ROWS) {
            sb_set_error("matmul_q4k_batch_tc: passes 4 takes 1 <= B <= %d, M %% 128 == 0",
                         SB_MV_MAX_ROWS);
            return -1;
        }
        return be_matmul_q4k_mv(Y, A, X, B, M, K);
    }
    if (passes == 2 && M % 128 == 0 && K % 256 == 0 && B >= 1 && K % 4 == 0)
        return be_matmul_q4k_exact(Y, A, X, B, M, K);
    {
        /* SLATE_TC_SK=1: three passes on the stream-K kernel */
        const char* e = getenv("SLATE_TC_SK");
        if (passes == 3 && e && e[0] == '1' && M % 128 == 0 && K % 256 == 0 && B >= 16)
            return be_matmul_q4k_sk(Y, A, X, B, M, K);
    }
    if (M % 128 || K % 256 || B < 16 || (passes != 1 && passes != 3)) {
        sb_set_error("matmul_q4k_batch_tc: unsupported shape or passes");
        return -1;
    }
    sb_matrix W = {SB_WT_Q4K, A, M, M, K, 0, 0};
    const int splits = sb_tc_splits_for(M, K);
    void *hi = NULL, *lo = NULL, *ws = NULL, *err = NULL;
    int rc = sb_cuda_check(cudaMallocAsync(&hi, (size_t)B * K * 2, g_stream), "alloc");
    if (!rc && passes == 3) rc = sb_cuda_check(cudaMallocAsync(&lo, (size_t)B * K * 2, g_stream), "alloc");
    if (!rc) rc = sb_cuda_check(cudaMallocAsync(&ws, (size_t)splits * B * M * 4, g_stream), "alloc");
    if (!rc) rc = sb_cuda_check(cudaMallocAsync(&err, 16, g_stream), "alloc");
    if (!rc) rc = sb_cuda_check(cudaMemsetAsync(err, 0, 16, g_stream), "memset");
    if (!rc) rc = sb_cuda_check(cudaStreamSynchronize(g_stream), "alloc sync");
    sb_tc_operand op;
    if (!rc && sb_tc_make_operand(&op, hi, lo, B, K, K)) rc = -1;
    if (!rc) rc = fin(sb_tc_split(X, K, B, &op, g_stream), "tc split");
    if (!rc) rc = fin(sb_tc_gemm(&W, &op, B, passes, splits, (float*)ws, Y, M, SB_EPI_STORE,
                                 (int*)err, g_stream), "matmul_q4k_batch_tc");
    int e = 0;
    if (!rc) rc = sb_cuda_check(cudaMemcpyAsync(&e, err, 4, cudaMemcpyDeviceToHost, g_stream), "err");
    if (!rc) rc = sb_cuda_check(cudaStreamSynchronize(g_stream), "matmul_q4k_batch_tc");
    if (!rc && e) {
        sb_set_error("tensor-core pipeline wait timed out (stage %d)", e);
        rc = -5;
    }
    if (hi) cudaFreeAsync(hi, g_stream);
    if (lo) cudaFreeAsync(lo, g_stream);
    if (ws) cudaFreeAsync(ws, g_stream);
    if (err) cudaFreeAsync(err, g_stream);
    return rc;
}

int slate_cuda_sample_rows(int32_t* out_tokens, const float* logits, int ld, int B, int V,
                           const slate_sampler_config_t* cfg, uint64_t* rng_state) {
    if (!out_tokens || !logits || !cfg || !rng_state || B < 1 || V < 1 || ld < V) {
        sb_set_error("sample_rows: bad arguments");
        return -1;
    }
    for (int r = 0; r < B; ++r)
        if (cfg[r].temperature > 0.0f && cfg[r].top_k > SB_SAMPLE_TOPK_MAX && cfg[r].top_k < V) {
            sb_set_error("top_k %d above the device sampler's %d", cfg[r].top_k, SB_SAMPLE_TOPK_MAX);
            return -1;
        }
    sb_sampler* hc = (sb_sampler*)malloc((size_t)B * sizeof(sb_sampler));
    if (!hc) return -5;
    for (int r = 0; r < B; ++r) hc[r] = (sb_sampler){cfg[r].temperature, cfg[r].top_k, cfg[r].top_p, 0};
    void *dc = NULL, *dr = NULL, *dout = NULL, *scr = NULL;
    int rc = sb_cuda_check(cudaDeviceSynchronize(), "sample_rows: pending work");
    if (!rc) rc = sb_cuda_check(cudaMalloc(&dc, (size_t)B * sizeof(sb_sampler)), "alloc");
    if (!rc) rc = sb_cuda_check(cudaMalloc(&dr, (size_t)B * 8), "alloc");
    if (!rc) rc = sb_cuda_check(cudaMalloc(&dout, (size_t)B * 4 + 16), "alloc");
    if (!rc) rc = sb_cuda_check(cudaMalloc(&scr, (size_t)B * V * 4), "alloc");
    if (!rc) rc = sb_cuda_check(cudaMemset(dout, 0, (size_t)B * 4 + 16), "memset");
    if (!rc) rc = sb_cuda_check(cudaMemcpy(dc, hc, (size_t)B * sizeof(sb_sampler), cudaMemcpyHostToDevice), "H2D");
    if (!rc) rc = sb_cuda_check(cudaMemcpy(dr, rng_state, (size_t)B * 8, cudaMemcpyHostToDevice), "H2D");
    int* err = dout ? (int*)((int32_t*)dout + B) : NULL;
    if (!rc && sb_sample_rows(logits, ld, V, B, (const sb_sampler*)dc, (uint64_t*)dr, (float*)scr,
                              (int32_t*)dout, NULL, NULL, NULL, NULL, err, 0))
        rc = -1;
    int e = 0;
    if (!rc) rc = sb_cuda_check(cudaMemcpy(out_tokens, dout, (size_t)B * 4, cudaMemcpyDeviceToHost), "D2H");
    if (!rc) rc = sb_cuda_check(cudaMemcpy(rng_state, dr, (size_t)B * 8, cudaMemcpyDeviceToHost), "D2H");
    if (!rc) rc = sb_cuda_check(cudaMemcpy(&e, err, 4, cudaMemcpyDeviceToHost), "D2H");
    if (!rc && e) {
        sb_set_error("sampler reported %d", e);
        rc = -1;
    }
    cudaFree(dc);
    cudaFree(dr);
    cudaFree(dout);
    cudaFree(scr);
    free(hc);
    return rc;
}

const slate_backend_cuda_t* slate_backend_cuda_create(int device) {
    pthread_mutex_lock(&g_init);
    const slate_backend_cuda_t* r = NULL;
    if (g_device >= 0) {
        r = g_device == device ? &g_be : NULL;
        if (!r) sb_set_error("backend already bound to device %d", g_device);
    } else {
        int n = 0;
        if (!sb_cuda_check(cudaGetDeviceCount(&n), "cudaGetDeviceCount") && device >= 0 &&
            device < n && !sb_cuda_check(cudaSetDevice(device), "cudaSetDevice") &&
            !sb_cuda_check(cudaStreamCreateWithFlags(&g_stream, cudaStreamNonBlocking), "stream")) {
            sb_gemm_prepare();
            memset(&g_be, 0, sizeof g_be);
            g_be.base.name = "cuda";
            g_be.base.alloc = be_alloc;
            g_be.base.release = be_release;
            g_be.base.copy_h2d = be_h2d;
            g_be.base.copy_d2h = be_d2h;
            g_be.base.matvec = be_matvec;
            g_be.base.linear_batch = be_linear_batch;
            g_be.base.matvec_q4k = be_matvec_q4k;
            g_be.base.rmsnorm_row = be_rmsnorm_row;
            g_be.base.silu_mul = be_silu_mul;
            g_be.base.add_inplace = be_add;
            g_be.base.embed_lookup = be_embed;
            g_be.base.attention_step = be_attention_step;
            g_be.base.sync = be_sync;
            g_be.abi_version = SLATE_CUDA_ABI_VERSION;
            g_be.device = device;
            g_be.matmul_q4k_batch = be_matmul_q4k;
            g_be.matmul_f32_batch = be_matmul_f32;
            g_be.rmsnorm_rows = be_rmsnorm_rows;
            g_be.argmax_rows = be_argmax_rows;
            g_be.rope_kv_append_paged = be_rope_kv;
            g_be.attention_paged_gqa = be_attention_paged;
            g_be.matmul_q4k_batch_tc = be_matmul_q4k_tc;
            sb_tc_prepare();
            g_device = device;
            r = &g_be;
        } else if (device < 0 || device >= n) {
            sb_set_error("no CUDA device %d (%d present)", device, n);
        }
    }
    pthread_mutex_unlock(&g_init);
    return r;
}

/* ---- host-coherent form ------------------------------------------------
 * The reference's GPT engine (src/infer/engine.c) uses its backend the way the
 * CPU backend allows: it memset()s and memcpy()s buffers returned by alloc on
 * the host (:276-277, 411-412, 586-591), hands host pointers to the entries
 * (the module's weights, calloc'd scratch at :446, the caller's logits) and
 * reads results right after a call without sync().  This form serves such a
 * caller unchanged: alloc returns managed memory (host and device see one
 * address), the copies go through cudaMemcpyDefault, and every entry waits for
 * its kernel before returning.  The kernels read the pointers they are given
 * directly, with plain loads only (no TMA): memory from this table's alloc,
 * pinned or registered host memory, or -- on a device that can access pageable
 * host memory (cudaDevAttrPageableMemoryAccess: HMM or ATS,
 * slate_cuda_pageable_memory_access) -- any host memory.  It shares the device
 * and stream of the main singleton. */
static slate_backend_t g_hc;

static void* hc_alloc(size_t bytes) {
    if (bytes == 0) return NULL;
    void* p = NULL;
    if (sb_cuda_check(cudaMallocManaged(&p, bytes, cudaMemAttachGlobal), "alloc (managed)"))
        return NULL;
    return p;
}
static void hc_copy(void* dst, const void* src, size_t bytes) {
    sb_cuda_check(cudaMemcpyAsync(dst, src, bytes, cudaMemcpyDefault, g_stream), "copy");
    be_sync();
}
static void hc_matvec(float* y, const float* A, const float* x, int M, int K) {
    note(sb_matvec_f32_generic(y, A, x, M, K, g_stream), "matvec");
    be_sync();
}
static void hc_linear_batch(float* C, const float* X, const float* W, int B, int K, int N) {
    be_linear_batch(C, X, W, B, K, N);
    be_sync();
}
static void hc_matvec_q4k(float* y, const void* A, const float* x, int M, int K) {
    be_matvec_q4k(y, A, x, M, K);
    be_sync();
}
static void hc_rmsnorm_row(float* y, const float* x, const float* w, int D, float eps) {
    be_rmsnorm_row(y, x, w, D, eps);
    be_sync();
}
static void hc_silu_mul(float* y, const float* g, const float* u, int H) {
    be_silu_mul(y, g, u, H);
    be_sync();
}
static void hc_add(float* y, const float* x, int D) {
    be_add(y, x, D);
    be_sync();
}
static void hc_embed(float* y, const float* W, int token, int D) {
    be_embed(y, W, token, D);
    be_sync();
}
static void hc_attention_step(float* out, const float* q, const float* K, const float* V,
                              float* scores, int L, int D) {
    be_attention_step(out, q, K, V, scores, L, D);
    be_sync();
}

int slate_cuda_pageable_memory_access(int device) {
    int v = 0;
    if (sb_cuda_check(cudaDeviceGetAttribute(&v, cudaDevAttrPageableMemoryAccess, device),
                      "cudaDeviceGetAttribute"))
        return -5;
    return v ? 1 : 0;
}

const slate_backend_t* slate_backend_cuda_host_coherent(int device) {
    if (!slate_backend_cuda_create(device)) return NULL;
    pthread_mutex_lock(&g_init);
    if (!g_hc.name) {
        g_hc.alloc = hc_alloc;
        g_hc.release = be_release;
        g_hc.copy_h2d = hc_copy;
        g_hc.copy_d2h = hc_copy;
        g_hc.matvec = hc_matvec;
        g_hc.linear_batch = hc_linear_batch;
        g_hc.matvec_q4k = hc_matvec_q4k;
        g_hc.rmsnorm_row = hc_rmsnorm_row;
        g_hc.silu_mul = hc_silu_mul;
        g_hc.add_inplace = hc_add;
        g_hc.embed_lookup = hc_embed;
        g_hc.attention_step = hc_attention_step;
        g_hc.sync = be_sync;
        g_hc.name = "cuda-host-coherent";
    }
    pthread_mutex_unlock(&g_init);
    return &g_hc;
}

const slate_backend_t* slate_backend_cuda(void) {
    const char* e = getenv("SLATE_CUDA_BACKEND");
    if (!e || strcmp(e, "1") != 0) return NULL;
    const char* d = getenv("SLATE_CUDA_DEVICE");
    const slate_backend_cuda_t* b = slate_backend_cuda_create(d ? atoi(d) : 0);
    return b ? &b->base : NULL;
}
