/*
 * llama_batch.c -- device-resident continuous-batching LLaMA decode engine.
 *
 * The reference decodes one session at a time (src/loader/llama_infer.c:
 * 134-206) with a dense host KV cache per session (:225-226); its only
 * batched step is the GPT engine's slate_infer_batch_step
 * (src/infer/engine.c:543-642).  This engine runs the LLaMA step for n
 * sequences at once on one GPU:
 *
 *   prologue   validate rows, allocate KV pages, gather embeddings    (1 kernel)
 *   per layer  rmsnorm -> QKV GEMM -> RoPE + paged KV append ->
 *              attention (partial + combine) -> Wo GEMM (+residual) ->
 *              rmsnorm -> gate/up GEMM (+SiLU*up) -> down GEMM (+residual)
 *                                                                  (9 kernels)
 *   final      rmsnorm -> LM head GEMM -> argmax + position advance (3 kernels)
 *
 * Host responsibilities are only: argument checks against host mirrors of the
 * positions, the per-step copy of (slot, token) metadata, and launching one
 * captured CUDA graph per batch size.  Positions, page tables and the page
 * free list live in device memory and are updated by the kernels.
 */
#define _GNU_SOURCE
#include "sb_internal.h"
#include "sb_kernels.h"
#include "sb_tc.h"

#include <math.h>
#include <pthread.h>
#include <stdio.h>
#include <stdlib.h>
#include <string.h>

typedef struct sb_layer {
    float* attn_norm;
    float* ffn_norm;
    sb_matrix wqkv, wo, wgu, wdown;
} sb_layer;

/* A lane runs the layers of a step for a contiguous range of the batch's rows.
 * A step runs one lane over all rows, or two lanes over the two halves on two
 * streams (independent chains: different sequences), so that one half's
 * attention, bound by HBM, runs beside the other half's projections, bound by
 * the tensor cores. */
typedef struct sb_lane {
    sb_tc_operand own[3];          /* half lanes: operands over the half's rows */
    const sb_tc_operand *op_d, *op_f, *op_a;   /* GEMM operands (K = D, F, Dq) */
    float* sk_ws;                  /* stream-K workspace of this lane */
    float* mv_ws;                  /* small-batch GEMM partials and counters */
    int* mv_cnt;
    int r0;                        /* first row */
    void* comm;                    /* NCCL communicator of this lane's all-reduces (tp > 1) */
    int xn_split, att_split;       /* enqueue time: the RMSNorm / attention wrote
                                      the f16 operand of the GEMM that follows */
} sb_lane;

/* Input of a step GEMM (which producer may already have written its f16 pair). */
enum { IN_XN, IN_ATT, IN_H, IN_OTHER };

struct slate_llama_batch {
    int device;
    cudaStream_t stream;
    cudaStream_t stream2;          /* second lane */
    cudaEvent_t ev_fork, ev_join;
    cudaEvent_t ev_a, ev_b;        /* lane order: a lane's attention of a layer done */
    pthread_mutex_t lock;
    /* model */
    int L, D, F, nq, nkv, hd, V, kvd, qkv_dim, max_seq;
    float theta, eps;
    float *emb, *out_norm;
    sb_matrix lm_head;
    sb_layer* layers;
    void** allocs;
    int n_allocs, cap_allocs;
    float *rope_cos, *rope_sin;
    /* KV */
    int kv_dtype, max_pages, max_slots;
    int64_t n_pages;
    void* pool;
    unsigned char kvmap[SB_KVMAP_BYTES];   /* tensor map of the pool */
    const void* kvmap_p;                   /* kvmap when the tensor-core attention runs */
    int32_t *pos, *page_table, *free_stack, *free_top, *status;
    /* activations */
    int max_batch, gemm_path, use_graphs;
    int ld_x, ld_qkv, ld_att, ld_h, ld_logits;
    float *x, *xn, *qkv, *att, *h, *logits, *scratch;
    int32_t *row_pos, *row_slot;
    int32_t *d_io;        /* [slots | tokens | out_tokens] of max_batch each */
    int32_t* h_io;        /* pinned mirror of d_io + one status word */
    /* host mirrors */
    int* h_pos;
    unsigned char* h_open;
    int pos_dirty;
    int64_t pages_used;
    /* graphs, one per batch size */
    cudaGraphExec_t* graphs;
    /* tensor-core GEMM path: f16 operands (hi/lo) with TMA maps, K-split
     * partials, device error word, split counts per weight */
    int tc_passes;                 /* 0 = off, 1 or 3 */
    sb_tc_operand op_d, op_f;      /* activations with K = d_model / ffn */
    float* tc_ws;
    int* tc_err;
    int* head_cnt;                 /* per-head row counts of the GEMV's RoPE epilogue (zeroed) */
    int sp_qkv, sp_wo, sp_gu, sp_dn;
    sb_tc_weight head_tc;          /* f32 LM head as an f16 pair (hi set when used) */
    sb_tc_operand op_a;            /* attention output, K = nq*hd (tensor parallel: local heads) */
    /* exact-weight Q4_K GEMM (gemm_path 0): operands over the same f16 hi/lo
     * buffers plus sub-block sums, stream-K partials and tile counters */
    int q4k_order;                 /* source Q4_K packing: 0 Slate, 1 ggml (repacked) */
    int q4_on;
    sb_q4_operand q4_d, q4_f, q4_a;
    float* q4_ws;
    int* q4_cnt;
    size_t q4_cnt_n;
    /* three-pass stream-K GEMM (gemm_sk.cu): workspace; sk_h: the gate/up
     * GEMM writes its SiLU output also as the down GEMM's f16 hi / lo operand */
    int sk_on, sk_h, sk_min;       /* sk_min: rows from which a GEMM uses it */
    int gv_on;                     /* Q4_K GEMMs of 1-2 rows on the CUDA-core GEMV */
    float* sk_ws;
    sb_lane full, half[2];         /* the whole batch; the two halves (dual) */
    int dual, half_rows;           /* dual: steps of > half_rows rows use two lanes */
    int chunk_step;                /* enqueue time: the step is a prompt chunk */
    /* tensor parallelism: nq, nkv, F above are this rank's shares, V the full
     * vocabulary of which the LM head holds rows [v0, v0 + V_l) */
    int tp, rank, V_l, v0, Dq;     /* Dq = nq * hd (local) */
    void* comm;                    /* NCCL communicator (tp > 1) */
    void* comm2;                   /* the second lane's (split from comm; two lanes, tp > 1) */
    void *pairs, *pairs_all;       /* per-row (max, index) of this rank / of all ranks */
    float* logits_all;             /* [tp][max_batch][ld_logits], gathered on request */
    /* stochastic sampling (allocated on first use): per-row configs and RNG
     * states (device + pinned host mirrors), softmax scratch, graphs per n */
    sb_sampler* d_samp;
    uint64_t* d_rng;
    float* samp_scratch;
    sb_sampler* h_samp;
    uint64_t* h_rng;
    cudaGraphExec_t* graphs_s;
    cudaGraphExec_t* graphs_c;     /* prompt-chunk steps (repeated slots), per n */
    cudaGraphExec_t* graphs_p;     /* the same without LM head (logits not wanted) */
};

/* Rows from which a Q4_K GEMM runs on the tensor cores (below: CUDA cores). */
#define SB_TC_MIN_ROWS 16
/* Rows from which the default path uses the stream-K kernel (gemm_sk.cu)
 * rather than gemm_tc.cu's tile-per-CTA kernel. */
#define SB_SK_MIN_ROWS 128

/* Whether the RMSNorm before a GEMM writes the tensor cores' f16 operand too
 * (the 3- or 1-pass split paths; the exact-weight path splits with sub-block
 * sums of its own). */
static int norm_splits(const slate_llama_batch_t* b, const sb_lane* L, int n) {
    return b->tc_passes && !b->q4_on && n >= SB_TC_MIN_ROWS && n <= L->op_d->rows &&
           !(L->mv_ws && n <= SB_MV_MAX_ROWS) &&
           b->D % 4 == 0 && b->D <= 8192 && b->ld_x % 4 == 0 && L->op_d->ld16 % 4 == 0;
}

/* RMSNorm of the lane's rows of x into xn (and, where the GEMMs take it, into
 * the lane's f16 operand). */
static int step_norm(slate_llama_batch_t* b, sb_lane* L, const float* w, int n, cudaStream_t s) {
    const size_t ro = (size_t)L->r0 * b->ld_x;
    L->xn_split = 0;
    /* -1 from the split kernel means the shape does not fit it (nothing was
     * launched) and the next form is tried; a failed launch is returned */
    int rc = -1;
    if (norm_splits(b, L, n)) {
        rc = sb_rmsnorm_rows_split(b->xn + ro, b->ld_x, b->x + ro, b->ld_x, w, n, b->D, b->eps,
                                   L->op_d->hi, L->op_d->lo, L->op_d->ld16, s);
        if (rc == 0) L->xn_split = 1;
        if (rc != -1) return rc;
    }
    /* f32 rows only, through the same kernel where the shape allows: it stays in
     * the programmatic launch chain, so the GEMM after it starts streaming its
     * weights while it runs */
    rc = sb_rmsnorm_rows_split(b->xn + ro, b->ld_x, b->x + ro, b->ld_x, w, n, b->D, b->eps, NULL,
                               NULL, 0, s);
    if (rc != -1) return rc;
    return sb_rmsnorm_rows(b->xn + ro, b->ld_x, b->x + ro, b->ld_x, w, n, b->D, b->eps, s);
}

/* Whether the GEMM after an RMSNorm takes the norm into its activation
 * staging (the one-/two-row GEMV), so no RMSNorm launch precedes it. */
static int norm_in_gemv(const slate_llama_batch_t* b, const sb_matrix* W, int n, int epi) {
    return b->gv_on && n <= SB_GV_MAX_ROWS && W->K == b->D && sb_gv_supported(W, n, epi);
}

/* Whether the f32 LM head runs on the tensor cores as its f16 hi/lo pair: from
 * SB_TC_MIN_ROWS rows, and from 4 rows where the operand's row box is small
 * (an engine of at most 64 rows), since the CUDA-core GEMV is FMA-bound from
 * about 4 rows while the tensor-core pass costs the same up to its box. */
static int head_on_tc(const slate_llama_batch_t* b, const sb_lane* L, int n) {
    return b->head_tc.hi && (n >= SB_TC_MIN_ROWS || (n >= 4 && L->op_d->n_box <= 64));
}

/* Whether a GEMM of this lane runs on the stream-K kernel. */
static int uses_sk(const slate_llama_batch_t* b, const sb_lane* L, const sb_matrix* W, int n,
                   int epi) {
    return b->sk_on && W->wtype == SB_WT_Q4K && W->M_pad % 128 == 0 &&
           (epi != SB_EPI_SILU || W->M % 128 == 0) &&
           (n >= b->sk_min || (L != &b->full && n >= SB_TC_MIN_ROWS));
}

/* Whether the lane's QKV projection of n rows carries RoPE and the paged KV
 * append in its output pass: it runs on the stream-K kernel, whose 128-row
 * tiles then hold whole heads. */
static int qkv_rope_fused(const slate_llama_batch_t* b, const sb_lane* L, int n) {
    const sb_matrix* W = &b->layers[0].wqkv;
    return uses_sk(b, L, W, n, SB_EPI_ROPE) && 128 % b->hd == 0 && b->hd % 2 == 0 &&
           L->op_d->K == W->K && W->M == (b->nq + 2 * b->nkv) * b->hd &&
           sb_sk_tiles(W->M_pad, n) <= sb_sk_tiles(b->layers[0].wgu.M_pad, n);
}

/* The lane's f16 operand for a GEMM input, chosen by what the input is (the
 * RMSNorm output, the SwiGLU rows, the attention output) rather than by K:
 * tensor-parallel shards can give two of them the same K (d_model = ffn / tp). */
static const sb_tc_operand* lane_op(const sb_lane* L, int in, int K) {
    if (in == IN_XN) return L->op_d;
    if (in == IN_H) return L->op_f;
    if (in == IN_ATT) return L->op_a;
    return K == L->op_d->K ? L->op_d : K == L->op_f->K ? L->op_f : L->op_a;
}

/* One weight GEMM of the step on the path chosen for (weight, rows); X and Y
 * point at the lane's first row, in names the input (IN_*). */
static int step_gemm(slate_llama_batch_t* b, sb_lane* L, const sb_matrix* W, const float* X,
                     int ldx, int in, int n, float* Y, int ldy, int epi, int splits,
                     cudaStream_t s) {
    /* the lane's operand already holds xn (att) as the f16 pair: RMSNorm (the
     * attention) wrote it */
    const int have_d = in == IN_XN && L->xn_split;
    const int have_a = in == IN_ATT && L->att_split;
    if (W == &b->lm_head && head_on_tc(b, L, n)) {
        int rc = have_d ? 0 : sb_tc_split(X, ldx, n, L->op_d, s);
        return rc ? rc : sb_tc_gemm_f16w(&b->head_tc, L->op_d, n, Y, ldy, epi, b->tc_err, s);
    }
    /* one or two rows: the CUDA-core GEMV (gemm_gv.cu), weight streaming bound */
    if (b->gv_on && n <= SB_GV_MAX_ROWS && sb_gv_supported(W, n, epi))
        return sb_gv_gemm(W, X, ldx, n, Y, ldy, epi, NULL, 0.f, NULL, NULL, b->tc_err, s);
    /* a few rows: weight streaming bound, gemm_mv.cu */
    if (L->mv_ws && W->wtype == SB_WT_Q4K && n <= SB_MV_MAX_ROWS &&
        sb_mv_gemm(W, X, ldx, n, Y, ldy, epi, L->mv_ws, L->mv_cnt, s) == 0)
        return 0;
    if (b->q4_on && W->wtype == SB_WT_Q4K && n >= SB_TC_MIN_ROWS && W->M_pad % 128 == 0) {
        const sb_q4_operand* op = in == IN_XN ? &b->q4_d : in == IN_H ? &b->q4_f
                                  : in == IN_ATT ? &b->q4_a
                                  : W->K == b->q4_d.K ? &b->q4_d
                                  : W->K == b->q4_f.K ? &b->q4_f : &b->q4_a;
        if (op->K != W->K) return -1;
        int rc = sb_q4_split(X, ldx, n, op, s);
        return rc ? rc : sb_q4_gemm(W, op, n, Y, ldy, epi, b->q4_ws, b->q4_cnt, b->tc_err, s);
    }
    const sb_tc_operand* op = lane_op(L, in, W->K);
    const int pre = (have_d && op->hi == L->op_d->hi) || (have_a && op->hi == L->op_a->hi);
    if (uses_sk(b, L, W, n, epi)) {
        if (op->K != W->K) return -1;
        /* the down GEMM's operand was written by the gate/up GEMM */
        int rc = (in == IN_H && b->sk_h) || pre ? 0 : sb_tc_split(X, ldx, n, op, s);
        const int fuse = epi == SB_EPI_SILU && b->sk_h;
        return rc ? rc : sb_sk_gemm(W, op, n, L->sk_ws, Y, ldy, epi, fuse ? L->op_f->hi : NULL,
                                    fuse ? L->op_f->lo : NULL, L->op_f->ld16, NULL, b->tc_err, s);
    }
    if (b->tc_passes && W->wtype == SB_WT_Q4K && n >= SB_TC_MIN_ROWS && W->M_pad % 128 == 0) {
        if (op->K != W->K) return -1;
        int rc = pre ? 0 : sb_tc_split(X, ldx, n, op, s);
        return rc ? rc : sb_tc_gemm(W, op, n, b->tc_passes, splits, b->tc_ws, Y, ldy, epi,
                                    b->tc_err, s);
    }
    return sb_gemm(W, X, ldx, n, Y, ldy, epi, b->gemm_path == 1 ? 1 : 0, s);
}

static int round_up(int x, int m) { return (x + m - 1) / m * m; }

static void* dalloc(slate_llama_batch_t* b, size_t bytes) {
    void* p = NULL;
    if (sb_cuda_check(cudaMalloc(&p, bytes ? bytes : 16), "cudaMalloc")) return NULL;
    if (b->n_allocs == b->cap_allocs) {
        b->cap_allocs = b->cap_allocs ? 2 * b->cap_allocs : 64;
        b->allocs = (void**)realloc(b->allocs, (size_t)b->cap_allocs * sizeof(void*));
    }
    b->allocs[b->n_allocs++] = p;
    return p;
}

/* ---- weight packing ------------------------------------------------------ */

/* Source rows of one logical matrix: rows [row0, row0 + rows) of a source
 * matrix with src_k columns, dtype 0|18, of which columns [k0, k0 + K) are
 * taken (a Q4_K column slice starts and ends on 256-column super-blocks). */
typedef struct { const void* p; int dtype; int rows; int row0; int src_k; int k0; } src_part;

static size_t q4k_row_bytes(int K) { return (size_t)(K / 256) * 144; }

/* Host staging buffer (pinned) reused across matrices. */
typedef struct { void* p; size_t cap; } stage_t;
static void* stage_get(stage_t* s, size_t bytes) {
    if (bytes > s->cap) {
        if (s->p) cudaFreeHost(s->p);
        s->p = NULL;
        if (cudaHostAlloc(&s->p, bytes, cudaHostAllocDefault) != cudaSuccess) {
            s->p = NULL;
            s->cap = 0;
            return NULL;
        }
        s->cap = bytes;
    }
    return s->p;
}

/* Packs parts (concatenated rows) into one device matrix.  interleave64 puts
 * part 0 (gate) and part 1 (up) in alternating 64-row groups for the fused
 * SwiGLU epilogue.  All-Q4_K groups stay Q4_K; any f32 part makes the whole
 * matrix f32 (Q4_K parts dequantised exactly). */
/* llama.cpp / ggml nibble packing of one Q4_K block -> Slate's
 * (util/quant.c:182-199): ggml byte 32g + e holds element e of sub-block 2g in
 * its low nibble and of 2g + 1 in its high nibble; Slate's byte 16s + i holds
 * elements i (low) and i + 16 (high) of sub-block s. */
static void q4k_from_ggml(uint8_t* dst, const uint8_t* src) {
    memcpy(dst, src, 16);                        /* d, dmin, packed scales: same */
    uint8_t e[8][32];
    for (int g = 0; g < 4; ++g)
        for (int i = 0; i < 32; ++i) {
            e[2 * g][i] = src[16 + 32 * g + i] & 15;
            e[2 * g + 1][i] = src[16 + 32 * g + i] >> 4;
        }
    for (int sb = 0; sb < 8; ++sb)
        for (int i = 0; i < 16; ++i) dst[16 + 16 * sb + i] = (uint8_t)(e[sb][i] | (e[sb][i + 16] << 4));
}

/* Exponent e (0..24) for the tensor-core split of a Q4_K matrix: the largest
 * with every weight below 2^13 after scaling by 2^e, from the block headers
 * (|d*sc*q - dmin*m| <= |d|*63*15 + |dmin|*63).  An f16 lo half of a weight
 * near 0.02 (~1e-5) is subnormal and keeps ~7 of its 11 bits; scaled, it
 * keeps all of them. */
static int q4k_wexp(const unsigned char* p, size_t nblocks) {
    float mx = 0.f;
    for (size_t i = 0; i < nblocks; ++i) {
        uint16_t dh, mh;
        memcpy(&dh, p + 144 * i, 2);
        memcpy(&mh, p + 144 * i + 2, 2);
        const float bnd = fabsf(sb_f16_to_f32(dh)) * 945.0f + fabsf(sb_f16_to_f32(mh)) * 63.0f;
        if (bnd > mx) mx = bnd;
    }
    if (!(mx > 0.f) || !isfinite(mx)) return 0;
    const int e = (int)floorf(log2f(8192.0f / mx));
    return e < 0 ? 0 : e > 24 ? 24 : e;
}

static int pack_matrix(slate_llama_batch_t* b, stage_t* st, sb_matrix* out, const src_part* parts,
                       int nparts, int K, int interleave64) {
    int all_q4k = 1, M = 0;
    for (int i = 0; i < nparts; ++i) {
        if (parts[i].dtype != 0 && parts[i].dtype != 1 && parts[i].dtype != 18) {
            sb_set_error("unsupported weight dtype %d", parts[i].dtype);
            return -1;
        }
        if (parts[i].dtype != 18) all_q4k = 0;
        M += parts[i].rows;
    }
    if (all_q4k && K % 256) all_q4k = 0;
    int per_part_pad = 0;
    if (interleave64) {
        per_part_pad = round_up(parts[0].rows, 64);
        M = 2 * per_part_pad;
    }
    const int M_pad = round_up(M, 128);
    out->wtype = all_q4k ? SB_WT_Q4K : SB_WT_F32;
    out->M = M;
    out->M_pad = M_pad;
    out->K = K;
    out->ldw = all_q4k ? 0 : round_up(K, 128);
    out->wexp = 0;
    const size_t row_bytes = all_q4k ? q4k_row_bytes(K) : (size_t)out->ldw * 4;
    const size_t bytes = row_bytes * (size_t)M_pad;
    if (nparts == 1 && !interleave64 && parts[0].src_k == K && !(all_q4k && b->q4k_order) &&
        (all_q4k || (parts[0].dtype == 0 && out->ldw == K))) {
        /* already in the device layout: copy rows straight from the source */
        unsigned char* dptr = (unsigned char*)dalloc(b, bytes);
        if (!dptr) return -5;
        const unsigned char* src = (const unsigned char*)parts[0].p + (size_t)parts[0].row0 * row_bytes;
        if (all_q4k) out->wexp = q4k_wexp(src, (size_t)M * (K / 256));
        SB_CU(cudaMemcpy(dptr, src, row_bytes * (size_t)M, cudaMemcpyHostToDevice));
        if (M_pad > M) SB_CU(cudaMemset(dptr + row_bytes * (size_t)M, 0, row_bytes * (size_t)(M_pad - M)));
        out->data = dptr;
        return 0;
    }
    unsigned char* h = (unsigned char*)stage_get(st, bytes);
    if (!h) {
        sb_set_error("pinned staging of %zu bytes failed", bytes);
        return -5;
    }
    memset(h, 0, bytes);
    /* destination row of source row r of part i */
    for (int i = 0, base = 0; i < nparts; ++i) {
        const src_part* sp = &parts[i];
        const size_t esz = sp->dtype == 1 ? 2 : 4;
        const size_t src_row = sp->dtype == 18 ? q4k_row_bytes(sp->src_k) : (size_t)sp->src_k * esz;
        const size_t col0 = sp->dtype == 18 ? q4k_row_bytes(sp->k0) : (size_t)sp->k0 * esz;
        for (int r = 0; r < sp->rows; ++r) {
            int dr;
            if (interleave64) dr = (r / 64) * 128 + (i ? 64 : 0) + r % 64;
            else dr = base + r;
            const unsigned char* s =
                (const unsigned char*)sp->p + (size_t)(sp->row0 + r) * src_row + col0;
            unsigned char* d = h + (size_t)dr * row_bytes;
            if (sp->dtype == 18 && b->q4k_order) {
                /* repack each block to Slate's order (into d, or a temp row
                 * that is then dequantised) */
                uint8_t* q = all_q4k ? (uint8_t*)d : (uint8_t*)malloc(q4k_row_bytes(K));
                if (!q) return -5;
                for (int blk = 0; blk < K / 256; ++blk) q4k_from_ggml(q + 144 * blk, s + 144 * blk);
                if (!all_q4k) {
                    sb_q4k_dequant_rows((float*)d, q, 1, K);
                    free(q);
                }
            } else if (all_q4k) {
                memcpy(d, s, q4k_row_bytes(K));
            } else if (sp->dtype == 0) {
                memcpy(d, s, (size_t)K * 4);
            } else if (sp->dtype == 1) {
                const uint16_t* h16 = (const uint16_t*)s;
                for (int k = 0; k < K; ++k) ((float*)d)[k] = sb_f16_to_f32(h16[k]);
            } else {
                sb_q4k_dequant_rows((float*)d, s, 1, K);
            }
        }
        base += sp->rows;
    }
    if (all_q4k) out->wexp = q4k_wexp(h, (size_t)M_pad * (K / 256));
    void* dptr = dalloc(b, bytes);
    if (!dptr) return -5;
    SB_CU(cudaMemcpy(dptr, h, bytes, cudaMemcpyHostToDevice));
    out->data = dptr;
    return 0;
}

static int upload_f32(slate_llama_batch_t* b, float** dst, const void* src, size_t n) {
    *dst = (float*)dalloc(b, n * 4);
    if (!*dst) return -5;
    SB_CU(cudaMemcpy(*dst, src, n * 4, cudaMemcpyHostToDevice));
    return 0;
}

/* ---- step enqueue ------------------------------------------------------- */

/* Layer l of a step for the lane's n rows (rows r0 .. r0 + n - 1), in three
 * parts: 0 = RMSNorm, QKV projection, RoPE + KV append; 1 = attention; 2 = Wo
 * (+ residual), RMSNorm, gate/up (SiLU), down (+ residual). */
static int enqueue_part(slate_llama_batch_t* b, sb_lane* L, int l, int part, int n, cudaStream_t s) {
    int rc = 0;
    /* Wo and down add into the residual stream; tensor parallel ranks hold
     * partial sums that are all-reduced into it, with rank 0 alone adding the
     * residual itself */
    const int res_epi = b->tp > 1 && b->rank != 0 ? SB_EPI_STORE : SB_EPI_ADD;
    const int r0 = L->r0;
    float* x = b->x + (size_t)r0 * b->ld_x;
    float* xn = b->xn + (size_t)r0 * b->ld_x;
    float* qkv = b->qkv + (size_t)r0 * b->ld_qkv;
    float* att = b->att + (size_t)r0 * b->ld_att;
    float* h = b->h + (size_t)r0 * b->ld_h;
    const int32_t* row_pos = b->row_pos + r0;
    const int32_t* row_slot = b->row_slot + r0;
    const sb_layer* ly = &b->layers[l];
    if (part == 0) {
        if (norm_in_gemv(b, &ly->wqkv, n, SB_EPI_ROPE)) {
            /* one launch: RMSNorm in the GEMV's staging of x, RoPE + the KV
             * append in its epilogue */
            const sb_rope_args ra = {row_pos, row_slot, b->page_table, b->pool, b->rope_cos,
                                     b->rope_sin, b->n_pages, b->max_pages, l, b->kv_dtype,
                                     b->nq, b->nkv, b->hd};
            L->xn_split = 0;
            rc |= sb_gv_gemm(&ly->wqkv, x, b->ld_x, n, qkv, b->ld_qkv, SB_EPI_ROPE, ly->attn_norm,
                             b->eps, &ra, b->head_cnt, b->tc_err, s);
            return rc;
        }
        rc |= step_norm(b, L, ly->attn_norm, n, s);
        if (qkv_rope_fused(b, L, n)) {
            /* RoPE and the KV append in the stream-K GEMM's output pass */
            const sb_tc_operand* op = L->op_d;
            const sb_rope_args ra = {row_pos, row_slot, b->page_table, b->pool, b->rope_cos,
                                     b->rope_sin, b->n_pages, b->max_pages, l, b->kv_dtype,
                                     b->nq, b->nkv, b->hd};
            if (!L->xn_split) rc |= sb_tc_split(xn, b->ld_x, n, op, s);
            rc |= sb_sk_gemm(&ly->wqkv, op, n, L->sk_ws, qkv, b->ld_qkv, SB_EPI_ROPE, NULL, NULL, 0,
                             &ra, b->tc_err, s);
        } else {
            rc |= step_gemm(b, L, &ly->wqkv, xn, b->ld_x, IN_XN, n, qkv, b->ld_qkv, SB_EPI_STORE,
                            b->sp_qkv, s);
            rc |= sb_rope_append(qkv, b->ld_qkv, n, b->nq, b->nkv, b->hd, row_pos, row_slot,
                                 b->page_table, b->max_pages, b->pool, b->n_pages, l, b->kv_dtype,
                                 b->rope_cos, b->rope_sin, s);
        }
    } else if (part == 1) {
        /* the second lane's partials sit after a whole batch's */
        float* scratch = b->scratch + (r0 ? sb_attention_scratch_floats(b->max_batch, b->nq, b->hd,
                                                                         b->max_seq)
                                          : 0);
        L->att_split = norm_splits(b, L, n) && L->op_a->ld16 >= b->Dq;
        if (b->chunk_step)   /* rows: consecutive positions of one sequence */
            rc |= sb_attention_paged_prefill(att, b->ld_att, qkv, b->ld_qkv, n, b->nq, b->nkv, b->hd,
                                             row_pos, row_slot, b->page_table, b->max_pages,
                                             b->pool, b->kvmap_p, b->n_pages, l, b->kv_dtype,
                                             b->max_seq, scratch, b->tc_err,
                                             L->att_split ? L->op_a->hi : NULL,
                                             L->att_split ? L->op_a->lo : NULL, L->op_a->ld16, s);
        else if (L->att_split)
            rc |= sb_attention_paged_split(att, b->ld_att, qkv, b->ld_qkv, n, b->nq, b->nkv, b->hd,
                                           row_pos, row_slot, b->page_table, b->max_pages, b->pool,
                                           b->kvmap_p, b->n_pages, l, b->kv_dtype, b->max_seq,
                                           scratch, b->tc_err, L->op_a->hi, L->op_a->lo,
                                           L->op_a->ld16, s);
        else
            rc |= sb_attention_paged(att, b->ld_att, qkv, b->ld_qkv, n, b->nq, b->nkv, b->hd, row_pos,
                                     row_slot, b->page_table, b->max_pages, b->pool, b->kvmap_p,
                                     b->n_pages, l, b->kv_dtype, b->max_seq, 0, scratch, b->tc_err,
                                     s);
    } else {
        rc |= step_gemm(b, L, &ly->wo, att, b->ld_att, IN_ATT, n, x, b->ld_x, res_epi, b->sp_wo, s);
        if (b->tp > 1) rc |= sb_tp_allreduce_sum(L->comm, x, (size_t)n * b->ld_x, s);
        if (norm_in_gemv(b, &ly->wgu, n, SB_EPI_SILU)) {
            /* RMSNorm in the GEMV's staging of x */
            L->xn_split = 0;
            rc |= sb_gv_gemm(&ly->wgu, x, b->ld_x, n, h, b->ld_h, SB_EPI_SILU, ly->ffn_norm, b->eps,
                             NULL, NULL, b->tc_err, s);
        } else {
            rc |= step_norm(b, L, ly->ffn_norm, n, s);
            rc |= step_gemm(b, L, &ly->wgu, xn, b->ld_x, IN_XN, n, h, b->ld_h, SB_EPI_SILU, b->sp_gu,
                            s);
        }
        rc |= step_gemm(b, L, &ly->wdown, h, b->ld_h, IN_H, n, x, b->ld_x, res_epi, b->sp_dn, s);
        if (b->tp > 1) rc |= sb_tp_allreduce_sum(L->comm, x, (size_t)n * b->ld_x, s);
    }
    return rc;
}

/* All layers of a step for one lane. */
static int enqueue_layers(slate_llama_batch_t* b, sb_lane* L, int n, cudaStream_t s) {
    int rc = 0;
    for (int l = 0; l < b->L && !rc; ++l)
        for (int part = 0; part < 3 && !rc; ++part) rc |= enqueue_part(b, L, l, part, n, s);
    return rc;
}

/* Two lanes, interleaved: the halves' attentions take turns (A's layer l,
 * then B's layer l, then A's layer l + 1, ...), so each runs beside the other
 * half's projections instead of beside the other attention. */
static int enqueue_lanes(slate_llama_batch_t* b, int n, cudaStream_t s) {
    sb_lane* A = &b->half[0];
    sb_lane* Bl = &b->half[1];
    const int na = b->half_rows, nb = n - b->half_rows;
    cudaStream_t s2 = b->stream2;
    int rc = sb_cuda_check(cudaEventRecord(b->ev_fork, s), "fork");
    rc |= sb_cuda_check(cudaStreamWaitEvent(s2, b->ev_fork, 0), "fork");
    for (int l = 0; l < b->L && !rc; ++l) {
        rc |= enqueue_part(b, A, l, 0, na, s);
        if (l > 0) rc |= sb_cuda_check(cudaStreamWaitEvent(s, b->ev_b, 0), "lane order");
        rc |= enqueue_part(b, A, l, 1, na, s);
        rc |= sb_cuda_check(cudaEventRecord(b->ev_a, s), "lane order");
        rc |= enqueue_part(b, A, l, 2, na, s);
        rc |= enqueue_part(b, Bl, l, 0, nb, s2);
        rc |= sb_cuda_check(cudaStreamWaitEvent(s2, b->ev_a, 0), "lane order");
        rc |= enqueue_part(b, Bl, l, 1, nb, s2);
        rc |= sb_cuda_check(cudaEventRecord(b->ev_b, s2), "lane order");
        rc |= enqueue_part(b, Bl, l, 2, nb, s2);
    }
    rc |= sb_cuda_check(cudaEventRecord(b->ev_join, s2), "join");
    rc |= sb_cuda_check(cudaStreamWaitEvent(s, b->ev_join, 0), "join");
    return rc;
}

/* Whether a step of n rows runs as two lanes. */
static int step_dual(const slate_llama_batch_t* b, int n) {
    return b->dual && n > b->half_rows;
}

static int enqueue_step(slate_llama_batch_t* b, int n, int sample, int chunk, int head,
                        cudaStream_t s) {
    int rc = 0;
    /* cudaGetLastError() below must only see this step's launches: a failure
     * left by an earlier unchecked call on this thread is cleared here (a
     * sticky device fault would still fail every call that follows). */
    (void)cudaGetLastError();
    const int32_t* slots = b->d_io;
    const int32_t* toks = b->d_io + b->max_batch;
    int32_t* out = b->d_io + 2 * b->max_batch;
    rc |= sb_step_prologue(slots, toks, n, b->pos, b->page_table, b->max_pages, b->free_stack,
                           b->free_top, b->max_slots, b->max_seq, b->V, b->emb, b->D, b->x,
                           b->ld_x, b->row_pos, b->row_slot, b->status, chunk, s);
    b->chunk_step = chunk;
    if (!chunk && step_dual(b, n)) {
        /* rows [0, half_rows) on this stream, [half_rows, n) on the second */
        rc |= enqueue_lanes(b, n, s);
    } else {
        rc |= enqueue_layers(b, &b->full, n, s);
    }
    if (!head) {
        /* a prompt chunk whose logits nobody reads: positions only */
        rc |= sb_step_advance(b->row_slot, b->row_pos, b->pos, b->status, n, s);
        if (rc) {
            sb_set_error("kernel launch rejected its arguments");
            return -1;
        }
        return sb_cuda_check(cudaGetLastError(), "step launch");
    }
    rc |= step_norm(b, &b->full, b->out_norm, n, s);
    rc |= step_gemm(b, &b->full, &b->lm_head, b->xn, b->ld_x, IN_XN, n, b->logits, b->ld_logits,
                    SB_EPI_STORE, 1, s);
    if (sample) {
        rc |= sb_sample_rows(b->logits, b->ld_logits, b->V, n, b->d_samp, b->d_rng, b->samp_scratch,
                             out, b->row_slot, b->row_pos, b->pos, b->status, b->tc_err, s);
    } else if (b->tp > 1) {
        rc |= sb_argmax_pairs(b->logits, b->ld_logits, b->V_l, n, b->v0, b->pairs, s);
        rc |= sb_tp_allgather(b->comm, b->pairs, b->pairs_all, (size_t)n * 8, s);
        rc |= sb_tp_epilogue(b->pairs_all, b->tp, n, b->row_slot, b->row_pos, b->pos, b->status,
                             out, s);
    } else {
        rc |= sb_step_epilogue(b->logits, b->ld_logits, b->V, n, b->row_slot, b->row_pos, b->pos,
                               b->status, out, s);
    }
    if (rc) {
        sb_set_error("kernel launch rejected its arguments");
        return -1;
    }
    return sb_cuda_check(cudaGetLastError(), "step launch");
}

/* Kernel launches step_gemm makes for (lane, W, n rows, epilogue, splits);
 * pre: the GEMM's input comes from a kernel that can write its f16 split
 * (RMSNorm, attention). */
static int gemm_launches(const slate_llama_batch_t* b, const sb_lane* L, const sb_matrix* W, int n,
                         int epi, int splits, int pre) {
    const int split = pre && norm_splits(b, L, n) ? 0 : 1;
    if (W == &b->lm_head && head_on_tc(b, L, n)) return split + 1;
    if (b->gv_on && n <= SB_GV_MAX_ROWS && sb_gv_supported(W, n, epi)) return 1;
    if (L->mv_ws && W->wtype == SB_WT_Q4K && n <= SB_MV_MAX_ROWS) return 1;
    if (b->q4_on && W->wtype == SB_WT_Q4K && n >= SB_TC_MIN_ROWS && W->M_pad % 128 == 0)
        return 2;                                                               /* split + GEMM */
    if (uses_sk(b, L, W, n, epi))
        return (W == &b->layers[0].wdown && b->sk_h ? 0 : split) +   /* split (down: fused) */
               sb_sk_kernels(W->M_pad, W->K, n, epi);              /* GEMM (+ output pass) */
    if (b->tc_passes && W->wtype == SB_WT_Q4K && n >= SB_TC_MIN_ROWS && W->M_pad % 128 == 0)
        return split + 1 + (splits == 1 && epi != SB_EPI_SILU ? 0 : 1);      /* + finish */
    return 1;
}

/* Kernel launches of one lane's layers for n rows. */
static int layer_launches(const slate_llama_batch_t* b, const sb_lane* L, int n) {
    const sb_layer* l0 = &b->layers[0];
    const int res_epi = b->tp > 1 && b->rank != 0 ? SB_EPI_STORE : SB_EPI_ADD;
    const int qkv = norm_in_gemv(b, &l0->wqkv, n, SB_EPI_ROPE) ? 1
                    : qkv_rope_fused(b, L, n)
                        ? (norm_splits(b, L, n) ? 0 : 1) + sb_sk_kernels(l0->wqkv.M_pad, l0->wqkv.K, n,
                                                                         SB_EPI_ROPE)
                        : 1 /* rope + append */ + gemm_launches(b, L, &l0->wqkv, n, SB_EPI_STORE,
                                                                b->sp_qkv, 1);
    const int norms = (norm_in_gemv(b, &l0->wqkv, n, SB_EPI_ROPE) ? 0 : 1) +
                      (norm_in_gemv(b, &l0->wgu, n, SB_EPI_SILU) ? 0 : 1);
    const int per_layer =
        norms /* rmsnorm */ + 2 /* attention */ + qkv +
        gemm_launches(b, L, &l0->wo, n, res_epi, b->sp_wo, L->op_a->ld16 >= b->Dq) +
        gemm_launches(b, L, &l0->wgu, n, SB_EPI_SILU, b->sp_gu, 1) +
        gemm_launches(b, L, &l0->wdown, n, res_epi, b->sp_dn, 0);
    return b->L * per_layer;
}

int slate_llama_batch_launches_per_step(const slate_llama_batch_t* b, int n) {
    if (!b || n < 1) return 0;
    const int layers = step_dual(b, n) ? layer_launches(b, &b->half[0], b->half_rows) +
                                             layer_launches(b, &b->half[1], n - b->half_rows)
                                       : layer_launches(b, &b->full, n);
    return 1 /* prologue */ + layers + 1 /* final rmsnorm */ +
           gemm_launches(b, &b->full, &b->lm_head, n, SB_EPI_STORE, 1, 1) + (b->tp > 1 ? 2 : 1);
}

/* Runs the step for n rows whose metadata is already in d_io; sample != 0
 * ends it with the stochastic sampler instead of the greedy argmax; chunk != 0
 * lets a slot occur several times (a prompt chunk, one lane), otherwise a
 * repeated slot is rejected (status -1) and the rows may run as two lanes. */
static int run_step_mode(slate_llama_batch_t* b, int n, int sample, int chunk, int head) {
    if (!b->use_graphs) return enqueue_step(b, n, sample, chunk, head, b->stream);
    cudaGraphExec_t* slot = chunk ? (head ? &b->graphs_c[n] : &b->graphs_p[n])
                            : sample ? &b->graphs_s[n] : &b->graphs[n];
    if (!*slot) {
        cudaGraph_t g = NULL;
        SB_CU(cudaStreamBeginCapture(b->stream, cudaStreamCaptureModeThreadLocal));
        int rc = enqueue_step(b, n, sample, chunk, head, b->stream);
        cudaError_t e = cudaStreamEndCapture(b->stream, &g);
        if (rc) {
            if (g) cudaGraphDestroy(g);
            return rc;
        }
        SB_CU(e);
        e = cudaGraphInstantiate(slot, g, 0);
        cudaGraphDestroy(g);
        SB_CU(e);
    }
    SB_CU(cudaGraphLaunch(*slot, b->stream));
    return 0;
}
static int run_step(slate_llama_batch_t* b, int n) { return run_step_mode(b, n, 0, 0, 1); }

/* ---- construction ------------------------------------------------------- */

void slate_llama_batch_free(slate_llama_batch_t* b) {
    if (!b) return;
    cudaSetDevice(b->device);
    if (b->stream) cudaStreamSynchronize(b->stream);
    if (b->stream2) cudaStreamSynchronize(b->stream2);
    if (b->graphs) {
        for (int i = 0; i <= b->max_batch; ++i)
            if (b->graphs[i]) cudaGraphExecDestroy(b->graphs[i]);
        free(b->graphs);
    }
    if (b->graphs_s) {
        for (int i = 0; i <= b->max_batch; ++i)
            if (b->graphs_s[i]) cudaGraphExecDestroy(b->graphs_s[i]);
        free(b->graphs_s);
    }
    if (b->graphs_c) {
        for (int i = 0; i <= b->max_batch; ++i)
            if (b->graphs_c[i]) cudaGraphExecDestroy(b->graphs_c[i]);
        free(b->graphs_c);
    }
    if (b->graphs_p) {
        for (int i = 0; i <= b->max_batch; ++i)
            if (b->graphs_p[i]) cudaGraphExecDestroy(b->graphs_p[i]);
        free(b->graphs_p);
    }
    if (b->h_samp) cudaFreeHost(b->h_samp);
    if (b->h_rng) cudaFreeHost(b->h_rng);
    sb_tc_free_weight(&b->head_tc);
    if (b->comm2) sb_tp_destroy(b->comm2);
    if (b->comm) sb_tp_destroy(b->comm);      /* after the graphs that hold its collectives */
    for (int i = 0; i < b->n_allocs; ++i) cudaFree(b->allocs[i]);
    free(b->allocs);
    if (b->h_io) cudaFreeHost(b->h_io);
    if (b->stream) cudaStreamDestroy(b->stream);
    if (b->stream2) cudaStreamDestroy(b->stream2);
    if (b->ev_fork) cudaEventDestroy(b->ev_fork);
    if (b->ev_join) cudaEventDestroy(b->ev_join);
    if (b->ev_a) cudaEventDestroy(b->ev_a);
    if (b->ev_b) cudaEventDestroy(b->ev_b);
    free(b->layers);
    free(b->h_pos);
    free(b->h_open);
    pthread_mutex_destroy(&b->lock);
    free(b);
}

slate_llama_batch_t* slate_llama_batch_new_desc(const slate_llama_desc_t* m,
                                                const slate_cuda_opts_t* o) {
    if (!m || !o) { sb_set_error("NULL model or options"); return NULL; }
    const int L = m->n_layers, D = m->d_model, F = m->ffn_hidden, nq = m->n_heads,
              nkv = m->n_kv_heads, hd = m->head_dim, V = m->vocab;
    if (L < 1 || D < 1 || F < 1 || nq < 1 || nkv < 1 || nq % nkv || hd * nq != D || V < 1 ||
        !m->token_embd || !m->output_norm || !m->output || !m->layers) {
        sb_set_error("inconsistent model description");
        return NULL;
    }
    if (hd != 8 && hd != 16 && hd != 32 && hd != 64 && hd != 128) {
        sb_set_error("head_dim %d unsupported (8, 16, 32, 64, 128)", hd);
        return NULL;
    }
    const int G = nq / nkv;
    if (G != 1 && G != 2 && G != 4 && G != 8) {
        sb_set_error("GQA group %d unsupported (1, 2, 4, 8)", G);
        return NULL;
    }
    if (m->token_embd_dtype != 0 && m->token_embd_dtype != 1) {
        sb_set_error("token_embd must be f32 or f16");
        return NULL;
    }
    if (o->max_batch < 1 || o->max_batch > 1024) {
        sb_set_error("max_batch %d out of range", o->max_batch);
        return NULL;
    }
    const int tp = o->tp_size > 1 ? o->tp_size : 1, rank = tp > 1 ? o->tp_rank : 0;
    if (tp > 1) {
        /* column slices of Wo (K = nq*hd) and down (K = F) must stay whole
         * Q4_K super-blocks; heads, kv heads and vocabulary split evenly */
        if (rank < 0 || rank >= tp || nkv % tp || V % tp || F % (256 * tp) ||
            ((nq / tp) * hd) % 256) {
            sb_set_error("tensor parallel %d (rank %d) needs n_kv_heads, vocab, ffn/256 and "
                         "(n_heads/tp)*head_dim/256 divisible", tp, rank);
            return NULL;
        }
    }
    /* the struct holds TMA descriptors, which must be 64-byte aligned */
    const size_t bsize = (sizeof(slate_llama_batch_t) + 63) / 64 * 64;
    slate_llama_batch_t* b = (slate_llama_batch_t*)aligned_alloc(64, bsize);
    if (!b) {
        sb_set_error("out of host memory");
        return NULL;
    }
    memset(b, 0, bsize);
    pthread_mutex_init(&b->lock, NULL);
    b->device = o->device;
    b->tp = tp;
    b->rank = rank;
    /* this rank's share: heads, kv heads, FFN units, vocabulary rows */
    b->L = L; b->D = D; b->F = F / tp; b->nq = nq / tp; b->nkv = nkv / tp; b->hd = hd; b->V = V;
    b->V_l = V / tp;
    b->v0 = rank * b->V_l;
    b->Dq = b->nq * hd;
    b->kvd = b->nkv * hd;
    b->qkv_dim = b->Dq + 2 * b->kvd;
    b->theta = m->theta_base;
    b->eps = m->rms_eps;
    b->max_seq = o->max_seq > 0 ? o->max_seq : m->max_seq;
    b->max_batch = o->max_batch;
    b->max_slots = o->max_slots > 0 ? o->max_slots : o->max_batch;
    b->kv_dtype = o->kv_dtype == SLATE_KV_F16 ? SLATE_KV_F16 : SLATE_KV_F32;
    b->gemm_path = o->gemm_path;
    b->q4k_order = o->q4k_order == 1;
    /* tensor-parallel steps are launched eagerly: their NCCL collectives set
     * up connections lazily, which stream capture does not allow */
    b->use_graphs = tp > 1 ? 0 : o->use_graphs;
    b->max_pages = (b->max_seq + SB_PAGE_TOKENS - 1) / SB_PAGE_TOKENS;
    stage_t stg = {NULL, 0};

    if (sb_cuda_check(cudaSetDevice(b->device), "cudaSetDevice") ||
        sb_cuda_check(cudaStreamCreateWithFlags(&b->stream, cudaStreamNonBlocking), "stream"))
        goto fail;
    if (tp > 1 && sb_tp_init(&b->comm, tp, rank, o->tp_id)) goto fail;
    sb_gemm_prepare();
    sb_tc_prepare();
    sb_gv_prepare();
    b->gv_on = o->gemm_path == 0;
    if (sb_attention_prepare(b->nq, b->nkv, hd, b->kv_dtype)) {
        sb_set_error("no attention kernel for head_dim %d, group %d", hd, nq / nkv);
        goto fail;
    }

    /* weights (an f16 embedding table is widened to f32 once, exactly) */
    if (m->token_embd_dtype == 1) {
        float* e32 = (float*)malloc((size_t)V * D * 4);
        if (!e32) { sb_set_error("host memory for the f16 embedding"); goto fail; }
        const uint16_t* e16 = (const uint16_t*)m->token_embd;
        for (size_t i = 0; i < (size_t)V * D; ++i) e32[i] = sb_f16_to_f32(e16[i]);
        const int rc_e = upload_f32(b, &b->emb, e32, (size_t)V * D);
        free(e32);
        if (rc_e) goto fail;
    } else if (upload_f32(b, &b->emb, m->token_embd, (size_t)V * D)) {
        goto fail;
    }
    if (upload_f32(b, &b->out_norm, m->output_norm, (size_t)D)) goto fail;
    if (m->output == m->token_embd && m->output_dtype == m->token_embd_dtype && D % 128 == 0 &&
        b->V_l % 128 == 0) {
        /* tied: share the table (this rank's vocabulary rows) */
        b->lm_head = (sb_matrix){SB_WT_F32, b->emb + (size_t)b->v0 * D, b->V_l, b->V_l, D, D, 0};
    } else {
        src_part p = {m->output, m->output_dtype, b->V_l, b->v0, D, 0};
        if (pack_matrix(b, &stg, &b->lm_head, &p, 1, D, 0)) goto fail;
    }
    b->layers = (sb_layer*)calloc((size_t)L, sizeof(sb_layer));
    for (int l = 0; l < L; ++l) {
        const slate_llama_layer_desc_t* s = m->layers[l];
        sb_layer* ly = &b->layers[l];
        if (!s) { sb_set_error("layer %d missing", l); goto fail; }
        if (upload_f32(b, &ly->attn_norm, s->attn_norm, (size_t)D) ||
            upload_f32(b, &ly->ffn_norm, s->ffn_norm, (size_t)D))
            goto fail;
        /* rows of this rank's heads / FFN units; Wo and down take the matching
         * column slice (with tp == 1 every part is the whole matrix) */
        const int Fl = b->F;
        src_part qkv[3] = {{s->attn_q, s->attn_q_dtype, b->Dq, rank * b->Dq, D, 0},
                           {s->attn_k, s->attn_k_dtype, b->kvd, rank * b->kvd, D, 0},
                           {s->attn_v, s->attn_v_dtype, b->kvd, rank * b->kvd, D, 0}};
        src_part wo = {s->attn_output, s->attn_output_dtype, D, 0, D, rank * b->Dq};
        src_part gu[2] = {{s->ffn_gate, s->ffn_gate_dtype, Fl, rank * Fl, D, 0},
                          {s->ffn_up, s->ffn_up_dtype, Fl, rank * Fl, D, 0}};
        src_part dn = {s->ffn_down, s->ffn_down_dtype, D, 0, F, rank * Fl};
        if (pack_matrix(b, &stg, &ly->wqkv, qkv, 3, D, 0) ||
            pack_matrix(b, &stg, &ly->wo, &wo, 1, b->Dq, 0) ||
            pack_matrix(b, &stg, &ly->wgu, gu, 2, D, 1) ||
            pack_matrix(b, &stg, &ly->wdown, &dn, 1, Fl, 0))
            goto fail;
    }
    if (stg.p) cudaFreeHost(stg.p);
    stg.p = NULL;

    /* RoPE tables with the reference's exact f32 expressions (llama_infer.c:83-85). */
    {
        const int half = hd / 2;
        size_t n = (size_t)b->max_seq * half;
        float* c = (float*)malloc(n * 4);
        float* sn = (float*)malloc(n * 4);
        for (int p = 0; p < b->max_seq; ++p)
            for (int i = 0; i < half; ++i) {
                float inv_freq = powf(b->theta, -2.0f * (float)i / (float)hd);
                float angle = (float)p * inv_freq;
                c[(size_t)p * half + i] = cosf(angle);
                sn[(size_t)p * half + i] = sinf(angle);
            }
        int rc = upload_f32(b, &b->rope_cos, c, n) | upload_f32(b, &b->rope_sin, sn, n);
        free(c);
        free(sn);
        if (rc) goto fail;
    }

    /* activations */
    {
        const int Dp = round_up(D, 128);
        const int B = b->max_batch;
        b->ld_x = Dp;
        b->ld_att = round_up(b->Dq, 128);
        b->ld_qkv = round_up(b->layers[0].wqkv.M_pad, 4);
        b->ld_h = round_up(b->layers[0].wgu.M_pad / 2, 128);
        b->ld_logits = round_up(b->lm_head.M_pad, 4);
        /* attention partials: one batch's, twice when the halves may run as lanes */
        size_t scr = sb_attention_scratch_floats(B, b->nq, hd, b->max_seq) * (o->lanes == 2 ? 2 : 1);
        b->x = (float*)dalloc(b, (size_t)B * b->ld_x * 4);
        b->xn = (float*)dalloc(b, (size_t)B * b->ld_x * 4);
        b->att = (float*)dalloc(b, (size_t)B * b->ld_att * 4);
        b->qkv = (float*)dalloc(b, (size_t)B * b->ld_qkv * 4);
        b->h = (float*)dalloc(b, (size_t)B * b->ld_h * 4);
        b->logits = (float*)dalloc(b, (size_t)B * b->ld_logits * 4);
        b->scratch = (float*)dalloc(b, scr * 4);
        b->row_pos = (int32_t*)dalloc(b, (size_t)B * 4);
        b->row_slot = (int32_t*)dalloc(b, (size_t)B * 4);
        b->d_io = (int32_t*)dalloc(b, (size_t)3 * B * 4);
        b->status = (int32_t*)dalloc(b, 16);
        b->tc_err = (int*)dalloc(b, 16);        /* pipeline-wait timeouts of any kernel */
        b->head_cnt = (int*)dalloc(b, (size_t)(b->nq + 2 * b->nkv) * 4);
        if (!b->x || !b->xn || !b->att || !b->qkv || !b->h || !b->logits || !b->scratch ||
            !b->row_pos || !b->row_slot || !b->d_io || !b->status || !b->tc_err || !b->head_cnt ||
            sb_cuda_check(cudaMemset(b->tc_err, 0, 16), "memset") ||
            sb_cuda_check(cudaMemset(b->head_cnt, 0, (size_t)(b->nq + 2 * b->nkv) * 4), "memset"))
            goto fail;
        /* zero padding columns are part of the GEMM contract */
        if (sb_cuda_check(cudaMemset(b->x, 0, (size_t)B * b->ld_x * 4), "memset") ||
            sb_cuda_check(cudaMemset(b->xn, 0, (size_t)B * b->ld_x * 4), "memset") ||
            sb_cuda_check(cudaMemset(b->att, 0, (size_t)B * b->ld_att * 4), "memset") ||
            sb_cuda_check(cudaMemset(b->h, 0, (size_t)B * b->ld_h * 4), "memset") ||
            sb_cuda_check(cudaMemset(b->qkv, 0, (size_t)B * b->ld_qkv * 4), "memset") ||
            sb_cuda_check(cudaMemset(b->status, 0, 16), "memset") ||
            sb_cuda_check(cudaMemset(b->d_io, 0, (size_t)3 * B * 4), "memset"))
            goto fail;
        if (sb_cuda_check(cudaHostAlloc((void**)&b->h_io, (size_t)(3 * B + 4) * 4,
                                        cudaHostAllocDefault), "cudaHostAlloc"))
            goto fail;
        if (tp > 1) {
            b->pairs = dalloc(b, (size_t)B * 8);
            b->pairs_all = dalloc(b, (size_t)tp * B * 8);
            if (!b->pairs || !b->pairs_all) goto fail;
        }
    }

    /* tensor-core path: gemm_path 0 (auto: the stream-K kernel from 128 rows,
     * gemm_tc.cu's kernel below), 3 (gemm_tc.cu's kernel only), 4 (exact-
     * weight kernel; 3-pass split for the f32 LM head) and 5 (stream-K kernel
     * from 16 rows) use the 3-pass split, 2 the single f16 pass, 1 keeps every
     * GEMM on the CUDA cores */
    b->tc_passes = o->gemm_path == 1 ? 0 : o->gemm_path == 2 ? 1 : 3;
    if (b->layers[0].wqkv.wtype != SB_WT_Q4K || D % 256 || b->F % 256 || b->Dq % 256)
        b->tc_passes = 0;
    if (b->tc_passes) {
        const int B = b->max_batch, lo = b->tc_passes == 3;
        /* f16 (hi, lo) staging of the GEMM inputs: K = d_model, the local FFN
         * width, and (tensor parallel) the local attention width */
        const int Ks[3] = {D, b->F, b->Dq};
        sb_tc_operand* ops[3] = {&b->op_d, &b->op_f, &b->op_a};
        for (int i = 0; i < 3; ++i) {
            if (i == 2 && b->Dq == D) {
                b->op_a = b->op_d;
                break;
            }
            const size_t nb = (size_t)B * Ks[i] * 2;
            void* hi = dalloc(b, nb);
            void* lw = lo ? dalloc(b, nb) : NULL;
            if (!hi || (lo && !lw) || sb_cuda_check(cudaMemset(hi, 0, nb), "memset") ||
                (lo && sb_cuda_check(cudaMemset(lw, 0, nb), "memset")) ||
                sb_tc_make_operand(ops[i], hi, lw, B, Ks[i], Ks[i]))
                goto fail;
        }
        const sb_layer* l0 = &b->layers[0];
        b->sp_qkv = sb_tc_splits_for(l0->wqkv.M_pad, D);
        b->sp_wo = sb_tc_splits_for(l0->wo.M_pad, b->Dq);
        b->sp_gu = sb_tc_splits_for(l0->wgu.M_pad, D);
        b->sp_dn = sb_tc_splits_for(l0->wdown.M_pad, b->F);
        size_t ws = 0, t;
        if ((t = (size_t)b->sp_qkv * l0->wqkv.M_pad) > ws) ws = t;
        if ((t = (size_t)b->sp_wo * l0->wo.M_pad) > ws) ws = t;
        if ((t = (size_t)b->sp_gu * l0->wgu.M_pad) > ws) ws = t;
        if ((t = (size_t)b->sp_dn * l0->wdown.M_pad) > ws) ws = t;
        if (b->lm_head.wtype == SB_WT_Q4K && (t = (size_t)b->lm_head.M_pad) > ws) ws = t;
        b->tc_ws = (float*)dalloc(b, ws * (size_t)B * 4);
        if (!b->tc_ws) goto fail;
        /* an f32 LM head runs on the tensor cores as an exact f16 hi/lo pair */
        if (b->tc_passes == 3 && b->lm_head.wtype == SB_WT_F32 &&
            (sb_tc_make_weight(&b->head_tc, (const float*)b->lm_head.data, b->lm_head.ldw, b->V_l,
                               D, b->stream) ||
             sb_cuda_check(cudaStreamSynchronize(b->stream), "head split")))
            goto fail;
        /* gemm_path 4: Q4_K weights on the exact-weight stream-K kernel (two f16
         * passes, block scales per super-block); 6: the same kernel with x
         * rounded once to f16 (one pass) */
        if (o->gemm_path == 4 || o->gemm_path == 6) {
            sb_q4_prepare();
            const int r_pad = (B + 127) / 128 * 128;
            const sb_tc_operand* src[3] = {&b->op_d, &b->op_f, &b->op_a};
            sb_q4_operand* dst[3] = {&b->q4_d, &b->q4_f, &b->q4_a};
            for (int i = 0; i < 3; ++i) {
                const size_t xs = (size_t)((src[i]->K / 256 + 1) & ~1) * r_pad * 8 * 2;
                void* xh = dalloc(b, xs);
                void* xl = dalloc(b, xs);
                if (!xh || !xl || sb_cuda_check(cudaMemset(xh, 0, xs), "memset") ||
                    sb_cuda_check(cudaMemset(xl, 0, xs), "memset") ||
                    sb_q4_make_operand(dst[i], src[i]->hi, src[i]->lo, xh, xl, B, r_pad, src[i]->K,
                                       src[i]->K))
                    goto fail;
                dst[i]->one_pass = o->gemm_path == 6;
            }
            int mp = l0->wqkv.M_pad;
            if (l0->wo.M_pad > mp) mp = l0->wo.M_pad;
            if (l0->wgu.M_pad > mp) mp = l0->wgu.M_pad;
            if (l0->wdown.M_pad > mp) mp = l0->wdown.M_pad;
            if (b->lm_head.wtype == SB_WT_Q4K && b->lm_head.M_pad > mp) mp = b->lm_head.M_pad;
            const size_t tiles = (size_t)sb_q4_tiles(mp, B);
            b->q4_ws = (float*)dalloc(b, sb_q4_ws_floats() * 4);
            b->q4_cnt = (int*)dalloc(b, tiles * 4);
            b->q4_cnt_n = tiles;
            if (!b->q4_ws || !b->q4_cnt || sb_cuda_check(cudaMemset(b->q4_cnt, 0, tiles * 4), "memset"))
                goto fail;
            b->q4_on = 1;
        }
        /* gemm_path 5: Q4_K weights on the three-pass stream-K kernel; the
         * default (0) uses it from 128 rows, where it is the faster kernel */
        if (o->gemm_path == 5 || o->gemm_path == 0) {
            b->sk_min = o->gemm_path == 5 ? SB_TC_MIN_ROWS : SB_SK_MIN_ROWS;
            sb_sk_prepare();
            b->sk_ws = (float*)dalloc(b, sb_sk_ws_floats(sb_sk_tiles(l0->wgu.M_pad, B)) * 4);
            if (!b->sk_ws) goto fail;
            b->sk_on = 1;
            /* gate/up on this kernel whenever down is: its output pass can
             * write down's f16 operand */
            b->sk_h = l0->wgu.M % 128 == 0 && l0->wdown.K == b->op_f.K && l0->wgu.M / 2 == b->op_f.K;
        }
    }

    /* lanes: the whole batch, and (one GPU, stream-K GEMMs) the two halves,
     * whose operands view the same f16 buffers from their first row on */
    b->full.op_d = &b->op_d;
    b->full.op_f = &b->op_f;
    b->full.op_a = &b->op_a;
    b->full.sk_ws = b->sk_ws;
    b->full.r0 = 0;
    b->full.comm = b->comm;
    b->half_rows = b->max_batch / 2;
    if (b->sk_on && !b->q4_on && o->lanes == 2 && b->half_rows >= SB_TC_MIN_ROWS) {
        /* tensor parallel: the second lane's all-reduces go through their own
         * communicator on the second stream, beside the first lane's work */
        if (b->tp > 1 && sb_tp_split(b->comm, b->rank, &b->comm2)) goto fail;
        b->half[0].comm = b->comm;
        b->half[1].comm = b->tp > 1 ? b->comm2 : NULL;
        const sb_tc_operand* fo[3] = {&b->op_d, &b->op_f, &b->op_a};
        for (int hh = 0; hh < 2; ++hh) {
            sb_lane* L = &b->half[hh];
            L->r0 = hh ? b->half_rows : 0;
            const int rows = hh ? b->max_batch - b->half_rows : b->half_rows;
            for (int i = 0; i < 3; ++i) {
                if (i == 2 && fo[2]->hi == fo[0]->hi) break;      /* op_a shares op_d */
                const size_t off = (size_t)L->r0 * fo[i]->ld16 * 2;
                if (sb_tc_make_operand(&L->own[i], (char*)fo[i]->hi + off,
                                       fo[i]->lo ? (char*)fo[i]->lo + off : NULL, rows, fo[i]->K,
                                       fo[i]->ld16))
                    goto fail;
            }
            L->op_d = &L->own[0];
            L->op_f = &L->own[1];
            L->op_a = fo[2]->hi == fo[0]->hi ? &L->own[0] : &L->own[2];
            L->sk_ws = hh ? (float*)dalloc(b, sb_sk_ws_floats(sb_sk_tiles(b->layers[0].wgu.M_pad,
                                                                          rows)) * 4)
                          : b->sk_ws;
            if (!L->sk_ws) goto fail;
        }
        if (sb_cuda_check(cudaStreamCreateWithFlags(&b->stream2, cudaStreamNonBlocking), "stream") ||
            sb_cuda_check(cudaEventCreateWithFlags(&b->ev_fork, cudaEventDisableTiming), "event") ||
            sb_cuda_check(cudaEventCreateWithFlags(&b->ev_join, cudaEventDisableTiming), "event") ||
            sb_cuda_check(cudaEventCreateWithFlags(&b->ev_a, cudaEventDisableTiming), "event") ||
            sb_cuda_check(cudaEventCreateWithFlags(&b->ev_b, cudaEventDisableTiming), "event"))
            goto fail;
        b->dual = 1;
    }

    /* small-batch Q4_K GEMMs (default path): partials and row-block counters
     * per lane that can run beside another (the full lane and the first half
     * never run at the same time) */
    if (o->gemm_path == 0 && b->layers[0].wqkv.wtype == SB_WT_Q4K) {
        const sb_matrix* mats[5] = {&b->layers[0].wqkv, &b->layers[0].wo, &b->layers[0].wgu,
                                    &b->layers[0].wdown, &b->lm_head};
        size_t wsf = 0;
        int blocks = 0;
        for (int i = 0; i < 5; ++i) {
            if (mats[i]->wtype != SB_WT_Q4K) continue;
            const size_t f = sb_mv_ws_floats(mats[i]->M_pad, mats[i]->K);
            if (f > wsf) wsf = f;
            if (mats[i]->M_pad / 128 > blocks) blocks = mats[i]->M_pad / 128;
        }
        sb_lane* lanes[2] = {&b->full, b->dual ? &b->half[1] : NULL};
        for (int i = 0; i < 2 && wsf && lanes[i]; ++i) {
            lanes[i]->mv_ws = (float*)dalloc(b, wsf * 4);
            lanes[i]->mv_cnt = (int*)dalloc(b, (size_t)blocks * 4);
            if (!lanes[i]->mv_ws || !lanes[i]->mv_cnt ||
                sb_cuda_check(cudaMemset(lanes[i]->mv_cnt, 0, (size_t)blocks * 4), "memset"))
                goto fail;
        }
        if (b->dual) {
            b->half[0].mv_ws = b->full.mv_ws;
            b->half[0].mv_cnt = b->full.mv_cnt;
        }
    }

    /* KV pool, page tables, free list */
    {
        const size_t esz = b->kv_dtype == SLATE_KV_F16 ? 2 : 4;
        const size_t page_bytes_all = (size_t)L * 2 * b->nkv * SB_PAGE_TOKENS * hd * esz;
        int64_t pages = o->kv_pages;
        if (pages <= 0) {
            size_t budget = o->kv_bytes;
            if (!budget) {
                size_t fr = 0, tot = 0;
                if (sb_cuda_check(cudaMemGetInfo(&fr, &tot), "cudaMemGetInfo")) goto fail;
                size_t tables = (size_t)b->max_slots * b->max_pages * 4;
                budget = fr > tables + (1u << 30) ? (size_t)((double)(fr - tables) * 0.90) : 0;
            }
            pages = (int64_t)(budget / page_bytes_all);
            int64_t want = (int64_t)b->max_slots * b->max_pages;
            if (pages > want) pages = want;
        }
        if (pages < 1 || pages > 0x7fffffff) {
            sb_set_error("KV pool of %lld pages not possible", (long long)pages);
            goto fail;
        }
        b->n_pages = pages;
        b->pool = dalloc(b, (size_t)pages * page_bytes_all);
        b->pos = (int32_t*)dalloc(b, (size_t)b->max_slots * 4);
        b->page_table = (int32_t*)dalloc(b, (size_t)b->max_slots * b->max_pages * 4);
        b->free_stack = (int32_t*)dalloc(b, (size_t)pages * 4);
        b->free_top = (int32_t*)dalloc(b, 16);
        if (!b->pool || !b->pos || !b->page_table || !b->free_stack || !b->free_top) goto fail;
        if (sb_cuda_check(cudaMemset(b->pos, 0, (size_t)b->max_slots * 4), "memset") ||
            sb_cuda_check(cudaMemset(b->page_table, 0xff, (size_t)b->max_slots * b->max_pages * 4),
                          "memset"))
            goto fail;
        if (sb_init_free_list(b->free_stack, b->free_top, pages, b->stream)) goto fail;
        if (o->attn_path != 1 && sb_attention_mma_supported(b->nq, b->nkv, hd, b->kv_dtype)) {
            if (sb_attention_make_map(b->kvmap, b->pool, pages, L, b->nkv, hd)) goto fail;
            b->kvmap_p = b->kvmap;
        }
    }
    b->h_pos = (int*)calloc((size_t)b->max_slots, sizeof(int));
    b->h_open = (unsigned char*)calloc((size_t)b->max_slots, 1);
    b->graphs = (cudaGraphExec_t*)calloc((size_t)b->max_batch + 1, sizeof(cudaGraphExec_t));
    b->graphs_c = (cudaGraphExec_t*)calloc((size_t)b->max_batch + 1, sizeof(cudaGraphExec_t));
    b->graphs_p = (cudaGraphExec_t*)calloc((size_t)b->max_batch + 1, sizeof(cudaGraphExec_t));
    if (!b->graphs || !b->graphs_c || !b->graphs_p) {
        sb_set_error("out of host memory");
        goto fail;
    }
    if (sb_cuda_check(cudaStreamSynchronize(b->stream), "init sync")) goto fail;
    return b;
fail:
    if (stg.p) cudaFreeHost(stg.p);
    slate_llama_batch_free(b);
    return NULL;
}

slate_llama_batch_t* slate_llama_batch_new_gguf(const char* path, const slate_cuda_opts_t* o) {
    slate_llama_desc_t d;
    slate_gguf_model_t* g = slate_gguf_model_open(path, &d);
    if (!g) return NULL;
    slate_llama_batch_t* b = slate_llama_batch_new_desc(&d, o);
    slate_gguf_model_close(g);
    return b;
}

/* ---- accessors ---------------------------------------------------------- */
int slate_llama_batch_vocab(const slate_llama_batch_t* b) { return b ? b->V : -1; }
int slate_llama_batch_max_batch(const slate_llama_batch_t* b) { return b ? b->max_batch : -1; }
int slate_llama_batch_max_seq(const slate_llama_batch_t* b) { return b ? b->max_seq : -1; }
int64_t slate_llama_batch_free_pages(const slate_llama_batch_t* b) {
    return b ? b->n_pages - b->pages_used : -1;
}
void* slate_llama_batch_stream(slate_llama_batch_t* b) { return b ? (void*)b->stream : NULL; }

/* Pulls device positions into the host mirror after device-API steps. */
static int refresh_positions(slate_llama_batch_t* b) {
    if (!b->pos_dirty) return 0;
    SB_CU(cudaMemcpyAsync(b->h_pos, b->pos, (size_t)b->max_slots * 4, cudaMemcpyDeviceToHost,
                          b->stream));
    SB_CU(cudaStreamSynchronize(b->stream));
    int64_t used = 0;
    for (int s = 0; s < b->max_slots; ++s)
        if (b->h_open[s]) used += (b->h_pos[s] + SB_PAGE_TOKENS - 1) / SB_PAGE_TOKENS;
    b->pages_used = used;
    b->pos_dirty = 0;
    return 0;
}

int slate_llama_batch_open(slate_llama_batch_t* b) {
    if (!b) return -1;
    pthread_mutex_lock(&b->lock);
    int slot = -2;
    for (int s = 0; s < b->max_slots; ++s)
        if (!b->h_open[s]) {
            b->h_open[s] = 1;
            b->h_pos[s] = 0;
            slot = s;
            break;
        }
    pthread_mutex_unlock(&b->lock);
    return slot;
}

int slate_llama_batch_close(slate_llama_batch_t* b, int slot) {
    if (!b || slot < 0 || slot >= b->max_slots || !b->h_open[slot]) return -1;
    pthread_mutex_lock(&b->lock);
    int rc = refresh_positions(b);
    if (!rc) {
        cudaSetDevice(b->device);
        rc = sb_release_slot(slot, b->pos, b->page_table, b->max_pages, b->free_stack,
                             b->free_top, b->stream);
        if (!rc) rc = sb_cuda_check(cudaGetLastError(), "release");
        b->pages_used -= (b->h_pos[slot] + SB_PAGE_TOKENS - 1) / SB_PAGE_TOKENS;
        b->h_open[slot] = 0;
        b->h_pos[slot] = 0;
    }
    pthread_mutex_unlock(&b->lock);
    return rc;
}

int slate_llama_batch_position(const slate_llama_batch_t* cb, int slot) {
    slate_llama_batch_t* b = (slate_llama_batch_t*)cb;
    if (!b || slot < 0 || slot >= b->max_slots || !b->h_open[slot]) return -1;
    pthread_mutex_lock(&b->lock);
    int rc = refresh_positions(b);
    int p = rc ? rc : b->h_pos[slot];
    pthread_mutex_unlock(&b->lock);
    return p;
}

/* ---- steps --------------------------------------------------------------- */

/* Enqueues the copy of the device status words (step status, tensor-core
 * wait status) into h_io[3B], h_io[3B+1] and their reset. */
static int status_readback(slate_llama_batch_t* b) {
    int32_t* h = b->h_io + 3 * b->max_batch;
    h[1] = 0;
    SB_CU(cudaMemcpyAsync(h, b->status, 4, cudaMemcpyDeviceToHost, b->stream));
    SB_CU(cudaMemsetAsync(b->status, 0, 4, b->stream));
    if (b->tc_err) {
        SB_CU(cudaMemcpyAsync(h + 1, b->tc_err, 4, cudaMemcpyDeviceToHost, b->stream));
        SB_CU(cudaMemsetAsync(b->tc_err, 0, 4, b->stream));
    }
    return 0;
}
/* After a synchronize: 0, the step's -1/-2/-3, or -5 when a tensor-core
 * kernel gave up waiting (which makes that step's results invalid). */
static int status_code(slate_llama_batch_t* b) {
    const int32_t* h = b->h_io + 3 * b->max_batch;
    if (h[1]) {
        /* a step that gave up may leave stream-K tile counters and the
         * GEMV's per-head counters raised */
        if (b->q4_cnt) cudaMemset(b->q4_cnt, 0, b->q4_cnt_n * 4);
        if (b->head_cnt) cudaMemset(b->head_cnt, 0, (size_t)(b->nq + 2 * b->nkv) * 4);
        sb_set_error("tensor-core GEMM pipeline wait timed out (stage %d)", h[1]);
        return -5;
    }
    if (h[0]) sb_set_error("device rejected the step (%d)", h[0]);
    return h[0];
}

/* Copies the step's logits [n][V] to dst (host or device).  A tensor-parallel
 * rank holds only its vocabulary slice: the slices of all ranks are gathered
 * first (a collective, so every rank asks for logits in the same steps). */
static int copy_logits(slate_llama_batch_t* b, int n, float* dst, enum cudaMemcpyKind kind) {
    const size_t ldl = (size_t)b->ld_logits;
    if (b->tp == 1)
        return sb_cuda_check(cudaMemcpy2DAsync(dst, (size_t)b->V * 4, b->logits, ldl * 4,
                                               (size_t)b->V * 4, (size_t)n, kind, b->stream),
                             "logits copy");
    if (!b->logits_all) {
        b->logits_all = (float*)dalloc(b, (size_t)b->tp * b->max_batch * ldl * 4);
        if (!b->logits_all) return -5;
    }
    int rc = sb_tp_allgather(b->comm, b->logits, b->logits_all, (size_t)n * ldl * 4, b->stream);
    for (int r = 0; r < b->tp && !rc && dst; ++r)
        rc = sb_cuda_check(cudaMemcpy2DAsync(dst + (size_t)r * b->V_l, (size_t)b->V * 4,
                                             b->logits_all + (size_t)r * n * ldl, ldl * 4,
                                             (size_t)b->V_l * 4, (size_t)n, kind, b->stream),
                           "logits copy");
    return rc;
}

/* Row n - 1 of the step's logits to host dst[V] (after copy_logits(.., NULL,
 * ..) has gathered them on a tensor-parallel rank). */
static int copy_last_logits(slate_llama_batch_t* b, int n, float* dst) {
    const size_t ldl = (size_t)b->ld_logits;
    if (b->tp == 1)
        return sb_cuda_check(cudaMemcpyAsync(dst, b->logits + (size_t)(n - 1) * ldl, (size_t)b->V * 4,
                                             cudaMemcpyDeviceToHost, b->stream), "logits copy");
    int rc = 0;
    for (int r = 0; r < b->tp && !rc; ++r)
        rc = sb_cuda_check(cudaMemcpyAsync(dst + (size_t)r * b->V_l,
                                           b->logits_all + ((size_t)r * n + (n - 1)) * ldl,
                                           (size_t)b->V_l * 4, cudaMemcpyDeviceToHost, b->stream),
                           "logits copy");
    return rc;
}

/* One step over host buffers.  allow_dup: a slot may occur several times (a
 * prompt chunk), its k-th occurrence at position pos + k.  out_logits gets all
 * n rows, last_logits (nullable) only row n - 1. */
static int step_host(slate_llama_batch_t* b, const int32_t* slots, int n, const int32_t* tokens,
                     int32_t* out_tokens, float* out_logits, float* last_logits, int allow_dup) {
    if (!b || !slots || !tokens || n < 1 || n > b->max_batch) return -1;
    pthread_mutex_lock(&b->lock);
    int rc = refresh_positions(b);
    /* host-side validation, same order and codes as engine.c:557-559 */
    int64_t new_pages = 0;
    for (int r = 0; r < n && !rc; ++r) {
        const int s = slots[r];
        if (s < 0 || s >= b->max_slots || !b->h_open[s]) { rc = -1; break; }
        int rank = 0;
        for (int q = 0; q < r; ++q) rank += slots[q] == s;
        if (rank && !allow_dup) { rc = -1; break; }
        if (b->h_pos[s] + rank >= b->max_seq) { rc = -2; break; }
        if (tokens[r] < 0 || tokens[r] >= b->V) { rc = -3; break; }
        if ((b->h_pos[s] + rank) % SB_PAGE_TOKENS == 0) ++new_pages;
    }
    if (!rc && b->pages_used + new_pages > b->n_pages) rc = -2;
    if (rc) {
        pthread_mutex_unlock(&b->lock);
        return rc;
    }
    cudaSetDevice(b->device);
    int32_t* h = b->h_io;
    memcpy(h, slots, (size_t)n * 4);
    memcpy(h + b->max_batch, tokens, (size_t)n * 4);
    rc = sb_cuda_check(cudaMemcpyAsync(b->d_io, h, (size_t)2 * b->max_batch * 4,
                                       cudaMemcpyHostToDevice, b->stream), "H2D metadata");
    /* a prompt chunk whose logits nobody reads runs without the LM head; tensor-
     * parallel ranks keep it, so that their collectives stay in step whatever
     * buffers each rank passes */
    const int head = !allow_dup || b->tp > 1 || out_tokens || out_logits || last_logits;
    if (!rc) rc = run_step_mode(b, n, 0, allow_dup, head);
    if (!rc)
        rc = sb_cuda_check(cudaMemcpyAsync(h + 2 * b->max_batch, b->d_io + 2 * b->max_batch,
                                           (size_t)n * 4, cudaMemcpyDeviceToHost, b->stream),
                           "D2H tokens");
    if (!rc) rc = status_readback(b);
    if (!rc && out_logits) rc = copy_logits(b, n, out_logits, cudaMemcpyDeviceToHost);
    if (!rc && last_logits) {
        if (b->tp > 1) {
            rc = copy_logits(b, n, NULL, cudaMemcpyDeviceToHost);   /* gathers only */
        }
        if (!rc) rc = copy_last_logits(b, n, last_logits);
    }
    if (!rc) rc = sb_cuda_check(cudaStreamSynchronize(b->stream), "step");
    if (!rc) {
        const int st = status_code(b);
        if (st) {
            rc = st;
        } else {
            for (int r = 0; r < n; ++r) {
                if (b->h_pos[slots[r]] % SB_PAGE_TOKENS == 0) ++b->pages_used;
                b->h_pos[slots[r]]++;
            }
            if (out_tokens) memcpy(out_tokens, h + 2 * b->max_batch, (size_t)n * 4);
        }
    }
    pthread_mutex_unlock(&b->lock);
    return rc;
}

int slate_llama_batch_step(slate_llama_batch_t* b, const int32_t* slots, int n,
                           const int32_t* tokens, int32_t* out_tokens, float* out_logits) {
    return step_host(b, slots, n, tokens, out_tokens, out_logits, NULL, 0);
}

/* Lazily creates the sampling buffers (outside any capture). */
static int sampling_ready(slate_llama_batch_t* b) {
    if (b->d_samp) return 0;
    const int B = b->max_batch;
    b->graphs_s = (cudaGraphExec_t*)calloc((size_t)B + 1, sizeof(cudaGraphExec_t));
    b->d_samp = (sb_sampler*)dalloc(b, (size_t)B * sizeof(sb_sampler));
    b->d_rng = (uint64_t*)dalloc(b, (size_t)B * 8);
    b->samp_scratch = (float*)dalloc(b, (size_t)B * b->V * 4);
    if (!b->graphs_s || !b->d_samp || !b->d_rng || !b->samp_scratch) return -5;
    SB_CU(cudaHostAlloc((void**)&b->h_samp, (size_t)B * sizeof(sb_sampler), cudaHostAllocDefault));
    SB_CU(cudaHostAlloc((void**)&b->h_rng, (size_t)B * 8, cudaHostAllocDefault));
    return 0;
}

int slate_llama_batch_step_sample(slate_llama_batch_t* b, const int32_t* slots, int n,
                                  const int32_t* tokens, const slate_sampler_config_t* cfg,
                                  uint64_t* rng_state, int32_t* out_tokens, float* out_logits) {
    if (!b || !slots || !tokens || !cfg || !rng_state || n < 1 || n > b->max_batch) return -1;
    if (b->tp > 1) {
        sb_set_error("sampling steps are not available with tensor parallelism");
        return -1;
    }
    for (int r = 0; r < n; ++r)
        if (cfg[r].temperature > 0.0f && cfg[r].top_k > SB_SAMPLE_TOPK_MAX && cfg[r].top_k < b->V) {
            sb_set_error("top_k %d above the device sampler's %d", cfg[r].top_k, SB_SAMPLE_TOPK_MAX);
            return -1;
        }
    pthread_mutex_lock(&b->lock);
    int rc = refresh_positions(b);
    int64_t new_pages = 0;
    for (int r = 0; r < n && !rc; ++r) {
        const int s = slots[r];
        if (s < 0 || s >= b->max_slots || !b->h_open[s]) { rc = -1; break; }
        for (int q = 0; q < r; ++q)
            if (slots[q] == s) { rc = -1; break; }
        if (rc) break;
        if (b->h_pos[s] >= b->max_seq) { rc = -2; break; }
        if (tokens[r] < 0 || tokens[r] >= b->V) { rc = -3; break; }
        if (b->h_pos[s] % SB_PAGE_TOKENS == 0) ++new_pages;
    }
    if (!rc && b->pages_used + new_pages > b->n_pages) rc = -2;
    if (!rc) {
        cudaSetDevice(b->device);
        rc = sampling_ready(b);
    }
    if (rc) {
        pthread_mutex_unlock(&b->lock);
        return rc;
    }
    int32_t* h = b->h_io;
    memcpy(h, slots, (size_t)n * 4);
    memcpy(h + b->max_batch, tokens, (size_t)n * 4);
    for (int r = 0; r < n; ++r) {
        b->h_samp[r] = (sb_sampler){cfg[r].temperature, cfg[r].top_k, cfg[r].top_p, 0};
        b->h_rng[r] = rng_state[r];
    }
    rc = sb_cuda_check(cudaMemcpyAsync(b->d_io, h, (size_t)2 * b->max_batch * 4,
                                       cudaMemcpyHostToDevice, b->stream), "H2D metadata");
    if (!rc) rc = sb_cuda_check(cudaMemcpyAsync(b->d_samp, b->h_samp, (size_t)n * sizeof(sb_sampler),
                                                cudaMemcpyHostToDevice, b->stream), "H2D sampler");
    if (!rc) rc = sb_cuda_check(cudaMemcpyAsync(b->d_rng, b->h_rng, (size_t)n * 8,
                                                cudaMemcpyHostToDevice, b->stream), "H2D rng");
    if (!rc) rc = run_step_mode(b, n, 1, 0, 1);
    if (!rc)
        rc = sb_cuda_check(cudaMemcpyAsync(h + 2 * b->max_batch, b->d_io + 2 * b->max_batch,
                                           (size_t)n * 4, cudaMemcpyDeviceToHost, b->stream),
                           "D2H tokens");
    if (!rc) rc = sb_cuda_check(cudaMemcpyAsync(b->h_rng, b->d_rng, (size_t)n * 8,
                                                cudaMemcpyDeviceToHost, b->stream), "D2H rng");
    if (!rc) rc = status_readback(b);
    if (!rc && out_logits) rc = copy_logits(b, n, out_logits, cudaMemcpyDeviceToHost);
    if (!rc) rc = sb_cuda_check(cudaStreamSynchronize(b->stream), "step");
    if (!rc) {
        const int st = status_code(b);
        if (st) {
            rc = st;
        } else {
            for (int r = 0; r < n; ++r) {
                if (b->h_pos[slots[r]] % SB_PAGE_TOKENS == 0) ++b->pages_used;
                b->h_pos[slots[r]]++;
                rng_state[r] = b->h_rng[r];
            }
            if (out_tokens) memcpy(out_tokens, h + 2 * b->max_batch, (size_t)n * 4);
        }
    }
    pthread_mutex_unlock(&b->lock);
    return rc;
}

int slate_llama_batch_step_device(slate_llama_batch_t* b, const int32_t* d_slots, int n,
                                  const int32_t* d_tokens, int32_t* d_out_tokens,
                                  float* d_out_logits, void* stream) {
    if (!b || !d_slots || !d_tokens || n < 1 || n > b->max_batch) return -1;
    pthread_mutex_lock(&b->lock);
    cudaSetDevice(b->device);
    cudaStream_t us = stream ? (cudaStream_t)stream : b->stream;
    int rc = 0;
    cudaEvent_t ev = NULL;
    if (us != b->stream) {
        /* order the engine stream after the caller's work and vice versa */
        rc = sb_cuda_check(cudaEventCreateWithFlags(&ev, cudaEventDisableTiming), "event");
        if (!rc) rc = sb_cuda_check(cudaEventRecord(ev, us), "event record");
        if (!rc) rc = sb_cuda_check(cudaStreamWaitEvent(b->stream, ev, 0), "event wait");
    }
    if (!rc) rc = sb_cuda_check(cudaMemcpyAsync(b->d_io, d_slots, (size_t)n * 4,
                                                cudaMemcpyDeviceToDevice, b->stream), "slots");
    if (!rc) rc = sb_cuda_check(cudaMemcpyAsync(b->d_io + b->max_batch, d_tokens, (size_t)n * 4,
                                                cudaMemcpyDeviceToDevice, b->stream), "tokens");
    if (!rc) rc = run_step(b, n);
    if (!rc && d_out_tokens)
        rc = sb_cuda_check(cudaMemcpyAsync(d_out_tokens, b->d_io + 2 * b->max_batch, (size_t)n * 4,
                                           cudaMemcpyDeviceToDevice, b->stream), "out tokens");
    if (!rc && d_out_logits) rc = copy_logits(b, n, d_out_logits, cudaMemcpyDeviceToDevice);
    if (!rc && ev) {
        rc = sb_cuda_check(cudaEventRecord(ev, b->stream), "event record");
        if (!rc) rc = sb_cuda_check(cudaStreamWaitEvent(us, ev, 0), "event wait");
    }
    if (ev) cudaEventDestroy(ev);
    b->pos_dirty = 1;
    pthread_mutex_unlock(&b->lock);
    return rc;
}

int slate_llama_batch_sync(slate_llama_batch_t* b) {
    if (!b) return -1;
    pthread_mutex_lock(&b->lock);
    cudaSetDevice(b->device);
    int rc = status_readback(b);
    if (!rc) rc = sb_cuda_check(cudaStreamSynchronize(b->stream), "sync");
    if (!rc) rc = status_code(b);
    pthread_mutex_unlock(&b->lock);
    return rc;
}

int slate_llama_batch_prefill(slate_llama_batch_t* b, int slot, const int32_t* tokens,
                              int n_tokens, float* out_logits) {
    if (!b || !tokens || n_tokens <= 0) return -1;
    /* chunks of up to max_batch prompt tokens, each one step whose rows are
     * consecutive positions of this slot: the GEMMs see a chunk of rows, each
     * row attends to everything before it (earlier chunks and earlier rows of
     * its own chunk, appended first in the step) */
    int32_t* slots = (int32_t*)malloc((size_t)b->max_batch * 4);
    if (!slots) return -5;
    for (int i = 0; i < b->max_batch; ++i) slots[i] = slot;
    int rc = 0;
    for (int i = 0; i < n_tokens && !rc; i += b->max_batch) {
        const int n = n_tokens - i < b->max_batch ? n_tokens - i : b->max_batch;
        const int last = i + n == n_tokens;
        rc = step_host(b, slots, n, tokens + i, NULL, NULL, last ? out_logits : NULL, 1);
    }
    free(slots);
    return rc;
}

int slate_llama_batch_seed_context(slate_llama_batch_t* b, int slot, int n_tokens, uint64_t seed) {
    if (!b || slot < 0 || slot >= b->max_slots || !b->h_open[slot] || n_tokens < 0) return -1;
    pthread_mutex_lock(&b->lock);
    int rc = refresh_positions(b);
    if (!rc && (b->h_pos[slot] != 0 || n_tokens > b->max_seq)) rc = -2;
    const int64_t need = (n_tokens + SB_PAGE_TOKENS - 1) / SB_PAGE_TOKENS;
    if (!rc && b->pages_used + need > b->n_pages) rc = -2;
    if (!rc) {
        cudaSetDevice(b->device);
        rc = sb_seed_context(slot, n_tokens, seed, b->L, b->nkv, b->hd, b->pos, b->page_table,
                             b->max_pages, b->free_stack, b->free_top, b->pool, b->n_pages,
                             b->kv_dtype, b->status, b->stream);
        if (!rc) rc = sb_cuda_check(cudaGetLastError(), "seed");
        if (!rc) rc = sb_cuda_check(cudaMemcpyAsync(b->h_io + 3 * b->max_batch, b->status, 4,
                                                    cudaMemcpyDeviceToHost, b->stream), "status");
        if (!rc) rc = sb_cuda_check(cudaMemsetAsync(b->status, 0, 4, b->stream), "status reset");
        if (!rc) rc = sb_cuda_check(cudaStreamSynchronize(b->stream), "seed sync");
        if (!rc) rc = b->h_io[3 * b->max_batch];
        if (!rc) {
            b->h_pos[slot] = n_tokens;
            b->pages_used += need;
        }
    }
    pthread_mutex_unlock(&b->lock);
    return rc;
}

int slate_llama_batch_read_kv(slate_llama_batch_t* b, int slot, int n, float* K, float* V) {
    if (!b || !K || !V || slot < 0 || slot >= b->max_slots || !b->h_open[slot] || n < 1) return -1;
    pthread_mutex_lock(&b->lock);
    int rc = refresh_positions(b);
    if (!rc && n > b->h_pos[slot]) rc = -1;
    float *dk = NULL, *dv = NULL;
    const size_t cnt = (size_t)b->L * n * b->kvd;
    if (!rc) {
        cudaSetDevice(b->device);
        rc = sb_cuda_check(cudaMalloc((void**)&dk, cnt * 4), "cudaMalloc");
        if (!rc) rc = sb_cuda_check(cudaMalloc((void**)&dv, cnt * 4), "cudaMalloc");
        if (!rc) rc = sb_read_kv(slot, n, b->L, b->nkv, b->hd, b->page_table, b->max_pages, b->pool,
                                 b->n_pages, b->kv_dtype, dk, dv, b->stream);
        if (!rc) rc = sb_cuda_check(cudaMemcpyAsync(K, dk, cnt * 4, cudaMemcpyDeviceToHost, b->stream), "K");
        if (!rc) rc = sb_cuda_check(cudaMemcpyAsync(V, dv, cnt * 4, cudaMemcpyDeviceToHost, b->stream), "V");
        if (!rc) rc = sb_cuda_check(cudaStreamSynchronize(b->stream), "read_kv");
    }
    if (dk) cudaFree(dk);
    if (dv) cudaFree(dv);
    pthread_mutex_unlock(&b->lock);
    return rc;
}

/* ---- profiling ---------------------------------------------------------- */
static int enqueue_kernel(slate_llama_batch_t* b, int kernel, int n, int layer, cudaStream_t s) {
    const sb_layer* ly = &b->layers[layer];
    float* scratch_y = b->logits;   /* [max_batch][ld_logits], >= any GEMM output row here */
    switch (kernel) {
        case SLATE_PROF_ATTENTION:
            return sb_attention_paged(b->att, b->ld_att, b->qkv, b->ld_qkv, n, b->nq, b->nkv, b->hd,
                                      b->row_pos, b->row_slot, b->page_table, b->max_pages,
                                      b->pool, b->kvmap_p, b->n_pages, layer, b->kv_dtype,
                                      b->max_seq, 0, b->scratch, b->tc_err, s);
        case SLATE_PROF_QKV:
            return step_gemm(b, &b->full, &ly->wqkv, b->xn, b->ld_x, IN_XN, n, scratch_y,
                             b->ld_logits, SB_EPI_STORE, b->sp_qkv, s);
        case SLATE_PROF_WO:
            return step_gemm(b, &b->full, &ly->wo, b->att, b->ld_att, IN_ATT, n, scratch_y,
                             b->ld_logits, SB_EPI_STORE, b->sp_wo, s);
        case SLATE_PROF_GATE_UP:
            return step_gemm(b, &b->full, &ly->wgu, b->xn, b->ld_x, IN_XN, n, b->h, b->ld_h,
                             SB_EPI_SILU, b->sp_gu, s);
        case SLATE_PROF_DOWN:
            return step_gemm(b, &b->full, &ly->wdown, b->h, b->ld_h, IN_H, n, scratch_y,
                             b->ld_logits, SB_EPI_STORE, b->sp_dn, s);
        case SLATE_PROF_LM_HEAD:
            return step_gemm(b, &b->full, &b->lm_head, b->xn, b->ld_x, IN_XN, n, b->logits,
                             b->ld_logits, SB_EPI_STORE, 1, s);
        case SLATE_PROF_STEP:
            return run_step(b, n);
        case SLATE_PROF_ALLREDUCE:
            /* the step's all-reduce after Wo / down: [n][ld_x] floats, here on
             * scratch rows (a collective: every rank makes the same call) */
            if (b->tp < 2) return -1;
            return sb_tp_allreduce_sum(b->comm, scratch_y, (size_t)n * b->ld_x, s);
    }
    return -1;
}

int slate_llama_batch_profile(slate_llama_batch_t* b, int kernel, int n, int layer, int iters,
                              float* ms) {
    if (!b || !ms || n < 1 || n > b->max_batch || layer < 0 || layer >= b->L || iters < 1 ||
        kernel < 0 || kernel > SLATE_PROF_ALLREDUCE || (kernel == SLATE_PROF_ALLREDUCE && b->tp < 2))
        return -1;
    if (b->ld_logits < b->D || (kernel == SLATE_PROF_QKV && b->ld_logits < b->layers[0].wqkv.M)) {
        sb_set_error("profile scratch too small for this model");
        return -1;
    }
    pthread_mutex_lock(&b->lock);
    cudaSetDevice(b->device);
    cudaEvent_t e0 = NULL, e1 = NULL;
    int rc = sb_cuda_check(cudaEventCreate(&e0), "event");
    if (!rc) rc = sb_cuda_check(cudaEventCreate(&e1), "event");
    if (!rc) rc = enqueue_kernel(b, kernel, n, layer, b->stream);   /* untimed */
    if (!rc) rc = sb_cuda_check(cudaEventRecord(e0, b->stream), "record");
    for (int i = 0; i < iters && !rc; ++i) rc = enqueue_kernel(b, kernel, n, layer, b->stream);
    if (!rc) rc = sb_cuda_check(cudaEventRecord(e1, b->stream), "record");
    if (!rc) rc = sb_cuda_check(cudaEventSynchronize(e1), "sync");
    float t = 0.f;
    if (!rc) rc = sb_cuda_check(cudaEventElapsedTime(&t, e0, e1), "elapsed");
    if (!rc) *ms = t / (float)iters;
    if (e0) cudaEventDestroy(e0);
    if (e1) cudaEventDestroy(e1);
    if (kernel == SLATE_PROF_STEP) b->pos_dirty = 1;
    pthread_mutex_unlock(&b->lock);
    return rc;
}
