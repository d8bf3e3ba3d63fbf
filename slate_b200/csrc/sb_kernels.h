/*
 * sb_kernels.h -- C-callable launchers for the sm_100a kernels (internal to
 * libslate_cuda.so; the public ABI is include/slate_cuda.h).  Every launcher
 * enqueues on the given stream and returns 0, or -1 for unsupported
 * arguments (checked before anything is launched).
 */
#ifndef SB_KERNELS_H
#define SB_KERNELS_H

#include <stddef.h>
#include <stdint.h>
#include <cuda_runtime_api.h>
#include "slate_cuda.h"

#ifdef __cplusplus
extern "C" {
#endif

#define SB_WT_F32 0
#define SB_WT_Q4K 18

#define SB_EPI_STORE 0   /* Y[n][m]  = acc                                   */
#define SB_EPI_ADD   1   /* Y[n][m] += acc (residual add, backend_cpu.c:99)  */
#define SB_EPI_SILU  2   /* rows interleaved by 64 (gate | up) per 128-row
                            tile: Y[n][t*64+r] = silu(g)*u (backend_cpu.c:78) */

#define SB_EPI_ROPE  3   /* fused Q|K|V projection: RoPE (llama_infer.c:77-92)
                            on the query heads in place, key heads rotated and
                            value heads copied into the paged cache at each
                            row's position (llama_infer.c:167-174) */

#define SB_PAGE_TOKENS 16

/* What the SB_EPI_ROPE epilogue needs: the rows' positions and slots, the
 * page table and KV pool (layout of slate_llama_batch_new_desc), the RoPE
 * tables [pos][head_dim/2], and the head counts of the projection. */
typedef struct sb_rope_args {
    const int32_t* row_pos;
    const int32_t* row_slot;
    const int32_t* page_table;
    void* pool;
    const float* rope_cos;
    const float* rope_sin;
    int64_t n_pages;
    int max_pages, layer, kv_dtype, nq, nkv, hd;
} sb_rope_args;

/* Weight matrix as the GEMMs consume it (packed once at upload):
 *   Q4_K: rows of K/256 super-blocks of 144 bytes (Slate's nibble order),
 *         row stride K/256*144 bytes, M_pad rows (zero blocks past M).
 *   f32 : row-major [M_pad][ldw] with ldw >= K, ldw % 32 == 0, zero padded. */
typedef struct sb_matrix {
    int wtype;
    const void* data;
    int M;       /* logical rows (for SILU: 2 * outputs, interleaved)      */
    int M_pad;   /* physical rows, multiple of 128                         */
    int K;       /* reduction length                                       */
    int ldw;     /* f32 row stride (floats); ignored for Q4_K              */
    int wexp;    /* Q4_K on the tensor cores (f16 hi/lo split of each weight):
                    weights are formed as w * 2^wexp -- exact, a power of two --
                    so that the lo halves stay normal f16 numbers, and the
                    accumulator is scaled by 2^-wexp; 0 = unscaled             */
} sb_matrix;

/* Y[n][·] (epi) X[n][0..K) · W[m][0..K)  for n < B.
 * X row stride ldx (floats); for f32 weights X must be zero in [K, ldw).
 * path: 0 = auto (GEMV for B <= 8, tiled otherwise), 1 = tiled only. */
/* One or two activation rows (gemm_gv.cu): Q4_K weights with K <= SB_GV_MAX_K,
 * M_pad % 128 == 0, on the CUDA cores (store / residual add / SiLU(gate)*up of
 * the interleaved gate|up weight), the weights streamed through shared memory
 * by bulk copies.  norm_w != NULL: X rows are RMSNorm-ed (weight norm_w[K],
 * eps) as they are staged.  SB_EPI_ROPE (the fused Q|K|V weight): Y stored,
 * then each head rotated / appended to the pool by the CTA that completes it
 * (head_cnt: nq + 2 nkv zeroed ints, left zeroed).  sb_gv_prepare() reads the SM count and opts the
 * kernels into their shared memory (per device, outside stream capture); a
 * ring wait that times out sets *err. */
#define SB_GV_MAX_ROWS 2
#define SB_GV_MAX_K 16384
void sb_gv_prepare(void);
int sb_gv_supported(const sb_matrix* W, int n, int epi);
int sb_gv_gemm(const sb_matrix* W, const float* X, int ldx, int n, float* Y, int ldy, int epi,
               const float* norm_w, float eps, const sb_rope_args* rope, int* head_cnt, int* err,
               cudaStream_t st);

/* Small batches (gemm_mv.cu): Q4_K weights, 1..SB_MV_MAX_ROWS activation
 * rows, tensor cores through mma.sync, weights streamed once.  ws holds
 * sb_mv_ws_floats(M_pad, K) floats; cnt M_pad / 128 zeroed ints (left zeroed).
 * X 16-byte aligned with ldx % 4 == 0.  Returns -1 (nothing launched) for
 * shapes it does not take. */
#define SB_MV_MAX_ROWS 16
size_t sb_mv_ws_floats(int M_pad, int K);
int sb_mv_gemm(const sb_matrix* W, const float* X, int ldx, int n, float* Y, int ldy, int epi,
               float* ws, int* cnt, cudaStream_t st);

int sb_gemm(const sb_matrix* W, const float* X, int ldx, int B, float* Y, int ldy,
            int epi, int path, cudaStream_t st);

/* Generic (any shape / alignment) f32 kernels for the reference vtable. */
int sb_matvec_f32_generic(float* y, const float* A, const float* x, int M, int K, cudaStream_t st);
int sb_linear_batch_generic(float* C, const float* X, const float* W, int B, int K, int N,
                            cudaStream_t st);
int sb_q4k_matmul_generic(float* Y, const void* A, const float* X, int B, int M, int K,
                          cudaStream_t st);

/* Row-wise RMSNorm (backend_cpu.c:48-76): Y[b] = X[b]*w*inv_rms(X[b]). */
int sb_rmsnorm_rows(float* Y, int ldy, const float* X, int ldx, const float* w, int B, int D,
                    float eps, cudaStream_t st);
/* The same rows also written as an f16 hi / lo pair (row stride ld16, lo
 * nullable; hi null: the f32 rows only) for the tensor-core GEMM operand, as a
 * programmatic dependent launch; D % 4 == 0, D <= 8192, ldx / ldy / ld16
 * multiples of 4 and 16-byte aligned X, Y, w (else -1, nothing launched); -5
 * when the launch itself fails. */
int sb_rmsnorm_rows_split(float* Y, int ldy, const float* X, int ldx, const float* w, int B, int D,
                          float eps, void* hi, void* lo, int ld16, cudaStream_t st);
int sb_silu_mul(float* y, const float* g, const float* u, int n, cudaStream_t st);
int sb_add_inplace(float* y, const float* x, int n, cudaStream_t st);
int sb_embed_lookup(float* y, const float* W, int token, int D, cudaStream_t st);
int sb_argmax_rows(int32_t* out, const float* logits, int ld, int B, int V, cudaStream_t st);
int sb_attention_step(float* out, const float* q, const float* K, const float* V, int L, int D,
                      cudaStream_t st);

/* Step prologue: validates rows, allocates KV pages on the device free list,
 * records row_pos/row_slot and gathers embeddings x[b] = emb[token[b]].
 * status (device int) receives -3 (bad token), -2 (position/pages) or -1
 * (bad slot) on failure; rows are then left without effect.  dup_ok: a slot
 * may occur several times (a prompt chunk: its k-th occurrence at position
 * pos + k); otherwise a repeated slot is a bad slot (-1). */
/* Positions of a step without LM head: pos[slot] = max(pos[slot], row_pos + 1)
 * per row when *status == 0. */
int sb_step_advance(const int32_t* row_slot, const int32_t* row_pos, int32_t* pos,
                    const int32_t* status, int B, cudaStream_t st);
int sb_step_prologue(const int32_t* slots, const int32_t* tokens, int B, int32_t* pos,
                     int32_t* page_table, int max_pages, int32_t* free_stack,
                     int32_t* free_top, int max_slots, int max_seq, int vocab,
                     const float* emb, int D, float* x, int ldx, int32_t* row_pos,
                     int32_t* row_slot, int32_t* status, int dup_ok, cudaStream_t st);
/* Step epilogue: out_tokens[b] = argmax(logits[b]) (first max), pos[slot]++
 * for every row when *status == 0. */
int sb_step_epilogue(const float* logits, int ldl, int V, int B, const int32_t* row_slot,
                     const int32_t* row_pos, int32_t* pos, const int32_t* status,
                     int32_t* out_tokens, cudaStream_t st);

/* RoPE with host-built tables cos/sin[pos][hd/2] (llama_infer.c:83-85 values)
 * on q and k in place, then K/V rows appended at row_pos into the paged pool
 * pool[layer][page][2][nkv][16][hd].  qkv rows: [q(nq*hd) | k | v], stride ld. */
int sb_rope_append(float* qkv, int ld, int B, int nq, int nkv, int hd, const int32_t* row_pos,
                   const int32_t* row_slot, const int32_t* page_table, int max_pages,
                   void* pool, int64_t n_pages, int layer, int kv_dtype,
                   const float* rope_cos, const float* rope_sin, cudaStream_t st);

/* Paged GQA attention (llama_infer.c:97-129): att[b][hq*hd+d] for ctx =
 * row_pos[b]+1.  Split over context chunks of ct tokens (one CTA per row, kv
 * head and chunk) into scratch partials (m, l, o[hd]), then combined.
 * sb_attention_chunk_tokens(B) picks ct from the row count: SB_ATTN_CHUNK from
 * 16 rows (at the 8B shape with 256 sequences 1024-token chunks ran 2-6%
 * faster per layer than 512, fewer per-CTA starts and partials, with ~10K
 * CTAs in flight; 4096 lost parallelism; at 16 rows 256-token chunks, 2.6
 * waves of CTAs, were slower than 1024), halving per halving of the rows down
 * to 128 tokens at 3 rows and 64 below, so that a few sequences still fill
 * one or more waves of CTAs whose pages are all in flight at once.  sb_attention_scratch_rows() is the scratch of B rows at chunk ct;
 * sb_attention_scratch_floats(max_batch) covers every B <= max_batch at its
 * own chunk (and any B <= max_batch at a longer chunk). */
#define SB_ATTN_CHUNK 1024
int sb_attention_chunk_tokens(int B);
size_t sb_attention_scratch_rows(int B, int nq, int hd, int max_seq, int ct);
size_t sb_attention_scratch_floats(int max_batch, int nq, int hd, int max_seq);
/* Opts the (head_dim, group, dtype) kernel into its shared-memory size on the
 * current device; call outside stream capture before the first launch. */
int sb_attention_prepare(int nq, int nkv, int hd, int kv_dtype);
/* kvmap: NULL, or a tensor map of the pool from sb_attention_make_map(); with
 * one, f16 pools of supported shapes take the tensor-core kernel.  ct: chunk
 * tokens (a multiple of 16 up to SB_ATTN_CHUNK), 0 = sb_attention_chunk_tokens(B). */
int sb_attention_paged(float* att, int ld_att, const float* qkv, int ld_qkv, int B, int nq,
                       int nkv, int hd, const int32_t* row_pos, const int32_t* row_slot,
                       const int32_t* page_table, int max_pages, const void* pool,
                       const void* kvmap, int64_t n_pages, int layer, int kv_dtype, int max_seq,
                       int ct, float* scratch, int* err, cudaStream_t st);
/* The same (chunks of sb_attention_chunk_tokens(B)), also writing the output
 * rows as the f16 hi / lo pair (row stride ld16 >= nq * hd, lo nullable) that
 * the following tensor-core GEMM takes. */
int sb_attention_paged_split(float* att, int ld_att, const float* qkv, int ld_qkv, int B, int nq,
                             int nkv, int hd, const int32_t* row_pos, const int32_t* row_slot,
                             const int32_t* page_table, int max_pages, const void* pool,
                             const void* kvmap, int64_t n_pages, int layer, int kv_dtype,
                             int max_seq, float* scratch, int* err, void* hi, void* lo, int ld16,
                             cudaStream_t st);

/* Tensor-core attention for f16 pools (head_dim 64 or 128, at most 8 query
 * heads per kv head).  The map is an opaque 128-byte CUtensorMap over the
 * pool viewed as [layers][n_pages*2*nkv*16][hd] f16. */
#define SB_KVMAP_BYTES 128
int sb_attention_mma_supported(int nq, int nkv, int hd, int kv_dtype);
int sb_attention_make_map(void* map, void* pool, int64_t n_pages, int layers, int nkv, int hd);
/* Chunk stage only (partials into `part`, same records as the CUDA-core
 * kernel; chunks of ct tokens, nchunk per row); prepare != 0 sets the
 * shared-memory attributes instead. */
int sb_attention_mma(int prepare, const void* map, const float* qkv, int ld_qkv, int B, int nq,
                     int nkv, int hd, const int32_t* row_pos, const int32_t* row_slot,
                     const int32_t* page_table, int max_pages, int64_t n_pages, int layer,
                     int nchunk, int ct, float* part, int* err, cudaStream_t st);
/* The causal prefill form of the same (attn_mma.cu): the B rows are
 * consecutive positions of one sequence (a prompt chunk); tiles of rows share
 * each streamed K/V page.  Same partial records. */
int sb_attention_prefill_mma(const void* map, const float* qkv, int ld_qkv, int B, int nq, int nkv,
                             int hd, const int32_t* row_pos, const int32_t* row_slot,
                             const int32_t* page_table, int max_pages, int64_t n_pages, int layer,
                             int nchunk, float* part, int* err, cudaStream_t st);
/* Paged attention for a prompt chunk (rows = consecutive positions of one
 * sequence) with the prefill kernel where the KV shape allows it (f16 KV,
 * a tensor map), else the decode kernels; output as sb_attention_paged_split
 * (hi may be null: f32 rows only). */
int sb_attention_paged_prefill(float* att, int ld_att, const float* qkv, int ld_qkv, int B, int nq,
                               int nkv, int hd, const int32_t* row_pos, const int32_t* row_slot,
                               const int32_t* page_table, int max_pages, const void* pool,
                               const void* kvmap, int64_t n_pages, int layer, int kv_dtype,
                               int max_seq, float* scratch, int* err, void* hi, void* lo, int ld16,
                               cudaStream_t st);

/* Tensor parallelism.  Per row, the (max logit, global index) pair of this
 * rank's vocabulary slice [v0, v0 + V) -> pairs[B] (8 bytes each); after an
 * all-gather of the pairs into all[T][B], every rank picks the first maximum
 * over the whole vocabulary and advances the positions. */
int sb_argmax_pairs(const float* logits, int ldl, int V, int B, int v0, void* pairs,
                    cudaStream_t st);
int sb_tp_epilogue(const void* all_pairs, int T, int B, const int32_t* row_slot,
                   const int32_t* row_pos, int32_t* pos, const int32_t* status,
                   int32_t* out_tokens, cudaStream_t st);
/* NCCL communicator of a tensor-parallel group (tp_nccl.c). */
int sb_tp_init(void** comm, int nranks, int rank, const void* unique_id);
int sb_tp_split(void* comm, int rank, void** out);
void sb_tp_destroy(void* comm);
int sb_tp_allreduce_sum(void* comm, float* buf, size_t n, cudaStream_t st);
int sb_tp_allgather(void* comm, const void* send, void* recv, size_t bytes, cudaStream_t st);

/* Stochastic sampling with the reference sampler's semantics
 * (util/sampling.c:9-83), one row of logits per CTA; rng[b] is advanced as
 * the reference advances its state.  scratch: B * V floats.  With pos != NULL
 * the positions advance like the greedy epilogue.  *err = 1 for a top_k above
 * SB_SAMPLE_TOPK_MAX. */
#define SB_SAMPLE_TOPK_MAX 2048
typedef struct sb_sampler { float temperature; int top_k; float top_p; int pad; } sb_sampler;
int sb_sample_rows(const float* logits, int ldl, int V, int B, const sb_sampler* cfg, uint64_t* rng,
                   float* scratch, int32_t* out, const int32_t* row_slot, const int32_t* row_pos,
                   int32_t* pos, const int32_t* status, int* err, cudaStream_t st);

/* Fills positions [0, n) of one slot with deterministic pseudo-random K/V
 * (benchmark stand-in for a prefilled prompt), allocating its pages. */
int sb_seed_context(int slot, int n, uint64_t seed, int n_layers, int nkv, int hd, int32_t* pos,
                    int32_t* page_table, int max_pages, int32_t* free_stack, int32_t* free_top,
                    void* pool, int64_t n_pages, int kv_dtype, int32_t* status,
                    cudaStream_t st);
/* Copies the first n K/V rows of one slot into dense f32 [n_layers][n][nkv*hd]. */
int sb_read_kv(int slot, int n, int n_layers, int nkv, int hd, const int32_t* page_table,
               int max_pages, const void* pool, int64_t n_pages, int kv_dtype, float* K,
               float* V, cudaStream_t st);
/* Returns the slot's pages to the device free list and zeroes its position. */
int sb_release_slot(int slot, int32_t* pos, int32_t* page_table, int max_pages,
                    int32_t* free_stack, int32_t* free_top, cudaStream_t st);
/* free_stack = [0, n_pages), free_top = n_pages. */
int sb_init_free_list(int32_t* free_stack, int32_t* free_top, int64_t n_pages, cudaStream_t st);

#ifdef __cplusplus
}
#endif
#endif
