/*
 * slate_cuda.h -- C ABI of slate-b200: a Blackwell (sm_100a) CUDA backend for
 * eating-and-drinking/slate's LLaMA-style Q4_K continuous-batching decode.
 *
 * Three layers, all plain C types (no CUDA or torch types in signatures):
 *
 *   1. The compute-backend vtable.  `slate_backend_t` is layout-identical to
 *      the reference's `struct slate_backend` (include/slate/backend.h:41-99)
 *      and `slate_backend_cuda()` replaces the reference's NULL stub
 *      (src/backend/backend_cuda_stub.c:33).  `slate_backend_cuda_t` appends
 *      status-returning batched entries after the 13 reference members, so a
 *      `const slate_backend_t*` taken from it works with unchanged callers.
 *   2. The device-resident LLaMA batch engine (`slate_llama_batch_*`): the
 *      batched counterpart of slate_llama_decode_step
 *      (src/loader/llama_infer.c:134-206) with the continuous-batching shape of
 *      slate_infer_batch_step (src/infer/engine.c:543-642, include/slate/
 *      infer.h:168-187).  Weights live in HBM, KV is paged on the GPU, and
 *      slots / page tables / positions are maintained on the device.
 *   3. A micro-batching scheduler over the batch engine with the contract of
 *      slate_scheduler_* (src/server/scheduler.c, include/slate/scheduler.h:
 *      40-60), plus helpers (GGUF loading, synthetic model writer, Q4_K
 *      quantiser) used by tests and benchmarks.
 *
 * Return codes follow the reference: 0 success, -1 bad arguments, -2 capacity
 * (cache / slots / pages / queue full), -3 bad token; -5 device error (the
 * message is available from slate_cuda_last_error()).
 *
 * When both this header and the reference's include/slate/backend.h are used
 * in one translation unit, include the reference header first.
 */
#ifndef SLATE_CUDA_H
#define SLATE_CUDA_H

#include <stddef.h>
#include <stdint.h>

#ifdef __cplusplus
extern "C" {
#endif

/* ------------------------------------------------------------------------ */
/* 1. Backend vtable                                                         */
/* ------------------------------------------------------------------------ */
#ifndef SLATE_BACKEND_H
#define SLATE_BACKEND_H
/* Identical member order and types to include/slate/backend.h:41-99. */
typedef struct slate_backend {
    const char* name;
    void* (*alloc)(size_t bytes);
    void  (*release)(void* dev_ptr);
    void  (*copy_h2d)(void* dst_dev, const void* src_host, size_t bytes);
    void  (*copy_d2h)(void* dst_host, const void* src_dev, size_t bytes);
    void  (*matvec)(float* y, const float* A, const float* x, int M, int K);
    void  (*linear_batch)(float* C, const float* X, const float* W, int B, int K, int N);
    void  (*matvec_q4k)(float* y, const void* A_q4k, const float* x, int M, int K);
    void  (*rmsnorm_row)(float* y, const float* x, const float* w, int D, float eps);
    void  (*silu_mul)(float* y, const float* gate, const float* up, int H);
    void  (*add_inplace)(float* y, const float* x, int D);
    void  (*embed_lookup)(float* y, const float* W, int token_id, int D);
    void  (*attention_step)(float* out, const float* q, const float* K_cache,
                            const float* V_cache, float* scores, int L, int D);
    void  (*sync)(void);
} slate_backend_t;
#endif

#define SLATE_CUDA_ABI_VERSION 1

/* KV element types for the paged cache. */
#define SLATE_KV_F32 0   /* the reference's dtype (llama_infer.c:225-226) */
#define SLATE_KV_F16 1   /* IEEE binary16, round-to-nearest-even on append */

/* Appended entries.  All pointers are device pointers; work is enqueued on the
 * backend's stream (sync() waits for it).  Each returns 0 or <0. */
typedef struct slate_backend_cuda {
    slate_backend_t base;          /* the 13 reference entries, same semantics */
    int abi_version;               /* SLATE_CUDA_ABI_VERSION */
    int device;                    /* CUDA ordinal the singleton is bound to */
    /* Y[B,M] = X[B,K] · Q4K(A)[M,K]ᵀ ; K % 256 == 0.  Batched matvec_q4k. */
    int (*matmul_q4k_batch)(float* Y, const void* A_q4k, const float* X, int B, int M, int K);
    /* Y[B,M] = X[B,K] · A[M,K]ᵀ (f32, A row-major [out, in] like matvec). */
    int (*matmul_f32_batch)(float* Y, const float* A, const float* X, int B, int M, int K);
    /* B independent rmsnorm_row calls over rows of stride D. */
    int (*rmsnorm_rows)(float* Y, const float* X, const float* w, int B, int D, float eps);
    /* First-max argmax per row (util/sampling.c:14-18): out[b] over logits[b*V..]. */
    int (*argmax_rows)(int32_t* out, const float* logits, int B, int V);
    /* RoPE (llama_infer.c:77-92) on q [B, nq*hd] and k [B, nkv*hd] in place at
     * per-row positions pos[B], then K/V append into the paged cache (layout
     * documented at slate_llama_batch_new_desc). */
    int (*rope_kv_append_paged)(float* q, float* k, const float* v, const int32_t* pos,
                                const int32_t* row_slot, const int32_t* page_table,
                                int max_pages, void* kv_pool, int64_t n_pages, int layer,
                                int B, int nq, int nkv, int hd, int kv_dtype,
                                const float* rope_cos, const float* rope_sin);
    /* GQA attention (llama_infer.c:97-129) of q [B, nq*hd] against paged KV
     * holding ctx = pos[b]+1 tokens per row; out [B, nq*hd]. */
    int (*attention_paged_gqa)(float* out, const float* q, const int32_t* pos,
                               const int32_t* row_slot, const int32_t* page_table,
                               int max_pages, const void* kv_pool, int64_t n_pages,
                               int layer, int B, int nq, int nkv, int hd, int kv_dtype);
    /* matmul_q4k_batch on the tensor cores (tcgen05, f32 accumulate):
     * passes 1 = f16 x f16 operands, 3 = f16 hi/lo split of both operands
     * (f32-level products), both for 16 <= B; 2 = exact f16 weights (sc*q)
     * against x as f16 hi/lo with the Q4_K block scales applied per
     * super-block (f32-level products), any B >= 1; 4 = the small-batch
     * kernel: the 4-bit quants (exact in f16) against x as f16 hi/lo through
     * mma.sync, per 32-element sub-block d*sc*sum(q*x) - dmin*m*sum(x) in f32
     * (the reference's own structure, util/quant.c:210-304), 1 <= B <= 16.
     * M % 128 == 0, K % 256 == 0.
     * Synchronous: returns -5 if the device reported a pipeline timeout. */
    int (*matmul_q4k_batch_tc)(float* Y, const void* A_q4k, const float* X, int B, int M, int K,
                               int passes);
} slate_backend_cuda_t;

/* Reference-compatible accessor.  Returns NULL (exactly like the stub at
 * src/backend/backend_cuda_stub.c:33) unless the environment variable
 * SLATE_CUDA_BACKEND=1 is set and a device is present, so that
 * slate_backend_default() (src/backend/backend_cpu.c:189-194) keeps choosing the
 * CPU for the reference's own oracle tests.  Explicit opt-in: below. */
const slate_backend_t* slate_backend_cuda(void);

/* Explicit constructor: binds the process-wide singleton to `device` (first
 * call wins; later calls with another device return NULL). */
const slate_backend_cuda_t* slate_backend_cuda_create(int device);

/* The 13 reference entries in a host-coherent form, for callers written
 * against the CPU backend's semantics -- the reference's GPT-style inference
 * engine (src/infer/engine.c: host memset / memcpy on alloc'd buffers at
 * :276-277, 411-412, 586-591; host weight, scratch and logits pointers passed
 * to the entries; results read without sync()).  alloc returns managed memory,
 * copies accept any pointers, and every entry returns only after its kernel has
 * finished.  Kernels read the pointers they are given directly: memory from
 * this alloc, pinned / registered host memory, or -- only where
 * slate_cuda_pageable_memory_access(device) is 1 (HMM / ATS) -- any host
 * memory, such as a module's own weights.  Same device and stream as
 * slate_backend_cuda_create(device), on which it calls first. */
const slate_backend_t* slate_backend_cuda_host_coherent(int device);
/* 1 if kernels on `device` may read pageable host memory (HMM / ATS), 0 if
 * not, -5 on error. */
int slate_cuda_pageable_memory_access(int device);

/* Text of the last device-side or argument error seen by this library on the
 * calling thread ("" if none). */
const char* slate_cuda_last_error(void);

struct slate_sampler_config;
/* Draws one token per row of DEVICE logits (B rows of V, row stride ld) with
 * the reference sampler's rules (slate_sample_token, util/sampling.c:9-83)
 * from HOST configurations and RNG states; out_tokens (host) and rng_state
 * (advanced as the reference advances it) are written back.  Synchronous. */
int slate_cuda_sample_rows(int32_t* out_tokens, const float* logits, int ld, int B, int V,
                           const struct slate_sampler_config* cfg, uint64_t* rng_state);

/* attention_paged_gqa for callers that cannot allocate device memory during
 * the call (an allocator that has already given all free HBM to its KV pool;
 * a latency-critical loop that must not enter the driver's allocator).  This
 * entry point has no counterpart in the reference.  Same arguments, kernels
 * and results as the vtable entry, plus the stream to run on (NULL = the
 * legacy default stream, which the call synchronises before returning).
 * Its scratch is one fixed device array per device of
 * SLATE_CUDA_NOALLOC_SCRATCH_FLOATS floats (8 MiB); a call needs
 * B * nq * ceil(max_pages * 16 / ct) * (hd + 2) of them, ct being the engine's
 * attention chunk for B rows (64 tokens below 3 rows, 128 at 3, up to 1024 from 16),
 * doubled up to 1024 tokens until the partials fit, and is rejected with -1
 * when even 1024-token chunks do not fit.  All calls on a device share the
 * array, so calls that overlap on the GPU race: serialise them.  The first
 * call on a device resolves the array's address (cudaGetSymbolAddress) with
 * that device current; make it before any stream capture.  Each call waits
 * for its stream before returning (it reads the kernels' error word).  No
 * cudaMalloc/cudaFree. */
#define SLATE_CUDA_NOALLOC_SCRATCH_FLOATS (1u << 21)
int slate_cuda_attention_paged_gqa_noalloc(float* out, const float* q, const int32_t* pos,
                                           const int32_t* row_slot, const int32_t* page_table,
                                           int max_pages, const void* kv_pool, int64_t n_pages,
                                           int layer, int B, int nq, int nkv, int hd,
                                           int kv_dtype, void* stream);

/* ------------------------------------------------------------------------ */
/* 2. Device-resident LLaMA batch engine                                     */
/* ------------------------------------------------------------------------ */

/* One transformer block's weights, member-for-member the reference's
 * slate_llama_layer_t (include/slate/llama.h:69-86).  Pointers are HOST
 * pointers (e.g. into the GGUF mmap); dtypes are slate_dtype_t values
 * (0 = f32, 18 = Q4_K). */
typedef struct slate_llama_layer_desc {
    const void* attn_norm;
    const void* attn_q;
    const void* attn_k;
    const void* attn_v;
    const void* attn_output;
    const void* ffn_norm;
    const void* ffn_gate;
    const void* ffn_up;
    const void* ffn_down;
    int attn_q_dtype, attn_k_dtype, attn_v_dtype, attn_output_dtype;
    int ffn_gate_dtype, ffn_up_dtype, ffn_down_dtype;
} slate_llama_layer_desc_t;

/* A model as the reference's loader exposes it: the fields of
 * slate_llama_config_t (include/slate/llama.h:53-65) plus the accessors
 * slate_llama_token_embd/_dtype, _output_norm, _output/_dtype, _layer. */
typedef struct slate_llama_desc {
    int n_layers, d_model, ffn_hidden, n_heads, n_kv_heads, head_dim, max_seq, vocab;
    float theta_base, rms_eps;
    int tied_output;
    const void* token_embd;  int token_embd_dtype;   /* f32 [vocab, d_model] */
    const void* output_norm;                          /* f32 [d_model] */
    const void* output;      int output_dtype;       /* [vocab, d_model] */
    const slate_llama_layer_desc_t* const* layers;    /* [n_layers] */
} slate_llama_desc_t;

typedef struct slate_cuda_opts {
    int device;          /* CUDA ordinal */
    int max_batch;       /* rows per step, 1..1024 */
    int max_slots;       /* concurrently open sequences (0 = max_batch) */
    int kv_dtype;        /* SLATE_KV_F32 or SLATE_KV_F16 */
    int max_seq;         /* per-sequence cap (0 = the model's max_seq) */
    int64_t kv_pages;    /* pool size in 16-token pages (0 = from kv_bytes) */
    size_t kv_bytes;     /* pool budget (0 = 90% of free HBM after weights) */
    int use_graphs;      /* capture one CUDA graph per batch size (1 = yes) */
    int gemm_path;       /* 0 auto (tcgen05 3-pass hi/lo split: the stream-K
                            kernel from 128 rows, the tile-per-CTA kernel below),
                            1 CUDA-core kernels only, 2 tcgen05 1-pass f16, 3 the
                            3-pass tile-per-CTA kernel only, 4 Q4_K on the
                            exact-weight stream-K tcgen05 kernel (2 f16 passes),
                            5 Q4_K on the 3-pass stream-K kernel from 16 rows,
                            6 as 4 with x rounded once to f16 (1 pass) */
    int attn_path;       /* 0 auto (tensor cores for f16 KV where the shape allows),
                            1 CUDA-core attention only */
    /* Tensor parallelism (the 70B plan): tp_size ranks, one process or thread
     * per GPU, each creating its engine with its tp_rank and the same tp_id
     * (from slate_cuda_tp_unique_id on one rank).  Wq/Wk/Wv and gate/up are
     * split by rows (heads / FFN units), Wo and down by columns with an
     * all-reduce(sum) of the [n, d_model] activations after each, the LM head
     * by vocabulary rows with a gathered (max, index) per row for the greedy
     * token.  Needs n_kv_heads, vocab and ffn_hidden / 256 divisible by
     * tp_size.  All ranks must make the same calls in the same order (steps,
     * opens, closes); logits are gathered when any is requested.  tp_size 0
     * or 1 = one GPU. */
    int tp_size;
    int tp_rank;
    unsigned char tp_id[128];
    /* Nibble packing of the model's Q4_K tensors: 0 = Slate's (sub-block j in
     * qs[16j..16j+15], low nibble element i, high nibble i + 16;
     * util/quant.c:182-199), 1 = llama.cpp / ggml's (64-element pairs: byte
     * 32g + e holds element e of sub-block 2g low and of 2g + 1 high), repacked
     * to Slate's at upload, so real llama.cpp Q4_K files decode as intended. */
    int q4k_order;
    /* 0 or 1: the whole batch as one chain of kernels.  2 (stream-K
     * tensor-core GEMMs, max_batch >= 32): a decode step of more than
     * max_batch / 2 rows runs its layers as two independent halves of the
     * batch on two streams, the halves' attentions taking turns, so that one
     * half's attention (bound by HBM) can run beside the other half's
     * projections (bound by the tensor cores).  With tensor parallelism each
     * half's all-reduces use their own communicator (split from the group's at
     * creation, a collective), so one half's all-reduce runs beside the other
     * half's GEMMs.  Prompt-chunk steps always run as one chain. */
    int lanes;
} slate_cuda_opts_t;

/* A fresh NCCL unique id (128 bytes) for a tensor-parallel group: create it on
 * one rank and hand it to every rank's slate_cuda_opts_t.tp_id. */
int slate_cuda_tp_unique_id(void* out, size_t n);

typedef struct slate_llama_batch slate_llama_batch_t;

#ifndef SLATE_SAMPLING_H
#define SLATE_SAMPLING_H
/* Identical to include/slate/sampling.h:15-20. */
typedef struct slate_sampler_config {
    float temperature;   /* 0 = greedy / argmax; > 0 = sample */
    int   top_k;         /* 0 = disabled; > 0 = restrict to top-k tokens */
    float top_p;         /* 0 = disabled; (0, 1] = nucleus sampling */
    uint64_t seed;
} slate_sampler_config_t;
#endif

/* Uploads the weights once and creates the KV page pool.
 * KV pool layout in HBM (one pool, layer-major):
 *   pool[layer][page][kv = 0 (K) | 1 (V)][kv_head][16 tokens][head_dim]
 * Returns NULL on failure (slate_cuda_last_error() says why). */
slate_llama_batch_t* slate_llama_batch_new_desc(const slate_llama_desc_t* model,
                                                const slate_cuda_opts_t* opts);
/* Convenience: open a LLaMA GGUF (the format the reference's
 * slate_gguf_open/slate_llama_open read) and upload it.  The file is only
 * needed during the call. */
slate_llama_batch_t* slate_llama_batch_new_gguf(const char* path, const slate_cuda_opts_t* opts);
void slate_llama_batch_free(slate_llama_batch_t* b);

/* Model/engine facts for callers sizing buffers. */
int slate_llama_batch_vocab(const slate_llama_batch_t* b);
int slate_llama_batch_max_batch(const slate_llama_batch_t* b);
int slate_llama_batch_max_seq(const slate_llama_batch_t* b);
int64_t slate_llama_batch_free_pages(const slate_llama_batch_t* b);

/* Sequence slots (the device-side counterpart of slate_llama_session_new /
 * _free / _position, llama_infer.c:212-260).  open -> slot >= 0 or -2. */
int slate_llama_batch_open(slate_llama_batch_t* b);
int slate_llama_batch_close(slate_llama_batch_t* b, int slot);
int slate_llama_batch_position(const slate_llama_batch_t* b, int slot);

/* One continuous-batching step over HOST buffers: row r appends tokens[r]
 * to sequence slots[r] (distinct slots) and yields its greedy next token in
 * out_tokens[r] (nullable) and, when out_logits != NULL, its logits in
 * out_logits[r*vocab ..].  1 <= n <= max_batch.  Returns 0 / -1 / -2 / -3 /
 * -5; on error no sequence advances. */
int slate_llama_batch_step(slate_llama_batch_t* b, const int32_t* slots, int n,
                           const int32_t* tokens, int32_t* out_tokens, float* out_logits);

/* One step whose next tokens are drawn by the reference sampler's rules
 * (slate_sample_token, util/sampling.c:9-83) on the device: per row a
 * sampler configuration and an RNG state, advanced exactly as the reference
 * advances it (rows with temperature <= 0 take the greedy token and keep their
 * state).  Same slots / positions / return codes as slate_llama_batch_step;
 * top_k up to 2048 (or >= vocab, i.e. off).  Not available with tensor
 * parallelism. */
int slate_llama_batch_step_sample(slate_llama_batch_t* b, const int32_t* slots, int n,
                                  const int32_t* tokens, const slate_sampler_config_t* cfg,
                                  uint64_t* rng_state, int32_t* out_tokens, float* out_logits);

/* The same step on DEVICE buffers, enqueued on `stream` (a cudaStream_t, or
 * NULL for the engine's stream) without host synchronisation; token / slot
 * validation happens on the device and is reported by
 * slate_llama_batch_sync(). */
int slate_llama_batch_step_device(slate_llama_batch_t* b, const int32_t* d_slots, int n,
                                  const int32_t* d_tokens, int32_t* d_out_tokens,
                                  float* d_out_logits, void* stream);

/* Waits for the engine's work; returns the first device-side status since the
 * last call (0, -2 or -3) or -5 on a CUDA error. */
int slate_llama_batch_sync(slate_llama_batch_t* b);

/* Token-by-token prompt processing for one slot, equivalent to n decode steps
 * (slate_llama_prefill, llama_infer.c:262-272).  Logits of the last position
 * go to out_logits (nullable). */
int slate_llama_batch_prefill(slate_llama_batch_t* b, int slot, const int32_t* tokens,
                              int n_tokens, float* out_logits);

/* Benchmark stand-in for a prefilled prompt: gives `slot` n_tokens positions
 * whose K/V rows are seeded pseudo-random values (|v| < 1, deterministic in
 * seed), so decode steps read a context of that length. */
int slate_llama_batch_seed_context(slate_llama_batch_t* b, int slot, int n_tokens,
                                   uint64_t seed);
/* Reads back the K/V rows of one slot ([n_layers][n][kv_dim] each, f32) for
 * tests; n <= position. */
int slate_llama_batch_read_kv(slate_llama_batch_t* b, int slot, int n, float* K, float* V);

/* Device stream the engine enqueues on (a cudaStream_t). */
void* slate_llama_batch_stream(slate_llama_batch_t* b);

/* Number of kernel launches one step of n rows enqueues (for accounting). */
int slate_llama_batch_launches_per_step(const slate_llama_batch_t* b, int n);

/* Kernel groups of the step that slate_llama_batch_profile can time. */
#define SLATE_PROF_ATTENTION 0   /* paged attention: partial + combine kernels */
#define SLATE_PROF_QKV       1   /* fused Q|K|V GEMM */
#define SLATE_PROF_WO        2   /* attention output GEMM */
#define SLATE_PROF_GATE_UP   3   /* fused gate|up GEMM with SiLU*up epilogue */
#define SLATE_PROF_DOWN      4   /* FFN down GEMM */
#define SLATE_PROF_LM_HEAD   5   /* vocabulary projection */
#define SLATE_PROF_STEP      6   /* one whole step (same graph as _step) */
#define SLATE_PROF_ALLREDUCE 7   /* tensor parallel only: the all-reduce(sum) of
                                    [n, d_model] activations that follows Wo and
                                    down (a collective: every rank calls it) */
/* Times `iters` back-to-back launches of one kernel group for the rows of the
 * most recent step (the first n rows; `layer` selects the layer's weights and
 * KV) on the engine stream with CUDA events, after one untimed launch; the
 * mean milliseconds per launch go to *ms.  GEMM groups write into scratch,
 * the attention group only rewrites its own output, so the sequences' state
 * is unchanged -- except PROF_STEP, which advances every row like a step.
 * Call only after slate_llama_batch_step/_step_device with the same n. */
int slate_llama_batch_profile(slate_llama_batch_t* b, int kernel, int n, int layer, int iters,
                              float* ms);

/* ------------------------------------------------------------------------ */
/* 3. Scheduler (single decoder thread, scheduler.c:45-99 contract)          */
/* ------------------------------------------------------------------------ */
typedef struct slate_llama_scheduler slate_llama_scheduler_t;
slate_llama_scheduler_t* slate_llama_scheduler_new(slate_llama_batch_t* b, int max_batch);
void slate_llama_scheduler_free(slate_llama_scheduler_t* s);
/* Blocks until the decoder thread has advanced `slot` by `token`; greedy
 * next token to *out_token (nullable), logits to out_logits (nullable).
 * Returns the step's code, or -2 when the queue (256) is full. */
int slate_llama_scheduler_decode(slate_llama_scheduler_t* s, int slot, int32_t token,
                                 int32_t* out_token, float* out_logits);
int      slate_llama_scheduler_pending(const slate_llama_scheduler_t* s);
uint64_t slate_llama_scheduler_total_batches(const slate_llama_scheduler_t* s);
double   slate_llama_scheduler_avg_batch_size(const slate_llama_scheduler_t* s);

/* ------------------------------------------------------------------------ */
/* Helpers: GGUF reading, Q4_K quantisation, synthetic models                */
/* ------------------------------------------------------------------------ */
typedef struct slate_gguf_model slate_gguf_model_t;
/* Parses a LLaMA GGUF (v2/v3; loader/gguf.c + loader/llama.c semantics) and
 * fills `desc` with pointers into its mmap.  NULL on failure. */
slate_gguf_model_t* slate_gguf_model_open(const char* path, slate_llama_desc_t* desc);
void slate_gguf_model_close(slate_gguf_model_t* g);

/* Quantises rows of f32 into Slate's Q4_K layout with the reference fixture
 * quantiser's arithmetic (tools/make_tiny_llama_q4k_gguf.py:39-87: per
 * sub-block min/max, round-half-even, f16 d/dmin).  K % 256 == 0. */
int slate_q4k_quantize_rows(void* dst, const float* src, int64_t rows, int K);

typedef struct slate_synth_config {
    int n_layers, d_model, ffn_hidden, n_heads, n_kv_heads, vocab, max_seq;
    float theta_base, rms_eps;
    int q4k;              /* 1: linear weights Q4_K; 0: all f32 */
    int tied_output;      /* 1: omit output.weight */
    uint64_t seed;
    int n_threads;        /* 0 = all online CPUs */
    int layer_period;     /* 0: every layer drawn independently; p > 0: layer l
                             repeats the weights of layer l % p (a file of a
                             large model written in a fraction of the time;
                             the engine still holds one copy per layer) */
    int q4k_order;        /* 0: Slate's nibble packing; 1: llama.cpp / ggml's */
    int embd_f16;         /* 0: f32 token_embd / output; 1: stored as f16;
                             2: f32 holding the f16-rounded values */
} slate_synth_config_t;
/* Writes a LLaMA GGUF with N(0, 0.02) weights (counter-based, deterministic
 * in seed), unit norm gains, f32 embedding/head.  Returns 0 or <0. */
int slate_synth_llama_gguf(const char* path, const slate_synth_config_t* cfg);

#ifdef __cplusplus
}
#endif
#endif /* SLATE_CUDA_H */
