/*
 * slate_oracle.h -- CPU restatement of eating-and-drinking/slate's LLaMA
 * Q4_K decode path.  TEST INFRASTRUCTURE ONLY: this is the checker that the
 * CUDA path is compared against.  Nothing in the product library links it;
 * only tests/, __graft_entry__.smoke() and bench.py's cpu_baseline leg load it.
 *
 * Every function names the reference file:line whose behaviour it restates.
 * Parity pin: the golden fixtures under tests/golden/ (produced by the
 * reference's own tools/make_*.py scripts) and, where the reference builds here, the
 * reference library compiled by oracle/Makefile into oracle/_ref/.
 */
#ifndef SLATE_ORACLE_H
#define SLATE_ORACLE_H

#include <stddef.h>
#include <stdint.h>

#ifdef __cplusplus
extern "C" {
#endif

/* ---- numerics primitives ---------------------------------------------- */
float orc_f16_to_f32(uint16_t h);                      /* util/precision.c:10-29 */
void  orc_dequant_q4k(float* dst, const void* src, int64_t n);   /* util/quant.c:168-202 */
float orc_dot_q4k(const void* blocks, const float* y, int64_t n); /* util/quant.c:210-304 */
void  orc_q4k_matvec(float* y, const void* A, const float* x, int M, int K); /* quant.c:306-313 */
void  orc_matvec_f32(float* y, const float* A, const float* x, int M, int K); /* backend_cpu.c:33-36 */
void  orc_linear_batch(float* C, const float* X, const float* W, int B, int K, int N); /* backend_cpu.c:38-42 */
void  orc_rmsnorm_row(float* y, const float* x, const float* w, int D, float eps); /* backend_cpu.c:48-76 */
void  orc_silu_mul(float* y, const float* g, const float* u, int H); /* backend_cpu.c:78-97 */
void  orc_rope_row(float* row, int n_heads, int head_dim, int pos, float theta); /* llama_infer.c:77-92 */
/* cos/sin[pos][hd/2] of the angles orc_rope_row uses (llama_infer.c:83-85). */
void  orc_rope_tables(float* cos_t, float* sin_t, int max_seq, int head_dim, float theta);
void  orc_attention_gqa(float* out, const float* q, const float* K, const float* V,
                        float* scores, int L, int nq, int nkv, int hd);   /* llama_infer.c:97-129 */
void  orc_attention_step(float* out, const float* q, const float* K, const float* V,
                         float* scores, int L, int D);                    /* backend_cpu.c:117-166 */
int   orc_argmax(const float* p, int n);                                  /* util/sampling.c:14-18 */

/* ---- model + session (loader/gguf.c, loader/llama.c, loader/llama_infer.c) */
typedef struct orc_model orc_model_t;
typedef struct orc_session orc_session_t;

typedef struct orc_config {
    int n_layers, d_model, ffn_hidden, n_heads, n_kv_heads, head_dim, max_seq, vocab;
    float theta_base, rms_eps;
    int tied_output;
} orc_config_t;

orc_model_t* orc_model_open(const char* gguf_path);     /* gguf.c:122-186 + llama.c:42-140 */
void         orc_model_close(orc_model_t* m);
const orc_config_t* orc_model_config(const orc_model_t* m);
/* Raw tensor access for tests: returns data pointer and GGML-side dtype
 * mapped to slate's enum (0 = f32, 18 = Q4_K), or NULL when absent. */
const void*  orc_model_tensor(const orc_model_t* m, const char* name, int* slate_dtype);

orc_session_t* orc_session_new(const orc_model_t* m, int max_seq_override);
void           orc_session_free(orc_session_t* s);
int            orc_session_position(const orc_session_t* s);
/* One token through the model; logits[vocab].  0 / -2 (full) / -3 (bad token).
 * llama_infer.c:134-206 */
int            orc_decode_step(orc_session_t* s, int32_t token, float* logits);
/* Seeds positions [0, n) of the session's cache with the given rows
 * (K, V: [n_layers][n][kv_dim]) and sets position = n.  Used to stand in for
 * a prefilled prompt when comparing long contexts. */
int            orc_session_seed_kv(orc_session_t* s, int n, const float* K, const float* V);

/* Runs n_sessions independent sessions in parallel pthreads (one reference
 * session per core), each decoding tokens[i*n_steps + t] (teacher forced),
 * writing logits when out != NULL ([n_sessions][n_steps][vocab]) and greedy
 * argmax to out_tok ([n_sessions][n_steps]).  Returns 0 or the first error. */
int orc_decode_many(const orc_model_t* m, int n_sessions, int n_steps,
                    const int32_t* tokens, float* out, int32_t* out_tok, int n_threads);

#ifdef __cplusplus
}
#endif
#endif
