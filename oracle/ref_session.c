/*
 * ref_session.c -- TEST INFRASTRUCTURE.  The reference's src/loader/llama_infer.c,
 * compiled unmodified (included whole), plus two accessors the CPU timing needs.
 *
 * bench.py times slate_llama_decode_step (src/loader/llama_infer.c:274-279) at
 * the benchmark's context lengths.  A real history of a few thousand tokens
 * would take hours to prefill on the CPU, and the reference exposes only a
 * position getter (slate_llama_session_position, :258-260).  The accessors
 * below work through the reference's own struct definition
 * (struct slate_llama_session, :52-71), so the layout is the compiler's, not a
 * hard-coded offset.  oracle/Makefile builds this translation unit in place of
 * the plain llama_infer.c object of _ref/libslate_ref.so.
 */
#include "loader/llama_infer.c"

/* Sets the session's position.  Attention then reads rows 0..position of the
 * session's KV cache (:167-179), whatever they hold. */
int slate_ref_session_set_position(slate_llama_session_t* s, int position) {
    if (!s || position < 0 || position >= slate_llama_config(s->model)->max_seq) return -1;
    s->position = position;
    return 0;
}

static uint64_t ref_mix64(uint64_t z) {
    z += 0x9e3779b97f4a7c15ull;
    z = (z ^ (z >> 30)) * 0xbf58476d1ce4e5b9ull;
    z = (z ^ (z >> 27)) * 0x94d049bb133111ebull;
    return z ^ (z >> 31);
}

/* Gives the session an n-token history: rows 0..n-1 of every layer's K and V
 * cache get the values the CUDA engine's slate_llama_batch_seed_context writes
 * for the same seed (element i of the [layer][K|V][token][kv_head][head_dim]
 * order is 2*u - 1, u the top 53 bits of splitmix64(seed ^ i*golden) scaled to
 * [0, 1), as f32), then the position becomes n.  Rows written with real values
 * also keep the CPU honest: never-written calloc rows all map the kernel's
 * shared zero page and would be served from cache. */
int slate_ref_session_seed_context(slate_llama_session_t* s, int n, uint64_t seed) {
    if (!s || n < 0 || n >= slate_llama_config(s->model)->max_seq) return -1;
    const slate_llama_config_t* c = slate_llama_config(s->model);
    const int64_t kv_dim = (int64_t)c->n_kv_heads * c->head_dim, max_seq = c->max_seq;
    for (int64_t layer = 0; layer < c->n_layers; ++layer)
        for (int64_t kv = 0; kv < 2; ++kv) {
            float* base = (kv ? s->V_cache : s->K_cache) + layer * max_seq * kv_dim;
            for (int64_t t = 0; t < n; ++t)
                for (int64_t e = 0; e < kv_dim; ++e) {
                    const uint64_t i = (uint64_t)(((layer * 2 + kv) * n + t) * kv_dim + e);
                    const uint64_t z = ref_mix64(seed ^ (i * 0x9e3779b97f4a7c15ull));
                    base[t * kv_dim + e] =
                        (float)((double)(z >> 11) * (1.0 / 9007199254740992.0)) * 2.0f - 1.0f;
                }
        }
    s->position = n;
    return 0;
}
