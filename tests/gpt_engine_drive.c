/*
 * gpt_engine_drive.c -- TEST INFRASTRUCTURE: runs the reference's GPT-style
 * inference engine (src/infer/engine.c, compiled unmodified into
 * oracle/_ref/libslate_ref.so) on a compute backend chosen by the caller, so a
 * test can compare the reference's CPU backend with this library's CUDA vtable
 * under the same, unchanged engine code.
 *
 * The model is the reference's own causal LM (slate_module_causal_lm_new,
 * include/slate/transformer.h:44-48) with seeded random weights, as in the
 * reference's tests/test_infer.c.  n_seq sessions each prefill a prompt of
 * prompt_len + s tokens (slate_infer_prefill), then advance together through
 * `steps` calls of slate_infer_batch_step (engine.c:543-642), teacher-forced
 * with a fixed token schedule so that both backends see the same inputs.
 * Logits go to out: per session its prefill logits, then per step the batch's
 * [n_seq][vocab] rows -- (1 + steps) * n_seq * vocab floats in all.
 *
 * oracle/Makefile builds this file against the reference headers into
 * oracle/_ref/libslate_gpt_drive.so.
 */
#include "slate/slate.h"
#include "slate/transformer.h"
#include "slate/infer.h"
#include "slate/backend.h"

#include <stdlib.h>

int gpt_engine_drive(const slate_backend_t* backend, int vocab, int max_seq, int d_model,
                     int n_layers, int ffn_hidden, int n_seq, int prompt_len, int steps,
                     float* out) {
    if (n_seq < 1 || prompt_len < 1 || steps < 0 || prompt_len + n_seq + steps > max_seq)
        return -1;
    if (!backend) backend = slate_backend_cpu();
    int rc = -1;
    slate_arena_t* arena = slate_arena_create((size_t)64 << 20);
    slate_module_t* model = arena ? slate_module_causal_lm_new(arena, vocab, max_seq, d_model,
                                                               n_layers, ffn_hidden, 1e-5f,
                                                               0xABCDull)
                                  : NULL;
    slate_infer_engine_t* eng = model ? slate_infer_engine_new_ex(model, n_layers, d_model, vocab,
                                                                  ffn_hidden, max_seq, backend)
                                      : NULL;
    slate_infer_session_t** sess = (slate_infer_session_t**)calloc((size_t)n_seq, sizeof(*sess));
    int32_t* tok = (int32_t*)malloc(sizeof(int32_t) * (size_t)(prompt_len + n_seq + steps));
    slate_infer_batch_t* batch = eng ? slate_infer_batch_new(eng, n_seq) : NULL;
    if (!batch || !sess || !tok) goto done;
    for (int s = 0; s < n_seq; ++s) {
        sess[s] = slate_infer_session_new(eng);
        if (!sess[s]) goto done;
        const int n = prompt_len + s;
        for (int i = 0; i < n; ++i) tok[i] = (int32_t)((i * 7 + s * 3 + 1) % vocab);
        if (slate_infer_prefill(sess[s], tok, n, out + (size_t)s * vocab) != 0) goto done;
    }
    for (int t = 0; t < steps; ++t) {
        for (int s = 0; s < n_seq; ++s) tok[s] = (int32_t)((t * 13 + s * 5 + 2) % vocab);
        if (slate_infer_batch_step(batch, sess, n_seq, tok,
                                   out + (size_t)(1 + t) * n_seq * vocab) != 0)
            goto done;
    }
    rc = 0;
done:
    if (sess)
        for (int s = 0; s < n_seq; ++s)
            if (sess[s]) slate_infer_session_free(sess[s]);
    if (batch) slate_infer_batch_free(batch);
    if (eng) slate_infer_engine_free(eng);
    if (model) slate_module_destroy(model);
    if (arena) slate_arena_destroy(arena);
    free(sess);
    free(tok);
    return rc;
}
