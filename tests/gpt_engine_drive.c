/*
 * gpt_engine_drive.c -- TEST INFRASTRUCTURE: runs the reference's GPT-style
 * inference engine (src/infer/engine.c, compiled unmodified into
 * oracle/_ref/libslate_ref.so) on a compute backend chosen by the caller, so a
 * test can compare the reference's CPU backend with this library's CUDA vtable
 * under the same, unchanged engine code.
 *
 * The model is the reference's own causal LM (slate_module_causal_lm_new,
 * include/slate/transformer.h:44-48) with seeded random weights, as in the
 * reference's tests/test_infer.c.  n_seq sessions take a prompt and then
 * advance together through `steps` calls of slate_infer_batch_step
 * (engine.c:543-642), teacher-forced with a fixed token schedule so that both
 * backends see the same inputs.
 *
 * relocate == 0: the engine as the reference's callers use it -- weights in
 * the module's host arena, prompts through slate_infer_prefill (whose scratch
 * is host calloc, engine.c:446), logits into the caller's buffer.  A GPU
 * backend then needs a device that reads pageable host memory.
 * relocate == 1: the model is first moved onto the backend (every parameter
 * copied into the backend's alloc'd memory with copy_h2d, the module's tensors
 * pointed at the copies), prompts run through slate_infer_batch_step token by
 * token, and logits land in an alloc'd buffer copied out with copy_d2h -- the
 * engine code is still the reference's, and it only hands the backend memory
 * the backend allocated.
 *
 * Logits go to out: per session its last prompt position's logits, then per
 * step the batch's [n_seq][vocab] rows -- (1 + steps) * n_seq * vocab floats.
 *
 * oracle/Makefile builds this file against the reference headers into
 * oracle/_ref/libslate_gpt_drive.so.
 */
#include "slate/slate.h"
#include "slate/transformer.h"
#include "slate/infer.h"
#include "slate/backend.h"

#include <stdlib.h>
#include <string.h>

static int32_t prompt_token(int s, int i, int vocab) { return (int32_t)((i * 7 + s * 3 + 1) % vocab); }

int gpt_engine_drive(const slate_backend_t* backend, int vocab, int max_seq, int d_model,
                     int n_layers, int ffn_hidden, int n_seq, int prompt_len, int steps,
                     int relocate, float* out) {
    if (n_seq < 1 || prompt_len < 1 || steps < 0 || prompt_len + n_seq + steps > max_seq)
        return -1;
    if (!backend) backend = slate_backend_cpu();
    int rc = -1;
    const size_t row = (size_t)vocab * sizeof(float);
    slate_arena_t* arena = slate_arena_create((size_t)64 << 20);
    slate_module_t* model = arena ? slate_module_causal_lm_new(arena, vocab, max_seq, d_model,
                                                               n_layers, ffn_hidden, 1e-5f,
                                                               0xABCDull)
                                  : NULL;
    slate_param_set_t ps;
    int have_ps = 0;
    void** moved = NULL;
    void** orig = NULL;
    float* lg = NULL;
    slate_infer_engine_t* eng = NULL;
    slate_infer_session_t** sess = (slate_infer_session_t**)calloc((size_t)n_seq, sizeof(*sess));
    int32_t* tok = (int32_t*)malloc(sizeof(int32_t) * (size_t)(prompt_len + n_seq + steps));
    slate_infer_batch_t* batch = NULL;
    if (!model || !sess || !tok) goto done;
    if (relocate) {
        if (slate_param_set_init(&ps) != 0) goto done;
        have_ps = 1;
        slate_module_register_params(model, &ps);
        moved = (void**)calloc((size_t)ps.n_params, sizeof(void*));
        orig = (void**)calloc((size_t)ps.n_params, sizeof(void*));
        if (!moved || !orig) goto done;
        for (int i = 0; i < ps.n_params; ++i) {
            slate_tensor_t* t = ps.params[i];
            const size_t bytes = slate_tensor_nbytes(t);
            moved[i] = backend->alloc(bytes);
            if (!moved[i]) goto done;
            backend->copy_h2d(moved[i], t->data, bytes);
            orig[i] = t->data;
            t->data = moved[i];
        }
        lg = (float*)backend->alloc((size_t)n_seq * row);
        if (!lg) goto done;
    }
    eng = slate_infer_engine_new_ex(model, n_layers, d_model, vocab, ffn_hidden, max_seq, backend);
    batch = eng ? slate_infer_batch_new(eng, n_seq) : NULL;
    if (!batch) goto done;
    for (int s = 0; s < n_seq; ++s)
        if (!(sess[s] = slate_infer_session_new(eng))) goto done;
    if (relocate) {
        /* the prompts through the batch step, one position per call */
        for (int i = 0; i < prompt_len; ++i) {
            for (int s = 0; s < n_seq; ++s) tok[s] = prompt_token(s, i, vocab);
            if (slate_infer_batch_step(batch, sess, n_seq, tok, lg) != 0) goto done;
        }
        backend->copy_d2h(out, lg, (size_t)n_seq * row);
    } else {
        for (int s = 0; s < n_seq; ++s) {
            for (int i = 0; i < prompt_len; ++i) tok[i] = prompt_token(s, i, vocab);
            if (slate_infer_prefill(sess[s], tok, prompt_len, out + (size_t)s * vocab) != 0) goto done;
        }
    }
    for (int t = 0; t < steps; ++t) {
        float* dst = out + (size_t)(1 + t) * n_seq * vocab;
        for (int s = 0; s < n_seq; ++s) tok[s] = (int32_t)((t * 13 + s * 5 + 2) % vocab);
        if (slate_infer_batch_step(batch, sess, n_seq, tok, relocate ? lg : dst) != 0) goto done;
        if (relocate) backend->copy_d2h(dst, lg, (size_t)n_seq * row);
    }
    rc = 0;
done:
    if (sess)
        for (int s = 0; s < n_seq; ++s)
            if (sess[s]) slate_infer_session_free(sess[s]);
    if (batch) slate_infer_batch_free(batch);
    if (eng) slate_infer_engine_free(eng);
    if (lg) backend->release(lg);
    if (moved && orig) {
        for (int i = 0; i < ps.n_params; ++i) {
            if (orig[i]) ps.params[i]->data = orig[i];    /* the arena's own buffer again */
            if (moved[i]) backend->release(moved[i]);
        }
    }
    free(moved);
    free(orig);
    if (have_ps) slate_param_set_destroy(&ps);
    if (model) slate_module_destroy(model);   /* the module frees nothing the arena owns */
    if (arena) slate_arena_destroy(arena);
    free(sess);
    free(tok);
    return rc;
}
