/*
 * slate_llama_cuda_shim.c -- the glue a slate build adds to run its LLaMA
 * models on libslate_cuda.so.  It is compiled inside the slate tree (it
 * includes slate's own headers) and linked with -lslate_cuda.
 *
 * slate_llama_batch_new() builds the engine from a model opened by slate's
 * loader (slate_gguf_open + slate_llama_open, src/loader/gguf.c:122-186 and
 * src/loader/llama.c:42-140): the description is filled through the public
 * accessors of include/slate/llama.h:93-107, so the GGUF mmap the model
 * borrows from is read once during the upload and is not needed afterwards.
 */
#include <stdlib.h>

#include "slate/llama.h"
#include "slate_cuda.h"

slate_llama_batch_t* slate_llama_batch_new(const slate_llama_t* m, const slate_cuda_opts_t* opts) {
    if (!m || !opts) return NULL;
    const slate_llama_config_t* c = slate_llama_config(m);
    slate_llama_layer_desc_t* layers =
        (slate_llama_layer_desc_t*)calloc((size_t)c->n_layers, sizeof(*layers));
    const slate_llama_layer_desc_t** ptrs =
        (const slate_llama_layer_desc_t**)calloc((size_t)c->n_layers, sizeof(*ptrs));
    if (!layers || !ptrs) {
        free(layers);
        free(ptrs);
        return NULL;
    }
    for (int i = 0; i < c->n_layers; ++i) {
        const slate_llama_layer_t* l = slate_llama_layer(m, i);
        slate_llama_layer_desc_t* d = &layers[i];
        d->attn_norm = l->attn_norm;
        d->attn_q = l->attn_q;
        d->attn_k = l->attn_k;
        d->attn_v = l->attn_v;
        d->attn_output = l->attn_output;
        d->ffn_norm = l->ffn_norm;
        d->ffn_gate = l->ffn_gate;
        d->ffn_up = l->ffn_up;
        d->ffn_down = l->ffn_down;
        d->attn_q_dtype = l->attn_q_dtype;
        d->attn_k_dtype = l->attn_k_dtype;
        d->attn_v_dtype = l->attn_v_dtype;
        d->attn_output_dtype = l->attn_output_dtype;
        d->ffn_gate_dtype = l->ffn_gate_dtype;
        d->ffn_up_dtype = l->ffn_up_dtype;
        d->ffn_down_dtype = l->ffn_down_dtype;
        ptrs[i] = d;
    }
    slate_llama_desc_t desc = {
        .n_layers = c->n_layers, .d_model = c->d_model, .ffn_hidden = c->ffn_hidden,
        .n_heads = c->n_heads, .n_kv_heads = c->n_kv_heads, .head_dim = c->head_dim,
        .max_seq = c->max_seq, .vocab = c->vocab, .theta_base = c->theta_base,
        .rms_eps = c->rms_eps, .tied_output = c->tied_output,
        .token_embd = slate_llama_token_embd(m), .token_embd_dtype = slate_llama_token_embd_dtype(m),
        .output_norm = slate_llama_output_norm(m),
        .output = slate_llama_output(m), .output_dtype = slate_llama_output_dtype(m),
        .layers = ptrs,
    };
    slate_llama_batch_t* b = slate_llama_batch_new_desc(&desc, opts);
    free(ptrs);
    free(layers);
    return b;
}
