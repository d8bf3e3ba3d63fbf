/*
 * gguf_load.c -- standalone LLaMA GGUF reader that fills a slate_llama_desc_t
 * (for callers that do not link the reference's loader).  It accepts what the
 * reference's src/loader/gguf.c:122-186 and src/loader/llama.c:42-140 accept:
 * GGUF v2/v3, general.alignment (default 32), the llama.* keys with the same
 * defaults (n_kv_heads = n_heads, context 2048, theta 10000, eps 1e-5), the
 * blk.N.* tensor names, and output.weight falling back to token_embd.weight.
 * Tensor data stay in the read-only mmap until slate_gguf_model_close().
 */
#define _GNU_SOURCE
#include "sb_internal.h"

#include <fcntl.h>
#include <stdio.h>
#include <stdlib.h>
#include <string.h>
#include <sys/mman.h>
#include <sys/stat.h>
#include <unistd.h>

typedef struct { char* name; int type; uint64_t off; } tinfo;
typedef struct { char* key; uint32_t type; uint64_t u; float f; } kvent;

struct slate_gguf_model {
    void* map;
    size_t size;
    int nt, nkv;
    tinfo* t;
    kvent* kv;
    const uint8_t* data;
    slate_llama_layer_desc_t* layers;
    const slate_llama_layer_desc_t** layer_ptrs;
};

typedef struct { const uint8_t *p, *e; } cur_t;
static int rd(cur_t* c, void* d, size_t n) {
    if ((size_t)(c->e - c->p) < n) return -1;
    memcpy(d, c->p, n);
    c->p += n;
    return 0;
}
static int rd_str(cur_t* c, char** out) {
    uint64_t n;
    if (rd(c, &n, 8) || n > (1u << 20) || (uint64_t)(c->e - c->p) < n) return -1;
    *out = (char*)malloc(n + 1);
    memcpy(*out, c->p, n);
    (*out)[n] = 0;
    c->p += n;
    return 0;
}
static int skip(cur_t* c, uint32_t t) {
    static const int sz[13] = {1, 1, 2, 2, 4, 4, 4, 1, 0, 0, 8, 8, 8};
    if (t == 8) { char* s; if (rd_str(c, &s)) return -1; free(s); return 0; }
    if (t == 9) {
        uint32_t et; uint64_t n;
        if (rd(c, &et, 4) || rd(c, &n, 8)) return -1;
        for (uint64_t i = 0; i < n; ++i) if (skip(c, et)) return -1;
        return 0;
    }
    if (t > 12 || !sz[t] || (c->e - c->p) < sz[t]) return -1;
    c->p += sz[t];
    return 0;
}

void slate_gguf_model_close(slate_gguf_model_t* g) {
    if (!g) return;
    for (int i = 0; i < g->nt; ++i) free(g->t[i].name);
    for (int i = 0; i < g->nkv; ++i) free(g->kv[i].key);
    free(g->t);
    free(g->kv);
    free(g->layers);
    free(g->layer_ptrs);
    if (g->map) munmap(g->map, g->size);
    free(g);
}

static const kvent* find(const slate_gguf_model_t* g, const char* k) {
    for (int i = 0; i < g->nkv; ++i) if (!strcmp(g->kv[i].key, k)) return &g->kv[i];
    return NULL;
}
static int get_u32(const slate_gguf_model_t* g, const char* k, int* out) {
    const kvent* e = find(g, k);
    if (!e || !(e->type == 4 || e->type == 5 || e->type == 10)) return -1;
    *out = (int)(uint32_t)e->u;
    return 0;
}
static void get_f32(const slate_gguf_model_t* g, const char* k, float* out) {
    const kvent* e = find(g, k);
    if (e && e->type == 6) *out = e->f;
}
static const void* tensor(const slate_gguf_model_t* g, const char* name, int* dtype) {
    for (int i = 0; i < g->nt; ++i)
        if (!strcmp(g->t[i].name, name)) {
            /* GGML type -> slate_dtype_t (gguf.c:102-111): F32 0, F16 1, Q8_0 16, Q4_0 17, Q4_K 18 */
            int ty = g->t[i].type;
            if (dtype) *dtype = ty == 0 ? 0 : ty == 1 ? 1 : ty == 8 ? 16 : ty == 2 ? 17 : ty == 12 ? 18 : 0;
            return g->data + g->t[i].off;
        }
    return NULL;
}

slate_gguf_model_t* slate_gguf_model_open(const char* path, slate_llama_desc_t* d) {
    if (!path || !d) return NULL;
    int fd = open(path, O_RDONLY);
    if (fd < 0) { sb_set_error("cannot open %s", path); return NULL; }
    struct stat st;
    if (fstat(fd, &st)) { close(fd); return NULL; }
    void* map = mmap(NULL, (size_t)st.st_size, PROT_READ, MAP_SHARED, fd, 0);
    close(fd);
    if (map == MAP_FAILED) { sb_set_error("mmap failed for %s", path); return NULL; }
    slate_gguf_model_t* g = (slate_gguf_model_t*)calloc(1, sizeof(*g));
    g->map = map;
    g->size = (size_t)st.st_size;
    cur_t c = {(const uint8_t*)map, (const uint8_t*)map + st.st_size};
    uint32_t magic, ver;
    uint64_t nt, nkv, align = 32;
    if (rd(&c, &magic, 4) || magic != 0x46554747u || rd(&c, &ver, 4) || ver < 2 || ver > 3 ||
        rd(&c, &nt, 8) || rd(&c, &nkv, 8) || nt > (1u << 24) || nkv > (1u << 24))
        goto bad;
    g->kv = (kvent*)calloc(nkv ? nkv : 1, sizeof(kvent));
    for (uint64_t i = 0; i < nkv; ++i, ++g->nkv) {
        kvent* e = &g->kv[i];
        if (rd_str(&c, &e->key) || rd(&c, &e->type, 4)) goto bad;
        if (e->type == 6) { if (rd(&c, &e->f, 4)) goto bad; }
        else if (e->type == 4 || e->type == 5) {
            uint32_t u; if (rd(&c, &u, 4)) goto bad; e->u = u;
            if (!strcmp(e->key, "general.alignment") && u) align = u;
        } else if (e->type == 10 || e->type == 11) { if (rd(&c, &e->u, 8)) goto bad; }
        else if (skip(&c, e->type)) goto bad;
    }
    g->t = (tinfo*)calloc(nt ? nt : 1, sizeof(tinfo));
    for (uint64_t i = 0; i < nt; ++i, ++g->nt) {
        uint32_t nd, ty;
        if (rd_str(&c, &g->t[i].name) || rd(&c, &nd, 4) || nd > 4) goto bad;
        for (uint32_t k = 0; k < nd; ++k) { uint64_t s; if (rd(&c, &s, 8)) goto bad; }
        if (rd(&c, &ty, 4) || rd(&c, &g->t[i].off, 8)) goto bad;
        g->t[i].type = (int)ty;
    }
    {
        size_t off = (size_t)(c.p - (const uint8_t*)map);
        off = (off + align - 1) / align * align;
        g->data = (const uint8_t*)map + off;
    }
    memset(d, 0, sizeof *d);
    d->theta_base = 10000.0f;
    d->rms_eps = 1e-5f;
    if (get_u32(g, "llama.block_count", &d->n_layers) || get_u32(g, "llama.embedding_length", &d->d_model) ||
        get_u32(g, "llama.feed_forward_length", &d->ffn_hidden) ||
        get_u32(g, "llama.attention.head_count", &d->n_heads) || d->n_heads <= 0) {
        sb_set_error("%s: missing llama.* metadata", path);
        goto bad;
    }
    if (get_u32(g, "llama.attention.head_count_kv", &d->n_kv_heads)) d->n_kv_heads = d->n_heads;
    if (get_u32(g, "llama.context_length", &d->max_seq)) d->max_seq = 2048;
    if (get_u32(g, "llama.vocab_size", &d->vocab)) d->vocab = 0;
    get_f32(g, "llama.rope.freq_base", &d->theta_base);
    get_f32(g, "llama.attention.layer_norm_rms_epsilon", &d->rms_eps);
    d->head_dim = d->d_model / d->n_heads;
    d->token_embd = tensor(g, "token_embd.weight", &d->token_embd_dtype);
    d->output_norm = tensor(g, "output_norm.weight", NULL);
    d->output = tensor(g, "output.weight", &d->output_dtype);
    if (!d->token_embd || !d->output_norm || d->vocab <= 0) {
        sb_set_error("%s: missing token_embd/output_norm or vocab", path);
        goto bad;
    }
    if (!d->output) {
        d->output = d->token_embd;
        d->output_dtype = d->token_embd_dtype;
        d->tied_output = 1;
    }
    g->layers = (slate_llama_layer_desc_t*)calloc((size_t)d->n_layers, sizeof(*g->layers));
    g->layer_ptrs = (const slate_llama_layer_desc_t**)calloc((size_t)d->n_layers, sizeof(void*));
    for (int l = 0; l < d->n_layers; ++l) {
        slate_llama_layer_desc_t* L = &g->layers[l];
        char nm[96];
#define T(field, suffix, dt)                                              \
        snprintf(nm, sizeof nm, "blk.%d." suffix, l);                      \
        L->field = tensor(g, nm, dt);                                      \
        if (!L->field) { sb_set_error("%s: missing %s", path, nm); goto bad; }
        T(attn_norm, "attn_norm.weight", NULL)
        T(attn_q, "attn_q.weight", &L->attn_q_dtype)
        T(attn_k, "attn_k.weight", &L->attn_k_dtype)
        T(attn_v, "attn_v.weight", &L->attn_v_dtype)
        T(attn_output, "attn_output.weight", &L->attn_output_dtype)
        T(ffn_norm, "ffn_norm.weight", NULL)
        T(ffn_gate, "ffn_gate.weight", &L->ffn_gate_dtype)
        T(ffn_up, "ffn_up.weight", &L->ffn_up_dtype)
        T(ffn_down, "ffn_down.weight", &L->ffn_down_dtype)
#undef T
        g->layer_ptrs[l] = L;
    }
    d->layers = g->layer_ptrs;
    return g;
bad:
    slate_gguf_model_close(g);
    return NULL;
}
