/*
 * slate_oracle.c -- CPU restatement of eating-and-drinking/slate's LLaMA
 * Q4_K decode path (TEST INFRASTRUCTURE: the checker, never the product).
 *
 * Scalar C11, written from the reference's documented behaviour; each
 * function cites the reference file:line it restates.  Accumulations that
 * the reference performs in AVX2 f32 lanes are done here in double (the
 * reference's own scalar fallback branches do the same, e.g.
 * util/quant.c:281-300), so this oracle is at least as accurate as the
 * reference; the tests' tolerances cover the difference.
 */
#define _GNU_SOURCE
#include "slate_oracle.h"

#include <fcntl.h>
#include <math.h>
#include <pthread.h>
#include <stdio.h>
#include <stdlib.h>
#include <string.h>
#include <sys/mman.h>
#include <sys/stat.h>
#include <unistd.h>

/* ------------------------------------------------------------------------ */
/* util/precision.c:10-29 -- IEEE binary16 -> binary32, subnormals expanded. */
float orc_f16_to_f32(uint16_t h) {
    uint32_t sign = ((uint32_t)h & 0x8000u) << 16;
    uint32_t e = (h >> 10) & 0x1fu, m = h & 0x3ffu, bits;
    if (e == 0) {
        if (m == 0) {
            bits = sign;
        } else {                       /* subnormal: renormalise */
            int shift = 0;
            while (!(m & 0x400u)) { m <<= 1; ++shift; }
            m &= 0x3ffu;
            bits = sign | ((uint32_t)(113 - shift) << 23) | (m << 13);
        }
    } else if (e == 31) {
        bits = sign | 0x7f800000u | (m << 13);
    } else {
        bits = sign | ((e + 112u) << 23) | (m << 13);
    }
    float f;
    memcpy(&f, &bits, 4);
    return f;
}

/* util/quant.c:157-166 -- GGML 12-byte packing of eight 6-bit (scale, min). */
static void q4k_scale_min(const uint8_t* s, int j, int* sc, int* mn) {
    if (j < 4) {
        *sc = s[j] & 63;
        *mn = s[j + 4] & 63;
    } else {
        *sc = (s[j + 4] & 15) | ((s[j - 4] >> 6) << 4);
        *mn = (s[j + 4] >> 4) | ((s[j] >> 6) << 4);
    }
}

static float rd_f16(const uint8_t* p) {
    uint16_t h;
    memcpy(&h, p, 2);
    return orc_f16_to_f32(h);
}

/* util/quant.c:168-202 -- Slate's nibble order: sub-block j's 32 weights live
 * in qs[16j .. 16j+15]; low nibbles are elements 0..15, high nibbles 16..31. */
void orc_dequant_q4k(float* dst, const void* src, int64_t n) {
    const uint8_t* p = (const uint8_t*)src;
    for (int64_t b = 0; b < n / 256; ++b) {
        const uint8_t* blk = p + b * 144;
        float d = rd_f16(blk), dmin = rd_f16(blk + 2);
        for (int j = 0; j < 8; ++j) {
            int sc, mn;
            q4k_scale_min(blk + 4, j, &sc, &mn);
            float sd = d * (float)sc, sm = dmin * (float)mn;
            const uint8_t* q = blk + 16 + 16 * j;
            float* o = dst + b * 256 + 32 * j;
            for (int i = 0; i < 16; ++i) {
                o[i] = sd * (float)(q[i] & 15) - sm;
                o[i + 16] = sd * (float)(q[i] >> 4) - sm;
            }
        }
    }
}

/* util/quant.c:210-304 -- sub-block factorisation
 *   Σ_blocks d·Σ_j sc_j·<q_j, y_j> − dmin·Σ_j mn_j·Σ y_j, block total in double. */
float orc_dot_q4k(const void* blocks, const float* y, int64_t n) {
    const uint8_t* p = (const uint8_t*)blocks;
    double total = 0.0;
    for (int64_t b = 0; b < n / 256; ++b) {
        const uint8_t* blk = p + b * 144;
        double d = rd_f16(blk), dmin = rd_f16(blk + 2);
        double dterm = 0.0, mterm = 0.0;
        for (int j = 0; j < 8; ++j) {
            int sc, mn;
            q4k_scale_min(blk + 4, j, &sc, &mn);
            const uint8_t* q = blk + 16 + 16 * j;
            const float* yj = y + b * 256 + 32 * j;
            double qy = 0.0, sy = 0.0;
            for (int i = 0; i < 16; ++i) {
                qy += (double)(q[i] & 15) * yj[i] + (double)(q[i] >> 4) * yj[i + 16];
                sy += (double)yj[i] + (double)yj[i + 16];
            }
            dterm += sc * qy;
            mterm += mn * sy;
        }
        total += d * dterm - dmin * mterm;
    }
    return (float)total;
}

/* util/quant.c:306-313 -- row-serial matvec over contiguous Q4_K rows. */
void orc_q4k_matvec(float* y, const void* A, const float* x, int M, int K) {
    size_t row_bytes = (size_t)(K / 256) * 144;
    for (int m = 0; m < M; ++m)
        y[m] = orc_dot_q4k((const uint8_t*)A + (size_t)m * row_bytes, x, K);
}

/* backend_cpu.c:33-36 -- y[M] = A[M,K]·x, A row-major [out, in]. */
void orc_matvec_f32(float* y, const float* A, const float* x, int M, int K) {
    for (int m = 0; m < M; ++m) {
        double s = 0.0;
        const float* a = A + (size_t)m * K;
        for (int k = 0; k < K; ++k) s += (double)a[k] * x[k];
        y[m] = (float)s;
    }
}

/* backend_cpu.c:38-42 -- C[B,N] = X[B,K]·W[K,N] (W is [in, out]). */
void orc_linear_batch(float* C, const float* X, const float* W, int B, int K, int N) {
    for (int b = 0; b < B; ++b)
        for (int n = 0; n < N; ++n) {
            double s = 0.0;
            for (int k = 0; k < K; ++k) s += (double)X[(size_t)b * K + k] * W[(size_t)k * N + n];
            C[(size_t)b * N + n] = (float)s;
        }
}

/* backend_cpu.c:48-76 -- Σx² accumulated wide, inverse RMS formed in f32. */
void orc_rmsnorm_row(float* y, const float* x, const float* w, int D, float eps) {
    double sq = 0.0;
    for (int d = 0; d < D; ++d) sq += (double)x[d] * x[d];
    float inv = 1.0f / sqrtf((float)(sq / (double)D) + eps);
    for (int d = 0; d < D; ++d) y[d] = x[d] * w[d] * inv;
}

/* backend_cpu.c:78-97 -- silu(g)·u = g/(1+e^{-g})·u. */
void orc_silu_mul(float* y, const float* g, const float* u, int H) {
    for (int i = 0; i < H; ++i) {
        float gi = g[i];
        y[i] = (gi / (1.0f + expf(-gi))) * u[i];
    }
}

/* loader/llama_infer.c:77-92 -- NeoX half-split rotation per head:
 * angle_i = (float)pos · θ^(−2i/hd) computed with powf/cosf/sinf in f32. */
void orc_rope_row(float* row, int n_heads, int hd, int pos, float theta) {
    int half = hd / 2;
    for (int h = 0; h < n_heads; ++h) {
        float* r = row + (size_t)h * hd;
        for (int i = 0; i < half; ++i) {
            float inv_freq = powf(theta, -2.0f * (float)i / (float)hd);
            float ang = (float)pos * inv_freq;
            float c = cosf(ang), s = sinf(ang);
            float a = r[i], b = r[i + half];
            r[i] = a * c - b * s;
            r[i + half] = a * s + b * c;
        }
    }
}

void orc_rope_tables(float* cos_t, float* sin_t, int max_seq, int hd, float theta) {
    int half = hd / 2;
    for (int p = 0; p < max_seq; ++p)
        for (int i = 0; i < half; ++i) {
            float inv_freq = powf(theta, -2.0f * (float)i / (float)hd);
            float ang = (float)p * inv_freq;
            cos_t[(size_t)p * half + i] = cosf(ang);
            sin_t[(size_t)p * half + i] = sinf(ang);
        }
}

/* loader/llama_infer.c:97-129 -- per q-head softmax(q·Kᵀ/√hd)·V over L rows;
 * q-head hq reads kv-head hq / (nq/nkv).  Max-subtracted expf, Σ in double. */
void orc_attention_gqa(float* out, const float* q, const float* K, const float* V,
                       float* scores, int L, int nq, int nkv, int hd) {
    int kvd = nkv * hd, group = nq / nkv;
    float scale = 1.0f / sqrtf((float)hd);
    for (int hq = 0; hq < nq; ++hq) {
        int hk = hq / group;
        const float* qh = q + (size_t)hq * hd;
        float m = -INFINITY;
        for (int t = 0; t < L; ++t) {
            const float* k = K + (size_t)t * kvd + (size_t)hk * hd;
            double s = 0.0;
            for (int d = 0; d < hd; ++d) s += (double)qh[d] * k[d];
            scores[t] = (float)s * scale;
            if (scores[t] > m) m = scores[t];
        }
        double S = 0.0;
        for (int t = 0; t < L; ++t) {
            scores[t] = expf(scores[t] - m);
            S += scores[t];
        }
        float invS = (float)(1.0 / S);
        for (int d = 0; d < hd; ++d) {
            double o = 0.0;
            for (int t = 0; t < L; ++t)
                o += (double)(scores[t] * invS) * V[(size_t)t * kvd + (size_t)hk * hd + d];
            out[(size_t)hq * hd + d] = (float)o;
        }
    }
}

/* backend_cpu.c:117-166 -- single-head attention_step vtable entry. */
void orc_attention_step(float* out, const float* q, const float* K, const float* V,
                        float* scores, int L, int D) {
    orc_attention_gqa(out, q, K, V, scores, L, 1, 1, D);
}

/* util/sampling.c:14-18 -- first index of the maximum (strict '>'). */
int orc_argmax(const float* p, int n) {
    int best = 0;
    float bv = p[0];
    for (int i = 1; i < n; ++i)
        if (p[i] > bv) { bv = p[i]; best = i; }
    return best;
}

/* ------------------------------------------------------------------------ */
/* GGUF v2/v3 reader -- loader/gguf.c:122-186 (header, KV table, tensor infos,
 * data section aligned to general.alignment, default 32). */
typedef struct { char* name; int64_t shape[4]; int n_dims, ggml_type; uint64_t off; } orc_tinfo;
typedef struct { char* key; uint32_t type; uint64_t u; float f; } orc_kv;

struct orc_model {
    void* map;
    size_t map_size;
    int n_t, n_kv;
    orc_tinfo* t;
    orc_kv* kv;
    const uint8_t* data;
    orc_config_t cfg;
    const void* tok_embd;
    const void* out_norm;
    const void* output;
    int output_dtype;
    struct orc_layer {
        const float *attn_norm, *ffn_norm;
        const void *w[7];  /* q, k, v, o, gate, up, down */
        int dt[7];
    } * layers;
};

typedef struct { const uint8_t *p, *end; } cur_t;
static int rd(cur_t* c, void* dst, size_t n) {
    if ((size_t)(c->end - c->p) < n) return -1;
    memcpy(dst, c->p, n);
    c->p += n;
    return 0;
}
static int rd_str(cur_t* c, char** out) {
    uint64_t n;
    if (rd(c, &n, 8) || (uint64_t)(c->end - c->p) < n) return -1;
    *out = (char*)malloc(n + 1);
    memcpy(*out, c->p, n);
    (*out)[n] = 0;
    c->p += n;
    return 0;
}
static size_t scalar_size(uint32_t t) {
    static const size_t sz[13] = {1, 1, 2, 2, 4, 4, 4, 1, 0, 0, 8, 8, 8};
    return t < 13 ? sz[t] : 0;
}
static int skip_val(cur_t* c, uint32_t t) {
    if (t == 8) { char* s; if (rd_str(c, &s)) return -1; free(s); return 0; }
    if (t == 9) {
        uint32_t et; uint64_t n;
        if (rd(c, &et, 4) || rd(c, &n, 8)) return -1;
        for (uint64_t i = 0; i < n; ++i) if (skip_val(c, et)) return -1;
        return 0;
    }
    size_t s = scalar_size(t);
    if (!s || (size_t)(c->end - c->p) < s) return -1;
    c->p += s;
    return 0;
}

static const orc_kv* find_kv(const orc_model_t* m, const char* k) {
    for (int i = 0; i < m->n_kv; ++i) if (!strcmp(m->kv[i].key, k)) return &m->kv[i];
    return NULL;
}
static int kv_u32(const orc_model_t* m, const char* k, int* out) {
    const orc_kv* v = find_kv(m, k);
    if (!v || !(v->type == 4 || v->type == 5 || v->type == 10)) return -1;
    *out = (int)(uint32_t)v->u;
    return 0;
}
static void kv_f32(const orc_model_t* m, const char* k, float* out) {
    const orc_kv* v = find_kv(m, k);
    if (v && v->type == 6) *out = v->f;
}

const void* orc_model_tensor(const orc_model_t* m, const char* name, int* dt) {
    for (int i = 0; i < m->n_t; ++i)
        if (!strcmp(m->t[i].name, name)) {
            if (dt) *dt = m->t[i].ggml_type == 12 ? 18 : (m->t[i].ggml_type == 0 ? 0 : -1);
            return m->data + m->t[i].off;
        }
    return NULL;
}

void orc_model_close(orc_model_t* m) {
    if (!m) return;
    for (int i = 0; i < m->n_t; ++i) free(m->t[i].name);
    for (int i = 0; i < m->n_kv; ++i) free(m->kv[i].key);
    free(m->t);
    free(m->kv);
    free(m->layers);
    if (m->map) munmap(m->map, m->map_size);
    free(m);
}

/* loader/llama.c:42-140 -- llama.* metadata with the reference's defaults
 * (n_kv_heads = n_heads, max_seq 2048, θ 10000, eps 1e-5) and blk.N.* names;
 * output.weight absent => tied to token_embd. */
orc_model_t* orc_model_open(const char* path) {
    int fd = open(path, O_RDONLY);
    if (fd < 0) return NULL;
    struct stat st;
    if (fstat(fd, &st)) { close(fd); return NULL; }
    void* map = mmap(NULL, (size_t)st.st_size, PROT_READ, MAP_SHARED, fd, 0);
    close(fd);
    if (map == MAP_FAILED) return NULL;
    orc_model_t* m = (orc_model_t*)calloc(1, sizeof(*m));
    m->map = map;
    m->map_size = (size_t)st.st_size;
    cur_t c = {(const uint8_t*)map, (const uint8_t*)map + st.st_size};
    uint32_t magic, ver;
    uint64_t nt, nkv, align = 32;
    if (rd(&c, &magic, 4) || magic != 0x46554747u || rd(&c, &ver, 4) || ver < 2 || ver > 3 ||
        rd(&c, &nt, 8) || rd(&c, &nkv, 8))
        goto bad;
    m->kv = (orc_kv*)calloc(nkv ? nkv : 1, sizeof(orc_kv));
    for (uint64_t i = 0; i < nkv; ++i, ++m->n_kv) {
        orc_kv* v = &m->kv[i];
        if (rd_str(&c, &v->key) || rd(&c, &v->type, 4)) goto bad;
        if (v->type == 6) {
            if (rd(&c, &v->f, 4)) goto bad;
        } else if (v->type == 4 || v->type == 5) {
            uint32_t u; if (rd(&c, &u, 4)) goto bad; v->u = u;
            if (!strcmp(v->key, "general.alignment")) align = u;
        } else if (v->type == 10 || v->type == 11) {
            if (rd(&c, &v->u, 8)) goto bad;
        } else if (skip_val(&c, v->type)) {
            goto bad;
        }
    }
    m->t = (orc_tinfo*)calloc(nt ? nt : 1, sizeof(orc_tinfo));
    for (uint64_t i = 0; i < nt; ++i, ++m->n_t) {
        orc_tinfo* t = &m->t[i];
        uint32_t nd, ty;
        if (rd_str(&c, &t->name) || rd(&c, &nd, 4) || nd > 4) goto bad;
        t->n_dims = (int)nd;
        for (uint32_t d = 0; d < nd; ++d) if (rd(&c, &t->shape[d], 8)) goto bad;
        if (rd(&c, &ty, 4) || rd(&c, &t->off, 8)) goto bad;
        t->ggml_type = (int)ty;
    }
    {
        size_t off = (size_t)(c.p - (const uint8_t*)map);
        off = (off + align - 1) / align * align;
        m->data = (const uint8_t*)map + off;
    }
    orc_config_t* g = &m->cfg;
    g->theta_base = 10000.0f;
    g->rms_eps = 1e-5f;
    if (kv_u32(m, "llama.block_count", &g->n_layers) || kv_u32(m, "llama.embedding_length", &g->d_model) ||
        kv_u32(m, "llama.feed_forward_length", &g->ffn_hidden) ||
        kv_u32(m, "llama.attention.head_count", &g->n_heads))
        goto bad;
    if (kv_u32(m, "llama.attention.head_count_kv", &g->n_kv_heads)) g->n_kv_heads = g->n_heads;
    if (kv_u32(m, "llama.context_length", &g->max_seq)) g->max_seq = 2048;
    if (kv_u32(m, "llama.vocab_size", &g->vocab)) g->vocab = 0;
    kv_f32(m, "llama.rope.freq_base", &g->theta_base);
    kv_f32(m, "llama.attention.layer_norm_rms_epsilon", &g->rms_eps);
    g->head_dim = g->d_model / g->n_heads;
    m->tok_embd = orc_model_tensor(m, "token_embd.weight", NULL);
    m->out_norm = orc_model_tensor(m, "output_norm.weight", NULL);
    if (!m->tok_embd || !m->out_norm) goto bad;
    m->output = orc_model_tensor(m, "output.weight", &m->output_dtype);
    if (!m->output) {
        m->output = m->tok_embd;
        m->output_dtype = 0;
        g->tied_output = 1;
    }
    if (g->vocab == 0) goto bad;
    m->layers = (struct orc_layer*)calloc((size_t)g->n_layers, sizeof(*m->layers));
    static const char* names[7] = {"attn_q", "attn_k", "attn_v", "attn_output",
                                   "ffn_gate", "ffn_up", "ffn_down"};
    for (int l = 0; l < g->n_layers; ++l) {
        char buf[96];
        snprintf(buf, sizeof buf, "blk.%d.attn_norm.weight", l);
        m->layers[l].attn_norm = (const float*)orc_model_tensor(m, buf, NULL);
        snprintf(buf, sizeof buf, "blk.%d.ffn_norm.weight", l);
        m->layers[l].ffn_norm = (const float*)orc_model_tensor(m, buf, NULL);
        if (!m->layers[l].attn_norm || !m->layers[l].ffn_norm) goto bad;
        for (int w = 0; w < 7; ++w) {
            snprintf(buf, sizeof buf, "blk.%d.%s.weight", l, names[w]);
            m->layers[l].w[w] = orc_model_tensor(m, buf, &m->layers[l].dt[w]);
            if (!m->layers[l].w[w]) goto bad;
        }
    }
    return m;
bad:
    orc_model_close(m);
    return NULL;
}

const orc_config_t* orc_model_config(const orc_model_t* m) { return m ? &m->cfg : NULL; }

/* ------------------------------------------------------------------------ */
/* loader/llama_infer.c:53-71, 212-256 -- dense per-session KV
 * [n_layers][max_seq][kv_dim] f32 plus single-token scratch. */
struct orc_session {
    const orc_model_t* m;
    int pos, max_seq;
    float *K, *V, *x, *xn, *q, *k, *v, *att, *g, *u, *tmp, *scores;
};

orc_session_t* orc_session_new(const orc_model_t* m, int max_seq_override) {
    const orc_config_t* c = &m->cfg;
    orc_session_t* s = (orc_session_t*)calloc(1, sizeof(*s));
    s->m = m;
    s->max_seq = max_seq_override > 0 ? max_seq_override : c->max_seq;
    size_t kvd = (size_t)c->n_kv_heads * c->head_dim;
    size_t cache = (size_t)c->n_layers * s->max_seq * kvd;
    s->K = (float*)calloc(cache, 4);
    s->V = (float*)calloc(cache, 4);
    s->x = (float*)calloc(c->d_model, 4);
    s->xn = (float*)calloc(c->d_model, 4);
    s->q = (float*)calloc(c->d_model, 4);
    s->k = (float*)calloc(kvd, 4);
    s->v = (float*)calloc(kvd, 4);
    s->att = (float*)calloc(c->d_model, 4);
    s->g = (float*)calloc(c->ffn_hidden, 4);
    s->u = (float*)calloc(c->ffn_hidden, 4);
    s->tmp = (float*)calloc(c->d_model, 4);
    s->scores = (float*)calloc(s->max_seq, 4);
    if (!s->K || !s->V || !s->x || !s->xn || !s->q || !s->k || !s->v || !s->att || !s->g ||
        !s->u || !s->tmp || !s->scores) {
        orc_session_free(s);
        return NULL;
    }
    return s;
}

void orc_session_free(orc_session_t* s) {
    if (!s) return;
    free(s->K); free(s->V); free(s->x); free(s->xn); free(s->q); free(s->k); free(s->v);
    free(s->att); free(s->g); free(s->u); free(s->tmp); free(s->scores);
    free(s);
}

int orc_session_position(const orc_session_t* s) { return s ? s->pos : -1; }

int orc_session_seed_kv(orc_session_t* s, int n, const float* K, const float* V) {
    const orc_config_t* c = &s->m->cfg;
    if (n < 0 || n > s->max_seq) return -2;
    size_t kvd = (size_t)c->n_kv_heads * c->head_dim;
    for (int l = 0; l < c->n_layers; ++l) {
        memcpy(s->K + (size_t)l * s->max_seq * kvd, K + (size_t)l * n * kvd, (size_t)n * kvd * 4);
        memcpy(s->V + (size_t)l * s->max_seq * kvd, V + (size_t)l * n * kvd, (size_t)n * kvd * 4);
    }
    s->pos = n;
    return 0;
}

/* llama_infer.c:43-51 -- Q4_K entry when dtype 18, f32 matvec otherwise. */
static void mv(float* y, const void* W, int dt, const float* x, int M, int K) {
    if (dt == 18) orc_q4k_matvec(y, W, x, M, K);
    else orc_matvec_f32(y, (const float*)W, x, M, K);
}

/* llama_infer.c:134-206 -- one decode step. */
int orc_decode_step(orc_session_t* s, int32_t token, float* logits) {
    const orc_model_t* m = s->m;
    const orc_config_t* c = &m->cfg;
    int D = c->d_model, H = c->ffn_hidden, hd = c->head_dim, p = s->pos;
    int kvd = c->n_kv_heads * hd;
    if (p >= s->max_seq) return -2;
    if (token < 0 || token >= c->vocab) return -3;
    memcpy(s->x, (const float*)m->tok_embd + (size_t)token * D, (size_t)D * 4);
    for (int l = 0; l < c->n_layers; ++l) {
        const struct orc_layer* L = &m->layers[l];
        orc_rmsnorm_row(s->xn, s->x, L->attn_norm, D, c->rms_eps);
        mv(s->q, L->w[0], L->dt[0], s->xn, D, D);
        mv(s->k, L->w[1], L->dt[1], s->xn, kvd, D);
        mv(s->v, L->w[2], L->dt[2], s->xn, kvd, D);
        orc_rope_row(s->q, c->n_heads, hd, p, c->theta_base);
        orc_rope_row(s->k, c->n_kv_heads, hd, p, c->theta_base);
        float* Kl = s->K + (size_t)l * s->max_seq * kvd;
        float* Vl = s->V + (size_t)l * s->max_seq * kvd;
        memcpy(Kl + (size_t)p * kvd, s->k, (size_t)kvd * 4);
        memcpy(Vl + (size_t)p * kvd, s->v, (size_t)kvd * 4);
        orc_attention_gqa(s->att, s->q, Kl, Vl, s->scores, p + 1, c->n_heads, c->n_kv_heads, hd);
        mv(s->tmp, L->w[3], L->dt[3], s->att, D, D);
        for (int i = 0; i < D; ++i) s->x[i] += s->tmp[i];
        orc_rmsnorm_row(s->xn, s->x, L->ffn_norm, D, c->rms_eps);
        mv(s->g, L->w[4], L->dt[4], s->xn, H, D);
        mv(s->u, L->w[5], L->dt[5], s->xn, H, D);
        orc_silu_mul(s->g, s->g, s->u, H);
        mv(s->tmp, L->w[6], L->dt[6], s->g, D, H);
        for (int i = 0; i < D; ++i) s->x[i] += s->tmp[i];
    }
    orc_rmsnorm_row(s->xn, s->x, (const float*)m->out_norm, D, c->rms_eps);
    mv(logits, m->output, m->output_dtype, s->xn, c->vocab, D);
    s->pos = p + 1;
    return 0;
}

/* ------------------------------------------------------------------------ */
typedef struct {
    const orc_model_t* m;
    int first, count, n_steps, rc;
    const int32_t* tokens;
    float* out;
    int32_t* out_tok;
} many_job;

static void* many_worker(void* arg) {
    many_job* j = (many_job*)arg;
    int V = j->m->cfg.vocab;
    float* lg = (float*)malloc((size_t)V * 4);
    for (int i = j->first; i < j->first + j->count && !j->rc; ++i) {
        orc_session_t* s = orc_session_new(j->m, j->n_steps);
        if (!s) { j->rc = -1; break; }
        for (int t = 0; t < j->n_steps; ++t) {
            int rc = orc_decode_step(s, j->tokens[(size_t)i * j->n_steps + t], lg);
            if (rc) { j->rc = rc; break; }
            if (j->out) memcpy(j->out + ((size_t)i * j->n_steps + t) * V, lg, (size_t)V * 4);
            if (j->out_tok) j->out_tok[(size_t)i * j->n_steps + t] = orc_argmax(lg, V);
        }
        orc_session_free(s);
    }
    free(lg);
    return NULL;
}

int orc_decode_many(const orc_model_t* m, int n, int n_steps, const int32_t* tokens,
                    float* out, int32_t* out_tok, int n_threads) {
    if (n_threads < 1) n_threads = 1;
    if (n_threads > n) n_threads = n;
    pthread_t th[256];
    many_job jobs[256];
    if (n_threads > 256) n_threads = 256;
    int per = (n + n_threads - 1) / n_threads, rc = 0;
    for (int i = 0; i < n_threads; ++i) {
        jobs[i] = (many_job){m, i * per, 0, n_steps, 0, tokens, out, out_tok};
        int cnt = n - i * per;
        jobs[i].count = cnt < 0 ? 0 : (cnt > per ? per : cnt);
        pthread_create(&th[i], NULL, many_worker, &jobs[i]);
    }
    for (int i = 0; i < n_threads; ++i) {
        pthread_join(th[i], NULL);
        if (!rc) rc = jobs[i].rc;
    }
    return rc;
}
