/*
 * synth.c -- Q4_K quantiser and synthetic LLaMA GGUF writer (benchmark and
 * test workload generator; not on the decode path).
 *
 * Quantiser: the arithmetic of the reference's fixture generators
 * (tools/make_tiny_llama_q4k_gguf.py:39-87, tools/make_q4k_test.py:7-63) under
 * NumPy 2 promotion rules, so files written here are byte-identical to what
 * those scripts would write for the same f32 weights:
 *   per 32-weight sub-block j:  scale_j = f32(wmax - wmin) / 15  (f32),
 *                               min_j   = -wmin,
 *                               q = clip(round_half_even(f64(w - wmin) / scale_j), 0, 15)
 *   per 256-weight block:       d = max_j scale_j / 63, dmin = max_j min_j / 63 (f64)
 *                               sc_j = clip(rhe(scale_j / d), 0, 63), mn_j likewise
 *                               header = f16_rne(d), f16_rne(dmin), GGML 12-byte packing
 *   nibbles: qs[16j + i] = q[j][i] | q[j][i + 16] << 4   (Slate's order, quant.c:182-199)
 *
 * Weights: N(0, 0.02) from a counter-based generator -- element i of tensor t
 * is 0.02 * z, z the Box-Muller normal of pair i/2 drawn from splitmix64
 * hashes of (seed, t, i/2) -- so any thread count writes the same bytes.
 * Norm gains are 1.0 as in the reference fixtures
 * (make_tiny_llama_q4k_gguf.py:117,122,127).
 *
 * Self-contained (libc, libm, pthreads): besides libslate_cuda.so, the oracle's
 * Makefile compiles this file alone into a CPU-only library, so that a process
 * timing the reference on the host can write the same workload file without
 * mapping the CUDA library.
 */
#define _GNU_SOURCE
#include "slate_cuda.h"

#include <fcntl.h>
#include <fenv.h>
#include <math.h>
#include <pthread.h>
#include <stdio.h>
#include <stdlib.h>
#include <string.h>
#include <unistd.h>

/* ---- f64 -> binary16, round to nearest even (numpy.float16(double)) ---- */
static uint16_t f64_to_f16(double x) {
    uint16_t sign = signbit(x) ? 0x8000u : 0;
    double a = fabs(x);
    if (isnan(x)) return 0x7e00u;
    if (a >= 65520.0) return sign | 0x7c00u;             /* rounds to infinity */
    if (a < 6.103515625e-05) {                           /* below 2^-14: subnormal */
        double q = nearbyint(a * 16777216.0);            /* units of 2^-24 */
        return sign | (uint16_t)q;                       /* q == 1024 -> min normal */
    }
    int e;
    frexp(a, &e);                                        /* a in [2^(e-1), 2^e) */
    double q = nearbyint(ldexp(a, 11 - e));              /* 11-bit significand */
    if (q >= 2048.0) { q /= 2.0; ++e; }
    int E = e - 1 + 15;
    if (E >= 31) return sign | 0x7c00u;
    return sign | (uint16_t)(E << 10) | (uint16_t)((uint32_t)q & 0x3ffu);
}

/* ---- binary16 -> f64, exact (subnormals included) ---- */
static double f16_to_f64(uint16_t h) {
    const int e = (h >> 10) & 0x1f, m = h & 0x3ff;
    double v = e == 0 ? ldexp((double)m, -24)
             : e == 31 ? (m ? NAN : INFINITY)
                       : ldexp((double)(m | 0x400), e - 25);
    return (h & 0x8000u) ? -v : v;
}

static void quant_block(uint8_t* out, const float* w) {
    double sub_scales[8], sub_mins[8];
    uint8_t q[8][32];
    for (int j = 0; j < 8; ++j) {
        const float* wj = w + 32 * j;
        float wmin = wj[0], wmax = wj[0];
        for (int i = 1; i < 32; ++i) {
            if (wj[i] < wmin) wmin = wj[i];
            if (wj[i] > wmax) wmax = wj[i];
        }
        float range = wmax - wmin;
        if (range < (float)1e-9) {
            sub_scales[j] = 1e-9;
            sub_mins[j] = -(double)wmin;
            memset(q[j], 0, 32);
        } else {
            float sc = range / 15.0f;
            sub_scales[j] = (double)sc;
            sub_mins[j] = -(double)wmin;
            for (int i = 0; i < 32; ++i) {
                double v = nearbyint((double)(wj[i] - wmin) / sub_scales[j]);
                if (v < 0) v = 0;
                if (v > 15) v = 15;
                q[j][i] = (uint8_t)v;
            }
        }
    }
    double smax = sub_scales[0], mmax = sub_mins[0];
    for (int j = 1; j < 8; ++j) {
        if (sub_scales[j] > smax) smax = sub_scales[j];
        if (sub_mins[j] > mmax) mmax = sub_mins[j];
    }
    double d = smax > 0 ? smax / 63.0 : 1e-9;
    double dmin = mmax > 0 ? mmax / 63.0 : 1e-9;
    uint8_t qs_[8], qm_[8];
    for (int j = 0; j < 8; ++j) {
        double a = nearbyint(sub_scales[j] / d), b = nearbyint(sub_mins[j] / dmin);
        a = a < 0 ? 0 : (a > 63 ? 63 : a);
        b = b < 0 ? 0 : (b > 63 ? 63 : b);
        qs_[j] = (uint8_t)a;
        qm_[j] = (uint8_t)b;
    }
    uint16_t dh = f64_to_f16(d), mh = f64_to_f16(dmin);
    memcpy(out, &dh, 2);
    memcpy(out + 2, &mh, 2);
    uint8_t* s = out + 4;
    memset(s, 0, 12);
    for (int j = 0; j < 4; ++j) {
        s[j] = qs_[j] & 63;
        s[j + 4] = qm_[j] & 63;
    }
    for (int j = 4; j < 8; ++j) {
        s[j + 4] = (uint8_t)((qs_[j] & 15) | ((qm_[j] & 15) << 4));
        s[j - 4] |= (uint8_t)(((qs_[j] >> 4) & 3) << 6);
        s[j] |= (uint8_t)(((qm_[j] >> 4) & 3) << 6);
    }
    uint8_t* qs = out + 16;
    for (int j = 0; j < 8; ++j)
        for (int i = 0; i < 16; ++i) qs[16 * j + i] = (uint8_t)((q[j][i] & 15) | ((q[j][i + 16] & 15) << 4));
}

int slate_q4k_quantize_rows(void* dst, const float* src, int64_t rows, int K) {
    if (!dst || !src || rows < 0 || K <= 0 || K % 256) return -1;
    int saved = fegetround();
    fesetround(FE_TONEAREST);
    const int64_t nb = rows * (K / 256);
    for (int64_t b = 0; b < nb; ++b) quant_block((uint8_t*)dst + b * 144, src + b * 256);
    fesetround(saved);
    return 0;
}

/* ---- counter-based N(0, 0.02) ------------------------------------------ */
static uint64_t mix64(uint64_t z) {
    z += 0x9e3779b97f4a7c15ull;
    z = (z ^ (z >> 30)) * 0xbf58476d1ce4e5b9ull;
    z = (z ^ (z >> 27)) * 0x94d049bb133111ebull;
    return z ^ (z >> 31);
}
static void gen_normal(float* out, int64_t first, int64_t n, uint64_t seed, int tensor) {
    const uint64_t key = mix64(seed ^ ((uint64_t)(tensor + 1) * 0xd1b54a32d192ed03ull));
    for (int64_t k = 0; k < n; ++k) {
        const int64_t i = first + k;
        const uint64_t pair = (uint64_t)(i >> 1);
        const uint64_t h1 = mix64(key ^ (2 * pair)), h2 = mix64(key ^ (2 * pair + 1));
        const double u1 = ((double)(h1 >> 11) + 1.0) * (1.0 / 9007199254740992.0);
        const double u2 = (double)(h2 >> 11) * (1.0 / 9007199254740992.0);
        const double r = sqrt(-2.0 * log(u1)), th = 6.283185307179586 * u2;
        out[k] = (float)(0.02 * ((i & 1) ? r * sin(th) : r * cos(th)));
    }
}

/* ---- GGUF writer --------------------------------------------------------- */
typedef struct {
    char name[64];
    int64_t rows, cols;   /* logical [rows, cols]; cols == 1 for vectors */
    int n_dims, ggml_type, kind, id;   /* kind 0 = normal, 1 = ones, 2 = embedding */
    int src;              /* >= 0: a copy of tensor src (layer_period) */
    uint64_t off;
    size_t bytes;
} tdesc;

typedef struct { uint8_t* p; size_t n, cap; } buf_t;
static void put(buf_t* b, const void* s, size_t n) {
    if (b->n + n > b->cap) {
        b->cap = (b->n + n) * 2 + 4096;
        b->p = (uint8_t*)realloc(b->p, b->cap);
    }
    memcpy(b->p + b->n, s, n);
    b->n += n;
}
static void put_u32(buf_t* b, uint32_t v) { put(b, &v, 4); }
static void put_u64(buf_t* b, uint64_t v) { put(b, &v, 8); }
static void put_str(buf_t* b, const char* s) { put_u64(b, strlen(s)); put(b, s, strlen(s)); }
static void kv_u32(buf_t* b, const char* k, uint32_t v) { put_str(b, k); put_u32(b, 4); put_u32(b, v); }
static void kv_f32(buf_t* b, const char* k, float v) { put_str(b, k); put_u32(b, 6); put(b, &v, 4); }

typedef struct {
    int fd;
    const tdesc* t;
    int nt;
    uint64_t data_off, seed;
    int tid, nthreads, rc;
    int q4k_order, embd_f16;
} job_t;

/* Slate's nibble packing of one block -> llama.cpp / ggml's: byte 32g + e
 * holds element e of sub-block 2g (low nibble) and of 2g + 1 (high). */
static void to_ggml_order(uint8_t* blk) {
    uint8_t* qs = blk + 16;
    uint8_t e[8][32], out[128];
    for (int s = 0; s < 8; ++s)
        for (int i = 0; i < 16; ++i) {
            e[s][i] = qs[16 * s + i] & 15;
            e[s][i + 16] = qs[16 * s + i] >> 4;
        }
    for (int g = 0; g < 4; ++g)
        for (int i = 0; i < 32; ++i) out[32 * g + i] = (uint8_t)(e[2 * g][i] | (e[2 * g + 1][i] << 4));
    memcpy(qs, out, 128);
}

static void* writer(void* arg) {
    job_t* j = (job_t*)arg;
    int saved = fegetround();
    fesetround(FE_TONEAREST);
    for (int ti = 0; ti < j->nt && !j->rc; ++ti) {
        const tdesc* t = &j->t[ti];
        if (t->src >= 0) continue;
        int64_t per = (t->rows + j->nthreads - 1) / j->nthreads;
        int64_t r0 = (int64_t)j->tid * per, r1 = r0 + per;
        if (r1 > t->rows) r1 = t->rows;
        if (r0 >= r1) continue;
        const int64_t chunk = 64;
        float* f = (float*)malloc((size_t)chunk * t->cols * 4);
        uint8_t* qb = (uint8_t*)malloc((size_t)chunk * (t->cols / 256 + 1) * 144 +
                                       (size_t)chunk * t->cols * 2);
        for (int64_t r = r0; r < r1 && !j->rc; r += chunk) {
            int64_t nr = r1 - r < chunk ? r1 - r : chunk;
            const int64_t n = nr * t->cols;
            if (t->kind == 1) for (int64_t i = 0; i < n; ++i) f[i] = 1.0f;
            else gen_normal(f, r * t->cols, n, j->seed, t->id);
            const void* src = f;
            size_t bytes = (size_t)n * 4, row_bytes = (size_t)t->cols * 4;
            if (t->ggml_type == 12) {
                for (int64_t b = 0; b < n / 256; ++b) {
                    quant_block(qb + b * 144, f + b * 256);
                    if (j->q4k_order == 1) to_ggml_order(qb + b * 144);
                }
                src = qb;
                row_bytes = (size_t)(t->cols / 256) * 144;
                bytes = row_bytes * (size_t)nr;
            } else if (t->ggml_type == 1) {              /* f16 storage */
                uint16_t* h16 = (uint16_t*)qb;
                for (int64_t i = 0; i < n; ++i) h16[i] = f64_to_f16((double)f[i]);
                src = qb;
                row_bytes = (size_t)t->cols * 2;
                bytes = row_bytes * (size_t)nr;
            } else if (t->kind == 2 && j->embd_f16 == 2) {   /* f32 of f16-rounded values */
                for (int64_t i = 0; i < n; ++i) f[i] = (float)f16_to_f64(f64_to_f16((double)f[i]));
            }
            off_t at = (off_t)(j->data_off + t->off + (uint64_t)r * row_bytes);
            if (pwrite(j->fd, src, bytes, at) != (ssize_t)bytes) j->rc = -6;
        }
        free(f);
        free(qb);
    }
    fesetround(saved);
    return NULL;
}

/* Copies repeated-layer tensors from their source tensor, one tensor per
 * thread in turn. */
static void* copier(void* arg) {
    job_t* j = (job_t*)arg;
    const size_t chunk = (size_t)64 << 20;
    unsigned char* buf = (unsigned char*)malloc(chunk);
    if (!buf) { j->rc = -6; return NULL; }
    for (int ti = j->tid; ti < j->nt && !j->rc; ti += j->nthreads) {
        const tdesc* t = &j->t[ti];
        if (t->src < 0) continue;
        const tdesc* s = &j->t[t->src];
        for (size_t done = 0; done < t->bytes && !j->rc; done += chunk) {
            size_t n = t->bytes - done < chunk ? t->bytes - done : chunk;
            if (pread(j->fd, buf, n, (off_t)(j->data_off + s->off + done)) != (ssize_t)n ||
                pwrite(j->fd, buf, n, (off_t)(j->data_off + t->off + done)) != (ssize_t)n)
                j->rc = -6;
        }
    }
    free(buf);
    return NULL;
}

int slate_synth_llama_gguf(const char* path, const slate_synth_config_t* c) {
    if (!path || !c || c->n_layers < 1 || c->d_model < 1 || c->n_heads < 1 ||
        c->d_model % c->n_heads || c->vocab < 1 || c->ffn_hidden < 1)
        return -1;
    const int D = c->d_model, F = c->ffn_hidden, V = c->vocab;
    const int nkv = c->n_kv_heads > 0 ? c->n_kv_heads : c->n_heads;
    const int kvd = nkv * (D / c->n_heads);
    const int nt = 2 + (c->tied_output ? 0 : 1) + 9 * c->n_layers;
    tdesc* t = (tdesc*)calloc((size_t)nt, sizeof(tdesc));
    int k = 0;
#define ADD(nm, R, C, nd, q, kd)                                                               \
    do {                                                                                       \
        snprintf(t[k].name, sizeof t[k].name, "%s", nm);                                       \
        t[k].rows = (R); t[k].cols = (C); t[k].n_dims = (nd); t[k].kind = (kd); t[k].id = k;   \
        t[k].ggml_type = ((q) && c->q4k && (C) % 256 == 0) ? 12 : 0;                           \
        t[k].src = -1;                                                                         \
        ++k;                                                                                   \
    } while (0)
    ADD("token_embd.weight", V, D, 2, 0, 2);
    ADD("output_norm.weight", 1, D, 1, 0, 1);
    if (!c->tied_output) ADD("output.weight", V, D, 2, 0, 2);
    if (c->embd_f16 == 1) {
        t[0].ggml_type = 1;
        if (!c->tied_output) t[2].ggml_type = 1;
    }
    for (int l = 0; l < c->n_layers; ++l) {
        char nm[64];
#define L_ADD(suffix, R, C, nd, q, kd) \
        snprintf(nm, sizeof nm, "blk.%d." suffix, l); ADD(nm, R, C, nd, q, kd)
        L_ADD("attn_norm.weight", 1, D, 1, 0, 1);
        L_ADD("attn_q.weight", D, D, 2, 1, 0);
        L_ADD("attn_k.weight", kvd, D, 2, 1, 0);
        L_ADD("attn_v.weight", kvd, D, 2, 1, 0);
        L_ADD("attn_output.weight", D, D, 2, 1, 0);
        L_ADD("ffn_norm.weight", 1, D, 1, 0, 1);
        L_ADD("ffn_gate.weight", F, D, 2, 1, 0);
        L_ADD("ffn_up.weight", F, D, 2, 1, 0);
        L_ADD("ffn_down.weight", D, F, 2, 1, 0);
#undef L_ADD
        if (c->layer_period > 0 && l >= c->layer_period)
            for (int j = 0; j < 9; ++j) t[k - 9 + j].src = k - 9 + j - 9 * (l - l % c->layer_period);
    }
#undef ADD
    uint64_t cur = 0;
    for (int i = 0; i < nt; ++i) {
        cur = (cur + 31) / 32 * 32;
        t[i].off = cur;
        t[i].bytes = t[i].ggml_type == 12 ? (size_t)t[i].rows * (t[i].cols / 256) * 144
                     : (size_t)t[i].rows * t[i].cols * (t[i].ggml_type == 1 ? 2 : 4);
        cur += t[i].bytes;
    }
    buf_t h = {0};
    put(&h, "GGUF", 4);
    put_u32(&h, 3);
    put_u64(&h, (uint64_t)nt);
    put_u64(&h, 11);
    put_str(&h, "general.architecture"); put_u32(&h, 8); put_str(&h, "llama");
    kv_u32(&h, "general.alignment", 32);
    kv_u32(&h, "llama.block_count", (uint32_t)c->n_layers);
    kv_u32(&h, "llama.embedding_length", (uint32_t)D);
    kv_u32(&h, "llama.feed_forward_length", (uint32_t)F);
    kv_u32(&h, "llama.attention.head_count", (uint32_t)c->n_heads);
    kv_u32(&h, "llama.attention.head_count_kv", (uint32_t)nkv);
    kv_u32(&h, "llama.context_length", (uint32_t)c->max_seq);
    kv_u32(&h, "llama.vocab_size", (uint32_t)V);
    kv_f32(&h, "llama.rope.freq_base", c->theta_base);
    kv_f32(&h, "llama.attention.layer_norm_rms_epsilon", c->rms_eps);
    for (int i = 0; i < nt; ++i) {
        put_str(&h, t[i].name);
        put_u32(&h, (uint32_t)t[i].n_dims);
        if (t[i].n_dims == 1) {
            put_u64(&h, (uint64_t)t[i].cols);
        } else {
            put_u64(&h, (uint64_t)t[i].cols);   /* GGUF lists the innermost dim first */
            put_u64(&h, (uint64_t)t[i].rows);
        }
        put_u32(&h, (uint32_t)t[i].ggml_type);
        put_u64(&h, t[i].off);
    }
    while (h.n % 32) put(&h, "", 1);
    const uint64_t data_off = h.n;
    int fd = open(path, O_CREAT | O_TRUNC | O_RDWR, 0644);
    int rc = 0;
    if (fd < 0) rc = -6;
    if (!rc && (ftruncate(fd, (off_t)(data_off + cur)) != 0 ||
                pwrite(fd, h.p, h.n, 0) != (ssize_t)h.n))
        rc = -6;
    if (!rc) {
        int nth = c->n_threads > 0 ? c->n_threads : (int)sysconf(_SC_NPROCESSORS_ONLN);
        if (nth < 1) nth = 1;
        if (nth > 256) nth = 256;
        pthread_t th[256];
        job_t jobs[256];
        for (int i = 0; i < nth; ++i) {
            jobs[i] = (job_t){fd, t, nt, data_off, c->seed, i, nth, 0, c->q4k_order, c->embd_f16};
            pthread_create(&th[i], NULL, writer, &jobs[i]);
        }
        for (int i = 0; i < nth; ++i) {
            pthread_join(th[i], NULL);
            if (!rc) rc = jobs[i].rc;
        }
        if (!rc && c->layer_period > 0 && c->layer_period < c->n_layers) {
            for (int i = 0; i < nth; ++i) {
                jobs[i] = (job_t){fd, t, nt, data_off, c->seed, i, nth, 0, c->q4k_order, c->embd_f16};
                pthread_create(&th[i], NULL, copier, &jobs[i]);
            }
            for (int i = 0; i < nth; ++i) {
                pthread_join(th[i], NULL);
                if (!rc) rc = jobs[i].rc;
            }
        }
    }
    if (fd >= 0) close(fd);
    free(h.p);
    free(t);
    return rc;
}
