// sampling.cu -- stochastic token sampling on the device with the exact
// semantics of the reference sampler (src/util/sampling.c:9-83), so that the
// same logits and RNG state give the same token and the same next state:
//
//   T <= 0            argmax, first maximum (:14-18); the RNG is not advanced
//   otherwise         p_i = (float)(expf((l_i - max) * (1/T)) / sum_double)
//   0 < top_k < V     top_k_indices (:20-31): a slot array seeded with 0..k-1,
//                     each later index replaces the first minimal slot when
//                     strictly larger; probabilities renormalised in that slot
//                     order; with 0 < top_p < 1 a stable descending insertion
//                     sort, the shortest prefix whose double cumulative sum
//                     reaches top_p, renormalised
//   sample_from (:33-41)  r = frand01 (one LCG step, 53 high bits / 2^53,
//                     rounded to float), first i with r <= float cumulative sum
//
// Every order-dependent sum is taken sequentially in the reference's order and
// type (double for the normalisers, float for the cumulative draw), so the
// result does not depend on a parallel reduction order.  expf is evaluated as
// the double-precision exp rounded to float, which is the correctly rounded
// value glibc's expf also returns.  One CTA per row: the element-wise work is
// spread over the CTA, the sequential passes run on one thread over chunks
// staged in shared memory.
#include <cuda_runtime.h>
#include <math.h>
#include <stdint.h>

#include "sb_internal.h"
#include "sb_kernels.h"

namespace {

constexpr int NT = 256;
constexpr int CHUNK = 4096;                // floats staged per sequential pass step
constexpr int KMAX = SB_SAMPLE_TOPK_MAX;

__device__ __forceinline__ float frand01(uint64_t* s) {
    *s = *s * 6364136223846793005ULL + 1442695040888963407ULL;
    return (float)((double)((*s >> 11) & ((1ULL << 53) - 1)) / (double)(1ULL << 53));
}

__device__ void block_max(float v, float* red, float& out) {
    for (int o = 16; o > 0; o >>= 1) v = fmaxf(v, __shfl_xor_sync(0xffffffffu, v, o));
    if ((threadIdx.x & 31) == 0) red[threadIdx.x >> 5] = v;
    __syncthreads();
    if (threadIdx.x == 0) {
        float m = red[0];
        for (int w = 1; w < NT / 32; ++w) m = fmaxf(m, red[w]);
        red[NT / 32] = m;
    }
    __syncthreads();
    out = red[NT / 32];
    __syncthreads();
}

__global__ void __launch_bounds__(NT) sample_rows_kernel(
    const float* __restrict__ logits, int ldl, int V, const sb_sampler* __restrict__ cfg,
    uint64_t* __restrict__ rng, float* __restrict__ scratch, int32_t* __restrict__ out,
    const int32_t* __restrict__ row_slot, const int32_t* __restrict__ row_pos,
    int32_t* __restrict__ pos, const int32_t* __restrict__ status, int* __restrict__ err) {
    __shared__ float stage[CHUNK];
    __shared__ float red[NT / 32 + 1];
    __shared__ int s_idx[KMAX];
    __shared__ float s_tp[KMAX];
    __shared__ int s_tok;
    const int b = blockIdx.x, tid = threadIdx.x;
    const float* l = logits + (size_t)b * ldl;
    float* p = scratch + (size_t)b * V;
    const sb_sampler c = cfg[b];

    if (c.temperature <= 0.0f) {
        // first maximum (strict >), as sampling.c:14-18; a NaN logits[0] is
        // the reference's best forever after (no value compares greater)
        float bv = -INFINITY;
        int bi = 0x7fffffff;
        for (int i = tid; i < V; i += NT) {
            const float v = l[i];
            if (v > bv || (v == bv && i < bi)) { bv = v; bi = i; }
        }
        for (int o = 16; o > 0; o >>= 1) {
            const float v2 = __shfl_xor_sync(0xffffffffu, bv, o);
            const int i2 = __shfl_xor_sync(0xffffffffu, bi, o);
            if (v2 > bv || (v2 == bv && i2 < bi)) { bv = v2; bi = i2; }
        }
        __shared__ float wv[NT / 32];
        __shared__ int wi[NT / 32];
        if ((tid & 31) == 0) { wv[tid >> 5] = bv; wi[tid >> 5] = bi; }
        __syncthreads();
        if (tid == 0) {
            for (int w = 1; w < NT / 32; ++w)
                if (wv[w] > bv || (wv[w] == bv && wi[w] < bi)) { bv = wv[w]; bi = wi[w]; }
            s_tok = (bi == 0x7fffffff || isnan(l[0])) ? 0 : bi;
        }
    } else {
        // ---- probabilities ----
        float mx = -INFINITY;
        for (int i = tid; i < V; i += NT) mx = fmaxf(mx, l[i]);
        block_max(mx, red, mx);
        const float inv_t = 1.0f / c.temperature;
        for (int i = tid; i < V; i += NT) p[i] = (float)exp((double)((l[i] - mx) * inv_t));
        __syncthreads();
        __shared__ double s_sum;
        // sequential double sum in index order
        double sum = 0.0;
        for (int c0 = 0; c0 < V; c0 += CHUNK) {
            const int n = min(CHUNK, V - c0);
            for (int i = tid; i < n; i += NT) stage[i] = p[c0 + i];
            __syncthreads();
            if (tid == 0)
                for (int i = 0; i < n; ++i) sum += (double)stage[i];
            __syncthreads();
        }
        if (tid == 0) s_sum = sum;
        __syncthreads();
        sum = s_sum;
        for (int i = tid; i < V; i += NT) p[i] = (float)((double)p[i] / sum);
        __syncthreads();

        uint64_t st = rng[b];
        if (c.top_k > 0 && c.top_k < V) {
            const int k = c.top_k;
            if (k > KMAX) {
                if (tid == 0) { atomicCAS(err, 0, 1); s_tok = 0; }
            } else {
                // top_k_indices, sequentially over staged chunks; s_tp holds
                // each slot's probability during the scan
                for (int i = tid; i < k; i += NT) {
                    s_idx[i] = i;
                    s_tp[i] = p[i];
                }
                __syncthreads();
                int mp = 0;
                if (tid == 0)
                    for (int i = 1; i < k; ++i)
                        if (s_tp[i] < s_tp[mp]) mp = i;
                for (int c0 = k; c0 < V; c0 += CHUNK) {
                    const int n = min(CHUNK, V - c0);
                    for (int i = tid; i < n; i += NT) stage[i] = p[c0 + i];
                    __syncthreads();
                    if (tid == 0) {
                        for (int i = 0; i < n; ++i) {
                            if (stage[i] > s_tp[mp]) {
                                s_idx[mp] = c0 + i;
                                s_tp[mp] = stage[i];
                                mp = 0;
                                for (int j = 1; j < k; ++j)
                                    if (s_tp[j] < s_tp[mp]) mp = j;
                            }
                        }
                    }
                    __syncthreads();
                }
                if (tid == 0) {
                    double s = 0.0;
                    for (int i = 0; i < k; ++i) s += (double)s_tp[i];
                    for (int i = 0; i < k; ++i) s_tp[i] = (float)((double)s_tp[i] / s);
                    int keep = k;
                    if (c.top_p > 0.0f && c.top_p < 1.0f) {
                        for (int i = 1; i < k; ++i) {              // stable, descending
                            const float pp = s_tp[i];
                            const int ii = s_idx[i];
                            int j = i - 1;
                            while (j >= 0 && s_tp[j] < pp) {
                                s_tp[j + 1] = s_tp[j];
                                s_idx[j + 1] = s_idx[j];
                                --j;
                            }
                            s_tp[j + 1] = pp;
                            s_idx[j + 1] = ii;
                        }
                        double cum = 0.0;
                        keep = 0;
                        for (int i = 0; i < k; ++i) {
                            cum += (double)s_tp[i];
                            ++keep;
                            if (cum >= (double)c.top_p) break;
                        }
                        double ns = 0.0;
                        for (int i = 0; i < keep; ++i) ns += (double)s_tp[i];
                        for (int i = 0; i < keep; ++i) s_tp[i] = (float)((double)s_tp[i] / ns);
                    }
                    const float r = frand01(&st);
                    float cum = 0.0f;
                    int tok = s_idx[keep - 1];
                    for (int i = 0; i < keep; ++i) {
                        cum += s_tp[i];
                        if (r <= cum) { tok = s_idx[i]; break; }
                    }
                    s_tok = tok;
                }
            }
        } else {
            // sample_from over the whole vocabulary, float cumulative sum
            __shared__ float s_r;
            __shared__ int s_done;
            if (tid == 0) {
                s_r = frand01(&st);
                s_done = 0;
                s_tok = V - 1;
            }
            __syncthreads();
            float cum = 0.0f;
            for (int c0 = 0; c0 < V; c0 += CHUNK) {
                const int n = min(CHUNK, V - c0);
                for (int i = tid; i < n; i += NT) stage[i] = p[c0 + i];
                __syncthreads();
                if (tid == 0 && !s_done) {
                    for (int i = 0; i < n; ++i) {
                        cum += stage[i];
                        if (s_r <= cum) { s_tok = c0 + i; s_done = 1; break; }
                    }
                }
                __syncthreads();
                if (s_done) break;
            }
        }
        if (tid == 0) rng[b] = st;
    }
    __syncthreads();
    if (tid == 0) {
        out[b] = s_tok;
        if (pos && (!status || *status == 0) && row_pos[b] >= 0)
            atomicMax(&pos[row_slot[b]], row_pos[b] + 1);
    }
}

}  // namespace

extern "C" int sb_sample_rows(const float* logits, int ldl, int V, int B, const sb_sampler* cfg,
                              uint64_t* rng, float* scratch, int32_t* out, const int32_t* row_slot,
                              const int32_t* row_pos, int32_t* pos, const int32_t* status, int* err,
                              cudaStream_t st) {
    if (B < 1 || V < 1 || !logits || !cfg || !rng || !scratch || !out || !err) return -1;
    sample_rows_kernel<<<B, NT, 0, st>>>(logits, ldl, V, cfg, rng, scratch, out, row_slot, row_pos,
                                         pos, status, err);
    return 0;
}
