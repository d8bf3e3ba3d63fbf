// attention.cu -- paged-KV GQA decode attention plus the per-token row kernels
// of the LLaMA decode step (sm_100a).
//
// Paged KV pool (one allocation, layer-major):
//   pool[layer][page][kv (0 = K, 1 = V)][kv_head][16 tokens][head_dim]
// f32 (the reference's cache dtype, src/loader/llama_infer.c:225-226) or f16.
// A sequence slot owns pages through page_table[slot][pos / 16]; the same page
// index serves every layer.  Pages come from a device-side free stack.
//
// The attention kernels themselves live in attn_paged.cu.
#include "sb_internal.h"
#include "sb_kernels.h"
#include "sb_pdl.h"
#include <cuda_fp16.h>
#include <math.h>

namespace {

__device__ __forceinline__ void set_status(int32_t* status, int code) {
    atomicCAS(status, 0, code);
}

// ------------------------------------------------------------------------
// KV element access helpers: DPL consecutive values starting at p.
template <int DPL>
__device__ __forceinline__ void load_row(const float* p, float (&v)[DPL]) {
    if (DPL == 4) {
        float4 t = __ldg((const float4*)p);
        v[0] = t.x; v[1 % DPL] = t.y; v[2 % DPL] = t.z; v[3 % DPL] = t.w;
    } else if (DPL == 2) {
        float2 t = __ldg((const float2*)p);
        v[0] = t.x; v[1 % DPL] = t.y;
    } else {
        v[0] = __ldg(p);
    }
}
template <int DPL>
__device__ __forceinline__ void load_row(const __half* p, float (&v)[DPL]) {
    if (DPL == 4) {
        uint2 t = __ldg((const uint2*)p);
        float2 a = __half22float2(*(const __half2*)&t.x);
        float2 b = __half22float2(*(const __half2*)&t.y);
        v[0] = a.x; v[1 % DPL] = a.y; v[2 % DPL] = b.x; v[3 % DPL] = b.y;
    } else if (DPL == 2) {
        uint32_t t = __ldg((const unsigned int*)p);
        float2 a = __half22float2(*(const __half2*)&t);
        v[0] = a.x; v[1 % DPL] = a.y;
    } else {
        v[0] = __half2float(p[0]);
    }
}

__device__ __forceinline__ float to_f(float v) { return v; }
__device__ __forceinline__ float to_f(__half v) { return __half2float(v); }
__device__ __forceinline__ void from_f(float& d, float v) { d = v; }
__device__ __forceinline__ void from_f(__half& d, float v) { d = __float2half_rn(v); }

// ------------------------------------------------------------------------
// RoPE + paged append.  One CTA per row.
template <typename KT>
__global__ void rope_append_kernel(float* __restrict__ qkv, int ld, int nq, int nkv, int hd,
                                   const int32_t* __restrict__ row_pos,
                                   const int32_t* __restrict__ row_slot,
                                   const int32_t* __restrict__ page_table, int max_pages,
                                   KT* __restrict__ pool, int64_t n_pages, int layer,
                                   const float* __restrict__ rc, const float* __restrict__ rs) {
    const int b = blockIdx.x;
    const int pos = row_pos[b];
    if (pos < 0) return;
    const int slot = row_slot[b];
    const int half = hd / 2;
    float* q = qkv + (size_t)b * ld;
    float* k = q + (size_t)nq * hd;
    const float* v = k + (size_t)nkv * hd;
    const float* cs = rc + (size_t)pos * half;
    const float* sn = rs + (size_t)pos * half;
    const int page = page_table[(size_t)slot * max_pages + pos / SB_PAGE_TOKENS];
    if (page < 0 || page >= n_pages) return;          // never allocated: skip, never fault
    const int t = pos % SB_PAGE_TOKENS;
    const size_t head_stride = (size_t)SB_PAGE_TOKENS * hd;
    KT* kbase = pool + ((size_t)layer * n_pages + page) * (size_t)2 * nkv * head_stride;
    KT* vbase = kbase + (size_t)nkv * head_stride;
    for (int i = threadIdx.x; i < (nq + nkv) * half; i += blockDim.x) {
        const int h = i / half, j = i % half;
        const float c = cs[j], s = sn[j];
        if (h < nq) {
            float* r = q + (size_t)h * hd;
            const float a = r[j], bb = r[j + half];
            r[j] = a * c - bb * s;
            r[j + half] = a * s + bb * c;
        } else {
            const int hk = h - nq;
            const float* r = k + (size_t)hk * hd;
            const float a = r[j], bb = r[j + half];
            KT* dst = kbase + (size_t)hk * head_stride + (size_t)t * hd;
            from_f(dst[j], a * c - bb * s);
            from_f(dst[j + half], a * s + bb * c);
        }
    }
    for (int i = threadIdx.x; i < nkv * hd; i += blockDim.x) {
        const int hk = i / hd, d = i % hd;
        from_f(vbase[(size_t)hk * head_stride + (size_t)t * hd + d], v[i]);
    }
}

// The same with one CTA per (row, head): blockIdx.y < nq rotates query head
// y in place, nq <= y < nq + nkv rotates key head y - nq into the cache, the
// rest copy value heads into the cache; thread j handles the pair (j, j + hd/2)
// (or, for values, elements j and j + hd/2).  ~(nq + 2 nkv) x rows small CTAs
// instead of one CTA per row keep the memory system busy.
template <typename KT>
__global__ void rope_append_heads_kernel(float* __restrict__ qkv, int ld, int nq, int nkv, int hd,
                                         const int32_t* __restrict__ row_pos,
                                         const int32_t* __restrict__ row_slot,
                                         const int32_t* __restrict__ page_table, int max_pages,
                                         KT* __restrict__ pool, int64_t n_pages, int layer,
                                         const float* __restrict__ rc, const float* __restrict__ rs) {
    sb_grid_release();
    sb_grid_wait();      // qkv: after the previous kernel (programmatic launch, sb_pdl.h)
    const int b = blockIdx.x, h = blockIdx.y, j = threadIdx.x;
    const int pos = row_pos[b];
    if (pos < 0) return;
    const int half = hd / 2;
    float* r = qkv + (size_t)b * ld + (size_t)h * hd;    // q, k and v heads are contiguous
    if (h < nq) {
        const float c = rc[(size_t)pos * half + j], sn = rs[(size_t)pos * half + j];
        const float a = r[j], bb = r[j + half];
        r[j] = a * c - bb * sn;
        r[j + half] = a * sn + bb * c;
        return;
    }
    const int slot = row_slot[b];
    const int page = page_table[(size_t)slot * max_pages + pos / SB_PAGE_TOKENS];
    if (page < 0 || page >= n_pages) return;          // never allocated: skip, never fault
    const int t = pos % SB_PAGE_TOKENS;
    const size_t head_stride = (size_t)SB_PAGE_TOKENS * hd;
    KT* kbase = pool + ((size_t)layer * n_pages + page) * (size_t)2 * nkv * head_stride;
    if (h < nq + nkv) {
        const float c = rc[(size_t)pos * half + j], sn = rs[(size_t)pos * half + j];
        const float a = r[j], bb = r[j + half];
        KT* dst = kbase + (size_t)(h - nq) * head_stride + (size_t)t * hd;
        from_f(dst[j], a * c - bb * sn);
        from_f(dst[j + half], a * sn + bb * c);
    } else {
        KT* dst = kbase + (size_t)nkv * head_stride + (size_t)(h - nq - nkv) * head_stride +
                  (size_t)t * hd;
        from_f(dst[j], r[j]);
        from_f(dst[j + half], r[j + half]);
    }
}

// ------------------------------------------------------------------------
// Row kernels.
__global__ void rmsnorm_kernel(float* __restrict__ Y, int ldy, const float* __restrict__ X,
                               int ldx, const float* __restrict__ w, int D, float eps) {
    const float* x = X + (size_t)blockIdx.x * ldx;
    float* y = Y + (size_t)blockIdx.x * ldy;
    float s = 0.f;
    for (int i = threadIdx.x; i < D; i += blockDim.x) s = fmaf(x[i], x[i], s);
    __shared__ double red[32];
    double sd = s;
    for (int o = 16; o > 0; o >>= 1) sd += __shfl_xor_sync(0xffffffffu, sd, o);
    if ((threadIdx.x & 31) == 0) red[threadIdx.x >> 5] = sd;
    __syncthreads();
    if (threadIdx.x < 32) {
        double v = threadIdx.x < blockDim.x / 32 ? red[threadIdx.x] : 0.0;
        for (int o = 16; o > 0; o >>= 1) v += __shfl_xor_sync(0xffffffffu, v, o);
        if (threadIdx.x == 0) red[0] = v;
    }
    __syncthreads();
    const float inv = 1.0f / sqrtf((float)(red[0] / (double)D) + eps);
    for (int i = threadIdx.x; i < D; i += blockDim.x) y[i] = x[i] * w[i] * inv;
}

// The same normalisation with the row held in registers (float4, up to
// RN_MAX * 4 * RN_T elements) and, besides the f32 row, the row as the f16
// hi / lo pair (hi = f16(y), lo = f16(y - hi)) that the tensor-core GEMMs take
// as their operand (hi null: f32 row only; lo may be null).  Sum of squares: f32 per thread, double
// across the block, as above.
constexpr int RN_T = 256, RN_MAX = 8;
__global__ void __launch_bounds__(RN_T) rmsnorm_split_kernel(
    float* __restrict__ Y, int ldy, const float* __restrict__ X, int ldx,
    const float* __restrict__ w, int D, float eps, __half* __restrict__ hi, __half* __restrict__ lo,
    int ld16) {
    sb_grid_release();   // the GEMM that follows may start its set-up
    sb_grid_wait();      // x: after the previous kernel (programmatic launch, sb_pdl.h)
    const int n = blockIdx.x, q4 = D / 4;
    const float4* x4 = (const float4*)(X + (size_t)n * ldx);
    float4 v[RN_MAX];
    float s = 0.f;
#pragma unroll
    for (int j = 0; j < RN_MAX; ++j) {
        const int i = threadIdx.x + j * RN_T;
        v[j] = i < q4 ? x4[i] : make_float4(0.f, 0.f, 0.f, 0.f);
        s = fmaf(v[j].x, v[j].x, s);
        s = fmaf(v[j].y, v[j].y, s);
        s = fmaf(v[j].z, v[j].z, s);
        s = fmaf(v[j].w, v[j].w, s);
    }
    __shared__ double red[32];
    double sd = s;
    for (int o = 16; o > 0; o >>= 1) sd += __shfl_xor_sync(0xffffffffu, sd, o);
    if ((threadIdx.x & 31) == 0) red[threadIdx.x >> 5] = sd;
    __syncthreads();
    if (threadIdx.x < 32) {
        double t = threadIdx.x < RN_T / 32 ? red[threadIdx.x] : 0.0;
        for (int o = 16; o > 0; o >>= 1) t += __shfl_xor_sync(0xffffffffu, t, o);
        if (threadIdx.x == 0) red[0] = t;
    }
    __syncthreads();
    const float inv = 1.0f / sqrtf((float)(red[0] / (double)D) + eps);
    const float4* w4 = (const float4*)w;
    float4* y4 = (float4*)(Y + (size_t)n * ldy);
    uint2* h2 = hi ? (uint2*)(hi + (size_t)n * ld16) : nullptr;
    uint2* l2 = hi && lo ? (uint2*)(lo + (size_t)n * ld16) : nullptr;
#pragma unroll
    for (int j = 0; j < RN_MAX; ++j) {
        const int i = threadIdx.x + j * RN_T;
        if (i >= q4) break;
        const float4 g = __ldg(w4 + i);
        const float4 y = make_float4(v[j].x * g.x * inv, v[j].y * g.y * inv, v[j].z * g.z * inv,
                                     v[j].w * g.w * inv);
        y4[i] = y;
        if (!h2) continue;
        const __half2 a = __floats2half2_rn(y.x, y.y), b = __floats2half2_rn(y.z, y.w);
        h2[i] = make_uint2(*(const uint32_t*)&a, *(const uint32_t*)&b);
        if (l2) {
            const float2 ab = __half22float2(a), bb = __half22float2(b);
            const __half2 la = __floats2half2_rn(y.x - ab.x, y.y - ab.y);
            const __half2 lb = __floats2half2_rn(y.z - bb.x, y.w - bb.y);
            l2[i] = make_uint2(*(const uint32_t*)&la, *(const uint32_t*)&lb);
        }
    }
}

__global__ void silu_mul_kernel(float* y, const float* g, const float* u, int n) {
    int i = blockIdx.x * blockDim.x + threadIdx.x;
    if (i < n) {
        float gi = g[i];
        y[i] = gi / (1.0f + expf(-gi)) * u[i];
    }
}
__global__ void add_kernel(float* y, const float* x, int n) {
    int i = blockIdx.x * blockDim.x + threadIdx.x;
    if (i < n) y[i] += x[i];
}
__global__ void embed_kernel(float* y, const float* W, int token, int D) {
    int i = blockIdx.x * blockDim.x + threadIdx.x;
    if (i < D) y[i] = W[(size_t)token * D + i];
}

// First index of the maximum (util/sampling.c:14-18); ties -> lower index.
__device__ __forceinline__ void am_merge(float& bv, int& bi, float v, int i) {
    if (v > bv || (v == bv && i < bi)) { bv = v; bi = i; }
}
__device__ void block_argmax(const float* row, int V, float& out_v, int& out_i) {
    float bv = -INFINITY;
    int bi = 0x7fffffff;
    if (((uintptr_t)row & 15) == 0) {
        // 16-byte loads, four in flight per thread (the logits are read once:
        // streaming loads); am_merge keeps the lowest index of the maximum
        // whatever order the elements arrive in
        const int V4 = V / 4;
        const float4* r4 = (const float4*)row;
#pragma unroll 4
        for (int j = threadIdx.x; j < V4; j += blockDim.x) {
            const float4 x = __ldcs(r4 + j);
            am_merge(bv, bi, x.x, 4 * j);
            am_merge(bv, bi, x.y, 4 * j + 1);
            am_merge(bv, bi, x.z, 4 * j + 2);
            am_merge(bv, bi, x.w, 4 * j + 3);
        }
        for (int i = 4 * V4 + threadIdx.x; i < V; i += blockDim.x) am_merge(bv, bi, row[i], i);
    } else {
        for (int i = threadIdx.x; i < V; i += blockDim.x) am_merge(bv, bi, row[i], i);
    }
    for (int o = 16; o > 0; o >>= 1) {
        float v2 = __shfl_xor_sync(0xffffffffu, bv, o);
        int i2 = __shfl_xor_sync(0xffffffffu, bi, o);
        am_merge(bv, bi, v2, i2);
    }
    __shared__ float sv[32];
    __shared__ int si[32];
    if ((threadIdx.x & 31) == 0) { sv[threadIdx.x >> 5] = bv; si[threadIdx.x >> 5] = bi; }
    __syncthreads();
    if (threadIdx.x < 32) {
        bv = threadIdx.x < blockDim.x / 32 ? sv[threadIdx.x] : -INFINITY;
        bi = threadIdx.x < blockDim.x / 32 ? si[threadIdx.x] : 0x7fffffff;
        for (int o = 16; o > 0; o >>= 1) {
            float v2 = __shfl_xor_sync(0xffffffffu, bv, o);
            int i2 = __shfl_xor_sync(0xffffffffu, bi, o);
            am_merge(bv, bi, v2, i2);
        }
    }
    out_v = bv;
    out_i = bi == 0x7fffffff ? 0 : bi;  // all -inf/NaN: index 0, like the reference
}
__global__ void argmax_kernel(int32_t* out, const float* logits, int ld, int V) {
    float v;
    int i;
    block_argmax(logits + (size_t)blockIdx.x * ld, V, v, i);
    if (threadIdx.x == 0) out[blockIdx.x] = i;
}

// Single-head attention_step (backend_cpu.c:117-166), one CTA, scores in smem.
__global__ void attention_step_kernel(float* out, const float* q, const float* K, const float* V,
                                      int L, int D) {
    extern __shared__ float sc[];
    __shared__ float red[32];
    __shared__ double dred[32];
    const float scale = 1.0f / sqrtf((float)D);
    const int lane = threadIdx.x & 31, wid = threadIdx.x >> 5, nw = blockDim.x >> 5;
    for (int t = wid; t < L; t += nw) {
        float s = 0.f;
        for (int d = lane; d < D; d += 32) s = fmaf(q[d], K[(size_t)t * D + d], s);
        for (int o = 16; o > 0; o >>= 1) s += __shfl_xor_sync(0xffffffffu, s, o);
        if (lane == 0) sc[t] = s * scale;
    }
    __syncthreads();
    float m = -INFINITY;
    for (int t = threadIdx.x; t < L; t += blockDim.x) m = fmaxf(m, sc[t]);
    for (int o = 16; o > 0; o >>= 1) m = fmaxf(m, __shfl_xor_sync(0xffffffffu, m, o));
    if (lane == 0) red[wid] = m;
    __syncthreads();
    m = -INFINITY;
    for (int i = 0; i < nw; ++i) m = fmaxf(m, red[i]);
    double S = 0.0;
    for (int t = threadIdx.x; t < L; t += blockDim.x) {
        float e = expf(sc[t] - m);
        sc[t] = e;
        S += e;
    }
    for (int o = 16; o > 0; o >>= 1) S += __shfl_xor_sync(0xffffffffu, S, o);
    if (lane == 0) dred[wid] = S;
    __syncthreads();
    S = 0.0;
    for (int i = 0; i < nw; ++i) S += dred[i];
    const float invS = (float)(1.0 / S);
    for (int d = threadIdx.x; d < D; d += blockDim.x) {
        float acc = 0.f;
        for (int t = 0; t < L; ++t) acc = fmaf(sc[t] * invS, V[(size_t)t * D + d], acc);
        out[d] = acc;
    }
}

// ------------------------------------------------------------------------
// Step prologue / epilogue and slot management.
__device__ int alloc_page(int32_t* free_stack, int32_t* free_top) {
    int idx = atomicSub(free_top, 1) - 1;
    if (idx < 0) {
        atomicAdd(free_top, 1);
        return -1;
    }
    return free_stack[idx];
}

__global__ void prologue_kernel(const int32_t* __restrict__ slots, const int32_t* __restrict__ tokens,
                                int32_t* pos, int32_t* page_table, int max_pages,
                                int32_t* free_stack, int32_t* free_top, int max_slots, int max_seq,
                                int vocab, const float* __restrict__ emb, int D, float* x, int ldx,
                                int32_t* row_pos, int32_t* row_slot, int32_t* status, int dup_ok) {
    __shared__ int s_ok, s_tok;
    const int b = blockIdx.x;
    if (threadIdx.x == 0) {
        int ok = 1;
        const int slot = slots[b], tok = tokens[b];
        int p = -1;
        if (slot < 0 || slot >= max_slots) { set_status(status, -1); ok = 0; }
        if (ok && (tok < 0 || tok >= vocab)) { set_status(status, -3); ok = 0; }
        // a slot may occur several times in one step (a prompt chunk): its
        // k-th occurrence takes position pos[slot] + k
        int rank = 0;
        if (ok)
            for (int r = 0; r < b; ++r) rank += slots[r] == slot;
        if (ok && rank && !dup_ok) { set_status(status, -1); ok = 0; }
        if (ok) {
            p = pos[slot] + rank;
            if (p >= max_seq) { set_status(status, -2); ok = 0; }
        }
        if (ok) {
            // the row at a page's first position allocates it (so rows of one
            // chunk never race for a page); a first occurrence also repairs a
            // missing entry
            int32_t* e = page_table + (size_t)slot * max_pages + p / SB_PAGE_TOKENS;
            if (*e < 0 && (p % SB_PAGE_TOKENS == 0 || rank == 0)) {
                int pg = alloc_page(free_stack, free_top);
                if (pg < 0) { set_status(status, -2); ok = 0; }
                else *e = pg;
            }
        }
        row_pos[b] = ok ? p : -1;
        row_slot[b] = ok ? slot : 0;
        s_ok = ok;
        s_tok = tok;
    }
    __syncthreads();
    float* xr = x + (size_t)b * ldx;
    if (!s_ok) {
        for (int i = threadIdx.x; i < D; i += blockDim.x) xr[i] = 0.f;
        return;
    }
    const float* er = emb + (size_t)s_tok * D;
    for (int i = threadIdx.x; i < D; i += blockDim.x) xr[i] = er[i];
}

__global__ void epilogue_kernel(const float* logits, int ldl, int V, const int32_t* row_slot,
                                const int32_t* row_pos, int32_t* pos, const int32_t* status,
                                int32_t* out_tokens) {
    float v;
    int i;
    block_argmax(logits + (size_t)blockIdx.x * ldl, V, v, i);
    if (threadIdx.x == 0) {
        if (out_tokens) out_tokens[blockIdx.x] = i;
        if (*status == 0 && row_pos[blockIdx.x] >= 0)
            atomicMax(&pos[row_slot[blockIdx.x]], row_pos[blockIdx.x] + 1);
    }
}

// Position advance of a step without an LM head (a prompt chunk whose logits
// nobody reads): pos[slot] = max(pos[slot], row_pos + 1) for every row when the
// step was accepted, as the epilogue does beside the argmax.
__global__ void advance_kernel(const int32_t* row_slot, const int32_t* row_pos, int32_t* pos,
                               const int32_t* status, int B) {
    const int r = blockIdx.x * blockDim.x + threadIdx.x;
    if (r < B && *status == 0 && row_pos[r] >= 0) atomicMax(&pos[row_slot[r]], row_pos[r] + 1);
}

// Tensor parallelism: each rank holds a vocabulary slice [v0, v0 + V) of the LM
// head; it reduces its logits to one (max, global index) pair per row, the pairs
// of all ranks are gathered, and every rank picks the same winner: the larger
// value, ties to the lower global index -- the first maximum over the whole
// vocabulary, as sampling.c:14-18 takes it.
struct sb_vi { float v; int i; };
__global__ void argmax_pairs_kernel(const float* logits, int ldl, int V, int v0, sb_vi* pairs) {
    float v;
    int i;
    block_argmax(logits + (size_t)blockIdx.x * ldl, V, v, i);
    if (threadIdx.x == 0) pairs[blockIdx.x] = sb_vi{v, v0 + i};
}
__global__ void tp_epilogue_kernel(const sb_vi* all, int T, int B, const int32_t* row_slot,
                                   const int32_t* row_pos, int32_t* pos, const int32_t* status,
                                   int32_t* out_tokens) {
    const int r = blockIdx.x * blockDim.x + threadIdx.x;
    if (r >= B) return;
    float bv = -INFINITY;
    int bi = 0x7fffffff;
    for (int t = 0; t < T; ++t) am_merge(bv, bi, all[(size_t)t * B + r].v, all[(size_t)t * B + r].i);
    if (out_tokens) out_tokens[r] = bi == 0x7fffffff ? 0 : bi;
    if (*status == 0 && row_pos[r] >= 0) atomicMax(&pos[row_slot[r]], row_pos[r] + 1);
}

__device__ __forceinline__ uint64_t mix64(uint64_t z) {
    z += 0x9e3779b97f4a7c15ull;
    z = (z ^ (z >> 30)) * 0xbf58476d1ce4e5b9ull;
    z = (z ^ (z >> 27)) * 0x94d049bb133111ebull;
    return z ^ (z >> 31);
}

__global__ void seed_alloc_kernel(int slot, int n, int32_t* pos, int32_t* page_table, int max_pages,
                                  int32_t* free_stack, int32_t* free_top, int32_t* status) {
    if (threadIdx.x != 0 || blockIdx.x != 0) return;
    const int np = (n + SB_PAGE_TOKENS - 1) / SB_PAGE_TOKENS;
    for (int i = 0; i < np; ++i) {
        int32_t* e = page_table + (size_t)slot * max_pages + i;
        if (*e < 0) {
            int pg = alloc_page(free_stack, free_top);
            if (pg < 0) { set_status(status, -2); return; }
            *e = pg;
        }
    }
    pos[slot] = n;
}

template <typename KT>
__global__ void seed_fill_kernel(int slot, int n, uint64_t seed, int n_layers, int nkv, int hd,
                                 const int32_t* page_table, int max_pages, KT* pool,
                                 int64_t n_pages, const int32_t* status) {
    if (*status != 0) return;
    const size_t row = (size_t)nkv * hd;          // values per token per K or V
    const size_t total = (size_t)n_layers * 2 * n * row;
    const size_t head_stride = (size_t)SB_PAGE_TOKENS * hd;
    for (size_t i = (size_t)blockIdx.x * blockDim.x + threadIdx.x; i < total;
         i += (size_t)gridDim.x * blockDim.x) {
        size_t r = i;
        const int d = (int)(r % hd); r /= hd;
        const int h = (int)(r % nkv); r /= nkv;
        const int t = (int)(r % n); r /= n;
        const int kv = (int)(r % 2); r /= 2;
        const int layer = (int)r;
        const int page = page_table[(size_t)slot * max_pages + t / SB_PAGE_TOKENS];
        if (page < 0 || page >= n_pages) continue;
        uint64_t z = mix64(seed ^ (i * 0x9e3779b97f4a7c15ull));
        float val = (float)((double)(z >> 11) * (1.0 / 9007199254740992.0)) * 2.0f - 1.0f;
        KT* dst = pool + ((size_t)layer * n_pages + page) * 2 * nkv * head_stride +
                  (size_t)kv * nkv * head_stride + (size_t)h * head_stride +
                  (size_t)(t % SB_PAGE_TOKENS) * hd + d;
        from_f(*dst, val);
    }
}

template <typename KT>
__global__ void read_kv_kernel(int slot, int n, int n_layers, int nkv, int hd,
                               const int32_t* page_table, int max_pages, const KT* pool,
                               int64_t n_pages, float* K, float* V) {
    const size_t row = (size_t)nkv * hd;
    const size_t total = (size_t)n_layers * n * row;
    const size_t head_stride = (size_t)SB_PAGE_TOKENS * hd;
    for (size_t i = (size_t)blockIdx.x * blockDim.x + threadIdx.x; i < total;
         i += (size_t)gridDim.x * blockDim.x) {
        size_t r = i;
        const int d = (int)(r % hd); r /= hd;
        const int h = (int)(r % nkv); r /= nkv;
        const int t = (int)(r % n); r /= n;
        const int layer = (int)r;
        const int page = page_table[(size_t)slot * max_pages + t / SB_PAGE_TOKENS];
        if (page < 0 || page >= n_pages) { K[i] = V[i] = 0.f; continue; }
        const KT* src = pool + ((size_t)layer * n_pages + page) * 2 * nkv * head_stride +
                        (size_t)h * head_stride + (size_t)(t % SB_PAGE_TOKENS) * hd + d;
        K[i] = to_f(src[0]);
        V[i] = to_f(src[(size_t)nkv * head_stride]);
    }
}

__global__ void release_kernel(int slot, int32_t* pos, int32_t* page_table, int max_pages,
                               int32_t* free_stack, int32_t* free_top) {
    for (int i = threadIdx.x; i < max_pages; i += blockDim.x) {
        int32_t* e = page_table + (size_t)slot * max_pages + i;
        const int pg = *e;
        if (pg >= 0) {
            const int idx = atomicAdd(free_top, 1);
            free_stack[idx] = pg;
            *e = -1;
        }
    }
    if (threadIdx.x == 0) pos[slot] = 0;
}

__global__ void init_free_kernel(int32_t* free_stack, int32_t* free_top, int64_t n) {
    for (int64_t i = (int64_t)blockIdx.x * blockDim.x + threadIdx.x; i < n;
         i += (int64_t)gridDim.x * blockDim.x)
        free_stack[i] = (int32_t)i;
    if (blockIdx.x == 0 && threadIdx.x == 0) *free_top = (int32_t)n;
}

}  // namespace

extern "C" int sb_rope_append(float* qkv, int ld, int B, int nq, int nkv, int hd,
                              const int32_t* row_pos, const int32_t* row_slot,
                              const int32_t* page_table, int max_pages, void* pool,
                              int64_t n_pages, int layer, int kv_dtype, const float* rope_cos,
                              const float* rope_sin, cudaStream_t st) {
    if (B < 1 || hd % 2) return -1;
    if (hd <= 2048 && B <= 0x7fffffff && nq + 2 * nkv <= 65535) {
        const dim3 grid((unsigned)B, (unsigned)(nq + 2 * nkv));
        const cudaError_t e =
            kv_dtype == SLATE_KV_F16
                ? sb_launch_pdl(rope_append_heads_kernel<__half>, grid, dim3(hd / 2), 0, st, qkv, ld,
                                nq, nkv, hd, row_pos, row_slot, page_table, max_pages, (__half*)pool,
                                n_pages, layer, rope_cos, rope_sin)
                : sb_launch_pdl(rope_append_heads_kernel<float>, grid, dim3(hd / 2), 0, st, qkv, ld,
                                nq, nkv, hd, row_pos, row_slot, page_table, max_pages, (float*)pool,
                                n_pages, layer, rope_cos, rope_sin);
        return e == cudaSuccess ? 0 : -1;
    }
    if (kv_dtype == SLATE_KV_F16)
        rope_append_kernel<__half><<<B, 128, 0, st>>>(qkv, ld, nq, nkv, hd, row_pos, row_slot,
                                                      page_table, max_pages, (__half*)pool, n_pages,
                                                      layer, rope_cos, rope_sin);
    else
        rope_append_kernel<float><<<B, 128, 0, st>>>(qkv, ld, nq, nkv, hd, row_pos, row_slot,
                                                     page_table, max_pages, (float*)pool, n_pages,
                                                     layer, rope_cos, rope_sin);
    return 0;
}

extern "C" int sb_rmsnorm_rows(float* Y, int ldy, const float* X, int ldx, const float* w, int B,
                               int D, float eps, cudaStream_t st) {
    if (B < 1 || D < 1) return -1;
    rmsnorm_kernel<<<B, 256, 0, st>>>(Y, ldy, X, ldx, w, D, eps);
    return 0;
}

extern "C" int sb_rmsnorm_rows_split(float* Y, int ldy, const float* X, int ldx, const float* w,
                                     int B, int D, float eps, void* hi, void* lo, int ld16,
                                     cudaStream_t st) {
    if (B < 1 || D < 1) return -1;
    if (D % 4 || D > RN_MAX * 4 * RN_T || ldx % 4 || ldy % 4 || ld16 % 4 || ((uintptr_t)X & 15) ||
        ((uintptr_t)Y & 15) || ((uintptr_t)w & 15) || B > 0x7fffffff)
        return -1;
    return sb_cuda_check(sb_launch_pdl(rmsnorm_split_kernel, dim3((unsigned)B), dim3(RN_T), 0, st,
                                       Y, ldy, X, ldx, w, D, eps, (__half*)hi, (__half*)lo, ld16),
                         "rmsnorm launch");
}
extern "C" int sb_silu_mul(float* y, const float* g, const float* u, int n, cudaStream_t st) {
    if (n < 1) return -1;
    silu_mul_kernel<<<(n + 255) / 256, 256, 0, st>>>(y, g, u, n);
    return 0;
}
extern "C" int sb_add_inplace(float* y, const float* x, int n, cudaStream_t st) {
    if (n < 1) return -1;
    add_kernel<<<(n + 255) / 256, 256, 0, st>>>(y, x, n);
    return 0;
}
extern "C" int sb_embed_lookup(float* y, const float* W, int token, int D, cudaStream_t st) {
    if (D < 1) return -1;
    embed_kernel<<<(D + 255) / 256, 256, 0, st>>>(y, W, token, D);
    return 0;
}
extern "C" int sb_argmax_rows(int32_t* out, const float* logits, int ld, int B, int V,
                              cudaStream_t st) {
    if (B < 1 || V < 1) return -1;
    argmax_kernel<<<B, 256, 0, st>>>(out, logits, ld, V);
    return 0;
}
extern "C" int sb_attention_step(float* out, const float* q, const float* K, const float* V, int L,
                                 int D, cudaStream_t st) {
    if (L < 1 || D < 1 || (size_t)L * 4 > 200 * 1024) return -1;
    size_t sm = (size_t)L * sizeof(float);
    if (sm > 48 * 1024)
        cudaFuncSetAttribute(attention_step_kernel, cudaFuncAttributeMaxDynamicSharedMemorySize,
                             (int)sm);
    attention_step_kernel<<<1, 256, sm, st>>>(out, q, K, V, L, D);
    return 0;
}

extern "C" int sb_step_prologue(const int32_t* slots, const int32_t* tokens, int B, int32_t* pos,
                                int32_t* page_table, int max_pages, int32_t* free_stack,
                                int32_t* free_top, int max_slots, int max_seq, int vocab,
                                const float* emb, int D, float* x, int ldx, int32_t* row_pos,
                                int32_t* row_slot, int32_t* status, int dup_ok, cudaStream_t st) {
    if (B < 1) return -1;
    prologue_kernel<<<B, 256, 0, st>>>(slots, tokens, pos, page_table, max_pages, free_stack,
                                       free_top, max_slots, max_seq, vocab, emb, D, x, ldx,
                                       row_pos, row_slot, status, dup_ok);
    return 0;
}
extern "C" int sb_argmax_pairs(const float* logits, int ldl, int V, int B, int v0, void* pairs,
                               cudaStream_t st) {
    if (B < 1 || V < 1) return -1;
    argmax_pairs_kernel<<<B, 512, 0, st>>>(logits, ldl, V, v0, (sb_vi*)pairs);
    return 0;
}

extern "C" int sb_step_advance(const int32_t* row_slot, const int32_t* row_pos, int32_t* pos,
                               const int32_t* status, int B, cudaStream_t st) {
    if (B < 1) return -1;
    advance_kernel<<<(B + 127) / 128, 128, 0, st>>>(row_slot, row_pos, pos, status, B);
    return 0;
}

extern "C" int sb_tp_epilogue(const void* all_pairs, int T, int B, const int32_t* row_slot,
                              const int32_t* row_pos, int32_t* pos, const int32_t* status,
                              int32_t* out_tokens, cudaStream_t st) {
    if (B < 1 || T < 1) return -1;
    tp_epilogue_kernel<<<(B + 127) / 128, 128, 0, st>>>((const sb_vi*)all_pairs, T, B, row_slot,
                                                          row_pos, pos, status, out_tokens);
    return 0;
}

extern "C" int sb_step_epilogue(const float* logits, int ldl, int V, int B,
                                     const int32_t* row_slot, const int32_t* row_pos, int32_t* pos,
                                     const int32_t* status, int32_t* out_tokens, cudaStream_t st) {
    if (B < 1) return -1;
    epilogue_kernel<<<B, 512, 0, st>>>(logits, ldl, V, row_slot, row_pos, pos, status, out_tokens);
    return 0;
}

extern "C" int sb_seed_context(int slot, int n, uint64_t seed, int n_layers, int nkv, int hd,
                               int32_t* pos, int32_t* page_table, int max_pages,
                               int32_t* free_stack, int32_t* free_top, void* pool,
                               int64_t n_pages, int kv_dtype, int32_t* status, cudaStream_t st) {
    if (n < 0) return -1;
    seed_alloc_kernel<<<1, 32, 0, st>>>(slot, n, pos, page_table, max_pages, free_stack, free_top,
                                        status);
    if (n == 0) return 0;
    if (kv_dtype == SLATE_KV_F16)
        seed_fill_kernel<__half><<<1184, 256, 0, st>>>(slot, n, seed, n_layers, nkv, hd, page_table,
                                                       max_pages, (__half*)pool, n_pages, status);
    else
        seed_fill_kernel<float><<<1184, 256, 0, st>>>(slot, n, seed, n_layers, nkv, hd, page_table,
                                                      max_pages, (float*)pool, n_pages, status);
    return 0;
}
extern "C" int sb_read_kv(int slot, int n, int n_layers, int nkv, int hd, const int32_t* page_table,
                          int max_pages, const void* pool, int64_t n_pages, int kv_dtype, float* K,
                          float* V, cudaStream_t st) {
    if (n < 1) return -1;
    if (kv_dtype == SLATE_KV_F16)
        read_kv_kernel<__half><<<592, 256, 0, st>>>(slot, n, n_layers, nkv, hd, page_table, max_pages,
                                                    (const __half*)pool, n_pages, K, V);
    else
        read_kv_kernel<float><<<592, 256, 0, st>>>(slot, n, n_layers, nkv, hd, page_table, max_pages,
                                                   (const float*)pool, n_pages, K, V);
    return 0;
}
extern "C" int sb_release_slot(int slot, int32_t* pos, int32_t* page_table, int max_pages,
                               int32_t* free_stack, int32_t* free_top, cudaStream_t st) {
    release_kernel<<<1, 256, 0, st>>>(slot, pos, page_table, max_pages, free_stack, free_top);
    return 0;
}
extern "C" int sb_init_free_list(int32_t* free_stack, int32_t* free_top, int64_t n_pages,
                                 cudaStream_t st) {
    if (n_pages < 1 || n_pages > 0x7fffffff) return -1;
    init_free_kernel<<<592, 256, 0, st>>>(free_stack, free_top, n_pages);
    return 0;
}
