// attn_mma.cu -- paged GQA decode attention for an f16 KV cache with the dot
// products on the tensor cores (sm_100a warp-level MMA, f16 x f16 -> f32).
//
// Same work split and partial-record format as attn_chunk (attn_paged.cu):
// one CTA per (row, kv head, chunk of ct tokens), a producer warp and four
// consumer warps that take pages round-robin.  Differences:
//   * each page's K and V blocks ([16 tokens][head_dim] f16) arrive by tiled
//     TMA in 64-column boxes with the 128-byte swizzle, so ldmatrix reads them
//     without bank conflicts;
//   * per page a warp computes S = Q K^T and O += P V with mma.m16n8k16.  The
//     16 rows of the A operand hold the f16 high halves of the G (<= 8) query
//     heads' q (or p) in rows 0..7 and the low halves (x - f16(x)) in rows
//     8..15, so one MMA yields both partial products and a head's value is
//     the sum of accumulator rows g and g + 8, which sit in the same lane.
//     q and p are thereby carried to ~22 bits; the only rounding relative to
//     f32 math is the f16 storage of K and V itself;
//   * the online softmax works on the accumulator fragments: a head's 16
//     scores sit in the 4 lanes of one quad, so its max and sum take two
//     shuffles, and the rescale of O is local to the lanes that hold the row.
// Reference semantics: src/loader/llama_infer.c:97-129 (scores q.k scaled by
// 1/sqrt(hd) after the dot, max-subtracted expf, normalised sum).
#include <cuda.h>
#include <cuda_fp16.h>
#include <cudaTypedefs.h>
#include <math.h>
#include <string.h>

#include "sb_internal.h"
#include "sb_kernels.h"
#include "sb_pdl.h"

namespace {

constexpr int NW = 4;
constexpr int STAGES = 8;                 // a multiple of NW: stage s belongs to warp s % NW
constexpr uint64_t WAIT_NS = 2000000000ull;

__device__ __forceinline__ uint32_t su32(const void* p) {
    return (uint32_t)__cvta_generic_to_shared(p);
}
__device__ __forceinline__ uint64_t gtimer() {
    uint64_t t;
    asm volatile("mov.u64 %0, %%globaltimer;" : "=l"(t));
    return t;
}
__device__ __forceinline__ void bar_init(uint64_t* b, uint32_t c) {
    asm volatile("mbarrier.init.shared::cta.b64 [%0], %1;" ::"r"(su32(b)), "r"(c));
}
__device__ __forceinline__ void bar_arrive(uint64_t* b) {
    asm volatile("mbarrier.arrive.shared::cta.b64 _, [%0];" ::"r"(su32(b)) : "memory");
}
__device__ __forceinline__ void bar_expect(uint64_t* b, uint32_t bytes) {
    asm volatile("mbarrier.arrive.expect_tx.shared::cta.b64 _, [%0], %1;" ::"r"(su32(b)), "r"(bytes)
                 : "memory");
}
__device__ __forceinline__ bool bar_try(uint64_t* b, uint32_t parity) {
    uint32_t ok;
    asm volatile(
        "{\n\t.reg .pred p;\n\tmbarrier.try_wait.parity.shared::cta.b64 p, [%1], %2;\n\t"
        "selp.u32 %0, 1, 0, p;\n\t}\n"
        : "=r"(ok)
        : "r"(su32(b)), "r"(parity)
        : "memory");
    return ok != 0;
}
__device__ bool bar_wait(uint64_t* b, uint32_t parity, int* err, int code) {
    if (bar_try(b, parity)) return true;
    const uint64_t t0 = gtimer();
    while (!bar_try(b, parity)) {
        if (*(volatile int*)err) return false;
        if (gtimer() - t0 > WAIT_NS) {
            atomicCAS(err, 0, code);
            return false;
        }
    }
    return true;
}
__device__ __forceinline__ void tma_3d(void* dst, const CUtensorMap* map, uint64_t* bar, int x, int y,
                                       int z) {
    asm volatile(
        "cp.async.bulk.tensor.3d.shared::cluster.global.tile.mbarrier::complete_tx::bytes "
        "[%0], [%1, {%3, %4, %5}], [%2];" ::"r"(su32(dst)),
        "l"(map), "r"(su32(bar)), "r"(x), "r"(y), "r"(z)
        : "memory");
}
__device__ __forceinline__ void ldsm_x4(uint32_t addr, uint32_t& r0, uint32_t& r1, uint32_t& r2,
                                        uint32_t& r3) {
    asm volatile("ldmatrix.sync.aligned.m8n8.x4.shared.b16 {%0, %1, %2, %3}, [%4];"
                 : "=r"(r0), "=r"(r1), "=r"(r2), "=r"(r3)
                 : "r"(addr));
}
__device__ __forceinline__ void ldsm_x4_t(uint32_t addr, uint32_t& r0, uint32_t& r1, uint32_t& r2,
                                          uint32_t& r3) {
    asm volatile("ldmatrix.sync.aligned.m8n8.x4.trans.shared.b16 {%0, %1, %2, %3}, [%4];"
                 : "=r"(r0), "=r"(r1), "=r"(r2), "=r"(r3)
                 : "r"(addr));
}
// D += A(16x16) * B(16x8).  A register r holds two f16 of row g (r = 0, 2) or
// row g + 8 (r = 1, 3) at columns 2t, 2t+1 (r = 0, 1) or 2t+8, 2t+9 (r = 2, 3).
__device__ __forceinline__ void mma16816(float (&d)[4], uint32_t a0, uint32_t a1, uint32_t a2,
                                         uint32_t a3, uint32_t b0, uint32_t b1) {
    asm volatile(
        "mma.sync.aligned.m16n8k16.row.col.f32.f16.f16.f32 "
        "{%0, %1, %2, %3}, {%4, %5, %6, %7}, {%8, %9}, {%0, %1, %2, %3};"
        : "+f"(d[0]), "+f"(d[1]), "+f"(d[2]), "+f"(d[3])
        : "r"(a0), "r"(a1), "r"(a2), "r"(a3), "r"(b0), "r"(b1));
}
__device__ __forceinline__ void split2(float x0, float x1, uint32_t& hi, uint32_t& lo) {
    const __half2 h = __floats2half2_rn(x0, x1);
    const float2 back = __half22float2(h);
    const __half2 l = __floats2half2_rn(x0 - back.x, x1 - back.y);
    hi = *(const uint32_t*)&h;
    lo = *(const uint32_t*)&l;
}

// Byte offset of (token row r, dim d) in a [16 rows][HD] f16 block stored as
// HD/64 boxes of [16][64] with the 128-byte swizzle (16-byte chunk c of row r
// sits at chunk c ^ (r % 8)).
__device__ __forceinline__ uint32_t swz(int r, int d) {
    return (uint32_t)((d >> 6) * 2048 + r * 128 + ((((d & 63) >> 3) ^ (r & 7)) << 4));
}

template <int HD, int G>
__global__ void __launch_bounds__(32 * (NW + 1), 3) attn_chunk_mma(
    const __grid_constant__ CUtensorMap kvmap, const float* __restrict__ qkv, int ld_qkv, int B,
    int nq, int nkv, const int32_t* __restrict__ row_pos, const int32_t* __restrict__ row_slot,
    const int32_t* __restrict__ page_table, int max_pages, int64_t n_pages, int layer,
    int nchunk_max, int ct, float* __restrict__ part, int* err) {
    static_assert(HD % 64 == 0 && G <= 8, "head_dim multiple of 64, at most 8 heads per group");
    constexpr int BLK = 16 * HD * 2;          // one K or V block, bytes
    constexpr int KC = HD / 16;               // 16-wide k chunks of head_dim
    constexpr int NT = HD / 8;                // 8-wide output tiles
    extern __shared__ __align__(1024) unsigned char smem_raw[];
    unsigned char* ring = (unsigned char*)(((uintptr_t)smem_raw + 1023) & ~(uintptr_t)1023);
    __shared__ uint64_t full[STAGES], empty[STAGES];
    __shared__ int pages_s[SB_ATTN_CHUNK / 16];

    sb_grid_release();
    sb_grid_wait();      // q, positions, pages: after the previous kernel (sb_pdl.h)
    const int tid = threadIdx.x, warp = tid >> 5, lane = tid & 31;
    const int g = lane >> 2, t4 = lane & 3;
    // chunk-major order: every row's first chunk is scheduled first, and the
    // shorter (partial or empty) later chunks fill the last waves
    const int chunk = blockIdx.x / (B * nkv);
    const int rest = blockIdx.x % (B * nkv);
    const int kvh = rest % nkv, b = rest / nkv;
    if (b >= B) return;
    const int pos = row_pos[b];
    if (pos < 0) return;
    const int ctx = pos + 1, t0 = chunk * ct;
    if (t0 >= ctx) return;
    const int t1 = min(ctx, t0 + ct);
    const int npg = (t1 - t0 + 15) / 16;
    const int slot = row_slot[b];

    if (tid == 0) {
        for (int s = 0; s < STAGES; ++s) {
            bar_init(&full[s], 1);
            bar_init(&empty[s], 1);
        }
        asm volatile("fence.mbarrier_init.release.cluster;" ::: "memory");
    }
    if (warp == NW) {
        for (int i = lane; i < npg; i += 32) {
            int page = page_table[(size_t)slot * max_pages + t0 / 16 + i];
            if (page < 0 || page >= n_pages) {
                atomicCAS(err, 0, 6);
                page = 0;
            }
            pages_s[i] = page;
        }
    }
    __syncthreads();

    // consumer state: O accumulators (row g: the p-high part, row g + 8: the
    // p-low part of head g), running max / sum of head g
    float o[NT][4];
    float m_run = -INFINITY, l_run = 0.f;
    if (warp == NW) {
        if (lane == 0) {
            int issued = 0;
            for (int i = 0; i < npg; ++i) {
                const int s = i % STAGES;
                if (i >= STAGES && !bar_wait(&empty[s], ((i / STAGES) - 1) & 1, err, 4)) break;
                // row of (page, K, kv head, token 0) in the layer's [rows][HD] view of the pool
                const int row = (pages_s[i] * 2 * nkv + kvh) * 16;
                const int vrow = row + nkv * 16;
                unsigned char* st = ring + (size_t)s * 2 * BLK;
                bar_expect(&full[s], 2 * BLK);
#pragma unroll
                for (int h = 0; h < HD / 64; ++h) {
                    tma_3d(st + h * 2048, &kvmap, &full[s], 64 * h, row, layer);
                    tma_3d(st + BLK + h * 2048, &kvmap, &full[s], 64 * h, vrow, layer);
                }
                issued = i + 1;
            }
            for (int i = issued - STAGES > 0 ? issued - STAGES : 0; i < issued; ++i)
                bar_wait(&full[i % STAGES], (i / STAGES) & 1, err, 5);
        }
    } else {
        // q of head g (rows >= G are zero) as f16 hi/lo A fragments
        uint32_t qa_hi[KC][2], qa_lo[KC][2];
        {
            const float* qp = qkv + (size_t)b * ld_qkv + (size_t)(kvh * G + (g < G ? g : 0)) * HD;
#pragma unroll
            for (int c = 0; c < KC; ++c) {
                float x0 = 0.f, x1 = 0.f, x2 = 0.f, x3 = 0.f;
                if (g < G) {
                    x0 = qp[16 * c + 2 * t4];
                    x1 = qp[16 * c + 2 * t4 + 1];
                    x2 = qp[16 * c + 8 + 2 * t4];
                    x3 = qp[16 * c + 8 + 2 * t4 + 1];
                }
                split2(x0, x1, qa_hi[c][0], qa_lo[c][0]);
                split2(x2, x3, qa_hi[c][1], qa_lo[c][1]);
            }
        }
#pragma unroll
        for (int j = 0; j < NT; ++j) o[j][0] = o[j][1] = o[j][2] = o[j][3] = 0.f;
        const float scale = 1.0f / sqrtf((float)HD);
        // ldmatrix row addresses: lane l feeds row (l % 8) of matrix (l / 8)
        const int mi = lane >> 3, mr = lane & 7;
        for (int i = warp; i < npg; i += NW) {
            const int s = i % STAGES;
            if (!bar_wait(&full[s], (i / STAGES) & 1, err, 7)) break;
            unsigned char* kblk = ring + (size_t)s * 2 * BLK;
            unsigned char* vblk = kblk + BLK;
            const int nval = min(16, t1 - (t0 + 16 * i));
            if (nval < 16) {
                // rows past the context may hold stale bits: clear them in V (P is 0 there,
                // but 0 * NaN would not be), then order the writes before the next TMA fill
                for (int e = lane; e < (16 - nval) * (HD / 8); e += 32) {
                    const int r = nval + e / (HD / 8), c8 = e % (HD / 8);
                    *(uint4*)(vblk + swz(r, 8 * c8)) = make_uint4(0, 0, 0, 0);
                }
                __syncwarp();
            }
            // ---- S = Q K^T: two n-tiles of 8 tokens ----
            float sc[2][4] = {{0.f, 0.f, 0.f, 0.f}, {0.f, 0.f, 0.f, 0.f}};
            const uint32_t kbase = su32(kblk);
#pragma unroll
            for (int c = 0; c < KC; ++c) {
                // matrices: (tok 0-7, d 16c..+7), (tok 0-7, d +8..), (tok 8-15, d 16c..), (tok 8-15, d +8..)
                const int r = (mi >> 1) * 8 + mr, d = 16 * c + (mi & 1) * 8;
                uint32_t b00, b01, b10, b11;
                ldsm_x4(kbase + swz(r, d), b00, b01, b10, b11);
                mma16816(sc[0], qa_hi[c][0], qa_lo[c][0], qa_hi[c][1], qa_lo[c][1], b00, b01);
                mma16816(sc[1], qa_hi[c][0], qa_lo[c][0], qa_hi[c][1], qa_lo[c][1], b10, b11);
            }
            // ---- online softmax on row g: tokens 8j + 2*t4 + e ----
            float sv[4];
            float mx = -INFINITY;
#pragma unroll
            for (int j = 0; j < 2; ++j)
#pragma unroll
                for (int e = 0; e < 2; ++e) {
                    const int tok = 8 * j + 2 * t4 + e;
                    const float v = tok < nval ? (sc[j][e] + sc[j][2 + e]) * scale : -INFINITY;
                    sv[2 * j + e] = v;
                    mx = fmaxf(mx, v);
                }
            mx = fmaxf(mx, __shfl_xor_sync(0xffffffffu, mx, 1));
            mx = fmaxf(mx, __shfl_xor_sync(0xffffffffu, mx, 2));
            const float m_new = fmaxf(m_run, mx);
            const float corr = expf(m_run - m_new);
            float p[4], ps = 0.f;
#pragma unroll
            for (int k = 0; k < 4; ++k) {
                const int tok = 8 * (k >> 1) + 2 * t4 + (k & 1);
                p[k] = tok < nval ? expf(sv[k] - m_new) : 0.f;
                ps += p[k];
            }
            ps += __shfl_xor_sync(0xffffffffu, ps, 1);
            ps += __shfl_xor_sync(0xffffffffu, ps, 2);
            l_run = l_run * corr + ps;
            m_run = m_new;
#pragma unroll
            for (int j = 0; j < NT; ++j) {
                o[j][0] *= corr;
                o[j][1] *= corr;
                o[j][2] *= corr;
                o[j][3] *= corr;
            }
            // P (row g, k = tokens) as hi/lo A fragments: a0 = tokens 2t..2t+1, a2 = 8+2t..
            uint32_t pa_hi0, pa_lo0, pa_hi2, pa_lo2;
            split2(p[0], p[1], pa_hi0, pa_lo0);
            split2(p[2], p[3], pa_hi2, pa_lo2);
            // ---- O += P V: NT tiles of 8 dims; V^T fragments via ldmatrix.trans ----
            const uint32_t vbase = su32(vblk);
#pragma unroll
            for (int j = 0; j < NT; j += 2) {
                // matrices: (tok 0-7, d 8j..), (tok 8-15, d 8j..), (tok 0-7, d 8j+8..), (tok 8-15, d 8j+8..)
                const int r = (mi & 1) * 8 + mr, d = 8 * j + (mi >> 1) * 8;
                uint32_t v00, v01, v10, v11;
                ldsm_x4_t(vbase + swz(r, d), v00, v01, v10, v11);
                mma16816(o[j], pa_hi0, pa_lo0, pa_hi2, pa_lo2, v00, v01);
                mma16816(o[j + 1], pa_hi0, pa_lo0, pa_hi2, pa_lo2, v10, v11);
            }
            asm volatile("fence.proxy.async.shared::cta;" ::: "memory");
            __syncwarp();
            if (lane == 0) bar_arrive(&empty[s]);
        }
    }
    __syncthreads();                              // ring drained: reuse it for the merge
    float* merge = (float*)ring;                  // [NW][G][2 + HD]
    if (warp < NW && g < G) {
        float* rec = merge + ((size_t)warp * G + g) * (HD + 2);
        if (t4 == 0) {
            rec[0] = m_run;
            rec[1] = l_run;
        }
#pragma unroll
        for (int j = 0; j < NT; ++j) {
            rec[2 + 8 * j + 2 * t4] = o[j][0] + o[j][2];
            rec[2 + 8 * j + 2 * t4 + 1] = o[j][1] + o[j][3];
        }
    }
    __syncthreads();
    for (int e = tid; e < G * HD; e += blockDim.x) {
        const int h = e / HD, d = e % HD;
        float M = -INFINITY;
#pragma unroll
        for (int w = 0; w < NW; ++w) M = fmaxf(M, merge[((size_t)w * G + h) * (HD + 2)]);
        float L = 0.f, O = 0.f;
#pragma unroll
        for (int w = 0; w < NW; ++w) {
            const float* rec = merge + ((size_t)w * G + h) * (HD + 2);
            const float f = rec[0] == -INFINITY ? 0.f : expf(rec[0] - M);
            L += rec[1] * f;
            O += rec[2 + d] * f;
        }
        float* out = part + (((size_t)b * nq + kvh * G + h) * nchunk_max + chunk) * (HD + 2);
        if (d == 0) {
            out[0] = M;
            out[1] = L;
        }
        out[2 + d] = O;
    }
}

// ---- causal prefill attention ---------------------------------------------
// A prompt chunk is a step whose rows are consecutive positions of one
// sequence.  The decode kernel above would stream every row's whole prefix on
// its own; here one CTA takes a tile of QT consecutive rows for one kv head and
// one context chunk, streams each K/V page of the chunk once, and every
// consumer warp applies it to its 16 query vectors (16 / G rows x G heads):
//   S = Q K^T with q split into f16 hi and lo (two MMAs, one accumulator),
//   causal mask (token <= the row's position), online softmax per vector
//   (two vectors per lane: accumulator rows g and g + 8), O += P V with p
//   split likewise.  V rows past the chunk's last token are masked in the
//   ldmatrix registers (the ring stage is shared by all warps).  The partial
//   records (m, l, o) have the decode kernel's format and layout, so
//   attn_combine finishes them.
template <int HD, int G>
__global__ void __launch_bounds__(32 * (NW + 1), 2) attn_prefill_mma(
    const __grid_constant__ CUtensorMap kvmap, const float* __restrict__ qkv, int ld_qkv, int B,
    int nq, int nkv, const int32_t* __restrict__ row_pos, const int32_t* __restrict__ row_slot,
    const int32_t* __restrict__ page_table, int max_pages, int64_t n_pages, int layer,
    int nchunk_max, float* __restrict__ part, int* err) {
    static_assert(HD % 64 == 0 && 16 % G == 0, "head_dim multiple of 64, G divides 16");
    constexpr int BLK = 16 * HD * 2;
    constexpr int KC = HD / 16;
    constexpr int NT = HD / 8;
    constexpr int RW = 16 / G;                // rows per consumer warp
    constexpr int QT = NW * RW;               // rows per CTA
    sb_grid_release();
    sb_grid_wait();      // q, positions, pages: after the previous kernel (sb_pdl.h)
    extern __shared__ __align__(1024) unsigned char smem_raw[];
    unsigned char* ring = (unsigned char*)(((uintptr_t)smem_raw + 1023) & ~(uintptr_t)1023);
    __shared__ uint64_t full[STAGES], empty[STAGES];
    __shared__ int pages_s[SB_ATTN_CHUNK / 16];
    __shared__ int s_ctx, s_slot;

    const int tid = threadIdx.x, warp = tid >> 5, lane = tid & 31;
    const int g = lane >> 2, t4 = lane & 3;
    const int chunk = blockIdx.x % nchunk_max;
    const int rest = blockIdx.x / nchunk_max;
    const int kvh = rest % nkv, tile = rest / nkv;
    const int r0 = tile * QT;
    if (r0 >= B) return;
    if (tid == 0) {
        // the tile's rows share one sequence; the chunk is needed up to the
        // last row's position
        int ctx = 0, slot = -1;
        for (int r = r0; r < min(B, r0 + QT); ++r) {
            const int p = row_pos[r];
            if (p >= 0) {
                ctx = max(ctx, p + 1);
                if (slot < 0) slot = row_slot[r];
            }
        }
        s_ctx = ctx;
        s_slot = slot;
        for (int s = 0; s < STAGES; ++s) {
            bar_init(&full[s], 1);
            bar_init(&empty[s], NW);            // every consumer warp reads every stage
        }
        asm volatile("fence.mbarrier_init.release.cluster;" ::: "memory");
    }
    __syncthreads();
    const int ctx = s_ctx, slot = s_slot, t0 = chunk * SB_ATTN_CHUNK;
    if (slot < 0 || t0 >= ctx) return;
    const int t1 = min(ctx, t0 + SB_ATTN_CHUNK);
    const int npg = (t1 - t0 + 15) / 16;
    if (warp == NW) {
        for (int i = lane; i < npg; i += 32) {
            int page = page_table[(size_t)slot * max_pages + t0 / 16 + i];
            if (page < 0 || page >= n_pages) {
                atomicCAS(err, 0, 6);
                page = 0;
            }
            pages_s[i] = page;
        }
    }
    __syncthreads();

    if (warp == NW) {
        if (lane == 0) {
            int issued = 0;
            for (int i = 0; i < npg; ++i) {
                const int s = i % STAGES;
                if (i >= STAGES && !bar_wait(&empty[s], ((i / STAGES) - 1) & 1, err, 4)) break;
                const int row = (pages_s[i] * 2 * nkv + kvh) * 16;
                const int vrow = row + nkv * 16;
                unsigned char* st = ring + (size_t)s * 2 * BLK;
                bar_expect(&full[s], 2 * BLK);
#pragma unroll
                for (int h = 0; h < HD / 64; ++h) {
                    tma_3d(st + h * 2048, &kvmap, &full[s], 64 * h, row, layer);
                    tma_3d(st + BLK + h * 2048, &kvmap, &full[s], 64 * h, vrow, layer);
                }
                issued = i + 1;
            }
            for (int i = issued - STAGES > 0 ? issued - STAGES : 0; i < issued; ++i)
                bar_wait(&full[i % STAGES], (i / STAGES) & 1, err, 5);
        }
        return;
    }

    // ---- consumer warp: vectors v = 0..15 -> row rw0 + v / G, head v % G;
    // this lane holds vectors g (accumulator rows 0..7) and g + 8 ----
    const int rw0 = r0 + warp * RW;
    int vrow[2], vpos[2], vhead[2];
#pragma unroll
    for (int u = 0; u < 2; ++u) {
        const int v = g + 8 * u;
        vrow[u] = rw0 + v / G;
        vhead[u] = kvh * G + v % G;
        vpos[u] = vrow[u] < B ? row_pos[vrow[u]] : -1;
    }
    uint32_t qa_hi[KC][4], qa_lo[KC][4];
#pragma unroll
    for (int c = 0; c < KC; ++c) {
#pragma unroll
        for (int u = 0; u < 2; ++u) {
            float x[4] = {0.f, 0.f, 0.f, 0.f};
            if (vpos[u] >= 0) {
                const float* qp = qkv + (size_t)vrow[u] * ld_qkv + (size_t)vhead[u] * HD + 16 * c;
                x[0] = qp[2 * t4];
                x[1] = qp[2 * t4 + 1];
                x[2] = qp[8 + 2 * t4];
                x[3] = qp[8 + 2 * t4 + 1];
            }
            // A registers: 0 = (row g, k 2t..), 1 = (row g+8, k 2t..), 2 = (row g, k 2t+8..),
            // 3 = (row g+8, k 2t+8..)
            split2(x[0], x[1], qa_hi[c][u], qa_lo[c][u]);
            split2(x[2], x[3], qa_hi[c][2 + u], qa_lo[c][2 + u]);
        }
    }
    float o[NT][4];
#pragma unroll
    for (int j = 0; j < NT; ++j) o[j][0] = o[j][1] = o[j][2] = o[j][3] = 0.f;
    float m_run[2] = {-INFINITY, -INFINITY}, l_run[2] = {0.f, 0.f};
    const float scale = 1.0f / sqrtf((float)HD);
    const int mi = lane >> 3, mr = lane & 7;
    for (int i = 0; i < npg; ++i) {
        const int s = i % STAGES;
        if (!bar_wait(&full[s], (i / STAGES) & 1, err, 7)) break;
        const unsigned char* kblk = ring + (size_t)s * 2 * BLK;
        const unsigned char* vblk = kblk + BLK;
        const int pt0 = t0 + 16 * i;                     // first token of the page
        const int nval = min(16, t1 - pt0);              // tokens of the page in the chunk
        // ---- S = Q K^T: two n-tiles of 8 tokens ----
        float sc[2][4] = {{0.f, 0.f, 0.f, 0.f}, {0.f, 0.f, 0.f, 0.f}};
        const uint32_t kbase = su32(kblk);
#pragma unroll
        for (int c = 0; c < KC; ++c) {
            const int r = (mi >> 1) * 8 + mr, d = 16 * c + (mi & 1) * 8;
            uint32_t b00, b01, b10, b11;
            ldsm_x4(kbase + swz(r, d), b00, b01, b10, b11);
            mma16816(sc[0], qa_hi[c][0], qa_hi[c][1], qa_hi[c][2], qa_hi[c][3], b00, b01);
            mma16816(sc[0], qa_lo[c][0], qa_lo[c][1], qa_lo[c][2], qa_lo[c][3], b00, b01);
            mma16816(sc[1], qa_hi[c][0], qa_hi[c][1], qa_hi[c][2], qa_hi[c][3], b10, b11);
            mma16816(sc[1], qa_lo[c][0], qa_lo[c][1], qa_lo[c][2], qa_lo[c][3], b10, b11);
        }
        // ---- causal mask, online softmax for vectors g (u = 0) and g + 8 (u = 1) ----
        float p[2][4];
#pragma unroll
        for (int u = 0; u < 2; ++u) {
            float sv[4], mx = -INFINITY;
#pragma unroll
            for (int k = 0; k < 4; ++k) {
                const int j = k >> 1, e = k & 1;
                const int tok = 8 * j + 2 * t4 + e;
                const bool ok = tok < nval && pt0 + tok <= vpos[u];
                sv[k] = ok ? sc[j][2 * u + e] * scale : -INFINITY;
                mx = fmaxf(mx, sv[k]);
            }
            mx = fmaxf(mx, __shfl_xor_sync(0xffffffffu, mx, 1));
            mx = fmaxf(mx, __shfl_xor_sync(0xffffffffu, mx, 2));
            const float m_new = fmaxf(m_run[u], mx);
            // a vector with nothing to attend to yet keeps m = -inf, l = 0, o = 0
            const float corr = m_new == -INFINITY ? 1.f : expf(m_run[u] - m_new);
            float ps = 0.f;
#pragma unroll
            for (int k = 0; k < 4; ++k) {
                p[u][k] = sv[k] == -INFINITY ? 0.f : expf(sv[k] - m_new);
                ps += p[u][k];
            }
            ps += __shfl_xor_sync(0xffffffffu, ps, 1);
            ps += __shfl_xor_sync(0xffffffffu, ps, 2);
            l_run[u] = l_run[u] * corr + ps;
            m_run[u] = m_new;
#pragma unroll
            for (int j = 0; j < NT; ++j) {
                o[j][2 * u] *= corr;
                o[j][2 * u + 1] *= corr;
            }
        }
        // P as A fragments (hi / lo): 0 = (g, tok 2t..), 1 = (g+8, tok 2t..),
        // 2 = (g, tok 8+2t..), 3 = (g+8, tok 8+2t..)
        uint32_t pa_hi[4], pa_lo[4];
        split2(p[0][0], p[0][1], pa_hi[0], pa_lo[0]);
        split2(p[1][0], p[1][1], pa_hi[1], pa_lo[1]);
        split2(p[0][2], p[0][3], pa_hi[2], pa_lo[2]);
        split2(p[1][2], p[1][3], pa_hi[3], pa_lo[3]);
        // V rows past nval may hold stale bits (0 * NaN is NaN): mask them in
        // the fragments; this lane's B registers hold tokens 2t, 2t+1 (b0)
        // and 8 + 2t, 9 + 2t (b1)
        const uint32_t m0 = (2 * t4 < nval ? 0xFFFFu : 0u) | (2 * t4 + 1 < nval ? 0xFFFF0000u : 0u);
        const uint32_t m1 = (8 + 2 * t4 < nval ? 0xFFFFu : 0u) | (9 + 2 * t4 < nval ? 0xFFFF0000u : 0u);
        const uint32_t vbase = su32(vblk);
#pragma unroll
        for (int j = 0; j < NT; j += 2) {
            const int r = (mi & 1) * 8 + mr, d = 8 * j + (mi >> 1) * 8;
            uint32_t v00, v01, v10, v11;
            ldsm_x4_t(vbase + swz(r, d), v00, v01, v10, v11);
            v00 &= m0;
            v01 &= m1;
            v10 &= m0;
            v11 &= m1;
            mma16816(o[j], pa_hi[0], pa_hi[1], pa_hi[2], pa_hi[3], v00, v01);
            mma16816(o[j], pa_lo[0], pa_lo[1], pa_lo[2], pa_lo[3], v00, v01);
            mma16816(o[j + 1], pa_hi[0], pa_hi[1], pa_hi[2], pa_hi[3], v10, v11);
            mma16816(o[j + 1], pa_lo[0], pa_lo[1], pa_lo[2], pa_lo[3], v10, v11);
        }
        __syncwarp();
        if (lane == 0) bar_arrive(&empty[s]);
    }
    // ---- partial records of this chunk for the vectors that attend to it ----
#pragma unroll
    for (int u = 0; u < 2; ++u) {
        if (vpos[u] < t0) continue;                 // row invalid or before this chunk
        float* out = part + (((size_t)vrow[u] * nq + vhead[u]) * nchunk_max + chunk) * (HD + 2);
        if (t4 == 0) {
            out[0] = m_run[u];
            out[1] = l_run[u];
        }
#pragma unroll
        for (int j = 0; j < NT; ++j) {
            out[2 + 8 * j + 2 * t4] = o[j][2 * u];
            out[2 + 8 * j + 2 * t4 + 1] = o[j][2 * u + 1];
        }
    }
}

template <int HD, int G>
size_t smem_bytes() {
    const size_t ring = (size_t)STAGES * 2 * 16 * HD * 2;
    const size_t merge = (size_t)NW * G * (HD + 2) * 4;
    return (ring > merge ? ring : merge) + 1024;
}

template <int HD, int G>
int launch(int prepare, const void* map, const float* qkv, int ld_qkv, int B, int nq, int nkv,
           const int32_t* row_pos, const int32_t* row_slot, const int32_t* page_table,
           int max_pages, int64_t n_pages, int layer, int nchunk, int ct, float* part, int* err,
           cudaStream_t st) {
    if (prepare) {
        cudaFuncSetAttribute(attn_chunk_mma<HD, G>, cudaFuncAttributeMaxDynamicSharedMemorySize,
                             (int)smem_bytes<HD, G>());
        cudaFuncSetAttribute(attn_chunk_mma<HD, G>, cudaFuncAttributePreferredSharedMemoryCarveout, 100);
        return 0;
    }
    const long ctas = (long)B * nkv * nchunk;
    CUtensorMap m;                      // the caller's copy need not be 64-byte aligned
    memcpy(&m, map, sizeof m);
    return sb_launch_pdl(attn_chunk_mma<HD, G>, dim3((unsigned)ctas), dim3(32 * (NW + 1)),
                         smem_bytes<HD, G>(), st, m, qkv, ld_qkv, B, nq, nkv, row_pos, row_slot,
                         page_table, max_pages, n_pages, layer, nchunk, ct, part, err) == cudaSuccess
               ? 0
               : -1;
}

template <int HD, int G>
int launch_prefill(int prepare, const void* map, const float* qkv, int ld_qkv, int B, int nq,
                   int nkv, const int32_t* row_pos, const int32_t* row_slot,
                   const int32_t* page_table, int max_pages, int64_t n_pages, int layer,
                   int nchunk, float* part, int* err, cudaStream_t st) {
    const size_t smem = (size_t)STAGES * 2 * 16 * HD * 2 + 1024;
    if (prepare) {
        cudaFuncSetAttribute(attn_prefill_mma<HD, G>, cudaFuncAttributeMaxDynamicSharedMemorySize,
                             (int)smem);
        return 0;
    }
    constexpr int QT = NW * (16 / G);
    const long ctas = (long)((B + QT - 1) / QT) * nkv * nchunk;
    CUtensorMap m;
    memcpy(&m, map, sizeof m);
    return sb_launch_pdl(attn_prefill_mma<HD, G>, dim3((unsigned)ctas), dim3(32 * (NW + 1)), smem,
                         st, m, qkv, ld_qkv, B, nq, nkv, row_pos, row_slot, page_table, max_pages,
                         n_pages, layer, nchunk, part, err) == cudaSuccess
               ? 0
               : -1;
}

template <int HD>
int launch_hd(int prepare, int prefill, int G, const void* map, const float* qkv, int ld_qkv,
              int B, int nq, int nkv, const int32_t* row_pos, const int32_t* row_slot,
              const int32_t* page_table, int max_pages, int64_t n_pages, int layer, int nchunk,
              int ct, float* part, int* err, cudaStream_t st) {
    switch (G) {
#define CASE(g)                                                                                 \
    case g:                                                                                     \
        return prefill ? launch_prefill<HD, g>(prepare, map, qkv, ld_qkv, B, nq, nkv, row_pos,  \
                                               row_slot, page_table, max_pages, n_pages, layer, \
                                               nchunk, part, err, st)                           \
                       : launch<HD, g>(prepare, map, qkv, ld_qkv, B, nq, nkv, row_pos, row_slot, \
                                       page_table, max_pages, n_pages, layer, nchunk, ct, part,  \
                                       err, st);
        CASE(1) CASE(2) CASE(4) CASE(8)
#undef CASE
    }
    return -1;
}

}  // namespace

extern "C" int sb_attention_mma_supported(int nq, int nkv, int hd, int kv_dtype) {
    if (kv_dtype != SLATE_KV_F16 || nkv < 1 || nq % nkv) return 0;
    const int G = nq / nkv;
    return (hd == 64 || hd == 128) && (G == 1 || G == 2 || G == 4 || G == 8);
}

extern "C" int sb_attention_make_map(void* map, void* pool, int64_t n_pages, int layers, int nkv,
                                     int hd) {
    cudaDriverEntryPointQueryResult q;
    void* p = nullptr;
    if (cudaGetDriverEntryPoint("cuTensorMapEncodeTiled", &p, cudaEnableDefault, &q) != cudaSuccess ||
        q != cudaDriverEntryPointSuccess) {
        sb_set_error("KV tensor map: cuTensorMapEncodeTiled not available");
        return -1;
    }
    auto enc = (PFN_cuTensorMapEncodeTiled_v12000)p;
    // the pool as a 3-D tensor [layer][row][head_dim] f16, one row per
    // (page, K|V, kv head, token)
    const uint64_t rows = (uint64_t)n_pages * 2 * nkv * 16;
    if (rows >= (1ull << 31) || hd % 64) {
        sb_set_error("KV tensor map: %llu rows of %d not addressable", (unsigned long long)rows, hd);
        return -1;
    }
    cuuint64_t dims[3] = {(cuuint64_t)hd, (cuuint64_t)rows, (cuuint64_t)layers};
    cuuint64_t strides[2] = {(cuuint64_t)hd * 2, (cuuint64_t)(rows * hd * 2)};
    cuuint32_t box[3] = {64, 16, 1};
    cuuint32_t estr[3] = {1, 1, 1};
    CUtensorMap m;
    CUresult r = enc(&m, CU_TENSOR_MAP_DATA_TYPE_FLOAT16, 3, pool, dims, strides, box, estr,
                     CU_TENSOR_MAP_INTERLEAVE_NONE, CU_TENSOR_MAP_SWIZZLE_128B,
                     CU_TENSOR_MAP_L2_PROMOTION_L2_256B, CU_TENSOR_MAP_FLOAT_OOB_FILL_NONE);
    if (r != CUDA_SUCCESS) {
        sb_set_error("KV tensor map: cuTensorMapEncodeTiled failed (%d)", (int)r);
        return -1;
    }
    memcpy(map, &m, sizeof m);
    return 0;
}

static int attention_mma(int prepare, int prefill, const void* map, const float* qkv, int ld_qkv,
                         int B, int nq, int nkv, int hd, const int32_t* row_pos,
                         const int32_t* row_slot, const int32_t* page_table, int max_pages,
                         int64_t n_pages, int layer, int nchunk, int ct, float* part, int* err,
                         cudaStream_t st) {
    const int G = nq / nkv;
    switch (hd) {
        case 64:
            return launch_hd<64>(prepare, prefill, G, map, qkv, ld_qkv, B, nq, nkv, row_pos,
                                 row_slot, page_table, max_pages, n_pages, layer, nchunk, ct,
                                 part, err, st);
        case 128:
            return launch_hd<128>(prepare, prefill, G, map, qkv, ld_qkv, B, nq, nkv, row_pos,
                                  row_slot, page_table, max_pages, n_pages, layer, nchunk, ct,
                                  part, err, st);
    }
    return -1;
}

extern "C" int sb_attention_mma(int prepare, const void* map, const float* qkv, int ld_qkv, int B,
                                int nq, int nkv, int hd, const int32_t* row_pos,
                                const int32_t* row_slot, const int32_t* page_table, int max_pages,
                                int64_t n_pages, int layer, int nchunk, int ct, float* part,
                                int* err, cudaStream_t st) {
    if (prepare)   // both kernels' shared-memory attributes
        return attention_mma(1, 0, nullptr, nullptr, 0, 0, nq, nkv, hd, nullptr, nullptr, nullptr,
                             0, 0, 0, 0, 0, nullptr, nullptr, 0) |
               attention_mma(1, 1, nullptr, nullptr, 0, 0, nq, nkv, hd, nullptr, nullptr, nullptr,
                             0, 0, 0, 0, 0, nullptr, nullptr, 0);
    if (ct < 16 || ct > SB_ATTN_CHUNK || ct % 16) return -1;
    return attention_mma(0, 0, map, qkv, ld_qkv, B, nq, nkv, hd, row_pos, row_slot, page_table,
                         max_pages, n_pages, layer, nchunk, ct, part, err, st);
}

extern "C" int sb_attention_prefill_mma(const void* map, const float* qkv, int ld_qkv, int B,
                                        int nq, int nkv, int hd, const int32_t* row_pos,
                                        const int32_t* row_slot, const int32_t* page_table,
                                        int max_pages, int64_t n_pages, int layer, int nchunk,
                                        float* part, int* err, cudaStream_t st) {
    return attention_mma(0, 1, map, qkv, ld_qkv, B, nq, nkv, hd, row_pos, row_slot, page_table,
                         max_pages, n_pages, layer, nchunk, SB_ATTN_CHUNK, part, err, st);
}
