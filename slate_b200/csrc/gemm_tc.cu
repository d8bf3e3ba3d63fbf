// gemm_tc.cu -- Q4_K weight GEMM on the 5th-generation tensor cores (sm_100a).
//
//   ws[s][n][m] = sum_{k in split s} X[n][k] * W[m][k]          (f32, TMEM)
//
// followed by sb_tc_finish(), which sums the K splits and applies the STORE /
// ADD (residual) / SILU (gate|up) epilogue.  Used for batched decode where
// the contraction is dense (B >= 16 rows): same weights and math as the
// reference's matvec_q4k (src/util/quant.c:306-313), B rows at a time.
//
// Per CTA: one 128-row weight tile x up to 256 activation rows, K in steps of
// 64 (128 bytes of f16 = one 128B-swizzle row).  Warps 0-3 are producers: each
// thread dequantises one weight row's 64 Q4_K values (d*sc*q - dmin*mn, the
// reference's f32 reconstruction, util/quant.c:187-199) to f16 and stores them
// in the canonical K-major SWIZZLE_128B layout; thread 0 also starts the TMA
// loads of the activation tile (f16, already in the same layout via the tensor
// map's 128B swizzle).  Warp 4 allocates TMEM and one elected thread issues
// tcgen05.mma (kind::f16, f32 accumulate, M=128, N=rows) per 16-wide K slice;
// tcgen05.commit on the stage's "empty" mbarrier hands the buffers back.
// After the last K step warps 0-3 read the accumulator with tcgen05.ld
// (warp w owns TMEM lanes 32w..32w+31 = weight rows) and write f32 partials.
//
// Precision: PASSES == 1 multiplies f16(w) by f16(x).  PASSES == 3 splits both
// operands into f16 hi + lo parts (v = hi + lo to 22 bits) and accumulates
// hi*hi + hi*lo + lo*hi, which reproduces f32 products to ~1e-6 relative.
//
// Every wait is bounded (2 s of %globaltimer); on timeout the kernel records
// an error code in *err, stops issuing work, and still frees its TMEM.
#include <cuda.h>
#include <cuda_fp16.h>
#include <cudaTypedefs.h>
#include <math.h>
#include <string.h>

#include "sb_internal.h"
#include "sb_kernels.h"
#include "sb_tc.h"

namespace {

constexpr int BM = 128;       // weight rows per CTA (TMEM lanes)
constexpr int BK = 64;        // K elements per stage (one 128-byte swizzle row)
constexpr int NPROD = 128;    // producer threads (warps 0-3)
constexpr int NTHREADS = 160; // + warp 4 (TMEM owner, MMA issuer)
constexpr uint64_t WAIT_NS = 2000000000ull;

__device__ __forceinline__ uint32_t smem_u32(const void* p) {
    return (uint32_t)__cvta_generic_to_shared(p);
}
__device__ __forceinline__ uint64_t gtimer() {
    uint64_t t;
    asm volatile("mov.u64 %0, %%globaltimer;" : "=l"(t));
    return t;
}
__device__ __forceinline__ void mbar_init(uint64_t* b, uint32_t count) {
    asm volatile("mbarrier.init.shared::cta.b64 [%0], %1;" ::"r"(smem_u32(b)), "r"(count));
}
__device__ __forceinline__ void mbar_arrive(uint64_t* b) {
    asm volatile("mbarrier.arrive.shared::cta.b64 _, [%0];" ::"r"(smem_u32(b)) : "memory");
}
__device__ __forceinline__ void mbar_expect_tx(uint64_t* b, uint32_t bytes) {
    asm volatile("mbarrier.arrive.expect_tx.shared::cta.b64 _, [%0], %1;" ::"r"(smem_u32(b)),
                 "r"(bytes)
                 : "memory");
}
__device__ __forceinline__ bool mbar_try(uint64_t* b, uint32_t parity) {
    uint32_t ok;
    asm volatile(
        "{\n\t.reg .pred p;\n\t"
        "mbarrier.try_wait.parity.shared::cta.b64 p, [%1], %2;\n\t"
        "selp.u32 %0, 1, 0, p;\n\t}\n"
        : "=r"(ok)
        : "r"(smem_u32(b)), "r"(parity)
        : "memory");
    return ok != 0;
}
// Bounded wait: false (and *err set) after WAIT_NS, or at once if another
// thread of the grid already failed.
__device__ bool mbar_wait(uint64_t* b, uint32_t parity, int* err, int code) {
    if (mbar_try(b, parity)) return true;
    const uint64_t t0 = gtimer();
    while (true) {
        if (mbar_try(b, parity)) return true;
        if (*(volatile int*)err) return false;
        if (gtimer() - t0 > WAIT_NS) {
            atomicCAS(err, 0, code);
            return false;
        }
    }
}
__device__ __forceinline__ void fence_async_smem() {
    asm volatile("fence.proxy.async.shared::cta;" ::: "memory");
}
__device__ __forceinline__ void tma_load_2d(void* dst, const CUtensorMap* map, uint64_t* bar, int x,
                                            int y) {
    asm volatile(
        "cp.async.bulk.tensor.2d.shared::cluster.global.tile.mbarrier::complete_tx::bytes "
        "[%0], [%1, {%3, %4}], [%2];" ::"r"(smem_u32(dst)),
        "l"(map), "r"(smem_u32(bar)), "r"(x), "r"(y)
        : "memory");
}
__device__ __forceinline__ void tc_fence_before() {
    asm volatile("tcgen05.fence::before_thread_sync;" ::: "memory");
}
__device__ __forceinline__ void tc_fence_after() {
    asm volatile("tcgen05.fence::after_thread_sync;" ::: "memory");
}
// K-major operand, SWIZZLE_128B: 8-row atoms of 128-byte rows, atoms 1024 B
// apart (SBO), LBO unused (1), descriptor version 1.
__device__ __forceinline__ uint64_t sw128_desc(uint32_t saddr) {
    return (uint64_t)((saddr & 0x3FFFFu) >> 4) | (1ull << 16) | ((uint64_t)(1024 >> 4) << 32) |
           (1ull << 46) | (2ull << 61);
}
__device__ __forceinline__ void mma_f16(uint32_t tmem_d, uint64_t a, uint64_t b, uint32_t idesc,
                                        uint32_t acc) {
    asm volatile(
        "{\n\t.reg .pred p;\n\t"
        "setp.ne.b32 p, %4, 0;\n\t"
        "tcgen05.mma.cta_group::1.kind::f16 [%0], %1, %2, %3, p;\n\t}\n" ::"r"(tmem_d),
        "l"(a), "l"(b), "r"(idesc), "r"(acc));
}
__device__ __forceinline__ void mma_commit(uint64_t* bar) {
    asm volatile(
        "tcgen05.commit.cta_group::1.mbarrier::arrive::one.shared::cluster.b64 [%0];" ::"r"(
            smem_u32(bar))
        : "memory");
}
__device__ __forceinline__ void tmem_ld16(uint32_t taddr, float (&v)[16]) {
    uint32_t r[16];
    asm volatile(
        "tcgen05.ld.sync.aligned.32x32b.x16.b32 "
        "{%0, %1, %2, %3, %4, %5, %6, %7, %8, %9, %10, %11, %12, %13, %14, %15}, [%16];"
        : "=r"(r[0]), "=r"(r[1]), "=r"(r[2]), "=r"(r[3]), "=r"(r[4]), "=r"(r[5]), "=r"(r[6]),
          "=r"(r[7]), "=r"(r[8]), "=r"(r[9]), "=r"(r[10]), "=r"(r[11]), "=r"(r[12]), "=r"(r[13]),
          "=r"(r[14]), "=r"(r[15])
        : "r"(taddr));
    asm volatile("tcgen05.wait::ld.sync.aligned;" ::: "memory");
#pragma unroll
    for (int i = 0; i < 16; ++i) v[i] = __uint_as_float(r[i]);
}

__device__ __forceinline__ float f16lo(uint32_t w) {
    return __half2float(__ushort_as_half((unsigned short)(w & 0xffffu)));
}
__device__ __forceinline__ float f16hi(uint32_t w) {
    return __half2float(__ushort_as_half((unsigned short)(w >> 16)));
}
__device__ __forceinline__ uint32_t hdr_byte(uint4 h, int i) {
    uint32_t w = i < 4 ? h.y : (i < 8 ? h.z : h.w);
    return (w >> ((i & 3) * 8)) & 0xffu;
}
__device__ __forceinline__ void sub_scale(uint4 h, int j, float& sd, float& sm) {
    const float d = f16lo(h.x), dmin = f16hi(h.x);
    uint32_t sc, mn;
    if (j < 4) {
        sc = hdr_byte(h, j) & 63u;
        mn = hdr_byte(h, j + 4) & 63u;
    } else {
        sc = (hdr_byte(h, j + 4) & 15u) | ((hdr_byte(h, j - 4) >> 6) << 4);
        mn = (hdr_byte(h, j + 4) >> 4) | ((hdr_byte(h, j) >> 6) << 4);
    }
    sd = d * (float)sc;
    sm = dmin * (float)mn;
}
__device__ __forceinline__ uint32_t pack_h2(float a, float b) {
    __half2 h = __floats2half2_rn(a, b);
    return *(uint32_t*)&h;
}

// Pulls one 144-byte Q4_K super-block into L2 ahead of use (the lines holding
// its first, middle and last byte).
__device__ __forceinline__ void l2_prefetch_block(const unsigned char* p) {
    asm volatile("prefetch.global.L2 [%0];" ::"l"(p));
    asm volatile("prefetch.global.L2 [%0];" ::"l"(p + 72));
    asm volatile("prefetch.global.L2 [%0];" ::"l"(p + 143));
}

// The low nibble of v as a float, exactly: 2^23 + q has q in its low mantissa
// bits, so subtracting 2^23 leaves q (an OR and an FADD on the full-rate
// pipes instead of an integer-to-float conversion).
__device__ __forceinline__ float nib_f32(uint32_t v) {
    return __uint_as_float(0x4B000000u | (v & 15u)) - 8388608.0f;
}

// Dequantises 32 weights (one Q4_K sub-block, 16 nibble bytes) into f16 hi
// (and lo) words: out[c] holds elements 2c, 2c+1.
template <int PASSES>
__device__ __forceinline__ void dequant32(uint4 q, float sd, float sm, uint32_t (&hi)[16],
                                          uint32_t (&lo)[16]) {
    const uint32_t qw[4] = {q.x, q.y, q.z, q.w};
    float w[32];
#pragma unroll
    for (int i = 0; i < 16; ++i) {
        const uint32_t b = qw[i >> 2] >> ((i & 3) * 8);
        w[i] = sd * nib_f32(b) - sm;
        w[i + 16] = sd * nib_f32(b >> 4) - sm;
    }
#pragma unroll
    for (int c = 0; c < 16; ++c) {
        const __half2 h = __floats2half2_rn(w[2 * c], w[2 * c + 1]);
        hi[c] = *(const uint32_t*)&h;
        if (PASSES == 3) {
            const float2 back = __half22float2(h);
            lo[c] = pack_h2(w[2 * c] - back.x, w[2 * c + 1] - back.y);
        }
    }
}

// AMODE 0: the A operand (weights) is Q4_K, dequantised by warps 0-3.
// AMODE 1: the A operand is an f16 hi (+ lo) weight pair in global memory,
//          loaded by TMA like the activations (f32 weights split once at load).
// direct 0: write f32 partials ws[split][n][m]; 1: Y[n][m] = acc; 2: Y += acc
// (direct modes need splits == 1).
template <int PASSES, int STAGES, int AMODE>
__global__ void __launch_bounds__(NTHREADS, 1)
    tc_kernel(const __grid_constant__ CUtensorMap xmap_hi, const __grid_constant__ CUtensorMap xmap_lo,
              const __grid_constant__ CUtensorMap amap_hi, const __grid_constant__ CUtensorMap amap_lo,
              const unsigned char* __restrict__ W, int M, int M_pad, int K, int n_rows, int n_box,
              int splits, float* __restrict__ ws, float* __restrict__ Y, int ldy, int direct,
              int* err, int wexp) {
    extern __shared__ __align__(1024) unsigned char smem_raw[];
    // weights enter the split as w * 2^wexp (exact); the epilogue scales back
    const float wsc = ldexpf(1.0f, wexp), wun = ldexpf(1.0f, -wexp);
    // 1024-aligned carve-up: per stage [A_hi | A_lo | B_hi | B_lo]
    unsigned char* base = (unsigned char*)(((uintptr_t)smem_raw + 1023) & ~(uintptr_t)1023);
    constexpr int PARTS = PASSES == 3 ? 2 : 1;
    const int a_bytes = BM * 128;            // 16 KB per operand part
    const int b_bytes = n_box * 128;
    const int stage_bytes = PARTS * (a_bytes + b_bytes);
    __shared__ uint64_t full_bar[STAGES], empty_bar[STAGES], done_bar;
    __shared__ uint32_t tmem_slot;

    const int tid = threadIdx.x, warp = tid >> 5, lane = tid & 31;
    const int m_tile = blockIdx.x, split = blockIdx.y, n_chunk = blockIdx.z;
    const int n0 = n_chunk * 256;
    const int n_here = min(n_rows - n0, 256);
    const int n_mma = (n_here + 15) & ~15;                 // tcgen05 N: multiple of 16
    const int nk = K / BK;
    const int ks0 = (int)((long)nk * split / splits), ks1 = (int)((long)nk * (split + 1) / splits);
    const uint32_t tmem_cols = n_mma <= 32 ? 32 : n_mma <= 64 ? 64 : n_mma <= 128 ? 128 : 256;

    if (tid == 0) {
        for (int s = 0; s < STAGES; ++s) {
            mbar_init(&full_bar[s], AMODE == 0 ? NPROD + 1 : 1);
            mbar_init(&empty_bar[s], 1);
        }
        mbar_init(&done_bar, 1);
        asm volatile("fence.mbarrier_init.release.cluster;" ::: "memory");
    }
    if (warp == 4) {
        asm volatile("tcgen05.alloc.cta_group::1.sync.aligned.shared::cta.b32 [%0], %1;" ::"r"(
                         smem_u32(&tmem_slot)),
                     "r"(tmem_cols));
        asm volatile("tcgen05.relinquish_alloc_permit.cta_group::1.sync.aligned;");
    }
    tc_fence_before();
    __syncthreads();
    tc_fence_after();
    const uint32_t tmem = tmem_slot;
    bool ok = true;

    if (warp < 4 && (AMODE == 0 || tid == 0)) {
        // ---------------- producers ----------------
        const int m = tid;                                   // tile row (AMODE 0)
        const size_t row_bytes = (size_t)(K / 256) * 144;
        const unsigned char* wrow = AMODE == 0 ? W + (size_t)(m_tile * BM + m) * row_bytes : nullptr;
        const uint32_t row_off = (uint32_t)((m >> 3) * 1024 + (m & 7) * 128);
        // Weight bytes are loaded one K step ahead (registers), so the DRAM
        // latency of step ks+1 overlaps the dequantisation of step ks.
        uint4 hdr = make_uint4(0, 0, 0, 0), q0 = hdr, q1 = hdr, nhdr = hdr, nq0 = hdr, nq1 = hdr;
        const int nsb = K / 256;
        if (AMODE == 0 && ks0 < ks1) {
            const unsigned char* p = wrow + (size_t)(ks0 >> 2) * 144;
            hdr = __ldg((const uint4*)p);
            q0 = __ldg((const uint4*)(p + 16 + 32 * (ks0 & 3)));
            q1 = __ldg((const uint4*)(p + 32 + 32 * (ks0 & 3)));
            // the next super-block goes to L2 now, the one after it on
            // entering each block (below): two blocks ahead
            if ((ks0 >> 2) + 1 < nsb) l2_prefetch_block(p + 144);
        }
        for (int ks = ks0; ks < ks1 && ok; ++ks) {
            const int it = ks - ks0, s = it % STAGES;
            if (it >= STAGES && !mbar_wait(&empty_bar[s], ((it / STAGES) - 1) & 1, err, 1)) {
                ok = false;
                break;
            }
            unsigned char* st = base + (size_t)s * stage_bytes;
            unsigned char* a_hi = st;
            unsigned char* a_lo = st + a_bytes;
            unsigned char* b_hi = st + PARTS * a_bytes;
            unsigned char* b_lo = b_hi + b_bytes;
            if (tid == 0) {
                mbar_expect_tx(&full_bar[s],
                               (uint32_t)(PARTS * b_bytes + (AMODE == 1 ? PARTS * a_bytes : 0)));
                if (AMODE == 1) {
                    tma_load_2d(a_hi, &amap_hi, &full_bar[s], ks * BK, m_tile * BM);
                    if (PASSES == 3) tma_load_2d(a_lo, &amap_lo, &full_bar[s], ks * BK, m_tile * BM);
                }
                tma_load_2d(b_hi, &xmap_hi, &full_bar[s], ks * BK, n0);
                if (PASSES == 3) tma_load_2d(b_lo, &xmap_lo, &full_bar[s], ks * BK, n0);
            }
            if (AMODE == 1) continue;
            const int j0 = (ks & 3) * 2;                     // 4 K-steps per super-block
            if ((ks & 3) == 0 && (ks >> 2) + 2 < nsb)
                l2_prefetch_block(wrow + (size_t)((ks >> 2) + 2) * 144);
            if (ks + 1 < ks1) {
                const unsigned char* p = wrow + (size_t)((ks + 1) >> 2) * 144;
                nhdr = ((ks + 1) & 3) == 0 ? __ldg((const uint4*)p) : hdr;
                nq0 = __ldg((const uint4*)(p + 16 + 32 * ((ks + 1) & 3)));
                nq1 = __ldg((const uint4*)(p + 32 + 32 * ((ks + 1) & 3)));
            }
            uint32_t hi[32], lo[32];
            {
                float sd, sm;
                uint32_t h16[16], l16[16];
                sub_scale(hdr, j0, sd, sm);
                dequant32<PASSES>(q0, sd * wsc, sm * wsc, h16, l16);
#pragma unroll
                for (int c = 0; c < 16; ++c) { hi[c] = h16[c]; lo[c] = l16[c]; }
                sub_scale(hdr, j0 + 1, sd, sm);
                dequant32<PASSES>(q1, sd * wsc, sm * wsc, h16, l16);
#pragma unroll
                for (int c = 0; c < 16; ++c) { hi[16 + c] = h16[c]; lo[16 + c] = l16[c]; }
            }
            // 8 chunks of 16 bytes (8 f16); chunk c lands at c ^ (row % 8)
#pragma unroll
            for (int c = 0; c < 8; ++c) {
                const uint32_t off = row_off + (uint32_t)(((c ^ (m & 7)) & 7) << 4);
                *(uint4*)(a_hi + off) = make_uint4(hi[4 * c], hi[4 * c + 1], hi[4 * c + 2], hi[4 * c + 3]);
                if (PASSES == 3)
                    *(uint4*)(a_lo + off) = make_uint4(lo[4 * c], lo[4 * c + 1], lo[4 * c + 2], lo[4 * c + 3]);
            }
            fence_async_smem();
            mbar_arrive(&full_bar[s]);
            hdr = nhdr;
            q0 = nq0;
            q1 = nq1;
        }
    } else if (warp == 4 && lane == 0) {
        // ---------------- MMA issuer ----------------
        const uint32_t idesc = (1u << 4) | ((uint32_t)(n_mma >> 3) << 17) | ((uint32_t)(BM >> 4) << 24);
        for (int ks = ks0; ks < ks1; ++ks) {
            const int it = ks - ks0, s = it % STAGES;
            if (!mbar_wait(&full_bar[s], (it / STAGES) & 1, err, 2)) {
                ok = false;
                break;
            }
            tc_fence_after();
            unsigned char* st = base + (size_t)s * stage_bytes;
            const uint32_t a_hi = smem_u32(st), a_lo = a_hi + a_bytes;
            const uint32_t b_hi = smem_u32(st + PARTS * a_bytes), b_lo = b_hi + b_bytes;
#pragma unroll
            for (int k = 0; k < BK / 16; ++k) {
                const uint32_t koff = 32u * k;                // 16 f16 = 32 bytes along K
                const uint32_t acc = (it > 0 || k > 0) ? 1u : 0u;
                mma_f16(tmem, sw128_desc(a_hi + koff), sw128_desc(b_hi + koff), idesc, acc);
                if (PASSES == 3) {
                    mma_f16(tmem, sw128_desc(a_hi + koff), sw128_desc(b_lo + koff), idesc, 1u);
                    mma_f16(tmem, sw128_desc(a_lo + koff), sw128_desc(b_hi + koff), idesc, 1u);
                }
            }
            mma_commit(&empty_bar[s]);
        }
        mma_commit(&done_bar);   // arrives once every MMA issued above has completed
    }
    __syncwarp();

    // ---------------- epilogue: TMEM -> f32 ----------------
    if (warp < 4) {
        bool have = ok && mbar_wait(&done_bar, 0, err, 3);
        have = __all_sync(0xffffffffu, have);   // tcgen05.ld is warp-collective
        tc_fence_after();
        if (have) {
            const int m = m_tile * BM + warp * 32 + lane;
            for (int c0 = 0; c0 < n_mma; c0 += 16) {
                float v[16];
                tmem_ld16(tmem + ((uint32_t)(warp * 32) << 16) + (uint32_t)c0, v);
#pragma unroll
                for (int j = 0; j < 16; ++j) v[j] *= wun;
#pragma unroll
                for (int j = 0; j < 16; ++j) {
                    const int n = c0 + j;
                    if (n >= n_here) continue;
                    if (direct == 0) {
                        ws[((size_t)split * n_rows + n0 + n) * M_pad + m] = v[j];
                    } else if (m < M) {
                        float* y = Y + (size_t)(n0 + n) * ldy + m;
                        *y = direct == 2 ? *y + v[j] : v[j];
                    }
                }
            }
        }
    }
    tc_fence_before();
    __syncthreads();
    if (warp == 4) {
        tc_fence_after();
        asm volatile("tcgen05.dealloc.cta_group::1.sync.aligned.b32 %0, %1;" ::"r"(tmem),
                     "r"(tmem_cols));
    }
}

// Sum of K-split partials plus the epilogue.
template <int EPI>
__global__ void tc_finish_kernel(const float* __restrict__ ws, int splits, int n_rows, int M_pad,
                                 int M, float* __restrict__ Y, int ldy) {
    const int n_out = EPI == SB_EPI_SILU ? M / 2 : M;
    const long total = (long)n_rows * n_out;
    for (long i = (long)blockIdx.x * blockDim.x + threadIdx.x; i < total;
         i += (long)gridDim.x * blockDim.x) {
        const int n = (int)(i / n_out), o = (int)(i % n_out);
        if (EPI == SB_EPI_SILU) {
            const int gm = (o / 64) * 128 + (o % 64);
            float g = 0.f, u = 0.f;
            for (int s = 0; s < splits; ++s) {
                const float* p = ws + ((size_t)s * n_rows + n) * M_pad;
                g += p[gm];
                u += p[gm + 64];
            }
            Y[(size_t)n * ldy + o] = g / (1.0f + expf(-g)) * u;
        } else {
            float v = 0.f;
            for (int s = 0; s < splits; ++s) v += ws[((size_t)s * n_rows + n) * M_pad + o];
            float* y = Y + (size_t)n * ldy + o;
            *y = EPI == SB_EPI_ADD ? *y + v : v;
        }
    }
}

// f32 activations -> f16 hi (and lo = f16(x - hi)) rows for the TMA operand:
// one row per blockIdx.y, four elements (one float4, one 8-byte hi word and one
// lo word) per thread.  Needs K % 4 == 0, ldx % 4 == 0, ld16 % 4 == 0 and a
// 16-byte aligned X.
__global__ void split_f16_rows_kernel(const float* __restrict__ X, int ldx, int K,
                                     __half* __restrict__ hi, __half* __restrict__ lo, int ld16) {
    const int n = blockIdx.y;
    const float4* x4 = (const float4*)(X + (size_t)n * ldx);
    uint2* h2 = (uint2*)(hi + (size_t)n * ld16);
    uint2* l2 = lo ? (uint2*)(lo + (size_t)n * ld16) : nullptr;
    for (int j = blockIdx.x * blockDim.x + threadIdx.x; j < K / 4; j += gridDim.x * blockDim.x) {
        const float4 v = __ldg(x4 + j);
        const __half2 a = __floats2half2_rn(v.x, v.y), b = __floats2half2_rn(v.z, v.w);
        h2[j] = make_uint2(*(const uint32_t*)&a, *(const uint32_t*)&b);
        if (l2) {
            const float2 ab = __half22float2(a), bb = __half22float2(b);
            const __half2 la = __floats2half2_rn(v.x - ab.x, v.y - ab.y);
            const __half2 lb = __floats2half2_rn(v.z - bb.x, v.w - bb.y);
            l2[j] = make_uint2(*(const uint32_t*)&la, *(const uint32_t*)&lb);
        }
    }
}

// Scalar form of the same split, for any strides and alignment.
__global__ void split_f16_kernel(const float* __restrict__ X, int ldx, int n_rows, int K,
                                 __half* __restrict__ hi, __half* __restrict__ lo, int ld16,
                                 float scale) {
    const long total = (long)n_rows * K;
    for (long i = (long)blockIdx.x * blockDim.x + threadIdx.x; i < total;
         i += (long)gridDim.x * blockDim.x) {
        const int n = (int)(i / K), k = (int)(i % K);
        const float x = X[(size_t)n * ldx + k] * scale;
        const __half h = __float2half_rn(x);
        hi[(size_t)n * ld16 + k] = h;
        if (lo) lo[(size_t)n * ld16 + k] = __float2half_rn(x - __half2float(h));
    }
}

template <int PASSES>
constexpr int stages_for() { return PASSES == 3 ? 2 : 4; }

template <int PASSES>
size_t smem_for(int n_box) {
    const int part = BM * 128 + n_box * 128;
    return (size_t)stages_for<PASSES>() * (PASSES == 3 ? 2 : 1) * part + 1024;
}

PFN_cuTensorMapEncodeTiled_v12000 encode_fn() {
    static PFN_cuTensorMapEncodeTiled_v12000 fn = nullptr;
    if (!fn) {
        cudaDriverEntryPointQueryResult q;
        void* p = nullptr;
        if (cudaGetDriverEntryPoint("cuTensorMapEncodeTiled", &p, cudaEnableDefault, &q) ==
                cudaSuccess &&
            q == cudaDriverEntryPointSuccess)
            fn = (PFN_cuTensorMapEncodeTiled_v12000)p;
    }
    return fn;
}

}  // namespace

extern "C" int sb_tc_make_operand(sb_tc_operand* op, void* hi, void* lo, int rows, int K, int ld16) {
    PFN_cuTensorMapEncodeTiled_v12000 enc = encode_fn();
    if (!enc || !op || !hi || K % BK || ld16 % 8 || rows < 1) return -1;
    op->hi = hi;
    op->lo = lo;
    op->rows = rows;
    op->K = K;
    op->ld16 = ld16;
    op->n_box = rows >= 256 ? 256 : (rows + 15) & ~15;
    for (int part = 0; part < 2; ++part) {
        void* g = part ? (lo ? lo : hi) : hi;
        cuuint64_t dims[2] = {(cuuint64_t)K, (cuuint64_t)rows};
        cuuint64_t strides[1] = {(cuuint64_t)ld16 * 2};
        cuuint32_t box[2] = {(cuuint32_t)BK, (cuuint32_t)op->n_box};
        cuuint32_t estr[2] = {1, 1};
        CUresult r = enc((CUtensorMap*)(part ? op->map_lo : op->map_hi), CU_TENSOR_MAP_DATA_TYPE_FLOAT16,
                         2, g, dims, strides, box, estr, CU_TENSOR_MAP_INTERLEAVE_NONE,
                         CU_TENSOR_MAP_SWIZZLE_128B, CU_TENSOR_MAP_L2_PROMOTION_L2_256B,
                         CU_TENSOR_MAP_FLOAT_OOB_FILL_NONE);
        if (r != CUDA_SUCCESS) {
            sb_set_error("cuTensorMapEncodeTiled failed (%d)", (int)r);
            return -1;
        }
    }
    return 0;
}

extern "C" int sb_tc_split(const float* X, int ldx, int n_rows, const sb_tc_operand* op,
                           cudaStream_t st) {
    if (n_rows < 1 || n_rows > op->rows) return -1;
    if (op->K % 4 == 0 && ldx % 4 == 0 && op->ld16 % 4 == 0 && ((uintptr_t)X & 15) == 0 &&
        n_rows <= 65535) {
        const int q = op->K / 4;
        dim3 grid((unsigned)((q + 255) / 256), (unsigned)n_rows);
        split_f16_rows_kernel<<<grid, 256, 0, st>>>(X, ldx, op->K, (__half*)op->hi,
                                                    (__half*)op->lo, op->ld16);
        return 0;
    }
    const long total = (long)n_rows * op->K;
    const int grid = (int)((total + 255) / 256 < 2368 ? (total + 255) / 256 : 2368);
    split_f16_kernel<<<grid, 256, 0, st>>>(X, ldx, n_rows, op->K, (__half*)op->hi,
                                           (__half*)op->lo, op->ld16, 1.0f);
    return 0;
}

// max |W| over M rows of K (row stride ldw) as the bits of a non-negative
// float (their order is the floats' order), for the weight pair's scale.
__global__ void absmax_kernel(const float* __restrict__ W, int ldw, int M, int K,
                              unsigned int* __restrict__ out) {
    float mx = 0.f;
    const long total = (long)M * K;
    for (long i = (long)blockIdx.x * blockDim.x + threadIdx.x; i < total;
         i += (long)gridDim.x * blockDim.x)
        mx = fmaxf(mx, fabsf(W[(size_t)(i / K) * ldw + i % K]));
    for (int o = 16; o; o >>= 1) mx = fmaxf(mx, __shfl_xor_sync(0xffffffffu, mx, o));
    if ((threadIdx.x & 31) == 0) atomicMax(out, __float_as_uint(mx));
}

extern "C" int sb_tc_make_weight(sb_tc_weight* w, const float* W32, int ldw, int M, int K,
                                 cudaStream_t st) {
    PFN_cuTensorMapEncodeTiled_v12000 enc = encode_fn();
    if (!enc || !w || K % BK) return -1;
    const int M_pad = (M + BM - 1) / BM * BM;
    void *hi = nullptr, *lo = nullptr;
    if (cudaMalloc(&hi, (size_t)M_pad * K * 2) != cudaSuccess ||
        cudaMalloc(&lo, (size_t)M_pad * K * 2) != cudaSuccess) {
        if (hi) cudaFree(hi);
        sb_set_error("cudaMalloc of %zu bytes for the f16 weight pair failed", (size_t)M_pad * K * 4);
        return -5;
    }
    cudaMemsetAsync(hi, 0, (size_t)M_pad * K * 2, st);
    cudaMemsetAsync(lo, 0, (size_t)M_pad * K * 2, st);
    const long total = (long)M * K;
    const int grid = (int)((total + 255) / 256 < 4736 ? (total + 255) / 256 : 4736);
    // the pair holds W * 2^wexp (exact), the largest power of two that keeps
    // every weight below 2^13, so that the lo halves stay normal f16 numbers
    // (a lo half of a weight near 0.02 is subnormal unscaled); the GEMM's
    // epilogue scales back by 2^-wexp
    unsigned int* d_mx = nullptr;
    unsigned int h_mx = 0;
    if (cudaMallocAsync((void**)&d_mx, sizeof(unsigned int), st) != cudaSuccess) {
        cudaFree(hi);
        cudaFree(lo);
        return -5;
    }
    cudaMemsetAsync(d_mx, 0, sizeof(unsigned int), st);
    absmax_kernel<<<grid, 256, 0, st>>>(W32, ldw, M, K, d_mx);
    cudaMemcpyAsync(&h_mx, d_mx, sizeof(unsigned int), cudaMemcpyDeviceToHost, st);
    cudaFreeAsync(d_mx, st);
    if (cudaStreamSynchronize(st) != cudaSuccess) {
        cudaFree(hi);
        cudaFree(lo);
        return -5;
    }
    float mx;
    memcpy(&mx, &h_mx, 4);
    int wexp = (mx > 0.f && isfinite(mx)) ? (int)floorf(log2f(8192.0f / mx)) : 0;
    wexp = wexp < 0 ? 0 : wexp > 24 ? 24 : wexp;
    split_f16_kernel<<<grid, 256, 0, st>>>(W32, ldw, M, K, (__half*)hi, (__half*)lo, K,
                                           ldexpf(1.0f, wexp));
    w->wexp = wexp;
    w->hi = hi;
    w->lo = lo;
    w->M = M;
    w->M_pad = M_pad;
    w->K = K;
    for (int part = 0; part < 2; ++part) {
        cuuint64_t dims[2] = {(cuuint64_t)K, (cuuint64_t)M_pad};
        cuuint64_t strides[1] = {(cuuint64_t)K * 2};
        cuuint32_t box[2] = {(cuuint32_t)BK, (cuuint32_t)BM};
        cuuint32_t estr[2] = {1, 1};
        CUresult r = enc((CUtensorMap*)(part ? w->map_lo : w->map_hi), CU_TENSOR_MAP_DATA_TYPE_FLOAT16,
                         2, part ? lo : hi, dims, strides, box, estr, CU_TENSOR_MAP_INTERLEAVE_NONE,
                         CU_TENSOR_MAP_SWIZZLE_128B, CU_TENSOR_MAP_L2_PROMOTION_L2_256B,
                         CU_TENSOR_MAP_FLOAT_OOB_FILL_NONE);
        if (r != CUDA_SUCCESS) {
            sb_set_error("cuTensorMapEncodeTiled failed (%d)", (int)r);
            return -1;
        }
    }
    return cudaGetLastError() == cudaSuccess ? 0 : -5;
}

extern "C" void sb_tc_free_weight(sb_tc_weight* w) {
    if (!w) return;
    if (w->hi) cudaFree(w->hi);
    if (w->lo) cudaFree(w->lo);
    w->hi = w->lo = nullptr;
}

extern "C" int sb_tc_gemm_f16w(const sb_tc_weight* W, const sb_tc_operand* X, int n_rows,
                               float* Y, int ldy, int epi, int* err, cudaStream_t st) {
    if (!W || !W->hi || !X || !X->lo || W->K != X->K || n_rows < 1 || n_rows > X->rows ||
        (epi != SB_EPI_STORE && epi != SB_EPI_ADD))
        return -1;
    dim3 grid((unsigned)(W->M_pad / BM), 1u, (unsigned)((n_rows + 255) / 256));
    tc_kernel<3, stages_for<3>(), 1><<<grid, NTHREADS, smem_for<3>(X->n_box), st>>>(
        *(const CUtensorMap*)X->map_hi, *(const CUtensorMap*)X->map_lo,
        *(const CUtensorMap*)W->map_hi, *(const CUtensorMap*)W->map_lo, nullptr, W->M, W->M_pad,
        W->K, n_rows, X->n_box, 1, nullptr, Y, ldy, epi == SB_EPI_ADD ? 2 : 1, err, W->wexp);
    return 0;
}

extern "C" int sb_tc_splits_for(int M_pad, int K) {
    const int tiles = M_pad / BM, nk = K / BK;
    int s = 148 / (tiles > 0 ? tiles : 1);
    if (s < 1) s = 1;
    if (s > nk / 4) s = nk / 4 > 0 ? nk / 4 : 1;
    return s;
}

extern "C" void sb_tc_prepare(void) {
    cudaFuncSetAttribute(tc_kernel<1, stages_for<1>(), 0>,
                         cudaFuncAttributeMaxDynamicSharedMemorySize, (int)smem_for<1>(256));
    cudaFuncSetAttribute(tc_kernel<3, stages_for<3>(), 0>,
                         cudaFuncAttributeMaxDynamicSharedMemorySize, (int)smem_for<3>(256));
    cudaFuncSetAttribute(tc_kernel<3, stages_for<3>(), 1>,
                         cudaFuncAttributeMaxDynamicSharedMemorySize, (int)smem_for<3>(256));
}

extern "C" int sb_tc_gemm(const sb_matrix* W, const sb_tc_operand* X, int n_rows, int passes,
                          int splits, float* ws, float* Y, int ldy, int epi, int* err,
                          cudaStream_t st) {
    if (!W || !X || W->wtype != SB_WT_Q4K || W->M_pad % BM || W->K % 256 || W->K != X->K ||
        n_rows < 1 || n_rows > X->rows || splits < 1 || (passes != 1 && passes != 3) ||
        (passes == 3 && !X->lo))
        return -1;
    dim3 grid((unsigned)(W->M_pad / BM), (unsigned)splits, (unsigned)((n_rows + 255) / 256));
    const unsigned char* w = (const unsigned char*)W->data;
    const CUtensorMap* xh = (const CUtensorMap*)X->map_hi;
    const CUtensorMap* xl = (const CUtensorMap*)(passes == 3 ? X->map_lo : X->map_hi);
    // one split and a STORE / ADD epilogue: write Y straight from TMEM
    const int direct = splits == 1 && epi != SB_EPI_SILU ? (epi == SB_EPI_ADD ? 2 : 1) : 0;
    if (passes == 1)
        tc_kernel<1, stages_for<1>(), 0><<<grid, NTHREADS, smem_for<1>(X->n_box), st>>>(
            *xh, *xl, *xh, *xh, w, W->M, W->M_pad, W->K, n_rows, X->n_box, splits, ws, Y, ldy,
            direct, err, W->wexp);
    else
        tc_kernel<3, stages_for<3>(), 0><<<grid, NTHREADS, smem_for<3>(X->n_box), st>>>(
            *xh, *xl, *xh, *xh, w, W->M, W->M_pad, W->K, n_rows, X->n_box, splits, ws, Y, ldy,
            direct, err, W->wexp);
    if (direct) return 0;
    const int n_out = epi == SB_EPI_SILU ? W->M / 2 : W->M;
    const long total = (long)n_rows * n_out;
    const int fg = (int)((total + 255) / 256 < 4736 ? (total + 255) / 256 : 4736);
    switch (epi) {
        case SB_EPI_STORE:
            tc_finish_kernel<SB_EPI_STORE><<<fg, 256, 0, st>>>(ws, splits, n_rows, W->M_pad, W->M, Y, ldy);
            break;
        case SB_EPI_ADD:
            tc_finish_kernel<SB_EPI_ADD><<<fg, 256, 0, st>>>(ws, splits, n_rows, W->M_pad, W->M, Y, ldy);
            break;
        case SB_EPI_SILU:
            tc_finish_kernel<SB_EPI_SILU><<<fg, 256, 0, st>>>(ws, splits, n_rows, W->M_pad, W->M, Y, ldy);
            break;
        default:
            return -1;
    }
    return 0;
}
