// gemm_q4k.cu -- Q4_K weight GEMM on the tcgen05 tensor cores with exact f16
// weights: two MMA passes instead of three.
//
// Reference arithmetic (src/util/quant.c:187-199, 210-304): a Q4_K weight is
//   w = d * sc_j * q - dmin * m_j      (q 4-bit, sc_j / m_j 6-bit, d / dmin f16)
// with d, dmin per 256-element super-block and sc_j, m_j per 32-element
// sub-block j.  sc_j * q <= 63 * 15 = 945 is an integer, exact in f16, so
//   y[n][m] = sum_b ( d_mb * P1_b[n][m] - dmin_mb * P2_b[n][m] )
//   P1_b = sum_{k in b} (sc*q)[m][k] * x[n][k]         (K = 256 per block)
//   P2_b = sum_{j in b} m_j[m]     * X_j[n]            X_j = sum of x over sub-block j
// The tensor cores compute P1 with A = f16(sc*q) (exact) against x split into
// f16 hi + lo (22 bits; two MMAs per K slice).  The dmin term needs no
// per-block scale: sum_b dmin_b * P2_b = sum_j c_j X_j with c_j = dmin * m_j
// (17 bits, exact as an f16 hi + lo pair), a GEMM over K/32 that three K=16
// MMAs per two super-blocks accumulate into one TMEM accumulator Q for the
// whole tile.  All products are exact in the f32 accumulator.  Four epilogue
// ("drain") warps read P1 out of TMEM after every super-block and accumulate
// d * P1 in f32 registers, then subtract Q, so the block scales are applied
// exactly as the reference applies them, in a different summation order.
//
// Operand placement follows the tensor core's shared-memory read budget: the
// dequantised weights never touch shared memory.  Producer thread m holds
// weight row m and writes its 64 f16 values of a K step straight into TMEM
// lane m (tcgen05.st), which is where an MMA with A in tensor memory reads
// row m; only the activations (B) stream through shared memory, so an MMA
// reads 4 KB of shared memory for 128 x 128 x 16 multiply-adds.
//
// Tiles are 128 weight rows x 128 activation rows.  The grid is persistent,
// one CTA per SM, over a stream-K schedule: the (tile, 64-wide K step) space
// is cut into equal contiguous ranges, one per CTA.  A tile covered by one CTA
// is written directly (store / residual add / fused SiLU(gate) * up); a tile
// shared by several CTAs is written as partials, and the last CTA to finish
// (per-tile arrival counter) sums them in a fixed order and applies the
// epilogue, so results do not depend on timing.
//
// Roles (320 threads): warps 0-3 dequantise (one weight row per thread) into
// TMEM and write c_j hi / lo into shared memory; warp 4 issues the MMAs; warp 5
// issues the TMA loads of x (hi, lo) and the bulk copies of the sub-block sums;
// warps 6-9 drain TMEM.  TMEM columns: P1 x2 [0, 256), Q [256, 384), A ring
// [384, 512) (4 stages x 32).  Every wait is bounded (2 s of %globaltimer); a
// timeout records an error code, the roles stop, in-flight copies are waited
// for and TMEM is freed.
#include <cuda.h>
#include <stdlib.h>
#include <string.h>
#include <cuda_fp16.h>
#include <cudaTypedefs.h>

#include "sb_internal.h"
#include "sb_kernels.h"
#include "sb_tc.h"

namespace {

constexpr int BM = 128;                 // weight rows per tile (TMEM lanes)
constexpr int BN = 128;                 // activation rows per tile (MMA N)
constexpr int BK = 64;                  // K per pipeline stage (one 128-byte swizzle row)
constexpr int STAGES = 4;               // A stages in TMEM (32 columns each), B stages in smem
constexpr int NPROD = 128;
constexpr int MMA_WARP = 4, TMA_WARP = 5, DRAIN_WARP0 = 6;
constexpr int NTHREADS = 320;
constexpr uint64_t WAIT_NS = 2000000000ull;
constexpr int B_BYTES = BN * 128;       // 16 KB per part (hi, lo)
constexpr int STAGE_BYTES = 2 * B_BYTES;
constexpr int QOP_BYTES = 128 * 32;     // [128 rows][16] f16, two 8-column core-matrix groups
constexpr int QGRP_BYTES = 4 * QOP_BYTES;   // c_hi, c_lo, X_hi, X_lo of one super-block pair
constexpr int XCH_FLOATS = 16 * 64;     // SiLU exchange: 16 columns x 64 rows
constexpr uint32_t COL_Q = 256, COL_A = 384;
constexpr int RAW_BYTES = BM * 144;     // one super-block of 128 Q4_K rows, by TMA
constexpr size_t SMEM = 2 * QGRP_BYTES + XCH_FLOATS * 4 + 2 * RAW_BYTES +
                        (size_t)STAGES * STAGE_BYTES + 1024;
static_assert((2 * QGRP_BYTES + XCH_FLOATS * 4 + 2 * RAW_BYTES) % 1024 == 0, "stage alignment");

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
// Bounded wait: false (and *err set) after WAIT_NS, or soon after any thread
// of the grid has failed.  try_wait suspends the thread in hardware until the
// phase completes or a short time limit passes; the error word and the clock
// are polled only every 32 tries so that waiting warps leave the issue slots
// (and the memory pipe) to the warps that share their scheduler.
__device__ bool bar_wait(uint64_t* b, uint32_t parity, int* err, int code) {
    if (bar_try(b, parity)) return true;
    const uint64_t t0 = gtimer();
    for (uint32_t n = 1;; ++n) {
        if (bar_try(b, parity)) return true;
        if ((n & 31) == 0) {
            if (*(volatile int*)err) return false;
            if (gtimer() - t0 > WAIT_NS) {
                atomicCAS(err, 0, code);
                return false;
            }
        }
    }
}
__device__ __forceinline__ void fence_async_smem() {
    asm volatile("fence.proxy.async.shared::cta;" ::: "memory");
}
__device__ __forceinline__ void tma_2d(void* dst, const CUtensorMap* map, uint64_t* bar, int x, int y) {
    asm volatile(
        "cp.async.bulk.tensor.2d.shared::cluster.global.tile.mbarrier::complete_tx::bytes "
        "[%0], [%1, {%3, %4}], [%2];" ::"r"(su32(dst)),
        "l"(map), "r"(su32(bar)), "r"(x), "r"(y)
        : "memory");
}
__device__ __forceinline__ void bulk_copy(void* dst, const void* src, uint32_t bytes, uint64_t* bar) {
    asm volatile(
        "cp.async.bulk.shared::cluster.global.mbarrier::complete_tx::bytes [%0], [%1], %2, [%3];" ::"r"(
            su32(dst)),
        "l"(src), "r"(bytes), "r"(su32(bar))
        : "memory");
}
__device__ __forceinline__ void tc_fence_before() {
    asm volatile("tcgen05.fence::before_thread_sync;" ::: "memory");
}
__device__ __forceinline__ void tc_fence_after() {
    asm volatile("tcgen05.fence::after_thread_sync;" ::: "memory");
}
// K-major, SWIZZLE_128B: 8-row atoms of 128-byte rows, 1024 B apart.
__device__ __forceinline__ uint64_t desc_sw128(uint32_t saddr) {
    return (uint64_t)((saddr & 0x3FFFFu) >> 4) | (1ull << 16) | ((uint64_t)(1024 >> 4) << 32) |
           (1ull << 46) | (2ull << 61);
}
// K-major, no swizzle: 8x16-byte core matrices; 8-row groups 128 B apart,
// the two 8-column K groups 2048 B apart (tile of 128 rows x 16 columns).
__device__ __forceinline__ uint64_t desc_plain(uint32_t saddr) {
    return (uint64_t)((saddr & 0x3FFFFu) >> 4) | ((uint64_t)(2048 >> 4) << 16) |
           ((uint64_t)(128 >> 4) << 32) | (1ull << 46);
}
__device__ __forceinline__ void mma_f16(uint32_t d, uint64_t a, uint64_t b, uint32_t idesc,
                                        uint32_t acc) {
    asm volatile(
        "{\n\t.reg .pred p;\n\tsetp.ne.b32 p, %4, 0;\n\t"
        "tcgen05.mma.cta_group::1.kind::f16 [%0], %1, %2, %3, p;\n\t}\n" ::"r"(d),
        "l"(a), "l"(b), "r"(idesc), "r"(acc));
}
// D (+)= A * B with A in tensor memory (lane = row, K pairs per column).
__device__ __forceinline__ void mma_f16_ta(uint32_t d, uint32_t a_tmem, uint64_t b, uint32_t idesc,
                                           uint32_t acc) {
    asm volatile(
        "{\n\t.reg .pred p;\n\tsetp.ne.b32 p, %4, 0;\n\t"
        "tcgen05.mma.cta_group::1.kind::f16 [%0], [%1], %2, %3, p;\n\t}\n" ::"r"(d),
        "r"(a_tmem), "l"(b), "r"(idesc), "r"(acc));
}
__device__ __forceinline__ void tmem_st32(uint32_t taddr, const uint32_t (&r)[32]) {
    asm volatile(
        "tcgen05.st.sync.aligned.32x32b.x32.b32 [%0], "
        "{%1, %2, %3, %4, %5, %6, %7, %8, %9, %10, %11, %12, %13, %14, %15, %16, "
        "%17, %18, %19, %20, %21, %22, %23, %24, %25, %26, %27, %28, %29, %30, %31, %32};" ::"r"(taddr),
        "r"(r[0]), "r"(r[1]), "r"(r[2]), "r"(r[3]), "r"(r[4]), "r"(r[5]), "r"(r[6]), "r"(r[7]),
        "r"(r[8]), "r"(r[9]), "r"(r[10]), "r"(r[11]), "r"(r[12]), "r"(r[13]), "r"(r[14]), "r"(r[15]),
        "r"(r[16]), "r"(r[17]), "r"(r[18]), "r"(r[19]), "r"(r[20]), "r"(r[21]), "r"(r[22]), "r"(r[23]),
        "r"(r[24]), "r"(r[25]), "r"(r[26]), "r"(r[27]), "r"(r[28]), "r"(r[29]), "r"(r[30]), "r"(r[31])
        : "memory");
    asm volatile("tcgen05.wait::st.sync.aligned;" ::: "memory");
}
__device__ __forceinline__ void mma_commit(uint64_t* bar) {
    asm volatile("tcgen05.commit.cta_group::1.mbarrier::arrive::one.shared::cluster.b64 [%0];" ::"r"(
                     su32(bar))
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
__device__ __forceinline__ void drain_sync() {
    asm volatile("bar.sync 1, 128;" ::: "memory");
}

// 6-bit scale and min of sub-block j from the 12 packed bytes (GGML packing,
// util/quant.c:157-166): header words h.y..h.w hold bytes 0..11.
__device__ __forceinline__ uint32_t hbyte(uint4 h, int i) {
    const uint32_t w = i < 4 ? h.y : (i < 8 ? h.z : h.w);
    return (w >> ((i & 3) * 8)) & 0xffu;
}
__device__ __forceinline__ void scale_min(uint4 h, int j, uint32_t& sc, uint32_t& mn) {
    if (j < 4) {
        sc = hbyte(h, j) & 63u;
        mn = hbyte(h, j + 4) & 63u;
    } else {
        sc = (hbyte(h, j + 4) & 15u) | ((hbyte(h, j - 4) >> 6) << 4);
        mn = (hbyte(h, j + 4) >> 4) | ((hbyte(h, j) >> 6) << 4);
    }
}

// Four elements' (pairs (b0,b1), (b2,b3) of one nibble plane) sc*q as two
// half2 words: (1024 + q) * sc - 1024 * sc is q * sc exactly (<= 945) after
// the single rounding of the fused multiply-add.
__device__ __forceinline__ void nib4(uint32_t nibs, __half2 sc2, __half2 off2, uint32_t& w0,
                                     uint32_t& w1) {
    // bytes [n0, 0x64, n1, 0x64]: the f16 pair (1024 + n0, 1024 + n1)
    const uint32_t p0 = __byte_perm(nibs, 0x64646464u, 0x4140);
    const uint32_t p1 = __byte_perm(nibs, 0x64646464u, 0x4342);
    const __half2 h0 = __hfma2(*(const __half2*)&p0, sc2, off2);
    const __half2 h1 = __hfma2(*(const __half2*)&p1, sc2, off2);
    w0 = *(const uint32_t*)&h0;
    w1 = *(const uint32_t*)&h1;
}
// One sub-block (16 nibble bytes, Slate order: byte i -> elements i (low
// nibble) and i + 16 (high)) -> 4 chunks of 8 f16 (elements 8c..8c+7).
__device__ __forceinline__ void subblock_sc_q(uint4 q, uint32_t sc, uint4 (&chunk)[4]) {
    const __half hs = __ushort2half_rn((unsigned short)sc);
    const __half2 sc2 = __halves2half2(hs, hs);
    const __half ho = __float2half_rn(-1024.0f * (float)sc);
    const __half2 off2 = __halves2half2(ho, ho);
    const uint32_t w[4] = {q.x, q.y, q.z, q.w};
    uint32_t lo[8], hi[8];
#pragma unroll
    for (int i = 0; i < 4; ++i) {
        nib4(w[i] & 0x0f0f0f0fu, sc2, off2, lo[2 * i], lo[2 * i + 1]);
        nib4((w[i] >> 4) & 0x0f0f0f0fu, sc2, off2, hi[2 * i], hi[2 * i + 1]);
    }
    chunk[0] = make_uint4(lo[0], lo[1], lo[2], lo[3]);   // elements 0-7
    chunk[1] = make_uint4(lo[4], lo[5], lo[6], lo[7]);   // 8-15
    chunk[2] = make_uint4(hi[0], hi[1], hi[2], hi[3]);   // 16-23
    chunk[3] = make_uint4(hi[4], hi[5], hi[6], hi[7]);   // 24-31
}

// ---- stream-K schedule ----------------------------------------------------
// CTA c of C owns units [u0(c), u0(c+1)) of the U = tiles * nk (tile, K step)
// units, tile-major.
__device__ __forceinline__ long long u_begin(int c, int C, long long U) {
    return U * c / C;
}
// The CTA whose range holds unit u.
__device__ int owner_of(long long u, int C, long long U) {
    int c = (int)((u * C) / U);
    while (c > 0 && u_begin(c, C, U) > u) --c;
    while (c + 1 < C && u_begin(c + 1, C, U) <= u) ++c;
    return c;
}

// Walks one CTA's schedule super-block segment by super-block segment: tile t,
// K steps [ka, kb) of it in this CTA's range, super-block sb.
struct SbsIt {
    long long u, u1;
    int nk, t, ka, kb, sb;
    __device__ __forceinline__ void set() {
        t = (int)(u / nk);
        ka = (int)(u - (long long)t * nk);
        kb = (int)min((long long)nk, u1 - (long long)t * nk);
        sb = ka / 4;
    }
    __device__ __forceinline__ void start(long long u0_, long long u1_, int nk_) {
        u = u0_;
        u1 = u1_;
        nk = nk_;
        t = ka = kb = sb = 0;
        if (u < u1) set();
    }
    __device__ __forceinline__ bool valid() const { return u < u1; }
    __device__ __forceinline__ void next() {
        if (sb < (kb - 1) / 4) {
            ++sb;
            return;
        }
        u = (long long)t * nk + kb;
        if (u < u1) set();
    }
};

struct Args {
    const unsigned char* W;   // Q4_K rows [M_pad][K/256 * 144]
    const __half* xs_hi;      // [K/256][r_pad][8]
    const __half* xs_lo;
    float* Y;
    float* ws;                // [C][2][BN][BM] partial tiles
    int* cnt;                 // [tiles] arrival counters (zero between launches)
    int* err;
    int M, M_pad, K, n_rows, r_pad, ldy, epi, NT;
    int one_pass;             // 1: x enters as its f16 rounding only (the lo part is not read)
};

// Epilogue of one finished 128x128 tile held in the drain threads' registers
// (thread = weight row m of the tile, v[j] = column n0 + j).
__device__ __forceinline__ void tile_out(const Args& a, float (&v)[BN], int mt, int n0, int m,
                                         float* xch) {
    const int row = mt * BM + m;
    if (a.epi != SB_EPI_SILU) {
#pragma unroll
        for (int j = 0; j < BN; ++j) {
            const int n = n0 + j;
            if (n < a.n_rows && row < a.M) {
                float* y = a.Y + (size_t)n * a.ldy + row;
                *y = a.epi == SB_EPI_ADD ? *y + v[j] : v[j];
            }
        }
        return;
    }
    // rows 0-63 of the tile are gate units, 64-127 the matching up rows
    const int unit = mt * 64 + (m & 63);
#pragma unroll
    for (int c0 = 0; c0 < BN; c0 += 16) {
        if (m >= 64) {
#pragma unroll
            for (int i = 0; i < 16; ++i) xch[i * 64 + (m - 64)] = v[c0 + i];
        }
        drain_sync();
        if (m < 64) {
#pragma unroll
            for (int i = 0; i < 16; ++i) {
                const int n = n0 + c0 + i;
                const float g = v[c0 + i], u = xch[i * 64 + m];
                if (n < a.n_rows && unit < a.M / 2) a.Y[(size_t)n * a.ldy + unit] = g / (1.0f + expf(-g)) * u;
            }
        }
        drain_sync();
    }
}

__global__ void __launch_bounds__(NTHREADS, 1)
    q4k_gemm_kernel(const __grid_constant__ CUtensorMap xmap_hi,
                    const __grid_constant__ CUtensorMap xmap_lo,
                    const __grid_constant__ CUtensorMap wmap, const Args a) {
    extern __shared__ __align__(1024) unsigned char smem_raw[];
    // [Q operand groups x2 | SiLU exchange | B stages], 1024-aligned; the small
    // no-swizzle operands come first so that every descriptor-addressed byte
    // lies well inside the allocation
    unsigned char* qbuf = (unsigned char*)(((uintptr_t)smem_raw + 1023) & ~(uintptr_t)1023);
    float* xch = (float*)(qbuf + 2 * QGRP_BYTES);
    unsigned char* rawbuf = (unsigned char*)(xch + XCH_FLOATS);       // [2][128 rows][144 B]
    unsigned char* bst = rawbuf + 2 * RAW_BYTES;
    __shared__ uint64_t full[STAGES], empty[STAGES], acc_full[2], acc_empty[2], qa_full[2],
        qa_empty[2], q_full, q_empty, raw_full[2], raw_empty[2];
    __shared__ uint32_t tmem_slot;
    __shared__ int last_flag;

    const int tid = threadIdx.x, warp = tid >> 5, lane = tid & 31;
    const int C = gridDim.x, c = blockIdx.x;
    const int nk = a.K / BK;
    const int MT = a.M_pad / BM;
    const long long U = (long long)MT * a.NT * nk;
    const long long u0 = u_begin(c, C, U), u1 = u_begin(c + 1, C, U);
    const size_t row_bytes = (size_t)(a.K / 256) * 144;

    if (tid == 0) {
        // producer warps arrive once per warp (elected lane)
        for (int s = 0; s < STAGES; ++s) {
            bar_init(&full[s], NPROD / 32 + 1);
            bar_init(&empty[s], 1);
        }
        for (int p = 0; p < 2; ++p) {
            bar_init(&acc_full[p], 1);
            bar_init(&acc_empty[p], 4);
            bar_init(&qa_full[p], NPROD / 32 + 1);
            bar_init(&qa_empty[p], 1);
            bar_init(&raw_full[p], 1);
            bar_init(&raw_empty[p], NPROD / 32);
        }
        bar_init(&q_full, 1);
        bar_init(&q_empty, 4);
        asm volatile("fence.mbarrier_init.release.cluster;" ::: "memory");
    }
    if (warp == MMA_WARP) {
        asm volatile("tcgen05.alloc.cta_group::1.sync.aligned.shared::cta.b32 [%0], %1;" ::"r"(
                         su32(&tmem_slot)),
                     "r"(512));
        asm volatile("tcgen05.relinquish_alloc_permit.cta_group::1.sync.aligned;");
    }
    tc_fence_before();
    __syncthreads();
    tc_fence_after();
    const uint32_t tmem = tmem_slot;
    bool ok = true;

    if (warp < 4) {
        // ---------------- producers ----------------
        // Thread m owns weight row m: per K step it converts 64 Q4_K values to
        // f16(sc * q) and stores them into its TMEM lane (A stage); per super-
        // block it writes c_j = dmin * m_j as f16 hi / lo into the Q operand.
        // The super-block's 128 x 144 bytes arrive by TMA into a two-slot ring
        // ahead of use, so the producers only read shared memory.
        const int m = tid;
        const uint32_t lane_a = tmem + ((uint32_t)(warp * 32) << 16) + COL_A;
        long long it = 0, gi = 0, si = 0;
        SbsIt cur;
        cur.start(u0, u1, nk);
        const uint4 zero4 = make_uint4(0, 0, 0, 0);
        while (cur.valid() && ok) {
            uint4 raw[9];
            {
                const int r = (int)(si & 1);
                if (!__all_sync(0xffffffffu, bar_wait(&raw_full[r], (uint32_t)((si >> 1) & 1), a.err, 22))) {
                    ok = false;
                    break;
                }
                const uint4* src = (const uint4*)(rawbuf + r * RAW_BYTES + m * 144);
#pragma unroll
                for (int i = 0; i < 9; ++i) raw[i] = src[i];
                __syncwarp();
                if (lane == 0) bar_arrive(&raw_empty[r]);
                ++si;
            }
            const int sb = cur.sb;
            const int ks = max(cur.ka, 4 * sb), ke = min(cur.kb, 4 * sb + 4);
            const bool first = sb == cur.ka / 4, last = sb == (cur.kb - 1) / 4;
            const bool opens = first || !(sb & 1), closes = last || (sb & 1);
            const int g = (int)(gi & 1);
            unsigned char* qg = qbuf + g * QGRP_BYTES;
            const uint4 hdr = raw[0];
            if (opens) {
                if (gi >= 2 &&
                    !__all_sync(0xffffffffu, bar_wait(&qa_empty[g], (uint32_t)(((gi >> 1) - 1) & 1), a.err, 11))) {
                    ok = false;
                    break;
                }
                if (sb & 1) {                // the pair's first block is outside this segment
                    *(uint4*)(qg + m * 16) = zero4;
                    *(uint4*)(qg + QOP_BYTES + m * 16) = zero4;
                }
            }
            {
                // c_j = dmin * m_j (exact in f32) as f16 hi + lo; sub-blocks
                // outside this segment's K steps are zero
                const float dmin = __half2float(__ushort_as_half((unsigned short)(hdr.x >> 16)));
                uint32_t hw[4], lw[4];
#pragma unroll
                for (int q = 0; q < 4; ++q) {
                    uint32_t sc0, mn0, sc1, mn1;
                    scale_min(hdr, 2 * q, sc0, mn0);
                    scale_min(hdr, 2 * q + 1, sc1, mn1);
                    const int kstep = 4 * sb + q;        // sub-blocks 2q, 2q+1
                    const bool in = kstep >= ks && kstep < ke;
                    const float c0 = in ? dmin * (float)mn0 : 0.f, c1 = in ? dmin * (float)mn1 : 0.f;
                    const __half2 h = __floats2half2_rn(c0, c1);
                    const float2 back = __half22float2(h);
                    const __half2 l = __floats2half2_rn(c0 - back.x, c1 - back.y);
                    hw[q] = *(const uint32_t*)&h;
                    lw[q] = *(const uint32_t*)&l;
                }
                const uint32_t kg = (uint32_t)(sb & 1) * 2048u;
                *(uint4*)(qg + kg + m * 16) = make_uint4(hw[0], hw[1], hw[2], hw[3]);
                *(uint4*)(qg + QOP_BYTES + kg + m * 16) = make_uint4(lw[0], lw[1], lw[2], lw[3]);
            }
            if (closes) {
                if (!(sb & 1)) {             // the pair's second block is outside this segment
                    *(uint4*)(qg + 2048 + m * 16) = zero4;
                    *(uint4*)(qg + QOP_BYTES + 2048 + m * 16) = zero4;
                }
                fence_async_smem();
                __syncwarp();
                if (lane == 0) bar_arrive(&qa_full[g]);
                ++gi;
            }
#pragma unroll
            for (int kk = 0; kk < 4; ++kk) {
                const int k = 4 * sb + kk;
                if (k < ks || k >= ke || !ok) continue;
                const int s = (int)(it % STAGES);
                if (it >= STAGES &&
                    !__all_sync(0xffffffffu, bar_wait(&empty[s], (uint32_t)(((it / STAGES) - 1) & 1), a.err, 12))) {
                    ok = false;
                    continue;
                }
                uint32_t sc0, mn0, sc1, mn1;
                scale_min(hdr, 2 * kk, sc0, mn0);
                scale_min(hdr, 2 * kk + 1, sc1, mn1);
                uint32_t w[32];
                {
                    uint4 c4[4];
                    subblock_sc_q(raw[1 + 2 * kk], sc0, c4);
#pragma unroll
                    for (int i = 0; i < 4; ++i) {
                        w[4 * i] = c4[i].x;
                        w[4 * i + 1] = c4[i].y;
                        w[4 * i + 2] = c4[i].z;
                        w[4 * i + 3] = c4[i].w;
                    }
                    subblock_sc_q(raw[2 + 2 * kk], sc1, c4);
#pragma unroll
                    for (int i = 0; i < 4; ++i) {
                        w[16 + 4 * i] = c4[i].x;
                        w[16 + 4 * i + 1] = c4[i].y;
                        w[16 + 4 * i + 2] = c4[i].z;
                        w[16 + 4 * i + 3] = c4[i].w;
                    }
                }
                tmem_st32(lane_a + (uint32_t)(32 * s), w);
                tc_fence_before();
                __syncwarp();
                if (lane == 0) bar_arrive(&full[s]);
                ++it;
            }
            cur.next();
        }
    } else if (warp == TMA_WARP) {
        // ---------------- x tiles (TMA) and sub-block sums (bulk copies) ----------------
        if (lane == 0) {
            long long it = 0, gi = 0, go = 0, ri = 0;
            SbsIt cur;
            cur.start(u0, u1, nk);
            // weight bytes of super-block segment `ri` (tile row block, block sb)
            SbsIt rw = cur;
            auto raw_issue = [&]() {
                const int r = (int)(ri & 1);
                if (ri >= 2 && !bar_wait(&raw_empty[r], (uint32_t)(((ri >> 1) - 1) & 1), a.err, 23))
                    return false;
                bar_expect(&raw_full[r], (uint32_t)RAW_BYTES);
                tma_2d(rawbuf + r * RAW_BYTES, &wmap, &raw_full[r], rw.sb * 144, (rw.t / a.NT) * BM);
                ++ri;
                rw.next();
                return true;
            };
            if (rw.valid() && !raw_issue()) ok = false;
            while (cur.valid() && ok) {
                if (rw.valid() && !raw_issue()) {
                    ok = false;
                    break;
                }
                const int sb = cur.sb;
                const int ks = max(cur.ka, 4 * sb), ke = min(cur.kb, 4 * sb + 4);
                const bool first = sb == cur.ka / 4, last = sb == (cur.kb - 1) / 4;
                const bool opens = first || !(sb & 1), closes = last || (sb & 1);
                const int g = (int)(gi & 1);
                const int n0 = (cur.t % a.NT) * BN;
                if (opens) {
                    if (gi >= 2 &&
                        !bar_wait(&qa_empty[g], (uint32_t)(((gi >> 1) - 1) & 1), a.err, 13)) {
                        ok = false;
                        break;
                    }
                    unsigned char* qg = qbuf + g * QGRP_BYTES;
                    bar_expect(&qa_full[g], (uint32_t)(2 * QOP_BYTES));
                    const int sb0 = sb & ~1;        // X of both blocks of the pair (buffers padded)
#pragma unroll
                    for (int h = 0; h < 2; ++h) {
                        const size_t off = ((size_t)(sb0 + h) * a.r_pad + n0) * 8;
                        bulk_copy(qg + 2 * QOP_BYTES + h * 2048, a.xs_hi + off, BN * 16, &qa_full[g]);
                        bulk_copy(qg + 3 * QOP_BYTES + h * 2048, a.xs_lo + off, BN * 16, &qa_full[g]);
                    }
                    ++go;
                }
                if (closes) ++gi;
                for (int k = ks; k < ke; ++k, ++it) {
                    const int s = (int)(it % STAGES);
                    if (it >= STAGES &&
                        !bar_wait(&empty[s], (uint32_t)(((it / STAGES) - 1) & 1), a.err, 14)) {
                        ok = false;
                        break;
                    }
                    unsigned char* st = bst + (size_t)s * STAGE_BYTES;
                    bar_expect(&full[s], (uint32_t)((a.one_pass ? 1 : 2) * B_BYTES));
                    tma_2d(st, &xmap_hi, &full[s], k * BK, n0);
                    if (!a.one_pass) tma_2d(st + B_BYTES, &xmap_lo, &full[s], k * BK, n0);
                }
                cur.next();
            }
            // no copy may still be in flight when the CTA exits
            for (long long i = it - STAGES > 0 ? it - STAGES : 0; i < it; ++i)
                bar_wait(&full[i % STAGES], (uint32_t)((i / STAGES) & 1), a.err, 15);
            for (long long i = go - 2 > 0 ? go - 2 : 0; i < go; ++i)
                bar_wait(&qa_full[i & 1], (uint32_t)((i >> 1) & 1), a.err, 15);
            for (long long i = ri - 2 > 0 ? ri - 2 : 0; i < ri; ++i)
                bar_wait(&raw_full[i & 1], (uint32_t)((i >> 1) & 1), a.err, 15);
        }
    } else if (warp == MMA_WARP) {
        // ---------------- MMA issue ----------------
        if (lane == 0) {
            const uint32_t idesc = (1u << 4) | ((uint32_t)(BN >> 3) << 17) | ((uint32_t)(BM >> 4) << 24);
            long long it = 0, si = 0, gi = 0, seg = 0;
            bool q_fresh = true;                      // next Q MMA starts a new accumulation
            SbsIt cur;
            cur.start(u0, u1, nk);
            while (cur.valid() && ok) {
                const int sb = cur.sb;
                const int ks = max(cur.ka, 4 * sb), ke = min(cur.kb, 4 * sb + 4);
                const bool first = sb == cur.ka / 4, last = sb == (cur.kb - 1) / 4;
                const bool closes = last || (sb & 1);
                const int p = (int)(si & 1), g = (int)(gi & 1);
                if (first) q_fresh = true;
                if (si >= 2 &&
                    !bar_wait(&acc_empty[p], (uint32_t)(((si >> 1) - 1) & 1), a.err, 16)) {
                    ok = false;
                    break;
                }
                tc_fence_after();
                const uint32_t p1 = tmem + (uint32_t)(p * 128);
                for (int k = ks; k < ke; ++k, ++it) {
                    const int s = (int)(it % STAGES);
                    if (!bar_wait(&full[s], (uint32_t)((it / STAGES) & 1), a.err, 17)) {
                        ok = false;
                        break;
                    }
                    tc_fence_after();
                    const uint32_t bh = su32(bst + (size_t)s * STAGE_BYTES), bl = bh + B_BYTES;
                    const uint32_t at = tmem + COL_A + (uint32_t)(32 * s);
#pragma unroll
                    for (int kk = 0; kk < BK / 16; ++kk) {
                        mma_f16_ta(p1, at + 8u * kk, desc_sw128(bh + 32u * kk), idesc,
                                   (k > ks || kk > 0) ? 1u : 0u);
                        if (!a.one_pass) mma_f16_ta(p1, at + 8u * kk, desc_sw128(bl + 32u * kk), idesc, 1u);
                    }
                    mma_commit(&empty[s]);
                }
                if (!ok) break;
                if (closes) {
                    if (!bar_wait(&qa_full[g], (uint32_t)((gi >> 1) & 1), a.err, 18) ||
                        (q_fresh && seg > 0 &&
                         !bar_wait(&q_empty, (uint32_t)((seg - 1) & 1), a.err, 20))) {
                        ok = false;
                        break;
                    }
                    tc_fence_after();
                    const uint32_t qg = su32(qbuf + g * QGRP_BYTES);
                    const uint32_t cq = tmem + COL_Q;
                    mma_f16(cq, desc_plain(qg), desc_plain(qg + 2 * QOP_BYTES), idesc, q_fresh ? 0u : 1u);
                    mma_f16(cq, desc_plain(qg), desc_plain(qg + 3 * QOP_BYTES), idesc, 1u);
                    mma_f16(cq, desc_plain(qg + QOP_BYTES), desc_plain(qg + 2 * QOP_BYTES), idesc, 1u);
                    q_fresh = false;
                    mma_commit(&qa_empty[g]);
                    ++gi;
                    if (last) {
                        mma_commit(&q_full);
                        ++seg;
                    }
                }
                mma_commit(&acc_full[p]);
                ++si;
                cur.next();
            }
        }
    } else {
        // ---------------- drain: acc += d * P1 per block, acc -= Q, epilogue ----------------
        // The four drain warps meet at named barriers (epilogue exchange, stream-K
        // fixup), so they never leave the schedule early: after a failed wait
        // they skip the TMEM reads (later waits fail at once) and still take
        // every barrier; the results are then invalid and *err says so.
        const int q = warp & 3, m = q * 32 + lane;
        const uint32_t lane_base = tmem + ((uint32_t)(q * 32) << 16);
        float acc[BN];
#pragma unroll
        for (int j = 0; j < BN; ++j) acc[j] = 0.f;
        long long si = 0, seg = 0;
        SbsIt cur;
        cur.start(u0, u1, nk);
        while (cur.valid()) {
            const int t = cur.t, ka = cur.ka, kb = cur.kb, sb = cur.sb;
            const bool last = sb == (kb - 1) / 4;
            const int mt = t / a.NT, n0 = (t % a.NT) * BN;
            const int p = (int)(si & 1);
            const uint32_t dd =
                __ldg((const uint32_t*)(a.W + (size_t)(mt * BM + m) * row_bytes + (size_t)sb * 144));
            const float d = __half2float(__ushort_as_half((unsigned short)(dd & 0xffffu)));
            bool have = ok && bar_wait(&acc_full[p], (uint32_t)((si >> 1) & 1), a.err, 19);
            have = __all_sync(0xffffffffu, have);
            if (have) {
                tc_fence_after();
#pragma unroll
                for (int c0 = 0; c0 < BN; c0 += 16) {
                    float v[16];
                    tmem_ld16(lane_base + (uint32_t)(p * 128 + c0), v);
#pragma unroll
                    for (int i = 0; i < 16; ++i) acc[c0 + i] = fmaf(d, v[i], acc[c0 + i]);
                }
            } else {
                ok = false;
            }
            tc_fence_before();
            __syncwarp();
            if (lane == 0) bar_arrive(&acc_empty[p]);
            ++si;
            if (last) {
                have = ok && bar_wait(&q_full, (uint32_t)(seg & 1), a.err, 21);
                have = __all_sync(0xffffffffu, have);
                if (have) {
                    tc_fence_after();
#pragma unroll
                    for (int c0 = 0; c0 < BN; c0 += 16) {
                        float v[16];
                        tmem_ld16(lane_base + COL_Q + (uint32_t)c0, v);
#pragma unroll
                        for (int i = 0; i < 16; ++i) acc[c0 + i] -= v[i];
                    }
                } else {
                    ok = false;
                }
                tc_fence_before();
                __syncwarp();
                if (lane == 0) bar_arrive(&q_empty);
                ++seg;
                // segment [ka, kb) of tile t is complete in acc
                if (ka == 0 && kb == nk) {
                    tile_out(a, acc, mt, n0, m, xch);
                } else {
                    const long long tu0 = (long long)t * nk;
                    const int slot = u0 >= tu0 ? 0 : 1;    // this CTA's first segment or its last
                    float* wsp = a.ws + ((size_t)c * 2 + slot) * (BN * BM);
#pragma unroll
                    for (int j = 0; j < BN; ++j) wsp[(size_t)j * BM + m] = acc[j];
                    __threadfence();
                    drain_sync();
                    const int cf = owner_of(tu0, C, U), cl = owner_of(tu0 + nk - 1, C, U);
                    if (warp == DRAIN_WARP0 && lane == 0) {
                        const int prev = atomicAdd(&a.cnt[t], 1);
                        last_flag = prev == cl - cf;
                    }
                    drain_sync();
                    if (last_flag) {
                        __threadfence();
#pragma unroll
                        for (int j = 0; j < BN; ++j) acc[j] = 0.f;
                        for (int cc = cf; cc <= cl; ++cc) {
                            const int sl = u_begin(cc, C, U) >= tu0 ? 0 : 1;
                            const float* src = a.ws + ((size_t)cc * 2 + sl) * (BN * BM);
#pragma unroll
                            for (int j = 0; j < BN; ++j) acc[j] += __ldcg(src + (size_t)j * BM + m);
                        }
                        tile_out(a, acc, mt, n0, m, xch);
                        if (warp == DRAIN_WARP0 && lane == 0) a.cnt[t] = 0;
                    }
                    drain_sync();
                }
#pragma unroll
                for (int j = 0; j < BN; ++j) acc[j] = 0.f;
            }
            cur.next();
        }
    }

    tc_fence_before();
    __syncthreads();
    if (warp == MMA_WARP) {
        tc_fence_after();
        asm volatile("tcgen05.dealloc.cta_group::1.sync.aligned.b32 %0, %1;" ::"r"(tmem), "r"(512));
    }
}

// ============================================================================
// Two-SM version (cta_group::2): a cluster of 2 CTAs computes a tile of 256
// weight rows x 128 activation rows.  CTA r holds weight rows [128 r, 128 r +
// 128) of the tile in its TMEM lanes (A, P1, Q) and activation rows [64 r, 64 r
// + 64) of the tile in its shared memory; the leader CTA (r = 0) issues MMAs of
// M = 256 that read both CTAs' operands, so each SM brings in half of the
// activation bytes per multiply-add of the one-SM kernel.  Completions are
// committed to both CTAs' barriers (tcgen05.commit multicast); producers of
// both CTAs arrive on the leader's barriers; the x tiles of both CTAs land on
// the leader's barrier (2-SM TMA form, no multicast).
constexpr int BN2 = 64;                    // activation rows per CTA (of 128 per pair)
constexpr int STAGES2 = 8;                 // x stages in shared memory
constexpr int B2_BYTES = BN2 * 128;        // 8 KB per part
constexpr int STAGE2_BYTES = 2 * B2_BYTES;
constexpr int QA2_BYTES = 128 * 32;        // c hi or lo: [128 rows][16]
constexpr int QB2_BYTES = BN2 * 32;        // X hi or lo: [64 rows][16]
constexpr int QGRP2_BYTES = 2 * QA2_BYTES + 2 * QB2_BYTES;
// (+ 8 KB of slack after the last stage: every operand read stays inside the
// allocation even if a descriptor spanned a whole 128-row tile)
constexpr size_t SMEM2 = 2 * QGRP2_BYTES + XCH_FLOATS * 4 + 2 * RAW_BYTES +
                         (size_t)STAGES2 * STAGE2_BYTES + 1024 + 8192;
static_assert((2 * QGRP2_BYTES + XCH_FLOATS * 4 + 2 * RAW_BYTES) % 1024 == 0, "stage alignment");

__device__ __forceinline__ uint32_t cluster_rank() {
    uint32_t r;
    asm volatile("mov.u32 %0, %%cluster_ctarank;" : "=r"(r));
    return r;
}
__device__ __forceinline__ void cluster_sync() {
    asm volatile("barrier.cluster.arrive.release.aligned;\n\tbarrier.cluster.wait.acquire.aligned;" ::: "memory");
}
// arrive on the barrier at the same offset in CTA 0 of the cluster
__device__ __forceinline__ void bar_arrive_leader(uint64_t* b) {
    asm volatile(
        "{\n\t.reg .b32 ra;\n\tmapa.shared::cluster.u32 ra, %0, 0;\n\t"
        "mbarrier.arrive.release.cluster.shared::cluster.b64 _, [ra];\n\t}" ::"r"(su32(b))
        : "memory");
}
__device__ __forceinline__ bool bar_try_cl(uint64_t* b, uint32_t parity) {
    uint32_t ok;
    asm volatile(
        "{\n\t.reg .pred p;\n\tmbarrier.try_wait.parity.acquire.cluster.shared::cta.b64 p, [%1], %2;\n\t"
        "selp.u32 %0, 1, 0, p;\n\t}\n"
        : "=r"(ok)
        : "r"(su32(b)), "r"(parity)
        : "memory");
    return ok != 0;
}
// bounded wait with cluster-scope acquire (barriers that receive remote arrivals)
__device__ bool bar_wait_cl(uint64_t* b, uint32_t parity, int* err, int code) {
    if (bar_try_cl(b, parity)) return true;
    const uint64_t t0 = gtimer();
    for (uint32_t n = 1;; ++n) {
        if (bar_try_cl(b, parity)) return true;
        if ((n & 31) == 0) {
            if (*(volatile int*)err) return false;
            if (gtimer() - t0 > WAIT_NS) {
                atomicCAS(err, 0, code);
                return false;
            }
        }
    }
}
// TMA tile load into this CTA's shared memory, completion counted on the
// leader CTA's barrier (2-SM form; no multicast)
__device__ __forceinline__ void tma_2d_2sm(void* dst, const CUtensorMap* map, uint64_t* bar, int x, int y) {
    const uint32_t b = su32(bar) & 0xFEFFFFFFu;
    asm volatile(
        "cp.async.bulk.tensor.2d.cta_group::2.shared::cluster.global.mbarrier::complete_tx::bytes "
        "[%0], [%1, {%3, %4}], [%2];" ::"r"(su32(dst)),
        "l"(map), "r"(b), "r"(x), "r"(y)
        : "memory");
}
__device__ __forceinline__ void mma2_ta(uint32_t d, uint32_t a_tmem, uint64_t b, uint32_t idesc,
                                        uint32_t acc) {
    asm volatile(
        "{\n\t.reg .pred p;\n\tsetp.ne.b32 p, %4, 0;\n\t"
        "tcgen05.mma.cta_group::2.kind::f16 [%0], [%1], %2, %3, p;\n\t}\n" ::"r"(d),
        "r"(a_tmem), "l"(b), "r"(idesc), "r"(acc));
}
__device__ __forceinline__ void mma2_ss(uint32_t d, uint64_t a, uint64_t b, uint32_t idesc,
                                        uint32_t acc) {
    asm volatile(
        "{\n\t.reg .pred p;\n\tsetp.ne.b32 p, %4, 0;\n\t"
        "tcgen05.mma.cta_group::2.kind::f16 [%0], %1, %2, %3, p;\n\t}\n" ::"r"(d),
        "l"(a), "l"(b), "r"(idesc), "r"(acc));
}
// commit to the barrier at this offset in both CTAs of the pair
__device__ __forceinline__ void commit2(uint64_t* bar) {
    asm volatile(
        "{\n\t.reg .b16 m;\n\tmov.b16 m, 3;\n\t"
        "tcgen05.commit.cta_group::2.mbarrier::arrive::one.shared::cluster.multicast::cluster.b64 [%0], m;\n\t}" ::"r"(
            su32(bar))
        : "memory");
}
// K-major, no swizzle, two 8-column K groups `lbo` bytes apart, 8-row groups 128 B apart
__device__ __forceinline__ uint64_t desc_plain_lbo(uint32_t saddr, uint32_t lbo) {
    return (uint64_t)((saddr & 0x3FFFFu) >> 4) | ((uint64_t)(lbo >> 4) << 16) |
           ((uint64_t)(128 >> 4) << 32) | (1ull << 46);
}

__global__ void __launch_bounds__(NTHREADS, 1)
    q4k_gemm2_kernel(const __grid_constant__ CUtensorMap xmap_hi,
                     const __grid_constant__ CUtensorMap xmap_lo,
                     const __grid_constant__ CUtensorMap xsmap_hi,
                     const __grid_constant__ CUtensorMap xsmap_lo,
                     const __grid_constant__ CUtensorMap wmap, const Args a) {
    extern __shared__ __align__(1024) unsigned char smem_raw[];
    // [Q groups x2 (c hi, c lo, X hi, X lo) | SiLU exchange | raw x2 | x stages]
    unsigned char* qbuf = (unsigned char*)(((uintptr_t)smem_raw + 1023) & ~(uintptr_t)1023);
    float* xch = (float*)(qbuf + 2 * QGRP2_BYTES);
    unsigned char* rawbuf = (unsigned char*)(xch + XCH_FLOATS);
    unsigned char* bst = rawbuf + 2 * RAW_BYTES;
    // full / qa_full / acc_empty / q_empty are used in the leader only (both
    // CTAs arrive there); the others are per CTA (multicast commits, local TMA)
    __shared__ uint64_t full[STAGES2], empty[STAGES2], acc_full[2], acc_empty[2], qa_full[2],
        qa_empty[2], q_full, q_empty, raw_full[2], raw_empty[2];
    __shared__ uint32_t tmem_slot;
    __shared__ int last_flag;

    const int tid = threadIdx.x, warp = tid >> 5, lane = tid & 31;
    const uint32_t rank = cluster_rank();
    const bool leader = rank == 0;
    const int C = gridDim.x >> 1, c = blockIdx.x >> 1;      // clusters, this cluster
    const int nk = a.K / BK;
    const int MT = a.M_pad / (2 * BM);
    const long long U = (long long)MT * a.NT * nk;
    const long long u0 = u_begin(c, C, U), u1 = u_begin(c + 1, C, U);
    const size_t row_bytes = (size_t)(a.K / 256) * 144;

    if (tid == 0) {
        // producer warps of both CTAs arrive once per warp (elected lane)
        for (int s = 0; s < STAGES2; ++s) {
            bar_init(&full[s], 2 * (NPROD / 32) + 1);
            bar_init(&empty[s], 1);
        }
        for (int p = 0; p < 2; ++p) {
            bar_init(&acc_full[p], 1);
            bar_init(&acc_empty[p], 8);
            bar_init(&qa_full[p], 2 * (NPROD / 32) + 1);
            bar_init(&qa_empty[p], 1);
            bar_init(&raw_full[p], 1);
            bar_init(&raw_empty[p], NPROD / 32);
        }
        bar_init(&q_full, 1);
        bar_init(&q_empty, 8);
        asm volatile("fence.mbarrier_init.release.cluster;" ::: "memory");
    }
    if (warp == MMA_WARP) {
        asm volatile("tcgen05.alloc.cta_group::2.sync.aligned.shared::cta.b32 [%0], %1;" ::"r"(
                         su32(&tmem_slot)),
                     "r"(512));
        asm volatile("tcgen05.relinquish_alloc_permit.cta_group::2.sync.aligned;");
    }
    tc_fence_before();
    cluster_sync();                 // barriers of both CTAs initialised, TMEM allocated
    tc_fence_after();
    const uint32_t tmem = tmem_slot;
    bool ok = true;

    if (warp < 4) {
        // ---------------- producers (both CTAs): own 128 weight rows ----------------
        const int m = tid;
        const uint32_t lane_a = tmem + ((uint32_t)(warp * 32) << 16) + COL_A;
        long long it = 0, gi = 0, si = 0;
        SbsIt cur;
        cur.start(u0, u1, nk);
        const uint4 zero4 = make_uint4(0, 0, 0, 0);
        while (cur.valid() && ok) {
            uint4 raw[9];
            {
                const int r = (int)(si & 1);
                if (!__all_sync(0xffffffffu, bar_wait(&raw_full[r], (uint32_t)((si >> 1) & 1), a.err, 22))) {
                    ok = false;
                    break;
                }
                const uint4* src = (const uint4*)(rawbuf + r * RAW_BYTES + m * 144);
#pragma unroll
                for (int i = 0; i < 9; ++i) raw[i] = src[i];
                __syncwarp();
                if (lane == 0) bar_arrive(&raw_empty[r]);
                ++si;
            }
            const int sb = cur.sb;
            const int ks = max(cur.ka, 4 * sb), ke = min(cur.kb, 4 * sb + 4);
            const bool first = sb == cur.ka / 4, last = sb == (cur.kb - 1) / 4;
            const bool opens = first || !(sb & 1), closes = last || (sb & 1);
            const int g = (int)(gi & 1);
            unsigned char* qg = qbuf + g * QGRP2_BYTES;
            const uint4 hdr = raw[0];
            if (opens) {
                if (gi >= 2 &&
                    !__all_sync(0xffffffffu, bar_wait_cl(&qa_empty[g], (uint32_t)(((gi >> 1) - 1) & 1), a.err, 11))) {
                    ok = false;
                    break;
                }
                if (sb & 1) {
                    *(uint4*)(qg + m * 16) = zero4;
                    *(uint4*)(qg + QA2_BYTES + m * 16) = zero4;
                }
            }
            {
                const float dmin = __half2float(__ushort_as_half((unsigned short)(hdr.x >> 16)));
                uint32_t hw[4], lw[4];
#pragma unroll
                for (int q = 0; q < 4; ++q) {
                    uint32_t sc0, mn0, sc1, mn1;
                    scale_min(hdr, 2 * q, sc0, mn0);
                    scale_min(hdr, 2 * q + 1, sc1, mn1);
                    const int kstep = 4 * sb + q;
                    const bool in = kstep >= ks && kstep < ke;
                    const float c0 = in ? dmin * (float)mn0 : 0.f, c1 = in ? dmin * (float)mn1 : 0.f;
                    const __half2 h = __floats2half2_rn(c0, c1);
                    const float2 back = __half22float2(h);
                    const __half2 l = __floats2half2_rn(c0 - back.x, c1 - back.y);
                    hw[q] = *(const uint32_t*)&h;
                    lw[q] = *(const uint32_t*)&l;
                }
                const uint32_t kg = (uint32_t)(sb & 1) * 2048u;
                *(uint4*)(qg + kg + m * 16) = make_uint4(hw[0], hw[1], hw[2], hw[3]);
                *(uint4*)(qg + QA2_BYTES + kg + m * 16) = make_uint4(lw[0], lw[1], lw[2], lw[3]);
            }
            if (closes) {
                if (!(sb & 1)) {
                    *(uint4*)(qg + 2048 + m * 16) = zero4;
                    *(uint4*)(qg + QA2_BYTES + 2048 + m * 16) = zero4;
                }
                fence_async_smem();
                __syncwarp();
                if (lane == 0) bar_arrive_leader(&qa_full[g]);
                ++gi;
            }
#pragma unroll
            for (int kk = 0; kk < 4; ++kk) {
                const int k = 4 * sb + kk;
                if (k < ks || k >= ke || !ok) continue;
                const int s = (int)(it % STAGES2);
                // The A ring has STAGES (4) TMEM slots, the x ring STAGES2 (8)
                // stages: slot it % 4 is free once the MMAs of K step it - 4
                // have completed, which empty[(it - 4) % 8] reports.
                const int sa = (int)(it % STAGES);
                if (it >= STAGES) {
                    const long long j = it - STAGES;
                    if (!__all_sync(0xffffffffu, bar_wait_cl(&empty[j % STAGES2], (uint32_t)((j / STAGES2) & 1), a.err, 12))) {
                        ok = false;
                        continue;
                    }
                }
                uint32_t sc0, mn0, sc1, mn1;
                scale_min(hdr, 2 * kk, sc0, mn0);
                scale_min(hdr, 2 * kk + 1, sc1, mn1);
                uint32_t w[32];
                {
                    uint4 c4[4];
                    subblock_sc_q(raw[1 + 2 * kk], sc0, c4);
#pragma unroll
                    for (int i = 0; i < 4; ++i) {
                        w[4 * i] = c4[i].x;
                        w[4 * i + 1] = c4[i].y;
                        w[4 * i + 2] = c4[i].z;
                        w[4 * i + 3] = c4[i].w;
                    }
                    subblock_sc_q(raw[2 + 2 * kk], sc1, c4);
#pragma unroll
                    for (int i = 0; i < 4; ++i) {
                        w[16 + 4 * i] = c4[i].x;
                        w[16 + 4 * i + 1] = c4[i].y;
                        w[16 + 4 * i + 2] = c4[i].z;
                        w[16 + 4 * i + 3] = c4[i].w;
                    }
                }
                tmem_st32(lane_a + (uint32_t)(32 * sa), w);
                tc_fence_before();
                __syncwarp();
                if (lane == 0) bar_arrive_leader(&full[s]);
                ++it;
            }
            cur.next();
        }
    } else if (warp == TMA_WARP) {
        // ---------------- x halves, sub-block sums (both CTAs), raw weights ----------------
        if (lane == 0) {
            long long it = 0, gi = 0, go = 0, ri = 0;
            SbsIt cur;
            cur.start(u0, u1, nk);
            SbsIt rw = cur;
            const int wrow0 = (int)rank * BM;
            auto raw_issue = [&]() {
                const int r = (int)(ri & 1);
                if (ri >= 2 && !bar_wait(&raw_empty[r], (uint32_t)(((ri >> 1) - 1) & 1), a.err, 23))
                    return false;
                bar_expect(&raw_full[r], (uint32_t)RAW_BYTES);
                tma_2d(rawbuf + r * RAW_BYTES, &wmap, &raw_full[r], rw.sb * 144,
                       (rw.t / a.NT) * 2 * BM + wrow0);
                ++ri;
                rw.next();
                return true;
            };
            if (rw.valid() && !raw_issue()) ok = false;
            while (cur.valid() && ok) {
                if (rw.valid() && !raw_issue()) {
                    ok = false;
                    break;
                }
                const int sb = cur.sb;
                const int ks = max(cur.ka, 4 * sb), ke = min(cur.kb, 4 * sb + 4);
                const bool first = sb == cur.ka / 4, last = sb == (cur.kb - 1) / 4;
                const bool opens = first || !(sb & 1), closes = last || (sb & 1);
                const int g = (int)(gi & 1);
                const int n0 = (cur.t % a.NT) * (2 * BN2) + (int)rank * BN2;   // this CTA's x rows
                if (opens) {
                    if (gi >= 2 &&
                        !bar_wait_cl(&qa_empty[g], (uint32_t)(((gi >> 1) - 1) & 1), a.err, 13)) {
                        ok = false;
                        break;
                    }
                    unsigned char* qg = qbuf + g * QGRP2_BYTES + 2 * QA2_BYTES;
                    if (leader) bar_expect(&qa_full[g], (uint32_t)(2 * 2 * QB2_BYTES));
                    const int sb0 = sb & ~1;
#pragma unroll
                    for (int h = 0; h < 2; ++h) {
                        const int y = (sb0 + h) * a.r_pad + n0;
                        tma_2d_2sm(qg + h * (QB2_BYTES / 2), &xsmap_hi, &qa_full[g], 0, y);
                        tma_2d_2sm(qg + QB2_BYTES + h * (QB2_BYTES / 2), &xsmap_lo, &qa_full[g], 0, y);
                    }
                    ++go;
                }
                if (closes) ++gi;
                for (int k = ks; k < ke; ++k, ++it) {
                    const int s = (int)(it % STAGES2);
                    if (it >= STAGES2 &&
                        !bar_wait_cl(&empty[s], (uint32_t)(((it / STAGES2) - 1) & 1), a.err, 14)) {
                        ok = false;
                        break;
                    }
                    unsigned char* st = bst + (size_t)s * STAGE2_BYTES;
                    if (leader) bar_expect(&full[s], (uint32_t)(a.one_pass ? 2 * B2_BYTES : 2 * STAGE2_BYTES));
                    tma_2d_2sm(st, &xmap_hi, &full[s], k * BK, n0);
                    if (!a.one_pass) tma_2d_2sm(st + B2_BYTES, &xmap_lo, &full[s], k * BK, n0);
                }
                cur.next();
            }
            // local copies must land before the CTA exits (the x halves and sums
            // complete on the leader's barriers, which the leader's MMA waits for)
            for (long long i = ri - 2 > 0 ? ri - 2 : 0; i < ri; ++i)
                bar_wait(&raw_full[i & 1], (uint32_t)((i >> 1) & 1), a.err, 15);
            (void)go;
        }
    } else if (warp == MMA_WARP) {
        // ---------------- MMA issue (leader only) ----------------
        if (lane == 0 && leader) {
            const uint32_t idesc = (1u << 4) | ((uint32_t)((2 * BN2) >> 3) << 17) |
                                   ((uint32_t)((2 * BM) >> 4) << 24);
            long long it = 0, si = 0, gi = 0, seg = 0;
            bool q_fresh = true;
            SbsIt cur;
            cur.start(u0, u1, nk);
            while (cur.valid() && ok) {
                const int sb = cur.sb;
                const int ks = max(cur.ka, 4 * sb), ke = min(cur.kb, 4 * sb + 4);
                const bool first = sb == cur.ka / 4, last = sb == (cur.kb - 1) / 4;
                const bool closes = last || (sb & 1);
                const int p = (int)(si & 1), g = (int)(gi & 1);
                if (first) q_fresh = true;
                if (si >= 2 &&
                    !bar_wait_cl(&acc_empty[p], (uint32_t)(((si >> 1) - 1) & 1), a.err, 16)) {
                    ok = false;
                    break;
                }
                tc_fence_after();
                const uint32_t p1 = tmem + (uint32_t)(p * 128);
                for (int k = ks; k < ke; ++k, ++it) {
                    const int s = (int)(it % STAGES2), sa = (int)(it % STAGES);
                    if (!bar_wait_cl(&full[s], (uint32_t)((it / STAGES2) & 1), a.err, 17)) {
                        ok = false;
                        break;
                    }
                    tc_fence_after();
                    const uint32_t bh = su32(bst + (size_t)s * STAGE2_BYTES), bl = bh + B2_BYTES;
                    const uint32_t at = tmem + COL_A + (uint32_t)(32 * sa);
#pragma unroll
                    for (int kk = 0; kk < BK / 16; ++kk) {
                        mma2_ta(p1, at + 8u * kk, desc_sw128(bh + 32u * kk), idesc,
                                (k > ks || kk > 0) ? 1u : 0u);
                        if (!a.one_pass) mma2_ta(p1, at + 8u * kk, desc_sw128(bl + 32u * kk), idesc, 1u);
                    }
                    commit2(&empty[s]);
                }
                if (!ok) break;
                if (closes) {
                    if (!bar_wait_cl(&qa_full[g], (uint32_t)((gi >> 1) & 1), a.err, 18) ||
                        (q_fresh && seg > 0 &&
                         !bar_wait_cl(&q_empty, (uint32_t)((seg - 1) & 1), a.err, 20))) {
                        ok = false;
                        break;
                    }
                    tc_fence_after();
                    const uint32_t qa = su32(qbuf + g * QGRP2_BYTES);
                    const uint32_t qb = qa + 2 * QA2_BYTES;
                    const uint32_t cq = tmem + COL_Q;
                    mma2_ss(cq, desc_plain_lbo(qa, 2048), desc_plain_lbo(qb, QB2_BYTES / 2), idesc,
                            q_fresh ? 0u : 1u);
                    mma2_ss(cq, desc_plain_lbo(qa, 2048), desc_plain_lbo(qb + QB2_BYTES, QB2_BYTES / 2),
                            idesc, 1u);
                    mma2_ss(cq, desc_plain_lbo(qa + QA2_BYTES, 2048), desc_plain_lbo(qb, QB2_BYTES / 2),
                            idesc, 1u);
                    q_fresh = false;
                    commit2(&qa_empty[g]);
                    ++gi;
                    if (last) {
                        commit2(&q_full);
                        ++seg;
                    }
                }
                commit2(&acc_full[p]);
                ++si;
                cur.next();
            }
        }
    } else {
        // ---------------- drain (both CTAs): own 128 rows x 128 columns ----------------
        const int q = warp & 3, m = q * 32 + lane;
        const uint32_t lane_base = tmem + ((uint32_t)(q * 32) << 16);
        const int mrow0 = (int)rank * BM;                 // this CTA's rows within the pair tile
        float acc[BN];
#pragma unroll
        for (int j = 0; j < BN; ++j) acc[j] = 0.f;
        long long si = 0, seg = 0;
        SbsIt cur;
        cur.start(u0, u1, nk);
        while (cur.valid()) {
            const int t = cur.t, ka = cur.ka, kb = cur.kb, sb = cur.sb;
            const bool last = sb == (kb - 1) / 4;
            const int mt = t / a.NT, n0 = (t % a.NT) * BN;
            const int p = (int)(si & 1);
            const int grow = mt * 2 * BM + mrow0 + m;     // global weight row
            const uint32_t dd = __ldg((const uint32_t*)(a.W + (size_t)grow * row_bytes + (size_t)sb * 144));
            const float d = __half2float(__ushort_as_half((unsigned short)(dd & 0xffffu)));
            bool have = ok && bar_wait_cl(&acc_full[p], (uint32_t)((si >> 1) & 1), a.err, 19);
            have = __all_sync(0xffffffffu, have);
            if (have) {
                tc_fence_after();
#pragma unroll
                for (int c0 = 0; c0 < BN; c0 += 16) {
                    float v[16];
                    tmem_ld16(lane_base + (uint32_t)(p * 128 + c0), v);
#pragma unroll
                    for (int i = 0; i < 16; ++i) acc[c0 + i] = fmaf(d, v[i], acc[c0 + i]);
                }
            } else {
                ok = false;
            }
            tc_fence_before();
            __syncwarp();
            if (lane == 0) bar_arrive_leader(&acc_empty[p]);
            ++si;
            if (last) {
                have = ok && bar_wait_cl(&q_full, (uint32_t)(seg & 1), a.err, 21);
                have = __all_sync(0xffffffffu, have);
                if (have) {
                    tc_fence_after();
#pragma unroll
                    for (int c0 = 0; c0 < BN; c0 += 16) {
                        float v[16];
                        tmem_ld16(lane_base + COL_Q + (uint32_t)c0, v);
#pragma unroll
                        for (int i = 0; i < 16; ++i) acc[c0 + i] -= v[i];
                    }
                } else {
                    ok = false;
                }
                tc_fence_before();
                __syncwarp();
                if (lane == 0) bar_arrive_leader(&q_empty);
                ++seg;
                // this CTA's 128-row slab of pair tile t behaves as one-SM tile mt*2 + rank
                const int mt1 = mt * 2 + (int)rank;
                if (ka == 0 && kb == nk) {
                    tile_out(a, acc, mt1, n0, m, xch);
                } else {
                    const long long tu0 = (long long)t * nk;
                    const int slot = u0 >= tu0 ? 0 : 1;
                    float* wsp = a.ws + (((size_t)c * 2 + slot) * 2 + rank) * (BN * BM);
#pragma unroll
                    for (int j = 0; j < BN; ++j) wsp[(size_t)j * BM + m] = acc[j];
                    __threadfence();
                    drain_sync();
                    const int cf = owner_of(tu0, C, U), cl = owner_of(tu0 + nk - 1, C, U);
                    if (warp == DRAIN_WARP0 && lane == 0) {
                        const int prev = atomicAdd(&a.cnt[t * 2 + (int)rank], 1);
                        last_flag = prev == cl - cf;
                    }
                    drain_sync();
                    if (last_flag) {
                        __threadfence();
#pragma unroll
                        for (int j = 0; j < BN; ++j) acc[j] = 0.f;
                        for (int cc = cf; cc <= cl; ++cc) {
                            const int sl = u_begin(cc, C, U) >= tu0 ? 0 : 1;
                            const float* src = a.ws + (((size_t)cc * 2 + sl) * 2 + rank) * (BN * BM);
#pragma unroll
                            for (int j = 0; j < BN; ++j) acc[j] += __ldcg(src + (size_t)j * BM + m);
                        }
                        tile_out(a, acc, mt1, n0, m, xch);
                        if (warp == DRAIN_WARP0 && lane == 0) a.cnt[t * 2 + (int)rank] = 0;
                    }
                    drain_sync();
                }
#pragma unroll
                for (int j = 0; j < BN; ++j) acc[j] = 0.f;
            }
            cur.next();
        }
    }

    tc_fence_before();
    __syncthreads();
    cluster_sync();                 // no CTA leaves while its peer may still address it
    if (warp == MMA_WARP) {
        tc_fence_after();
        asm volatile("tcgen05.dealloc.cta_group::2.sync.aligned.b32 %0, %1;" ::"r"(tmem), "r"(512));
    }
}

// f32 activations -> f16 hi / lo rows plus the per-sub-block sums X_j as f16
// hi / lo in [K/256][r_pad][8] (one thread per (row, sub-block)).
__global__ void q4_split_kernel(const float* __restrict__ X, int ldx, int n_rows, int K,
                                __half* __restrict__ hi, __half* __restrict__ lo, int ld16,
                                __half* __restrict__ xs_hi, __half* __restrict__ xs_lo, int r_pad) {
    const int nsub = K / 32;
    const long total = (long)n_rows * nsub;
    for (long i = (long)blockIdx.x * blockDim.x + threadIdx.x; i < total;
         i += (long)gridDim.x * blockDim.x) {
        const int n = (int)(i / nsub), j = (int)(i % nsub);
        const float4* src = (const float4*)(X + (size_t)n * ldx + 32 * j);
        float s = 0.f;
        uint32_t h[16], l[16];
#pragma unroll
        for (int v = 0; v < 8; ++v) {
            const float4 f = src[v];
            s += f.x;
            s += f.y;
            s += f.z;
            s += f.w;
            const __half2 a = __floats2half2_rn(f.x, f.y), b = __floats2half2_rn(f.z, f.w);
            const float2 fa = __half22float2(a), fb = __half22float2(b);
            const __half2 la = __floats2half2_rn(f.x - fa.x, f.y - fa.y);
            const __half2 lb = __floats2half2_rn(f.z - fb.x, f.w - fb.y);
            h[2 * v] = *(const uint32_t*)&a;
            h[2 * v + 1] = *(const uint32_t*)&b;
            l[2 * v] = *(const uint32_t*)&la;
            l[2 * v + 1] = *(const uint32_t*)&lb;
        }
        uint4* dh = (uint4*)(hi + (size_t)n * ld16 + 32 * j);
        uint4* dl = (uint4*)(lo + (size_t)n * ld16 + 32 * j);
#pragma unroll
        for (int v = 0; v < 4; ++v) {
            dh[v] = make_uint4(h[4 * v], h[4 * v + 1], h[4 * v + 2], h[4 * v + 3]);
            dl[v] = make_uint4(l[4 * v], l[4 * v + 1], l[4 * v + 2], l[4 * v + 3]);
        }
        const __half sh = __float2half_rn(s);
        const size_t o = ((size_t)(j >> 3) * r_pad + n) * 8 + (j & 7);
        xs_hi[o] = sh;
        xs_lo[o] = __float2half_rn(s - __half2float(sh));
    }
}

int g_sms = 0;

}  // namespace

extern "C" int sb_q4_make_operand(sb_q4_operand* op, void* hi, void* lo, void* xs_hi, void* xs_lo,
                                  int rows, int r_pad, int K, int ld16) {
    cudaDriverEntryPointQueryResult qr;
    void* fp = nullptr;
    if (cudaGetDriverEntryPoint("cuTensorMapEncodeTiled", &fp, cudaEnableDefault, &qr) != cudaSuccess ||
        qr != cudaDriverEntryPointSuccess)
        return -1;
    auto enc = (PFN_cuTensorMapEncodeTiled_v12000)fp;
    if (!op || !hi || !lo || !xs_hi || !xs_lo || K % 256 || ld16 % 8 || rows < 1 || r_pad % BN ||
        r_pad < rows)
        return -1;
    op->hi = hi;
    op->lo = lo;
    op->xs_hi = xs_hi;
    op->xs_lo = xs_lo;
    op->rows = rows;
    op->r_pad = r_pad;
    op->K = K;
    op->ld16 = ld16;
    op->one_pass = 0;
    const cuuint64_t nsb = (cuuint64_t)((K / 256 + 1) & ~1);
    for (int part = 0; part < 6; ++part) {
        // parts 0-1: x hi / lo, 64 x 128 boxes; 2-3: x hi / lo, 64 x 64 boxes;
        // 4-5: sub-block sums hi / lo as [nsb * r_pad][8] with 8 x 64 boxes
        unsigned char* maps[6] = {op->map_hi, op->map_lo, op->map2_hi, op->map2_lo, op->xsmap_hi,
                                  op->xsmap_lo};
        void* base[6] = {hi, lo, hi, lo, xs_hi, xs_lo};
        const bool xs = part >= 4;
        cuuint64_t dims[2] = {xs ? 8 : (cuuint64_t)K, xs ? nsb * (cuuint64_t)r_pad : (cuuint64_t)rows};
        cuuint64_t strides[1] = {xs ? 16 : (cuuint64_t)ld16 * 2};
        cuuint32_t box[2] = {xs ? 8u : (cuuint32_t)BK, part < 2 ? (cuuint32_t)BN : (cuuint32_t)BN2};
        cuuint32_t estr[2] = {1, 1};
        CUresult r = enc((CUtensorMap*)maps[part], CU_TENSOR_MAP_DATA_TYPE_FLOAT16, 2, base[part], dims,
                         strides, box, estr, CU_TENSOR_MAP_INTERLEAVE_NONE,
                         xs ? CU_TENSOR_MAP_SWIZZLE_NONE : CU_TENSOR_MAP_SWIZZLE_128B,
                         CU_TENSOR_MAP_L2_PROMOTION_L2_256B, CU_TENSOR_MAP_FLOAT_OOB_FILL_NONE);
        if (r != CUDA_SUCCESS) {
            sb_set_error("cuTensorMapEncodeTiled failed (%d)", (int)r);
            return -1;
        }
    }
    return 0;
}

extern "C" int sb_q4_split(const float* X, int ldx, int n_rows, const sb_q4_operand* op,
                           cudaStream_t st) {
    if (!op || n_rows < 1 || n_rows > op->rows || ldx % 4) return -1;
    const long total = (long)n_rows * (op->K / 32);
    const int grid = (int)((total + 127) / 128 < 4736 ? (total + 127) / 128 : 4736);
    q4_split_kernel<<<grid, 128, 0, st>>>(X, ldx, n_rows, op->K, (__half*)op->hi, (__half*)op->lo,
                                          op->ld16, (__half*)op->xs_hi, (__half*)op->xs_lo,
                                          op->r_pad);
    return 0;
}

extern "C" size_t sb_q4_ws_floats(void) {
    return (size_t)(g_sms > 0 ? g_sms : 256) * 2 * BN * BM;
}

extern "C" int sb_q4_tiles(int M_pad, int n_rows) {
    return M_pad / BM * ((n_rows + BN - 1) / BN);
}

extern "C" void sb_q4_prepare(void) {
    int dev = 0;
    cudaGetDevice(&dev);
    cudaDeviceGetAttribute(&g_sms, cudaDevAttrMultiProcessorCount, dev);
    cudaFuncSetAttribute(q4k_gemm_kernel, cudaFuncAttributeMaxDynamicSharedMemorySize, (int)SMEM);
    cudaFuncSetAttribute(q4k_gemm2_kernel, cudaFuncAttributeMaxDynamicSharedMemorySize, (int)SMEM2);
}

extern "C" int sb_q4_gemm(const sb_matrix* W, const sb_q4_operand* X, int n_rows, float* Y, int ldy,
                          int epi, float* ws, int* cnt, int* err, cudaStream_t st) {
    if (!W || !X || W->wtype != SB_WT_Q4K || W->M_pad % BM || W->K % 256 || W->K != X->K ||
        n_rows < 1 || n_rows > X->rows || !ws || !cnt || !err || g_sms < 1 ||
        (epi != SB_EPI_STORE && epi != SB_EPI_ADD && epi != SB_EPI_SILU))
        return -1;
    Args a;
    a.W = (const unsigned char*)W->data;
    a.xs_hi = (const __half*)X->xs_hi;
    a.xs_lo = (const __half*)X->xs_lo;
    a.Y = Y;
    a.ws = ws;
    a.cnt = cnt;
    a.err = err;
    a.M = W->M;
    a.M_pad = W->M_pad;
    a.K = W->K;
    a.n_rows = n_rows;
    a.r_pad = X->r_pad;
    a.ldy = ldy;
    a.epi = epi;
    a.NT = (n_rows + BN - 1) / BN;
    a.one_pass = X->one_pass;
    // the Q4_K rows as a 2-D byte tensor [M_pad][K/256 * 144], boxes of one
    // super-block x 128 rows (encoded per call; a captured graph keeps it)
    CUtensorMap wmap;
    {
        cudaDriverEntryPointQueryResult qr;
        void* fp = nullptr;
        if (cudaGetDriverEntryPoint("cuTensorMapEncodeTiled", &fp, cudaEnableDefault, &qr) != cudaSuccess ||
            qr != cudaDriverEntryPointSuccess)
            return -1;
        auto enc = (PFN_cuTensorMapEncodeTiled_v12000)fp;
        const cuuint64_t rb = (cuuint64_t)(W->K / 256) * 144;
        cuuint64_t dims[2] = {rb, (cuuint64_t)W->M_pad};
        cuuint64_t strides[1] = {rb};
        cuuint32_t box[2] = {144, (cuuint32_t)BM};
        cuuint32_t estr[2] = {1, 1};
        CUresult r = enc(&wmap, CU_TENSOR_MAP_DATA_TYPE_UINT8, 2, (void*)W->data, dims, strides, box,
                         estr, CU_TENSOR_MAP_INTERLEAVE_NONE, CU_TENSOR_MAP_SWIZZLE_NONE,
                         CU_TENSOR_MAP_L2_PROMOTION_L2_256B, CU_TENSOR_MAP_FLOAT_OOB_FILL_NONE);
        if (r != CUDA_SUCCESS) {
            sb_set_error("Q4_K tensor map: cuTensorMapEncodeTiled failed (%d)", (int)r);
            return -1;
        }
    }
    const char* one = getenv("SLATE_Q4_ONE_SM");
    if (W->M_pad % (2 * BM) == 0 && !(one && one[0] == '1') && g_sms >= 2) {
        // pairs of CTAs over tiles of 256 weight rows x 128 activation rows
        const long long U = (long long)(W->M_pad / (2 * BM)) * a.NT * (W->K / BK);
        const int C = (int)(U < g_sms / 2 ? U : g_sms / 2);
        cudaLaunchConfig_t cfg = {};
        cfg.gridDim = dim3((unsigned)(2 * C));
        cfg.blockDim = dim3(NTHREADS);
        cfg.dynamicSmemBytes = SMEM2;
        cfg.stream = st;
        cudaLaunchAttribute attr[1];
        attr[0].id = cudaLaunchAttributeClusterDimension;
        attr[0].val.clusterDim.x = 2;
        attr[0].val.clusterDim.y = 1;
        attr[0].val.clusterDim.z = 1;
        cfg.attrs = attr;
        cfg.numAttrs = 1;
        CUtensorMap m2h, m2l, xsh, xsl;
        memcpy(&m2h, X->map2_hi, sizeof m2h);
        memcpy(&m2l, X->map2_lo, sizeof m2l);
        memcpy(&xsh, X->xsmap_hi, sizeof xsh);
        memcpy(&xsl, X->xsmap_lo, sizeof xsl);
        return cudaLaunchKernelEx(&cfg, q4k_gemm2_kernel, m2h, m2l, xsh, xsl, wmap, a) == cudaSuccess
                   ? 0
                   : -5;
    }
    const long long U = (long long)(W->M_pad / BM) * a.NT * (W->K / BK);
    const int C = (int)(U < g_sms ? U : g_sms);
    q4k_gemm_kernel<<<C, NTHREADS, SMEM, st>>>(*(const CUtensorMap*)X->map_hi,
                                               *(const CUtensorMap*)X->map_lo, wmap, a);
    return 0;
}
