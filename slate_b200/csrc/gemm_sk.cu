// gemm_sk.cu -- Q4_K weight GEMM on the tcgen05 tensor cores: three f16
// passes, dequantised weights in tensor memory, persistent stream-K schedule.
//
//   Y[n][m] (op)= sum_k X[n][k] * W[m][k]       (op: store, residual add, or
//                                                SiLU(gate) * up for the fused FFN)
//
// W is Q4_K (src/util/quant.c:187-199: w = d * sc_j * q - dmin * m_j in f32,
// the reference's own reconstruction); X is f32, staged as an f16 hi + lo pair
// (x = hi + lo to ~22 bits) by sb_tc_split().  Each weight is also split into
// f16 hi + lo, and the tensor cores accumulate hi*hi + hi*lo + lo*hi in f32,
// which reproduces f32 products to ~1e-6 relative (the same numerics as
// gemm_tc.cu's three-pass kernel).  The weights are split as w * 2^wexp (a
// power of two per matrix, chosen at upload) so that their lo halves stay
// normal f16 numbers; the drain scales the accumulator back by 2^-wexp.
//
// Work decomposition: a tile is 128 weight rows (TMEM lanes) x up to 256
// activation rows (MMA N); the (tile, 64-wide K step) space is cut into one
// contiguous range per CTA, one CTA per SM.  A STORE / ADD tile covered by
// one CTA is written from TMEM with its epilogue; the parts of a tile shared
// by several CTAs, and every tile of the fused SiLU(gate) * up projection, go
// to a workspace as f32, and a second launch spread over the whole GPU sums
// the parts in CTA order -- results do not depend on timing -- and applies the
// epilogue.  This keeps every SM busy whatever the tile count
// (the 224 tiles of the 8B gate/up projection are 1.5 waves of 148 SMs as a
// plain grid), and the accumulator is released as soon as it is copied out.
//
// Operand placement: the dequantised weights go register -> TMEM
// (tcgen05.st; MMA with A in tensor memory), so shared memory holds only the
// activation ring, deep enough (3 x 64 KB; 4 x 32 KB for operands of up to
// 128 rows) to keep the TMA stream ahead of the MMAs, and the tensor core
// reads only B from shared memory.
//
// Roles (512 threads): warps 0-7 dequantise (warp w, lane l: weight row
// 32 (w % 4) + l, sub-block w / 4 of the K step's two; each thread copies the
// Q4_K bytes of the next two K steps into its own shared-memory ring slots
// with cp.async while the current step converts; two producer warps per
// scheduler hide each other's latency); warp 8 issues the MMAs; warp 9
// issues the TMA loads of x; warps 12-15 drain the accumulator (warp 12 + q
// reads TMEM lanes 32q..32q+31).  TMEM: the
// accumulator in columns [0, 256), the A ring (4 stages x (32 hi + 32 lo)
// columns) in [256, 512).  Every wait is bounded (2 s of %globaltimer): a
// timeout records an error code in *err and the roles stop; copies and MMAs
// in flight are waited for and TMEM is freed before the CTA exits.
#include <cuda.h>
#include <cuda_fp16.h>
#include <cudaTypedefs.h>

#include "sb_internal.h"
#include "sb_kernels.h"
#include "sb_pdl.h"
#include "sb_tc.h"

namespace {

constexpr int BM = 128;                 // weight rows per tile
constexpr int BN = 256;                 // activation rows per tile (max MMA N)
constexpr int BK = 64;                  // K per step (one 128-byte swizzle row of f16)
constexpr int ASTAGES = 4;              // A stages in TMEM
constexpr int BSTAGES = 4;              // x stages in shared memory (at most; see sk_stages)
constexpr int NPROD = 256;             // 8 producer warps: two per weight row, one sub-block each
constexpr int MMA_WARP = 8, TMA_WARP = 9, DRAIN_WARP0 = 12;
constexpr int NTHREADS = 512;
constexpr uint32_t COL_A = 256;
constexpr int WSTAGES = 3;              // per-thread ring of Q4_K bytes (cp.async)
constexpr int W_STAGE = 2 * NPROD * 16; // [header | nibbles][producer thread] x 16 B
// x stages: 3 of 64 KB for 256-row operand boxes, 4 of 32 KB for boxes of up
// to 128 rows -- the latter leave room on the SM for an attention CTA of the
// other half of the batch.
__host__ __device__ constexpr int sk_stages(int n_box) { return n_box <= 128 ? 4 : 3; }
__host__ __device__ constexpr size_t sk_smem(int n_box) {
    return (size_t)sk_stages(n_box) * 2 * n_box * 128 + (size_t)WSTAGES * W_STAGE + 1024;
}
constexpr size_t SMEM_MAX = sk_smem(BN);
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
// Bounded wait: false (and *err set) after WAIT_NS, or soon after another
// thread of the grid has failed (the error word is polled every 32 tries).
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
// Wait used before the CTA exits for its own copies / MMAs in flight: bounded
// by time only (not cut short by another CTA's error), so that nothing still
// writes into this CTA's shared or tensor memory once it has gone.
__device__ void bar_wait_exit(uint64_t* b, uint32_t parity, int* err) {
    const uint64_t t0 = gtimer();
    while (!bar_try(b, parity)) {
        if (gtimer() - t0 > WAIT_NS) {
            atomicCAS(err, 0, 9);
            return;
        }
    }
}
__device__ __forceinline__ void tma_2d(void* dst, const CUtensorMap* map, uint64_t* bar, int x, int y) {
    asm volatile(
        "cp.async.bulk.tensor.2d.shared::cluster.global.tile.mbarrier::complete_tx::bytes "
        "[%0], [%1, {%3, %4}], [%2];" ::"r"(su32(dst)),
        "l"(map), "r"(su32(bar)), "r"(x), "r"(y)
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
// D (+)= A * B, A in tensor memory (lane = weight row, column c = K pair 2c, 2c+1).
__device__ __forceinline__ void mma_ta(uint32_t d, uint32_t a_tmem, uint64_t b, uint32_t idesc,
                                       uint32_t acc) {
    asm volatile(
        "{\n\t.reg .pred p;\n\tsetp.ne.b32 p, %4, 0;\n\t"
        "tcgen05.mma.cta_group::1.kind::f16 [%0], [%1], %2, %3, p;\n\t}\n" ::"r"(d),
        "r"(a_tmem), "l"(b), "r"(idesc), "r"(acc));
}
__device__ __forceinline__ void mma_commit(uint64_t* bar) {
    asm volatile("tcgen05.commit.cta_group::1.mbarrier::arrive::one.shared::cluster.b64 [%0];" ::"r"(
                     su32(bar))
                 : "memory");
}
// 16 columns of this warp's 32 lanes (no wait: the caller waits once).
__device__ __forceinline__ void tmem_st16(uint32_t taddr, const uint32_t* r) {
    asm volatile(
        "tcgen05.st.sync.aligned.32x32b.x16.b32 [%0], "
        "{%1, %2, %3, %4, %5, %6, %7, %8, %9, %10, %11, %12, %13, %14, %15, %16};" ::"r"(taddr),
        "r"(r[0]), "r"(r[1]), "r"(r[2]), "r"(r[3]), "r"(r[4]), "r"(r[5]), "r"(r[6]), "r"(r[7]),
        "r"(r[8]), "r"(r[9]), "r"(r[10]), "r"(r[11]), "r"(r[12]), "r"(r[13]), "r"(r[14]), "r"(r[15])
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

// 16 bytes global -> shared without a register (L2 only; completion by group)
// with an L2 eviction policy (createpolicy): the weights are read once per
// GEMM, so they are marked to leave L2 first and the workspace written by the
// drain stays there for the output pass.
__device__ __forceinline__ uint64_t l2_evict_first() {
    uint64_t pol;
    asm volatile("createpolicy.fractional.L2::evict_first.b64 %0, 1.0;" : "=l"(pol));
    return pol;
}
__device__ __forceinline__ void cp_async16_pol(void* dst, const void* src, uint64_t pol) {
    asm volatile("cp.async.cg.shared.global.L2::cache_hint [%0], [%1], 16, %2;" ::"r"(su32(dst)),
                 "l"(src), "l"(pol)
                 : "memory");
}
__device__ __forceinline__ void cp_async_commit() {
    asm volatile("cp.async.commit_group;" ::: "memory");
}
template <int N>
__device__ __forceinline__ void cp_async_wait() {
    asm volatile("cp.async.wait_group %0;" ::"n"(N) : "memory");
}

// ---- Q4_K dequantisation (util/quant.c:157-166 scale packing, :187-199 values)
__device__ __forceinline__ float f16_lo(uint32_t w) {
    return __half2float(__ushort_as_half((unsigned short)(w & 0xffffu)));
}
__device__ __forceinline__ float f16_hi(uint32_t w) {
    return __half2float(__ushort_as_half((unsigned short)(w >> 16)));
}
__device__ __forceinline__ uint32_t hbyte(uint4 h, int i) {
    const uint32_t w = i < 4 ? h.y : (i < 8 ? h.z : h.w);
    return (w >> ((i & 3) * 8)) & 0xffu;
}
// d * sc_j and dmin * m_j of sub-block j, in f32 as the reference forms them.
__device__ __forceinline__ void sub_scale(uint4 h, int j, float& sd, float& sm) {
    uint32_t sc, mn;
    if (j < 4) {
        sc = hbyte(h, j) & 63u;
        mn = hbyte(h, j + 4) & 63u;
    } else {
        sc = (hbyte(h, j + 4) & 15u) | ((hbyte(h, j - 4) >> 6) << 4);
        mn = (hbyte(h, j + 4) >> 4) | ((hbyte(h, j) >> 6) << 4);
    }
    sd = f16_lo(h.x) * (float)sc;
    sm = f16_hi(h.x) * (float)mn;
}
// One sub-block (16 nibble bytes, Slate order: byte i holds element i in its
// low nibble and element i + 16 in its high nibble) -> 16 columns of f16 pairs
// (column c = elements 2c, 2c+1) as hi = f16(w) and lo = f16(w - hi), with
// w = sd * q - sm formed in f32 by one fused multiply-add per element.
// A nibble q becomes the float 2^23 + q by a byte permute (q in the low
// mantissa byte under the exponent byte 0x4B), and subtracting 2^23 leaves q
// exactly; the element pairs go through the paired f32 pipes (FADD2 / FFMA2,
// round-to-nearest like their scalar forms).
__device__ __forceinline__ void dequant_sub(uint4 q, float sd, float sm, uint32_t* hi, uint32_t* lo) {
    const uint32_t qw[4] = {q.x, q.y, q.z, q.w};
    const float2 sd2 = make_float2(sd, sd), nsm2 = make_float2(-sm, -sm);
    const float2 off2 = make_float2(-8388608.0f, -8388608.0f);
#pragma unroll
    for (int h = 0; h < 2; ++h) {                        // low nibbles, then high
#pragma unroll
        for (int wi = 0; wi < 4; ++wi) {
            const uint32_t nb = (h ? qw[wi] >> 4 : qw[wi]) & 0x0f0f0f0fu;
#pragma unroll
            for (int pr = 0; pr < 2; ++pr) {             // bytes 2pr, 2pr+1 of the word
                const float2 mg = make_float2(
                    __uint_as_float(__byte_perm(nb, 0x4B000000u, 0x7440u + 2 * pr)),
                    __uint_as_float(__byte_perm(nb, 0x4B000000u, 0x7441u + 2 * pr)));
                const float2 w = __ffma2_rn(sd2, __fadd2_rn(mg, off2), nsm2);
                const __half2 hh = __floats2half2_rn(w.x, w.y);
                const float2 back = __half22float2(hh);
                const __half2 ll = __floats2half2_rn(w.x - back.x, w.y - back.y);
                const int c = h * 8 + wi * 2 + pr;       // elements 2c, 2c+1
                hi[c] = *(const uint32_t*)&hh;
                lo[c] = *(const uint32_t*)&ll;
            }
        }
    }
}

// ---- stream-K schedule ----------------------------------------------------
// CTA c of C owns units [U*c/C, U*(c+1)/C) of the U = tiles * nk (tile, K step)
// units, tile-major; a segment is one tile's part of that range.
__device__ __forceinline__ long long u_begin(int c, int C, long long U) {
    return U * c / C;
}
__device__ int owner_of(long long u, int C, long long U) {
    int c = (int)((u * C) / U);
    while (c > 0 && u_begin(c, C, U) > u) --c;
    while (c + 1 < C && u_begin(c + 1, C, U) <= u) ++c;
    return c;
}
struct Seg {
    long long u, u1;
    int nk, t, ka, kb;
    __device__ __forceinline__ void set() {
        t = (int)(u / nk);
        ka = (int)(u - (long long)t * nk);
        kb = (int)min((long long)nk, u1 - (long long)t * nk);
    }
    __device__ __forceinline__ void start(long long a, long long b, int nk_) {
        u = a;
        u1 = b;
        nk = nk_;
        t = ka = kb = 0;
        if (u < u1) set();
    }
    __device__ __forceinline__ bool valid() const { return u < u1; }
    __device__ __forceinline__ void next() {
        u = (long long)t * nk + kb;
        if (u < u1) set();
    }
};

// RoPE + paged-cache epilogue of the fused Q|K|V projection (SB_EPI_ROPE).
struct SkRope {
    const int32_t* row_pos;
    const int32_t* row_slot;
    const int32_t* page_table;
    void* pool;
    const float* rcos;
    const float* rsin;
    long long n_pages;
    int max_pages, layer, kv_f16, nq, nkv, hd;
};

struct SkArgs {
    const unsigned char* W;   // Q4_K rows [M_pad][K/256 * 144]
    float* Y;
    float* ws;                // partial tile slots (ws_slot), SiLU tile areas (ws_tile)
    __half* h_hi;             // SiLU: optional f16 hi / lo copy of the output
    __half* h_lo;
    int* err;
    int M, M_pad, K, n_rows, NT, n_box, ldy, epi, ld16;
    float wscale, wunscale;   // 2^wexp applied to the weights before the split, 2^-wexp after
    SkRope r;                 // SB_EPI_ROPE only
};

// Workspace: a 128 x 256 tile is stored as [BN/4][BM] float4 (column group
// c/4, row m), so that a warp's 32 rows of one column group are 512
// contiguous bytes.  CTA cc has two slots for the parts of shared tiles
// (slot 0: its first segment, slot 1: its last); after the C * 2 slots, each
// tile of a fused SiLU GEMM has an area for the accumulator of a CTA that
// computed it alone.
__device__ __forceinline__ float4* ws_slot(const float* ws, int cc, int slot) {
    return (float4*)(ws + ((size_t)cc * 2 + slot) * (BN * BM));
}
__device__ __forceinline__ float4* ws_tile(const float* ws, int C, int t) {
    return (float4*)(ws + ((size_t)C * 2 + t) * (BN * BM));
}

// SiLU(g) * u = g / (1 + e^-g) * u (backend_cpu.c:78-87) with the fast
// exponential and division (__expf, __fdividef: a few ulp of f32 apart from
// expf and the IEEE quotient); the output pass evaluates it for every FFN unit
// of every row, and the exact forms made that pass instruction-bound.
__device__ __forceinline__ float silu_mul(float g, float u) {
    return __fdividef(g, 1.0f + __expf(-g)) * u;
}
__device__ __forceinline__ void store_h(const SkArgs& a, int n, int unit, float h) {
    a.Y[(size_t)n * a.ldy + unit] = h;
    if (a.h_hi) {
        const __half hh = __float2half_rn(h);
        a.h_hi[(size_t)n * a.ld16 + unit] = hh;
        a.h_lo[(size_t)n * a.ld16 + unit] = __float2half_rn(h - __half2float(hh));
    }
}

// STORE / ADD epilogue of a tile this CTA computed alone, straight from TMEM,
// by the four drain warps (thread m = weight row m, 16 columns per round; ADD
// loads the next 16 values of Y while the current ones are written).
__device__ __forceinline__ void alone_out(const SkArgs& a, uint32_t lane_base, int mt, int n0,
                                          int n_mma, int m) {
    const int row = mt * BM + m;
    const bool live = row < a.M;
    float y[16];
    auto load_y = [&](int c0) {
#pragma unroll
        for (int i = 0; i < 16; ++i) {
            const int n = n0 + c0 + i;
            y[i] = (live && n < a.n_rows) ? a.Y[(size_t)n * a.ldy + row] : 0.f;
        }
    };
    if (a.epi == SB_EPI_ADD) load_y(0);
    for (int c0 = 0; c0 < n_mma; c0 += 16) {
        float v[16];
        tmem_ld16(lane_base + (uint32_t)c0, v);
        float o[16];
#pragma unroll
        for (int i = 0; i < 16; ++i) {
            const float r = v[i] * a.wunscale;
            o[i] = a.epi == SB_EPI_ADD ? y[i] + r : r;
        }
        if (a.epi == SB_EPI_ADD && c0 + 16 < n_mma) load_y(c0 + 16);
        if (live) {
#pragma unroll
            for (int i = 0; i < 16; ++i) {
                const int n = n0 + c0 + i;
                if (n < a.n_rows) a.Y[(size_t)n * a.ldy + row] = o[i];
            }
        }
    }
}

// ---- output passes (second launch) -----------------------------------------
// STORE / ADD: CTA (t, g) finishes column group g (4 columns) of shared tile t,
// thread m weight row m; tiles that one CTA of the GEMM computed alone were
// written by it and are skipped.  The parts of CTAs cf..cl are summed in that
// order (the result does not depend on timing), then the epilogue is applied.
// The CTAs whose ranges cover tile t (cf..cl) and the slot holding cf's part
// (0 if cf's range starts in the tile; every later CTA's part is its first
// segment, slot 0).  Computed by one thread of the output-pass CTA.
struct TileSrc {
    int cf, cl, slot0;
};
__device__ TileSrc tile_sources(int t, int nk, int C, long long U) {
    const long long tu0 = (long long)t * nk;
    TileSrc r;
    r.cf = owner_of(tu0, C, U);
    r.cl = owner_of(tu0 + nk - 1, C, U);
    r.slot0 = u_begin(r.cf, C, U) >= tu0 ? 0 : 1;
    return r;
}

__global__ void __launch_bounds__(BM) sk_out_kernel(const SkArgs a, int C, long long U) {
    sb_grid_release();
    sb_grid_wait();      // the GEMM's workspace: after it (sb_pdl.h)
    __shared__ TileSrc ts;
    const int t = blockIdx.x, g4 = blockIdx.y, m = threadIdx.x;
    if (m == 0) ts = tile_sources(t, a.K / BK, C, U);
    __syncthreads();
    const int cf = ts.cf, cl = ts.cl;
    const int mt = t / a.NT, n0 = (t % a.NT) * BN;
    const int row = mt * BM + m;
    if (cf == cl || n0 + 4 * g4 >= a.n_rows || row >= a.M) return;
    float4 acc = make_float4(0.f, 0.f, 0.f, 0.f);
#pragma unroll 4
    for (int cc = cf; cc <= cl; ++cc) {
        const float4* src = ws_slot(a.ws, cc, cc == cf ? ts.slot0 : 0) + (size_t)g4 * BM;
        const float4 p = __ldcg(src + m);
        acc.x += p.x; acc.y += p.y; acc.z += p.z; acc.w += p.w;
    }
    const float v[4] = {acc.x, acc.y, acc.z, acc.w};
#pragma unroll
    for (int j = 0; j < 4; ++j) {
        const int n = n0 + 4 * g4 + j;
        if (n >= a.n_rows) continue;
        float* y = a.Y + (size_t)n * a.ldy + row;
        *y = a.epi == SB_EPI_ADD ? *y + v[j] : v[j];
    }
}

// SiLU: CTA (t, q) finishes columns [64 q, 64 q + 64) of every tile t (the
// GEMM leaves all its SiLU tiles in the workspace: a tile computed alone in
// its own area, the parts of a shared tile in the CTAs' slots); item (column
// group, gate row m < 64) reads gate row m and up row m + 64, four items per
// thread with their loads issued together.
constexpr int ST = 256;
__global__ void __launch_bounds__(ST) sk_silu_out_kernel(const SkArgs a, int C, long long U) {
    sb_grid_release();   // the down GEMM may start its set-up
    sb_grid_wait();      // the GEMM's workspace: after it (sb_pdl.h)
    __shared__ TileSrc ts;
    const int t = blockIdx.x, q = blockIdx.y;
    if (threadIdx.x == 0) ts = tile_sources(t, a.K / BK, C, U);
    __syncthreads();
    const int cf = ts.cf, cl = ts.cl;
    const int mt = t / a.NT, n0 = (t % a.NT) * BN;
    const int groups = (min(a.n_rows - n0, BN) + 3) / 4;
    const int g_lo = q * 16, g_hi = min(groups, g_lo + 16);
    if (g_lo >= g_hi) return;
    const int items = (g_hi - g_lo) * 64;
    for (int base = threadIdx.x; base < items; base += 4 * ST) {
        float4 acc[4], acc2[4];
        int g4[4], mm[4];
        bool live[4];
#pragma unroll
        for (int j = 0; j < 4; ++j) {
            const int it = base + j * ST;
            live[j] = it < items;
            g4[j] = g_lo + (live[j] ? it / 64 : 0);
            mm[j] = live[j] ? it % 64 : 0;
            acc[j] = make_float4(0.f, 0.f, 0.f, 0.f);
            acc2[j] = acc[j];
        }
        for (int cc = cf; cc <= cl; ++cc) {
            const float4* src = cf == cl ? ws_tile(a.ws, C, t)
                                         : ws_slot(a.ws, cc, cc == cf ? ts.slot0 : 0);
            float4 p[4], p2[4];
#pragma unroll
            for (int j = 0; j < 4; ++j) {
                if (!live[j]) continue;
                p[j] = __ldcg(src + (size_t)g4[j] * BM + mm[j]);
                p2[j] = __ldcg(src + (size_t)g4[j] * BM + mm[j] + 64);
            }
#pragma unroll
            for (int j = 0; j < 4; ++j) {
                if (!live[j]) continue;
                acc[j].x += p[j].x; acc[j].y += p[j].y; acc[j].z += p[j].z; acc[j].w += p[j].w;
                acc2[j].x += p2[j].x; acc2[j].y += p2[j].y; acc2[j].z += p2[j].z; acc2[j].w += p2[j].w;
            }
        }
#pragma unroll
        for (int j = 0; j < 4; ++j) {
            if (!live[j]) continue;
            const float v[4] = {acc[j].x, acc[j].y, acc[j].z, acc[j].w};
            const float u[4] = {acc2[j].x, acc2[j].y, acc2[j].z, acc2[j].w};
            const int unit = mt * 64 + mm[j];
            if (unit >= a.M / 2) continue;
#pragma unroll
            for (int e = 0; e < 4; ++e) {
                const int n = n0 + 4 * g4[j] + e;
                if (n < a.n_rows) store_h(a, n, unit, silu_mul(v[e], u[e]));
            }
        }
    }
}

// RoPE epilogue of the fused Q|K|V projection (src/loader/llama_infer.c:160-174):
// CTA (t, g4) finishes columns [4 g4, 4 g4 + 4) of tile t, thread m weight row
// m.  Every tile goes through the workspace (a tile computed alone in its own
// area, the parts of a shared one in the CTAs' slots), and a 128-row tile holds
// 128 / head_dim whole heads, so the NeoX pair (d, d + head_dim / 2) of a head
// is in the tile: query heads are rotated in place in Y, key heads rotated and
// value heads copied into the paged cache at each row's position, exactly as
// rope_append_heads_kernel does with the projection written out first.
__global__ void __launch_bounds__(BM) sk_rope_out_kernel(const SkArgs a, int C, long long U) {
    sb_grid_release();   // the attention may start its set-up
    sb_grid_wait();      // the GEMM's workspace: after it (sb_pdl.h)
    __shared__ TileSrc ts;
    __shared__ float xs[BM][4];
    const int t = blockIdx.x, g4 = blockIdx.y, m = threadIdx.x;
    if (m == 0) ts = tile_sources(t, a.K / BK, C, U);
    __syncthreads();
    const int cf = ts.cf, cl = ts.cl;
    const int mt = t / a.NT, n0 = (t % a.NT) * BN;
    if (n0 + 4 * g4 >= a.n_rows) return;          // the same for every thread of the CTA
    float4 acc = make_float4(0.f, 0.f, 0.f, 0.f);
    for (int cc = cf; cc <= cl; ++cc) {
        const float4* src = (cf == cl ? ws_tile(a.ws, C, t) : ws_slot(a.ws, cc, cc == cf ? ts.slot0 : 0)) +
                            (size_t)g4 * BM;
        const float4 p = __ldcg(src + m);
        acc.x += p.x; acc.y += p.y; acc.z += p.z; acc.w += p.w;
    }
    xs[m][0] = acc.x;
    xs[m][1] = acc.y;
    xs[m][2] = acc.z;
    xs[m][3] = acc.w;
    __syncthreads();
    const SkRope& r = a.r;
    const int row = mt * BM + m;
    if (row >= a.M) return;                       // zero padding rows
    const int hd = r.hd, half = hd / 2, h = row / hd, d = row % hd;
    const bool rotate = h < r.nq + r.nkv;
    if (rotate && d >= half) return;              // the pair is the thread of element d - half
    const size_t hs = (size_t)SB_PAGE_TOKENS * hd;
#pragma unroll
    for (int j = 0; j < 4; ++j) {
        const int n = n0 + 4 * g4 + j;
        if (n >= a.n_rows) break;
        const int pos = r.row_pos[n];
        if (pos < 0) continue;
        float o0 = xs[m][j], o1 = 0.f;
        if (rotate) {
            const float c = r.rcos[(size_t)pos * half + d], sn = r.rsin[(size_t)pos * half + d];
            const float x0 = xs[m][j], x1 = xs[m + half][j];
            o0 = x0 * c - x1 * sn;
            o1 = x0 * sn + x1 * c;
            if (h < r.nq) {
                a.Y[(size_t)n * a.ldy + row] = o0;
                a.Y[(size_t)n * a.ldy + row + half] = o1;
                continue;
            }
        }
        const int slot = r.row_slot[n];
        const int page = r.page_table[(size_t)slot * r.max_pages + pos / SB_PAGE_TOKENS];
        if (page < 0 || page >= r.n_pages) continue;   // never allocated: skip, never fault
        const int kv = rotate ? 0 : 1, hk = rotate ? h - r.nq : h - r.nq - r.nkv;
        const size_t off = ((((size_t)r.layer * r.n_pages + page) * 2 + kv) * r.nkv + hk) * hs +
                           (size_t)(pos % SB_PAGE_TOKENS) * hd + d;
        if (r.kv_f16) {
            __half* dst = (__half*)r.pool + off;
            dst[0] = __float2half_rn(o0);
            if (rotate) dst[half] = __float2half_rn(o1);
        } else {
            float* dst = (float*)r.pool + off;
            dst[0] = o0;
            if (rotate) dst[half] = o1;
        }
    }
}

__global__ void __launch_bounds__(NTHREADS, 1)
    sk_kernel(const __grid_constant__ CUtensorMap xmap_hi, const __grid_constant__ CUtensorMap xmap_lo,
              const SkArgs a) {
    extern __shared__ __align__(1024) unsigned char smem_raw[];
    unsigned char* bst = (unsigned char*)(((uintptr_t)smem_raw + 1023) & ~(uintptr_t)1023);
    const int nbs = sk_stages(a.n_box);
    const size_t b_part = (size_t)a.n_box * 128, b_stage = 2 * b_part;   // hi | lo
    uint4* wring = (uint4*)(bst + (size_t)nbs * b_stage);     // [WSTAGES][2][NPROD]
    __shared__ uint64_t a_full[ASTAGES], a_empty[ASTAGES], b_full[BSTAGES], b_empty[BSTAGES];
    __shared__ uint64_t acc_full, acc_empty, done_bar;
    __shared__ uint32_t tmem_slot;

    sb_grid_release();   // the output pass may be scheduled (it waits for this grid)
    const int tid = threadIdx.x, warp = tid >> 5, lane = tid & 31;
    const int C = gridDim.x, c = blockIdx.x;
    const int nk = a.K / BK;
    const long long U = (long long)(a.M_pad / BM) * a.NT * nk;
    const long long u0 = u_begin(c, C, U), u1 = u_begin(c + 1, C, U);

    if (tid == 0) {
        for (int s = 0; s < ASTAGES; ++s) {
            bar_init(&a_full[s], NPROD / 32);      // one arrival per producer warp
            bar_init(&a_empty[s], 1);
        }
        for (int s = 0; s < nbs; ++s) {
            bar_init(&b_full[s], 1);
            bar_init(&b_empty[s], 1);
        }
        bar_init(&acc_full, 1);
        bar_init(&acc_empty, 4);                  // one arrival per drain warp
        bar_init(&done_bar, 1);
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

    if (warp < 8) {
        // ---------------- producers: Q4_K -> f16 hi | lo in TMEM ----------------
        const int m = (warp & 3) * 32 + lane, half = warp >> 2;
        const uint32_t lane_a = tmem + ((uint32_t)((warp & 3) * 32) << 16) + COL_A + 16u * half;
        const size_t row_bytes = (size_t)(a.K / 256) * 144;
        const uint64_t wpol = l2_evict_first();
        long long it = 0;
        Seg sg;
        sg.start(u0, u1, nk);
        while (sg.valid() && ok) {
            const int mt = sg.t / a.NT;
            const unsigned char* wrow = a.W + (size_t)(mt * BM + m) * row_bytes;
            // The Q4_K bytes (header, this thread's 16 nibble bytes) of K steps
            // k+1 and k+2 are in flight into this thread's ring slots while
            // step k converts (cp.async: no register waits on the copies).
            auto issue = [&](int kk, long long slot) {
                const unsigned char* p = wrow + (size_t)(kk >> 2) * 144;
                uint4* d = wring + (size_t)(slot % WSTAGES) * 2 * NPROD + tid;
                cp_async16_pol(d, p, wpol);
                cp_async16_pol(d + NPROD, p + 16 + 32 * (kk & 3) + 16 * half, wpol);
            };
            long long wi = 0;                      // ring position of step sg.ka
            for (int j = 0; j < WSTAGES - 1; ++j) {
                if (sg.ka + j < sg.kb) issue(sg.ka + j, wi + j);
                cp_async_commit();
            }
            for (int k = sg.ka; k < sg.kb; ++k, ++it, ++wi) {
                const int s = (int)(it % ASTAGES);
                if (it >= ASTAGES &&
                    !__all_sync(0xffffffffu,
                                bar_wait(&a_empty[s], (uint32_t)(((it / ASTAGES) - 1) & 1), a.err, 31))) {
                    ok = false;
                    break;
                }
                if (k + WSTAGES - 1 < sg.kb) issue(k + WSTAGES - 1, wi + WSTAGES - 1);
                cp_async_commit();
                cp_async_wait<WSTAGES - 1>();     // step k's copies have landed
                const uint4* src = wring + (size_t)(wi % WSTAGES) * 2 * NPROD + tid;
                const uint4 h0 = src[0], q0 = src[NPROD];
                uint32_t hi[16], lo[16];
                float sd, sm;
                sub_scale(h0, (k & 3) * 2 + half, sd, sm);
                dequant_sub(q0, sd * a.wscale, sm * a.wscale, hi, lo);
                tmem_st16(lane_a + (uint32_t)(64 * s), hi);
                tmem_st16(lane_a + (uint32_t)(64 * s + 32), lo);
                asm volatile("tcgen05.wait::st.sync.aligned;" ::: "memory");
                tc_fence_before();
                __syncwarp();
                if (lane == 0) bar_arrive(&a_full[s]);
            }
            cp_async_wait<0>();                    // nothing in flight past the segment
            sg.next();
        }
    } else if (warp == TMA_WARP) {
        // ---------------- x hi / lo tiles by TMA ----------------
        if (lane == 0) {
            // x is the previous kernel's output: wait for that grid (this one
            // may start early, see sb_sk_gemm)
            sb_grid_wait();
            long long it = 0;
            Seg sg;
            sg.start(u0, u1, nk);
            const uint32_t bytes = 2u * (uint32_t)a.n_box * 128u;
            while (sg.valid() && ok) {
                const int n0 = (sg.t % a.NT) * BN;
                for (int k = sg.ka; k < sg.kb; ++k, ++it) {
                    const int s = (int)(it % nbs);
                    if (it >= nbs &&
                        !bar_wait(&b_empty[s], (uint32_t)(((it / nbs) - 1) & 1), a.err, 32)) {
                        ok = false;
                        break;
                    }
                    unsigned char* st = bst + (size_t)s * b_stage;
                    bar_expect(&b_full[s], bytes);
                    tma_2d(st, &xmap_hi, &b_full[s], k * BK, n0);
                    tma_2d(st + b_part, &xmap_lo, &b_full[s], k * BK, n0);
                }
                sg.next();
            }
            // no copy may still be in flight when the CTA exits
            for (long long i = it - nbs > 0 ? it - nbs : 0; i < it; ++i)
                bar_wait_exit(&b_full[i % nbs], (uint32_t)((i / nbs) & 1), a.err);
        }
    } else if (warp == MMA_WARP) {
        // ---------------- MMA issue ----------------
        if (lane == 0) {
            long long it = 0, seg = 0;
            Seg sg;
            sg.start(u0, u1, nk);
            while (sg.valid() && ok) {
                const int n0 = (sg.t % a.NT) * BN;
                const int n_here = min(a.n_rows - n0, BN);
                const int n_mma = (n_here + 15) & ~15;
                const uint32_t idesc =
                    (1u << 4) | ((uint32_t)(n_mma >> 3) << 17) | ((uint32_t)(BM >> 4) << 24);
                if (seg > 0 && !bar_wait(&acc_empty, (uint32_t)((seg - 1) & 1), a.err, 33)) {
                    ok = false;
                    break;
                }
                tc_fence_after();
                for (int k = sg.ka; k < sg.kb; ++k, ++it) {
                    const int sa = (int)(it % ASTAGES), sb = (int)(it % nbs);
                    if (!bar_wait(&a_full[sa], (uint32_t)((it / ASTAGES) & 1), a.err, 34) ||
                        !bar_wait(&b_full[sb], (uint32_t)((it / nbs) & 1), a.err, 35)) {
                        ok = false;
                        break;
                    }
                    tc_fence_after();
                    const uint32_t bh = su32(bst + (size_t)sb * b_stage), bl = bh + (uint32_t)b_part;
                    const uint32_t ah = tmem + COL_A + (uint32_t)(64 * sa), al = ah + 32;
#pragma unroll
                    for (int kk = 0; kk < BK / 16; ++kk) {
                        mma_ta(tmem, ah + 8u * kk, desc_sw128(bh + 32u * kk), idesc,
                               (k > sg.ka || kk > 0) ? 1u : 0u);
                        mma_ta(tmem, ah + 8u * kk, desc_sw128(bl + 32u * kk), idesc, 1u);
                        mma_ta(tmem, al + 8u * kk, desc_sw128(bh + 32u * kk), idesc, 1u);
                    }
                    mma_commit(&a_empty[sa]);
                    mma_commit(&b_empty[sb]);
                }
                if (!ok) break;
                mma_commit(&acc_full);
                ++seg;
                sg.next();
            }
            // every MMA issued above has completed before TMEM is freed
            mma_commit(&done_bar);
            bar_wait_exit(&done_bar, 0, a.err);
        }
    } else if (warp >= DRAIN_WARP0) {
        // ---------------- drain: TMEM -> output or workspace ----------------
        // A STORE / ADD tile computed alone is written from TMEM with its
        // epilogue; the part of a shared tile, and every SiLU tile, goes to the
        // workspace for the output pass.  The accumulator is released right
        // after.
        const int q = warp & 3, m = q * 32 + lane;
        const uint32_t lane_base = tmem + ((uint32_t)(q * 32) << 16);
        sb_grid_wait();      // Y / workspace: after the previous grid
        long long seg = 0;
        Seg sg;
        sg.start(u0, u1, nk);
        while (sg.valid()) {
            const int t = sg.t, mt = t / a.NT, n0 = (t % a.NT) * BN;
            const int n_mma = (min(a.n_rows - n0, BN) + 15) & ~15;
            bool have = ok && bar_wait(&acc_full, (uint32_t)(seg & 1), a.err, 36);
            have = __all_sync(0xffffffffu, have);
            if (!have) ok = false;
            tc_fence_after();
            const bool alone = sg.ka == 0 && sg.kb == nk;
            if (have && alone && a.epi != SB_EPI_SILU && a.epi != SB_EPI_ROPE) {
                alone_out(a, lane_base, mt, n0, n_mma, m);
            } else if (have) {
                float4* wsp = (alone ? ws_tile(a.ws, C, t)
                                     : ws_slot(a.ws, c, u0 >= (long long)t * nk ? 0 : 1)) + m;
                for (int c0 = 0; c0 < n_mma; c0 += 16) {
                    float v[16];
                    tmem_ld16(lane_base + (uint32_t)c0, v);
                    const float u = a.wunscale;
#pragma unroll
                    for (int j = 0; j < 4; ++j)
                        wsp[(size_t)((c0 >> 2) + j) * BM] = make_float4(
                            v[4 * j] * u, v[4 * j + 1] * u, v[4 * j + 2] * u, v[4 * j + 3] * u);
                }
            }
            tc_fence_before();
            __syncwarp();
            if (lane == 0) bar_arrive(&acc_empty);
            ++seg;
            sg.next();
        }
    }

    tc_fence_before();
    __syncthreads();
    if (warp == MMA_WARP) {
        tc_fence_after();
        asm volatile("tcgen05.dealloc.cta_group::1.sync.aligned.b32 %0, %1;" ::"r"(tmem), "r"(512));
    }
}

int g_sms = 0;

}  // namespace

extern "C" size_t sb_sk_ws_floats(int max_silu_tiles) {
    int dev = 0, sms = 148;
    if (cudaGetDevice(&dev) == cudaSuccess)
        cudaDeviceGetAttribute(&sms, cudaDevAttrMultiProcessorCount, dev);
    return ((size_t)sms * 2 + (size_t)(max_silu_tiles > 0 ? max_silu_tiles : 0)) * BN * BM;
}

extern "C" int sb_sk_tiles(int M_pad, int n_rows) {
    return (M_pad / BM) * ((n_rows + BN - 1) / BN);
}

// Grid size and whether the output pass runs, as sb_sk_gemm decides them.
static bool sk_plan(int M_pad, int K, int n_rows, int epi, int* C_out, long long* U_out) {
    const int NT = (n_rows + BN - 1) / BN, nk = K / BK;
    const long long U = (long long)(M_pad / BM) * NT * nk;
    const int C = (int)(U < g_sms ? U : g_sms);
    bool pass = epi == SB_EPI_SILU || epi == SB_EPI_ROPE;
    for (int c = 1; c < C && !pass; ++c) pass = (U * c / C) % nk != 0;
    if (C_out) *C_out = C;
    if (U_out) *U_out = U;
    return pass;
}

extern "C" int sb_sk_kernels(int M_pad, int K, int n_rows, int epi) {
    if (!g_sms) sb_sk_prepare();
    return 1 + (sk_plan(M_pad, K, n_rows, epi, NULL, NULL) ? 1 : 0);
}

extern "C" void sb_sk_prepare(void) {
    cudaFuncSetAttribute(sk_kernel, cudaFuncAttributeMaxDynamicSharedMemorySize, (int)SMEM_MAX);
    int dev = 0;
    if (cudaGetDevice(&dev) == cudaSuccess)
        cudaDeviceGetAttribute(&g_sms, cudaDevAttrMultiProcessorCount, dev);
}

extern "C" int sb_sk_gemm(const sb_matrix* W, const sb_tc_operand* X, int n_rows, float* ws,
                          float* Y, int ldy, int epi, void* h_hi, void* h_lo, int ld16,
                          const sb_rope_args* rope, int* err, cudaStream_t st) {
    if (!W || !X || !X->lo || W->wtype != SB_WT_Q4K || W->M_pad % BM || W->K % 256 ||
        W->K != X->K || n_rows < 1 || n_rows > X->rows || !ws || !Y || !err ||
        (epi != SB_EPI_STORE && epi != SB_EPI_ADD && epi != SB_EPI_SILU && epi != SB_EPI_ROPE) ||
        (epi == SB_EPI_SILU && W->M % 128) || (h_hi && (!h_lo || epi != SB_EPI_SILU || ld16 < W->M / 2)))
        return -1;
    if (epi == SB_EPI_ROPE &&
        (!rope || rope->hd < 2 || rope->hd % 2 || BM % rope->hd ||
         W->M != (rope->nq + 2 * rope->nkv) * rope->hd || !rope->pool || !rope->row_pos ||
         !rope->row_slot || !rope->page_table || !rope->rope_cos || !rope->rope_sin))
        return -1;
    if (!g_sms) sb_sk_prepare();
    SkArgs a;
    a.W = (const unsigned char*)W->data;
    a.Y = Y;
    a.ws = ws;
    a.err = err;
    a.M = W->M;
    a.M_pad = W->M_pad;
    a.K = W->K;
    a.n_rows = n_rows;
    a.NT = (n_rows + BN - 1) / BN;
    a.n_box = X->n_box;
    a.ldy = ldy;
    a.epi = epi;
    a.h_hi = (__half*)h_hi;
    a.h_lo = (__half*)h_lo;
    a.ld16 = ld16;
    a.wscale = ldexpf(1.0f, W->wexp);
    a.wunscale = ldexpf(1.0f, -W->wexp);
    a.r = SkRope{};
    if (epi == SB_EPI_ROPE)
        a.r = SkRope{rope->row_pos, rope->row_slot, rope->page_table, rope->pool, rope->rope_cos,
                     rope->rope_sin, (long long)rope->n_pages, rope->max_pages, rope->layer,
                     rope->kv_dtype == SLATE_KV_F16, rope->nq, rope->nkv, rope->hd};
    const int MT = W->M_pad / BM;
    int C = 0;
    long long U = 0;
    // the output pass: every SiLU tile; shared tiles exist only when some CTA
    // boundary falls inside a tile
    const bool pass = sk_plan(W->M_pad, W->K, n_rows, epi, &C, &U);
    // Programmatic dependent launch (sb_pdl.h): the weight producers and the
    // MMA issuer touch nothing earlier kernels write and start at once; the x
    // loads and the drain wait for the previous grid.
    if (sb_launch_pdl(sk_kernel, dim3((unsigned)C), dim3(NTHREADS), sk_smem(X->n_box), st,
                      *(const CUtensorMap*)X->map_hi, *(const CUtensorMap*)X->map_lo, a) !=
        cudaSuccess)
        return -1;
    cudaError_t e = cudaSuccess;
    if (epi == SB_EPI_ROPE)
        e = sb_launch_pdl(sk_rope_out_kernel,
                          dim3((unsigned)(MT * a.NT), (unsigned)((min(n_rows, BN) + 3) / 4)), dim3(BM),
                          0, st, a, C, U);
    else if (pass && epi == SB_EPI_SILU)
        e = sb_launch_pdl(sk_silu_out_kernel, dim3((unsigned)(MT * a.NT), 4u), dim3(ST), 0, st, a, C,
                          U);
    else if (pass)
        e = sb_launch_pdl(sk_out_kernel,
                          dim3((unsigned)(MT * a.NT), (unsigned)((min(n_rows, BN) + 3) / 4)), dim3(BM),
                          0, st, a, C, U);
    if (e != cudaSuccess) return -1;
    return 0;
}
