// gemm_mv.cu -- Q4_K weight GEMM for small batches (1..16 activation rows):
// the weights stream from HBM once, the tensor cores (mma.sync m16n8k16) do
// the multiply-adds.
//
//   Y[n][m] (op)= sum_k X[n][k] * W[m][k]       n <= 16; op: store, residual
//                                               add, or SiLU(gate) * up
//
// Numerics follow the structure of the reference's Q4_K dot product
// (src/util/quant.c:210-304): per 32-element sub-block j of a super-block it
// forms sum(q * x) and sum(x) and combines them as
//     d * sc_j * sum(q * x) - dmin * m_j * sum(x).
// The 4-bit quants q (0..15) are exact in f16, so the tensor cores form
// sum(q * x) per sub-block with x as an f16 hi + lo pair (two MMAs; every
// product q * hi and q * lo is exact, the sums are f32), and the CUDA cores
// apply d * sc_j (exact in f32) and subtract dmin * m_j * sum(x) in f32.  No
// weight is dequantised to floating point, so the per-weight work is a mask,
// an OR and one packed f16 subtraction per two weights.  Each activation row
// is scaled by a power of two per K chunk (largest |x| just below 2^14) before
// the split, so small activations keep their low bits in the lo half; the
// scale is divided out exactly at the end.
//
// Work decomposition: a CTA (8 warps) owns 256 weight rows and a K chunk of
// KC columns (a multiple of 256); a warp owns 32 rows (two m16 tiles) and
// walks the chunk's super-blocks through a ring of two shared-memory stages
// (32 rows x 144 bytes each, copied with coalesced 16-byte cp.async, one
// super-block ahead of the one being computed; 16 warps per SM hide the
// rest).  Lane (g, t) reads 32-bit word t of every sub-block of rows g and
// g + 8 of each tile (bank-conflict
// free at the 144-byte row stride): the low nibbles of that word are the
// lane's four A elements of the sub-block's first MMA, the high nibbles those
// of its second, so every MMA covers exactly one sub-block (the k order inside
// a sub-block is permuted the same way in A and in the staged x fragments).
// The header of each row's super-block is decoded once per warp (lane l: row
// l) into shared memory.
// With more than one K chunk, each CTA writes its 256 x n partial sums to a
// workspace and the last CTA of the row block (an atomic counter; no CTA
// waits on another) sums the chunks in chunk order -- results do not depend
// on timing -- and applies the epilogue.
//
// The weights of the first super-block are requested before the grid waits
// for the previous kernel of the stream (programmatic dependent launch), so
// the weight stream starts while the producer of X finishes.
#include <cuda_fp16.h>

#include "sb_internal.h"
#include "sb_kernels.h"
#include "sb_pdl.h"

namespace {

constexpr int WARPS = 8;
constexpr int NTHREADS = 32 * WARPS;
constexpr int ROWS = 32 * WARPS;        // weight rows per CTA
constexpr int TROW = ROWS + 4;          // output tile row stride (floats): conflict-free stores
constexpr int SROW = 9;                 // scale scratch row stride (float2): conflict-free loads
constexpr int MAX_KC = 512;             // x fragments of a chunk: 16 KB of shared memory
constexpr int WSTAGES = 2;              // weight ring stages per warp
constexpr int WSTAGE = 32 * 144;        // bytes: 32 rows x one super-block

struct MvArgs {
    const unsigned char* W;
    int M, M_pad, K;
    const float* X;
    int ldx, n;
    float* Y;
    int ldy;
    float* ws;
    int* cnt;
    int KC, nkc;
};

// (1024 + n) with n in bits 0-3 / 16-19 -> exact n in both halves.
__device__ __forceinline__ uint32_t nib_lo(uint32_t q) {
    uint32_t h = (q & 0x000F000Fu) | 0x64006400u;
    __half2 r = __hsub2(*reinterpret_cast<__half2*>(&h), __half2half2(__ushort_as_half(0x6400)));
    return *reinterpret_cast<uint32_t*>(&r);
}
// (1024 + 16 n) with n in bits 4-7 / 20-23 -> (1024 + 16 n) / 16 - 64 = n, exact.
__device__ __forceinline__ uint32_t nib_hi(uint32_t q) {
    uint32_t h = (q & 0x00F000F0u) | 0x64006400u;
    __half2 r = __hfma2(*reinterpret_cast<__half2*>(&h), __half2half2(__ushort_as_half(0x2C00)),
                        __half2half2(__ushort_as_half(0xD400)));   // x * 1/16 - 64
    return *reinterpret_cast<uint32_t*>(&r);
}

__device__ __forceinline__ void mma16816(float (&d)[4], const uint32_t (&a)[4], uint32_t b0,
                                         uint32_t b1) {
    asm("mma.sync.aligned.m16n8k16.row.col.f32.f16.f16.f32 {%0,%1,%2,%3}, {%4,%5,%6,%7}, "
        "{%8,%9}, {%0,%1,%2,%3};"
        : "+f"(d[0]), "+f"(d[1]), "+f"(d[2]), "+f"(d[3])
        : "r"(a[0]), "r"(a[1]), "r"(a[2]), "r"(a[3]), "r"(b0), "r"(b1));
}

__device__ __forceinline__ float byte_f(uint32_t w, int i) { return (float)((w >> (8 * i)) & 0xffu); }

// Effective scale d*sc_j and min dmin*m_j of the 8 sub-blocks of a super-block
// header (f16 d, f16 dmin, 12 packed 6-bit scale / min bytes;
// src/util/quant.c:157-166).
__device__ __forceinline__ void decode_header(uint4 h, float2* out) {
    const float d = __half2float(__ushort_as_half((unsigned short)(h.x & 0xffffu)));
    const float dmin = __half2float(__ushort_as_half((unsigned short)(h.x >> 16)));
    const uint32_t sc03 = h.y & 0x3F3F3F3Fu, m03 = h.z & 0x3F3F3F3Fu;
    const uint32_t sc47 = (h.w & 0x0F0F0F0Fu) | ((h.y >> 2) & 0x30303030u);
    const uint32_t m47 = ((h.w >> 4) & 0x0F0F0F0Fu) | ((h.z >> 2) & 0x30303030u);
#pragma unroll
    for (int i = 0; i < 4; ++i) {
        out[i] = make_float2(d * byte_f(sc03, i), dmin * byte_f(m03, i));
        out[4 + i] = make_float2(d * byte_f(sc47, i), dmin * byte_f(m47, i));
    }
}

__device__ __forceinline__ float silu_mul(float g, float u) { return g / (1.0f + expf(-g)) * u; }

__device__ __forceinline__ void cp_async16(void* dst, const void* src) {
    const unsigned d = (unsigned)__cvta_generic_to_shared(dst);
    asm volatile("cp.async.cg.shared.global [%0], [%1], 16;" ::"r"(d), "l"(src) : "memory");
}
__device__ __forceinline__ void cp_commit() { asm volatile("cp.async.commit_group;" ::: "memory"); }
template <int N>
__device__ __forceinline__ void cp_wait() { asm volatile("cp.async.wait_group %0;" ::"n"(N) : "memory"); }

// Super-block kb of the warp's 32 rows -> stage (row r at r * 144): 288
// 16-byte pieces, 9 per lane, consecutive lanes on consecutive pieces (piece
// i = 9 r + c lands at 16 i; off[k] is its offset in the matrix).
__device__ __forceinline__ void stage_weights(unsigned char* stage, const unsigned char* wrow0,
                                              const uint32_t (&off)[9], int kb, int lane) {
    const unsigned char* src = wrow0 + (size_t)kb * 144;
#pragma unroll
    for (int k = 0; k < 9; ++k) cp_async16(stage + 16 * (lane + 32 * k), src + off[k]);
}

template <int NT, int EPI>
__global__ void __launch_bounds__(NTHREADS, 2) mv_kernel(const MvArgs a) {
    extern __shared__ __align__(16) unsigned char smem[];
    const int KC = a.KC;
    const int nsub = KC / 32;
    uint4* xf = reinterpret_cast<uint4*>(smem);                               // [nsub][2][NT][32]
    float* xs = reinterpret_cast<float*>(smem + (size_t)nsub * 2 * NT * 512);  // [nsub][8 NT]
    float2* sc = reinterpret_cast<float2*>(xs + nsub * 8 * NT);               // [WARPS][32][SROW]
    float* cs = reinterpret_cast<float*>(sc + WARPS * 32 * SROW);             // [8 NT] x scale
    unsigned char* ring = reinterpret_cast<unsigned char*>(cs + 16);          // [WARPS][WSTAGES][WSTAGE]
    float* tile = reinterpret_cast<float*>(smem);                             // [8 NT][TROW], after the loop
    __shared__ int s_last;
    __shared__ int rmax[16];

    const int tid = threadIdx.x, warp = tid >> 5, lane = tid & 31;
    const int g = lane >> 2, t = lane & 3;
    const int rb = blockIdx.x, kc = blockIdx.y;
    const int row0 = rb * ROWS;
    const int k0 = kc * KC;
    const size_t rbytes = (size_t)(a.K / 256) * 144;
    const unsigned char* wrow0 = a.W + (size_t)(row0 + 32 * warp) * rbytes;
    const int kb0 = k0 / 256, nsb = KC / 256;
    const bool wvalid = row0 + 32 * warp < a.M_pad;   // the last CTA may hold 128 rows only
    uint32_t off[9];
#pragma unroll
    for (int k = 0; k < 9; ++k) {
        const int i = lane + 32 * k, r = i / 9;
        off[k] = (uint32_t)(r * rbytes + 16 * (i - 9 * r));
    }

    // weights of the first two super-blocks: independent of the previous kernel
    unsigned char* wring = ring + (size_t)warp * WSTAGES * WSTAGE;
#pragma unroll
    for (int p = 0; p < WSTAGES - 1; ++p) {
        if (wvalid && p < nsb) stage_weights(wring + p * WSTAGE, wrow0, off, kb0 + p, lane);
        cp_commit();
    }
    sb_grid_release();
    sb_grid_wait();

    // ---- activations of the chunk: per-row power-of-two scale, f16 hi/lo
    // fragments in MMA order, sub-block sums.  A thread's float4s of the chunk
    // (rows < n; at most 16: 8 NT rows x KC / 4) are all requested at once.
    constexpr int U = (8 * NT * (MAX_KC / NT) / 4 + NTHREADS - 1) / NTHREADS;
    const int q4 = KC / 4, total = a.n * q4;
    for (int i = tid; i < nsub * 2 * NT * 32; i += NTHREADS) xf[i] = make_uint4(0u, 0u, 0u, 0u);
    for (int i = tid; i < nsub * 8 * NT; i += NTHREADS) xs[i] = 0.f;
    if (tid < 8 * NT) rmax[tid] = 0;
    float4 v[U];
#pragma unroll
    for (int u = 0; u < U; ++u) {
        const int f = tid + NTHREADS * u;
        if (f < total) {
            const int c = f / q4, e = 4 * (f - c * q4);
            v[u] = *reinterpret_cast<const float4*>(a.X + (size_t)c * a.ldx + k0 + e);
        }
    }
    __syncthreads();
#pragma unroll
    for (int u = 0; u < U; ++u) {
        const int f = tid + NTHREADS * u;
        if (f < total) {
            const float m = fmaxf(fmaxf(fabsf(v[u].x), fabsf(v[u].y)), fmaxf(fabsf(v[u].z), fabsf(v[u].w)));
            atomicMax(&rmax[f / q4], __float_as_int(m));     // m >= 0: int order = float order
        }
    }
    __syncthreads();
    if (tid < 8 * NT) {
        const float m = __int_as_float(rmax[tid]);
        int e = 0;
        const bool ok = m > 0.f && m <= 3.0e38f;
        if (ok) {
            frexpf(m, &e);                       // m < 2^e
            e = max(-100, min(100, e));
        }
        cs[tid] = ok ? ldexpf(1.0f, 14 - e) : 1.0f;
    }
    __syncthreads();
#pragma unroll
    for (int u = 0; u < U; ++u) {
        const int f = tid + NTHREADS * u;
        // the 8 float4s of a sub-block sit in 8 consecutive lanes (q4 % 8 == 0),
        // all inside or all outside the chunk
        float ps = 0.f;
        int c = 0, e = 0;
        if (f < total) {
            c = f / q4;
            e = 4 * (f - c * q4);
            const float sc_ = cs[c];
            float4 x = v[u];
            x.x *= sc_; x.y *= sc_; x.z *= sc_; x.w *= sc_;
            ps = ((x.x + x.y) + x.z) + x.w;
            // k slots (2t, 2t+1) <- elements (0, 2); (2t+8, 2t+9) <- (1, 3)
            __half2 h02 = __floats2half2_rn(x.x, x.z), h13 = __floats2half2_rn(x.y, x.w);
            float2 r02 = __half22float2(h02), r13 = __half22float2(h13);
            __half2 l02 = __floats2half2_rn(x.x - r02.x, x.z - r02.y);
            __half2 l13 = __floats2half2_rn(x.y - r13.x, x.w - r13.y);
            uint4 fr;
            fr.x = *reinterpret_cast<uint32_t*>(&h02);
            fr.y = *reinterpret_cast<uint32_t*>(&h13);
            fr.z = *reinterpret_cast<uint32_t*>(&l02);
            fr.w = *reinterpret_cast<uint32_t*>(&l13);
            // fragment (2 * sub + half, nt, lane g * 4 + t) holds x[nt * 8 + g][16 * hs + 4 t ..]
            xf[((e >> 4) * NT + (c >> 3)) * 32 + (c & 7) * 4 + ((e >> 2) & 3)] = fr;
        }
        ps += __shfl_xor_sync(0xffffffffu, ps, 1);
        ps += __shfl_xor_sync(0xffffffffu, ps, 2);
        ps += __shfl_xor_sync(0xffffffffu, ps, 4);
        if (f < total && (lane & 7) == 0) xs[(e >> 5) * 8 * NT + c] = ps;
    }
    __syncthreads();

    float acc[2][NT][4];
#pragma unroll
    for (int rt = 0; rt < 2; ++rt)
#pragma unroll
        for (int nt = 0; nt < NT; ++nt)
#pragma unroll
            for (int c = 0; c < 4; ++c) acc[rt][nt][c] = 0.f;

    float2* wsc = sc + warp * 32 * SROW;
    for (int sb = 0; sb < (wvalid ? nsb : 0); ++sb) {
        cp_wait<WSTAGES - 2>();   // this lane's pieces of super-block sb have landed
        __syncwarp();             // ... and every lane's; stage (sb - 1) is free again
        if (sb + WSTAGES - 1 < nsb)
            stage_weights(wring + ((sb + WSTAGES - 1) % WSTAGES) * WSTAGE, wrow0, off,
                          kb0 + sb + WSTAGES - 1, lane);
        cp_commit();
        const unsigned char* cur = wring + (sb % WSTAGES) * WSTAGE;
        float2 dm[8];
        decode_header(*reinterpret_cast<const uint4*>(cur + lane * 144), dm);
#pragma unroll
        for (int j = 0; j < 8; ++j) wsc[lane * SROW + j] = dm[j];
        __syncwarp();
#pragma unroll
        for (int j = 0; j < 8; ++j) {
            const int sub = sb * 8 + j;
            uint4 xb[2][NT];
            float2 xsum[NT];
#pragma unroll
            for (int hs = 0; hs < 2; ++hs)
#pragma unroll
                for (int nt = 0; nt < NT; ++nt) xb[hs][nt] = xf[((2 * sub + hs) * NT + nt) * 32 + lane];
#pragma unroll
            for (int nt = 0; nt < NT; ++nt)
                xsum[nt] = *reinterpret_cast<const float2*>(xs + sub * 8 * NT + nt * 8 + 2 * t);
#pragma unroll
            for (int rt = 0; rt < 2; ++rt) {
                const uint32_t q0 = *reinterpret_cast<const uint32_t*>(
                    cur + (16 * rt + g) * 144 + 16 + 16 * j + 4 * t);
                const uint32_t q1 = *reinterpret_cast<const uint32_t*>(
                    cur + (16 * rt + g + 8) * 144 + 16 + 16 * j + 4 * t);
                const uint32_t q0s = q0 >> 8, q1s = q1 >> 8;
                const uint32_t alo[4] = {nib_lo(q0), nib_lo(q1), nib_lo(q0s), nib_lo(q1s)};
                const uint32_t ahi[4] = {nib_hi(q0), nib_hi(q1), nib_hi(q0s), nib_hi(q1s)};
                const float2 s0 = wsc[(16 * rt + g) * SROW + j];
                const float2 s1 = wsc[(16 * rt + g + 8) * SROW + j];
#pragma unroll
                for (int nt = 0; nt < NT; ++nt) {
                    float d[4] = {0.f, 0.f, 0.f, 0.f};
                    mma16816(d, alo, xb[0][nt].x, xb[0][nt].y);
                    mma16816(d, alo, xb[0][nt].z, xb[0][nt].w);
                    mma16816(d, ahi, xb[1][nt].x, xb[1][nt].y);
                    mma16816(d, ahi, xb[1][nt].z, xb[1][nt].w);
                    acc[rt][nt][0] = fmaf(s0.x, d[0], fmaf(-s0.y, xsum[nt].x, acc[rt][nt][0]));
                    acc[rt][nt][1] = fmaf(s0.x, d[1], fmaf(-s0.y, xsum[nt].y, acc[rt][nt][1]));
                    acc[rt][nt][2] = fmaf(s1.x, d[2], fmaf(-s1.y, xsum[nt].x, acc[rt][nt][2]));
                    acc[rt][nt][3] = fmaf(s1.x, d[3], fmaf(-s1.y, xsum[nt].y, acc[rt][nt][3]));
                }
            }
        }
    }
    cp_wait<0>();

    // ---- partial sums of the CTA -> tile[col][row] (x scale divided out)
    __syncthreads();   // the x fragments are dead; the tile reuses their space
#pragma unroll
    for (int rt = 0; rt < 2; ++rt)
#pragma unroll
        for (int nt = 0; nt < NT; ++nt)
#pragma unroll
            for (int c = 0; c < 4; ++c) {
                const int col = nt * 8 + 2 * t + (c & 1);
                const int r = 32 * warp + 16 * rt + g + 8 * (c >> 1);
                tile[col * TROW + r] = acc[rt][nt][c] / cs[col];
            }
    __syncthreads();

    if (a.nkc > 1) {
        // write this chunk's part; the last CTA of the row block sums them
        float* part = a.ws + ((size_t)kc * gridDim.x + rb) * (8 * NT) * ROWS;
        for (int col = 0; col < a.n; ++col) part[col * ROWS + tid] = tile[col * TROW + tid];
        // the CTA's writes reach thread 0 through the barrier; its GPU-scope
        // fence orders them (cumulatively) before the count, and after the
        // count for the CTA that finishes the row block
        __syncthreads();
        if (tid == 0) {
            __threadfence();
            s_last = atomicAdd(&a.cnt[rb], 1) == a.nkc - 1;
            if (s_last) __threadfence();
        }
        __syncthreads();
        if (!s_last) return;
        float sum[8 * NT];
#pragma unroll
        for (int col = 0; col < 8 * NT; ++col) sum[col] = 0.f;
        for (int c0 = 0; c0 < a.nkc; c0 += 4) {      // chunk order; 4 x 8 NT loads in flight
            float pv[4][8 * NT];
#pragma unroll
            for (int cc = 0; cc < 4; ++cc)
#pragma unroll
                for (int col = 0; col < 8 * NT; ++col)
                    pv[cc][col] = (c0 + cc < a.nkc && col < a.n)
                                      ? __ldcg(a.ws + (((size_t)(c0 + cc) * gridDim.x + rb) * (8 * NT) +
                                                       col) * ROWS + tid)
                                      : 0.f;
#pragma unroll
            for (int cc = 0; cc < 4; ++cc)
#pragma unroll
                for (int col = 0; col < 8 * NT; ++col) sum[col] += pv[cc][col];
        }
#pragma unroll
        for (int col = 0; col < 8 * NT; ++col)
            if (col < a.n) tile[col * TROW + tid] = sum[col];
        if (tid == 0) a.cnt[rb] = 0;     // every CTA of the row block has counted
        __syncthreads();
    }

    // ---- epilogue: thread = row of the block (SiLU: output of the block)
    if (EPI == SB_EPI_SILU) {
        // 128-row groups (gate rows 0-63, up rows 64-127): ROWS / 2 outputs
        if (tid < ROWS / 2) {
            const int o = rb * (ROWS / 2) + tid;
            const int gr = (tid / 64) * 128 + tid % 64;
            if (o < a.M / 2)
                for (int col = 0; col < a.n; ++col)
                    a.Y[(size_t)col * a.ldy + o] =
                        silu_mul(tile[col * TROW + gr], tile[col * TROW + gr + 64]);
        }
    } else {
        const int m = row0 + tid;
        if (m < a.M)
            for (int col = 0; col < a.n; ++col) {
                float* y = a.Y + (size_t)col * a.ldy + m;
                const float v = tile[col * TROW + tid];
                *y = EPI == SB_EPI_ADD ? *y + v : v;
            }
    }
}

size_t mv_smem(int KC, int NT) {
    const size_t nsub = KC / 32;
    size_t loop = nsub * 2 * NT * 512 + nsub * 8 * NT * 4 + WARPS * 32 * SROW * 8 + 16 * 4 +
                  (size_t)WARPS * WSTAGES * WSTAGE;
    size_t out = (size_t)8 * NT * TROW * 4;
    return loop > out ? loop : out;
}

// K chunk: s super-blocks, s dividing K / 256, at most MAX_KC / NT columns;
// the s with the least (waves of 2 CTAs per SM) x (s + 1 super-block times,
// the one for staging x and the partial sums), larger s on ties.
int mv_plan(int M_pad, int K, int NT) {
    const long slots = 2L * 148;
    const int blocks = (M_pad + ROWS - 1) / ROWS, nsb = K / 256, kmax = MAX_KC / NT / 256;
    int best = 0;
    long best_cost = 0;
    for (int s = 1; s <= nsb && s <= kmax; ++s) {
        if (nsb % s) continue;
        const long ctas = (long)blocks * (nsb / s);
        const long cost = (ctas + slots - 1) / slots * (s + 1);
        if (best == 0 || cost <= best_cost) {
            best = s;
            best_cost = cost;
        }
    }
    return best * 256;
}

template <int NT, int EPI>
int launch(const MvArgs& a, int blocks, cudaStream_t st) {
    const size_t smem = mv_smem(a.KC, NT);
    static unsigned long long ready = 0;     // per device ordinal (< 64)
    int dev = 0;
    if (cudaGetDevice(&dev) != cudaSuccess || dev < 0 || dev >= 64) return -1;
    if (!(__atomic_load_n(&ready, __ATOMIC_RELAXED) >> dev & 1ull)) {
        if (cudaFuncSetAttribute(mv_kernel<NT, EPI>, cudaFuncAttributeMaxDynamicSharedMemorySize,
                                 (int)mv_smem(MAX_KC / NT, NT)) != cudaSuccess)
            return -1;
        __atomic_fetch_or(&ready, 1ull << dev, __ATOMIC_RELAXED);
    }
    return sb_launch_pdl(mv_kernel<NT, EPI>, dim3(blocks, a.nkc), dim3(NTHREADS), smem, st, a) ==
                   cudaSuccess
               ? 0
               : -1;
}

template <int NT>
int dispatch(const MvArgs& a, int blocks, int epi, cudaStream_t st) {
    switch (epi) {
        case SB_EPI_STORE: return launch<NT, SB_EPI_STORE>(a, blocks, st);
        case SB_EPI_ADD: return launch<NT, SB_EPI_ADD>(a, blocks, st);
        case SB_EPI_SILU: return launch<NT, SB_EPI_SILU>(a, blocks, st);
    }
    return -1;
}

}  // namespace

extern "C" size_t sb_mv_ws_floats(int M_pad, int K) {
    if (M_pad % 128 || K % 256) return 0;
    const size_t blocks = (M_pad + ROWS - 1) / ROWS;
    size_t best = 0;
    for (int NT = 1; NT <= 2; ++NT) {
        const int KC = mv_plan(M_pad, K, NT);
        const size_t f = (size_t)(K / KC) * blocks * ROWS * 8 * NT;
        if (f > best) best = f;
    }
    return best;
}

extern "C" int sb_mv_gemm(const sb_matrix* W, const float* X, int ldx, int n, float* Y, int ldy,
                          int epi, float* ws, int* cnt, cudaStream_t st) {
    if (!W || !X || !Y || !ws || !cnt || n < 1 || n > SB_MV_MAX_ROWS) return -1;
    if (W->wtype != SB_WT_Q4K || W->K % 256 || W->M_pad % 128 || ldx % 4 ||
        (reinterpret_cast<uintptr_t>(X) & 15))
        return -1;
    const int NT = n <= 8 ? 1 : 2;
    MvArgs a;
    a.W = static_cast<const unsigned char*>(W->data);
    a.M = W->M;
    a.M_pad = W->M_pad;
    a.K = W->K;
    a.X = X;
    a.ldx = ldx;
    a.n = n;
    a.Y = Y;
    a.ldy = ldy;
    a.ws = ws;
    a.cnt = cnt;
    a.KC = mv_plan(W->M_pad, W->K, NT);
    if (a.KC == 0) return -1;
    a.nkc = W->K / a.KC;
    const int blocks = (W->M_pad + ROWS - 1) / ROWS;
    return NT == 1 ? dispatch<1>(a, blocks, epi, st) : dispatch<2>(a, blocks, epi, st);
}
