// gemm_cc.cu -- Q4_K / f32 weight GEMMs on the CUDA cores (sm_100a).
//
//   Y[n][m] (epi)= sum_k X[n][k] * W[m][k]      n < B (batch rows), m < M
//
// This is the batched form of the reference's matvec_q4k / matvec entries
// (src/backend/backend_cpu.c:33-36, 44-46 -> src/util/quant.c:306-313): the
// same row-major [out, in] weights, applied to B activation rows at once so
// each weight byte is read from HBM once per step instead of once per row.
//
// Two kernels:
//   * gemv_kernel  (B <= 8): weight-bandwidth bound.  A warp owns 4 weight
//     rows; lane l covers 8 weights of every Q4_K super-block (sub-block l/4,
//     32-bit word l%4 of its 16 nibble bytes), so a warp reads each block's
//     128 nibble bytes as one coalesced 128-byte line.  Activations come
//     through L1 and are reused across the 4 rows.
//   * gemm_tiled   (B > 8): 128 weight rows x BN batch rows per CTA, K in
//     32-element steps (one Q4_K sub-block).  Warps 0-3 dequantise the
//     sub-block (d*sc*q - dmin*mn, the reference's reconstruction,
//     util/quant.c:187-199) into shared memory, warps 4-7 stage activations;
//     all 8 warps run an 8x8 (or 8x4) register tile.  Double-buffered.
//
// Numerics: f32 products, f32 accumulation; dequantised weights are exactly
// the reference's f32 reconstruction.
#include "sb_kernels.h"
#include "sb_internal.h"
#include <cuda_fp16.h>

namespace {

__device__ __forceinline__ float f16_lo(uint32_t w) {
    return __half2float(__ushort_as_half((unsigned short)(w & 0xffffu)));
}
__device__ __forceinline__ float f16_hi(uint32_t w) {
    return __half2float(__ushort_as_half((unsigned short)(w >> 16)));
}
__device__ __forceinline__ uint32_t byte_of(uint4 h, int i) {  // scales byte i (0..11)
    uint32_t w = i < 4 ? h.y : (i < 8 ? h.z : h.w);
    return (w >> ((i & 3) * 8)) & 0xffu;
}
// Sub-block j's effective scale and min from a block header
// (bytes 0..15: f16 d, f16 dmin, 12 packed scale bytes; util/quant.c:157-166).
__device__ __forceinline__ void q4k_sub(uint4 h, int j, float& sd, float& sm) {
    float d = f16_lo(h.x), dmin = f16_hi(h.x);
    uint32_t sc, mn;
    if (j < 4) {
        sc = byte_of(h, j) & 63u;
        mn = byte_of(h, j + 4) & 63u;
    } else {
        sc = (byte_of(h, j + 4) & 15u) | ((byte_of(h, j - 4) >> 6) << 4);
        mn = (byte_of(h, j + 4) >> 4) | ((byte_of(h, j) >> 6) << 4);
    }
    sd = d * (float)sc;
    sm = dmin * (float)mn;
}

__device__ __forceinline__ float silu_mul1(float g, float u) { return g / (1.0f + expf(-g)) * u; }

// ------------------------------------------------------------------------
// GEMV: NB batch rows (1..8), 4 weight rows per warp.
// For EPI == SILU the warp's 4 rows are 2 (gate, up) pairs -> 2 outputs.
template <int WT, int NB, int EPI>
__global__ void __launch_bounds__(256) gemv_kernel(sb_matrix W, const float* __restrict__ X,
                                                   int ldx, float* __restrict__ Y, int ldy) {
    constexpr int R = 4;
    const int lane = threadIdx.x & 31;
    const long warp = (long)blockIdx.x * 8 + (threadIdx.x >> 5);
    long rows[R];
    if (EPI == SB_EPI_SILU) {
        // outputs o0 = 2*warp, o1 = 2*warp+1; gate row of output o is
        // (o/64)*128 + o%64 and its up row sits 64 rows later.
        for (int p = 0; p < 2; ++p) {
            long o = 2 * warp + p;
            long g = (o / 64) * 128 + (o % 64);
            rows[2 * p] = g;
            rows[2 * p + 1] = g + 64;
        }
    } else {
        for (int r = 0; r < R; ++r) rows[r] = warp * R + r;
    }
    bool live[R];
    for (int r = 0; r < R; ++r) live[r] = rows[r] < W.M_pad;
    if (!live[0]) return;

    float acc[R][NB];
#pragma unroll
    for (int r = 0; r < R; ++r)
#pragma unroll
        for (int b = 0; b < NB; ++b) acc[r][b] = 0.f;

    if (WT == SB_WT_Q4K) {
        const int nblk = W.K / 256;
        const size_t rb = (size_t)nblk * 144;
        const int j = lane >> 2, wd = lane & 3;
        const unsigned char* base = (const unsigned char*)W.data;
        for (int kb = 0; kb < nblk; ++kb) {
            float xa[NB][8];
            const int k0 = kb * 256 + 32 * j + 4 * wd;
#pragma unroll
            for (int b = 0; b < NB; ++b) {
                float4 a = *(const float4*)(X + (size_t)b * ldx + k0);
                float4 c = *(const float4*)(X + (size_t)b * ldx + k0 + 16);
                xa[b][0] = a.x; xa[b][1] = a.y; xa[b][2] = a.z; xa[b][3] = a.w;
                xa[b][4] = c.x; xa[b][5] = c.y; xa[b][6] = c.z; xa[b][7] = c.w;
            }
#pragma unroll
            for (int r = 0; r < R; ++r) {
                if (!live[r]) continue;
                const unsigned char* blk = base + (size_t)rows[r] * rb + (size_t)kb * 144;
                uint4 h = __ldg((const uint4*)blk);
                uint32_t q = __ldg((const uint32_t*)(blk + 16 + 16 * j + 4 * wd));
                float sd, sm;
                q4k_sub(h, j, sd, sm);
                float w[8];
#pragma unroll
                for (int i = 0; i < 4; ++i) {
                    w[i] = sd * (float)((q >> (8 * i)) & 15u) - sm;
                    w[4 + i] = sd * (float)((q >> (8 * i + 4)) & 15u) - sm;
                }
#pragma unroll
                for (int b = 0; b < NB; ++b)
#pragma unroll
                    for (int i = 0; i < 8; ++i) acc[r][b] = fmaf(w[i], xa[b][i], acc[r][b]);
            }
        }
    } else {
        const float* base = (const float*)W.data;
        for (int k0 = lane * 4; k0 < W.ldw; k0 += 128) {
            float4 xa[NB];
#pragma unroll
            for (int b = 0; b < NB; ++b) xa[b] = *(const float4*)(X + (size_t)b * ldx + k0);
#pragma unroll
            for (int r = 0; r < R; ++r) {
                if (!live[r]) continue;
                float4 w = __ldg((const float4*)(base + (size_t)rows[r] * W.ldw + k0));
#pragma unroll
                for (int b = 0; b < NB; ++b) {
                    acc[r][b] = fmaf(w.x, xa[b].x, acc[r][b]);
                    acc[r][b] = fmaf(w.y, xa[b].y, acc[r][b]);
                    acc[r][b] = fmaf(w.z, xa[b].z, acc[r][b]);
                    acc[r][b] = fmaf(w.w, xa[b].w, acc[r][b]);
                }
            }
        }
    }
#pragma unroll
    for (int r = 0; r < R; ++r)
#pragma unroll
        for (int b = 0; b < NB; ++b)
#pragma unroll
            for (int o = 16; o > 0; o >>= 1) acc[r][b] += __shfl_xor_sync(0xffffffffu, acc[r][b], o);
    if (lane != 0) return;
    if (EPI == SB_EPI_SILU) {
        for (int p = 0; p < 2; ++p) {
            long o = 2 * warp + p;
            if (!live[2 * p] || o >= W.M / 2) continue;
            for (int b = 0; b < NB; ++b)
                Y[(size_t)b * ldy + o] = silu_mul1(acc[2 * p][b], acc[2 * p + 1][b]);
        }
    } else {
        for (int r = 0; r < R; ++r) {
            if (!live[r] || rows[r] >= W.M) continue;
            for (int b = 0; b < NB; ++b) {
                float* y = Y + (size_t)b * ldy + rows[r];
                *y = (EPI == SB_EPI_ADD) ? *y + acc[r][b] : acc[r][b];
            }
        }
    }
}

// ------------------------------------------------------------------------
// Tiled GEMM: 128 weight rows x BN batch rows per CTA, 256 threads.
template <int WT, int BN, int EPI>
__global__ void __launch_bounds__(256) gemm_tiled(sb_matrix W, const float* __restrict__ X,
                                                  int ldx, int B, float* __restrict__ Y, int ldy) {
    constexpr int BM = 128, BK = 32;
    constexpr int TN = BN / 16;            // n values per thread (8 or 4)
    constexpr int XCH = 8 * BN / 128;      // float4 chunks of X per loader thread
    extern __shared__ float4 smem4[];
    float* smem = (float*)smem4;
    float* As = smem;                      // [2][BK][BM]
    float* Xs = smem + 2 * BK * BM;        // [2][BK][BN]

    const int tid = threadIdx.x;
    const int tx = tid & 15, ty = tid >> 4;
    const long m0 = (long)blockIdx.x * BM;
    const long n0 = (long)blockIdx.y * BN;
    const int nsteps = (WT == SB_WT_Q4K) ? W.K / BK : W.ldw / BK;

    // register staging for the next k-step
    uint4 rh = make_uint4(0, 0, 0, 0), rq = make_uint4(0, 0, 0, 0);
    float4 ra[8];
    float4 rx[XCH];
    const bool a_loader = tid < 128;
    const long arow = m0 + tid;
    const bool arow_ok = a_loader && arow < W.M_pad;
    const int xt = tid - 128;
    const int xn = a_loader ? 0 : (xt % BN);
    const int xc0 = a_loader ? 0 : (xt / BN) * XCH;
    const bool xrow_ok = !a_loader && (n0 + xn) < B;

    auto load = [&](int s) {
        if (a_loader) {
            if (WT == SB_WT_Q4K) {
                if (arow_ok) {
                    const unsigned char* blk = (const unsigned char*)W.data +
                                               (size_t)arow * (size_t)(W.K / 256) * 144 +
                                               (size_t)(s >> 3) * 144;
                    rh = __ldg((const uint4*)blk);
                    rq = __ldg((const uint4*)(blk + 16 + 16 * (s & 7)));
                } else {
                    rh = make_uint4(0, 0, 0, 0);
                    rq = make_uint4(0, 0, 0, 0);
                }
            } else {
                const float* src = (const float*)W.data + (size_t)arow * W.ldw + (size_t)s * BK;
#pragma unroll
                for (int c = 0; c < 8; ++c)
                    ra[c] = arow_ok ? __ldg((const float4*)(src + 4 * c)) : make_float4(0, 0, 0, 0);
            }
        } else {
            const float* src = X + (size_t)(n0 + xn) * ldx + (size_t)s * BK;
#pragma unroll
            for (int c = 0; c < XCH; ++c)
                rx[c] = xrow_ok ? *(const float4*)(src + 4 * (xc0 + c)) : make_float4(0, 0, 0, 0);
        }
    };
    auto store = [&](int s, int buf) {
        if (a_loader) {
            float* as = As + buf * BK * BM + tid;
            if (WT == SB_WT_Q4K) {
                float sd, sm;
                q4k_sub(rh, s & 7, sd, sm);
                uint32_t q[4] = {rq.x, rq.y, rq.z, rq.w};
#pragma unroll
                for (int i = 0; i < 16; ++i) {
                    uint32_t b = (q[i >> 2] >> ((i & 3) * 8)) & 0xffu;
                    as[i * BM] = sd * (float)(b & 15u) - sm;
                    as[(i + 16) * BM] = sd * (float)(b >> 4) - sm;
                }
            } else {
#pragma unroll
                for (int c = 0; c < 8; ++c) {
                    as[(4 * c + 0) * BM] = ra[c].x;
                    as[(4 * c + 1) * BM] = ra[c].y;
                    as[(4 * c + 2) * BM] = ra[c].z;
                    as[(4 * c + 3) * BM] = ra[c].w;
                }
            }
        } else {
            float* xs = Xs + buf * BK * BN + xn;
#pragma unroll
            for (int c = 0; c < XCH; ++c) {
                int k = 4 * (xc0 + c);
                xs[(k + 0) * BN] = rx[c].x;
                xs[(k + 1) * BN] = rx[c].y;
                xs[(k + 2) * BN] = rx[c].z;
                xs[(k + 3) * BN] = rx[c].w;
            }
        }
    };

    float acc[8][TN];
#pragma unroll
    for (int i = 0; i < 8; ++i)
#pragma unroll
        for (int j = 0; j < TN; ++j) acc[i][j] = 0.f;

    load(0);
    store(0, 0);
    __syncthreads();
    for (int s = 0; s < nsteps; ++s) {
        const int buf = s & 1;
        if (s + 1 < nsteps) load(s + 1);
        const float* as = As + buf * BK * BM;
        const float* xs = Xs + buf * BK * BN;
#pragma unroll 8
        for (int kk = 0; kk < BK; ++kk) {
            float4 a0 = *(const float4*)(as + kk * BM + ty * 4);
            float4 a1 = *(const float4*)(as + kk * BM + 64 + ty * 4);
            float a[8] = {a0.x, a0.y, a0.z, a0.w, a1.x, a1.y, a1.z, a1.w};
            float x[TN];
            float4 b0 = *(const float4*)(xs + kk * BN + tx * 4);
            x[0] = b0.x; x[1] = b0.y; x[2] = b0.z; x[3] = b0.w;
            if (TN == 8) {
                float4 b1 = *(const float4*)(xs + kk * BN + BN / 2 + tx * 4);
                x[4 % TN] = b1.x; x[5 % TN] = b1.y; x[6 % TN] = b1.z; x[7 % TN] = b1.w;
            }
#pragma unroll
            for (int i = 0; i < 8; ++i)
#pragma unroll
                for (int j = 0; j < TN; ++j) acc[i][j] = fmaf(a[i], x[j], acc[i][j]);
        }
        if (s + 1 < nsteps) store(s + 1, buf ^ 1);
        __syncthreads();
    }

    // epilogue
#pragma unroll
    for (int j = 0; j < TN; ++j) {
        const long n = n0 + (j < 4 ? tx * 4 + j : BN / 2 + tx * 4 + (j - 4));
        if (n >= B) continue;
        float* yrow = Y + (size_t)n * ldy;
        if (EPI == SB_EPI_SILU) {
            const long o0 = m0 / 2 + ty * 4;
#pragma unroll
            for (int i = 0; i < 4; ++i)
                if (o0 + i < W.M / 2) yrow[o0 + i] = silu_mul1(acc[i][j], acc[4 + i][j]);
        } else {
#pragma unroll
            for (int h = 0; h < 2; ++h) {
                const long mb = m0 + h * 64 + ty * 4;
#pragma unroll
                for (int i = 0; i < 4; ++i) {
                    if (mb + i >= W.M) continue;
                    float v = acc[h * 4 + i][j];
                    yrow[mb + i] = (EPI == SB_EPI_ADD) ? yrow[mb + i] + v : v;
                }
            }
        }
    }
}

template <int WT, int EPI>
int launch_gemv(const sb_matrix* W, const float* X, int ldx, int B, float* Y, int ldy,
                cudaStream_t st) {
    long warps = (EPI == SB_EPI_SILU) ? (W->M_pad / 2 + 1) / 2 : (W->M_pad + 3) / 4;
    dim3 grid((unsigned)((warps + 7) / 8));
    switch (B) {
#define CASE(nb) \
    case nb: gemv_kernel<WT, nb, EPI><<<grid, 256, 0, st>>>(*W, X, ldx, Y, ldy); break;
        CASE(1) CASE(2) CASE(3) CASE(4) CASE(5) CASE(6) CASE(7) CASE(8)
#undef CASE
        default: return -1;
    }
    return 0;
}

template <int WT, int EPI>
int launch_tiled(const sb_matrix* W, const float* X, int ldx, int B, float* Y, int ldy,
                 cudaStream_t st) {
    const int BM = 128;
    unsigned gm = (unsigned)((W->M_pad + BM - 1) / BM);
    if (B > 64) {
        const int BN = 128;
        size_t sm = (size_t)(2 * 32 * BM + 2 * 32 * BN) * sizeof(float);
        dim3 grid(gm, (unsigned)((B + BN - 1) / BN));
        gemm_tiled<WT, BN, EPI><<<grid, 256, sm, st>>>(*W, X, ldx, B, Y, ldy);
    } else {
        const int BN = 64;  // 48 KB of shared memory: within the default limit
        size_t sm = (size_t)(2 * 32 * BM + 2 * 32 * BN) * sizeof(float);
        dim3 grid(gm, (unsigned)((B + BN - 1) / BN));
        gemm_tiled<WT, BN, EPI><<<grid, 256, sm, st>>>(*W, X, ldx, B, Y, ldy);
    }
    return 0;
}

template <int WT>
int dispatch_epi(const sb_matrix* W, const float* X, int ldx, int B, float* Y, int ldy, int epi,
                 bool gemv, cudaStream_t st) {
    switch (epi) {
        case SB_EPI_STORE:
            return gemv ? launch_gemv<WT, SB_EPI_STORE>(W, X, ldx, B, Y, ldy, st)
                        : launch_tiled<WT, SB_EPI_STORE>(W, X, ldx, B, Y, ldy, st);
        case SB_EPI_ADD:
            return gemv ? launch_gemv<WT, SB_EPI_ADD>(W, X, ldx, B, Y, ldy, st)
                        : launch_tiled<WT, SB_EPI_ADD>(W, X, ldx, B, Y, ldy, st);
        case SB_EPI_SILU:
            return gemv ? launch_gemv<WT, SB_EPI_SILU>(W, X, ldx, B, Y, ldy, st)
                        : launch_tiled<WT, SB_EPI_SILU>(W, X, ldx, B, Y, ldy, st);
    }
    return -1;
}

// ------------------------------------------------------------------------
// Generic f32 kernels for arbitrary shapes (reference vtable entries).
__global__ void matvec_generic(float* y, const float* A, const float* x, int M, int K) {
    int row = blockIdx.x * 8 + (threadIdx.x >> 5), lane = threadIdx.x & 31;
    if (row >= M) return;
    float s = 0.f;
    for (int k = lane; k < K; k += 32) s = fmaf(A[(size_t)row * K + k], x[k], s);
    for (int o = 16; o > 0; o >>= 1) s += __shfl_xor_sync(0xffffffffu, s, o);
    if (lane == 0) y[row] = s;
}
__global__ void linear_batch_generic(float* C, const float* X, const float* W, int B, int K,
                                     int N) {
    long i = (long)blockIdx.x * blockDim.x + threadIdx.x;
    if (i >= (long)B * N) return;
    int b = (int)(i / N), n = (int)(i % N);
    float s = 0.f;
    for (int k = 0; k < K; ++k) s = fmaf(X[(size_t)b * K + k], W[(size_t)k * N + n], s);
    C[i] = s;
}

template <int WT, int EPI>
void prepare_one() {
    const int sm = (2 * 32 * 128 + 2 * 32 * 128) * (int)sizeof(float);
    cudaFuncSetAttribute(gemm_tiled<WT, 128, EPI>, cudaFuncAttributeMaxDynamicSharedMemorySize, sm);
}

}  // namespace

// The BN=128 tiles use 64 KB of dynamic shared memory, above the 48 KB default;
// the attribute is per device and may not be set inside a stream capture.
extern "C" void sb_gemm_prepare(void) {
    prepare_one<SB_WT_Q4K, SB_EPI_STORE>();
    prepare_one<SB_WT_Q4K, SB_EPI_ADD>();
    prepare_one<SB_WT_Q4K, SB_EPI_SILU>();
    prepare_one<SB_WT_F32, SB_EPI_STORE>();
    prepare_one<SB_WT_F32, SB_EPI_ADD>();
    prepare_one<SB_WT_F32, SB_EPI_SILU>();
}

extern "C" int sb_gemm(const sb_matrix* W, const float* X, int ldx, int B, float* Y, int ldy,
                       int epi, int path, cudaStream_t st) {
    if (!W || !X || !Y || B < 1 || W->M < 1) return -1;
    if (W->wtype == SB_WT_Q4K) {
        if (W->K % 256) return -1;
    } else if (W->wtype == SB_WT_F32) {
        if (W->ldw % 128 || W->ldw < W->K) return -1;
    } else {
        return -1;
    }
    if (epi == SB_EPI_SILU && W->M_pad % 128) return -1;
    bool gemv = (path == 0) && B <= 8;
    return W->wtype == SB_WT_Q4K ? dispatch_epi<SB_WT_Q4K>(W, X, ldx, B, Y, ldy, epi, gemv, st)
                                 : dispatch_epi<SB_WT_F32>(W, X, ldx, B, Y, ldy, epi, gemv, st);
}

extern "C" int sb_matvec_f32_generic(float* y, const float* A, const float* x, int M, int K,
                                     cudaStream_t st) {
    if (M < 1 || K < 1) return -1;
    matvec_generic<<<(M + 7) / 8, 256, 0, st>>>(y, A, x, M, K);
    return 0;
}

extern "C" int sb_linear_batch_generic(float* C, const float* X, const float* W, int B, int K,
                                       int N, cudaStream_t st) {
    if (B < 1 || K < 1 || N < 1) return -1;
    long n = (long)B * N;
    linear_batch_generic<<<(unsigned)((n + 255) / 256), 256, 0, st>>>(C, X, W, B, K, N);
    return 0;
}

extern "C" int sb_q4k_matmul_generic(float* Y, const void* A, const float* X, int B, int M, int K,
                                     cudaStream_t st) {
    if (K % 256 || B < 1 || M < 1) return -1;
    sb_matrix W = {SB_WT_Q4K, A, M, M, K, 0};
    return sb_gemm(&W, X, K, B, Y, M, SB_EPI_STORE, 0, st);
}
