// gemm_gv.cu -- Q4_K weight GEMV for one or two activation rows on the CUDA
// cores: the weights stream from HBM once, with about two instructions per
// weight, so the kernel keeps pace with the memory system.
//
//   Y[n][m] (op)= sum_k X[n][k] * W[m][k]      n < NR (1 or 2); op: store,
//                                              residual add, SiLU(gate) * up
//
// A decode step of one or two sequences (the latency-bound regime of the
// reference server, which decodes one token per session per step) multiplies
// every weight by one or two activations.  The tensor-core small-batch kernel
// (gemm_mv.cu) wastes 7/8 of each m16n8k16 MMA there and is bound by its
// instruction stream; this kernel does the multiply-adds on the paired f32
// pipe instead.
//
// Numerics: the structure of the reference's Q4_K dot product
// (src/util/quant.c:210-304): per 32-element sub-block j of a super-block
//     d * sc_j * sum(q * x) - dmin * m_j * sum(x)
// with every q * x product exact in f32 (q a 4-bit integer, x f32) and the
// sums in f32.  A nibble q becomes the float 2^23 + q by a byte permute under
// the exponent byte 0x4B and the paired subtraction of 2^23 leaves q exactly.
//
// Work decomposition: a "quad" is four weight rows -- m..m+3, or for the fused
// SwiGLU weight (gate and up interleaved in 64-row groups, the upload's
// layout) the gate rows g, g+1 and their up rows g+64, g+65 -- so that each x
// value loaded into registers serves four rows.  LQ lanes (the power of two
// >= K/256, at most 32) share a quad, lane l taking super-blocks l, l+LQ, ...;
// a warp holds 32/LQ quads, a CTA 4 warps.  x (NR rows of K floats) and its
// sub-block sums are staged once per CTA in shared memory; the weights are
// read with 16-byte loads, the next sub-block's while the current one is
// computed.  The lanes of a quad then sum their parts with shuffles and lane
// 0 applies the epilogue.
//
// The first super-block headers are requested before the grid waits for the
// previous kernel of the stream (programmatic dependent launch): weights do
// not depend on it, x does.
#include <cuda_fp16.h>
#include <stdint.h>

#include "sb_internal.h"
#include "sb_kernels.h"
#include "sb_pdl.h"

namespace {

constexpr int WARPS = 4;
constexpr int NTHREADS = 32 * WARPS;

struct GvArgs {
    const unsigned char* W;   // Q4_K rows [M_pad][K/256 * 144]
    const float* X;
    float* Y;
    int ldx, ldy, M, K, nb, LQ, QW, n_quads;
};

__host__ __device__ constexpr size_t gv_smem(int nr, int K) {
    return (size_t)nr * K * 4 + (size_t)nr * (K / 32) * 4;
}

// d * sc_j and dmin * m_j of sub-block j from a super-block header
// (util/quant.c:157-166 packing; f16 d / dmin in the first word).
__device__ __forceinline__ float2 sub_scale(uint4 h, int j) {
    const uint32_t w[3] = {h.y, h.z, h.w};
    auto byte = [&](int i) { return (w[i >> 2] >> ((i & 3) * 8)) & 0xffu; };
    uint32_t sc, mn;
    if (j < 4) {
        sc = byte(j) & 63u;
        mn = byte(j + 4) & 63u;
    } else {
        sc = (byte(j + 4) & 15u) | ((byte(j - 4) >> 6) << 4);
        mn = (byte(j + 4) >> 4) | ((byte(j) >> 6) << 4);
    }
    const float d = __half2float(__ushort_as_half((unsigned short)(h.x & 0xffffu)));
    const float dmin = __half2float(__ushort_as_half((unsigned short)(h.x >> 16)));
    return make_float2(d * (float)sc, dmin * (float)mn);
}

// The four nibbles (low if hi == 0, else high) of word `w` as exact floats.
__device__ __forceinline__ void nibbles(uint32_t w, int hi, float2& a, float2& b) {
    const uint32_t nb = (hi ? w >> 4 : w) & 0x0f0f0f0fu;
    const float2 off = make_float2(-8388608.0f, -8388608.0f);
    a = __fadd2_rn(make_float2(__uint_as_float(__byte_perm(nb, 0x4B000000u, 0x7440u)),
                               __uint_as_float(__byte_perm(nb, 0x4B000000u, 0x7441u))), off);
    b = __fadd2_rn(make_float2(__uint_as_float(__byte_perm(nb, 0x4B000000u, 0x7442u)),
                               __uint_as_float(__byte_perm(nb, 0x4B000000u, 0x7443u))), off);
}

__device__ __forceinline__ float silu_mul(float g, float u) { return g / (1.0f + expf(-g)) * u; }

template <int NR, int EPI>
__global__ void __launch_bounds__(NTHREADS, 4) gv_kernel(const GvArgs a) {
    extern __shared__ __align__(16) float xs[];   // [NR][K] x, then [NR][K/32] sub-block sums
    float* xsum = xs + (size_t)NR * a.K;
    sb_grid_release();   // the next kernel may start its set-up
    const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
    const int qq = lane / a.LQ, l = lane % a.LQ;
    const int quad = (blockIdx.x * WARPS + warp) * a.QW + qq;
    const bool live = quad < a.n_quads;
    int rows[4];
    if (EPI == SB_EPI_SILU) {
        const int t = quad >> 5, g = (quad & 31) * 2;
        rows[0] = t * 128 + g;
        rows[1] = rows[0] + 1;
        rows[2] = rows[0] + 64;
        rows[3] = rows[0] + 65;
    } else {
#pragma unroll
        for (int r = 0; r < 4; ++r) rows[r] = quad * 4 + r;
    }
    const size_t row_bytes = (size_t)a.nb * 144;
    const unsigned char* wr[4];
#pragma unroll
    for (int r = 0; r < 4; ++r) wr[r] = a.W + (size_t)(live ? rows[r] : 0) * row_bytes;
    // the first block's headers before x is ready (weights are not written by
    // the previous kernel)
    uint4 hdr[4];
#pragma unroll
    for (int r = 0; r < 4; ++r)
        hdr[r] = live && l < a.nb ? __ldg((const uint4*)(wr[r] + (size_t)l * 144)) : make_uint4(0, 0, 0, 0);

    sb_grid_wait();      // x: after the previous kernel (sb_pdl.h)
    for (int i = threadIdx.x; i < NR * a.K; i += NTHREADS) {
        const int nr = i / a.K, k = i - nr * a.K;
        xs[i] = a.X[(size_t)nr * a.ldx + k];
    }
    __syncthreads();
    for (int i = threadIdx.x; i < NR * (a.K / 32); i += NTHREADS) {
        const float4* p = (const float4*)(xs + (size_t)i * 32);
        float s = 0.f;
#pragma unroll
        for (int c = 0; c < 8; ++c) {
            const float4 v = p[c];
            s += (v.x + v.y) + (v.z + v.w);
        }
        xsum[i] = s;
    }
    __syncthreads();

    float acc[4][NR];
#pragma unroll
    for (int r = 0; r < 4; ++r)
#pragma unroll
        for (int nr = 0; nr < NR; ++nr) acc[r][nr] = 0.f;
    if (live) {
        for (int b = l; b < a.nb; b += a.LQ) {
            if (b != l) {
#pragma unroll
                for (int r = 0; r < 4; ++r) hdr[r] = __ldg((const uint4*)(wr[r] + (size_t)b * 144));
            }
            uint4 q[4];
#pragma unroll
            for (int r = 0; r < 4; ++r) q[r] = __ldg((const uint4*)(wr[r] + (size_t)b * 144 + 16));
#pragma unroll
            for (int j = 0; j < 8; ++j) {
                uint4 qn[4];
                if (j < 7) {
#pragma unroll
                    for (int r = 0; r < 4; ++r)
                        qn[r] = __ldg((const uint4*)(wr[r] + (size_t)b * 144 + 32 + 16 * j));
                }
                float2 dot[4][NR];
#pragma unroll
                for (int r = 0; r < 4; ++r)
#pragma unroll
                    for (int nr = 0; nr < NR; ++nr) dot[r][nr] = make_float2(0.f, 0.f);
                const int k0 = b * 256 + j * 32;
#pragma unroll
                for (int w = 0; w < 4; ++w) {
                    // elements 4w..4w+3 (low nibbles) and 16+4w..16+4w+3 (high)
                    float4 xl[NR], xh[NR];
#pragma unroll
                    for (int nr = 0; nr < NR; ++nr) {
                        xl[nr] = *(const float4*)(xs + (size_t)nr * a.K + k0 + 4 * w);
                        xh[nr] = *(const float4*)(xs + (size_t)nr * a.K + k0 + 16 + 4 * w);
                    }
#pragma unroll
                    for (int r = 0; r < 4; ++r) {
                        const uint32_t word = w == 0 ? q[r].x : w == 1 ? q[r].y : w == 2 ? q[r].z : q[r].w;
                        float2 l0, l1, h0, h1;
                        nibbles(word, 0, l0, l1);
                        nibbles(word, 1, h0, h1);
#pragma unroll
                        for (int nr = 0; nr < NR; ++nr) {
                            float2 d2 = dot[r][nr];
                            d2 = __ffma2_rn(l0, make_float2(xl[nr].x, xl[nr].y), d2);
                            d2 = __ffma2_rn(l1, make_float2(xl[nr].z, xl[nr].w), d2);
                            d2 = __ffma2_rn(h0, make_float2(xh[nr].x, xh[nr].y), d2);
                            d2 = __ffma2_rn(h1, make_float2(xh[nr].z, xh[nr].w), d2);
                            dot[r][nr] = d2;
                        }
                    }
                }
#pragma unroll
                for (int r = 0; r < 4; ++r) {
                    const float2 s = sub_scale(hdr[r], j);
#pragma unroll
                    for (int nr = 0; nr < NR; ++nr) {
                        const float dq = dot[r][nr].x + dot[r][nr].y;
                        acc[r][nr] = fmaf(s.x, dq, fmaf(-s.y, xsum[(size_t)nr * (a.K / 32) + b * 8 + j],
                                                        acc[r][nr]));
                    }
                }
                if (j < 7) {
#pragma unroll
                    for (int r = 0; r < 4; ++r) q[r] = qn[r];
                }
            }
        }
    }
    // the quad's lanes sum their super-blocks
#pragma unroll
    for (int o = 16; o >= 1; o >>= 1) {
        if (o < a.LQ) {
#pragma unroll
            for (int r = 0; r < 4; ++r)
#pragma unroll
                for (int nr = 0; nr < NR; ++nr) acc[r][nr] += __shfl_xor_sync(0xffffffffu, acc[r][nr], o);
        }
    }
    if (!live || l != 0) return;
#pragma unroll
    for (int nr = 0; nr < NR; ++nr) {
        float* y = a.Y + (size_t)nr * a.ldy;
        if (EPI == SB_EPI_SILU) {
            const int unit = (rows[0] >> 7) * 64 + (rows[0] & 63);
            if (unit < a.M / 2) y[unit] = silu_mul(acc[0][nr], acc[2][nr]);
            if (unit + 1 < a.M / 2) y[unit + 1] = silu_mul(acc[1][nr], acc[3][nr]);
        } else {
#pragma unroll
            for (int r = 0; r < 4; ++r) {
                if (rows[r] >= a.M) continue;
                y[rows[r]] = EPI == SB_EPI_ADD ? y[rows[r]] + acc[r][nr] : acc[r][nr];
            }
        }
    }
}

template <int NR, int EPI>
int launch(const GvArgs& a, cudaStream_t st) {
    const size_t smem = gv_smem(NR, a.K);
    const int quads_per_cta = WARPS * a.QW;
    const unsigned grid = (unsigned)((a.n_quads + quads_per_cta - 1) / quads_per_cta);
    return sb_launch_pdl(gv_kernel<NR, EPI>, dim3(grid), dim3(NTHREADS), smem, st, a) == cudaSuccess
               ? 0
               : -5;
}

template <int NR>
int dispatch(const GvArgs& a, int epi, cudaStream_t st) {
    switch (epi) {
        case SB_EPI_STORE: return launch<NR, SB_EPI_STORE>(a, st);
        case SB_EPI_ADD: return launch<NR, SB_EPI_ADD>(a, st);
        case SB_EPI_SILU: return launch<NR, SB_EPI_SILU>(a, st);
    }
    return -1;
}

}  // namespace

// The shared-memory opt-in of every instantiation (per device, outside any
// stream capture).
extern "C" void sb_gv_prepare(void) {
    const int smem = (int)gv_smem(2, SB_GV_MAX_K);
    cudaFuncSetAttribute(gv_kernel<1, SB_EPI_STORE>, cudaFuncAttributeMaxDynamicSharedMemorySize, smem);
    cudaFuncSetAttribute(gv_kernel<1, SB_EPI_ADD>, cudaFuncAttributeMaxDynamicSharedMemorySize, smem);
    cudaFuncSetAttribute(gv_kernel<1, SB_EPI_SILU>, cudaFuncAttributeMaxDynamicSharedMemorySize, smem);
    cudaFuncSetAttribute(gv_kernel<2, SB_EPI_STORE>, cudaFuncAttributeMaxDynamicSharedMemorySize, smem);
    cudaFuncSetAttribute(gv_kernel<2, SB_EPI_ADD>, cudaFuncAttributeMaxDynamicSharedMemorySize, smem);
    cudaFuncSetAttribute(gv_kernel<2, SB_EPI_SILU>, cudaFuncAttributeMaxDynamicSharedMemorySize, smem);
}

extern "C" int sb_gv_supported(const sb_matrix* W, int n, int epi) {
    return W && W->wtype == SB_WT_Q4K && n >= 1 && n <= SB_GV_MAX_ROWS && W->K % 256 == 0 &&
           W->K <= SB_GV_MAX_K && W->M_pad % 128 == 0 &&
           (epi == SB_EPI_STORE || epi == SB_EPI_ADD || (epi == SB_EPI_SILU && W->M % 128 == 0));
}

extern "C" int sb_gv_gemm(const sb_matrix* W, const float* X, int ldx, int n, float* Y, int ldy,
                          int epi, cudaStream_t st) {
    if (!sb_gv_supported(W, n, epi) || !X || !Y || ldx < W->K ||
        (n > 1 && ldy < (epi == SB_EPI_SILU ? W->M / 2 : W->M)))
        return -1;
    GvArgs a;
    a.W = (const unsigned char*)W->data;
    a.X = X;
    a.Y = Y;
    a.ldx = ldx;
    a.ldy = ldy;
    a.M = W->M;
    a.K = W->K;
    a.nb = W->K / 256;
    int lq = 1;
    while (lq < a.nb && lq < 32) lq *= 2;
    a.LQ = lq;
    a.QW = 32 / lq;
    a.n_quads = W->M_pad / 4;
    return n == 1 ? dispatch<1>(a, epi, st) : dispatch<2>(a, epi, st);
}
