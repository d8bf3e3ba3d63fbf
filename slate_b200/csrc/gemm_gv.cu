// gemm_gv.cu -- Q4_K weight GEMV for one or two activation rows on the CUDA
// cores, bound by the weight stream from HBM.
//
//   Y[n][m] (op)= sum_k X[n][k] * W[m][k]      n < NR (1 or 2); op: store,
//                                              residual add, SiLU(gate) * up,
//                                              or store + RoPE + KV append
//
// A decode step of one or two sequences (the latency-bound regime of the
// reference server, which decodes one token per session per step) multiplies
// every weight by one or two activations; the tensor-core small-batch kernel
// (gemm_mv.cu) would waste 7/8 of each m16n8k16 MMA here.
//
// Numerics: the structure of the reference's Q4_K dot product
// (src/util/quant.c:210-304): per 32-element sub-block s of a super-block
//     d * sc_s * sum(q * x) - dmin * m_s * sum(x)
// with every q * x product exact in f32 (q a 4-bit integer, x f32) and the
// sums in f32.  A nibble q becomes the float 2^23 + q by a byte permute under
// the exponent byte 0x4B, and a paired subtraction of 2^23 leaves q exactly.
//
// Memory pipeline: one persistent CTA per SM owns a contiguous range of
// "stages" (RS weight rows each, RS * K/256 * 144 contiguous bytes; for the
// SwiGLU weight, whose gate and up rows are interleaved in 64-row groups, a
// stage is RS/2 gate rows and their RS/2 up rows).  A producer warp streams
// the stages through an NS-deep shared-memory ring with cp.async.bulk (TMA
// bulk copies completing on mbarriers), so ~100 KB per SM are in flight
// whatever the consumers do; it starts before the grid waits for the previous
// kernel of the stream (programmatic dependent launch), since weights are not
// written by it.  x (NR rows of K floats, stored 64-float groups 68 floats
// apart so the consumers' loads hit distinct banks) and its 32-element sums
// are staged once per CTA; with a norm weight, the staged rows are RMSNorm-ed
// in place first (the step's RMSNorm launch before this GEMM is then not
// needed).
//
// Consumers: NG groups of 8 warps take the stages in turn.  In a stage, WPR
// warps share a row (WPR = the power of two >= K/4096), each summing a
// contiguous part of its super-blocks; a lane takes one 32-byte quant group
// of a super-block (64 weights: all of sub-blocks 2j and 2j+1, Slate's
// nibble order), so the sub-block scales are unpacked once per 64 weights.  Each warp's part is
// reduced by shuffles and stored to shared memory; after the last stage the
// parts of every row are summed in a fixed order (deterministic results) and
// the epilogue writes Y.
//
// Waits on the ring are bounded (2 s): a timeout sets *err, the CTA stops
// consuming, and the producer waits (bounded) for its copies in flight before
// the CTA exits.
#include <cuda_fp16.h>
#include <stdint.h>

#include "sb_internal.h"
#include "sb_kernels.h"
#include "sb_pdl.h"

namespace {

constexpr int CW = 8;                      // consumer warps per group
constexpr int NG = 2;                      // consumer groups
constexpr int NCONS = 32 * CW * NG;        // consumer threads
constexpr int NTHREADS = NCONS + 32;       // + the producer warp
constexpr int MAX_NS = 12;
constexpr int STATIC_SMEM = 1024;          // bound on the kernel's static shared memory
constexpr uint64_t WAIT_NS = 2000000000ull;

struct GvArgs {
    const unsigned char* W;   // Q4_K rows [M_pad][K/256 * 144]
    const float* X;
    float* Y;
    int* err;
    const float* nw;          // RMSNorm weight applied to X while it is staged (null: none)
    float eps;
    sb_rope_args r;           // SB_EPI_ROPE: positions, page table, pool, RoPE tables
    int* head_cnt;            // SB_EPI_ROPE: rows written per head (zero between launches)
    int ldx, ldy, M, K, nb;
    int RS, WPR, CH;          // rows per stage, warps per row, super-blocks per part
    int n_stages, NS;         // stages in the matrix, ring depth
    int stage_bytes, max_local;   // bytes per stage, stages per CTA at most
};

// ---- shared-memory layout (host and device) ----
__host__ __device__ constexpr int xs_floats(int K) { return K / 64 * 68; }
__host__ __device__ constexpr size_t gv_smem(int nr, int K, int ns, int stage_bytes, int max_local,
                                             int rs, int wpr) {
    return (size_t)ns * stage_bytes + (size_t)nr * xs_floats(K) * 4 + (size_t)nr * (K / 32) * 4 +
           (size_t)max_local * rs * wpr * nr * 4 + (size_t)2 * ns * 8 + 16;
}

__device__ __forceinline__ uint32_t su32(const void* p) { return (uint32_t)__cvta_generic_to_shared(p); }
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
__device__ __forceinline__ void bulk_g2s(void* dst, const void* src, uint32_t bytes, uint64_t* bar) {
    asm volatile(
        "cp.async.bulk.shared::cluster.global.mbarrier::complete_tx::bytes [%0], [%1], %2, [%3];" ::"r"(
            su32(dst)),
        "l"(src), "r"(bytes), "r"(su32(bar))
        : "memory");
}
// the consumer threads only (the producer warp may have left)
__device__ __forceinline__ void cons_sync() { asm volatile("bar.sync 1, %0;" ::"n"(NCONS) : "memory"); }

// Memory row of the r-th row of stage `st`.
template <int EPI>
__device__ __forceinline__ int stage_row(int st, int r, int RS) {
    if (EPI == SB_EPI_SILU) {
        const int half = RS / 2;
        const int unit = st * half + (r < half ? r : r - half);
        return (unit >> 6) * 128 + (unit & 63) + (r < half ? 0 : 64);
    }
    return st * RS + r;
}

// Four nibbles of `nb` (already masked to one nibble per byte) as floats.
__device__ __forceinline__ void nib4(uint32_t nb, float2& a, float2& b) {
    const float2 off = make_float2(-8388608.0f, -8388608.0f);
    a = __fadd2_rn(make_float2(__uint_as_float(__byte_perm(nb, 0x4B000000u, 0x7440u)),
                               __uint_as_float(__byte_perm(nb, 0x4B000000u, 0x7441u))), off);
    b = __fadd2_rn(make_float2(__uint_as_float(__byte_perm(nb, 0x4B000000u, 0x7442u)),
                               __uint_as_float(__byte_perm(nb, 0x4B000000u, 0x7443u))), off);
}

__device__ __forceinline__ float silu_mul(float g, float u) { return g / (1.0f + expf(-g)) * u; }

__device__ __forceinline__ void put_kv(void* pool, int kv_dtype, size_t i, float v) {
    if (kv_dtype == 1) ((__half*)pool)[i] = __float2half_rn(v);
    else ((float*)pool)[i] = v;
}

// RoPE of head h of the fused Q|K|V rows (llama_infer.c:77-92, pairs (j, j +
// hd/2) at the row's position) and the KV append (llama_infer.c:169-175): a
// query head is rotated in place, a key head rotated into the pool, a value
// head copied into it.  The rows were written by several CTAs: read through L2.
template <int NR>
__device__ void rope_head(const GvArgs& a, int h) {
    const sb_rope_args& r = a.r;
    const int half = r.hd / 2;
    for (int t = threadIdx.x; t < NR * half; t += NCONS) {
        const int nr = t / half, j = t - nr * half;
        const int pos = r.row_pos[nr];
        if (pos < 0) continue;
        float* row = a.Y + (size_t)nr * a.ldy + (size_t)h * r.hd;
        const float x0 = __ldcg(row + j), x1 = __ldcg(row + j + half);
        if (h < r.nq) {
            const float c = r.rope_cos[(size_t)pos * half + j], sn = r.rope_sin[(size_t)pos * half + j];
            row[j] = x0 * c - x1 * sn;
            row[j + half] = x0 * sn + x1 * c;
            continue;
        }
        const int slot = r.row_slot[nr];
        const int page = r.page_table[(size_t)slot * r.max_pages + pos / SB_PAGE_TOKENS];
        if (page < 0 || page >= r.n_pages) continue;          // never allocated: skip, never fault
        const size_t hs = (size_t)SB_PAGE_TOKENS * r.hd;
        const size_t base = ((size_t)r.layer * r.n_pages + page) * 2 * r.nkv * hs +
                            (size_t)(pos % SB_PAGE_TOKENS) * r.hd;
        if (h < r.nq + r.nkv) {
            const float c = r.rope_cos[(size_t)pos * half + j], sn = r.rope_sin[(size_t)pos * half + j];
            const size_t o = base + (size_t)(h - r.nq) * hs;
            put_kv(r.pool, r.kv_dtype, o + j, x0 * c - x1 * sn);
            put_kv(r.pool, r.kv_dtype, o + j + half, x0 * sn + x1 * c);
        } else {
            const size_t o = base + (size_t)r.nkv * hs + (size_t)(h - r.nq - r.nkv) * hs;
            put_kv(r.pool, r.kv_dtype, o + j, x0);
            put_kv(r.pool, r.kv_dtype, o + j + half, x1);
        }
    }
}

template <int NR, int EPI>
__global__ void __launch_bounds__(NTHREADS, 1) gv_kernel(const GvArgs a) {
    extern __shared__ __align__(128) unsigned char smem[];
    unsigned char* ring = smem;
    float* xs = (float*)(smem + (size_t)a.NS * a.stage_bytes);
    const int xsn = xs_floats(a.K);
    float* xsum = xs + (size_t)NR * xsn;
    float* part = xsum + (size_t)NR * (a.K / 32);
    uint64_t* full = (uint64_t*)(((uintptr_t)(part + (size_t)a.max_local * a.RS * a.WPR * NR) + 7) & ~(uintptr_t)7);
    uint64_t* empty = full + a.NS;

    sb_grid_release();   // the next kernel may start its set-up
    const int G = gridDim.x;
    const int s0 = (int)((long long)a.n_stages * blockIdx.x / G);
    const int s1 = (int)((long long)a.n_stages * (blockIdx.x + 1) / G);
    const int n_local = s1 - s0;
    const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
    if (threadIdx.x == 0) {
        for (int s = 0; s < a.NS; ++s) {
            bar_init(&full[s], 1);
            bar_init(&empty[s], CW);
        }
        asm volatile("fence.mbarrier_init.release.cluster;" ::: "memory");
    }
    __syncthreads();

    const size_t row_bytes = (size_t)a.nb * 144;
    if (warp == CW * NG) {
        // ---------------- producer ----------------
        if (lane == 0) {
            int issued = 0;
            for (int i = 0; i < n_local; ++i) {
                const int s = i % a.NS;
                if (i >= a.NS && !bar_wait(&empty[s], ((i / a.NS) - 1) & 1, a.err, 21)) break;
                unsigned char* dst = ring + (size_t)s * a.stage_bytes;
                bar_expect(&full[s], (uint32_t)a.stage_bytes);
                if (EPI == SB_EPI_SILU) {
                    const int half = a.RS / 2;
                    const uint32_t hb = (uint32_t)(half * row_bytes);
                    bulk_g2s(dst, a.W + (size_t)stage_row<EPI>(s0 + i, 0, a.RS) * row_bytes, hb, &full[s]);
                    bulk_g2s(dst + hb, a.W + (size_t)stage_row<EPI>(s0 + i, half, a.RS) * row_bytes, hb,
                             &full[s]);
                } else {
                    bulk_g2s(dst, a.W + (size_t)(s0 + i) * a.RS * row_bytes, (uint32_t)a.stage_bytes,
                             &full[s]);
                }
                ++issued;
            }
            // every copy this CTA issued has landed before it exits (on the
            // normal path the consumers waited for them already)
            for (int i = issued > a.NS ? issued - a.NS : 0; i < issued; ++i)
                if (!bar_wait(&full[i % a.NS], (i / a.NS) & 1, a.err, 22)) break;
        }
        return;
    }

    // ---------------- consumers ----------------
    sb_grid_wait();      // x: after the previous kernel (sb_pdl.h)
    {
        const bool vec = (((uintptr_t)a.X | ((uintptr_t)a.ldx * 4)) & 15) == 0;
        for (int nr = 0; nr < NR; ++nr) {
            const float* xr = a.X + (size_t)nr * a.ldx;
            float* xd = xs + (size_t)nr * xsn;
            if (vec) {
                for (int i = threadIdx.x; i < a.K / 4; i += NCONS) {
                    const int k = 4 * i;
                    *(float4*)(xd + (k >> 6) * 68 + (k & 63)) = __ldg((const float4*)(xr + k));
                }
            } else {
                for (int k = threadIdx.x; k < a.K; k += NCONS) xd[(k >> 6) * 68 + (k & 63)] = xr[k];
            }
        }
    }
    cons_sync();
    if (a.nw) {
        // RMSNorm of each staged row (llama_infer.c:157, 186): y = x * w / sqrt(mean(x^2) + eps),
        // the sum of squares in f32 per thread and in double across the block
        __shared__ double red[CW * NG][NR];
        __shared__ float inv_s[NR];
        for (int nr = 0; nr < NR; ++nr) {
            const float* xd = xs + (size_t)nr * xsn;
            float sq = 0.f;
            for (int k = threadIdx.x; k < a.K; k += NCONS) {
                const float v = xd[(k >> 6) * 68 + (k & 63)];
                sq = fmaf(v, v, sq);
            }
            double sd = sq;
#pragma unroll
            for (int o = 16; o > 0; o >>= 1) sd += __shfl_xor_sync(0xffffffffu, sd, o);
            if ((threadIdx.x & 31) == 0) red[threadIdx.x >> 5][nr] = sd;
        }
        cons_sync();
        if (threadIdx.x < NR) {
            double t = 0.0;
            for (int w = 0; w < CW * NG; ++w) t += red[w][threadIdx.x];
            inv_s[threadIdx.x] = 1.0f / sqrtf((float)(t / (double)a.K) + a.eps);
        }
        cons_sync();
        for (int nr = 0; nr < NR; ++nr) {
            float* xd = xs + (size_t)nr * xsn;
            const float inv = inv_s[nr];
            for (int k = threadIdx.x; k < a.K; k += NCONS) {
                float* p = xd + (k >> 6) * 68 + (k & 63);
                *p = *p * __ldg(a.nw + k) * inv;
            }
        }
        cons_sync();
    }
    for (int i = threadIdx.x; i < NR * (a.K / 32); i += NCONS) {
        const int nr = i / (a.K / 32), sbk = i - nr * (a.K / 32);
        const float4* p = (const float4*)(xs + (size_t)nr * xsn + (sbk >> 1) * 68 + (sbk & 1) * 32);
        float s = 0.f;
#pragma unroll
        for (int c = 0; c < 8; ++c) {
            const float4 v = p[c];
            s += (v.x + v.y) + (v.z + v.w);
        }
        xsum[i] = s;
    }
    cons_sync();

    const int grp = warp / CW, cw = warp % CW;
    const int rr = cw / a.WPR, pw = cw % a.WPR;
    const int j = lane & 3;                      // quant group: sub-blocks 2j, 2j+1
    const int sb_lo = pw * a.CH;
    const int sb_hi = min(a.nb, sb_lo + a.CH);
    // scale-unpacking constants of this lane's sub-block pair (quant.c:157-166:
    // sub-blocks 0-3 hold 6-bit scale / min in bytes 0-3 / 4-7; 4-7 take their
    // low 4 bits from bytes 8-11 and their top 2 from the top bits of 0-7)
    const bool upper = j >= 2;
    const uint32_t t8 = upper ? 8u * (2 * j - 4) : 16u * j;   // byte offset of the pair
    const uint32_t mlo = upper ? 0x000F000Fu : 0x003F003Fu;
    const uint32_t mhi = upper ? 0x00300030u : 0u;

    for (int i = grp; i < n_local; i += NG) {
        const int s = i % a.NS;
        if (!bar_wait(&full[s], (i / a.NS) & 1, a.err, 23)) break;
        const unsigned char* rowp = ring + (size_t)s * a.stage_bytes + (size_t)rr * row_bytes;
        float acc[NR];
#pragma unroll
        for (int nr = 0; nr < NR; ++nr) acc[nr] = 0.f;
        for (int sb = sb_lo + (lane >> 2); sb < sb_hi; sb += 8) {
            const unsigned char* blk = rowp + (size_t)sb * 144;
            const uint4 h = *(const uint4*)blk;
            const uint4 q0 = *(const uint4*)(blk + 16 + 32 * j);
            const uint4 q1 = *(const uint4*)(blk + 32 + 32 * j);
            // sc / m of sub-blocks 2j, 2j+1 in the two 16-bit halves
            const uint32_t A = upper ? h.w : h.y;
            const uint32_t scw = (__byte_perm(A >> t8, 0, 0x5150) & mlo) |
                                 ((__byte_perm(h.y >> t8, 0, 0x5150) >> 2) & mhi);
            const uint32_t B = upper ? (h.w >> 4) : h.z;
            const uint32_t mw = (__byte_perm(B >> t8, 0, 0x5150) & mlo) |
                                ((__byte_perm(h.z >> t8, 0, 0x5150) >> 2) & mhi);
            const float2 off = make_float2(-8388608.0f, -8388608.0f);
            const float2 scf = __fadd2_rn(make_float2(__uint_as_float(__byte_perm(scw, 0x4B000000u, 0x7440u)),
                                                      __uint_as_float(__byte_perm(scw, 0x4B000000u, 0x7442u))),
                                          off);
            const float2 mf = __fadd2_rn(make_float2(__uint_as_float(__byte_perm(mw, 0x4B000000u, 0x7440u)),
                                                     __uint_as_float(__byte_perm(mw, 0x4B000000u, 0x7442u))),
                                         off);
            const float d = __half2float(__ushort_as_half((unsigned short)(h.x & 0xffffu)));
            const float dmin = __half2float(__ushort_as_half((unsigned short)(h.x >> 16)));
            const int k0 = sb * 256 + 64 * j;          // first element of the group
            const uint32_t qw[8] = {q0.x, q0.y, q0.z, q0.w, q1.x, q1.y, q1.z, q1.w};
            float2 dl[NR], dh[NR];
#pragma unroll
            for (int nr = 0; nr < NR; ++nr) dl[nr] = dh[nr] = make_float2(0.f, 0.f);
            const float* xg = xs + (k0 >> 6) * 68;     // the group's 64 floats (row nr: + nr * xsn)
#pragma unroll
            for (int w = 0; w < 8; ++w) {
                // word w of the group: sub-block 2j (w < 4) or 2j+1; in a
                // sub-block's 16 bytes the low nibbles are its elements 0..15
                // and the high nibbles 16..31 (quant.c:168-202)
                const int e = (w >> 2) * 32 + 4 * (w & 3);
                float2 l0, l1, h0, h1;
                nib4(qw[w] & 0x0f0f0f0fu, l0, l1);
                nib4((qw[w] >> 4) & 0x0f0f0f0fu, h0, h1);
#pragma unroll
                for (int nr = 0; nr < NR; ++nr) {
                    const float4 xl = *(const float4*)(xg + (size_t)nr * xsn + e);
                    const float4 xh = *(const float4*)(xg + (size_t)nr * xsn + e + 16);
                    float2& dd = w < 4 ? dl[nr] : dh[nr];
                    dd = __ffma2_rn(l0, make_float2(xl.x, xl.y), dd);
                    dd = __ffma2_rn(l1, make_float2(xl.z, xl.w), dd);
                    dd = __ffma2_rn(h0, make_float2(xh.x, xh.y), dd);
                    dd = __ffma2_rn(h1, make_float2(xh.z, xh.w), dd);
                }
            }
#pragma unroll
            for (int nr = 0; nr < NR; ++nr) {
                const float2 xsm = *(const float2*)(xsum + (size_t)nr * (a.K / 32) + sb * 8 + 2 * j);
                float v = d * (scf.x * (dl[nr].x + dl[nr].y)) - dmin * (mf.x * xsm.x);
                v += d * (scf.y * (dh[nr].x + dh[nr].y)) - dmin * (mf.y * xsm.y);
                acc[nr] += v;
            }
        }
        __syncwarp();
        if (lane == 0) bar_arrive(&empty[s]);   // this warp is done with the stage
#pragma unroll
        for (int nr = 0; nr < NR; ++nr) {
#pragma unroll
            for (int o = 16; o >= 1; o >>= 1) acc[nr] += __shfl_xor_sync(0xffffffffu, acc[nr], o);
        }
        if (lane == 0) {
#pragma unroll
            for (int nr = 0; nr < NR; ++nr)
                part[((size_t)(i * a.RS + rr) * a.WPR + pw) * NR + nr] = acc[nr];
        }
    }
    cons_sync();
    if (*(volatile int*)a.err) return;

    // ---------------- epilogue: the parts of each row in a fixed order ----------------
    const float* pp = part;
    const int wpr = a.WPR;
    if (EPI == SB_EPI_SILU) {
        const int half = a.RS / 2;
        for (int t = threadIdx.x; t < n_local * half * NR; t += NCONS) {
            const int nr = t / (n_local * half), u = t - nr * (n_local * half);
            const int ls = u / half, r = u - ls * half;
            const int unit = (s0 + ls) * half + r;
            if (unit >= a.M / 2) continue;
            const float* pg = pp + (size_t)(ls * a.RS + r) * wpr * NR + nr;
            const float* pu = pg + (size_t)half * wpr * NR;
            float g = 0.f, u2 = 0.f;
            for (int p = 0; p < wpr; ++p) {
                g += pg[p * NR];
                u2 += pu[p * NR];
            }
            a.Y[(size_t)nr * a.ldy + unit] = silu_mul(g, u2);
        }
    } else {
        for (int t = threadIdx.x; t < n_local * a.RS * NR; t += NCONS) {
            const int nr = t / (n_local * a.RS), lr = t - nr * (n_local * a.RS);
            const int m = s0 * a.RS + lr;
            if (m >= a.M) continue;
            const float* pr = pp + (size_t)lr * wpr * NR + nr;
            float v = 0.f;
            for (int p = 0; p < wpr; ++p) v += pr[p * NR];
            float* y = a.Y + (size_t)nr * a.ldy + m;
            *y = EPI == SB_EPI_ADD ? *y + v : v;
        }
    }
    if (EPI == SB_EPI_ROPE) {
        // heads are 128-ish rows, written by two to four CTAs: the CTA that
        // completes a head (per-head counters of rows written) rotates it
        __shared__ int is_fin;
        __threadfence();                  // this CTA's rows, before its counts
        const int m0 = s0 * a.RS, m1 = min(a.M, s1 * a.RS);
        for (int h = m0 / a.r.hd; m1 > m0 && h <= (m1 - 1) / a.r.hd; ++h) {
            cons_sync();
            if (threadIdx.x == 0) {
                const int lo = max(m0, h * a.r.hd), hi = min(m1, (h + 1) * a.r.hd);
                is_fin = atomicAdd(&a.head_cnt[h], hi - lo) + (hi - lo) == a.r.hd;
                if (is_fin) __threadfence();   // the other CTAs' rows, after their counts
            }
            cons_sync();
            if (is_fin) {
                rope_head<NR>(a, h);
                if (threadIdx.x == 0) a.head_cnt[h] = 0;   // every row of the head has counted
            }
        }
    }
}

int g_sms = 0;
int g_smem_max = 0;

template <int NR, int EPI>
int launch(const GvArgs& a, size_t smem, cudaStream_t st) {
    const unsigned grid = (unsigned)min(g_sms, a.n_stages);
    return sb_cuda_check(sb_launch_pdl(gv_kernel<NR, EPI>, dim3(grid), dim3(NTHREADS), smem, st, a),
                         "gv_kernel launch");
}

template <int NR>
int dispatch(const GvArgs& a, size_t smem, int epi, cudaStream_t st) {
    switch (epi) {
        case SB_EPI_STORE: return launch<NR, SB_EPI_STORE>(a, smem, st);
        case SB_EPI_ADD: return launch<NR, SB_EPI_ADD>(a, smem, st);
        case SB_EPI_SILU: return launch<NR, SB_EPI_SILU>(a, smem, st);
        case SB_EPI_ROPE: return launch<NR, SB_EPI_ROPE>(a, smem, st);
    }
    return -1;
}

// Stage geometry of a K: warps per row, rows per stage, super-blocks per part.
void geometry(int K, int& wpr, int& rs, int& ch, int& stage_bytes) {
    const int nb = K / 256;
    wpr = 1;
    while (wpr * 16 < nb && wpr < CW) wpr *= 2;
    rs = CW / wpr;
    ch = (nb + wpr - 1) / wpr;
    stage_bytes = rs * nb * 144;
}

template <int NR>
void set_smem(int smem) {
    cudaFuncSetAttribute(gv_kernel<NR, SB_EPI_STORE>, cudaFuncAttributeMaxDynamicSharedMemorySize, smem);
    cudaFuncSetAttribute(gv_kernel<NR, SB_EPI_ADD>, cudaFuncAttributeMaxDynamicSharedMemorySize, smem);
    cudaFuncSetAttribute(gv_kernel<NR, SB_EPI_SILU>, cudaFuncAttributeMaxDynamicSharedMemorySize, smem);
    cudaFuncSetAttribute(gv_kernel<NR, SB_EPI_ROPE>, cudaFuncAttributeMaxDynamicSharedMemorySize, smem);
}

}  // namespace

// SM count and the shared-memory opt-in of every instantiation (per device,
// outside any stream capture).
extern "C" void sb_gv_prepare(void) {
    int dev = 0;
    cudaGetDevice(&dev);
    cudaDeviceGetAttribute(&g_sms, cudaDevAttrMultiProcessorCount, dev);
    cudaDeviceGetAttribute(&g_smem_max, cudaDevAttrMaxSharedMemoryPerBlockOptin, dev);
    g_smem_max -= STATIC_SMEM;          // the kernel's static shared memory comes on top
    const int smem = g_smem_max;
    set_smem<1>(smem);
    set_smem<2>(smem);
}

// The ring depth that fits beside x for (n, K, M), 0 if fewer than 3 stages fit.
static int gv_ring(int n, int K, int M, int epi, size_t* smem_out, int* n_stages_out, int* max_local_out) {
    if (g_sms <= 0 || g_smem_max <= 0) return 0;
    int wpr, rs, ch, sbytes;
    geometry(K, wpr, rs, ch, sbytes);
    if (epi == SB_EPI_SILU && rs < 2) return 0;
    const int rows = epi == SB_EPI_SILU ? M : M;
    const int n_stages = (rows + rs - 1) / rs;
    const int grid = n_stages < g_sms ? n_stages : g_sms;
    const int max_local = (n_stages + grid - 1) / grid;
    const size_t fixed = gv_smem(n, K, 0, sbytes, max_local, rs, wpr);
    if ((size_t)g_smem_max <= fixed) return 0;
    int ns = (int)(((size_t)g_smem_max - fixed) / ((size_t)sbytes + 16));
    if (ns > MAX_NS) ns = MAX_NS;
    if (ns < 3) return 0;
    if (smem_out) *smem_out = gv_smem(n, K, ns, sbytes, max_local, rs, wpr);
    if (n_stages_out) *n_stages_out = n_stages;
    if (max_local_out) *max_local_out = max_local;
    return ns;
}

extern "C" int sb_gv_supported(const sb_matrix* W, int n, int epi) {
    return W && W->wtype == SB_WT_Q4K && n >= 1 && n <= SB_GV_MAX_ROWS && W->K % 256 == 0 &&
           W->K <= SB_GV_MAX_K && W->M_pad % 128 == 0 &&
           (epi == SB_EPI_STORE || epi == SB_EPI_ADD || epi == SB_EPI_ROPE ||
            (epi == SB_EPI_SILU && W->M % 128 == 0)) &&
           gv_ring(n, W->K, W->M, epi, NULL, NULL, NULL) > 0;
}

extern "C" int sb_gv_gemm(const sb_matrix* W, const float* X, int ldx, int n, float* Y, int ldy,
                          int epi, const float* norm_w, float eps, const sb_rope_args* rope,
                          int* head_cnt, int* err, cudaStream_t st) {
    if (!sb_gv_supported(W, n, epi) || !X || !Y || !err || ldx < W->K ||
        (n > 1 && ldy < (epi == SB_EPI_SILU ? W->M / 2 : W->M)))
        return -1;
    if (epi == SB_EPI_ROPE &&
        (!rope || !head_cnt || rope->hd % 2 || rope->hd / 2 > NCONS || rope->nq < 1 || rope->nkv < 1 ||
         W->M != (rope->nq + 2 * rope->nkv) * rope->hd))
        return -1;
    GvArgs a;
    a.W = (const unsigned char*)W->data;
    a.X = X;
    a.Y = Y;
    a.err = err;
    a.nw = norm_w;
    a.eps = eps;
    a.r = rope ? *rope : sb_rope_args{};
    a.head_cnt = head_cnt;
    a.ldx = ldx;
    a.ldy = ldy;
    a.M = W->M;
    a.K = W->K;
    a.nb = W->K / 256;
    geometry(a.K, a.WPR, a.RS, a.CH, a.stage_bytes);
    size_t smem = 0;
    a.NS = gv_ring(n, a.K, a.M, epi, &smem, &a.n_stages, &a.max_local);
    if (a.NS <= 0) return -1;
    switch (n) {
        case 1: return dispatch<1>(a, smem, epi, st);
        case 2: return dispatch<2>(a, smem, epi, st);
    }
    return -1;
}
