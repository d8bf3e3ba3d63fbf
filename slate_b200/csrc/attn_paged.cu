// attn_paged.cu -- paged-KV GQA decode attention (src/loader/llama_infer.c:97-129)
// for a batch of sequences at their own positions (sm_100a).
//
// Pool layout: pool[layer][page][kv (0 = K, 1 = V)][kv_head][16 tokens][head_dim],
// so one (page, kv, head) block -- 16 rows of head_dim -- is contiguous
// (4 KB for f16 / 8 KB for f32 at head_dim 128).
//
// One CTA per (row, kv_head, SB_ATTN_CHUNK-token chunk).  A producer warp streams the
// chunk's pages with cp.async.bulk (TMA bulk copies, one for K and one for V,
// completion on an mbarrier) into a ring of ~64 KB (4-16 stages) in
// shared memory.  Four consumer warps take pages round-robin; each handles
// all G = n_heads / n_kv_heads query heads of the group, lane l holding
// head_dim/32 consecutive dims, so every K/V byte crosses HBM once and shared
// memory once per step.  Per page a warp forms the 16 x G partial dots,
// reduces them across lanes with a transpose-reduction (lane l ends up with
// entries l*VPL .. of the [head][token] grid), applies an online softmax
// (running max / sum, expf, as the reference's max-subtracted softmax) and
// accumulates p*V with probabilities broadcast through shared memory.  The
// warps' (m, l, o) states are merged in the CTA, then across chunks by
// attn_combine.  A prompt chunk (rows at consecutive positions of one
// sequence, f32 K/V or any cache the tensor-core prefill kernel does not take)
// runs the same kernel on tiles of four rows: each warp owns one row and reads
// every page, so the chunk's K/V is streamed once per four rows.  Waits are
// bounded (2 s); a timeout sets *err and the CTA drains its copies before
// exiting.
#include <cuda_fp16.h>
#include <math.h>

#include "sb_kernels.h"
#include "sb_pdl.h"

namespace {

constexpr int NW = 4;                     // consumer warps per CTA
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
__device__ __forceinline__ void bulk_g2s(void* dst, const void* src, uint32_t bytes, uint64_t* bar) {
    asm volatile(
        "cp.async.bulk.shared::cluster.global.mbarrier::complete_tx::bytes [%0], [%1], %2, [%3];" ::"r"(
            su32(dst)),
        "l"(src), "r"(bytes), "r"(su32(bar))
        : "memory");
}

template <int DPL>
__device__ __forceinline__ void ld_row(const float* p, float (&v)[DPL]) {
    if constexpr (DPL == 4) {
        const float4 t = *(const float4*)p;
        v[0] = t.x; v[1] = t.y; v[2] = t.z; v[3] = t.w;
    } else if constexpr (DPL == 2) {
        const float2 t = *(const float2*)p;
        v[0] = t.x; v[1] = t.y;
    } else {
        v[0] = p[0];
    }
}
template <int DPL>
__device__ __forceinline__ void ld_row(const __half* p, float (&v)[DPL]) {
    if constexpr (DPL == 4) {
        const uint2 t = *(const uint2*)p;
        const float2 a = __half22float2(*(const __half2*)&t.x), b = __half22float2(*(const __half2*)&t.y);
        v[0] = a.x; v[1] = a.y; v[2] = b.x; v[3] = b.y;
    } else if constexpr (DPL == 2) {
        const uint32_t t = *(const uint32_t*)p;
        const float2 a = __half22float2(*(const __half2*)&t);
        v[0] = a.x; v[1] = a.y;
    } else {
        v[0] = __half2float(p[0]);
    }
}

// Sum of v[NV] over the warp's 32 lanes, spread so that lane l keeps the
// entries [l*NV/32, (l+1)*NV/32) when NV >= 32, or entry l >> log2(32/NV)
// (held by 32/NV lanes each) when NV < 32.  log2(32)=5 shuffle rounds; each
// round halves what a lane holds until one entry is left, then adds copies.
template <int NV>
__device__ __forceinline__ void transpose_reduce(float (&v)[NV], float (&out)[NV >= 32 ? NV / 32 : 1],
                                                 int lane) {
    int n = NV;
#pragma unroll
    for (int o = 16; o >= 1; o >>= 1) {
        if (n > 1) {
            const bool up = lane & o;
            const int h = n / 2;
#pragma unroll
            for (int i = 0; i < NV / 2; ++i) {
                if (i < h) {
                    const float send = up ? v[i] : v[i + h];
                    const float keep = up ? v[i + h] : v[i];
                    v[i] = keep + __shfl_xor_sync(0xffffffffu, send, o);
                }
            }
            n = h;
        } else {
            v[0] += __shfl_xor_sync(0xffffffffu, v[0], o);
        }
    }
#pragma unroll
    for (int i = 0; i < (NV >= 32 ? NV / 32 : 1); ++i) out[i] = v[i];
}

constexpr int ilog2(int x) { return x <= 1 ? 0 : 1 + ilog2(x / 2); }

template <int HD, int G, typename KT>
struct AttnShape {
    static constexpr int DPL = HD >= 32 ? HD / 32 : 1;
    static constexpr int ACTIVE = HD / DPL;
    // Page i uses stage i % STAGES and is consumed by warp i % NW.  With
    // STAGES a multiple of NW a stage always belongs to one warp, which waits
    // for its phases in order; otherwise a warp could wait two phases ahead of
    // another warp's pending use and the parity wait would alias.
    static constexpr int HEAD_ELEMS = 16 * HD;
    static constexpr int HEAD_BYTES = HEAD_ELEMS * (int)sizeof(KT);
    // about 64 KB of K/V in flight per CTA whatever the head size (8 KB pages
    // of a 64-wide f32 head get 8 stages, 16 KB ones 4), a multiple of NW
    static constexpr int STAGES_RAW = 65536 / (2 * HEAD_BYTES);
    static constexpr int STAGES = STAGES_RAW >= 16 ? 16 : STAGES_RAW >= 8 ? 8 : 4;
    static_assert(STAGES % NW == 0, "each ring stage must belong to one consumer warp");
    // scores are formed 8 tokens (half a page) at a time
    static constexpr int TOK = 8;
    static constexpr int NV = TOK * G;
    static constexpr int VPL = NV >= 32 ? NV / 32 : 1;       // entries per lane
    static constexpr int SH = NV >= 32 ? 0 : ilog2(32 / NV); // lanes per entry = 1 << SH
    static constexpr int GL = NV >= 32 ? TOK / VPL : (TOK << SH);  // lanes per head
    static constexpr size_t RING = (size_t)STAGES * 2 * HEAD_BYTES;
    static constexpr size_t MERGE = (size_t)NW * G * (HD + 2) * sizeof(float);
    static constexpr size_t SMEM = RING > MERGE ? RING : MERGE;
};

// ROWS (prompt chunks): one CTA per (NW consecutive rows of one sequence,
// kv_head, chunk).  Consumer warp w owns row b0 + w and every warp takes every
// page of the chunk (the empty barrier counts NW arrivals), masking tokens past
// its own row's position, so the chunk's K/V crosses HBM once for NW rows and
// each warp writes its row's (m, l, o) partial without a CTA merge.
template <int HD, int G, typename KT, bool ROWS>
__global__ void __launch_bounds__(32 * (NW + 1), G >= 8 ? 2 : 3) attn_chunk(
    const float* __restrict__ qkv, int ld_qkv, int B, int nq, int nkv,
    const int32_t* __restrict__ row_pos, const int32_t* __restrict__ row_slot,
    const int32_t* __restrict__ page_table, int max_pages, const KT* __restrict__ pool,
    int64_t n_pages, int layer, int nchunk_max, int ct, float* __restrict__ part, int* err) {
    using S = AttnShape<HD, G, KT>;
    constexpr int DPL = S::DPL, STAGES = S::STAGES, TOK = S::TOK, NV = S::NV, VPL = S::VPL,
                  SH = S::SH, GL = S::GL;
    extern __shared__ __align__(128) unsigned char smem_raw[];
    KT* ring = (KT*)smem_raw;                        // [STAGES][2][16][HD]; reused for the merge
    __shared__ uint64_t full[STAGES], empty[STAGES];
    __shared__ __align__(16) float p_s[NW][TOK * G]; // probabilities [token][head]
    __shared__ int pages_s[SB_ATTN_CHUNK / 16];

    const int tid = threadIdx.x, warp = tid >> 5, lane = tid & 31;
    sb_grid_release();   // the combine kernel may start its set-up
    sb_grid_wait();      // q, positions, pages, the appended K/V: after the previous kernel (sb_pdl.h)
    // chunk-major order: every row's first chunk is scheduled first, and the
    // shorter (partial or empty) later chunks fill the last waves
    const int nunit = ROWS ? (B + NW - 1) / NW : B;   // rows, or tiles of NW rows
    const int chunk = blockIdx.x / (nunit * nkv);
    const int rest = blockIdx.x % (nunit * nkv);
    const int kvh = rest % nkv, unit = rest / nkv;
    if (unit >= nunit) return;
    const int b0 = ROWS ? unit * NW : unit;
    // the longest context of the unit's rows, and the sequence of its first row
    // with a position (a row without one has no slot to trust)
    int ctx = 0, slot = -1;
#pragma unroll
    for (int w = 0; w < (ROWS ? NW : 1); ++w) {
        const int p = b0 + w < B ? row_pos[b0 + w] : -1;
        if (p >= 0) {
            ctx = max(ctx, p + 1);
            if (slot < 0) slot = row_slot[b0 + w];
        }
    }
    const int t0 = chunk * ct;
    if (t0 >= ctx) return;                            // also: no row with a position
    const int t1 = min(ctx, t0 + ct);
    const int npg = (t1 - t0 + 15) / 16;

    if (tid == 0) {
        for (int s = 0; s < STAGES; ++s) {
            bar_init(&full[s], 1);
            bar_init(&empty[s], ROWS ? NW : 1);
        }
        asm volatile("fence.mbarrier_init.release.cluster;" ::: "memory");
    }
    if (warp == NW) {
        // the chunk's page ids, fetched once so no copy waits on a table read
        for (int i = lane; i < npg; i += 32) {
            int page = page_table[(size_t)slot * max_pages + t0 / 16 + i];
            if (page < 0 || page >= n_pages) {      // never allocated: read page 0, flag it
                atomicCAS(err, 0, 6);
                page = 0;
            }
            pages_s[i] = page;
        }
    }
    __syncthreads();

    float* merge = (float*)smem_raw;                 // [NW][G][2 + HD] after the ring drains
    const bool dl = lane < S::ACTIVE;
    const int d0 = dl ? lane * DPL : 0;
    float q[G][DPL], o[G][DPL], m[G], l[G];          // consumer state
    if (warp == NW) {
        // ---------------- producer ----------------
        if (lane == 0) {
            const size_t hs = (size_t)S::HEAD_ELEMS;
            int issued = 0;
            for (int i = 0; i < npg; ++i) {
                const int s = i % STAGES;
                if (i >= STAGES && !bar_wait(&empty[s], ((i / STAGES) - 1) & 1, err, 4)) break;
                const KT* src = pool + (((size_t)layer * n_pages + pages_s[i]) * 2 * nkv + kvh) * hs;
                KT* dst = ring + (size_t)s * 2 * hs;
                bar_expect(&full[s], 2 * S::HEAD_BYTES);
                bulk_g2s(dst, src, S::HEAD_BYTES, &full[s]);
                bulk_g2s(dst + hs, src + (size_t)nkv * hs, S::HEAD_BYTES, &full[s]);
                issued = i + 1;
            }
            // no copy may still be landing when the ring is reused or the CTA exits
            for (int i = issued - STAGES > 0 ? issued - STAGES : 0; i < issued; ++i)
                bar_wait(&full[i % STAGES], (i / STAGES) & 1, err, 5);
        }
    } else {
        // ---------------- consumers ----------------
        // this warp's row and the end of its context inside the chunk
        const int b = ROWS ? b0 + warp : b0;
        int r1 = t1;
        if (ROWS) {
            r1 = b < B ? min(row_pos[b] + 1, t1) : 0;
            if (r1 > t0 && row_slot[b] != slot) {     // rows of another sequence: not a prompt chunk
                atomicCAS(err, 0, 8);
                r1 = 0;
            }
        }
        const bool live = r1 > t0;
#pragma unroll
        for (int h = 0; h < G; ++h) {
            const float* qp = qkv + (size_t)b * ld_qkv + (size_t)(kvh * G + h) * HD + d0;
#pragma unroll
            for (int i = 0; i < DPL; ++i) {
                q[h][i] = dl && live ? qp[i] : 0.f;
                o[h][i] = 0.f;
            }
            m[h] = -INFINITY;
            l[h] = 0.f;
        }
        const float scale = 1.0f / sqrtf((float)HD);
        for (int i = ROWS ? 0 : warp; i < npg; i += ROWS ? 1 : NW) {
            const int s = i % STAGES;
            if (!bar_wait(&full[s], (i / STAGES) & 1, err, 7)) break;
            const KT* kp0 = ring + (size_t)s * 2 * S::HEAD_ELEMS + d0;
            const KT* vp0 = kp0 + S::HEAD_ELEMS;
            const int nval_page = min(16, r1 - (t0 + 16 * i));   // <= 0: past this row's position
#pragma unroll 1
            for (int half = 0; half < 2; ++half) {
                const int nval = nval_page - TOK * half;   // valid tokens in this half (may be <= 0)
                if (nval <= 0) break;
                const KT* kp = kp0 + TOK * half * HD;
                const KT* vp = vp0 + TOK * half * HD;
                float part_s[NV];
                {
                    float kr[TOK][DPL];
#pragma unroll
                    for (int t = 0; t < TOK; ++t) {
                        if (dl && t < nval) ld_row<DPL>(kp + t * HD, kr[t]);
                        else
#pragma unroll
                            for (int c = 0; c < DPL; ++c) kr[t][c] = 0.f;
                    }
#pragma unroll
                    for (int h = 0; h < G; ++h)
#pragma unroll
                        for (int t = 0; t < TOK; ++t) {
                            if constexpr (DPL % 2 == 0) {
                                // dims in pairs on the paired f32 pipe (FMUL2 / FFMA2)
                                float2 a2 = __fmul2_rn(make_float2(q[h][0], q[h][1]),
                                                       make_float2(kr[t][0], kr[t][1]));
#pragma unroll
                                for (int c = 2; c < DPL; c += 2)
                                    a2 = __ffma2_rn(make_float2(q[h][c], q[h][c + 1]),
                                                    make_float2(kr[t][c], kr[t][c + 1]), a2);
                                part_s[h * TOK + t] = a2.x + a2.y;
                            } else {
                                float a = 0.f;
#pragma unroll
                                for (int c = 0; c < DPL; ++c) a = fmaf(q[h][c], kr[t][c], a);
                                part_s[h * TOK + t] = a;
                            }
                        }
                }
                float sv[VPL];
                transpose_reduce<NV>(part_s, sv, lane);
                float pmax = -INFINITY;
                int hh = 0;
#pragma unroll
                for (int j = 0; j < VPL; ++j) {
                    const int idx = NV >= 32 ? lane * VPL + j : lane >> SH;
                    hh = idx / TOK;
                    sv[j] = (idx % TOK) < nval ? sv[j] * scale : -INFINITY;
                    pmax = fmaxf(pmax, sv[j]);
                }
#pragma unroll
                for (int off = 1; off < GL; off <<= 1)
                    pmax = fmaxf(pmax, __shfl_xor_sync(0xffffffffu, pmax, off));
                float mloc = -INFINITY;
#pragma unroll
                for (int h = 0; h < G; ++h)
                    if (h == hh) mloc = fmaxf(m[h], pmax);
                float psum = 0.f;
#pragma unroll
                for (int j = 0; j < VPL; ++j) {
                    const int idx = NV >= 32 ? lane * VPL + j : lane >> SH;
                    const int t = idx % TOK;
                    const float pe = t < nval ? expf(sv[j] - mloc) : 0.f;
                    psum += pe;
                    p_s[warp][t * G + idx / TOK] = pe;     // copies write the same value
                }
#pragma unroll
                for (int off = 1 << SH; off < GL; off <<= 1)
                    psum += __shfl_xor_sync(0xffffffffu, psum, off);
#pragma unroll
                for (int h = 0; h < G; ++h) {
                    const float mn = __shfl_sync(0xffffffffu, mloc, h * GL);
                    const float sm = __shfl_sync(0xffffffffu, psum, h * GL);
                    const float corr = expf(m[h] - mn);
                    l[h] = l[h] * corr + sm;
                    if constexpr (DPL % 2 == 0) {
#pragma unroll
                        for (int c = 0; c < DPL; c += 2) {
                            const float2 r2 = __fmul2_rn(make_float2(o[h][c], o[h][c + 1]),
                                                         make_float2(corr, corr));
                            o[h][c] = r2.x;
                            o[h][c + 1] = r2.y;
                        }
                    } else {
#pragma unroll
                        for (int c = 0; c < DPL; ++c) o[h][c] *= corr;
                    }
                    m[h] = mn;
                }
                __syncwarp();
#pragma unroll
                for (int t = 0; t < TOK; ++t) {
                    float vr[DPL];
                    if (dl && t < nval) ld_row<DPL>(vp + t * HD, vr);
                    else
#pragma unroll
                        for (int c = 0; c < DPL; ++c) vr[c] = 0.f;
#pragma unroll
                    for (int h = 0; h < G; ++h) {
                        const float p = p_s[warp][t * G + h];
                        if constexpr (DPL % 2 == 0) {
#pragma unroll
                            for (int c = 0; c < DPL; c += 2) {
                                const float2 r2 = __ffma2_rn(make_float2(p, p), make_float2(vr[c], vr[c + 1]),
                                                             make_float2(o[h][c], o[h][c + 1]));
                                o[h][c] = r2.x;
                                o[h][c + 1] = r2.y;
                            }
                        } else {
#pragma unroll
                            for (int c = 0; c < DPL; ++c) o[h][c] = fmaf(p, vr[c], o[h][c]);
                        }
                    }
                }
                __syncwarp();
            }
            if (lane == 0) bar_arrive(&empty[s]);
        }
    }
    __syncthreads();                                  // ring drained: reuse it for the merge
    if constexpr (ROWS) {
        // each row's partial straight from its warp (the combine drops chunks
        // at or past a row's position, so a row without tokens here writes none)
        if (warp < NW && b0 + warp < B && t0 <= row_pos[b0 + warp]) {
#pragma unroll
            for (int h = 0; h < G; ++h) {
                float* out = part + (((size_t)(b0 + warp) * nq + kvh * G + h) * nchunk_max + chunk) *
                                        (HD + 2);
                if (lane == 0) {
                    out[0] = m[h];
                    out[1] = l[h];
                }
                if (dl)
#pragma unroll
                    for (int c = 0; c < DPL; ++c) out[2 + d0 + c] = o[h][c];
            }
        }
        return;
    }
    if (warp < NW) {
#pragma unroll
        for (int h = 0; h < G; ++h) {
            float* rec = merge + ((size_t)warp * G + h) * (HD + 2);
            if (lane == 0) {
                rec[0] = m[h];
                rec[1] = l[h];
            }
            if (dl)
#pragma unroll
                for (int c = 0; c < DPL; ++c) rec[2 + d0 + c] = o[h][c];
        }
    }
    __syncthreads();
    // merge the consumer warps: one thread per (head, dim)
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
        float* out = part + (((size_t)b0 * nq + kvh * G + h) * nchunk_max + chunk) * (HD + 2);
        if (d == 0) {
            out[0] = M;
            out[1] = L;
        }
        out[2 + d] = O;
    }
}

// Merge chunk partials: out = Σ_c o_c e^{m_c-M} / Σ_c l_c e^{m_c-M}, one CTA
// per (row, query head): warp 0 forms the chunk weights e^{m_c-M} / L (the
// chunks spread over its lanes), then thread d sums dim d over the chunks in
// chunk order with independent loads.  With hi != null the rows are also
// written as the f16 pair hi = f16(out), lo = f16(out - hi) (row stride ld16)
// that the next tensor-core GEMM takes.
constexpr int COMBINE_T = 128;            // threads per CTA: head_dim <= 128
constexpr int COMBINE_MAXCH = 12288;      // chunk weights in the default 48 KB of shared memory
template <int HD>
__global__ void __launch_bounds__(COMBINE_T) attn_combine(const float* __restrict__ part, int B, int nq,
                                                          const int32_t* __restrict__ row_pos,
                                                          int nchunk_max, int ct,
                                                          float* __restrict__ att, int ld_att,
                                                          __half* __restrict__ hi,
                                                          __half* __restrict__ lo, int ld16) {
    sb_grid_release();   // the Wo GEMM may start its set-up
    sb_grid_wait();      // chunk partials: after the previous kernel (sb_pdl.h)
    extern __shared__ float wch[];        // [nchunk_max] chunk weights
    const int tid = threadIdx.x, lane = tid & 31;
    const int hq = (int)(blockIdx.x % nq);
    const int b = (int)(blockIdx.x / nq);
    if (b >= B) return;
    const int pos = row_pos[b];
    if (pos < 0) return;
    const int nch = min((pos + ct) / ct, nchunk_max);    // ceil((pos + 1) / ct)
    const float* rec0 = part + ((size_t)b * nq + hq) * nchunk_max * (HD + 2);
    if (tid < 32) {
        float M = -INFINITY;
        for (int c = lane; c < nch; c += 32) M = fmaxf(M, rec0[(size_t)c * (HD + 2)]);
#pragma unroll
        for (int o = 16; o > 0; o >>= 1) M = fmaxf(M, __shfl_xor_sync(0xffffffffu, M, o));
        double L = 0.0;
        for (int c = lane; c < nch; c += 32) {
            const float* r = rec0 + (size_t)c * (HD + 2);
            const float e = expf(r[0] - M);
            wch[c] = e;
            L += (double)r[1] * (double)e;
        }
#pragma unroll
        for (int o = 16; o > 0; o >>= 1) L += __shfl_xor_sync(0xffffffffu, L, o);
        const float invL = (float)(1.0 / L);
        __syncwarp();
        for (int c = lane; c < nch; c += 32) wch[c] *= invL;
    }
    __syncthreads();
    const int d = tid;
    if (d >= HD) return;
    float acc = 0.f;
    const float* r = rec0 + 2 + d;
#pragma unroll 8
    for (int c = 0; c < nch; ++c) acc = fmaf(r[(size_t)c * (HD + 2)], wch[c], acc);
    att[(size_t)b * ld_att + (size_t)hq * HD + d] = acc;
    if (hi) {
        const __half h = __float2half_rn(acc);
        hi[(size_t)b * ld16 + (size_t)hq * HD + d] = h;
        if (lo) lo[(size_t)b * ld16 + (size_t)hq * HD + d] = __float2half_rn(acc - __half2float(h));
    }
}

// The same merge with one warp per (row, query head), four per CTA: for large
// batches, where there are (row, head) pairs enough to fill the GPU with warps
// and a CTA per pair would only add scheduling and a barrier.
template <int HD>
__global__ void __launch_bounds__(128) attn_combine_warp(const float* __restrict__ part, int B, int nq,
                                                    const int32_t* __restrict__ row_pos,
                                                    int nchunk_max, int ct, float* __restrict__ att,
                                                    int ld_att, __half* __restrict__ hi,
                                                    __half* __restrict__ lo, int ld16) {
    sb_grid_release();   // the Wo GEMM may start its set-up
    sb_grid_wait();      // chunk partials: after the previous kernel (sb_pdl.h)
    const int lane = threadIdx.x & 31;
    const long w = (long)blockIdx.x * 4 + (threadIdx.x >> 5);
    const int hq = (int)(w % nq);
    const int b = (int)(w / nq);
    if (b >= B) return;
    const int pos = row_pos[b];
    if (pos < 0) return;
    const int nch = (pos + ct) / ct;                      // ceil((pos + 1) / ct)
    const float* rec0 = part + ((size_t)b * nq + hq) * nchunk_max * (HD + 2);
    // the chunks' maxima and weighted sums, spread over the lanes
    float M = -INFINITY;
    for (int c = lane; c < nch; c += 32) M = fmaxf(M, rec0[(size_t)c * (HD + 2)]);
#pragma unroll
    for (int o = 16; o > 0; o >>= 1) M = fmaxf(M, __shfl_xor_sync(0xffffffffu, M, o));
    double L = 0.0;
    for (int c = lane; c < nch; c += 32) {
        const float* r = rec0 + (size_t)c * (HD + 2);
        L += (double)r[1] * (double)expf(r[0] - M);
    }
#pragma unroll
    for (int o = 16; o > 0; o >>= 1) L += __shfl_xor_sync(0xffffffffu, L, o);
    const float invL = (float)(1.0 / L);
    // out[d] = sum_c o_c[d] e^{m_c - M}, chunks in order: lane c0 + j holds
    // chunk c0 + j's weight, broadcast to the warp; the loads of successive
    // chunks are independent of one another
    constexpr int DPL = (HD + 31) / 32;
    float acc[DPL];
#pragma unroll
    for (int i = 0; i < DPL; ++i) acc[i] = 0.f;
    for (int c0 = 0; c0 < nch; c0 += 32) {
        const int cl = c0 + lane;
        const float wl = cl < nch ? expf(rec0[(size_t)cl * (HD + 2)] - M) : 0.f;
        const int cn = min(32, nch - c0);
#pragma unroll 8
        for (int j = 0; j < cn; ++j) {
            const float wj = __shfl_sync(0xffffffffu, wl, j);
            const float* r = rec0 + (size_t)(c0 + j) * (HD + 2) + 2;
#pragma unroll
            for (int i = 0; i < DPL; ++i) {
                const int d = lane + 32 * i;
                if (d < HD) acc[i] = fmaf(r[d], wj, acc[i]);
            }
        }
    }
#pragma unroll
    for (int i = 0; i < DPL; ++i) {
        const int d = lane + 32 * i;
        if (d >= HD) break;
        const float o = acc[i] * invL;
        att[(size_t)b * ld_att + (size_t)hq * HD + d] = o;
        if (hi) {
            const __half h = __float2half_rn(o);
            hi[(size_t)b * ld16 + (size_t)hq * HD + d] = h;
            if (lo) lo[(size_t)b * ld16 + (size_t)hq * HD + d] = __float2half_rn(o - __half2float(h));
        }
    }
}

// prepare != 0: only opt the instantiation into its shared-memory size (the
// dynamic ring plus static state can exceed the 48 KB default); this happens
// per device and outside any stream capture.
struct HiLo {
    __half* hi;
    __half* lo;
    int ld16;
};

// The merge of the chunk partials: a CTA per (row, query head) while there
// are few such pairs (small batches, many chunks each), a warp per pair beyond
// COMBINE_CTA_MAX of them (chunk kernel + merge per layer on B200 at the 8B
// shape, f32 KV: at 1 row 12.0 against 14.0 us, at 64 rows even, at 256 rows
// 0.711 against 0.708 ms).
#ifndef COMBINE_CTA_MAX
#define COMBINE_CTA_MAX 2048
#endif
template <int HD>
int launch_combine(const float* scratch, int B, int nq, const int32_t* row_pos, int nchunk, int ct,
                   float* att, int ld_att, HiLo hl, cudaStream_t st) {
    const long cw = (long)B * nq;
    const cudaError_t e =
        cw > COMBINE_CTA_MAX
            ? sb_launch_pdl(attn_combine_warp<HD>, dim3((unsigned)((cw + 3) / 4)), dim3(128), 0, st,
                            scratch, B, nq, row_pos, nchunk, ct, att, ld_att, hl.hi, hl.lo, hl.ld16)
            : sb_launch_pdl(attn_combine<HD>, dim3((unsigned)cw), dim3(COMBINE_T), (size_t)nchunk * 4,
                            st, scratch, B, nq, row_pos, nchunk, ct, att, ld_att, hl.hi, hl.lo,
                            hl.ld16);
    return e == cudaSuccess ? 0 : -1;
}

template <int HD, int G, typename KT>
int launch_g(int prepare, int rows, float* att, int ld_att, const float* qkv, int ld_qkv, int B,
             int nq, int nkv, const int32_t* row_pos, const int32_t* row_slot,
             const int32_t* page_table, int max_pages, const void* pool, int64_t n_pages, int layer,
             int nchunk, int ct, float* scratch, int* err, HiLo hl, cudaStream_t st) {
    using S = AttnShape<HD, G, KT>;
    if (prepare) {
        for (auto f : {attn_chunk<HD, G, KT, false>, attn_chunk<HD, G, KT, true>}) {
            cudaFuncSetAttribute(f, cudaFuncAttributeMaxDynamicSharedMemorySize, (int)S::SMEM);
            cudaFuncSetAttribute(f, cudaFuncAttributePreferredSharedMemoryCarveout, 100);
        }
        return 0;
    }
    const long ctas = (long)(rows ? (B + NW - 1) / NW : B) * nkv * nchunk;
    if (sb_launch_pdl(rows ? attn_chunk<HD, G, KT, true> : attn_chunk<HD, G, KT, false>,
                      dim3((unsigned)ctas), dim3(32 * (NW + 1)), S::SMEM, st, qkv, ld_qkv, B, nq,
                      nkv, row_pos, row_slot, page_table, max_pages, (const KT*)pool, n_pages,
                      layer, nchunk, ct, scratch, err) != cudaSuccess)
        return -1;
    return launch_combine<HD>(scratch, B, nq, row_pos, nchunk, ct, att, ld_att, hl, st);
}

template <int HD, typename KT>
int launch_hd(int prepare, int rows, int G, float* att, int ld_att, const float* qkv, int ld_qkv, int B,
              int nq, int nkv, const int32_t* row_pos, const int32_t* row_slot,
              const int32_t* page_table, int max_pages, const void* pool, int64_t n_pages,
              int layer, int nchunk, int ct, float* scratch, int* err, HiLo hl, cudaStream_t st) {
    switch (G) {
#define CASE(g)                                                                                  \
    case g:                                                                                      \
        return launch_g<HD, g, KT>(prepare, rows, att, ld_att, qkv, ld_qkv, B, nq, nkv, row_pos,       \
                                   row_slot, page_table, max_pages, pool, n_pages, layer,        \
                                   nchunk, ct, scratch, err, hl, st);
        CASE(1) CASE(2) CASE(4) CASE(8)
#undef CASE
    }
    return -1;
}

template <typename KT>
int launch_kt(int prepare, int rows, int hd, int G, float* att, int ld_att, const float* qkv, int ld_qkv,
              int B, int nq, int nkv, const int32_t* row_pos, const int32_t* row_slot,
              const int32_t* page_table, int max_pages, const void* pool, int64_t n_pages,
              int layer, int nchunk, int ct, float* scratch, int* err, HiLo hl, cudaStream_t st) {
    switch (hd) {
#define CASE(h)                                                                                  \
    case h:                                                                                      \
        return launch_hd<h, KT>(prepare, rows, G, att, ld_att, qkv, ld_qkv, B, nq, nkv, row_pos,       \
                                row_slot, page_table, max_pages, pool, n_pages, layer, nchunk,   \
                                ct, scratch, err, hl, st);
        CASE(8) CASE(16) CASE(32) CASE(64) CASE(128)
#undef CASE
    }
    return -1;
}

int combine(int hd, const float* scratch, int B, int nq, const int32_t* row_pos, int nchunk,
            int ct, float* att, int ld_att, HiLo hl, cudaStream_t st) {
    switch (hd) {
        case 64: return launch_combine<64>(scratch, B, nq, row_pos, nchunk, ct, att, ld_att, hl, st);
        case 128: return launch_combine<128>(scratch, B, nq, row_pos, nchunk, ct, att, ld_att, hl, st);
    }
    return -1;
}

int dispatch(int prepare, int rows, float* att, int ld_att, const float* qkv, int ld_qkv, int B,
             int nq, int nkv, int hd, const int32_t* row_pos, const int32_t* row_slot,
             const int32_t* page_table, int max_pages, const void* pool, const void* kvmap,
             int64_t n_pages, int layer, int kv_dtype, int max_seq, int ct, float* scratch,
             int* err, HiLo hl, cudaStream_t st) {
    if (nkv < 1 || nq % nkv) return -1;
    const int G = nq / nkv;
    if (ct <= 0) ct = sb_attention_chunk_tokens(B);
    if (ct < 16 || ct > SB_ATTN_CHUNK || ct % 16) return -1;
    const int nchunk = (max_seq + ct - 1) / ct;
    if (nchunk > COMBINE_MAXCH) return -1;
    if (sb_attention_mma_supported(nq, nkv, hd, kv_dtype)) {
        if (prepare) {
            const int rc = sb_attention_mma(1, nullptr, nullptr, 0, 0, nq, nkv, hd, nullptr, nullptr,
                                            nullptr, 0, 0, 0, 0, 0, nullptr, nullptr, 0);
            if (rc) return rc;          // the CUDA-core kernel is prepared too (calls without a map)
        } else if (kvmap) {
            const int rc = sb_attention_mma(0, kvmap, qkv, ld_qkv, B, nq, nkv, hd, row_pos, row_slot,
                                            page_table, max_pages, n_pages, layer, nchunk, ct,
                                            scratch, err, st);
            return rc ? rc : combine(hd, scratch, B, nq, row_pos, nchunk, ct, att, ld_att, hl, st);
        }
    }
    // a prompt chunk of fewer than NW rows gains nothing from row tiles
    rows = rows && B >= NW;
    return kv_dtype == SLATE_KV_F16
               ? launch_kt<__half>(prepare, rows, hd, G, att, ld_att, qkv, ld_qkv, B, nq, nkv, row_pos,
                                   row_slot, page_table, max_pages, pool, n_pages, layer, nchunk,
                                   ct, scratch, err, hl, st)
               : launch_kt<float>(prepare, rows, hd, G, att, ld_att, qkv, ld_qkv, B, nq, nkv, row_pos,
                                  row_slot, page_table, max_pages, pool, n_pages, layer, nchunk,
                                  ct, scratch, err, hl, st);
}

}  // namespace

extern "C" int sb_attention_chunk_tokens(int B) {
    return B >= 16 ? SB_ATTN_CHUNK : B >= 8 ? SB_ATTN_CHUNK / 2 : B >= 4 ? SB_ATTN_CHUNK / 4
                                   : B >= 3 ? SB_ATTN_CHUNK / 8 : SB_ATTN_CHUNK / 16;
}

extern "C" size_t sb_attention_scratch_rows(int B, int nq, int hd, int max_seq, int ct) {
    return (size_t)B * nq * ((max_seq + ct - 1) / ct) * (hd + 2);
}

extern "C" size_t sb_attention_scratch_floats(int max_batch, int nq, int hd, int max_seq) {
    size_t best = 0;
    for (int B = 1; B <= max_batch; ++B) {
        const size_t f = sb_attention_scratch_rows(B, nq, hd, max_seq, sb_attention_chunk_tokens(B));
        if (f > best) best = f;
    }
    return best;
}

extern "C" int sb_attention_prepare(int nq, int nkv, int hd, int kv_dtype) {
    return dispatch(1, 0, nullptr, 0, nullptr, 0, 0, nq, nkv, hd, nullptr, nullptr, nullptr, 0,
                    nullptr, nullptr, 0, 0, kv_dtype, 0, SB_ATTN_CHUNK, nullptr, nullptr,
                    HiLo{nullptr, nullptr, 0}, 0);
}

extern "C" int sb_attention_paged(float* att, int ld_att, const float* qkv, int ld_qkv, int B,
                                  int nq, int nkv, int hd, const int32_t* row_pos,
                                  const int32_t* row_slot, const int32_t* page_table,
                                  int max_pages, const void* pool, const void* kvmap,
                                  int64_t n_pages, int layer, int kv_dtype, int max_seq, int ct,
                                  float* scratch, int* err, cudaStream_t st) {
    if (B < 1 || !err) return -1;
    return dispatch(0, 0, att, ld_att, qkv, ld_qkv, B, nq, nkv, hd, row_pos, row_slot, page_table,
                    max_pages, pool, kvmap, n_pages, layer, kv_dtype, max_seq, ct, scratch, err,
                    HiLo{nullptr, nullptr, 0}, st);
}

extern "C" int sb_attention_paged_prefill(float* att, int ld_att, const float* qkv, int ld_qkv,
                                          int B, int nq, int nkv, int hd, const int32_t* row_pos,
                                          const int32_t* row_slot, const int32_t* page_table,
                                          int max_pages, const void* pool, const void* kvmap,
                                          int64_t n_pages, int layer, int kv_dtype, int max_seq,
                                          float* scratch, int* err, void* hi, void* lo, int ld16,
                                          cudaStream_t st) {
    if (B < 1 || !err || (hi && ld16 < nq * hd)) return -1;
    const HiLo hl{(__half*)hi, (__half*)lo, hi ? ld16 : 0};
    if (!kvmap || !sb_attention_mma_supported(nq, nkv, hd, kv_dtype))
        return dispatch(0, 1, att, ld_att, qkv, ld_qkv, B, nq, nkv, hd, row_pos, row_slot, page_table,
                        max_pages, pool, kvmap, n_pages, layer, kv_dtype, max_seq, 0, scratch, err,
                        hl, st);
    const int nchunk = (max_seq + SB_ATTN_CHUNK - 1) / SB_ATTN_CHUNK;
    const int rc = sb_attention_prefill_mma(kvmap, qkv, ld_qkv, B, nq, nkv, hd, row_pos, row_slot,
                                            page_table, max_pages, n_pages, layer, nchunk, scratch,
                                            err, st);
    return rc ? rc : combine(hd, scratch, B, nq, row_pos, nchunk, SB_ATTN_CHUNK, att, ld_att, hl,
                             st);
}

extern "C" int sb_attention_paged_split(float* att, int ld_att, const float* qkv, int ld_qkv, int B,
                                        int nq, int nkv, int hd, const int32_t* row_pos,
                                        const int32_t* row_slot, const int32_t* page_table,
                                        int max_pages, const void* pool, const void* kvmap,
                                        int64_t n_pages, int layer, int kv_dtype, int max_seq,
                                        float* scratch, int* err, void* hi, void* lo, int ld16,
                                        cudaStream_t st) {
    if (B < 1 || !err || !hi || ld16 < nq * hd) return -1;
    return dispatch(0, 0, att, ld_att, qkv, ld_qkv, B, nq, nkv, hd, row_pos, row_slot, page_table,
                    max_pages, pool, kvmap, n_pages, layer, kv_dtype, max_seq, 0, scratch, err,
                    HiLo{(__half*)hi, (__half*)lo, ld16}, st);
}
