// attn_noalloc.cu -- paged GQA attention that allocates no device memory.
//
// The vtable's attention_paged_gqa takes its chunk partials and error word
// from cudaMallocAsync on every call.  Some callers cannot allocate device
// memory at that point: a serving process whose allocator has already handed
// all free HBM to its KV page pool (a cudaMalloc at decode time would fail),
// or a latency-critical loop that must not let the driver's allocator
// synchronise or grow a memory pool mid-step.  This entry point runs the same
// kernels with their scratch in a fixed file-scope device array instead.
//
// Scratch: SLATE_CUDA_NOALLOC_SCRATCH_FLOATS floats of partial records plus
// one error word.  A call needs B * n_heads * ceil(max_pages * 16 / ct) *
// (head_dim + 2) floats, ct being the engine's attention chunk for B rows
// (sb_attention_chunk_tokens: 64 tokens below 3 rows, 128 at 3, up to 1024 from 16),
// doubled up to 1024 tokens until the partials fit; a request that does not
// fit even with 1024-token chunks is rejected with -1 and a message before
// any device work.  Every call on a device shares the one
// array: calls whose kernels overlap on the GPU (two host threads, or two
// streams) race on it, so the caller serialises them.
//
// Set-up: the first call on a device (with that device current) resolves the
// array's device address with cudaGetSymbolAddress and keeps it; make that
// first call before any stream capture.  Every call is synchronous: it waits
// for its stream to read the kernels' error word before it returns.  The error word is cleared on the
// stream before each launch; the partials need no clearing (each record the
// combine reads is written first by the same call).
#include <cuda_runtime.h>
#include <stdint.h>
#include <stdlib.h>

#include <mutex>

#include "sb_internal.h"
#include "sb_kernels.h"

namespace {

constexpr int kMaxDevices = 64;
static __device__ __align__(256) float g_scratch[SLATE_CUDA_NOALLOC_SCRATCH_FLOATS + 64];
std::mutex g_mu;
float* g_base[kMaxDevices];

// Device address of g_scratch on the current device (resolved once per device).
float* scratch_base(int* rc) {
    int dev = -1;
    if ((*rc = sb_cuda_check(cudaGetDevice(&dev), "cudaGetDevice"))) return nullptr;
    if (dev < 0 || dev >= kMaxDevices) {
        sb_set_error("attention (no-alloc): device ordinal %d above %d", dev, kMaxDevices - 1);
        *rc = -1;
        return nullptr;
    }
    std::lock_guard<std::mutex> g(g_mu);
    if (!g_base[dev]) {
        void* p = nullptr;
        if ((*rc = sb_cuda_check(cudaGetSymbolAddress(&p, g_scratch), "cudaGetSymbolAddress")))
            return nullptr;
        g_base[dev] = (float*)p;
    }
    return g_base[dev];
}

}  // namespace

extern "C" int slate_cuda_attention_paged_gqa_noalloc(float* out, const float* q,
                                                      const int32_t* pos, const int32_t* row_slot,
                                                      const int32_t* page_table, int max_pages,
                                                      const void* kv_pool, int64_t n_pages,
                                                      int layer, int B, int nq, int nkv, int hd,
                                                      int kv_dtype, void* stream) {
    if (!out || !q || !pos || !row_slot || !page_table || !kv_pool || max_pages < 1 ||
        n_pages < 1 || layer < 0 || B < 1 || nq < 1 || nkv < 1 || nq % nkv || hd < 1 ||
        (kv_dtype != SLATE_KV_F32 && kv_dtype != SLATE_KV_F16)) {
        sb_set_error("attention (no-alloc): bad arguments");
        return -1;
    }
    const int max_seq = max_pages * 16;
    // the engine's chunk for B rows, lengthened until the partials fit
    int ct = sb_attention_chunk_tokens(B);
    while (ct < SB_ATTN_CHUNK &&
           sb_attention_scratch_rows(B, nq, hd, max_seq, ct) > (size_t)SLATE_CUDA_NOALLOC_SCRATCH_FLOATS)
        ct *= 2;
    const size_t need = sb_attention_scratch_rows(B, nq, hd, max_seq, ct);
    if (need > (size_t)SLATE_CUDA_NOALLOC_SCRATCH_FLOATS) {
        sb_set_error("attention (no-alloc): %zu scratch floats needed (B %d x heads %d x %d chunks "
                     "x %d), limit %zu",
                     need, B, nq, (max_seq + ct - 1) / ct, hd + 2,
                     (size_t)SLATE_CUDA_NOALLOC_SCRATCH_FLOATS);
        return -1;
    }
    int rc = 0;
    float* scr = scratch_base(&rc);
    if (!scr) return rc;
    int* err = (int*)(scr + SLATE_CUDA_NOALLOC_SCRATCH_FLOATS);
    cudaStream_t st = (cudaStream_t)stream;
    if (sb_attention_prepare(nq, nkv, hd, kv_dtype)) {
        sb_set_error("attention (no-alloc): no kernel for head_dim %d, group %d", hd, nq / nkv);
        return -1;
    }
    if ((rc = sb_cuda_check(cudaMemsetAsync(err, 0, sizeof(int), st), "clear error word")))
        return rc;
    // same kernel choice as attention_paged_gqa: tensor cores for supported f16 shapes
    unsigned char map[SB_KVMAP_BYTES];
    const void* mapp = nullptr;
    const char* path = getenv("SLATE_CUDA_ATTN_PATH");
    if (sb_attention_mma_supported(nq, nkv, hd, kv_dtype) && !(path && path[0] == '1')) {
        if (sb_attention_make_map(map, (void*)kv_pool, n_pages, layer + 1, nkv, hd)) return -1;
        mapp = map;
    }
    if (sb_attention_paged(out, nq * hd, q, nq * hd, B, nq, nkv, hd, pos, row_slot, page_table,
                           max_pages, kv_pool, mapp, n_pages, layer, kv_dtype, max_seq, ct, scr,
                           err, st)) {
        sb_set_error("attention (no-alloc): unsupported shape");
        return -1;
    }
    if ((rc = sb_cuda_check(cudaGetLastError(), "attention (no-alloc) launch"))) return rc;
    int e = 0;
    if ((rc = sb_cuda_check(cudaMemcpyAsync(&e, err, sizeof(int), cudaMemcpyDeviceToHost, st),
                            "read error word")))
        return rc;
    if ((rc = sb_cuda_check(cudaStreamSynchronize(st), "attention (no-alloc)"))) return rc;
    if (e) {
        sb_set_error("attention (no-alloc): pipeline reported %d", e);
        return -5;
    }
    return 0;
}
