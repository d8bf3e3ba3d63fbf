/*
 * sb_internal.h -- shared host-side helpers of libslate_cuda.so (not public).
 */
#ifndef SB_INTERNAL_H
#define SB_INTERNAL_H

#include <stdarg.h>
#include <stdint.h>
#include <cuda_runtime_api.h>
#include "slate_cuda.h"

#ifdef __cplusplus
extern "C" {
#endif

/* Records a message retrievable by slate_cuda_last_error() (thread-local). */
void sb_set_error(const char* fmt, ...);
/* Records the CUDA error text for `what` and returns -5 when e != success. */
int sb_cuda_check(cudaError_t e, const char* what);
#define SB_CU(call) do { int rc_ = sb_cuda_check((call), #call); if (rc_) return rc_; } while (0)

/* f16 bits -> f32 (exact), host side. */
float sb_f16_to_f32(uint16_t h);
/* Dequantises `rows` Q4_K rows of K elements (Slate layout) into f32. */
void sb_q4k_dequant_rows(float* dst, const void* src, int64_t rows, int K);

/* Sets the shared-memory attributes of every GEMM instantiation on the
 * current device (must happen outside stream capture). */
void sb_gemm_prepare(void);

#ifdef __cplusplus
}
#endif
#endif
