/*
 * sb_tc.h -- tensor-core (tcgen05) Q4_K GEMM launchers (internal).
 */
#ifndef SB_TC_H
#define SB_TC_H

#include <stdint.h>
#include <cuda_runtime_api.h>
#include "sb_kernels.h"

#ifdef __cplusplus
extern "C" {
#endif

/* An f16 activation operand [rows][K] (row stride ld16 elements) with its
 * TMA tensor maps (SWIZZLE_128B boxes of 64 x n_box).  `lo` (nullable) holds
 * f16(x - hi) for the 3-pass split. */
#ifdef __cplusplus
#define SB_ALIGN64 alignas(64)
#else
#define SB_ALIGN64 _Alignas(64)
#endif
typedef struct sb_tc_operand {
    SB_ALIGN64 unsigned char map_hi[128];   /* CUtensorMap */
    SB_ALIGN64 unsigned char map_lo[128];
    void* hi;
    void* lo;
    int rows, K, ld16, n_box;
} sb_tc_operand;

int sb_tc_make_operand(sb_tc_operand* op, void* hi, void* lo, int rows, int K, int ld16);
/* X (f32, stride ldx) -> op->hi / op->lo for the first n_rows rows. */
int sb_tc_split(const float* X, int ldx, int n_rows, const sb_tc_operand* op, cudaStream_t st);
/* K-split count that fills the GPU for a weight of M_pad rows. */
int sb_tc_splits_for(int M_pad, int K);
/* ws: splits * n_rows * W->M_pad floats.  passes: 1 (f16 x f16) or 3 (hi/lo). */
int sb_tc_gemm(const sb_matrix* W, const sb_tc_operand* X, int n_rows, int passes, int splits,
               float* ws, float* Y, int ldy, int epi, int* err, cudaStream_t st);
/* Shared-memory attributes (outside stream capture). */
void sb_tc_prepare(void);

/* An f32 weight [M][K] held as an f16 pair (hi = f16(w), lo = f16(w - hi),
 * M padded to 128 with zeros) with TMA maps, for the 3-pass tensor-core GEMM
 * without dequantisation (the f32 LM head). */
typedef struct sb_tc_weight {
    SB_ALIGN64 unsigned char map_hi[128];
    SB_ALIGN64 unsigned char map_lo[128];
    void* hi;
    void* lo;
    int M, M_pad, K;
    int wexp;    /* the pair holds W * 2^wexp (exact; keeps the lo halves normal) */
} sb_tc_weight;
/* Splits the device f32 matrix W32 (row stride ldw) into a new pair. */
int sb_tc_make_weight(sb_tc_weight* w, const float* W32, int ldw, int M, int K, cudaStream_t st);
void sb_tc_free_weight(sb_tc_weight* w);
/* Y[n][m] (=, +=) X[n] . W[m] for m < M with the 3-pass split (epi STORE / ADD). */
int sb_tc_gemm_f16w(const sb_tc_weight* W, const sb_tc_operand* X, int n_rows, float* Y, int ldy,
                    int epi, int* err, cudaStream_t st);

/* Operand of the exact-weight Q4_K GEMM (gemm_q4k.cu): f16 hi / lo rows
 * [rows][ld16] with TMA maps of 64 x 128 boxes, plus the per-sub-block sums
 * of x as f16 hi / lo in [K/256 rounded up to even][r_pad][8] (r_pad: rows
 * rounded up to 128; zero-filled once, the padding block stays zero). */
typedef struct sb_q4_operand {
    SB_ALIGN64 unsigned char map_hi[128];    /* x boxes 64 x 128 (one-SM kernel) */
    SB_ALIGN64 unsigned char map_lo[128];
    SB_ALIGN64 unsigned char map2_hi[128];   /* x boxes 64 x 64 (two-SM kernel) */
    SB_ALIGN64 unsigned char map2_lo[128];
    SB_ALIGN64 unsigned char xsmap_hi[128];  /* sub-block sums, boxes 8 x 64 */
    SB_ALIGN64 unsigned char xsmap_lo[128];
    void *hi, *lo, *xs_hi, *xs_lo;
    int rows, r_pad, K, ld16;
    int one_pass;                            /* 1: the GEMM reads x's f16 rounding only */
} sb_q4_operand;
int sb_q4_make_operand(sb_q4_operand* op, void* hi, void* lo, void* xs_hi, void* xs_lo, int rows,
                       int r_pad, int K, int ld16);
/* X (f32, stride ldx, ldx % 4 == 0) -> hi / lo / sub-block sums, n_rows rows. */
int sb_q4_split(const float* X, int ldx, int n_rows, const sb_q4_operand* op, cudaStream_t st);
/* Y[n][m] (=, +=, SiLU(gate)*up) over Q4_K W for n < n_rows, two f16 passes with
 * exact weights; weights with M_pad % 256 == 0 run on CTA pairs (cta_group::2)
 * unless SLATE_Q4_ONE_SM=1.  ws: sb_q4_ws_floats() floats; cnt: sb_q4_tiles(M_pad, n_rows)
 * ints, zero before the first call (the kernel leaves them zero). */
int sb_q4_gemm(const sb_matrix* W, const sb_q4_operand* X, int n_rows, float* Y, int ldy, int epi,
               float* ws, int* cnt, int* err, cudaStream_t st);
size_t sb_q4_ws_floats(void);
int sb_q4_tiles(int M_pad, int n_rows);
/* SM count and shared-memory attribute on the current device (outside capture;
 * before sb_q4_ws_floats). */
void sb_q4_prepare(void);

/* Three-pass Q4_K GEMM on a persistent stream-K grid (gemm_sk.cu): Y[n][m]
 * (=, +=, SiLU(gate)*up) over Q4_K W for n < n_rows with X's f16 hi / lo pair.
 * Tiles split between CTAs, and SiLU tiles, are finished by a second launch.
 * ws: sb_sk_ws_floats(t) floats, t >= sb_sk_tiles(M_pad, n_rows) of every
 * SiLU weight it is used with (0 if none).  SiLU needs W->M % 128 == 0 (gate rows 0-63 and up
 * rows 64-127 of every 128-row tile) and may also write the result as an f16
 * hi / lo pair (h_hi / h_lo, row stride ld16; NULL: not written), the operand
 * of the GEMM that follows.  SB_EPI_ROPE (the fused Q|K|V weight, `rope`
 * non-NULL, 128 % head_dim == 0) rotates the query heads in place in Y and
 * writes the rotated keys and the values into the paged cache instead of Y;
 * its tiles also need the workspace's tile areas (t >= the QKV tiles). */
int sb_sk_gemm(const sb_matrix* W, const sb_tc_operand* X, int n_rows, float* ws, float* Y,
               int ldy, int epi, void* h_hi, void* h_lo, int ld16, const sb_rope_args* rope,
               int* err, cudaStream_t st);
size_t sb_sk_ws_floats(int max_silu_tiles);
/* Kernel launches of one sb_sk_gemm call (1, or 2 with the output pass). */
int sb_sk_kernels(int M_pad, int K, int n_rows, int epi);
int sb_sk_tiles(int M_pad, int n_rows);
/* SM count and shared-memory attribute on the current device (outside capture). */
void sb_sk_prepare(void);

#ifdef __cplusplus
}
#endif
#endif
