/*
 * common.c -- error reporting and small host-side numerics shared by the
 * engine, the backend vtable and the helpers.
 */
#include "sb_internal.h"

#include <stdio.h>
#include <string.h>

static __thread char g_err[512];

void sb_set_error(const char* fmt, ...) {
    va_list ap;
    va_start(ap, fmt);
    vsnprintf(g_err, sizeof g_err, fmt, ap);
    va_end(ap);
}

const char* slate_cuda_last_error(void) { return g_err; }

int sb_cuda_check(cudaError_t e, const char* what) {
    if (e == cudaSuccess) return 0;
    sb_set_error("%s: %s", what, cudaGetErrorString(e));
    return -5;
}

/* IEEE binary16 -> binary32 (exact; subnormals renormalised), the conversion
 * of the reference's util/precision.c:10-29. */
float sb_f16_to_f32(uint16_t h) {
    uint32_t sign = ((uint32_t)h & 0x8000u) << 16;
    uint32_t e = (h >> 10) & 0x1fu, m = h & 0x3ffu, bits;
    if (e == 0) {
        if (m == 0) {
            bits = sign;
        } else {
            int sh = 0;
            while (!(m & 0x400u)) { m <<= 1; ++sh; }
            bits = sign | ((uint32_t)(113 - sh) << 23) | ((m & 0x3ffu) << 13);
        }
    } else if (e == 31) {
        bits = sign | 0x7f800000u | (m << 13);
    } else {
        bits = sign | ((e + 112u) << 23) | (m << 13);
    }
    float f;
    memcpy(&f, &bits, 4);
    return f;
}

/* Q4_K reconstruction d*sc*q - dmin*mn in Slate's nibble order
 * (util/quant.c:168-202), used when a fused weight group mixes dtypes. */
void sb_q4k_dequant_rows(float* dst, const void* src, int64_t rows, int K) {
    const uint8_t* p = (const uint8_t*)src;
    const int64_t nb = (int64_t)rows * (K / 256);
    for (int64_t b = 0; b < nb; ++b) {
        const uint8_t* blk = p + b * 144;
        uint16_t dh, mh;
        memcpy(&dh, blk, 2);
        memcpy(&mh, blk + 2, 2);
        const float d = sb_f16_to_f32(dh), dmin = sb_f16_to_f32(mh);
        const uint8_t* s = blk + 4;
        for (int j = 0; j < 8; ++j) {
            int sc, mn;
            if (j < 4) {
                sc = s[j] & 63;
                mn = s[j + 4] & 63;
            } else {
                sc = (s[j + 4] & 15) | ((s[j - 4] >> 6) << 4);
                mn = (s[j + 4] >> 4) | ((s[j] >> 6) << 4);
            }
            const float sd = d * (float)sc, sm = dmin * (float)mn;
            const uint8_t* q = blk + 16 + 16 * j;
            float* o = dst + b * 256 + 32 * j;
            for (int i = 0; i < 16; ++i) {
                o[i] = sd * (float)(q[i] & 15) - sm;
                o[i + 16] = sd * (float)(q[i] >> 4) - sm;
            }
        }
    }
}
