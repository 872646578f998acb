/*
 * Build shim for compiling the reference's own kernel sources in place.
 *
 * TEST INFRASTRUCTURE ONLY: used by oracle/Makefile to build oracle/_ref
 * (the reference's scalar/AVX2 CPU kernels) as a checker and CPU baseline.
 *
 * The reference includes "ds4f/simd.h" from src/kernels.c:3 and
 * src/simd.c, but does not ship the header (its include/ds4f/ holds only
 * attn.h ds4f.h gpu.h kernels.h moe.h tokenizer.h). This file supplies the
 * six ds4f_simd_* prototypes those sources call, with the signatures they
 * are defined with in src/simd.c (:81, :92, :114, :139, :222, :266, :397),
 * plus the group-size constant that src/simd.c uses in its AVX2 branch
 * (:654) but defines only in its aarch64 branch (:137).
 */
#ifndef DS4F_REF_SIMD_SHIM_H
#define DS4F_REF_SIMD_SHIM_H

#include <stdint.h>

#ifndef DS4F_MLX4_GROUP_LOCAL
#define DS4F_MLX4_GROUP_LOCAL 64
#endif

int  ds4f_simd_available(void);
void ds4f_simd_mxfp4_decode(const uint8_t *vals, const uint8_t *scales,
                            int n, int bsize, float *out);
void ds4f_simd_mxfp4_matvec(const uint8_t *vals, const uint8_t *scales,
                            int R, int C, int bsize, const float *x,
                            float *y, float *scratch);
void ds4f_simd_bf16_matvec(const uint16_t *W, int R, int C,
                           const float *x, const float *bias, float *y);
void ds4f_simd_mlx4_matvec(const uint32_t *vals, const uint16_t *scales,
                           const uint16_t *biases, int R, int C,
                           const float *x, float *y, int r0, int r1);
void ds4f_simd_i8_matvec(const uint8_t *W, const uint8_t *scales,
                         int R, int C, int SR, int SC, const float *x,
                         float *y);
void ds4f_simd_f8_matvec(const uint8_t *W, const uint8_t *scales,
                         int R, int C, int SR, int SC, const float *x,
                         float *y, int r0, int r1);

#endif
