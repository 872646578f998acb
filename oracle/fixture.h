/*
 * fixture.h -- seeded synthetic inputs for the routed-expert path (CPU).
 *
 * TEST INFRASTRUCTURE ONLY. The product library carries a device copy of
 * the same generator (ds4f_gpu_synth_*); tests check the two agree byte
 * for byte. To make that possible every step uses only IEEE operations
 * that are correctly rounded on both CPU and GPU (+ - * / sqrt, integer
 * ops), evaluated in a fixed order with no FMA contraction:
 *
 *   key      = mix(mix(seed) ^ tid)                  per tensor
 *   element i: base = mix(key + i); draw pairs z = mix(base + k*G),
 *              v = (z >> 11) * 2^-52 - 1 in [-1, 1)
 *              Marsaglia polar: accept s = v1^2 + v2^2 in (0, 1)
 *              g = v1 * sqrt(-2 ln(s) / s)            (N(0,1))
 *   ln(s)    = e ln2 + 2 atanh-series of (m-1)/(m+1), m in [1/sqrt2, sqrt2)
 *   value    = (float)(g * sigma)
 * where mix(x) is the splitmix64 step (x + G, then the finaliser) and
 * G = 0x9E3779B97F4A7C15.
 *
 * Quantisers:
 *   bf16   round-to-nearest-even of the fp32 bits.
 *   FP8    per 128x128 block s = amax / 448 (fp32); byte = the nearest
 *          value of the reference decode table (src/kernels.c:228-241)
 *          among canonical bytes (e <= 14, or 0x7E = 448), ties to the
 *          even byte. Canonical bytes decode identically under the
 *          reference table and under IEEE-style E4M3FN hardware decode.
 *   MXFP4  per 32 elements along K: k = ceil(log2(amax / 6)), clamped to
 *          [-127, 127], scale byte k + 127, nibble = nearest E2M1
 *          magnitude of x / 2^k (ties to the smaller), sign bit 3, even
 *          index in the low nibble -- the encoder of the reference's gate
 *          test (tests/test_kernels.c:19-54) and converter
 *          (tools/convert-ds4f.py:1024-1044, :1081-1110). ceil(log2) is
 *          computed exactly from the float's bits.
 */
#ifndef DS4F_FIXTURE_H
#define DS4F_FIXTURE_H

#include <stdint.h>

#ifdef __cplusplus
extern "C" {
#endif

#define FX_KIND_ROUTER  1u
#define FX_KIND_SHARED  2u      /* t: 0 gate, 1 up, 2 down, 3 gate weight */
#define FX_KIND_EXPERT  3u      /* x = expert, t: 0 gate, 1 up, 2 down    */
#define FX_KIND_ACT     4u      /* x = token / step                        */

uint64_t fx_mix64(uint64_t x);
uint64_t fx_tid(uint32_t layer, uint32_t kind, uint32_t x, uint32_t t);
uint64_t fx_key(uint64_t seed, uint64_t tid);
double   fx_ln(double s);
double   fx_gauss(uint64_t key, uint64_t i);
float    fx_value(uint64_t key, uint64_t i, double sigma);
uint16_t fx_bf16_rne(float f);
uint8_t  fx_f8_encode(float v);
int      fx_ceil_log2(float y);
int      fx_e2m1_encode(float q);

void fx_fill_f32(float *dst, int64_t n, uint64_t key, double sigma);
void fx_fill_bf16(uint16_t *dst, int64_t n, uint64_t key, double sigma);
/* [R x C] matrix, element (r, c) = fx_value(key, r*C + c, sigma). */
int  fx_quant_fp8(int R, int C, uint64_t key, double sigma, uint8_t *vals,
                  float *scales /* [R/128][C/128] */);
int  fx_quant_mxfp4(int R, int C, uint64_t key, double sigma, uint8_t *vals,
                    uint8_t *scales /* [R*C/32] */);

/* One expert slot (layout of orc_expert_layout), sigma 0.02 by default. */
int  fx_expert(int fmt, int H, int M, uint64_t seed, uint32_t layer,
               uint32_t expert, double sigma, uint8_t *slot);
/* Layer trunk: norm = 1.0, router/shared ~ N(0, sigma) in bf16. */
void fx_trunk(int H, int M, int E, uint64_t seed, uint32_t layer,
              double sigma, uint16_t *norm, uint16_t *router,
              uint16_t *sh_gate, uint16_t *sh_up, uint16_t *sh_down,
              uint16_t *sh_gw);

#ifdef __cplusplus
}
#endif

#endif
