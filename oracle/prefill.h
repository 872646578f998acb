/* prefill.h -- CPU restatement of the GPU batched prefill's arithmetic
 * (test infrastructure only). See prefill.c. */
#ifndef DS4F_ORACLE_PREFILL_H
#define DS4F_ORACLE_PREFILL_H

#include <stdint.h>

#ifdef __cplusplus
extern "C" {
#endif

/* The activation quantiser of ds4f_gpu_quant_f8_digits, bit for bit:
 * x [N][C] fp32 -> q [ND][N][C] E4M3 digit planes, s [N][C/128]. */
int orc_quant_f8_digits(const float *x, int N, int C, int ND, uint8_t *q, float *s);

/* The block-scaled digit GEMM of ds4f_gpu_f8_gemm, in double:
 * Y [N][R] = per 128-column block kb, sW[r/128][kb] sX[n][kb] times the
 * block's sum of W[r][c] (d0 + d1/16 + d2/256)[n][c]. */
int orc_f8_gemm_digits(const uint8_t *W, const float *sW, const uint8_t *X, const float *sX, double *Y,
                       int R, int C, int N, int ND);

/* One layer of the GPU batched prefill (prefill.cu / ds4f_gpu_moe_prefill),
 * restated (FP8 pools, or MXFP4 pools through their exact FP8 copy): the
 * same quantisation points (3 E4M3 digits per routed
 * activation and chain element, bf16 hi/lo digits in the shared expert),
 * block sums in double, promotion, combine and residual in the GPU's fp32
 * order. states [T][H] in/out; sel / w [T][K] (sel < 0: skipped). */
struct OrcLayerW;
struct OrcExpertLayout;
int orc_prefill_layer(int fmt, int H, int M, int K, const struct OrcLayerW *lw,
                      const struct OrcExpertLayout *lay, int T, float *states, const int *sel, const float *w);


#ifdef __cplusplus
}
#endif

#endif
