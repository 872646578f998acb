/* prefill.c -- CPU restatement of the batched-prefill arithmetic of the GPU
 * build (test infrastructure only: tests, smoke() and the bench's CPU arm
 * use it as the checker).
 *
 * The reference's batched path (ds4f_moe_step_batch, src/moe.c:1480-1707)
 * multiplies fp32 activations by the dequantised weights. The GPU feeds the
 * FP8 tensor cores instead, so its activations pass through a quantiser
 * that has no reference counterpart; it is restated here bit for bit (the
 * same fp32 operations, correctly rounded, and the same round-to-nearest-
 * even E4M3 encoding) so the GPU's digits can be compared byte for byte,
 * and the GEMM it feeds is restated in double precision as the tolerance
 * reference.
 */
#include "prefill.h"

#include <math.h>
#include <stdlib.h>
#include <string.h>

#include "ds4f_oracle.h"
#include "fixture.h"

/* Per (row, 128-column block): a = max |x|, r = 240 / a, s = a / 240
 * (a = 0: r = 0, s = 1), y = x r; d0 = E4M3(y), y = (y - d0) 16, d1 = ...
 * Every digit lies in [-240, 240], where fx_f8_encode (nearest, ties to
 * even) is the standard E4M3 encoding and orc_f8_value its exact value. */
int orc_quant_f8_digits(const float *x, int N, int C, int ND, uint8_t *q, float *s) {
    if (N <= 0 || C <= 0 || C % 128 || ND < 1 || ND > 3) return -1;
    for (int n = 0; n < N; n++)
        for (int b = 0; b < C / 128; b++) {
            const float *xb = x + (int64_t)n * C + b * 128;
            float a = 0.0f;
            for (int i = 0; i < 128; i++) a = fmaxf(a, fabsf(xb[i]));
            const float r = a > 0.0f ? 240.0f / a : 0.0f;
            s[(int64_t)n * (C / 128) + b] = a > 0.0f ? a / 240.0f : 1.0f;
            for (int i = 0; i < 128; i++) {
                float y = xb[i] * r;
                for (int d = 0; d < ND; d++) {
                    uint8_t byte = fx_f8_encode(y);
                    if (byte == 0 && signbit(y)) byte = 0x80;      /* E4M3(-0) = -0 */
                    q[((int64_t)d * N + n) * C + b * 128 + i] = byte;
                    y = (y - orc_f8_value(byte)) * 16.0f;
                }
            }
        }
    return 0;
}

/* Y[n][r] = sum_kb sW[r/128][kb] sX[n][kb] sum_{c in kb} W[r][c] x~[n][c],
 * x~ = sum_d X[d][n][c] 16^-d, evaluated in double. */
int orc_f8_gemm_digits(const uint8_t *W, const float *sW, const uint8_t *X, const float *sX, double *Y,
                       int R, int C, int N, int ND) {
    if (R % 128 || C % 128 || ND < 1 || ND > 3) return -1;
    const int KB = C / 128;
    double *xv = (double *)malloc((size_t)C * sizeof(double));
    if (!xv) return -1;
    for (int n = 0; n < N; n++) {
        for (int c = 0; c < C; c++) {
            double v = 0.0, f = 1.0;
            for (int d = 0; d < ND; d++, f /= 16.0) v += f * orc_f8_value(X[((int64_t)d * N + n) * C + c]);
            xv[c] = v;
        }
        for (int r = 0; r < R; r++) {
            double acc = 0.0;
            for (int kb = 0; kb < KB; kb++) {
                double part = 0.0;
                for (int c = kb * 128; c < kb * 128 + 128; c++)
                    part += (double)orc_f8_value(W[(int64_t)r * C + c]) * xv[c];
                acc += part * (double)sW[(r / 128) * KB + kb] * (double)sX[(int64_t)n * KB + kb];
            }
            Y[(int64_t)n * R + r] = acc;
        }
    }
    free(xv);
    return 0;
}
