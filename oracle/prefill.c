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

/* ---- one layer of the GPU batched prefill (prefill.cu), restated ------ */

/* sum over one K block of W[c] (E4M3 bytes) times the digit planes' values
 * of one activation row, per digit, each rounded to float from double --
 * the tensor core's exact-product fp32 sums up to their summation order. */
static void f8_block_digits(const uint8_t *w, const uint8_t *const *xd, int ND, int c0, float *D) {
    for (int d = 0; d < ND; d++) {
        double s = 0.0;
        for (int c = c0; c < c0 + 128; c++) s += (double)orc_f8_value(w[c]) * (double)orc_f8_value(xd[d][c]);
        D[d] = (float)s;
    }
}

/* The GPU's promotion: v = (D0 + D1/16) + D2/256 in fp32, then
 * acc = fma(v, sW * sX, acc) per 128-column block, blocks in order. */
static float f8_row_dot(const uint8_t *w, const float *sw_row, const uint8_t *const *xd, const float *sx,
                        int C, int ND) {
    float acc = 0.0f;
    for (int kb = 0; kb < C / 128; kb++) {
        float D[3];
        f8_block_digits(w, xd, ND, kb * 128, D);
        float v = D[0];
        if (ND > 1) v = v + D[1] * 0.0625f;
        if (ND > 2) v = v + D[2] * 0.00390625f;
        acc = fmaf(v, sw_row[kb] * sx[kb], acc);
    }
    return acc;
}

/* The same for an MXFP4 row (E2M1 nibbles, E8M0 scale per 32): the weights
 * exactly dequantised (wrow, C floats, from orc_mxfp4_decode), each 128-column
 * block's sum with each digit plane in double rounded to float (the
 * block-scaled MMA applies the weights' scales to exact products), the
 * digits combined as above and acc = fma(v, sX, acc): the weight scale is
 * already inside the sums. */
static float mx_row_dot(const float *wrow, const uint8_t *const *xd, const float *sx, int C, int ND) {
    float acc = 0.0f;
    for (int kb = 0; kb < C / 128; kb++) {
        float D[3];
        for (int d = 0; d < ND; d++) {
            double sum = 0.0;
            for (int c = kb * 128; c < kb * 128 + 128; c++) sum += (double)wrow[c] * (double)orc_f8_value(xd[d][c]);
            D[d] = (float)sum;
        }
        float v = D[0];
        if (ND > 1) v = v + D[1] * 0.0625f;
        if (ND > 2) v = v + D[2] * 0.00390625f;
        acc = fmaf(v, 1.0f * sx[kb], acc);
    }
    return acc;
}

/* bf16 hi/lo digits of x */
static void bf16_digits(float x, float *hi, float *lo) {
    *hi = orc_bf16_to_f32(fx_bf16_rne(x));
    *lo = orc_bf16_to_f32(fx_bf16_rne(x - *hi));
}

/* The shared expert's bf16 GEMM row: per 64-column block, D_d = sum of
 * w x digit_d in double, rounded to float; acc += D0 + D1 in fp32. */
static float bf16_row_dot(const uint16_t *w, const float *hi, const float *lo, int C) {
    float acc = 0.0f;
    for (int kb = 0; kb < C / 64; kb++) {
        double s0 = 0.0, s1 = 0.0;
        for (int c = kb * 64; c < kb * 64 + 64; c++) {
            const double wv = (double)orc_bf16_to_f32(w[c]);
            s0 += wv * (double)hi[c];
            s1 += wv * (double)lo[c];
        }
        acc = acc + ((float)s0 + (float)s1);
    }
    return acc;
}


int orc_prefill_layer(int fmt, int H, int M, int K, const OrcLayerW *lw, const OrcExpertLayout *lay, int T,
                      float *states, const int *sel, const float *w) {
    const int ND = 3;
    int rc = -1;
    float *xin = (float *)malloc((size_t)T * H * sizeof(float));
    uint8_t *xq = (uint8_t *)malloc((size_t)ND * T * H);
    float *sx = (float *)malloc((size_t)T * (H / 128) * sizeof(float));
    float *gu = (float *)malloc((size_t)2 * M * sizeof(float));
    float *ch = (float *)malloc((size_t)M * sizeof(float));
    uint8_t *cq = (uint8_t *)malloc((size_t)ND * M);
    float *sc = (float *)malloc((size_t)(M / 128) * sizeof(float));
    float *out = (float *)malloc((size_t)K * H * sizeof(float));
    float *hi = (float *)malloc((size_t)H * sizeof(float)), *lo = (float *)malloc((size_t)H * sizeof(float));
    float *so = (float *)malloc((size_t)H * sizeof(float));
    /* MXFP4: one dequantised row (the widest, H or M columns) */
    float *wrow = (float *)malloc((size_t)(H > M ? H : M) * sizeof(float));
    if (!xin || !xq || !sx || !gu || !ch || !cq || !sc || !out || !hi || !lo || !so || !wrow) goto done;
    memcpy(xin, states, (size_t)T * H * sizeof(float));
    for (int t = 0; t < T; t++) orc_rmsnorm(lw->norm, H, xin + (int64_t)t * H);
    if (orc_quant_f8_digits(xin, T, H, ND, xq, sx)) goto done;
    for (int t = 0; t < T; t++) {
        const uint8_t *xd[3];
        for (int d = 0; d < ND; d++) xd[d] = xq + ((int64_t)d * T + t) * H;
        const float *sxt = sx + (int64_t)t * (H / 128);
        /* routed selections, each one chain */
        for (int j = 0; j < K; j++) {
            const int e = sel[(int64_t)t * K + j];
            if (e < 0) continue;
            const uint8_t *slot = lw->experts + (int64_t)e * lay->nbytes;
            if (fmt == ORC_FMT_MXFP4) {
                /* gate, up: rows of H nibbles (H / 2 bytes, H / 32 scales) */
                for (int mat = 0; mat < 2; mat++)
                    for (int m = 0; m < M; m++) {
                        orc_mxfp4_decode(slot + lay->rel_v[mat] + (int64_t)m * (H / 2),
                                         slot + lay->rel_s[mat] + (int64_t)m * (H / 32), H, 32, wrow);
                        gu[mat * M + m] = mx_row_dot(wrow, xd, sxt, H, ND);
                    }
            } else {
                for (int mat = 0; mat < 2; mat++)
                    for (int m = 0; m < M; m++)
                        gu[mat * M + m] = f8_row_dot(slot + lay->rel_v[mat] + (int64_t)m * H,
                                                     (const float *)(slot + lay->rel_s[mat]) + (m / 128) * (H / 128),
                                                     xd, sxt, H, ND);
            }
            for (int m = 0; m < M; m++) ch[m] = orc_silu_mul(gu[m], gu[M + m]);
            if (orc_quant_f8_digits(ch, 1, M, ND, cq, sc)) goto done;
            const uint8_t *cd[3] = {cq, cq + M, cq + 2 * M};
            for (int r = 0; r < H; r++) {
                if (fmt == ORC_FMT_MXFP4) {
                    orc_mxfp4_decode(slot + lay->rel_v[2] + (int64_t)r * (M / 2),
                                     slot + lay->rel_s[2] + (int64_t)r * (M / 32), M, 32, wrow);
                    out[(int64_t)j * H + r] = mx_row_dot(wrow, cd, sc, M, ND);
                } else {
                    out[(int64_t)j * H + r] = f8_row_dot(slot + lay->rel_v[2] + (int64_t)r * M,
                                                         (const float *)(slot + lay->rel_s[2]) + (r / 128) * (M / 128),
                                                         cd, sc, M, ND);
                }
            }
        }
        /* shared expert (bf16 hi/lo digits) and its gate */
        const float *x = xin + (int64_t)t * H;
        for (int c = 0; c < H; c++) bf16_digits(x[c], hi + c, lo + c);
        for (int m = 0; m < M; m++) {
            gu[m] = bf16_row_dot(lw->sh_gate + (int64_t)m * H, hi, lo, H);
            gu[M + m] = bf16_row_dot(lw->sh_up + (int64_t)m * H, hi, lo, H);
        }
        for (int m = 0; m < M; m++) bf16_digits(orc_silu_mul(gu[m], gu[M + m]), hi + m, lo + m);
        for (int r = 0; r < H; r++) so[r] = bf16_row_dot(lw->sh_down + (int64_t)r * M, hi, lo, M);
        double g = 0.0;
        for (int c = 0; c < H; c++) g += (double)orc_bf16_to_f32(lw->sh_gw[c]) * (double)x[c];
        const float sig = 1.0f / (1.0f + expf(-(float)g));
        /* combine in selection order, then the shared expert, then the residual */
        float *st = states + (int64_t)t * H;
        for (int r = 0; r < H; r++) {
            float acc = 0.0f;
            for (int j = 0; j < K; j++) {
                const float wj = w[(int64_t)t * K + j];
                if (sel[(int64_t)t * K + j] < 0 || wj == 0.0f) continue;
                acc = acc + wj * out[(int64_t)j * H + r];
            }
            acc = acc + sig * so[r];
            st[r] = st[r] + acc;
        }
    }
    rc = 0;
done:
    free(xin); free(xq); free(sx); free(gu); free(ch); free(cq); free(sc); free(out);
    free(hi); free(lo); free(so); free(wrow);
    return rc;
}
