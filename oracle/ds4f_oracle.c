/*
 * ds4f_oracle.c -- CPU restatement of the reference's routed-expert path.
 *
 * TEST INFRASTRUCTURE ONLY (the parity checker; see ds4f_oracle.h).
 * Written from the reference's behaviour, function by function, citing
 * the file:line each one follows. Scalar, single-threaded, -std=c99
 * -ffp-contract=off so the evaluation order is the reference's.
 */
#include "ds4f_oracle.h"

#include <math.h>
#include <stdlib.h>
#include <string.h>

/* ---- element decode ------------------------------------------------ */

/* 2^(b-127) via ldexpf; b = 0 gives the subnormal 2^-127 and b = 255
 * gives +inf (src/kernels.c:24-26). */
float orc_e8m0_value(uint8_t b) { return ldexpf(1.0f, (int)b - 127); }

/* E4M3 byte -> fp32 with the reference's table rule
 * (src/kernels.c:228-241): e = 0 -> m * 2^-9; e = 15 -> 448 for every
 * mantissa (not IEEE-style NaN/extended range); else (1 + m/8) 2^(e-7);
 * bit 7 is the sign. */
static float f8_rule(int b) {
    int s = (b >> 7) & 1, e = (b >> 3) & 0xF, m = b & 7;
    float v;
    if (e == 0)
        v = (float)m * 0.001953125f;
    else if (e == 0xF)
        v = 448.0f;
    else
        v = (1.0f + (float)m / 8.0f) * ldexpf(1.0f, e - 7);
    return s ? -v : v;
}

static float g_f8_lut[256];
static int g_f8_ready = 0;

static void f8_lut_init(void) {
    if (g_f8_ready) return;
    for (int b = 0; b < 256; b++) g_f8_lut[b] = f8_rule(b);
    g_f8_ready = 1;            /* idempotent: identical values either way */
}

float orc_f8_value(uint8_t b) {          /* src/kernels.c:308-311 */
    f8_lut_init();
    return g_f8_lut[b];
}

float orc_bf16_to_f32(uint16_t h) {      /* src/kernels.c:84-89 */
    uint32_t bits = (uint32_t)h << 16;
    float f;
    memcpy(&f, &bits, sizeof f);
    return f;
}

/* E2M1 magnitudes, index = nibble & 7 (src/kernels.c:28-32). */
static const float k_e2m1[8] = {0.0f, 0.5f, 1.0f, 1.5f,
                                2.0f, 3.0f, 4.0f, 6.0f};

/* Flat decode: nibble i is byte i>>1, low nibble for even i; bit 3 is the
 * sign; times the E8M0 scale of block i / bsize (src/kernels.c:34-46). */
void orc_mxfp4_decode(const uint8_t *vals, const uint8_t *scales, int64_t n,
                      int bsize, float *out) {
    for (int64_t i = 0; i < n; i++) {
        int nib = (vals[i >> 1] >> ((i & 1) ? 4 : 0)) & 0xF;
        float v = k_e2m1[nib & 7];
        if (nib & 8) v = -v;
        out[i] = v * orc_e8m0_value(scales[i / bsize]);
    }
}

static float block_scale(int kind, const void *scales, int idx) {
    if (!scales) return 1.0f;
    if (kind == ORC_SCALE_F32) return ((const float *)scales)[idx];
    return orc_e8m0_value(((const uint8_t *)scales)[idx]);
}

/* src/kernels.c:294-306, generalised to a row range: element (r, c) uses
 * scale[r*SR/R][c*SC/C] (integer division in int64). */
void orc_f8_decode_rows(const uint8_t *W, int scale_kind, const void *scales,
                        int R, int C, int SR, int SC, int r0, int r1,
                        float *out) {
    f8_lut_init();
    if (SR < 1) SR = 1;
    if (SC < 1) SC = 1;
    for (int r = r0; r < r1; r++) {
        const uint8_t *wr = W + (int64_t)r * C;
        int sr = (int)(((int64_t)r * SR) / R);
        float *o = out + (int64_t)(r - r0) * C;
        for (int c = 0; c < C; c++) {
            int sc = (int)(((int64_t)c * SC) / C);
            float s = block_scale(scale_kind, scales, sr * SC + sc);
            o[c] = g_f8_lut[wr[c]] * s;
        }
    }
}

/* ---- matvec -------------------------------------------------------- */

/* Scalar branch of ds4f_f8_matvec (src/kernels.c:255-269): per row an
 * fp32 accumulator, columns ascending, acc += (lut[W] * s) * x. */
void orc_f8_matvec(const uint8_t *W, int scale_kind, const void *scales,
                   int R, int C, int SR, int SC, const float *x, float *y) {
    f8_lut_init();
    if (SR < 1) SR = 1;
    if (SC < 1) SC = 1;
    for (int r = 0; r < R; r++) {
        float acc = 0.0f;
        int sr = (int)(((int64_t)r * SR) / R);
        const uint8_t *wr = W + (int64_t)r * C;
        for (int c = 0; c < C; c++) {
            int sc = (int)(((int64_t)c * SC) / C);
            float s = block_scale(scale_kind, scales, sr * SC + sc);
            acc += g_f8_lut[wr[c]] * s * x[c];
        }
        y[r] = acc;
    }
}

/* Scalar ds4f_mxfp4_matvec (src/kernels.c:48-62): decode the whole matrix
 * into scratch, then a row-by-row fp32 dot, columns ascending. */
void orc_mxfp4_matvec(const uint8_t *vals, const uint8_t *scales, int R,
                      int C, int bsize, const float *x, float *y,
                      float *scratch) {
    orc_mxfp4_decode(vals, scales, (int64_t)R * C, bsize, scratch);
    for (int r = 0; r < R; r++) {
        float acc = 0.0f;
        const float *wr = scratch + (int64_t)r * C;
        for (int c = 0; c < C; c++) acc += wr[c] * x[c];
        y[r] = acc;
    }
}

/* Scalar fallback of ds4f_mlx4_matvec (src/kernels.c:201-221). Element
 * k = r*C + c is nibble k%8 of word k/8; group g = k/64 rebuilds the table
 * lut[q] = (float)q * s + b when g changes. */
void orc_mlx4_matvec(const uint32_t *vals, const uint16_t *scales,
                     const uint16_t *biases, int R, int C, const float *x,
                     float *y) {
    float lut[16];
    long gcur = -1;
    for (int r = 0; r < R; r++) {
        float acc = 0.0f;
        for (int c = 0; c < C; c++) {
            long k = (long)r * C + c;
            long g = k / 64;
            if (g != gcur) {
                gcur = g;
                float s = orc_bf16_to_f32(scales[g]);
                float b = biases ? orc_bf16_to_f32(biases[g]) : 0.0f;
                for (int q = 0; q < 16; q++) lut[q] = (float)q * s + b;
            }
            int q = (int)((vals[k >> 3] >> (4 * (int)(k & 7))) & 0xFu);
            acc += lut[q] * x[c];
        }
        y[r] = acc;
    }
}

/* Scalar ds4f_bf16_matvec (src/kernels.c:97-102). */
void orc_bf16_matvec(const uint16_t *W, int R, int C, const float *x,
                     const float *bias, float *y) {
    for (int r = 0; r < R; r++) {
        float acc = 0.0f;
        const uint16_t *wr = W + (int64_t)r * C;
        for (int c = 0; c < C; c++) acc += orc_bf16_to_f32(wr[c]) * x[c];
        y[r] = acc + (bias ? bias[r] : 0.0f);
    }
}

/* ---- MoE pieces ---------------------------------------------------- */

/* rmsnorm_moe (src/moe.c:841-851): ss in double, r = sqrtf(float(ss/dim)
 * + 1e-6f), x = x / r * w. */
void orc_rmsnorm(const uint16_t *w, int dim, float *x) {
    double ss = 0.0;
    for (int i = 0; i < dim; i++) ss += (double)x[i] * x[i];
    float r = sqrtf((float)(ss / (double)dim) + 1e-6f);
    for (int i = 0; i < dim; i++) x[i] = x[i] / r * orc_bf16_to_f32(w[i]);
}

/* ds4f_topk (src/moe.c:531-561). Insertion into a descending list: a new
 * score moves above entry j only when strictly greater, so an equal score
 * that arrives later (higher index) stays below. Then softmax over all E
 * scores in double with the max subtracted; the selected probabilities
 * are kept raw. */
void orc_topk(const float *scores, int E, int k, int *idx, float *w) {
    if (k > E) k = E;
    for (int j = 0; j < k; j++) { idx[j] = -1; w[j] = 0.0f; }
    for (int e = 0; e < E; e++) {
        float s = scores[e];
        int j = k - 1;
        while (j >= 0 && (idx[j] < 0 || s > w[j])) j--;
        if (j < k - 1) {
            for (int q = k - 2; q > j; q--) {
                idx[q + 1] = idx[q];
                w[q + 1] = w[q];
            }
            idx[j + 1] = e;
            w[j + 1] = s;
        }
    }
    double mx = -1e30, sw = 0.0;
    for (int e = 0; e < E; e++)
        if ((double)scores[e] > mx) mx = (double)scores[e];
    for (int e = 0; e < E; e++) sw += exp((double)scores[e] - mx);
    for (int j = 0; j < k && idx[j] >= 0; j++)
        w[j] = (float)(exp((double)w[j] - mx) / sw);
}

void orc_topk_renorm(int k, float *w) {
    float s = 0.0f;
    for (int j = 0; j < k; j++) s += w[j];
    if (s > 0.0f)
        for (int j = 0; j < k; j++) w[j] = w[j] / s;
}

/* src/moe.c:645-649 */
float orc_silu_mul(float g, float u) {
    float sig = 1.0f / (1.0f + expf(-g));
    return g * sig * u;
}

/* ---- expert pool --------------------------------------------------- */

int orc_expert_layout(int fmt, int H, int M, OrcExpertLayout *lay) {
    int64_t vb[3], sb[3];
    int64_t mh = (int64_t)M * H;
    if (H <= 0 || M <= 0) return -1;
    if (fmt == ORC_FMT_FP8) {
        if (H % 128 || M % 128) return -1;
        int64_t nsc = (int64_t)(M / 128) * (H / 128);
        for (int t = 0; t < 3; t++) { vb[t] = mh; sb[t] = nsc * 4; }
    } else if (fmt == ORC_FMT_MXFP4) {
        if (H % 32 || M % 32) return -1;
        for (int t = 0; t < 3; t++) { vb[t] = mh / 2; sb[t] = mh / 32; }
    } else {
        return -1;
    }
    int64_t off = 0;
    for (int t = 0; t < 3; t++) {
        lay->rel_v[t] = off; off += vb[t];
        lay->rel_s[t] = off; off += sb[t];
    }
    lay->nbytes = off;
    return 0;
}

static void fmt_matvec(int fmt, const uint8_t *slot, const OrcExpertLayout *lay,
                       int t, int R, int C, const float *x, float *y,
                       float *scratch) {
    const uint8_t *v = slot + lay->rel_v[t];
    const uint8_t *s = slot + lay->rel_s[t];
    if (fmt == ORC_FMT_FP8)
        orc_f8_matvec(v, ORC_SCALE_F32, s, R, C, R / 128, C / 128, x, y);
    else
        orc_mxfp4_matvec(v, s, R, C, 32, x, y, scratch);
}

/* exp_run, Qwen3 branch (src/moe.c:598-753): gate and up read the same
 * input, silu(gate)*up is the chain, down maps it back to H. */
int orc_expert_chain(int fmt, const uint8_t *slot, const OrcExpertLayout *lay,
                     int H, int M, const float *x, float *out) {
    float *gx = (float *)malloc((size_t)M * sizeof(float));
    float *ux = (float *)malloc((size_t)M * sizeof(float));
    float *scratch = NULL;
    if (fmt == ORC_FMT_MXFP4)
        scratch = (float *)malloc((size_t)M * H * sizeof(float));
    if (!gx || !ux || (fmt == ORC_FMT_MXFP4 && !scratch)) {
        free(gx); free(ux); free(scratch);
        return -1;
    }
    fmt_matvec(fmt, slot, lay, 0, M, H, x, gx, scratch);
    fmt_matvec(fmt, slot, lay, 1, M, H, x, ux, scratch);
    for (int i = 0; i < M; i++) gx[i] = orc_silu_mul(gx[i], ux[i]);
    fmt_matvec(fmt, slot, lay, 2, H, M, gx, out, scratch);
    free(gx); free(ux); free(scratch);
    return 0;
}

/* Shared expert (src/moe.c:1235-1293) with the bf16 matvec in place of
 * the reference's MLX4 one: acc += sigmoid(gw . xin) * down(silu(gate
 * xin) * up xin). */
int orc_shared_add(const OrcLayerW *lw, int H, int M, const float *xin,
                   float *acc) {
    float *sg = (float *)malloc((size_t)(3 * M + H) * sizeof(float));
    if (!sg) return -1;
    float *upv = sg + M, *chain = sg + 2 * M, *sout = sg + 3 * M;
    float sgate[1];
    orc_bf16_matvec(lw->sh_gate, M, H, xin, NULL, sg);
    orc_bf16_matvec(lw->sh_up, M, H, xin, NULL, upv);
    for (int i = 0; i < M; i++) chain[i] = orc_silu_mul(sg[i], upv[i]);
    orc_bf16_matvec(lw->sh_down, H, M, chain, NULL, sout);
    orc_bf16_matvec(lw->sh_gw, 1, H, xin, NULL, sgate);
    float sg2 = 1.0f / (1.0f + expf(-sgate[0]));
    for (int i = 0; i < H; i++) acc[i] += sg2 * sout[i];
    free(sg);
    return 0;
}

/* Router for one token: RMSNorm of the state (src/main.c:1014-1033), bf16
 * gate matvec with no bias (:1080-1083), ds4f_topk (:1088), then the
 * BASELINE renormalisation. xin receives the normed input. */
static void route(int H, int E, int K, int renorm, const OrcLayerW *lw,
                  const float *state, float *xin, float *scores, int *idx,
                  float *w) {
    memcpy(xin, state, (size_t)H * sizeof(float));
    orc_rmsnorm(lw->norm, H, xin);
    orc_bf16_matvec(lw->router, E, H, xin, NULL, scores);
    orc_topk(scores, E, K, idx, w);
    if (renorm) orc_topk_renorm(K, w);
}

int orc_moe_layer(int fmt, int H, int M, int E, int K, int renorm,
                  const OrcLayerW *lw, const OrcExpertLayout *lay,
                  float *state, int *idx, float *w, float *scores,
                  float *acc_out) {
    int rc = -1;
    float *xin = (float *)malloc((size_t)H * sizeof(float));
    float *acc = (float *)calloc((size_t)H, sizeof(float));
    float *out = (float *)malloc((size_t)H * sizeof(float));
    float *sc = (float *)malloc((size_t)E * sizeof(float));
    if (!xin || !acc || !out || !sc || K > E) goto done;
    route(H, E, K, renorm, lw, state, xin, sc, idx, w);
    if (scores) memcpy(scores, sc, (size_t)E * sizeof(float));
    /* src/moe.c:1162-1227: chains per selection, combined in j order */
    for (int j = 0; j < K; j++) {
        const uint8_t *slot = lw->experts + (int64_t)idx[j] * lay->nbytes;
        if (orc_expert_chain(fmt, slot, lay, H, M, xin, out) != 0) goto done;
        for (int i = 0; i < H; i++) acc[i] += w[j] * out[i];
    }
    if (orc_shared_add(lw, H, M, xin, acc) != 0) goto done;
    if (acc_out) memcpy(acc_out, acc, (size_t)H * sizeof(float));
    for (int i = 0; i < H; i++) state[i] += acc[i];    /* src/moe.c:1424 */
    rc = 0;
done:
    free(xin); free(acc); free(out); free(sc);
    return rc;
}

typedef struct { int eid, b, j; } OrcSel;

static int sel_cmp(const void *a, const void *b) {
    const OrcSel *x = (const OrcSel *)a, *y = (const OrcSel *)b;
    if (x->eid != y->eid) return x->eid - y->eid;
    if (x->b != y->b) return x->b - y->b;   /* deterministic within group */
    return x->j - y->j;
}

/* ds4f_moe_step_batch (src/moe.c:1480-1707) over B tokens: (token,
 * selection) pairs sorted by expert (:1516-1529), each distinct expert
 * run over its group (:1545-1613) with per-selection outputs, combined
 * per token in selection order skipping zero weights (:1614-1630), the
 * shared expert per token (:1636-1698), then the residual (:1700-1705).
 * Router per token as orc_moe_layer. */
int orc_moe_batch(int fmt, int H, int M, int E, int K, int renorm,
                  const OrcLayerW *lw, const OrcExpertLayout *lay, int B,
                  float *states, int *idx, float *w) {
    float *xin = (float *)malloc((size_t)H * sizeof(float));
    float *sc = (float *)malloc((size_t)E * sizeof(float));
    if (!xin || !sc || K > E) { free(xin); free(sc); return -1; }
    for (int b = 0; b < B; b++)
        route(H, E, K, renorm, lw, states + (int64_t)b * H, xin, sc,
              idx + (int64_t)b * K, w + (int64_t)b * K);
    free(xin); free(sc);
    return orc_moe_batch_sel(fmt, H, M, K, lw, lay, B, states, idx, w);
}

int orc_moe_batch_sel(int fmt, int H, int M, int K, const OrcLayerW *lw,
                      const OrcExpertLayout *lay, int B, float *states,
                      const int *idx, const float *w) {
    int rc = -1;
    int64_t ns = (int64_t)B * K;
    float *xins = (float *)malloc((size_t)B * H * sizeof(float));
    float *acc = (float *)calloc((size_t)B * H, sizeof(float));
    float *dy = (float *)calloc((size_t)ns * H, sizeof(float));
    OrcSel *sl = (OrcSel *)malloc((size_t)ns * sizeof(OrcSel));
    int64_t *pos = (int64_t *)malloc((size_t)ns * sizeof(int64_t));
    if (!xins || !acc || !dy || !sl || !pos) goto done;
    /* the caller's RMSNorm of each token (src/main.c:1014-1033) */
    memcpy(xins, states, (size_t)B * H * sizeof(float));
    for (int b = 0; b < B; b++) orc_rmsnorm(lw->norm, H, xins + (int64_t)b * H);
    int64_t n = 0;
    for (int b = 0; b < B; b++)
        for (int j = 0; j < K; j++) {
            int eid = idx[(int64_t)b * K + j];
            if (eid < 0) continue;
            sl[n].eid = eid; sl[n].b = b; sl[n].j = j; n++;
        }
    qsort(sl, (size_t)n, sizeof(OrcSel), sel_cmp);
    for (int64_t s = 0; s < n; s++) {
        const uint8_t *slot = lw->experts + (int64_t)sl[s].eid * lay->nbytes;
        if (orc_expert_chain(fmt, slot, lay, H, M,
                             xins + (int64_t)sl[s].b * H,
                             dy + s * H) != 0)
            goto done;
        pos[(int64_t)sl[s].b * K + sl[s].j] = s;
    }
    for (int b = 0; b < B; b++)
        for (int j = 0; j < K; j++) {
            if (idx[(int64_t)b * K + j] < 0) continue;
            float wj = w[(int64_t)b * K + j];
            if (wj == 0.0f) continue;
            const float *d = dy + pos[(int64_t)b * K + j] * H;
            float *a = acc + (int64_t)b * H;
            for (int i = 0; i < H; i++) a[i] += wj * d[i];
        }
    for (int b = 0; b < B; b++)
        if (orc_shared_add(lw, H, M, xins + (int64_t)b * H,
                       acc + (int64_t)b * H) != 0)
            goto done;
    for (int64_t i = 0; i < (int64_t)B * H; i++) states[i] += acc[i];
    rc = 0;
done:
    free(xins); free(acc); free(dy); free(sl); free(pos);
    return rc;
}
