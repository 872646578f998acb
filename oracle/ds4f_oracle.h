/*
 * ds4f_oracle.h -- CPU restatement of the reference's routed-expert path.
 *
 * TEST INFRASTRUCTURE ONLY. This is the parity checker for libds4f_cuda:
 * only tests/, __graft_entry__.smoke() and bench.py's cpu_baseline leg may
 * load it, and never as the thing measured or shipped.
 *
 * Every function restates the reference's *scalar* C path
 * (ds4f_kernels_set_simd(0), src/kernels.c:16) and cites the file:line it
 * follows. Parity is pinned two ways (tests/test_oracle_golden.py):
 *   - the known-answer vectors of the reference's own gate test
 *     (tests/test_kernels.c:57-76, :79-101, :104-137, :258-276, :320-355);
 *   - bit-for-bit agreement with the reference's own kernels.c/moe.c,
 *     compiled from its sources into oracle/_ref by oracle/Makefile, on
 *     seeded random inputs (E8M0-scale FP8, MXFP4, bf16, top-k).
 *
 * Compiled with -std=c99 -O2 -ffp-contract=off: ISO C evaluation, no FMA
 * contraction, like the reference Makefile (Makefile:16).
 */
#ifndef DS4F_ORACLE_H
#define DS4F_ORACLE_H

#include <stdint.h>

#ifdef __cplusplus
extern "C" {
#endif

/* ---- element decode ------------------------------------------------ */
float orc_e8m0_value(uint8_t b);          /* src/kernels.c:24-26        */
float orc_f8_value(uint8_t b);            /* src/kernels.c:228-241,308  */
float orc_bf16_to_f32(uint16_t h);        /* src/kernels.c:84-89        */
void  orc_mxfp4_decode(const uint8_t *vals, const uint8_t *scales,
                       int64_t n, int bsize, float *out);  /* :34-46 */

/* Scale kinds for the FP8 block-scaled format. */
#define ORC_SCALE_E8M0 0   /* reference: one E8M0 byte per block        */
#define ORC_SCALE_F32  1   /* BASELINE:  one fp32 per 128x128 block     */

/* Dequantised rows [r0, r1) of an FP8 E4M3 [R x C] matrix with [SR x SC]
 * block scales; out is (r1-r0) x C fp32.  src/kernels.c:294-306. */
void orc_f8_decode_rows(const uint8_t *W, int scale_kind, const void *scales,
                        int R, int C, int SR, int SC, int r0, int r1,
                        float *out);

/* ---- matvec -------------------------------------------------------- */
/* y[r] = sum_c lut[W]*s*x, c ascending, (lut*s)*x then +=.
 * src/kernels.c:243-270 (scalar branch :255-269). */
void orc_f8_matvec(const uint8_t *W, int scale_kind, const void *scales,
                   int R, int C, int SR, int SC, const float *x, float *y);
/* Two-pass decode-then-dot.  src/kernels.c:48-62. scratch: R*C floats. */
void orc_mxfp4_matvec(const uint8_t *vals, const uint8_t *scales, int R,
                      int C, int bsize, const float *x, float *y,
                      float *scratch);
/* Scalar ds4f_mlx4_matvec (src/kernels.c:201-221): per 64-element group a
 * 16-entry table lut[q] = q*s + b (bf16 scale/bias), acc += lut[q]*x. */
void orc_mlx4_matvec(const uint32_t *vals, const uint16_t *scales,
                     const uint16_t *biases, int R, int C, const float *x,
                     float *y);
/* src/kernels.c:91-103 (scalar branch :97-102). bias may be NULL. */
void orc_bf16_matvec(const uint16_t *W, int R, int C, const float *x,
                     const float *bias, float *y);

/* ---- MoE pieces ---------------------------------------------------- */
/* In-place RMSNorm, bf16 weight, eps 1e-6, double sum of squares.
 * src/moe.c:841-851 (identical to the router's copy, src/main.c:1014-1033). */
void orc_rmsnorm(const uint16_t *w, int dim, float *x);
/* Insertion top-k (strict >, lower index wins ties) + softmax over all E
 * in double, selected probabilities kept raw.  src/moe.c:531-561. */
void orc_topk(const float *scores, int E, int k, int *idx, float *w);
/* norm_topk_prob: w[j] /= sum_j w[j] (fp32, j ascending). Not in the
 * reference (removed there, docs/fidelity-audit.md:40-42); BASELINE asks
 * for it. */
void orc_topk_renorm(int k, float *w);
/* silu(g)*u exactly as src/moe.c:645-649: s*(1/(1+expf(-s)))*u. */
float orc_silu_mul(float g, float u);

/* ---- expert pool --------------------------------------------------- */
/* Expert formats. */
#define ORC_FMT_MXFP4 0    /* e2m1, E8M0 per 32 along K (fmt 0, moe.h:28) */
#define ORC_FMT_FP8   2    /* E4M3, fp32 scale per 128x128 block         */

/* One expert slot: gate [M x H], up [M x H], down [H x M], each stored as
 * values then scales, in manifest order (tools/convert-ds4f.py:1321-1356,
 * src/moe.c:600-605). Offsets relative to the slot start. */
typedef struct OrcExpertLayout {
    int64_t rel_v[3];     /* gate, up, down values   */
    int64_t rel_s[3];     /* gate, up, down scales   */
    int64_t nbytes;       /* fixed-rate slot size    */
} OrcExpertLayout;

/* Fill the canonical slot layout for (fmt, H, M). Returns 0, -1 if the
 * shape does not fit the format (FP8: H, M multiples of 128; MXFP4:
 * multiples of 32). */
int orc_expert_layout(int fmt, int H, int M, OrcExpertLayout *lay);

/* The Qwen3 expert chain for one expert: gx = Wg x, ux = Wu x,
 * c = silu(gx)*ux, out = Wd c.  src/moe.c:598-753 with the format's
 * matvec (FP8: orc_f8_matvec with fp32 scales; MXFP4: orc_mxfp4_matvec). */
int orc_expert_chain(int fmt, const uint8_t *slot, const OrcExpertLayout *lay,
                     int H, int M, const float *x, float *out);

/* Per-layer resident ("trunk") weights, all bf16. */
typedef struct OrcLayerW {
    const uint16_t *norm;       /* [H]    post_attention_layernorm     */
    const uint16_t *router;     /* [E x H]                              */
    const uint16_t *sh_gate;    /* [M x H] shared expert gate_proj     */
    const uint16_t *sh_up;      /* [M x H]                              */
    const uint16_t *sh_down;    /* [H x M]                              */
    const uint16_t *sh_gw;      /* [1 x H] shared_expert_gate          */
    const uint8_t  *experts;    /* [E] slots of lay.nbytes             */
} OrcLayerW;

/* One token through one MoE layer (the Qwen3.5 no-mHC branch of
 * ds4f_moe_step, src/moe.c:948-1456, with the router of
 * src/main.c:1014-1088):
 *   xin = rmsnorm(state); scores = router xin; top-k; renorm (if renorm);
 *   acc = sum_j w[j] chain_j(xin)  (selection order, moe.c:1224-1225);
 *   acc += sigmoid(gw.xin) * shared(xin)  (moe.c:1235-1293, bf16 matvec);
 *   state += acc  (moe.c:1424).
 * Outputs idx[K], w[K] (the weights actually used), optionally the raw
 * router scores[E] and the pre-residual acc[H]. Returns 0 / -1. */
int orc_moe_layer(int fmt, int H, int M, int E, int K, int renorm,
                  const OrcLayerW *lw, const OrcExpertLayout *lay,
                  float *state, int *idx, float *w, float *scores,
                  float *acc_out);

/* acc += sigmoid(gw . xin) * shared_down(silu(gate xin) * up xin): the
 * shared expert of one token (src/moe.c:1235-1293, bf16 weights). */
int orc_shared_add(const OrcLayerW *lw, int H, int M, const float *xin, float *acc);

/* Batched variant (prefill; src/moe.c:1480-1707): B tokens, states [B][H]
 * row-major, each token routed by its own router pass; grouped by expert,
 * combined in selection order.  idx/w are [B][K]. Per (token, selection)
 * the arithmetic is that of orc_moe_layer, so results are bit-identical
 * to B independent orc_moe_layer calls (as moe.c:1462-1464 states for the
 * reference). */
int orc_moe_batch(int fmt, int H, int M, int E, int K, int renorm,
                  const OrcLayerW *lw, const OrcExpertLayout *lay, int B,
                  float *states, int *idx, float *w);

/* The batched step with the routing given (the reference's
 * ds4f_moe_step_batch proper, src/moe.c:1480-1707, whose caller routes):
 * RMSNorm of each state, then chains grouped by expert, selection-order
 * combine, shared expert, residual. idx / w [B][K]; idx < 0 skipped. */
int orc_moe_batch_sel(int fmt, int H, int M, int K, const OrcLayerW *lw,
                      const OrcExpertLayout *lay, int B, float *states,
                      const int *idx, const float *w);

#ifdef __cplusplus
}
#endif

#endif
