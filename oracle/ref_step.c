/* ref_step.c -- TEST INFRASTRUCTURE ONLY: a caller of the reference's own
 * ds4f_moe_step (src/moe.c:948-1456), compiled against the reference's
 * headers into oracle/_ref/libds4f_ref.so beside the reference's objects.
 *
 * The reference step is usable as built only with a trunk layout and a pool
 * layout from its converter's JSON; this file builds both in memory for one
 * Qwen3.5 layer of MXFP4 experts (the format its expert chain reads,
 * src/moe.c:619-640): the post-attention norm as the layer's only trunk
 * tensor, no shared expert, no mHC, no latent projections. The step then
 * takes the Qwen3.5 branch: xin = rmsnorm(state), the K routed chains on
 * their own threads, the selection-order combine, state += acc
 * (src/moe.c:986-993, 1162-1227, 1424). tests/test_oracle_step.py compares
 * it with the oracle's restated step.
 */
#include <stdint.h>
#include <stdlib.h>
#include <string.h>

#include "ds4f/moe.h"

/* state[H] in/out; norm [H] bf16; experts [E][slot_bytes]: gate [M x H],
 * up [M x H], down [H x M], each e2m1 values at rel_v[i] then E8M0 scales
 * per 32 at rel_s[i]; sel / wsel [K] the routing (as the engine's router
 * call site hands it over, src/main.c:1088-1132). Returns the step's
 * status, -1 on an allocation failure. */
int orcref_moe_step_mxfp4(int H, int M, int E, int K, const uint16_t *norm, const uint8_t *experts,
                          const int64_t rel_v[3], const int64_t rel_s[3], int64_t slot_bytes,
                          const int *sel, const float *wsel, float *state) {
    Ds4fCfg cfg;
    memset(&cfg, 0, sizeof cfg);
    cfg.n_layers = 1;
    cfg.n_experts = E;
    cfg.topk = K;
    cfg.hidden = H;
    cfg.latent = H;            /* no latent projection: latent = xin */
    cfg.moe_inter = M;
    cfg.expert_nbytes = slot_bytes;

    Ds4fTrunkTensor tn;
    memset(&tn, 0, sizeof tn);
    strcpy(tn.name, "post_attention_layernorm.weight");
    tn.dtype = 4;              /* BF16 */
    tn.rank = 1;
    tn.dims[0] = H;
    tn.off = 0;
    tn.nbytes = (long)H * 2;
    int t_off[2] = {0, 1};
    Ds4fTrunkLayout *tl = (Ds4fTrunkLayout *)malloc(sizeof *tl);
    if (!tl) return -1;
    memset(tl, 0xFF, sizeof *tl);       /* every role index -1: absent */
    tl->n_layers = 1;
    tl->t = &tn;
    tl->t_off = t_off;
    tl->ffn_norm[0] = 0;

    Ds4fExpertLayout *el = (Ds4fExpertLayout *)calloc((size_t)E, sizeof *el);
    if (!el) { free(tl); return -1; }
    const long dims[3][2] = {{M, H}, {M, H}, {H, M}};
    for (int x = 0; x < E; x++) {
        el[x].n = 3;
        el[x].chain = 1;       /* Qwen3: gate || up -> silu -> down */
        for (int i = 0; i < 3; i++) {
            Ds4fMoETensor *t = &el[x].t[i];
            t->rank = 2;
            t->dims[0] = dims[i][0];
            t->dims[1] = dims[i][1];
            t->rel_v = (long)rel_v[i];
            t->rel_s = (long)rel_s[i];
            t->rel_b = -1;
            t->v_nbytes = dims[i][0] * dims[i][1] / 2;
            t->s_nbytes = dims[i][0] * dims[i][1] / 32;
            t->bsize = 32;
            t->fmt = 0;        /* mxfp4 */
        }
    }
    Ds4fPoolLayout pl;
    pl.n_layers = 1;
    pl.n_experts = E;
    pl.expert_nbytes = slot_bytes;
    pl.max_rc = (int64_t)M * H;
    pl.exp = el;

    const uint8_t *es[64];
    float *js[64];
    float *scratch = (float *)malloc((size_t)M * H * sizeof(float));
    int rc = scratch ? 0 : -1;
    int nj = 0;
    for (int j = 0; j < K && j < 64 && !rc; j++) {
        es[j] = experts + (int64_t)sel[j] * slot_bytes;
        if (j > 0) {
            js[nj] = (float *)malloc((size_t)M * H * sizeof(float));
            if (!js[nj]) rc = -1;
            else nj++;
        }
    }
    int64_t nmv = 0, ndec = 0;
    if (!rc)
        rc = ds4f_moe_step(&cfg, tl, 0, (const uint8_t *)norm, &pl, es, sel, wsel, state, scratch,
                           (long)M * H, js, &nmv, &ndec);
    for (int j = 0; j < nj; j++) free(js[j]);
    free(scratch);
    free(el);
    free(tl);
    return rc;
}
