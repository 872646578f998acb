// moe.cu -- one Qwen3.5 MoE layer for one token on the GPU: RMSNorm,
// router logits, certified top-k + softmax + renorm, fused gate/up +
// SiLU-mul for the top-k experts and the shared expert, fused down +
// selection-order combine + shared-gate + residual.
//
// Reference: ds4f_moe_step (src/moe.c:948-1456, Qwen3.5 no-mHC branch),
// its router call site (src/main.c:1014-1088) and ds4f_topk
// (src/moe.c:531-561). The host/GPU round trips of the reference's Metal
// path (two dispatches plus a CPU SiLU per layer, src/moe.c:1105-1150)
// become four kernels that never leave the device.
#include "../../include/ds4f/gpu_cuda.h"
#include "model.cuh"

#include <algorithm>
#include <mutex>

namespace ds4f {

namespace {

constexpr int kRouteWarps = 8;
constexpr double kUnitRoundoff = 5.9604644775390625e-08;   // 2^-24

// ---------------------------------------------------------------------------
// RMSNorm into shared memory (src/moe.c:841-851; the router's copy
// src/main.c:1014-1033 is identical): sum of squares in double, r =
// sqrtf(float(ss / H) + 1e-6f), x / r * w with IEEE division. The sum
// order is a fixed tree (thread-strided partials, xor-butterfly, warps in
// order), so every CTA and every run gets the same bits.
// ---------------------------------------------------------------------------
__device__ void rmsnorm_smem(const float *__restrict__ state,
                             const uint16_t *__restrict__ norm, int H,
                             float *xs, double *red, float prescale) {
    double ss = 0.0;
    for (int i = threadIdx.x; i < H; i += blockDim.x) {
        double v = (double)state[i];
        ss = __dadd_rn(ss, __dmul_rn(v, v));
    }
    ss = warp_sum_d(ss);
    int nw = blockDim.x >> 5;
    if ((threadIdx.x & 31) == 0) red[threadIdx.x >> 5] = ss;
    __syncthreads();
    if (threadIdx.x == 0) {
        double t = 0.0;
        for (int k = 0; k < nw; k++) t = __dadd_rn(t, red[k]);
        red[32] = t;
    }
    __syncthreads();
    float r = __fsqrt_rn(__fadd_rn(__double2float_rn(__ddiv_rn(red[32], (double)H)),
                                   1e-6f));
    for (int i = threadIdx.x; i < H; i += blockDim.x)
        xs[i] = __fmul_rn(__fmul_rn(__fdiv_rn(state[i], r), bf16_to_f32(norm[i])),
                          prescale);
    __syncthreads();
}

// ---------------------------------------------------------------------------
// Router logits with a certificate. The reference sums each row
// sequentially in fp32: s_c = fl(s_{c-1} + p_c), p_c = fl(w_c x_c)
// (ds4f_bf16_matvec scalar, src/kernels.c:97-102). Here S = sum p_c in
// double (products bit-identical to the reference's), and
//   |s_n - S| <= u sum_c |S_c| / (1 - n u),   S_c = exact prefix sums,
// bounded per 8-element chunk q (prefix P_q) by 8|P_q| + sum_t |p_t|(8-t).
// Bnd = 1.001 u * that sum (the 1.001 covers 1/(1-nu) and double rounding).
// k_topk decides the top-k from [S - Bnd, S + Bnd] and recomputes exact
// fp32 sums only when two candidates' intervals overlap.
// Token b = blockIdx.y of a batch: state [b][H], xin [b][H], S / Bnd [b][E].
// ---------------------------------------------------------------------------
__global__ void __launch_bounds__(256)
k_route(const float *__restrict__ state, const uint16_t *__restrict__ trunk_l,
        TrunkLayout tr, int H, int E, float *__restrict__ xin_out,
        double *__restrict__ S, double *__restrict__ Bnd) {
    extern __shared__ float xs[];
    __shared__ double red[33];
    state += (int64_t)blockIdx.y * H;
    xin_out += (int64_t)blockIdx.y * H;
    S += (int64_t)blockIdx.y * E;
    Bnd += (int64_t)blockIdx.y * E;
    rmsnorm_smem(state, trunk_l + tr.norm, H, xs, red, 1.0f);
    if (blockIdx.x == 0)
        for (int i = threadIdx.x; i < H; i += blockDim.x) xin_out[i] = xs[i];
    const int lane = threadIdx.x & 31, warp = threadIdx.x >> 5;
    const int e = blockIdx.x * kRouteWarps + warp;
    if (e >= E) return;
    const uint16_t *row = trunk_l + tr.router + (int64_t)e * H;
    const int rounds = H / 256;
    double base = 0.0, bsum = 0.0;
    for (int k = 0; k < rounds; k++) {
        int q = lane + 32 * k;
        uint4 w = ldg_stream(row + q * 8);
        const float *x = xs + q * 8;
        uint32_t ww[4] = {w.x, w.y, w.z, w.w};
        double T = 0.0, A = 0.0;
#pragma unroll
        for (int t = 0; t < 8; t++) {
            uint32_t h = (t & 1) ? (ww[t >> 1] & 0xFFFF0000u) : (ww[t >> 1] << 16);
            float p = __fmul_rn(__uint_as_float(h), x[t]);
            T = __dadd_rn(T, (double)p);
            A = __dadd_rn(A, (double)fabsf(p) * (double)(8 - t));
        }
        double incl = T;
#pragma unroll
        for (int o = 1; o < 32; o <<= 1) {
            double y = __shfl_up_sync(0xFFFFFFFFu, incl, o);
            if (lane >= o) incl = __dadd_rn(incl, y);
        }
        double excl = __shfl_up_sync(0xFFFFFFFFu, incl, 1);
        if (lane == 0) excl = 0.0;
        double P = __dadd_rn(base, excl);
        bsum = __dadd_rn(bsum, __dadd_rn(8.0 * fabs(P), A));
        base = __dadd_rn(base, __shfl_sync(0xFFFFFFFFu, incl, 31));
    }
    bsum = warp_sum_d(bsum);
    if (lane == 0) {
        S[e] = base;
        Bnd[e] = 1.001 * kUnitRoundoff * bsum + 1e-300;
    }
}

// Exact reference-order fp32 logit of router row e (the fallback).
__device__ float exact_logit(const uint16_t *__restrict__ row,
                             const float *__restrict__ xs, int H) {
    float acc = 0.0f;
    for (int c = 0; c < H; c++)
        acc = __fadd_rn(acc, __fmul_rn(bf16_to_f32(row[c]), xs[c]));
    return acc;   // + 0.0f bias (src/kernels.c:101) changes nothing but -0
}

// ---------------------------------------------------------------------------
// Top-k (src/moe.c:531-561) from the certified logits, one CTA.
// Selection: descending, lower index first among equal values. Weights:
// softmax over all E in double with the max subtracted, the selected
// probabilities kept, then (renorm) divided by their fp32 sum in j order.
// Token b = blockIdx.x of a batch: S / Bnd [b][E], xin [b][H], idx / w [b][K].
// ---------------------------------------------------------------------------
__global__ void __launch_bounds__(256)
k_topk(const double *__restrict__ S, const double *__restrict__ Bnd,
       const float *__restrict__ xin, const uint16_t *__restrict__ router,
       int H, int E, int K, int renorm, int exact_all, int *__restrict__ idx_out,
       float *__restrict__ w_out, unsigned *__restrict__ diag) {
    S += (int64_t)blockIdx.x * E;
    Bnd += (int64_t)blockIdx.x * E;
    xin += (int64_t)blockIdx.x * H;
    idx_out += (int64_t)blockIdx.x * K;
    w_out += (int64_t)blockIdx.x * K;
    extern __shared__ unsigned char sm[];
    double *lo = (double *)sm;
    double *hi = lo + E;
    float *v = (float *)(hi + E);
    int *cand = (int *)(v + E);
    int *rk = cand + E;
    float *xs = (float *)(rk + E);
    __shared__ double lk_s, red[8];
    __shared__ int ncand_s, cert_s, fast_s, nonfin_s, sel_s[64];
    const int tid = threadIdx.x;
    if (tid == 0) { ncand_s = 0; cert_s = 1; fast_s = 0; nonfin_s = 0; }
    __syncthreads();
    for (int e = tid; e < E; e += blockDim.x) {
        double b = exact_all ? 0.0 : Bnd[e];
        lo[e] = S[e] - b;
        hi[e] = S[e] + b;
        v[e] = (float)S[e];
        if (!isfinite(S[e]) || !isfinite(b)) nonfin_s = 1;
    }
    __syncthreads();
    // a logit that is not finite (NaN or inf state): no interval orders it,
    // so every expert's exact logit goes through the reference's own
    // insertion rule below
    const bool nonfin = nonfin_s != 0;
    // Fast path (top-8 of at most 256): warp 0 proposes the 8 by a sorting
    // network on 32-bit keys of the logits and certifies them on the
    // intervals rounded outward to fp32 (consecutive selections separate,
    // and only the 8 reach the last one's lower bound); the general path
    // below runs only when that fails. Both select by the same rule, so a
    // certified proposal is the general path's selection.
    if (K == 8 && E % 32 == 0 && E <= 256 && !exact_all && !nonfin) {
        if (tid < 32) {
            const int lane = tid, NE = E / 32;
            uint32_t k8[8];
#pragma unroll
            for (int i = 0; i < 8; i++)
                k8[i] = i < NE ? tk_key(__double2float_rn(S[lane + 32 * i]), lane + 32 * i) : 0u;
            tk_sort8(k8);
            tk_warp_top8(k8);
            int er = 0;
#pragma unroll
            for (int j = 0; j < 8; j++) if (j == lane) er = tk_expert(k8[j]);
            float lor = 3.0e38f, hir = -3.0e38f;
            if (lane < 8) {
                lor = __double2float_rd(__dsub_rd(S[er], Bnd[er]));
                hir = __double2float_ru(__dadd_ru(S[er], Bnd[er]));
            }
            const float hin = __shfl_down_sync(0xFFFFFFFFu, hir, 1);
            const bool sep = lane >= 7 || lor > hin;
            const float lo8 = __shfl_sync(0xFFFFFFFFu, lor, 7);
            int nmine = 0;
            for (int i = 0; i < NE; i++)
                nmine += __double2float_ru(__dadd_ru(S[lane + 32 * i], Bnd[lane + 32 * i])) >= lo8;
            const int nreach = (int)__reduce_add_sync(0xFFFFFFFFu, (unsigned)nmine);
            const bool cert = __all_sync(0xFFFFFFFFu, sep) && nreach == 8;
            if (cert && lane < 8) sel_s[lane] = er;
            if (lane == 0) fast_s = cert ? 1 : 0;
        }
        __syncthreads();
    }
    if (!exact_all && !fast_s && !nonfin) {
        // K-th largest lower bound
        for (int e = tid; e < E; e += blockDim.x) {
            int r = 0;
            double le = lo[e];
            for (int f = 0; f < E; f++) r += (lo[f] > le) || (lo[f] == le && f < e);
            if (r == K - 1) lk_s = le;
        }
        __syncthreads();
        double lk = lk_s;
        for (int e = tid; e < E; e += blockDim.x) {
            cand[e] = hi[e] >= lk;
            if (cand[e]) atomicAdd(&ncand_s, 1);
        }
        __syncthreads();
        if (ncand_s != K) cert_s = 0;
        __syncthreads();
        if (cert_s) {
            // order by S among candidates; adjacent intervals must separate
            for (int e = tid; e < E; e += blockDim.x) {
                rk[e] = -1;
                if (!cand[e]) continue;
                int r = 0;
                for (int f = 0; f < E; f++)
                    r += cand[f] && (S[f] > S[e] || (S[f] == S[e] && f < e));
                rk[e] = r;
                sel_s[r] = e;
            }
            __syncthreads();
            for (int r = tid; r + 1 < K; r += blockDim.x)
                if (!(lo[sel_s[r]] > hi[sel_s[r + 1]])) cert_s = 0;
            __syncthreads();
        }
    }
    if (nonfin || (!fast_s && (exact_all || !cert_s))) {
        // exact reference-order logits for every candidate (all experts in
        // exact mode or with a non-finite logit), then select on them
        for (int i = tid; i < H; i += blockDim.x) xs[i] = xin[i];
        __syncthreads();
        for (int e = tid; e < E; e += blockDim.x) {
            if (exact_all || nonfin) cand[e] = 1;
            if (cand[e]) v[e] = exact_logit(router + (int64_t)e * H, xs, H);
        }
        __syncthreads();
        if (nonfin) {
            if (tid == 0) tk_insertion(v, E, K, sel_s);
        } else {
            for (int e = tid; e < E; e += blockDim.x) {
                if (!cand[e]) continue;
                int r = 0;
                for (int f = 0; f < E; f++)
                    r += cand[f] && (v[f] > v[e] || (v[f] == v[e] && f < e));
                if (r < K) sel_s[r] = e;
            }
        }
        if (tid == 0 && !exact_all) atomicAdd(diag + 1, 1u);
        __syncthreads();
    }
    // softmax over all E in double, max subtracted (the max as a block
    // reduction: the same value in any order)
    double mx = -1e300;
    for (int e = tid; e < E; e += blockDim.x) mx = fmax(mx, (double)v[e]);
#pragma unroll
    for (int o = 16; o > 0; o >>= 1) mx = fmax(mx, __shfl_xor_sync(0xFFFFFFFFu, mx, o));
    if ((tid & 31) == 0) red[tid >> 5] = mx;
    __syncthreads();
    mx = red[0];
    for (int k = 1; k < (int)(blockDim.x >> 5); k++) mx = fmax(mx, red[k]);
    __syncthreads();
    double part = 0.0;
    for (int e = tid; e < E; e += blockDim.x) part += exp((double)v[e] - mx);
    part = warp_sum_d(part);
    if ((tid & 31) == 0) red[tid >> 5] = part;
    __syncthreads();
    // the K selected probabilities in parallel, their fp32 sum in j order
    __shared__ float wj_s[64];
    if (tid < K) {
        double sw = 0.0;
        for (int k = 0; k < (int)(blockDim.x >> 5); k++) sw += red[k];
        wj_s[tid] = (float)(exp((double)v[sel_s[tid]] - mx) / sw);
    }
    __syncthreads();
    if (tid == 0) {
        float s = 0.0f;
        for (int j = 0; j < K; j++) s = __fadd_rn(s, wj_s[j]);
        for (int j = 0; j < K; j++) {
            idx_out[j] = sel_s[j];
            w_out[j] = (renorm && s > 0.0f) ? __fdiv_rn(wj_s[j], s) : wj_s[j];
        }
        atomicAdd(diag, 1u);
    }
}


// ---------------------------------------------------------------------------
// Row-dot building blocks. A lane holds its columns of x in registers and
// dots them with 16-byte chunks of a weight row of C elements:
//   FP8   chunk = 16 E4M3,  MXFP4 chunk = 32 E2M1,  BF16 chunk = 8 bf16.
// lpr = lanes per row = min(32, C / chunk); a warp covers 32 / lpr rows per
// step; lane chunks are q = lane % lpr + lpr * k, k < kch. x is pre-scaled
// by 2^64 (common.cuh) so every product stays a normal float; each
// chunk's partial dot is rescaled with its block scale.
// ---------------------------------------------------------------------------
template <int FMT> struct Chunk;
template <> struct Chunk<DS4F_FMT_FP8>   { static constexpr int ce = 16; };
template <> struct Chunk<DS4F_FMT_MXFP4> { static constexpr int ce = 32; };
template <> struct Chunk<3>              { static constexpr int ce = 8; };   // bf16
constexpr int kBF16 = 3;

template <int FMT, int C>
struct RowGeom {
    static constexpr int ce = Chunk<FMT>::ce;
    static constexpr int nq = C / ce;
    static constexpr int lpr = nq < 32 ? nq : 32;
    static constexpr int kch = nq / lpr;
    static constexpr int rps = 32 / lpr;
    static constexpr int bytes = FMT == DS4F_FMT_FP8 ? C : FMT == DS4F_FMT_MXFP4 ? C / 2 : 2 * C;
    static_assert(nq * ce == C && kch * lpr == nq && (lpr & (lpr - 1)) == 0,
                  "row length must split into power-of-two lane groups");
};

template <int FMT, int C>
__device__ __forceinline__ void load_x(float (&x)[RowGeom<FMT, C>::kch * RowGeom<FMT, C>::ce],
                                       const float *xs) {
    using G = RowGeom<FMT, C>;
    const int ql = (threadIdx.x & 31) % G::lpr;
#pragma unroll
    for (int k = 0; k < G::kch; k++) {
        const float4 *src = (const float4 *)(xs + (ql + G::lpr * k) * G::ce);
#pragma unroll
        for (int e = 0; e < G::ce / 4; e++) {
            float4 v = src[e];
            x[k * G::ce + 4 * e] = v.x;     x[k * G::ce + 4 * e + 1] = v.y;
            x[k * G::ce + 4 * e + 2] = v.z; x[k * G::ce + 4 * e + 3] = v.w;
        }
    }
}

template <int FMT, int C>
__device__ __forceinline__ void load_row(uint4 (&b)[RowGeom<FMT, C>::kch],
                                         const uint8_t *row) {
    using G = RowGeom<FMT, C>;
    const int ql = (threadIdx.x & 31) % G::lpr;
#pragma unroll
    for (int k = 0; k < G::kch; k++) b[k] = ldg_stream(row + (ql + G::lpr * k) * 16);
}

// Sum over the row of chunk_dot * scale(q); returned per lane (reduce over
// the lpr lanes of the row with row_reduce).
template <int FMT, int C, typename ScaleFn>
__device__ __forceinline__ float row_partial(const uint4 (&b)[RowGeom<FMT, C>::kch],
                                             const float (&x)[RowGeom<FMT, C>::kch * RowGeom<FMT, C>::ce],
                                             ScaleFn scale) {
    using G = RowGeom<FMT, C>;
    const int ql = (threadIdx.x & 31) % G::lpr;
    float acc = 0.f;
#pragma unroll
    for (int k = 0; k < G::kch; k++) {
        const int q = ql + G::lpr * k;
        if constexpr (FMT == DS4F_FMT_FP8) {
            acc = fmaf(f8_dot16(b[k], x + k * G::ce) * DS4F_F8_POST, scale(q), acc);
        } else if constexpr (FMT == DS4F_FMT_MXFP4) {
            acc = fmaf(e2m1_dot32(b[k], x + k * G::ce) * DS4F_E2M1_POST, scale(q), acc);
        } else {
            acc += bf16_dot8(b[k], x + k * G::ce);
        }
    }
    return acc;
}

template <int LPR>
__device__ __forceinline__ float row_reduce(float v) {
#pragma unroll
    for (int o = LPR >> 1; o > 0; o >>= 1) v += __shfl_xor_sync(0xFFFFFFFFu, v, o);
    return v;
}

// FP8 fp32 128x128 block scale for (row r, chunk q) of a [R x C] matrix.
template <int C>
__device__ __forceinline__ float f8s(const float *s, int r, int q) {
    return __ldg(s + (r >> 7) * (C / 128) + (q >> 3));
}
// MXFP4 E8M0 scale for (row r, chunk q): flat block (r*C + 32q) / 32.
template <int C>
__device__ __forceinline__ float mxs(const uint8_t *s, int r, int q) {
    return e8m0_to_f32(__ldg(s + r * (C / 32) + q));
}

struct LayerArgs {
    const uint8_t *pool_l;       // expert slots of layer L (first expert = efirst)
    int64_t slot_bytes;
    SlotLayout slot;
    const uint16_t *trunk_l;
    TrunkLayout tr;
    int E, K, efirst, ecount;
    const int *idx;
    const float *w;
    const float *xin;
    float *chain;                // [(K+1) M]
    float *sgate;
    float *state;                // [H] in/out
    float *acc_out;              // [H] or null
    const int *slot_of;          // streaming: selection j's arena slot (pool_l = the arena);
                                 //   null: expert idx[j] at pool_l + (idx[j] - efirst) slots
    int partial;                 // 1: expert-parallel shard step -- only selections in
                                 //    [efirst, efirst + ecount) count, acc_out gets the
                                 //    shard's partial sum, the state is left alone
    int add_shared;              // shared expert included (partial: on one rank only)
};

// ---------------------------------------------------------------------------
// gate/up + SiLU-mul. Static partition: CTA c of G owns routed (selection,
// row) pairs [c KM/G, (c+1) KM/G) and shared rows [c M/G, (c+1) M/G); each
// warp takes two pairs at a time (gate and up rows of both in flight). The
// shared_expert_gate dot (1 x H bf16) goes to the last CTA.
// chain[j M + i] = silu(gate_j x)_i * (up_j x)_i   (src/moe.c:619-649)
// ---------------------------------------------------------------------------
template <int FMT, int H, int M>
__global__ void __launch_bounds__(256)
k_gateup(LayerArgs a) {
    __shared__ __align__(16) float xs[H];
    using G = RowGeom<FMT, H>;
    using GB = RowGeom<kBF16, H>;
    static_assert(G::lpr == 32 && GB::lpr == 32, "gate/up rows span a warp");
    const int lane = threadIdx.x & 31, warp = threadIdx.x >> 5;
    for (int i = threadIdx.x; i < H; i += blockDim.x) xs[i] = a.xin[i] * DS4F_X_PRESCALE;
    __syncthreads();
    // the selections held here, in selection order (all of them unless
    // this is an expert-parallel shard step)
    __shared__ int loc[16];
    __shared__ int nloc;
    if (threadIdx.x == 0) {
        int n = 0;
        for (int j = 0; j < a.K; j++)
            if (a.idx[j] >= a.efirst && a.idx[j] < a.efirst + a.ecount) loc[n++] = j;
        nloc = n;
    }
    __syncthreads();
    const int nb = gridDim.x, cb = blockIdx.x;
    const int P = nloc * M;
    const int p0 = (int)((int64_t)cb * P / nb), p1 = (int)((int64_t)(cb + 1) * P / nb);
    {
        float x[G::kch * G::ce];
        load_x<FMT, H>(x, xs);
        for (int pp = p0 + 2 * warp; pp < p1; pp += 16) {
            uint4 bg[2][G::kch], bu[2][G::kch];
            const uint8_t *base[2];
            int ii[2], jj[2];
#pragma unroll
            for (int t = 0; t < 2; t++) {
                int p = min(pp + t, p1 - 1);
                jj[t] = loc[p / M]; ii[t] = p % M;
                base[t] = a.pool_l + (int64_t)(a.slot_of ? a.slot_of[jj[t]] : a.idx[jj[t]] - a.efirst) * a.slot_bytes;
                load_row<FMT, H>(bg[t], base[t] + a.slot.rel_v[0] + (int64_t)ii[t] * G::bytes);
                load_row<FMT, H>(bu[t], base[t] + a.slot.rel_v[1] + (int64_t)ii[t] * G::bytes);
            }
#pragma unroll
            for (int t = 0; t < 2; t++) {
                float g, u;
                if constexpr (FMT == DS4F_FMT_FP8) {
                    const float *sg = (const float *)(base[t] + a.slot.rel_s[0]);
                    const float *su = (const float *)(base[t] + a.slot.rel_s[1]);
                    g = row_partial<FMT, H>(bg[t], x, [&](int q) { return f8s<H>(sg, ii[t], q); });
                    u = row_partial<FMT, H>(bu[t], x, [&](int q) { return f8s<H>(su, ii[t], q); });
                } else {
                    const uint8_t *sg = base[t] + a.slot.rel_s[0];
                    const uint8_t *su = base[t] + a.slot.rel_s[1];
                    g = row_partial<FMT, H>(bg[t], x, [&](int q) { return mxs<H>(sg, ii[t], q); });
                    u = row_partial<FMT, H>(bu[t], x, [&](int q) { return mxs<H>(su, ii[t], q); });
                }
                g = warp_sum(g);
                u = warp_sum(u);
                if (lane == 0 && pp + t < p1) a.chain[jj[t] * M + ii[t]] = silu_mul(g, u);
            }
        }
    }
    if (a.add_shared) {
        float x[GB::kch * GB::ce];
        load_x<kBF16, H>(x, xs);
        const int s0 = (int)((int64_t)cb * M / nb), s1 = (int)((int64_t)(cb + 1) * M / nb);
        const uint8_t *tg = (const uint8_t *)(a.trunk_l + a.tr.sh_gate);
        const uint8_t *tu = (const uint8_t *)(a.trunk_l + a.tr.sh_up);
        auto none = [](int) { return 1.0f; };
        for (int i = s0 + warp; i < s1; i += 8) {
            uint4 bg[GB::kch], bu[GB::kch];
            load_row<kBF16, H>(bg, tg + (int64_t)i * GB::bytes);
            load_row<kBF16, H>(bu, tu + (int64_t)i * GB::bytes);
            float g = warp_sum(row_partial<kBF16, H>(bg, x, none)) * DS4F_BF16_POST;
            float u = warp_sum(row_partial<kBF16, H>(bu, x, none)) * DS4F_BF16_POST;
            if (lane == 0) a.chain[a.K * M + i] = silu_mul(g, u);
        }
        if (cb == nb - 1 && warp == 7) {
            uint4 bw[GB::kch];
            load_row<kBF16, H>(bw, (const uint8_t *)(a.trunk_l + a.tr.sh_gw));
            float g = warp_sum(row_partial<kBF16, H>(bw, x, none)) * DS4F_BF16_POST;
            if (lane == 0) *a.sgate = g;
        }
    }
}

// ---------------------------------------------------------------------------
// down + combine + shared gate + residual. CTA c owns output rows
// [c H/G, (c+1) H/G). Warp j < K computes down_j(chain_j) for those rows,
// warp K the shared expert's bf16 down; then one thread per row combines
// in selection order (src/moe.c:1203-1227), adds sigmoid(sgate) * shared
// (:1279-1282) and the residual (:1424).
// ---------------------------------------------------------------------------
constexpr int kDownMaxRows = 32;

template <int FMT, int H, int M>
__global__ void __launch_bounds__(544)
k_down(LayerArgs a) {
    __shared__ __align__(16) float cs[17][M];
    __shared__ float outs[17][kDownMaxRows];
    using G = RowGeom<FMT, M>;
    using GB = RowGeom<kBF16, M>;
    const int lane = threadIdx.x & 31, warp = threadIdx.x >> 5;
    const int K = a.K;
    for (int i = threadIdx.x; i < (K + 1) * M; i += blockDim.x)
        cs[i / M][i % M] = a.chain[i] * DS4F_X_PRESCALE;
    __syncthreads();
    const int nb = gridDim.x, cb = blockIdx.x;
    const int r0 = (int)((int64_t)cb * H / nb), r1 = (int)((int64_t)(cb + 1) * H / nb);
    const int nr = r1 - r0;
    const bool held = warp < K && a.idx[warp] >= a.efirst && a.idx[warp] < a.efirst + a.ecount;
    if (warp < K && !held) {
        for (int t = lane; t < nr; t += 32) outs[warp][t] = 0.0f;    // another rank's selection
    } else if (warp < K) {
        float x[G::kch * G::ce];
        load_x<FMT, M>(x, cs[warp]);
        const uint8_t *base = a.pool_l + (int64_t)(a.slot_of ? a.slot_of[warp] : a.idx[warp] - a.efirst) * a.slot_bytes;
        const uint8_t *dv = base + a.slot.rel_v[2];
        const int sub = lane / G::lpr;
        for (int rr = 0; rr < nr; rr += 4 * G::rps) {
            uint4 b[4][G::kch];
            int rows[4];
#pragma unroll
            for (int t = 0; t < 4; t++) {
                rows[t] = min(r0 + rr + t * G::rps + sub, r1 - 1);
                load_row<FMT, M>(b[t], dv + (int64_t)rows[t] * G::bytes);
            }
#pragma unroll
            for (int t = 0; t < 4; t++) {
                float v;
                if constexpr (FMT == DS4F_FMT_FP8) {
                    const float *sd = (const float *)(base + a.slot.rel_s[2]);
                    v = row_partial<FMT, M>(b[t], x, [&](int q) { return f8s<M>(sd, rows[t], q); });
                } else {
                    const uint8_t *sd = base + a.slot.rel_s[2];
                    v = row_partial<FMT, M>(b[t], x, [&](int q) { return mxs<M>(sd, rows[t], q); });
                }
                v = row_reduce<G::lpr>(v);
                int lr = rr + t * G::rps + sub;
                if (lane % G::lpr == 0 && lr < nr) outs[warp][lr] = v;
            }
        }
    } else if (warp == K && !a.add_shared) {
        for (int t = lane; t < nr; t += 32) outs[K][t] = 0.0f;
    } else if (warp == K) {
        float x[GB::kch * GB::ce];
        load_x<kBF16, M>(x, cs[K]);
        const uint8_t *dv = (const uint8_t *)(a.trunk_l + a.tr.sh_down);
        const int sub = lane / GB::lpr;
        auto none = [](int) { return 1.0f; };
        for (int rr = 0; rr < nr; rr += 4 * GB::rps) {
            uint4 b[4][GB::kch];
#pragma unroll
            for (int t = 0; t < 4; t++)
                load_row<kBF16, M>(b[t], dv + (int64_t)min(r0 + rr + t * GB::rps + sub, r1 - 1) * GB::bytes);
#pragma unroll
            for (int t = 0; t < 4; t++) {
                float v = row_reduce<GB::lpr>(row_partial<kBF16, M>(b[t], x, none)) * DS4F_BF16_POST;
                int lr = rr + t * GB::rps + sub;
                if (lane % GB::lpr == 0 && lr < nr) outs[K][lr] = v;
            }
        }
    }
    __syncthreads();
    if (threadIdx.x < nr) {
        const int t = threadIdx.x, r = r0 + t;
        float acc = 0.0f;
        for (int j = 0; j < K; j++)
            if (a.idx[j] >= a.efirst && a.idx[j] < a.efirst + a.ecount)
                acc = __fadd_rn(acc, __fmul_rn(a.w[j], outs[j][t]));
        if (a.add_shared) acc = __fadd_rn(acc, __fmul_rn(sigmoid_ref(*a.sgate), outs[K][t]));
        if (a.acc_out) a.acc_out[r] = acc;
        if (!a.partial) a.state[r] = __fadd_rn(a.state[r], acc);
    }
}

int num_sms() {
    int dev = 0, sms = 148;
    cudaGetDevice(&dev);
    cudaDeviceGetAttribute(&sms, cudaDevAttrMultiProcessorCount, dev);
    return sms;
}

template <int FMT, int H, int M>
int launch_chain(const LayerArgs &a, cudaStream_t st) {
    int G = num_sms();
    k_gateup<FMT, H, M><<<G, 256, 0, st>>>(a);
    DS4F_CUDA(cudaGetLastError());
    int Gd = std::max(G, (H + kDownMaxRows - 1) / kDownMaxRows);
    k_down<FMT, H, M><<<Gd, 32 * (a.K + 1), 0, st>>>(a);
    DS4F_CUDA(cudaGetLastError());
    return 0;
}

}  // namespace

int slot_layout(int fmt, int H, int M, SlotLayout *s) {
    int64_t mh = (int64_t)M * H, vb, sb;
    if (fmt == DS4F_FMT_FP8) {
        DS4F_REQUIRE(H % 128 == 0 && M % 128 == 0, "FP8 pool needs H, M multiples of 128");
        vb = mh; sb = (int64_t)(M / 128) * (H / 128) * 4;
    } else if (fmt == DS4F_FMT_MXFP4) {
        DS4F_REQUIRE(H % 32 == 0 && M % 32 == 0, "MXFP4 pool needs H, M multiples of 32");
        vb = mh / 2; sb = mh / 32;
    } else {
        DS4F_REQUIRE(false, "unknown expert format %d", fmt);
    }
    int64_t off = 0;
    for (int t = 0; t < 3; t++) {
        s->rel_v[t] = off; off += vb;
        s->rel_s[t] = off; off += sb;
    }
    s->nbytes = off;
    return 0;
}

int trunk_layout(int H, int M, int E, TrunkLayout *t) {
    auto al = [](int64_t n) { return (n + 127) / 128 * 128; };   // 256 B
    int64_t o = 0;
    t->norm = o; o += al(H);
    t->router = o; o += al((int64_t)E * H);
    t->sh_gate = o; o += al((int64_t)M * H);
    t->sh_up = o; o += al((int64_t)M * H);
    t->sh_down = o; o += al((int64_t)H * M);
    t->sh_gw = o; o += al(H);
    t->n = o;
    return 0;
}

int route_batch_launch(Model *m, int L, const float *states, int B, float *xin, double *S, double *Bnd,
                       int *idx, float *w, cudaStream_t st) {
    const ModelDesc &d = m->d;
    const int H = d.hidden, E = d.n_experts, K = d.topk;
    DS4F_REQUIRE(B > 0 && B <= 65535, "route: batch %d out of range", B);
    const uint16_t *trunk_l = m->trunk + (int64_t)L * m->tr.n;
    k_route<<<dim3((E + kRouteWarps - 1) / kRouteWarps, B), 256, H * sizeof(float), st>>>(
        states, trunk_l, m->tr, H, E, xin, S, Bnd);
    DS4F_CUDA(cudaGetLastError());
    const size_t tk_smem = (size_t)E * (8 + 8 + 4 + 4 + 4) + (size_t)H * 4;
    k_topk<<<B, 256, tk_smem, st>>>(S, Bnd, xin, trunk_l + m->tr.router, H, E, K, d.renorm, d.router_exact,
                                    idx, w, m->w.diag);
    DS4F_CUDA(cudaGetLastError());
    return 0;
}

int moe_layer_launch(Model *m, int L, float *state, int *idx_out, float *w_out,
                     cudaStream_t st) {
    return moe_layer_launch_ex(m, L, state, idx_out, w_out, nullptr, false, true, st);
}

int moe_layer_launch_ex(Model *m, int L, float *state, int *idx_out, float *w_out, float *acc_out,
                        bool partial, bool add_shared, cudaStream_t st) {
    const ModelDesc &d = m->d;
    const int H = d.hidden, M = d.moe_inter, E = d.n_experts, K = d.topk;
    const uint16_t *trunk_l = m->trunk + (int64_t)L * m->tr.n;
    Work &w = m->w;
    k_route<<<(E + kRouteWarps - 1) / kRouteWarps, 256, H * sizeof(float), st>>>(
        state, trunk_l, m->tr, H, E, w.xin, w.S, w.Bnd);
    DS4F_CUDA(cudaGetLastError());
    size_t tk_smem = (size_t)E * (8 + 8 + 4 + 4 + 4) + (size_t)H * 4;
    k_topk<<<1, 256, tk_smem, st>>>(w.S, w.Bnd, w.xin, trunk_l + m->tr.router, H, E,
                                    K, d.renorm, d.router_exact, w.idx, w.w, w.diag);
    DS4F_CUDA(cudaGetLastError());
    LayerArgs a;
    a.pool_l = m->pool + (int64_t)L * d.expert_count * m->slot.nbytes;
    a.slot_bytes = m->slot.nbytes;
    a.slot = m->slot;
    a.trunk_l = trunk_l;
    a.tr = m->tr;
    a.E = E; a.K = K; a.efirst = d.expert_first; a.ecount = d.expert_count;
    a.idx = w.idx; a.w = w.w; a.xin = w.xin; a.chain = w.chain; a.sgate = w.sgate;
    a.state = state; a.acc_out = acc_out ? acc_out : w.acc;
    a.partial = partial ? 1 : 0; a.add_shared = add_shared ? 1 : 0;
    a.slot_of = nullptr;
    if (m->cache) {             // streaming: the selections come through the slot cache
        if (stream_fetch(m, L, st)) return -1;
        a.pool_l = m->pool;
        a.slot_of = m->slot_dev;
    }
    int rc;
    if (d.fmt == DS4F_FMT_FP8 && H == 2048 && M == 512) rc = launch_chain<DS4F_FMT_FP8, 2048, 512>(a, st);
    else if (d.fmt == DS4F_FMT_MXFP4 && H == 2048 && M == 512) rc = launch_chain<DS4F_FMT_MXFP4, 2048, 512>(a, st);
    else if (d.fmt == DS4F_FMT_FP8 && H == 1024 && M == 256) rc = launch_chain<DS4F_FMT_FP8, 1024, 256>(a, st);
    else if (d.fmt == DS4F_FMT_MXFP4 && H == 1024 && M == 256) rc = launch_chain<DS4F_FMT_MXFP4, 1024, 256>(a, st);
    else { set_error("moe layer: no kernel for fmt %d H %d M %d", d.fmt, H, M); return -1; }
    if (rc) return rc;
    if (idx_out) DS4F_CUDA(cudaMemcpyAsync(idx_out, w.idx, K * sizeof(int), cudaMemcpyDeviceToDevice, st));
    if (w_out) DS4F_CUDA(cudaMemcpyAsync(w_out, w.w, K * sizeof(float), cudaMemcpyDeviceToDevice, st));
    return 0;
}

}  // namespace ds4f

// ===========================================================================
// Allocation-free variant of the one-token layer step.
//
// Some hosts cannot let this library call cudaMalloc: an engine that owns
// every byte of device memory through its own pre-sized arena (as the
// reference engine plans and caps its memory before it starts, and never
// allocates in its per-token loop), or a caller working inside a memory
// budget it must not exceed behind its own back. For them the per-call
// workspace of the layer step (normed input, router logits and bounds,
// routing, SiLU chains, shared-gate logit, counters) lives in the static
// device array below instead of a Model's cudaMalloc'd workspace; the
// caller passes the weights, the state and the outputs as device pointers.
//
// The array is a file-scope __device__ object: every GPU that loads this
// library holds kStaticScratchBytes of it until the process exits. Its
// name is not a device address in host code, so the address is looked up
// with cudaGetSymbolAddress once per device, on the first call made with
// that device current (make that first call before any stream capture).
// All calls on a device share the array and it keeps the last call's
// contents; calls that overlap on the GPU (different streams, no ordering
// between them) race on it.
// ===========================================================================
namespace ds4f {
namespace {

constexpr int kStaticMaxH = 2048, kStaticMaxM = 512, kStaticMaxE = 256, kStaticMaxK = 16;
constexpr size_t al256s(size_t n) { return (n + 255) & ~(size_t)255; }
constexpr size_t kStaticScratchBytes =
    al256s(kStaticMaxH * 4) + 2 * al256s(kStaticMaxE * 8) + 2 * al256s(kStaticMaxK * 4) +
    al256s((size_t)(kStaticMaxK + 1) * kStaticMaxM * 4) + al256s(4) + al256s(kStaticMaxH * 4) +
    al256s(16);

__device__ __align__(256) unsigned char g_static_scratch[kStaticScratchBytes];

std::mutex g_static_mu;
void *g_static_addr[64];            // per device ordinal, looked up once

}  // namespace
}  // namespace ds4f

extern "C" int ds4f_gpu_moe_layer_static(const Ds4fLayerDev *ld, float *state, int *idx,
                                         float *w, void *stream) {
    using namespace ds4f;
    DS4F_REQUIRE(ld && state, "moe_layer_static: null argument");
    const int H = ld->hidden, M = ld->moe_inter, E = ld->n_experts, K = ld->topk;
    DS4F_REQUIRE(H <= kStaticMaxH && M <= kStaticMaxM && E <= kStaticMaxE && K <= kStaticMaxK,
                 "moe_layer_static: sizes H %d, M %d, E %d, K %d exceed the static scratch "
                 "maximum (H <= %d, M <= %d, E <= %d, K <= %d)",
                 H, M, E, K, kStaticMaxH, kStaticMaxM, kStaticMaxE, kStaticMaxK);
    DS4F_REQUIRE(K >= 1 && K <= E, "moe_layer_static: topk %d of %d experts", K, E);
    DS4F_REQUIRE(ld->fmt == DS4F_FMT_FP8 || ld->fmt == DS4F_FMT_MXFP4,
                 "moe_layer_static: expert format %d (FP8 or MXFP4)", ld->fmt);
    DS4F_REQUIRE((H == 2048 && M == 512) || (H == 1024 && M == 256),
                 "moe_layer_static: kernels are built for (H, M) = (2048, 512) or (1024, 256)");
    DS4F_REQUIRE(ld->experts && ld->norm && ld->router && ld->sh_gate && ld->sh_up &&
                     ld->sh_down && ld->sh_gw,
                 "moe_layer_static: null weight pointer");
    SlotLayout slot;
    if (slot_layout(ld->fmt, H, M, &slot)) return -1;
    DS4F_REQUIRE(ld->slot_bytes >= slot.nbytes && ld->slot_bytes % 16 == 0,
                 "moe_layer_static: slot_bytes %lld (need >= %lld, multiple of 16)",
                 (long long)ld->slot_bytes, (long long)slot.nbytes);
    const void *ptrs[7] = {ld->experts, ld->norm, ld->router, ld->sh_gate,
                           ld->sh_up, ld->sh_down, ld->sh_gw};
    for (const void *p : ptrs)
        DS4F_REQUIRE(((uintptr_t)p % 16) == 0, "moe_layer_static: weights must be 16-byte aligned");

    int dev = 0;
    DS4F_CUDA(cudaGetDevice(&dev));
    DS4F_REQUIRE(dev >= 0 && dev < 64, "moe_layer_static: device ordinal %d", dev);
    unsigned char *base;
    {
        std::lock_guard<std::mutex> lk(g_static_mu);
        if (!g_static_addr[dev]) {
            void *p = nullptr;
            DS4F_CUDA(cudaGetSymbolAddress(&p, g_static_scratch));
            g_static_addr[dev] = p;
        }
        base = (unsigned char *)g_static_addr[dev];
    }
    Work wk;
    unsigned char *p = base;
    auto take = [&](size_t n) { unsigned char *r = p; p += al256s(n); return r; };
    wk.xin = (float *)take(kStaticMaxH * 4);
    wk.S = (double *)take(kStaticMaxE * 8);
    wk.Bnd = (double *)take(kStaticMaxE * 8);
    wk.idx = (int *)take(kStaticMaxK * 4);
    wk.w = (float *)take(kStaticMaxK * 4);
    wk.chain = (float *)take((size_t)(kStaticMaxK + 1) * kStaticMaxM * 4);
    wk.sgate = (float *)take(4);
    wk.acc = (float *)take(kStaticMaxH * 4);
    wk.diag = (unsigned *)take(16);

    // the bf16 trunk tensors as element offsets from the norm pointer: the
    // caller's buffers may be separate allocations, so the distance is taken
    // between addresses (CUDA's unified virtual address space), not by
    // subtracting pointers into different objects
    const uint16_t *tb = ld->norm;
    auto elems_from_norm = [&](const uint16_t *p) {
        return (int64_t)((intptr_t)(uintptr_t)p - (intptr_t)(uintptr_t)tb) / (int64_t)sizeof(uint16_t);
    };
    TrunkLayout tr;
    tr.norm = 0;
    tr.router = elems_from_norm(ld->router);
    tr.sh_gate = elems_from_norm(ld->sh_gate);
    tr.sh_up = elems_from_norm(ld->sh_up);
    tr.sh_down = elems_from_norm(ld->sh_down);
    tr.sh_gw = elems_from_norm(ld->sh_gw);
    tr.n = 0;
    cudaStream_t st = (cudaStream_t)stream;

    k_route<<<(E + kRouteWarps - 1) / kRouteWarps, 256, H * sizeof(float), st>>>(
        state, tb, tr, H, E, wk.xin, wk.S, wk.Bnd);
    DS4F_CUDA(cudaGetLastError());
    size_t tk_smem = (size_t)E * (8 + 8 + 4 + 4 + 4) + (size_t)H * 4;
    k_topk<<<1, 256, tk_smem, st>>>(wk.S, wk.Bnd, wk.xin, ld->router, H, E, K,
                                    ld->renorm, 0, wk.idx, wk.w, wk.diag);
    DS4F_CUDA(cudaGetLastError());
    LayerArgs a;
    a.pool_l = (const uint8_t *)ld->experts;
    a.slot_bytes = ld->slot_bytes;
    a.slot = slot;
    a.trunk_l = tb;
    a.tr = tr;
    a.E = E; a.K = K; a.efirst = 0; a.ecount = E;
    a.idx = wk.idx; a.w = wk.w; a.xin = wk.xin; a.chain = wk.chain; a.sgate = wk.sgate;
    a.state = state; a.acc_out = wk.acc;
    a.partial = 0; a.add_shared = 1; a.slot_of = nullptr;
    int rc;
    if (ld->fmt == DS4F_FMT_FP8 && H == 2048) rc = launch_chain<DS4F_FMT_FP8, 2048, 512>(a, st);
    else if (ld->fmt == DS4F_FMT_MXFP4 && H == 2048) rc = launch_chain<DS4F_FMT_MXFP4, 2048, 512>(a, st);
    else if (ld->fmt == DS4F_FMT_FP8) rc = launch_chain<DS4F_FMT_FP8, 1024, 256>(a, st);
    else rc = launch_chain<DS4F_FMT_MXFP4, 1024, 256>(a, st);
    if (rc) return rc;
    if (idx) DS4F_CUDA(cudaMemcpyAsync(idx, wk.idx, K * sizeof(int), cudaMemcpyDeviceToDevice, st));
    if (w) DS4F_CUDA(cudaMemcpyAsync(w, wk.w, K * sizeof(float), cudaMemcpyDeviceToDevice, st));
    return 0;
}
