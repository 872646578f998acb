// prefill.cu -- the batched prefill of one MoE layer on the tensor cores:
// ds4f_moe_step_batch (src/moe.c:1480-1707) for B tokens with the routing
// given, restated for B200.
//
//  1. RMSNorm of every token (src/moe.c:841-851 arithmetic), then the
//     activation digits (gemm.cu quantiser: 3 E4M3 digits per element).
//  2. Group the (token, selection) pairs by expert: counts, offsets, the
//     tile list (expert, first row, rows) of 64-row tiles, and each
//     selection's row in its expert's range (the reference sorts with
//     qsort, src/moe.c:1527, whose order within a group does not matter as
//     each selection keeps its own output row, :1606-1607).
//  3. Gather each selection's digit rows; grouped GEMMs: gate and up
//     (tcgen05, per expert), SiLU-mul (src/moe.c:645-649) into the chain's
//     digits, down.
//  4. Shared expert in bf16 on the tensor cores (tcgen05 kind::f16, the
//     activations as two bf16 digits hi + lo), its sigmoid gate logit.
//  5. Combine in selection order (src/moe.c:1614-1630: acc += w_j out_j,
//     then acc += sigmoid(g) shared, state += acc).
#include <cuda_bf16.h>

#include "common.cuh"
#include "gemm.cuh"
#include "model.cuh"
#include "../../include/ds4f/gpu_cuda.h"

namespace ds4f {
namespace {

constexpr int kND = 3;           // E4M3 digits per routed activation

// ---- 2. grouping -------------------------------------------------------------------
__global__ void k_count(const int *sel, int n, int first, int count, int *cnt) {
    const int i = blockIdx.x * blockDim.x + threadIdx.x;
    if (i >= n) return;
    const int e = sel[i] - first;
    if (e >= 0 && e < count) atomicAdd(cnt + e, 1);
}

// Exclusive prefix sum over one block (blockDim <= 1024); returns the total.
__device__ int block_excl_scan(int v, int *out_excl, int *sh) {
    const int lane = threadIdx.x & 31, warp = threadIdx.x >> 5, nw = (blockDim.x + 31) >> 5;
    int incl = v;
#pragma unroll
    for (int o = 1; o < 32; o <<= 1) {
        const int y = __shfl_up_sync(0xFFFFFFFFu, incl, o);
        if (lane >= o) incl += y;
    }
    if (lane == 31) sh[warp] = incl;
    __syncthreads();
    if (threadIdx.x == 0) {
        int run = 0;
        for (int k = 0; k < nw; k++) { const int t = sh[k]; sh[k] = run; run += t; }
        sh[32] = run;
    }
    __syncthreads();
    *out_excl = sh[warp] + incl - v;
    const int tot = sh[32];
    __syncthreads();
    return tot;
}

// One block of >= count threads: offsets, the 64-row tile list, totals.
__global__ void k_plan(const int *cnt, int count, int slot0, int *off, int *tiles, int *ntiles, int *nrows) {
    __shared__ int sh[33];
    const int e = threadIdx.x;
    const int c = e < count ? cnt[e] : 0, nt = (c + kGemmBN - 1) / kGemmBN;
    int o, t0;
    const int rows = block_excl_scan(c, &o, sh);
    const int tiles_n = block_excl_scan(nt, &t0, sh);
    if (e < count) {
        off[e] = o;
        for (int i = 0; i < nt; i++) {
            tiles[3 * (t0 + i)] = slot0 + e;
            tiles[3 * (t0 + i) + 1] = o + kGemmBN * i;
            tiles[3 * (t0 + i) + 2] = min(kGemmBN, c - kGemmBN * i);
        }
    }
    if (e == 0) { *ntiles = tiles_n; *nrows = rows; }
}

// Each in-shard selection takes the next row of its expert's range:
// pos[selection] = row. The order of rows inside an expert's range does not
// change any result (every output column of the tensor-core GEMM depends on
// its own row only; the combine reads rows by pos), as in the reference
// whose qsort leaves it open (src/moe.c:1527).
__global__ void k_place(const int *sel, int n, int first, int count, const int *off, int *fill, int *pos) {
    const int i = blockIdx.x * blockDim.x + threadIdx.x;
    if (i >= n) return;
    const int e = sel[i] - first;
    if (e < 0 || e >= count) return;
    pos[i] = off[e] + atomicAdd(fill + e, 1);
}

// ---- 1. the token's front end ------------------------------------------------------
// One block per token, one warp per 128-column block (4 columns per lane):
// RMSNorm (src/moe.c:841-851: double sum of squares, x / r * w), the E4M3
// digits and scale of every block written straight into the row of each of
// the token's in-shard selections (its expert's range of the grouped B
// planes), and, for the shared expert, the bf16 (hi, lo) digits and the
// shared_expert_gate logit (fp32 products of the bf16 matvec,
// src/kernels.c:84-103).
__global__ void k_front(const float *st, const uint16_t *nw, int H, const int *sel, int K, int first, int count,
                        const int *pos, uint8_t *Xg, float *sxg, int64_t rows_cap, uint16_t *Xb, int64_t xb_plane,
                        const uint16_t *gw, float *sg) {
    __shared__ double part[32];
    __shared__ float gpart[32];
    __shared__ int rows[16];
    const int t = blockIdx.x, warp = threadIdx.x >> 5, lane = threadIdx.x & 31, nwp = blockDim.x >> 5;
    const int c = warp * 128 + 4 * lane;
    const int64_t off = (int64_t)t * H + c;
    if (threadIdx.x < K) {
        const int i = t * K + threadIdx.x, e = sel ? sel[i] - first : -1;
        rows[threadIdx.x] = (e >= 0 && e < count) ? pos[i] : -1;
    }
    const float4 v = *(const float4 *)(st + off);
    double ss = __dadd_rn(__dadd_rn(__dmul_rn((double)v.x, (double)v.x), __dmul_rn((double)v.y, (double)v.y)),
                          __dadd_rn(__dmul_rn((double)v.z, (double)v.z), __dmul_rn((double)v.w, (double)v.w)));
    ss = warp_sum_d(ss);
    if (lane == 0) part[warp] = ss;
    __syncthreads();
    double tot = 0.0;
    for (int k = 0; k < nwp; k++) tot = __dadd_rn(tot, part[k]);
    const float r = __fsqrt_rn(__fadd_rn(__double2float_rn(__ddiv_rn(tot, (double)H)), 1e-6f));
    const uint2 nw4 = *(const uint2 *)(nw + c);
    const float4 x = make_float4(__fmul_rn(__fdiv_rn(v.x, r), __uint_as_float(nw4.x << 16)),
                                 __fmul_rn(__fdiv_rn(v.y, r), __uint_as_float(nw4.x & 0xFFFF0000u)),
                                 __fmul_rn(__fdiv_rn(v.z, r), __uint_as_float(nw4.y << 16)),
                                 __fmul_rn(__fdiv_rn(v.w, r), __uint_as_float(nw4.y & 0xFFFF0000u)));
    uint32_t wd[3];
    const float s = quant_block_words(x, kND, wd);
    for (int j = 0; j < K; j++) {
        const int p = rows[j];
        if (p < 0) continue;
#pragma unroll
        for (int d = 0; d < kND; d++) *(uint32_t *)(Xg + ((int64_t)d * rows_cap + p) * H + c) = wd[d];
        if (lane == 0) sxg[(int64_t)p * (H / 128) + warp] = s;
    }
    if (Xb) {
        uint32_t hi[2], lo[2];
        const float xs[4] = {x.x, x.y, x.z, x.w};
#pragma unroll
        for (int i = 0; i < 4; i += 2) {
            const __nv_bfloat16 h0 = __float2bfloat16_rn(xs[i]), h1 = __float2bfloat16_rn(xs[i + 1]);
            const __nv_bfloat16 l0 = __float2bfloat16_rn(__fsub_rn(xs[i], __bfloat162float(h0)));
            const __nv_bfloat16 l1 = __float2bfloat16_rn(__fsub_rn(xs[i + 1], __bfloat162float(h1)));
            hi[i >> 1] = __bfloat16_as_ushort(h0) | ((uint32_t)__bfloat16_as_ushort(h1) << 16);
            lo[i >> 1] = __bfloat16_as_ushort(l0) | ((uint32_t)__bfloat16_as_ushort(l1) << 16);
        }
        *(uint2 *)(Xb + off) = make_uint2(hi[0], hi[1]);
        *(uint2 *)(Xb + xb_plane + off) = make_uint2(lo[0], lo[1]);
        const uint2 g4 = *(const uint2 *)(gw + c);
        float a = __fmul_rn(__uint_as_float(g4.x << 16), x.x);
        a = fmaf(__uint_as_float(g4.x & 0xFFFF0000u), x.y, a);
        a = fmaf(__uint_as_float(g4.y << 16), x.z, a);
        a = fmaf(__uint_as_float(g4.y & 0xFFFF0000u), x.w, a);
        a = warp_sum(a);
        if (lane == 0) gpart[warp] = a;
        __syncthreads();
        if (threadIdx.x == 0) {
            float sum = 0.f;
            for (int k = 0; k < nwp; k++) sum += gpart[k];
            sg[t] = sum;
        }
    }
}

// ---- 3. SiLU-mul into the chain's digits --------------------------------------------
// GU [rows][2M] (gate, up) -> Cq [ND][rows_cap][M], sc [rows][M/128]
__global__ void k_silu_digits(const float *GU, int M, const int *nrows, uint8_t *Cq, float *sc, int rows_cap) {
    const int nb = M / 128;
    const int64_t blk = ((int64_t)blockIdx.x * blockDim.x + threadIdx.x) >> 5;
    const int lane = threadIdx.x & 31;
    const int p = (int)(blk / nb), b = (int)(blk % nb);
    if (p >= *nrows) return;
    const float *g = GU + (int64_t)p * 2 * M + b * 128 + 4 * lane;
    const float4 gv = *(const float4 *)g, uv = *(const float4 *)(g + M);
    const float4 c = make_float4(silu_mul(gv.x, uv.x), silu_mul(gv.y, uv.y), silu_mul(gv.z, uv.z),
                                 silu_mul(gv.w, uv.w));
    const float s = quant_block_digits(c, kND, Cq, (int64_t)rows_cap * M, (int64_t)p * M + b * 128 + 4 * lane);
    if (lane == 0) sc[blk] = s;
}

// ---- 4. shared expert ----------------------------------------------------------------
// Two bf16 digits: hi = bf16(x), lo = bf16(x - hi) (round to nearest even),
// planes q[0] = hi, q[1] = lo, each n elements.
__device__ __forceinline__ void bf16_digits(float x, uint16_t *q, int64_t n, int64_t i) {
    const __nv_bfloat16 hi = __float2bfloat16_rn(x);
    const __nv_bfloat16 lo = __float2bfloat16_rn(__fsub_rn(x, __bfloat162float(hi)));
    q[i] = __bfloat16_as_ushort(hi);
    q[n + i] = __bfloat16_as_ushort(lo);
}
// GS [T][2M] -> chain digits [2][T][M]
__global__ void k_silu_bf16_digits(const float *GS, int M, int64_t T, uint16_t *q) {
    const int64_t i = (int64_t)blockIdx.x * blockDim.x + threadIdx.x;
    if (i >= T * M) return;
    const int64_t t = i / M, m = i % M;
    bf16_digits(silu_mul(GS[t * 2 * M + m], GS[t * 2 * M + M + m]), q, T * M, i);
}
// ---- 5. combine ------------------------------------------------------------------------
// One block per token: its in-shard selections (j order, zero weights
// skipped) staged in shared memory, then 4 output columns per thread.
__global__ void k_combine(float *states, float *acc_out, const float *O, const float *OS, const float *sg,
                          const int *sel, const float *w, const int *pos, int first, int count, int K, int H) {
    __shared__ int prow[16];
    __shared__ float pw[16];
    __shared__ int np;
    const int t = blockIdx.x;
    if (threadIdx.x == 0) {
        int n = 0;
        for (int j = 0; j < K && sel; j++) {
            const int i = t * K + j, e = sel[i] - first;
            if (e < 0 || e >= count || w[i] == 0.0f) continue;
            prow[n] = pos[i];
            pw[n] = w[i];
            n++;
        }
        np = n;
    }
    __syncthreads();
    const float sig = OS ? sigmoid_ref(sg[t]) : 0.f;
    const int n = np;
    for (int c = threadIdx.x; c < H / 4; c += blockDim.x) {
        float4 acc = make_float4(0.f, 0.f, 0.f, 0.f);
#pragma unroll 4
        for (int k = 0; k < n; k++) {
            const float4 o = *(const float4 *)(O + (int64_t)prow[k] * H + 4 * c);
            const float wk = pw[k];
            acc.x = __fadd_rn(acc.x, __fmul_rn(wk, o.x));
            acc.y = __fadd_rn(acc.y, __fmul_rn(wk, o.y));
            acc.z = __fadd_rn(acc.z, __fmul_rn(wk, o.z));
            acc.w = __fadd_rn(acc.w, __fmul_rn(wk, o.w));
        }
        if (OS) {
            const float4 so = *(const float4 *)(OS + (int64_t)t * H + 4 * c);
            acc.x = __fadd_rn(acc.x, __fmul_rn(sig, so.x));
            acc.y = __fadd_rn(acc.y, __fmul_rn(sig, so.y));
            acc.z = __fadd_rn(acc.z, __fmul_rn(sig, so.z));
            acc.w = __fadd_rn(acc.w, __fmul_rn(sig, so.w));
        }
        if (acc_out) {                       // expert-parallel partial: acc only
            *((float4 *)(acc_out + (int64_t)t * H) + c) = acc;
            continue;
        }
        float4 *st = (float4 *)(states + (int64_t)t * H) + c;
        float4 v = *st;
        v.x = __fadd_rn(v.x, acc.x);
        v.y = __fadd_rn(v.y, acc.y);
        v.z = __fadd_rn(v.z, acc.z);
        v.w = __fadd_rn(v.w, acc.w);
        *st = v;
    }
}

// ---- MXFP4 pools: the exact FP8 copy ---------------------------------------------------
// ---- workspace -----------------------------------------------------------------------
struct PfWs {
    int *cnt, *off, *tiles, *ntiles, *nrows, *pos;
    uint8_t *Xg; float *sxg; float *GU; uint8_t *Cq; float *sc; float *O;
    uint16_t *Xb; float *GS; uint16_t *Cb; float *OS; float *sg;
    unsigned *err;
    // batched decode: the routing computed on the device
    float *rxin; double *rS, *rB; int *ridx; float *rw;
    int tiles_max;
};

size_t al(size_t n) { return (n + 255) / 256 * 256; }

int pf_workspace(Model *m, int T, PfWs *w) {
    const int H = m->d.hidden, M = m->d.moe_inter, K = m->d.topk, count = m->d.expert_count;
    const int E = m->d.n_experts;
    const int64_t R = (int64_t)T * K;
    const int tiles_max = (int)(R / kGemmBN) + count;
    // the error word first: its place does not depend on T, so calls with
    // different token counts share it
    const size_t sizes[] = {
        al(4), al(count * 4), al(count * 4), al((size_t)tiles_max * 12), al(4), al(4), al(R * 4),
        al((size_t)kND * R * H), al((size_t)R * (H / 128) * 4), al((size_t)R * 2 * M * 4),
        al((size_t)kND * R * M), al((size_t)R * (M / 128) * 4), al((size_t)R * H * 4),
        al((size_t)2 * T * H * 2), al((size_t)T * 2 * M * 4), al((size_t)2 * T * M * 2),
        al((size_t)T * H * 4), al((size_t)T * 4), al(4),
        al((size_t)T * H * 4), al((size_t)T * E * 8), al((size_t)T * E * 8), al(R * 4), al(R * 4)};
    size_t total = 0;
    bool fresh = false;
    for (size_t s : sizes) total += s;
    if (total > m->pf_bytes) {
        if (m->pf_ws) { DS4F_CUDA(cudaFree(m->pf_ws)); m->pf_ws = nullptr; m->pf_bytes = 0; }
        size_t fre = 0, tot = 0;
        DS4F_CUDA(cudaMemGetInfo(&fre, &tot));
        DS4F_REQUIRE((double)total <= 0.95 * (double)fre,
                     "prefill: workspace of %.2f GB for %d tokens, %.2f GB free", total / 1e9, T, fre / 1e9);
        DS4F_CUDA(cudaMalloc(&m->pf_ws, total));
        m->pf_bytes = total;
        fresh = true;
    }
    uint8_t *p = (uint8_t *)m->pf_ws;
    int k = 0;
    auto take = [&]() { uint8_t *r = p; p += sizes[k++]; return r; };
    w->err = (unsigned *)take();
    w->cnt = (int *)take(); w->off = (int *)take(); w->tiles = (int *)take(); w->ntiles = (int *)take();
    w->nrows = (int *)take(); w->pos = (int *)take();
    w->Xg = take(); w->sxg = (float *)take(); w->GU = (float *)take(); w->Cq = take(); w->sc = (float *)take();
    w->O = (float *)take(); w->Xb = (uint16_t *)take(); w->GS = (float *)take(); w->Cb = (uint16_t *)take();
    w->OS = (float *)take(); w->sg = (float *)take(); take();
    w->rxin = (float *)take(); w->rS = (double *)take(); w->rB = (double *)take(); w->ridx = (int *)take();
    w->rw = (float *)take();
    w->tiles_max = tiles_max;
    if (fresh) DS4F_CUDA(cudaMemset(w->err, 0, 4));
    return 0;
}

// Asynchronous steps (the expert-parallel partial calls, made once per layer
// between collectives) do not synchronise: each copies the pipeline error
// word to pinned host memory after its kernels, and a later call reports
// what an earlier step left there (then clears it).
int async_begin(Model *m, const PfWs &ws, cudaStream_t st) {
    if (!m->pf_err_h) {
        DS4F_CUDA(cudaHostAlloc((void **)&m->pf_err_h, 4, cudaHostAllocDefault));
        *m->pf_err_h = 0;
    }
    const unsigned h = *(volatile unsigned *)m->pf_err_h;
    if (h) {
        *m->pf_err_h = 0;
        DS4F_CUDA(cudaMemsetAsync(ws.err, 0, 4, st));
        set_error("prefill: a tensor-core pipeline wait gave up (code %u) in an earlier asynchronous step", h);
        return -1;
    }
    return 0;
}
int async_end(Model *m, const PfWs &ws, cudaStream_t st) {
    DS4F_CUDA(cudaMemcpyAsync(m->pf_err_h, ws.err, 4, cudaMemcpyDeviceToHost, st));
    return 0;
}

}  // namespace

int prefill_layer(Model *m, int L, float *states, int T, const int *sel, const float *w, cudaStream_t st,
                  bool first_layer, bool last_layer, float *acc_out, bool add_shared) {
    DS4F_REQUIRE(T > 0 && L >= 0 && L < m->d.n_layers, "prefill: layer %d / tokens %d", L, T);
    DS4F_REQUIRE(!m->cache, "prefill: not available for a streaming model (its experts are not resident)");
    // the tensor core reads the pool itself: FP8 bytes (their fp32 block
    // scales applied in the epilogue) or MXFP4 nibbles (their E8M0 scales
    // applied by the block-scaled MMA)
    const bool mx = m->d.fmt == DS4F_FMT_MXFP4;
    const uint8_t *pool = m->pool;
    const SlotLayout &sl = m->slot;
    const int H = m->d.hidden, M = m->d.moe_inter, K = m->d.topk;
    const int first = m->d.expert_first, count = m->d.expert_count;
    DS4F_REQUIRE(count <= 1024, "prefill: at most 1024 experts per shard");
    DS4F_REQUIRE(H % 128 == 0 && H <= 4096 && M % 128 == 0 && K <= 16,
                 "prefill: hidden %d / moe_inter %d must be multiples of 128 (hidden <= 4096), top-k %d <= 16", H, M, K);
    PfWs ws;
    if (pf_workspace(m, T, &ws)) return -1;
    const int64_t R = (int64_t)T * K;
    const uint16_t *tl = m->trunk + (int64_t)L * m->tr.n;
    const int64_t total_slots = (int64_t)m->d.n_layers * count;

    // sel == nullptr: the shared expert alone (the expert-parallel prefill's
    // own tokens; their routed selections run on the experts' ranks)
    const bool routed = sel != nullptr;
    DS4F_REQUIRE(routed || add_shared, "prefill: neither routed selections nor the shared expert");
    if (first_layer) DS4F_CUDA(cudaMemsetAsync(ws.err, 0, 4, st));
    // 1: grouping (it depends on the routing only)
    if (routed) {
    DS4F_CUDA(cudaMemsetAsync(ws.cnt, 0, count * 4, st));
    k_count<<<(unsigned)((R + 255) / 256), 256, 0, st>>>(sel, (int)R, first, count, ws.cnt);
    k_plan<<<1, ((count + 31) / 32) * 32, 0, st>>>(ws.cnt, count, L * count, ws.off, ws.tiles, ws.ntiles,
                                                   ws.nrows);
    DS4F_CUDA(cudaMemsetAsync(ws.cnt, 0, count * 4, st));       // now the per-expert fill counters
    k_place<<<(unsigned)((R + 255) / 256), 256, 0, st>>>(sel, (int)R, first, count, ws.off, ws.cnt, ws.pos);
    }
    // 2: RMSNorm, digits into the grouped rows, the shared expert's inputs
    k_front<<<T, 32 * (H / 128), 0, st>>>(states, tl + m->tr.norm, H, sel, K, first, count, ws.pos, ws.Xg, ws.sxg,
                                           R, add_shared ? ws.Xb : nullptr, (int64_t)T * H, tl + m->tr.sh_gw,
                                           ws.sg);
    // 3: gate, up, SiLU digits, down
    if (routed) {
    {   // gate and up in one launch
        GemmArgs g{};
        g.sX = ws.sxg; g.Y = ws.GU; g.ldy = 2 * M; g.ycol0 = 0; g.ycol2 = M;
        g.R = M; g.C = H; g.tiles = ws.tiles; g.ntiles = ws.ntiles; g.err = ws.err;
        if (mx) {
            g.sfa = pool + sl.rel_s[0];
            g.sfa2 = pool + sl.rel_s[1];
            g.sfa_slot = sl.nbytes;
            if (gemm_launch_mx<kND>(pool + sl.rel_v[0], total_slots, sl.nbytes, ws.Xg, R, g, ws.tiles_max, st,
                                    pool + sl.rel_v[1]))
                return -1;
        } else {
            g.sW = (const float *)(pool + sl.rel_s[0]);
            g.sW2 = (const float *)(pool + sl.rel_s[1]);
            g.sw_slot = sl.nbytes / 4;
            if (gemm_launch<kND, false>(pool + sl.rel_v[0], total_slots, sl.nbytes, ws.Xg, R, g,
                                        ws.tiles_max, st, pool + sl.rel_v[1]))
                return -1;
        }
    }
    k_silu_digits<<<(unsigned)((R * (M / 128) * 32 + 255) / 256), 256, 0, st>>>(ws.GU, M, ws.nrows, ws.Cq,
                                                                                ws.sc, (int)R);
    {
        GemmArgs g{};
        g.sX = ws.sc; g.Y = ws.O; g.ldy = H; g.ycol0 = 0;
        g.R = H; g.C = M; g.tiles = ws.tiles; g.ntiles = ws.ntiles; g.err = ws.err;
        if (mx) {
            g.sfa = pool + sl.rel_s[2];
            g.sfa_slot = sl.nbytes;
            if (gemm_launch_mx<kND>(pool + sl.rel_v[2], total_slots, sl.nbytes, ws.Cq, R, g, ws.tiles_max, st))
                return -1;
        } else {
            g.sW = (const float *)(pool + sl.rel_s[2]);
            g.sw_slot = sl.nbytes / 4;
            if (gemm_launch<kND, false>(pool + sl.rel_v[2], total_slots, sl.nbytes, ws.Cq, R, g, ws.tiles_max,
                                        st))
                return -1;
        }
    }
    }
    // 4: shared expert
    if (add_shared) {
    {   // shared gate and up in one launch
        GemmArgs g{};
        g.Y = ws.GS; g.ldy = 2 * M; g.ycol0 = 0; g.ycol2 = M; g.R = M; g.C = H; g.N = T; g.err = ws.err;
        if (bf16_gemm_launch(tl + m->tr.sh_gate, ws.Xb, g, st, tl + m->tr.sh_up)) return -1;
    }
    k_silu_bf16_digits<<<(unsigned)(((int64_t)T * M + 255) / 256), 256, 0, st>>>(ws.GS, M, T, ws.Cb);
    {
        GemmArgs g{};
        g.Y = ws.OS; g.ldy = H; g.ycol0 = 0; g.R = H; g.C = M; g.N = T; g.err = ws.err;
        if (bf16_gemm_launch(tl + m->tr.sh_down, ws.Cb, g, st)) return -1;
    }
    }
    // 5
    k_combine<<<T, 256, 0, st>>>(states, acc_out, ws.O, add_shared ? ws.OS : nullptr, ws.sg, sel, w, ws.pos,
                                 first, count, K, H);
    DS4F_CUDA(cudaGetLastError());
    if (last_layer) {
        // the pipeline waits of every layer since first_layer report here
        unsigned h = 0;
        DS4F_CUDA(cudaMemcpyAsync(&h, ws.err, 4, cudaMemcpyDeviceToHost, st));
        DS4F_CUDA(cudaStreamSynchronize(st));
        DS4F_REQUIRE(h == 0, "prefill: a tensor-core pipeline wait gave up (code %u)", h);
    }
    return 0;
}

int prefill_pre_size(Model *m, int T) {
    PfWs ws;
    return pf_workspace(m, T, &ws);
}

int prefill_check(Model *m, cudaStream_t st) {
    DS4F_REQUIRE(m->pf_ws, "prefill: no workspace");
    PfWs ws;
    if (pf_workspace(m, 1, &ws)) return -1;          // the current layout, no regrowth
    unsigned h = 0;
    DS4F_CUDA(cudaMemcpyAsync(&h, ws.err, 4, cudaMemcpyDeviceToHost, st));
    DS4F_CUDA(cudaStreamSynchronize(st));
    if (h) DS4F_CUDA(cudaMemsetAsync(ws.err, 0, 4, st));
    DS4F_REQUIRE(h == 0, "prefill: a tensor-core pipeline wait gave up (code %u)", h);
    return 0;
}

// Batched decode of one layer: the certified router and top-K of every
// token on the device (the per-token route of src/main.c:1014-1088 and
// ds4f_topk, src/moe.c:531-561, B at once), then the grouped chain of the
// batched step (ds4f_moe_step_batch, src/moe.c:1480-1707) on the tensor
// cores with that routing. idx / w (device, may be null) receive the routing.
// async: no synchronisation (errors reported by a later call, async_begin);
// otherwise first_layer / last_layer as in prefill_layer.
int decode_batch_layer(Model *m, int L, float *states, int B, int *idx, float *w, cudaStream_t st,
                       bool first_layer, bool last_layer, float *acc_out, bool add_shared, bool async) {
    DS4F_REQUIRE(B > 0 && L >= 0 && L < m->d.n_layers, "decode batch: layer %d / tokens %d", L, B);
    const int K = m->d.topk;
    PfWs ws;
    if (pf_workspace(m, B, &ws)) return -1;
    if (async && async_begin(m, ws, st)) return -1;
    if (route_batch_launch(m, L, states, B, ws.rxin, ws.rS, ws.rB, ws.ridx, ws.rw, st)) return -1;
    if (idx) DS4F_CUDA(cudaMemcpyAsync(idx, ws.ridx, (size_t)B * K * 4, cudaMemcpyDeviceToDevice, st));
    if (w) DS4F_CUDA(cudaMemcpyAsync(w, ws.rw, (size_t)B * K * 4, cudaMemcpyDeviceToDevice, st));
    if (prefill_layer(m, L, states, B, ws.ridx, ws.rw, st, async ? false : first_layer, async ? false : last_layer,
                      acc_out, add_shared))
        return -1;
    return async ? async_end(m, ws, st) : 0;
}

}  // namespace ds4f

extern "C" {

int ds4f_gpu_moe_layer_batch_dev(Ds4fGpuModel *h, int layer, float *states_dev, int B, int *idx_dev,
                                 float *w_dev, void *stream) {
    DS4F_REQUIRE(h && states_dev, "moe_layer_batch: null argument");
    DS4F_REQUIRE(!h->m.cache, "moe_layer_batch: not available for a streaming model (its experts are not resident)");
    return ds4f::decode_batch_layer(&h->m, layer, states_dev, B, idx_dev, w_dev, (cudaStream_t)stream, true, true,
                                    nullptr, true, false);
}

int ds4f_gpu_moe_layer_batch_partial_dev(Ds4fGpuModel *h, int layer, const float *states_dev, int B,
                                         float *acc_dev, int add_shared, void *stream) {
    DS4F_REQUIRE(h && states_dev && acc_dev, "moe_layer_batch_partial: null argument");
    DS4F_REQUIRE(!h->m.cache, "moe_layer_batch_partial: not available for a streaming model (its experts are not resident)");
    return ds4f::decode_batch_layer(&h->m, layer, const_cast<float *>(states_dev), B, nullptr, nullptr,
                                    (cudaStream_t)stream, false, false, acc_dev, add_shared != 0, true);
}

// The first step runs eagerly (it sizes the workspace, builds an MXFP4
// pool's FP8 copy and sets the kernels' attributes); the later steps replay
// one CUDA graph of a whole step (every layer's launches), kept while the
// states buffer, the batch and the workspace stay the same. One pipeline
// check after the last step.
// The work runs on the model's own stream (a capture needs a stream of
// its own), ordered after and before the caller's stream.
static int stack_batch(ds4f::Model *m, float *states_dev, int B, int n_steps, cudaStream_t st) {
    const int NL = m->d.n_layers;
    ds4f::PfWs ws;
    if (ds4f::pf_workspace(m, B, &ws)) return -1;
    DS4F_CUDA(cudaMemsetAsync(ws.err, 0, 4, st));
    int s = 0;
    const bool fresh = !m->bgraph || m->bgraph_state != states_dev || m->bgraph_B != B || m->bgraph_ws != m->pf_ws;
    if (fresh) {
        for (int L = 0; L < NL; L++)
            if (ds4f::decode_batch_layer(m, L, states_dev, B, nullptr, nullptr, st, false, false, nullptr, true,
                                         false))
                return -1;
        s = 1;
        if (s < n_steps) {
            if (m->bgraph) { cudaGraphExecDestroy(m->bgraph); m->bgraph = nullptr; }
            if (ds4f::pf_workspace(m, B, &ws)) return -1;     // the eager step left it sized
            cudaGraph_t g;
            DS4F_CUDA(cudaStreamBeginCapture(st, cudaStreamCaptureModeThreadLocal));
            int rc = 0;
            for (int L = 0; L < NL && !rc; L++)
                rc = ds4f::decode_batch_layer(m, L, states_dev, B, nullptr, nullptr, st, false, false, nullptr, true,
                                              false);
            cudaError_t e = cudaStreamEndCapture(st, &g);
            if (rc) { if (e == cudaSuccess) cudaGraphDestroy(g); return -1; }
            DS4F_CUDA(e);
            e = cudaGraphInstantiate(&m->bgraph, g, 0);
            cudaGraphDestroy(g);
            DS4F_CUDA(e);
            m->bgraph_state = states_dev;
            m->bgraph_B = B;
            m->bgraph_ws = m->pf_ws;
        }
    }
    for (; s < n_steps; s++) DS4F_CUDA(cudaGraphLaunch(m->bgraph, st));
    unsigned e = 0;
    DS4F_CUDA(cudaMemcpyAsync(&e, ws.err, 4, cudaMemcpyDeviceToHost, st));
    DS4F_CUDA(cudaStreamSynchronize(st));
    DS4F_REQUIRE(e == 0, "moe_stack_batch: a tensor-core pipeline wait gave up (code %u)", e);
    return 0;
}

int ds4f_gpu_moe_stack_batch_dev(Ds4fGpuModel *h, float *states_dev, int B, int n_steps, void *stream) {
    DS4F_REQUIRE(h && states_dev && n_steps > 0 && B > 0, "moe_stack_batch: bad arguments");
    DS4F_REQUIRE(!h->m.cache, "moe_stack_batch: not available for a streaming model (its experts are not resident)");
    return ds4f::on_model_stream(h->m, stream,
                                 [&](cudaStream_t st) { return stack_batch(&h->m, states_dev, B, n_steps, st); });
}

int ds4f_gpu_moe_prefill(Ds4fGpuModel *h, int layer, float *states_dev, int T, const int *sel_dev,
                         const float *w_dev, void *stream) {
    DS4F_REQUIRE(h && states_dev && sel_dev && w_dev, "moe_prefill: null argument");
    return ds4f::prefill_layer(&h->m, layer, states_dev, T, sel_dev, w_dev, (cudaStream_t)stream, true, true,
                               nullptr, true);
}

int ds4f_gpu_prefill(Ds4fGpuModel *h, float *states_dev, int T, const int *sel_dev, const float *w_dev,
                     void *stream) {
    DS4F_REQUIRE(h && states_dev && sel_dev && w_dev, "prefill: null argument");
    const ds4f::Model &m = h->m;
    const int64_t per = (int64_t)T * m.d.topk;
    // one synchronisation (and error check) for the whole stack
    for (int L = 0; L < m.d.n_layers; L++)
        if (ds4f::prefill_layer(&h->m, L, states_dev, T, sel_dev + L * per, w_dev + L * per, (cudaStream_t)stream,
                                L == 0, L == m.d.n_layers - 1, nullptr, true))
            return -1;
    return 0;
}

int ds4f_gpu_moe_prefill_partial(Ds4fGpuModel *h, int layer, const float *states_dev, int T, const int *sel_dev,
                                 const float *w_dev, float *acc_dev, int add_shared, void *stream) {
    DS4F_REQUIRE(h && states_dev && sel_dev && w_dev && acc_dev && T > 0, "moe_prefill_partial: bad arguments");
    ds4f::Model *m = &h->m;
    cudaStream_t st = (cudaStream_t)stream;
    ds4f::PfWs ws;
    if (ds4f::pf_workspace(m, T, &ws) || ds4f::async_begin(m, ws, st)) return -1;
    if (ds4f::prefill_layer(m, layer, const_cast<float *>(states_dev), T, sel_dev, w_dev, st, false, false, acc_dev,
                            add_shared != 0))
        return -1;
    return ds4f::async_end(m, ws, st);
}

}  // extern "C"
