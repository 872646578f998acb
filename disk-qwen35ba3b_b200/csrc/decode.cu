// decode.cu -- persistent decode kernel: every layer of a decode step (and
// several steps) for one token in ONE cooperative launch, one CTA per SM.
//
// Per layer, each CTA c of G owns a static slice of every phase:
//   router rows   [c E/G, (c+1) E/G)     shared gate/up rows [c M/G, ...)
//   routed (selection, row) pairs [c K M/G, ...)    output rows [c H/G, ...)
// and runs
//   (A) wait for the layer's input state        (flag: state counter)
//   (B) RMSNorm of the full state into shared memory
//   (C) its router rows: S, bound (certified logits, see moe.cu); its shared
//       gate/up rows -> shared SiLU chain; publish      (flag: route counter)
//   (E) TMA-prefetch the next layer's router and shared gate/up rows
//   (F) wait for all router rows; top-k + softmax + renorm (every CTA, same
//       bits); exact reference-order logits for near-ties
//   (G) TMA the selected experts' gate/up rows (2-stage ring) and down rows
//   (H) gate/up dots + SiLU-mul -> chains; publish      (flag: chain counter)
//   (J) down rows (routed + shared, prefetched) -> selection-order combine,
//       shared gate, residual on its output rows        (flag: state counter)
//   (K) TMA-prefetch the next layer's shared down rows
// Weights never round-trip through the host; the router and shared-expert
// bytes stream during the routing bubble, the routed bytes right after it.
// Reference: ds4f_moe_step (src/moe.c:948-1456) and its router call site
// (src/main.c:1014-1088), per layer, for the decode loop (src/main.c:848).
//
// Waits are bounded (flag spins and mbarrier waits give up after ~2 s,
// record an error code and drain this CTA's copies before returning).
// Data written by other CTAs is read with ld.global.cg (L2), never through
// the incoherent L1 / read-only paths.
#include "model.cuh"

#include <algorithm>

namespace ds4f {

namespace {

constexpr int kThreads = 512;
constexpr int kWarps = kThreads / 32;
constexpr int kGmin = 128;                 // smem is sized for grids >= this
constexpr int kStagePairs = 8;
constexpr long kSpinLimit = 1L << 25;      // x ~64 ns sleep: ~2 s
constexpr double kU = 5.9604644775390625e-08;

// ---- PTX helpers ------------------------------------------------------------
__device__ __forceinline__ uint32_t sa(const void *p) {
    return (uint32_t)__cvta_generic_to_shared(p);
}
__device__ __forceinline__ void mbar_init(uint64_t *b, uint32_t n) {
    asm volatile("mbarrier.init.shared::cta.b64 [%0], %1;" ::"r"(sa(b)), "r"(n) : "memory");
}
__device__ __forceinline__ void mbar_expect(uint64_t *b, uint32_t bytes) {
    asm volatile("mbarrier.arrive.expect_tx.shared::cta.b64 _, [%0], %1;" ::"r"(sa(b)),
                 "r"(bytes) : "memory");
}
__device__ __forceinline__ bool mbar_test(uint64_t *b, uint32_t parity) {
    uint32_t ok;
    asm volatile(
        "{ .reg .pred p; mbarrier.try_wait.parity.shared::cta.b64 p, [%1], %2; "
        "selp.u32 %0, 1, 0, p; }"
        : "=r"(ok) : "r"(sa(b)), "r"(parity) : "memory");
    return ok != 0;
}
// global -> this CTA's shared memory, completion counted on mbarrier b
__device__ __forceinline__ void bulk(void *dst, const void *src, uint32_t bytes, uint64_t *b) {
    asm volatile(
        "cp.async.bulk.shared::cluster.global.mbarrier::complete_tx::bytes [%0], [%1], %2, [%3];"
        ::"r"(sa(dst)), "l"(src), "r"(bytes), "r"(sa(b)) : "memory");
}
__device__ __forceinline__ void fence_async() {
    asm volatile("fence.proxy.async.shared::cta;" ::: "memory");
}
// 16-byte shared-memory load (asm volatile: not hoisted across the
// mbarrier waits that publish the TMA-written bytes)
__device__ __forceinline__ uint4 lds16(const void *p) {
    uint4 r;
    asm volatile("ld.shared.v4.u32 {%0,%1,%2,%3}, [%4];"
                 : "=r"(r.x), "=r"(r.y), "=r"(r.z), "=r"(r.w) : "r"(sa(p)) : "memory");
    return r;
}

// ---- shapes -------------------------------------------------------------------
template <int FMT, int H, int M>
struct Shape {
    static constexpr int row_b = FMT == DS4F_FMT_FP8 ? H : H / 2;     // gate/up row bytes
    static constexpr int drow_b = FMT == DS4F_FMT_FP8 ? M : M / 2;    // down row bytes
    static constexpr int ce = FMT == DS4F_FMT_FP8 ? 16 : 32;          // elements / 16 B
    static constexpr int gq = H / ce;                                  // chunks per gate row
    static constexpr int gk = gq / 32;                                 // chunks per lane
    static constexpr int dq = M / ce;                                  // chunks per down row
    static constexpr int dlpr = dq < 32 ? dq : 32;                     // lanes per down row
    static constexpr int dk = dq / dlpr;
    static constexpr int bq = M / 8;                                   // bf16 down chunks
    static constexpr int blpr = bq < 32 ? bq : 32;
    static constexpr int bk = bq / blpr;
    // FP8: whole scale blocks; MXFP4: E8M0 per 32 along K, per row
    static constexpr int gsc_b = FMT == DS4F_FMT_FP8 ? (M / 128) * (H / 128) * 4 : H / 32;
    static constexpr int dsc_b = FMT == DS4F_FMT_FP8 ? (H / 128) * (M / 128) * 4 : M / 32;
    static_assert(gk >= 1 && gq % 32 == 0, "gate/up rows must span the warp");
};

template <int FMT, int H, int M, int E, int K>
struct Smem {
    using S = Shape<FMT, H, M>;
    static constexpr int RT = (E + kGmin - 1) / kGmin;          // router rows per CTA
    static constexpr int SG = (M + kGmin - 1) / kGmin;          // shared rows per CTA
    static constexpr int RR = (H + kGmin - 1) / kGmin;          // output rows per CTA
    static constexpr int GSC_SEG = FMT == DS4F_FMT_FP8 ? S::gsc_b : kStagePairs * S::gsc_b;
    static constexpr int DSC = FMT == DS4F_FMT_FP8 ? S::dsc_b : (RR * S::dsc_b + 48 + 15) / 16 * 16;
    // byte offsets (16-byte aligned)
    static constexpr int a16(int n) { return (n + 15) / 16 * 16; }
    static constexpr int o_bar = 0;                                   // 8 mbarriers
    static constexpr int o_xin = 128;
    static constexpr int o_rt = o_xin + a16(H * 4);
    static constexpr int o_sgu = o_rt + a16(RT * H * 2);
    static constexpr int o_sd = o_sgu + a16(SG * 2 * H * 2);
    static constexpr int o_dn = o_sd + a16(RR * M * 2);
    static constexpr int o_dsc = o_dn + a16(K * RR * S::drow_b);
    static constexpr int o_stage = o_dsc + a16(K * DSC);
    static constexpr int stage_w = kStagePairs * S::row_b;           // gate rows of a stage
    static constexpr int stage_b = a16(2 * stage_w + 2 * 2 * GSC_SEG);
    static constexpr int o_red = o_stage + 2 * stage_b;
    static constexpr int o_out = o_red + 1024;                        // (K+1) x RR floats
    static constexpr int o_chain = o_out + a16((K + 1) * RR * 4);     // (K+1) x M floats
    static constexpr int o_topk = o_chain + a16((K + 1) * M * 4);     // tk[E] doubles
    static constexpr int o_cand = o_topk + a16(E * 8);                // candf[E] ints
    static constexpr int o_sel = o_cand + a16(E * 4);                 // sel[64], wsel[64], ctl[16]
    static constexpr int bytes = o_sel + 64 * 4 + 64 * 4 + 16 * 4;
};

struct DecodeArgs {
    const uint8_t *pool;        // [L][E] expert slots
    int64_t slot_bytes;
    SlotLayout slot;
    const uint16_t *trunk;      // [L] trunk blocks
    int64_t trunk_n;            // elements per layer block
    TrunkLayout tr;
    int n_layers, n_steps, E, renorm, exact_all;
    float *state;               // [H] in/out
    double *S, *B;              // [E]
    float *chain;               // [(K+1) M]
    float *sgate;
    unsigned *ctr;              // [3 * 32]: route, chain, state counters (128 B apart)
    unsigned *diag;             // [4]: layers, fallbacks, error code, failing CTA
    unsigned long long *trace;  // optional [T][G][kTracePts] %globaltimer stamps
};

constexpr int kTracePts = 10;
__device__ __forceinline__ unsigned long long gtimer() {
    unsigned long long t;
    asm volatile("mov.u64 %0, %globaltimer;" : "=l"(t));
    return t;
}

__device__ __forceinline__ bool aborted(const DecodeArgs &a) {
    return *(volatile unsigned *)(a.diag + 2) != 0;
}

// thread 0 only: spin until *ctr >= target; false on abort / timeout
__device__ bool flag_wait(const DecodeArgs &a, const unsigned *ctr, unsigned target, unsigned code) {
    long it = 0;
    while (true) {
        unsigned v;
        asm volatile("ld.acquire.gpu.global.u32 %0, [%1];" : "=r"(v) : "l"(ctr) : "memory");
        if (v >= target) return true;
        if (aborted(a)) return false;
        if (++it > kSpinLimit) {
            if (atomicCAS(a.diag + 2, 0u, code) == 0u) a.diag[3] = blockIdx.x;
            return false;
        }
        __nanosleep(64);
    }
}

__device__ __forceinline__ void flag_arrive(unsigned *ctr) {
    __threadfence();
    atomicAdd(ctr, 1u);
}

// all threads: wait for mbarrier phase; false on timeout (error recorded)
__device__ bool mbar_wait(const DecodeArgs &a, uint64_t *b, uint32_t parity, unsigned code) {
    long it = 0;
    while (!mbar_test(b, parity)) {
        if (++it > kSpinLimit) {
            if (atomicCAS(a.diag + 2, 0u, code) == 0u) a.diag[3] = blockIdx.x;
            return false;
        }
        __nanosleep(32);
    }
    return true;
}

template <int FMT, int H, int M, int E, int K>
__global__ void __launch_bounds__(kThreads, 1)
k_decode(DecodeArgs a) {
    using S = Shape<FMT, H, M>;
    using L = Smem<FMT, H, M, E, K>;
    extern __shared__ __align__(128) unsigned char sm[];
    uint64_t *bar = (uint64_t *)(sm + L::o_bar);
    // bar[0]: router + shared gate/up rows; bar[1]: shared down rows;
    // bar[2], bar[3]: gate/up ring; bar[4]: routed down rows
    float *xin = (float *)(sm + L::o_xin);
    uint16_t *rt = (uint16_t *)(sm + L::o_rt);
    uint16_t *sgu = (uint16_t *)(sm + L::o_sgu);
    uint16_t *sd = (uint16_t *)(sm + L::o_sd);
    uint8_t *dn = sm + L::o_dn;
    uint8_t *dsc = sm + L::o_dsc;
    uint8_t *stage = sm + L::o_stage;
    float *red = (float *)(sm + L::o_red);          // 256 floats of scratch
    float *outs = (float *)(sm + L::o_out);
    float *cs = (float *)(sm + L::o_chain);         // staged chains
    double *tk = (double *)(sm + L::o_topk);        // [E] logit used for softmax
    int *candf = (int *)(sm + L::o_cand);           // [E] exact-path candidates
    int *sel = (int *)(sm + L::o_sel);              // [64] selection order
    float *wsel = (float *)(sel + 64);              // [64] weights
    int *ctl = (int *)(wsel + 64);                  // control words

    const int tid = threadIdx.x, lane = tid & 31, warp = tid >> 5;
    const int G = gridDim.x, c = blockIdx.x;
    const int rt0 = c * E / G, rt1 = (c + 1) * E / G;
    const int sg0 = c * M / G, sg1 = (c + 1) * M / G;
    const int p0 = c * (K * M) / G, p1 = (c + 1) * (K * M) / G;
    const int r0 = c * H / G, r1 = (c + 1) * H / G, nr = r1 - r0;
    const int nstages = (p1 - p0 + kStagePairs - 1) / kStagePairs;
    unsigned *c_route = a.ctr, *c_chain = a.ctr + 32, *c_state = a.ctr + 64;

    uint32_t ph[5] = {0, 0, 0, 0, 0};          // next parity to wait per barrier
    bool pend[5] = {false, false, false, false, false};
    bool ok = true;

    if (tid == 0) {
        for (int i = 0; i < 5; i++) mbar_init(bar + i, 1);
        asm volatile("fence.mbarrier_init.release.cluster;" ::: "memory");
    }
    __syncthreads();

    auto trunk_l = [&](int l) { return a.trunk + (int64_t)l * a.trunk_n; };
    auto expert = [&](int l, int e) { return a.pool + ((int64_t)l * a.E + e) * a.slot_bytes; };

    // TMA: router + shared gate/up rows of layer l (bar 0)
    auto prefetch_rt = [&](int l) {
        const uint16_t *t = trunk_l(l);
        uint32_t b1 = (rt1 - rt0) * H * 2, b2 = (sg1 - sg0) * H * 2;
        mbar_expect(bar + 0, b1 + 2 * b2);
        if (b1) bulk(rt, t + a.tr.router + (int64_t)rt0 * H, b1, bar + 0);
        if (b2) {
            bulk(sgu, t + a.tr.sh_gate + (int64_t)sg0 * H, b2, bar + 0);
            bulk(sgu + L::SG * H, t + a.tr.sh_up + (int64_t)sg0 * H, b2, bar + 0);
        }
    };
    // TMA: shared down rows of layer l (bar 1)
    auto prefetch_sd = [&](int l) {
        uint32_t b = nr * M * 2;
        mbar_expect(bar + 1, b);
        if (b) bulk(sd, trunk_l(l) + a.tr.sh_down + (int64_t)r0 * M, b, bar + 1);
    };
    // TMA: gate/up stage s of layer l into ring slot s & 1 (bar 2 + slot)
    auto issue_stage = [&](int l, int s) {
        uint8_t *st = stage + (s & 1) * L::stage_b;
        uint8_t *wg = st, *wu = st + L::stage_w, *sc = st + 2 * L::stage_w;
        int q0 = p0 + s * kStagePairs, q1 = min(q0 + kStagePairs, p1);
        uint32_t total = 0;
        int seg = 0;
        struct { int j, i0, i1, slot; } sgs[2];
        for (int q = q0; q < q1;) {
            int j = q / M, i0 = q % M, n = min(q1 - q, M - i0);
            sgs[seg] = {j, i0, i0 + n, q - q0};
            seg++;
            q += n;
        }
        for (int g = 0; g < seg; g++) {
            int n = sgs[g].i1 - sgs[g].i0;
            total += 2 * n * S::row_b;
            total += FMT == DS4F_FMT_FP8 ? 2 * S::gsc_b : 2 * n * S::gsc_b;
        }
        mbar_expect(bar + 2 + (s & 1), total);
        for (int g = 0; g < seg; g++) {
            const uint8_t *ex = expert(l, sel[sgs[g].j]);
            int n = sgs[g].i1 - sgs[g].i0, sl = sgs[g].slot;
            bulk(wg + sl * S::row_b, ex + a.slot.rel_v[0] + (int64_t)sgs[g].i0 * S::row_b,
                 n * S::row_b, bar + 2 + (s & 1));
            bulk(wu + sl * S::row_b, ex + a.slot.rel_v[1] + (int64_t)sgs[g].i0 * S::row_b,
                 n * S::row_b, bar + 2 + (s & 1));
            if (FMT == DS4F_FMT_FP8) {
                bulk(sc + g * L::GSC_SEG, ex + a.slot.rel_s[0], S::gsc_b, bar + 2 + (s & 1));
                bulk(sc + (2 + g) * L::GSC_SEG, ex + a.slot.rel_s[1], S::gsc_b, bar + 2 + (s & 1));
            } else {
                bulk(sc + sl * S::gsc_b, ex + a.slot.rel_s[0] + (int64_t)sgs[g].i0 * S::gsc_b,
                     n * S::gsc_b, bar + 2 + (s & 1));
                bulk(sc + L::GSC_SEG * 2 + sl * S::gsc_b,
                     ex + a.slot.rel_s[1] + (int64_t)sgs[g].i0 * S::gsc_b, n * S::gsc_b,
                     bar + 2 + (s & 1));
            }
        }
    };
    // TMA: routed down rows [r0, r1) of the K selected experts (bar 4)
    auto issue_down = [&](int l) {
        uint32_t total = K * nr * S::drow_b;
        int64_t sa0 = 0, sab = 0;
        if (FMT == DS4F_FMT_FP8) {
            total += K * S::dsc_b;
        } else {
            sa0 = ((int64_t)r0 * S::dsc_b) / 16 * 16;
            sab = (((int64_t)r1 * S::dsc_b + 15) / 16) * 16 - sa0;
            total += K * (uint32_t)sab;
        }
        mbar_expect(bar + 4, total);
        for (int j = 0; j < K; j++) {
            const uint8_t *ex = expert(l, sel[j]);
            if (nr)
                bulk(dn + j * L::RR * S::drow_b, ex + a.slot.rel_v[2] + (int64_t)r0 * S::drow_b,
                     nr * S::drow_b, bar + 4);
            if (FMT == DS4F_FMT_FP8)
                bulk(dsc + j * L::DSC, ex + a.slot.rel_s[2], S::dsc_b, bar + 4);
            else
                bulk(dsc + j * L::DSC, ex + a.slot.rel_s[2] + sa0, (uint32_t)sab, bar + 4);
        }
    };

    // layer-0 prefetches
    if (tid == 0) {
        prefetch_rt(0);
        prefetch_sd(0);
    }
    pend[0] = pend[1] = true;

    const int T = a.n_layers * a.n_steps;
    // phase stamps: 0 start, 1 state ready, 2 normed, 3 router+shared done,
    // 4 routes visible, 5 top-k done, 6 copies issued + softmax, 7 chains done,
    // 8 chains visible, 9 state rows written
#define DS4F_TRACE(k) \
    if (a.trace && tid == 0) a.trace[((int64_t)t * G + c) * kTracePts + (k)] = gtimer()
    for (int t = 0; t < T && ok; t++) {
        const int l = t % a.n_layers;
        DS4F_TRACE(0);
        const int ln = (t + 1) % a.n_layers;
        const bool more = t + 1 < T;
        // (A) input state of this layer
        if (t > 0) {
            if (tid == 0) ctl[0] = flag_wait(a, c_state, (unsigned)(t * G), 1);
            __syncthreads();
            if (!ctl[0]) { ok = false; break; }
        }
        DS4F_TRACE(1);
        // (B) RMSNorm (src/moe.c:841-851): double sum of squares, fixed tree
        {
            double ss = 0.0;
            for (int i = tid; i < H; i += kThreads) {
                float v = __ldcg(a.state + i);
                xin[i] = v;
                double d = (double)v;
                ss = __dadd_rn(ss, __dmul_rn(d, d));
            }
            ss = warp_sum_d(ss);
            double *rd = (double *)red;
            if (lane == 0) rd[warp] = ss;
            __syncthreads();
            if (tid == 0) {
                double s2 = 0.0;
                for (int k = 0; k < kWarps; k++) s2 = __dadd_rn(s2, rd[k]);
                rd[16] = s2;
            }
            __syncthreads();
            float r = __fsqrt_rn(__fadd_rn(__double2float_rn(__ddiv_rn(rd[16], (double)H)), 1e-6f));
            const uint16_t *nw = trunk_l(l) + a.tr.norm;
            for (int i = tid; i < H; i += kThreads)
                xin[i] = __fmul_rn(__fdiv_rn(xin[i], r), bf16_to_f32(__ldg(nw + i)));
            __syncthreads();
        }
        DS4F_TRACE(2);
        // (C) router rows + shared gate/up rows (weights prefetched, bar 0)
        if (!__syncthreads_and(mbar_wait(a, bar + 0, ph[0], 2))) { ok = false; break; }
        ph[0] ^= 1; pend[0] = false;
        if (warp < rt1 - rt0) {
            const int e = rt0 + warp;
            const uint16_t *row = rt + warp * H;
            double base = 0.0, bsum = 0.0;
            for (int k = 0; k < H / 256; k++) {
                int q = lane + 32 * k;
                uint4 w = lds16(row + q * 8);
                uint32_t ww[4] = {w.x, w.y, w.z, w.w};
                double Tq = 0.0, Aq = 0.0;
#pragma unroll
                for (int u = 0; u < 8; u++) {
                    uint32_t h = (u & 1) ? (ww[u >> 1] & 0xFFFF0000u) : (ww[u >> 1] << 16);
                    float p = __fmul_rn(__uint_as_float(h), xin[q * 8 + u]);
                    Tq = __dadd_rn(Tq, (double)p);
                    Aq = __dadd_rn(Aq, (double)fabsf(p) * (double)(8 - u));
                }
                double incl = Tq;
#pragma unroll
                for (int o = 1; o < 32; o <<= 1) {
                    double y = __shfl_up_sync(0xFFFFFFFFu, incl, o);
                    if (lane >= o) incl = __dadd_rn(incl, y);
                }
                double excl = __shfl_up_sync(0xFFFFFFFFu, incl, 1);
                if (lane == 0) excl = 0.0;
                bsum = __dadd_rn(bsum, __dadd_rn(8.0 * fabs(__dadd_rn(base, excl)), Aq));
                base = __dadd_rn(base, __shfl_sync(0xFFFFFFFFu, incl, 31));
            }
            bsum = warp_sum_d(bsum);
            if (lane == 0) {
                __stcg(a.S + e, base);
                __stcg(a.B + e, 1.001 * kU * bsum + 1e-300);
            }
        } else if (warp >= L::RT && warp < L::RT + 2 * (sg1 - sg0)) {
            // shared gate (even) / up (odd) row dots, bf16, x unscaled
            const int w2 = warp - L::RT, i = w2 >> 1, m = w2 & 1;
            const uint16_t *row = sgu + m * L::SG * H + i * H;
            float acc = 0.f;
#pragma unroll
            for (int k = 0; k < H / 256; k++) {
                int q = lane + 32 * k;
                acc += bf16_dot8(lds16(row + q * 8), xin + q * 8);
            }
            acc = warp_sum(acc);
            if (lane == 0) red[64 + w2] = acc;
        } else if (warp == kWarps - 1 && c == G - 1) {
            const uint16_t *gw = trunk_l(l) + a.tr.sh_gw;
            float acc = 0.f;
            for (int k = 0; k < H / 256; k++) {
                int q = lane + 32 * k;
                acc += bf16_dot8(__ldg((const uint4 *)(gw + q * 8)), xin + q * 8);
            }
            acc = warp_sum(acc);
            if (lane == 0) __stcg(a.sgate, acc);
        }
        __syncthreads();
        if (tid < sg1 - sg0)
            __stcg(a.chain + K * M + sg0 + tid, silu_mul(red[64 + 2 * tid], red[64 + 2 * tid + 1]));
        __syncthreads();
        if (tid == 0) {
            flag_arrive(c_route);
            // (E) next layer's router + shared gate/up rows into the freed buffers
            if (more) { fence_async(); prefetch_rt(ln); }
        }
        pend[0] = more;
        DS4F_TRACE(3);
        // (F) routing: every CTA, identical bits
        if (tid == 0) ctl[0] = flag_wait(a, c_route, (unsigned)((t + 1) * G), 3);
        __syncthreads();
        if (!ctl[0]) { ok = false; break; }
        DS4F_TRACE(4);
        if (warp == 0) {
            // certified top-K from [S - B, S + B]; lane holds e = lane + 32 i
            constexpr int NE = (E + 31) / 32;
            double sv[NE], lo[NE], hi[NE];
#pragma unroll
            for (int i = 0; i < NE; i++) {
                int e = lane + 32 * i;
                if (e < E) {
                    double s = __ldcg(a.S + e), b = a.exact_all ? 0.0 : __ldcg(a.B + e);
                    sv[i] = s; lo[i] = s - b; hi[i] = s + b;
                } else {
                    sv[i] = lo[i] = hi[i] = -1e300;
                }
            }
            // K rounds of arg-max of lo (lower index wins ties)
            unsigned taken = 0;
            double lk = 0.0;
            for (int k = 0; k < K; k++) {
                double bv = -2e300; int be = 0x7FFFFFFF;
#pragma unroll
                for (int i = 0; i < NE; i++) {
                    int e = lane + 32 * i;
                    if (!(taken >> i & 1) && e < E && (lo[i] > bv || (lo[i] == bv && e < be))) { bv = lo[i]; be = e; }
                }
#pragma unroll
                for (int o = 16; o > 0; o >>= 1) {
                    double ov = __shfl_xor_sync(0xFFFFFFFFu, bv, o);
                    int oe = __shfl_xor_sync(0xFFFFFFFFu, be, o);
                    if (ov > bv || (ov == bv && oe < be)) { bv = ov; be = oe; }
                }
                if ((be & 31) == lane) taken |= 1u << (be >> 5);
                lk = bv;
            }
            int mine = 0;
#pragma unroll
            for (int i = 0; i < NE; i++) mine += (lane + 32 * i < E) && hi[i] >= lk;
            int ncand = mine;
#pragma unroll
            for (int o = 16; o > 0; o >>= 1) ncand += __shfl_xor_sync(0xFFFFFFFFu, ncand, o);
            bool cert = !a.exact_all && ncand == K;
            double prev_lo = 0.0;
            if (cert) {
                // order the K candidates (= the taken set) by S, check separation
                unsigned used = 0;
                for (int k = 0; k < K; k++) {
                    double bv = -2e300; int be = 0x7FFFFFFF; double blo = 0.0, bhi = 0.0;
#pragma unroll
                    for (int i = 0; i < NE; i++) {
                        int e = lane + 32 * i;
                        if ((taken >> i & 1) && !(used >> i & 1) && (sv[i] > bv || (sv[i] == bv && e < be))) {
                            bv = sv[i]; be = e; blo = lo[i]; bhi = hi[i];
                        }
                    }
#pragma unroll
                    for (int o = 16; o > 0; o >>= 1) {
                        double ov = __shfl_xor_sync(0xFFFFFFFFu, bv, o);
                        int oe = __shfl_xor_sync(0xFFFFFFFFu, be, o);
                        double ol = __shfl_xor_sync(0xFFFFFFFFu, blo, o);
                        double oh = __shfl_xor_sync(0xFFFFFFFFu, bhi, o);
                        if (ov > bv || (ov == bv && oe < be)) { bv = ov; be = oe; blo = ol; bhi = oh; }
                    }
                    if ((be & 31) == lane) used |= 1u << (be >> 5);
                    if (k > 0 && !(prev_lo > bhi)) cert = false;
                    prev_lo = blo;
                    if (lane == 0) sel[k] = be;
                }
            }
            // tk[e] = value used for softmax; candidate flags for the exact path
#pragma unroll
            for (int i = 0; i < NE; i++) {
                int e = lane + 32 * i;
                if (e < E) {
                    tk[e] = (double)(float)sv[i];
                    candf[e] = a.exact_all || hi[i] >= lk;
                }
            }
            if (lane == 0) { ctl[1] = cert ? 1 : 0; ctl[2] = ncand; }
        }
        __syncthreads();
        if (!ctl[1]) {
            // exact reference-order logits (src/kernels.c:97-102) of every
            // candidate, one thread each, then select on them
            const uint16_t *router = trunk_l(l) + a.tr.router;
            for (int e = tid; e < E; e += kThreads) {
                if (!candf[e]) continue;
                const uint16_t *row = router + (int64_t)e * H;
                float acc = 0.0f;
                for (int cc = 0; cc < H; cc++)
                    acc = __fadd_rn(acc, __fmul_rn(bf16_to_f32(__ldg(row + cc)), xin[cc]));
                tk[e] = (double)acc;
            }
            __syncthreads();
            for (int e = tid; e < E; e += kThreads) {
                if (!candf[e]) continue;
                int r = 0;
                double ve = tk[e];
                for (int f = 0; f < E; f++) r += candf[f] && (tk[f] > ve || (tk[f] == ve && f < e));
                if (r < K) sel[r] = e;
            }
            if (tid == 0 && !a.exact_all && c == 0) atomicAdd(a.diag + 1, 1u);
            __syncthreads();
        }
        DS4F_TRACE(5);
        // (G) stream the selected experts: gate/up ring + down rows
        if (tid == 0) {
            fence_async();
            for (int s = 0; s < 2 && s < nstages; s++) issue_stage(l, s);
            issue_down(l);
        }
        pend[2] = nstages > 0; pend[3] = nstages > 1; pend[4] = true;
        // softmax over all E (double, max subtracted) + renorm, while the
        // copies fly
        {
            double *rd = (double *)red;
            double mx = tid < E ? tk[tid] : -1e300;
#pragma unroll
            for (int o = 16; o > 0; o >>= 1) mx = fmax(mx, __shfl_xor_sync(0xFFFFFFFFu, mx, o));
            if (lane == 0) rd[16 + warp] = mx;
            __syncthreads();
            mx = rd[16];
            for (int k = 1; k < kWarps; k++) mx = fmax(mx, rd[16 + k]);
            double part = 0.0;
            if (tid < E) part = exp(tk[tid] - mx);
            part = warp_sum_d(part);
            if (lane == 0) rd[warp] = part;
            __syncthreads();
            if (tid == 0) {
                double sw = 0.0;
                for (int k = 0; k < kWarps; k++) sw += rd[k];
                float s = 0.0f;
                for (int j = 0; j < K; j++) {
                    wsel[j] = (float)(exp(tk[sel[j]] - mx) / sw);
                    s = __fadd_rn(s, wsel[j]);
                }
                if (a.renorm && s > 0.0f)
                    for (int j = 0; j < K; j++) wsel[j] = __fdiv_rn(wsel[j], s);
                if (c == 0) atomicAdd(a.diag, 1u);
            }
            __syncthreads();
        }
        DS4F_TRACE(6);
        // (H) gate/up dots: warp w -> slot w/2 of the stage, gate (even) / up
        {
            float xr[S::gk * S::ce];
#pragma unroll
            for (int k = 0; k < S::gk; k++)
#pragma unroll
                for (int e = 0; e < S::ce; e += 4) {
                    float4 v = *(const float4 *)(xin + (lane + 32 * k) * S::ce + e);
                    xr[k * S::ce + e] = v.x * DS4F_X_PRESCALE;
                    xr[k * S::ce + e + 1] = v.y * DS4F_X_PRESCALE;
                    xr[k * S::ce + e + 2] = v.z * DS4F_X_PRESCALE;
                    xr[k * S::ce + e + 3] = v.w * DS4F_X_PRESCALE;
                }
            for (int s = 0; s < nstages; s++) {
                const int slot = s & 1;
                if (!__syncthreads_and(mbar_wait(a, bar + 2 + slot, ph[2 + slot], 4))) { ok = false; break; }
                ph[2 + slot] ^= 1;
                uint8_t *st = stage + slot * L::stage_b;
                const int q0 = p0 + s * kStagePairs, nq = min(kStagePairs, p1 - q0);
                const int ps = warp >> 1, m = warp & 1;
                if (ps < nq) {
                    const int q = q0 + ps, i = q % M;
                    const int jfirst = q0 / M;
                    const int g = q / M - jfirst;                  // segment 0 or 1
                    const uint8_t *row = st + m * L::stage_w + ps * S::row_b;
                    float acc = 0.f;
#pragma unroll
                    for (int k = 0; k < S::gk; k++) {
                        const int qq = lane + 32 * k;
                        uint4 w = lds16(row + qq * 16);
                        if constexpr (FMT == DS4F_FMT_FP8) {
                            const float *sc = (const float *)(st + 2 * L::stage_w + (2 * m + g) * L::GSC_SEG);
                            float s8 = sc[(i >> 7) * (H / 128) + (qq >> 3)];
                            acc = fmaf(f8_dot16(w, xr + k * S::ce) * DS4F_F8_POST, s8, acc);
                        } else {
                            // gate scales at [0, GSC_SEG), up at [2 GSC_SEG, 3 GSC_SEG),
                            // one E8M0 byte per 32-element chunk, row by slot
                            const uint8_t *sc = st + 2 * L::stage_w + m * 2 * L::GSC_SEG;
                            float s4 = e8m0_to_f32(sc[ps * S::gsc_b + qq]);
                            acc = fmaf(e2m1_dot32(w, xr + k * S::ce) * DS4F_E2M1_POST, s4, acc);
                        }
                    }
                    acc = warp_sum(acc);
                    if (lane == 0) red[2 * ps + m] = acc;
                }
                __syncthreads();
                if (tid < nq) {
                    const int q = q0 + tid;
                    __stcg(a.chain + (q / M) * M + (q % M), silu_mul(red[2 * tid], red[2 * tid + 1]));
                }
                __syncthreads();
                if (tid == 0 && s + 2 < nstages) { fence_async(); issue_stage(l, s + 2); }
                pend[2 + slot] = s + 2 < nstages;
            }
            if (!ok) break;
        }
        __syncthreads();
        DS4F_TRACE(7);
        if (tid == 0) flag_arrive(c_chain);
        // (I) all chains
        if (tid == 0) ctl[0] = flag_wait(a, c_chain, (unsigned)((t + 1) * G), 5);
        __syncthreads();
        if (!ctl[0]) { ok = false; break; }
        DS4F_TRACE(8);
        for (int i = tid; i < (K + 1) * M; i += kThreads) cs[i] = __ldcg(a.chain + i);
        // (J) down rows: routed (bar 4) and shared (bar 1)
        if (!__syncthreads_and(mbar_wait(a, bar + 4, ph[4], 6))) { ok = false; break; }
        ph[4] ^= 1; pend[4] = false;
        if (!__syncthreads_and(mbar_wait(a, bar + 1, ph[1], 7))) { ok = false; break; }
        ph[1] ^= 1; pend[1] = false;
        {
            // row-dots (j, r), j-major, j = K the shared expert; warp w takes
            // a contiguous range so its chain registers change at most twice
            const int ndots = (K + 1) * nr;
            const int d0 = warp * ndots / kWarps, d1 = (warp + 1) * ndots / kWarps;
            int jcur = -1;
            float xr[S::dk * S::ce];          // routed chain (pre-scaled by 2^64)
            float xb[S::bk * 8];              // shared chain (bf16 chunk layout)
            for (int d = d0; d < d1; d++) {
                const int j = d / nr, rr = d % nr;
                if (j != jcur) {
                    jcur = j;
                    if (j < K) {
#pragma unroll
                        for (int k = 0; k < S::dk; k++)
#pragma unroll
                            for (int e = 0; e < S::ce; e++)
                                xr[k * S::ce + e] =
                                    cs[j * M + ((lane % S::dlpr) + S::dlpr * k) * S::ce + e] * DS4F_X_PRESCALE;
                    } else {
#pragma unroll
                        for (int k = 0; k < S::bk; k++)
#pragma unroll
                            for (int e = 0; e < 8; e++)
                                xb[k * 8 + e] = cs[K * M + ((lane % S::blpr) + S::blpr * k) * 8 + e];
                    }
                }
                float v = 0.f;
                if (j < K) {
                    // rows shorter than a warp: lane groups repeat the row and
                    // only lane 0's sum is kept
                    const uint8_t *row = dn + (j * L::RR + rr) * S::drow_b;
                    const int ql = lane % S::dlpr;
#pragma unroll
                    for (int k = 0; k < S::dk; k++) {
                        const int q = ql + S::dlpr * k;
                        uint4 w = lds16(row + q * 16);
                        if constexpr (FMT == DS4F_FMT_FP8) {
                            const float *sc = (const float *)(dsc + j * L::DSC);
                            float s8 = sc[((r0 + rr) >> 7) * (M / 128) + (q >> 3)];
                            v = fmaf(f8_dot16(w, xr + k * S::ce) * DS4F_F8_POST, s8, v);
                        } else {
                            const int sa0 = (r0 * S::dsc_b) / 16 * 16;
                            const uint8_t *sc = dsc + j * L::DSC;
                            float s4 = e8m0_to_f32(sc[(r0 + rr) * S::dsc_b - sa0 + q]);
                            v = fmaf(e2m1_dot32(w, xr + k * S::ce) * DS4F_E2M1_POST, s4, v);
                        }
                    }
#pragma unroll
                    for (int o = S::dlpr >> 1; o > 0; o >>= 1) v += __shfl_xor_sync(0xFFFFFFFFu, v, o);
                } else {
                    const uint16_t *row = sd + rr * M;
                    const int ql = lane % S::blpr;
#pragma unroll
                    for (int k = 0; k < S::bk; k++) {
                        const int q = ql + S::blpr * k;
                        v += bf16_dot8(lds16(row + q * 8), xb + k * 8);
                    }
#pragma unroll
                    for (int o = S::blpr >> 1; o > 0; o >>= 1) v += __shfl_xor_sync(0xFFFFFFFFu, v, o);
                }
                if (lane == 0) outs[j * L::RR + rr] = v;
            }
            __syncthreads();
            // selection-order combine (src/moe.c:1224-1225), shared gate
            // (:1279-1282), residual (:1424)
            if (tid < nr) {
                const int r = r0 + tid;
                float acc = 0.0f;
                for (int j = 0; j < K; j++) acc = __fadd_rn(acc, __fmul_rn(wsel[j], outs[j * L::RR + tid]));
                float sg = sigmoid_ref(__ldcg(a.sgate));
                acc = __fadd_rn(acc, __fmul_rn(sg, outs[K * L::RR + tid]));
                __stcg(a.state + r, __fadd_rn(__ldcg(a.state + r), acc));
            }
            __syncthreads();
        }
        DS4F_TRACE(9);
        if (tid == 0) {
            flag_arrive(c_state);
            if (more) { fence_async(); prefetch_sd(ln); }
        }
        pend[1] = more;
    }
#undef DS4F_TRACE
    // drain this CTA's copies before exit (bounded)
    for (int i = 0; i < 5; i++)
        if (pend[i]) mbar_wait(a, bar + i, ph[i], 8);
}

}  // namespace
}  // namespace ds4f

namespace ds4f {
namespace {

template <int FMT, int H, int M, int E, int K>
int launch_t(Model *m, float *state, int n_steps, cudaStream_t st) {
    using L = Smem<FMT, H, M, E, K>;
    static_assert(L::bytes <= 227 * 1024, "decode kernel shared memory over budget");
    static bool attr = false;
    auto kern = k_decode<FMT, H, M, E, K>;
    if (!attr) {
        DS4F_CUDA(cudaFuncSetAttribute(kern, cudaFuncAttributeMaxDynamicSharedMemorySize, L::bytes));
        attr = true;
    }
    int dev = 0, sms = 0;
    DS4F_CUDA(cudaGetDevice(&dev));
    DS4F_CUDA(cudaDeviceGetAttribute(&sms, cudaDevAttrMultiProcessorCount, dev));
    DS4F_REQUIRE(sms >= kGmin, "decode: %d SMs, the persistent kernel needs >= %d", sms, kGmin);
    DecodeArgs a;
    a.pool = m->pool;
    a.slot_bytes = m->slot.nbytes;
    a.slot = m->slot;
    a.trunk = m->trunk;
    a.trunk_n = m->tr.n;
    a.tr = m->tr;
    a.n_layers = m->d.n_layers;
    a.n_steps = n_steps;
    a.E = E;
    a.renorm = m->d.renorm;
    a.exact_all = m->d.router_exact;
    a.state = state;
    a.S = m->w.S;
    a.B = m->w.Bnd;
    a.chain = m->w.chain;
    a.sgate = m->w.sgate;
    a.ctr = m->w.ctr;
    a.diag = m->w.diag;
    a.trace = nullptr;
    if (m->trace && (int64_t)m->d.n_layers * n_steps * sms * kTracePts <= m->trace_n) a.trace = m->trace;
    DS4F_CUDA(cudaMemsetAsync(m->w.ctr, 0, 3 * 128, st));
    DS4F_CUDA(cudaMemsetAsync(m->w.diag + 2, 0, 2 * sizeof(unsigned), st));
    cudaLaunchConfig_t cfg = {};
    cfg.gridDim = dim3(sms);
    cfg.blockDim = dim3(kThreads);
    cfg.dynamicSmemBytes = L::bytes;
    cfg.stream = st;
    cudaLaunchAttribute at[1];
    at[0].id = cudaLaunchAttributeCooperative;
    at[0].val.cooperative = 1;
    cfg.attrs = at;
    cfg.numAttrs = 1;
    DS4F_CUDA(cudaLaunchKernelEx(&cfg, kern, a));
    return 0;
}

}  // namespace

bool decode_eligible(const Model *m) {
    const ModelDesc &d = m->d;
    if (d.expert_count != d.n_experts || d.topk != 8) return false;
    if (!((d.hidden == 2048 && d.moe_inter == 512) || (d.hidden == 1024 && d.moe_inter == 256)))
        return false;
    return d.n_experts == 256 || d.n_experts == 64;
}

int decode_launch(Model *m, float *state, int n_steps, cudaStream_t st) {
    const ModelDesc &d = m->d;
    DS4F_REQUIRE(decode_eligible(m), "decode: shape not supported by the persistent kernel");
    const bool f8 = d.fmt == DS4F_FMT_FP8;
    if (d.hidden == 2048 && d.n_experts == 256)
        return f8 ? launch_t<DS4F_FMT_FP8, 2048, 512, 256, 8>(m, state, n_steps, st)
                  : launch_t<DS4F_FMT_MXFP4, 2048, 512, 256, 8>(m, state, n_steps, st);
    if (d.hidden == 2048 && d.n_experts == 64)
        return f8 ? launch_t<DS4F_FMT_FP8, 2048, 512, 64, 8>(m, state, n_steps, st)
                  : launch_t<DS4F_FMT_MXFP4, 2048, 512, 64, 8>(m, state, n_steps, st);
    if (d.n_experts == 256)
        return f8 ? launch_t<DS4F_FMT_FP8, 1024, 256, 256, 8>(m, state, n_steps, st)
                  : launch_t<DS4F_FMT_MXFP4, 1024, 256, 256, 8>(m, state, n_steps, st);
    return f8 ? launch_t<DS4F_FMT_FP8, 1024, 256, 64, 8>(m, state, n_steps, st)
              : launch_t<DS4F_FMT_MXFP4, 1024, 256, 64, 8>(m, state, n_steps, st);
}

}  // namespace ds4f
