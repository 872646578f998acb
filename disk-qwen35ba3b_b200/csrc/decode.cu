// decode.cu -- persistent decode kernel: every layer of a decode step (and
// several steps) for one token in ONE cooperative launch, one CTA per SM.
//
// Per layer, CTA c of G owns a static slice of every phase: router rows
// [cE/G, (c+1)E/G), shared gate/up rows [cM/G, ...), routed (selection,
// row) pairs [cKM/G, ...) and output rows [cH/G, ...). A layer is
//   (A) the layer's input state (tagged words, see below)
//   (B) RMSNorm of the full state (src/moe.c:841-851)
//   (C) its router rows -> certified logits S and bounds B, published
//   (D) its shared-expert gate/up rows -> shared SiLU chain, published
//   (F) every CTA: poll all S/B, top-k + softmax + renorm (same bits in
//       every CTA); exact reference-order logits only for near-ties
//   (G) TMA bulk copies of ALL of its routed gate/up rows and down rows
//       (about 176 KB per SM for FP8, in flight at once), 4 sub-barriers
//   (H) gate/up dots + SiLU-mul as the bytes land -> chains, published
//   (I) down rows (routed + prefetched shared) against the polled chains,
//       selection-order combine, shared gate, residual -> state, published
// The next layer's router rows + norm weights and shared down rows are
// prefetched by TMA during the current layer.
//
// Publication: a value written by one CTA for the others is an 8-byte word
// (tag << 32 | bits) stored with st.relaxed.gpu; a reader polls the word
// with ld.relaxed.gpu until the tag is the one of this layer, so the data
// itself is the signal (one L2 round trip, no counters or atomics). Tags
// are (launch epoch << 16) | (layer-step + 1). Every wait is bounded: a
// poll or copy wait that gives up records an error code, the CTA drains its
// own copies and returns; the host reports it.
//
// Reference: ds4f_moe_step (src/moe.c:948-1456) and its router call site
// (src/main.c:1014-1088), per layer of the decode loop (src/main.c:848).
#include "model.cuh"

#include <algorithm>

namespace ds4f {

namespace {

constexpr int kThreads = 512;
constexpr int kWarps = kThreads / 32;
constexpr int kGmin = 144;                 // shared memory is sized for G >= this
constexpr int kGroupPairs = 8;             // gate/up pairs per copy group
constexpr int kGroups = 4;
constexpr long kSpin = 1L << 24;           // default polls (with backoff) before giving up
constexpr double kU = 5.9604644775390625e-08;
constexpr int kTracePts = 32;
constexpr int kMaxRanks = 8;

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
__device__ __forceinline__ void bulk(void *dst, const void *src, uint32_t bytes, uint64_t *b) {
    asm volatile(
        "cp.async.bulk.shared::cluster.global.mbarrier::complete_tx::bytes [%0], [%1], %2, [%3];"
        ::"r"(sa(dst)), "l"(src), "r"(bytes), "r"(sa(b)) : "memory");
}
__device__ __forceinline__ void fence_async() {
    asm volatile("fence.proxy.async.shared::cta;" ::: "memory");
}
__device__ __forceinline__ uint4 lds16(const void *p) {
    uint4 r;
    asm volatile("ld.shared.v4.u32 {%0,%1,%2,%3}, [%4];"
                 : "=r"(r.x), "=r"(r.y), "=r"(r.z), "=r"(r.w) : "r"(sa(p)) : "memory");
    return r;
}
__device__ __forceinline__ void st_tag(uint64_t *p, uint32_t tag, uint32_t bits) {
    uint64_t w = ((uint64_t)tag << 32) | bits;
    asm volatile("st.relaxed.gpu.global.u64 [%0], %1;" ::"l"(p), "l"(w) : "memory");
}
// After a thread's last tagged store of a phase: push its stores out to L2
// now (readers poll with bulk copies; a relaxed store may otherwise linger
// in the SM's write path for microseconds). It blocks the storing thread
// for ~0.5-1.5 us, so it is used where that thread waits anyway (the chain
// and state publishes), not where it issues the next copies.
__device__ __forceinline__ void publish_flush() {
    asm volatile("fence.acq_rel.gpu;" ::: "memory");
}
// A tagged word stored into another GPU's memory (a peer mapping; visible
// there ~1 us later, measured on B200 over NVLink, fence or not), and a
// load of such a word from this GPU's memory.
__device__ __forceinline__ void st_tag_sys(uint64_t *p, uint32_t tag, uint32_t bits) {
    uint64_t w = ((uint64_t)tag << 32) | bits;
    asm volatile("st.relaxed.sys.global.u64 [%0], %1;" ::"l"(p), "l"(w) : "memory");
}
__device__ __forceinline__ uint64_t ld_sys(const uint64_t *p) {
    uint64_t w;
    asm volatile("ld.relaxed.sys.global.u64 %0, [%1];" : "=l"(w) : "l"(p) : "memory");
    return w;
}
__device__ __forceinline__ unsigned long long gtimer() {
    unsigned long long t;
    asm volatile("mov.u64 %0, %globaltimer;" : "=l"(t));
    return t;
}
// ---- shapes -------------------------------------------------------------------
template <int FMT, int H, int M>
struct Shape {
    static constexpr int row_b = FMT == DS4F_FMT_FP8 ? H : H / 2;     // gate/up row bytes
    static constexpr int drow_b = FMT == DS4F_FMT_FP8 ? M : M / 2;    // down row bytes
    static constexpr int cpl = H / 32;                                 // router cols per lane
    // 4-byte weight granules: lane l of a row-dot reads granules 32 j + l
    static constexpr int gb = FMT == DS4F_FMT_FP8 ? 4 : 8;             // elements / granule
    static constexpr int ng = H / (32 * gb);                           // gate/up granules / lane
    static constexpr int dg = M / (32 * gb);                           // down granules / lane
    static constexpr int bn = M / 128;                                 // bf16 8-byte granules / lane
    static_assert(ng >= 1 && H % (32 * gb) == 0 && dg >= 1 && M % (32 * gb) == 0 && M % 128 == 0,
                  "granules span the warp");
    static constexpr int gsc_b = FMT == DS4F_FMT_FP8 ? (M / 128) * (H / 128) * 4 : H / 32;
    static constexpr int dsc_b = FMT == DS4F_FMT_FP8 ? (H / 128) * (M / 128) * 4 : M / 32;
    static_assert(cpl % 8 == 0, "router rows: whole 8-element chunks per lane");
};

// The exact fallback's selection, out of line (rarely run, so kept out of
// the layer loop's instruction stream): every candidate's logit in the
// reference's sequential order (src/kernels.c:97-102), one thread each,
// then the top K among the candidates -- or, when a logit is not finite,
// the reference's insertion rule over every expert. CTA-wide.
template <int H, int E, int K>
__device__ __noinline__ void exact_select(const uint16_t *router, const float *xin, const int *candf, double *tk,
                                          int *sel, bool nonfin) {
    const int tid = threadIdx.x;
    for (int e = tid; e < E; e += kThreads) {
        if (!candf[e]) continue;
        const uint16_t *row = router + (int64_t)e * H;
        float acc = 0.0f;
        for (int cc = 0; cc < H; cc++) acc = __fadd_rn(acc, __fmul_rn(bf16_to_f32(__ldg(row + cc)), xin[cc]));
        tk[e] = (double)acc;
    }
    __syncthreads();
    if (nonfin) {
        if (tid == 0) tk_insertion(tk, E, K, sel);
    } else {
        for (int e = tid; e < E; e += kThreads) {
            if (!candf[e]) continue;
            int r = 0;
            const double ve = tk[e];
            for (int f = 0; f < E; f++) r += candf[f] && (tk[f] > ve || (tk[f] == ve && f < e));
            if (r < K) sel[r] = e;
        }
    }
}

template <int FMT, int H, int M, int E, int K>
struct Smem {
    using S = Shape<FMT, H, M>;
    static constexpr int a16(int n) { return (n + 15) / 16 * 16; }
    static constexpr int RT = (E + kGmin - 1) / kGmin;          // router rows per CTA
    static constexpr int RR = (H + kGmin - 1) / kGmin;          // output rows per CTA
    static constexpr int PP = (K * M + kGmin - 1) / kGmin;      // gate/up pairs per CTA
    static constexpr int GSC = FMT == DS4F_FMT_FP8 ? kGroups * 2 * 2 * S::gsc_b   // [group][seg][mat]
                                                   : PP * 2 * S::gsc_b;          // [mat][pair]
    static constexpr int DSC = FMT == DS4F_FMT_FP8 ? S::dsc_b : a16(RR * S::dsc_b + 48);
    static_assert(PP <= kGroups * kGroupPairs, "gate/up pairs exceed the copy groups");
    static_assert(4 * RT <= 8 && M < 4 * kGmin && 2 * ((M + kGmin - 1) / kGmin) <= 8,
                  "warp roles: router rows in warps 0-7, shared rows in 8-15, gate logit in CTA 0 warp 15");
    static constexpr int o_bar = 0;                                   // 9 mbarriers (of 16 slots)
    static constexpr int o_xin = 128;
    static constexpr int o_nw = o_xin + a16(H * 4);
    static constexpr int o_rt = o_nw + a16(H * 2);
    static constexpr int o_sd = o_rt + a16(RT * H * 2);
    static constexpr int o_dn = o_sd + a16(RR * M * 2);
    static constexpr int o_dsc = o_dn + a16(K * RR * S::drow_b);
    // gate rows then up rows; between uses it receives the tagged-word
    // gathers (state, router logits, chains)
    // (the chain gather: (K+1) M chain words, the shared-gate logit and a
    // pad word)
    static constexpr int NCWP = (K + 1) * M + 2;
    static constexpr int GATH = 8 * ((H > 4 * E ? H : 4 * E) > NCWP ? (H > 4 * E ? H : 4 * E) : NCWP);
    // + the chains unpacked to floats after the tagged words
    static constexpr int UNP = GATH + 4 * ((K + 1) * M + 4);
    // + the next layer's shared gate/up rows and the shared-gate row, past
    // the gathers (they land during the down phase, are read in the router
    // phase, and are overwritten by the gate/up copies after that)
    static constexpr int NSG = (M + kGmin - 1) / kGmin;
    static constexpr int SHO = a16(UNP);
    static constexpr int SHB = 2 * NSG * H * 2 + H * 2;
    static constexpr int GU0 = 2 * PP * S::row_b > UNP ? 2 * PP * S::row_b : UNP;
    static constexpr int GU = GU0 > SHO + SHB ? GU0 : SHO + SHB;
    static constexpr int o_gu = o_dsc + a16(K * DSC);
    static constexpr int o_gsc = o_gu + a16(GU);
    static constexpr int o_srow = o_gsc + a16(GSC);
    static constexpr int o_outs = o_srow + a16(RR * 4);
    // 1 KB scratch: doubles [0, 64) for reductions and the top-k ranks,
    // floats [192, 200) for the shared gate/up partial sums
    static constexpr int o_red = o_outs + a16((K + 1) * RR * 4);
    static constexpr int o_tk = o_red + 1024;                         // [E] doubles
    static constexpr int o_cand = o_tk + a16(E * 8);                  // [E] ints
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
    uint32_t epoch;             // 1..65535, distinct from the previous launch's
    long spin;                  // polls of a copy barrier before giving up
    long rounds;                // copy rounds of a tagged-word gather before giving up
    int stall_cta, stall_t;     // test hook: this CTA withholds its state words
                                // at this layer-step (-1: off)
    int stall_peer_t;           // test hook (several GPUs): no down rows stored to the
                                // other GPUs at this layer-step (-1: off)
    // expert parallelism: this GPU's pool holds experts [efirst, efirst +
    // ecount) of every layer; world > 1: every rank's [2][K][H] tagged
    // down-output words (pout[rank] is this GPU's, the others peer mappings)
    int efirst, ecount, rank, world;
    int split_sel;              // 1: every GPU holds the whole pool and takes selections
                                // [rank K / world, (rank + 1) K / world); 0: its shard's
    int par0;                   // parity of this launch's first layer-step, counted over
                                // every fused launch (the words' buffer alternates per step)
    uint64_t *pout[kMaxRanks];
    float *state;               // [H] in (read at layer 0) / out (last layer)
    uint64_t *st_ll;            // [H] tagged state words
    uint64_t *sb_ll;            // [E][4] tagged words: S, its interval's ends (fp32), 0
    uint64_t *ch_ll;            // [(K+1) M + 2] tagged chains, the shared-gate logit, a pad word
    unsigned *diag;             // [4]: layers, fallbacks, error code, failing CTA
    unsigned long long *trace;  // optional [T][G][kTracePts] %globaltimer stamps
    int *log_idx;               // optional route log, layer-steps t < log_n:
    float *log_w;               //   selections [t][K], weights [t][K],
    float *log_state;           //   the layer's output state [t][H]
    int log_n;
};

__device__ __forceinline__ bool aborted(const DecodeArgs &a) {
    return *(volatile unsigned *)(a.diag + 2) != 0;
}
__device__ void give_up(const DecodeArgs &a, unsigned code) {
    if (atomicCAS(a.diag + 2, 0u, code) == 0u) a.diag[3] = blockIdx.x;
}

__device__ bool mbar_wait(const DecodeArgs &a, uint64_t *b, uint32_t parity, unsigned code) {
    long it = 0;
    while (!mbar_test(b, parity)) {
        if (++it > a.spin) { give_up(a, code); return false; }
        if (it > 16) __nanosleep(32);
    }
    return true;
}

// One thread: wait (bounded) until the word at p, written by another GPU,
// carries `tag`; its value in v. false after the limit or an abort.
__device__ bool poll_word(const DecodeArgs &a, const uint64_t *p, uint32_t tag, float &v) {
    for (long it = 0;; it++) {
        uint64_t w;
        asm volatile("ld.relaxed.sys.global.u64 %0, [%1];" : "=l"(w) : "l"(p) : "memory");
        if ((uint32_t)(w >> 32) == tag) { v = __uint_as_float((uint32_t)w); return true; }
        if (it > a.spin || ((it & 1023) == 1023 && aborted(a))) {
            if (!aborted(a)) give_up(a, 11);
            v = 0.f;
            return false;
        }
        if (it > 16) __nanosleep(64);
    }
}

// CTA-wide, every thread calls it: TMA-copy the tagged words src[0, n)
// into shared memory until the first `ncheck` of them carry `tag` (re-copy
// while any is still from an earlier layer); n is even (16-byte copies).
// One bulk copy per round instead of per-thread polls. false (uniformly)
// on timeout or abort.
// The first copy of a gather, issued ahead so the block can work while it
// is in flight (gather_ll with issued = true then waits for it).
__device__ __forceinline__ void gather_issue(uint64_t *bar, uint32_t &pendb, uint64_t *dst, const uint64_t *src,
                                             int n) {
    if (threadIdx.x == 0) {
        fence_async();
        mbar_expect(bar, n * 8);
        bulk(dst, src, n * 8, bar);
    }
    pendb |= 1u << 7;
}

// Copy n tagged words into dst until the first ncheck carry `tag`. Each
// round is one bulk copy and two block barriers (the copy's round trip
// spaces the polls); every 16th round also checks the limit and an abort.
// Words i < km belong to selection i >> mshift and are checked only where
// bit (i >> mshift) of locmask is set (a sharded model's chains of the
// selections another GPU holds are never written here).
__device__ bool gather_ll(const DecodeArgs &a, uint64_t *bar, uint32_t &phb, uint32_t &pendb,
                          uint64_t *dst, const uint64_t *src, int n, int ncheck, uint32_t tag,
                          unsigned code, unsigned long long *rounds = nullptr, bool issued = false,
                          int km = 0, int mshift = 0, unsigned locmask = ~0u) {
    const int tid = threadIdx.x;
    for (long it = 0;; it++) {
        if (rounds && tid == 0) *rounds = (unsigned long long)(it + 1);
        if (it > 0 || !issued) gather_issue(bar, pendb, dst, src, n);
        if (!__syncthreads_and(mbar_wait(a, bar, (phb >> 7) & 1u, code))) return false;
        phb ^= 1u << 7;
        pendb &= ~(1u << 7);
        bool all = true;
        for (int i = tid; i < ncheck; i += kThreads)
            all = all && ((i < km && !((locmask >> (i >> mshift)) & 1u)) || (uint32_t)(dst[i] >> 32) == tag);
        if (__syncthreads_and(all)) return true;
        if ((it & 15) == 15 && __syncthreads_or(it > a.rounds || aborted(a))) {
            if (tid == 0 && !aborted(a)) give_up(a, code);
            return false;
        }
    }
}

// EP: this GPU holds a shard of every layer's experts and exchanges the
// down outputs with the other GPUs (world > 1); false: the whole pool here.
// TR: record the phase trace. A separate instance: a layer's code does not
// fit in the instruction cache, and the ~30 stamps' code alone, branched
// over, cost 3.7 % of the step (1,343 vs 1,393 tok/s measured).
template <int FMT, int H, int M, int E, int K, bool EP, bool TR>
__global__ void __launch_bounds__(kThreads, 1)
k_decode(DecodeArgs a) {
    using S = Shape<FMT, H, M>;
    using L = Smem<FMT, H, M, E, K>;
    extern __shared__ __align__(128) unsigned char sm[];
    // bar 0: router rows + norm weights; 1: shared down rows;
    // 2..5: gate/up copy groups; 6: routed down rows; 7: tagged gathers
    uint64_t *bar = (uint64_t *)(sm + L::o_bar);
    float *xin = (float *)(sm + L::o_xin);
    uint16_t *nw = (uint16_t *)(sm + L::o_nw);
    uint16_t *rt = (uint16_t *)(sm + L::o_rt);
    uint16_t *sd = (uint16_t *)(sm + L::o_sd);
    uint8_t *dn = sm + L::o_dn;
    uint8_t *dsc = sm + L::o_dsc;
    uint8_t *gu = sm + L::o_gu;
    uint8_t *gsc = sm + L::o_gsc;
    float *srow = (float *)(sm + L::o_srow);
    float *outs = (float *)(sm + L::o_outs);
    float *red = (float *)(sm + L::o_red);
    double *tk = (double *)(sm + L::o_tk);
    int *candf = (int *)(sm + L::o_cand);
    int *sel = (int *)(sm + L::o_sel);
    float *wsel = (float *)(sel + 64);
    int *ctl = (int *)(wsel + 64);
    int *locs = ctl + 8;      // the selections held here, in selection order (ctl[4]: count, ctl[5]: mask)

    const int tid = threadIdx.x, lane = tid & 31, warp = tid >> 5;
    const int G = gridDim.x, c = blockIdx.x;
    const int rt0 = c * E / G, nrt = (c + 1) * E / G - rt0;
    const int sg0 = c * M / G, nsg = (c + 1) * M / G - sg0;
    // routed (selection, row) pairs: the CTA's slice of the nloc M pairs of
    // the selections this GPU holds (all K with every expert here), set per
    // layer once the routing is known (set_pairs)
    int nloc = K, p0 = c * (K * M) / G, np = (c + 1) * (K * M) / G - p0;
    unsigned lmask = (1u << K) - 1;     // bit j: selection j's expert is here
    const int r0 = c * H / G, nr = (c + 1) * H / G - r0;
    int ngroups = (np + kGroupPairs - 1) / kGroupPairs;
    auto set_pairs = [&](int nl) {
        nloc = nl;
        p0 = c * (nl * M) / G;
        np = (c + 1) * (nl * M) / G - p0;
        ngroups = (np + kGroupPairs - 1) / kGroupPairs;
    };

    // mbarrier i: its phase parity (bit i of phb) and whether a copy on it
    // is still in flight (bit i of pendb) -- two registers, not sixteen
    uint32_t phb = 0, pendb = 0;
#define PH(i) ((phb >> (i)) & 1u)
#define FLIP(i) (phb ^= 1u << (i))
#define PEND(i, v) (pendb = (v) ? (pendb | (1u << (i))) : (pendb & ~(1u << (i))))
    bool ok = true;

    if (tid == 0) {
        for (int i = 0; i < 9; i++) mbar_init(bar + i, 1);
        asm volatile("fence.mbarrier_init.release.cluster;" ::: "memory");
    }
    __syncthreads();

    auto trunk_l = [&](int l) { return a.trunk + (int64_t)l * a.trunk_n; };
    auto expert = [&](int l, int e) {
        return a.pool + ((int64_t)l * a.ecount + (e - a.efirst)) * a.slot_bytes;
    };
    auto tag_of = [&](int t) { return (a.epoch << 16) | (uint32_t)(t + 1); };

    // one thread: router rows + norm weights of layer l (bar 0)
    auto prefetch_rt = [&](int l) {
        const uint16_t *t = trunk_l(l);
        uint32_t b1 = nrt * H * 2;
        mbar_expect(bar + 0, b1 + H * 2);
        bulk(nw, t + a.tr.norm, H * 2, bar + 0);
        if (b1) bulk(rt, t + a.tr.router + (int64_t)rt0 * H, b1, bar + 0);
    };
    // one thread: shared gate rows, up rows of layer l (and the shared-gate
    // row in CTA 0) into gu + SHO (bar 8)
    auto prefetch_sh = [&](int l) {
        const uint16_t *t = trunk_l(l);
        const uint32_t b = nsg * H * 2;
        mbar_expect(bar + 8, 2 * b + (c == 0 ? H * 2 : 0));
        if (b) {
            bulk(gu + L::SHO, t + a.tr.sh_gate + (int64_t)sg0 * H, b, bar + 8);
            bulk(gu + L::SHO + L::NSG * H * 2, t + a.tr.sh_up + (int64_t)sg0 * H, b, bar + 8);
        }
        if (c == 0) bulk(gu + L::SHO + 2 * L::NSG * H * 2, t + a.tr.sh_gw, H * 2, bar + 8);
    };
    // one thread: shared down rows of layer l (bar 1)
    auto prefetch_sd = [&](int l) {
        uint32_t b = nr * M * 2;
        mbar_expect(bar + 1, b);
        if (b) bulk(sd, trunk_l(l) + a.tr.sh_down + (int64_t)r0 * M, b, bar + 1);
    };
    // Copies are issued two or three per warp by every warp: a warp's
    // lanes get one bulk copy accepted every ~57 cycles whatever its size,
    // while different warps issue side by side (32 copies: ~1,840 cycles
    // from one warp, ~400-800 from sixteen, measured on B200).
    // Copy k of gate/up group g of layer l (bar 2 + g), for
    // L = 8 g + k: a group is <= 2 segments (one per expert), each gate
    // rows (k & 3 == 0), up rows (1), gate scales (2), up scales (3).
    // Thread g of warp 0 sets group g's byte count first (expect_groups).
    // warp 0, once the routing is final: which selections' experts this GPU
    // holds (mask and count into ctl[5], ctl[4], their list in selection
    // order into locs) and this thread's pair slice
    auto route_local = [&]() {
        if constexpr (!EP) return;
        const bool here = lane < K && (a.split_sel ? lane >= a.rank * K / a.world && lane < (a.rank + 1) * K / a.world
                                                   : sel[lane] >= a.efirst && sel[lane] < a.efirst + a.ecount);
        const unsigned mk = __ballot_sync(0xFFFFFFFFu, here);
        if (here) locs[__popc(mk & ((1u << lane) - 1u))] = lane;
        if (lane == 0) { ctl[4] = __popc(mk); ctl[5] = (int)mk; }
        lmask = mk;
        set_pairs(__popc(mk));
        __syncwarp();
    };
    auto expect_groups = [&](int g) {
        const int q0 = p0 + g * kGroupPairs, q1 = min(q0 + kGroupPairs, p0 + np);
        if (g < ngroups) {
            uint32_t total = 0;
            for (int q = q0; q < q1;) {
                int i0 = q % M, n = min(q1 - q, M - i0);
                total += 2 * n * S::row_b + (FMT == DS4F_FMT_FP8 ? 2 * S::gsc_b : 2 * n * S::gsc_b);
                q += n;
            }
            mbar_expect(bar + 2 + g, total);
        }
    };
    auto issue_group_copy = [&](int l, int L) {
        const int g = L >> 3, sg = (L >> 2) & 1, kind = L & 3;
        const int q0 = p0 + g * kGroupPairs, q1 = min(q0 + kGroupPairs, p0 + np);
        const int split = min(q1, (q0 / M + 1) * M);
        if (g >= ngroups) return;
        const int qa = sg == 0 ? q0 : split, qb = sg == 0 ? split : q1;
        if (qa >= qb) return;
        const int j = EP ? locs[qa / M] : qa / M, i0 = qa % M, n = qb - qa, slot = qa - p0, mat = kind & 1;
        const uint8_t *ex = expert(l, sel[j]);
        if (kind < 2)
            bulk(gu + (mat * L::PP + slot) * S::row_b, ex + a.slot.rel_v[mat] + (int64_t)i0 * S::row_b,
                 n * S::row_b, bar + 2 + g);
        else if (FMT == DS4F_FMT_FP8)
            bulk(gsc + ((g * 2 + sg) * 2 + mat) * S::gsc_b, ex + a.slot.rel_s[mat], S::gsc_b, bar + 2 + g);
        else
            bulk(gsc + (mat * L::PP + slot) * S::gsc_b, ex + a.slot.rel_s[mat] + (int64_t)i0 * S::gsc_b,
                 n * S::gsc_b, bar + 2 + g);
    };
    // bytes of the routed down copies (rows + scales of K experts)
    const int sa0 = FMT == DS4F_FMT_FP8 ? 0 : (r0 * S::dsc_b) / 16 * 16;
    const int sab = FMT == DS4F_FMT_FP8 ? S::dsc_b : ((r0 + nr) * S::dsc_b + 15) / 16 * 16 - sa0;
    const uint32_t dn_sel = nr * S::drow_b + sab;      // per selection held here
    // copy 2 j + h < 2 K: down rows (h = 0) or scales (h = 1) of
    // selection j (bar 6)
    auto issue_down_copy = [&](int l, int L) {
        const int j = L >> 1;
        if (EP && !((lmask >> j) & 1u)) return;
        const uint8_t *ex = expert(l, sel[j]);
        if ((L & 1) == 0) {
            if (nr)
                bulk(dn + j * L::RR * S::drow_b, ex + a.slot.rel_v[2] + (int64_t)r0 * S::drow_b,
                     nr * S::drow_b, bar + 6);
        } else {
            bulk(dsc + j * L::DSC, ex + a.slot.rel_s[2] + sa0, sab, bar + 6);
        }
    };

    if (tid == 0) {
        prefetch_rt(0);
        prefetch_sd(0);
        prefetch_sh(0);
    }
    pendb |= 3u | (1u << 8);

    const int T = a.n_layers * a.n_steps;
#define DS4F_TRACE(k) \
    if constexpr (TR) { if (tid == 0) a.trace[((int64_t)t * G + c) * kTracePts + (k)] = gtimer(); }
#define DS4F_ROUNDS(k) (TR ? a.trace + ((int64_t)t * G + c) * kTracePts + (k) : nullptr)
    for (int t = 0; t < T; t++) {
        const int l = t % a.n_layers, ln = (t + 1) % a.n_layers;
        const bool more = t + 1 < T;
        const uint32_t tg = tag_of(t);            // words this layer publishes
        DS4F_TRACE(0);
        // (A) input state: PER words per thread
        {
            constexpr int PER = (H + kThreads - 1) / kThreads;
            float v[PER];
            bool got = true;
            if (t == 0) {
#pragma unroll
                for (int k = 0; k < PER; k++)
                    v[k] = (tid + k * kThreads < H) ? __ldcg(a.state + tid + k * kThreads) : 0.f;
            } else {
                static_assert(H % kThreads == 0, "state words split evenly over threads");
                const uint64_t *sw = (const uint64_t *)gu;
                got = gather_ll(a, bar + 7, phb, pendb, (uint64_t *)gu, a.st_ll, H, H,
                                tag_of(t - 1), 1, DS4F_ROUNDS(14));
#pragma unroll
                for (int k = 0; k < PER; k++) v[k] = __uint_as_float((uint32_t)sw[tid + k * kThreads]);
            }
            double ss = 0.0;
#pragma unroll
            for (int k = 0; k < PER; k++) {
                const int i = tid + k * kThreads;
                if (i < H) {
                    xin[i] = v[k];
                    if (i >= r0 && i < r0 + nr) srow[i - r0] = v[k];
                    double d = (double)v[k];
                    ss = __dadd_rn(ss, __dmul_rn(d, d));
                }
            }
            ss = warp_sum_d(ss);
            double *rd = (double *)red;
            if (lane == 0) rd[warp] = ss;
            if (!got) { ok = false; break; }          // uniform: gather_ll's result
            __syncthreads();
            DS4F_TRACE(1);
            if (tid == 0) {
                double s2 = 0.0;
                for (int k = 0; k < kWarps; k++) s2 = __dadd_rn(s2, rd[k]);
                rd[16] = s2;
            }
            // (B) norm weights arrive with the router rows (bar 0)
            bool okb = mbar_wait(a, bar + 0, PH(0), 2);
            if (!__syncthreads_and(okb)) { ok = false; break; }
            FLIP(0); PEND(0, false);
            float r = __fsqrt_rn(__fadd_rn(__double2float_rn(__ddiv_rn(rd[16], (double)H)), 1e-6f));
            for (int i = tid; i < H; i += kThreads)
                xin[i] = __fmul_rn(__fdiv_rn(xin[i], r), bf16_to_f32(nw[i]));
            __syncthreads();
        }
        DS4F_TRACE(2);
        // (C) router rows: warps RW r .. RW r + RW - 1 take row r (r < nrt),
        //     warp q the columns [q H/RW, (q+1) H/RW), lane l 8 contiguous
        //     columns of them (RW = H / 256). The chunk sums and each warp's
        //     total give each lane its exact column-order prefix for the
        //     bound (named barrier over the router warps only).
        constexpr int RW = H / 256;
        static_assert(RW * 2 <= kWarps, "two router rows per CTA at most");
        if (warp < RW * nrt) {
            constexpr int CQ = H / RW;
            static_assert(CQ == 256, "router rows: one 8-element chunk per lane");
            const int rr = warp / RW, q = warp % RW, e = rt0 + rr, nrw = 32 * RW * nrt;
            const int c0 = q * CQ + lane * 8;
            const uint16_t *row = rt + rr * H + c0;
            uint4 w = lds16(row);
            const uint32_t ww[4] = {w.x, w.y, w.z, w.w};
            const float4 x0 = *(const float4 *)(xin + c0);
            const float4 x1 = *(const float4 *)(xin + c0 + 4);
            const float x[8] = {x0.x, x0.y, x0.z, x0.w, x1.x, x1.y, x1.z, x1.w};
            double p8[8];
            // the bound's |p| (8 - u) terms: positive, summed in fp32 (8 terms
            // per lane, relative error < 1e-6, inside the 1.001 margin)
            float ab = 0.f;
#pragma unroll
            for (int u = 0; u < 8; u++) {
                uint32_t h = (u & 1) ? (ww[u >> 1] & 0xFFFF0000u) : (ww[u >> 1] << 16);
                float pr = __fmul_rn(__uint_as_float(h), x[u]);   // the reference's product
                p8[u] = (double)pr;
                ab = fmaf(fabsf(pr), (float)(8 - u), ab);
            }
            const double tot = __dadd_rn(__dadd_rn(__dadd_rn(p8[0], p8[1]), __dadd_rn(p8[2], p8[3])),
                                         __dadd_rn(__dadd_rn(p8[4], p8[5]), __dadd_rn(p8[6], p8[7])));
            double incl = tot;
#pragma unroll
            for (int o = 1; o < 32; o <<= 1) {
                double y = __shfl_up_sync(0xFFFFFFFFu, incl, o);
                if (lane >= o) incl = __dadd_rn(incl, y);
            }
            double *rx = (double *)red + 32;      // [row][warp] totals, then at +2 RW bound parts
            if (lane == 31) rx[rr * RW + q] = incl;
            asm volatile("bar.sync 1, %0;" ::"r"(nrw) : "memory");
            double P = __dsub_rn(incl, tot);      // prefix before this lane within the warp
            for (int k = 0; k < q; k++) P = __dadd_rn(rx[rr * RW + k], P);
            double bs = __dadd_rn(8.0 * fabs(P), (double)ab);
            bs = warp_sum_d(bs);
            if (lane == 0) rx[2 * RW + rr * RW + q] = bs;
            asm volatile("bar.sync 1, %0;" ::"r"(nrw) : "memory");
            if (q == 0 && lane < 4) {
                double Sv = 0.0, Bs = 0.0;
                for (int k = 0; k < RW; k++) {
                    Sv = __dadd_rn(Sv, rx[rr * RW + k]);
                    Bs = __dadd_rn(Bs, rx[2 * RW + rr * RW + k]);
                }
                // the prefixes carry double rounding of their own: widen by 1e-12
                const double Bv = 1.001 * kU * (Bs * (1.0 + 1e-12)) + 1e-300;
                // published as fp32: S rounded to nearest (the softmax input and
                // the selection key), the interval [S - B, S + B] rounded
                // outward (still a certificate, wider by at most an ulp)
                const float sf = __double2float_rn(Sv);
                const float lf = __double2float_rd(__dsub_rd(Sv, Bv));
                const float hf = __double2float_ru(__dadd_ru(Sv, Bv));
                const uint32_t word = lane == 0 ? __float_as_uint(sf) : lane == 1 ? __float_as_uint(lf)
                                    : lane == 2 ? __float_as_uint(hf) : 0u;
                st_tag(a.sb_ll + 4 * e + lane, tg, word);
            }
        }
        DS4F_TRACE(3);
        static_assert(E % 32 == 0 && (4 * E * 8) % 16 == 0, "router width: whole warps of experts");
        // (D) shared gate (even) / up (odd) rows and, CTA 0 warp 15, the
        //     shared-gate row: prefetched into shared memory (bar 8)
        if (warp < 2 * nsg || (warp == kWarps - 1 && c == 0)) {
            const bool okd = mbar_wait(a, bar + 8, PH(8), 9);
            const bool gl = warp == kWarps - 1 && c == 0;   // CTA 0 has < 4 shared rows
            const int w2 = warp, m = w2 & 1;
            const uint16_t *row = (const uint16_t *)(gu + L::SHO) +
                                  (gl ? 2 * L::NSG * H : (m * L::NSG + (w2 >> 1)) * H);
            float acc = 0.f;
            if (okd) {
#pragma unroll
                for (int k = 0; k < H / 256; k++)
                    acc += bf16_dot8(lds16(row + (lane + 32 * k) * 8), xin + (lane + 32 * k) * 8);
            }
            acc = warp_sum(acc);
            if (lane == 0 && okd) {
                if (gl) {
                    st_tag(a.ch_ll + (K + 1) * M, tg, __float_as_uint(acc));
                    st_tag(a.ch_ll + (K + 1) * M + 1, tg, 0u);     // the pad word
                }
                else red[192 + w2] = acc;       // bytes 768..: clear of rd[0..63]
            }
        }
        FLIP(8);
        PEND(8, false);
        // the router-logit gather's first copy goes out only now: issued
        // before the shared rows (to fly while they are computed) it landed
        // before most CTAs' words were visible and nearly always needed a
        // second round (1.95 vs 1.38 rounds; 1,318 -> 1,341 tok/s). Its words
        // land in the gathers' region, clear of the shared rows; the last
        // reads of that region, the state words, were ordered by the
        // barriers of (B).
        gather_issue(bar + 7, pendb, (uint64_t *)gu, a.sb_ll, 4 * E);
        // (F) routing: gather every S/B word, then warp 0 takes the
        //     certified top-K
        if (!gather_ll(a, bar + 7, phb, pendb, (uint64_t *)gu, a.sb_ll, 4 * E, 4 * E, tg, 3,
                       DS4F_ROUNDS(15), true)) {
            ok = false;
            break;
        }
        DS4F_TRACE(18);        // every router word visible; the top-K follows
        if (warp == 0) {
            constexpr int NE = E / 32;
            static_assert(K == 8 && NE <= 8, "the sorting network selects 8");
            // expert e's words 4e .. 4e+2: S, and its interval's ends (fp32)
            const uint64_t *sbw = (const uint64_t *)gu;
            auto word_f = [&](int w) { return __uint_as_float((uint32_t)sbw[w]); };
            // the first 8 by key in selection order, in every lane (lane l
            // starts from experts l + 32 i)
            static_assert(E <= 256, "expert index in the key's low byte");
            uint32_t k8[8];
            bool fin = true;
#pragma unroll
            for (int i = 0; i < 8; i++) {
                k8[i] = 0u;
                if (i < NE) {
                    const int e = lane + 32 * i;
                    const float sv = word_f(4 * e);
                    k8[i] = tk_key(sv, e);
                    tk[e] = (double)sv;
                    fin = fin && isfinite(sv) && isfinite(word_f(4 * e + 1)) && isfinite(word_f(4 * e + 2));
                }
            }
            // a logit that is not finite: no interval orders it; every
            // expert's exact logit then goes through the reference's own
            // insertion rule (tk_insertion) in the fallback below
            const bool nonfin = !__all_sync(0xFFFFFFFFu, fin);
            if (lane == 0) { ctl[3] = 1; ctl[1] = 0; ctl[2] = nonfin ? 1 : 0; }
            DS4F_TRACE(27);
            tk_sort8(k8);
            tk_warp_top8(k8);
            DS4F_TRACE(28);
            // lane r < 8: the r-th selection's interval
            int er = 0;
#pragma unroll
            for (int j = 0; j < 8; j++) if (j == lane) er = tk_expert(k8[j]);
            float lor = 3.0e38f, hir = -3.0e38f;
            if (lane < K) {
                lor = word_f(4 * er + 1);
                hir = word_f(4 * er + 2);
            }
            // certified when consecutive selections' intervals separate and
            // only the 8 selections reach the last one's lower bound (then
            // every reference-order logit ranks the same); otherwise the
            // exact fallback recomputes every expert whose interval reaches
            // the lowest lower bound among the 8 (a superset of the true 8)
            const float hin = __shfl_down_sync(0xFFFFFFFFu, hir, 1);
            const bool sep = lane >= K - 1 || lor > hin;
            const float lo8 = __shfl_sync(0xFFFFFFFFu, lor, K - 1);
            float lmin = lor;
#pragma unroll
            for (int o = 16; o > 0; o >>= 1) lmin = fminf(lmin, __shfl_xor_sync(0xFFFFFFFFu, lmin, o));
            int nmine = 0;
#pragma unroll
            for (int i = 0; i < NE; i++) {
                const int e = lane + 32 * i;
                const float hi = word_f(4 * e + 2);
                nmine += hi >= lo8;
                candf[e] = a.exact_all || nonfin || hi >= lmin;
            }
            const int nreach = (int)__reduce_add_sync(0xFFFFFFFFu, (unsigned)nmine);
            const bool cert = !a.exact_all && !nonfin && __all_sync(0xFFFFFFFFu, sep) && nreach == K;
            DS4F_TRACE(29);
            if (cert && lane < K) sel[lane] = er;
            if (lane == 0) ctl[1] = cert ? 1 : 0;
            if (cert) {
                // the routing is final: the selections held here, the byte
                // counts of this layer's copies, then group 0's copies at
                // once (the other groups follow from the other warps after
                // the barrier below, the down rows after group 0's dots: the
                // first group lands first)
                __syncwarp();
                route_local();
                if (lane < kGroups) expect_groups(lane);
                if (lane == kGroups) mbar_expect(bar + 6, (EP ? nloc : K) * dn_sel);
                __syncwarp();
                DS4F_TRACE(30);
                if (lane < 8) { fence_async(); issue_group_copy(l, lane); }
                DS4F_TRACE(31);
            }
        }
        // ctl[] is read after the barrier (a __syncthreads_and predicate
        // would be evaluated before warp 0 wrote it)
        __syncthreads();
        if (!ctl[3]) { ok = false; break; }
        DS4F_TRACE(4);
        if (tid < nsg)          // needed in the down phase only: no flush
            st_tag(a.ch_ll + K * M + sg0 + tid, tg,
                   __float_as_uint(silu_mul(red[192 + 2 * tid], red[192 + 2 * tid + 1])));
        if (!ctl[1]) {
            exact_select<H, E, K>(trunk_l(l) + a.tr.router, xin, candf, tk, sel, ctl[2] != 0);
            if (tid == 0 && !a.exact_all && c == 0) atomicAdd(a.diag + 1, 1u);
            __syncthreads();
            if (warp == 0) {
                route_local();
                if (lane < kGroups) expect_groups(lane);
                if (lane == kGroups) mbar_expect(bar + 6, (EP ? nloc : K) * dn_sel);
            }
            __syncthreads();
            if (tid < 8) { fence_async(); issue_group_copy(l, tid); }
        }
        // every thread: this layer's selections held here and its pairs
        if constexpr (EP) {
            lmask = (unsigned)ctl[5];
            set_pairs(ctl[4]);
        }
        DS4F_TRACE(5);
        // (G) the gate/up copies of groups 1.. (group 0's went out with the
        //     routing): warp w >= 1 issues copies 8 + 2 (w - 1) + (0, 1)
        //     (lanes 0, 1); the last warp also the next layer's router rows +
        //     norm weights (buffers (B) and (C) are done with). Their last
        //     readers (the previous layer's gate/up, the top-k's look at the
        //     router words) are ordered by the barriers above. The down copies
        //     go out after group 0's dots (every warp's lane 2, copy w), or
        //     here when the CTA has no gate/up pairs.
        static_assert(kGroups * 8 <= 8 + 2 * (kWarps - 1) && 2 * K == kWarps, "copy roles");
        if (warp >= 1 && lane < 2 && 8 + 2 * (warp - 1) + lane < kGroups * 8) {
            fence_async();
            issue_group_copy(l, 8 + 2 * (warp - 1) + lane);
        } else if (lane == 2 && ngroups == 0) {
            fence_async();
            issue_down_copy(l, warp);
        } else if (lane == 3 && warp == kWarps - 1 && more) {
            fence_async();
            prefetch_rt(ln);
        }
#pragma unroll
        for (int g = 0; g < kGroups; g++) PEND(2 + g, g < ngroups);
        PEND(6, true);
        PEND(0, more);
        DS4F_TRACE(6);
        asm volatile("" ::: "memory");        // keep the x loads below the issue code
        // x registers of the gate/up granules: warp w covers column half
        // w / 8; lane l holds elements (32 j + l) gb + u of its granules j,
        // pre-scaled by 2^64 (16-byte reads, consecutive lanes consecutive
        // addresses)
        constexpr int NGH = S::ng / 2;
        static_assert(S::ng % 2 == 0 && kWarps == 2 * kGroupPairs, "two column halves per pair");
        const int hcol = warp >> 3;
        float xr[NGH * S::gb];
#pragma unroll
        for (int j = 0; j < NGH; j++)
#pragma unroll
            for (int u = 0; u < S::gb; u += 4) {
                const float4 v = *(const float4 *)(xin + (32 * (hcol * NGH + j) + lane) * S::gb + u);
                xr[j * S::gb + u] = v.x * DS4F_X_PRESCALE;
                xr[j * S::gb + u + 1] = v.y * DS4F_X_PRESCALE;
                xr[j * S::gb + u + 2] = v.z * DS4F_X_PRESCALE;
                xr[j * S::gb + u + 3] = v.w * DS4F_X_PRESCALE;
            }
        if (warp == kWarps - 1) {
            // softmax over all E (double, max subtracted) and the renorm
            // (src/moe.c:531-561 + norm_topk_prob); wsel is read after the
            // gate/up phase's barriers
            constexpr int NE = E / 32;
            double mx = -1e300;
#pragma unroll
            for (int i = 0; i < NE; i++) mx = fmax(mx, tk[lane + 32 * i]);
#pragma unroll
            for (int o = 16; o > 0; o >>= 1) mx = fmax(mx, __shfl_xor_sync(0xFFFFFFFFu, mx, o));
            double sw = 0.0;
#pragma unroll
            for (int i = 0; i < NE; i++) sw += exp(tk[lane + 32 * i] - mx);
            sw = warp_sum_d(sw);
            const float wj = lane < K ? (float)(exp(tk[sel[lane]] - mx) / sw) : 0.0f;
            float s = 0.0f;
            for (int j = 0; j < K; j++) s = __fadd_rn(s, __shfl_sync(0xFFFFFFFFu, wj, j));
            if (lane < K) wsel[lane] = (a.renorm && s > 0.0f) ? __fdiv_rn(wj, s) : wj;
            if (lane == 0 && c == 0) atomicAdd(a.diag, 1u);
            if (a.log_idx && c == 0 && t < a.log_n && lane < K) {
                a.log_idx[(int64_t)t * K + lane] = sel[lane];
                a.log_w[(int64_t)t * K + lane] = wsel[lane];
            }
        }
        DS4F_TRACE(7);
        // (H) gate/up: warp w -> pair w % 8 of every group, gate and up
        //     rows over column half w / 8 (the two halves meet in red[]);
        //     each warp takes a group as soon as it has landed (its own wait,
        //     no block barrier)
        {
            unsigned landed = 0;
            if (TR && tid == 0)
                for (int g = 0; g < ngroups; g++) landed |= (unsigned)mbar_test(bar + 2 + g, PH(2 + g)) << g;
            if (TR && tid == 0) a.trace[((int64_t)t * G + c) * kTracePts + 17] = landed;
            const int ps = warp & 7;
            bool okg = true;
#pragma unroll 1
            for (int g = 0; g < ngroups; g++) {
                okg = mbar_wait(a, bar + 2 + g, PH(2 + g), 4);
                if (!okg) break;
                if (g == 0) {
                    DS4F_TRACE(8);
                } else {
                    DS4F_TRACE(20 + g);
                }
                // rows past the CTA's pairs read slot 0 and are dropped
                const int q0 = p0 + g * kGroupPairs;
                const bool valid = ps < min(kGroupPairs, p0 + np - q0);
                const int q = valid ? q0 + ps : p0, slot = q - p0;
                const uint8_t *rg = gu + slot * S::row_b, *ru = gu + (L::PP + slot) * S::row_b;
                float ag, au;
                if constexpr (FMT == DS4F_FMT_FP8) {
                    // granule j lies in column block j: one scale per warp
                    const int seg = valid ? q / M - q0 / M : 0;
                    const int sb = (((valid ? g : 0) * 2 + seg) * 2) * S::gsc_b;
                    const float *sg = (const float *)(gsc + sb) + ((q % M) >> 7) * (H / 128) + hcol * NGH;
                    const float *su = (const float *)(gsc + sb + S::gsc_b) + ((q % M) >> 7) * (H / 128) + hcol * NGH;
                    float2 g2 = make_float2(0.f, 0.f), u2 = make_float2(0.f, 0.f);
#pragma unroll
                    for (int j = 0; j < NGH; j++) {
                        const int off = (32 * (hcol * NGH + j) + lane) * 4;
                        const float2 x01 = make_float2(xr[4 * j], xr[4 * j + 1]);
                        const float2 x23 = make_float2(xr[4 * j + 2], xr[4 * j + 3]);
                        g2 = f8_fma4(*(const uint32_t *)(rg + off), x01, x23, sg[j], g2);
                        u2 = f8_fma4(*(const uint32_t *)(ru + off), x01, x23, su[j], u2);
                    }
                    ag = (g2.x + g2.y) * DS4F_X_UNSCALE;
                    au = (u2.x + u2.y) * DS4F_X_UNSCALE;
                } else {
                    const uint8_t *s4g = gsc + slot * S::gsc_b, *s4u = gsc + (L::PP + slot) * S::gsc_b;
                    float eg = 0.f, eu = 0.f;
#pragma unroll
                    for (int j = 0; j < NGH; j++) {
                        const int gi = 32 * (hcol * NGH + j) + lane;
                        eg = fmaf(e2m1_dot8c(*(const uint32_t *)(rg + 4 * gi), xr + 8 * j), e8m0_to_f32(s4g[gi >> 2]), eg);
                        eu = fmaf(e2m1_dot8c(*(const uint32_t *)(ru + 4 * gi), xr + 8 * j), e8m0_to_f32(s4u[gi >> 2]), eu);
                    }
                    ag = eg * DS4F_E2M1_POST;
                    au = eu * DS4F_E2M1_POST;
                }
#pragma unroll
                for (int o = 16; o > 0; o >>= 1) {
                    ag += __shfl_xor_sync(0xFFFFFFFFu, ag, o);
                    au += __shfl_xor_sync(0xFFFFFFFFu, au, o);
                }
                // red[] floats: [half][group][pair][gate, up]
                if (lane == 0) {
                    red[((hcol * kGroups + g) * kGroupPairs + ps) * 2] = ag;
                    red[((hcol * kGroups + g) * kGroupPairs + ps) * 2 + 1] = au;
                }
                if (g == 0 && lane == 2) { fence_async(); issue_down_copy(l, warp); }
            }
            DS4F_TRACE(24);
            if (!__syncthreads_and(okg)) { ok = false; break; }
            DS4F_TRACE(25);
#pragma unroll
            for (int g = 0; g < kGroups; g++)
                if (g < ngroups) { FLIP(2 + g); PEND(2 + g, false); }
            // the gate/up rows are consumed: the next layer's shared rows
            // may land past the gathers' region of the buffer
            if (tid == 0 && more) { fence_async(); prefetch_sh(ln); }
            PEND(8, more);
            if (tid < np) {
                constexpr int HALF = kGroups * kGroupPairs * 2;
                const int q = p0 + tid;
                st_tag(a.ch_ll + (EP ? locs[q / M] : q / M) * M + (q % M), tg,
                       __float_as_uint(silu_mul(red[2 * tid] + red[HALF + 2 * tid],
                                                red[2 * tid + 1] + red[HALF + 2 * tid + 1])));
                publish_flush();
            }
        }
        DS4F_TRACE(9);
        // (I) down rows: routed (bar 6) and shared (bar 1); chains polled
        {
            const bool okd = mbar_wait(a, bar + 6, PH(6), 6) && mbar_wait(a, bar + 1, PH(1), 7);
            if (!__syncthreads_and(okd)) { ok = false; break; }
            FLIP(6); PEND(6, false);
            FLIP(1); PEND(1, false);
            DS4F_TRACE(10);
            // every chain word (routed, shared, then the shared-gate logit)
            // into shared memory, over the gate/up rows (H) is done with
            // (K+1) M chain words + the logit, copied as an even count (the
            // workspace allocation is padded past the last word)
            constexpr int NCW = (K + 1) * M + 1;
            static_assert(L::NCWP == NCW + 1 && L::NCWP % 2 == 0, "even gathers");
            static_assert((M & (M - 1)) == 0, "chain words of selection j: j << log2 M ..");
            constexpr int MSH = __builtin_ctz(M);
            if (!gather_ll(a, bar + 7, phb, pendb, (uint64_t *)gu, a.ch_ll, L::NCWP, NCW, tg, 5, DS4F_ROUNDS(16), false, EP ? K * M : 0, MSH, lmask)) {
                ok = false;
                break;
            }
            // the values next to the words, routed chains pre-scaled by 2^64
            float *chf = (float *)(gu + L::GATH);
            {
                const uint64_t *chw = (const uint64_t *)gu;
                for (int i = tid; i < NCW; i += kThreads) {
                    const float v = __uint_as_float((uint32_t)chw[i]);
                    chf[i] = i < K * M ? v * DS4F_X_PRESCALE : v;
                }
            }
            __syncthreads();
            DS4F_TRACE(12);
            // row-dots: warp w takes up to 8 of the CTA's output rows of
            // routed selection w / 2 (rows [(w & 1) hr, ...), hr = ceil(nr / 2))
            // and shared-expert row w. Lane l reads granules 32 g + l of each
            // row against the chain's matching floats, held in registers; the
            // 8 rows' lane partials then meet in one butterfly (9 shuffles for
            // 8 sums), the shared row's in a warp sum.
            static_assert(kWarps == 2 * K && L::RR <= 16 && L::RR <= kWarps, "row-dot warp roles");
            constexpr int XC = S::dg * S::gb;
            static_assert(4 * S::bn <= 16 && XC <= 16, "at most 16 chain floats per lane");
            {
                const int jw = warp >> 1, hr = (nr + 1) >> 1;
                const int rw0 = (warp & 1) * hr, nrw = (!EP || ((lmask >> jw) & 1u)) ? min(hr, nr - rw0) : 0;
                float xc[XC], xs[4 * S::bn];
#pragma unroll
                for (int g = 0; g < S::dg; g++)
#pragma unroll
                    for (int u = 0; u < S::gb; u += 4) {
                        const float4 v4 = *(const float4 *)(chf + jw * M + (32 * g + lane) * S::gb + u);
                        xc[g * S::gb + u] = v4.x; xc[g * S::gb + u + 1] = v4.y;
                        xc[g * S::gb + u + 2] = v4.z; xc[g * S::gb + u + 3] = v4.w;
                    }
#pragma unroll
                for (int g = 0; g < S::bn; g++) {
                    const float4 v4 = *(const float4 *)(chf + K * M + 4 * (32 * g + lane));
                    xs[4 * g] = v4.x; xs[4 * g + 1] = v4.y; xs[4 * g + 2] = v4.z; xs[4 * g + 3] = v4.w;
                }
                // the lane partial of routed row rr of selection jw
                auto row_part = [&](int rr) -> float {
                    const uint8_t *row = dn + (jw * L::RR + rr) * S::drow_b;
                    if constexpr (FMT == DS4F_FMT_FP8) {
                        // granule g lies in column block g
                        const float *sc = (const float *)(dsc + jw * L::DSC) + ((r0 + rr) >> 7) * (M / 128);
                        float2 a2 = make_float2(0.f, 0.f);
#pragma unroll
                        for (int g = 0; g < S::dg; g++)
                            a2 = f8_fma4(*(const uint32_t *)(row + 4 * (32 * g + lane)),
                                         make_float2(xc[4 * g], xc[4 * g + 1]),
                                         make_float2(xc[4 * g + 2], xc[4 * g + 3]), sc[g], a2);
                        return (a2.x + a2.y) * DS4F_X_UNSCALE;
                    } else {
                        const uint8_t *s4 = dsc + jw * L::DSC + (r0 + rr) * S::dsc_b - sa0;
                        float v = 0.f;
#pragma unroll
                        for (int g = 0; g < S::dg; g++) {
                            const int q = 32 * g + lane;
                            v = fmaf(e2m1_dot8c(*(const uint32_t *)(row + 4 * q), xc + 8 * g),
                                     e8m0_to_f32(s4[q >> 2]), v);
                        }
                        return v * DS4F_E2M1_POST;
                    }
                };
                float pv[8];
#pragma unroll
                for (int i = 0; i < 8; i++) pv[i] = i < nrw ? row_part(rw0 + i) : 0.f;
                float sh = 0.f;
                if (warp < nr) {
                    const uint16_t *row = sd + warp * M;
#pragma unroll
                    for (int g = 0; g < S::bn; g++)
                        sh += bf16_dot4(*(const uint2 *)(row + 4 * (32 * g + lane)),
                                        make_float4(xs[4 * g], xs[4 * g + 1], xs[4 * g + 2], xs[4 * g + 3]));
                }
                if (warp == 0) DS4F_TRACE(26);
                // butterfly: after the step at offset 16 a lane holds 4 rows'
                // partials (bit 4 picks the half), at 8 two, at 4 one; offsets
                // 2 and 1 finish that row's sum, row = 4 b4 + 2 b3 + b2
                const bool b4 = lane & 16, b3 = lane & 8, b2 = lane & 4;
                float w4[4];
#pragma unroll
                for (int i = 0; i < 4; i++) {
                    const float r = __shfl_xor_sync(0xFFFFFFFFu, b4 ? pv[i] : pv[i + 4], 16);
                    w4[i] = (b4 ? pv[i + 4] : pv[i]) + r;
                }
                float w2[2];
#pragma unroll
                for (int i = 0; i < 2; i++) {
                    const float r = __shfl_xor_sync(0xFFFFFFFFu, b3 ? w4[i] : w4[i + 2], 8);
                    w2[i] = (b3 ? w4[i + 2] : w4[i]) + r;
                }
                float z = (b2 ? w2[1] : w2[0]) + __shfl_xor_sync(0xFFFFFFFFu, b2 ? w2[0] : w2[1], 4);
                z += __shfl_xor_sync(0xFFFFFFFFu, z, 2);
                z += __shfl_xor_sync(0xFFFFFFFFu, z, 1);
                sh = warp_sum(sh);
                const int slot = (b4 ? 4 : 0) + (b3 ? 2 : 0) + (b2 ? 1 : 0);
                if ((lane & 3) == 0 && slot < nrw) {
                    outs[jw * L::RR + rw0 + slot] = z;
                    if constexpr (EP) {
                        // several GPUs: the row goes to every other GPU at once
                        // (their words for layer parity (par0 + t) & 1), plain
                        // stores into its memory; the others' arrive in ours
                        const int64_t par = (int64_t)((a.par0 + t) & 1) * K * H;
                        for (int p = 0; p < a.world; p++)
                            if (p != a.rank && t != a.stall_peer_t)
                                st_tag_sys(a.pout[p] + par + jw * H + r0 + rw0 + slot, tg, __float_as_uint(z));
                    }
                }
                if (lane == 0 && warp < nr) outs[K * L::RR + warp] = sh;
            }
            DS4F_TRACE(13);
            if (tid == 0) red[0] = sigmoid_ref(chf[(K + 1) * M]);
            __syncthreads();
            // several GPUs: the other GPUs' rows of this CTA's selections
            // they hold into outs[] (read below exactly as this GPU's own)
            if (EP && tid < nr) {
                DS4F_TRACE(19);
                // every word read at once (one round trip), then only the
                // ones not yet there polled
                const uint64_t *base = a.pout[a.rank] + (int64_t)((a.par0 + t) & 1) * K * H + r0 + tid;
                uint64_t w[K];
#pragma unroll
                for (int j = 0; j < K; j++) w[j] = ((lmask >> j) & 1u) ? 0ull : ld_sys(base + (int64_t)j * H);
#pragma unroll
                for (int j = 0; j < K; j++) {
                    if ((lmask >> j) & 1u) continue;
                    float v = __uint_as_float((uint32_t)w[j]);
                    if ((uint32_t)(w[j] >> 32) != tg) poll_word(a, base + (int64_t)j * H, tg, v);
                    outs[j * L::RR + tid] = v;
                }
                DS4F_TRACE(20);
            }
            // selection-order combine (src/moe.c:1224-1225), shared gate
            // (:1279-1282), residual (:1424); a selection held elsewhere
            // contributes the word its GPU stored here
            if (tid < nr) {
                const int r = r0 + tid;
                float acc = 0.0f;
                for (int j = 0; j < K; j++) acc = __fadd_rn(acc, __fmul_rn(wsel[j], outs[j * L::RR + tid]));
                acc = __fadd_rn(acc, __fmul_rn(red[0], outs[K * L::RR + tid]));
                const float ns = __fadd_rn(srow[tid], acc);
                if (c != a.stall_cta || t != a.stall_t) {
                    st_tag(a.st_ll + r, tg, __float_as_uint(ns));
                    publish_flush();
                }
                if (!more) __stcg(a.state + r, ns);
                if (a.log_state && t < a.log_n) __stcg(a.log_state + (int64_t)t * H + r, ns);
            }
            __syncthreads();
        }
        DS4F_TRACE(11);        // (stamps 12, 13: inside the down phase, above)
        if (tid == 0 && more) { fence_async(); prefetch_sd(ln); }
        PEND(1, more);
    }
    // drain this CTA's copies before exit (bounded)
    for (int i = 0; i < 9; i++)
        if ((pendb >> i) & 1u) mbar_wait(a, bar + i, PH(i), 8);
#undef DS4F_TRACE
#undef DS4F_ROUNDS
#undef PH
#undef FLIP
#undef PEND
}

template <int FMT, int H, int M, int E, int K>
int launch_t(Model *m, float *state, int n_steps, cudaStream_t st, const DecodePeers *pe) {
    using L = Smem<FMT, H, M, E, K>;
    static_assert(L::bytes <= 227 * 1024, "decode kernel shared memory over budget");
    static SmemOptIn opt[4];
    const bool ep = pe && pe->world > 1;
    decltype(&k_decode<FMT, H, M, E, K, false, false>) kerns[4] = {
        k_decode<FMT, H, M, E, K, false, false>, k_decode<FMT, H, M, E, K, true, false>,
        k_decode<FMT, H, M, E, K, false, true>, k_decode<FMT, H, M, E, K, true, true>};
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
    a.E = E;
    a.efirst = m->d.expert_first;
    a.ecount = m->d.expert_count;
    a.rank = pe ? pe->rank : 0;
    a.world = pe ? pe->world : 1;
    a.split_sel = pe ? pe->split_sel : 0;
    for (int p = 0; p < kMaxRanks; p++) a.pout[p] = pe && p < pe->world ? pe->out[p] : nullptr;
    int *epoch = pe ? pe->epoch : &m->epoch;
    int64_t lsteps0 = 0;
    int64_t *lsteps = pe ? pe->lsteps : &lsteps0;
    a.renorm = m->d.renorm;
    a.exact_all = m->d.router_exact;
    a.st_ll = m->w.st_ll;
    a.sb_ll = m->w.sb_ll;
    a.ch_ll = m->w.ch_ll;
    a.diag = m->w.diag;
    a.spin = m->wait_limit > 0 ? (long)m->wait_limit : kSpin;
    a.rounds = std::max(16L, a.spin / 16);
    a.stall_cta = m->stall_cta;
    a.stall_t = m->stall_t;
    a.stall_peer_t = m->stall_peer_t;
    DS4F_CUDA(cudaMemsetAsync(m->w.diag + 2, 0, 2 * sizeof(unsigned), st));
    // tags carry 16 bits of layer-step: split long runs into launches
    const int per = std::max(1, 65000 / m->d.n_layers);
    for (int s0 = 0; s0 < n_steps; s0 += per) {
        const int ns = std::min(per, n_steps - s0);
        *epoch = *epoch % 65535 + 1;
        a.epoch = (uint32_t)*epoch;
        a.par0 = (int)(*lsteps & 1);
        *lsteps += (int64_t)ns * m->d.n_layers;
        a.n_steps = ns;
        a.state = state;
        a.trace = nullptr;
        a.log_n = m->log_n > 0 ? std::max(0, m->log_n - s0 * m->d.n_layers) : 0;
        a.log_idx = a.log_n ? m->log_idx + (int64_t)s0 * m->d.n_layers * K : nullptr;
        a.log_w = a.log_n ? m->log_w + (int64_t)s0 * m->d.n_layers * K : nullptr;
        a.log_state = a.log_n ? m->log_state + (int64_t)s0 * m->d.n_layers * H : nullptr;
        if (m->trace && (int64_t)m->d.n_layers * ns * sms * kTracePts <= m->trace_n) a.trace = m->trace;
        const int ki = (ep ? 1 : 0) + (a.trace ? 2 : 0);
        auto kern = kerns[ki];
        if (opt[ki].set(kern, L::bytes)) return -1;
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
    }
    return 0;
}

}  // namespace

namespace {
bool decode_shape_ok(const Model *m) {
    const ModelDesc &d = m->d;
    if (d.topk != 8 || m->cache) return false;
    if (m->slot.nbytes % 16) return false;       // every slot 16-byte aligned (bulk copies)
    if (!((d.hidden == 2048 && d.moe_inter == 512) || (d.hidden == 1024 && d.moe_inter == 256)))
        return false;
    return d.n_experts == 256 || d.n_experts == 64;
}
}  // namespace

bool decode_eligible(const Model *m) {
    return m->d.expert_first == 0 && m->d.expert_count == m->d.n_experts && decode_shape_ok(m);
}

bool decode_eligible_ep(const Model *m, int rank, int world, int split_sel) {
    const int E = m->d.n_experts;
    if (world < 1 || world > kMaxRanks || !decode_shape_ok(m)) return false;
    if (split_sel) return m->d.expert_first == 0 && m->d.expert_count == E;
    return E % world == 0 && m->d.expert_first == rank * (E / world) && m->d.expert_count == E / world;
}

int decode_launch(Model *m, float *state, int n_steps, cudaStream_t st, const DecodePeers *pe) {
    const ModelDesc &d = m->d;
    DS4F_REQUIRE(pe ? decode_eligible_ep(m, pe->rank, pe->world, pe->split_sel) : decode_eligible(m),
                 "decode: shape or shard not supported by the persistent kernel");
    const bool f8 = d.fmt == DS4F_FMT_FP8;
    if (d.hidden == 2048 && d.n_experts == 256)
        return f8 ? launch_t<DS4F_FMT_FP8, 2048, 512, 256, 8>(m, state, n_steps, st, pe)
                  : launch_t<DS4F_FMT_MXFP4, 2048, 512, 256, 8>(m, state, n_steps, st, pe);
    if (d.hidden == 2048 && d.n_experts == 64)
        return f8 ? launch_t<DS4F_FMT_FP8, 2048, 512, 64, 8>(m, state, n_steps, st, pe)
                  : launch_t<DS4F_FMT_MXFP4, 2048, 512, 64, 8>(m, state, n_steps, st, pe);
    if (d.n_experts == 256)
        return f8 ? launch_t<DS4F_FMT_FP8, 1024, 256, 256, 8>(m, state, n_steps, st, pe)
                  : launch_t<DS4F_FMT_MXFP4, 1024, 256, 256, 8>(m, state, n_steps, st, pe);
    return f8 ? launch_t<DS4F_FMT_FP8, 1024, 256, 64, 8>(m, state, n_steps, st, pe)
              : launch_t<DS4F_FMT_MXFP4, 1024, 256, 64, 8>(m, state, n_steps, st, pe);
}

}  // namespace ds4f
