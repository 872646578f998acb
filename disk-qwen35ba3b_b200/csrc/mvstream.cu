// mvstream.cu -- the expert-shaped jobs of a dequant-matvec plan streamed
// through shared memory by TMA (config 1: 8 experts x gate/up/down at batch 1;
// ds4f_f8_matvec src/kernels.c:243-270, ds4f_mxfp4_matvec :48-62,
// ds4f_bf16_matvec :91-103).
//
// A batch-1 matvec reads every weight byte once: it is bound by HBM, and a
// short job list (25 MB for config 1) by how soon every SM has enough bytes
// in flight. The vector path of matvec.cu loads a 64-row item's x and then
// its rows two at a time, each round waiting a full HBM latency. Here one
// persistent CTA per SM owns a contiguous range of units (up to 64 rows of
// one job, <= 32 KB), balanced by bytes over the CTAs; one thread keeps
// kSlots units in flight as bulk copies into a ring of shared-memory slots,
// and 16 warps compute each unit as it lands, one row per warp at a time:
// lane l takes 16-byte chunks l, l + 32, ... of the row (consecutive lanes,
// consecutive addresses), decodes in registers against x (held in registers,
// pre-scaled by 2^64, reloaded only when the job changes) and the warp sums
// the row. The arithmetic per chunk is the vector path's, so results are
// identical to it.
#include "matvec.cuh"
#include "tc.cuh"

#include <algorithm>
#include <vector>

namespace ds4f {

namespace {

constexpr int kSThreads = 512;
constexpr int kSWarps = kSThreads / 32;
constexpr int kSlotBytes = 32 * 1024;
constexpr int kSlots = 6;
constexpr int kXRegs = 64;          // x floats per lane: 4 FP8 / 2 MXFP4 / 8 BF16 chunks

__device__ __forceinline__ int row_bytes_of(const MvJob &J) {
    return J.fmt == DS4F_FMT_FP8 ? J.C : J.fmt == DS4F_FMT_MXFP4 ? J.C / 2 : 2 * J.C;
}

// One row r of job J from shared memory (its bytes at `row`), x of the
// lane's chunks in xr; every lane returns the row's sum.
template <int FMT>
__device__ __forceinline__ float row_dot(const MvJob &J, const uint8_t *row, int r, const float *xr) {
    constexpr int CE = FMT == DS4F_FMT_FP8 ? 16 : FMT == DS4F_FMT_MXFP4 ? 32 : 8;
    constexpr int KCH = kXRegs / CE;
    const int lane = threadIdx.x & 31, nq = J.C / CE;
    float acc = 0.f;
#pragma unroll
    for (int k = 0; k < KCH; k++) {
        const int q = lane + 32 * k;
        if (q >= nq) break;
        uint4 b;
        asm volatile("ld.shared.v4.u32 {%0,%1,%2,%3}, [%4];"
                     : "=r"(b.x), "=r"(b.y), "=r"(b.z), "=r"(b.w) : "r"(tc::sa(row + 16 * q)));
        if constexpr (FMT == DS4F_FMT_FP8) {
            if (J.canon) b = f8_canon16(b);
            const int sr = (int)(((int64_t)r * J.SR) / J.R), sc = (int)(((int64_t)q * 16 * J.SC) / J.C);
            const int si = sr * J.SC + sc;
            const float s = !J.s ? 1.0f
                            : J.scale_kind == DS4F_SCALE_F32 ? __ldg((const float *)J.s + si)
                                                             : e8m0_to_f32(__ldg((const uint8_t *)J.s + si));
            acc += (f8_dot16(b, xr + 16 * k) * DS4F_F8_POST) * s;
        } else if constexpr (FMT == DS4F_FMT_MXFP4) {
            const int64_t bi = ((int64_t)r * J.C + (int64_t)q * 32) / 32;
            acc += (e2m1_dot32(b, xr + 32 * k) * DS4F_E2M1_POST) * e8m0_to_f32(__ldg((const uint8_t *)J.s + bi));
        } else {
            acc += bf16_dot8(b, xr + 8 * k);
        }
    }
    return warp_sum(acc);
}

template <int FMT>
__device__ __forceinline__ void load_x(const MvJob &J, float *xr) {
    constexpr int CE = FMT == DS4F_FMT_FP8 ? 16 : FMT == DS4F_FMT_MXFP4 ? 32 : 8;
    constexpr int KCH = kXRegs / CE;
    const float pre = FMT == DS4F_FMT_BF16 ? 1.0f : DS4F_X_PRESCALE;
    const int lane = threadIdx.x & 31, nq = J.C / CE;
#pragma unroll
    for (int k = 0; k < KCH; k++) {
        const int q = lane + 32 * k;
#pragma unroll
        for (int e = 0; e < CE; e += 4) {
            float4 v = make_float4(0.f, 0.f, 0.f, 0.f);
            if (q < nq) v = __ldg((const float4 *)(J.x + q * CE + e));
            xr[CE * k + e] = v.x * pre;
            xr[CE * k + e + 1] = v.y * pre;
            xr[CE * k + e + 2] = v.z * pre;
            xr[CE * k + e + 3] = v.w * pre;
        }
    }
}

__global__ void __launch_bounds__(kSThreads, 1)
k_mv_stream(const MvJob *__restrict__ jobs, const MvUnit *__restrict__ units, const int *__restrict__ ranges,
            unsigned *err) {
    extern __shared__ __align__(128) unsigned char sm[];
    uint64_t *bar = (uint64_t *)sm;                       // kSlots mbarriers
    uint8_t *ring = sm + 128;
    const int tid = threadIdx.x, warp = tid >> 5, lane = tid & 31;
    const int u0 = ranges[blockIdx.x], n = ranges[blockIdx.x + 1] - u0;
    if (tid == 0) {
        for (int i = 0; i < kSlots; i++) tc::mbar_init(bar + i, 1);
        tc::mbar_fence_init();
    }
    __syncthreads();
    // thread 0: unit k's rows into slot k % kSlots
    auto issue = [&](int k) {
        const MvUnit u = units[u0 + k];
        const MvJob &J = jobs[u.job];
        const int rb = row_bytes_of(J);
        uint64_t *b = bar + k % kSlots;
        tc::mbar_expect(b, (uint32_t)u.bytes);
        asm volatile(
            "cp.async.bulk.shared::cluster.global.mbarrier::complete_tx::bytes [%0], [%1], %2, [%3];"
            ::"r"(tc::sa(ring + (size_t)(k % kSlots) * kSlotBytes)),
              "l"((const uint8_t *)J.v + (int64_t)u.row0 * rb), "r"((uint32_t)u.bytes), "r"(tc::sa(b))
            : "memory");
    };
    if (tid == 0)
        for (int k = 0; k < n && k < kSlots; k++) issue(k);
    float xr[kXRegs];
    int cur = -1;
    bool ok = true;
    int k = 0;
    for (; k < n; k++) {
        const MvUnit u = units[u0 + k];
        const MvJob J = jobs[u.job];
        if (u.job != cur) {
            if (J.fmt == DS4F_FMT_FP8) load_x<DS4F_FMT_FP8>(J, xr);
            else if (J.fmt == DS4F_FMT_MXFP4) load_x<DS4F_FMT_MXFP4>(J, xr);
            else load_x<DS4F_FMT_BF16>(J, xr);
            cur = u.job;
        }
        ok = tc::mbar_wait(bar + k % kSlots, (uint32_t)((k / kSlots) & 1), err, 1u);
        if (!__syncthreads_and(ok)) break;
        const uint8_t *slot = ring + (size_t)(k % kSlots) * kSlotBytes;
        const int rb = row_bytes_of(J);
        for (int i = warp; i < u.nrows; i += kSWarps) {
            const int r = u.row0 + i;
            float v;
            if (J.fmt == DS4F_FMT_FP8) v = row_dot<DS4F_FMT_FP8>(J, slot + (size_t)i * rb, r, xr);
            else if (J.fmt == DS4F_FMT_MXFP4) v = row_dot<DS4F_FMT_MXFP4>(J, slot + (size_t)i * rb, r, xr);
            else v = row_dot<DS4F_FMT_BF16>(J, slot + (size_t)i * rb, r, xr) +
                     (J.s ? __ldg((const float *)J.s + r) : 0.0f);
            if (lane == 0) J.y[r] = v;
        }
        __syncthreads();                                  // the slot is free again
        if (tid == 0 && k + kSlots < n) {
            asm volatile("fence.proxy.async.shared::cta;" ::: "memory");
            issue(k + kSlots);
        }
    }
    // a CTA that stopped at unit k drains the copies still in flight, units
    // k .. k + kSlots - 1 (bounded; each on its slot's phase)
    if (!ok && tid == 0)
        for (int i = k; i < n && i < k + kSlots; i++)
            tc::mbar_wait(bar + i % kSlots, (uint32_t)((i / kSlots) & 1), err, 1u, true, 1L << 22);
}

}  // namespace

bool stream_eligible(const MvJob &J) {
    if (!((uintptr_t)J.v % 16 == 0 && (uintptr_t)J.x % 16 == 0 && J.R >= 1 && J.C % 128 == 0 && J.C <= 2048))
        return false;
    if (J.fmt == DS4F_FMT_FP8) return J.SR >= 1 && J.SC >= 1 && J.C % J.SC == 0 && (J.C / J.SC) % 16 == 0;
    if (J.fmt == DS4F_FMT_MXFP4) return J.bsize == 32 && J.s;
    return J.fmt == DS4F_FMT_BF16 && J.C <= 2048;
}

int stream_plan(MvJob *jobs, int njobs, MvStream *sp) {
    *sp = MvStream{};
    std::vector<MvUnit> units;
    std::vector<int64_t> start;
    int64_t total = 0;
    for (int j = 0; j < njobs; j++) {
        MvJob &J = jobs[j];
        if (J.SR < 1) J.SR = 1;
        if (J.SC < 1) J.SC = 1;
        J.streamed = stream_eligible(J) ? 1 : 0;
        if (!J.streamed) continue;
        const int rb = J.fmt == DS4F_FMT_FP8 ? J.C : J.fmt == DS4F_FMT_MXFP4 ? J.C / 2 : 2 * J.C;
        const int per = std::max(1, std::min(64, kSlotBytes / rb));
        for (int r = 0; r < J.R; r += per) {
            MvUnit u;
            u.job = j;
            u.row0 = r;
            u.nrows = std::min(per, J.R - r);
            u.bytes = u.nrows * rb;
            start.push_back(total);
            total += u.bytes;
            units.push_back(u);
        }
    }
    if (units.empty()) return 0;
    int dev = 0, sms = 148;
    DS4F_CUDA(cudaGetDevice(&dev));
    DS4F_CUDA(cudaDeviceGetAttribute(&sms, cudaDevAttrMultiProcessorCount, dev));
    const int G = (int)std::min<int64_t>(sms, (int64_t)units.size());
    // CTA c: the units whose first byte lies in [c total / G, (c+1) total / G)
    std::vector<int> ranges(G + 1, 0);
    size_t u = 0;
    for (int c = 0; c < G; c++) {
        ranges[c] = (int)u;
        const int64_t end = (int64_t)((__int128)(c + 1) * total / G);
        while (u < units.size() && start[u] < end) u++;
    }
    ranges[G] = (int)units.size();
    const size_t ub = units.size() * sizeof(MvUnit), rbb = ranges.size() * sizeof(int);
    if (cudaMalloc(&sp->base, ub + rbb + 256) != cudaSuccess) {
        set_error("mv_plan: device allocation failed");
        return -1;
    }
    sp->units = (MvUnit *)sp->base;
    sp->ranges = (int *)((uint8_t *)sp->base + ub);
    sp->err = (unsigned *)((uint8_t *)sp->base + (ub + rbb + 15) / 16 * 16);
    DS4F_CUDA(cudaMemcpy(sp->units, units.data(), ub, cudaMemcpyHostToDevice));
    DS4F_CUDA(cudaMemcpy(sp->ranges, ranges.data(), rbb, cudaMemcpyHostToDevice));
    DS4F_CUDA(cudaMemset(sp->err, 0, 4));
    sp->nunits = (int)units.size();
    sp->grid = G;
    return 0;
}

void stream_free(MvStream *sp) {
    if (sp->base) cudaFree(sp->base);
    *sp = MvStream{};
}

int stream_launch(const MvJob *jobs_dev, const MvStream &sp, cudaStream_t st) {
    if (!sp.nunits) return 0;
    static SmemOptIn opt;
    const int bytes = 128 + kSlots * kSlotBytes;
    if (opt.set(k_mv_stream, bytes)) return -1;
    k_mv_stream<<<sp.grid, kSThreads, bytes, st>>>(jobs_dev, sp.units, sp.ranges, sp.err);
    DS4F_CUDA(cudaGetLastError());
    return 0;
}

int stream_check(const MvStream &sp) {
    if (!sp.nunits) return 0;
    unsigned e = 0;
    DS4F_CUDA(cudaMemcpy(&e, sp.err, 4, cudaMemcpyDeviceToHost));
    if (e) {
        cudaMemset(sp.err, 0, 4);
        set_error("matvec: a weight copy did not complete (the stream kernel gave up waiting)");
        return -1;
    }
    return 0;
}

}  // namespace ds4f
