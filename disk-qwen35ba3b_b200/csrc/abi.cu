// abi.cu -- the extern "C" boundary of libds4f_cuda (include/ds4f/gpu_cuda.h).
#include "../../include/ds4f/gpu_cuda.h"
#include "matvec.cuh"
#include "model.cuh"

#include <algorithm>
#include <cstdarg>
#include <cstdio>
#include <cstring>
#include <mutex>
#include <unordered_map>
#include <vector>

#include <fcntl.h>
#include <unistd.h>

namespace ds4f {

static thread_local char g_err[512] = "";

void set_error(const char *fmt, ...) {
    va_list ap;
    va_start(ap, fmt);
    vsnprintf(g_err, sizeof g_err, fmt, ap);
    va_end(ap);
}

int cuda_fail(cudaError_t e, const char *what, const char *file, int line) {
    const char *f = strrchr(file, '/');
    set_error("CUDA error %s (%s) in %s at %s:%d", cudaGetErrorName(e),
              cudaGetErrorString(e), what, f ? f + 1 : file, line);
    return -1;
}

namespace {

struct DevState {
    cudaStream_t stream = nullptr;
    void *scratch = nullptr;
    size_t scratch_cap = 0;
    // MLX4 weight arena keyed by the caller's stable tensor id (the
    // reference's Metal arena, src/gpu_metal.mm:186-254): first sight of
    // an id copies its weights, later calls reuse them.
    std::unordered_map<const void *, uint8_t *> arena;
    std::vector<void *> arena_blocks;
};

std::mutex g_mu;
std::unordered_map<int, DevState> g_dev;

DevState *dev_state() {
    int dev = 0;
    if (cudaGetDevice(&dev) != cudaSuccess) return nullptr;
    std::lock_guard<std::mutex> lk(g_mu);
    DevState &s = g_dev[dev];
    if (!s.stream && cudaStreamCreateWithFlags(&s.stream, cudaStreamNonBlocking) != cudaSuccess)
        return nullptr;
    return &s;
}

int stream_of(void *st, cudaStream_t *out) {
    if (st) { *out = (cudaStream_t)st; return 0; }
    DevState *s = dev_state();
    DS4F_REQUIRE(s, "no CUDA device / stream");
    *out = s->stream;
    return 0;
}

// Device scratch for the host-buffer calls: grown, never shrunk.
void *scratch(size_t bytes) {
    DevState *s = dev_state();
    if (!s) return nullptr;
    if (bytes > s->scratch_cap) {
        if (s->scratch) cudaFree(s->scratch);
        s->scratch = nullptr;
        s->scratch_cap = 0;
        size_t cap = bytes < ((size_t)1 << 20) ? ((size_t)1 << 20) : bytes;
        if (cudaMalloc(&s->scratch, cap) != cudaSuccess) {
            set_error("out of device memory for %zu scratch bytes", cap);
            return nullptr;
        }
        s->scratch_cap = cap;
    }
    return s->scratch;
}

size_t al256(size_t n) { return (n + 255) & ~(size_t)255; }

int run_one(MvJob J, const void *hv, size_t vbytes, const void *hs, size_t sbytes,
            const void *hb, size_t bbytes, const float *hx, float *hy) {
    DevState *ds = dev_state();
    DS4F_REQUIRE(ds, "no CUDA device");
    size_t ox = 0, ov = al256(ox + (size_t)J.C * 4), os = al256(ov + vbytes),
           ob = al256(os + sbytes), oy = al256(ob + bbytes), oj = al256(oy + (size_t)J.R * 4),
           tot = oj + sizeof(MvJob);
    uint8_t *base = (uint8_t *)scratch(tot);
    if (!base) return -1;
    cudaStream_t st = ds->stream;
    DS4F_CUDA(cudaMemcpyAsync(base + ox, hx, (size_t)J.C * 4, cudaMemcpyHostToDevice, st));
    DS4F_CUDA(cudaMemcpyAsync(base + ov, hv, vbytes, cudaMemcpyHostToDevice, st));
    if (hs && sbytes) DS4F_CUDA(cudaMemcpyAsync(base + os, hs, sbytes, cudaMemcpyHostToDevice, st));
    if (hb && bbytes) DS4F_CUDA(cudaMemcpyAsync(base + ob, hb, bbytes, cudaMemcpyHostToDevice, st));
    J.x = (const float *)(base + ox);
    J.v = base + ov;
    J.s = (hs && sbytes) ? base + os : nullptr;
    J.b = (hb && bbytes) ? base + ob : nullptr;
    J.y = (float *)(base + oy);
    int n = plan_jobs(&J, 1);
    if (n < 0) return -1;
    DS4F_CUDA(cudaMemcpyAsync(base + oj, &J, sizeof J, cudaMemcpyHostToDevice, st));
    if (launch_jobs((const MvJob *)(base + oj), 1, n, st)) return -1;
    DS4F_CUDA(cudaMemcpyAsync(hy, base + oy, (size_t)J.R * 4, cudaMemcpyDeviceToHost, st));
    DS4F_CUDA(cudaStreamSynchronize(st));
    return 0;
}

MvJob job_of(int fmt, int R, int C) {
    MvJob J;
    memset(&J, 0, sizeof J);
    J.fmt = fmt; J.R = R; J.C = C; J.SR = 1; J.SC = 1; J.bsize = 32;
    return J;
}

}  // namespace
}  // namespace ds4f

using namespace ds4f;

struct Ds4fMvPlan {
    MvJob *jobs_dev;
    int njobs, nitems, device;
    MvStream sp;          // the expert-shaped jobs, streamed by TMA (mvstream.cu)
    unsigned *err_h;      // pinned copy of sp.err after each run, read by the next
};

namespace ds4f {

}  // namespace ds4f

extern "C" {

const char *ds4f_gpu_last_error(void) { return g_err; }

int ds4f_gpu_init(void) {
    int n = 0;
    cudaError_t e = cudaGetDeviceCount(&n);
    if (e != cudaSuccess || n < 1) {
        set_error("no CUDA device (%s)", e == cudaSuccess ? "count 0" : cudaGetErrorString(e));
        return -1;
    }
    DS4F_CUDA(cudaFree(0));
    DS4F_REQUIRE(dev_state(), "cannot create the library stream");
    return 0;
}

void ds4f_gpu_free(void) {
    std::lock_guard<std::mutex> lk(g_mu);
    int cur = 0;
    cudaGetDevice(&cur);
    for (auto &kv : g_dev) {
        cudaSetDevice(kv.first);
        DevState &s = kv.second;
        if (s.stream) cudaStreamSynchronize(s.stream);
        if (s.scratch) cudaFree(s.scratch);
        for (void *p : s.arena_blocks) cudaFree(p);
        if (s.stream) cudaStreamDestroy(s.stream);
    }
    g_dev.clear();
    cudaSetDevice(cur);
}

int ds4f_gpu_f8_matvec(const uint8_t *W, int scale_kind, const void *scales, int R,
                       int C, int SR, int SC, const float *x, float *y) {
    DS4F_REQUIRE(W && x && y && R >= 0 && C > 0, "f8_matvec: bad arguments");
    if (R == 0) return 0;
    MvJob J = job_of(DS4F_FMT_FP8, R, C);
    J.SR = SR < 1 ? 1 : SR; J.SC = SC < 1 ? 1 : SC;
    J.scale_kind = scale_kind; J.canon = 1;
    size_t sb = scales ? (size_t)J.SR * J.SC * (scale_kind == DS4F_SCALE_F32 ? 4 : 1) : 0;
    return run_one(J, W, (size_t)R * C, scales, sb, nullptr, 0, x, y);
}

int ds4f_gpu_mxfp4_matvec(const uint8_t *vals, const uint8_t *scales, int R, int C,
                          int bsize, const float *x, float *y) {
    DS4F_REQUIRE(vals && scales && x && y && R >= 0 && C > 0, "mxfp4_matvec: bad arguments");
    DS4F_REQUIRE(bsize == 16 || bsize == 32, "mxfp4_matvec: bsize %d (16 or 32)", bsize);
    if (R == 0) return 0;
    MvJob J = job_of(DS4F_FMT_MXFP4, R, C);
    J.bsize = bsize;
    int64_t n = (int64_t)R * C;
    return run_one(J, vals, (size_t)(n + 1) / 2, scales, (size_t)((n + bsize - 1) / bsize),
                   nullptr, 0, x, y);
}

int ds4f_gpu_bf16_matvec(const uint16_t *W, int R, int C, const float *x,
                         const float *bias, float *y) {
    DS4F_REQUIRE(W && x && y && R >= 0 && C > 0, "bf16_matvec: bad arguments");
    if (R == 0) return 0;
    MvJob J = job_of(DS4F_FMT_BF16, R, C);
    return run_one(J, W, (size_t)R * C * 2, bias, bias ? (size_t)R * 4 : 0, nullptr, 0, x, y);
}

int ds4f_gpu_mlx4_matvec(const uint32_t *vals, const uint16_t *scales,
                         const uint16_t *biases, int R, int C, const float *x,
                         float *y) {
    DS4F_REQUIRE(vals && scales && x && y && R >= 0 && C > 0, "mlx4_matvec: bad arguments");
    if (R == 0) return 0;
    MvJob J = job_of(DS4F_FMT_MLX4, R, C);
    int64_t n = (int64_t)R * C;
    size_t ng = (size_t)((n + 63) / 64);
    return run_one(J, vals, (size_t)((n + 7) / 8) * 4, scales, ng * 2, biases,
                   biases ? ng * 2 : 0, x, y);
}

int ds4f_gpu_mlx4_batch(const uint32_t *const *vals, const uint16_t *const *scales,
                        const uint16_t *const *biases, const float *const *xs,
                        float *const *ys, const void *const *ids, int R, int C,
                        int njobs) {
    DS4F_REQUIRE(vals && scales && xs && ys && ids && R > 0 && C > 0 && njobs >= 0,
                 "mlx4_batch: bad arguments");
    if (njobs == 0) return 0;
    DevState *ds = dev_state();
    DS4F_REQUIRE(ds, "no CUDA device");
    cudaStream_t st = ds->stream;
    int64_t n = (int64_t)R * C;
    size_t vb = (size_t)((n + 7) / 8) * 4, gb = (size_t)((n + 63) / 64) * 2;
    size_t slot = al256(vb) + al256(gb) + al256(gb);
    std::vector<MvJob> jobs(njobs);
    for (int j = 0; j < njobs; j++) {
        auto it = ds->arena.find(ids[j]);
        uint8_t *w;
        if (it == ds->arena.end()) {
            void *p = nullptr;
            DS4F_CUDA(cudaMalloc(&p, slot));
            ds->arena_blocks.push_back(p);
            w = (uint8_t *)p;
            DS4F_CUDA(cudaMemcpyAsync(w, vals[j], vb, cudaMemcpyHostToDevice, st));
            DS4F_CUDA(cudaMemcpyAsync(w + al256(vb), scales[j], gb, cudaMemcpyHostToDevice, st));
            if (biases && biases[j])
                DS4F_CUDA(cudaMemcpyAsync(w + al256(vb) + al256(gb), biases[j], gb,
                                          cudaMemcpyHostToDevice, st));
            ds->arena[ids[j]] = w;
        } else {
            w = it->second;
        }
        jobs[j] = job_of(DS4F_FMT_MLX4, R, C);
        jobs[j].v = w;
        jobs[j].s = w + al256(vb);
        jobs[j].b = (biases && biases[j]) ? w + al256(vb) + al256(gb) : nullptr;
    }
    size_t ox = 0, oy = al256((size_t)njobs * C * 4), oj = oy + al256((size_t)njobs * R * 4);
    uint8_t *base = (uint8_t *)scratch(oj + sizeof(MvJob) * njobs);
    if (!base) return -1;
    for (int j = 0; j < njobs; j++) {
        DS4F_CUDA(cudaMemcpyAsync(base + ox + (size_t)j * C * 4, xs[j], (size_t)C * 4,
                                  cudaMemcpyHostToDevice, st));
        jobs[j].x = (const float *)(base + ox + (size_t)j * C * 4);
        jobs[j].y = (float *)(base + oy + (size_t)j * R * 4);
    }
    int items = plan_jobs(jobs.data(), njobs);
    if (items < 0) return -1;
    DS4F_CUDA(cudaMemcpyAsync(base + oj, jobs.data(), sizeof(MvJob) * njobs,
                              cudaMemcpyHostToDevice, st));
    if (launch_jobs((const MvJob *)(base + oj), njobs, items, st)) return -1;
    for (int j = 0; j < njobs; j++)
        DS4F_CUDA(cudaMemcpyAsync(ys[j], base + oy + (size_t)j * R * 4, (size_t)R * 4,
                                  cudaMemcpyDeviceToHost, st));
    DS4F_CUDA(cudaStreamSynchronize(st));
    return 0;
}

int ds4f_gpu_f8_decode_rows(const uint8_t *W, int scale_kind, const void *scales, int R,
                            int C, int SR, int SC, int r0, int r1, float *out) {
    DS4F_REQUIRE(W && out && R > 0 && C > 0 && 0 <= r0 && r0 <= r1 && r1 <= R,
                 "f8_decode_rows: bad arguments");
    DevState *ds = dev_state();
    DS4F_REQUIRE(ds, "no CUDA device");
    SR = SR < 1 ? 1 : SR; SC = SC < 1 ? 1 : SC;
    size_t vb = (size_t)R * C, sb = scales ? (size_t)SR * SC * (scale_kind == DS4F_SCALE_F32 ? 4 : 1) : 0;
    size_t ob = (size_t)(r1 - r0) * C * 4;
    uint8_t *base = (uint8_t *)scratch(al256(vb) + al256(sb) + ob);
    if (!base) return -1;
    cudaStream_t st = ds->stream;
    DS4F_CUDA(cudaMemcpyAsync(base, W, vb, cudaMemcpyHostToDevice, st));
    if (sb) DS4F_CUDA(cudaMemcpyAsync(base + al256(vb), scales, sb, cudaMemcpyHostToDevice, st));
    float *o = (float *)(base + al256(vb) + al256(sb));
    if (launch_f8_decode(base, scale_kind, sb ? base + al256(vb) : nullptr, R, C, SR, SC, r0,
                         r1, o, st))
        return -1;
    DS4F_CUDA(cudaMemcpyAsync(out, o, ob, cudaMemcpyDeviceToHost, st));
    DS4F_CUDA(cudaStreamSynchronize(st));
    return 0;
}

int ds4f_gpu_mxfp4_decode(const uint8_t *vals, const uint8_t *scales, int64_t n, int bsize,
                          float *out) {
    DS4F_REQUIRE(vals && scales && out && n >= 0 && bsize > 0, "mxfp4_decode: bad arguments");
    if (n == 0) return 0;
    DevState *ds = dev_state();
    DS4F_REQUIRE(ds, "no CUDA device");
    size_t vb = (size_t)(n + 1) / 2, sb = (size_t)((n + bsize - 1) / bsize);
    uint8_t *base = (uint8_t *)scratch(al256(vb) + al256(sb) + (size_t)n * 4);
    if (!base) return -1;
    cudaStream_t st = ds->stream;
    DS4F_CUDA(cudaMemcpyAsync(base, vals, vb, cudaMemcpyHostToDevice, st));
    DS4F_CUDA(cudaMemcpyAsync(base + al256(vb), scales, sb, cudaMemcpyHostToDevice, st));
    float *o = (float *)(base + al256(vb) + al256(sb));
    if (launch_mx_decode(base, base + al256(vb), n, bsize, o, st)) return -1;
    DS4F_CUDA(cudaMemcpyAsync(out, o, (size_t)n * 4, cudaMemcpyDeviceToHost, st));
    DS4F_CUDA(cudaStreamSynchronize(st));
    return 0;
}

int ds4f_gpu_mv_plan(const Ds4fMvJob *jobs, int njobs, Ds4fMvPlan **plan) {
    DS4F_REQUIRE(jobs && plan && njobs > 0, "mv_plan: bad arguments");
    *plan = nullptr;
    std::vector<MvJob> v(njobs);
    for (int j = 0; j < njobs; j++) {
        MvJob &J = v[j];
        memset(&J, 0, sizeof J);
        J.v = jobs[j].w; J.s = jobs[j].scales; J.x = jobs[j].x; J.y = jobs[j].y;
        J.R = jobs[j].R; J.C = jobs[j].C; J.SR = jobs[j].SR; J.SC = jobs[j].SC;
        J.fmt = jobs[j].fmt; J.scale_kind = jobs[j].scale_kind; J.bsize = jobs[j].bsize;
        J.canon = jobs[j].canon;
        DS4F_REQUIRE(J.fmt != DS4F_FMT_MLX4, "mv_plan: MLX4 jobs go through ds4f_gpu_mlx4_batch");
    }
    Ds4fMvPlan *p = new Ds4fMvPlan();
    memset(p, 0, sizeof *p);
    // the expert-shaped jobs go to the stream kernel, the rest to k_mv_jobs
    if (stream_plan(v.data(), njobs, &p->sp)) { delete p; return -1; }
    int items = plan_jobs(v.data(), njobs);
    if (items < 0) { stream_free(&p->sp); delete p; return -1; }
    p->njobs = njobs; p->nitems = items;
    cudaGetDevice(&p->device);
    if (cudaMalloc(&p->jobs_dev, sizeof(MvJob) * njobs) != cudaSuccess ||
        cudaMemcpy(p->jobs_dev, v.data(), sizeof(MvJob) * njobs, cudaMemcpyHostToDevice) !=
            cudaSuccess ||
        cudaHostAlloc((void **)&p->err_h, 4, cudaHostAllocDefault) != cudaSuccess) {
        cudaFree(p->jobs_dev);
        stream_free(&p->sp);
        delete p;
        set_error("mv_plan: device allocation failed");
        return -1;
    }
    *p->err_h = 0;
    *plan = p;
    return 0;
}

int ds4f_gpu_mv_run(const Ds4fMvPlan *plan, void *stream) {
    DS4F_REQUIRE(plan, "mv_run: null plan");
    cudaStream_t st;
    if (stream_of(stream, &st)) return -1;
    if (*(volatile unsigned *)plan->err_h) {
        *plan->err_h = 0;
        cudaMemsetAsync(plan->sp.err, 0, 4, st);
        set_error("mv_run: a weight copy of an earlier run did not complete (its outputs are invalid)");
        return -1;
    }
    if (stream_launch(plan->jobs_dev, plan->sp, st)) return -1;
    if (plan->sp.nunits) DS4F_CUDA(cudaMemcpyAsync(plan->err_h, plan->sp.err, 4, cudaMemcpyDeviceToHost, st));
    return launch_jobs(plan->jobs_dev, plan->njobs, plan->nitems, st);
}

void ds4f_gpu_mv_plan_free(Ds4fMvPlan *plan) {
    if (!plan) return;
    cudaSetDevice(plan->device);
    cudaDeviceSynchronize();
    cudaFree(plan->jobs_dev);
    stream_free(&plan->sp);
    if (plan->err_h) cudaFreeHost(plan->err_h);
    delete plan;
}

// ---- model --------------------------------------------------------------

// pool_slots < 0: the whole shard resident; else an arena of that many slots
// (a streaming model)
static int model_create_impl(const Ds4fGpuModelDesc *desc, int64_t pool_slots, Ds4fGpuModel **out) {
    DS4F_REQUIRE(desc && out, "model_create: null argument");
    *out = nullptr;
    ModelDesc d;
    d.fmt = desc->fmt; d.n_layers = desc->n_layers; d.hidden = desc->hidden;
    d.moe_inter = desc->moe_inter; d.n_experts = desc->n_experts; d.topk = desc->topk;
    d.renorm = desc->renorm; d.expert_first = desc->expert_first;
    d.expert_count = desc->expert_count; d.router_exact = desc->router_exact;
    DS4F_REQUIRE(d.fmt == DS4F_FMT_FP8 || d.fmt == DS4F_FMT_MXFP4,
                 "model: expert format %d (FP8 or MXFP4)", d.fmt);
    DS4F_REQUIRE(d.n_layers > 0 && d.n_experts > 0 && d.topk > 0 && d.topk <= 16 &&
                     d.topk <= d.n_experts && d.n_experts <= 4096,
                 "model: bad sizes (layers %d experts %d topk %d)", d.n_layers, d.n_experts,
                 d.topk);
    DS4F_REQUIRE((d.hidden == 2048 && d.moe_inter == 512) ||
                     (d.hidden == 1024 && d.moe_inter == 256),
                 "model: kernels are built for (H, M) = (2048, 512) or (1024, 256), got (%d, %d)",
                 d.hidden, d.moe_inter);
    DS4F_REQUIRE(d.expert_first >= 0 && d.expert_count > 0 &&
                     d.expert_first + d.expert_count <= d.n_experts,
                 "model: expert shard [%d, %d) outside [0, %d)", d.expert_first,
                 d.expert_first + d.expert_count, d.n_experts);
    Model m;
    memset(&m, 0, sizeof m);
    m.d = d;
    m.stall_cta = m.stall_t = -1;
    m.stall_peer_t = -1;
    if (slot_layout(d.fmt, d.hidden, d.moe_inter, &m.slot)) return -1;
    trunk_layout(d.hidden, d.moe_inter, d.n_experts, &m.tr);
    DS4F_CUDA(cudaGetDevice(&m.device));
    const int H = d.hidden, M = d.moe_inter, E = d.n_experts, K = d.topk;
    // + 4 KB: bulk copies of small scale runs round up to 16 bytes
    size_t pool_b = (size_t)(pool_slots < 0 ? (int64_t)d.n_layers * d.expert_count : pool_slots) * m.slot.nbytes +
                    4096;
    size_t trunk_b = (size_t)d.n_layers * m.tr.n * 2;
    m.bmax = 64;
    size_t ws_b = al256(H * 4) + al256(E * 8) * 2 + al256(K * 4) * 2 +
                  al256((size_t)(K + 1) * M * 4) + al256(4) + al256(H * 4) + al256(16) +
                  al256((size_t)m.bmax * H * 4) + al256((size_t)m.bmax * K * 4) * 2 +
                  al256((size_t)H * 8) + al256((size_t)E * 32) + al256(((size_t)(K + 1) * M + 2) * 8);
    // memory plan first (invariant 5 of the reference, ds4f.h:32-35 /
    // mem.c): refuse past 95% of free device memory, allocate nothing.
    size_t fre = 0, tot = 0;
    DS4F_CUDA(cudaMemGetInfo(&fre, &tot));
    size_t need = pool_b + trunk_b + ws_b;
    DS4F_REQUIRE((double)need <= 0.95 * (double)fre,
                 "model: needs %.2f GB of device memory, %.2f GB free (refusing past 95%%)",
                 need / 1e9, fre / 1e9);
    DS4F_CUDA(cudaMalloc(&m.pool, pool_b));
    if (cudaMalloc(&m.trunk, trunk_b) != cudaSuccess || cudaMalloc(&m.ws_base, ws_b) != cudaSuccess) {
        cudaFree(m.pool); cudaFree(m.trunk);
        set_error("model: device allocation failed");
        return -1;
    }
    uint8_t *p = (uint8_t *)m.ws_base;
    auto take = [&](size_t n) { uint8_t *r = p; p += al256(n); return r; };
    m.w.xin = (float *)take(H * 4);
    m.w.S = (double *)take(E * 8);
    m.w.Bnd = (double *)take(E * 8);
    m.w.idx = (int *)take(K * 4);
    m.w.w = (float *)take(K * 4);
    m.w.chain = (float *)take((size_t)(K + 1) * M * 4);
    m.w.sgate = (float *)take(4);
    m.w.acc = (float *)take(H * 4);
    m.w.diag = (unsigned *)take(16);
    m.state_dev = (float *)take((size_t)m.bmax * H * 4);
    m.idx_dev = (int *)take((size_t)m.bmax * K * 4);
    m.w_dev = (float *)take((size_t)m.bmax * K * 4);
    m.w.st_ll = (uint64_t *)take((size_t)H * 8);
    m.w.sb_ll = (uint64_t *)take((size_t)E * 32);
    m.w.ch_ll = (uint64_t *)take(((size_t)(K + 1) * M + 2) * 8);   // + pad word
    if ((size_t)(p - (uint8_t *)m.ws_base) != ws_b) {       // the size above and the layout agree
        cudaFree(m.pool); cudaFree(m.trunk); cudaFree(m.ws_base);
        set_error("model: workspace layout (%zu bytes) differs from its size (%zu)",
                  (size_t)(p - (uint8_t *)m.ws_base), ws_b);
        return -1;
    }
    cudaMemset(m.ws_base, 0, ws_b);
    if (cudaStreamCreateWithFlags(&m.stream, cudaStreamNonBlocking) != cudaSuccess) {
        cudaFree(m.pool); cudaFree(m.trunk); cudaFree(m.ws_base);
        set_error("model: stream creation failed");
        return -1;
    }
    Ds4fGpuModel *h = new Ds4fGpuModel();
    h->m = m;
    *out = h;
    return 0;
}

int ds4f_gpu_model_create(const Ds4fGpuModelDesc *desc, Ds4fGpuModel **out) {
    return model_create_impl(desc, -1, out);
}

int ds4f_gpu_model_create_streaming(const Ds4fGpuModelDesc *desc, const uint8_t *host_pool, int n_slots,
                                    Ds4fGpuModel **out) {
    DS4F_REQUIRE(desc && host_pool && out, "model_create_streaming: null argument");
    *out = nullptr;
    DS4F_REQUIRE(desc->expert_first == 0 && desc->expert_count == desc->n_experts,
                 "model_create_streaming: the host pool holds every expert (no shard)");
    DS4F_REQUIRE(n_slots >= desc->topk, "model_create_streaming: %d slots, at least top-k = %d needed", n_slots,
                 desc->topk);
    n_slots = (int)std::min<int64_t>(n_slots, (int64_t)desc->n_layers * desc->n_experts);   // no unused slots
    Ds4fGpuModel *h = nullptr;
    if (model_create_impl(desc, n_slots, &h)) return -1;
    Model &m = h->m;
    const size_t host_b = (size_t)m.d.n_layers * m.d.n_experts * m.slot.nbytes;
    cudaError_t e = cudaHostRegister(const_cast<uint8_t *>(host_pool), host_b, cudaHostRegisterReadOnly);
    if (e != cudaSuccess) e = cudaHostRegister(const_cast<uint8_t *>(host_pool), host_b, cudaHostRegisterDefault);
    if (e != cudaSuccess) {
        ds4f_gpu_model_destroy(h);
        set_error("model_create_streaming: pinning the %.2f GB host pool failed (%s)", host_b / 1e9,
                  cudaGetErrorString(e));
        return -1;
    }
    m.host_pool = host_pool;
    m.stream_slots = n_slots;
    m.cache = slot_cache_new(n_slots);
    const int K = m.d.topk;
    if (!m.cache || cudaMalloc(&m.slot_dev, K * 4) != cudaSuccess ||
        cudaHostAlloc((void **)&m.idx_h, K * 4, cudaHostAllocDefault) != cudaSuccess ||
        cudaHostAlloc((void **)&m.slot_h, K * 4, cudaHostAllocDefault) != cudaSuccess) {
        ds4f_gpu_model_destroy(h);
        set_error("model_create_streaming: allocation failed");
        return -1;
    }
    *out = h;
    return 0;
}

int ds4f_gpu_stream_stats(const Ds4fGpuModel *h, int64_t *requests, int64_t *hits, int64_t *fetched) {
    DS4F_REQUIRE(h && h->m.cache, "stream_stats: not a streaming model");
    slot_cache_stats(h->m.cache, requests, hits, nullptr, fetched);
    return 0;
}

void ds4f_gpu_model_destroy(Ds4fGpuModel *h) {
    if (!h) return;
    Model &m = h->m;
    int cur = 0;
    cudaGetDevice(&cur);
    cudaSetDevice(m.device);
    if (m.stream) cudaStreamSynchronize(m.stream);
    ep_free(&m);
    if (m.graph) cudaGraphExecDestroy(m.graph);
    if (m.trace) cudaFree(m.trace);
    if (m.log_base) cudaFree(m.log_base);
    if (m.pf_ws) cudaFree(m.pf_ws);
    if (m.pf_err_h) cudaFreeHost(m.pf_err_h);
    if (m.bgraph) cudaGraphExecDestroy(m.bgraph);
    if (m.host_pool) cudaHostUnregister(const_cast<uint8_t *>(m.host_pool));
    if (m.cache) slot_cache_delete(m.cache);
    if (m.slot_dev) cudaFree(m.slot_dev);
    if (m.idx_h) cudaFreeHost(m.idx_h);
    if (m.slot_h) cudaFreeHost(m.slot_h);
    cudaFree(m.pool);
    cudaFree(m.trunk);
    cudaFree(m.ws_base);
    if (m.stream) cudaStreamDestroy(m.stream);
    cudaSetDevice(cur);
    delete h;
}

int ds4f_gpu_model_slot(const Ds4fGpuModel *h, int64_t rel_v[3], int64_t rel_s[3],
                        int64_t *nbytes) {
    DS4F_REQUIRE(h, "model_slot: null model");
    for (int t = 0; t < 3; t++) {
        if (rel_v) rel_v[t] = h->m.slot.rel_v[t];
        if (rel_s) rel_s[t] = h->m.slot.rel_s[t];
    }
    if (nbytes) *nbytes = h->m.slot.nbytes;
    return 0;
}

int ds4f_gpu_model_synth(Ds4fGpuModel *h, uint64_t seed) {
    DS4F_REQUIRE(h, "model_synth: null model");
    DS4F_REQUIRE(!h->m.cache, "model_synth: a streaming model's experts are the caller's host pool");
    if (synth_model(&h->m, seed, 0.02, h->m.stream)) return -1;
    DS4F_CUDA(cudaStreamSynchronize(h->m.stream));
    return 0;
}

static int trunk_io(const Model &m, int layer, uint16_t *const host[6], bool up) {
    DS4F_REQUIRE(layer >= 0 && layer < m.d.n_layers, "trunk: layer %d out of range", layer);
    const int64_t H = m.d.hidden, M = m.d.moe_inter, E = m.d.n_experts;
    const int64_t off[6] = {m.tr.norm, m.tr.router, m.tr.sh_gate, m.tr.sh_up, m.tr.sh_down,
                            m.tr.sh_gw};
    const int64_t n[6] = {H, E * H, M * H, M * H, H * M, H};
    uint16_t *t = m.trunk + (int64_t)layer * m.tr.n;
    for (int i = 0; i < 6; i++) {
        if (!host[i]) continue;
        if (up)
            DS4F_CUDA(cudaMemcpyAsync(t + off[i], host[i], n[i] * 2, cudaMemcpyHostToDevice, m.stream));
        else
            DS4F_CUDA(cudaMemcpyAsync(host[i], t + off[i], n[i] * 2, cudaMemcpyDeviceToHost, m.stream));
    }
    DS4F_CUDA(cudaStreamSynchronize(m.stream));
    return 0;
}

int ds4f_gpu_model_set_trunk(Ds4fGpuModel *h, int layer, const uint16_t *norm,
                             const uint16_t *router, const uint16_t *sh_gate,
                             const uint16_t *sh_up, const uint16_t *sh_down,
                             const uint16_t *sh_gw) {
    DS4F_REQUIRE(h, "set_trunk: null model");
    uint16_t *const p[6] = {(uint16_t *)norm, (uint16_t *)router, (uint16_t *)sh_gate,
                            (uint16_t *)sh_up, (uint16_t *)sh_down, (uint16_t *)sh_gw};
    return trunk_io(h->m, layer, p, true);
}

int ds4f_gpu_model_get_trunk(const Ds4fGpuModel *h, int layer, uint16_t *norm,
                             uint16_t *router, uint16_t *sh_gate, uint16_t *sh_up,
                             uint16_t *sh_down, uint16_t *sh_gw) {
    DS4F_REQUIRE(h, "get_trunk: null model");
    uint16_t *const p[6] = {norm, router, sh_gate, sh_up, sh_down, sh_gw};
    return trunk_io(h->m, layer, p, false);
}

static int canon_slot(Model &m, uint8_t *slot_dev) {
    if (m.d.fmt != DS4F_FMT_FP8) return 0;
    for (int t = 0; t < 3; t++)
        if (launch_f8_canon(slot_dev + m.slot.rel_v[t], m.slot.rel_s[t] - m.slot.rel_v[t],
                            m.stream))
            return -1;
    return 0;
}

int ds4f_gpu_model_set_expert(Ds4fGpuModel *h, int layer, int expert, const uint8_t *slot) {
    DS4F_REQUIRE(h && slot, "set_expert: null argument");
    Model &m = h->m;
    DS4F_REQUIRE(!m.cache, "set_expert: a streaming model's experts are the caller's host pool");
    DS4F_REQUIRE(layer >= 0 && layer < m.d.n_layers, "set_expert: layer %d out of range", layer);
    DS4F_REQUIRE(expert >= m.d.expert_first && expert < m.d.expert_first + m.d.expert_count,
                 "set_expert: expert %d not in this shard", expert);
    uint8_t *dst = (uint8_t *)expert_ptr(&m, layer, expert);
    DS4F_CUDA(cudaMemcpyAsync(dst, slot, m.slot.nbytes, cudaMemcpyHostToDevice, m.stream));
    if (canon_slot(m, dst)) return -1;
    DS4F_CUDA(cudaStreamSynchronize(m.stream));
    return 0;
}

int ds4f_gpu_model_get_expert(const Ds4fGpuModel *h, int layer, int expert, uint8_t *slot) {
    DS4F_REQUIRE(h && slot, "get_expert: null argument");
    const Model &m = h->m;
    DS4F_REQUIRE(!m.cache, "get_expert: a streaming model's experts are the caller's host pool");
    DS4F_REQUIRE(layer >= 0 && layer < m.d.n_layers, "get_expert: layer %d out of range", layer);
    DS4F_REQUIRE(expert >= m.d.expert_first && expert < m.d.expert_first + m.d.expert_count,
                 "get_expert: expert %d not in this shard", expert);
    DS4F_CUDA(cudaMemcpyAsync(slot, expert_ptr(&m, layer, expert), m.slot.nbytes,
                              cudaMemcpyDeviceToHost, m.stream));
    DS4F_CUDA(cudaStreamSynchronize(m.stream));
    return 0;
}

int ds4f_gpu_pool_load(Ds4fGpuModel *h, const char *path) {
    DS4F_REQUIRE(h && path, "pool_load: null argument");
    Model &m = h->m;
    DS4F_REQUIRE(!m.cache, "pool_load: a streaming model reads its experts from the caller's host pool");
    int fd = open(path, O_RDONLY);
    DS4F_REQUIRE(fd >= 0, "pool_load: cannot open %s", path);
    uint8_t hdr[24];
    if (pread(fd, hdr, 24, 0) != 24) { close(fd); set_error("pool_load: short header in %s", path); return -1; }
    auto rd = [&](int o) { uint64_t v = 0; for (int i = 7; i >= 0; i--) v = (v << 8) | hdr[o + i]; return v; };
    uint64_t nb = rd(0), nl = rd(8), ne = rd(16);
    if ((int64_t)nb != m.slot.nbytes || (int)nl != m.d.n_layers || (int)ne != m.d.n_experts) {
        close(fd);
        set_error("pool_load: header (nbytes %llu, %llu layers x %llu experts) does not match "
                  "the model (%lld, %d x %d)", (unsigned long long)nb, (unsigned long long)nl,
                  (unsigned long long)ne, (long long)m.slot.nbytes, m.d.n_layers, m.d.n_experts);
        return -1;
    }
    off_t sz = lseek(fd, 0, SEEK_END);
    if (sz != (off_t)(24 + nb * nl * ne)) {
        close(fd);
        set_error("pool_load: size %lld, expected %llu", (long long)sz,
                  (unsigned long long)(24 + nb * nl * ne));
        return -1;
    }
    // stream the shard through two pinned staging buffers
    const size_t chunk = (size_t)64 << 20;
    void *stg[2] = {nullptr, nullptr};
    cudaEvent_t ev[2] = {nullptr, nullptr};
    int rc = -1;
    if (cudaMallocHost(&stg[0], chunk) != cudaSuccess || cudaMallocHost(&stg[1], chunk) != cudaSuccess ||
        cudaEventCreate(&ev[0]) != cudaSuccess || cudaEventCreate(&ev[1]) != cudaSuccess) {
        set_error("pool_load: pinned staging allocation failed");
        goto out;
    }
    {
        int b = 0;
        for (int L = 0; L < m.d.n_layers; L++) {
            // this shard's experts of layer L are contiguous in the file
            int64_t src = 24 + ((int64_t)L * m.d.n_experts + m.d.expert_first) * m.slot.nbytes;
            int64_t len = (int64_t)m.d.expert_count * m.slot.nbytes;
            uint8_t *dst = m.pool + (int64_t)L * m.d.expert_count * m.slot.nbytes;
            for (int64_t o = 0; o < len; o += chunk) {
                size_t n = (size_t)std::min<int64_t>(chunk, len - o);
                if (cudaEventSynchronize(ev[b]) != cudaSuccess) { set_error("pool_load: event"); goto out; }
                size_t got = 0;
                while (got < n) {
                    ssize_t r = pread(fd, (uint8_t *)stg[b] + got, n - got, src + o + got);
                    if (r <= 0) { set_error("pool_load: read error in %s", path); goto out; }
                    got += (size_t)r;
                }
                if (cudaMemcpyAsync(dst + o, stg[b], n, cudaMemcpyHostToDevice, m.stream) != cudaSuccess ||
                    cudaEventRecord(ev[b], m.stream) != cudaSuccess) {
                    set_error("pool_load: copy failed");
                    goto out;
                }
                b ^= 1;
            }
        }
        for (int L = 0; L < m.d.n_layers; L++)
            for (int e = 0; e < m.d.expert_count; e++)
                if (canon_slot(m, m.pool + ((int64_t)L * m.d.expert_count + e) * m.slot.nbytes))
                    goto out;
        if (cudaStreamSynchronize(m.stream) != cudaSuccess) { set_error("pool_load: sync failed"); goto out; }
        rc = 0;
    }
out:
    cudaStreamSynchronize(m.stream);
    if (ev[0]) cudaEventDestroy(ev[0]);
    if (ev[1]) cudaEventDestroy(ev[1]);
    if (stg[0]) cudaFreeHost(stg[0]);
    if (stg[1]) cudaFreeHost(stg[1]);
    close(fd);
    return rc;
}

int ds4f_gpu_moe_layer_dev(Ds4fGpuModel *h, int layer, float *state, int *idx, float *w,
                           void *stream) {
    DS4F_REQUIRE(h && state, "moe_layer: null argument");
    Model &m = h->m;
    DS4F_REQUIRE(layer >= 0 && layer < m.d.n_layers, "moe_layer: layer %d out of range", layer);
    DS4F_REQUIRE(m.d.expert_count == m.d.n_experts,
                 "moe_layer: model holds a shard; use the expert-parallel path");
    return on_model_stream(m, stream, [&](cudaStream_t st) {
        return moe_layer_launch(&m, layer, state, idx, w, st);
    });
}

int ds4f_gpu_moe_layer_partial_dev(Ds4fGpuModel *h, int layer, const float *state, int B, float *acc,
                                   int add_shared, void *stream) {
    DS4F_REQUIRE(h && state && acc && B > 0, "moe_layer_partial: bad arguments");
    Model &m = h->m;
    DS4F_REQUIRE(layer >= 0 && layer < m.d.n_layers, "moe_layer_partial: layer %d out of range", layer);
    const int H = m.d.hidden;
    return on_model_stream(m, stream, [&](cudaStream_t st) {
        for (int b = 0; b < B; b++)
            if (moe_layer_launch_ex(&m, layer, const_cast<float *>(state) + (int64_t)b * H, nullptr, nullptr,
                                    acc + (int64_t)b * H, true, add_shared != 0, st))
                return -1;
        return 0;
    });
}

int ds4f_gpu_moe_layer(Ds4fGpuModel *h, int layer, float *state, int *idx, float *w) {
    DS4F_REQUIRE(h && state, "moe_layer: null argument");
    Model &m = h->m;
    const int H = m.d.hidden, K = m.d.topk;
    DS4F_CUDA(cudaMemcpyAsync(m.state_dev, state, H * 4, cudaMemcpyHostToDevice, m.stream));
    if (ds4f_gpu_moe_layer_dev(h, layer, m.state_dev, m.idx_dev, m.w_dev, m.stream)) return -1;
    DS4F_CUDA(cudaMemcpyAsync(state, m.state_dev, H * 4, cudaMemcpyDeviceToHost, m.stream));
    if (idx) DS4F_CUDA(cudaMemcpyAsync(idx, m.idx_dev, K * 4, cudaMemcpyDeviceToHost, m.stream));
    if (w) DS4F_CUDA(cudaMemcpyAsync(w, m.w_dev, K * 4, cudaMemcpyDeviceToHost, m.stream));
    DS4F_CUDA(cudaStreamSynchronize(m.stream));
    return 0;
}

// One decode step of the layer stack, captured once into a CUDA graph per
// state buffer and replayed.
static int stack_step(Model &m, float *state, cudaStream_t st) {
    if (m.path != 1 && decode_eligible(&m)) return decode_launch(&m, state, 1, st);
    DS4F_REQUIRE(m.path != 2, "moe_stack: the persistent decode kernel does not cover this model");
    if (m.cache) {              // streaming: every layer waits for its routing on the host
        for (int L = 0; L < m.d.n_layers; L++)
            if (moe_layer_launch(&m, L, state, nullptr, nullptr, st)) return -1;
        return 0;
    }
    if (!m.graph || m.graph_state != state) {
        if (m.graph) { cudaGraphExecDestroy(m.graph); m.graph = nullptr; }
        cudaGraph_t g;
        DS4F_CUDA(cudaStreamBeginCapture(st, cudaStreamCaptureModeThreadLocal));
        int rc = 0;
        for (int L = 0; L < m.d.n_layers && !rc; L++)
            rc = moe_layer_launch(&m, L, state, nullptr, nullptr, st);
        cudaError_t e = cudaStreamEndCapture(st, &g);
        if (rc) { if (e == cudaSuccess) cudaGraphDestroy(g); return -1; }
        DS4F_CUDA(e);
        e = cudaGraphInstantiate(&m.graph, g, 0);
        cudaGraphDestroy(g);
        DS4F_CUDA(e);
        m.graph_state = state;
    }
    DS4F_CUDA(cudaGraphLaunch(m.graph, st));
    return 0;
}

int ds4f_gpu_moe_stack_dev(Ds4fGpuModel *h, float *state, int n_steps, void *stream) {
    DS4F_REQUIRE(h && state && n_steps >= 0, "moe_stack: bad arguments");
    Model &m = h->m;
    DS4F_REQUIRE(m.d.expert_count == m.d.n_experts,
                 "moe_stack: model holds a shard; use the expert-parallel path");
    return on_model_stream(m, stream, [&](cudaStream_t st) {
        if (n_steps > 0 && m.path != 1 && decode_eligible(&m))
            return decode_launch(&m, state, n_steps, st);
        for (int s = 0; s < n_steps; s++)
            if (stack_step(m, state, st)) return -1;
        return 0;
    });
}

// Error word of the persistent kernel (set on a barrier or copy timeout).
static int check_decode_error(const Model &m) {
    unsigned d[4];
    DS4F_CUDA(cudaMemcpy(d, m.w.diag, sizeof d, cudaMemcpyDeviceToHost));
    DS4F_REQUIRE(d[2] == 0, "decode kernel gave up waiting (code %u at CTA %u): a phase "
                 "barrier or weight copy did not complete", d[2], d[3]);
    return 0;
}

int ds4f_gpu_model_trace(Ds4fGpuModel *h, int64_t n_stamps) {
    DS4F_REQUIRE(h && n_stamps >= 0, "model_trace: bad arguments");
    Model &m = h->m;
    DS4F_CUDA(cudaStreamSynchronize(m.stream));
    if (m.trace) { cudaFree(m.trace); m.trace = nullptr; m.trace_n = 0; }
    if (n_stamps == 0) return 0;
    DS4F_CUDA(cudaMalloc(&m.trace, (size_t)n_stamps * 8));
    DS4F_CUDA(cudaMemset(m.trace, 0, (size_t)n_stamps * 8));
    m.trace_n = n_stamps;
    return 0;
}

int ds4f_gpu_model_route_log(Ds4fGpuModel *h, int n_layer_steps) {
    DS4F_REQUIRE(h && n_layer_steps >= 0, "model_route_log: bad arguments");
    Model &m = h->m;
    DS4F_CUDA(cudaStreamSynchronize(m.stream));
    if (m.log_base) { cudaFree(m.log_base); m.log_base = nullptr; }
    m.log_idx = nullptr; m.log_w = m.log_state = nullptr; m.log_n = 0;
    if (n_layer_steps == 0) return 0;
    const size_t n = (size_t)n_layer_steps, K = m.d.topk, H = m.d.hidden;
    const size_t b0 = al256(n * K * 4), b1 = al256(n * K * 4), b2 = al256(n * H * 4);
    DS4F_CUDA(cudaMalloc(&m.log_base, b0 + b1 + b2));
    DS4F_CUDA(cudaMemset(m.log_base, 0xFF, b0 + b1 + b2));      // -1 / NaN: not written
    m.log_idx = (int *)m.log_base;
    m.log_w = (float *)((char *)m.log_base + b0);
    m.log_state = (float *)((char *)m.log_base + b0 + b1);
    m.log_n = n_layer_steps;
    return 0;
}

int ds4f_gpu_model_route_log_read(const Ds4fGpuModel *h, int *idx, float *w, float *states, int n_layer_steps) {
    DS4F_REQUIRE(h && h->m.log_base && n_layer_steps >= 0 && n_layer_steps <= h->m.log_n,
                 "model_route_log_read: bad arguments (log of %d layer-steps)", h ? h->m.log_n : 0);
    const Model &m = h->m;
    const size_t n = (size_t)n_layer_steps, K = m.d.topk, H = m.d.hidden;
    DS4F_CUDA(cudaStreamSynchronize(m.stream));
    if (idx) DS4F_CUDA(cudaMemcpy(idx, m.log_idx, n * K * 4, cudaMemcpyDeviceToHost));
    if (w) DS4F_CUDA(cudaMemcpy(w, m.log_w, n * K * 4, cudaMemcpyDeviceToHost));
    if (states) DS4F_CUDA(cudaMemcpy(states, m.log_state, n * H * 4, cudaMemcpyDeviceToHost));
    return 0;
}

int ds4f_gpu_model_trace_read(const Ds4fGpuModel *h, uint64_t *out, int64_t n_stamps) {
    DS4F_REQUIRE(h && out && h->m.trace && n_stamps <= h->m.trace_n, "model_trace_read: bad arguments");
    DS4F_CUDA(cudaStreamSynchronize(h->m.stream));
    DS4F_CUDA(cudaMemcpy(out, h->m.trace, (size_t)n_stamps * 8, cudaMemcpyDeviceToHost));
    return 0;
}

int ds4f_gpu_model_set_wait_limit(Ds4fGpuModel *h, int64_t polls) {
    DS4F_REQUIRE(h && polls >= 0, "model_set_wait_limit: bad arguments");
    h->m.wait_limit = polls;
    return 0;
}

int ds4f_gpu_model_inject_peer_stall(Ds4fGpuModel *h, int layer_step) {
    DS4F_REQUIRE(h, "model_inject_peer_stall: null model");
    h->m.stall_peer_t = layer_step < 0 ? -1 : layer_step;
    return 0;
}

int ds4f_gpu_model_inject_stall(Ds4fGpuModel *h, int cta, int layer_step) {
    DS4F_REQUIRE(h && (cta < 0 || layer_step >= 0), "model_inject_stall: bad arguments");
    h->m.stall_cta = cta < 0 ? -1 : cta;
    h->m.stall_t = cta < 0 ? -1 : layer_step;
    return 0;
}

int ds4f_gpu_model_set_path(Ds4fGpuModel *h, int path) {
    DS4F_REQUIRE(h && path >= 0 && path <= 2, "model_set_path: bad arguments");
    DS4F_REQUIRE(path != 2 || decode_eligible(&h->m),
                 "model_set_path: the persistent decode kernel does not cover this model");
    h->m.path = path;
    return 0;
}

int ds4f_gpu_moe_stack(Ds4fGpuModel *h, float *state, int n_steps) {
    DS4F_REQUIRE(h && state, "moe_stack: null argument");
    Model &m = h->m;
    const int H = m.d.hidden;
    DS4F_CUDA(cudaMemcpyAsync(m.state_dev, state, H * 4, cudaMemcpyHostToDevice, m.stream));
    if (ds4f_gpu_moe_stack_dev(h, m.state_dev, n_steps, m.stream)) return -1;
    DS4F_CUDA(cudaMemcpyAsync(state, m.state_dev, H * 4, cudaMemcpyDeviceToHost, m.stream));
    DS4F_CUDA(cudaStreamSynchronize(m.stream));
    return check_decode_error(m);
}

int ds4f_gpu_model_stats(const Ds4fGpuModel *h, uint64_t out[2]) {
    DS4F_REQUIRE(h && out, "model_stats: null argument");
    unsigned d[4];
    DS4F_CUDA(cudaStreamSynchronize(h->m.stream));
    DS4F_CUDA(cudaMemcpy(d, h->m.w.diag, sizeof d, cudaMemcpyDeviceToHost));
    out[0] = d[0];
    out[1] = d[1];
    return check_decode_error(h->m);
}

int ds4f_gpu_synth_f32(float *dst, int64_t n, uint64_t seed, uint32_t layer, uint32_t kind,
                       uint32_t x, uint32_t t, double sigma, void *stream) {
    DS4F_REQUIRE(dst && n >= 0, "synth_f32: bad arguments");
    cudaStream_t st;
    if (stream_of(stream, &st)) return -1;
    uint64_t tid = ((uint64_t)layer << 40) | ((uint64_t)(kind & 0xFF) << 32) |
                   ((uint64_t)(x & 0xFFFFFF) << 8) | (uint64_t)(t & 0xFF);
    auto mix = [](uint64_t z) {
        z += 0x9E3779B97F4A7C15ull;
        z = (z ^ (z >> 30)) * 0xBF58476D1CE4E5B9ull;
        z = (z ^ (z >> 27)) * 0x94D049BB133111EBull;
        return z ^ (z >> 31);
    };
    return synth_f32(dst, n, mix(mix(seed) ^ tid), sigma, st);
}

}  // extern "C"
