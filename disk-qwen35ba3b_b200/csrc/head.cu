// head.cu -- the step after the MoE path: the output head's logits over the
// vocabulary and the greedy pick (ds4f_head_logits, src/head.c:243-299;
// ds4f_argmax, src/head.c:303-309), the head's weights resident in HBM.
//
// The matvec is k_head_bf16 below for BF16 heads of width 1024, 2048 or 4096,
// else the job kernel of matvec.cu on one job of R = vocabulary rows
// (HBM-bound: the weight bytes are read once per call). The pick is a
// two-stage reduction with the reference's rule: start from logits[0], take
// an index only if its logit is strictly greater -- so the lowest index wins
// ties, NaN logits are never taken, and a NaN logits[0] is the answer.
#include <algorithm>
#include <climits>
#include <cstring>

#include "common.cuh"
#include "matvec.cuh"
#include "../../include/ds4f/gpu_cuda.h"

namespace ds4f {
namespace {

constexpr int kArgThreads = 1024;
constexpr int kArgBlocks = 148;         // one per SM: 248k logits are ~1 MB

struct Best {
    float v;
    int i;                              // INT_MAX: no candidate yet
};

__device__ __forceinline__ Best better(Best a, Best b) {
    if (b.i == INT_MAX) return a;
    if (a.i == INT_MAX) return b;
    if (b.v > a.v || (b.v == a.v && b.i < a.i)) return b;
    return a;
}

__device__ Best block_best(Best m) {
    __shared__ float sv[kArgThreads / 32];
    __shared__ int si[kArgThreads / 32];
    for (int o = 16; o > 0; o >>= 1) {
        Best t{__shfl_xor_sync(0xFFFFFFFFu, m.v, o), __shfl_xor_sync(0xFFFFFFFFu, m.i, o)};
        m = better(m, t);
    }
    const int w = threadIdx.x >> 5, lane = threadIdx.x & 31;
    if (lane == 0) { sv[w] = m.v; si[w] = m.i; }
    __syncthreads();
    if (w == 0) {
        m = lane < (int)(blockDim.x >> 5) ? Best{sv[lane], si[lane]} : Best{0.f, INT_MAX};
        for (int o = 16; o > 0; o >>= 1) {
            Best t{__shfl_xor_sync(0xFFFFFFFFu, m.v, o), __shfl_xor_sync(0xFFFFFFFFu, m.i, o)};
            m = better(m, t);
        }
    }
    return m;                           // valid in warp 0
}

__global__ void __launch_bounds__(kArgThreads) k_argmax_part(const float *__restrict__ y, int n,
                                                             float *__restrict__ pv, int *__restrict__ pi) {
    Best m{0.f, INT_MAX};
    for (int i = blockIdx.x * blockDim.x + threadIdx.x; i < n; i += gridDim.x * blockDim.x) {
        const float v = y[i];
        if (v == v && (m.i == INT_MAX || v > m.v)) m = Best{v, i};   // indices rise: first max kept
    }
    m = block_best(m);
    if (threadIdx.x == 0) { pv[blockIdx.x] = m.v; pi[blockIdx.x] = m.i; }
}

__global__ void __launch_bounds__(kArgThreads) k_argmax_final(const float *__restrict__ y, const float *__restrict__ pv,
                                                              const int *__restrict__ pi, int nparts,
                                                              int *__restrict__ out) {
    Best m{0.f, INT_MAX};
    for (int p = threadIdx.x; p < nparts; p += blockDim.x) m = better(m, Best{pv[p], pi[p]});
    m = block_best(m);
    if (threadIdx.x == 0) {
        const float y0 = y[0];
        *out = (y0 != y0 || m.i == INT_MAX) ? 0 : m.i;
    }
}

// BF16 head rows: one warp per row, the row's H/256 16-byte chunks per lane
// loaded together (lane-contiguous, so each load instruction of a warp covers
// 512 contiguous bytes), x staged once per block in shared memory. About 50
// registers a thread: four 256-thread blocks per SM, 32 warps streaming.
template <int CPL>
__global__ void __launch_bounds__(256, 4) k_head_bf16(const uint16_t *__restrict__ W, const float *__restrict__ x,
                                                      float *__restrict__ y, int V) {
    constexpr int H = CPL * 256;
    __shared__ __align__(16) float xs[H];
    for (int i = threadIdx.x; i < H; i += blockDim.x) xs[i] = x[i];
    __syncthreads();
    const int lane = threadIdx.x & 31;
    const int warps = gridDim.x * (blockDim.x >> 5);
    for (int r = blockIdx.x * (blockDim.x >> 5) + (threadIdx.x >> 5); r < V; r += warps) {
        const uint8_t *row = (const uint8_t *)W + (int64_t)r * H * 2;
        uint4 c[CPL];
#pragma unroll
        for (int k = 0; k < CPL; k++) c[k] = ldg_stream(row + (size_t)(lane + 32 * k) * 16);
        float acc = 0.f;
#pragma unroll
        for (int k = 0; k < CPL; k++) {
            const float4 *xv = (const float4 *)(xs + (lane + 32 * k) * 8);
            const float4 x0 = xv[0], x1 = xv[1];
            const uint32_t w[4] = {c[k].x, c[k].y, c[k].z, c[k].w};
            const float xx[8] = {x0.x, x0.y, x0.z, x0.w, x1.x, x1.y, x1.z, x1.w};
#pragma unroll
            for (int j = 0; j < 4; j++) {
                acc = fmaf(__uint_as_float(w[j] << 16), xx[2 * j], acc);
                acc = fmaf(__uint_as_float(w[j] & 0xFFFF0000u), xx[2 * j + 1], acc);
            }
        }
        for (int o = 16; o > 0; o >>= 1) acc += __shfl_xor_sync(0xFFFFFFFFu, acc, o);
        if (lane == 0) y[r] = acc;
    }
}

int argmax_launch(const float *y, int n, float *pv, int *pi, int *out, cudaStream_t st) {
    const int nb = std::max(1, std::min(kArgBlocks, (n + kArgThreads - 1) / kArgThreads));
    k_argmax_part<<<nb, kArgThreads, 0, st>>>(y, n, pv, pi);
    DS4F_CUDA(cudaGetLastError());
    k_argmax_final<<<1, kArgThreads, 0, st>>>(y, pv, pi, nb, out);
    DS4F_CUDA(cudaGetLastError());
    return 0;
}

}  // namespace
}  // namespace ds4f

struct Ds4fGpuHead {
    int dtype = 0, V = 0, H = 0, device = 0, nitems = 0;
    int rows_kernel = 0;                // BF16 with H = 1024 / 2048 / 4096: k_head_bf16
    int grid = 0;
    const void *wdev = nullptr;
    void *wbuf = nullptr;               // weights, scales, biases, x, logits, job, partials
    float *x = nullptr, *y = nullptr, *pv = nullptr;
    int *pi = nullptr, *best = nullptr;
    ds4f::MvJob *job = nullptr;
    float *host_x = nullptr, *host_y = nullptr;
    int *host_best = nullptr;
    cudaStream_t stream = nullptr;
};

extern "C" {

int ds4f_gpu_head_create(int dtype, const void *w, const void *scales, const void *biases, int V, int H,
                         int SR, int SC, Ds4fGpuHead **out) {
    using namespace ds4f;
    DS4F_REQUIRE(out && w && V > 0 && H > 0, "head_create: bad arguments");
    *out = nullptr;
    int fmt;
    size_t wb, sb = 0, bb = 0;
    const int64_t n = (int64_t)V * H;
    if (dtype == 2) {                                   // F8_E4M3, E8M0 block scales [SR x SC]
        fmt = DS4F_FMT_FP8;
        wb = (size_t)n;
        if (scales) sb = (size_t)std::max(SR, 1) * std::max(SC, 1);
    } else if (dtype == 6) {                            // MLX 4-bit: H is the decoded width
        DS4F_REQUIRE(scales && H % 8 == 0, "head_create: MLX4 head needs scales and H %% 8 == 0");
        fmt = DS4F_FMT_MLX4;
        wb = (size_t)(n / 8) * 4;
        sb = (size_t)((n + 63) / 64) * 2;
        if (biases) bb = sb;
    } else if (dtype == 4 || dtype == 3) {              // BF16 (the reference's default branch)
        fmt = DS4F_FMT_BF16;
        wb = (size_t)n * 2;
    } else {
        DS4F_REQUIRE(false, "head_create: head dtype %d (%s) is not built here; FP8 (2), BF16 (4) and MLX4 (6) are",
                     dtype, dtype == 0 ? "F32" : dtype == 1 ? "I8" : dtype == 5 ? "F16" : "unknown");
    }
    auto al = [](size_t v) { return (v + 255) & ~(size_t)255; };
    const int nparts = 148;
    size_t ow = 0, os = al(ow + wb), ob = al(os + sb), ox = al(ob + bb), oy = al(ox + (size_t)H * 4),
           oj = al(oy + (size_t)V * 4), opv = al(oj + sizeof(MvJob)), opi = al(opv + nparts * 4),
           obest = al(opi + nparts * 4), tot = al(obest + 4);
    size_t fre = 0, totm = 0;
    DS4F_CUDA(cudaMemGetInfo(&fre, &totm));
    DS4F_REQUIRE((double)tot <= 0.95 * (double)fre, "head_create: needs %.2f GB, %.2f GB free", tot / 1e9,
                 fre / 1e9);
    Ds4fGpuHead *h = new Ds4fGpuHead();
    h->dtype = dtype; h->V = V; h->H = H;
    cudaGetDevice(&h->device);
    auto fail = [&](const char *what) {
        ds4f_gpu_head_free(h);
        set_error("head_create: %s", what);
        return -1;
    };
    if (cudaMalloc(&h->wbuf, tot) != cudaSuccess) return fail("device allocation failed");
    if (cudaStreamCreateWithFlags(&h->stream, cudaStreamNonBlocking) != cudaSuccess) return fail("stream");
    if (cudaHostAlloc((void **)&h->host_x, (size_t)H * 4, cudaHostAllocDefault) != cudaSuccess ||
        cudaHostAlloc((void **)&h->host_y, (size_t)V * 4, cudaHostAllocDefault) != cudaSuccess ||
        cudaHostAlloc((void **)&h->host_best, 4, cudaHostAllocDefault) != cudaSuccess)
        return fail("pinned host buffers");
    uint8_t *base = (uint8_t *)h->wbuf;
    if (cudaMemcpy(base + ow, w, wb, cudaMemcpyHostToDevice) != cudaSuccess ||
        (sb && cudaMemcpy(base + os, scales, sb, cudaMemcpyHostToDevice) != cudaSuccess) ||
        (bb && cudaMemcpy(base + ob, biases, bb, cudaMemcpyHostToDevice) != cudaSuccess))
        return fail("weight upload failed");
    h->x = (float *)(base + ox);
    h->y = (float *)(base + oy);
    h->job = (MvJob *)(base + oj);
    h->pv = (float *)(base + opv);
    h->pi = (int *)(base + opi);
    h->best = (int *)(base + obest);
    MvJob J;
    memset(&J, 0, sizeof J);
    J.fmt = fmt; J.R = V; J.C = H; J.SR = std::max(SR, 1); J.SC = std::max(SC, 1); J.bsize = 32;
    J.scale_kind = DS4F_SCALE_E8M0;
    J.canon = fmt == DS4F_FMT_FP8;                     // the reference table's e=15 rule in-kernel
    J.v = base + ow;
    J.s = sb ? base + os : nullptr;
    J.b = bb ? base + ob : nullptr;
    J.x = h->x;
    J.y = h->y;
    h->wdev = base + ow;
    if (fmt == DS4F_FMT_BF16 && (H == 1024 || H == 2048 || H == 4096)) {
        int sms = 0;
        cudaDeviceGetAttribute(&sms, cudaDevAttrMultiProcessorCount, h->device);
        h->rows_kernel = 1;
        h->grid = std::max(1, std::min(4 * sms, (V + 7) / 8));   // every block resident
    }
    h->nitems = plan_jobs(&J, 1);
    if (h->nitems < 0) { ds4f_gpu_head_free(h); return -1; }
    if (cudaMemcpy(h->job, &J, sizeof J, cudaMemcpyHostToDevice) != cudaSuccess) return fail("job upload");
    *out = h;
    return 0;
}

void ds4f_gpu_head_free(Ds4fGpuHead *h) {
    if (!h) return;
    int cur = 0;
    cudaGetDevice(&cur);
    cudaSetDevice(h->device);
    if (h->stream) cudaStreamSynchronize(h->stream);
    if (h->wbuf) cudaFree(h->wbuf);
    if (h->host_x) cudaFreeHost(h->host_x);
    if (h->host_y) cudaFreeHost(h->host_y);
    if (h->host_best) cudaFreeHost(h->host_best);
    if (h->stream) cudaStreamDestroy(h->stream);
    cudaSetDevice(cur);
    delete h;
}

static int head_matvec(Ds4fGpuHead *h, cudaStream_t st) {
    using namespace ds4f;
    if (!h->rows_kernel) return launch_jobs(h->job, 1, h->nitems, st);
    const uint16_t *w = (const uint16_t *)h->wdev;
    if (h->H == 1024) k_head_bf16<4><<<h->grid, 256, 0, st>>>(w, h->x, h->y, h->V);
    else if (h->H == 2048) k_head_bf16<8><<<h->grid, 256, 0, st>>>(w, h->x, h->y, h->V);
    else k_head_bf16<16><<<h->grid, 256, 0, st>>>(w, h->x, h->y, h->V);
    DS4F_CUDA(cudaGetLastError());
    return 0;
}

int ds4f_gpu_head_logits_dev(Ds4fGpuHead *h, const float *state_dev, float *logits_dev, int *argmax_dev,
                             void *stream) {
    using namespace ds4f;
    DS4F_REQUIRE(h && state_dev, "head_logits: null argument");
    cudaStream_t st = (cudaStream_t)stream;           // NULL: the default stream, as every _dev call
    DS4F_CUDA(cudaMemcpyAsync(h->x, state_dev, (size_t)h->H * 4, cudaMemcpyDeviceToDevice, st));
    if (head_matvec(h, st)) return -1;
    if (argmax_dev && argmax_launch(h->y, h->V, h->pv, h->pi, argmax_dev, st)) return -1;
    if (logits_dev)
        DS4F_CUDA(cudaMemcpyAsync(logits_dev, h->y, (size_t)h->V * 4, cudaMemcpyDeviceToDevice, st));
    return 0;
}

int ds4f_gpu_head_logits(Ds4fGpuHead *h, const float *state, float *logits, int *argmax) {
    using namespace ds4f;
    DS4F_REQUIRE(h && state, "head_logits: null argument");
    cudaStream_t st = h->stream;
    memcpy(h->host_x, state, (size_t)h->H * 4);
    DS4F_CUDA(cudaMemcpyAsync(h->x, h->host_x, (size_t)h->H * 4, cudaMemcpyHostToDevice, st));
    if (head_matvec(h, st)) return -1;
    if (argmax) {
        if (argmax_launch(h->y, h->V, h->pv, h->pi, h->best, st)) return -1;
        DS4F_CUDA(cudaMemcpyAsync(h->host_best, h->best, 4, cudaMemcpyDeviceToHost, st));
    }
    if (logits) DS4F_CUDA(cudaMemcpyAsync(h->host_y, h->y, (size_t)h->V * 4, cudaMemcpyDeviceToHost, st));
    DS4F_CUDA(cudaStreamSynchronize(st));
    if (argmax) *argmax = *h->host_best;
    if (logits) memcpy(logits, h->host_y, (size_t)h->V * 4);
    return 0;
}

int ds4f_gpu_argmax_dev(const float *logits_dev, int n, int *out_dev, void *stream) {
    using namespace ds4f;
    DS4F_REQUIRE(logits_dev && out_dev && n > 0, "argmax: bad arguments");
    cudaStream_t st = (cudaStream_t)stream;
    float *pv;
    int *pi;
    DS4F_CUDA(cudaMallocAsync((void **)&pv, 148 * 8, st));
    pi = (int *)(pv + 148);
    int rc = argmax_launch(logits_dev, n, pv, pi, out_dev, st);
    cudaFreeAsync(pv, st);
    return rc;
}

}  // extern "C"
