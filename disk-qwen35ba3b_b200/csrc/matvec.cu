// matvec.cu -- fused dequant + matvec for FP8-E4M3 (block-scaled), MXFP4
// (E2M1 + E8M0 per 32) and bf16, batch 1, on CUDA cores.
//
// Replaces the reference's ds4f_f8_matvec (src/kernels.c:243-270),
// ds4f_mxfp4_matvec (:48-62, a decode-to-scratch then dot two-pass design)
// and ds4f_bf16_matvec (:91-103) with one pass over the packed weights:
// 16-byte streaming loads, in-register decode, fp32 FMA against x held in
// registers, warp-shuffle reduction. The reference accumulates each row
// sequentially in fp32; this kernel sums in a different order, so results
// agree within fp32 reassociation error (tests: max rel 2e-3 of max |y|;
// observed ~1e-6). Dequantised values themselves are bit-exact
// (launch_f8_decode / launch_mx_decode).
//
// Work is a flat list of 64-row items over all jobs in the launch (the 24
// matvecs of an 8-expert layer run as one launch); a persistent grid walks
// the items.
#include "matvec.cuh"

#include <algorithm>

namespace ds4f {

namespace {

template <int FMT> struct Fmt;
template <> struct Fmt<DS4F_FMT_FP8>  { static constexpr int CE = 16, KMAX = 4; };
template <> struct Fmt<DS4F_FMT_MXFP4> { static constexpr int CE = 32, KMAX = 2; };
template <> struct Fmt<DS4F_FMT_BF16> { static constexpr int CE = 8,  KMAX = 8; };
template <> struct Fmt<DS4F_FMT_MLX4> { static constexpr int CE = 32, KMAX = 2; };

// MLX4 nibble q (0..15) of word w at position k -> q * 2^-130 exactly (an
// fp32 denormal with mantissa q << 19); x pre-scaled by 2^64 keeps the
// products normal; DS4F_MLX4_POST = 2^130 / 2^64 undoes both.
template <int K>
__device__ __forceinline__ float mlx4_raw(uint32_t w) {
    constexpr int sh = 4 * K - 19;
    uint32_t t = sh >= 0 ? (w >> sh) : (w << -sh);
    return __uint_as_float(t & 0x00780000u);
}
#define DS4F_MLX4_POST 7.378697629483821e+19f   // 2^66

__device__ __forceinline__ float mlx4_word_dot(uint32_t w, const float *x) {
    float a = 0.f, b = 0.f;
    a = fmaf(mlx4_raw<0>(w), x[0], a); b = fmaf(mlx4_raw<1>(w), x[1], b);
    a = fmaf(mlx4_raw<2>(w), x[2], a); b = fmaf(mlx4_raw<3>(w), x[3], b);
    a = fmaf(mlx4_raw<4>(w), x[4], a); b = fmaf(mlx4_raw<5>(w), x[5], b);
    a = fmaf(mlx4_raw<6>(w), x[6], a); b = fmaf(mlx4_raw<7>(w), x[7], b);
    return a + b;
}

__device__ __forceinline__ float f8_scale(const MvJob &J, int r, int c) {
    int sr = (int)(((int64_t)r * J.SR) / J.R);
    int sc = (int)(((int64_t)c * J.SC) / J.C);
    int i = sr * J.SC + sc;
    if (!J.s) return 1.0f;
    if (J.scale_kind == DS4F_SCALE_F32) return __ldg((const float *)J.s + i);
    return e8m0_to_f32(__ldg((const uint8_t *)J.s + i));
}

template <int FMT>
__device__ __forceinline__ float chunk_dot(uint4 q, const float *x) {
    if constexpr (FMT == DS4F_FMT_FP8) return f8_dot16(q, x);
    else if constexpr (FMT == DS4F_FMT_MXFP4) return e2m1_dot32(q, x);
    else if constexpr (FMT == DS4F_FMT_MLX4)
        return mlx4_word_dot(q.x, x) + mlx4_word_dot(q.y, x + 8) +
               mlx4_word_dot(q.z, x + 16) + mlx4_word_dot(q.w, x + 24);
    else return bf16_dot8(q, x);
}

// Scale applied to one chunk's raw dot (units documented in common.cuh).
template <int FMT>
__device__ __forceinline__ float chunk_scaled(const MvJob &J, int r, int q,
                                              float d) {
    if constexpr (FMT == DS4F_FMT_FP8) {
        return (d * DS4F_F8_POST) * f8_scale(J, r, q * 16);
    } else if constexpr (FMT == DS4F_FMT_MXFP4) {
        int64_t bi = ((int64_t)r * J.C + (int64_t)q * 32) / J.bsize;
        return (d * DS4F_E2M1_POST) *
               e8m0_to_f32(__ldg((const uint8_t *)J.s + bi));
    } else if constexpr (FMT == DS4F_FMT_MLX4) {
        int64_t g = ((int64_t)r * J.C + (int64_t)q * 32) / 64;
        return (d * DS4F_MLX4_POST) *
               bf16_to_f32(__ldg((const uint16_t *)J.s + g));
    } else {
        return d;
    }
}

// MLX4 bias term of one chunk: b_g * sum(x over the chunk's 32 columns).
__device__ __forceinline__ float mlx4_bias(const MvJob &J, int r, int q, float xsum) {
    if (!J.b) return 0.0f;
    int64_t g = ((int64_t)r * J.C + (int64_t)q * 32) / 64;
    return bf16_to_f32(__ldg((const uint16_t *)J.b + g)) * xsum;
}

template <int FMT>
__device__ __forceinline__ const uint8_t *row_ptr(const MvJob &J, int r) {
    const uint8_t *v = (const uint8_t *)J.v;
    if constexpr (FMT == DS4F_FMT_FP8) return v + (int64_t)r * J.C;
    else if constexpr (FMT == DS4F_FMT_MXFP4 || FMT == DS4F_FMT_MLX4)
        return v + (int64_t)r * J.C / 2;
    else return v + (int64_t)r * J.C * 2;
}

// Vector path: lanes_per_row (lpr) lanes cover a row, each lane holds its
// columns of x in registers for a tile of up to KMAX chunks per lane, and
// each warp owns up to 8 row slots of the 64-row item.
template <int FMT>
__device__ void item_fast(const MvJob &J, int row0) {
    constexpr int CE = Fmt<FMT>::CE, KMAX = Fmt<FMT>::KMAX;
    const int lane = threadIdx.x & 31, warp = threadIdx.x >> 5;
    const int lpr = J.lpr, rps = 32 / lpr;
    const int sub = lane / lpr, ql = lane % lpr;
    const int nslots = kMvRowsPerItem / rps;
    const int nq = J.nq;
    float acc[8];
#pragma unroll
    for (int s = 0; s < 8; s++) acc[s] = 0.f;
    const float pre = (FMT == DS4F_FMT_BF16) ? 1.0f : DS4F_X_PRESCALE;
    for (int t0 = 0; t0 < nq; t0 += lpr * KMAX) {
        float xr[KMAX][CE];
        float xsum[KMAX];
#pragma unroll
        for (int k = 0; k < KMAX; k++) {
            int q = t0 + ql + lpr * k;
#pragma unroll
            for (int e = 0; e < CE; e += 4) {
                float4 v = make_float4(0.f, 0.f, 0.f, 0.f);
                if (q < nq) v = __ldg((const float4 *)(J.x + q * CE + e));
                xr[k][e] = v.x * pre; xr[k][e + 1] = v.y * pre;
                xr[k][e + 2] = v.z * pre; xr[k][e + 3] = v.w * pre;
            }
            xsum[k] = 0.f;
            if constexpr (FMT == DS4F_FMT_MLX4) {
#pragma unroll
                for (int e = 0; e < CE; e++) xsum[k] += xr[k][e];
                xsum[k] *= 1.0f / DS4F_X_PRESCALE;
            }
        }
#pragma unroll
        for (int s = 0; s < 8; s += 2) {
            int sl0 = warp + 8 * s, sl1 = warp + 8 * (s + 1);
            int r0 = row0 + sl0 * rps + sub, r1 = row0 + sl1 * rps + sub;
            bool ok0 = sl0 < nslots && r0 < J.R, ok1 = sl1 < nslots && r1 < J.R;
            uint4 b0[KMAX], b1[KMAX];
#pragma unroll
            for (int k = 0; k < KMAX; k++) {
                int q = t0 + ql + lpr * k;
                b0[k] = b1[k] = make_uint4(0, 0, 0, 0);
                if (ok0 && q < nq) b0[k] = ldg_stream(row_ptr<FMT>(J, r0) + (int64_t)q * 16);
                if (ok1 && q < nq) b1[k] = ldg_stream(row_ptr<FMT>(J, r1) + (int64_t)q * 16);
            }
#pragma unroll
            for (int k = 0; k < KMAX; k++) {
                int q = t0 + ql + lpr * k;
                if (q >= nq) continue;
                if constexpr (FMT == DS4F_FMT_FP8) {
                    if (J.canon) { b0[k] = f8_canon16(b0[k]); b1[k] = f8_canon16(b1[k]); }
                }
                if (ok0) acc[s] += chunk_scaled<FMT>(J, r0, q, chunk_dot<FMT>(b0[k], xr[k]));
                if (ok1) acc[s + 1] += chunk_scaled<FMT>(J, r1, q, chunk_dot<FMT>(b1[k], xr[k]));
                if constexpr (FMT == DS4F_FMT_MLX4) {
                    if (ok0) acc[s] += mlx4_bias(J, r0, q, xsum[k]);
                    if (ok1) acc[s + 1] += mlx4_bias(J, r1, q, xsum[k]);
                }
            }
        }
    }
#pragma unroll
    for (int s = 0; s < 8; s++) {
        float v = acc[s];
        for (int o = lpr >> 1; o > 0; o >>= 1) v += __shfl_xor_sync(0xFFFFFFFFu, v, o);
        int sl = warp + 8 * s, r = row0 + sl * rps + sub;
        if (ql == 0 && sl < nslots && r < J.R) {
            if constexpr (FMT == DS4F_FMT_BF16) {
                J.y[r] = v + (J.s ? ((const float *)J.s)[r] : 0.0f);
            } else {
                J.y[r] = v;
            }
        }
    }
}

// Any-shape path: warp per row, lanes stride the columns one element at a
// time with the reference's per-element scale index.
template <int FMT>
__device__ void item_generic(const MvJob &J, int row0) {
    const int lane = threadIdx.x & 31, warp = threadIdx.x >> 5;
    for (int r = row0 + warp; r < min(row0 + kMvRowsPerItem, J.R); r += 8) {
        float acc = 0.f;
        for (int c = lane; c < J.C; c += 32) {
            float w;
            if constexpr (FMT == DS4F_FMT_FP8) {
                uint32_t b = ((const uint8_t *)J.v)[(int64_t)r * J.C + c];
                if (J.canon && (b & 0x78u) == 0x78u) b = (b & 0x80u) | 0x7Eu;
                w = (f8_raw<0>(b) * DS4F_F8_UNSCALE) * f8_scale(J, r, c);
            } else if constexpr (FMT == DS4F_FMT_MXFP4) {
                int64_t i = (int64_t)r * J.C + c;
                uint32_t nib = (((const uint8_t *)J.v)[i >> 1] >> ((i & 1) ? 4 : 0)) & 0xFu;
                w = (e2m1_raw(nib) * DS4F_E2M1_UNSCALE) *
                    e8m0_to_f32(((const uint8_t *)J.s)[i / J.bsize]);
            } else if constexpr (FMT == DS4F_FMT_MLX4) {
                int64_t k = (int64_t)r * J.C + c;
                uint32_t q = (((const uint32_t *)J.v)[k >> 3] >> (4 * (k & 7))) & 0xFu;
                float sc = bf16_to_f32(((const uint16_t *)J.s)[k / 64]);
                float bi = J.b ? bf16_to_f32(((const uint16_t *)J.b)[k / 64]) : 0.0f;
                w = fmaf((float)q, sc, bi);
            } else {
                w = bf16_to_f32(((const uint16_t *)J.v)[(int64_t)r * J.C + c]);
            }
            acc = fmaf(w, __ldg(J.x + c), acc);
        }
        acc = warp_sum(acc);
        if (lane == 0) {
            if constexpr (FMT == DS4F_FMT_BF16)
                acc += J.s ? ((const float *)J.s)[r] : 0.0f;
            J.y[r] = acc;
        }
    }
}

__global__ void __launch_bounds__(kMvThreads)
k_mv_jobs(const MvJob *__restrict__ jobs, int njobs, int nitems) {
    __shared__ MvJob sj;
    for (int item = blockIdx.x; item < nitems; item += gridDim.x) {
        __syncthreads();
        if (threadIdx.x == 0) {
            int lo = 0, hi = njobs - 1;
            while (lo < hi) {                      // last job with item0 <= item
                int mid = (lo + hi + 1) >> 1;
                if (jobs[mid].item0 <= item) lo = mid; else hi = mid - 1;
            }
            sj = jobs[lo];
        }
        __syncthreads();
        const MvJob J = sj;
        int row0 = (item - J.item0) * kMvRowsPerItem;
        if (J.fast) {
            if (J.fmt == DS4F_FMT_FP8) item_fast<DS4F_FMT_FP8>(J, row0);
            else if (J.fmt == DS4F_FMT_MXFP4) item_fast<DS4F_FMT_MXFP4>(J, row0);
            else if (J.fmt == DS4F_FMT_MLX4) item_fast<DS4F_FMT_MLX4>(J, row0);
            else item_fast<DS4F_FMT_BF16>(J, row0);
        } else {
            if (J.fmt == DS4F_FMT_FP8) item_generic<DS4F_FMT_FP8>(J, row0);
            else if (J.fmt == DS4F_FMT_MXFP4) item_generic<DS4F_FMT_MXFP4>(J, row0);
            else if (J.fmt == DS4F_FMT_MLX4) item_generic<DS4F_FMT_MLX4>(J, row0);
            else item_generic<DS4F_FMT_BF16>(J, row0);
        }
    }
}

__global__ void k_f8_decode(const uint8_t *W, int kind, const void *scales,
                            int R, int C, int SR, int SC, int r0, int r1,
                            float *out) {
    int64_t n = (int64_t)(r1 - r0) * C;
    for (int64_t i = blockIdx.x * (int64_t)blockDim.x + threadIdx.x; i < n;
         i += (int64_t)gridDim.x * blockDim.x) {
        int r = r0 + (int)(i / C), c = (int)(i % C);
        uint32_t b = W[(int64_t)r * C + c];
        if ((b & 0x78u) == 0x78u) b = (b & 0x80u) | 0x7Eu;
        float v = f8_raw<0>(b) * DS4F_F8_UNSCALE;          // exact
        int sr = (int)(((int64_t)r * (SR < 1 ? 1 : SR)) / R);
        int sc = (int)(((int64_t)c * (SC < 1 ? 1 : SC)) / C);
        int si = sr * (SC < 1 ? 1 : SC) + sc;
        float s = !scales ? 1.0f
                  : kind == DS4F_SCALE_F32 ? ((const float *)scales)[si]
                                           : e8m0_to_f32(((const uint8_t *)scales)[si]);
        out[i] = __fmul_rn(v, s);
    }
}

__global__ void k_mx_decode(const uint8_t *vals, const uint8_t *scales,
                            int64_t n, int bsize, float *out) {
    for (int64_t i = blockIdx.x * (int64_t)blockDim.x + threadIdx.x; i < n;
         i += (int64_t)gridDim.x * blockDim.x) {
        uint32_t nib = (vals[i >> 1] >> ((i & 1) ? 4 : 0)) & 0xFu;
        float v = e2m1_raw(nib) * DS4F_E2M1_UNSCALE;       // exact
        out[i] = __fmul_rn(v, e8m0_to_f32(scales[i / bsize]));
    }
}

__global__ void k_f8_canon(uint8_t *buf, int64_t n) {
    int64_t n16 = n / 16;
    uint4 *b4 = (uint4 *)buf;
    for (int64_t i = blockIdx.x * (int64_t)blockDim.x + threadIdx.x; i < n16;
         i += (int64_t)gridDim.x * blockDim.x)
        b4[i] = f8_canon16(b4[i]);
    if (blockIdx.x == 0)
        for (int64_t i = n16 * 16 + threadIdx.x; i < n; i += blockDim.x) {
            uint32_t b = buf[i];
            if ((b & 0x78u) == 0x78u) buf[i] = (uint8_t)((b & 0x80u) | 0x7Eu);
        }
}

int grid_for(int64_t work, int per_block) {
    int dev = 0, sms = 148;
    cudaGetDevice(&dev);
    cudaDeviceGetAttribute(&sms, cudaDevAttrMultiProcessorCount, dev);
    int64_t g = (work + per_block - 1) / per_block;
    return (int)std::max<int64_t>(1, std::min<int64_t>(g, (int64_t)sms * 8));
}

}  // namespace

int plan_jobs(MvJob *jobs, int njobs) {
    int items = 0;
    for (int j = 0; j < njobs; j++) {
        MvJob &J = jobs[j];
        DS4F_REQUIRE(J.R >= 0 && J.C >= 1, "matvec: bad shape %d x %d", J.R, J.C);
        if (J.streamed) {                       // the stream kernel's job: no items here
            J.item0 = items;
            continue;
        }
        DS4F_REQUIRE(J.fmt == DS4F_FMT_FP8 || J.fmt == DS4F_FMT_MXFP4 ||
                     J.fmt == DS4F_FMT_BF16 || J.fmt == DS4F_FMT_MLX4,
                     "matvec: unknown format %d", J.fmt);
        if (J.fmt == DS4F_FMT_MXFP4)
            DS4F_REQUIRE(J.bsize == 16 || J.bsize == 32,
                         "matvec: MXFP4 block size %d (16 or 32)", J.bsize);
        if (J.SR < 1) J.SR = 1;
        if (J.SC < 1) J.SC = 1;
        int ce = J.fmt == DS4F_FMT_FP8 ? 16 : J.fmt == DS4F_FMT_BF16 ? 8 : 32;
        bool al = ((uintptr_t)J.v % 16) == 0 && ((uintptr_t)J.x % 16) == 0;
        bool fast = al && J.C % ce == 0;
        if (J.fmt == DS4F_FMT_FP8)
            fast = fast && J.C % J.SC == 0 && (J.C / J.SC) % 16 == 0;
        if (J.fmt == DS4F_FMT_MXFP4) fast = fast && J.bsize == 32;
        if (J.fmt == DS4F_FMT_MLX4) fast = fast && J.C % 64 == 0;
        int nq = J.C / ce;
        int lpr = 32;
        if (fast && nq < 32) {
            lpr = 1;
            while (lpr * 2 <= nq) lpr *= 2;
            fast = (lpr == nq);                     // power-of-two short rows
        }
        J.fast = fast ? 1 : 0;
        J.lpr = lpr;
        J.nq = nq;
        J.item0 = items;
        items += (J.R + kMvRowsPerItem - 1) / kMvRowsPerItem;
    }
    return items;
}

int launch_jobs(const MvJob *jobs_dev, int njobs, int nitems, cudaStream_t st) {
    if (nitems <= 0) return 0;
    k_mv_jobs<<<grid_for(nitems, 1), kMvThreads, 0, st>>>(jobs_dev, njobs, nitems);
    DS4F_CUDA(cudaGetLastError());
    return 0;
}

int launch_f8_decode(const uint8_t *W, int scale_kind, const void *scales,
                     int R, int C, int SR, int SC, int r0, int r1, float *out,
                     cudaStream_t st) {
    DS4F_REQUIRE(R > 0 && C > 0 && r0 >= 0 && r1 <= R && r0 <= r1,
                 "f8 decode: bad rows [%d, %d) of %d", r0, r1, R);
    int64_t n = (int64_t)(r1 - r0) * C;
    if (n == 0) return 0;
    k_f8_decode<<<grid_for(n, 256), 256, 0, st>>>(W, scale_kind, scales, R, C,
                                                 SR, SC, r0, r1, out);
    DS4F_CUDA(cudaGetLastError());
    return 0;
}

int launch_mx_decode(const uint8_t *vals, const uint8_t *scales, int64_t n,
                     int bsize, float *out, cudaStream_t st) {
    DS4F_REQUIRE(n >= 0 && bsize > 0, "mxfp4 decode: bad args");
    if (n == 0) return 0;
    k_mx_decode<<<grid_for(n, 256), 256, 0, st>>>(vals, scales, n, bsize, out);
    DS4F_CUDA(cudaGetLastError());
    return 0;
}

int launch_f8_canon(uint8_t *buf, int64_t n, cudaStream_t st) {
    DS4F_REQUIRE(((uintptr_t)buf % 16) == 0, "f8 canon: buffer not 16-byte aligned");
    if (n == 0) return 0;
    k_f8_canon<<<grid_for(n / 16 + 1, 256), 256, 0, st>>>(buf, n);
    DS4F_CUDA(cudaGetLastError());
    return 0;
}

}  // namespace ds4f
