// synth.cu -- seeded synthetic expert pools on the device.
//
// The BASELINE workloads are synthetic (no checkpoint): weights ~N(0, 0.02)
// quantised to FP8 (fp32 scale per 128x128 block) or MXFP4 (E8M0 per 32),
// bf16 router/shared expert, RMSNorm weight 1. A 40-layer FP8 pool is
// ~32 GB, too slow to generate on the host, so the generator runs here.
// Every step uses IEEE-exact operations in a fixed order (explicit _rn
// intrinsics, no contraction) so the bytes equal the CPU generator's in
// the test suite's checker, operation for operation:
//   key = mix(mix(seed) ^ tid);  element i: base = mix(key + i); Marsaglia
//   polar draws v = (z >> 11) 2^-52 - 1 from z = mix(base + k G);
//   g = v1 sqrt(-2 ln(s) / s) with ln from an atanh series; value =
//   float(g sigma). Quantisers: bf16 RNE; FP8 s = amax / 448 and the
//   nearest canonical byte of the reference decode table (ties to even);
//   MXFP4 k = ceil(log2(amax / 6)) exactly, nearest E2M1 magnitude.
#include "model.cuh"

namespace ds4f {

namespace {

constexpr uint64_t kG = 0x9E3779B97F4A7C15ull;

__host__ __device__ __forceinline__ uint64_t mix64(uint64_t x) {
    x += kG;
    x = (x ^ (x >> 30)) * 0xBF58476D1CE4E5B9ull;
    x = (x ^ (x >> 27)) * 0x94D049BB133111EBull;
    return x ^ (x >> 31);
}

__host__ __device__ __forceinline__ uint64_t tid_of(uint32_t layer, uint32_t kind,
                                                    uint32_t x, uint32_t t) {
    return ((uint64_t)layer << 40) | ((uint64_t)(kind & 0xFF) << 32) |
           ((uint64_t)(x & 0xFFFFFF) << 8) | (uint64_t)(t & 0xFF);
}

__host__ __device__ __forceinline__ uint64_t key_of(uint64_t seed, uint64_t tid) {
    return mix64(mix64(seed) ^ tid);
}

__device__ double ln_series(double s) {
    uint64_t b = (uint64_t)__double_as_longlong(s);
    int ex = (int)((b >> 52) & 0x7FF), adj = 0;
    if (ex == 0) {
        s = __dmul_rn(s, 18014398509481984.0);
        b = (uint64_t)__double_as_longlong(s);
        ex = (int)((b >> 52) & 0x7FF);
        adj = 54;
    }
    int e = ex - 1023 - adj;
    double m = __longlong_as_double((long long)((b & 0x000FFFFFFFFFFFFFull) |
                                                0x3FF0000000000000ull));
    if (m > 1.4142135623730951) { m = __dmul_rn(m, 0.5); e += 1; }
    double t = __ddiv_rn(__dsub_rn(m, 1.0), __dadd_rn(m, 1.0));
    double t2 = __dmul_rn(t, t);
    double p = 1.0 / 23.0;
    p = __dadd_rn(__dmul_rn(p, t2), 1.0 / 21.0);
    p = __dadd_rn(__dmul_rn(p, t2), 1.0 / 19.0);
    p = __dadd_rn(__dmul_rn(p, t2), 1.0 / 17.0);
    p = __dadd_rn(__dmul_rn(p, t2), 1.0 / 15.0);
    p = __dadd_rn(__dmul_rn(p, t2), 1.0 / 13.0);
    p = __dadd_rn(__dmul_rn(p, t2), 1.0 / 11.0);
    p = __dadd_rn(__dmul_rn(p, t2), 1.0 / 9.0);
    p = __dadd_rn(__dmul_rn(p, t2), 1.0 / 7.0);
    p = __dadd_rn(__dmul_rn(p, t2), 1.0 / 5.0);
    p = __dadd_rn(__dmul_rn(p, t2), 1.0 / 3.0);
    p = __dadd_rn(__dmul_rn(p, t2), 1.0);
    double lt = __dmul_rn(__dmul_rn(2.0, t), p);
    return __dadd_rn(__dmul_rn((double)e, 0.6931471805599453), lt);
}

__device__ double gauss(uint64_t key, uint64_t i) {
    uint64_t base = mix64(key + i);
    for (uint64_t k = 0; k < 64; k++) {
        uint64_t z1 = mix64(base + (2 * k) * kG);
        uint64_t z2 = mix64(base + (2 * k + 1) * kG);
        double v1 = __dsub_rn(__dmul_rn((double)(z1 >> 11), 2.220446049250313e-16), 1.0);
        double v2 = __dsub_rn(__dmul_rn((double)(z2 >> 11), 2.220446049250313e-16), 1.0);
        double s = __dadd_rn(__dmul_rn(v1, v1), __dmul_rn(v2, v2));
        if (s > 0.0 && s < 1.0) {
            double f = __dsqrt_rn(__ddiv_rn(__dmul_rn(-2.0, ln_series(s)), s));
            return __dmul_rn(v1, f);
        }
    }
    return 0.0;
}

__device__ __forceinline__ float value(uint64_t key, uint64_t i, double sigma) {
    return __double2float_rn(__dmul_rn(gauss(key, i), sigma));
}

__device__ __forceinline__ uint16_t bf16_rne(float f) {
    uint32_t b = __float_as_uint(f);
    if ((b & 0x7FFFFFFFu) > 0x7F800000u) return (uint16_t)((b >> 16) | 0x40);
    b += 0x7FFFu + ((b >> 16) & 1u);
    return (uint16_t)(b >> 16);
}

__device__ __forceinline__ float f8_mag(int b) {
    return f8_raw<0>((uint32_t)b) * DS4F_F8_UNSCALE;   // exact table value
}

__device__ uint8_t f8_encode(float v) {
    int neg = v < 0.0f;
    float a = fabsf(v);
    int byte;
    if (!(a < 448.0f)) {
        byte = 0x7E;
    } else {
        int lo = 0, hi = 0x77;
        while (lo < hi) {
            int mid = (lo + hi + 1) >> 1;
            if (f8_mag(mid) <= a) lo = mid; else hi = mid - 1;
        }
        int b0 = lo, b1 = (lo == 0x77) ? 0x7E : lo + 1;
        double d0 = __dsub_rn((double)a, (double)f8_mag(b0));
        double d1 = __dsub_rn((double)f8_mag(b1), (double)a);
        if (d0 < d1) byte = b0;
        else if (d1 < d0) byte = b1;
        else byte = (b0 & 1) ? b1 : b0;
    }
    return (uint8_t)(byte | (neg ? 0x80 : 0));
}

__device__ int ceil_log2(float y) {
    uint32_t b = __float_as_uint(y);
    int ex = (int)((b >> 23) & 0xFF), adj = 0;
    if (ex == 0) {
        y = __fmul_rn(y, 4294967296.0f);
        b = __float_as_uint(y);
        ex = (int)((b >> 23) & 0xFF);
        adj = 32;
    }
    int e = ex - 127 - adj;
    return (b & 0x7FFFFFu) ? e + 1 : e;
}

__device__ int e2m1_encode(float q) {
    const float mags[8] = {0.0f, 0.5f, 1.0f, 1.5f, 2.0f, 3.0f, 4.0f, 6.0f};
    float a = fabsf(q);
    int best = 0;
    float bd = a;
#pragma unroll
    for (int i = 1; i < 8; i++) {
        float d = fabsf(__fsub_rn(a, mags[i]));
        if (d < bd) { bd = d; best = i; }
    }
    return (q < 0.0f ? 8 : 0) | best;
}

// Where a tensor's key comes from: (seed, layer, kind, x, t).
struct KeySpec { uint64_t seed; uint32_t layer, kind, x0, t; };

__global__ void k_synth_f32(float *dst, int64_t n, uint64_t key, double sigma) {
    for (int64_t i = blockIdx.x * (int64_t)blockDim.x + threadIdx.x; i < n;
         i += (int64_t)gridDim.x * blockDim.x)
        dst[i] = value(key, (uint64_t)i, sigma);
}

__global__ void k_synth_bf16(uint16_t *dst, int64_t n, uint64_t key, double sigma) {
    for (int64_t i = blockIdx.x * (int64_t)blockDim.x + threadIdx.x; i < n;
         i += (int64_t)gridDim.x * blockDim.x)
        dst[i] = bf16_rne(value(key, (uint64_t)i, sigma));
}

__global__ void k_fill_u16(uint16_t *dst, int64_t n, uint16_t v) {
    for (int64_t i = blockIdx.x * (int64_t)blockDim.x + threadIdx.x; i < n;
         i += (int64_t)gridDim.x * blockDim.x)
        dst[i] = v;
}

// FP8 [R x C], one CTA per 128x128 block, blockIdx.y = expert within the
// shard (slot stride slot_bytes). Block values staged in shared memory.
__global__ void __launch_bounds__(256)
k_synth_fp8(uint8_t *slots, int64_t slot_bytes, int64_t rel_v, int64_t rel_s,
            int R, int C, KeySpec ks, double sigma) {
    extern __shared__ float blk[];                 // 128 * 128
    __shared__ float red[8];
    const int SC = C / 128;
    const int br = blockIdx.x / SC, bc = blockIdx.x % SC;
    const uint32_t expert = ks.x0 + blockIdx.y;
    const uint64_t key = key_of(ks.seed, tid_of(ks.layer, ks.kind, expert, ks.t));
    uint8_t *slot = slots + (int64_t)blockIdx.y * slot_bytes;
    float amax = 0.0f;
    for (int k = threadIdx.x; k < 128 * 128; k += blockDim.x) {
        int r = br * 128 + k / 128, c = bc * 128 + k % 128;
        float w = value(key, (uint64_t)r * C + c, sigma);
        blk[k] = w;
        amax = fmaxf(amax, fabsf(w));
    }
#pragma unroll
    for (int o = 16; o > 0; o >>= 1) amax = fmaxf(amax, __shfl_xor_sync(0xFFFFFFFFu, amax, o));
    if ((threadIdx.x & 31) == 0) red[threadIdx.x >> 5] = amax;
    __syncthreads();
    if (threadIdx.x == 0) {
        float m = 0.0f;
        for (int k = 0; k < (int)(blockDim.x >> 5); k++) m = fmaxf(m, red[k]);
        red[0] = m > 0.0f ? __fdiv_rn(m, 448.0f) : 1.0f;
        ((float *)(slot + rel_s))[br * SC + bc] = red[0];
    }
    __syncthreads();
    const float s = red[0];
    for (int k = threadIdx.x; k < 128 * 128; k += blockDim.x) {
        int r = br * 128 + k / 128, c = bc * 128 + k % 128;
        slot[rel_v + (int64_t)r * C + c] = f8_encode(__fdiv_rn(blk[k], s));
    }
}

// MXFP4 [R x C], one warp per 32-element block along K.
__global__ void __launch_bounds__(256)
k_synth_mx(uint8_t *slots, int64_t slot_bytes, int64_t rel_v, int64_t rel_s,
           int R, int C, KeySpec ks, double sigma) {
    const int lane = threadIdx.x & 31;
    const int64_t nblk = (int64_t)R * C / 32;
    const uint32_t expert = ks.x0 + blockIdx.y;
    const uint64_t key = key_of(ks.seed, tid_of(ks.layer, ks.kind, expert, ks.t));
    uint8_t *slot = slots + (int64_t)blockIdx.y * slot_bytes;
    for (int64_t bi = (blockIdx.x * (int64_t)blockDim.x + threadIdx.x) >> 5; bi < nblk;
         bi += ((int64_t)gridDim.x * blockDim.x) >> 5) {
        float x = value(key, (uint64_t)(bi * 32 + lane), sigma);
        float m = fabsf(x);
#pragma unroll
        for (int o = 16; o > 0; o >>= 1) m = fmaxf(m, __shfl_xor_sync(0xFFFFFFFFu, m, o));
        int k = m > 0.0f ? ceil_log2(__fdiv_rn(m, 6.0f)) : -127;
        k = k < -127 ? -127 : (k > 127 ? 127 : k);
        uint32_t sb = (uint32_t)((k + 127) & 0xFF);
        float s = e8m0_to_f32(sb);
        int nib = e2m1_encode(s != 0.0f ? __fdiv_rn(x, s) : 0.0f);
        int hi = __shfl_down_sync(0xFFFFFFFFu, nib, 1);
        if ((lane & 1) == 0) slot[rel_v + (bi * 32 + lane) / 2] = (uint8_t)(nib | (hi << 4));
        if (lane == 0) slot[rel_s + bi] = (uint8_t)sb;
    }
}

int grid1d(int64_t n) {
    int64_t g = (n + 255) / 256;
    return (int)(g < 1 ? 1 : (g > 65535 ? 65535 : g));
}

}  // namespace

int synth_f32(float *dst, int64_t n, uint64_t key, double sigma, cudaStream_t st) {
    if (n <= 0) return 0;
    k_synth_f32<<<grid1d(n), 256, 0, st>>>(dst, n, key, sigma);
    DS4F_CUDA(cudaGetLastError());
    return 0;
}

int synth_model(Model *m, uint64_t seed, double sigma, cudaStream_t st) {
    const ModelDesc &d = m->d;
    const int H = d.hidden, M = d.moe_inter, E = d.n_experts;
    static SmemOptIn opt;
    if (opt.set(k_synth_fp8, 128 * 128 * 4)) return -1;
    for (int L = 0; L < d.n_layers; L++) {
        uint16_t *t = m->trunk + (int64_t)L * m->tr.n;
        k_fill_u16<<<grid1d(H), 256, 0, st>>>(t + m->tr.norm, H, 0x3F80);   // 1.0
        struct { int64_t off, n; uint32_t kind, tt; } parts[5] = {
            {m->tr.router, (int64_t)E * H, 1, 0},
            {m->tr.sh_gate, (int64_t)M * H, 2, 0},
            {m->tr.sh_up, (int64_t)M * H, 2, 1},
            {m->tr.sh_down, (int64_t)H * M, 2, 2},
            {m->tr.sh_gw, (int64_t)H, 2, 3}};
        for (auto &p : parts)
            k_synth_bf16<<<grid1d(p.n), 256, 0, st>>>(
                t + p.off, p.n, key_of(seed, tid_of(L, p.kind, 0, p.tt)), sigma);
        DS4F_CUDA(cudaGetLastError());
        uint8_t *slots = m->pool + (int64_t)L * d.expert_count * m->slot.nbytes;
        for (int tt = 0; tt < 3; tt++) {
            int R = tt < 2 ? M : H, C = tt < 2 ? H : M;
            KeySpec ks{seed, (uint32_t)L, 3u, (uint32_t)d.expert_first, (uint32_t)tt};
            if (d.fmt == DS4F_FMT_FP8) {
                dim3 grid((R / 128) * (C / 128), d.expert_count);
                k_synth_fp8<<<grid, 256, 128 * 128 * 4, st>>>(
                    slots, m->slot.nbytes, m->slot.rel_v[tt], m->slot.rel_s[tt], R, C, ks, sigma);
            } else {
                int64_t nblk = (int64_t)R * C / 32;
                dim3 grid((unsigned)((nblk + 7) / 8 < 4096 ? (nblk + 7) / 8 : 4096), d.expert_count);
                k_synth_mx<<<grid, 256, 0, st>>>(slots, m->slot.nbytes, m->slot.rel_v[tt],
                                                 m->slot.rel_s[tt], R, C, ks, sigma);
            }
            DS4F_CUDA(cudaGetLastError());
        }
    }
    return 0;
}

}  // namespace ds4f
