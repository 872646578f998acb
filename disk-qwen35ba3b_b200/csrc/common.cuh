// common.cuh -- shared device helpers for libds4f_cuda (sm_100a).
//
// Decode rules follow the reference's scalar kernels:
//   E4M3  src/kernels.c:228-241 (e = 15 decodes to +-448 for every mantissa)
//   E2M1  src/kernels.c:28-46   (even index = low nibble, bit 3 = sign)
//   E8M0  src/kernels.c:24-26   (2^(b-127), b = 0 subnormal, 255 = inf)
//   bf16  src/kernels.c:84-89   (top half of fp32)
// Built without --use_fast_math, -ftz=false, IEEE div/sqrt: subnormal scales
// and weights survive, as the reference's do.
#pragma once

#include <cuda_runtime.h>
#include <stdint.h>

#include <atomic>

#define DS4F_FMT_MXFP4 0
#define DS4F_FMT_FP8 2
#define DS4F_SCALE_E8M0 0
#define DS4F_SCALE_F32 1

namespace ds4f {

// ---- host-side error plumbing (thread-local last error) ---------------
void set_error(const char *fmt, ...);
int cuda_fail(cudaError_t e, const char *what, const char *file, int line);

#define DS4F_CUDA(call)                                                     \
    do {                                                                    \
        cudaError_t _e = (call);                                            \
        if (_e != cudaSuccess)                                              \
            return ::ds4f::cuda_fail(_e, #call, __FILE__, __LINE__);        \
    } while (0)

// A kernel's opt-in to more than 48 KB of dynamic shared memory, made once
// per device: the attribute belongs to the current device, and one process
// may drive several GPUs (devices past 64 set it on every launch).
struct SmemOptIn {
    std::atomic<uint64_t> done{0};
    template <class F>
    int set(F *kernel, int bytes) {
        int dev = 0;
        DS4F_CUDA(cudaGetDevice(&dev));
        const uint64_t bit = dev < 64 ? (1ull << dev) : 0;
        if (bit && (done.load(std::memory_order_acquire) & bit)) return 0;
        DS4F_CUDA(cudaFuncSetAttribute(kernel, cudaFuncAttributeMaxDynamicSharedMemorySize, bytes));
        done.fetch_or(bit, std::memory_order_release);
        return 0;
    }
};

#define DS4F_REQUIRE(cond, ...)                                             \
    do {                                                                    \
        if (!(cond)) {                                                      \
            ::ds4f::set_error(__VA_ARGS__);                                 \
            return -1;                                                      \
        }                                                                   \
    } while (0)

// ---- element decode ------------------------------------------------------

__device__ __forceinline__ float bf16_to_f32(uint16_t h) {
    return __uint_as_float((uint32_t)h << 16);
}

// E8M0 scale 2^(b-127) built from bits: b >= 1 is a normal float with
// exponent field b; b = 0 is the subnormal 2^-127 (mantissa bit 22); b =
// 255 is +inf. Same values as ldexpf(1, b - 127).
__device__ __forceinline__ float e8m0_to_f32(uint32_t b) {
    return b ? __uint_as_float(b << 23) : __uint_as_float(0x00400000u);
}

// Reference E4M3 rule applied to 4 packed bytes: every byte whose
// exponent field is 15 becomes 0x7E (+-448) with its sign kept. The
// result decodes identically under the reference table and under
// IEEE-style E4M3FN decode (no NaN encodings remain).
__device__ __forceinline__ uint32_t f8_canon4(uint32_t w) {
    uint32_t mag = w & 0x7F7F7F7Fu;
    // bytes with mag >= 0x78: add 0x08 to each byte's low 7 bits and look
    // at bit 7 (no carry out of a byte since mag <= 0x7F, 0x7F + 0x08 <
    // 0x100).
    uint32_t hi = ((mag + 0x08080808u) & 0x80808080u);
    uint32_t m = (hi >> 7) * 0xFFu;                      // 0xFF per e=15 byte
    return (w & ~m) | ((w & 0x80808080u) | 0x7E7E7E7Eu) & m;
}

// E4M3 byte k of word w (canonical) -> fp32 times 2^-120, exactly:
// bits (b & 0x7F) << 20 put e in the fp32 exponent field and m in the top
// mantissa bits, so normals are (1 + m/8) 2^(e-127) and e = 0 bytes are
// the denormal m 2^-129 -- both the true value times 2^-120. Callers fold
// 2^120 into the block scale.
template <int K>
__device__ __forceinline__ float f8_raw(uint32_t w) {
    uint32_t t = (K == 3) ? w : (w << (24 - 8 * K));   // byte K -> bits 24..31
    return __uint_as_float((t & 0x80000000u) | ((t >> 4) & 0x07F00000u));
}
#define DS4F_F8_UNSCALE 1.329227995784916e+36f   // 2^120
#define DS4F_F8_POST 7.205759403792794e+16f      // 2^120 / 2^64 = 2^56

// E2M1 nibble -> fp32 times 2^-126, exactly: bits (n & 7) << 22 put the
// 2-bit exponent in the fp32 exponent field and the mantissa bit at bit
// 22, giving 2^(e-127)(1 + m/2) for e >= 1 and m 2^-127 for e = 0 -- the
// magnitudes {0, .5, 1, 1.5, 2, 3, 4, 6} times 2^-126. Bit 3 -> sign.
// The multiply by 0x10400000 spreads nibble bits 0..3 to 22..25 and 28..31
// without overlap; the mask keeps 22..24 and 31.
__device__ __forceinline__ float e2m1_raw(uint32_t nib) {
    return __uint_as_float((nib * 0x10400000u) & 0x81C00000u);
}
#define DS4F_E2M1_UNSCALE 8.507059173023462e+37f   // 2^126

// x pre-scaled by 2^64 keeps the E2M1 and E4M3 products (raw magnitudes
// down to 2^-129) in the normal fp32 range; the 2^-64 goes back with the
// block scale (DS4F_F8_POST, DS4F_E2M1_POST, DS4F_BF16_POST).
#define DS4F_X_PRESCALE 1.8446744073709552e+19f    // 2^64
#define DS4F_E2M1_POST 4.611686018427388e+18f      // 2^126 / 2^64 = 2^62
#define DS4F_BF16_POST 5.421010862427522e-20f      // 2^-64
#define DS4F_X_UNSCALE 5.421010862427522e-20f      // 2^-64: undoes DS4F_X_PRESCALE

// ---- top-8 by a warp sorting network ------------------------------------------
// Candidates for the selection are ordered by a 32-bit key: the logit's
// order-preserving float key with its low 8 bits replaced by 255 - expert
// (so the lower index comes first among equal keys, as in ds4f_topk,
// src/moe.c:537-545). The key only proposes the 8 to certify: the
// certificate itself compares the exact intervals, so two logits too close
// for the key cannot pass it and go to the exact fallback instead.
__device__ __forceinline__ uint32_t tk_key(float s, int e) {
    const uint32_t u = __float_as_uint(s);
    const uint32_t k = (u & 0x80000000u) ? ~u : (u | 0x80000000u);
    return (k & 0xFFFFFF00u) | (uint32_t)(255 - e);
}
__device__ __forceinline__ int tk_expert(uint32_t key) { return 255 - (int)(key & 0xFFu); }
// The reference's insertion top-k (ds4f_topk, src/moe.c:531-546), one
// thread, on fp32 logits v[e] (held as float or double): a slot is passed
// over while it is empty or the new logit is strictly greater. Used when a
// logit is not finite: NaN never passes a filled slot and an all-NaN row
// selects experts 0..K-1, exactly as the reference does; every sel[j] < K
// then holds a valid expert whenever E >= K.
template <typename V>
__device__ void tk_insertion(const V *v, int E, int K, int *sel) {
    float wk[64];
    if (K > E) K = E;
    for (int j = 0; j < K; j++) { sel[j] = -1; wk[j] = 0.0f; }
    for (int e = 0; e < E; e++) {
        const float s = (float)v[e];
        int j = K - 1;
        while (j >= 0 && (sel[j] < 0 || s > wk[j])) j--;
        if (j < K - 1) {
            for (int q = K - 2; q > j; q--) { sel[q + 1] = sel[q]; wk[q + 1] = wk[q]; }
            sel[j + 1] = e;
            wk[j + 1] = s;
        }
    }
}
// Bitonic sort of 8 keys, largest first.
__device__ __forceinline__ void tk_sort8(uint32_t (&k8)[8]) {
#pragma unroll
    for (int k = 2; k <= 8; k <<= 1)
#pragma unroll
        for (int j = k >> 1; j > 0; j >>= 1)
#pragma unroll
            for (int i = 0; i < 8; i++) {
                const int l = i ^ j;
                if (l > i) {
                    const uint32_t hi = max(k8[i], k8[l]), lo = min(k8[i], k8[l]);
                    k8[i] = (i & k) == 0 ? hi : lo;
                    k8[l] = (i & k) == 0 ? lo : hi;
                }
            }
}
// Every lane holds its own sorted 8; after the five butterfly merges every
// lane holds the warp's largest 8, sorted (the larger of each list against
// the reverse of the other is the pair's largest 8 as a bitonic sequence,
// sorted again by three half-cleaner rounds).
__device__ __forceinline__ void tk_warp_top8(uint32_t (&k8)[8]) {
#pragma unroll
    for (int m = 1; m < 32; m <<= 1) {
        uint32_t p[8];
#pragma unroll
        for (int j = 0; j < 8; j++) p[j] = __shfl_xor_sync(0xFFFFFFFFu, k8[j], m);
#pragma unroll
        for (int j = 0; j < 8; j++) k8[j] = max(k8[j], p[7 - j]);
#pragma unroll
        for (int j = 4; j > 0; j >>= 1)
#pragma unroll
            for (int i = 0; i < 8; i++) {
                const int l = i ^ j;
                if (l > i) {
                    const uint32_t hi = max(k8[i], k8[l]), lo = min(k8[i], k8[l]);
                    k8[i] = hi;
                    k8[l] = lo;
                }
            }
    }
}

// ---- reductions ----------------------------------------------------------

__device__ __forceinline__ float warp_sum(float v) {
#pragma unroll
    for (int o = 16; o > 0; o >>= 1) v += __shfl_xor_sync(0xFFFFFFFFu, v, o);
    return v;
}

__device__ __forceinline__ double warp_sum_d(double v) {
#pragma unroll
    for (int o = 16; o > 0; o >>= 1) v += __shfl_xor_sync(0xFFFFFFFFu, v, o);
    return v;
}

// 16-byte streaming load of weights: read once, do not keep in L1.
__device__ __forceinline__ uint4 ldg_stream(const void *p) {
    uint4 r;
    asm volatile("ld.global.nc.L1::no_allocate.v4.u32 {%0,%1,%2,%3}, [%4];"
                 : "=r"(r.x), "=r"(r.y), "=r"(r.z), "=r"(r.w)
                 : "l"(p));
    return r;
}

// Dot of 16 canonical E4M3 bytes with 16 floats, in units of 2^-120.
__device__ __forceinline__ float f8_dot16(uint4 q, const float *x) {
    float a = 0.f, b = 0.f;
    a = fmaf(f8_raw<0>(q.x), x[0], a);  b = fmaf(f8_raw<1>(q.x), x[1], b);
    a = fmaf(f8_raw<2>(q.x), x[2], a);  b = fmaf(f8_raw<3>(q.x), x[3], b);
    a = fmaf(f8_raw<0>(q.y), x[4], a);  b = fmaf(f8_raw<1>(q.y), x[5], b);
    a = fmaf(f8_raw<2>(q.y), x[6], a);  b = fmaf(f8_raw<3>(q.y), x[7], b);
    a = fmaf(f8_raw<0>(q.z), x[8], a);  b = fmaf(f8_raw<1>(q.z), x[9], b);
    a = fmaf(f8_raw<2>(q.z), x[10], a); b = fmaf(f8_raw<3>(q.z), x[11], b);
    a = fmaf(f8_raw<0>(q.w), x[12], a); b = fmaf(f8_raw<1>(q.w), x[13], b);
    a = fmaf(f8_raw<2>(q.w), x[14], a); b = fmaf(f8_raw<3>(q.w), x[15], b);
    return a + b;
}

// Dot of the 4 canonical E4M3 bytes of w (byte k = element k) with x[0..3],
// in units of 2^-120 (x pre-scaled by 2^64: result in units of 2^-56).
__device__ __forceinline__ float f8_dot4(uint32_t w, const float *x) {
    float a = f8_raw<0>(w) * x[0], b = f8_raw<1>(w) * x[1];
    a = fmaf(f8_raw<2>(w), x[2], a);
    b = fmaf(f8_raw<3>(w), x[3], b);
    return a + b;
}

// Two canonical E4M3 bytes (the low 16 bits of w16) -> their fp32 values,
// exactly: the hardware conversion to f16x2 (every E4M3 value, subnormals
// included, is an f16; canonical bytes hold no NaN code), then to fp32.
// Four instructions for two bytes, against three per byte by shifts.
__device__ __forceinline__ float2 f8_cvt2(uint32_t w16) {
    uint32_t h;
    asm("{ .reg .b16 t; cvt.u16.u32 t, %1; cvt.rn.f16x2.e4m3x2 %0, t; }" : "=r"(h) : "r"(w16));
    float lo, hi;
    asm("{ .reg .b16 a, b; mov.b32 {a, b}, %2; cvt.f32.f16 %0, a; cvt.f32.f16 %1, b; }"
        : "=f"(lo), "=f"(hi) : "r"(h));
    return make_float2(lo, hi);
}
// acc + (Σ of the 4 products of w's bytes with x01, x23) * s, as two lanes
// of packed fp32 (sm_100 FFMA2). With x pre-scaled by 2^64 the result is
// in units of 2^-64 (DS4F_X_UNSCALE brings it back).
__device__ __forceinline__ float2 f8_fma4(uint32_t w, float2 x01, float2 x23, float s, float2 acc) {
    float2 p = __fmul2_rn(f8_cvt2(w & 0xFFFFu), x01);
    p = __ffma2_rn(f8_cvt2(w >> 16), x23, p);
    return __ffma2_rn(p, make_float2(s, s), acc);
}

// Two E2M1 nibbles (the low byte of w8, the even element in the low nibble)
// -> their fp32 values, exactly, by the hardware conversion to f16x2.
__device__ __forceinline__ float2 e2m1_cvt2(uint32_t w8) {
    uint32_t h;
    asm("{ .reg .b8 t; cvt.u8.u32 t, %1; cvt.rn.f16x2.e2m1x2 %0, t; }" : "=r"(h) : "r"(w8));
    float lo, hi;
    asm("{ .reg .b16 a, b; mov.b32 {a, b}, %2; cvt.f32.f16 %0, a; cvt.f32.f16 %1, b; }"
        : "=f"(lo), "=f"(hi) : "r"(h));
    return make_float2(lo, hi);
}
// e2m1_dot8 by the hardware conversion: the same even / odd partial sums in
// packed fp32, scaled to units of 2^-126 once at the end (the products are
// the same up to that power of two).
__device__ __forceinline__ float e2m1_dot8c(uint32_t w, const float *x) {
    float2 p = __fmul2_rn(e2m1_cvt2(w & 0xFFu), make_float2(x[0], x[1]));
    p = __ffma2_rn(e2m1_cvt2((w >> 8) & 0xFFu), make_float2(x[2], x[3]), p);
    p = __ffma2_rn(e2m1_cvt2((w >> 16) & 0xFFu), make_float2(x[4], x[5]), p);
    p = __ffma2_rn(e2m1_cvt2(w >> 24), make_float2(x[6], x[7]), p);
    return (p.x + p.y) * 1.1754943508222875e-38f;      // 2^-126
}
// Dot of the 8 E2M1 nibbles of w (even index low nibble) with x[0..7], in
// units of 2^-126.
__device__ __forceinline__ float e2m1_dot8(uint32_t w, const float *x) {
    float a = e2m1_raw(w & 0xFu) * x[0], b = e2m1_raw((w >> 4) & 0xFu) * x[1];
#pragma unroll
    for (int k = 2; k < 8; k += 2) {
        a = fmaf(e2m1_raw((w >> (4 * k)) & 0xFu), x[k], a);
        b = fmaf(e2m1_raw((w >> (4 * k + 4)) & 0xFu), x[k + 1], b);
    }
    return a + b;
}

// Dot of 4 bf16 (q.x low, q.x high, q.y low, q.y high) with x.
__device__ __forceinline__ float bf16_dot4(uint2 q, float4 x) {
    float a = __uint_as_float(q.x << 16) * x.x, b = __uint_as_float(q.x & 0xFFFF0000u) * x.y;
    a = fmaf(__uint_as_float(q.y << 16), x.z, a);
    b = fmaf(__uint_as_float(q.y & 0xFFFF0000u), x.w, b);
    return a + b;
}

__device__ __forceinline__ uint4 f8_canon16(uint4 q) {
    return make_uint4(f8_canon4(q.x), f8_canon4(q.y), f8_canon4(q.z),
                      f8_canon4(q.w));
}

// Dot of 32 E2M1 nibbles (16 bytes, even index low nibble) with 32 floats
// pre-scaled by 2^64; result in units of 2^-62.
__device__ __forceinline__ float e2m1_dot32(uint4 q, const float *x) {
    float a = 0.f, b = 0.f;
    const uint32_t w[4] = {q.x, q.y, q.z, q.w};
#pragma unroll
    for (int i = 0; i < 4; i++) {
#pragma unroll
        for (int k = 0; k < 8; k += 2) {
            a = fmaf(e2m1_raw((w[i] >> (4 * k)) & 0xFu), x[8 * i + k], a);
            b = fmaf(e2m1_raw((w[i] >> (4 * k + 4)) & 0xFu), x[8 * i + k + 1], b);
        }
    }
    return a + b;
}

// Dot of 8 bf16 with 8 floats.
__device__ __forceinline__ float bf16_dot8(uint4 q, const float *x) {
    float a = 0.f, b = 0.f;
    a = fmaf(__uint_as_float(q.x << 16), x[0], a);
    b = fmaf(__uint_as_float(q.x & 0xFFFF0000u), x[1], b);
    a = fmaf(__uint_as_float(q.y << 16), x[2], a);
    b = fmaf(__uint_as_float(q.y & 0xFFFF0000u), x[3], b);
    a = fmaf(__uint_as_float(q.z << 16), x[4], a);
    b = fmaf(__uint_as_float(q.z & 0xFFFF0000u), x[5], b);
    a = fmaf(__uint_as_float(q.w << 16), x[6], a);
    b = fmaf(__uint_as_float(q.w & 0xFFFF0000u), x[7], b);
    return a + b;
}

// silu(g) * u in the reference's form s * (1 / (1 + exp(-s))) * u
// (src/moe.c:645-649), IEEE division, CUDA expf.
__device__ __forceinline__ float silu_mul(float g, float u) {
    float sig = __fdiv_rn(1.0f, __fadd_rn(1.0f, expf(-g)));
    return __fmul_rn(__fmul_rn(g, sig), u);
}

__device__ __forceinline__ float sigmoid_ref(float g) {
    return __fdiv_rn(1.0f, __fadd_rn(1.0f, expf(-g)));
}

}  // namespace ds4f
