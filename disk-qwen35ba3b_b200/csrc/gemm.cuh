// gemm.cuh -- the tensor-core GEMM and the quantisers of the batched
// prefill (gemm.cu), as used by its orchestration (prefill.cu).
#pragma once

#include <cuda.h>

#include "common.cuh"

namespace ds4f {

constexpr int kGemmBN = 64;                // B columns (tokens) per tile

struct GemmArgs {
    const float *sW;          // FP8: scales of slot 0, [R/128][KB] floats
    const float *sW2;         // the second A matrix's (gemm_launch with A2)
    int ycol2;                // the second A matrix's output column offset
    int64_t sw_slot;          // floats between consecutive slots' scales
    const float *sX;          // FP8: [rows][KB] activation scales
    float *Y;                 // Y[(first row + n) * ldy + ycol0 + r]
    int64_t ldy;
    int ycol0, R, C, KB;      // KB: K blocks of 128 bytes (set by gemm_launch)
    int row_scales;           // 1: sW holds a scale per (row, K block), [R][KB];
                              //    0: per 128x128 block
    const uint8_t *sfa;       // MXFP4 A (gemm_launch_mx): E8M0 scales of slot 0,
    const uint8_t *sfa2;      //   [R][C/32] bytes (the second A matrix's in sfa2),
    int64_t sfa_slot;         //   bytes between consecutive slots' scales
    const int *tiles;         // grouped: [*ntiles][3] = slot, first B row, valid rows
    const int *ntiles;
    int N;                    // dense: B rows
    int nmat;                 // A matrices (2: A2 given; set by gemm_launch)
    unsigned *err;
};

// FP8 digit GEMM (persistent, tcgen05): A = slots x [R][C] E4M3 bytes,
// `slot_stride` bytes apart (A2: a second matrix of the same shape and
// slots, the up projection beside the gate: scales sW2, output columns
// ycol2 + r); X = ND digit planes [xrows][C]. At most `ntiles_max` B tiles
// (the grouped mode reads the count from *g.ntiles). BF must be false.
template <int ND, bool BF>
int gemm_launch(const void *A, int64_t slots, int64_t slot_stride, const void *X, int64_t xrows,
                GemmArgs g, int ntiles_max, cudaStream_t st, const void *A2 = nullptr);

// The same GEMM with MXFP4 A (E2M1 nibbles [R][C] per slot, C / 2 bytes a
// row, `slot_stride` bytes apart; E8M0 scales per 32 in g.sfa / g.sfa2): the
// tensor core's block-scaled MMA (kind::mxf8f6f4.block_scale) applies the
// weights' scales itself, the epilogue only the activations'.
template <int ND>
int gemm_launch_mx(const void *A, int64_t slots, int64_t slot_stride, const void *X, int64_t xrows,
                   GemmArgs g, int ntiles_max, cudaStream_t st, const void *A2 = nullptr);
// bf16 GEMM (tcgen05 kind::f16): Y = A . X~, A [R][C] bf16 (A2 as above),
// X~ = hi + lo, two bf16 planes [N][C]; dense over g.N rows.
int bf16_gemm_launch(const uint16_t *A, const uint16_t *X, GemmArgs g, cudaStream_t st,
                     const uint16_t *A2 = nullptr);

int quant_f8_digits_launch(const float *x, int N, int C, int ND, uint8_t *q, float *s, cudaStream_t st);

// ---- the quantisers' per-lane step ------------------------------------------------
// Two fp32 -> E4M3 bytes (round to nearest even, saturating), lo in the low byte.
__device__ __forceinline__ uint32_t e4m3_2(float lo, float hi) {
    uint16_t r;
    asm("cvt.rn.satfinite.e4m3x2.f32 %0, %1, %2;" : "=h"(r) : "f"(hi), "f"(lo));
    return r;
}
__device__ __forceinline__ float e4m3_val(uint32_t b) {      // exact
    return __int_as_float(((int)(b << 24) >> 4) & (int)0x87F00000) * DS4F_F8_UNSCALE;
}
// A warp holds one 128-column block, 4 values per lane (columns 4 lane ..):
// a = max |v|, r = 240 / a, y = v r, then ND (<= 3) E4M3 digits, the lane's
// 4 bytes of digit d in wd[d]; returns the block scale.
__device__ __forceinline__ float quant_block_words(float4 v, int ND, uint32_t (&wd)[3]) {
    float a = fmaxf(fmaxf(fabsf(v.x), fabsf(v.y)), fmaxf(fabsf(v.z), fabsf(v.w)));
#pragma unroll
    for (int o = 16; o > 0; o >>= 1) a = fmaxf(a, __shfl_xor_sync(0xFFFFFFFFu, a, o));
    const float r = a > 0.f ? __fdiv_rn(240.0f, a) : 0.f;
    float y[4] = {__fmul_rn(v.x, r), __fmul_rn(v.y, r), __fmul_rn(v.z, r), __fmul_rn(v.w, r)};
#pragma unroll
    for (int d = 0; d < 3; d++) {
        wd[d] = 0;
        if (d >= ND) continue;
        const uint32_t w = e4m3_2(y[0], y[1]) | (e4m3_2(y[2], y[3]) << 16);
        wd[d] = w;
#pragma unroll
        for (int i = 0; i < 4; i++) y[i] = __fmul_rn(__fsub_rn(y[i], e4m3_val((w >> (8 * i)) & 0xFF)), 16.0f);
    }
    return a > 0.f ? __fdiv_rn(a, 240.0f) : 1.0f;
}
// The same, each digit written to its plane q + d * plane at byte offset `off`.
__device__ __forceinline__ float quant_block_digits(float4 v, int ND, uint8_t *q, int64_t plane,
                                                    int64_t off) {
    uint32_t wd[3];
    const float s = quant_block_words(v, ND, wd);
#pragma unroll
    for (int d = 0; d < 3; d++)
        if (d < ND) *(uint32_t *)(q + (int64_t)d * plane + off) = wd[d];
    return s;
}

}  // namespace ds4f
