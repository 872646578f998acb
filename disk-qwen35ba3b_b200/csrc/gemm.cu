// gemm.cu -- block-scaled FP8 GEMM on the 5th-generation tensor cores
// (tcgen05, TMEM accumulators, TMA-fed 128-byte-swizzled tiles), the
// building block of the batched prefill (the grouped-by-expert chains of
// ds4f_moe_step_batch, src/moe.c:1480-1707), and the activation quantiser
// whose outputs it consumes.
//
//   Y[n][r] = sum_kb sW[r/128][kb] sX[n][kb] sum_{c in kb} W[r][c] x~[n][c]
//
// W: [R][C] canonical E4M3 (the expert pool's bytes), sW fp32 per 128x128
// block (the pool's scales). The activations are fp32 in the reference
// (src/moe.c:1480-1707); here each row's 128-column block is scaled into
// [-240, 240] and written as ND E4M3 "digits", x~ = d0 + d1/16 + d2/256
// (relative error <= 2^-13 at ND = 3, against 2^-4 for one digit), so the
// tensor core works on native FP8 on both sides while the chain keeps the
// reference's precision. The digits are planes [ND][N][C]; one 3-D TMA box
// brings a tile's ND x BN rows, and the MMA's N dimension is ND x BN.
//
// The tensor core sums each 128-column block exactly as E4M3 x E4M3
// products in fp32 (tcgen05.mma kind::f8f6f4, 4 instructions of K = 32);
// the block's two scales differ per output element, so each block's partial
// sums are read back from TMEM, the digits combined, and added into fp32
// registers with the scales ("promotion") while the tensor core already
// works on the next block in the other TMEM buffer. The FP8 GEMMs run on
// one persistent kernel (k_gemm_p); the shared expert's bf16 GEMMs
// (k_gemm_bf16) accumulate their whole K in TMEM instead.
#include <cuda.h>
#include <cudaTypedefs.h>

#include "common.cuh"
#include "tc.cuh"
#include "gemm.cuh"
#include "../../include/ds4f/gpu_cuda.h"

namespace ds4f {

// ---- host: tensor maps -----------------------------------------------------------
static PFN_cuTensorMapEncodeTiled_v12000 encode_fn() {
    static PFN_cuTensorMapEncodeTiled_v12000 fn = nullptr;
    if (!fn) {
        void *p = nullptr;
        cudaDriverEntryPointQueryResult q;
        if (cudaGetDriverEntryPoint("cuTensorMapEncodeTiled", &p, cudaEnableDefault, &q) == cudaSuccess &&
            q == cudaDriverEntryPointSuccess)
            fn = (PFN_cuTensorMapEncodeTiled_v12000)p;
    }
    return fn;
}

// 8-bit tensor [rows][inner] (row stride `stride` bytes), boxes of
// [box_rows][128 bytes] with the 128-byte swizzle; rows past the end read 0.
int tmap_u8_2d(CUtensorMap *m, const void *base, uint64_t inner, uint64_t rows, uint64_t stride,
               uint32_t box_rows) {
    auto fn = encode_fn();
    if (!fn) { set_error("cuTensorMapEncodeTiled is unavailable"); return -1; }
    if (((uintptr_t)base & 15) || (stride & 15) || inner % 128 || box_rows < 1 || box_rows > 256) {
        set_error("tensor map: base/stride must be 16-byte aligned, inner a multiple of 128");
        return -1;
    }
    cuuint64_t dims[2] = {inner, rows};
    cuuint64_t strides[1] = {stride};
    cuuint32_t box[2] = {128, box_rows};
    cuuint32_t es[2] = {1, 1};
    CUresult r = fn(m, CU_TENSOR_MAP_DATA_TYPE_UINT8, 2, const_cast<void *>(base), dims, strides, box, es,
                    CU_TENSOR_MAP_INTERLEAVE_NONE, CU_TENSOR_MAP_SWIZZLE_128B,
                    CU_TENSOR_MAP_L2_PROMOTION_L2_256B, CU_TENSOR_MAP_FLOAT_OOB_FILL_NONE);
    if (r != CUDA_SUCCESS) { set_error("cuTensorMapEncodeTiled failed (%d)", (int)r); return -1; }
    return 0;
}

// 8-bit tensor [planes][rows][inner], boxes of [planes][box_rows][128 bytes].
int tmap_u8_3d(CUtensorMap *m, const void *base, uint64_t inner, uint64_t rows, uint64_t planes,
               uint64_t row_stride, uint64_t plane_stride, uint32_t box_rows, uint32_t box_planes) {
    auto fn = encode_fn();
    if (!fn) { set_error("cuTensorMapEncodeTiled is unavailable"); return -1; }
    if (((uintptr_t)base & 15) || (row_stride & 15) || (plane_stride & 15) || inner % 128 ||
        box_rows < 1 || box_rows > 256 || box_planes < 1 || box_planes > 256) {
        set_error("tensor map: base/strides must be 16-byte aligned, inner a multiple of 128");
        return -1;
    }
    cuuint64_t dims[3] = {inner, rows, planes};
    cuuint64_t strides[2] = {row_stride, plane_stride};
    cuuint32_t box[3] = {128, box_rows, box_planes};
    cuuint32_t es[3] = {1, 1, 1};
    CUresult r = fn(m, CU_TENSOR_MAP_DATA_TYPE_UINT8, 3, const_cast<void *>(base), dims, strides, box, es,
                    CU_TENSOR_MAP_INTERLEAVE_NONE, CU_TENSOR_MAP_SWIZZLE_128B,
                    CU_TENSOR_MAP_L2_PROMOTION_L2_256B, CU_TENSOR_MAP_FLOAT_OOB_FILL_NONE);
    if (r != CUDA_SUCCESS) { set_error("cuTensorMapEncodeTiled failed (%d)", (int)r); return -1; }
    return 0;
}

// 4-bit tensor [planes][rows][inner] (E2M1 nibbles, two to a byte, row
// stride `row_stride` bytes), boxes of [1][box_rows][128 elements] landing in
// shared memory unpacked (each 16 nibbles in a 16-byte chunk, the layout the
// block-scaled MMA reads 4-bit operands in: a 128-byte row holds 128
// elements, as for 8-bit ones) with the 128-byte swizzle.
int tmap_u4_3d(CUtensorMap *m, const void *base, uint64_t inner, uint64_t rows, uint64_t planes,
               uint64_t row_stride, uint64_t plane_stride, uint32_t box_rows) {
    auto fn = encode_fn();
    if (!fn) { set_error("cuTensorMapEncodeTiled is unavailable"); return -1; }
    if (((uintptr_t)base & 31) || (row_stride & 31) || (plane_stride & 31) || inner % 128 || box_rows < 1 ||
        box_rows > 256) {
        set_error("tensor map (4-bit): base and strides must be 32-byte aligned, inner a multiple of 128");
        return -1;
    }
    cuuint64_t dims[3] = {inner, rows, planes};
    cuuint64_t strides[2] = {row_stride, plane_stride};
    cuuint32_t box[3] = {128, box_rows, 1};
    cuuint32_t es[3] = {1, 1, 1};
    CUresult r = fn(m, CU_TENSOR_MAP_DATA_TYPE_16U4_ALIGN16B, 3, const_cast<void *>(base), dims, strides, box, es,
                    CU_TENSOR_MAP_INTERLEAVE_NONE, CU_TENSOR_MAP_SWIZZLE_128B,
                    CU_TENSOR_MAP_L2_PROMOTION_L2_256B, CU_TENSOR_MAP_FLOAT_OOB_FILL_NONE);
    if (r != CUDA_SUCCESS) { set_error("cuTensorMapEncodeTiled (4-bit) failed (%d)", (int)r); return -1; }
    return 0;
}

namespace {

// ---- activation quantiser -------------------------------------------------------
// Per (row, 128-column block): a = max |x|; r = 240 / a and s = a / 240 (fp32,
// correctly rounded; a = 0: r = 0, s = 1); y = x * r; then ND digits
//   d0 = E4M3(y),  e = (y - d0) * 16,  d1 = E4M3(e),  e = (e - d1) * 16, ...
// E4M3() rounds to nearest even, saturating. Every digit stays within
// [-240, 240] (exponent field <= 14), where the reference's E4M3 table and
// standard E4M3 agree. Output planes q[d][row][col].
__global__ void k_quant_f8_digits(const float *x, int N, int C, int ND, uint8_t *q, float *s) {
    const int nb = C / 128;
    const int64_t blk = (int64_t)blockIdx.x * (blockDim.x / 32) + threadIdx.x / 32;   // one warp per block
    if (blk >= (int64_t)N * nb) return;
    const int lane = threadIdx.x & 31;
    const int64_t off = (blk / nb) * (int64_t)C + (blk % nb) * 128 + 4 * lane;
    const float sc = quant_block_digits(*(const float4 *)(x + off), ND, q, (int64_t)N * C, off);
    if (lane == 0) s[blk] = sc;
}

constexpr int kEpiWarps = 16;              // four per TMEM lane quadrant, 16 columns each
constexpr int kEpiCols = kGemmBN / (kEpiWarps / 4);
constexpr int kGemmThreads = 64 + 32 * kEpiWarps;   // warp 0 TMA, warp 1 MMA + TMEM, warps 2.. epilogue
static_assert(kEpiCols == 16, "one 16-column TMEM load per warp");

// ---- bf16 GEMM (the shared expert) ------------------------------------------------
// tcgen05 kind::f16 on bf16, 64-column K blocks (4 MMAs of K = 16), no
// scales, 2 digits (hi, lo) as 2 x 64 MMA columns; the whole K sum stays
// in TMEM and is read once. A is [R][C] bf16 (A2: a second matrix of the
// same shape into columns ycol2 + r), B the digit planes [2][N][C]; one CTA
// per (row tile, 64-row B tile): tile = blockIdx.y, rows 64 blockIdx.y.
constexpr int kBStages = 4;
struct BfSmem {
    static constexpr int NM = 2 * kGemmBN;            // MMA N: the two digit planes
    static constexpr int A = 128 * 128;
    static constexpr int STAGE = A + NM * 128;
    static constexpr int o_bar = kBStages * STAGE;    // full[S], empty[S], tfull, done
    static constexpr int o_slot = o_bar + ((2 * kBStages + 2) * 8 + 127) / 128 * 128;
    static constexpr int bytes = o_slot + 16 + 1024;
    static constexpr uint32_t ID = tc::idesc(128, NM, 1, 1);
};

__global__ void __launch_bounds__(kGemmThreads, 1)
k_gemm_bf16(const __grid_constant__ CUtensorMap tW, const __grid_constant__ CUtensorMap tW2,
            const __grid_constant__ CUtensorMap tX, GemmArgs g) {
    using L = BfSmem;
    constexpr int BN = kGemmBN;
    extern __shared__ uint8_t smem_raw[];
    uint8_t *sm = smem_raw + ((1024 - (tc::sa(smem_raw) & 1023)) & 1023);
    uint64_t *full = (uint64_t *)(sm + L::o_bar), *empty = full + kBStages;
    uint64_t *tfull = empty + kBStages, *done = tfull + 1;
    uint32_t *slot = (uint32_t *)(sm + L::o_slot);

    const int n0 = blockIdx.y * BN, nv = min(BN, g.N - n0);
    const int tid = threadIdx.x, warp = tid >> 5, lane = tid & 31;
    const int MT = g.R / 128, mat = blockIdx.x / MT;
    const int r0 = (blockIdx.x % MT) * 128, KB = g.KB;
    const CUtensorMap *tA = mat ? &tW2 : &tW;
    unsigned *err = g.err;

    if (warp == 1) tc::tmem_alloc(slot, 128);
    if (tid == 0) {
        for (int s = 0; s < kBStages; s++) { tc::mbar_init(full + s, 1); tc::mbar_init(empty + s, 1); }
        tc::mbar_init(tfull, 1);
        tc::mbar_init(done, 1);
        tc::mbar_fence_init();
        tc::prefetch_tmap(tA);
        tc::prefetch_tmap(&tX);
    }
    tc::fence_before_sync();
    __syncthreads();
    tc::fence_after_sync();
    const uint32_t taddr = *slot;

    if (warp == 0) {
        if (lane == 0) {
            int kb = 0;
            for (; kb < KB; kb++) {
                const int s = kb % kBStages;
                if (kb >= kBStages && !tc::mbar_wait(empty + s, ((kb / kBStages) - 1) & 1, err, 1)) break;
                uint8_t *a = sm + s * L::STAGE;
                tc::mbar_expect(full + s, L::STAGE);
                tc::tma_load_3d(a, tA, kb * 128, r0, 0, full + s);
                tc::tma_load_3d(a + L::A, &tX, kb * 128, n0, 0, full + s);
            }
            // every issued load has landed before the CTA may exit
            for (int k = kb - 1; k >= 0 && k >= kb - kBStages; k--)
                tc::mbar_wait(full + k % kBStages, (k / kBStages) & 1, err, 2, true);
        }
    } else if (warp == 1) {
        if (lane == 0) {
            for (int kb = 0; kb < KB; kb++) {
                const int s = kb % kBStages;
                if (!tc::mbar_wait(full + s, (kb / kBStages) & 1, err, 3)) break;
                tc::fence_after_sync();
                const uint8_t *a = sm + s * L::STAGE;
#pragma unroll
                for (int k = 0; k < 4; k++)
                    tc::mma_f16(taddr, tc::sdesc_sw128(a + 32 * k), tc::sdesc_sw128(a + L::A + 32 * k), L::ID,
                                kb > 0 || k > 0);
                tc::commit(empty + s);
                if (kb == KB - 1) tc::commit(tfull);
            }
            tc::commit(done);
            tc::mbar_wait(done, 0, err, 5, true);      // every MMA finished
        }
    } else {
        // warp quadrant q reads TMEM lanes 32q .. 32q + 31 = rows; the four
        // warps of a quadrant take 16 columns each: D0 + D1 per column
        const int q = warp & 3, c0 = ((warp - 2) >> 2) * kEpiCols, row = q * 32 + lane;
        if (tc::mbar_wait(tfull, 0, err, 6)) {
            tc::fence_after_sync();
            const uint32_t tq = taddr + ((uint32_t)(q * 32) << 16);
            uint32_t r[2][16];
            tc::tmem_ld16_nowait(tq + c0, r[0]);
            tc::tmem_ld16_nowait(tq + BN + c0, r[1]);
            tc::tmem_wait_ld();
            tc::tmem_regs_ready(r[0]);
            tc::tmem_regs_ready(r[1]);
            if (r0 + row < g.R) {
                float *y = g.Y + (int64_t)(n0 + c0) * g.ldy + (mat ? g.ycol2 : g.ycol0) + r0 + row;
#pragma unroll
                for (int j = 0; j < kEpiCols; j++)
                    if (c0 + j < nv) y[(int64_t)j * g.ldy] = __fadd_rn(__uint_as_float(r[0][j]), __uint_as_float(r[1][j]));
            }
        }
    }
    tc::fence_before_sync();
    __syncthreads();
    if (warp == 1) {
        tc::fence_after_sync();
        tc::tmem_dealloc(taddr, 128);
    }
}

// ---- persistent FP8 GEMM ------------------------------------------------------------
// One CTA per SM walks the items (B tile t, A row tile m), item i = t RT + m,
// i = blockIdx.x, + gridDim.x, ...; the load ring and the two TMEM buffers run
// on across item boundaries, so the next item's first K blocks land while the
// tensor core and the epilogue finish the current one (a CTA per item pays the
// pipeline fill every time: the down projection has only 4 K blocks). Each
// item loads and multiplies only its valid B rows rounded up to 16 (one tensor
// map per width), so narrow expert groups do not stream 64 digit rows.
constexpr int kPStages = 5;

template <int ND>
struct PSmem {
    static constexpr int NMX = kGemmBN * ND;          // widest MMA N (one TMEM buffer)
    static constexpr int A = 128 * 128;
    static constexpr int STAGE = A + NMX * 128;
    // full[S], empty[S], tfull[2], tempty[2], done, sfull[S] (block-scaled)
    static constexpr int o_bar = kPStages * STAGE;
    static constexpr int o_slot = o_bar + ((3 * kPStages + 5) * 8 + 127) / 128 * 128;
    // TMEM: two accumulator buffers, then (block-scaled) the A scale factors
    // of each stage in 4 columns, then 8 columns of B scale factors (1.0)
    static constexpr uint32_t SFA = 2 * NMX, SFB = SFA + 4 * kPStages;
    static_assert(SFB + 16 <= 512, "TMEM columns for the scale factors");
    static constexpr int o_sx = o_slot + 16;          // two [kb][64] activation-scale tiles
    static constexpr int bytes(int kb) { return o_sx + 2 * kGemmBN * kb * 4 + 1024; }
    static_assert(STAGE % 1024 == 0 && 2 * NMX <= 512, "stage alignment and TMEM columns");
};

struct PItem { int zs, n0, nv, w, mat, r0; };

// Item i of RT row tiles per B tile (MT per A matrix); false past the end.
__device__ __forceinline__ bool p_item(const GemmArgs &g, int i, int n_items, int RT, int MT, PItem &it) {
    if (i >= n_items) return false;
    const int t = i / RT, m = i % RT;
    if (g.tiles) {
        it.zs = g.tiles[3 * t]; it.n0 = g.tiles[3 * t + 1]; it.nv = g.tiles[3 * t + 2];
    } else {
        it.zs = 0; it.n0 = t * kGemmBN; it.nv = min(kGemmBN, g.N - it.n0);
    }
    it.w = (it.nv + 15) & ~15;
    it.mat = m / MT;
    it.r0 = (m % MT) * 128;
    return true;
}

// Epilogue of one K block for columns [c0, c0 + kEpiCols) of a tile w rows
// wide: digit d of column n sits at TMEM column d w + n; otherwise as promote().
template <int ND>
__device__ __forceinline__ void promote_w(uint32_t t, int w, int c0, const float *sxk, float sw,
                                          float2 (&acc)[kEpiCols / 2]) {
#pragma unroll
    for (int c = 0; c < kEpiCols / 16; c++) {
        const uint32_t col = c0 + c * 16;
        uint32_t r[3][16];
        tc::tmem_ld16_nowait(t + col, r[0]);
        if (ND > 1) tc::tmem_ld16_nowait(t + w + col, r[1]);
        if (ND > 2) tc::tmem_ld16_nowait(t + 2 * w + col, r[2]);
        float sc[16];
#pragma unroll
        for (int i = 0; i < 16; i += 4) {
            const float4 s4 = *(const float4 *)(sxk + col + i);
            sc[i] = __fmul_rn(sw, s4.x); sc[i + 1] = __fmul_rn(sw, s4.y);
            sc[i + 2] = __fmul_rn(sw, s4.z); sc[i + 3] = __fmul_rn(sw, s4.w);
        }
        tc::tmem_wait_ld();
        tc::tmem_regs_ready(r[0]);
        if (ND > 1) tc::tmem_regs_ready(r[1]);
        if (ND > 2) tc::tmem_regs_ready(r[2]);
#pragma unroll
        for (int i = 0; i < 16; i += 2) {
            float v0 = __uint_as_float(r[0][i]), v1 = __uint_as_float(r[0][i + 1]);
            if (ND > 1) {
                v0 = fmaf(__uint_as_float(r[1][i]), 0.0625f, v0);
                v1 = fmaf(__uint_as_float(r[1][i + 1]), 0.0625f, v1);
            }
            if (ND > 2) {
                v0 = fmaf(__uint_as_float(r[2][i]), 0.00390625f, v0);
                v1 = fmaf(__uint_as_float(r[2][i + 1]), 0.00390625f, v1);
            }
            float2 &a2 = acc[(c * 16 + i) >> 1];
            a2 = __ffma2_rn(make_float2(v0, v1), make_float2(sc[i], sc[i + 1]), a2);
        }
    }
}

// The activation scales of item `it` that thread e of the epilogue holds:
// entries e + 32 kEpiWarps p of the tile's [kb][64] table (0 past nv).
constexpr int kPSxRegs = 4;                // KB <= 32
__device__ __forceinline__ void p_sx_load(const GemmArgs &g, const PItem &it, bool valid, int e,
                                          float (&v)[kPSxRegs]) {
    const int KB = g.KB;
#pragma unroll
    for (int p = 0; p < kPSxRegs; p++) {
        const int i = e + p * 32 * kEpiWarps, kb = i / kGemmBN, col = i % kGemmBN;
        v[p] = (valid && kb < KB && col < it.nv) ? __ldg(g.sX + (int64_t)(it.n0 + col) * KB + kb) : 0.f;
    }
}
__device__ __forceinline__ void p_sx_store(float *sxt, int KB, int e, const float (&v)[kPSxRegs]) {
#pragma unroll
    for (int p = 0; p < kPSxRegs; p++) {
        const int i = e + p * 32 * kEpiWarps;
        if (i < kGemmBN * KB) sxt[i] = v[p];
    }
}

// MX: A is MXFP4 (unpacked E2M1 tiles, block-scaled MMA); four more warps,
// one per TMEM lane quadrant, write each stage's A scale factors into TMEM.
template <int ND, bool MX>
__global__ void __launch_bounds__(MX ? kGemmThreads + 128 : kGemmThreads, 1)
k_gemm_p(const __grid_constant__ CUtensorMap tW, const __grid_constant__ CUtensorMap tW2,
         const __grid_constant__ CUtensorMap tX16, const __grid_constant__ CUtensorMap tX32,
         const __grid_constant__ CUtensorMap tX48, const __grid_constant__ CUtensorMap tX64, GemmArgs g) {
    using L = PSmem<ND>;
    extern __shared__ uint8_t smem_raw[];
    uint8_t *sm = smem_raw + ((1024 - (tc::sa(smem_raw) & 1023)) & 1023);
    uint64_t *full = (uint64_t *)(sm + L::o_bar), *empty = full + kPStages;
    uint64_t *tfull = empty + kPStages, *tempty = tfull + 2, *done = tempty + 2, *sfull = done + 1;
    uint32_t *slot = (uint32_t *)(sm + L::o_slot);
    float *sxt = (float *)(sm + L::o_sx);
    constexpr uint32_t kTmemCols = (MX || 2 * L::NMX > 256) ? 512 : 256;

    const int MT = g.R / 128, RT = MT * g.nmat, KB = g.KB;
    const int n_items = (g.tiles ? *g.ntiles : (g.N + kGemmBN - 1) / kGemmBN) * RT;
    if ((int)blockIdx.x >= n_items) return;                 // uniform: before any barrier
    const int tid = threadIdx.x, warp = tid >> 5, lane = tid & 31;
    unsigned *err = g.err;

    if (warp == 1) tc::tmem_alloc(slot, kTmemCols);
    if (tid == 0) {
        for (int s = 0; s < kPStages; s++) { tc::mbar_init(full + s, 1); tc::mbar_init(empty + s, 1); }
        if (MX)
            for (int s = 0; s < kPStages; s++) tc::mbar_init(sfull + s, 4);
        for (int b = 0; b < 2; b++) { tc::mbar_init(tfull + b, 1); tc::mbar_init(tempty + b, kEpiWarps); }
        tc::mbar_init(done, 1);
        tc::mbar_fence_init();
        tc::prefetch_tmap(&tW);
        if (g.nmat > 1) tc::prefetch_tmap(&tW2);
    }
    tc::fence_before_sync();
    __syncthreads();
    tc::fence_after_sync();
    const uint32_t taddr = *slot;
    PItem it;

    if (warp == 0) {
        if (lane == 0) {
            int k = 0;
            bool ok = true;
            for (int i = blockIdx.x; ok && p_item(g, i, n_items, RT, MT, it); i += gridDim.x) {
                const CUtensorMap *tA = it.mat ? &tW2 : &tW;
                const CUtensorMap *tB = it.w == 16 ? &tX16 : it.w == 32 ? &tX32 : it.w == 48 ? &tX48 : &tX64;
                // a 4-bit A tile lands unpacked (16 KB of shared memory) but
                // its transaction counts the 8 KB read
                const uint32_t bytes = (MX ? L::A / 2 : L::A) + ND * it.w * 128;
                for (int kb = 0; kb < KB; kb++, k++) {
                    const int s = k % kPStages;
                    if (k >= kPStages && !tc::mbar_wait(empty + s, ((k / kPStages) - 1) & 1, err, 1)) {
                        ok = false;
                        break;
                    }
                    uint8_t *a = sm + s * L::STAGE;
                    tc::mbar_expect(full + s, bytes);
                    tc::tma_load_3d(a, tA, kb * 128, it.r0, it.zs, full + s);
                    tc::tma_load_3d(a + L::A, tB, kb * 128, it.n0, 0, full + s);
                }
            }
            // every issued load has landed before the CTA may exit
            for (int j = k - 1; j >= 0 && j >= k - kPStages; j--)
                tc::mbar_wait(full + j % kPStages, (j / kPStages) & 1, err, 2, true);
        }
    } else if (warp == 1) {
        if (lane == 0) {
            int k = 0;
            bool ok = true;
            for (int i = blockIdx.x; ok && p_item(g, i, n_items, RT, MT, it); i += gridDim.x) {
                const uint32_t id = tc::idesc(128, ND * it.w, 0, 0);
                for (int kb = 0; kb < KB; kb++, k++) {
                    const int s = k % kPStages, b = k & 1;
                    if (!tc::mbar_wait(full + s, (k / kPStages) & 1, err, 3) ||
                        (MX && !tc::mbar_wait(sfull + s, (k / kPStages) & 1, err, 7)) ||
                        (k >= 2 && !tc::mbar_wait(tempty + b, ((k >> 1) - 1) & 1, err, 4))) {
                        ok = false;
                        break;
                    }
                    tc::fence_after_sync();
                    const uint8_t *a = sm + s * L::STAGE;
#pragma unroll
                    for (int q = 0; q < 4; q++) {
                        if constexpr (MX)
                            // K step q: byte q of each row's scale word (the 4
                            // sub-blocks of 32 in this 128-column block)
                            tc::mma_mx_bs(taddr + b * L::NMX, tc::sdesc_sw128(a + 32 * q),
                                          tc::sdesc_sw128(a + L::A + 32 * q), tc::idesc_bs(128, ND * it.w, 5, 0, q),
                                          (taddr + L::SFA + 4 * s) | ((uint32_t)q << 30),
                                          (taddr + L::SFB) | ((uint32_t)q << 30), q > 0);
                        else
                            tc::mma_f8f6f4(taddr + b * L::NMX, tc::sdesc_sw128(a + 32 * q),
                                           tc::sdesc_sw128(a + L::A + 32 * q), id, q > 0);
                    }
                    tc::commit(empty + s);
                    tc::commit(tfull + b);
                }
            }
            tc::commit(done);
            tc::mbar_wait(done, 0, err, 5, true);      // every MMA finished
        }
    } else if (warp < 2 + kEpiWarps) {
        // epilogue: warp quadrant q reads TMEM lanes 32q .. 32q + 31 = rows;
        // the four warps of a quadrant take 16 columns each. After a failed
        // wait the warps keep walking the items without waiting, so every
        // one of them reaches each named barrier.
        const int q = warp & 3, c0 = ((warp - 2) >> 2) * kEpiCols, row = q * 32 + lane, e = tid - 64;
        const uint32_t tq = taddr + ((uint32_t)(q * 32) << 16);
        float pre[kPSxRegs];
        bool ok = true;
        int k = 0, j = 0;
        p_item(g, blockIdx.x, n_items, RT, MT, it);
        p_sx_load(g, it, true, e, pre);
        p_sx_store(sxt, KB, e, pre);
        asm volatile("bar.sync 1, %0;" ::"r"(32 * kEpiWarps) : "memory");
        for (int i = blockIdx.x; i < n_items; i += gridDim.x, j++) {
            p_item(g, i, n_items, RT, MT, it);
            PItem nx;
            const bool has_next = p_item(g, i + gridDim.x, n_items, RT, MT, nx);
            p_sx_load(g, nx, has_next, e, pre);
            const float *sxi = sxt + (j & 1) * kGemmBN * KB;
            // the weights' block scales (MX: applied by the tensor core)
            const float *swr = MX ? nullptr
                                  : (it.mat ? g.sW2 : g.sW) + it.zs * g.sw_slot +
                                        (g.row_scales ? (int64_t)(it.r0 + row) * KB : (int64_t)(it.r0 / 128) * KB);
            float2 acc[kEpiCols / 2];
#pragma unroll
            for (int c = 0; c < kEpiCols / 2; c++) acc[c] = make_float2(0.f, 0.f);
            for (int kb = 0; kb < KB; kb++, k++) {
                const int b = k & 1;
                if (ok) ok = tc::mbar_wait(tfull + b, (k >> 1) & 1, err, 6);
                if (ok) {
                    tc::fence_after_sync();
                    if (c0 < it.w)
                        promote_w<ND>(tq + b * L::NMX, it.w, c0, sxi + kb * kGemmBN, MX ? 1.0f : __ldg(swr + kb),
                                      acc);
                    tc::fence_before_sync();
                }
                __syncwarp();
                if (lane == 0) tc::mbar_arrive(tempty + b);
            }
            if (ok && c0 < it.nv && it.r0 + row < g.R) {
                float *y = g.Y + (int64_t)(it.n0 + c0) * g.ldy + (it.mat ? g.ycol2 : g.ycol0) + it.r0 + row;
#pragma unroll
                for (int c = 0; c < kEpiCols; c++)
                    if (c0 + c < it.nv) y[(int64_t)c * g.ldy] = (c & 1) ? acc[c >> 1].y : acc[c >> 1].x;
            }
            p_sx_store(sxt + ((j + 1) & 1) * kGemmBN * KB, KB, e, pre);
            asm volatile("bar.sync 1, %0;" ::"r"(32 * kEpiWarps) : "memory");
        }
    } else if constexpr (MX) {
        // scale factors: warp quadrant q writes rows 32q .. 32q + 31 of A's
        // E8M0 scales, for each stage one 32-bit word per row (the 4 scales
        // of the 128-column K block, byte i = sub-block i) into 4 columns
        // of its lanes, once the stage's previous MMAs are done; B's are 1.0
        // (127) in 16 columns of every lane, written once
        const int q = warp & 3;
        const uint32_t tq = taddr + ((uint32_t)(q * 32) << 16);
#pragma unroll
        for (int c = 0; c < 16; c += 4) tc::tmem_st4(tq + L::SFB + c, 0x7F7F7F7Fu);
        const int rb = g.C / 32;                            // scale bytes per row
        int k = 0;
        bool ok = true;
        for (int i = blockIdx.x; ok && p_item(g, i, n_items, RT, MT, it); i += gridDim.x) {
            const uint8_t *sr = (it.mat ? g.sfa2 : g.sfa) + (int64_t)it.zs * g.sfa_slot +
                                (int64_t)(it.r0 + q * 32 + lane) * rb;
            for (int kb = 0; kb < KB; kb++, k++) {
                const int s = k % kPStages;
                bool okw = true;
                if (k >= kPStages && lane == 0) okw = tc::mbar_wait(empty + s, ((k / kPStages) - 1) & 1, err, 8);
                if (!__shfl_sync(0xFFFFFFFFu, okw, 0)) { ok = false; break; }
                tc::fence_after_sync();
                tc::tmem_st4(tq + L::SFA + 4 * s, __ldg((const uint32_t *)(sr + 4 * kb)));
                tc::tmem_wait_st();
                tc::fence_before_sync();
                __syncwarp();
                if (lane == 0) tc::mbar_arrive(sfull + s);
            }
        }
    }
    tc::fence_before_sync();
    __syncthreads();
    if (warp == 1) {
        tc::fence_after_sync();
        tc::tmem_dealloc(taddr, kTmemCols);
    }
}

// SMs of the current device (cached per device).
int sm_count() {
    static std::atomic<int> cache[64];
    int dev = 0;
    if (cudaGetDevice(&dev) != cudaSuccess) return 148;
    int n = dev < 64 ? cache[dev].load() : 0;
    if (n <= 0) {
        if (cudaDeviceGetAttribute(&n, cudaDevAttrMultiProcessorCount, dev) != cudaSuccess || n <= 0) n = 148;
        if (dev < 64) cache[dev].store(n);
    }
    return n;
}

}  // namespace

// A: slots x [R][C] E4M3 bytes, `slot_stride` bytes apart; B: ND digit
// planes [xrows][C]. At most `ntiles_max` B tiles (the grouped mode reads the
// count from *g.ntiles). The persistent kernel, one B tensor map per tile width.
template <int ND, bool BF>
int gemm_launch(const void *A, int64_t slots, int64_t slot_stride, const void *X, int64_t xrows,
                GemmArgs g, int ntiles_max, cudaStream_t st, const void *A2) {
    static_assert(!BF, "bf16 GEMMs: bf16_gemm_launch");
    if (g.R <= 0 || g.C <= 0 || g.R % 128 || g.C % 128 || ntiles_max <= 0) {
        set_error("gemm: R and C must be positive multiples of 128");
        return -1;
    }
    CUtensorMap tW, tW2, tX;
    if (tmap_u8_3d(&tW, A, (uint64_t)g.C, g.R, slots, (uint64_t)g.C, slot_stride, 128, 1) ||
        tmap_u8_3d(&tW2, A2 ? A2 : A, (uint64_t)g.C, g.R, slots, (uint64_t)g.C, slot_stride, 128, 1) ||
        tmap_u8_3d(&tX, X, (uint64_t)g.C, xrows, ND, (uint64_t)g.C, (uint64_t)xrows * g.C, kGemmBN, ND))
        return -1;
    g.KB = g.C / 128;
    using P = PSmem<ND>;
    CUtensorMap tX16, tX32, tX48;
    if (tmap_u8_3d(&tX16, X, (uint64_t)g.C, xrows, ND, (uint64_t)g.C, (uint64_t)xrows * g.C, 16, ND) ||
        tmap_u8_3d(&tX32, X, (uint64_t)g.C, xrows, ND, (uint64_t)g.C, (uint64_t)xrows * g.C, 32, ND) ||
        tmap_u8_3d(&tX48, X, (uint64_t)g.C, xrows, ND, (uint64_t)g.C, (uint64_t)xrows * g.C, 48, ND))
        return -1;
    const int psmem = P::bytes(g.KB);
    if (psmem > 227 * 1024 || kGemmBN * g.KB > kPSxRegs * 32 * kEpiWarps) {
        set_error("gemm: C too large for the scale tiles");
        return -1;
    }
    static SmemOptIn opt;
    if (opt.set(k_gemm_p<ND, false>, 227 * 1024)) return -1;
    g.nmat = A2 ? 2 : 1;
    const int64_t items = (int64_t)ntiles_max * (g.R / 128) * (A2 ? 2 : 1);
    const int grid = (int)std::min<int64_t>(items, sm_count());
    k_gemm_p<ND, false><<<grid, kGemmThreads, psmem, st>>>(tW, tW2, tX16, tX32, tX48, tX, g);
    DS4F_CUDA(cudaGetLastError());
    return 0;
}
template int gemm_launch<3, false>(const void *, int64_t, int64_t, const void *, int64_t, GemmArgs, int,
                                   cudaStream_t, const void *);

template <int ND>
int gemm_launch_mx(const void *A, int64_t slots, int64_t slot_stride, const void *X, int64_t xrows, GemmArgs g,
                   int ntiles_max, cudaStream_t st, const void *A2) {
    if (g.R <= 0 || g.C <= 0 || g.R % 128 || g.C % 128 || ntiles_max <= 0 || !g.sfa || (A2 && !g.sfa2)) {
        set_error("gemm (MXFP4): R and C must be positive multiples of 128, scales given");
        return -1;
    }
    CUtensorMap tW, tW2, tX16, tX32, tX48, tX64;
    if (tmap_u4_3d(&tW, A, (uint64_t)g.C, g.R, slots, (uint64_t)g.C / 2, slot_stride, 128) ||
        tmap_u4_3d(&tW2, A2 ? A2 : A, (uint64_t)g.C, g.R, slots, (uint64_t)g.C / 2, slot_stride, 128) ||
        tmap_u8_3d(&tX16, X, (uint64_t)g.C, xrows, ND, (uint64_t)g.C, (uint64_t)xrows * g.C, 16, ND) ||
        tmap_u8_3d(&tX32, X, (uint64_t)g.C, xrows, ND, (uint64_t)g.C, (uint64_t)xrows * g.C, 32, ND) ||
        tmap_u8_3d(&tX48, X, (uint64_t)g.C, xrows, ND, (uint64_t)g.C, (uint64_t)xrows * g.C, 48, ND) ||
        tmap_u8_3d(&tX64, X, (uint64_t)g.C, xrows, ND, (uint64_t)g.C, (uint64_t)xrows * g.C, kGemmBN, ND))
        return -1;
    g.KB = g.C / 128;
    using P = PSmem<ND>;
    const int psmem = P::bytes(g.KB);
    if (psmem > 227 * 1024 || kGemmBN * g.KB > kPSxRegs * 32 * kEpiWarps) {
        set_error("gemm: C too large for the scale tiles");
        return -1;
    }
    static SmemOptIn opt;
    if (opt.set(k_gemm_p<ND, true>, 227 * 1024)) return -1;
    g.nmat = A2 ? 2 : 1;
    const int64_t items = (int64_t)ntiles_max * (g.R / 128) * (A2 ? 2 : 1);
    const int grid = (int)std::min<int64_t>(items, sm_count());
    k_gemm_p<ND, true><<<grid, kGemmThreads + 128, psmem, st>>>(tW, tW2, tX16, tX32, tX48, tX64, g);
    DS4F_CUDA(cudaGetLastError());
    return 0;
}
template int gemm_launch_mx<3>(const void *, int64_t, int64_t, const void *, int64_t, GemmArgs, int, cudaStream_t,
                               const void *);

int bf16_gemm_launch(const uint16_t *A, const uint16_t *X, GemmArgs g, cudaStream_t st, const uint16_t *A2) {
    using L = BfSmem;
    if (g.R <= 0 || g.C <= 0 || g.R % 128 || g.C % 64 || g.N <= 0) {
        set_error("bf16 gemm: R must be a positive multiple of 128, C of 64");
        return -1;
    }
    const uint64_t cb = (uint64_t)g.C * 2;
    CUtensorMap tW, tW2, tX;
    if (tmap_u8_3d(&tW, A, cb, g.R, 1, cb, (uint64_t)g.R * cb, 128, 1) ||
        tmap_u8_3d(&tW2, A2 ? A2 : A, cb, g.R, 1, cb, (uint64_t)g.R * cb, 128, 1) ||
        tmap_u8_3d(&tX, X, cb, g.N, 2, cb, (uint64_t)g.N * cb, kGemmBN, 2))
        return -1;
    g.KB = (int)(cb / 128);
    static SmemOptIn opt;
    if (opt.set(k_gemm_bf16, L::bytes)) return -1;
    dim3 grid((g.R / 128) * (A2 ? 2 : 1), (g.N + kGemmBN - 1) / kGemmBN);
    k_gemm_bf16<<<grid, kGemmThreads, L::bytes, st>>>(tW, tW2, tX, g);
    DS4F_CUDA(cudaGetLastError());
    return 0;
}

int f8_gemm_launch(const uint8_t *W, const float *sW, const uint8_t *X, const float *sX, float *Y,
                   int R, int C, int N, int ND, unsigned *err, cudaStream_t st) {
    if (R <= 0 || C <= 0 || N <= 0 || R % 128 || C % 128) {
        set_error("f8_gemm: R and C must be positive multiples of 128, N > 0");
        return -1;
    }
    GemmArgs g{};
    g.sW = sW; g.sw_slot = 0; g.sX = sX; g.Y = Y; g.ldy = R; g.ycol0 = 0;
    g.R = R; g.C = C; g.N = N; g.err = err;
    const int nt = (N + kGemmBN - 1) / kGemmBN;
    switch (ND) {
    case 1: return gemm_launch<1, false>(W, 1, (int64_t)R * C, X, N, g, nt, st);
    case 2: return gemm_launch<2, false>(W, 1, (int64_t)R * C, X, N, g, nt, st);
    case 3: return gemm_launch<3, false>(W, 1, (int64_t)R * C, X, N, g, nt, st);
    }
    set_error("f8_gemm: digits must be 1, 2 or 3");
    return -1;
}

int quant_f8_digits_launch(const float *x, int N, int C, int ND, uint8_t *q, float *s, cudaStream_t st) {
    if (N <= 0 || C <= 0 || C % 128 || ND < 1 || ND > 3) {
        set_error("quant_f8_digits: C must be a positive multiple of 128, digits 1..3");
        return -1;
    }
    const int64_t blocks = (int64_t)N * (C / 128);
    k_quant_f8_digits<<<(unsigned)((blocks + 7) / 8), 256, 0, st>>>(x, N, C, ND, q, s);
    DS4F_CUDA(cudaGetLastError());
    return 0;
}

}  // namespace ds4f

namespace ds4f { namespace {
__device__ unsigned g_gemm_err;
}  // namespace
}  // namespace ds4f

extern "C" {

int ds4f_gpu_quant_f8_digits(const float *x, int N, int C, int ND, uint8_t *q, float *s, void *stream) {
    cudaStream_t st = (cudaStream_t)stream;
    if (ds4f::quant_f8_digits_launch(x, N, C, ND, q, s, st)) return -1;
    DS4F_CUDA(cudaStreamSynchronize(st));
    return 0;
}

int ds4f_gpu_f8_gemm(const uint8_t *W, const float *sW, const uint8_t *X, const float *sX, float *Y,
                     int R, int C, int N, int ND, void *stream) {
    cudaStream_t st = (cudaStream_t)stream;
    unsigned *err = nullptr;
    DS4F_CUDA(cudaGetSymbolAddress((void **)&err, ds4f::g_gemm_err));
    DS4F_CUDA(cudaMemsetAsync(err, 0, sizeof(unsigned), st));
    if (ds4f::f8_gemm_launch(W, sW, X, sX, Y, R, C, N, ND, err, st)) return -1;
    unsigned h = 0;
    DS4F_CUDA(cudaMemcpyAsync(&h, err, sizeof(unsigned), cudaMemcpyDeviceToHost, st));
    DS4F_CUDA(cudaStreamSynchronize(st));
    if (h) { ds4f::set_error("f8_gemm: a pipeline wait gave up (code %u)", h); return -1; }
    return 0;
}

}  // extern "C"
