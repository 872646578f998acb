// tc.cuh -- sm_100a building blocks for the tensor-core kernels: mbarriers,
// TMA tensor loads, and the tcgen05 MMA / TMEM instructions, as inline PTX.
//
// Operand layout used throughout: K-major tiles of 8-bit (or 16-bit)
// elements, 128-byte rows, loaded by TMA with the 128-byte swizzle (16-byte
// chunk c of row r stored at chunk c ^ (r & 7) within each 1024-byte group
// of 8 rows). The UMMA shared-memory descriptor for that layout has the
// start address (>> 4), leading-byte offset 16 (unused: one MMA never spans
// two 128-byte K atoms), stride-byte offset 1024 (next group of 8 rows),
// version 1, layout type 2 (SWIZZLE_128B); a K step of 32 bytes inside the
// atom advances the start address by 32.
#pragma once

#include <cuda_runtime.h>
#include <stdint.h>

namespace ds4f {
namespace tc {

__device__ __forceinline__ uint32_t sa(const void *p) {
    return (uint32_t)__cvta_generic_to_shared(p);
}

// ---- mbarriers ---------------------------------------------------------------
__device__ __forceinline__ void mbar_init(uint64_t *b, uint32_t n) {
    asm volatile("mbarrier.init.shared::cta.b64 [%0], %1;" ::"r"(sa(b)), "r"(n) : "memory");
}
__device__ __forceinline__ void mbar_fence_init() {
    asm volatile("fence.mbarrier_init.release.cluster;" ::: "memory");
}
__device__ __forceinline__ void mbar_expect(uint64_t *b, uint32_t bytes) {
    asm volatile("mbarrier.arrive.expect_tx.shared::cta.b64 _, [%0], %1;" ::"r"(sa(b)), "r"(bytes)
                 : "memory");
}
__device__ __forceinline__ void mbar_arrive(uint64_t *b) {
    asm volatile("mbarrier.arrive.shared::cta.b64 _, [%0];" ::"r"(sa(b)) : "memory");
}
__device__ __forceinline__ bool mbar_test(uint64_t *b, uint32_t parity) {
    uint32_t ok;
    asm volatile(
        "{ .reg .pred p; mbarrier.try_wait.parity.shared::cta.b64 p, [%1], %2; "
        "selp.u32 %0, 1, 0, p; }"
        : "=r"(ok) : "r"(sa(b)), "r"(parity) : "memory");
    return ok != 0;
}
// Bounded wait: false (and *err set to `code` if it was 0) after `limit`
// polls, or early when another thread already failed (unless `drain`: the
// waits that keep a CTA alive until its own copies / MMAs have finished
// only end at the limit).
__device__ __forceinline__ bool mbar_wait(uint64_t *b, uint32_t parity, unsigned *err, unsigned code,
                                          bool drain = false, long limit = 1L << 26) {
    long it = 0;
    while (!mbar_test(b, parity)) {
        ++it;
        if (!drain && (it & 1023) == 0 && *(volatile unsigned *)err) return false;
        if (it > limit) { atomicCAS(err, 0u, code); return false; }
        if (it > 64) __nanosleep(20);
    }
    return true;
}

// ---- TMA tensor loads --------------------------------------------------------
// tmap: generic address of a CUtensorMap kernel parameter (__grid_constant__).
// The innermost coordinate x times the element size must be a multiple of 16
// bytes; callers only pass multiples of 128 bytes.
__device__ __forceinline__ void tma_load_2d(void *dst, const void *tmap, int x, int y, uint64_t *b) {
    asm volatile(
        "cp.async.bulk.tensor.2d.shared::cluster.global.mbarrier::complete_tx::bytes [%0], [%1, {%2, %3}], [%4];"
        ::"r"(sa(dst)), "l"(tmap), "r"(x), "r"(y), "r"(sa(b)) : "memory");
}
__device__ __forceinline__ void tma_load_3d(void *dst, const void *tmap, int x, int y, int z, uint64_t *b) {
    asm volatile(
        "cp.async.bulk.tensor.3d.shared::cluster.global.mbarrier::complete_tx::bytes [%0], [%1, {%2, %3, %4}], [%5];"
        ::"r"(sa(dst)), "l"(tmap), "r"(x), "r"(y), "r"(z), "r"(sa(b)) : "memory");
}
__device__ __forceinline__ void prefetch_tmap(const void *tmap) {
    asm volatile("prefetch.tensormap [%0];" ::"l"(tmap) : "memory");
}

// ---- tcgen05 -----------------------------------------------------------------
// TMEM allocation: one whole warp; the base address lands in *slot (shared).
__device__ __forceinline__ void tmem_alloc(uint32_t *slot, uint32_t ncols) {
    asm volatile("tcgen05.alloc.cta_group::1.sync.aligned.shared::cta.b32 [%0], %1;" ::"r"(sa(slot)),
                 "r"(ncols) : "memory");
    asm volatile("tcgen05.relinquish_alloc_permit.cta_group::1.sync.aligned;" ::: "memory");
}
__device__ __forceinline__ void tmem_dealloc(uint32_t taddr, uint32_t ncols) {
    asm volatile("tcgen05.dealloc.cta_group::1.sync.aligned.b32 %0, %1;" ::"r"(taddr), "r"(ncols)
                 : "memory");
}
__device__ __forceinline__ void fence_before_sync() {
    asm volatile("tcgen05.fence::before_thread_sync;" ::: "memory");
}
__device__ __forceinline__ void fence_after_sync() {
    asm volatile("tcgen05.fence::after_thread_sync;" ::: "memory");
}

// Shared-memory matrix descriptor: K-major, 128-byte swizzle (see top).
__device__ __forceinline__ uint64_t sdesc_sw128(const void *p) {
    const uint64_t addr = sa(p);
    return ((addr & 0x3FFFFull) >> 4) | ((uint64_t)(16 >> 4) << 16) | ((uint64_t)(1024 >> 4) << 32) |
           (1ull << 46) | (2ull << 61);
}

// Instruction descriptor: fp32 accumulator, A/B formats, both K-major,
// N >> 3 at bits 17..22, M >> 4 at bits 24..28.
//   kind::f8f6f4 formats: 0 E4M3, 1 E5M2;  kind::f16 formats: 0 F16, 1 BF16
__host__ __device__ constexpr uint32_t idesc(int M, int N, uint32_t afmt, uint32_t bfmt) {
    return (1u << 4) | (afmt << 7) | (bfmt << 10) | ((uint32_t)(N >> 3) << 17) |
           ((uint32_t)(M >> 4) << 24);
}

// D[tmem] (+)= A[smem] . B[smem]^T, one instruction (K = 32 bytes of
// 8-bit elements, 16 of 16-bit), issued by a single thread.
__device__ __forceinline__ void mma_f8f6f4(uint32_t d, uint64_t a, uint64_t b, uint32_t id, uint32_t acc) {
    asm volatile(
        "{ .reg .pred p; setp.ne.b32 p, %4, 0; "
        "tcgen05.mma.cta_group::1.kind::f8f6f4 [%0], %1, %2, %3, p; }"
        ::"r"(d), "l"(a), "l"(b), "r"(id), "r"(acc) : "memory");
}
__device__ __forceinline__ void mma_f16(uint32_t d, uint64_t a, uint64_t b, uint32_t id, uint32_t acc) {
    asm volatile(
        "{ .reg .pred p; setp.ne.b32 p, %4, 0; "
        "tcgen05.mma.cta_group::1.kind::f16 [%0], %1, %2, %3, p; }"
        ::"r"(d), "l"(a), "l"(b), "r"(id), "r"(acc) : "memory");
}
// Block-scaled instruction descriptor (kind::mxf8f6f4.block_scale, fp32
// accumulator, both K-major): B scale-factor byte id at bits 4..5, A/B
// formats at 7..9 / 10..12 (0 E4M3, 5 E2M1), N >> 3 at 17..22, scale format
// E8M0 at bit 23, M >> 4 at 24..28, A scale-factor byte id at 29..30; K = 32.
__host__ __device__ constexpr uint32_t idesc_bs(int M, int N, uint32_t afmt, uint32_t bfmt, uint32_t sfid) {
    return (sfid << 4) | (afmt << 7) | (bfmt << 10) | ((uint32_t)(N >> 3) << 17) | (1u << 23) |
           ((uint32_t)(M >> 4) << 24) | (sfid << 29);
}
// D[tmem] (+)= (A . sA)[smem] . (B . sB)[smem]^T with UE8M0 scale factors per
// 32 K-elements read from TMEM (byte `sfid` of each lane's 32-bit word at
// sfa / sfb, the byte id also in the address's top bits), one instruction.
__device__ __forceinline__ void mma_mx_bs(uint32_t d, uint64_t a, uint64_t b, uint32_t id, uint32_t sfa,
                                          uint32_t sfb, uint32_t acc) {
    asm volatile(
        "{ .reg .pred p; setp.ne.b32 p, %4, 0; "
        "tcgen05.mma.cta_group::1.kind::mxf8f6f4.block_scale [%0], %1, %2, %3, [%5], [%6], p; }"
        ::"r"(d), "l"(a), "l"(b), "r"(id), "r"(acc), "r"(sfa), "r"(sfb) : "memory");
}
// The warp's 32 TMEM lanes (its lane quadrant), 4 consecutive 32-bit
// columns from taddr, all given the value w; tmem_wait_st before relying on it.
__device__ __forceinline__ void tmem_st4(uint32_t taddr, uint32_t w) {
    asm volatile("tcgen05.st.sync.aligned.32x32b.x4.b32 [%0], {%1, %1, %1, %1};" ::"r"(taddr), "r"(w)
                 : "memory");
}
__device__ __forceinline__ void tmem_wait_st() {
    asm volatile("tcgen05.wait::st.sync.aligned;" ::: "memory");
}

// Arrive on *b once every tcgen05 op this thread issued so far is done.
__device__ __forceinline__ void commit(uint64_t *b) {
    asm volatile("tcgen05.commit.cta_group::1.mbarrier::arrive::one.shared::cluster.b64 [%0];" ::"r"(sa(b))
                 : "memory");
}
// 16 consecutive 32-bit columns of this thread's TMEM lane, without the
// wait (tmem_wait_ld before using any of them).
__device__ __forceinline__ void tmem_ld16_nowait(uint32_t taddr, uint32_t (&r)[16]) {
    asm volatile(
        "tcgen05.ld.sync.aligned.32x32b.x16.b32 {%0,%1,%2,%3,%4,%5,%6,%7,%8,%9,%10,%11,%12,%13,%14,%15}, [%16];"
        : "=r"(r[0]), "=r"(r[1]), "=r"(r[2]), "=r"(r[3]), "=r"(r[4]), "=r"(r[5]), "=r"(r[6]), "=r"(r[7]),
          "=r"(r[8]), "=r"(r[9]), "=r"(r[10]), "=r"(r[11]), "=r"(r[12]), "=r"(r[13]), "=r"(r[14]), "=r"(r[15])
        : "r"(taddr));
}
__device__ __forceinline__ void tmem_wait_ld() {
    asm volatile("tcgen05.wait::ld.sync.aligned;" ::: "memory");
}
// After tmem_wait_ld: an empty asm that "rewrites" the loaded registers, so
// no use of them can be scheduled above the wait (tcgen05.ld fills its
// destination registers asynchronously).
__device__ __forceinline__ void tmem_regs_ready(uint32_t (&r)[16]) {
    asm volatile(""
                 : "+r"(r[0]), "+r"(r[1]), "+r"(r[2]), "+r"(r[3]), "+r"(r[4]), "+r"(r[5]), "+r"(r[6]),
                   "+r"(r[7]), "+r"(r[8]), "+r"(r[9]), "+r"(r[10]), "+r"(r[11]), "+r"(r[12]), "+r"(r[13]),
                   "+r"(r[14]), "+r"(r[15]));
}
// 16 consecutive fp32 columns of this thread's TMEM lane.
__device__ __forceinline__ void tmem_ld16(uint32_t taddr, float (&v)[16]) {
    uint32_t r[16];
    asm volatile(
        "tcgen05.ld.sync.aligned.32x32b.x16.b32 {%0,%1,%2,%3,%4,%5,%6,%7,%8,%9,%10,%11,%12,%13,%14,%15}, [%16];"
        : "=r"(r[0]), "=r"(r[1]), "=r"(r[2]), "=r"(r[3]), "=r"(r[4]), "=r"(r[5]), "=r"(r[6]), "=r"(r[7]),
          "=r"(r[8]), "=r"(r[9]), "=r"(r[10]), "=r"(r[11]), "=r"(r[12]), "=r"(r[13]), "=r"(r[14]), "=r"(r[15])
        : "r"(taddr));
    tmem_wait_ld();
    tmem_regs_ready(r);
#pragma unroll
    for (int i = 0; i < 16; i++) v[i] = __uint_as_float(r[i]);
}

}  // namespace tc
}  // namespace ds4f
