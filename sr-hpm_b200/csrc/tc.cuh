// tcgen05 (5th-generation tensor core) helpers for sm_100a: tensor-memory allocation, shared-memory matrix
// descriptors, instruction descriptors, MMA issue / commit, tensor-memory loads and stores, fences.
//
// Only the SWIZZLE_NONE canonical layouts are used. In 16-byte units ("rows" of a core matrix):
//   K-major : core matrix = 8 rows (M or N) x 16 bytes along K, the 8 rows 16 bytes apart (128 contiguous bytes);
//             SBO = byte distance between consecutive 8-row groups along M/N,
//             LBO = byte distance between the two 16-byte K halves of one instruction's K extent (32 bytes).
//   MN-major: core matrix = 8 K-rows x 16 bytes along M/N (8 16-bit elements), the K-rows 16 bytes apart;
//             SBO = byte distance between consecutive 8-element groups along M/N,
//             LBO = byte distance between consecutive 8-row groups along K.
// Accumulators (M = 128, one CTA): row i of D is tensor-memory lane i, column j of D is column (base + j), 32 bits.
// A warp reads the 32 lanes of its quarter (warp % 4) of tensor memory.
#pragma once
#include <cstdint>

namespace srhpm {
namespace tc {

// ---- descriptors ------------------------------------------------------------------------------------------------

// shared-memory matrix descriptor: SWIZZLE_NONE, descriptor version 1 (sm_100), base offset 0
__device__ __forceinline__ uint64_t sdesc(uint32_t saddr, uint32_t lbo, uint32_t sbo) {
    return (uint64_t) ((saddr >> 4) & 0x3FFFu) | ((uint64_t) ((lbo >> 4) & 0x3FFFu) << 16) |
           ((uint64_t) ((sbo >> 4) & 0x3FFFu) << 32) | (1ull << 46);
}

// instruction descriptor fields (kind::f16 and kind::i8)
enum : uint32_t { kD_F16 = 0, kD_F32 = 1, kD_S32 = 2 };
enum : uint32_t { kAB_F16 = 0, kAB_BF16 = 1, kAB_U8 = 0, kAB_S8 = 1 };
enum : uint32_t { kKMajor = 0, kMNMajor = 1 };

__host__ __device__ constexpr uint32_t idesc(uint32_t dfmt, uint32_t afmt, uint32_t bfmt, uint32_t amajor, uint32_t bmajor, uint32_t N,
                         uint32_t M) {
    return (dfmt << 4) | (afmt << 7) | (bfmt << 10) | (amajor << 15) | (bmajor << 16) | ((N >> 3) << 17) |
           ((M >> 4) << 24);
}

// ---- tensor memory -----------------------------------------------------------------------------------------------

// one full warp: allocate `ncols` columns (power of two >= 32); the base address is written to *dst (shared)
__device__ __forceinline__ void tmem_alloc(uint32_t * dst, uint32_t ncols) {
    const uint32_t a = (uint32_t) __cvta_generic_to_shared(dst);
    asm volatile("tcgen05.alloc.cta_group::1.sync.aligned.shared::cta.b32 [%0], %1;" ::"r"(a), "r"(ncols) : "memory");
    asm volatile("tcgen05.relinquish_alloc_permit.cta_group::1.sync.aligned;" ::: "memory");
}
// one full warp (the allocating one)
__device__ __forceinline__ void tmem_free(uint32_t base, uint32_t ncols) {
    asm volatile("tcgen05.dealloc.cta_group::1.sync.aligned.b32 %0, %1;" ::"r"(base), "r"(ncols) : "memory");
}

__device__ __forceinline__ void fence_before() { asm volatile("tcgen05.fence::before_thread_sync;" ::: "memory"); }
__device__ __forceinline__ void fence_after() { asm volatile("tcgen05.fence::after_thread_sync;" ::: "memory"); }

// ---- MMA (issued by one thread) ----------------------------------------------------------------------------------

__device__ __forceinline__ void mma_i8(uint32_t d, uint64_t a, uint64_t b, uint32_t id, uint32_t accumulate) {
    asm volatile(
        "{\n\t.reg .pred p;\n\tsetp.ne.b32 p, %4, 0;\n\t"
        "tcgen05.mma.cta_group::1.kind::i8 [%0], %1, %2, %3, {%5, %5, %5, %5}, p;\n\t}" ::"r"(d),
        "l"(a), "l"(b), "r"(id), "r"(accumulate), "r"(0u)
        : "memory");
}
__device__ __forceinline__ void mma_f16(uint32_t d, uint64_t a, uint64_t b, uint32_t id, uint32_t accumulate) {
    asm volatile(
        "{\n\t.reg .pred p;\n\tsetp.ne.b32 p, %4, 0;\n\t"
        "tcgen05.mma.cta_group::1.kind::f16 [%0], %1, %2, %3, {%5, %5, %5, %5}, p;\n\t}" ::"r"(d),
        "l"(a), "l"(b), "r"(id), "r"(accumulate), "r"(0u)
        : "memory");
}
// the mbarrier receives one arrival when every MMA this thread issued before has completed
__device__ __forceinline__ void commit(uint64_t * bar) {
    const uint32_t a = (uint32_t) __cvta_generic_to_shared(bar);
    asm volatile("tcgen05.commit.cta_group::1.mbarrier::arrive::one.shared::cluster.b64 [%0];" ::"r"(a) : "memory");
}

// ---- tensor memory <-> registers (whole warp; lane = warp quarter base + lane id) ----------------------------------

__device__ __forceinline__ void ld16(uint32_t taddr, uint32_t (&r)[16]) {
    asm volatile(
        "tcgen05.ld.sync.aligned.32x32b.x16.b32 {%0,%1,%2,%3,%4,%5,%6,%7,%8,%9,%10,%11,%12,%13,%14,%15}, [%16];"
        : "=r"(r[0]), "=r"(r[1]), "=r"(r[2]), "=r"(r[3]), "=r"(r[4]), "=r"(r[5]), "=r"(r[6]), "=r"(r[7]),
          "=r"(r[8]), "=r"(r[9]), "=r"(r[10]), "=r"(r[11]), "=r"(r[12]), "=r"(r[13]), "=r"(r[14]), "=r"(r[15])
        : "r"(taddr));
}
__device__ __forceinline__ void ld8(uint32_t taddr, uint32_t (&r)[8]) {
    asm volatile("tcgen05.ld.sync.aligned.32x32b.x8.b32 {%0,%1,%2,%3,%4,%5,%6,%7}, [%8];"
                 : "=r"(r[0]), "=r"(r[1]), "=r"(r[2]), "=r"(r[3]), "=r"(r[4]), "=r"(r[5]), "=r"(r[6]), "=r"(r[7])
                 : "r"(taddr));
}
__device__ __forceinline__ void st16(uint32_t taddr, const uint32_t (&r)[16]) {
    asm volatile(
        "tcgen05.st.sync.aligned.32x32b.x16.b32 [%0], {%1,%2,%3,%4,%5,%6,%7,%8,%9,%10,%11,%12,%13,%14,%15,%16};" ::
            "r"(taddr),
        "r"(r[0]), "r"(r[1]), "r"(r[2]), "r"(r[3]), "r"(r[4]), "r"(r[5]), "r"(r[6]), "r"(r[7]), "r"(r[8]), "r"(r[9]),
        "r"(r[10]), "r"(r[11]), "r"(r[12]), "r"(r[13]), "r"(r[14]), "r"(r[15])
        : "memory");
}
__device__ __forceinline__ void st8(uint32_t taddr, const uint32_t (&r)[8]) {
    asm volatile("tcgen05.st.sync.aligned.32x32b.x8.b32 [%0], {%1,%2,%3,%4,%5,%6,%7,%8};" ::"r"(taddr), "r"(r[0]),
                 "r"(r[1]), "r"(r[2]), "r"(r[3]), "r"(r[4]), "r"(r[5]), "r"(r[6]), "r"(r[7])
                 : "memory");
}
__device__ __forceinline__ void ld4(uint32_t taddr, uint32_t (&r)[4]) {
    asm volatile("tcgen05.ld.sync.aligned.32x32b.x4.b32 {%0,%1,%2,%3}, [%4];"
                 : "=r"(r[0]), "=r"(r[1]), "=r"(r[2]), "=r"(r[3])
                 : "r"(taddr));
}
__device__ __forceinline__ void st4(uint32_t taddr, const uint32_t (&r)[4]) {
    asm volatile("tcgen05.st.sync.aligned.32x32b.x4.b32 [%0], {%1,%2,%3,%4};" ::"r"(taddr), "r"(r[0]), "r"(r[1]),
                 "r"(r[2]), "r"(r[3])
                 : "memory");
}
// NC (a multiple of 4, at most 28) consecutive columns of this warp's lane quarter
template <int NC> __device__ __forceinline__ void ld_cols(uint32_t taddr, uint32_t * r) {
    if constexpr (NC >= 16) ld16(taddr, *reinterpret_cast<uint32_t(*)[16]>(r));
    if constexpr ((NC & 8) != 0) ld8(taddr + (NC & 16), *reinterpret_cast<uint32_t(*)[8]>(r + (NC & 16)));
    if constexpr ((NC & 4) != 0) ld4(taddr + (NC & 24), *reinterpret_cast<uint32_t(*)[4]>(r + (NC & 24)));
}
template <int NC> __device__ __forceinline__ void st_cols(uint32_t taddr, const uint32_t * r) {
    if constexpr (NC >= 16) st16(taddr, *reinterpret_cast<const uint32_t(*)[16]>(r));
    if constexpr ((NC & 8) != 0) st8(taddr + (NC & 16), *reinterpret_cast<const uint32_t(*)[8]>(r + (NC & 16)));
    if constexpr ((NC & 4) != 0) st4(taddr + (NC & 24), *reinterpret_cast<const uint32_t(*)[4]>(r + (NC & 24)));
}
__device__ __forceinline__ void wait_ld() { asm volatile("tcgen05.wait::ld.sync.aligned;" ::: "memory"); }
__device__ __forceinline__ void wait_st() { asm volatile("tcgen05.wait::st.sync.aligned;" ::: "memory"); }

// lane-quarter base address of warp w (row 32 * (w % 4) of the accumulator)
__device__ __forceinline__ uint32_t taddr(uint32_t base, uint32_t warp, uint32_t col) {
    return base + ((32u * (warp & 3u)) << 16) + col;
}

}  // namespace tc
}  // namespace srhpm
