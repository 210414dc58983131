// Thin wrappers over the sm_100a PTX this library uses: mbarriers with bounded waits, 1-D bulk async copies
// (global -> shared, completion counted on an mbarrier), int8 tensor-core MMA, programmatic dependent launch.
#pragma once
#include <cstdint>
#include <cuda_fp16.h>

namespace srhpm {

// Bound of every mbarrier wait: kWaitLimit probes of try_wait (each blocks for a hardware-defined interval while
// the phase is incomplete). A wait that runs out sets the kernel's error word and the kernel finishes without
// hanging.
constexpr uint32_t kWaitLimit = 1u << 22;
// The stage waits of the GEMM pipeline pass a suspend-time hint instead: the waiting thread sleeps until the phase
// completes or kSuspendNs elapse (no spinning that takes issue slots from the other warps); bound kSuspendLimit
// probes, ~2 s at most.
constexpr uint32_t kSuspendNs    = 20000;
constexpr uint32_t kSuspendLimit = 100000;

// error words written to the context's device status slot
enum : int32_t {
    kErrNone        = 0,
    kErrWaitFull    = 1,
    kErrWaitEmpty   = 2,
    kErrWaitDrain   = 3,
    kErrPeerWait    = 4,
    kErrClusterWait = 5,
    kErrGridWait    = 6,
};

__device__ __forceinline__ uint32_t smem_u32(const void * p) {
    return static_cast<uint32_t>(__cvta_generic_to_shared(p));
}

__device__ __forceinline__ void mbar_init(uint64_t * bar, uint32_t count) {
    asm volatile("mbarrier.init.shared::cta.b64 [%0], %1;" ::"r"(smem_u32(bar)), "r"(count) : "memory");
}

__device__ __forceinline__ void fence_mbar_init() {
    asm volatile("fence.mbarrier_init.release.cluster;" ::: "memory");
}

__device__ __forceinline__ void mbar_arrive(uint64_t * bar) {
    asm volatile("mbarrier.arrive.release.cta.shared::cta.b64 _, [%0];" ::"r"(smem_u32(bar)) : "memory");
}

__device__ __forceinline__ void mbar_arrive_expect_tx(uint64_t * bar, uint32_t tx) {
    asm volatile("mbarrier.arrive.expect_tx.release.cta.shared::cta.b64 _, [%0], %1;" ::"r"(smem_u32(bar)), "r"(tx)
                 : "memory");
}

__device__ __forceinline__ bool mbar_try_wait(uint64_t * bar, uint32_t parity) {
    uint32_t ok;
    asm volatile(
        "{\n\t.reg .pred p;\n\t"
        "mbarrier.try_wait.parity.acquire.cta.shared::cta.b64 p, [%1], %2;\n\t"
        "selp.u32 %0, 1, 0, p;\n\t}"
        : "=r"(ok)
        : "r"(smem_u32(bar)), "r"(parity)
        : "memory");
    return ok != 0;
}

__device__ __forceinline__ bool mbar_try_wait_hint(uint64_t * bar, uint32_t parity) {
    uint32_t ok;
    asm volatile(
        "{\n\t.reg .pred p;\n\t"
        "mbarrier.try_wait.parity.acquire.cta.shared::cta.b64 p, [%1], %2, %3;\n\t"
        "selp.u32 %0, 1, 0, p;\n\t}"
        : "=r"(ok)
        : "r"(smem_u32(bar)), "r"(parity), "n"(kSuspendNs)
        : "memory");
    return ok != 0;
}

// bounded wait with the suspend hint; false when the limit ran out
__device__ __forceinline__ bool mbar_wait_sleep(uint64_t * bar, uint32_t parity) {
    for (uint32_t i = 0; i < kSuspendLimit; i++) {
        if (mbar_try_wait_hint(bar, parity)) {
            return true;
        }
    }
    return false;
}

// bounded wait for the phase with the given parity to complete; false when the limit ran out
__device__ __forceinline__ bool mbar_wait(uint64_t * bar, uint32_t parity) {
    for (uint32_t i = 0; i < kWaitLimit; i++) {
        if (mbar_try_wait(bar, parity)) {
            return true;
        }
    }
    return false;
}

// 1-D bulk copy global -> shared of `bytes` (multiple of 16, both addresses 16-byte aligned), completion counted on bar
__device__ __forceinline__ void bulk_g2s(void * dst, const void * src, uint32_t bytes, uint64_t * bar) {
    asm volatile(
        "cp.async.bulk.shared::cluster.global.mbarrier::complete_tx::bytes [%0], [%1], %2, [%3];" ::"r"(smem_u32(dst)),
        "l"(src), "r"(bytes), "r"(smem_u32(bar))
        : "memory");
}

// 2-D tiled TMA load of one box at element coordinates (x, y), completion counted on bar (no multicast)
__device__ __forceinline__ void tma_load_2d(void * dst, const void * tmap, int x, int y, uint64_t * bar) {
    asm volatile(
        "cp.async.bulk.tensor.2d.shared::cluster.global.tile.mbarrier::complete_tx::bytes [%0], [%1, {%2, %3}], [%4];" ::
            "r"(smem_u32(dst)),
        "l"(tmap), "r"(x), "r"(y), "r"(smem_u32(bar))
        : "memory");
}

__device__ __forceinline__ void prefetch_tmap(const void * tmap) {
    asm volatile("prefetch.tensormap [%0];" ::"l"(tmap) : "memory");
}

// ---- thread-block clusters: distributed shared memory and remote mbarrier arrivals
__device__ __forceinline__ uint32_t mapa_shared(uint32_t saddr, uint32_t rank) {
    uint32_t r;
    asm volatile("mapa.shared::cluster.u32 %0, %1, %2;" : "=r"(r) : "r"(saddr), "r"(rank));
    return r;
}
__device__ __forceinline__ void cluster_sync_all() {
    asm volatile("barrier.cluster.arrive.release.aligned;\n\tbarrier.cluster.wait.acquire.aligned;" ::: "memory");
}
__device__ __forceinline__ void fence_acq_rel_cluster() { asm volatile("fence.acq_rel.cluster;" ::: "memory"); }
__device__ __forceinline__ void mbar_arrive_cluster(uint32_t cluster_addr) {
    asm volatile("mbarrier.arrive.release.cluster.shared::cluster.b64 _, [%0];" ::"r"(cluster_addr) : "memory");
}
__device__ __forceinline__ float ld_dsmem_f32(uint32_t cluster_addr) {
    float v;
    asm volatile("ld.shared::cluster.f32 %0, [%1];" : "=f"(v) : "r"(cluster_addr) : "memory");
    return v;
}
// bounded wait on a local mbarrier whose arrivals come from other CTAs of the cluster (acquire at cluster scope)
__device__ __forceinline__ bool mbar_wait_cluster(uint64_t * bar, uint32_t parity) {
    for (uint32_t i = 0; i < kWaitLimit; i++) {
        uint32_t ok;
        asm volatile(
            "{\n\t.reg .pred p;\n\t"
            "mbarrier.try_wait.parity.acquire.cluster.shared::cta.b64 p, [%1], %2;\n\t"
            "selp.u32 %0, 1, 0, p;\n\t}"
            : "=r"(ok)
            : "r"(smem_u32(bar)), "r"(parity)
            : "memory");
        if (ok) return true;
    }
    return false;
}

// barrier among `count` threads (a multiple of 32) on hardware barrier `id` (id 0 is __syncthreads)
__device__ __forceinline__ void named_bar_sync(int id, int count) {
    asm volatile("bar.sync %0, %1;" ::"r"(id), "r"(count) : "memory");
}

// orders this thread's generic-proxy shared-memory writes before later async-proxy (bulk copy) accesses
__device__ __forceinline__ void fence_proxy_async_smem() {
    asm volatile("fence.proxy.async.shared::cta;" ::: "memory");
}

// orders generic-proxy global-memory accesses with async-proxy (bulk copy / TMA) accesses of the same locations
__device__ __forceinline__ void fence_proxy_async_global() {
    asm volatile("fence.proxy.async.global;" ::: "memory");
}

// barrier arrival without waiting (the waiting side calls named_bar_sync with the same id and count)
__device__ __forceinline__ void named_bar_arrive(int id, int count) {
    asm volatile("bar.arrive %0, %1;" ::"r"(id), "r"(count) : "memory");
}

__device__ __forceinline__ uint32_t ld_acquire_gpu(const uint32_t * p) {
    uint32_t v;
    asm volatile("ld.acquire.gpu.global.u32 %0, [%1];" : "=r"(v) : "l"(p) : "memory");
    return v;
}

__device__ __forceinline__ uint64_t globaltimer_ns() {
    uint64_t t;
    asm volatile("mov.u64 %0, %%globaltimer;" : "=l"(t));
    return t;
}

// programmatic dependent launch: wait for the preceding grid's writes / let the next grid start its prologue
__device__ __forceinline__ void pdl_wait() { asm volatile("griddepcontrol.wait;" ::: "memory"); }
__device__ __forceinline__ void pdl_launch_dependents() { asm volatile("griddepcontrol.launch_dependents;" :::); }

// D = A(16x32, row) * B(32x8, col) + C, int8 operands, int32 accumulators. A unsigned (u8) or signed (s8), B signed.
// Fragments (g = lane/4, t = lane%4): a0 = A[g][4t..4t+3], a1 = A[g+8][4t..], a2 = A[g][16+4t..], a3 = A[g+8][16+4t..];
// b0 = B[4t..4t+3][g], b1 = B[16+4t..][g]; c0 = C[g][2t], c1 = C[g][2t+1], c2 = C[g+8][2t], c3 = C[g+8][2t+1].
template <bool A_UNSIGNED>
__device__ __forceinline__ void mma_k32(int (&c)[4], uint32_t a0, uint32_t a1, uint32_t a2, uint32_t a3, uint32_t b0,
                                        uint32_t b1) {
    if constexpr (A_UNSIGNED) {
        asm volatile(
            "mma.sync.aligned.m16n8k32.row.col.s32.u8.s8.s32 {%0,%1,%2,%3}, {%4,%5,%6,%7}, {%8,%9}, {%0,%1,%2,%3};"
            : "+r"(c[0]), "+r"(c[1]), "+r"(c[2]), "+r"(c[3])
            : "r"(a0), "r"(a1), "r"(a2), "r"(a3), "r"(b0), "r"(b1));
    } else {
        asm volatile(
            "mma.sync.aligned.m16n8k32.row.col.s32.s8.s8.s32 {%0,%1,%2,%3}, {%4,%5,%6,%7}, {%8,%9}, {%0,%1,%2,%3};"
            : "+r"(c[0]), "+r"(c[1]), "+r"(c[2]), "+r"(c[3])
            : "r"(a0), "r"(a1), "r"(a2), "r"(a3), "r"(b0), "r"(b1));
    }
}

// D = A(16x32) * B(32x8) with a zero accumulator input (no per-call register zeroing)
template <bool A_UNSIGNED>
__device__ __forceinline__ void mma_k32_z(int (&d)[4], uint32_t a0, uint32_t a1, uint32_t a2, uint32_t a3,
                                          uint32_t b0, uint32_t b1) {
    const int z = 0;
    if constexpr (A_UNSIGNED) {
        asm volatile(
            "mma.sync.aligned.m16n8k32.row.col.s32.u8.s8.s32 {%0,%1,%2,%3}, {%4,%5,%6,%7}, {%8,%9}, {%10,%10,%10,%10};"
            : "=r"(d[0]), "=r"(d[1]), "=r"(d[2]), "=r"(d[3])
            : "r"(a0), "r"(a1), "r"(a2), "r"(a3), "r"(b0), "r"(b1), "r"(z));
    } else {
        asm volatile(
            "mma.sync.aligned.m16n8k32.row.col.s32.s8.s8.s32 {%0,%1,%2,%3}, {%4,%5,%6,%7}, {%8,%9}, {%10,%10,%10,%10};"
            : "=r"(d[0]), "=r"(d[1]), "=r"(d[2]), "=r"(d[3])
            : "r"(a0), "r"(a1), "r"(a2), "r"(a3), "r"(b0), "r"(b1), "r"(z));
    }
}

// D = A(16x32) * B(32x8) + c in every accumulator (the same constant for the 4 outputs)
template <bool A_UNSIGNED>
__device__ __forceinline__ void mma_k32_c(int (&d)[4], uint32_t a0, uint32_t a1, uint32_t a2, uint32_t a3,
                                          uint32_t b0, uint32_t b1, int c) {
    if constexpr (A_UNSIGNED) {
        asm volatile(
            "mma.sync.aligned.m16n8k32.row.col.s32.u8.s8.s32 {%0,%1,%2,%3}, {%4,%5,%6,%7}, {%8,%9}, {%10,%10,%10,%10};"
            : "=r"(d[0]), "=r"(d[1]), "=r"(d[2]), "=r"(d[3])
            : "r"(a0), "r"(a1), "r"(a2), "r"(a3), "r"(b0), "r"(b1), "r"(c));
    } else {
        asm volatile(
            "mma.sync.aligned.m16n8k32.row.col.s32.s8.s8.s32 {%0,%1,%2,%3}, {%4,%5,%6,%7}, {%8,%9}, {%10,%10,%10,%10};"
            : "=r"(d[0]), "=r"(d[1]), "=r"(d[2]), "=r"(d[3])
            : "r"(a0), "r"(a1), "r"(a2), "r"(a3), "r"(b0), "r"(b1), "r"(c));
    }
}

// packed f32 pairs (sm_100 f32x2 instructions: one issue for two lanes of arithmetic, each rounded as the scalar
// instruction rounds)
typedef unsigned long long f2;
__device__ __forceinline__ f2 f2_pack(float a, float b) {
    f2 r;
    asm("mov.b64 %0, {%1, %2};" : "=l"(r) : "f"(a), "f"(b));
    return r;
}
__device__ __forceinline__ void f2_unpack(f2 r, float & a, float & b) {
    asm("mov.b64 {%0, %1}, %2;" : "=f"(a), "=f"(b) : "l"(r));
}
__device__ __forceinline__ f2 f2_add(f2 a, f2 b) {
    f2 r;
    asm("add.rn.f32x2 %0, %1, %2;" : "=l"(r) : "l"(a), "l"(b));
    return r;
}
__device__ __forceinline__ f2 f2_mul(f2 a, f2 b) {
    f2 r;
    asm("mul.rn.f32x2 %0, %1, %2;" : "=l"(r) : "l"(a), "l"(b));
    return r;
}
__device__ __forceinline__ f2 f2_fma(f2 a, f2 b, f2 c) {
    f2 r;
    asm("fma.rn.f32x2 %0, %1, %2, %3;" : "=l"(r) : "l"(a), "l"(b), "l"(c));
    return r;
}

// D = A(16x16) * B(16x8) with a zero accumulator input
template <bool A_UNSIGNED>
__device__ __forceinline__ void mma_k16_z(int (&d)[4], uint32_t a0, uint32_t a1, uint32_t b0) {
    const int z = 0;
    if constexpr (A_UNSIGNED) {
        asm volatile("mma.sync.aligned.m16n8k16.row.col.s32.u8.s8.s32 {%0,%1,%2,%3}, {%4,%5}, {%6}, {%7,%7,%7,%7};"
                     : "=r"(d[0]), "=r"(d[1]), "=r"(d[2]), "=r"(d[3])
                     : "r"(a0), "r"(a1), "r"(b0), "r"(z));
    } else {
        asm volatile("mma.sync.aligned.m16n8k16.row.col.s32.s8.s8.s32 {%0,%1,%2,%3}, {%4,%5}, {%6}, {%7,%7,%7,%7};"
                     : "=r"(d[0]), "=r"(d[1]), "=r"(d[2]), "=r"(d[3])
                     : "r"(a0), "r"(a1), "r"(b0), "r"(z));
    }
}

// explicit shared-space loads at 32-bit shared addresses (generic pointers into shared memory can compile to generic
// loads once their provenance is lost)
__device__ __forceinline__ uint32_t sld32(uint32_t a) {
    uint32_t v;
    asm volatile("ld.shared.b32 %0, [%1];" : "=r"(v) : "r"(a));
    return v;
}
// 4 bytes at a shared address that is 4-byte aligned (A4), or any even one (two aligned words and a funnel shift)
template <bool A4>
__device__ __forceinline__ uint32_t sld4_a2(uint32_t a) {
    if constexpr (A4) {
        return sld32(a);
    } else {
        const uint32_t b = a & ~3u;
        return __funnelshift_r(sld32(b), sld32(b + 4), (a & 3u) * 8);
    }
}
// 32-bit shared load at base + OFF (OFF folded into the instruction)
template <int OFF>
__device__ __forceinline__ uint32_t sld32o(uint32_t base) {
    uint32_t v;
    asm volatile("ld.shared.b32 %0, [%1+%2];" : "=r"(v) : "r"(base), "n"(OFF));
    return v;
}
// 8 bytes at shared address base + OFF: base 4-byte aligned (A4), or any even address (three aligned words and two
// funnel shifts by sh = 8 * (address mod 4))
template <bool A4, int OFF>
__device__ __forceinline__ uint2 sld8o(uint32_t base, uint32_t sh) {
    if constexpr (A4) {
        return make_uint2(sld32o<OFF>(base), sld32o<OFF + 4>(base));
    } else {
        const uint32_t w0 = sld32o<OFF>(base), w1 = sld32o<OFF + 4>(base), w2 = sld32o<OFF + 8>(base);
        return make_uint2(__funnelshift_r(w0, w1, sh), __funnelshift_r(w1, w2, sh));
    }
}
__device__ __forceinline__ float half_bits_to_float(uint16_t h) { return __half2float(__ushort_as_half(h)); }

__device__ __forceinline__ uint16_t lds_u16(const uint8_t * p) { return *reinterpret_cast<const uint16_t *>(p); }

}  // namespace srhpm
