// The peer-memory exchange across the GPUs of one box: the all-reduce of the tensor-parallel decoder step (inside the
// next RMSNorm: add_rms_norm_ar_kernel in decoder_ops.cu, add_rms_norm_ar_q8K_kernel in srv_gemm.cu).
//
// All-reduce (flag-in-word exchange). Every rank's row-parallel GEMM (attention output, FFN down) writes its partial
// sums into slot `slot` of its own symmetric buffer (mapped on every peer): [2 slots][kArRows rows][d] f32, followed by
// a receive area [2 slots][kArRows rows][kArMaxRanks source ranks][d] of 8-byte words. For row i, the rank's threads
// store each partial value with the (slot, row) epoch into the receive area of every rank (its own included) as ONE
// 64-bit word (value bits low, epoch high), then read its own receive area until each word from each rank carries the
// epoch, and add the values in rank order, so every rank sums the same values in the same order. An aligned 64-bit
// store is single-copy atomic: a word that shows the epoch shows the value written with it, so no fence and no flag
// round trip is needed, on either side. The partial rows themselves come from this rank's previous kernel (complete
// at griddepcontrol.wait). Waits are bounded (2 s, then an error status). A slot's words are rewritten by a rank only
// after its next exchange on the other slot, which needs this rank's words of that exchange, sent after it had read
// the slot: two slots suffice.
//
// The attention's record merge over peer memory (fa_merge_peers_kernel) exchanges its records the same way.
#pragma once
#include <cstdint>

#include "internal.h"
#include "ptx.cuh"

namespace srhpm {

constexpr int kArMaxRanks = 8;
constexpr int kArRows     = 16;

// bytes of one slot's partial rows
__host__ __device__ inline size_t ar_part_bytes(int64_t d) { return (size_t) kArRows * d * sizeof(float); }

// ---- all-reduce by flag-in-word exchange ------------------------------------------------------------------------

// byte offset of the receive area, and of word (slot, row, source rank, element 0)
__host__ __device__ inline size_t ar_recv_off(int64_t d) { return 2 * ar_part_bytes(d); }
__host__ __device__ inline size_t ar_recv_word(int64_t d, int slot, int row, int src) {
    return ar_recv_off(d) + ((((size_t) slot * kArRows + row) * kArMaxRanks + src) * (size_t) d) * sizeof(uint64_t);
}

__device__ __forceinline__ uint64_t ll_word(float v, uint32_t e) {
    return (uint64_t) __float_as_uint(v) | ((uint64_t) e << 32);
}
__device__ __forceinline__ void st_relaxed_sys_v2(void * p, uint64_t a, uint64_t b) {
    asm volatile("st.relaxed.sys.global.v2.b64 [%0], {%1, %2};" ::"l"(p), "l"(a), "l"(b) : "memory");
}
__device__ __forceinline__ void ld_relaxed_sys_v2(const void * p, uint64_t & a, uint64_t & b) {
    asm volatile("ld.relaxed.sys.global.v2.b64 {%0, %1}, [%2];" : "=l"(a), "=l"(b) : "l"(p) : "memory");
}

// the (slot, row) epoch of this exchange: thread 0 bumps the rank's counter, the CTA reads it after a barrier
__device__ inline uint32_t ar_epoch(uint32_t * epochs, int slot, int row, uint32_t * e_s) {
    if (threadIdx.x == 0) *e_s = ++epochs[slot * kArRows + row];
    __syncthreads();
    return *e_s;
}

// The thread's float4 j of row i: store this rank's partial values, with epoch e, into every rank's receive area
// (source = this rank). Each 8-byte word is single-copy atomic; the two words of a 16-byte store need not be.
__device__ __forceinline__ void ar_push4(const uint64_t * peers, int world, int rank, int slot, int i, int64_t d,
                                         int64_t j, uint32_t e) {
    const float4 p = reinterpret_cast<const float4 *>(peers[rank] + (size_t) slot * ar_part_bytes(d))[i * (d >> 2) + j];
    const uint64_t w0 = ll_word(p.x, e), w1 = ll_word(p.y, e), w2 = ll_word(p.z, e), w3 = ll_word(p.w, e);
    const size_t   o  = ar_recv_word(d, slot, i, rank) + (size_t) j * 4 * sizeof(uint64_t);
    for (int r = 0; r < world; r++) {
        uint8_t * q = reinterpret_cast<uint8_t *>(peers[r] + o);
        st_relaxed_sys_v2(q, w0, w1);
        st_relaxed_sys_v2(q + 16, w2, w3);
    }
}

// a += the ranks' values of float4 j of row i, in rank order, each read from this rank's receive area once its word
// carries epoch e (bounded: 2 s from t0, then the status word is set and the missing values count as 0)
__device__ __forceinline__ void ar_gather4(float4 & a, const uint64_t * peers, int world, int rank, int slot, int i,
                                           int64_t d, int64_t j, uint32_t e, uint64_t t0, bool & ok, int32_t * status) {
    for (int r = 0; r < world; r++) {
        const uint8_t * q = reinterpret_cast<const uint8_t *>(peers[rank] + ar_recv_word(d, slot, i, r)) +
                            (size_t) j * 4 * sizeof(uint64_t);
        uint64_t w[4];
        for (;;) {
            ld_relaxed_sys_v2(q, w[0], w[1]);
            ld_relaxed_sys_v2(q + 16, w[2], w[3]);
            if ((uint32_t) (w[0] >> 32) == e && (uint32_t) (w[1] >> 32) == e && (uint32_t) (w[2] >> 32) == e &&
                (uint32_t) (w[3] >> 32) == e) {
                break;
            }
            if (!ok || globaltimer_ns() - t0 > 2000000000ull) {
                if (ok) atomicExch(status, kErrPeerWait);
                ok = false;
                w[0] = w[1] = w[2] = w[3] = 0;
                break;
            }
            __nanosleep(32);
        }
        a.x += __uint_as_float((uint32_t) w[0]);
        a.y += __uint_as_float((uint32_t) w[1]);
        a.z += __uint_as_float((uint32_t) w[2]);
        a.w += __uint_as_float((uint32_t) w[3]);
    }
}

}  // namespace srhpm
