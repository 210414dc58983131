// The peer-memory flag barrier across the GPUs of one box, and the all-reduce of the tensor-parallel decoder step built
// on it (add_rms_norm_ar_kernel in decoder_ops.cu, add_rms_norm_q8K_kernel in srv_gemm.cu); the attention's record
// merge over peer memory (fa_merge_peers_kernel in fa_decode.cu) uses the same barrier.
//
// Every rank's row-parallel GEMM (attention output, FFN down) writes its partial sums into slot `slot` of its own
// symmetric buffer (mapped on every peer): [2 slots][kArRows rows][d] f32, then flags [2][kArRows][kArMaxRanks] u32.
// For row i, one thread bumps this rank's epoch of (slot, row), publishes it into every peer's flag (slot, i, rank),
// and waits until every peer's flag in its own buffer has reached it (bounded: 2 s, then an error status). The row is
// then summed over ranks in rank order, so every rank adds the same values in the same order. Each slot is rewritten
// only after a later barrier of the same rows, so two suffice.
//
// Ordering (PTX memory model, system scope): the partial rows were written by the previous kernel of each rank,
// complete and visible to this grid once it passes griddepcontrol.wait. The waiting thread issues one
// fence.acq_rel.sys before its relaxed flag stores (a release: the rows are ordered before the flags every peer
// polls) and one after its polls have seen every peer's flag (an acquire: the peers' rows are ordered before the
// loads that follow); the CTA barrier after the wait carries that order to the CTA's other threads. The peer rows
// are read uncached (ld.global.cv).
#pragma once
#include <cstdint>

#include "internal.h"
#include "ptx.cuh"

namespace srhpm {

constexpr int kArMaxRanks = 8;
constexpr int kArRows     = 16;

__device__ __forceinline__ uint64_t global_timer_ns() {
    uint64_t t;
    asm volatile("mov.u64 %0, %%globaltimer;" : "=l"(t));
    return t;
}
__device__ __forceinline__ void st_relaxed_sys(uint32_t * p, uint32_t v) {
    asm volatile("st.relaxed.sys.global.u32 [%0], %1;" ::"l"(p), "r"(v) : "memory");
}
__device__ __forceinline__ uint32_t ld_relaxed_sys(const uint32_t * p) {
    uint32_t v;
    asm volatile("ld.relaxed.sys.global.u32 %0, [%1];" : "=r"(v) : "l"(p) : "memory");
    return v;
}

// bytes of one slot's partial rows
__host__ __device__ inline size_t ar_part_bytes(int64_t d) { return (size_t) kArRows * d * sizeof(float); }

// One flag round of `row` (one thread calls it): publish epoch e into flag [row][rank] of every rank's buffer (flags
// [rows][kArMaxRanks] u32 at byte offset flag_off), then wait until every rank's flag [row][j] in this rank's buffer
// has reached e. Release before the stores, acquire after the polls (see above). Returns false (and sets the status
// word) when a peer's flag did not arrive within 2 s.
__device__ inline bool peer_row_barrier(const uint64_t * peers, int world, int rank, size_t flag_off, int row,
                                        uint32_t e, int32_t * status) {
    const size_t fo = flag_off + ((size_t) row * kArMaxRanks + rank) * sizeof(uint32_t);
    fence_acq_rel_sys();  // release: this rank's data before its flags
    for (int j = 0; j < world; j++) st_relaxed_sys(reinterpret_cast<uint32_t *>(peers[j] + fo), e);
    const uint32_t * mine = reinterpret_cast<const uint32_t *>(peers[rank] + flag_off) + (size_t) row * kArMaxRanks;
    const uint64_t   t0   = global_timer_ns();
    bool             ok   = true;
    for (int j = 0; j < world && ok; j++) {
        while ((int32_t) (ld_relaxed_sys(mine + j) - e) < 0) {
            if (global_timer_ns() - t0 > 2000000000ull) {
                ok = false;
                atomicExch(status, kErrPeerWait);
                break;
            }
            __nanosleep(64);
        }
    }
    fence_acq_rel_sys();  // acquire: every peer's data after its flag
    return ok;
}

// The flag barrier of row i of the all-reduce (one thread calls it).
__device__ inline bool ar_row_barrier(const uint64_t * peers, int world, int rank, int slot, uint32_t * epochs, int i,
                                      int64_t d, int32_t * status) {
    const uint32_t e = ++epochs[slot * kArRows + i];
    return peer_row_barrier(peers, world, rank, 2 * ar_part_bytes(d), slot * kArRows + i, e, status);
}

// x4 += the ranks' partial sums of float4 j of row i, in rank order
__device__ __forceinline__ void ar_add_row4(float4 & a, const uint64_t * peers, int world, int slot, int i, int64_t d4,
                                            int64_t j) {
    const size_t pb = ar_part_bytes(d4 * 4);
    for (int r = 0; r < world; r++) {
        const float4 b = __ldcv(reinterpret_cast<const float4 *>(peers[r] + slot * pb) + i * d4 + j);
        a.x += b.x;
        a.y += b.y;
        a.z += b.z;
        a.w += b.w;
    }
}

}  // namespace srhpm
