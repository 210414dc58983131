// Small-batch quantized matmul for speculative verification on sm_100a (the GPU counterpart of the reference's
// SRV kernels, patch/srhpm.patch:5448-6680, and of its dGPU co-verifier, dgpu/dgpu.cu:107-191).
//
// Y[t][r] = sum_k W[r][k] X[t][k] for N = 1..16 activation rows against GGUF-packed weight rows.
//
//   1. quant_q8K_kernel / quant_q80_kernel: each activation row is quantized per 256 columns to int8 with one f32
//      scale (bit-identical to srv_quantize_row, patch/srhpm.patch:5518-5575) -- or per 32 columns to q8_0 for Q8_0
//      weights -- into "activation records": for each super-block, NT = 8 or 16 token rows of 256 int8 values at a
//      288-byte stride (so that consecutive tokens fall on different shared-memory banks), then the scales. Only the
//      N real token rows are written: the padding rows (N..NT-1) reach only MMA output columns that are never stored.
//      srhpm_mul_mat_fused_quant does the same work in the GEMM kernel's own prologue (fq_quantize, fq_grid_meet).
//   2. srv_gemm_kernel: persistent CTAs over (64-row block, K range) units. A producer warp streams each unit
//      through a 3-4 stage shared-memory ring, one super-block column at a time: 2-D TMA boxes of the 64 row
//      segments (rows grouped G at a time when the row stride is not a multiple of 16 bytes; the < G rows past
//      the tensor map come by 1-D bulk copies) plus the column's activation record, completion counted on an
//      mbarrier. Four consumer warps each own 16 rows. Every super-block is decoded once in registers into int8 MMA
//      fragments (A = 16 rows x 32 (or 16) weights) and multiplied with all activation rows at once on the tensor
//      cores (B = 32 x 8 tokens), int32 exact; the integer block scales multiply the int32 fragments, the Q4_K/Q5_K
//      minimum term is a second MMA against the replicated 6-bit mins, and one f32 FMA per super-block and token
//      applies d_w * d_x -- the same integer arithmetic as the reference's srv_row (patch/srhpm.patch:6119-6226).
//
// The k order inside an MMA is free as long as A and B agree: Q4_K / Q5_K use "thread t holds weights 8t..8t+7"
// (one 8-byte load per row and nibble plane), the others the natural fragment order.
#include <algorithm>
#include <atomic>
#include <map>
#include <mutex>
#include <tuple>

#include <cuda.h>
#include <cstring>

#include "allreduce.cuh"
#include "internal.h"
#include "launch.cuh"
#include "ptx.cuh"

namespace srhpm {
namespace {

constexpr int     QK         = 256;
constexpr int     kMagic32   = 0x4B400000;        // the bits of 12582912.0f (1.5 * 2^23)
constexpr int     kNCW       = 4;                 // consumer warps, one per 16-row slice
constexpr int     kThreads   = (kNCW + 1) * 32;   // + 1 producer warp
constexpr int     kTileRows  = 16 * kNCW;         // weight rows per CTA tile
constexpr int     kTokStride = 288;               // bytes per token row inside an activation record
constexpr int     kMaxStages = 6;
constexpr int     kMaxSplit  = 8;                 // K ranges per product at most
constexpr int     kBarBytes  = 128;               // room for the 2 * kMaxStages + 2 mbarriers

__host__ __device__ constexpr int rec_nscales(bool q80, int NT) { return q80 ? 8 * NT : NT; }
// [NT token rows of kTokStride bytes][f32 scales][K-quant records: NT int32 sums of each token's 256 codes]
__host__ __device__ constexpr int rec_bytes(bool q80, int NT) {
    return (NT * kTokStride + 4 * rec_nscales(q80, NT) + (q80 ? 0 : 4 * NT) + 15) / 16 * 16;
}

// ---------------------------------------------------------------------------------------------------------------
// activation quantizers

// Warm L2 with this warp's activation segment (256 floats: one 128-byte line per 4 lanes) while the previous grid is
// still finishing. A hint only: the loads after griddepcontrol.wait still return what that grid wrote (L2 is the
// point of coherence the writes reach), so X may be the previous kernel's output.
__device__ __forceinline__ void prefetch_act_l2(const float * X, int64_t ldx, int N, int nsb, int TT, int lane) {
    const int64_t wid = (int64_t) blockIdx.x * 8 + (threadIdx.x >> 5);
    if (wid >= (int64_t) nsb * TT || (lane & 3) != 0) return;
    const int sb = (int) (wid / TT), t = (int) (wid % TT);
    if (t < N) asm volatile("prefetch.global.L2 [%0];" ::"l"(X + (int64_t) t * ldx + (int64_t) sb * QK + 8 * lane));
}

// one warp per (super-block, token); lane l owns columns 8l..8l+7
__device__ __forceinline__ void load8(const float * __restrict__ xp, float (&v)[8]) {
    if ((reinterpret_cast<uintptr_t>(xp) & 15) == 0) {
        const float4 a = *reinterpret_cast<const float4 *>(xp);
        const float4 b = *reinterpret_cast<const float4 *>(xp + 4);
        v[0] = a.x; v[1] = a.y; v[2] = a.z; v[3] = a.w; v[4] = b.x; v[5] = b.y; v[6] = b.z; v[7] = b.w;
    } else {
#pragma unroll
        for (int j = 0; j < 8; j++) v[j] = xp[j];
    }
}

__device__ __forceinline__ uint2 pack8(const int (&q)[8]) {
    uint2 r;
    r.x = (uint32_t) (q[0] & 0xff) | ((uint32_t) (q[1] & 0xff) << 8) | ((uint32_t) (q[2] & 0xff) << 16) |
          ((uint32_t) (q[3] & 0xff) << 24);
    r.y = (uint32_t) (q[4] & 0xff) | ((uint32_t) (q[5] & 0xff) << 8) | ((uint32_t) (q[6] & 0xff) << 16) |
          ((uint32_t) (q[7] & 0xff) << 24);
    return r;
}

// srv_quantize_row: amax = max |x| over 256; the first element of that magnitude (with its sign) gives
// iscale = -127 / max; q = min(round_half_even(iscale * x), 127); d = 1 / iscale. IEEE division, no contraction.
// One warp per (super-block, token); lane l holds columns 8l..8l+7 in v.
__device__ __forceinline__ void q8K_quantize_warp(const float (&v)[8], int lane, int (&qv)[8], float & dv) {
    float amax = 0.0f;  // fmaxf from 0 drops NaNs, so the lane maxima are non-negative, NaN-free floats, which order
#pragma unroll          // as their bit patterns: one integer warp reduction gives the maximum
    for (int j = 0; j < 8; j++) amax = fmaxf(amax, fabsf(v[j]));
    amax = __uint_as_float(__reduce_max_sync(0xffffffffu, __float_as_uint(amax)));
    dv   = 0.0f;
    if (amax == 0.0f) {
#pragma unroll
        for (int j = 0; j < 8; j++) qv[j] = 0;
    } else {
        int first = QK, jf = 0;
#pragma unroll
        for (int j = 7; j >= 0; j--) {
            if (fabsf(v[j]) == amax) {
                first = 8 * lane + j;
                jf    = j;
            }
        }
        float mine = v[0];
#pragma unroll
        for (int j = 1; j < 8; j++) mine = (j == jf) ? v[j] : mine;
        const int   fmin   = __reduce_min_sync(0xffffffffu, first);
        const float mx     = __shfl_sync(0xffffffffu, mine, fmin >> 3);
        const float iscale = __fdiv_rn(-127.0f, mx);
#pragma unroll
        for (int j = 0; j < 8; j++) qv[j] = min(__float2int_rn(__fmul_rn(iscale, v[j])), 127);
        dv = __fdiv_rn(1.0f, iscale);
    }
}

// record byte orders (the k order inside an MMA is free as long as weights and activations agree): natural; Q3_K:
// each lane's 8 columns in the order 0 4 1 5 2 6 3 7; IQ4_XS: in each 32-column sub-block, the pairs (l, l + 16)
// interleaved so that bytes 4t..4t+3 hold columns 4t, 4t+16, 4t+1, 4t+17 and bytes 16+4t.. hold 4t+2, 4t+18, 4t+3,
// 4t+19 (the order of the decoder's table lookups)
enum : int { kPermNone = 0, kPermQ3K = 1, kPermIQ4XS = 2 };
__host__ __device__ constexpr int record_perm(int wtype) {
    return wtype == SRHPM_TYPE_Q3_K ? kPermQ3K : wtype == SRHPM_TYPE_IQ4_XS ? kPermIQ4XS : kPermNone;
}

// the token row t of one super-block's activation record: the lane's 8 codes (perm: stored in the order
// 0 4 1 5 2 6 3 7, the k order of its decoder), the scale, the per-32 sums split into int8 halves s = 128 hi + lo
// (lo in 0..127) in the row's padding (hi at 256 + sub-block, lo at 264 + sub-block: the Q4_K / Q5_K minimum term),
// and the sum over all 256 after the scales (the Q3_K offset term)
__device__ __forceinline__ void q8K_store_record(const int (&qv)[8], float dv, uint8_t * rec, int t, int NT, int lane,
                                                 int perm) {
    const uint2 pk = pack8(qv);
    uint2       st = pk;
    if (perm == kPermQ3K) {
        st = make_uint2(__byte_perm(pk.x, pk.y, 0x5140), __byte_perm(pk.x, pk.y, 0x7362));
    } else if (perm == kPermIQ4XS) {
        // lane 4b + k holds columns 8k..8k+7 of sub-block b; lanes k < 2 write bytes 8k.. from the low halves of
        // their own and lane k + 2's words, lanes k >= 2 from the high halves of lane k - 2's and their own
        const uint32_t ox = __shfl_xor_sync(0xffffffffu, pk.x, 2), oy = __shfl_xor_sync(0xffffffffu, pk.y, 2);
        const bool     lo = (lane & 2) == 0;
        const uint2    A = lo ? pk : make_uint2(ox, oy), B = lo ? make_uint2(ox, oy) : pk;
        const uint32_t sel = lo ? 0x5140u : 0x7362u;
        st = make_uint2(__byte_perm(A.x, B.x, sel), __byte_perm(A.y, B.y, sel));
    }
    *reinterpret_cast<uint2 *>(rec + t * kTokStride + 8 * lane) = st;
    if (lane == 0) reinterpret_cast<float *>(rec + NT * kTokStride)[t] = dv;
    int s32 = 0;
#pragma unroll
    for (int j = 0; j < 8; j++) s32 += qv[j];
    s32 += __shfl_xor_sync(0xffffffffu, s32, 1);
    s32 += __shfl_xor_sync(0xffffffffu, s32, 2);
    if ((lane & 3) == 0) {
        rec[t * kTokStride + 256 + lane / 4] = (uint8_t) (int8_t) (s32 >> 7);
        rec[t * kTokStride + 264 + lane / 4] = (uint8_t) (s32 & 127);
    }
    // s32 is the sum of the lane's group of 4: the 8 groups' sums are the quarter of the lanes' total
    const int s256 = __reduce_add_sync(0xffffffffu, s32) >> 2;
    if (lane == 0) reinterpret_cast<int32_t *>(rec + NT * kTokStride + 4 * NT)[t] = s256;
}

template <bool DENSE>
__global__ void __launch_bounds__(256) quant_q8K_kernel(const float * __restrict__ X, int64_t ldx, int N, int nsb,
                                                         int NT, uint8_t * __restrict__ recs, int8_t * __restrict__ q,
                                                         float * __restrict__ d, int16_t * __restrict__ b32,
                                                         int16_t * __restrict__ b16, int32_t * __restrict__ cnt,
                                                         int ncnt, int perm) {
    // launched early behind the previous call's GEMM: let the next GEMM get resident, then wait for the previous
    // grid (it may still read the records and counters this kernel rewrites, or write the X it reads)
    pdl_launch_dependents();
    if (X) prefetch_act_l2(X, ldx, N, nsb, N, threadIdx.x & 31);
    pdl_wait();
    for (int i = blockIdx.x * blockDim.x + threadIdx.x; i < ncnt; i += gridDim.x * blockDim.x) cnt[i] = 0;
    const int     lane = threadIdx.x & 31;
    const int     TT   = N;  // records: the padding token rows are never read into a stored output
    const int64_t wid  = (int64_t) blockIdx.x * 8 + (threadIdx.x >> 5);
    if (wid >= (int64_t) nsb * TT) {
        return;
    }
    const int sb = (int) (wid / TT), t = (int) (wid % TT);
    float     v[8];
    if (t < N) {
        load8(X + (int64_t) t * ldx + (int64_t) sb * QK + 8 * lane, v);
    } else {
#pragma unroll
        for (int j = 0; j < 8; j++) v[j] = 0.0f;
    }
    int   qv[8];
    float dv;
    q8K_quantize_warp(v, lane, qv, dv);
    if constexpr (DENSE) {
        const uint2   pk = pack8(qv);
        const int64_t K  = (int64_t) nsb * QK;
        *reinterpret_cast<uint2 *>(q + (int64_t) t * K + (int64_t) sb * QK + 8 * lane) = pk;
        if (lane == 0) d[(int64_t) t * nsb + sb] = dv;
        int s = 0;
#pragma unroll
        for (int j = 0; j < 8; j++) s += qv[j];
        const int s16 = s + __shfl_xor_sync(0xffffffffu, s, 1);
        const int s32 = s16 + __shfl_xor_sync(0xffffffffu, s16, 2);
        if (b16 && (lane & 1) == 0) b16[(int64_t) t * (K / 16) + (int64_t) sb * 16 + lane / 2] = (int16_t) s16;
        if (b32 && (lane & 3) == 0) b32[(int64_t) t * (K / 32) + (int64_t) sb * 8 + lane / 4] = (int16_t) s32;
    } else {
        q8K_store_record(qv, dv, recs + (size_t) sb * rec_bytes(false, NT), t, NT, lane, perm);
    }
}

// SwiGLU fused with the activation quantizer of the GEMM that consumes h (the FFN down projection): one warp per
// (super-block, token); h = silu(gate) * up for its 256 values (as swiglu_kernel: g / (1 + expf(-g)) * u), written to
// h and quantized into the GEMM's records exactly as quant_q8K_kernel does; tokens N..NT-1 get zero rows; the first
// CTA zeroes the split-K counters.
__global__ void __launch_bounds__(256) swiglu_q8K_kernel(const float * __restrict__ gate, const float * __restrict__ up,
                                                         int64_t ld_in, float * __restrict__ h, int64_t ld_out, int N,
                                                         int nsb, int NT, uint8_t * __restrict__ recs, int perm,
                                                         int32_t * __restrict__ cnt, int ncnt) {
    pdl_launch_dependents();
    pdl_wait();
    if (blockIdx.x == 0) {
        for (int i = threadIdx.x; i < ncnt; i += blockDim.x) cnt[i] = 0;
    }
    const int     lane = threadIdx.x & 31;
    const int64_t wid  = (int64_t) blockIdx.x * 8 + (threadIdx.x >> 5);
    if (wid >= (int64_t) nsb * NT) return;
    const int sb = (int) (wid / NT), t = (int) (wid % NT);
    float     v[8];
    if (t < N) {
        const int64_t c0 = (int64_t) sb * QK + 8 * lane;
        float         g8[8], u8[8];
        load8(gate + (int64_t) t * ld_in + c0, g8);
        load8(up + (int64_t) t * ld_in + c0, u8);
#pragma unroll
        for (int j = 0; j < 8; j++) v[j] = g8[j] / (1.0f + expf(-g8[j])) * u8[j];
        float * hp = h + (int64_t) t * ld_out + c0;
        if (!h) {  // the records only (srhpm_mul_mat_swiglu)
        } else if ((reinterpret_cast<uintptr_t>(hp) & 15) == 0) {
            reinterpret_cast<float4 *>(hp)[0] = make_float4(v[0], v[1], v[2], v[3]);
            reinterpret_cast<float4 *>(hp)[1] = make_float4(v[4], v[5], v[6], v[7]);
        } else {
#pragma unroll
            for (int j = 0; j < 8; j++) hp[j] = v[j];
        }
    } else {
#pragma unroll
        for (int j = 0; j < 8; j++) v[j] = 0.0f;
    }
    int   qv[8];
    float dv;
    q8K_quantize_warp(v, lane, qv, dv);
    q8K_store_record(qv, dv, recs + (size_t) sb * rec_bytes(false, NT), t, NT, lane, perm);
}

// residual add + RMSNorm fused with the activation quantizer of the GEMM that consumes y (a fused GEMM
// prologue): CTA t < N: x += delta; y = x / sqrt(mean(x^2) + eps) * w (as add_rms_norm); the row of y is staged in
// shared memory and each warp quantizes super-blocks of it into the GEMM's activation records exactly as
// quant_q8K_kernel does (same functions); CTAs N..NT-1 write the zero padding rows; CTA 0 zeroes the split-K counters.
// add_rms_norm_ar_q8K_kernel below is the form whose delta is the tensor-parallel all-reduce of the ranks' partial
// rows (the flag-in-word exchange and the rank-order sum of allreduce.cuh, as add_rms_norm_ar_kernel does):
// all-reduce, residual add, norm and the next GEMM's activation records in one kernel.
struct NormAr {
    const uint64_t * peers;  // null: no all-reduce
    int              world, rank, slot;
    uint32_t *       epochs;
    int32_t *        status;
};

constexpr int kNormQThreads = 1024;
__global__ void __launch_bounds__(kNormQThreads) add_rms_norm_q8K_kernel(float * x, const float * delta,
                                                                          const float * w, float eps, float * y,
                                                                          int N, int64_t d, int NT, uint8_t * recs,
                                                                          int perm, int32_t * cnt, int ncnt) {
    pdl_launch_dependents();
    pdl_wait();
    extern __shared__ float ys[];
    const int     t  = blockIdx.x;
    const int64_t d4 = d >> 2;
    if (blockIdx.x == 0) {
        for (int i = threadIdx.x; i < ncnt; i += blockDim.x) cnt[i] = 0;
    }
    if (t < N) {
        float * xr = x + (int64_t) t * d;
        float   ss = 0.0f;
        float4  v[4];
#pragma unroll
        for (int k = 0; k < 4; k++) {
            const int64_t j = threadIdx.x + (int64_t) k * kNormQThreads;
            if (j < d4) {
                float4 a = reinterpret_cast<const float4 *>(xr)[j];
                if (delta) {
                    const float4 b = reinterpret_cast<const float4 *>(delta + (int64_t) t * d)[j];
                    a.x += b.x; a.y += b.y; a.z += b.z; a.w += b.w;
                    reinterpret_cast<float4 *>(xr)[j] = a;
                }
                v[k] = a;
                ss = fmaf(a.x, a.x, fmaf(a.y, a.y, fmaf(a.z, a.z, fmaf(a.w, a.w, ss))));
            }
        }
        __shared__ float part[32];
#pragma unroll
        for (int o = 16; o > 0; o >>= 1) ss += __shfl_xor_sync(0xffffffffu, ss, o);
        if ((threadIdx.x & 31) == 0) part[threadIdx.x >> 5] = ss;
        __syncthreads();
        if (threadIdx.x < 32) {
            ss = part[threadIdx.x];
#pragma unroll
            for (int o = 16; o > 0; o >>= 1) ss += __shfl_xor_sync(0xffffffffu, ss, o);
            if (threadIdx.x == 0) part[0] = ss;
        }
        __syncthreads();
        const float scale = 1.0f / sqrtf(part[0] / (float) d + eps);
#pragma unroll
        for (int k = 0; k < 4; k++) {
            const int64_t j = threadIdx.x + (int64_t) k * kNormQThreads;
            if (j < d4) {
                const float4 ww = reinterpret_cast<const float4 *>(w)[j];
                float4       o;
                o.x = v[k].x * scale * ww.x;
                o.y = v[k].y * scale * ww.y;
                o.z = v[k].z * scale * ww.z;
                o.w = v[k].w * scale * ww.w;
                reinterpret_cast<float4 *>(y + (int64_t) t * d)[j] = o;
                reinterpret_cast<float4 *>(ys)[j] = o;
            }
        }
    } else {
        for (int64_t j = threadIdx.x; j < d4; j += kNormQThreads) reinterpret_cast<float4 *>(ys)[j] = make_float4(0, 0, 0, 0);
    }
    __syncthreads();
    const int lane = threadIdx.x & 31, warp = threadIdx.x >> 5;
    const int nsb  = (int) (d / QK);
    for (int sb = warp; sb < nsb; sb += kNormQThreads / 32) {
        float v8[8];
        const float4 a = reinterpret_cast<const float4 *>(ys + (int64_t) sb * QK + 8 * lane)[0];
        const float4 b = reinterpret_cast<const float4 *>(ys + (int64_t) sb * QK + 8 * lane)[1];
        v8[0] = a.x; v8[1] = a.y; v8[2] = a.z; v8[3] = a.w; v8[4] = b.x; v8[5] = b.y; v8[6] = b.z; v8[7] = b.w;
        int   qv[8];
        float dv;
        q8K_quantize_warp(v8, lane, qv, dv);
        q8K_store_record(qv, dv, recs + (size_t) sb * rec_bytes(false, NT), t, NT, lane, perm);
    }
}

// The all-reduce form of add_rms_norm_q8K_kernel, spread over a cluster of kArC CTAs per token row, so that the
// exchange's stores to the peers and the loads of the receive area run on kArC SMs per row instead of one (a rank
// sends (world - 1) x d x 8 bytes per row). CTA c of row t handles the float4 columns 128 c + v + 1024 k (thread v,
// k = 0..3): the columns thread 128 c + v of the one-CTA kernel handles. So each warp is a warp of that kernel, and
// the sum of squares is reduced in the same order (each thread's chain, the warp's butterfly, then one butterfly over
// the 32 warp partials gathered over distributed shared memory): the rows are bit-identical to the one-CTA kernel's.
// The super-blocks of y that a CTA quantizes (2 c + 16 k, + 1) lie inside its own columns. Every CTA reads the row's
// epoch; CTA 0 advances it after the cluster's last barrier. Rows N..NT-1 write the zero padding records.
constexpr int kArC  = 8;
constexpr int kArCT = 128;
__global__ void __cluster_dims__(kArC, 1, 1) __launch_bounds__(kArCT)
    add_rms_norm_ar_q8K_kernel(float * x, const float * w, float eps, float * y, int N, int64_t d, int NT,
                               uint8_t * recs, int perm, int32_t * cnt, int ncnt, const NormAr ar) {
    pdl_launch_dependents();
    pdl_wait();  // this rank's GEMM has written its partial rows
    __shared__ float4   ys[4 * kArCT];  // this CTA's columns of y: [k][v]
    __shared__ float    part[kArCT / 32];
    __shared__ float    tot_s;
    __shared__ uint32_t e_s;
    const int     c = blockIdx.x, t = blockIdx.y, tid = threadIdx.x, lane = tid & 31, warp = tid >> 5;
    const int64_t d4   = d >> 2;
    const bool    real = t < N;
    if (c == 0 && t == 0) {
        for (int i = tid; i < ncnt; i += kArCT) cnt[i] = 0;
    }
    float    ss = 0.0f;
    float4   v[4];
    uint32_t e  = 0;
    if (real) {
        if (tid == 0) e_s = __ldcg(&ar.epochs[ar.slot * kArRows + t]) + 1u;
        __syncthreads();
        e = e_s;
        {  // send this rank's values of the CTA's columns to every rank (ar_push4, all columns per rank in turn)
            const float4 * mine = reinterpret_cast<const float4 *>(ar.peers[ar.rank] + (size_t) ar.slot * ar_part_bytes(d)) +
                                  (int64_t) t * d4;
            float4 pv[4];
#pragma unroll
            for (int k = 0; k < 4; k++) {
                const int64_t j = kArCT * c + tid + (int64_t) k * 1024;
                if (j < d4) pv[k] = mine[j];
            }
            const size_t o = ar_recv_word(d, ar.slot, t, ar.rank);
            for (int r = 0; r < ar.world; r++) {
                uint8_t * q = reinterpret_cast<uint8_t *>(ar.peers[r] + o);
#pragma unroll
                for (int k = 0; k < 4; k++) {
                    const int64_t j = kArCT * c + tid + (int64_t) k * 1024;
                    if (j < d4) {
                        st_relaxed_sys_v2(q + j * 32, ll_word(pv[k].x, e), ll_word(pv[k].y, e));
                        st_relaxed_sys_v2(q + j * 32 + 16, ll_word(pv[k].z, e), ll_word(pv[k].w, e));
                    }
                }
            }
        }
        float *        xr = x + (int64_t) t * d;
        bool           ok = true;
        const uint64_t t0 = globaltimer_ns();
#pragma unroll
        for (int k = 0; k < 4; k++) {
            const int64_t j = kArCT * c + tid + (int64_t) k * 1024;
            if (j < d4) {
                float4 a = reinterpret_cast<const float4 *>(xr)[j];
                ar_gather4(a, ar.peers, ar.world, ar.rank, ar.slot, t, d, j, e, t0, ok, ar.status);
                reinterpret_cast<float4 *>(xr)[j] = a;
                v[k] = a;
                ss = fmaf(a.x, a.x, fmaf(a.y, a.y, fmaf(a.z, a.z, fmaf(a.w, a.w, ss))));
            }
        }
    }
#pragma unroll
    for (int o = 16; o > 0; o >>= 1) ss += __shfl_xor_sync(0xffffffffu, ss, o);
    if (lane == 0) part[warp] = ss;
    cluster_sync_all();  // every CTA's warp partials are written
    if (warp == 0) {
        // lane l: the partial of warp l of the one-CTA kernel = warp l % 4 of cluster CTA l / 4
        float p = ld_dsmem_f32(mapa_shared(smem_u32(&part[lane & 3]), (uint32_t) (lane >> 2)));
#pragma unroll
        for (int o = 16; o > 0; o >>= 1) p += __shfl_xor_sync(0xffffffffu, p, o);
        if (lane == 0) tot_s = p;
    }
    __syncthreads();
    const float scale = 1.0f / sqrtf(tot_s / (float) d + eps);
#pragma unroll
    for (int k = 0; k < 4; k++) {
        const int64_t j = kArCT * c + tid + (int64_t) k * 1024;
        float4        o = make_float4(0, 0, 0, 0);
        if (real && j < d4) {
            const float4 ww = reinterpret_cast<const float4 *>(w)[j];
            o.x = v[k].x * scale * ww.x;
            o.y = v[k].y * scale * ww.y;
            o.z = v[k].z * scale * ww.z;
            o.w = v[k].w * scale * ww.w;
            reinterpret_cast<float4 *>(y + (int64_t) t * d)[j] = o;
        }
        ys[k * kArCT + tid] = o;
    }
    __syncthreads();
    const int nsb = (int) (d / QK);
    for (int q = warp; q < 8; q += kArCT / 32) {  // the CTA's super-blocks: 2 c + 16 k + h, q = 2 k + h
        const int k = q >> 1, h = q & 1, sb = 2 * c + 16 * k + h;
        if (sb >= nsb) continue;
        const float * src = reinterpret_cast<const float *>(ys + k * kArCT + h * 64) + 8 * lane;
        const float4  a   = reinterpret_cast<const float4 *>(src)[0];
        const float4  b   = reinterpret_cast<const float4 *>(src)[1];
        float         v8[8];
        v8[0] = a.x; v8[1] = a.y; v8[2] = a.z; v8[3] = a.w; v8[4] = b.x; v8[5] = b.y; v8[6] = b.z; v8[7] = b.w;
        int   qv[8];
        float dv;
        q8K_quantize_warp(v8, lane, qv, dv);
        q8K_store_record(qv, dv, recs + (size_t) sb * rec_bytes(false, NT), t, NT, lane, perm);
    }
    cluster_sync_all();  // no CTA exits while a peer may read its partials; every CTA has read the epoch
    if (real && c == 0 && tid == 0) ar.epochs[ar.slot * kArRows + t] = e;
}

// q8_0 quantizer, per 32 columns (4 lanes per block): d = amax / 127 stored as f16. SIMD mode: id = 127 / amax,
// q = round_half_even(x * id); REF mode: id = 1 / d (f32 d), q = roundf(x * id).
// q8_0 quantization of one warp's 256 values (lane l holds columns 8l..8l+7: 32-block l / 4) with the context's
// q8_0 mode; returns the codes packed and the block's f16 scale
__device__ __forceinline__ uint2 q80_quantize_warp(const float (&v)[8], int mode, __half & dh) {
    float amax = 0.0f;
#pragma unroll
    for (int j = 0; j < 8; j++) amax = fmaxf(amax, fabsf(v[j]));
    amax = fmaxf(amax, __shfl_xor_sync(0xffffffffu, amax, 1));
    amax = fmaxf(amax, __shfl_xor_sync(0xffffffffu, amax, 2));
    const float dd = __fdiv_rn(amax, 127.0f);
    dh             = __float2half_rn(dd);
    int qv[8];
    if (mode == SRHPM_Q8_0_ACT_SIMD) {
        const float id = amax != 0.0f ? __fdiv_rn(127.0f, amax) : 0.0f;
#pragma unroll
        for (int j = 0; j < 8; j++) qv[j] = __float2int_rn(__fmul_rn(v[j], id));
    } else {
        const float id = dd != 0.0f ? __fdiv_rn(1.0f, dd) : 0.0f;
#pragma unroll
        for (int j = 0; j < 8; j++) qv[j] = (int) roundf(__fmul_rn(v[j], id));
    }
    return pack8(qv);
}

// token row t of one super-block's q8_0 activation record: the codes, then the 8 block scales at [blk * NT + t]
__device__ __forceinline__ void q80_store_record(uint2 pk, __half dh, uint8_t * rec, int t, int NT, int lane) {
    *reinterpret_cast<uint2 *>(rec + t * kTokStride + 8 * lane) = pk;
    if ((lane & 3) == 0) reinterpret_cast<float *>(rec + NT * kTokStride)[(lane >> 2) * NT + t] = __half2float(dh);
}

template <bool DENSE>
__global__ void __launch_bounds__(256) quant_q80_kernel(const float * __restrict__ X, int64_t ldx, int N, int nsb,
                                                         int NT, int mode, uint8_t * __restrict__ recs,
                                                         uint8_t * __restrict__ blocks, int32_t * __restrict__ cnt,
                                                         int ncnt) {
    // launched early behind the previous call's GEMM: let the next GEMM get resident, then wait for the previous
    // grid (it may still read the records and counters this kernel rewrites, or write the X it reads)
    pdl_launch_dependents();
    prefetch_act_l2(X, ldx, N, nsb, N, threadIdx.x & 31);
    pdl_wait();
    for (int i = blockIdx.x * blockDim.x + threadIdx.x; i < ncnt; i += gridDim.x * blockDim.x) cnt[i] = 0;
    const int     lane = threadIdx.x & 31;
    const int     TT   = N;  // records: the padding token rows are never read into a stored output
    const int64_t wid  = (int64_t) blockIdx.x * 8 + (threadIdx.x >> 5);
    if (wid >= (int64_t) nsb * TT) {
        return;
    }
    const int sb = (int) (wid / TT), t = (int) (wid % TT);
    float     v[8];
    if (t < N) {
        load8(X + (int64_t) t * ldx + (int64_t) sb * QK + 8 * lane, v);
    } else {
#pragma unroll
        for (int j = 0; j < 8; j++) v[j] = 0.0f;
    }
    __half      dh;
    const uint2 pk  = q80_quantize_warp(v, mode, dh);
    const int   blk = lane >> 2;  // 32-block inside the super-block
    if constexpr (DENSE) {
        const int64_t nb32 = (int64_t) nsb * 8;
        uint8_t *     out  = blocks + ((int64_t) t * nb32 + (int64_t) sb * 8 + blk) * 34;
        if ((lane & 3) == 0) *reinterpret_cast<__half *>(out) = dh;
        uint16_t * qs = reinterpret_cast<uint16_t *>(out + 2 + 8 * (lane & 3));
        qs[0] = (uint16_t) (pk.x & 0xffff);
        qs[1] = (uint16_t) (pk.x >> 16);
        qs[2] = (uint16_t) (pk.y & 0xffff);
        qs[3] = (uint16_t) (pk.y >> 16);
    } else {
        q80_store_record(pk, dh, recs + (size_t) sb * rec_bytes(true, NT), t, NT, lane);
    }
}

// ---------------------------------------------------------------------------------------------------------------
// per-type super-block decoders
//
// prep(): one lane unpacks the scales of one (row, super-block) into a "scale record" in shared memory (integer block
//         scales as int32, Q4_K/Q5_K mins replicated over the 4 bytes of an MMA operand word, f32 super-block
//         scales), so the four lanes that share a row read them instead of each unpacking them again.
// sb():   consumes one super-block of rows (g, g+8) of the warp's 16-row slice: wa / wb point at the two rows'
//         blocks in shared memory, ra / rb at their scale records, xr at the super-block's activation record.

__device__ __forceinline__ uint32_t lds32(const uint8_t * p) { return *reinterpret_cast<const uint32_t *>(p); }
__device__ __forceinline__ uint2    lds64(const uint8_t * p) { return *reinterpret_cast<const uint2 *>(p); }
__device__ __forceinline__ int4     lds128i(const uint8_t * p) { return *reinterpret_cast<const int4 *>(p); }
__device__ __forceinline__ float    ldh(const uint8_t * p) { return half_bits_to_float(lds_u16(p)); }

__device__ __forceinline__ uint32_t prmt(uint32_t a, uint32_t b, uint32_t sel) {
    uint32_t r;
    asm("prmt.b32 %0, %1, %2, %3;" : "=r"(r) : "r"(a), "r"(b), "r"(sel));
    return r;
}
__device__ __forceinline__ int ubyte(uint32_t w, int j) { return (int) __byte_perm(w, 0u, 0x4440u | (uint32_t) j); }
__device__ __forceinline__ int sbyte(uint32_t w, int j) { return ((int32_t) (w << (24 - 8 * j))) >> 24; }

// per-byte a - k for bytes holding 0..127 (no borrow between bytes)
__device__ __forceinline__ uint32_t vsub_small(uint32_t a, uint32_t k) { return ((a | 0x80808080u) - k) ^ 0x80808080u; }

__device__ __forceinline__ int sel4(const int4 & v, int j) { return j == 0 ? v.x : j == 1 ? v.y : j == 2 ? v.z : v.w; }

struct DbgOut {
    int32_t * isum;
    int32_t * imin;
    int64_t   rows;
    int       N;
    int       nblk;
};

template <int NG>
__device__ __forceinline__ void dbg_store(const DbgOut & o, const int (&v)[NG][4], bool is_min, int64_t rg, int blk,
                                          int lane) {
    int32_t * dst = is_min ? o.imin : o.isum;
    if (!dst) return;
    const int t = lane & 3;
#pragma unroll
    for (int grp = 0; grp < NG; grp++) {
#pragma unroll
        for (int e = 0; e < 4; e++) {
            const int     tok = 8 * grp + 2 * t + (e & 1);
            const int64_t row = e < 2 ? rg : rg + 8;
            if (tok < o.N && row < o.rows) dst[((int64_t) tok * o.rows + row) * o.nblk + blk] = v[grp][e];
        }
    }
}

template <int NG>
__device__ __forceinline__ void zero(int (&v)[NG][4]) {
#pragma unroll
    for (int grp = 0; grp < NG; grp++) v[grp][0] = v[grp][1] = v[grp][2] = v[grp][3] = 0;
}

// f32 update of one super-block: acc += (d_row * x_tok) * isum  [- (dmin_row * x_tok) * imin], in f32 pairs (the
// two tokens of a thread: one f32x2 multiply and one f32x2 fused multiply-add per row, each lane rounded as the
// scalar pair would be)
template <int NG, bool MIN>
__device__ __forceinline__ void sb_update(float (&acc)[NG][4], const int (&im)[NG][4], const int (&in)[NG][4],
                                          float dA, float dB, float mA, float mB, const float * xs, int t) {
#pragma unroll
    for (int grp = 0; grp < NG; grp++) {
        const float2 x  = *reinterpret_cast<const float2 *>(xs + 8 * grp + 2 * t);
        const f2     xx = f2_pack(x.x, x.y);
        f2           a01 = f2_pack(acc[grp][0], acc[grp][1]), a23 = f2_pack(acc[grp][2], acc[grp][3]);
        a01 = f2_fma(f2_mul(f2_pack(dA, dA), xx), f2_pack((float) im[grp][0], (float) im[grp][1]), a01);
        a23 = f2_fma(f2_mul(f2_pack(dB, dB), xx), f2_pack((float) im[grp][2], (float) im[grp][3]), a23);
        if constexpr (MIN) {
            a01 = f2_fma(f2_mul(f2_pack(-mA, -mA), xx), f2_pack((float) in[grp][0], (float) in[grp][1]), a01);
            a23 = f2_fma(f2_mul(f2_pack(-mB, -mB), xx), f2_pack((float) in[grp][2], (float) in[grp][3]), a23);
        }
        f2_unpack(a01, acc[grp][0], acc[grp][1]);
        f2_unpack(a23, acc[grp][2], acc[grp][3]);
    }
}

// im += sA * c[0..1] (row g), sB * c[2..3] (row g + 8)
template <int NG>
__device__ __forceinline__ void scale_acc(int (&im)[NG][4], int grp, int sA, int sB, const int (&c)[4]) {
    im[grp][0] += sA * c[0];
    im[grp][1] += sA * c[1];
    im[grp][2] += sB * c[2];
    im[grp][3] += sB * c[3];
}

// Q4_K / Q5_K minimum term of one super-block through one MMA pair over k = sub-block index: A = the 8 6-bit mins
// of each row (thread t = 0 holds sub-blocks 0..3, t = 1 holds 4..7, others zero), B = the per-sub-block activation
// sums split as s = 128 hi + lo (int8 each, from the record's padding). Returns sum_b m_b * s_b.
template <int NG>
__device__ __forceinline__ void mins_mma(int (&in)[NG][4], uint32_t mlA, uint32_t mhA, uint32_t mlB, uint32_t mhB,
                                         const uint8_t * xr, int lane) {
    const int      t  = lane & 3, g = lane >> 2;
    const uint32_t a0 = t == 0 ? mlA : t == 1 ? mhA : 0u;
    const uint32_t a1 = t == 0 ? mlB : t == 1 ? mhB : 0u;
#pragma unroll
    for (int grp = 0; grp < NG; grp++) {
        const uint8_t * tok = xr + (8 * grp + g) * kTokStride;
        const uint32_t  bh  = t < 2 ? lds32(tok + 256 + 4 * t) : 0u;
        const uint32_t  bl  = t < 2 ? lds32(tok + 264 + 4 * t) : 0u;
        int             ch[4], cl[4];
        mma_k32_z<true>(ch, a0, a1, 0u, 0u, bh, 0u);
        mma_k32_z<true>(cl, a0, a1, 0u, 0u, bl, 0u);
#pragma unroll
        for (int e = 0; e < 4; e++) in[grp][e] = ch[e] * 128 + cl[e];
    }
}

// Q4_K (144 B: d, dmin, 12 bytes of 6-bit scales/mins, 128 bytes of nibbles) and Q5_K (176 B: + 32 bytes of 5th
// bits before the nibbles). Pair p of sub-blocks (2p, 2p+1) shares 32 code bytes: low nibble = sub-block 2p, high
// nibble = sub-block 2p+1; the 5th bit of sub-block b, weight l is bit b of qh[l]. Thread t holds weights 8t..8t+7
// of each sub-block (one 8-byte load per row and pair). Q4_K feeds the high nibbles unshifted (16 x the code) into
// the MMA and divides that accumulator by 16 once per super-block (exact: every term is a multiple of 16).
// Scale record: int32 sc[8] | the 8 mins as bytes (2 words) | f32 d, dmin.
template <bool Q5>
struct DecK45 {
    static constexpr int  BS   = Q5 ? 176 : 144;
    static constexpr int  KC   = 2;
    static constexpr int  RECB = 48;
    static constexpr bool Q80  = false;
    static constexpr int  MINB = 2;  // resident CTAs per SM the kernel is compiled for
    static constexpr int  QS   = Q5 ? 48 : 16;

    __device__ __forceinline__ static void prep(const uint8_t * blk, uint8_t * rec) {
        const uint32_t s0 = lds32(blk + 4), s1 = lds32(blk + 8), s2 = lds32(blk + 12);
        const uint32_t sl = s0 & 0x3F3F3F3Fu, sh = (s2 & 0x0F0F0F0Fu) | ((s0 >> 2) & 0x30303030u);
        const uint32_t ml = s1 & 0x3F3F3F3Fu, mh = ((s2 >> 4) & 0x0F0F0F0Fu) | ((s1 >> 2) & 0x30303030u);
        int4 * ri = reinterpret_cast<int4 *>(rec);
        ri[0]     = make_int4(ubyte(sl, 0), ubyte(sl, 1), ubyte(sl, 2), ubyte(sl, 3));
        ri[1]     = make_int4(ubyte(sh, 0), ubyte(sh, 1), ubyte(sh, 2), ubyte(sh, 3));
        const float2 dd = make_float2(ldh(blk), ldh(blk + 2));
        ri[2] = make_int4((int) ml, (int) mh, __float_as_int(dd.x), __float_as_int(dd.y));
    }

    __device__ __forceinline__ static uint32_t hbit(uint32_t qh, int b) { return ((qh >> b) << 4) & 0x10101010u; }

    template <int NG, bool DBG>
    __device__ __forceinline__ static void sb(const uint8_t * wa, const uint8_t * wb, const uint8_t * ra,
                                              const uint8_t * rb, const uint8_t * xr, int lane, float (&acc)[NG][4],
                                              const DbgOut & dbg, int64_t rg, int sbi) {
        constexpr int NT = 8 * NG;
        const int     t = lane & 3, g = lane >> 2;
        const int4    scA[2] = { lds128i(ra), lds128i(ra + 16) }, scB[2] = { lds128i(rb), lds128i(rb + 16) };
        const int4    tA = lds128i(ra + 32), tB = lds128i(rb + 32);  // mins (2 words), d, dmin
        uint2         ha = make_uint2(0, 0), hb = make_uint2(0, 0);
        if constexpr (Q5) {
            ha = lds64(wa + 16 + 8 * t);
            hb = lds64(wb + 16 + 8 * t);
        }
        int im[NG][4], ih[NG][4], in[NG][4];
        zero<NG>(im);
        zero<NG>(ih);
        mins_mma<NG>(in, (uint32_t) tA.x, (uint32_t) tA.y, (uint32_t) tB.x, (uint32_t) tB.y, xr, lane);
#pragma unroll
        for (int p = 0; p < 4; p++) {
            const uint2 va = lds64(wa + QS + 32 * p + 8 * t);
            const uint2 vb = lds64(wb + QS + 32 * p + 8 * t);
#pragma unroll
            for (int h = 0; h < 2; h++) {
                const int b = 2 * p + h;
                uint32_t  a0, a1, a2, a3;
                if constexpr (Q5) {
                    a0 = ((va.x >> (4 * h)) & 0x0F0F0F0Fu) | hbit(ha.x, b);
                    a2 = ((va.y >> (4 * h)) & 0x0F0F0F0Fu) | hbit(ha.y, b);
                    a1 = ((vb.x >> (4 * h)) & 0x0F0F0F0Fu) | hbit(hb.x, b);
                    a3 = ((vb.y >> (4 * h)) & 0x0F0F0F0Fu) | hbit(hb.y, b);
                } else {
                    const uint32_t m = h ? 0xF0F0F0F0u : 0x0F0F0F0Fu;
                    a0 = va.x & m;
                    a2 = va.y & m;
                    a1 = vb.x & m;
                    a3 = vb.y & m;
                }
                const int sA = sel4(scA[b >> 2], b & 3), sB = sel4(scB[b >> 2], b & 3);
#pragma unroll
                for (int grp = 0; grp < NG; grp++) {
                    const uint2 x = lds64(xr + (8 * grp + g) * kTokStride + 32 * b + 8 * t);
                    int         c[4];
                    mma_k32_z<true>(c, a0, a1, a2, a3, x.x, x.y);
                    if (!Q5 && h) {
                        scale_acc<NG>(ih, grp, sA, sB, c);
                    } else {
                        scale_acc<NG>(im, grp, sA, sB, c);
                    }
                }
            }
        }
        if constexpr (!Q5) {
#pragma unroll
            for (int grp = 0; grp < NG; grp++) {
#pragma unroll
                for (int e = 0; e < 4; e++) im[grp][e] += ih[grp][e] >> 4;
            }
        }
        if constexpr (DBG) {
            dbg_store<NG>(dbg, im, false, rg, sbi, lane);
            dbg_store<NG>(dbg, in, true, rg, sbi, lane);
        } else {
            const float * xs = reinterpret_cast<const float *>(xr + NT * kTokStride);
            sb_update<NG, true>(acc, im, in, __int_as_float(tA.z), __int_as_float(tB.z), __int_as_float(tA.w),
                                __int_as_float(tB.w), xs, t);
        }
    }
};

// Q6_K (210 B: 128 bytes low nibbles, 64 bytes of 2-bit highs, 16 int8 scales per 16 weights, d). Weight
// 128n + 32j + l: nibble (j >> 1) of ql[64n + 32(j & 1) + l], bits 2j of qh[32n + l], minus 32; scale 8n + 2j + l/16.
// One k16 MMA per 16-weight group. Scale record: int32 sc[16] | f32 d.
struct DecQ6K {
    static constexpr int  BS   = 210;
    static constexpr int  KC   = 1;
    static constexpr int  RECB = 80;
    static constexpr bool Q80  = false;
    static constexpr int  MINB = 4;  // resident CTAs per SM the kernel is compiled for (measured: 4 beats 2 here)

    __device__ __forceinline__ static void prep(const uint8_t * blk, uint8_t * rec) {
        int4 *         ri = reinterpret_cast<int4 *>(rec);
        const uint32_t a = smem_u32(blk + 192), b = a & ~3u, sh = (a & 3u) * 8;
        uint32_t       wd[5];
#pragma unroll
        for (int i = 0; i < 5; i++) wd[i] = sld32(b + 4 * i);
#pragma unroll
        for (int i = 0; i < 4; i++) {
            const uint32_t w = __funnelshift_r(wd[i], wd[i + 1], sh);
            ri[i]            = make_int4(sbyte(w, 0), sbyte(w, 1), sbyte(w, 2), sbyte(w, 3));
        }
        *reinterpret_cast<float *>(rec + 64) = ldh(blk + 208);
    }

    template <int NG, bool DBG, bool A4>
    __device__ __forceinline__ static void sb_impl(uint32_t pa, uint32_t pb, const uint8_t * ra, const uint8_t * rb,
                                                   const uint8_t * xr, int lane, float (&acc)[NG][4],
                                                   const DbgOut & dbg, int64_t rg, int sbi) {
        constexpr int NT = 8 * NG;
        const int     t = lane & 3, g = lane >> 2;
        int           im[NG][4], in[NG][4];
        zero<NG>(im);
        zero<NG>(in);
#pragma unroll
        for (int n = 0; n < 2; n++) {
            const int4 sA4[2] = { lds128i(ra + 32 * n), lds128i(ra + 32 * n + 16) };
            const int4 sB4[2] = { lds128i(rb + 32 * n), lds128i(rb + 32 * n + 16) };
#pragma unroll
            for (int h = 0; h < 2; h++) {
                const int      off = 16 * h + 4 * t;
                const uint32_t l0a = sld4_a2<A4>(pa + 64 * n + off), l1a = sld4_a2<A4>(pa + 64 * n + 32 + off);
                const uint32_t l0b = sld4_a2<A4>(pb + 64 * n + off), l1b = sld4_a2<A4>(pb + 64 * n + 32 + off);
                const uint32_t qha = sld4_a2<A4>(pa + 128 + 32 * n + off), qhb = sld4_a2<A4>(pb + 128 + 32 * n + off);
#pragma unroll
                for (int j = 0; j < 4; j++) {
                    const uint32_t la = (j & 1) ? l1a : l0a, lb = (j & 1) ? l1b : l0b;
                    const int      sh = 4 * (j >> 1);
                    const uint32_t ua = vsub_small(((la >> sh) & 0x0F0F0F0Fu) | (((qha >> (2 * j)) & 0x03030303u) << 4),
                                                   0x20202020u);
                    const uint32_t ub = vsub_small(((lb >> sh) & 0x0F0F0F0Fu) | (((qhb >> (2 * j)) & 0x03030303u) << 4),
                                                   0x20202020u);
                    const int is = 2 * j + h;  // scale index within this half
                    const int sA = sel4(sA4[is >> 2], is & 3), sB = sel4(sB4[is >> 2], is & 3);
                    const int b  = 4 * n + j;
#pragma unroll
                    for (int grp = 0; grp < NG; grp++) {
                        const uint32_t x    = lds32(xr + (8 * grp + g) * kTokStride + 32 * b + off);
                        int            c[4];
                        mma_k16_z<false>(c, ua, ub, x);
                        scale_acc<NG>(im, grp, sA, sB, c);
                    }
                }
            }
        }
        if constexpr (DBG) {
            dbg_store<NG>(dbg, im, false, rg, sbi, lane);
        } else {
            const float * xs = reinterpret_cast<const float *>(xr + NT * kTokStride);
            sb_update<NG, false>(acc, im, in, *reinterpret_cast<const float *>(ra + 64),
                                 *reinterpret_cast<const float *>(rb + 64), 0.f, 0.f, xs, t);
        }
    }

    template <int NG, bool DBG>
    __device__ __forceinline__ static void sb(const uint8_t * wa, const uint8_t * wb, const uint8_t * ra,
                                              const uint8_t * rb, const uint8_t * xr, int lane, float (&acc)[NG][4],
                                              const DbgOut & dbg, int64_t rg, int sbi) {
        // the choice must be warp-uniform: sb_impl issues mma.sync (rows of one warp can differ in alignment)
        const uint32_t pa = smem_u32(wa), pb = smem_u32(wb);
        if (__all_sync(0xffffffffu, ((pa | pb) & 3u) == 0)) {
            sb_impl<NG, DBG, true>(pa, pb, ra, rb, xr, lane, acc, dbg, rg, sbi);
        } else {
            sb_impl<NG, DBG, false>(pa, pb, ra, rb, xr, lane, acc, dbg, rg, sbi);
        }
    }
};

// Q3_K (110 B: 32 bytes of high bits, 64 bytes of 2-bit codes, 12 bytes of 6-bit scales, d). Weight 128n + 32j + l:
// code c = bits 2j of qs[32n + l], high bit hb = bit (4n + j) of hmask[l] (set = +0, clear = -4), so q = i - 4 with
// the 3-bit index i = c + 4 hb; scale s = 6 bits - 32 at index 8n + 2j + l/16.
//
// Every weight goes into the MMA already scaled, as the unsigned byte 128 - s q (s q in [-124, 128]): one prmt per 4
// weights looks the indices up in the sub-block's 8-entry table, so a super-block is 8 k32 MMAs per row pair with the
// sub-block scales inside, and the exact integer sum is recovered as sum s q x = 128 sum x - sum (128 - s q) x with
// the token's code sum from the activation record.
// Thread t takes l = 8t..8t+7 (one sub-block half h = t / 2) of every (n, j); two 32-bit words per 8 bytes of qs and
// hmask are spread into nibble indices (nibble 2k: l = 8t + k, nibble 2k + 1: l = 8t + 4 + k), so its A registers
// hold l = 8t + {0,4,1,5} and 8t + {2,6,3,7} -- the order in which the quantizer stores Q3_K activation records.
// Scale record: 16 tables of 8 bytes, [h][n][j] | f32 d. Table of scale u = s + 32 (entry i = 128 - s (i - 4)):
// bytes 0-3 = u * 0x01020304 + 0x60402000, bytes 4-7 = 0xE0C0A080 - u * 0x03020100 (no byte leaves 0..255).
struct DecQ3K {
    static constexpr int  BS   = 110;
    static constexpr int  KC   = 2;
    static constexpr int  RECB = 144;
    static constexpr bool Q80  = false;
    static constexpr int  MINB = 2;  // resident CTAs per SM the kernel is compiled for

    __device__ __forceinline__ static void prep(const uint8_t * blk, uint8_t * rec) {
        const uint32_t a  = smem_u32(blk + 96);
        const uint32_t b  = a & ~3u, sh = (a & 3u) * 8;
        const uint32_t w0 = sld32(b), w1 = sld32(b + 4), w2 = sld32(b + 8), w3 = sld32(b + 12);
        const uint32_t s0 = __funnelshift_r(w0, w1, sh), s1 = __funnelshift_r(w1, w2, sh);
        const uint32_t s2 = __funnelshift_r(w2, w3, sh);
        uint32_t       w[4];  // byte k of w[i] = u of scale index 4i + k
        w[0] = (s0 & 0x0F0F0F0Fu) | ((s2 << 4) & 0x30303030u);
        w[1] = (s1 & 0x0F0F0F0Fu) | ((s2 << 2) & 0x30303030u);
        w[2] = ((s0 >> 4) & 0x0F0F0F0Fu) | (s2 & 0x30303030u);
        w[3] = ((s1 >> 4) & 0x0F0F0F0Fu) | ((s2 >> 2) & 0x30303030u);
        uint4 * rt = reinterpret_cast<uint4 *>(rec);
#pragma unroll
        for (int h = 0; h < 2; h++) {
#pragma unroll
            for (int n = 0; n < 2; n++) {
#pragma unroll
                for (int jp = 0; jp < 2; jp++) {  // tables j = 2 jp, 2 jp + 1: scale indices 8n + 4jp + h, + 2
                    const uint32_t u0 = __byte_perm(w[2 * n + jp], 0u, 0x4440u | (uint32_t) h);
                    const uint32_t u1 = __byte_perm(w[2 * n + jp], 0u, 0x4440u | (uint32_t) (2 + h));
                    rt[4 * h + 2 * n + jp] = make_uint4(u0 * 0x01020304u + 0x60402000u, 0xE0C0A080u - u0 * 0x03020100u,
                                                        u1 * 0x01020304u + 0x60402000u, 0xE0C0A080u - u1 * 0x03020100u);
                }
            }
        }
        *reinterpret_cast<float *>(rec + 128) = half_bits_to_float((uint16_t) __funnelshift_r(w3, w3, sh));
    }

    // the four selectors (j = 0..3) of one row and half n from its qs words q0 (l = 8t..8t+3), q1 (8t+4..8t+7) and
    // hmask words h0, h1: nibble = c | hb << 2, bit 3 clear
    __device__ __forceinline__ static void selectors(uint32_t q0, uint32_t q1, uint32_t h0, uint32_t h1, int n,
                                                     uint32_t (&y)[4]) {
        const uint32_t elo = (q0 & 0x0F0F0F0Fu) | ((q1 << 4) & 0xF0F0F0F0u);   // c0 c1 per nibble pair
        const uint32_t ehi = ((q0 >> 4) & 0x0F0F0F0Fu) | (q1 & 0xF0F0F0F0u);   // c2 c3
        const uint32_t f   = n == 0 ? (h0 & 0x0F0F0F0Fu) | ((h1 << 4) & 0xF0F0F0F0u)
                                    : ((h0 >> 4) & 0x0F0F0F0Fu) | (h1 & 0xF0F0F0F0u);  // hb of j = 0..3 per nibble
        const uint32_t f02 = f & 0x55555555u, f13 = (f >> 1) & 0x55555555u;
        y[0] = (elo & 0x33333333u) | ((f02 << 2) & 0xCCCCCCCCu);
        y[1] = ((elo >> 2) & 0x33333333u) | ((f13 << 2) & 0xCCCCCCCCu);
        y[2] = (ehi & 0x33333333u) | (f02 & 0xCCCCCCCCu);
        y[3] = ((ehi >> 2) & 0x33333333u) | (f13 & 0xCCCCCCCCu);
    }

    // pa, pb: the rows' byte 8t rounded down to 4 bytes (A4: already aligned), sha, shb: 8 * the remainder
    template <bool A4>
    __device__ __forceinline__ static void load(uint32_t pa, uint32_t pb, uint32_t sha, uint32_t shb, uint2 & ha,
                                                uint2 & hb, uint2 (&qa)[2], uint2 (&qb)[2]) {
        ha    = sld8o<A4, 0>(pa, sha);
        hb    = sld8o<A4, 0>(pb, shb);
        qa[0] = sld8o<A4, 32>(pa, sha);
        qa[1] = sld8o<A4, 64>(pa, sha);
        qb[0] = sld8o<A4, 32>(pb, shb);
        qb[1] = sld8o<A4, 64>(pb, shb);
    }

    template <int NG, bool DBG>
    __device__ __forceinline__ static void sb(const uint8_t * wa, const uint8_t * wb, const uint8_t * ra,
                                              const uint8_t * rb, const uint8_t * xr, int lane, float (&acc)[NG][4],
                                              const DbgOut & dbg, int64_t rg, int sbi) {
        constexpr int  NT = 8 * NG;
        const int      t = lane & 3, g = lane >> 2, h = t >> 1;
        const uint32_t pa = smem_u32(wa) + 8 * t, pb = smem_u32(wb) + 8 * t;
        uint2          ha, hb, qa[2], qb[2];
        if (__all_sync(0xffffffffu, ((pa | pb) & 3u) == 0)) {  // warp-uniform: no divergence around the loads
            load<true>(pa, pb, 0, 0, ha, hb, qa, qb);
        } else {
            load<false>(pa & ~3u, pb & ~3u, (pa & 3u) * 8, (pb & 3u) * 8, ha, hb, qa, qb);
        }
        const uint8_t * ta = ra + 64 * h;
        const uint8_t * tb = rb + 64 * h;
        const uint8_t * xt = xr + g * kTokStride + 8 * t;
        int            im[2][NG][4];  // one accumulator chain per half n
#pragma unroll
        for (int n = 0; n < 2; n++) {
            zero<NG>(im[n]);
            uint32_t ya[4], yb[4];
            selectors(qa[n].x, qa[n].y, ha.x, ha.y, n, ya);
            selectors(qb[n].x, qb[n].y, hb.x, hb.y, n, yb);
#pragma unroll
            for (int jp = 0; jp < 2; jp++) {
                const int4 TA = lds128i(ta + 32 * n + 16 * jp), TB = lds128i(tb + 32 * n + 16 * jp);
#pragma unroll
                for (int e = 0; e < 2; e++) {
                    const int      j   = 2 * jp + e;
                    const uint32_t alo = (uint32_t) (e ? TA.z : TA.x), ahi = (uint32_t) (e ? TA.w : TA.y);
                    const uint32_t blo = (uint32_t) (e ? TB.z : TB.x), bhi = (uint32_t) (e ? TB.w : TB.y);
                    const uint32_t a0 = prmt(alo, ahi, ya[j]), a2 = prmt(alo, ahi, ya[j] >> 16);
                    const uint32_t a1 = prmt(blo, bhi, yb[j]), a3 = prmt(blo, bhi, yb[j] >> 16);
#pragma unroll
                    for (int grp = 0; grp < NG; grp++) {
                        const uint2 x = lds64(xt + 8 * grp * kTokStride + 32 * (4 * n + j));
                        mma_k32<true>(im[n][grp], a0, a1, a2, a3, x.x, x.y);
                    }
                }
            }
        }
        const uint8_t * xsum = xr + NT * kTokStride + 4 * NT + 8 * t;  // code sums of tokens 2t, 2t + 1
        int             is[NG][4];
#pragma unroll
        for (int grp = 0; grp < NG; grp++) {
            const uint2 s2 = lds64(xsum + 32 * grp);
            const int   x0 = 128 * (int) s2.x, x1 = 128 * (int) s2.y;
            is[grp][0]     = x0 - (im[0][grp][0] + im[1][grp][0]);
            is[grp][1]     = x1 - (im[0][grp][1] + im[1][grp][1]);
            is[grp][2]     = x0 - (im[0][grp][2] + im[1][grp][2]);
            is[grp][3]     = x1 - (im[0][grp][3] + im[1][grp][3]);
        }
        if constexpr (DBG) {
            dbg_store<NG>(dbg, is, false, rg, sbi, lane);
        } else {
            const float * xs = reinterpret_cast<const float *>(xr + NT * kTokStride);
            sb_update<NG, false>(acc, is, is, *reinterpret_cast<const float *>(ra + 128),
                                 *reinterpret_cast<const float *>(rb + 128), 0.f, 0.f, xs, t);
        }
    }
};

// IQ4_XS (136 B: d, 2 high bits of 8 scales, 4 bits of 8 scales, 128 bytes of code-book indices). Sub-block b,
// weight l: index = nibble (l >= 16) of qs[16b + (l & 15)], value kvalues_iq4nl[index]; scale = 6 bits - 32.
// Scale record: int32 sc[8] | f32 d.
struct DecIQ4XS {
    static constexpr int  BS   = 136;
    static constexpr int  KC   = 2;
    static constexpr int  RECB = 48;
    static constexpr bool Q80  = false;
    static constexpr int  MINB = 2;  // resident CTAs per SM the kernel is compiled for

    // the 16-entry code book as four words of int8 lanes (GGUF constant kvalues_iq4nl)
    static constexpr uint32_t T0 = 0xBFAD9881u, T1 = 0xF6EADDCFu, T2 = 0x26190D01u, T3 = 0x71594535u;

    // v holds 8 indices (byte j: low nibble = weight j, high nibble = weight j + 16) -> the values in nibble order:
    // r0 = weights 0, 16, 1, 17 and r1 = 2, 18, 3, 19 (the activation records are stored in this order, kPermIQ4XS)
    __device__ __forceinline__ static void lookup(uint32_t v, uint32_t & r0, uint32_t & r1) {
        const uint32_t v7  = v & 0x77777777u;
        const uint32_t sel = 0x32103210u | ((v & 0x88888888u) >> 1);  // bit 2 set: take the upper table's byte
        r0                 = prmt(prmt(T0, T1, v7), prmt(T2, T3, v7), sel);
        r1                 = prmt(prmt(T0, T1, v7 >> 16), prmt(T2, T3, v7 >> 16), sel >> 16);
    }

    __device__ __forceinline__ static void prep(const uint8_t * blk, uint8_t * rec) {
        const uint32_t H = lds_u16(blk + 2), L = lds32(blk + 4);
        int4 *         ri = reinterpret_cast<int4 *>(rec);
        int            v[8];
#pragma unroll
        for (int b = 0; b < 8; b++) v[b] = (int) (((L >> (4 * b)) & 0xFu) | (((H >> (2 * b)) & 3u) << 4)) - 32;
        ri[0]                                = make_int4(v[0], v[1], v[2], v[3]);
        ri[1]                                = make_int4(v[4], v[5], v[6], v[7]);
        *reinterpret_cast<float *>(rec + 32) = ldh(blk);
    }

    template <int NG, bool DBG>
    __device__ __forceinline__ static void sb(const uint8_t * wa, const uint8_t * wb, const uint8_t * ra,
                                              const uint8_t * rb, const uint8_t * xr, int lane, float (&acc)[NG][4],
                                              const DbgOut & dbg, int64_t rg, int sbi) {
        constexpr int NT = 8 * NG;
        const int     t = lane & 3, g = lane >> 2;
        const int4    sA4[2] = { lds128i(ra), lds128i(ra + 16) }, sB4[2] = { lds128i(rb), lds128i(rb + 16) };
        int           im[NG][4], in[NG][4];
        zero<NG>(im);
        zero<NG>(in);
#pragma unroll
        for (int b = 0; b < 8; b++) {
            const int sA = sel4(sA4[b >> 2], b & 3), sB = sel4(sB4[b >> 2], b & 3);
            uint32_t  a0, a2, a1, a3;
            lookup(lds32(wa + 8 + 16 * b + 4 * t), a0, a2);
            lookup(lds32(wb + 8 + 16 * b + 4 * t), a1, a3);
#pragma unroll
            for (int grp = 0; grp < NG; grp++) {
                const uint8_t * xp   = xr + (8 * grp + g) * kTokStride + 32 * b + 4 * t;
                int             c[4];
                mma_k32_z<false>(c, a0, a1, a2, a3, lds32(xp), lds32(xp + 16));
                scale_acc<NG>(im, grp, sA, sB, c);
            }
        }
        if constexpr (DBG) {
            dbg_store<NG>(dbg, im, false, rg, sbi, lane);
        } else {
            const float * xs = reinterpret_cast<const float *>(xr + NT * kTokStride);
            sb_update<NG, false>(acc, im, in, *reinterpret_cast<const float *>(ra + 32),
                                 *reinterpret_cast<const float *>(rb + 32), 0.f, 0.f, xs, t);
        }
    }
};

// Q8_0 (34 B per 32 weights: f16 d, 32 int8). A "super-block" here is 8 consecutive blocks (272 bytes); each block
// has its own weight and activation scale, so the f32 update happens per block. Scale record: f32 d[8].
struct DecQ80 {
    static constexpr int  BS   = 272;
    static constexpr int  KC   = 1;
    static constexpr int  RECB = 32;
    static constexpr bool Q80  = true;
    static constexpr int  MINB = 2;  // resident CTAs per SM the kernel is compiled for

    __device__ __forceinline__ static void prep(const uint8_t * blk, uint8_t * rec) {
        float4 * rf = reinterpret_cast<float4 *>(rec);
        rf[0]       = make_float4(ldh(blk), ldh(blk + 34), ldh(blk + 68), ldh(blk + 102));
        rf[1]       = make_float4(ldh(blk + 136), ldh(blk + 170), ldh(blk + 204), ldh(blk + 238));
    }

    // 4 quant bytes at byte offset o of block i; rows are 16-byte aligned in practice (Q8_0 rows are multiples of
    // 272 bytes), so block i's quants (at 34 i + 2) are 4-byte aligned for odd i and 2 mod 4 for even i
    template <bool A4>
    __device__ __forceinline__ static uint32_t q4(uint32_t base, int i, int o) {
        const uint32_t a = base + 34 * i + o;
        if constexpr (A4) {
            if (i & 1) return sld32(a);
            return __funnelshift_r(sld32(a - 2), sld32(a + 2), 16);
        } else {
            return sld4_a2<false>(a);
        }
    }

    template <int NG, bool DBG, bool A4>
    __device__ __forceinline__ static void sb_impl(uint32_t pa, uint32_t pb, const uint8_t * ra, const uint8_t * rb,
                                                   const uint8_t * xr, int lane, float (&acc)[NG][4],
                                                   const DbgOut & dbg, int64_t rg, int sbi) {
        constexpr int NT = 8 * NG;
        const int     t = lane & 3, g = lane >> 2;
        const float * xsb = reinterpret_cast<const float *>(xr + NT * kTokStride);
        const float4  dA4[2] = { *reinterpret_cast<const float4 *>(ra), *reinterpret_cast<const float4 *>(ra + 16) };
        const float4  dB4[2] = { *reinterpret_cast<const float4 *>(rb), *reinterpret_cast<const float4 *>(rb + 16) };
#pragma unroll
        for (int i = 0; i < 8; i++) {
            const uint32_t a0 = q4<A4>(pa, i, 2 + 4 * t), a2 = q4<A4>(pa, i, 18 + 4 * t);
            const uint32_t a1 = q4<A4>(pb, i, 2 + 4 * t), a3 = q4<A4>(pb, i, 18 + 4 * t);
            int            c[NG][4];
#pragma unroll
            for (int grp = 0; grp < NG; grp++) {
                const uint8_t * xp = xr + (8 * grp + g) * kTokStride + 32 * i + 4 * t;
                if constexpr (DBG) {
                    mma_k32_z<false>(c[grp], a0, a1, a2, a3, lds32(xp), lds32(xp + 16));
                } else {
                    // the block sum i (|i| <= 32 * 128 * 127 < 2^22) on top of 0x4B400000 reads as the float
                    // 12582912 + i exactly: one f32x2 subtraction per pair gives the sums as floats
                    mma_k32_c<false>(c[grp], a0, a1, a2, a3, lds32(xp), lds32(xp + 16), kMagic32);
                }
            }
            if constexpr (DBG) {
                dbg_store<NG>(dbg, c, false, rg, 8 * sbi + i, lane);
            } else {
                const float4 & qa = dA4[i >> 2];
                const float4 & qb = dB4[i >> 2];
                const float    dA = (i & 3) == 0 ? qa.x : (i & 3) == 1 ? qa.y : (i & 3) == 2 ? qa.z : qa.w;
                const float    dB = (i & 3) == 0 ? qb.x : (i & 3) == 1 ? qb.y : (i & 3) == 2 ? qb.z : qb.w;
                const float *  xs = xsb + i * NT;
                const f2       nm = f2_pack(-12582912.0f, -12582912.0f);
#pragma unroll
                for (int grp = 0; grp < NG; grp++) {
                    const float2 x  = *reinterpret_cast<const float2 *>(xs + 8 * grp + 2 * t);
                    const f2     xx = f2_pack(x.x, x.y);
                    const f2     c01 = f2_add(f2_pack(__int_as_float(c[grp][0]), __int_as_float(c[grp][1])), nm);
                    const f2     c23 = f2_add(f2_pack(__int_as_float(c[grp][2]), __int_as_float(c[grp][3])), nm);
                    f2           a01 = f2_pack(acc[grp][0], acc[grp][1]), a23 = f2_pack(acc[grp][2], acc[grp][3]);
                    a01 = f2_fma(f2_mul(f2_pack(dA, dA), xx), c01, a01);
                    a23 = f2_fma(f2_mul(f2_pack(dB, dB), xx), c23, a23);
                    f2_unpack(a01, acc[grp][0], acc[grp][1]);
                    f2_unpack(a23, acc[grp][2], acc[grp][3]);
                }
            }
        }
    }

    template <int NG, bool DBG>
    __device__ __forceinline__ static void sb(const uint8_t * wa, const uint8_t * wb, const uint8_t * ra,
                                              const uint8_t * rb, const uint8_t * xr, int lane, float (&acc)[NG][4],
                                              const DbgOut & dbg, int64_t rg, int sbi) {
        // the choice must be warp-uniform: sb_impl issues mma.sync (rows of one warp can differ in alignment)
        const uint32_t pa = smem_u32(wa), pb = smem_u32(wb);
        if (__all_sync(0xffffffffu, ((pa | pb) & 3u) == 0)) {
            sb_impl<NG, DBG, true>(pa, pb, ra, rb, xr, lane, acc, dbg, rg, sbi);
        } else {
            sb_impl<NG, DBG, false>(pa, pb, ra, rb, xr, lane, acc, dbg, rg, sbi);
        }
    }
};

// ---------------------------------------------------------------------------------------------------------------
// the kernel
//
// Work unit = (block of 64 weight rows, K range). CTAs are persistent: CTA c takes units c, c + grid, ... and the
// grid is a multiple of the number of K ranges, so a CTA keeps one K range. Each unit streams through the stage ring
// in chunks of kc super-blocks; a stage holds the chunk's 64 row segments (TMA boxes) and its kc activation records.
// With one K range the consumers write Y; otherwise each unit writes its partial sums to the work buffer and the
// last of the unit's K ranges to arrive (an atomic counter, no waiting) adds them up in K order and writes Y.

struct GemmArgs {
    const uint8_t * W;           // weight rows, 16-byte aligned
    int64_t         rows;
    int64_t         row_bytes;
    int64_t         w_bytes;     // rows * row_bytes
    int64_t         rows_main;   // rows reachable through the tensor map: (rows / G) * G
    int             nsb;         // 256-column super-blocks per row
    int             kc;          // super-blocks per stage
    int             G;           // weight rows per tensor-map row (G * row_bytes is a multiple of 16)
    int             gshift;      // log2(G)
    int             rbm16;       // row_bytes mod 16
    int             Wbox;        // bytes per row segment in a stage (TMA box width)
    int             S;           // stages in the ring
    int             ksplit;      // K ranges
    int             kr_sbs;      // super-blocks per K range (the last one may be shorter)
    int             units;
    int             stage_bytes;
    int             left_off;    // leftover-row slots (rows >= rows_main) inside a stage
    int             LSR;         // leftover slot stride
    int             rec_off;     // activation records inside a stage
    int             scr_off;     // per-warp scale-record scratch (after the stages)
    int             red_off;     // cluster split K: this CTA's partial sums [NT][64] f32 (after the scratch)
    int             cluster;     // the K ranges of a row block form a thread-block cluster (split-K in DSMEM)
    const uint8_t * recs;
    float *         part;        // split-K partial sums [ksplit][N][rows]
    int32_t *       cnt;         // split-K arrival counters, one per row block (zeroed by the quantizer kernel)
    float *         Y;
    int64_t         ldy;         // elements
    int             N;
    int32_t *       status;
    int32_t *       isum;        // integer outputs (srhpm_mul_mat_isums), else null
    int32_t *       imin;
    int             nblk;        // blocks per row in the integer outputs
    // fused quantization: the consumer warps of the whole grid quantize X into the records themselves (one job per
    // (super-block, token) and warp), zero the split-K counters, and the grid meets at *sync before any CTA loads a
    // record; otherwise a separate quantizer kernel ran before this one
    int             fq;
    const float *   X;
    const float *   X2;          // non-null: X and X2 are the SwiGLU inputs (gate, up), the records are of
                                 // silu(X) * X2 as swiglu_q8K_kernel computes it
    int64_t         ldx;
    int             perm;        // record byte order (record_perm)
    int             q80mode;     // the context's q8_0 mode (Q8_0 weights)
    int             ncnt;        // split-K counters to zero
    uint32_t *      sync;        // this work buffer's arrival counter: every launch adds exactly 2^20 to it
};

// The consumer warps' share of the activation quantization (fused form): warp w of the grid quantizes the
// (super-block, token) pairs w, w + warps, ... of the N real tokens (the records' padding tokens feed only output
// columns that are never stored) and the grid zeroes the split-K counters. Same device functions and records as
// quant_q8K_kernel / quant_q80_kernel.
template <class D, int NG>
__device__ __forceinline__ void fq_quantize(const GemmArgs & a, int warp, int lane) {
    constexpr int NT = 8 * NG;
    constexpr int RB = rec_bytes(D::Q80, NT);
    const int     nw = (int) gridDim.x * kNCW;
    const int     jobs = a.nsb * a.N;
    for (int j = (int) blockIdx.x * kNCW + warp; j < jobs; j += nw) {
        const int     sb = j / a.N, t = j - sb * a.N;
        const int64_t c0 = (int64_t) t * a.ldx + (int64_t) sb * QK + 8 * lane;
        float         v[8];
        load8(a.X + c0, v);
        if (a.X2) {  // h = silu(gate) * up, as swiglu_q8K_kernel
            float u8[8];
            load8(a.X2 + c0, u8);
#pragma unroll
            for (int jj = 0; jj < 8; jj++) v[jj] = v[jj] / (1.0f + expf(-v[jj])) * u8[jj];
        }
        uint8_t * rec = const_cast<uint8_t *>(a.recs) + (size_t) sb * RB;
        if constexpr (D::Q80) {
            __half      dh;
            const uint2 pk = q80_quantize_warp(v, a.q80mode, dh);
            q80_store_record(pk, dh, rec, t, NT, lane);
        } else {
            int   qv[8];
            float dv;
            q8K_quantize_warp(v, lane, qv, dv);
            q8K_store_record(qv, dv, rec, t, NT, lane, a.perm);
        }
    }
    for (int i = (int) blockIdx.x * (kNCW * 32) + (int) threadIdx.x; i < a.ncnt; i += (int) gridDim.x * (kNCW * 32)) {
        a.cnt[i] = 0;
    }
    // the records are read by other CTAs' bulk copies (async proxy)
    fence_proxy_async_global();
}

// Fused form, producer lane 0 of every CTA, after the CTA's consumers finished their quantization jobs: publish the
// CTA's arrival (release) and wait (acquire, bounded: 2 s, then an error status) until every CTA of the grid has
// arrived. Each launch adds exactly 2^20 to the counter (CTA 0 adds the remainder of the equal shares), so the counter
// is a multiple of 2^20 between launches, the value a CTA reads before adding its own share lies in its launch's
// epoch, and the launch is complete at the next multiple (modulo 2^32). All CTAs are resident together (the grid is
// sized to the resident CTA slots), and the launch before this one on the stream never waits for this one.
__device__ __forceinline__ void fq_grid_meet(const GemmArgs & a) {
    __threadfence();
    const uint32_t q   = (1u << 20) / gridDim.x;
    const uint32_t inc = blockIdx.x == 0 ? (1u << 20) - (gridDim.x - 1) * q : q;
    const uint32_t old = atomicAdd(a.sync, inc);
    const uint32_t target = ((old >> 20) + 1u) << 20;
    const uint64_t t0 = globaltimer_ns();
    while ((int32_t) (ld_acquire_gpu(a.sync) - target) < 0) {
        if (globaltimer_ns() - t0 > 2000000000ull) {
            atomicExch(a.status, kErrGridWait);
            break;
        }
        __nanosleep(32);
    }
    __threadfence();
    fence_proxy_async_global();  // the bulk copies that follow read what other CTAs wrote
}

// 1-D copy of the row segment [start, end) of W into dst (16-byte aligned, holding the segment at its own 16-byte
// phase): bulk bytes below the last 16-byte boundary of W, hand copy of the ragged end. Returns the bulk bytes.
__device__ __forceinline__ uint32_t row_segment_copy(const GemmArgs & a, uint8_t * dst, int64_t start, int64_t end,
                                                     uint64_t * bar, bool issue) {
    const int64_t wlim = a.w_bytes & ~int64_t(15);
    const int64_t a0 = start & ~int64_t(15), be = min((end + 15) & ~int64_t(15), wlim);
    uint32_t      tx = 0;
    if (be > a0) {
        if (issue) bulk_g2s(dst, a.W + a0, (uint32_t) (be - a0), bar);
        tx = (uint32_t) (be - a0);
    }
    if (!issue) {
        for (int64_t p = max(a0, be); p < end; p++) dst[p - a0] = a.W[p];
    }
    return tx;
}

template <class D, int NG>
__device__ __forceinline__ void produce_stage(const GemmArgs & a, const CUtensorMap * wmap, uint8_t * st,
                                              uint64_t * bar, int64_t row0, int sb0, int kcc, int lane,
                                              bool defer_records) {
    constexpr int RB = rec_bytes(D::Q80, 8 * NG);
    // leftover rows (at most G - 1, never reached by the tensor map): one lane each, 1-D copies
    uint32_t      tx = 0;
    const int64_t lr = row0 + lane;
    const bool    left = lane < kTileRows && lr >= a.rows_main && lr < a.rows && lr < row0 + kTileRows;
    if (left) {
        const int64_t start = lr * a.row_bytes + (int64_t) sb0 * D::BS;
        tx = row_segment_copy(a, st + a.left_off + (int) (lr - a.rows_main) * a.LSR, start,
                              start + (int64_t) kcc * D::BS, bar, false);
    }
    tx = __reduce_add_sync(0xffffffffu, tx);
    const bool tma = a.rows_main > 0;
    if (tma) tx += (uint32_t) (kTileRows * a.Wbox);
    tx += (uint32_t) (kcc * RB);  // the records, issued here or (deferred) once the quantizer grid has finished
    fence_proxy_async_smem();
    __syncwarp();
    if (lane == 0) mbar_arrive_expect_tx(bar, tx);
    __syncwarp();
    if (left) {
        const int64_t start = lr * a.row_bytes + (int64_t) sb0 * D::BS;
        row_segment_copy(a, st + a.left_off + (int) (lr - a.rows_main) * a.LSR, start, start + (int64_t) kcc * D::BS,
                         bar, true);
    }
    if (lane == 0) {
        if (tma) {
            const int rpb = kTileRows >> a.gshift;  // tensor-map rows per box
            for (int j = 0; j < a.G; j++) {
                const int64_t xb = ((int64_t) j * a.row_bytes + (int64_t) sb0 * D::BS) & ~int64_t(15);
                tma_load_2d(st + j * rpb * a.Wbox, wmap, (int) (xb >> 2), (int) (row0 >> a.gshift), bar);
            }
        }
        if (!defer_records) bulk_g2s(st + a.rec_off, a.recs + (size_t) sb0 * RB, (uint32_t) (kcc * RB), bar);
    }
}

template <class D, int NG>
__device__ __forceinline__ void producer(const GemmArgs & a, const CUtensorMap * wmap, uint64_t * full,
                                         uint64_t * empty, uint8_t * stage0, int lane) {
    constexpr int RB  = rec_bytes(D::Q80, 8 * NG);
    const int     kr  = blockIdx.x % a.ksplit;
    const int     sbA = kr * a.kr_sbs, sbB = min(a.nsb, sbA + a.kr_sbs);
    const int     nck = (sbB - sbA + a.kc - 1) / a.kc;
    if (lane == 0 && a.rows_main > 0) prefetch_tmap(wmap);
    int  n = 0, s = 0;  // stages issued; ring slot of the next one
    int  ph     = 0;    // parity of the slot's next empty-barrier phase to wait for
    bool ok     = true;
    bool waited = false;
    for (int u = blockIdx.x; u < a.units && ok; u += gridDim.x) {
        const int64_t row0 = (int64_t) (u / a.ksplit) * kTileRows;
        for (int c = 0; c < nck; c++) {
            if (n >= a.S && !mbar_wait_sleep(&empty[s], ph)) {
                ok = false;
                break;
            }
            const int sb0 = sbA + c * a.kc, kcc = min(a.kc, sbB - sb0);
            // the first stages' weights go out before the activation records exist (programmatic dependent
            // launch); their records follow once the quantizer grid has finished
            const bool pre = !waited;
            produce_stage<D, NG>(a, wmap, stage0 + (size_t) s * a.stage_bytes, &full[s], row0, sb0, kcc, lane, pre);
            n++;
            if (++s == a.S) {
                s = 0;
                if (n > a.S) ph ^= 1;
            }
            if (n == a.S) ph = 0;
            if (pre && (n == a.S || (c + 1 == nck && u + (int) gridDim.x >= a.units))) {
                pdl_wait();
                waited = true;
                if (a.fq) {
                    named_bar_sync(2, kThreads);  // this CTA's consumers have written their records
                    if (lane == 0) fq_grid_meet(a);
                    __syncwarp();
                }
                if (lane == 0) {
                    for (int m = 0; m < n; m++) {  // the records of the stages issued so far (slot m, first use)
                        const int sbm = sbA + (m % nck) * a.kc, kcm = min(a.kc, sbB - sbm);
                        bulk_g2s(stage0 + (size_t) m * a.stage_bytes + a.rec_off, a.recs + (size_t) sbm * RB,
                                 (uint32_t) (kcm * RB), &full[m]);
                    }
                }
            }
        }
    }
    if (!waited) {
        pdl_wait();
        if (a.fq) {  // the grid's counter takes this CTA's share in every case
            named_bar_sync(2, kThreads);
            if (lane == 0) fq_grid_meet(a);
            __syncwarp();
        }
    }
    // drain: every copy this warp issued has landed before the CTA may exit
    for (int m = max(0, n - a.S); m < n; m++) {
        if (!mbar_wait(&full[m % a.S], (m / a.S) & 1)) ok = false;
    }
    if (!ok && lane == 0) atomicExch(a.status, kErrWaitEmpty);
}

// shared-memory address of local row r (0..63) of the tile in a stage; rows past the matrix map to the stage base
template <class D>
__device__ __forceinline__ const uint8_t * row_ptr(const GemmArgs & a, const uint8_t * st, int64_t row0, int r,
                                                   int sb0) {
    const int64_t R = row0 + r;
    if (R < a.rows_main) {
        const int j = r & (a.G - 1), q = r >> a.gshift;
        const int ph = (j * a.rbm16 + sb0 * (D::BS & 15)) & 15;
        return st + (j * (kTileRows >> a.gshift) + q) * a.Wbox + ph;
    }
    if (R < a.rows) {
        const int ph = (int) ((R * a.row_bytes + (int64_t) sb0 * D::BS) & 15);
        return st + a.left_off + (int) (R - a.rows_main) * a.LSR + ph;
    }
    return st;
}

template <class D, int NG, bool DBG>
__global__ void __launch_bounds__(kThreads, D::MINB) srv_gemm_kernel(const __grid_constant__ CUtensorMap wmap,
                                                            const GemmArgs a) {
    extern __shared__ __align__(128) uint8_t smem[];
    uint64_t * full       = reinterpret_cast<uint64_t *>(smem);
    uint64_t * empty      = full + kMaxStages;
    uint64_t * part_ready = full + 2 * kMaxStages;  // cluster split K, K range 0: the other ranges' partials are in
    uint64_t * part_free  = part_ready + 1;         // cluster split K, K range > 0: range 0 has read this CTA's partials
    uint8_t *  stage0     = smem + kBarBytes;
    const int  warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
    if (threadIdx.x == 0) {
        for (int s = 0; s < a.S; s++) {
            mbar_init(&full[s], 1);
            mbar_init(&empty[s], kNCW * 32);
        }
        if (a.cluster) {
            mbar_init(part_ready, a.ksplit - 1);
            mbar_init(part_free, 1);
        }
        fence_mbar_init();
    }
    __syncthreads();
    if (a.cluster) cluster_sync_all();  // every CTA's barriers exist before any remote arrival
    if (warp == kNCW) {
        producer<D, NG>(a, &wmap, full, empty, stage0, lane);
        if (a.cluster) cluster_sync_all();  // no CTA exits while a peer may still use its shared memory
        return;
    }
    pdl_launch_dependents();  // the next call's quantizer may start; it waits for this grid before touching data
    if (a.fq) {  // warm L2 with the activation segment of this warp's first quantization job (a hint, as above)
        const int j = (int) blockIdx.x * kNCW + warp;
        if (j < a.nsb * a.N && (lane & 3) == 0) {
            const int     sb = j / a.N, t = j - sb * a.N;
            const int64_t c0 = (int64_t) t * a.ldx + (int64_t) sb * QK + 8 * lane;
            asm volatile("prefetch.global.L2 [%0];" ::"l"(a.X + c0));
            if (a.X2) asm volatile("prefetch.global.L2 [%0];" ::"l"(a.X2 + c0));
        }
    }
    pdl_wait();  // the split-K counters and partials are written below; the quantizer grid zeroes the counters
    if (a.fq) {
        fq_quantize<D, NG>(a, warp, lane);
        named_bar_arrive(2, kThreads);  // the producer meets the grid for this CTA, then loads the records
    }
    constexpr int  RB  = rec_bytes(D::Q80, 8 * NG);
    const int      g = lane >> 2, t = lane & 3;
    const int      rl  = warp * 16 + g;
    const int      kr  = blockIdx.x % a.ksplit;
    const int      sbA = kr * a.kr_sbs, sbB = min(a.nsb, sbA + a.kr_sbs);
    const int      nck = (sbB - sbA + a.kc - 1) / a.kc;
    const DbgOut   dbg = { a.isum, a.imin, a.rows, a.N, a.nblk };
    uint8_t *      scr = smem + a.scr_off + warp * (D::KC * 16 * D::RECB);  // this warp's scale records
    __shared__ int last_flag;
    int            s = 0, ph = 0;
    uint32_t       uidx = 0;  // units done (phase parity of the cluster split-K barriers)
    bool           bad = false;  // a wait ran out: skip further waits and work, keep meeting the barriers
    // a row's place in a stage: fixed offset + 16-byte phase (j * row_bytes + sb0 * BS) mod 16, j = row mod G
    const int      bsm = D::BS & 15;
    auto           row_off = [&](int r, int & jterm) -> int {
        const int j = r & (a.G - 1), q = r >> a.gshift;
        jterm       = j * a.rbm16;
        return (j * (kTileRows >> a.gshift) + q) * a.Wbox;
    };
    int       ja, jb, jp;
    const int offa = row_off(rl, ja), offb = row_off(rl + 8, jb), offp = row_off(warp * 16 + (lane & 15), jp);
    for (int u = blockIdx.x; u < a.units; u += gridDim.x) {
        const int64_t rb = u / a.ksplit, row0 = rb * kTileRows, rg = row0 + rl;
        const bool    edge = row0 + kTileRows > a.rows_main;  // rows past the tensor map in this tile
        float         acc[NG][4];
#pragma unroll
        for (int grp = 0; grp < NG; grp++) acc[grp][0] = acc[grp][1] = acc[grp][2] = acc[grp][3] = 0.0f;
        for (int c = 0; c < nck; c++) {
            const int slot = s, par = ph;
            if (++s == a.S) {
                s = 0;
                ph ^= 1;
            }
            if (!bad && !mbar_wait_sleep(&full[slot], par)) {
                if (lane == 0) atomicExch(a.status, kErrWaitFull);
                bad = true;
            }
            if (bad) {
                mbar_arrive(&empty[slot]);
                continue;
            }
            const uint8_t * st  = stage0 + (size_t) slot * a.stage_bytes;
            const int       sb0 = sbA + c * a.kc, kcc = min(a.kc, sbB - sb0);
            const uint8_t * wa;
            const uint8_t * wb;
            const uint8_t * wp;
            if (!edge) {
                const int sbt = sb0 * bsm;
                wa            = st + offa + ((ja + sbt) & 15);
                wb            = st + offb + ((jb + sbt) & 15);
                wp            = st + offp + ((jp + sbt) & 15);
            } else {
                wa = row_ptr<D>(a, st, row0, rl, sb0);
                wb = row_ptr<D>(a, st, row0, rl + 8, sb0);
                wp = row_ptr<D>(a, st, row0, warp * 16 + (lane & 15), sb0);
            }
            // scale records of this warp's 16 rows x kcc super-blocks, one (row, super-block) per lane: lane l takes
            // row l & 15 of super-block l >> 4 (clamped to the chunk, so every lane runs the same code)
            {
                const int kb = min(lane >> 4, kcc - 1);
                D::prep(wp + kb * D::BS, scr + (kb * 16 + (lane & 15)) * D::RECB);
            }
            __syncwarp();
            const uint8_t * xr = st + a.rec_off;
            if (kcc == D::KC) {  // a full stage: straight-line code, so the super-blocks' loads and math can overlap
#pragma unroll
                for (int kb = 0; kb < D::KC; kb++) {
                    D::template sb<NG, DBG>(wa + kb * D::BS, wb + kb * D::BS, scr + (kb * 16 + g) * D::RECB,
                                            scr + (kb * 16 + g + 8) * D::RECB, xr + kb * RB, lane, acc, dbg, rg,
                                            sb0 + kb);
                }
            } else {
                for (int kb = 0; kb < kcc; kb++) {
                    D::template sb<NG, DBG>(wa + kb * D::BS, wb + kb * D::BS, scr + (kb * 16 + g) * D::RECB,
                                            scr + (kb * 16 + g + 8) * D::RECB, xr + kb * RB, lane, acc, dbg, rg,
                                            sb0 + kb);
                }
            }
            mbar_arrive(&empty[slot]);  // every consumer thread arrives: no divergent branch per stage
        }
        if constexpr (!DBG) {
            if (a.ksplit == 1) {
                if (bad) continue;
#pragma unroll
                for (int grp = 0; grp < NG; grp++) {
#pragma unroll
                    for (int e = 0; e < 4; e++) {
                        const int     tok = 8 * grp + 2 * t + (e & 1);
                        const int64_t row = e < 2 ? rg : rg + 8;
                        if (tok < a.N && row < a.rows) a.Y[(int64_t) tok * a.ldy + row] = acc[grp][e];
                    }
                }
            } else if (a.cluster) {
                // split K inside a cluster: every K range keeps its partial sums in its own shared memory; K range 0
                // (cluster rank 0) waits for the others' arrivals, adds their partials over DSMEM in K order and
                // writes Y, then releases them
                float * red = reinterpret_cast<float *>(smem + a.red_off);  // [8 NG tokens][64 rows]
#pragma unroll
                for (int grp = 0; grp < NG; grp++) {
#pragma unroll
                    for (int e = 0; e < 4; e++) {
                        red[(8 * grp + 2 * t + (e & 1)) * kTileRows + (e < 2 ? rl : rl + 8)] = acc[grp][e];
                    }
                }
                named_bar_sync(1, kNCW * 32);
                const uint32_t par = uidx & 1;
                if (kr != 0) {
                    if (threadIdx.x == 0) {
                        fence_acq_rel_cluster();
                        mbar_arrive_cluster(mapa_shared(smem_u32(part_ready), 0));
                        if (!mbar_wait_cluster(part_free, par)) atomicExch(a.status, kErrClusterWait);
                    }
                    named_bar_sync(1, kNCW * 32);  // the partial buffer is free again
                } else {
                    if (threadIdx.x == 0 && !mbar_wait_cluster(part_ready, par)) atomicExch(a.status, kErrClusterWait);
                    named_bar_sync(1, kNCW * 32);
                    if (!bad) {
#pragma unroll
                        for (int grp = 0; grp < NG; grp++) {
#pragma unroll
                            for (int e = 0; e < 4; e++) {
                                const int     tok = 8 * grp + 2 * t + (e & 1);
                                const int     rlo = e < 2 ? rl : rl + 8;
                                const int64_t row = row0 + rlo;
                                if (tok < a.N && row < a.rows) {
                                    const uint32_t ad = smem_u32(&red[tok * kTileRows + rlo]);
                                    float          sum = acc[grp][e];
                                    for (int k = 1; k < a.ksplit; k++) sum += ld_dsmem_f32(mapa_shared(ad, k));
                                    a.Y[(int64_t) tok * a.ldy + row] = sum;
                                }
                            }
                        }
                    }
                    named_bar_sync(1, kNCW * 32);  // every remote read is done
                    if (threadIdx.x == 0) {
                        for (int k = 1; k < a.ksplit; k++) mbar_arrive_cluster(mapa_shared(smem_u32(part_free), k));
                    }
                }
                uidx++;
            } else {
                // split K: partial sums out, then the last K range of this row block reduces them in K order
                if (!bad) {
#pragma unroll
                    for (int grp = 0; grp < NG; grp++) {
#pragma unroll
                        for (int e = 0; e < 4; e++) {
                            const int     tok = 8 * grp + 2 * t + (e & 1);
                            const int64_t row = e < 2 ? rg : rg + 8;
                            if (tok < a.N && row < a.rows) {
                                a.part[((int64_t) kr * a.N + tok) * a.rows + row] = acc[grp][e];
                            }
                        }
                    }
                }
                __threadfence();
                named_bar_sync(1, kNCW * 32);
                if (threadIdx.x == 0) last_flag = atomicAdd(&a.cnt[rb], 1) == a.ksplit - 1;
                named_bar_sync(1, kNCW * 32);
                if (last_flag && !bad) {
                    __threadfence();
#pragma unroll
                    for (int grp = 0; grp < NG; grp++) {
#pragma unroll
                        for (int e = 0; e < 4; e++) {
                            const int     tok = 8 * grp + 2 * t + (e & 1);
                            const int64_t row = e < 2 ? rg : rg + 8;
                            if (tok < a.N && row < a.rows) {
                                float sum = 0.0f;
                                for (int k = 0; k < a.ksplit; k++) {
                                    sum += __ldcg(&a.part[((int64_t) k * a.N + tok) * a.rows + row]);
                                }
                                a.Y[(int64_t) tok * a.ldy + row] = sum;
                            }
                        }
                    }
                }
                named_bar_sync(1, kNCW * 32);  // last_flag is rewritten by the next unit
            }
        }
    }
    if (a.cluster) cluster_sync_all();
}

// ---------------------------------------------------------------------------------------------------------------
// host side

int slot_stride(int need) {
    int s = (need + 15) / 16 * 16;
    while (s % 128 != 32 && s % 128 != 96) s += 16;
    return s;
}

using EncodeTiled = CUresult (*)(CUtensorMap *, CUtensorMapDataType, cuuint32_t, void *, const cuuint64_t *,
                                 const cuuint64_t *, const cuuint32_t *, const cuuint32_t *, CUtensorMapInterleave,
                                 CUtensorMapSwizzle, CUtensorMapL2promotion, CUtensorMapFloatOOBfill);

EncodeTiled encode_fn() {
    static EncodeTiled fn = [] {
        void *                          p = nullptr;
        cudaDriverEntryPointQueryResult q;
        if (cudaGetDriverEntryPoint("cuTensorMapEncodeTiled", &p, cudaEnableDefault, &q) != cudaSuccess ||
            q != cudaDriverEntryPointSuccess) {
            p = nullptr;
        }
        return reinterpret_cast<EncodeTiled>(p);
    }();
    return fn;
}

// the separate activation quantizer (records and zeroed split-K counters), launched before the GEMM when the GEMM
// does not quantize in its own prologue
int launch_quantizer(srhpm_ctx * ctx, const GemmArgs & a, int NT, bool q80, cudaStream_t stream) {
    const int64_t      warps  = (int64_t) a.nsb * a.N;  // one per (super-block, real token)
    const int          blocks = (int) ((warps + 7) / 8);
    cudaLaunchConfig_t cfg    = {};
    cfg.gridDim               = dim3((unsigned) blocks);
    cfg.blockDim              = dim3(256);
    cfg.stream                = stream;
    cudaLaunchAttribute attr[1];
    attr[0].id                                         = cudaLaunchAttributeProgrammaticStreamSerialization;
    attr[0].val.programmaticStreamSerializationAllowed = 1;
    cfg.attrs                                          = attr;
    cfg.numAttrs                                       = 1;
    uint8_t *   recs = const_cast<uint8_t *>(a.recs);
    cudaError_t e;
    if (a.X2) {  // SwiGLU inputs: the SwiGLU kernel writes the records (K-quant weights; h is not stored)
        cfg.gridDim = dim3((unsigned) (((int64_t) a.nsb * NT + 7) / 8));
        e = cudaLaunchKernelEx(&cfg, swiglu_q8K_kernel, a.X, a.X2, a.ldx, (float *) nullptr, (int64_t) 0, a.N, a.nsb,
                               NT, recs, a.perm, a.cnt, a.ncnt);
    } else if (q80) {
        e = cudaLaunchKernelEx(&cfg, quant_q80_kernel<false>, a.X, a.ldx, a.N, a.nsb, NT, a.q80mode, recs,
                               (uint8_t *) nullptr, a.cnt, a.ncnt);
    } else {
        e = cudaLaunchKernelEx(&cfg, quant_q8K_kernel<false>, a.X, a.ldx, a.N, a.nsb, NT, recs, (int8_t *) nullptr,
                               (float *) nullptr, (int16_t *) nullptr, (int16_t *) nullptr, a.cnt, a.ncnt, a.perm);
    }
    ctx->launches.fetch_add(1);
    return cuda_status(e);
}

template <class D, int NG, bool DBG>
int launch_gemm(srhpm_ctx * ctx, GemmArgs a, cudaStream_t stream) {
    constexpr int RB = rec_bytes(D::Q80, 8 * NG);
    a.kc             = std::min(D::KC, a.nsb);
    a.G              = 1;
    a.gshift         = 0;
    while ((a.G * a.row_bytes) % 16 != 0) {  // row sizes are even, so G <= 8
        a.G *= 2;
        a.gshift++;
    }
    a.rbm16            = (int) (a.row_bytes & 15);
    a.rows_main        = (a.rows / a.G) * a.G;
    const bool aligned = a.G == 1 && D::BS % 16 == 0;
    // box width: the segment (plus its 16-byte phase) widened to 32 or 96 mod 128, so that the rows of a quad
    // group land on different shared-memory banks (the extra bytes are the next segment's, read from L2)
    a.Wbox             = slot_stride((aligned ? 0 : 14) + a.kc * D::BS);
    a.LSR              = slot_stride((aligned ? 0 : 14) + a.kc * D::BS);
    a.left_off         = kTileRows * a.Wbox;
    a.rec_off          = (a.left_off + (a.G > 1 ? (a.G - 1) * a.LSR : 0) + 127) / 128 * 128;
    a.stage_bytes      = (a.rec_off + a.kc * RB + 127) / 128 * 128;
    const int scr      = kNCW * D::KC * 16 * D::RECB;
    const int red      = kTileRows * 8 * NG * (int) sizeof(float);  // cluster split K: the CTA's partial sums
    // the most resident CTAs per SM the decoder is compiled for (D::MINB: 2, or 4 for Q6_K; 228 KB of shared memory per
    // SM, 1 KB of it reserved per CTA, a few bytes of static shared memory), then the most stages (4..2) that still
    // fit them. Measured: 4 CTAs with 2-3 stages streamed slower than 2 CTAs with 3-4 stages for every type but Q6_K.
    a.S = 0;
    for (int c = D::MINB; c >= 2 && a.S == 0; c--) {
        const int lim = 233472 / c - 1024 - 256;
        for (int st = 4; st >= 2; st--) {
            if (kBarBytes + st * a.stage_bytes + scr + red <= lim) {
                a.S = st;
                break;
            }
        }
    }
    if (a.S == 0) a.S = 2;
    a.scr_off         = kBarBytes + a.S * a.stage_bytes;
    a.red_off         = a.scr_off + scr;
    const size_t smem = (size_t) a.red_off + red;
    if (smem > 200 * 1024 || a.Wbox > 1024) return SRHPM_ERR_INVALID;

    CUtensorMap wmap;
    memset(&wmap, 0, sizeof(wmap));
    if (a.rows_main > 0) {
        EncodeTiled enc = encode_fn();
        if (!enc) return SRHPM_ERR_CUDA;
        const cuuint64_t dims[2]    = { (cuuint64_t) (a.G * a.row_bytes / 4), (cuuint64_t) (a.rows / a.G) };
        const cuuint64_t strides[1] = { (cuuint64_t) (a.G * a.row_bytes) };
        const cuuint32_t box[2]     = { (cuuint32_t) (a.Wbox / 4), (cuuint32_t) (kTileRows / a.G) };
        const cuuint32_t estr[2]    = { 1, 1 };
        const CUresult   r = enc(&wmap, CU_TENSOR_MAP_DATA_TYPE_UINT32, 2, const_cast<uint8_t *>(a.W), dims, strides,
                                 box, estr, CU_TENSOR_MAP_INTERLEAVE_NONE, CU_TENSOR_MAP_SWIZZLE_NONE,
                                 CU_TENSOR_MAP_L2_PROMOTION_L2_256B, CU_TENSOR_MAP_FLOAT_OOB_FILL_NONE);
        if (r != CUDA_SUCCESS) return SRHPM_ERR_INVALID;
    }

    auto kern = srv_gemm_kernel<D, NG, DBG>;
    // the shared-memory opt-in is per kernel and per device; every configuration needs under 200 KB
    static std::atomic<unsigned> attr_done{ 0 };
    int                          dev = 0;
    cudaGetDevice(&dev);
    if (!(attr_done.load() & (1u << (dev & 31)))) {
        const int st = cuda_status(cudaFuncSetAttribute(kern, cudaFuncAttributeMaxDynamicSharedMemorySize, 200 * 1024));
        if (st != SRHPM_OK) return st;
        attr_done.fetch_or(1u << (dev & 31));
    }
    int per_sm = 0;
    cudaOccupancyMaxActiveBlocksPerMultiprocessor(&per_sm, kern, kThreads, smem);
    const int     slots  = std::max(1, per_sm) * ctx->num_sms;
    const int64_t nrb    = (a.rows + kTileRows - 1) / kTileRows;
    cudaLaunchConfig_t cfg = {};
    cfg.blockDim           = dim3(kThreads);
    cfg.dynamicSmemBytes   = smem;
    cfg.stream             = stream;
    cudaLaunchAttribute attr[2];
    attr[0].id                                         = cudaLaunchAttributeProgrammaticStreamSerialization;
    attr[0].val.programmaticStreamSerializationAllowed = 1;
    attr[1].id                                         = cudaLaunchAttributeClusterDimension;
    attr[1].val.clusterDim.y                           = 1;
    attr[1].val.clusterDim.z                           = 1;
    cfg.attrs                                          = attr;
    // CTA slots usable by clusters of ks CTAs (placed whole inside a GPC, so maybe fewer than single CTAs); cached
    // per (device, kernel, shared memory, ks)
    auto cluster_slots = [&](int ks) -> int {
        static std::mutex                            mu;
        static std::map<std::tuple<int, size_t, int>, int> cache;
        const auto                                   key = std::make_tuple(dev, smem, ks);
        {
            std::lock_guard<std::mutex> lk(mu);
            const auto                  it = cache.find(key);
            if (it != cache.end()) return it->second;
        }
        attr[1].val.clusterDim.x = (unsigned) ks;
        cfg.gridDim              = dim3((unsigned) ks);
        cfg.numAttrs             = 2;
        int clusters             = 0;
        if (cudaOccupancyMaxActiveClusters(&clusters, kern, &cfg) != cudaSuccess) {
            cudaGetLastError();
            clusters = 0;
        }
        const int v = std::min(slots, clusters * ks);
        std::lock_guard<std::mutex> lk(mu);
        cache[key] = v;
        return v;
    };
    // split K so that the units fill the resident CTA slots in ONE round (measured: two rounds of half-size units
    // cost far more than one round of full ones). In units of a full-K row block a one-round split of ks ranges takes
    // about 1 / ks plus its epilogue: ~0.10 when the K ranges of a row block form a cluster and reduce in distributed
    // shared memory (if cluster occupancy holds all units), ~0.18 through global memory (fence, arrival counter,
    // reduction). Take the cheapest (the fewest ranges among equals), K ranges of >= 2 super-blocks. Products with a
    // row block for every slot are not split.
    a.ksplit  = 1;
    a.cluster = 0;
    int usable = slots;
    if (!DBG && a.part && nrb < slots) {
        const int most = std::max(1, std::min(kMaxSplit, a.nsb / 2));
        double    best = 1.0;  // ks = 1: one round of full-K units
        for (int ks = 2; ks <= most; ks++) {
            const int     sbs   = (a.nsb + ks - 1) / ks;
            const int     eff   = (a.nsb + sbs - 1) / sbs;  // non-empty ranges
            const int64_t units = nrb * eff;
            int           cl    = -1;
            if (eff > 1 && units <= cluster_slots(eff)) {
                cl = 1;
            } else if (units <= slots) {
                cl = 0;
            }
            if (cl < 0 || eff < 2) continue;
            const double cost = 1.0 / eff + (cl ? 0.10 : 0.18);
            if (cost < best * 0.999) {
                best      = cost;
                a.ksplit  = eff;
                a.cluster = cl;
                usable    = cl ? cluster_slots(eff) : slots;
            }
        }
    }
    a.kr_sbs = (a.nsb + a.ksplit - 1) / a.ksplit;
    a.units  = (int) (nrb * a.ksplit);
    attr[1].val.clusterDim.x = (unsigned) a.ksplit;
    cfg.numAttrs             = a.cluster ? 2 : 1;
    // persistent grid: balanced rounds, a multiple of the K ranges
    const int rounds = (a.units + usable - 1) / usable;
    int       grid   = (a.units + rounds - 1) / rounds;
    grid             = (grid + a.ksplit - 1) / a.ksplit * a.ksplit;
    cfg.gridDim      = dim3((unsigned) grid);
    // activations: quantized in the GEMM's own prologue (one launch per product) when the grid's consumer warps get
    // at most two (super-block, token) jobs each; else by the separate quantizer kernel first (a.X null: the records
    // were written by a fused norm / SwiGLU prologue)
    if (a.fq && (int64_t) a.nsb * a.N > 2LL * grid * kNCW) a.fq = 0;
    if (a.X && !a.fq) {
        const int st = launch_quantizer(ctx, a, 8 * NG, D::Q80, stream);
        if (st != SRHPM_OK) return st;
    }
    ctx->launches.fetch_add(1);
    return cuda_status(cudaLaunchKernelEx(&cfg, kern, wmap, a));
}

template <class D>
int dispatch_ng(srhpm_ctx * ctx, const GemmArgs & a, bool dbg, cudaStream_t stream) {
    if (a.N <= 8) {
        return dbg ? launch_gemm<D, 1, true>(ctx, a, stream) : launch_gemm<D, 1, false>(ctx, a, stream);
    }
    return dbg ? launch_gemm<D, 2, true>(ctx, a, stream) : launch_gemm<D, 2, false>(ctx, a, stream);
}

uint8_t * align256(void * p) {
    return reinterpret_cast<uint8_t *>((reinterpret_cast<uintptr_t>(p) + 255) & ~uintptr_t(255));
}


}  // namespace

// work buffer: [activation records][split-K partials][split-K counters]
struct WorkLayout {
    size_t recs, part, cnt, total;
};

WorkLayout work_layout(int wtype, int64_t rows, int64_t K, int64_t N) {
    const int  NT  = N <= 8 ? 8 : 16;
    WorkLayout w   = {};
    w.recs         = 0;
    w.part         = ((size_t) (K / QK) * rec_bytes(wtype == SRHPM_TYPE_Q8_0, NT) + 255) / 256 * 256;
    // the most K ranges a product can be split into: kMaxSplit, or more when the direct kernel's resident records of
    // a K range would exceed ~50 KB
    const int     max_sbs = std::max(1, (50 * 1024) / rec_bytes(wtype == SRHPM_TYPE_Q8_0, NT));
    const int64_t splits  = std::max<int64_t>(kMaxSplit, (K / QK + max_sbs - 1) / max_sbs);
    w.cnt          = w.part + ((size_t) splits * N * rows * 4 + 255) / 256 * 256;
    const int64_t nrb = (rows + kTileRows - 1) / kTileRows;
    w.total        = w.cnt + (size_t) nrb * 4 + 256;  // + 256: room to align the caller's pointer
    return w;
}

// the same buffer without split-K partials (products are not split along K)
WorkLayout work_layout_unsplit(int wtype, int64_t rows, int64_t K, int64_t N) {
    WorkLayout w      = work_layout(wtype, rows, K, N);
    const size_t cnts = w.total - w.cnt;
    w.cnt             = w.part;
    w.total           = w.cnt + cnts;
    return w;
}

size_t gemm_work_size(int wtype, int64_t rows, int64_t K, int64_t N) { return work_layout(wtype, rows, K, N).total; }

size_t gemm_work_size_unsplit(int wtype, int64_t rows, int64_t K, int64_t N) {
    return work_layout_unsplit(wtype, rows, K, N).total;
}

namespace {

// the arrival counter of the grids that use this work buffer (one per buffer, so that calls with different buffers
// may run concurrently on other streams); null when the context's table is full
uint32_t * sync_counter(srhpm_ctx * ctx, const void * work) {
    if (!ctx->d_sync) return nullptr;
    std::lock_guard<std::mutex> lk(ctx->sync_mu);
    const uintptr_t             key = reinterpret_cast<uintptr_t>(work);
    const auto                  it  = ctx->sync_slots.find(key);
    if (it != ctx->sync_slots.end()) return ctx->d_sync + it->second;
    if (ctx->sync_next >= kSyncSlots) return nullptr;
    const int slot        = ctx->sync_next++;
    ctx->sync_slots[key] = slot;
    return ctx->d_sync + slot;
}

int gemm_run_impl(srhpm_ctx * ctx, int wtype, const uint8_t * W, int64_t rows, int64_t K, size_t row_bytes,
                  const float * X, int64_t ldx, int64_t N, float * Y, int64_t ldy, void * wdata, size_t wsize,
                  int32_t * isum, int32_t * imin, bool split, cudaStream_t stream, bool prequant = false,
                  bool fused_ok = false, const float * X2 = nullptr) {
    const WorkLayout wl = split ? work_layout(wtype, rows, K, N) : work_layout_unsplit(wtype, rows, K, N);
    if (wsize < wl.total || !wdata) return SRHPM_ERR_WORKSPACE;
    const int  nsb  = (int) (K / QK);
    const bool q80  = wtype == SRHPM_TYPE_Q8_0;
    uint8_t *  base = align256(wdata);
    uint8_t *  recs = base + wl.recs;
    int32_t *  cnt  = reinterpret_cast<int32_t *>(base + wl.cnt);
    const int  nrb  = (int) ((rows + kTileRows - 1) / kTileRows);
    // the activation records (and zeroed split-K counters) come from the GEMM's own prologue or a quantizer kernel
    // launched just before it (launch_gemm); prequant: written by the preceding fused norm / SwiGLU
    GemmArgs a  = {};
    if (!prequant) {
        a.X       = X;
        a.X2      = X2;
        a.ldx     = ldx;
        a.perm    = record_perm(wtype);
        a.q80mode = ctx->q8_0_act_mode;
        a.ncnt    = nrb;
        a.fq      = fused_ok ? 1 : 0;
        if (a.fq) {
            a.sync = sync_counter(ctx, recs);
            if (!a.sync) a.fq = 0;
        }
    }
    a.W         = W;
    a.rows      = rows;
    a.row_bytes = (int64_t) row_bytes;
    a.w_bytes   = rows * (int64_t) row_bytes;
    a.nsb       = nsb;
    a.recs      = recs;
    a.part      = split ? reinterpret_cast<float *>(base + wl.part) : nullptr;  // null: one K range
    a.cnt       = cnt;
    a.Y         = Y;
    a.ldy       = ldy;
    a.N         = (int) N;
    a.status    = ctx->d_status;
    a.isum      = isum;
    a.imin      = imin;
    a.nblk      = q80 ? nsb * 8 : nsb;
    const bool dbg = isum != nullptr;
    switch (wtype) {
        case SRHPM_TYPE_Q4_K: return dispatch_ng<DecK45<false>>(ctx, a, dbg, stream);
        case SRHPM_TYPE_Q5_K: return dispatch_ng<DecK45<true>>(ctx, a, dbg, stream);
        case SRHPM_TYPE_Q6_K: return dispatch_ng<DecQ6K>(ctx, a, dbg, stream);
        case SRHPM_TYPE_Q3_K: return dispatch_ng<DecQ3K>(ctx, a, dbg, stream);
        case SRHPM_TYPE_IQ4_XS: return dispatch_ng<DecIQ4XS>(ctx, a, dbg, stream);
        case SRHPM_TYPE_Q8_0: return dispatch_ng<DecQ80>(ctx, a, dbg, stream);
        default: return SRHPM_UNSUPPORTED;
    }
}

}  // namespace

int gemm_run_prequant(srhpm_ctx * ctx, int wtype, const uint8_t * W, int64_t rows, int64_t K, size_t row_bytes,
                      int64_t N, float * Y, int64_t ldy, void * wdata, size_t wsize, cudaStream_t stream) {
    if (wtype == SRHPM_TYPE_Q8_0) return SRHPM_UNSUPPORTED;
    return gemm_run_impl(ctx, wtype, W, rows, K, row_bytes, nullptr, K, N, Y, ldy, wdata, wsize, nullptr, nullptr,
                         true, stream, true);
}

int norm_quant_run(srhpm_ctx * ctx, int wtype, int64_t rows, int64_t K, int64_t N, float * x, const float * delta,
                   const float * w, float eps, float * y, void * wdata, size_t wsize, cudaStream_t stream,
                   const uint64_t * peers, int world, int rank, int slot, uint32_t * epochs) {
    if (wtype == SRHPM_TYPE_Q8_0) return SRHPM_UNSUPPORTED;
    if (K % QK != 0 || K > 4 * 4 * kNormQThreads || N < 1 || N > 16) return SRHPM_ERR_INVALID;
    if (peers && (N > kArRows || world < 1 || world > kArMaxRanks || rank < 0 || rank >= world || slot < 0 ||
                  slot > 1 || !epochs)) {
        return SRHPM_ERR_INVALID;
    }
    const NormAr ar = { peers, world, rank, slot, epochs, ctx->d_status };
    const WorkLayout wl = work_layout(wtype, rows, K, N);
    if (wsize < wl.total || !wdata) return SRHPM_ERR_WORKSPACE;
    uint8_t * base = align256(wdata);
    const int NT   = N <= 8 ? 8 : 16;
    const int nrb  = (int) ((rows + kTileRows - 1) / kTileRows);
    static std::atomic<unsigned> attr_done{ 0 };
    int                          dev = 0;
    cudaGetDevice(&dev);
    if (!(attr_done.load() & (1u << (dev & 31)))) {
        const int st = cuda_status(cudaFuncSetAttribute(add_rms_norm_q8K_kernel,
                                                        cudaFuncAttributeMaxDynamicSharedMemorySize, 64 * 1024));
        if (st != SRHPM_OK) return st;
        attr_done.fetch_or(1u << (dev & 31));
    }
    cudaError_t e;
    if (peers) {  // a cluster of kArC CTAs per row (compile-time cluster shape)
        e = launch_k_pdl(add_rms_norm_ar_q8K_kernel, dim3(kArC, NT), dim3(kArCT), 0, stream, x, w, eps, y, (int) N, K,
                         NT, base + wl.recs, record_perm(wtype), reinterpret_cast<int32_t *>(base + wl.cnt), nrb, ar);
    } else {
        e = launch_k_pdl(add_rms_norm_q8K_kernel, dim3(NT), dim3(kNormQThreads), (size_t) K * 4, stream, x, delta, w,
                         eps, y, (int) N, K, NT, base + wl.recs, record_perm(wtype),
                         reinterpret_cast<int32_t *>(base + wl.cnt), nrb);
    }
    ctx->launches.fetch_add(1);
    return cuda_status(e);
}

int swiglu_quant_run(srhpm_ctx * ctx, int wtype, int64_t rows, int64_t K, int64_t N, const float * gate,
                     const float * up, int64_t ld_in, float * h, int64_t ld_out, void * wdata, size_t wsize,
                     cudaStream_t stream) {
    if (wtype == SRHPM_TYPE_Q8_0) return SRHPM_UNSUPPORTED;
    if (K % QK != 0 || N < 1 || N > 16) return SRHPM_ERR_INVALID;
    const WorkLayout wl = work_layout(wtype, rows, K, N);
    if (wsize < wl.total || !wdata) return SRHPM_ERR_WORKSPACE;
    uint8_t *     base   = align256(wdata);
    const int     NT     = N <= 8 ? 8 : 16;
    const int     nrb    = (int) ((rows + kTileRows - 1) / kTileRows);
    const int     nsb    = (int) (K / QK);
    const int64_t warps  = (int64_t) nsb * NT;
    const int     blocks = (int) ((warps + 7) / 8);
    const cudaError_t e = launch_k_pdl(swiglu_q8K_kernel, dim3(blocks), dim3(256), 0, stream, gate, up, ld_in, h,
                                       ld_out, (int) N, nsb, NT, base + wl.recs, record_perm(wtype),
                                       reinterpret_cast<int32_t *>(base + wl.cnt), nrb);
    ctx->launches.fetch_add(1);
    return cuda_status(e);
}

int gemm_run(srhpm_ctx * ctx, int wtype, const uint8_t * W, int64_t rows, int64_t K, size_t row_bytes,
             const float * X, int64_t ldx, int64_t N, float * Y, int64_t ldy, void * wdata, size_t wsize,
             int32_t * isum, int32_t * imin, cudaStream_t stream, bool fused_quant) {
    return gemm_run_impl(ctx, wtype, W, rows, K, row_bytes, X, ldx, N, Y, ldy, wdata, wsize, isum, imin, true, stream,
                         false, fused_quant);
}

int gemm_run_swiglu(srhpm_ctx * ctx, int wtype, const uint8_t * W, int64_t rows, int64_t K, size_t row_bytes,
                    const float * gate, const float * up, int64_t ld_in, int64_t N, float * Y, int64_t ldy,
                    void * wdata, size_t wsize, cudaStream_t stream) {
    if (wtype == SRHPM_TYPE_Q8_0) return SRHPM_UNSUPPORTED;  // the SwiGLU record writer is the q8_K one
    return gemm_run_impl(ctx, wtype, W, rows, K, row_bytes, gate, ld_in, N, Y, ldy, wdata, wsize, nullptr, nullptr,
                         true, stream, false, true, up);
}

int gemm_run_unsplit(srhpm_ctx * ctx, int wtype, const uint8_t * W, int64_t rows, int64_t K, size_t row_bytes,
                     const float * X, int64_t ldx, int64_t N, float * Y, int64_t ldy, void * wdata, size_t wsize,
                     cudaStream_t stream) {
    return gemm_run_impl(ctx, wtype, W, rows, K, row_bytes, X, ldx, N, Y, ldy, wdata, wsize, nullptr, nullptr, false,
                         stream);
}

int quantize_q8K_dense(srhpm_ctx * ctx, const float * X, int64_t ldx, int64_t N, int64_t K, int8_t * q, float * d,
                       int16_t * b32, int16_t * b16, cudaStream_t stream) {
    const int     nsb    = (int) (K / QK);
    const int64_t warps  = (int64_t) nsb * N;
    const int     blocks = (int) ((warps + 7) / 8);
    quant_q8K_kernel<true><<<blocks, 256, 0, stream>>>(X, ldx, (int) N, nsb, 0, nullptr, q, d, b32, b16,
                                                       nullptr, 0, 0);
    ctx->launches.fetch_add(1);
    return cuda_status(cudaGetLastError());
}

int quantize_q8_0_dense(srhpm_ctx * ctx, const float * X, int64_t ldx, int64_t N, int64_t K, void * blocks,
                        cudaStream_t stream) {
    const int     nsb    = (int) (K / QK);
    const int64_t warps  = (int64_t) nsb * N;
    const int     nblk   = (int) ((warps + 7) / 8);
    quant_q80_kernel<true><<<nblk, 256, 0, stream>>>(X, ldx, (int) N, nsb, 0, ctx->q8_0_act_mode, nullptr,
                                                     reinterpret_cast<uint8_t *>(blocks), nullptr, 0);
    ctx->launches.fetch_add(1);
    return cuda_status(cudaGetLastError());
}

}  // namespace srhpm
