// Small-batch quantized matmul for speculative verification on sm_100a (the GPU counterpart of the reference's
// SRV kernels, patch/srhpm.patch:5448-6680, and of its dGPU co-verifier, dgpu/dgpu.cu:107-191).
//
// Y[t][r] = sum_k W[r][k] X[t][k] for N = 1..16 activation rows against GGUF-packed weight rows.
//
//   1. quant_q8K_kernel / quant_q80_kernel: each activation row is quantized per 256 columns to int8 with one f32
//      scale (bit-identical to srv_quantize_row, patch/srhpm.patch:5518-5575) -- or per 32 columns to q8_0 for Q8_0
//      weights -- into "activation records": for each super-block, NT = 8 or 16 token rows of 256 int8 values at a
//      288-byte stride (so that consecutive tokens fall on different shared-memory banks), then the scales.
//   2. srv_gemm_kernel: one CTA per 64-row tile. A producer warp streams the tile through a 4-stage shared-memory
//      ring, kc super-blocks at a time: one 1-D bulk async copy per weight row (16-byte aligned, ragged bytes at the
//      very end of the matrix copied by hand) plus one copy of the kc activation records, completion counted on an
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

#include "internal.h"
#include "ptx.cuh"

namespace srhpm {
namespace {

constexpr int     QK         = 256;
constexpr int     kNCW       = 4;                 // consumer warps
constexpr int     kThreads   = (kNCW + 1) * 32;   // + 1 producer warp
constexpr int     kTileRows  = 16 * kNCW;         // weight rows per CTA
constexpr int     kTokStride = 288;               // bytes per token row inside an activation record
constexpr int     kStages    = 4;
constexpr int     kBarBytes  = 128;               // room for the 2 * kStages mbarriers

__host__ __device__ constexpr int rec_nscales(bool q80, int NT) { return q80 ? 8 * NT : NT; }
__host__ __device__ constexpr int rec_bytes(bool q80, int NT) {
    return (NT * kTokStride + 4 * rec_nscales(q80, NT) + 15) / 16 * 16;
}

struct GemmArgs {
    const uint8_t * W;
    int64_t         rows;
    int64_t         row_bytes;
    int64_t         w_bytes;     // valid bytes of W (rows * row_bytes)
    int             nsb;         // 256-column super-blocks per row
    int             kc;          // super-blocks per stage
    int             SR;          // shared-memory bytes per weight row slot
    int             stage_bytes;
    const uint8_t * recs;        // activation records, nsb of them
    float *         Y;
    int64_t         ldy;         // elements
    int             N;
    int32_t *       status;
    int32_t *       isum;        // integer outputs (srhpm_mul_mat_isums), else null
    int32_t *       imin;
    int             nblk;        // blocks per row in the integer outputs
};

// ---------------------------------------------------------------------------------------------------------------
// activation quantizers

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
template <bool DENSE>
__global__ void __launch_bounds__(256) quant_q8K_kernel(const float * __restrict__ X, int64_t ldx, int N, int nsb,
                                                         int NT, uint8_t * __restrict__ recs, int8_t * __restrict__ q,
                                                         float * __restrict__ d, int16_t * __restrict__ b32,
                                                         int16_t * __restrict__ b16) {
    pdl_launch_dependents();
    const int     lane = threadIdx.x & 31;
    const int     TT   = DENSE ? N : NT;
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
    float amax = 0.0f;
#pragma unroll
    for (int j = 0; j < 8; j++) amax = fmaxf(amax, fabsf(v[j]));
#pragma unroll
    for (int o = 16; o > 0; o >>= 1) amax = fmaxf(amax, __shfl_xor_sync(0xffffffffu, amax, o));
    int   qv[8];
    float dv = 0.0f;
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
    const uint2 pk = pack8(qv);
    if constexpr (DENSE) {
        const int64_t K = (int64_t) nsb * QK;
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
        uint8_t * rec = recs + (size_t) sb * rec_bytes(false, NT);
        *reinterpret_cast<uint2 *>(rec + t * kTokStride + 8 * lane) = pk;
        if (lane == 0) reinterpret_cast<float *>(rec + NT * kTokStride)[t] = dv;
    }
}

// q8_0 quantizer, per 32 columns (4 lanes per block): d = amax / 127 stored as f16. SIMD mode: id = 127 / amax,
// q = round_half_even(x * id); REF mode: id = 1 / d (f32 d), q = roundf(x * id).
template <bool DENSE>
__global__ void __launch_bounds__(256) quant_q80_kernel(const float * __restrict__ X, int64_t ldx, int N, int nsb,
                                                         int NT, int mode, uint8_t * __restrict__ recs,
                                                         uint8_t * __restrict__ blocks) {
    pdl_launch_dependents();
    const int     lane = threadIdx.x & 31;
    const int     TT   = DENSE ? N : NT;
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
    float amax = 0.0f;
#pragma unroll
    for (int j = 0; j < 8; j++) amax = fmaxf(amax, fabsf(v[j]));
    amax = fmaxf(amax, __shfl_xor_sync(0xffffffffu, amax, 1));
    amax = fmaxf(amax, __shfl_xor_sync(0xffffffffu, amax, 2));
    const float  dd = __fdiv_rn(amax, 127.0f);
    const __half dh = __float2half_rn(dd);
    int          qv[8];
    if (mode == SRHPM_Q8_0_ACT_SIMD) {
        const float id = amax != 0.0f ? __fdiv_rn(127.0f, amax) : 0.0f;
#pragma unroll
        for (int j = 0; j < 8; j++) qv[j] = __float2int_rn(__fmul_rn(v[j], id));
    } else {
        const float id = dd != 0.0f ? __fdiv_rn(1.0f, dd) : 0.0f;
#pragma unroll
        for (int j = 0; j < 8; j++) qv[j] = (int) roundf(__fmul_rn(v[j], id));
    }
    const uint2 pk  = pack8(qv);
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
        uint8_t * rec = recs + (size_t) sb * rec_bytes(true, NT);
        *reinterpret_cast<uint2 *>(rec + t * kTokStride + 8 * lane) = pk;
        if ((lane & 3) == 0) reinterpret_cast<float *>(rec + NT * kTokStride)[blk * NT + t] = __half2float(dh);
    }
}

// ---------------------------------------------------------------------------------------------------------------
// per-type super-block decoders. sb<NG>() consumes one super-block of rows (g, g+8) of the warp's 16-row slice:
// wa / wb point at the two rows' blocks in shared memory, xr at the super-block's activation record.

__device__ __forceinline__ uint32_t lds32(const uint8_t * p) { return *reinterpret_cast<const uint32_t *>(p); }
__device__ __forceinline__ uint2    lds64(const uint8_t * p) { return *reinterpret_cast<const uint2 *>(p); }
__device__ __forceinline__ float    ldh(const uint8_t * p) { return half_bits_to_float(lds_u16(p)); }

__device__ __forceinline__ uint32_t prmt(uint32_t a, uint32_t b, uint32_t sel) {
    uint32_t r;
    asm("prmt.b32 %0, %1, %2, %3;" : "=r"(r) : "r"(a), "r"(b), "r"(sel));
    return r;
}
__device__ __forceinline__ int ubyte(uint32_t w, int j) { return (int) ((w >> (8 * j)) & 0xffu); }
__device__ __forceinline__ int sbyte(uint32_t w, int j) { return ((int32_t) (w << (24 - 8 * j))) >> 24; }

// per-byte a - k for bytes holding 0..127 (no borrow between bytes)
__device__ __forceinline__ uint32_t vsub_small(uint32_t a, uint32_t k) { return ((a | 0x80808080u) - k) ^ 0x80808080u; }

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

// f32 update of one super-block: acc += (d_row * x_tok) * isum  [- (dmin_row * x_tok) * imin]
template <int NG, bool MIN>
__device__ __forceinline__ void sb_update(float (&acc)[NG][4], const int (&im)[NG][4], const int (&in)[NG][4],
                                          float dA, float dB, float mA, float mB, const float * xs, int t) {
#pragma unroll
    for (int grp = 0; grp < NG; grp++) {
        const float x0 = xs[8 * grp + 2 * t], x1 = xs[8 * grp + 2 * t + 1];
        acc[grp][0] += (dA * x0) * (float) im[grp][0];
        acc[grp][1] += (dA * x1) * (float) im[grp][1];
        acc[grp][2] += (dB * x0) * (float) im[grp][2];
        acc[grp][3] += (dB * x1) * (float) im[grp][3];
        if constexpr (MIN) {
            acc[grp][0] -= (mA * x0) * (float) in[grp][0];
            acc[grp][1] -= (mA * x1) * (float) in[grp][1];
            acc[grp][2] -= (mB * x0) * (float) in[grp][2];
            acc[grp][3] -= (mB * x1) * (float) in[grp][3];
        }
    }
}

// Q4_K (144 B: d, dmin, 12 bytes of 6-bit scales/mins, 128 bytes of nibbles) and Q5_K (176 B: + 32 bytes of 5th
// bits before the nibbles). Pair p of sub-blocks (2p, 2p+1) shares 32 code bytes: low nibble = sub-block 2p, high
// nibble = sub-block 2p+1; the 5th bit of sub-block b, weight l is bit b of qh[l].
template <bool Q5>
struct DecK45 {
    static constexpr int  BS  = Q5 ? 176 : 144;
    static constexpr bool Q80 = false;
    static constexpr int  QS  = Q5 ? 48 : 16;

    __device__ __forceinline__ static uint32_t hbit(uint32_t qh, int b) { return ((qh >> b) << 4) & 0x10101010u; }

    template <int NG, bool DBG>
    __device__ __forceinline__ static void sb(const uint8_t * wa, const uint8_t * wb, const uint8_t * xr, int lane,
                                              float (&acc)[NG][4], const DbgOut & dbg, int64_t rg, int sbi) {
        constexpr int NT = 8 * NG;
        const int     t = lane & 3, g = lane >> 2;
        const uint32_t a0w = lds32(wa + 4), a1w = lds32(wa + 8), a2w = lds32(wa + 12);
        const uint32_t b0w = lds32(wb + 4), b1w = lds32(wb + 8), b2w = lds32(wb + 12);
        // 6-bit scales of sub-blocks 0..3 / 4..7 and mins, one byte each
        const uint32_t scA[2] = { a0w & 0x3F3F3F3Fu, (a2w & 0x0F0F0F0Fu) | ((a0w >> 2) & 0x30303030u) };
        const uint32_t mnA[2] = { a1w & 0x3F3F3F3Fu, ((a2w >> 4) & 0x0F0F0F0Fu) | ((a1w >> 2) & 0x30303030u) };
        const uint32_t scB[2] = { b0w & 0x3F3F3F3Fu, (b2w & 0x0F0F0F0Fu) | ((b0w >> 2) & 0x30303030u) };
        const uint32_t mnB[2] = { b1w & 0x3F3F3F3Fu, ((b2w >> 4) & 0x0F0F0F0Fu) | ((b1w >> 2) & 0x30303030u) };
        uint2 ha = make_uint2(0, 0), hb = make_uint2(0, 0);
        if constexpr (Q5) {
            ha = lds64(wa + 16 + 8 * t);
            hb = lds64(wb + 16 + 8 * t);
        }
        int im[NG][4], in[NG][4];
#pragma unroll
        for (int grp = 0; grp < NG; grp++) {
#pragma unroll
            for (int e = 0; e < 4; e++) im[grp][e] = in[grp][e] = 0;
        }
#pragma unroll
        for (int p = 0; p < 4; p++) {
            const uint2 va = lds64(wa + QS + 32 * p + 8 * t);
            const uint2 vb = lds64(wb + QS + 32 * p + 8 * t);
#pragma unroll
            for (int h = 0; h < 2; h++) {
                const int b  = 2 * p + h;
                uint32_t  a0 = (va.x >> (4 * h)) & 0x0F0F0F0Fu, a2 = (va.y >> (4 * h)) & 0x0F0F0F0Fu;
                uint32_t  a1 = (vb.x >> (4 * h)) & 0x0F0F0F0Fu, a3 = (vb.y >> (4 * h)) & 0x0F0F0F0Fu;
                if constexpr (Q5) {
                    a0 |= hbit(ha.x, b);
                    a2 |= hbit(ha.y, b);
                    a1 |= hbit(hb.x, b);
                    a3 |= hbit(hb.y, b);
                }
                const int      sA = ubyte(scA[b >> 2], b & 3), sB = ubyte(scB[b >> 2], b & 3);
                const uint32_t mA = prmt(mnA[b >> 2], 0, 0x1111u * (b & 3));
                const uint32_t mB = prmt(mnB[b >> 2], 0, 0x1111u * (b & 3));
#pragma unroll
                for (int grp = 0; grp < NG; grp++) {
                    const uint2 x = lds64(xr + (8 * grp + g) * kTokStride + 32 * b + 8 * t);
                    int         c[4] = { 0, 0, 0, 0 };
                    mma_k32<true>(c, a0, a1, a2, a3, x.x, x.y);
                    im[grp][0] += sA * c[0];
                    im[grp][1] += sA * c[1];
                    im[grp][2] += sB * c[2];
                    im[grp][3] += sB * c[3];
                    mma_k32<true>(in[grp], mA, mB, mA, mB, x.x, x.y);
                }
            }
        }
        if constexpr (DBG) {
            dbg_store<NG>(dbg, im, false, rg, sbi, lane);
            dbg_store<NG>(dbg, in, true, rg, sbi, lane);
        } else {
            const float * xs = reinterpret_cast<const float *>(xr + NT * kTokStride);
            sb_update<NG, true>(acc, im, in, ldh(wa), ldh(wb), ldh(wa + 2), ldh(wb + 2), xs, t);
        }
    }
};

// Q6_K (210 B: 128 bytes low nibbles, 64 bytes of 2-bit highs, 16 int8 scales per 16 weights, d). Weight
// 128n + 32j + l: nibble (j >> 1) of ql[64n + 32(j & 1) + l], bits 2j of qh[32n + l], minus 32; scale 8n + 2j + l/16.
// One k16 MMA per 16-weight group.
struct DecQ6K {
    static constexpr int  BS  = 210;
    static constexpr bool Q80 = false;

    template <int NG, bool DBG>
    __device__ __forceinline__ static void sb(const uint8_t * wa, const uint8_t * wb, const uint8_t * xr, int lane,
                                              float (&acc)[NG][4], const DbgOut & dbg, int64_t rg, int sbi) {
        constexpr int NT = 8 * NG;
        const int     t = lane & 3, g = lane >> 2;
        uint32_t      SA[4], SB[4];
#pragma unroll
        for (int i = 0; i < 4; i++) {
            SA[i] = lds_u32_a2(wa + 192 + 4 * i);
            SB[i] = lds_u32_a2(wb + 192 + 4 * i);
        }
        int im[NG][4], in[NG][4];
#pragma unroll
        for (int grp = 0; grp < NG; grp++) {
#pragma unroll
            for (int e = 0; e < 4; e++) im[grp][e] = in[grp][e] = 0;
        }
#pragma unroll
        for (int n = 0; n < 2; n++) {
#pragma unroll
            for (int h = 0; h < 2; h++) {
                const int      off = 16 * h + 4 * t;
                const uint32_t l0a = lds_u32_a2(wa + 64 * n + off), l1a = lds_u32_a2(wa + 64 * n + 32 + off);
                const uint32_t l0b = lds_u32_a2(wb + 64 * n + off), l1b = lds_u32_a2(wb + 64 * n + 32 + off);
                const uint32_t qha = lds_u32_a2(wa + 128 + 32 * n + off), qhb = lds_u32_a2(wb + 128 + 32 * n + off);
#pragma unroll
                for (int j = 0; j < 4; j++) {
                    const uint32_t la = (j & 1) ? l1a : l0a, lb = (j & 1) ? l1b : l0b;
                    const int      sh = 4 * (j >> 1);
                    uint32_t       ua = ((la >> sh) & 0x0F0F0F0Fu) | (((qha >> (2 * j)) & 0x03030303u) << 4);
                    uint32_t       ub = ((lb >> sh) & 0x0F0F0F0Fu) | (((qhb >> (2 * j)) & 0x03030303u) << 4);
                    ua                = vsub_small(ua, 0x20202020u);
                    ub                = vsub_small(ub, 0x20202020u);
                    const int is = 8 * n + 2 * j + h;
                    const int sA = sbyte(SA[is >> 2], is & 3), sB = sbyte(SB[is >> 2], is & 3);
                    const int b  = 4 * n + j;
#pragma unroll
                    for (int grp = 0; grp < NG; grp++) {
                        const uint32_t x    = lds32(xr + (8 * grp + g) * kTokStride + 32 * b + off);
                        int            c[4] = { 0, 0, 0, 0 };
                        mma_k16<false>(c, ua, ub, x);
                        im[grp][0] += sA * c[0];
                        im[grp][1] += sA * c[1];
                        im[grp][2] += sB * c[2];
                        im[grp][3] += sB * c[3];
                    }
                }
            }
        }
        if constexpr (DBG) {
            dbg_store<NG>(dbg, im, false, rg, sbi, lane);
        } else {
            const float * xs = reinterpret_cast<const float *>(xr + NT * kTokStride);
            sb_update<NG, false>(acc, im, in, ldh(wa + 208), ldh(wb + 208), 0.f, 0.f, xs, t);
        }
    }
};

// Q3_K (110 B: 32 bytes of high bits, 64 bytes of 2-bit codes, 12 bytes of 6-bit scales, d). Weight 128n + 32j + l:
// bits 2j of qs[32n + l], high bit (4n + j) of hmask[l] (set = +0, clear = -4); scale index 8n + 2j + l/16, minus 32.
struct DecQ3K {
    static constexpr int  BS  = 110;
    static constexpr bool Q80 = false;

    template <int NG, bool DBG>
    __device__ __forceinline__ static void sb(const uint8_t * wa, const uint8_t * wb, const uint8_t * xr, int lane,
                                              float (&acc)[NG][4], const DbgOut & dbg, int64_t rg, int sbi) {
        constexpr int NT = 8 * NG;
        const int     t = lane & 3, g = lane >> 2;
        uint32_t      SA[4], SB[4];
        {
            const uint32_t s0 = lds_u32_a2(wa + 96), s1 = lds_u32_a2(wa + 100), s2 = lds_u32_a2(wa + 104);
            const uint32_t r0 = lds_u32_a2(wb + 96), r1 = lds_u32_a2(wb + 100), r2 = lds_u32_a2(wb + 104);
            const uint32_t loA[4] = { s0 & 0x0F0F0F0Fu, s1 & 0x0F0F0F0Fu, (s0 >> 4) & 0x0F0F0F0Fu, (s1 >> 4) & 0x0F0F0F0Fu };
            const uint32_t loB[4] = { r0 & 0x0F0F0F0Fu, r1 & 0x0F0F0F0Fu, (r0 >> 4) & 0x0F0F0F0Fu, (r1 >> 4) & 0x0F0F0F0Fu };
#pragma unroll
            for (int i = 0; i < 4; i++) {
                SA[i] = vsub_small(loA[i] | (((s2 >> (2 * i)) & 0x03030303u) << 4), 0x20202020u);
                SB[i] = vsub_small(loB[i] | (((r2 >> (2 * i)) & 0x03030303u) << 4), 0x20202020u);
            }
        }
        int im[NG][4], in[NG][4];
#pragma unroll
        for (int grp = 0; grp < NG; grp++) {
#pragma unroll
            for (int e = 0; e < 4; e++) im[grp][e] = in[grp][e] = 0;
        }
#pragma unroll
        for (int h = 0; h < 2; h++) {
            const int      off = 16 * h + 4 * t;
            const uint32_t hma = lds_u32_a2(wa + off), hmb = lds_u32_a2(wb + off);
#pragma unroll
            for (int n = 0; n < 2; n++) {
                const uint32_t qa = lds_u32_a2(wa + 32 + 32 * n + off), qb = lds_u32_a2(wb + 32 + 32 * n + off);
#pragma unroll
                for (int j = 0; j < 4; j++) {
                    const int      hs = 4 * n + j;
                    const uint32_t ua = vsub_small(((qa >> (2 * j)) & 0x03030303u) | (((hma >> hs) & 0x01010101u) << 2),
                                                   0x04040404u);
                    const uint32_t ub = vsub_small(((qb >> (2 * j)) & 0x03030303u) | (((hmb >> hs) & 0x01010101u) << 2),
                                                   0x04040404u);
                    const int is = 8 * n + 2 * j + h;
                    const int sA = sbyte(SA[is >> 2], is & 3), sB = sbyte(SB[is >> 2], is & 3);
                    const int b  = 4 * n + j;
#pragma unroll
                    for (int grp = 0; grp < NG; grp++) {
                        const uint32_t x    = lds32(xr + (8 * grp + g) * kTokStride + 32 * b + off);
                        int            c[4] = { 0, 0, 0, 0 };
                        mma_k16<false>(c, ua, ub, x);
                        im[grp][0] += sA * c[0];
                        im[grp][1] += sA * c[1];
                        im[grp][2] += sB * c[2];
                        im[grp][3] += sB * c[3];
                    }
                }
            }
        }
        if constexpr (DBG) {
            dbg_store<NG>(dbg, im, false, rg, sbi, lane);
        } else {
            const float * xs = reinterpret_cast<const float *>(xr + NT * kTokStride);
            sb_update<NG, false>(acc, im, in, ldh(wa + 108), ldh(wb + 108), 0.f, 0.f, xs, t);
        }
    }
};

// IQ4_XS (136 B: d, 2 high bits of 8 scales, 4 bits of 8 scales, 128 bytes of code-book indices). Sub-block b,
// weight l: index = nibble (l >= 16) of qs[16b + (l & 15)], value kvalues_iq4nl[index]; scale = 6 bits - 32.
struct DecIQ4XS {
    static constexpr int  BS  = 136;
    static constexpr bool Q80 = false;

    // the 16-entry code book as four words of int8 lanes (GGUF constant kvalues_iq4nl)
    static constexpr uint32_t T0 = 0xBFAD9881u, T1 = 0xF6EADDCFu, T2 = 0x26190D01u, T3 = 0x71594535u;

    // v holds 8 indices (byte j: low nibble = weight j, high nibble = weight j + 16) -> lo / hi value words
    __device__ __forceinline__ static void lookup(uint32_t v, uint32_t & lo, uint32_t & hi) {
        const uint32_t v7  = v & 0x77777777u;
        const uint32_t sel = 0x32103210u | ((v & 0x88888888u) >> 1);  // bit 2 set: take the upper table's byte
        const uint32_t r0  = prmt(prmt(T0, T1, v7), prmt(T2, T3, v7), sel & 0xffffu);
        const uint32_t r1  = prmt(prmt(T0, T1, v7 >> 16), prmt(T2, T3, v7 >> 16), sel >> 16);
        lo                 = prmt(r0, r1, 0x6420u);
        hi                 = prmt(r0, r1, 0x7531u);
    }

    template <int NG, bool DBG>
    __device__ __forceinline__ static void sb(const uint8_t * wa, const uint8_t * wb, const uint8_t * xr, int lane,
                                              float (&acc)[NG][4], const DbgOut & dbg, int64_t rg, int sbi) {
        constexpr int  NT = 8 * NG;
        const int      t = lane & 3, g = lane >> 2;
        const uint32_t HA = lds_u16(wa + 2), HB = lds_u16(wb + 2);
        const uint32_t LA = lds32(wa + 4), LB = lds32(wb + 4);
        int            im[NG][4], in[NG][4];
#pragma unroll
        for (int grp = 0; grp < NG; grp++) {
#pragma unroll
            for (int e = 0; e < 4; e++) im[grp][e] = in[grp][e] = 0;
        }
#pragma unroll
        for (int b = 0; b < 8; b++) {
            const int sA = (int) (((LA >> (4 * b)) & 0xFu) | (((HA >> (2 * b)) & 3u) << 4)) - 32;
            const int sB = (int) (((LB >> (4 * b)) & 0xFu) | (((HB >> (2 * b)) & 3u) << 4)) - 32;
            uint32_t  a0, a2, a1, a3;
            lookup(lds32(wa + 8 + 16 * b + 4 * t), a0, a2);
            lookup(lds32(wb + 8 + 16 * b + 4 * t), a1, a3);
#pragma unroll
            for (int grp = 0; grp < NG; grp++) {
                const uint8_t * xp   = xr + (8 * grp + g) * kTokStride + 32 * b + 4 * t;
                int             c[4] = { 0, 0, 0, 0 };
                mma_k32<false>(c, a0, a1, a2, a3, lds32(xp), lds32(xp + 16));
                im[grp][0] += sA * c[0];
                im[grp][1] += sA * c[1];
                im[grp][2] += sB * c[2];
                im[grp][3] += sB * c[3];
            }
        }
        if constexpr (DBG) {
            dbg_store<NG>(dbg, im, false, rg, sbi, lane);
        } else {
            const float * xs = reinterpret_cast<const float *>(xr + NT * kTokStride);
            sb_update<NG, false>(acc, im, in, ldh(wa), ldh(wb), 0.f, 0.f, xs, t);
        }
    }
};

// Q8_0 (34 B per 32 weights: f16 d, 32 int8). A "super-block" here is 8 consecutive blocks (272 bytes); each block
// has its own weight and activation scale, so the f32 update happens per block.
struct DecQ80 {
    static constexpr int  BS  = 272;
    static constexpr bool Q80 = true;

    template <int NG, bool DBG>
    __device__ __forceinline__ static void sb(const uint8_t * wa, const uint8_t * wb, const uint8_t * xr, int lane,
                                              float (&acc)[NG][4], const DbgOut & dbg, int64_t rg, int sbi) {
        constexpr int NT = 8 * NG;
        const int     t = lane & 3, g = lane >> 2;
        const float * xsb = reinterpret_cast<const float *>(xr + NT * kTokStride);
#pragma unroll
        for (int i = 0; i < 8; i++) {
            const uint8_t * ba = wa + 34 * i;
            const uint8_t * bb = wb + 34 * i;
            const uint32_t  a0 = lds_u32_a2(ba + 2 + 4 * t), a2 = lds_u32_a2(ba + 18 + 4 * t);
            const uint32_t  a1 = lds_u32_a2(bb + 2 + 4 * t), a3 = lds_u32_a2(bb + 18 + 4 * t);
            int             c[NG][4];
#pragma unroll
            for (int grp = 0; grp < NG; grp++) {
                const uint8_t * xp = xr + (8 * grp + g) * kTokStride + 32 * i + 4 * t;
                c[grp][0] = c[grp][1] = c[grp][2] = c[grp][3] = 0;
                mma_k32<false>(c[grp], a0, a1, a2, a3, lds32(xp), lds32(xp + 16));
            }
            if constexpr (DBG) {
                dbg_store<NG>(dbg, c, false, rg, 8 * sbi + i, lane);
            } else {
                const float   dA = ldh(ba), dB = ldh(bb);
                const float * xs = xsb + i * NT;
#pragma unroll
                for (int grp = 0; grp < NG; grp++) {
                    const float x0 = xs[8 * grp + 2 * t], x1 = xs[8 * grp + 2 * t + 1];
                    acc[grp][0] += (dA * x0) * (float) c[grp][0];
                    acc[grp][1] += (dA * x1) * (float) c[grp][1];
                    acc[grp][2] += (dB * x0) * (float) c[grp][2];
                    acc[grp][3] += (dB * x1) * (float) c[grp][3];
                }
            }
        }
    }
};

// ---------------------------------------------------------------------------------------------------------------
// the kernel

template <class D, int NG>
__device__ __forceinline__ void producer(const GemmArgs & a, uint64_t * full, uint64_t * empty, uint8_t * stage0,
                                         int64_t row0, int nchunks, int lane) {
    constexpr int  RB   = rec_bytes(D::Q80, 8 * NG);
    const int64_t  wlim = a.w_bytes & ~int64_t(15);  // bytes below this are reachable by 16-byte bulk copies
    // weight part of chunk c: tail bytes by hand (issue = false, returns this lane's bulk bytes) or the bulk copies
    auto w_part = [&](int c, uint8_t * st, uint64_t * bar, bool issue) -> uint32_t {
        uint32_t      tx  = 0;
        const int     sb0 = c * a.kc, kcc = min(a.kc, a.nsb - sb0);
        for (int i = lane; i < kTileRows; i += 32) {
            const int64_t r = row0 + i;
            if (r >= a.rows) continue;
            const int64_t start = r * a.row_bytes + (int64_t) sb0 * D::BS, end = start + (int64_t) kcc * D::BS;
            const int64_t a0 = start & ~int64_t(15), be = min((end + 15) & ~int64_t(15), wlim);
            uint8_t *     dst = st + i * a.SR;
            if (be > a0) {
                if (issue) bulk_g2s(dst, a.W + a0, (uint32_t) (be - a0), bar);
                tx += (uint32_t) (be - a0);
            }
            if (!issue) {
                for (int64_t p = max(a0, be); p < end; p++) dst[p - a0] = a.W[p];
            }
        }
        return tx;
    };
    const int npre   = min(kStages, nchunks);
    int       issued = 0;
    bool      ok     = true;
    // prologue: weight copies of the first stages go out before the activation records exist (PDL overlap)
    for (int c = 0; c < npre; c++) {
        uint8_t *      st  = stage0 + (size_t) c * a.stage_bytes;
        const int      kcc = min(a.kc, a.nsb - c * a.kc);
        const uint32_t tx  = __reduce_add_sync(0xffffffffu, w_part(c, st, &full[c], false)) + (uint32_t) (kcc * RB);
        fence_proxy_async_smem();
        __syncwarp();
        if (lane == 0) mbar_arrive_expect_tx(&full[c], tx);
        __syncwarp();
        w_part(c, st, &full[c], true);
    }
    pdl_wait();
    if (lane == 0) {
        for (int c = 0; c < npre; c++) {
            const int kcc = min(a.kc, a.nsb - c * a.kc);
            bulk_g2s(stage0 + (size_t) c * a.stage_bytes + kTileRows * a.SR, a.recs + (size_t) c * a.kc * RB,
                     (uint32_t) (kcc * RB), &full[c]);
        }
    }
    issued = npre;
    for (int c = npre; c < nchunks; c++) {
        const int s = c % kStages;
        if (!mbar_wait(&empty[s], ((c / kStages) - 1) & 1)) {
            ok = false;
            break;
        }
        uint8_t *      st  = stage0 + (size_t) s * a.stage_bytes;
        const int      kcc = min(a.kc, a.nsb - c * a.kc);
        const uint32_t tx  = __reduce_add_sync(0xffffffffu, w_part(c, st, &full[s], false)) + (uint32_t) (kcc * RB);
        fence_proxy_async_smem();
        __syncwarp();
        if (lane == 0) mbar_arrive_expect_tx(&full[s], tx);
        __syncwarp();
        w_part(c, st, &full[s], true);
        if (lane == 0) {
            bulk_g2s(st + kTileRows * a.SR, a.recs + (size_t) c * a.kc * RB, (uint32_t) (kcc * RB), &full[s]);
        }
        issued = c + 1;
    }
    // drain: every copy this warp issued has landed before the CTA may exit
    for (int c = max(0, issued - kStages); c < issued; c++) {
        if (!mbar_wait(&full[c % kStages], (c / kStages) & 1)) {
            ok = false;
        }
    }
    if (!ok && lane == 0) atomicExch(a.status, kErrWaitEmpty);
}

template <class D, int NG, bool DBG>
__global__ void __launch_bounds__(kThreads) srv_gemm_kernel(const GemmArgs a) {
    extern __shared__ __align__(128) uint8_t smem[];
    uint64_t *    full   = reinterpret_cast<uint64_t *>(smem);
    uint64_t *    empty  = full + kStages;
    uint8_t *     stage0 = smem + kBarBytes;
    constexpr int RB     = rec_bytes(D::Q80, 8 * NG);
    const int     warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
    const int64_t row0    = (int64_t) blockIdx.x * kTileRows;
    const int     nchunks = (a.nsb + a.kc - 1) / a.kc;
    if (threadIdx.x == 0) {
        for (int s = 0; s < kStages; s++) {
            mbar_init(&full[s], 1);
            mbar_init(&empty[s], kNCW);
        }
        fence_mbar_init();
    }
    __syncthreads();
    if (warp == kNCW) {
        producer<D, NG>(a, full, empty, stage0, row0, nchunks, lane);
        return;
    }
    const int     g = lane >> 2, t = lane & 3;
    const int     rl = warp * 16 + g;
    const int64_t rg = row0 + rl;
    float         acc[NG][4];
#pragma unroll
    for (int grp = 0; grp < NG; grp++) acc[grp][0] = acc[grp][1] = acc[grp][2] = acc[grp][3] = 0.0f;
    const DbgOut dbg = { a.isum, a.imin, a.rows, a.N, a.nblk };
    for (int c = 0; c < nchunks; c++) {
        const int s = c % kStages;
        if (!mbar_wait(&full[s], (c / kStages) & 1)) {
            if (lane == 0) atomicExch(a.status, kErrWaitFull);
            return;
        }
        const uint8_t * st  = stage0 + (size_t) s * a.stage_bytes;
        const int       sb0 = c * a.kc, kcc = min(a.kc, a.nsb - sb0);
        const int       pa  = rg < a.rows ? (int) ((rg * a.row_bytes + (int64_t) sb0 * D::BS) & 15) : 0;
        const int       pb  = rg + 8 < a.rows ? (int) (((rg + 8) * a.row_bytes + (int64_t) sb0 * D::BS) & 15) : 0;
        const uint8_t * wa  = st + rl * a.SR + pa;
        const uint8_t * wb  = st + (rl + 8) * a.SR + pb;
        const uint8_t * xr  = st + kTileRows * a.SR;
        for (int kb = 0; kb < kcc; kb++) {
            D::template sb<NG, DBG>(wa + kb * D::BS, wb + kb * D::BS, xr + kb * RB, lane, acc, dbg, rg, sb0 + kb);
        }
        __syncwarp();
        if (lane == 0) mbar_arrive(&empty[s]);
    }
    if constexpr (!DBG) {
#pragma unroll
        for (int grp = 0; grp < NG; grp++) {
#pragma unroll
            for (int e = 0; e < 4; e++) {
                const int     tok = 8 * grp + 2 * t + (e & 1);
                const int64_t row = e < 2 ? rg : rg + 8;
                if (tok < a.N && row < a.rows) a.Y[(int64_t) tok * a.ldy + row] = acc[grp][e];
            }
        }
    }
}

// ---------------------------------------------------------------------------------------------------------------
// host side

int slot_stride(int need) {
    int s = (need + 15) / 16 * 16;
    while (s % 128 != 32 && s % 128 != 96) s += 16;
    return s;
}

template <class D>
int choose_kc() {
    return std::max(1, 20000 / (kTileRows * D::BS));
}

template <class D, int NG, bool DBG>
int launch_gemm(srhpm_ctx * ctx, GemmArgs a, cudaStream_t stream) {
    constexpr int RB      = rec_bytes(D::Q80, 8 * NG);
    const bool    aligned = (a.row_bytes % 16 == 0) && ((a.kc * D::BS) % 16 == 0);
    const int     need    = (aligned ? 0 : 14) + a.kc * D::BS;
    a.SR                  = slot_stride(need);
    a.stage_bytes         = (kTileRows * a.SR + a.kc * RB + 127) / 128 * 128;
    const size_t smem     = kBarBytes + (size_t) kStages * a.stage_bytes;
    if (smem > 200 * 1024) return SRHPM_ERR_INVALID;
    auto         kern     = srv_gemm_kernel<D, NG, DBG>;
    // the shared-memory opt-in is per kernel and per device
    static std::atomic<unsigned> attr_done{ 0 };
    int                          dev = 0;
    cudaGetDevice(&dev);
    if (!(attr_done.load() & (1u << (dev & 31)))) {
        // every configuration of this kernel needs well under 200 KB (checked below); the opt-in covers them all
        const int st = cuda_status(cudaFuncSetAttribute(kern, cudaFuncAttributeMaxDynamicSharedMemorySize, 200 * 1024));
        if (st != SRHPM_OK) return st;
        attr_done.fetch_or(1u << (dev & 31));
    }
    cudaLaunchConfig_t cfg = {};
    cfg.gridDim            = dim3((unsigned) ((a.rows + kTileRows - 1) / kTileRows));
    cfg.blockDim           = dim3(kThreads);
    cfg.dynamicSmemBytes   = smem;
    cfg.stream             = stream;
    cudaLaunchAttribute attr[1];
    attr[0].id                                         = cudaLaunchAttributeProgrammaticStreamSerialization;
    attr[0].val.programmaticStreamSerializationAllowed = 1;
    cfg.attrs                                          = attr;
    cfg.numAttrs                                       = 1;
    ctx->launches.fetch_add(1);
    return cuda_status(cudaLaunchKernelEx(&cfg, kern, a));
}

template <class D>
int dispatch_ng(srhpm_ctx * ctx, const GemmArgs & a, bool dbg, cudaStream_t stream) {
    if (a.N <= 8) {
        return dbg ? launch_gemm<D, 1, true>(ctx, a, stream) : launch_gemm<D, 1, false>(ctx, a, stream);
    }
    return dbg ? launch_gemm<D, 2, true>(ctx, a, stream) : launch_gemm<D, 2, false>(ctx, a, stream);
}

template <class D>
int kc_for() { return choose_kc<D>(); }

int kc_of(int wtype) {
    switch (wtype) {
        case SRHPM_TYPE_Q4_K: return kc_for<DecK45<false>>();
        case SRHPM_TYPE_Q5_K: return kc_for<DecK45<true>>();
        case SRHPM_TYPE_Q6_K: return kc_for<DecQ6K>();
        case SRHPM_TYPE_Q3_K: return kc_for<DecQ3K>();
        case SRHPM_TYPE_IQ4_XS: return kc_for<DecIQ4XS>();
        case SRHPM_TYPE_Q8_0: return kc_for<DecQ80>();
        default: return 1;
    }
}

uint8_t * align256(void * p) {
    return reinterpret_cast<uint8_t *>((reinterpret_cast<uintptr_t>(p) + 255) & ~uintptr_t(255));
}

}  // namespace

size_t gemm_work_size(int wtype, int64_t K, int64_t N) {
    const int NT = N <= 8 ? 8 : 16;
    return (size_t) (K / QK) * rec_bytes(wtype == SRHPM_TYPE_Q8_0, NT) + 256;
}

int gemm_run(srhpm_ctx * ctx, int wtype, const uint8_t * W, int64_t rows, int64_t K, size_t row_bytes,
             const float * X, int64_t ldx, int64_t N, float * Y, int64_t ldy, void * wdata, size_t wsize,
             int32_t * isum, int32_t * imin, cudaStream_t stream) {
    if (wsize < gemm_work_size(wtype, K, N) || !wdata) return SRHPM_ERR_WORKSPACE;
    const int  nsb  = (int) (K / QK);
    const int  NT   = N <= 8 ? 8 : 16;
    const bool q80  = wtype == SRHPM_TYPE_Q8_0;
    uint8_t *  recs = align256(wdata);
    // 1. activation records
    {
        const int64_t warps  = (int64_t) nsb * NT;
        const int     blocks = (int) ((warps + 7) / 8);
        if (q80) {
            quant_q80_kernel<false><<<blocks, 256, 0, stream>>>(X, ldx, (int) N, nsb, NT, ctx->q8_0_act_mode, recs,
                                                                nullptr);
        } else {
            quant_q8K_kernel<false><<<blocks, 256, 0, stream>>>(X, ldx, (int) N, nsb, NT, recs, nullptr, nullptr,
                                                                nullptr, nullptr);
        }
        ctx->launches.fetch_add(1);
        const int st = cuda_status(cudaGetLastError());
        if (st != SRHPM_OK) return st;
    }
    // 2. the matmul
    GemmArgs a    = {};
    a.W           = W;
    a.rows        = rows;
    a.row_bytes   = (int64_t) row_bytes;
    a.w_bytes     = rows * (int64_t) row_bytes;
    a.nsb         = nsb;
    a.kc          = std::min(kc_of(wtype), nsb);
    a.recs        = recs;
    a.Y           = Y;
    a.ldy         = ldy;
    a.N           = (int) N;
    a.status      = ctx->d_status;
    a.isum        = isum;
    a.imin        = imin;
    a.nblk        = q80 ? nsb * 8 : nsb;
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

int quantize_q8K_dense(srhpm_ctx * ctx, const float * X, int64_t ldx, int64_t N, int64_t K, int8_t * q, float * d,
                       int16_t * b32, int16_t * b16, cudaStream_t stream) {
    const int     nsb    = (int) (K / QK);
    const int64_t warps  = (int64_t) nsb * N;
    const int     blocks = (int) ((warps + 7) / 8);
    quant_q8K_kernel<true><<<blocks, 256, 0, stream>>>(X, ldx, (int) N, nsb, 0, nullptr, q, d, b32, b16);
    ctx->launches.fetch_add(1);
    return cuda_status(cudaGetLastError());
}

int quantize_q8_0_dense(srhpm_ctx * ctx, const float * X, int64_t ldx, int64_t N, int64_t K, void * blocks,
                        cudaStream_t stream) {
    const int     nsb    = (int) (K / QK);
    const int64_t warps  = (int64_t) nsb * N;
    const int     nblk   = (int) ((warps + 7) / 8);
    quant_q80_kernel<true><<<nblk, 256, 0, stream>>>(X, ldx, (int) N, nsb, 0, ctx->q8_0_act_mode, nullptr,
                                                     reinterpret_cast<uint8_t *>(blocks));
    ctx->launches.fetch_add(1);
    return cuda_status(cudaGetLastError());
}

}  // namespace srhpm
