// Multi-query attention over a q8_0 KV cache for a few query tokens (speculative verification), on the 5th-generation
// tensor cores. Computes ggml_flash_attn_ext as the reference's grouped path does
// (ggml_compute_forward_flash_attn_ext_gqa_small, patch/srhpm.patch:581-824): all R = G * N query rows of one KV head
// (G query heads per KV head, N query tokens) form one tile, Q is quantized per row to q8_0 (the vec_dot type of a
// q8_0 cache, P:670-673) and Q.K is the exact integer q8_0 dot product (P:700-706), scaled, soft-capped and masked
// (P:732-746); softmax is online over KV tiles (P:748-764) and the KV range is split into chunks whose partial
// (max, sum, V-weighted sum) records are merged afterwards (P:787-823).
//
// One CTA per (KV head, row group of <= 48 rows, KV chunk). Per tile of 128 KV tokens:
//   * producer warp: TMA of the K tile as two 128-byte SWIZZLE_128B planes + one 32-byte SWIZZLE_32B plane (the
//     K-major operand layout the tensor core reads directly) and of the V tile as plain 272-byte rows, through a
//     3-slot shared-memory ring;
//   * MMA warp (one thread): S_b = K_b . Q_b^T for the 8 q8_0 blocks b (kind::i8, M = 128 tokens, N = rows, int32 in
//     tensor memory). The 32 quant bytes of block b sit at row bytes 34b+2..34b+33, which straddle two 32-byte
//     windows of the row; each window is one MMA against a Q operand that holds Q's block-b bytes at the same
//     positions and zeros elsewhere (the interleaved d bytes meet zeros), so S_b is the exact block sum. After
//     softmax, O^T += V^T . P^T (kind::f16, M = 128 dv per half, N = rows, f32 in tensor memory);
//   * 4 compute warps, thread = KV token: read S_b, apply d_k * d_q (+ scale, softcap, mask), row maxima with
//     redux.sync, p = 2^(s - m) as f16 into P^T, and V dequantized to f16 (d * q) into the MN-major V^T operand.
//     The running maximum is raised only when a tile's maximum exceeds it by 2^8 (then O and the row sums are
//     rescaled in place); p <= 256 otherwise, and the final division by the row sum makes the result the same.
// A chunk writes its normalized output directly, or (several chunks) its (max, sum, acc) record for fa_combine.
#include <cuda.h>
#include <cuda_fp16.h>

#include <algorithm>
#include <atomic>
#include <cmath>

#include "allreduce.cuh"
#include "internal.h"
#include "launch.cuh"
#include "ptx.cuh"
#include "tc.cuh"

namespace srhpm {
namespace {

constexpr int   kT       = 128;                 // KV tokens per tile
constexpr int   kD       = 256;                 // DK = DV
constexpr int   kRowB    = 272;                 // q8_0 bytes of one 256-value row
constexpr int   kPlane   = kT * 128;            // one SWIZZLE_128B plane of a K tile
constexpr int   kKTile   = 2 * kPlane + kT * 32;  // 36864: planes of row bytes 0-127, 128-255, 256-287
constexpr int   kVTile   = kT * kRowB;          // 34816
constexpr int   kSlot    = kKTile;
constexpr int   kNSlot   = 5;                  // ring slots (a K or a V tile each)
constexpr int   kRG      = 48;                  // rows per row group (tensor memory: 8 * 48 + 2 * 48 columns)
constexpr int   kCW      = 16;                  // compute warps (4 token quarters x 4 row quarters)
constexpr int   kFaThreads = (kCW + 2) * 32;    // + producer warp + MMA warp
constexpr float kLog2e   = 1.4426950408889634f;
constexpr float kLazy    = 8.0f;                // raise the running maximum only beyond 2^8

struct FaArgs {
    const float *   q;
    int64_t         qnb1, qnb2;  // bytes: token, head
    int             N, H, G, R;  // query tokens, heads, heads per KV head, rows per KV head (G * N)
    int             L, Hkv, nrg;
    int             chunk_len, n_chunks;
    const uint8_t * mask;  // f16 or null
    int64_t         mnb1, mnb2;
    int             mne2, mne0;
    int             mask_mode;   // 0 none, 1 one mask row per query token (staged per tile), 2 per-head rows
    float           qscale;      // folded into the Q block scales: scale*log2e, or scale/softcap with a softcap
    float           softcap_l2;  // softcap*log2e, 0 = none
    float           max_bias, m0, m1;
    int             n_head_log2;
    const float *   sinks;       // f32 [H] or null
    float *         dst;
    int64_t         dnb1, dnb2;  // bytes: head, token
    float *         part_acc;    // [Hkv * R][n_chunks][256]
    float2 *        part_ms;     // [Hkv * R][n_chunks] (max in log2 units, sum)
    // what fa_combine reads: record (row, c) at part_ms[row * ms_row + c * ms_chunk] and
    // part_acc[row * acc_row + c * acc_chunk + dv] (the layout above, or the record sets of several devices)
    int64_t         ms_row, ms_chunk, acc_row, acc_chunk;
    int             parts_out;   // 1: write this KV range's merged record (rec_ms, rec_acc), not dst; no sinks
    float2 *        rec_ms;      // [Hkv * R]
    float *         rec_acc;     // [Hkv * R][256]
    int32_t *       status;
    int             q8mode;
};

// shared-memory layout (bytes from a 1024-aligned base)
template <int RP> struct Smem {
    static constexpr int ring = 0;
    static constexpr int p    = ring + kNSlot * kSlot;
    static constexpr int qop  = p + RP * kT * 2;      // Q operands of the 9 K windows, [2][rows][16] each
    static constexpr int qopb = 16 * RP * 32;         // their bytes
    static constexpr int dq   = qop + qopb;           // f32 [8][RP]
    static constexpr int red  = dq + 8 * RP * 4;      // f32 [2][4][RP] (per tile parity, per token quarter)
    static constexpr int mu   = red + 2 * 4 * RP * 4; // f32 [RP] running maximum (log2 units)
    static constexpr int al   = mu + RP * 4;          // f32 [RP] rescale factor of this tile
    static constexpr int fac  = al + RP * 4;          // f32 [RP] final factor
    static constexpr int slope = fac + RP * 4;        // f32 [RP] ALiBi slope * log2e
    static constexpr int moff = slope + RP * 4;       // int64 [RP] mask row offsets
    static constexpr int mslot = moff + RP * 8;       // int32 [RP] staged mask row of each row (its query token)
    static constexpr int MBR  = RP == 48 ? 8 : 16;    // staged mask rows (query tokens); 48-row groups: no room for 16
    static constexpr int mbuf = (mslot + RP * 4 + 15) / 16 * 16;  // f16 [2][MBR][kT] staged mask tiles
    static constexpr int bar  = mbuf + 2 * MBR * kT * 2;
    static constexpr int nbar = 2 * kNSlot + 4;       // full[], empty[], s_full, s_free, pv_ready, pv_done
    static constexpr int misc = bar + nbar * 8;       // tmem base, flags[3]
    static constexpr int total = misc + 16;
    static constexpr int alloc = total + 1024;
};

__device__ __forceinline__ void tma3(uint8_t * dst, const CUtensorMap * m, int x, int y, int z, uint64_t * bar) {
    asm volatile(
        "cp.async.bulk.tensor.3d.shared::cluster.global.tile.mbarrier::complete_tx::bytes [%0], [%1, {%2, %3, %4}], "
        "[%5];" ::"r"(smem_u32(dst)),
        "l"(m), "r"(x), "r"(y), "r"(z), "r"(smem_u32(bar))
        : "memory");
}

__device__ __forceinline__ float redux_max(float v) {
    float r;
    asm("redux.sync.max.f32 %0, %1, 0xffffffff;" : "=f"(r) : "f"(v));
    return r;
}

__device__ __forceinline__ uint32_t prmt(uint32_t a, uint32_t b, uint32_t sel) {
    uint32_t r;
    asm("prmt.b32 %0, %1, %2, %3;" : "=r"(r) : "r"(a), "r"(b), "r"(sel));
    return r;
}

__device__ __forceinline__ bool wait_or_flag(uint64_t * bar, uint32_t parity, int32_t * status, bool & bad) {
    if (bad) return false;
    if (!mbar_wait(bar, parity)) {
        bad = true;
        atomicExch(status, kErrWaitFull);
        return false;
    }
    return true;
}

// a 32-bit word of f16x2 from two int8 held in bytes (hi ? 2,3 : 0,1) of w ^ 0x80808080: 1024 + (q + 128) each
template <int HI> __device__ __forceinline__ uint32_t magic_pair(uint32_t wx) {
    return prmt(wx, 0x64u, HI ? 0x4342u : 0x4140u);
}

__device__ __forceinline__ float ex2(float x) {
    float r;
    asm("ex2.approx.ftz.f32 %0, %1;" : "=f"(r) : "f"(x));
    return r;
}

// The Q.K accumulators start at kMagic: an int32 sum i (|i| <= 32 * 127 * 127 < 2^22) then reads as the float
// 12582912 + i exactly, and one subtraction gives i as a float (no integer-to-float conversion instruction).
constexpr uint32_t kMagic  = 0x4B400000u;
constexpr float    kMagicF = 12582912.0f;

// K window w (row bytes 32w..32w+31) holds quant bytes of blocks w-1 and w (w = 1..7), of block 0 (w = 0) or of
// block 7 (w = 8); its Q operand has the rows of those blocks (RP or 2 RP rows), so one MMA per window fills the score
// columns of both blocks (block b at columns RP * b)
template <int RP> __host__ __device__ constexpr int qwin_rows(int w) { return (w == 0 || w == 8) ? RP : 2 * RP; }
template <int RP> __host__ __device__ constexpr int qwin_off(int w) {
    return w == 0 ? 0 : RP * 32 + (w - 1) * 2 * RP * 32;
}

template <int RP> __device__ __forceinline__ void arm_scores(uint32_t tS, int q, int rbase) {
    constexpr int RH = RP / 4;
    uint32_t      m[RH];
#pragma unroll
    for (int j = 0; j < RH; j++) m[j] = kMagic;
#pragma unroll
    for (int b = 0; b < 8; b++) tc::st_cols<RH>(tc::taddr(tS, q, RP * b + rbase), m);
}

// 1 thread = a quarter of one KV token's V row: blocks 2*qr, 2*qr+1 ([d | 32 q] each, row bytes 68*qr..68*qr+67).
// load_v_part reads the 80 bytes from 64*qr (16-byte loads, conflict-free across consecutive tokens); the quarter
// starts WS = qr words into them. convert_v_part writes 64 f16 = d * q into the V^T operand of the dv half the blocks
// belong to ([dv group of 8 (16 per half)][token][8 f16]).
__device__ __forceinline__ void load_v_part(const uint8_t * row, int qr, uint32_t (&w)[20]) {
    const uint4 * src = reinterpret_cast<const uint4 *>(row + 64 * qr);
#pragma unroll
    for (int c = 0; c < 5; c++) {
        const uint4 u = src[c];
        w[4 * c] = u.x; w[4 * c + 1] = u.y; w[4 * c + 2] = u.z; w[4 * c + 3] = u.w;
    }
}
template <int WS> __device__ __forceinline__ void convert_v_part(const uint32_t (&w)[20], uint8_t * vch, int t) {
    const __half2 bias = __halves2half2(__ushort_as_half(0x6480u), __ushort_as_half(0x6480u));  // 1152
#pragma unroll
    for (int bb = 0; bb < 2; bb++) {
        const int      od    = 4 * WS + 34 * bb;
        const uint32_t dbits = (w[od >> 2] >> (8 * (od & 3))) & 0xffffu;
        const __half2  dd    = __halves2half2(__ushort_as_half((unsigned short) dbits),
                                              __ushort_as_half((unsigned short) dbits));
        uint32_t       f[16];
#pragma unroll
        for (int m = 0; m < 16; m++) {
            const int      o  = od + 2 + 2 * m;  // even: the pair sits in one word
            const uint32_t wx = w[o >> 2] ^ 0x80808080u;
            const uint32_t mg = ((o >> 1) & 1) ? magic_pair<1>(wx) : magic_pair<0>(wx);
            __half2        h  = __hsub2(*reinterpret_cast<const __half2 *>(&mg), bias);
            h                 = __hmul2(h, dd);
            f[m]              = *reinterpret_cast<const uint32_t *>(&h);
        }
        const int jb = 4 * ((2 * WS + bb) & 3);  // dv group of block 2 qr + bb inside its half (qr = WS)
#pragma unroll
        for (int qd = 0; qd < 4; qd++) {
            *reinterpret_cast<uint4 *>(vch + ((jb + qd) * kT + t) * 16) =
                make_uint4(f[4 * qd], f[4 * qd + 1], f[4 * qd + 2], f[4 * qd + 3]);
        }
    }
}

// P^T rows rbase..rbase+RH-1 (f16 pairs in pk) of token t: MN-major [row group of 8][token][8 f16], 4 rows per store
template <int RH> __device__ __forceinline__ void store_p(uint8_t * pbase, int rbase, int t, const uint32_t * pk) {
#pragma unroll
    for (int u = 0; u < RH / 4; u++) {
        const int row = rbase + 4 * u;
        *reinterpret_cast<uint2 *>(pbase + ((row >> 3) * kT + t) * 16 + (row & 7) * 2) = make_uint2(pk[2 * u], pk[2 * u + 1]);
    }
}

// staged mask tile (mask_mode 1, N <= MBR): row tq, tokens tok0..tok0+127 -> f16 [MBR][kT]; thread p < N * 16 moves 8 tokens
__device__ __forceinline__ uint4 mask_piece(const FaArgs & a, int p, int tok0) {
    const int  tq = p >> 4, e0 = tok0 + 8 * (p & 15);
    const uint8_t * src = a.mask + (int64_t) tq * a.mnb1 + 2 * (int64_t) e0;
    if (e0 + 8 <= a.mne0) return __ldg(reinterpret_cast<const uint4 *>(src));
    uint16_t v[8];
#pragma unroll
    for (int e = 0; e < 8; e++) v[e] = e0 + e < a.mne0 ? __ldg(reinterpret_cast<const unsigned short *>(src) + e) : 0;
    return make_uint4(v[0] | (uint32_t) v[1] << 16, v[2] | (uint32_t) v[3] << 16, v[4] | (uint32_t) v[5] << 16,
                      v[6] | (uint32_t) v[7] << 16);
}

template <int RP>
__global__ void __launch_bounds__(kFaThreads, 1)
    fa_q80_kernel(const __grid_constant__ CUtensorMap mk128, const __grid_constant__ CUtensorMap mk32,
                  const __grid_constant__ CUtensorMap mv, const FaArgs a) {
    using S           = Smem<RP>;
    constexpr int RH  = RP / 4;  // rows per compute thread
    extern __shared__ uint8_t smem_raw[];
    // 1024-byte aligned base, by pointer arithmetic on the shared array (an integer round trip would make every
    // access through `sm` a generic load / store)
    uint8_t * sm = smem_raw + ((1024u - (smem_u32(smem_raw) & 1023u)) & 1023u);
    uint64_t * full    = reinterpret_cast<uint64_t *>(sm + S::bar);
    uint64_t * empty   = full + kNSlot;
    uint64_t * s_full  = empty + kNSlot;
    uint64_t * s_free  = s_full + 1;
    uint64_t * pv_rdy  = s_full + 2;
    uint64_t * pv_done = s_full + 3;
    uint32_t * tptr    = reinterpret_cast<uint32_t *>(sm + S::misc);
    int *      flags   = reinterpret_cast<int *>(sm + S::misc + 4);
    float *    dq      = reinterpret_cast<float *>(sm + S::dq);
    float *    red     = reinterpret_cast<float *>(sm + S::red);
    float *    mu      = reinterpret_cast<float *>(sm + S::mu);
    float *    al      = reinterpret_cast<float *>(sm + S::al);
    float *    fac     = reinterpret_cast<float *>(sm + S::fac);
    float *    slope2  = reinterpret_cast<float *>(sm + S::slope);
    int64_t *  moff    = reinterpret_cast<int64_t *>(sm + S::moff);
    int *      mslot   = reinterpret_cast<int *>(sm + S::mslot);
    uint16_t * mbuf    = reinterpret_cast<uint16_t *>(sm + S::mbuf);

    const int tid = threadIdx.x, warp = tid >> 5, lane = tid & 31;
    const int chunk = blockIdx.x;
    const int g = blockIdx.y / a.nrg, rg = blockIdx.y % a.nrg;
    const int t0 = chunk * a.chunk_len, t1 = min(a.L, t0 + a.chunk_len);
    const int nt = (t1 - t0 + kT - 1) / kT;
    const int row0 = rg * RP;               // first row (of the KV head's R) of this group
    const int rows = min(RP, a.R - row0);   // valid rows
    // compute threads: lane quarter q (KV token t = 32 q + lane of the tile), row quarter qr (rows rbase..rbase+RH-1)
    const int q = warp & 3, qr = (warp >> 2) & 3, t = 32 * q + lane, rbase = qr * RH;
    bool      bad = false;

    if (tid == 0) {
        for (int i = 0; i < kNSlot; i++) {
            mbar_init(&full[i], 1);
            mbar_init(&empty[i], 1);  // released by the commit of the tile's P.V
        }
        mbar_init(s_full, 1);
        mbar_init(s_free, kCW);
        mbar_init(pv_rdy, kCW);
        mbar_init(pv_done, 1);
        fence_mbar_init();
        flags[0] = flags[1] = flags[2] = 0;
    }
    if (warp == 0) tc::tmem_alloc(tptr, 512);
    if (tid < kCW * 32) {
        uint4 * z = reinterpret_cast<uint4 *>(sm + S::qop);
        for (int i = tid; i < S::qopb / 16; i += kCW * 32) z[i] = make_uint4(0, 0, 0, 0);
    }
    tc::fence_before();
    __syncthreads();
    tc::fence_after();
    const uint32_t tbase = *tptr;
    const uint32_t tS    = tbase;           // S_b at columns RP * b
    const uint32_t tO    = tbase + 8 * RP;  // O^T halves at tO, tO + RP

    // producer: the first loads of the ring need no empty-slot wait
    auto produce = [&](int n) {
        const int slot = n % kNSlot;
        uint8_t * dst  = sm + S::ring + slot * kSlot;
        const int tok  = t0 + (n >> 1) * kT;
        if ((n & 1) == 0) {
            mbar_arrive_expect_tx(&full[slot], kKTile);
            tma3(dst, &mk128, 0, tok, g, &full[slot]);
            tma3(dst + kPlane, &mk128, 32, tok, g, &full[slot]);
            tma3(dst + 2 * kPlane, &mk32, 64, tok, g, &full[slot]);
        } else {
            mbar_arrive_expect_tx(&full[slot], kVTile);
            tma3(dst, &mv, 0, tok, g, &full[slot]);
        }
    };
    const int nload = 2 * nt;
    if (warp == kCW && lane == 0) {
        prefetch_tmap(&mk128);
        prefetch_tmap(&mk32);
        prefetch_tmap(&mv);
    }
    // launched behind the kernel that wrote the newest K/V rows and Q (programmatic dependent launch): everything
    // above overlapped its tail; from here on its writes are visible
    pdl_wait();
    if (warp == kCW && lane == 0) {
        for (int n = 0; n < min(kNSlot, nload); n++) produce(n);
    }
    __syncwarp();

    // Q rows -> q8_0 (the cache type's vec_dot type), scattered into the 16 window operands; per-row constants;
    // the score accumulators armed with the magic offset
    if (warp < kCW) {
        for (int u = tid; u < 8 * RP; u += kCW * 32) {
            const int r = u >> 3, b = u & 7;
            int8_t    qv[32];
            float     dqs = 0.0f;
            if (r < rows) {
                const int     rr  = row0 + r;
                const int     h   = g * a.G + rr / a.N, tq = rr % a.N;
                const float * src = reinterpret_cast<const float *>(reinterpret_cast<const uint8_t *>(a.q) +
                                                                     tq * a.qnb1 + h * a.qnb2) + 32 * b;
                float x[32], amax = 0.0f;
#pragma unroll
                for (int j = 0; j < 32; j++) {
                    x[j] = src[j];
                    amax = fmaxf(amax, fabsf(x[j]));
                }
                const float  dd = __fdiv_rn(amax, 127.0f);
                const __half dh = __float2half_rn(dd);
                if (a.q8mode == SRHPM_Q8_0_ACT_SIMD) {
                    const float id = amax != 0.0f ? __fdiv_rn(127.0f, amax) : 0.0f;
#pragma unroll
                    for (int j = 0; j < 32; j++) qv[j] = (int8_t) __float2int_rn(__fmul_rn(x[j], id));
                } else {
                    const float id = dd != 0.0f ? __fdiv_rn(1.0f, dd) : 0.0f;
#pragma unroll
                    for (int j = 0; j < 32; j++) qv[j] = (int8_t) (int) roundf(__fmul_rn(x[j], id));
                }
                dqs = __half2float(dh) * a.qscale;
            } else {
#pragma unroll
                for (int j = 0; j < 32; j++) qv[j] = 0;
            }
            dq[b * RP + r] = dqs;
#pragma unroll
            for (int j = 0; j < 32; j++) {
                const int pos = 34 * b + 2 + j, x = pos & 31, w = pos >> 5;
                const int row = (w >= 1 && w <= 7 && b == w) ? RP + r : r;  // second block of a shared window
                sm[S::qop + qwin_off<RP>(w) + (x >> 4) * qwin_rows<RP>(w) * 16 + row * 16 + (x & 15)] =
                    (uint8_t) qv[j];
            }
        }
        if (tid < RP) {
            const int r = tid, rr = row0 + min(r, rows - 1);
            const int h = g * a.G + rr / a.N, tq = rr % a.N;
            float     sl = 1.0f;
            if (a.max_bias > 0.0f) {
                sl = h < a.n_head_log2 ? powf(a.m0, (float) (h + 1)) : powf(a.m1, (float) (2 * (h - a.n_head_log2) + 1));
            }
            slope2[r] = sl * kLog2e;
            moff[r]   = a.mask ? (int64_t) tq * a.mnb1 + (int64_t) (h % a.mne2) * a.mnb2 : 0;
            mslot[r]  = tq;
            mu[r]     = -INFINITY;
        }
        if (a.mask_mode == 1 && tid < a.N * 16) {  // N <= MBR
            *reinterpret_cast<uint4 *>(mbuf + (tid >> 4) * kT + 8 * (tid & 15)) = mask_piece(a, tid, t0);
        }
        arm_scores<RP>(tS, q, rbase);
        tc::wait_st();
    }
    asm volatile("fence.proxy.async.shared::cta;" ::: "memory");
    tc::fence_before();
    __syncthreads();
    tc::fence_after();

    const uint32_t qop_s = smem_u32(sm + S::qop);
    const uint32_t p_s   = smem_u32(sm + S::p);

    if (warp == kCW) {
        // ---------------- producer ----------------
        if (lane == 0) {
            for (int n = kNSlot; n < nload; n++) {
                const int slot = n % kNSlot;
                if (!wait_or_flag(&empty[slot], ((n / kNSlot) - 1) & 1, a.status, bad)) break;
                produce(n);
            }
        }
        __syncwarp();
    } else if (warp == kCW + 1) {
        // ---------------- MMA issuer ----------------
        if (lane == 0) {
            constexpr uint32_t id8  = tc::idesc(tc::kD_S32, tc::kAB_S8, tc::kAB_S8, tc::kKMajor, tc::kKMajor, RP, 128);
            constexpr uint32_t id8w = tc::idesc(tc::kD_S32, tc::kAB_S8, tc::kAB_S8, tc::kKMajor, tc::kKMajor, 2 * RP,
                                                128);
            constexpr uint32_t id16 = tc::idesc(tc::kD_F32, tc::kAB_F16, tc::kAB_F16, tc::kMNMajor, tc::kMNMajor, RP,
                                                128);
            auto issue_qk = [&](int i) {
                const int n = 2 * i, slot = n % kNSlot;
                wait_or_flag(&full[slot], (n / kNSlot) & 1, a.status, bad);
                tc::fence_after();
                const uint32_t kb = smem_u32(sm + S::ring + slot * kSlot);
#pragma unroll
                for (int w = 0; w < 9; w++) {
                    uint64_t ad;
                    if (w < 8) {
                        ad = tc::sdesc(kb + (w >> 2) * kPlane + (w & 3) * 32, 16, 1024) | (2ull << 61);
                    } else {
                        ad = tc::sdesc(kb + 2 * kPlane, 16, 256) | (6ull << 61);
                    }
                    const uint64_t bd = tc::sdesc(qop_s + qwin_off<RP>(w), qwin_rows<RP>(w) * 16, 128);
                    tc::mma_i8(tS + (w == 0 ? 0 : RP * (w - 1)), ad, bd, (w == 0 || w == 8) ? id8 : id8w,
                               1u);  // onto the armed magic offset
                }
                tc::commit(s_full);
            };
            issue_qk(0);
            for (int i = 0; i < nt; i++) {
                if (i + 1 < nt) {
                    wait_or_flag(s_free, i & 1, a.status, bad);
                    issue_qk(i + 1);
                }
                wait_or_flag(pv_rdy, i & 1, a.status, bad);
                tc::fence_after();
                const int ks = (2 * i) % kNSlot, vs = (2 * i + 1) % kNSlot;  // V^T halves live in these slots
#pragma unroll
                for (int hf = 0; hf < 2; hf++) {
                    const uint32_t vb = smem_u32(sm + S::ring + (hf ? vs : ks) * kSlot);
#pragma unroll
                    for (int k = 0; k < kT / 16; k++) {
                        const uint64_t ad = tc::sdesc(vb + k * 256, 128, kT * 16);
                        const uint64_t bd = tc::sdesc(p_s + k * 256, 128, kT * 16);
                        tc::mma_f16(tO + hf * RP, ad, bd, id16, (uint32_t) (i > 0 || k > 0));
                    }
                }
                tc::commit(pv_done);
                tc::commit(&empty[ks]);
                tc::commit(&empty[vs]);
            }
        }
        __syncwarp();
    } else {
        // ---------------- compute warps ----------------
        const f2 negC = f2_pack(-kMagicF, -kMagicF);
        float    l[RH];  // row sums of this thread's token
#pragma unroll
        for (int r = 0; r < RH; r++) l[r] = 0.0f;
        uint32_t msl[RH / 4];  // staged mask row of each of this thread's rows, 4 per word
#pragma unroll
        for (int j = 0; j < RH / 4; j++) {
            msl[j] = 0;
#pragma unroll
            for (int e = 0; e < 4; e++) msl[j] |= (uint32_t) (mslot[rbase + 4 * j + e] & 0xff) << (8 * e);
        }
        for (int i = 0; i < nt; i++) {
            const int n = 2 * i, kslot = n % kNSlot, vslot = (n + 1) % kNSlot;
            // next tile's staged mask piece: loaded now, stored before this tile's first barrier (which orders it before
            // the next tile's reads)
            uint4      mnext = make_uint4(0, 0, 0, 0);
            const bool stage = a.mask_mode == 1 && i + 1 < nt && tid < a.N * 16;  // N <= MBR
            if (stage) mnext = mask_piece(a, tid, t0 + (i + 1) * kT);
            wait_or_flag(s_full, i & 1, a.status, bad);
            wait_or_flag(&full[kslot], (n / kNSlot) & 1, a.status, bad);  // (complete already) the d bytes
            tc::fence_after();
            const uint8_t * kb = sm + S::ring + kslot * kSlot;
            float           dk[8];
#pragma unroll
            for (int b = 0; b < 8; b++) {
                const int       o  = 34 * b, oo = o & 127;
                const uint8_t * pr = kb + (o >> 7) * kPlane + t * 128 + ((((oo >> 4) ^ (t & 7))) << 4) + (oo & 15);
                dk[b]              = half_bits_to_float(*reinterpret_cast<const uint16_t *>(pr));
            }
            // s[r] = sum_b d_k[b] * d_q[b][r] * isum_b[r] (d_q carries scale * log2e)
            f2 s2[RH / 2];
#pragma unroll
            for (int j = 0; j < RH / 2; j++) s2[j] = 0ull;
            {
                // two blocks per tensor-memory round trip, the next pair loading while this one is scaled
                uint32_t v[2][2 * RH];
                tc::ld_cols<RH>(tc::taddr(tS, q, rbase), v[0]);
                tc::ld_cols<RH>(tc::taddr(tS, q, RP + rbase), v[0] + RH);
#pragma unroll
                for (int bp = 0; bp < 4; bp++) {
                    tc::wait_ld();
                    if (bp < 3) {
                        tc::ld_cols<RH>(tc::taddr(tS, q, RP * (2 * bp + 2) + rbase), v[(bp + 1) & 1]);
                        tc::ld_cols<RH>(tc::taddr(tS, q, RP * (2 * bp + 3) + rbase), v[(bp + 1) & 1] + RH);
                    }
#pragma unroll
                    for (int e = 0; e < 2; e++) {
                        const int        b   = 2 * bp + e;
                        const float4 *   dqc = reinterpret_cast<const float4 *>(dq + b * RP + rbase);
                        const f2         dk2 = f2_pack(dk[b], dk[b]);
                        const uint32_t * vb  = v[bp & 1] + e * RH;
#pragma unroll
                        for (int j4 = 0; j4 < RH / 4; j4++) {
                            const float4 d4 = dqc[j4];
                            const f2 x0 = f2_add(f2_pack(__uint_as_float(vb[4 * j4]), __uint_as_float(vb[4 * j4 + 1])), negC);
                            const f2 x1 = f2_add(f2_pack(__uint_as_float(vb[4 * j4 + 2]), __uint_as_float(vb[4 * j4 + 3])), negC);
                            s2[2 * j4]     = f2_fma(x0, f2_mul(f2_pack(d4.x, d4.y), dk2), s2[2 * j4]);
                            s2[2 * j4 + 1] = f2_fma(x1, f2_mul(f2_pack(d4.z, d4.w), dk2), s2[2 * j4 + 1]);
                        }
                    }
                }
            }
            // re-arm the accumulators, then release them (next Q.K) and the K slot
            arm_scores<RP>(tS, q, rbase);
            tc::wait_st();
            tc::fence_before();
            __syncwarp();
            if (lane == 0) mbar_arrive(s_free);
            float s[RH];
#pragma unroll
            for (int j = 0; j < RH / 2; j++) f2_unpack(s2[j], s[2 * j], s[2 * j + 1]);

            const int  tok   = t0 + i * kT + t;
            const bool valid = tok < t1;
            if (a.softcap_l2 != 0.0f) {
#pragma unroll
                for (int r = 0; r < RH; r++) s[r] = a.softcap_l2 * tanhf(s[r]);
            }
            if (a.mask_mode == 1) {
                const uint16_t * mb = mbuf + (i & 1) * S::MBR * kT + t;
#pragma unroll
                for (int r = 0; r < RH; r++) {
                    const float sl = a.max_bias > 0.0f ? slope2[rbase + r] : kLog2e;
                    const int   sl_r = (msl[r >> 2] >> (8 * (r & 3))) & 0xff;
                    s[r] = fmaf(sl, half_bits_to_float(mb[sl_r * kT]), s[r]);
                }
            } else if (a.mask_mode == 2 && valid) {
#pragma unroll
                for (int r = 0; r < RH; r++) {
                    const uint16_t mv16 = __ldg(reinterpret_cast<const unsigned short *>(a.mask + moff[rbase + r] +
                                                                                         2 * (int64_t) tok));
                    s[r] = fmaf(slope2[rbase + r], half_bits_to_float(mv16), s[r]);
                }
            }
            if (!valid) {
#pragma unroll
                for (int r = 0; r < RH; r++) s[r] = -INFINITY;
            }
            // tile maxima; the running maximum rises (second barrier) only when some row's tile maximum exceeds it
            // by more than 2^8
            float * redb = red + (i & 1) * 4 * RP;
            bool    up   = false;
            float   mx[RH];
#pragma unroll
            for (int r = 0; r < RH; r++) mx[r] = redux_max(s[r]);  // independent: all in flight together
#pragma unroll
            for (int r = 0; r < RH; r++) {
                if (lane == 0) redb[q * RP + rbase + r] = mx[r];
                up |= mx[r] > mu[rbase + r] + kLazy;
            }
            if (lane == 0 && up) flags[i % 3] = 1;
            // this thread's half of the tile's raw V row, read before the barrier: after it, the K and V slots are
            // rewritten with the f16 V^T halves
            uint32_t vw[20];
            wait_or_flag(&full[vslot], ((n + 1) / kNSlot) & 1, a.status, bad);
            load_v_part(sm + S::ring + vslot * kSlot + t * kRowB, qr, vw);
            if (stage) {
                *reinterpret_cast<uint4 *>(mbuf + ((i + 1) & 1) * S::MBR * kT + (tid >> 4) * kT + 8 * (tid & 15)) = mnext;
            }
            named_bar_sync(1, kCW * 32);
            if (tid == 0) flags[(i + 2) % 3] = 0;
            const bool resc = flags[i % 3] != 0;
            if (resc) {
                if (tid < RP) {
                    float mt = redb[tid];
#pragma unroll
                    for (int w = 1; w < 4; w++) mt = fmaxf(mt, redb[w * RP + tid]);
                    const float mo = mu[tid];
                    if (mt > mo + kLazy) {
                        mu[tid] = mt;
                        al[tid] = exp2f(mo - mt);
                    } else {
                        al[tid] = 1.0f;
                    }
                }
                named_bar_sync(1, kCW * 32);
            }
            if (i > 0) {
                wait_or_flag(pv_done, (i - 1) & 1, a.status, bad);
                tc::fence_after();
            }
            if (resc) {
#pragma unroll
                for (int r = 0; r < RH; r++) l[r] *= al[rbase + r];
                if (i > 0) {
#pragma unroll
                    for (int hf = 0; hf < 2; hf++) {
                        uint32_t       o[RH];
                        const uint32_t ta = tc::taddr(tO + hf * RP, q, rbase);
                        tc::ld_cols<RH>(ta, o);
                        tc::wait_ld();
#pragma unroll
                        for (int j = 0; j < RH; j++) o[j] = __float_as_uint(__uint_as_float(o[j]) * al[rbase + j]);
                        tc::st_cols<RH>(ta, o);
                    }
                    tc::wait_st();
                }
            }
            // P^T (MN-major: [row group of 8][token][8 f16])
            {
                uint32_t pk[RH / 2];
#pragma unroll
                for (int j = 0; j < RH / 2; j++) {
                    const int   r  = 2 * j, row = rbase + r;
                    const float m0 = mu[row], m1 = mu[row + 1];
                    const float p0 = ex2(s[r] - (m0 == -INFINITY ? 0.0f : m0));
                    const float p1 = ex2(s[r + 1] - (m1 == -INFINITY ? 0.0f : m1));
                    l[r] += p0;
                    l[r + 1] += p1;
                    const __half2 hp = __floats2half2_rn(p0, p1);
                    pk[j]            = *reinterpret_cast<const uint32_t *>(&hp);
                }
                store_p<RH>(sm + S::p, rbase, t, pk);
            }
            // V^T of blocks 2qr, 2qr+1: dv half 0 into the tile's K slot, half 1 into its V slot
            {
                uint8_t * vch = sm + S::ring + (qr >= 2 ? vslot : kslot) * kSlot;
                switch (qr) {
                    case 0: convert_v_part<0>(vw, vch, t); break;
                    case 1: convert_v_part<1>(vw, vch, t); break;
                    case 2: convert_v_part<2>(vw, vch, t); break;
                    default: convert_v_part<3>(vw, vch, t); break;
                }
            }
            asm volatile("fence.proxy.async.shared::cta;" ::: "memory");
            tc::fence_before();
            __syncwarp();
            if (lane == 0) mbar_arrive(pv_rdy);
        }

        // ---------------- epilogue ----------------
        // every CTA of the grid is resident by now: the chunk merge may launch (it waits for this grid to finish)
        pdl_launch_dependents();
        wait_or_flag(pv_done, (nt - 1) & 1, a.status, bad);
        tc::fence_after();
#pragma unroll
        for (int r = 0; r < RH; r++) {
            float v = l[r];
#pragma unroll
            for (int o = 16; o > 0; o >>= 1) v += __shfl_xor_sync(0xffffffffu, v, o);
            if (lane == 0) red[(nt & 1) * 4 * RP + q * RP + rbase + r] = v;
        }
        named_bar_sync(1, kCW * 32);
        const bool single = a.n_chunks == 1 && !a.parts_out;
        if (tid < rows) {
            const float * rs = red + (nt & 1) * 4 * RP;
            float Ssum = rs[tid];
#pragma unroll
            for (int w = 1; w < 4; w++) Ssum += rs[w * RP + tid];
            const int rr = row0 + tid;
            float     M  = mu[tid];
            if (single) {
                if (Ssum == 0.0f) M = -INFINITY;
                float ms = 1.0f;
                if (a.sinks) {
                    const int   h   = g * a.G + rr / a.N;
                    const float sk2 = a.sinks[h] * kLog2e;
                    if (sk2 > M) {
                        ms   = exp2f(M - sk2);
                        Ssum = Ssum * ms + 1.0f;
                    } else {
                        Ssum += exp2f(sk2 - M);
                    }
                }
                fac[tid] = Ssum == 0.0f ? 0.0f : ms / Ssum;
            } else {
                a.part_ms[(int64_t) (g * a.R + rr) * a.n_chunks + chunk] = make_float2(M, Ssum);
            }
        }
        named_bar_sync(1, kCW * 32);
#pragma unroll
        for (int hf = 0; hf < 2; hf++) {
            const int dv = hf * 128 + 32 * q + lane;
            uint32_t  o[RH];
            tc::ld_cols<RH>(tc::taddr(tO + hf * RP, q, rbase), o);
            tc::wait_ld();
#pragma unroll
            for (int j = 0; j < RH; j++) {
                const int r = rbase + j;
                if (r < rows) {
                    const int   rr  = row0 + r;
                    const float val = __uint_as_float(o[j]);
                    if (single) {
                        const int h = g * a.G + rr / a.N, tq = rr % a.N;
                        float * out = reinterpret_cast<float *>(reinterpret_cast<uint8_t *>(a.dst) + h * a.dnb1 +
                                                                tq * a.dnb2);
                        out[dv] = val * fac[r];
                    } else {
                        a.part_acc[((int64_t) (g * a.R + rr) * a.n_chunks + chunk) * kD + dv] = val;
                    }
                }
            }
        }
    }

    tc::fence_before();
    __syncthreads();
    if (warp == 0) tc::tmem_free(tbase, 512);
}

// ---------------------------------------------------------------------------------------------------------------
// f16 KV cache: the same pipeline without per-block scales. Q.K on kind::f16 with Q split into f16 hi + lo parts
// (exact to ~2^-22 of Q, so the scores carry f32-level accuracy as the reference's f32 GEMM does); the K tile arrives
// as SWIZZLE_128B planes of 64 dims (K-major operand), the V tile likewise and is the MN-major V^T operand as it lands
// (no conversion). Ring: 4 slots of 32 KB per tile (K dims 0-127, 128-255, V dims 0-127, 128-255); K slots return to
// the producer when Q.K completes, V slots when P.V does.

constexpr int kSlotF = kT * 256;  // 32768: 128 tokens x 128 dims of f16

template <int RP> struct SmemF {
    static constexpr int ring  = 0;                   // 4 slots
    static constexpr int p     = ring + 4 * kSlotF;
    static constexpr int qop   = p + RP * kT * 2;     // 16 dim-steps x {hi, lo} x [2][RP][16]
    static constexpr int red   = qop + 32 * RP * 32;  // f32 [2][4][RP]
    static constexpr int mu    = red + 2 * 4 * RP * 4;
    static constexpr int al    = mu + RP * 4;
    static constexpr int fac   = al + RP * 4;
    static constexpr int slope = fac + RP * 4;
    static constexpr int moff  = slope + RP * 4;      // int64 [RP]
    static constexpr int mslot = moff + RP * 8;       // int32 [RP]
    static constexpr int MBR   = 16;                  // staged mask rows (query tokens)
    static constexpr int mbuf  = (mslot + RP * 4 + 15) / 16 * 16;  // f16 [2][MBR][kT]
    static constexpr int bar   = mbuf + 2 * MBR * kT * 2;
    static constexpr int misc  = bar + 12 * 8;        // tmem base, flags[3]
    static constexpr int total = misc + 16;
    static constexpr int alloc = total + 1024;
};

__device__ __forceinline__ void tma3h(uint8_t * dst, const CUtensorMap * m, int x, int y, int z, uint64_t * bar) {
    tma3(dst, m, x, y, z, bar);
}

template <int RP>
__global__ void __launch_bounds__(kFaThreads, 1)
    fa_f16_kernel(const __grid_constant__ CUtensorMap mk, const __grid_constant__ CUtensorMap mv, const FaArgs a) {
    using S          = SmemF<RP>;
    constexpr int RH = RP / 4;
    extern __shared__ uint8_t smem_raw[];
    // 1024-byte aligned base, by pointer arithmetic on the shared array (an integer round trip would make every
    // access through `sm` a generic load / store)
    uint8_t * sm = smem_raw + ((1024u - (smem_u32(smem_raw) & 1023u)) & 1023u);
    uint64_t * full    = reinterpret_cast<uint64_t *>(sm + S::bar);
    uint64_t * empty   = full + 4;
    uint64_t * s_full  = empty + 4;
    uint64_t * s_free  = s_full + 1;
    uint64_t * pv_rdy  = s_full + 2;
    uint64_t * pv_done = s_full + 3;
    uint32_t * tptr    = reinterpret_cast<uint32_t *>(sm + S::misc);
    int *      flags   = reinterpret_cast<int *>(sm + S::misc + 4);
    float *    red     = reinterpret_cast<float *>(sm + S::red);
    float *    mu      = reinterpret_cast<float *>(sm + S::mu);
    float *    al      = reinterpret_cast<float *>(sm + S::al);
    float *    fac     = reinterpret_cast<float *>(sm + S::fac);
    float *    slope2  = reinterpret_cast<float *>(sm + S::slope);
    int64_t *  moff    = reinterpret_cast<int64_t *>(sm + S::moff);
    int *      mslot   = reinterpret_cast<int *>(sm + S::mslot);
    uint16_t * mbuf    = reinterpret_cast<uint16_t *>(sm + S::mbuf);

    const int tid = threadIdx.x, warp = tid >> 5, lane = tid & 31;
    const int chunk = blockIdx.x;
    const int g = blockIdx.y / a.nrg, rg = blockIdx.y % a.nrg;
    const int t0 = chunk * a.chunk_len, t1 = min(a.L, t0 + a.chunk_len);
    const int nt = (t1 - t0 + kT - 1) / kT;
    const int row0 = rg * RP;
    const int rows = min(RP, a.R - row0);
    const int q = warp & 3, qr = (warp >> 2) & 3, t = 32 * q + lane, rbase = qr * RH;
    bool      bad = false;

    if (tid == 0) {
        for (int i = 0; i < 4; i++) {
            mbar_init(&full[i], 1);
            mbar_init(&empty[i], 1);  // released by a tcgen05.commit
        }
        mbar_init(s_full, 1);
        mbar_init(s_free, kCW);
        mbar_init(pv_rdy, kCW);
        mbar_init(pv_done, 1);
        fence_mbar_init();
        flags[0] = flags[1] = flags[2] = 0;
    }
    if (warp == 0) tc::tmem_alloc(tptr, 256);
    tc::fence_before();
    __syncthreads();
    tc::fence_after();
    const uint32_t tbase = *tptr;
    const uint32_t tS    = tbase;        // S^T [token][row] at columns 0..RP-1 (f32)
    const uint32_t tO    = tbase + RP;   // O^T halves at tO, tO + RP

    // tile i uses slot s for: K dims 128 s.. (s = 0, 1), V dims 128 (s - 2).. (s = 2, 3); two 64-dim planes each
    auto produce = [&](int i, int sl) {
        uint8_t * dst = sm + S::ring + sl * kSlotF;
        const int tok = t0 + i * kT;
        mbar_arrive_expect_tx(&full[sl], kSlotF);
        const CUtensorMap * m  = sl < 2 ? &mk : &mv;
        const int           x0 = 128 * (sl & 1);
        tma3h(dst, m, x0, tok, g, &full[sl]);
        tma3h(dst + kPlane, m, x0 + 64, tok, g, &full[sl]);
    };
    if (warp == kCW && lane == 0) {
        prefetch_tmap(&mk);
        prefetch_tmap(&mv);
    }
    pdl_wait();  // programmatic dependent launch: the writer of Q and of the newest K/V rows has finished
    if (warp == kCW && lane == 0) {
        for (int sl = 0; sl < 4; sl++) produce(0, sl);
    }
    __syncwarp();

    // Q rows -> f16 hi + lo parts into the 16 dim-step operands; per-row constants
    if (warp < kCW) {
        for (int u = tid; u < RP * 64; u += kCW * 32) {  // 4 dims per unit
            const int r = u >> 6, d0 = (u & 63) * 4;
            float     x[4] = { 0.0f, 0.0f, 0.0f, 0.0f };
            if (r < rows) {
                const int     rr  = row0 + r;
                const int     h   = g * a.G + rr / a.N, tq = rr % a.N;
                const float * src = reinterpret_cast<const float *>(reinterpret_cast<const uint8_t *>(a.q) +
                                                                     tq * a.qnb1 + h * a.qnb2);
#pragma unroll
                for (int e = 0; e < 4; e++) x[e] = src[d0 + e];
            }
#pragma unroll
            for (int e = 0; e < 4; e++) {
                const int    d = d0 + e, j = d >> 4, xx = d & 15;
                const __half hi = __float2half_rn(x[e]);
                const __half lo = __float2half_rn(x[e] - __half2float(hi));
                const int    o  = (xx >> 3) * RP * 16 + r * 16 + (xx & 7) * 2;
                *reinterpret_cast<__half *>(sm + S::qop + (2 * j) * RP * 32 + o)     = hi;
                *reinterpret_cast<__half *>(sm + S::qop + (2 * j + 1) * RP * 32 + o) = lo;
            }
        }
        if (tid < RP) {
            const int r = tid, rr = row0 + min(r, rows - 1);
            const int h = g * a.G + rr / a.N, tq = rr % a.N;
            float     sl = 1.0f;
            if (a.max_bias > 0.0f) {
                sl = h < a.n_head_log2 ? powf(a.m0, (float) (h + 1)) : powf(a.m1, (float) (2 * (h - a.n_head_log2) + 1));
            }
            slope2[r] = sl * kLog2e;
            moff[r]   = a.mask ? (int64_t) tq * a.mnb1 + (int64_t) (h % a.mne2) * a.mnb2 : 0;
            mslot[r]  = tq;
            mu[r]     = -INFINITY;
        }
        if (a.mask_mode == 1 && tid < a.N * 16) {  // N <= MBR
            *reinterpret_cast<uint4 *>(mbuf + (tid >> 4) * kT + 8 * (tid & 15)) = mask_piece(a, tid, t0);
        }
    }
    asm volatile("fence.proxy.async.shared::cta;" ::: "memory");
    tc::fence_before();
    __syncthreads();
    tc::fence_after();

    const uint32_t qop_s = smem_u32(sm + S::qop);
    const uint32_t p_s   = smem_u32(sm + S::p);

    if (warp == kCW) {
        // ---------------- producer ----------------
        if (lane == 0) {
            for (int i = 1; i < nt && !bad; i++) {
                for (int sl = 0; sl < 4; sl++) {
                    if (!wait_or_flag(&empty[sl], (i - 1) & 1, a.status, bad)) break;
                    produce(i, sl);
                }
            }
        }
        __syncwarp();
    } else if (warp == kCW + 1) {
        // ---------------- MMA issuer ----------------
        if (lane == 0) {
            constexpr uint32_t idqk = tc::idesc(tc::kD_F32, tc::kAB_F16, tc::kAB_F16, tc::kKMajor, tc::kKMajor, RP, 128);
            constexpr uint32_t idpv = tc::idesc(tc::kD_F32, tc::kAB_F16, tc::kAB_F16, tc::kMNMajor, tc::kMNMajor, RP,
                                                128);
            auto issue_qk = [&](int i) {
                wait_or_flag(&full[0], i & 1, a.status, bad);
                wait_or_flag(&full[1], i & 1, a.status, bad);
                tc::fence_after();
                const uint32_t kb = smem_u32(sm + S::ring);
#pragma unroll
                for (int j = 0; j < 16; j++) {  // 16 dims per MMA: 32 bytes of a 128-byte swizzled row
                    const int      jj = j & 7;
                    const uint64_t ad = tc::sdesc(kb + (j >> 3) * kSlotF + (jj >> 2) * kPlane + (jj & 3) * 32, 16,
                                                  1024) | (2ull << 61);
                    tc::mma_f16(tS, ad, tc::sdesc(qop_s + (2 * j) * RP * 32, RP * 16, 128), idqk, (uint32_t) (j > 0));
                    tc::mma_f16(tS, ad, tc::sdesc(qop_s + (2 * j + 1) * RP * 32, RP * 16, 128), idqk, 1u);
                }
                tc::commit(s_full);
                tc::commit(&empty[0]);
                tc::commit(&empty[1]);
            };
            issue_qk(0);
            for (int i = 0; i < nt; i++) {
                if (i + 1 < nt) {
                    wait_or_flag(s_free, i & 1, a.status, bad);
                    issue_qk(i + 1);
                }
                wait_or_flag(pv_rdy, i & 1, a.status, bad);
                wait_or_flag(&full[2], i & 1, a.status, bad);
                wait_or_flag(&full[3], i & 1, a.status, bad);
                tc::fence_after();
#pragma unroll
                for (int hf = 0; hf < 2; hf++) {
                    const uint32_t vb = smem_u32(sm + S::ring + (2 + hf) * kSlotF);
#pragma unroll
                    for (int k = 0; k < kT / 16; k++) {  // 16 tokens = two 8-row groups of the swizzled planes
                        const uint64_t ad = tc::sdesc(vb + k * 2048, kPlane, 1024) | (2ull << 61);
                        const uint64_t bd = tc::sdesc(p_s + k * 256, 128, kT * 16);
                        tc::mma_f16(tO + hf * RP, ad, bd, idpv, (uint32_t) (i > 0 || k > 0));
                    }
                }
                tc::commit(pv_done);
                tc::commit(&empty[2]);
                tc::commit(&empty[3]);
            }
        }
        __syncwarp();
    } else {
        // ---------------- compute warps ----------------
        float l[RH];
#pragma unroll
        for (int r = 0; r < RH; r++) l[r] = 0.0f;
        uint32_t msl[RH / 4];
#pragma unroll
        for (int j = 0; j < RH / 4; j++) {
            msl[j] = 0;
#pragma unroll
            for (int e = 0; e < 4; e++) msl[j] |= (uint32_t) (mslot[rbase + 4 * j + e] & 0xff) << (8 * e);
        }
        for (int i = 0; i < nt; i++) {
            uint4      mnext = make_uint4(0, 0, 0, 0);
            const bool stage = a.mask_mode == 1 && i + 1 < nt && tid < a.N * 16;
            if (stage) mnext = mask_piece(a, tid, t0 + (i + 1) * kT);
            wait_or_flag(s_full, i & 1, a.status, bad);
            tc::fence_after();
            float s[RH];
            {
                uint32_t v[RH];
                tc::ld_cols<RH>(tc::taddr(tS, q, rbase), v);
                tc::wait_ld();
#pragma unroll
                for (int r = 0; r < RH; r++) s[r] = __uint_as_float(v[r]);
            }
            tc::fence_before();
            __syncwarp();
            if (lane == 0) mbar_arrive(s_free);
            if (a.softcap_l2 != 0.0f) {
#pragma unroll
                for (int r = 0; r < RH; r++) s[r] = a.softcap_l2 * tanhf(s[r] * a.qscale);
            } else {
#pragma unroll
                for (int r = 0; r < RH; r++) s[r] *= a.qscale;
            }
            const int  tok   = t0 + i * kT + t;
            const bool valid = tok < t1;
            if (a.mask_mode == 1) {
                const uint16_t * mb = mbuf + (i & 1) * S::MBR * kT + t;
#pragma unroll
                for (int r = 0; r < RH; r++) {
                    const float sl   = a.max_bias > 0.0f ? slope2[rbase + r] : kLog2e;
                    const int   sl_r = (msl[r >> 2] >> (8 * (r & 3))) & 0xff;
                    s[r] = fmaf(sl, half_bits_to_float(mb[sl_r * kT]), s[r]);
                }
            } else if (a.mask_mode == 2 && valid) {
#pragma unroll
                for (int r = 0; r < RH; r++) {
                    const uint16_t mv16 = __ldg(reinterpret_cast<const unsigned short *>(a.mask + moff[rbase + r] +
                                                                                         2 * (int64_t) tok));
                    s[r] = fmaf(slope2[rbase + r], half_bits_to_float(mv16), s[r]);
                }
            }
            if (!valid) {
#pragma unroll
                for (int r = 0; r < RH; r++) s[r] = -INFINITY;
            }
            float * redb = red + (i & 1) * 4 * RP;
            bool    up   = false;
            float   mx[RH];
#pragma unroll
            for (int r = 0; r < RH; r++) mx[r] = redux_max(s[r]);
#pragma unroll
            for (int r = 0; r < RH; r++) {
                if (lane == 0) redb[q * RP + rbase + r] = mx[r];
                up |= mx[r] > mu[rbase + r] + kLazy;
            }
            if (lane == 0 && up) flags[i % 3] = 1;
            if (stage) {
                *reinterpret_cast<uint4 *>(mbuf + ((i + 1) & 1) * S::MBR * kT + (tid >> 4) * kT + 8 * (tid & 15)) = mnext;
            }
            named_bar_sync(1, kCW * 32);
            if (tid == 0) flags[(i + 2) % 3] = 0;
            const bool resc = flags[i % 3] != 0;
            if (resc) {
                if (tid < RP) {
                    float mt = redb[tid];
#pragma unroll
                    for (int w = 1; w < 4; w++) mt = fmaxf(mt, redb[w * RP + tid]);
                    const float mo = mu[tid];
                    if (mt > mo + kLazy) {
                        mu[tid] = mt;
                        al[tid] = exp2f(mo - mt);
                    } else {
                        al[tid] = 1.0f;
                    }
                }
                named_bar_sync(1, kCW * 32);
            }
            if (i > 0) {
                wait_or_flag(pv_done, (i - 1) & 1, a.status, bad);
                tc::fence_after();
            }
            if (resc) {
#pragma unroll
                for (int r = 0; r < RH; r++) l[r] *= al[rbase + r];
                if (i > 0) {
#pragma unroll
                    for (int hf = 0; hf < 2; hf++) {
                        uint32_t       o[RH];
                        const uint32_t ta = tc::taddr(tO + hf * RP, q, rbase);
                        tc::ld_cols<RH>(ta, o);
                        tc::wait_ld();
#pragma unroll
                        for (int j = 0; j < RH; j++) o[j] = __float_as_uint(__uint_as_float(o[j]) * al[rbase + j]);
                        tc::st_cols<RH>(ta, o);
                    }
                    tc::wait_st();
                }
            }
            {
                uint32_t pk[RH / 2];
#pragma unroll
                for (int j = 0; j < RH / 2; j++) {
                    const int   r  = 2 * j, row = rbase + r;
                    const float m0 = mu[row], m1 = mu[row + 1];
                    const float p0 = ex2(s[r] - (m0 == -INFINITY ? 0.0f : m0));
                    const float p1 = ex2(s[r + 1] - (m1 == -INFINITY ? 0.0f : m1));
                    l[r] += p0;
                    l[r + 1] += p1;
                    const __half2 hp = __floats2half2_rn(p0, p1);
                    pk[j]            = *reinterpret_cast<const uint32_t *>(&hp);
                }
                store_p<RH>(sm + S::p, rbase, t, pk);
            }
            asm volatile("fence.proxy.async.shared::cta;" ::: "memory");
            tc::fence_before();
            __syncwarp();
            if (lane == 0) mbar_arrive(pv_rdy);
        }

        // ---------------- epilogue ----------------
        // every CTA of the grid is resident by now: the chunk merge may launch (it waits for this grid to finish)
        pdl_launch_dependents();
        wait_or_flag(pv_done, (nt - 1) & 1, a.status, bad);
        tc::fence_after();
#pragma unroll
        for (int r = 0; r < RH; r++) {
            float v = l[r];
#pragma unroll
            for (int o = 16; o > 0; o >>= 1) v += __shfl_xor_sync(0xffffffffu, v, o);
            if (lane == 0) red[(nt & 1) * 4 * RP + q * RP + rbase + r] = v;
        }
        named_bar_sync(1, kCW * 32);
        const bool single = a.n_chunks == 1 && !a.parts_out;
        if (tid < rows) {
            const float * rs   = red + (nt & 1) * 4 * RP;
            float         Ssum = rs[tid];
#pragma unroll
            for (int w = 1; w < 4; w++) Ssum += rs[w * RP + tid];
            const int rr = row0 + tid;
            float     M  = mu[tid];
            if (single) {
                if (Ssum == 0.0f) M = -INFINITY;
                float ms = 1.0f;
                if (a.sinks) {
                    const int   h   = g * a.G + rr / a.N;
                    const float sk2 = a.sinks[h] * kLog2e;
                    if (sk2 > M) {
                        ms   = exp2f(M - sk2);
                        Ssum = Ssum * ms + 1.0f;
                    } else {
                        Ssum += exp2f(sk2 - M);
                    }
                }
                fac[tid] = Ssum == 0.0f ? 0.0f : ms / Ssum;
            } else {
                a.part_ms[(int64_t) (g * a.R + rr) * a.n_chunks + chunk] = make_float2(M, Ssum);
            }
        }
        named_bar_sync(1, kCW * 32);
#pragma unroll
        for (int hf = 0; hf < 2; hf++) {
            const int dv = hf * 128 + 32 * q + lane;
            uint32_t  o[RH];
            tc::ld_cols<RH>(tc::taddr(tO + hf * RP, q, rbase), o);
            tc::wait_ld();
#pragma unroll
            for (int j = 0; j < RH; j++) {
                const int r = rbase + j;
                if (r < rows) {
                    const int   rr  = row0 + r;
                    const float val = __uint_as_float(o[j]);
                    if (single) {
                        const int h = g * a.G + rr / a.N, tq = rr % a.N;
                        float * out = reinterpret_cast<float *>(reinterpret_cast<uint8_t *>(a.dst) + h * a.dnb1 +
                                                                tq * a.dnb2);
                        out[dv] = val * fac[r];
                    } else {
                        a.part_acc[((int64_t) (g * a.R + rr) * a.n_chunks + chunk) * kD + dv] = val;
                    }
                }
            }
        }
    }

    tc::fence_before();
    __syncthreads();
    if (warp == 0) tc::tmem_free(tbase, 256);
}

// merge of the chunk records of one row (P:787-823), then sinks and normalization; one CTA per (KV head, row).
// The same merge combines the record sets of several devices (each the merged record of its KV range) and, with
// parts_out, leaves this device's merged record unnormalized for such a merge.
__global__ void __launch_bounds__(256) fa_combine_kernel(const FaArgs a) {
    // the next kernel (the attention output projection) may become resident and stream its first weights now; it
    // waits for this grid before it reads the output
    pdl_launch_dependents();
    pdl_wait();
    const int row = blockIdx.x, g = row / a.R, rr = row % a.R;
    const int h = g * a.G + rr / a.N, tq = rr % a.N;
    __shared__ float w_s[256];  // per chunk: weight 2^(M_c - M) (0 for empty chunks)
    __shared__ float s_s[256];
    __shared__ float mf_s;
    const float2 * ms = a.part_ms + (int64_t) row * a.ms_row;
    const int      nc = a.n_chunks;  // <= 256 (fa_plan: one chunk per CTA of a wave at most; merge: checked)
    const int      dv  = threadIdx.x;
    const float *  src = a.part_acc + (int64_t) row * a.acc_row + dv;
    const int64_t  ac  = a.acc_chunk, mc = a.ms_chunk;
    // the first kPre chunks' partial outputs do not depend on the (max, sum) records: in flight with them
    constexpr int kPre = 32;
    float         pre[kPre];
#pragma unroll
    for (int c = 0; c < kPre; c++) pre[c] = c < nc ? __ldcg(src + c * ac) : 0.0f;
    if (threadIdx.x < 32) {
        float m = -INFINITY;
        for (int c = threadIdx.x; c < nc; c += 32) {
            const float2 v = ms[c * mc];
            if (v.y != 0.0f) m = fmaxf(m, v.x);
        }
#pragma unroll
        for (int o = 16; o > 0; o >>= 1) m = fmaxf(m, __shfl_xor_sync(0xffffffffu, m, o));
        if (threadIdx.x == 0) mf_s = m;
    }
    __syncthreads();
    const float Mf = mf_s;
    for (int c = threadIdx.x; c < nc; c += blockDim.x) {
        const float2 v = ms[c * mc];
        w_s[c]         = v.y != 0.0f ? exp2f(v.x - Mf) : 0.0f;
        s_s[c]         = v.y;
    }
    __syncthreads();
    float acc = 0.0f, S = 0.0f;
#pragma unroll
    for (int c = 0; c < kPre; c++) {
        if (c < nc) {
            const float w = w_s[c];
            acc           = fmaf(w, w != 0.0f ? pre[c] : 0.0f, acc);
            S             = fmaf(w, s_s[c], S);
        }
    }
#pragma unroll 8
    for (int c = kPre; c < nc; c++) {
        const float w = w_s[c];
        acc           = fmaf(w, w != 0.0f ? src[c * ac] : 0.0f, acc);
        S             = fmaf(w, s_s[c], S);
    }
    if (a.parts_out) {  // an empty range leaves (-inf, 0) and zeros: skipped by the merge
        if (dv == 0) a.rec_ms[row] = make_float2(Mf, S);
        a.rec_acc[(int64_t) row * kD + dv] = acc;
        return;
    }
    if (a.sinks) {
        const float sk2 = a.sinks[h] * kLog2e;
        if (sk2 > Mf) {
            const float m2 = exp2f(Mf - sk2);
            acc *= m2;
            S = S * m2 + 1.0f;
        } else {
            S += exp2f(sk2 - Mf);
        }
    }
    const float inv = S == 0.0f ? 0.0f : 1.0f / S;
    float * out = reinterpret_cast<float *>(reinterpret_cast<uint8_t *>(a.dst) + h * a.dnb1 + tq * a.dnb2);
    out[dv]     = acc * inv;
}

using EncodeTiled = CUresult (*)(CUtensorMap *, CUtensorMapDataType, cuuint32_t, void *, const cuuint64_t *,
                                 const cuuint64_t *, const cuuint32_t *, const cuuint32_t *, CUtensorMapInterleave,
                                 CUtensorMapSwizzle, CUtensorMapL2promotion, CUtensorMapFloatOOBfill);

EncodeTiled fa_encode_fn() {
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

struct Plan {
    int nrg, rp, n_chunks, chunk_len;
};

Plan fa_plan(int num_sms, int R, int L, int Hkv) {
    Plan      p;
    const int max_ch = (L + kT - 1) / kT;
    if (Hkv * max_ch >= num_sms) {
        // long caches: the fewest row groups of <= 48 rows (each group reads every KV byte), rows split evenly
        // between them (54 rows: 2 x 32, not 48 + 16: equal groups advance through the same tiles together, so the
        // second read of a tile comes from L2, and neither carries a mostly empty tile); as many chunks of at least
        // two tiles as fill the SMs in ONE wave (one CTA per SM: a CTA more than the SMs runs as a second wave)
        p.nrg            = (R + kRG - 1) / kRG;
        p.rp             = ((R + p.nrg - 1) / p.nrg + 15) / 16 * 16;
        const int groups = Hkv * p.nrg;
        int       want   = std::max(1, std::min(max_ch, num_sms / groups));
        if (max_ch >= 2) want = std::min(want, max_ch / 2);
        want             = std::max(1, want);
        const int per    = (L + want - 1) / want;
        p.chunk_len      = (per + kT - 1) / kT * kT;
    } else {
        // short caches (fewer 128-token tiles than SMs): one wave of CTAs with the fewest tiles each; among row-group
        // sizes with equal tiles per CTA the one with the fewest padded rows, then the fewest groups (K/V reads)
        int best_tpc = 1 << 30, best_pad = 0;
        for (const int rp : { 16, 32, kRG }) {
            const int nrg    = (R + rp - 1) / rp;
            const int groups = Hkv * nrg;
            const int want   = std::max(1, std::min(max_ch, num_sms / groups));
            const int tpc    = (max_ch + want - 1) / want;
            if (tpc < best_tpc || (tpc == best_tpc && nrg * rp < best_pad) ||
                (tpc == best_tpc && nrg * rp == best_pad && nrg < p.nrg)) {
                best_tpc = tpc;
                best_pad = nrg * rp;
                p.rp     = rp;
                p.nrg    = nrg;
            }
        }
        p.chunk_len = best_tpc * kT;
    }
    p.n_chunks = (L + p.chunk_len - 1) / p.chunk_len;
    return p;
}

int launch_combine(srhpm_ctx * ctx, const FaArgs & a, cudaStream_t stream) {
    cudaLaunchConfig_t  cfg = {};
    cudaLaunchAttribute attr[1];
    cfg.gridDim                                        = dim3(a.Hkv * a.R);
    cfg.blockDim                                       = dim3(kD);
    cfg.dynamicSmemBytes                               = 0;
    cfg.stream                                         = stream;
    attr[0].id                                         = cudaLaunchAttributeProgrammaticStreamSerialization;
    attr[0].val.programmaticStreamSerializationAllowed = 1;
    cfg.attrs                                          = attr;
    cfg.numAttrs                                       = 1;
    const int st = cuda_status(cudaLaunchKernelEx(&cfg, fa_combine_kernel, a));
    ctx->launches.fetch_add(1);
    return st;
}

template <class K> int set_smem(srhpm_ctx * ctx, K kern, int bytes, std::atomic<unsigned> & done) {
    if (!(done.load() & (1u << ctx->device))) {
        const int st = cuda_status(cudaFuncSetAttribute(kern, cudaFuncAttributeMaxDynamicSharedMemorySize, bytes));
        if (st != SRHPM_OK) return st;
        done.fetch_or(1u << ctx->device);
    }
    return SRHPM_OK;
}

template <int RP>
int launch_fa(srhpm_ctx * ctx, const FaArgs & a, const CUtensorMap & mk128, const CUtensorMap & mk32,
              const CUtensorMap & mv, cudaStream_t stream) {
    static std::atomic<unsigned> done{ 0 };
    int st = set_smem(ctx, fa_q80_kernel<RP>, Smem<RP>::alloc, done);
    if (st != SRHPM_OK) return st;
    st = cuda_status(launch_k_pdl(fa_q80_kernel<RP>, dim3(a.n_chunks, a.Hkv * a.nrg), dim3(kFaThreads),
                                Smem<RP>::alloc, stream, mk128, mk32, mv, a));
    ctx->launches.fetch_add(1);
    if (st != SRHPM_OK || a.n_chunks == 1) return st;
    return launch_combine(ctx, a, stream);
}

template <int RP>
int launch_fa_f16(srhpm_ctx * ctx, const FaArgs & a, const CUtensorMap & mk, const CUtensorMap & mv,
                  cudaStream_t stream) {
    static std::atomic<unsigned> done{ 0 };
    int st = set_smem(ctx, fa_f16_kernel<RP>, SmemF<RP>::alloc, done);
    if (st != SRHPM_OK) return st;
    st = cuda_status(launch_k_pdl(fa_f16_kernel<RP>, dim3(a.n_chunks, a.Hkv * a.nrg), dim3(kFaThreads),
                                SmemF<RP>::alloc, stream, mk, mv, a));
    ctx->launches.fetch_add(1);
    if (st != SRHPM_OK || a.n_chunks == 1) return st;
    return launch_combine(ctx, a, stream);
}

}  // namespace

size_t fa_work_size(int num_sms, int R, int L, int Hkv) {
    const Plan p = fa_plan(num_sms, R, L, Hkv);
    if (p.n_chunks == 1) return 0;
    const size_t rows = (size_t) Hkv * R * p.n_chunks;
    return rows * kD * sizeof(float) + rows * sizeof(float2) + 256;
}

int fa_run(srhpm_ctx * ctx, const FaView & v, float scale, float max_bias, float softcap, void * wdata, size_t wsize,
           cudaStream_t stream, void * rec) {
    const int  G   = v.H / v.Hkv;
    const int  R   = G * v.N;
    const Plan p   = fa_plan(ctx->num_sms, R, v.L, v.Hkv);
    const size_t need = fa_work_size(ctx->num_sms, R, v.L, v.Hkv);
    if (need > 0 && (wdata == nullptr || wsize < need)) return SRHPM_ERR_WORKSPACE;

    FaArgs a   = {};
    a.q        = v.q;
    a.qnb1     = v.qnb1;
    a.qnb2     = v.qnb2;
    a.N        = v.N;
    a.H        = v.H;
    a.G        = G;
    a.R        = R;
    a.L        = v.L;
    a.Hkv      = v.Hkv;
    a.nrg      = p.nrg;
    a.chunk_len = p.chunk_len;
    a.n_chunks = p.n_chunks;
    a.mask     = v.mask;
    a.mnb1     = v.mnb1;
    a.mnb2     = v.mnb2;
    a.mne2     = v.mne2;
    a.mne0     = v.mne0;
    a.mask_mode = 0;
    if (v.mask) {
        const int  mbr    = v.kv_type == SRHPM_TYPE_F16 ? SmemF<16>::MBR : (p.rp == 48 ? Smem<48>::MBR : Smem<16>::MBR);
        const bool staged = v.mne2 == 1 && v.N <= mbr && reinterpret_cast<uintptr_t>(v.mask) % 16 == 0 &&
                            v.mnb1 % 16 == 0;
        a.mask_mode = staged ? 1 : 2;
    }
    if (softcap != 0.0f) {
        a.qscale     = scale / softcap;
        a.softcap_l2 = softcap * kLog2e;
    } else {
        a.qscale     = scale * kLog2e;
        a.softcap_l2 = 0.0f;
    }
    a.max_bias    = max_bias;
    a.n_head_log2 = 1 << (int) floor(log2((double) v.H));
    a.m0          = powf(2.0f, -(max_bias) / a.n_head_log2);
    a.m1          = powf(2.0f, -(max_bias / 2.0f) / a.n_head_log2);
    a.sinks       = v.sinks;
    a.dst         = v.dst;
    a.dnb1        = v.dnb1;
    a.dnb2        = v.dnb2;
    if (p.n_chunks > 1) {
        const size_t rows = (size_t) v.Hkv * R * p.n_chunks;
        a.part_acc        = reinterpret_cast<float *>(wdata);
        a.part_ms = reinterpret_cast<float2 *>(reinterpret_cast<uint8_t *>(wdata) + rows * kD * sizeof(float));
    }
    a.ms_row    = p.n_chunks;
    a.ms_chunk  = 1;
    a.acc_row   = (int64_t) p.n_chunks * kD;
    a.acc_chunk = kD;
    if (rec) {
        // record set of this KV range: {max, sum} per row, then the rows' unnormalized outputs; sinks belong to the
        // merge of all ranges
        a.parts_out = 1;
        a.sinks     = nullptr;
        a.rec_ms    = reinterpret_cast<float2 *>(rec);
        a.rec_acc   = reinterpret_cast<float *>(reinterpret_cast<uint8_t *>(rec) + fa_part_ms_bytes(v.H, v.N));
        if (p.n_chunks == 1) {  // the one chunk's record is the range's record
            a.part_ms  = a.rec_ms;
            a.part_acc = a.rec_acc;
        }
    }
    a.status = ctx->d_status;
    a.q8mode = ctx->q8_0_act_mode;

    EncodeTiled enc = fa_encode_fn();
    if (!enc) return SRHPM_ERR_CUDA;
    if (v.kv_type == SRHPM_TYPE_F16) {
        a.qscale = softcap != 0.0f ? scale / softcap : scale * kLog2e;  // applied to the f32 scores
        CUtensorMap      mk, mv;
        const cuuint64_t dims[3] = { kD, (cuuint64_t) v.L, (cuuint64_t) v.Hkv };
        const cuuint64_t kst[2]  = { (cuuint64_t) v.knb1, (cuuint64_t) v.knb2 };
        const cuuint64_t vst[2]  = { (cuuint64_t) v.vnb1, (cuuint64_t) v.vnb2 };
        const cuuint32_t box[3]  = { 64, kT, 1 }, es[3] = { 1, 1, 1 };
        if (enc(&mk, CU_TENSOR_MAP_DATA_TYPE_UINT16, 3, const_cast<uint8_t *>(v.k), dims, kst, box, es,
                CU_TENSOR_MAP_INTERLEAVE_NONE, CU_TENSOR_MAP_SWIZZLE_128B, CU_TENSOR_MAP_L2_PROMOTION_L2_256B,
                CU_TENSOR_MAP_FLOAT_OOB_FILL_NONE) != CUDA_SUCCESS ||
            enc(&mv, CU_TENSOR_MAP_DATA_TYPE_UINT16, 3, const_cast<uint8_t *>(v.v), dims, vst, box, es,
                CU_TENSOR_MAP_INTERLEAVE_NONE, CU_TENSOR_MAP_SWIZZLE_128B, CU_TENSOR_MAP_L2_PROMOTION_L2_256B,
                CU_TENSOR_MAP_FLOAT_OOB_FILL_NONE) != CUDA_SUCCESS) {
            return SRHPM_ERR_INVALID;
        }
        switch (p.rp) {
            case 16: return launch_fa_f16<16>(ctx, a, mk, mv, stream);
            case 32: return launch_fa_f16<32>(ctx, a, mk, mv, stream);
            default: return launch_fa_f16<48>(ctx, a, mk, mv, stream);
        }
    }
    CUtensorMap      mk128, mk32, mv;
    const cuuint64_t kdims[3] = { kRowB / 4, (cuuint64_t) v.L, (cuuint64_t) v.Hkv };
    const cuuint64_t kstr[2]  = { (cuuint64_t) v.knb1, (cuuint64_t) v.knb2 };
    const cuuint64_t vstr[2]  = { (cuuint64_t) v.vnb1, (cuuint64_t) v.vnb2 };
    const cuuint32_t b128[3] = { 32, kT, 1 }, b32[3] = { 8, kT, 1 }, bv[3] = { kRowB / 4, kT, 1 };
    const cuuint32_t es[3]   = { 1, 1, 1 };
    if (enc(&mk128, CU_TENSOR_MAP_DATA_TYPE_UINT32, 3, const_cast<uint8_t *>(v.k), kdims, kstr, b128, es,
            CU_TENSOR_MAP_INTERLEAVE_NONE, CU_TENSOR_MAP_SWIZZLE_128B, CU_TENSOR_MAP_L2_PROMOTION_L2_256B,
            CU_TENSOR_MAP_FLOAT_OOB_FILL_NONE) != CUDA_SUCCESS ||
        enc(&mk32, CU_TENSOR_MAP_DATA_TYPE_UINT32, 3, const_cast<uint8_t *>(v.k), kdims, kstr, b32, es,
            CU_TENSOR_MAP_INTERLEAVE_NONE, CU_TENSOR_MAP_SWIZZLE_32B, CU_TENSOR_MAP_L2_PROMOTION_L2_256B,
            CU_TENSOR_MAP_FLOAT_OOB_FILL_NONE) != CUDA_SUCCESS ||
        enc(&mv, CU_TENSOR_MAP_DATA_TYPE_UINT32, 3, const_cast<uint8_t *>(v.v), kdims, vstr, bv, es,
            CU_TENSOR_MAP_INTERLEAVE_NONE, CU_TENSOR_MAP_SWIZZLE_NONE, CU_TENSOR_MAP_L2_PROMOTION_L2_256B,
            CU_TENSOR_MAP_FLOAT_OOB_FILL_NONE) != CUDA_SUCCESS) {
        return SRHPM_ERR_INVALID;
    }
    switch (p.rp) {
        case 16: return launch_fa<16>(ctx, a, mk128, mk32, mv, stream);
        case 32: return launch_fa<32>(ctx, a, mk128, mk32, mv, stream);
        default: return launch_fa<48>(ctx, a, mk128, mk32, mv, stream);
    }
}

// record set: {max, sum} pairs [H * N] padded to 16 bytes, then acc [H * N][256]
size_t fa_part_ms_bytes(int64_t H, int64_t N) { return ((size_t) (H * N) * sizeof(float2) + 15) / 16 * 16; }
size_t fa_part_bytes(int64_t H, int64_t N) { return fa_part_ms_bytes(H, N) + (size_t) (H * N) * kD * sizeof(float); }

// ---- the record merge over peer memory ---------------------------------------------------------------------------
// Every rank's buffer (mapped on every rank) holds its record set (fa_part_bytes(H, N), written by
// srhpm_flash_attn_ext_partial), then a receive area [2 slots][kArMaxRanks source ranks][H * N rows][258] of 8-byte
// words (value bits low, epoch high): the row's 256 unnormalized outputs, then its max and sum. CTA = row
// r = h * N + t. The CTA stores its record row, with the row's epoch, into every rank's receive area (source = this
// rank), then reads its own until each word from each rank carries the epoch (the flag-in-word exchange of
// allreduce.cuh: an aligned 64-bit store is single-copy atomic, so no fence or flag round is needed), merges the rows
// in rank order with fa_combine_kernel's arithmetic, adds the sinks and normalizes into dst. Slot = epoch parity: a
// rank sends its next-but-one exchange of a row only after this rank's words of the next one reached it, which this
// rank sends after reading the slot, so two slots suffice.
constexpr int kRecWords = kD + 2;

__host__ __device__ inline size_t fa_recv_word(size_t set, int rows, int slot, int src, int row) {
    return (set + 15) / 16 * 16 + ((((size_t) slot * kArMaxRanks + src) * rows + row) * kRecWords) * sizeof(uint64_t);
}

__device__ __forceinline__ uint64_t rec_word(float v, uint32_t e) {
    return (uint64_t) __float_as_uint(v) | ((uint64_t) e << 32);
}
__device__ __forceinline__ void st_relaxed_sys_b64(void * p, uint64_t v) {
    asm volatile("st.relaxed.sys.global.b64 [%0], %1;" ::"l"(p), "l"(v) : "memory");
}
__device__ __forceinline__ uint64_t ld_relaxed_sys_b64(const void * p) {
    uint64_t v;
    asm volatile("ld.relaxed.sys.global.b64 %0, [%1];" : "=l"(v) : "l"(p) : "memory");
    return v;
}
// the word's value once it carries epoch e (bounded: 2 s from t0, then the status word is set, ok cleared, 0)
__device__ __forceinline__ float wait_word(const uint8_t * p, uint32_t e, uint64_t t0, bool & ok, int32_t * status) {
    for (;;) {
        const uint64_t w = ld_relaxed_sys_b64(p);
        if ((uint32_t) (w >> 32) == e) return __uint_as_float((uint32_t) w);
        if (!ok || globaltimer_ns() - t0 > 2000000000ull) {
            if (ok) atomicExch(status, kErrPeerWait);
            ok = false;
            return 0.0f;
        }
        __nanosleep(32);
    }
}

__global__ void __launch_bounds__(256) fa_merge_peers_kernel(const uint64_t * peers, int world, int rank,
                                                             uint32_t * epochs, int N, int H, size_t ms_bytes,
                                                             size_t set, const float * sinks, float * dst,
                                                             int64_t dnb1, int64_t dnb2, int32_t * status) {
    pdl_launch_dependents();
    pdl_wait();  // this rank's partial records are complete
    const int row = blockIdx.x, h = row / N, tq = row % N, rows = H * N, dv = threadIdx.x;
    __shared__ uint32_t e_s;
    __shared__ int      ok_s;
    __shared__ float    w_s[kArMaxRanks], s_s[kArMaxRanks];
    __shared__ float    mf_s;
    if (dv == 0) e_s = ++epochs[row];
    __syncthreads();
    const uint32_t e = e_s;
    const int      slot = (int) (e & 1u);
    {  // send this rank's record row to every rank
        const float2 ms = reinterpret_cast<const float2 *>(peers[rank])[row];
        const float  v  = reinterpret_cast<const float *>(peers[rank] + ms_bytes)[(int64_t) row * kD + dv];
        for (int r = 0; r < world; r++) {
            uint8_t * q = reinterpret_cast<uint8_t *>(peers[r] + fa_recv_word(set, rows, slot, rank, row));
            st_relaxed_sys_b64(q + (size_t) dv * sizeof(uint64_t), rec_word(v, e));
            if (dv == 0) {
                st_relaxed_sys_b64(q + (size_t) kD * sizeof(uint64_t), rec_word(ms.x, e));
                st_relaxed_sys_b64(q + (size_t) (kD + 1) * sizeof(uint64_t), rec_word(ms.y, e));
            }
        }
    }
    const uint8_t * mine = reinterpret_cast<const uint8_t *>(peers[rank]);
    const uint64_t  t0   = globaltimer_ns();
    bool            ok   = true;
    if (dv == 0) {  // the ranks' (max, sum) pairs, their weights 2^(M_r - M)
        float m = -INFINITY;
        for (int r = 0; r < world; r++) {
            const uint8_t * q = mine + fa_recv_word(set, rows, slot, r, row);
            w_s[r]            = wait_word(q + (size_t) kD * sizeof(uint64_t), e, t0, ok, status);
            s_s[r]            = wait_word(q + (size_t) (kD + 1) * sizeof(uint64_t), e, t0, ok, status);
            if (s_s[r] != 0.0f) m = fmaxf(m, w_s[r]);
        }
        mf_s = m;
        for (int r = 0; r < world; r++) w_s[r] = s_s[r] != 0.0f ? exp2f(w_s[r] - m) : 0.0f;
        ok_s = ok;
    }
    __syncthreads();
    float acc = 0.0f, S = 0.0f;
    if (ok_s) {
        const float Mf = mf_s;
        for (int r = 0; r < world; r++) {
            const float w = w_s[r];
            const float v = wait_word(mine + fa_recv_word(set, rows, slot, r, row) + (size_t) dv * sizeof(uint64_t),
                                      e, t0, ok, status);
            acc = fmaf(w, w != 0.0f ? v : 0.0f, acc);
            S   = fmaf(w, s_s[r], S);
        }
        if (sinks) {
            const float sk2 = sinks[h] * kLog2e;
            if (sk2 > Mf) {
                const float m2 = exp2f(Mf - sk2);
                acc *= m2;
                S = S * m2 + 1.0f;
            } else {
                S += exp2f(sk2 - Mf);
            }
        }
    }
    const float inv = S == 0.0f ? 0.0f : 1.0f / S;
    float * out = reinterpret_cast<float *>(reinterpret_cast<uint8_t *>(dst) + h * dnb1 + tq * dnb2);
    out[dv]     = acc * inv;
}

size_t fa_peer_buffer_bytes(int64_t H, int64_t N) {
    const size_t set = fa_part_bytes(H, N);
    return (set + 15) / 16 * 16 + 2 * (size_t) kArMaxRanks * (size_t) (H * N) * kRecWords * sizeof(uint64_t);
}

int fa_merge_peers_run(srhpm_ctx * ctx, const uint64_t * peers, int world, int rank, uint32_t * epochs, int N, int H,
                       const float * sinks, float * dst, int64_t dnb1, int64_t dnb2, cudaStream_t stream) {
    if (world < 1 || world > kArMaxRanks || rank < 0 || rank >= world || N < 1 || H < 1) return SRHPM_ERR_INVALID;
    const cudaError_t e = launch_k_pdl(fa_merge_peers_kernel, dim3((unsigned) (H * N)), dim3(kD), 0, stream, peers,
                                       world, rank, epochs, N, H, fa_part_ms_bytes(H, N), fa_part_bytes(H, N), sinks,
                                       dst, dnb1, dnb2, ctx->d_status);
    ctx->launches.fetch_add(1);
    return cuda_status(e);
}

int fa_merge_run(srhpm_ctx * ctx, const void * parts, int n_parts, int N, int H, const float * sinks, float * dst,
                 int64_t dnb1, int64_t dnb2, cudaStream_t stream) {
    // one "KV head" holding every head: row = h * N + t, as in the record sets
    const size_t  set  = fa_part_bytes(H, N);
    FaArgs        a    = {};
    a.N         = N;
    a.H         = H;
    a.G         = H;
    a.R         = H * N;
    a.Hkv       = 1;
    a.n_chunks  = n_parts;
    a.part_ms   = reinterpret_cast<float2 *>(const_cast<void *>(parts));
    a.part_acc  = reinterpret_cast<float *>(reinterpret_cast<uint8_t *>(const_cast<void *>(parts)) + fa_part_ms_bytes(H, N));
    a.ms_row    = 1;
    a.ms_chunk  = (int64_t) (set / sizeof(float2));
    a.acc_row   = kD;
    a.acc_chunk = (int64_t) (set / sizeof(float));
    a.sinks     = sinks;
    a.dst       = dst;
    a.dnb1      = dnb1;
    a.dnb2      = dnb2;
    a.status    = ctx->d_status;
    return launch_combine(ctx, a, stream);
}

}  // namespace srhpm
