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

#include "internal.h"
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
constexpr int   kNSlot   = 3;
constexpr int   kVC      = (kD / 8) * kT * 16;  // V^T operand: [dv group of 8][token][8 f16]
constexpr int   kRG      = 48;                  // rows per row group (tensor memory: 8 * 48 + 2 * 48 columns)
constexpr int   kCW      = 4;                   // compute warps
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
    int             mne2;
    float           qscale;      // folded into the Q block scales: scale*log2e, or scale/softcap with a softcap
    float           softcap_l2;  // softcap*log2e, 0 = none
    float           max_bias, m0, m1;
    int             n_head_log2;
    const float *   sinks;       // f32 [H] or null
    float *         dst;
    int64_t         dnb1, dnb2;  // bytes: head, token
    float *         part_acc;    // [Hkv * R][n_chunks][256]
    float2 *        part_ms;     // [Hkv * R][n_chunks] (max in log2 units, sum)
    int32_t *       status;
    int             q8mode;
};

// shared-memory layout (bytes from a 1024-aligned base)
template <int RP> struct Smem {
    static constexpr int ring = 0;
    static constexpr int vc   = ring + kNSlot * kSlot;
    static constexpr int p    = vc + kVC;
    static constexpr int qop  = p + RP * kT * 2;      // 16 Q operands of [2][RP][16]
    static constexpr int qopb = 2 * RP * 16;          // bytes per Q operand
    static constexpr int dq   = qop + 16 * qopb;      // f32 [8][RP]
    static constexpr int red  = dq + 8 * RP * 4;      // f32 [4][RP]
    static constexpr int mu   = red + kCW * RP * 4;   // f32 [RP] running maximum (log2 units)
    static constexpr int al   = mu + RP * 4;          // f32 [RP] rescale factor of this tile
    static constexpr int fac  = al + RP * 4;          // f32 [RP] final factor
    static constexpr int slope = fac + RP * 4;        // f32 [RP] ALiBi slope * log2e
    static constexpr int moff = slope + RP * 4;       // int64 [RP] mask row offsets
    static constexpr int bar  = (moff + RP * 8 + 7) / 8 * 8;
    static constexpr int nbar = 2 * kNSlot + 4;       // full[3], empty[3], s_full, s_free, pv_ready, pv_done
    static constexpr int misc = bar + nbar * 8;       // tmem base, flags[2]
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
    asm volatile("redux.sync.max.f32 %0, %1, 0xffffffff;" : "=f"(r) : "f"(v));
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

// 1 thread = 1 KV token of the tile; V row (272 bytes, [d | 32 q] x 8) -> 256 f16 = d * q into the V^T operand
__device__ __forceinline__ void convert_v_row(const uint8_t * row, uint8_t * vc, int t) {
    uint32_t w[68];
#pragma unroll
    for (int c = 0; c < 17; c++) {
        const uint4 u = *reinterpret_cast<const uint4 *>(row + 16 * c);
        w[4 * c] = u.x; w[4 * c + 1] = u.y; w[4 * c + 2] = u.z; w[4 * c + 3] = u.w;
    }
    const __half2 bias = __halves2half2(__ushort_as_half(0x6480u), __ushort_as_half(0x6480u));  // 1152
#pragma unroll
    for (int b = 0; b < 8; b++) {
        const int      od = 34 * b;
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
#pragma unroll
        for (int qd = 0; qd < 4; qd++) {
            *reinterpret_cast<uint4 *>(vc + ((4 * b + qd) * kT + t) * 16) =
                make_uint4(f[4 * qd], f[4 * qd + 1], f[4 * qd + 2], f[4 * qd + 3]);
        }
    }
}

template <int RP>
__global__ void __launch_bounds__(kFaThreads, 1)
    fa_q80_kernel(const __grid_constant__ CUtensorMap mk128, const __grid_constant__ CUtensorMap mk32,
                  const __grid_constant__ CUtensorMap mv, const FaArgs a) {
    using S = Smem<RP>;
    extern __shared__ uint8_t smem_raw[];
    uint8_t * sm = reinterpret_cast<uint8_t *>((reinterpret_cast<uintptr_t>(smem_raw) + 1023) & ~uintptr_t(1023));
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

    const int tid = threadIdx.x, warp = tid >> 5, lane = tid & 31;
    const int chunk = blockIdx.x;
    const int g = blockIdx.y / a.nrg, rg = blockIdx.y % a.nrg;
    const int t0 = chunk * a.chunk_len, t1 = min(a.L, t0 + a.chunk_len);
    const int nt = (t1 - t0 + kT - 1) / kT;
    const int row0 = rg * kRG;                       // first row (of the KV head's R) of this group
    const int rows = min(RP, a.R - row0);            // valid rows
    bool      bad  = false;

    if (tid == 0) {
        for (int i = 0; i < kNSlot; i++) {
            mbar_init(&full[i], 1);
            mbar_init(&empty[i], kCW);
        }
        mbar_init(s_full, 1);
        mbar_init(s_free, kCW);
        mbar_init(pv_rdy, kCW);
        mbar_init(pv_done, 1);
        fence_mbar_init();
        flags[0] = flags[1] = 0;
    }
    if (warp == 0) tc::tmem_alloc(tptr, 512);
    if (tid < kCW * 32) {
        uint4 * z = reinterpret_cast<uint4 *>(sm + S::qop);
        for (int i = tid; i < 16 * S::qopb / 16; i += kCW * 32) z[i] = make_uint4(0, 0, 0, 0);
    }
    tc::fence_before();
    __syncthreads();
    tc::fence_after();
    const uint32_t tbase = *tptr;

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
        for (int n = 0; n < min(kNSlot, nload); n++) produce(n);
    }
    __syncwarp();

    // Q rows -> q8_0 (the cache type's vec_dot type), scattered into the 16 window operands; per-row constants
    if (tid < kCW * 32) {
        for (int u = tid; u < 8 * RP; u += kCW * 32) {
            const int r = u >> 3, b = u & 7;
            int8_t    qv[32];
            float     dqs = 0.0f;
            if (r < rows) {
                const int     rr = row0 + r;
                const int     h  = g * a.G + rr / a.N, tq = rr % a.N;
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
            dq[b * RP + r]   = dqs;
            const int w0     = (34 * b + 2) >> 5;
#pragma unroll
            for (int j = 0; j < 32; j++) {
                const int pos = 34 * b + 2 + j, x = pos & 31, s = (pos >> 5) - w0;
                sm[S::qop + (2 * b + s) * S::qopb + (x >> 4) * RP * 16 + r * 16 + (x & 15)] = (uint8_t) qv[j];
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
            mu[r]     = -INFINITY;
        }
    }
    asm volatile("fence.proxy.async.shared::cta;" ::: "memory");
    tc::fence_before();
    __syncthreads();
    tc::fence_after();

    const uint32_t qop_s = smem_u32(sm + S::qop);
    const uint32_t vc_s  = smem_u32(sm + S::vc);
    const uint32_t p_s   = smem_u32(sm + S::p);
    const uint32_t tS    = tbase;             // S_b at columns RP * b
    const uint32_t tO    = tbase + 8 * RP;    // O^T halves at tO, tO + RP

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
            constexpr uint32_t id16 = tc::idesc(tc::kD_F32, tc::kAB_F16, tc::kAB_F16, tc::kMNMajor, tc::kMNMajor, RP,
                                                128);
            auto issue_qk = [&](int i) {
                const int n = 2 * i, slot = n % kNSlot;
                wait_or_flag(&full[slot], (n / kNSlot) & 1, a.status, bad);
                tc::fence_after();
                const uint32_t kb = smem_u32(sm + S::ring + slot * kSlot);
#pragma unroll
                for (int b = 0; b < 8; b++) {
                    const int w0 = (34 * b + 2) >> 5;
#pragma unroll
                    for (int s = 0; s < 2; s++) {
                        const int j = w0 + s;
                        uint64_t  ad;
                        if (j < 8) {
                            ad = tc::sdesc(kb + (j >> 2) * kPlane + (j & 3) * 32, 16, 1024) | (2ull << 61);
                        } else {
                            ad = tc::sdesc(kb + 2 * kPlane, 16, 256) | (6ull << 61);
                        }
                        const uint64_t bd = tc::sdesc(qop_s + (2 * b + s) * S::qopb, RP * 16, 128);
                        tc::mma_i8(tS + RP * b, ad, bd, id8, (uint32_t) s);
                    }
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
#pragma unroll
                for (int hf = 0; hf < 2; hf++) {
#pragma unroll
                    for (int k = 0; k < kT / 16; k++) {
                        const uint64_t ad = tc::sdesc(vc_s + hf * 16 * kT * 16 + k * 256, 128, kT * 16);
                        const uint64_t bd = tc::sdesc(p_s + k * 256, 128, kT * 16);
                        tc::mma_f16(tO + hf * RP, ad, bd, id16, (uint32_t) (i > 0 || k > 0));
                    }
                }
                tc::commit(pv_done);
            }
        }
        __syncwarp();
    } else {
        // ---------------- compute warps: thread = KV token of the tile ----------------
        float l[RP];
#pragma unroll
        for (int r = 0; r < RP; r++) l[r] = 0.0f;
        for (int i = 0; i < nt; i++) {
            const int n = 2 * i, kslot = n % kNSlot, vslot = (n + 1) % kNSlot;
            wait_or_flag(s_full, i & 1, a.status, bad);
            wait_or_flag(&full[kslot], (n / kNSlot) & 1, a.status, bad);  // (complete already) the d bytes
            tc::fence_after();
            const uint8_t * kb = sm + S::ring + kslot * kSlot;
            float           dk[8];
#pragma unroll
            for (int b = 0; b < 8; b++) {
                const int o = 34 * b, oo = o & 127;
                const uint8_t * pr = kb + (o >> 7) * kPlane + tid * 128 + ((((oo >> 4) ^ (tid & 7))) << 4) + (oo & 15);
                dk[b] = half_bits_to_float(*reinterpret_cast<const uint16_t *>(pr));
            }
            float s[RP];
#pragma unroll
            for (int r = 0; r < RP; r++) s[r] = 0.0f;
#pragma unroll
            for (int b = 0; b < 8; b++) {
                uint32_t v[RP];
#pragma unroll
                for (int c = 0; c < RP / 16; c++) {
                    tc::ld16(tc::taddr(tS, warp, RP * b + 16 * c), *reinterpret_cast<uint32_t(*)[16]>(&v[16 * c]));
                }
                tc::wait_ld();
                const float * dqb = dq + b * RP;
#pragma unroll
                for (int r = 0; r < RP; r++) s[r] = fmaf((float) (int) v[r], dqb[r] * dk[b], s[r]);
            }
            tc::fence_before();
            __syncwarp();
            if (lane == 0) {
                mbar_arrive(s_free);
                mbar_arrive(&empty[kslot]);
            }

            const int  tok   = t0 + i * kT + tid;
            const bool valid = tok < t1;
            if (a.softcap_l2 != 0.0f) {
#pragma unroll
                for (int r = 0; r < RP; r++) s[r] = a.softcap_l2 * tanhf(s[r]);
            }
            if (a.mask != nullptr && valid) {
#pragma unroll
                for (int r = 0; r < RP; r++) {
                    const uint16_t mb = __ldg(reinterpret_cast<const unsigned short *>(a.mask + moff[r] + 2 * (int64_t) tok));
                    s[r] = fmaf(slope2[r], half_bits_to_float(mb), s[r]);
                }
            }
            if (!valid) {
#pragma unroll
                for (int r = 0; r < RP; r++) s[r] = -INFINITY;
            }
#pragma unroll
            for (int r = 0; r < RP; r++) {
                const float m = redux_max(s[r]);
                if (lane == 0) red[warp * RP + r] = m;
            }
            named_bar_sync(1, kCW * 32);
            if (tid < RP) {
                float mt = red[tid];
#pragma unroll
                for (int w = 1; w < kCW; w++) mt = fmaxf(mt, red[w * RP + tid]);
                const float mo = mu[tid];
                if (mt > mo + kLazy) {
                    mu[tid]         = mt;
                    al[tid]         = exp2f(mo - mt);
                    flags[i & 1]    = 1;
                } else {
                    al[tid] = 1.0f;
                }
            }
            named_bar_sync(1, kCW * 32);
            const bool resc = flags[i & 1] != 0;
            if (tid == 0) flags[(i + 1) & 1] = 0;
            if (i > 0) {
                wait_or_flag(pv_done, (i - 1) & 1, a.status, bad);
                tc::fence_after();
            }
            if (resc) {
#pragma unroll
                for (int r = 0; r < RP; r++) l[r] *= al[r];
                if (i > 0) {
#pragma unroll
                    for (int hf = 0; hf < 2; hf++) {
#pragma unroll
                        for (int c = 0; c < RP / 16; c++) {
                            uint32_t o[16];
                            const uint32_t ta = tc::taddr(tO + hf * RP, warp, 16 * c);
                            tc::ld16(ta, o);
                            tc::wait_ld();
#pragma unroll
                            for (int j = 0; j < 16; j++) o[j] = __float_as_uint(__uint_as_float(o[j]) * al[16 * c + j]);
                            tc::st16(ta, o);
                        }
                    }
                    tc::wait_st();
                }
            }
            // P^T (MN-major: [row group of 8][token][8 f16])
#pragma unroll
            for (int rg8 = 0; rg8 < RP / 8; rg8++) {
                uint32_t pk[4];
#pragma unroll
                for (int j = 0; j < 4; j++) {
                    const int   r0 = 8 * rg8 + 2 * j;
                    const float p0 = s[r0] == -INFINITY ? 0.0f : exp2f(s[r0] - mu[r0]);
                    const float p1 = s[r0 + 1] == -INFINITY ? 0.0f : exp2f(s[r0 + 1] - mu[r0 + 1]);
                    l[r0] += p0;
                    l[r0 + 1] += p1;
                    const __half2 hp = __floats2half2_rn(p0, p1);
                    pk[j]            = *reinterpret_cast<const uint32_t *>(&hp);
                }
                *reinterpret_cast<uint4 *>(sm + S::p + (rg8 * kT + tid) * 16) = make_uint4(pk[0], pk[1], pk[2], pk[3]);
            }
            // V^T
            wait_or_flag(&full[vslot], ((n + 1) / kNSlot) & 1, a.status, bad);
            convert_v_row(sm + S::ring + vslot * kSlot + tid * kRowB, sm + S::vc, tid);
            __syncwarp();
            if (lane == 0) mbar_arrive(&empty[vslot]);
            asm volatile("fence.proxy.async.shared::cta;" ::: "memory");
            tc::fence_before();
            __syncwarp();
            if (lane == 0) mbar_arrive(pv_rdy);
        }

        // ---------------- epilogue ----------------
        wait_or_flag(pv_done, (nt - 1) & 1, a.status, bad);
        tc::fence_after();
#pragma unroll
        for (int r = 0; r < RP; r++) {
            float v = l[r];
#pragma unroll
            for (int o = 16; o > 0; o >>= 1) v += __shfl_xor_sync(0xffffffffu, v, o);
            if (lane == 0) red[warp * RP + r] = v;
        }
        named_bar_sync(1, kCW * 32);
        const bool single = a.n_chunks == 1;
        if (tid < rows) {
            float Ssum = red[tid];
#pragma unroll
            for (int w = 1; w < kCW; w++) Ssum += red[w * RP + tid];
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
            const int dv = hf * 128 + warp * 32 + lane;
#pragma unroll
            for (int c = 0; c < RP / 16; c++) {
                uint32_t o[16];
                tc::ld16(tc::taddr(tO + hf * RP, warp, 16 * c), o);
                tc::wait_ld();
#pragma unroll
                for (int j = 0; j < 16; j++) {
                    const int r = 16 * c + j;
                    if (r < rows) {
                        const int rr = row0 + r;
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
    }

    tc::fence_before();
    __syncthreads();
    if (warp == 0) tc::tmem_free(tbase, 512);
}

// merge of the chunk records of one row (P:787-823), then sinks and normalization; one CTA per (KV head, row)
__global__ void __launch_bounds__(256) fa_combine_kernel(const FaArgs a) {
    pdl_wait();
    const int row = blockIdx.x, g = row / a.R, rr = row % a.R;
    const int h = g * a.G + rr / a.N, tq = rr % a.N;
    const float2 * ms = a.part_ms + (int64_t) row * a.n_chunks;
    float Mf = -INFINITY;
    for (int c = 0; c < a.n_chunks; c++) {
        const float2 m = ms[c];
        if (m.y != 0.0f) Mf = fmaxf(Mf, m.x);
    }
    const int dv = threadIdx.x;
    float     acc = 0.0f, S = 0.0f;
    for (int c = 0; c < a.n_chunks; c++) {
        const float2 m = ms[c];
        if (m.y == 0.0f) continue;
        const float w = exp2f(m.x - Mf);
        acc = fmaf(w, a.part_acc[((int64_t) row * a.n_chunks + c) * kD + dv], acc);
        S   = fmaf(w, m.y, S);
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
    Plan p;
    p.nrg              = (R + kRG - 1) / kRG;
    p.rp               = p.nrg > 1 ? kRG : (R + 15) / 16 * 16;
    const int groups   = Hkv * p.nrg;
    const int max_ch   = (L + kT - 1) / kT;
    const int want     = std::max(1, std::min(max_ch, (num_sms + groups - 1) / groups));
    const int per      = (L + want - 1) / want;
    p.chunk_len        = (per + kT - 1) / kT * kT;
    p.n_chunks         = (L + p.chunk_len - 1) / p.chunk_len;
    return p;
}

template <int RP>
int launch_fa(srhpm_ctx * ctx, const FaArgs & a, const CUtensorMap & mk128, const CUtensorMap & mk32,
              const CUtensorMap & mv, cudaStream_t stream) {
    auto                         kern = fa_q80_kernel<RP>;
    static std::atomic<unsigned> attr_done{ 0 };
    if (!(attr_done.load() & (1u << ctx->device))) {
        const int st = cuda_status(cudaFuncSetAttribute(kern, cudaFuncAttributeMaxDynamicSharedMemorySize,
                                                        Smem<RP>::alloc));
        if (st != SRHPM_OK) return st;
        attr_done.fetch_or(1u << ctx->device);
    }
    kern<<<dim3(a.n_chunks, a.Hkv * a.nrg), kFaThreads, Smem<RP>::alloc, stream>>>(mk128, mk32, mv, a);
    ctx->launches.fetch_add(1);
    int st = cuda_status(cudaGetLastError());
    if (st != SRHPM_OK || a.n_chunks == 1) return st;

    cudaLaunchConfig_t   cfg = {};
    cudaLaunchAttribute  attr[1];
    cfg.gridDim          = dim3(a.Hkv * a.R);
    cfg.blockDim         = dim3(kD);
    cfg.dynamicSmemBytes = 0;
    cfg.stream           = stream;
    attr[0].id                                         = cudaLaunchAttributeProgrammaticStreamSerialization;
    attr[0].val.programmaticStreamSerializationAllowed = 1;
    cfg.attrs                                          = attr;
    cfg.numAttrs                                       = 1;
    st = cuda_status(cudaLaunchKernelEx(&cfg, fa_combine_kernel, a));
    ctx->launches.fetch_add(1);
    return st;
}

}  // namespace

size_t fa_work_size(int num_sms, int R, int L, int Hkv) {
    const Plan p = fa_plan(num_sms, R, L, Hkv);
    if (p.n_chunks == 1) return 0;
    const size_t rows = (size_t) Hkv * R * p.n_chunks;
    return rows * kD * sizeof(float) + rows * sizeof(float2) + 256;
}

int fa_run(srhpm_ctx * ctx, const FaView & v, float scale, float max_bias, float softcap, void * wdata, size_t wsize,
           cudaStream_t stream) {
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
    a.status = ctx->d_status;
    a.q8mode = ctx->q8_0_act_mode;

    EncodeTiled enc = fa_encode_fn();
    if (!enc) return SRHPM_ERR_CUDA;
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

}  // namespace srhpm
