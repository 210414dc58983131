// The element-wise operators around the verify GEMMs of a dense decoder step (ggml semantics):
//   get_rows   token embeddings: rows of an f16 / f32 table -> f32 (ggml_get_rows)
//   add_rms_norm  residual stream x += delta (ggml_add), then y = x / sqrt(mean(x^2) + eps) * w
//                 (ggml_rms_norm followed by ggml_mul with the norm weight)
//   rope_kv    NeoX rotary embedding of the query and key heads of a fused QKV row (ggml_rope_ext, mode NEOX,
//              theta_i = pos * base^(-2i/d)); the rotated keys and the values are written into the KV cache at their
//              positions as f16 or q8_0 (ggml_cpy of f32 rows into the cache view; q8_0 with the context's q8_0 mode)
//   swiglu     silu(gate) * up (ggml_swiglu); gate and up may be the two halves of one fused gate|up GEMM output
// All rows are short (N <= 16 tokens): one CTA per (row, chunk) and grid-stride loops; these ops move a few hundred KB
// per step against the ~12 GB of weights. Each is launched with programmatic dependent launch: it lets its successor
// get resident at once and waits for its predecessor's writes before reading.
#include <cuda_fp16.h>
#include <cuda_runtime.h>

#include <cmath>

#include "allreduce.cuh"
#include "internal.h"
#include "launch.cuh"
#include "ptx.cuh"

namespace srhpm {
namespace {

__global__ void get_rows_kernel(const uint8_t * table, int64_t row_bytes, int is_f16, const int32_t * ids, int64_t d,
                                float * out) {
    pdl_launch_dependents();
    pdl_wait();
    const int64_t   i   = blockIdx.y;
    const uint8_t * src = table + (int64_t) ids[i] * row_bytes;
    for (int64_t j = blockIdx.x * blockDim.x + threadIdx.x; j < d; j += (int64_t) gridDim.x * blockDim.x) {
        out[i * d + j] = is_f16 ? __half2float(reinterpret_cast<const __half *>(src)[j])
                                : reinterpret_cast<const float *>(src)[j];
    }
}

// one CTA per row; the row (d <= 4 * 4 * blockDim) stays in registers between the sum and the scaling
constexpr int kNormThreads = 1024;
__global__ void __launch_bounds__(kNormThreads) add_rms_norm_kernel(float * x, const float * delta, const float * w,
                                                                     float eps, float * y, int64_t d) {
    pdl_launch_dependents();
    pdl_wait();
    const int64_t i  = blockIdx.x;
    float *       xr = x + i * d;
    const bool    vec = (d & 3) == 0 && (reinterpret_cast<uintptr_t>(xr) & 15) == 0 &&
                     (delta == nullptr || (reinterpret_cast<uintptr_t>(delta + i * d) & 15) == 0) &&
                     (reinterpret_cast<uintptr_t>(y + i * d) & 15) == 0 && (reinterpret_cast<uintptr_t>(w) & 15) == 0;
    float         ss = 0.0f;
    float4        v[4];
    const int64_t d4 = d >> 2;
    if (vec) {
#pragma unroll
        for (int k = 0; k < 4; k++) {
            const int64_t j = threadIdx.x + (int64_t) k * kNormThreads;
            if (j < d4) {
                float4 a = reinterpret_cast<const float4 *>(xr)[j];
                if (delta) {
                    const float4 b = reinterpret_cast<const float4 *>(delta + i * d)[j];
                    a.x += b.x; a.y += b.y; a.z += b.z; a.w += b.w;
                    reinterpret_cast<float4 *>(xr)[j] = a;
                }
                v[k] = a;
                ss = fmaf(a.x, a.x, fmaf(a.y, a.y, fmaf(a.z, a.z, fmaf(a.w, a.w, ss))));
            }
        }
    } else {
        for (int64_t j = threadIdx.x; j < d; j += kNormThreads) {
            float a = xr[j];
            if (delta) {
                a += delta[i * d + j];
                xr[j] = a;
            }
            ss = fmaf(a, a, ss);
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
    if (vec) {
#pragma unroll
        for (int k = 0; k < 4; k++) {
            const int64_t j = threadIdx.x + (int64_t) k * kNormThreads;
            if (j < d4) {
                const float4 ww = reinterpret_cast<const float4 *>(w)[j];
                float4       o;
                o.x = v[k].x * scale * ww.x;
                o.y = v[k].y * scale * ww.y;
                o.z = v[k].z * scale * ww.z;
                o.w = v[k].w * scale * ww.w;
                reinterpret_cast<float4 *>(y + i * d)[j] = o;
            }
        }
    } else {
        for (int64_t j = threadIdx.x; j < d; j += kNormThreads) y[i * d + j] = xr[j] * scale * w[j];
    }
}

// ---- residual add of a tensor-parallel partial sum + RMSNorm, the all-reduce done in the same kernel ------------
// CTA i (row i): the flag-in-word exchange of allreduce.cuh (each thread sends its values of the rank's partial row to
// every rank, then adds the ranks' values in rank order), x += the sum, and the norm.
__global__ void __launch_bounds__(kNormThreads) add_rms_norm_ar_kernel(float * x, const uint64_t * peers, int world,
                                                                        int rank, int slot, uint32_t * epochs,
                                                                        const float * w, float eps, float * y,
                                                                        int64_t d, int32_t * status) {
    pdl_launch_dependents();
    pdl_wait();  // this rank's GEMM has written its partial rows
    const int64_t i = blockIdx.x;
    __shared__ uint32_t e_s;
    const uint32_t      e  = ar_epoch(epochs, slot, (int) i, &e_s);
    const int64_t       d4 = d >> 2;
#pragma unroll
    for (int k = 0; k < 4; k++) {
        const int64_t j = threadIdx.x + (int64_t) k * kNormThreads;
        if (j < d4) ar_push4(peers, world, rank, slot, (int) i, d, j, e);
    }
    float *        xr = x + i * d;
    float          ss = 0.0f;
    float4         v[4];
    bool           ok = true;
    const uint64_t t0 = globaltimer_ns();
#pragma unroll
    for (int k = 0; k < 4; k++) {
        const int64_t j = threadIdx.x + (int64_t) k * kNormThreads;
        if (j < d4) {
            float4 a = reinterpret_cast<const float4 *>(xr)[j];
            ar_gather4(a, peers, world, rank, slot, (int) i, d, j, e, t0, ok, status);
            reinterpret_cast<float4 *>(xr)[j] = a;
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
        const int64_t j = threadIdx.x + (int64_t) k * kNormThreads;
        if (j < d4) {
            const float4 ww = reinterpret_cast<const float4 *>(w)[j];
            float4       o;
            o.x = v[k].x * scale * ww.x;
            o.y = v[k].y * scale * ww.y;
            o.z = v[k].z * scale * ww.z;
            o.w = v[k].w * scale * ww.w;
            reinterpret_cast<float4 *>(y + i * d)[j] = o;
        }
    }
}

struct RopeArgs {
    float *         qkv;         // [n][ld]: q heads (H x hd) | k heads (Hkv x hd) | v heads (Hkv x hd)
    int64_t         ld;
    int             n, H, Hkv, hd;
    const int32_t * pos;         // [n]
    float           theta_scale; // base^(-2/hd)
    uint8_t *       kc;          // cache rows: token p, head g at kc + p * knb1 + g * knb2
    uint8_t *       vc;
    int64_t         knb1, knb2, vnb1, vnb2;
    int             cache_type;  // SRHPM_TYPE_F16 or SRHPM_TYPE_Q8_0
    int             q8mode;
};

// rotate the pair (j, j + hd/2) of one head row in place
__device__ __forceinline__ void rope_pair(float * h, int j, int half, float p, float theta_scale) {
    const float theta = p * powf(theta_scale, (float) j);
    float       s, c;
    sincosf(theta, &s, &c);
    const float x0 = h[j], x1 = h[j + half];
    h[j]        = x0 * c - x1 * s;
    h[j + half] = x0 * s + x1 * c;
}

// q8_0 of 32 values (one warp lane per value; lanes of a block = a full warp), bytes to dst (34 bytes)
__device__ __forceinline__ void q80_store_warp(float v, uint8_t * dst, int mode) {
    const int lane = threadIdx.x & 31;
    float     amax = fabsf(v);
#pragma unroll
    for (int o = 16; o > 0; o >>= 1) amax = fmaxf(amax, __shfl_xor_sync(0xffffffffu, amax, o));
    const float  dd = __fdiv_rn(amax, 127.0f);
    const __half dh = __float2half_rn(dd);
    int          qv;
    if (mode == SRHPM_Q8_0_ACT_SIMD) {
        const float id = amax != 0.0f ? __fdiv_rn(127.0f, amax) : 0.0f;
        qv             = __float2int_rn(__fmul_rn(v, id));
    } else {
        const float id = dd != 0.0f ? __fdiv_rn(1.0f, dd) : 0.0f;
        qv             = (int) roundf(__fmul_rn(v, id));
    }
    if (lane == 0) *reinterpret_cast<__half *>(dst) = dh;
    dst[2 + lane] = (uint8_t) (int8_t) qv;
}

// grid: (token, head of q + k + v); one CTA of hd/2 threads (f16 cache) or hd threads (q8_0: a warp per block)
__global__ void rope_kv_kernel(const RopeArgs a) {
    pdl_launch_dependents();
    pdl_wait();
    const int t = blockIdx.x, hh = blockIdx.y, half = a.hd / 2;
    float *   row = a.qkv + (int64_t) t * a.ld;
    const float p = (float) a.pos[t];
    if (hh < a.H) {  // query head: rotate in place
        float * h = row + (int64_t) hh * a.hd;
        for (int j = threadIdx.x; j < half; j += blockDim.x) rope_pair(h, j, half, p, a.theta_scale);
        return;
    }
    const bool isk = hh < a.H + a.Hkv;
    const int  g   = isk ? hh - a.H : hh - a.H - a.Hkv;
    float *    h   = row + (int64_t) (a.H + (isk ? 0 : a.Hkv) + g) * a.hd;
    if (isk) {
        for (int j = threadIdx.x; j < half; j += blockDim.x) rope_pair(h, j, half, p, a.theta_scale);
        __syncthreads();
    }
    uint8_t * dst = (isk ? a.kc + (int64_t) a.pos[t] * a.knb1 + (int64_t) g * a.knb2
                         : a.vc + (int64_t) a.pos[t] * a.vnb1 + (int64_t) g * a.vnb2);
    if (a.cache_type == SRHPM_TYPE_F16) {
        for (int j = threadIdx.x; j < a.hd; j += blockDim.x) reinterpret_cast<__half *>(dst)[j] = __float2half_rn(h[j]);
    } else {
        for (int j = threadIdx.x; j < a.hd; j += blockDim.x) {  // blockDim = hd: one warp per 32-value block
            q80_store_warp(h[j], dst + (j >> 5) * 34, a.q8mode);
        }
    }
}

__global__ void swiglu_kernel(const float * gate, const float * up, int64_t ld_in, float * out, int64_t ld_out,
                              int64_t cols) {
    pdl_launch_dependents();
    pdl_wait();
    const int64_t r = blockIdx.y;
    for (int64_t j = blockIdx.x * (int64_t) blockDim.x + threadIdx.x; j < cols; j += (int64_t) gridDim.x * blockDim.x) {
        const float g   = gate[r * ld_in + j];
        out[r * ld_out + j] = g / (1.0f + expf(-g)) * up[r * ld_in + j];
    }
}

}  // namespace

int get_rows_run(srhpm_ctx * ctx, const uint8_t * table, int64_t row_bytes, int is_f16, const int32_t * ids, int n,
                 int64_t d, float * out, cudaStream_t stream) {
    const cudaError_t e = launch_k_pdl(get_rows_kernel, dim3((unsigned) std::min<int64_t>(8, (d + 255) / 256), n),
                                       dim3(256), 0, stream, table, row_bytes, is_f16, ids, d, out);
    ctx->launches.fetch_add(1);
    return cuda_status(e);
}

int add_rms_norm_run(srhpm_ctx * ctx, float * x, const float * delta, const float * w, float eps, float * y, int n,
                     int64_t d, cudaStream_t stream) {
    if (d > 4 * 4 * kNormThreads) return SRHPM_UNSUPPORTED;
    const cudaError_t e = launch_k_pdl(add_rms_norm_kernel, dim3(n), dim3(kNormThreads), 0, stream, x, delta, w, eps,
                                       y, d);
    ctx->launches.fetch_add(1);
    return cuda_status(e);
}

int add_rms_norm_ar_run(srhpm_ctx * ctx, float * x, const uint64_t * peers, int world, int rank, int slot,
                        uint32_t * epochs, const float * w, float eps, float * y, int n, int64_t d,
                        cudaStream_t stream) {
    if (d > 4 * 4 * kNormThreads || (d & 3) != 0) return SRHPM_UNSUPPORTED;
    if (n < 1 || n > kArRows || world < 1 || world > kArMaxRanks || rank < 0 || rank >= world || slot < 0 ||
        slot > 1) {
        return SRHPM_ERR_INVALID;
    }
    const cudaError_t e = launch_k_pdl(add_rms_norm_ar_kernel, dim3(n), dim3(kNormThreads), 0, stream, x, peers,
                                       world, rank, slot, epochs, w, eps, y, d, ctx->d_status);
    ctx->launches.fetch_add(1);
    return cuda_status(e);
}

size_t allreduce_buffer_bytes(int64_t d) {
    // the two slots of partial rows, then the receive area of 8-byte (value, epoch) words
    return 2 * ar_part_bytes(d) + 2 * (size_t) kArRows * kArMaxRanks * d * sizeof(uint64_t);
}

int rope_kv_run(srhpm_ctx * ctx, float * qkv, int64_t ld, int n, int H, int Hkv, int hd, const int32_t * pos,
                float theta_base, uint8_t * kc, int64_t knb1, int64_t knb2, uint8_t * vc, int64_t vnb1, int64_t vnb2,
                int cache_type, cudaStream_t stream) {
    RopeArgs a;
    a.qkv         = qkv;
    a.ld          = ld;
    a.n           = n;
    a.H           = H;
    a.Hkv         = Hkv;
    a.hd          = hd;
    a.pos         = pos;
    a.theta_scale = powf(theta_base, -2.0f / (float) hd);
    a.kc          = kc;
    a.vc          = vc;
    a.knb1        = knb1;
    a.knb2        = knb2;
    a.vnb1        = vnb1;
    a.vnb2        = vnb2;
    a.cache_type  = cache_type;
    a.q8mode      = ctx->q8_0_act_mode;
    const cudaError_t e = launch_k_pdl(rope_kv_kernel, dim3(n, H + 2 * Hkv),
                                       dim3(cache_type == SRHPM_TYPE_F16 ? hd / 2 : hd), 0, stream, a);
    ctx->launches.fetch_add(1);
    return cuda_status(e);
}

int swiglu_run(srhpm_ctx * ctx, const float * gate, const float * up, int64_t ld_in, float * out, int64_t ld_out,
               int rows, int64_t cols, cudaStream_t stream) {
    const int blocks = (int) std::min<int64_t>(std::max(1, 4 * ctx->num_sms / rows), (cols + 255) / 256);
    const cudaError_t e = launch_k_pdl(swiglu_kernel, dim3(blocks, rows), dim3(256), 0, stream, gate, up, ld_in, out,
                                       ld_out, cols);
    ctx->launches.fetch_add(1);
    return cuda_status(e);
}

}  // namespace srhpm
