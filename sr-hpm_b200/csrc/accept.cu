// Greedy verification of a draft: per-row argmax of the target logits over the vocabulary and the longest accepted
// prefix, as common_sampler_sample_and_accept_n does with a greedy sampler (upstream; the reference's relaxed
// acceptance at patch/srhpm.patch:9-35): for i < n_draft, id_i = argmax(logits row i); with relax > 0 a drafted token
// whose logit is within relax of the best replaces it; id_i is emitted and the scan stops at the first id_i != draft_i;
// when every drafted token is accepted the argmax of row n_draft is emitted as well.
//
// argmax semantics are those of the sequential greedy scan (best = element 0; element i replaces best when strictly
// greater): the first index of the maximum over the non-NaN values, or 0 when the row starts with NaN.
//
// Kernels: argmax_part_kernel (grid = segments x rows, 16-byte loads where the row allows, one (max, index) per
// segment), then a one-CTA kernel launched with programmatic stream serialization: either the acceptance
// (accept_final_kernel) or, for a vocabulary shard, the per-row record {max, index, logit of the drafted token}
// (shard_final_kernel); accept_merge_kernel merges the records of all shards and runs the acceptance.
#include <cuda_runtime.h>

#include <cmath>

#include "internal.h"
#include "ptx.cuh"

namespace srhpm {
namespace {

constexpr int kArgThreads = 256;
constexpr int kMaxRows    = 17;  // n_draft <= 16

struct ArgPair {
    float v;
    int   i;  // INT32_MAX: empty
};

// combine: larger value wins, equal values go to the lower index; NaN never enters
__device__ __forceinline__ ArgPair arg_better(ArgPair a, ArgPair b) {
    if (b.v > a.v || (b.v == a.v && b.i < a.i)) return b;
    return a;
}

__device__ __forceinline__ ArgPair warp_argmax(ArgPair p) {
#pragma unroll
    for (int o = 16; o > 0; o >>= 1) {
        ArgPair q;
        q.v = __shfl_xor_sync(0xffffffffu, p.v, o);
        q.i = __shfl_xor_sync(0xffffffffu, p.i, o);
        p   = arg_better(p, q);
    }
    return p;
}

__device__ __forceinline__ void consider(ArgPair & p, float x, int i) {
    if (!isnan(x) && (x > p.v || (x == p.v && i < p.i))) {
        p.v = x;
        p.i = i;
    }
}

struct ArgArgs {
    const uint8_t * logits;
    int64_t         ldb;  // row stride in bytes
    int             n_vocab, n_rows, nseg, seg_len;
    ArgPair *       part;  // [n_rows][nseg]
};

__global__ void __launch_bounds__(kArgThreads) argmax_part_kernel(const ArgArgs a) {
    pdl_launch_dependents();
    const int     seg = blockIdx.x, row = blockIdx.y;
    const float * x   = reinterpret_cast<const float *>(a.logits + (int64_t) row * a.ldb);
    const int     i0  = seg * a.seg_len, i1 = min(a.n_vocab, i0 + a.seg_len);
    ArgPair       p{ -INFINITY, INT32_MAX };
    if ((reinterpret_cast<uintptr_t>(x) & 15) == 0 && (i0 & 3) == 0) {
        const int n4 = (i1 - i0) >> 2;
        for (int k = threadIdx.x; k < n4; k += kArgThreads) {
            const float4 v = __ldcs(reinterpret_cast<const float4 *>(x + i0) + k);
            const int    i = i0 + 4 * k;
            consider(p, v.x, i);
            consider(p, v.y, i + 1);
            consider(p, v.z, i + 2);
            consider(p, v.w, i + 3);
        }
        for (int i = i0 + 4 * n4 + threadIdx.x; i < i1; i += kArgThreads) consider(p, x[i], i);
    } else {
        for (int i = i0 + threadIdx.x; i < i1; i += kArgThreads) consider(p, x[i], i);
    }
    p = warp_argmax(p);
    __shared__ ArgPair sp[kArgThreads / 32];
    if ((threadIdx.x & 31) == 0) sp[threadIdx.x >> 5] = p;
    __syncthreads();
    if (threadIdx.x < 32) {
        p = threadIdx.x < kArgThreads / 32 ? sp[threadIdx.x] : ArgPair{ -INFINITY, INT32_MAX };
        p = warp_argmax(p);
        if (threadIdx.x == 0) a.part[row * a.nseg + seg] = p;
    }
}

// argmax of row r from its segment records (one warp); index 0 when the row starts with NaN or is all NaN
__device__ __forceinline__ int row_argmax(const ArgArgs & a, int r, float * vmax) {
    ArgPair p{ -INFINITY, INT32_MAX };
    for (int s = threadIdx.x & 31; s < a.nseg; s += 32) p = arg_better(p, a.part[r * a.nseg + s]);
    p                = warp_argmax(p);
    const float * x0 = reinterpret_cast<const float *>(a.logits + (int64_t) r * a.ldb);
    if (isnan(x0[0]) || p.i == INT32_MAX) {
        *vmax = x0[0];
        return 0;
    }
    *vmax = p.v;
    return p.i;
}

// the sequential acceptance over per-row argmax ids and logits (thread 0)
__device__ void accept_scan(const int * am, const float * amv, const float * dlog, const int * has_dlog,
                            const int32_t * draft, int n_draft, float relax, int32_t * out_ids, int32_t * out_n) {
    int n = 0, i = 0;
    for (; i < n_draft; i++) {
        int id = am[i];
        if (relax > 0.0f && draft[i] != id && has_dlog[i] && amv[i] - dlog[i] <= relax) id = draft[i];
        out_ids[n++] = id;
        if (draft[i] != id) break;
    }
    if (i == n_draft) out_ids[n++] = am[n_draft];
    *out_n = n;
}

__global__ void __launch_bounds__(32 * kMaxRows) accept_final_kernel(const ArgArgs a, const int32_t * draft,
                                                                       int n_draft, float relax, int32_t * out_ids,
                                                                       int32_t * out_n) {
    pdl_wait();
    __shared__ int   am[kMaxRows], has[kMaxRows];
    __shared__ float amv[kMaxRows], dl[kMaxRows];
    const int        r = threadIdx.x >> 5;
    if (r < a.n_rows) {
        float     v;
        const int id = row_argmax(a, r, &v);
        if ((threadIdx.x & 31) == 0) {
            am[r]  = id;
            amv[r] = v;
            has[r] = 0;
            dl[r]  = 0.0f;
            if (r < n_draft) {
                const int d = draft[r];
                if (d >= 0 && d < a.n_vocab) {
                    dl[r]  = reinterpret_cast<const float *>(a.logits + (int64_t) r * a.ldb)[d];
                    has[r] = 1;
                }
            }
        }
    }
    __syncthreads();
    if (threadIdx.x == 0) accept_scan(am, amv, dl, has, draft, n_draft, relax, out_ids, out_n);
}

// record of a vocabulary shard: {max, global index of the first maximum (-1: the shard starts the vocabulary with
// NaN), logit of the drafted token when the shard holds it, 1 if it does}
__global__ void __launch_bounds__(32 * kMaxRows) shard_final_kernel(const ArgArgs a, int64_t vocab_offset,
                                                                      const int32_t * draft, int n_draft,
                                                                      srhpm_argmax_record * out) {
    pdl_wait();
    const int r = threadIdx.x >> 5;
    if (r >= a.n_rows) return;
    ArgPair p{ -INFINITY, INT32_MAX };
    for (int s = threadIdx.x & 31; s < a.nseg; s += 32) p = arg_better(p, a.part[r * a.nseg + s]);
    p = warp_argmax(p);
    if ((threadIdx.x & 31) == 0) {
        const float *       x = reinterpret_cast<const float *>(a.logits + (int64_t) r * a.ldb);
        srhpm_argmax_record rec;
        rec.vmax      = p.v;
        rec.imax      = p.i == INT32_MAX ? -2 : (int32_t) (vocab_offset + p.i);
        if (vocab_offset == 0 && isnan(x[0])) rec.imax = -1;
        rec.vdraft    = 0.0f;
        rec.has_draft = 0;
        if (draft != nullptr && r < n_draft) {
            const int64_t d = (int64_t) draft[r] - vocab_offset;
            if (d >= 0 && d < a.n_vocab) {
                rec.vdraft    = x[d];
                rec.has_draft = 1;
            }
        }
        out[r] = rec;
    }
}

__global__ void __launch_bounds__(32 * kMaxRows) accept_merge_kernel(const srhpm_argmax_record * recs, int n_shards,
                                                                       int n_rows, const int32_t * draft, int n_draft,
                                                                       float relax, int32_t * out_ids,
                                                                       int32_t * out_n) {
    pdl_wait();
    __shared__ int   am[kMaxRows], has[kMaxRows];
    __shared__ float amv[kMaxRows], dl[kMaxRows];
    if (threadIdx.x < n_rows) {
        const int r = threadIdx.x;
        ArgPair   p{ -INFINITY, INT32_MAX };
        bool      first_nan = false;
        has[r]              = 0;
        dl[r]               = 0.0f;
        for (int s = 0; s < n_shards; s++) {
            const srhpm_argmax_record rec = recs[s * n_rows + r];
            if (rec.imax == -1) first_nan = true;
            if (rec.imax >= 0) p = arg_better(p, ArgPair{ rec.vmax, rec.imax });
            if (rec.has_draft) {
                dl[r]  = rec.vdraft;
                has[r] = 1;
            }
        }
        am[r]  = (first_nan || p.i == INT32_MAX) ? 0 : p.i;
        amv[r] = p.v;
    }
    __syncthreads();
    if (threadIdx.x == 0) accept_scan(am, amv, dl, has, draft, n_draft, relax, out_ids, out_n);
}

int launch_pdl(const void * fn, void ** args, dim3 grid, dim3 block, cudaStream_t stream) {
    cudaLaunchConfig_t  cfg = {};
    cudaLaunchAttribute attr[1];
    cfg.gridDim                                        = grid;
    cfg.blockDim                                       = block;
    cfg.stream                                         = stream;
    attr[0].id                                         = cudaLaunchAttributeProgrammaticStreamSerialization;
    attr[0].val.programmaticStreamSerializationAllowed = 1;
    cfg.attrs                                          = attr;
    cfg.numAttrs                                       = 1;
    return cuda_status(cudaLaunchKernelExC(&cfg, fn, args));
}

ArgArgs arg_plan(int num_sms, const uint8_t * logits, int64_t ldb, int n_vocab, int n_rows, void * wdata) {
    ArgArgs a;
    a.logits   = logits;
    a.ldb      = ldb;
    a.n_vocab  = n_vocab;
    a.n_rows   = n_rows;
    const int want = std::max(1, (2 * num_sms + n_rows - 1) / n_rows);
    a.seg_len  = std::max(1024, ((n_vocab + want - 1) / want + 3) / 4 * 4);
    a.nseg     = (n_vocab + a.seg_len - 1) / a.seg_len;
    a.part     = reinterpret_cast<ArgPair *>(wdata);
    return a;
}

}  // namespace

size_t argmax_work_size(int num_sms, int n_vocab, int n_rows) {
    const ArgArgs a = arg_plan(num_sms, nullptr, 0, n_vocab, n_rows, nullptr);
    return (size_t) a.nseg * n_rows * sizeof(ArgPair);
}

int accept_run(srhpm_ctx * ctx, const uint8_t * logits, int64_t ldb, int n_vocab, int n_rows, const int32_t * draft,
               int n_draft, float relax, int32_t * out_ids, int32_t * out_n, int64_t vocab_offset,
               srhpm_argmax_record * out_recs, void * wdata, size_t wsize, cudaStream_t stream) {
    if (n_rows > kMaxRows) return SRHPM_UNSUPPORTED;
    ArgArgs a = arg_plan(ctx->num_sms, logits, ldb, n_vocab, n_rows, wdata);
    if (wdata == nullptr || wsize < argmax_work_size(ctx->num_sms, n_vocab, n_rows)) return SRHPM_ERR_WORKSPACE;
    argmax_part_kernel<<<dim3(a.nseg, n_rows), kArgThreads, 0, stream>>>(a);
    ctx->launches.fetch_add(1);
    int st = cuda_status(cudaGetLastError());
    if (st != SRHPM_OK) return st;
    if (out_recs == nullptr) {
        void * args[] = { &a, &draft, &n_draft, &relax, &out_ids, &out_n };
        st = launch_pdl((const void *) accept_final_kernel, args, dim3(1), dim3(32 * kMaxRows), stream);
    } else {
        void * args[] = { &a, &vocab_offset, &draft, &n_draft, &out_recs };
        st = launch_pdl((const void *) shard_final_kernel, args, dim3(1), dim3(32 * kMaxRows), stream);
    }
    ctx->launches.fetch_add(1);
    return st;
}

int accept_merge_run(srhpm_ctx * ctx, const srhpm_argmax_record * recs, int n_shards, int n_rows,
                     const int32_t * draft, int n_draft, float relax, int32_t * out_ids, int32_t * out_n,
                     cudaStream_t stream) {
    if (n_rows > kMaxRows) return SRHPM_UNSUPPORTED;
    void * args[] = { &recs, &n_shards, &n_rows, &draft, &n_draft, &relax, &out_ids, &out_n };
    const int st  = launch_pdl((const void *) accept_merge_kernel, args, dim3(1), dim3(32 * kMaxRows), stream);
    ctx->launches.fetch_add(1);
    return st;
}

}  // namespace srhpm
