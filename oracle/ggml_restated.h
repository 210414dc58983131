// TEST INFRASTRUCTURE (oracle). Restatements of the upstream ggml/ggml-cpu routines (llama.cpp @ d05706b, not
// available here) that the reference's FA-GQA function (patch/srhpm.patch:581-824) calls, plus the minimal tensor /
// thread-pool types it reads. Each routine states the upstream behaviour it follows; none is copied source.
#pragma once
#include "ref_shim.h"
#include <algorithm>
#include <atomic>
#include <cmath>
#include <cstdio>
#include <cstdlib>
#include <thread>
#include <vector>

#ifndef GGML_FA_TILE_KV
// KV tile of the grouped FA path (patch/srhpm.patch:621, :678). The upstream value is not in the container; the
// output depends on it only through the f32 summation order and chunk rounding.
#define GGML_FA_TILE_KV 32
#endif
#define CACHE_LINE_SIZE 64
#define CACHE_LINE_SIZE_F32 (CACHE_LINE_SIZE / sizeof(float))

#define GGML_ASSERT(x)                                                                   \
    do {                                                                                 \
        if (!(x)) {                                                                      \
            fprintf(stderr, "oracle GGML_ASSERT failed: %s (%s:%d)\n", #x, __FILE__, __LINE__); \
            abort();                                                                     \
        }                                                                                \
    } while (0)
#define GGML_UNUSED(x) (void) (x)

// ggml_type numbering (GGUF)
enum ggml_type {
    GGML_TYPE_F32 = 0, GGML_TYPE_F16 = 1, GGML_TYPE_Q8_0 = 8, GGML_TYPE_Q3_K = 11, GGML_TYPE_Q4_K = 12,
    GGML_TYPE_Q5_K = 13, GGML_TYPE_Q6_K = 14, GGML_TYPE_Q8_K = 15, GGML_TYPE_IQ4_XS = 23, GGML_TYPE_COUNT = 40,
};

struct ggml_tensor {
    enum ggml_type type;
    int64_t        ne[4];
    size_t         nb[4];
    int32_t        op_params[16];
    ggml_tensor *  src[10];
    void *         data;
};

// GGML_TENSOR_LOCALS(type, prefix, tensor, field): prefix0..prefix3 = tensor->field[0..3]
#define GGML_TENSOR_LOCALS(T, P, X, F)          \
    const T P##0 = (X)->F[0]; GGML_UNUSED(P##0); \
    const T P##1 = (X)->F[1]; GGML_UNUSED(P##1); \
    const T P##2 = (X)->F[2]; GGML_UNUSED(P##2); \
    const T P##3 = (X)->F[3]; GGML_UNUSED(P##3);

// thread pool: a shared work counter (fetch-add returns the previous value, as upstream) and a spin barrier
struct ggml_threadpool {
    std::atomic<int> chunk{0};
    std::atomic<int> arrived{0};
    std::atomic<int> phase{0};
    int              n_threads = 1;
};
static inline void ggml_threadpool_chunk_set(ggml_threadpool * tp, int v) { tp->chunk.store(v); }
static inline int ggml_threadpool_chunk_add(ggml_threadpool * tp, int v) { return tp->chunk.fetch_add(v); }
static inline void ggml_barrier(ggml_threadpool * tp) {
    if (tp->n_threads == 1) {
        return;
    }
    const int ph = tp->phase.load();
    if (tp->arrived.fetch_add(1) == tp->n_threads - 1) {
        tp->arrived.store(0);
        tp->phase.fetch_add(1);
    } else {
        while (tp->phase.load() == ph) {
            std::this_thread::yield();
        }
    }
}

struct ggml_compute_params {
    int               ith, nth;
    size_t            wsize;
    void *            wdata;
    ggml_threadpool * threadpool;
    bool              use_ref;
};

// --- q8_0 (the vec_dot type of a q8_0 KV cache) ----------------------------------------------------------------
// Selects which q8_0 activation quantizer from_float runs (see oracle.h: ORC_Q8_0_SIMD / ORC_Q8_0_REF).
extern int g_ref_q8_0_mode;

// from_float of q8_0. Mode 0 follows ggml-cpu's x86 SIMD quantizer: d = amax/127 stored as f16,
// id = 127/amax, q = round-half-even(x*id). Mode 1 follows ggml's scalar quantize_row_q8_0_ref:
// id = 1/d (f32 d before the f16 store), q = roundf(x*id) (half away from zero).
static inline void ref_quantize_row_q8_0(const float * x, void * vy, int64_t k) {
    block_q8_0 * y  = (block_q8_0 *) vy;
    const int64_t nb = k / QK8_0;
    for (int64_t i = 0; i < nb; i++) {
        float amax = 0.0f;
        for (int j = 0; j < QK8_0; j++) {
            amax = std::max(amax, fabsf(x[i * QK8_0 + j]));
        }
        const float d = amax / 127.f;
        y[i].d        = ref_fp32_to_fp16(d);
        if (g_ref_q8_0_mode == 0) {
            const float id = amax != 0.0f ? 127.f / amax : 0.0f;
            for (int j = 0; j < QK8_0; j++) {
                y[i].qs[j] = (int8_t) lrintf(x[i * QK8_0 + j] * id);  // default rounding mode: nearest-even
            }
        } else {
            const float id = d != 0.0f ? 1.0f / d : 0.0f;
            for (int j = 0; j < QK8_0; j++) {
                y[i].qs[j] = (int8_t) roundf(x[i * QK8_0 + j] * id);
            }
        }
    }
}

static inline void ref_dequantize_row_q8_0(const void * vx, float * y, int64_t k) {
    const block_q8_0 * x = (const block_q8_0 *) vx;
    for (int64_t i = 0; i < k / QK8_0; i++) {
        const float d = ref_fp16_to_fp32(x[i].d);
        for (int j = 0; j < QK8_0; j++) {
            y[i * QK8_0 + j] = x[i].qs[j] * d;
        }
    }
}

// 8-lane f32 horizontal sum in the order of the x86 path: (l0+l4, l1+l5, l2+l6, l3+l7), then pairs, then the two
static inline float ref_hsum8(const float a[8]) {
    const float s0 = a[0] + a[4], s1 = a[1] + a[5], s2 = a[2] + a[6], s3 = a[3] + a[7];
    return (s0 + s2) + (s1 + s3);
}

// vec_dot of q8_0 x q8_0 as ggml-cpu's x86 path accumulates it: per 32-block, 8 int32 lanes of 4 products each,
// converted to f32 and fused-multiply-added with d_x*d_y into 8 f32 lane accumulators; then ref_hsum8.
static inline void ref_vec_dot_q8_0_q8_0(int n, float * s, size_t bs, const void * vx, size_t bx, const void * vy,
                                         size_t by, int nrc) {
    GGML_UNUSED(bs); GGML_UNUSED(bx); GGML_UNUSED(by); GGML_UNUSED(nrc);
    const block_q8_0 * x = (const block_q8_0 *) vx;
    const block_q8_0 * y = (const block_q8_0 *) vy;
    float acc[8] = { 0 };
    for (int ib = 0; ib < n / QK8_0; ib++) {
        const float d = ref_fp16_to_fp32(x[ib].d) * ref_fp16_to_fp32(y[ib].d);
        for (int l = 0; l < 8; l++) {
            int p = 0;
            for (int j = 4 * l; j < 4 * l + 4; j++) {
                p += (int) x[ib].qs[j] * (int) y[ib].qs[j];
            }
            acc[l] = fmaf(d, (float) p, acc[l]);
        }
    }
    *s = ref_hsum8(acc);
}

static inline void ref_fp16_row_to_fp32(const void * vx, float * y, int64_t k) {
    const ggml_half * x = (const ggml_half *) vx;
    for (int64_t i = 0; i < k; i++) {
        y[i] = ref_fp16_to_fp32(x[i]);
    }
}

struct ggml_type_traits {
    int64_t blck_size;
    size_t  type_size;
    void (*to_float)(const void *, float *, int64_t);
};
struct ggml_type_traits_cpu {
    void (*from_float)(const float *, void *, int64_t);
    void (*vec_dot)(int, float *, size_t, const void *, size_t, const void *, size_t, int);
    enum ggml_type vec_dot_type;
};

static inline const ggml_type_traits * ggml_get_type_traits(enum ggml_type t) {
    static const ggml_type_traits f32  = { 1, 4, nullptr };
    static const ggml_type_traits f16  = { 1, 2, ref_fp16_row_to_fp32 };
    static const ggml_type_traits q8_0 = { 32, 34, ref_dequantize_row_q8_0 };
    switch (t) {
        case GGML_TYPE_F32: return &f32;
        case GGML_TYPE_F16: return &f16;
        case GGML_TYPE_Q8_0: return &q8_0;
        default: GGML_ASSERT(false && "type not supported by the oracle"); return nullptr;
    }
}
static inline const ggml_type_traits_cpu * ggml_get_type_traits_cpu(enum ggml_type t) {
    static const ggml_type_traits_cpu f32  = { nullptr, nullptr, GGML_TYPE_F32 };
    static const ggml_type_traits_cpu f16  = { nullptr, nullptr, GGML_TYPE_F16 };
    static const ggml_type_traits_cpu q8_0 = { ref_quantize_row_q8_0, ref_vec_dot_q8_0_q8_0, GGML_TYPE_Q8_0 };
    switch (t) {
        case GGML_TYPE_F32: return &f32;
        case GGML_TYPE_F16: return &f16;
        case GGML_TYPE_Q8_0: return &q8_0;
        default: GGML_ASSERT(false && "type not supported by the oracle"); return nullptr;
    }
}
static inline int64_t ggml_blck_size(enum ggml_type t) { return ggml_get_type_traits(t)->blck_size; }
static inline size_t ggml_row_size(enum ggml_type t, int64_t n) {
    const ggml_type_traits * tt = ggml_get_type_traits(t);
    return tt->type_size * (size_t) (n / tt->blck_size);
}

// C[M x N] += A[M x K] * B[K x N], all row-major f32: for each output row, for each k, a broadcast of A[i][k]
// fused-multiply-added across the row of B (the order of a SIMD implementation vectorised over N)
static inline void simd_gemm(float * C, const float * A, const float * B, int64_t M, int64_t K, int64_t N) {
    for (int64_t i = 0; i < M; i++) {
        float * c = C + i * N;
        for (int64_t k = 0; k < K; k++) {
            const float a = A[i * K + k];
            const float * b = B + k * N;
            for (int64_t j = 0; j < N; j++) {
                c[j] = fmaf(a, b[j], c[j]);
            }
        }
    }
}

static inline void ggml_vec_scale_f32(int64_t n, float * y, float v) {
    for (int64_t i = 0; i < n; i++) y[i] *= v;
}
static inline void ggml_vec_tanh_f32(int64_t n, float * y, const float * x) {
    for (int64_t i = 0; i < n; i++) y[i] = tanhf(x[i]);
}
static inline void ggml_vec_add_f32(int64_t n, float * z, const float * x, const float * y) {
    for (int64_t i = 0; i < n; i++) z[i] = x[i] + y[i];
}
static inline void ggml_vec_max_f32(int64_t n, float * s, const float * x) {
    float m = -INFINITY;
    for (int64_t i = 0; i < n; i++) m = std::max(m, x[i]);
    *s = m;
}
// y = exp(x - max), returns the sum in double (upstream returns ggml_float = double)
static inline double ggml_vec_soft_max_f32(int64_t n, float * y, const float * x, float max) {
    double sum = 0;
    for (int64_t i = 0; i < n; i++) {
        const float v = expf(x[i] - max);
        sum += (double) v;
        y[i] = v;
    }
    return sum;
}
static inline void ggml_cpu_fp16_to_fp32(const ggml_fp16_t * x, float * y, int64_t n) {
    for (int64_t i = 0; i < n; i++) y[i] = ref_fp16_to_fp32(x[i]);
}
