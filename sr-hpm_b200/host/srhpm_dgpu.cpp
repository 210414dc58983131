// libsrhpm_dgpu.so: the reference's dGPU library interface (dgpu/dgpu.cu:17-312), which ggml-cpu loads by name next
// to itself and binds with dlsym / GetProcAddress (patch/srhpm.patch:5034-5055): dgpu_init, dgpu_launch,
// dgpu_collect, dgpu_mem_info, plus dgpu_pinned_bytes. The same contract on the B200 kernels, over the C ABI:
//   - dgpu_launch(kind 0 = IQ4_XS / 1 = Q3_K, key, rows, nrows, K, M <= 8, x, x_nb, max_pinned) takes the first nrows
//     rows of the tensor identified by `key`, copies them once per key (re-copied when a launch needs more rows), and
//     starts Y = rows . x^T asynchronously; status 0, or -1 bad arguments, -2 the copies would exceed max_pinned,
//     -3 no memory for the copy, -4 no memory for the staging buffers, -5 the launch failed, -6 Q3_K rows of an odd
//     number of super-blocks (as the reference, whose rows would not be 4-byte aligned); nothing runs on failure;
//   - dgpu_collect(M, nrows, dst, dst_nb) waits for the last launch and writes y[t][0..nrows) to dst + t * dst_nb
//     (M and nrows those of the launch; -1 otherwise, -5 when the launch failed on the device).
// Two differences, both from the B200's design:
//   - the copies live in HBM (device memory) instead of pinned host memory read over PCIe, so max_pinned bounds
//     their HBM bytes;
//   - the activations are quantized per 256 columns exactly as the CPU's SRV rows are (srv_quantize_row), so the rows
//     of a product split between the CPU and this library agree with each other bit for bit in their integer sums;
//     the reference's dGPU kernels work on the f32 activations instead.
// Thread-safe: launches and collects are serialised by one mutex, as the reference's launches are.
#include <cuda_runtime_api.h>

#include <cstdint>
#include <cstdio>
#include <cstdlib>
#include <cstring>
#include <mutex>
#include <unordered_map>

#include "srhpm_b200.h"
#include "srhpm_dgpu.h"

#define DGPU_API extern "C" __attribute__((visibility("default")))

namespace {

constexpr int     kMaxM = 8;    // MMAX of the reference's kernels
constexpr int64_t kQK   = 256;

struct Copy {
    void * dev;
    size_t bytes;
};

std::mutex                               g_mtx;
srhpm_ctx *                              g_ctx    = nullptr;
cudaStream_t                             g_stream = nullptr;
cudaEvent_t                              g_done   = nullptr;
std::unordered_map<const void *, Copy>   g_w;
size_t                                   g_held = 0;
// staging: x (pinned) -> x (device); y (device) -> y (pinned); the GEMM's work buffer
float *  g_xh = nullptr, * g_xd = nullptr, * g_yd = nullptr, * g_yh = nullptr;
size_t   g_xcap = 0, g_ycap = 0;
void *   g_work = nullptr;
size_t   g_wcap = 0;
bool     g_launched = false;
int      g_last_m   = 0;   // shape of the last launch (the layout of the staged result)
int64_t  g_last_rows = 0;

bool grow_device(void ** p, size_t * cap, size_t need) {
    if (need <= *cap) return true;
    cudaFree(*p);
    *p = nullptr;
    *cap = 0;
    if (cudaMalloc(p, need) != cudaSuccess) {
        cudaGetLastError();
        return false;
    }
    *cap = need;
    return true;
}

bool ensure_stage(size_t xn, size_t yn, size_t wbytes) {
    if (xn > g_xcap) {
        cudaFreeHost(g_xh);
        cudaFree(g_xd);
        g_xh = g_xd = nullptr;
        g_xcap      = 0;
        if (cudaHostAlloc(reinterpret_cast<void **>(&g_xh), xn * sizeof(float), cudaHostAllocDefault) != cudaSuccess ||
            cudaMalloc(reinterpret_cast<void **>(&g_xd), xn * sizeof(float)) != cudaSuccess) {
            cudaGetLastError();
            return false;
        }
        g_xcap = xn;
    }
    if (yn > g_ycap) {
        cudaFreeHost(g_yh);
        cudaFree(g_yd);
        g_yh = g_yd = nullptr;
        g_ycap      = 0;
        if (cudaHostAlloc(reinterpret_cast<void **>(&g_yh), yn * sizeof(float), cudaHostAllocDefault) != cudaSuccess ||
            cudaMalloc(reinterpret_cast<void **>(&g_yd), yn * sizeof(float)) != cudaSuccess) {
            cudaGetLastError();
            return false;
        }
        g_ycap = yn;
    }
    return grow_device(&g_work, &g_wcap, wbytes > 0 ? wbytes : 256);
}

}  // namespace

DGPU_API int dgpu_init() {
    std::lock_guard<std::mutex> lk(g_mtx);
    if (g_ctx) {
        return 0;
    }
    int dev = 0;
    if (cudaGetDevice(&dev) != cudaSuccess) {
        cudaGetLastError();
        return -1;
    }
    srhpm_ctx * ctx = nullptr;
    if (srhpm_ctx_create(dev, &ctx) != SRHPM_OK) {
        return -1;
    }
    if (cudaStreamCreateWithFlags(&g_stream, cudaStreamNonBlocking) != cudaSuccess ||
        cudaEventCreateWithFlags(&g_done, cudaEventDisableTiming) != cudaSuccess) {
        cudaGetLastError();
        srhpm_ctx_destroy(ctx);
        return -1;
    }
    g_ctx = ctx;
    return 0;
}

DGPU_API size_t dgpu_pinned_bytes() {
    std::lock_guard<std::mutex> lk(g_mtx);
    return g_held;
}

DGPU_API void dgpu_mem_info(size_t * free_b, size_t * total_b) {
    if (cudaMemGetInfo(free_b, total_b) != cudaSuccess) {
        cudaGetLastError();
        *free_b = *total_b = 0;
    }
}

DGPU_API int dgpu_launch(int kind, const void * key, const void * rows, int64_t nrows, int64_t K, int M,
                         const float * x, size_t x_nb, size_t max_pinned) {
    if ((kind != 0 && kind != 1) || M < 1 || M > kMaxM || K <= 0 || K % kQK || nrows < 1 || !rows || !x ||
        x_nb < (size_t) K * sizeof(float)) {
        return -1;
    }
    const int     type  = kind == 0 ? SRHPM_TYPE_IQ4_XS : SRHPM_TYPE_Q3_K;
    const int64_t nsb   = K / kQK;
    if (kind == 1 && (nsb & 1)) {
        return -6;
    }
    const size_t  rowb  = srhpm_row_size(type, K);
    const size_t  bytes = (size_t) nrows * rowb;
    std::lock_guard<std::mutex> lk(g_mtx);
    if (!g_ctx) {
        return -5;  // dgpu_init has not succeeded
    }
    // the previous launch may still read the copies and the staging buffers
    if (cudaStreamSynchronize(g_stream) != cudaSuccess) {
        cudaGetLastError();
        return -5;
    }
    auto it = g_w.find(key);
    if (it == g_w.end() || it->second.bytes < bytes) {
        const size_t old = it == g_w.end() ? 0 : it->second.bytes;
        if (g_held - old + bytes > max_pinned) {
            return -2;
        }
        void * d = nullptr;
        if (cudaMalloc(&d, bytes) != cudaSuccess) {
            cudaGetLastError();
            return -3;
        }
        // pageable source: complete before the launch below reads it
        if (cudaMemcpyAsync(d, rows, bytes, cudaMemcpyHostToDevice, g_stream) != cudaSuccess ||
            cudaStreamSynchronize(g_stream) != cudaSuccess) {
            cudaGetLastError();
            cudaFree(d);
            return -3;
        }
        if (it != g_w.end()) {
            cudaFree(it->second.dev);
        }
        g_w[key] = { d, bytes };
        g_held   = g_held - old + bytes;
        it       = g_w.find(key);
    }
    srhpm_tensor W = {}, X = {}, Y = {};
    W.type  = type;
    W.ne[0] = K;
    W.ne[1] = nrows;
    W.ne[2] = W.ne[3] = 1;
    W.nb[0] = srhpm_type_size(type);
    W.nb[1] = rowb;
    W.nb[2] = W.nb[3] = rowb * (size_t) nrows;
    W.data  = it->second.dev;
    X.type  = SRHPM_TYPE_F32;
    X.ne[0] = K;
    X.ne[1] = M;
    X.ne[2] = X.ne[3] = 1;
    X.nb[0] = sizeof(float);
    X.nb[1] = (size_t) K * sizeof(float);
    X.nb[2] = X.nb[3] = X.nb[1] * (size_t) M;
    Y.type  = SRHPM_TYPE_F32;
    Y.ne[0] = nrows;
    Y.ne[1] = M;
    Y.ne[2] = Y.ne[3] = 1;
    Y.nb[0] = sizeof(float);
    Y.nb[1] = (size_t) nrows * sizeof(float);
    Y.nb[2] = Y.nb[3] = Y.nb[1] * (size_t) M;
    size_t ws = 0;
    X.data    = reinterpret_cast<void *>(16);  // the work size reads shapes only
    if (srhpm_mul_mat_work_size(&W, &X, &ws) != SRHPM_OK) {
        return -1;
    }
    if (!ensure_stage((size_t) M * K, (size_t) M * nrows, ws)) {
        return -4;
    }
    for (int t = 0; t < M; t++) {
        memcpy(g_xh + (size_t) t * K, reinterpret_cast<const char *>(x) + t * x_nb, (size_t) K * sizeof(float));
    }
    X.data = g_xd;
    Y.data = g_yd;
    if (cudaMemcpyAsync(g_xd, g_xh, (size_t) M * K * sizeof(float), cudaMemcpyHostToDevice, g_stream) != cudaSuccess) {
        cudaGetLastError();
        return -5;
    }
    if (srhpm_mul_mat(g_ctx, &W, &X, &Y, g_work, g_wcap, g_stream) != SRHPM_OK) {
        return -5;
    }
    if (cudaMemcpyAsync(g_yh, g_yd, (size_t) M * nrows * sizeof(float), cudaMemcpyDeviceToHost, g_stream) !=
            cudaSuccess ||
        cudaEventRecord(g_done, g_stream) != cudaSuccess) {
        cudaGetLastError();
        return -5;
    }
    g_launched  = true;
    g_last_m    = M;
    g_last_rows = nrows;
    return 0;
}

DGPU_API int dgpu_collect(int M, int64_t nrows, char * dst, size_t dst_nb) {
    std::lock_guard<std::mutex> lk(g_mtx);
    if (!g_launched || M < 1 || M > g_last_m || nrows != g_last_rows || !dst) {
        return -1;  // not the shape of the last launch
    }
    if (cudaEventSynchronize(g_done) != cudaSuccess) {
        cudaGetLastError();
        return -5;
    }
    for (int t = 0; t < M; t++) {
        memcpy(dst + (size_t) t * dst_nb, g_yh + (size_t) t * nrows, (size_t) nrows * sizeof(float));
    }
    return 0;
}
