// srhpm_mul_mat_static: the quantized matmul without a caller-provided work buffer.
//
// Its scratch (the activation records and the row-block counters of srv_gemm.cu) lives in g_static_work, a
// file-scope device array that every GPU loading this library holds until the process exits. Host code cannot use
// the array's name as a device address (in host code it is only a stand-in for the symbol), so the first call on a
// device looks up the real address with cudaGetSymbolAddress, with that device current, and caches it. That first
// call should therefore come before any stream capture. Every call shares the array and leaves the last call's
// contents in it; the parts that must start at zero are cleared by each call's own quantizer kernel. Calls whose
// kernels overlap on the GPU (other streams, other host threads) race on the array.
#include <mutex>

#include "internal.h"

namespace srhpm {

constexpr size_t kStaticWorkBytes = size_t(1) << 20;  // 1 MiB

static __device__ __align__(256) uint8_t g_static_work[kStaticWorkBytes];

namespace {

constexpr int kMaxDevices = 64;
std::mutex    g_static_mu;
void *        g_static_ptr[kMaxDevices] = {};

// device address of g_static_work on `device` (looked up once per device, with that device current)
int static_work_ptr(int device, void ** out) {
    if (device < 0 || device >= kMaxDevices) return SRHPM_ERR_INVALID;
    std::lock_guard<std::mutex> lk(g_static_mu);
    if (!g_static_ptr[device]) {
        int prev = 0;
        int st   = cuda_status(cudaGetDevice(&prev));
        if (st != SRHPM_OK) return st;
        if (prev != device && (st = cuda_status(cudaSetDevice(device))) != SRHPM_OK) return st;
        void * p = nullptr;
        st       = cuda_status(cudaGetSymbolAddress(&p, g_static_work));
        if (prev != device) cudaSetDevice(prev);
        if (st != SRHPM_OK) return st;
        g_static_ptr[device] = p;
    }
    *out = g_static_ptr[device];
    return SRHPM_OK;
}

}  // namespace

size_t static_work_bytes() { return kStaticWorkBytes; }

int gemm_run_static(srhpm_ctx * ctx, int wtype, const uint8_t * W, int64_t rows, int64_t K, size_t row_bytes,
                    const float * X, int64_t ldx, int64_t N, float * Y, int64_t ldy, cudaStream_t stream) {
    const size_t need = gemm_work_size_unsplit(wtype, rows, K, N);
    if (need > kStaticWorkBytes) return SRHPM_ERR_TOO_LARGE;
    // the kernels launch on the calling thread's current device: it must be the context's, or they would use the
    // other device's copy of the array through a peer address
    int cur = -1;
    int st  = cuda_status(cudaGetDevice(&cur));
    if (st != SRHPM_OK) return st;
    if (cur != ctx->device) return SRHPM_ERR_INVALID;
    void * work = nullptr;
    st          = static_work_ptr(ctx->device, &work);
    if (st != SRHPM_OK) return st;
    return gemm_run_unsplit(ctx, wtype, W, rows, K, row_bytes, X, ldx, N, Y, ldy, work, kStaticWorkBytes, stream);
}

}  // namespace srhpm
