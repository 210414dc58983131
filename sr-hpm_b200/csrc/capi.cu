// The C ABI of libsrhpm_b200: argument validation against the ggml operator contracts, context management, and
// dispatch to the kernels. Every check that fails returns a status code; nothing aborts.
#include <cstdio>

#include "internal.h"

namespace srhpm {

static thread_local int g_last_cuda_error = 0;

void set_last_cuda_error(cudaError_t e) { g_last_cuda_error = (int) e; }

bool is_weight_type(int type) {
    switch (type) {
        case SRHPM_TYPE_Q4_K:
        case SRHPM_TYPE_Q5_K:
        case SRHPM_TYPE_Q6_K:
        case SRHPM_TYPE_Q3_K:
        case SRHPM_TYPE_IQ4_XS:
        case SRHPM_TYPE_Q8_0: return true;
        default: return false;
    }
}

int weight_block_bytes(int type) { return (int) srhpm_type_size(type); }

}  // namespace srhpm

using namespace srhpm;

namespace {

bool aligned(const void * p, size_t a) { return (reinterpret_cast<uintptr_t>(p) % a) == 0; }

// ggml_mul_mat(W, X) -> Y contract of the verify path (patch/srhpm.patch:6400-6407, :6474)
int check_mul_mat(const srhpm_tensor * W, const srhpm_tensor * X, const srhpm_tensor * Y) {
    if (!W || !X) return SRHPM_ERR_INVALID;
    if (!is_weight_type(W->type)) return SRHPM_UNSUPPORTED;
    if (X->type != SRHPM_TYPE_F32) return SRHPM_UNSUPPORTED;
    const int64_t K = W->ne[0], rows = W->ne[1], N = X->ne[1];
    if (W->ne[2] != 1 || W->ne[3] != 1 || X->ne[2] != 1 || X->ne[3] != 1) return SRHPM_UNSUPPORTED;
    if (N < 1 || N > 16) return SRHPM_UNSUPPORTED;  // larger batches: the stock path (SRV_MAXM = 16)
    if (K <= 0 || K % 256 != 0 || rows <= 0) return SRHPM_UNSUPPORTED;
    if (X->ne[0] != K) return SRHPM_ERR_INVALID;
    if (W->nb[0] != srhpm_type_size(W->type) || W->nb[1] != srhpm_row_size(W->type, K)) return SRHPM_ERR_INVALID;
    if (X->nb[0] != 4 || X->nb[1] % 4 != 0 || X->nb[1] < (size_t) K * 4) return SRHPM_ERR_INVALID;
    if (!W->data || !X->data) return SRHPM_ERR_INVALID;
    if (!aligned(W->data, 16)) return SRHPM_ERR_ALIGN;
    if (!aligned(X->data, 4)) return SRHPM_ERR_ALIGN;
    if (Y) {
        if (Y->type != SRHPM_TYPE_F32 || Y->ne[0] != rows || Y->ne[1] != N || !Y->data) return SRHPM_ERR_INVALID;
        if (Y->nb[0] != 4 || Y->nb[1] % 4 != 0 || Y->nb[1] < (size_t) rows * 4 || !aligned(Y->data, 4)) {
            return SRHPM_ERR_INVALID;
        }
    }
    return SRHPM_OK;
}

int check_act(const srhpm_tensor * X) {
    if (!X || X->type != SRHPM_TYPE_F32 || !X->data) return SRHPM_ERR_INVALID;
    if (X->ne[0] <= 0 || X->ne[0] % 256 != 0 || X->ne[1] < 1 || X->ne[2] != 1 || X->ne[3] != 1) return SRHPM_ERR_INVALID;
    if (X->nb[0] != 4 || X->nb[1] % 4 != 0 || X->nb[1] < (size_t) X->ne[0] * 4) return SRHPM_ERR_INVALID;
    return SRHPM_OK;
}

}  // namespace

extern "C" {

int srhpm_ctx_create(int device, srhpm_ctx ** out) {
    if (!out) return SRHPM_ERR_INVALID;
    *out = nullptr;
    int n = 0;
    int st = cuda_status(cudaGetDeviceCount(&n));
    if (st != SRHPM_OK) return st;
    if (device < 0 || device >= n) return SRHPM_ERR_INVALID;
    int prev = 0;
    cudaGetDevice(&prev);
    st = cuda_status(cudaSetDevice(device));
    if (st != SRHPM_OK) return st;
    srhpm_ctx * c = new srhpm_ctx();
    c->device     = device;
    cudaDeviceGetAttribute(&c->num_sms, cudaDevAttrMultiProcessorCount, device);
    st = cuda_status(cudaMalloc(&c->d_status, 64));
    if (st == SRHPM_OK) st = cuda_status(cudaMemset(c->d_status, 0, 64));
    cudaSetDevice(prev);
    if (st != SRHPM_OK) {
        if (c->d_status) cudaFree(c->d_status);
        delete c;
        return st;
    }
    *out = c;
    return SRHPM_OK;
}

int srhpm_ctx_destroy(srhpm_ctx * ctx) {
    if (!ctx) return SRHPM_ERR_INVALID;
    if (ctx->d_status) cudaFree(ctx->d_status);
    delete ctx;
    return SRHPM_OK;
}

int srhpm_ctx_set_q8_0_act_mode(srhpm_ctx * ctx, int mode) {
    if (!ctx || (mode != SRHPM_Q8_0_ACT_SIMD && mode != SRHPM_Q8_0_ACT_REF)) return SRHPM_ERR_INVALID;
    ctx->q8_0_act_mode = mode;
    return SRHPM_OK;
}

int64_t srhpm_ctx_launch_count(const srhpm_ctx * ctx, int reset) {
    if (!ctx) return -1;
    srhpm_ctx * c = const_cast<srhpm_ctx *>(ctx);
    return reset ? c->launches.exchange(0) : c->launches.load();
}

int srhpm_ctx_check(srhpm_ctx * ctx, int32_t * device_code) {
    if (!ctx) return SRHPM_ERR_INVALID;
    int32_t code = 0;
    int     st   = cuda_status(cudaMemcpy(&code, ctx->d_status, 4, cudaMemcpyDeviceToHost));
    if (st != SRHPM_OK) return st;
    if (device_code) *device_code = code;
    if (code != 0) {
        cudaMemset(ctx->d_status, 0, 4);
        return SRHPM_ERR_DEVICE;
    }
    return SRHPM_OK;
}

int srhpm_last_cuda_error(void) { return g_last_cuda_error; }

const char * srhpm_status_str(int status) {
    switch (status) {
        case SRHPM_OK: return "ok";
        case SRHPM_UNSUPPORTED: return "unsupported (use the stock path)";
        case SRHPM_ERR_INVALID: return "invalid argument";
        case SRHPM_ERR_ALIGN: return "misaligned pointer or stride";
        case SRHPM_ERR_WORKSPACE: return "work buffer missing or too small";
        case SRHPM_ERR_CUDA: return "CUDA runtime error";
        case SRHPM_ERR_DEVICE: return "a kernel reported an error";
        case SRHPM_ERR_TOO_LARGE: return "product too large for the static work buffer";
        default: return "unknown status";
    }
}

int srhpm_blck_size(int type) {
    switch (type) {
        case SRHPM_TYPE_F32:
        case SRHPM_TYPE_F16:
        case SRHPM_TYPE_I32: return 1;
        case SRHPM_TYPE_Q8_0: return 32;
        case SRHPM_TYPE_Q3_K:
        case SRHPM_TYPE_Q4_K:
        case SRHPM_TYPE_Q5_K:
        case SRHPM_TYPE_Q6_K:
        case SRHPM_TYPE_Q8_K:
        case SRHPM_TYPE_IQ4_XS: return 256;
        default: return 0;
    }
}

size_t srhpm_type_size(int type) {
    switch (type) {
        case SRHPM_TYPE_F32: return 4;
        case SRHPM_TYPE_F16: return 2;
        case SRHPM_TYPE_I32: return 4;
        case SRHPM_TYPE_Q8_0: return 34;
        case SRHPM_TYPE_Q3_K: return 110;
        case SRHPM_TYPE_Q4_K: return 144;
        case SRHPM_TYPE_Q5_K: return 176;
        case SRHPM_TYPE_Q6_K: return 210;
        case SRHPM_TYPE_Q8_K: return 292;
        case SRHPM_TYPE_IQ4_XS: return 136;
        default: return 0;
    }
}

size_t srhpm_row_size(int type, int64_t n) {
    const int bs = srhpm_blck_size(type);
    if (bs <= 0 || n % bs) return 0;
    return srhpm_type_size(type) * (size_t) (n / bs);
}

int srhpm_mul_mat_work_size(const srhpm_tensor * W, const srhpm_tensor * X, size_t * size) {
    if (!size) return SRHPM_ERR_INVALID;
    const int st = check_mul_mat(W, X, nullptr);
    if (st != SRHPM_OK) return st;
    *size = gemm_work_size(W->type, W->ne[1], W->ne[0], X->ne[1]);
    return SRHPM_OK;
}

int srhpm_mul_mat(srhpm_ctx * ctx, const srhpm_tensor * W, const srhpm_tensor * X, srhpm_tensor * Y, void * wdata,
                  size_t wsize, void * stream) {
    if (!ctx || !Y) return SRHPM_ERR_INVALID;
    const int st = check_mul_mat(W, X, Y);
    if (st != SRHPM_OK) return st;
    return gemm_run(ctx, W->type, (const uint8_t *) W->data, W->ne[1], W->ne[0], W->nb[1], (const float *) X->data,
                    (int64_t) (X->nb[1] / 4), X->ne[1], (float *) Y->data, (int64_t) (Y->nb[1] / 4), wdata, wsize,
                    nullptr, nullptr, (cudaStream_t) stream);
}

int srhpm_mul_mat_static(srhpm_ctx * ctx, const srhpm_tensor * W, const srhpm_tensor * X, srhpm_tensor * Y,
                         void * stream) {
    if (!ctx || !Y) return SRHPM_ERR_INVALID;
    const int st = check_mul_mat(W, X, Y);
    if (st != SRHPM_OK) return st;
    return gemm_run_static(ctx, W->type, (const uint8_t *) W->data, W->ne[1], W->ne[0], W->nb[1],
                           (const float *) X->data, (int64_t) (X->nb[1] / 4), X->ne[1], (float *) Y->data,
                           (int64_t) (Y->nb[1] / 4), (cudaStream_t) stream);
}

int srhpm_mul_mat_isums(srhpm_ctx * ctx, const srhpm_tensor * W, const srhpm_tensor * X, int32_t * isum,
                        int32_t * imin, void * wdata, size_t wsize, void * stream) {
    if (!ctx || !isum) return SRHPM_ERR_INVALID;
    const int st = check_mul_mat(W, X, nullptr);
    if (st != SRHPM_OK) return st;
    return gemm_run(ctx, W->type, (const uint8_t *) W->data, W->ne[1], W->ne[0], W->nb[1], (const float *) X->data,
                    (int64_t) (X->nb[1] / 4), X->ne[1], nullptr, 0, wdata, wsize, isum, imin, (cudaStream_t) stream);
}

int srhpm_quantize_rows_q8_K(srhpm_ctx * ctx, const srhpm_tensor * X, int8_t * q, float * d, int16_t * bsum32,
                             int16_t * bsum16, void * stream) {
    if (!ctx || !q || !d) return SRHPM_ERR_INVALID;
    const int st = check_act(X);
    if (st != SRHPM_OK) return st;
    if (!aligned(q, 8)) return SRHPM_ERR_ALIGN;
    return quantize_q8K_dense(ctx, (const float *) X->data, (int64_t) (X->nb[1] / 4), X->ne[1], X->ne[0], q, d, bsum32,
                              bsum16, (cudaStream_t) stream);
}

int srhpm_quantize_rows_q8_0(srhpm_ctx * ctx, const srhpm_tensor * X, void * blocks, void * stream) {
    if (!ctx || !blocks) return SRHPM_ERR_INVALID;
    const int st = check_act(X);
    if (st != SRHPM_OK) return st;
    if (!aligned(blocks, 2)) return SRHPM_ERR_ALIGN;
    return quantize_q8_0_dense(ctx, (const float *) X->data, (int64_t) (X->nb[1] / 4), X->ne[1], X->ne[0], blocks,
                               (cudaStream_t) stream);
}

}  // extern "C"
