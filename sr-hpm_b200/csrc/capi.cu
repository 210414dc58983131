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

// ggml_flash_attn_ext(q, k, v, mask, sinks) contract of the reference's grouped path (patch/srhpm.patch:833-841) and
// of this kernel: q f32 [DK, N, H], k / v q8_0 [256, L, Hkv] (token and head strides multiples of 16 bytes), mask f16
// [>= L, >= N, ne2] broadcast over heads (h % ne2), sinks f32 [H], dst f32 [DV, H, N]
int check_fa(const srhpm_tensor * q, const srhpm_tensor * k, const srhpm_tensor * v, const srhpm_tensor * mask,
             const srhpm_tensor * sinks, const srhpm_tensor * dst, FaView * fv) {
    if (!q || !k || !v) return SRHPM_ERR_INVALID;
    if (q->type != SRHPM_TYPE_F32 || k->type != v->type) return SRHPM_UNSUPPORTED;
    if (k->type != SRHPM_TYPE_Q8_0 && k->type != SRHPM_TYPE_F16) return SRHPM_UNSUPPORTED;
    if (q->ne[3] != 1 || k->ne[3] != 1 || v->ne[3] != 1) return SRHPM_UNSUPPORTED;
    const int64_t DK = k->ne[0], DV = v->ne[0], L = k->ne[1], Hkv = k->ne[2], N = q->ne[1], H = q->ne[2];
    if (q->ne[0] != DK) return SRHPM_ERR_INVALID;
    if (DK != 256 || DV != 256) return SRHPM_UNSUPPORTED;
    if (N < 1 || N > 16) return SRHPM_UNSUPPORTED;
    if (L < 1 || L > INT32_MAX || Hkv < 1 || H < 1 || H > 65536 || H % Hkv != 0) return SRHPM_ERR_INVALID;
    if (v->ne[1] != L || v->ne[2] != Hkv) return SRHPM_ERR_INVALID;
    const size_t rowb = srhpm_row_size(k->type, 256);
    if (k->nb[0] != srhpm_type_size(k->type) || v->nb[0] != srhpm_type_size(v->type)) return SRHPM_ERR_INVALID;
    if (k->nb[1] < rowb || v->nb[1] < rowb || k->nb[2] < rowb || v->nb[2] < rowb) return SRHPM_ERR_INVALID;
    if (k->nb[1] % 16 || k->nb[2] % 16 || v->nb[1] % 16 || v->nb[2] % 16) return SRHPM_ERR_ALIGN;
    if (!k->data || !v->data || !q->data) return SRHPM_ERR_INVALID;
    if (!aligned(k->data, 16) || !aligned(v->data, 16) || !aligned(q->data, 4)) return SRHPM_ERR_ALIGN;
    if (q->nb[0] != 4 || q->nb[1] % 4 || q->nb[2] % 4) return SRHPM_ERR_INVALID;
    if (!dst || dst->type != SRHPM_TYPE_F32 || !dst->data) return SRHPM_ERR_INVALID;
    if (dst->ne[0] != DV || dst->ne[1] != H || dst->ne[2] != N || dst->ne[3] != 1) return SRHPM_ERR_INVALID;
    if (dst->nb[0] != 4 || dst->nb[1] % 4 || dst->nb[2] % 4 || !aligned(dst->data, 4)) return SRHPM_ERR_INVALID;
    fv->mask = nullptr;
    fv->mnb1 = fv->mnb2 = 0;
    fv->mne2 = 1;
    fv->mne0 = 0;
    if (mask) {
        if (mask->type != SRHPM_TYPE_F16 || !mask->data || mask->nb[0] != 2) return SRHPM_ERR_INVALID;
        if (mask->ne[0] < L || mask->ne[1] < N || mask->ne[2] < 1 || mask->ne[3] != 1) return SRHPM_ERR_INVALID;
        if (mask->nb[1] % 2 || mask->nb[2] % 2 || !aligned(mask->data, 2)) return SRHPM_ERR_ALIGN;
        fv->mask = (const uint8_t *) mask->data;
        fv->mnb1 = (int64_t) mask->nb[1];
        fv->mnb2 = (int64_t) mask->nb[2];
        fv->mne2 = (int) mask->ne[2];
        fv->mne0 = mask->ne[0];
    }
    fv->sinks = nullptr;
    if (sinks) {
        if (sinks->type != SRHPM_TYPE_F32 || sinks->ne[0] != H || sinks->nb[0] != 4 || !sinks->data) {
            return SRHPM_ERR_INVALID;
        }
        fv->sinks = (const float *) sinks->data;
    }
    fv->q    = (const float *) q->data;
    fv->qnb1 = (int64_t) q->nb[1];
    fv->qnb2 = (int64_t) q->nb[2];
    fv->N    = (int) N;
    fv->H    = (int) H;
    fv->k    = (const uint8_t *) k->data;
    fv->knb1 = (int64_t) k->nb[1];
    fv->knb2 = (int64_t) k->nb[2];
    fv->v    = (const uint8_t *) v->data;
    fv->vnb1 = (int64_t) v->nb[1];
    fv->vnb2 = (int64_t) v->nb[2];
    fv->L       = (int) L;
    fv->Hkv     = (int) Hkv;
    fv->kv_type = k->type;
    fv->dst  = (float *) dst->data;
    fv->dnb1 = (int64_t) dst->nb[1];
    fv->dnb2 = (int64_t) dst->nb[2];
    return SRHPM_OK;
}

// logits f32 [n_vocab, rows], rows contiguous in the vocabulary (nb[0] = 4), any row stride
int check_logits(const srhpm_tensor * lg, int min_rows) {
    if (!lg || lg->type != SRHPM_TYPE_F32 || !lg->data) return SRHPM_ERR_INVALID;
    if (lg->ne[0] < 1 || lg->ne[0] > INT32_MAX || lg->ne[1] < min_rows || lg->ne[2] != 1 || lg->ne[3] != 1) {
        return SRHPM_ERR_INVALID;
    }
    if (lg->nb[0] != 4 || lg->nb[1] % 4 || lg->nb[1] < (size_t) lg->ne[0] * 4 || !aligned(lg->data, 4)) {
        return SRHPM_ERR_INVALID;
    }
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
    // the status word (64 bytes), then the GEMM grids' arrival counters
    const size_t dev_bytes = 64 + (size_t) kSyncSlots * sizeof(uint32_t);
    st = cuda_status(cudaMalloc(&c->d_status, dev_bytes));
    if (st == SRHPM_OK) st = cuda_status(cudaMemset(c->d_status, 0, dev_bytes));
    if (st == SRHPM_OK) c->d_sync = reinterpret_cast<uint32_t *>(reinterpret_cast<uint8_t *>(c->d_status) + 64);
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

int srhpm_mul_mat_fused_quant(srhpm_ctx * ctx, const srhpm_tensor * W, const srhpm_tensor * X, srhpm_tensor * Y,
                              void * wdata, size_t wsize, void * stream) {
    if (!ctx || !Y) return SRHPM_ERR_INVALID;
    const int st = check_mul_mat(W, X, Y);
    if (st != SRHPM_OK) return st;
    return gemm_run(ctx, W->type, (const uint8_t *) W->data, W->ne[1], W->ne[0], W->nb[1], (const float *) X->data,
                    (int64_t) (X->nb[1] / 4), X->ne[1], (float *) Y->data, (int64_t) (Y->nb[1] / 4), wdata, wsize,
                    nullptr, nullptr, (cudaStream_t) stream, true);
}

int srhpm_mul_mat_swiglu(srhpm_ctx * ctx, const srhpm_tensor * W, const srhpm_tensor * gate, const srhpm_tensor * up,
                         srhpm_tensor * Y, void * wdata, size_t wsize, void * stream) {
    if (!ctx || !Y || !up) return SRHPM_ERR_INVALID;
    const int st = check_mul_mat(W, gate, Y);
    if (st != SRHPM_OK) return st;
    if (up->type != SRHPM_TYPE_F32 || up->ne[0] != gate->ne[0] || up->ne[1] != gate->ne[1] || up->ne[2] != 1 ||
        up->ne[3] != 1 || up->nb[0] != 4 || up->nb[1] != gate->nb[1] || !up->data) {
        return SRHPM_ERR_INVALID;
    }
    if (!aligned(up->data, 4)) return SRHPM_ERR_ALIGN;
    return gemm_run_swiglu(ctx, W->type, (const uint8_t *) W->data, W->ne[1], W->ne[0], W->nb[1],
                           (const float *) gate->data, (const float *) up->data, (int64_t) (gate->nb[1] / 4),
                           gate->ne[1], (float *) Y->data, (int64_t) (Y->nb[1] / 4), wdata, wsize,
                           (cudaStream_t) stream);
}

int srhpm_add_rms_norm_quant(srhpm_ctx * ctx, float * x, const float * delta, const float * w, float eps, float * y,
                             int n, const srhpm_tensor * W_next, void * wdata, size_t wsize, void * stream) {
    if (!ctx || !x || !w || !y || !W_next || n < 1 || n > 16) return SRHPM_ERR_INVALID;
    if ((reinterpret_cast<uintptr_t>(x) | reinterpret_cast<uintptr_t>(w) | reinterpret_cast<uintptr_t>(y) |
         reinterpret_cast<uintptr_t>(delta)) & 15) {
        return SRHPM_ERR_ALIGN;
    }
    const int64_t K = W_next->ne[0];
    if (W_next->type != SRHPM_TYPE_Q4_K && W_next->type != SRHPM_TYPE_Q5_K && W_next->type != SRHPM_TYPE_Q6_K &&
        W_next->type != SRHPM_TYPE_Q3_K && W_next->type != SRHPM_TYPE_IQ4_XS) {
        return SRHPM_UNSUPPORTED;
    }
    return norm_quant_run(ctx, W_next->type, W_next->ne[1], K, n, x, delta, w, eps, y, wdata, wsize,
                          (cudaStream_t) stream);
}

int srhpm_add_rms_norm_allreduce_quant(srhpm_ctx * ctx, float * x, const uint64_t * peer_buffers, int world,
                                       int rank, int slot, uint32_t * epochs, const float * w, float eps, float * y,
                                       int n, const srhpm_tensor * W_next, void * wdata, size_t wsize, void * stream) {
    if (!ctx || !x || !peer_buffers || !epochs || !w || !y || !W_next || n < 1 || n > 16) return SRHPM_ERR_INVALID;
    if ((reinterpret_cast<uintptr_t>(x) | reinterpret_cast<uintptr_t>(w) | reinterpret_cast<uintptr_t>(y)) & 15) {
        return SRHPM_ERR_ALIGN;
    }
    if (W_next->type != SRHPM_TYPE_Q4_K && W_next->type != SRHPM_TYPE_Q5_K && W_next->type != SRHPM_TYPE_Q6_K &&
        W_next->type != SRHPM_TYPE_Q3_K && W_next->type != SRHPM_TYPE_IQ4_XS) {
        return SRHPM_UNSUPPORTED;
    }
    return norm_quant_run(ctx, W_next->type, W_next->ne[1], W_next->ne[0], n, x, nullptr, w, eps, y, wdata, wsize,
                          (cudaStream_t) stream, peer_buffers, world, rank, slot, epochs);
}

int srhpm_swiglu_quant(srhpm_ctx * ctx, const float * gate, const float * up, int64_t ld_in, float * out,
                       int64_t ld_out, int n, const srhpm_tensor * W_next, void * wdata, size_t wsize, void * stream) {
    if (!ctx || !gate || !up || !out || !W_next || n < 1 || n > 16 || ld_in < W_next->ne[0] ||
        ld_out < W_next->ne[0]) {
        return SRHPM_ERR_INVALID;
    }
    if (W_next->type != SRHPM_TYPE_Q4_K && W_next->type != SRHPM_TYPE_Q5_K && W_next->type != SRHPM_TYPE_Q6_K &&
        W_next->type != SRHPM_TYPE_Q3_K && W_next->type != SRHPM_TYPE_IQ4_XS) {
        return SRHPM_UNSUPPORTED;
    }
    return swiglu_quant_run(ctx, W_next->type, W_next->ne[1], W_next->ne[0], n, gate, up, ld_in, out, ld_out, wdata,
                            wsize, (cudaStream_t) stream);
}

int srhpm_mul_mat_prequantized(srhpm_ctx * ctx, const srhpm_tensor * W, const srhpm_tensor * X, srhpm_tensor * Y,
                               void * wdata, size_t wsize, void * stream) {
    if (!ctx || !Y) return SRHPM_ERR_INVALID;
    const int st = check_mul_mat(W, X, Y);
    if (st != SRHPM_OK) return st;
    return gemm_run_prequant(ctx, W->type, (const uint8_t *) W->data, W->ne[1], W->ne[0], W->nb[1], X->ne[1],
                             (float *) Y->data, (int64_t) (Y->nb[1] / 4), wdata, wsize, (cudaStream_t) stream);
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

int srhpm_flash_attn_ext_work_size(const srhpm_ctx * ctx, const srhpm_tensor * q, const srhpm_tensor * k,
                                   const srhpm_tensor * v, size_t * size) {
    if (!ctx || !size || !q || !k || !v) return SRHPM_ERR_INVALID;
    FaView             fv;
    srhpm_tensor       d = {};
    d.type               = SRHPM_TYPE_F32;
    d.ne[0]              = v->ne[0];
    d.ne[1]              = q->ne[2];
    d.ne[2]              = q->ne[1];
    d.ne[3]              = 1;
    d.nb[0]              = 4;
    d.nb[1]              = 4 * (size_t) d.ne[0];
    d.nb[2]              = d.nb[1] * (size_t) d.ne[1];
    d.nb[3]              = d.nb[2] * (size_t) d.ne[2];
    d.data               = (void *) 16;  // shape check only
    const int st         = check_fa(q, k, v, nullptr, nullptr, &d, &fv);
    if (st != SRHPM_OK) return st;
    *size = fa_work_size(ctx->num_sms, (fv.H / fv.Hkv) * fv.N, fv.L, fv.Hkv);
    return SRHPM_OK;
}

int srhpm_flash_attn_ext(srhpm_ctx * ctx, const srhpm_tensor * q, const srhpm_tensor * k, const srhpm_tensor * v,
                         const srhpm_tensor * mask, const srhpm_tensor * sinks, float scale, float max_bias,
                         float softcap, srhpm_tensor * dst, void * wdata, size_t wsize, void * stream) {
    if (!ctx) return SRHPM_ERR_INVALID;
    FaView    fv;
    const int st = check_fa(q, k, v, mask, sinks, dst, &fv);
    if (st != SRHPM_OK) return st;
    return fa_run(ctx, fv, scale, max_bias, softcap, wdata, wsize, (cudaStream_t) stream);
}

size_t srhpm_flash_attn_part_size(int64_t n_head, int64_t n_tokens) {
    if (n_head < 1 || n_tokens < 1) return 0;
    return fa_part_bytes(n_head, n_tokens);
}

int srhpm_flash_attn_ext_partial(srhpm_ctx * ctx, const srhpm_tensor * q, const srhpm_tensor * k,
                                 const srhpm_tensor * v, const srhpm_tensor * mask, float scale, float max_bias,
                                 float softcap, void * part, void * wdata, size_t wsize, void * stream) {
    if (!ctx || !q || !k || !v || !part) return SRHPM_ERR_INVALID;
    if (!aligned(part, 16)) return SRHPM_ERR_ALIGN;
    if (q->type != SRHPM_TYPE_F32 || q->ne[1] < 1 || q->ne[1] > 16 || q->ne[2] < 1 || q->ne[2] > 65536) {
        return SRHPM_ERR_INVALID;
    }
    const size_t bytes = fa_part_bytes(q->ne[2], q->ne[1]);
    if (k->ne[1] == 0 && v->ne[1] == 0) {  // an empty KV range: sums 0, skipped by the merge
        return cuda_status(cudaMemsetAsync(part, 0, bytes, (cudaStream_t) stream));
    }
    srhpm_tensor d = {};  // dst is not written; its shape is checked like srhpm_flash_attn_ext's
    d.type         = SRHPM_TYPE_F32;
    d.ne[0]        = v->ne[0];
    d.ne[1]        = q->ne[2];
    d.ne[2]        = q->ne[1];
    d.ne[3]        = 1;
    d.nb[0]        = 4;
    d.nb[1]        = 4 * (size_t) d.ne[0];
    d.nb[2]        = d.nb[1] * (size_t) d.ne[1];
    d.nb[3]        = d.nb[2] * (size_t) d.ne[2];
    d.data         = part;
    FaView    fv;
    const int st = check_fa(q, k, v, mask, nullptr, &d, &fv);
    if (st != SRHPM_OK) return st;
    return fa_run(ctx, fv, scale, max_bias, softcap, wdata, wsize, (cudaStream_t) stream, part);
}

int srhpm_flash_attn_merge(srhpm_ctx * ctx, const void * parts, int n_parts, const srhpm_tensor * sinks,
                           srhpm_tensor * dst, void * stream) {
    if (!ctx || !parts || !dst || n_parts < 1 || n_parts > 256) return SRHPM_ERR_INVALID;
    if (!aligned(parts, 16)) return SRHPM_ERR_ALIGN;
    if (dst->type != SRHPM_TYPE_F32 || !dst->data || dst->ne[0] != 256 || dst->ne[1] < 1 || dst->ne[1] > 65536 ||
        dst->ne[2] < 1 || dst->ne[2] > 16 || dst->ne[3] != 1) {
        return SRHPM_ERR_INVALID;
    }
    if (dst->nb[0] != 4 || dst->nb[1] % 4 || dst->nb[2] % 4 || !aligned(dst->data, 4)) return SRHPM_ERR_INVALID;
    const int H = (int) dst->ne[1], N = (int) dst->ne[2];
    const float * sk = nullptr;
    if (sinks) {
        if (sinks->type != SRHPM_TYPE_F32 || sinks->ne[0] != H || sinks->nb[0] != 4 || !sinks->data) {
            return SRHPM_ERR_INVALID;
        }
        sk = (const float *) sinks->data;
    }
    return fa_merge_run(ctx, parts, n_parts, N, H, sk, (float *) dst->data, (int64_t) dst->nb[1],
                        (int64_t) dst->nb[2], (cudaStream_t) stream);
}

size_t srhpm_flash_attn_peer_buffer_size(int64_t n_head, int64_t n_tokens) {
    if (n_head < 1 || n_tokens < 1) return 0;
    return fa_peer_buffer_bytes(n_head, n_tokens);
}

int srhpm_flash_attn_merge_peers(srhpm_ctx * ctx, const uint64_t * peer_buffers, int world, int rank,
                                 uint32_t * epochs, const srhpm_tensor * sinks, srhpm_tensor * dst, void * stream) {
    if (!ctx || !peer_buffers || !epochs || !dst) return SRHPM_ERR_INVALID;
    if (dst->type != SRHPM_TYPE_F32 || !dst->data || dst->ne[0] != 256 || dst->ne[1] < 1 || dst->ne[1] > 65536 ||
        dst->ne[2] < 1 || dst->ne[2] > 16 || dst->ne[3] != 1) {
        return SRHPM_ERR_INVALID;
    }
    if (dst->nb[0] != 4 || dst->nb[1] % 4 || dst->nb[2] % 4 || !aligned(dst->data, 4)) return SRHPM_ERR_INVALID;
    const int H = (int) dst->ne[1], N = (int) dst->ne[2];
    const float * sk = nullptr;
    if (sinks) {
        if (sinks->type != SRHPM_TYPE_F32 || sinks->ne[0] != H || sinks->nb[0] != 4 || !sinks->data) {
            return SRHPM_ERR_INVALID;
        }
        sk = (const float *) sinks->data;
    }
    return fa_merge_peers_run(ctx, peer_buffers, world, rank, epochs, N, H, sk, (float *) dst->data,
                              (int64_t) dst->nb[1], (int64_t) dst->nb[2], (cudaStream_t) stream);
}

int srhpm_verify_accept_work_size(const srhpm_ctx * ctx, const srhpm_tensor * logits, size_t * size) {
    if (!ctx || !size) return SRHPM_ERR_INVALID;
    const int st = check_logits(logits, 1);
    if (st != SRHPM_OK) return st;
    if (logits->ne[1] > 17) return SRHPM_UNSUPPORTED;
    *size = argmax_work_size(ctx->num_sms, (int) logits->ne[0], (int) logits->ne[1]);
    return SRHPM_OK;
}

int srhpm_verify_accept(srhpm_ctx * ctx, const srhpm_tensor * logits, const int32_t * draft, int n_draft, float relax,
                        int32_t * out_ids, int32_t * out_n, void * wdata, size_t wsize, void * stream) {
    if (!ctx || !out_ids || !out_n || n_draft < 0 || (n_draft > 0 && !draft)) return SRHPM_ERR_INVALID;
    if (n_draft > 16) return SRHPM_UNSUPPORTED;
    const int st = check_logits(logits, n_draft + 1);
    if (st != SRHPM_OK) return st;
    return accept_run(ctx, (const uint8_t *) logits->data, (int64_t) logits->nb[1], (int) logits->ne[0], n_draft + 1,
                      draft, n_draft, relax, out_ids, out_n, 0, nullptr, wdata, wsize, (cudaStream_t) stream);
}

int srhpm_argmax_shard(srhpm_ctx * ctx, const srhpm_tensor * logits, int64_t vocab_offset, const int32_t * draft,
                       int n_draft, srhpm_argmax_record * out, void * wdata, size_t wsize, void * stream) {
    if (!ctx || !out || vocab_offset < 0 || n_draft < 0 || (n_draft > 0 && !draft)) return SRHPM_ERR_INVALID;
    const int st = check_logits(logits, 1);
    if (st != SRHPM_OK) return st;
    if (logits->ne[1] > 17 || n_draft > 16) return SRHPM_UNSUPPORTED;
    return accept_run(ctx, (const uint8_t *) logits->data, (int64_t) logits->nb[1], (int) logits->ne[0],
                      (int) logits->ne[1], draft, n_draft, 0.0f, nullptr, nullptr, vocab_offset, out, wdata, wsize,
                      (cudaStream_t) stream);
}

int srhpm_accept_merge(srhpm_ctx * ctx, const srhpm_argmax_record * recs, int n_shards, int n_rows,
                       const int32_t * draft, int n_draft, float relax, int32_t * out_ids, int32_t * out_n,
                       void * stream) {
    if (!ctx || !recs || !out_ids || !out_n || n_shards < 1 || n_draft < 0 || n_rows < n_draft + 1) {
        return SRHPM_ERR_INVALID;
    }
    if (n_draft > 0 && !draft) return SRHPM_ERR_INVALID;
    if (n_rows > 17) return SRHPM_UNSUPPORTED;
    return accept_merge_run(ctx, recs, n_shards, n_rows, draft, n_draft, relax, out_ids, out_n, (cudaStream_t) stream);
}

int srhpm_get_rows(srhpm_ctx * ctx, const srhpm_tensor * table, const int32_t * ids, int n, float * out, void * stream) {
    if (!ctx || !table || !table->data || !ids || !out || n < 1 || n > 16) return SRHPM_ERR_INVALID;
    if (table->type != SRHPM_TYPE_F16 && table->type != SRHPM_TYPE_F32) return SRHPM_UNSUPPORTED;
    if (table->nb[0] != srhpm_type_size(table->type) || table->ne[0] < 1) return SRHPM_ERR_INVALID;
    return get_rows_run(ctx, (const uint8_t *) table->data, (int64_t) table->nb[1], table->type == SRHPM_TYPE_F16, ids,
                        n, table->ne[0], out, (cudaStream_t) stream);
}

int srhpm_add_rms_norm(srhpm_ctx * ctx, float * x, const float * delta, const float * w, float eps, float * y, int n,
                       int64_t d, void * stream) {
    if (!ctx || !x || !w || !y || n < 1 || n > 16 || d < 1) return SRHPM_ERR_INVALID;
    return add_rms_norm_run(ctx, x, delta, w, eps, y, n, d, (cudaStream_t) stream);
}

size_t srhpm_allreduce_buffer_size(int64_t d) { return d > 0 ? allreduce_buffer_bytes(d) : 0; }

int srhpm_add_rms_norm_allreduce(srhpm_ctx * ctx, float * x, const uint64_t * peer_buffers, int world, int rank,
                                 int slot, uint32_t * epochs, const float * w, float eps, float * y, int n, int64_t d,
                                 void * stream) {
    if (!ctx || !x || !peer_buffers || !epochs || !w || !y || d < 1) return SRHPM_ERR_INVALID;
    if ((reinterpret_cast<uintptr_t>(x) | reinterpret_cast<uintptr_t>(w) | reinterpret_cast<uintptr_t>(y)) & 15) {
        return SRHPM_ERR_ALIGN;
    }
    return add_rms_norm_ar_run(ctx, x, peer_buffers, world, rank, slot, epochs, w, eps, y, n, d,
                               (cudaStream_t) stream);
}

int srhpm_rope_kv(srhpm_ctx * ctx, float * qkv, int64_t ld, int n, int n_head, int n_head_kv, int head_dim,
                  const int32_t * pos, float theta_base, const srhpm_tensor * k_cache, const srhpm_tensor * v_cache,
                  void * stream) {
    if (!ctx || !qkv || !pos || !k_cache || !v_cache || n < 1 || n > 16 || n_head < 1 || n_head_kv < 1) {
        return SRHPM_ERR_INVALID;
    }
    if (head_dim != 256 || ld < (int64_t) (n_head + 2 * n_head_kv) * head_dim) return SRHPM_ERR_INVALID;
    if (k_cache->type != v_cache->type || (k_cache->type != SRHPM_TYPE_F16 && k_cache->type != SRHPM_TYPE_Q8_0)) {
        return SRHPM_UNSUPPORTED;
    }
    if (k_cache->ne[0] != head_dim || v_cache->ne[0] != head_dim || k_cache->ne[2] != n_head_kv ||
        v_cache->ne[2] != n_head_kv || !k_cache->data || !v_cache->data) {
        return SRHPM_ERR_INVALID;
    }
    return rope_kv_run(ctx, qkv, ld, n, n_head, n_head_kv, head_dim, pos, theta_base, (uint8_t *) k_cache->data,
                       (int64_t) k_cache->nb[1], (int64_t) k_cache->nb[2], (uint8_t *) v_cache->data,
                       (int64_t) v_cache->nb[1], (int64_t) v_cache->nb[2], k_cache->type, (cudaStream_t) stream);
}

int srhpm_swiglu(srhpm_ctx * ctx, const float * gate, const float * up, int64_t ld_in, float * out, int64_t ld_out,
                 int n, int64_t n_ff, void * stream) {
    if (!ctx || !gate || !up || !out || n < 1 || n > 16 || n_ff < 1 || ld_in < n_ff || ld_out < n_ff) {
        return SRHPM_ERR_INVALID;
    }
    return swiglu_run(ctx, gate, up, ld_in, out, ld_out, n, n_ff, (cudaStream_t) stream);
}

}  // extern "C"
