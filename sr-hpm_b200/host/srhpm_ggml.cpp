// The reference's C++ operator interface for the verify path (tensor_traits_srv, srv_traits_for, the grouped
// flash-attention entry points, greedy acceptance) over the C ABI of srhpm_b200.h. See include/srhpm_ggml.hpp.
#include "srhpm_ggml.hpp"

#include <cuda_runtime_api.h>

#include <algorithm>
#include <cstdio>
#include <cstdlib>
#include <cstring>
#include <string>

namespace srhpm::ggml {
namespace {

// GGML_ASSERT / GGML_ABORT: print where and why, then abort (ggml's behaviour for a violated precondition)
[[noreturn]] void ggml_abort(const char * file, int line, const char * what) {
    fflush(stdout);
    fprintf(stderr, "%s:%d: %s\n", file, line, what);
    fflush(stderr);
    abort();
}

#define SRHPM_GGML_ASSERT(x)                                         \
    do {                                                             \
        if (!(x)) ggml_abort(__FILE__, __LINE__, "GGML_ASSERT(" #x ") failed"); \
    } while (0)

// a failed device call: no CPU counterpart, no error channel in the interface
void check_status(int st, const char * what, const char * file, int line) {
    if (st == SRHPM_OK) return;
    char msg[256];
    snprintf(msg, sizeof msg, "%s failed: %s (CUDA error %d)", what, srhpm_status_str(st), srhpm_last_cuda_error());
    ggml_abort(file, line, msg);
}

#define SRHPM_CHECK(call, what) check_status((call), (what), __FILE__, __LINE__)

void check_cuda(cudaError_t e, const char * what, const char * file, int line) {
    if (e == cudaSuccess) return;
    char msg[256];
    snprintf(msg, sizeof msg, "%s failed: %s", what, cudaGetErrorString(e));
    ggml_abort(file, line, msg);
}

#define SRHPM_CUDA(call) check_cuda((call), #call, __FILE__, __LINE__)

srhpm_tensor to_view(const ggml_tensor * t) {
    srhpm_tensor v = {};
    v.type         = t->type;
    for (int i = 0; i < GGML_MAX_DIMS; i++) {
        v.ne[i] = t->ne[i];
        v.nb[i] = t->nb[i];
    }
    v.data = t->data;
    return v;
}

const char * type_name(ggml_type t) {  // ggml_type_name
    switch (t) {
        case GGML_TYPE_F32: return "f32";
        case GGML_TYPE_F16: return "f16";
        case GGML_TYPE_Q8_0: return "q8_0";
        case GGML_TYPE_Q3_K: return "q3_K";
        case GGML_TYPE_Q4_K: return "q4_K";
        case GGML_TYPE_Q5_K: return "q5_K";
        case GGML_TYPE_Q6_K: return "q6_K";
        case GGML_TYPE_IQ4_XS: return "iq4_xs";
        case GGML_TYPE_I32: return "i32";
    }
    return "?";
}

bool is_srv_type(ggml_type t) {
    switch (t) {
        case GGML_TYPE_Q3_K:
        case GGML_TYPE_Q4_K:
        case GGML_TYPE_Q5_K:
        case GGML_TYPE_Q6_K:
        case GGML_TYPE_IQ4_XS:
        case GGML_TYPE_Q8_0: return true;
        default: return false;
    }
}

}  // namespace

int64_t ggml_nrows(const ggml_tensor * t) { return t->ne[1] * t->ne[2] * t->ne[3]; }

size_t ggml_nbytes(const ggml_tensor * t) {
    const int blck = srhpm_blck_size(t->type);
    if (blck <= 0) return 0;
    size_t n = (size_t) t->ne[0] * t->nb[0] / (size_t) blck;
    for (int i = 1; i < GGML_MAX_DIMS; i++) n += (size_t) (t->ne[i] - 1) * t->nb[i];
    return n;
}

ggml_tensor ggml_tensor_view(ggml_type type, int64_t ne0, int64_t ne1, int64_t ne2, int64_t ne3, void * data) {
    ggml_tensor t;
    t.type  = type;
    t.ne[0] = ne0;
    t.ne[1] = ne1;
    t.ne[2] = ne2;
    t.ne[3] = ne3;
    t.nb[0] = srhpm_type_size(type);
    t.nb[1] = srhpm_row_size(type, ne0);
    t.nb[2] = t.nb[1] * (size_t) ne1;
    t.nb[3] = t.nb[2] * (size_t) ne2;
    t.data  = data;
    return t;
}

// ---- tensor_traits_srv -------------------------------------------------------------------------------------------

bool tensor_traits_srv_b200::work_size(int /* n_threads */, const ggml_tensor * op, size_t & size) {
    if (op->op != GGML_OP_MUL_MAT || ggml_nrows(op->src[1]) > SRV_MAXM) {
        return false;
    }
    const srhpm_tensor W = to_view(op->src[0]), X = to_view(op->src[1]);
    size_t             s = 0;
    if (srhpm_mul_mat_work_size(&W, &X, &s) != SRHPM_OK) {
        return false;
    }
    size = s;
    return true;
}

bool tensor_traits_srv_b200::compute_forward(ggml_compute_params * params, ggml_tensor * op) {
    if (op->op != GGML_OP_MUL_MAT || ggml_nrows(op->src[1]) > SRV_MAXM) {
        return false;  // large batches: stock path
    }
    const ggml_tensor * src0 = op->src[0];
    const ggml_tensor * src1 = op->src[1];
    SRHPM_GGML_ASSERT(src1->type == GGML_TYPE_F32);
    SRHPM_GGML_ASSERT(src1->ne[2] == 1 && src1->ne[3] == 1 && op->ne[2] == 1 && op->ne[3] == 1);
    SRHPM_GGML_ASSERT(src0->nb[1] == srhpm_row_size(src0->type, src0->ne[0]));
    srhpm_tensor W = to_view(src0), X = to_view(src1), Y = to_view(op);
    size_t       need = 0;
    // every thread answers alike: shapes the kernels do not take go to the stock path on all of them
    if (srhpm_mul_mat_work_size(&W, &X, &need) == SRHPM_UNSUPPORTED) {
        return false;
    }
    if (params->ith != 0) {
        return true;
    }
    SRHPM_GGML_ASSERT(be_ != nullptr && be_->ctx != nullptr);
    const int st = srhpm_mul_mat(be_->ctx, &W, &X, &Y, params->wdata, params->wsize, be_->stream);
    if (st == SRHPM_UNSUPPORTED) {
        return false;
    }
    SRHPM_CHECK(st, "srhpm_mul_mat");
    return true;
}

int tensor_traits_srv_b200::repack(ggml_tensor * t, const void * data, size_t data_size) {
    if (t == nullptr || t->data == nullptr || (data_size > 0 && data == nullptr)) {
        return -1;
    }
    // ordered on the backend's stream and complete on return: a copy from pageable memory may otherwise still be in
    // flight when a kernel on another stream reads the rows
    cudaStream_t s = be_ ? static_cast<cudaStream_t>(be_->stream) : nullptr;
    if (cudaMemcpyAsync(t->data, data, data_size, cudaMemcpyHostToDevice, s) != cudaSuccess) {
        return -1;
    }
    return cudaStreamSynchronize(s) == cudaSuccess ? 0 : -1;
}

// ---- extra buffer type ---------------------------------------------------------------------------------------------

tensor_traits * extra_buffer_type_b200::srv_traits_for(const ggml_tensor * cur) {
    if (cur == nullptr || cur->ne[0] % QK_K != 0 || cur->ne[2] != 1 || cur->ne[3] != 1) {
        return nullptr;
    }
    static const std::string srv_types = [] {
        const char * e = getenv("GGML_SRV_TYPES");
        return std::string(e ? e : "");
    }();
    if (!srv_types.empty() &&
        ("," + srv_types + ",").find("," + std::string(type_name(cur->type)) + ",") == std::string::npos) {
        return nullptr;
    }
    return is_srv_type(cur->type) ? &srv_ : nullptr;
}

bool extra_buffer_type_b200::supports_op(const ggml_tensor * op) {
    if (op == nullptr || op->op != GGML_OP_MUL_MAT || op->src[0] == nullptr || op->src[1] == nullptr) {
        return false;
    }
    const ggml_tensor * src1 = op->src[1];
    return srv_traits_for(op->src[0]) != nullptr && src1->type == GGML_TYPE_F32 && src1->ne[2] == 1 &&
           src1->ne[3] == 1 && ggml_nrows(src1) <= SRV_MAXM;
}

tensor_traits * extra_buffer_type_b200::get_tensor_traits(const ggml_tensor * op) {
    return supports_op(op) ? srv_traits_for(op->src[0]) : nullptr;
}

// ---- grouped flash attention ---------------------------------------------------------------------------------------

size_t fa_gqa_small_work_size(const backend & be, const ggml_tensor * op, int /* n_threads */) {
    if (op == nullptr || op->op != GGML_OP_FLASH_ATTN_EXT || be.ctx == nullptr) {
        return 0;
    }
    if (op->src[0] == nullptr || op->src[1] == nullptr || op->src[2] == nullptr) {
        return 0;
    }
    const srhpm_tensor q = to_view(op->src[0]), k = to_view(op->src[1]), v = to_view(op->src[2]);
    size_t             s = 0;
    if (srhpm_flash_attn_ext_work_size(be.ctx, &q, &k, &v, &s) != SRHPM_OK) {
        return 0;
    }
    return std::max<size_t>(s, 256);
}

bool compute_forward_flash_attn_ext_gqa_small(const backend & be, const ggml_compute_params * params,
                                              ggml_tensor * dst) {
    const size_t need = fa_gqa_small_work_size(be, dst, params->nth);
    if (need == 0 || params->wsize < need) {
        return false;
    }
    if (params->ith != 0) {
        return true;
    }
    float scale = 1.0f, max_bias = 0.0f, softcap = 0.0f;
    memcpy(&scale, (const float *) dst->op_params + 0, sizeof(float));
    memcpy(&max_bias, (const float *) dst->op_params + 1, sizeof(float));
    memcpy(&softcap, (const float *) dst->op_params + 2, sizeof(float));
    const srhpm_tensor q = to_view(dst->src[0]), k = to_view(dst->src[1]), v = to_view(dst->src[2]);
    srhpm_tensor       m = {}, s = {}, d = to_view(dst);
    if (dst->src[3]) m = to_view(dst->src[3]);
    if (dst->src[4]) s = to_view(dst->src[4]);
    const int st = srhpm_flash_attn_ext(be.ctx, &q, &k, &v, dst->src[3] ? &m : nullptr, dst->src[4] ? &s : nullptr,
                                        scale, max_bias, softcap, &d, params->wdata, params->wsize, be.stream);
    SRHPM_CHECK(st, "srhpm_flash_attn_ext");
    return true;
}

// ---- greedy acceptance ---------------------------------------------------------------------------------------------

common_sampler_b200::common_sampler_b200(const backend & be, int64_t n_vocab) : be_(be), n_vocab_(n_vocab) {
    SRHPM_GGML_ASSERT(be.ctx != nullptr && n_vocab > 0);
    // the work buffer of the largest call: 17 rows (16 drafted tokens + 1)
    ggml_tensor        lg = ggml_tensor_view(GGML_TYPE_F32, n_vocab, 17, 1, 1, reinterpret_cast<void *>(256));
    const srhpm_tensor v  = to_view(&lg);
    size_t             ws = 0;
    SRHPM_CHECK(srhpm_verify_accept_work_size(be.ctx, &v, &ws), "srhpm_verify_accept_work_size");
    wsize_ = std::max<size_t>(ws, 256);
    SRHPM_CUDA(cudaMalloc(&work_, wsize_));
    SRHPM_CUDA(cudaMalloc(reinterpret_cast<void **>(&draft_), 16 * sizeof(int32_t)));
    SRHPM_CUDA(cudaMalloc(reinterpret_cast<void **>(&ids_), 17 * sizeof(int32_t)));
    SRHPM_CUDA(cudaMalloc(reinterpret_cast<void **>(&n_), sizeof(int32_t)));
}

common_sampler_b200::~common_sampler_b200() {
    cudaFree(work_);
    cudaFree(draft_);
    cudaFree(ids_);
    cudaFree(n_);
}

std::vector<int32_t> common_sampler_b200::sample_and_accept_n(const ggml_tensor * logits,
                                                              const std::vector<int32_t> & draft, float relax) {
    const int nd = (int) draft.size();
    SRHPM_GGML_ASSERT(nd <= 16);
    SRHPM_GGML_ASSERT(logits != nullptr && logits->type == GGML_TYPE_F32 && logits->ne[0] == n_vocab_);
    SRHPM_GGML_ASSERT(logits->ne[1] >= nd + 1);
    cudaStream_t s = static_cast<cudaStream_t>(be_.stream);
    if (nd > 0) {
        SRHPM_CUDA(cudaMemcpyAsync(draft_, draft.data(), nd * sizeof(int32_t), cudaMemcpyHostToDevice, s));
    }
    const srhpm_tensor v = to_view(logits);
    SRHPM_CHECK(srhpm_verify_accept(be_.ctx, &v, draft_, nd, relax, ids_, n_, work_, wsize_, be_.stream),
                "srhpm_verify_accept");
    int32_t host[17] = {};
    int32_t n        = 0;
    SRHPM_CUDA(cudaMemcpyAsync(host, ids_, sizeof host, cudaMemcpyDeviceToHost, s));
    SRHPM_CUDA(cudaMemcpyAsync(&n, n_, sizeof n, cudaMemcpyDeviceToHost, s));
    SRHPM_CUDA(cudaStreamSynchronize(s));
    SRHPM_GGML_ASSERT(n >= 1 && n <= nd + 1);
    return std::vector<int32_t>(host, host + n);
}

}  // namespace srhpm::ggml
