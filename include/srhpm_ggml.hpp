// srhpm_ggml: the reference's C++ operator interface for the verify path, on the B200 kernels of srhpm_b200.h.
//
// SR-HPM plugs its kernels into ggml-cpu as an extra buffer type whose tensor_traits (tensor_traits_srv,
// patch/srhpm.patch:6363-6632) take over ggml_mul_mat for the weights srv_traits_for selects (:6634-6676). The
// grouped attention path is a pair of functions behind a gate inside ggml_compute_forward_flash_attn_ext
// (:555-824, gate :833-841), and acceptance is upstream's common_sampler_sample_and_accept_n. This header keeps those
// names, argument meanings and error behaviour on a device backend:
//   - tensor_traits::work_size / compute_forward return false where the reference does ("use the stock path": not a
//     MUL_MAT, more than SRV_MAXM activation rows) and for shapes the kernels do not take; a violated GGML_ASSERT of
//     the reference (activations not f32, 3-D operands, a padded weight row) aborts here too; a CUDA or kernel error,
//     which has no counterpart on the CPU, aborts with its status;
//   - tensor data are device pointers; params->wdata is a device buffer of work_size bytes; only thread 0 (ith == 0)
//     launches, on the backend's stream, and the call returns without waiting (ggml backends synchronise per graph);
//   - repack copies the native GGUF rows to the device (the reference's memcpy, :6613-6621) and waits for the copy.
// The structures below mirror the ggml fields this path reads (same names and meanings; the op numbering is this
// header's). Everything goes through the C ABI of srhpm_b200.h.
#ifndef SRHPM_GGML_HPP
#define SRHPM_GGML_HPP

#include <cstddef>
#include <cstdint>
#include <vector>

#include "srhpm_b200.h"

namespace srhpm::ggml {

// ggml_type ids (GGUF numbering) of the tensors on this path
enum ggml_type : int32_t {
    GGML_TYPE_F32    = 0,
    GGML_TYPE_F16    = 1,
    GGML_TYPE_Q8_0   = 8,
    GGML_TYPE_Q3_K   = 11,
    GGML_TYPE_Q4_K   = 12,
    GGML_TYPE_Q5_K   = 13,
    GGML_TYPE_Q6_K   = 14,
    GGML_TYPE_IQ4_XS = 23,
    GGML_TYPE_I32    = 26,
};

// the operators of this path
enum ggml_op : int32_t {
    GGML_OP_NONE = 0,
    GGML_OP_MUL_MAT,
    GGML_OP_FLASH_ATTN_EXT,
};

constexpr int     GGML_MAX_DIMS      = 4;
constexpr int     GGML_MAX_SRC       = 10;
constexpr int     GGML_MAX_OP_PARAMS = 64;
constexpr int     GGML_MAX_NAME      = 64;
constexpr int64_t QK_K               = 256;
constexpr int64_t SRV_MAXM           = 16;  // activation rows the SRV path takes (patch/srhpm.patch:5466)

struct ggml_tensor {
    ggml_type     type                                          = GGML_TYPE_F32;
    int64_t       ne[GGML_MAX_DIMS]                             = { 1, 1, 1, 1 };  // elements, ne[0] innermost
    size_t        nb[GGML_MAX_DIMS]                             = { 0, 0, 0, 0 };  // bytes per step
    ggml_op       op                                            = GGML_OP_NONE;
    int32_t       op_params[GGML_MAX_OP_PARAMS / sizeof(int32_t)] = {};
    ggml_tensor * src[GGML_MAX_SRC]                             = {};
    void *        data                                          = nullptr;  // device memory
    char          name[GGML_MAX_NAME]                           = {};
};

// the fields of ggml_compute_params a tensor_traits reads
struct ggml_compute_params {
    int    ith   = 0;  // thread index: thread 0 launches, the others return at once
    int    nth   = 1;
    size_t wsize = 0;  // device work buffer
    void * wdata = nullptr;
};

int64_t ggml_nrows(const ggml_tensor * t);   // ne[1] * ne[2] * ne[3]
size_t  ggml_nbytes(const ggml_tensor * t);
// a contiguous tensor of `type` over `data` (nb from the type's block size, as ggml_new_tensor lays it out)
ggml_tensor ggml_tensor_view(ggml_type type, int64_t ne0, int64_t ne1, int64_t ne2, int64_t ne3, void * data);

// ggml::cpu::tensor_traits
class tensor_traits {
  public:
    virtual ~tensor_traits() = default;
    virtual bool work_size(int n_threads, const ggml_tensor * op, size_t & size)  = 0;
    virtual bool compute_forward(ggml_compute_params * params, ggml_tensor * op)  = 0;
    virtual int  repack(ggml_tensor * t, const void * data, size_t data_size)     = 0;
};

// One device of the backend: its context and the stream every call is ordered on.
struct backend {
    srhpm_ctx * ctx    = nullptr;
    void *      stream = nullptr;  // cudaStream_t; nullptr = the legacy default stream
};

// tensor_traits_srv for every SRV weight type at once (the type is read from src[0] at each call):
// op = ggml_mul_mat(src[0] = W [K, rows], src[1] = X f32 [K, M]) -> f32 [rows, M], M <= SRV_MAXM.
class tensor_traits_srv_b200 final : public tensor_traits {
  public:
    explicit tensor_traits_srv_b200(const backend * be) : be_(be) {}
    // patch/srhpm.patch:6366-6374: false for another op or M > SRV_MAXM; else the device work bytes
    bool work_size(int n_threads, const ggml_tensor * op, size_t & size) override;
    // patch/srhpm.patch:6400-6611: false for another op, M > SRV_MAXM or a shape the kernels do not take
    bool compute_forward(ggml_compute_params * params, ggml_tensor * op) override;
    // patch/srhpm.patch:6613-6621: the native rows, copied to t->data on the device (on the backend's stream,
    // complete on return); 0, or -1 when the copy failed
    int  repack(ggml_tensor * t, const void * data, size_t data_size) override;

  private:
    const backend * be_;
};

// The extra buffer type of the device: selects the traits of weight tensors (ggml::cpu::extra_buffer_type).
class extra_buffer_type_b200 {
  public:
    explicit extra_buffer_type_b200(backend be) : be_(be), srv_(&be_) {}
    extra_buffer_type_b200(const extra_buffer_type_b200 &)             = delete;  // srv_ points at be_
    extra_buffer_type_b200 & operator=(const extra_buffer_type_b200 &) = delete;
    // srv_traits_for (patch/srhpm.patch:6634-6676): the traits of weight `cur`, or nullptr. Takes 2-D weights with
    // ne[0] a multiple of 256 of type Q3_K, Q4_K, Q5_K, Q6_K, IQ4_XS, and Q8_0 (which the reference leaves to ggml's
    // stock mul_mat; a device backend has no stock path, so the same traits run the stock algorithm). The reference's
    // GGML_SRV_TYPES=<type>,<type>... restricts the types as there; its GGML_SRV=1 opt-in is the CPU's and does not
    // apply to a device backend.
    tensor_traits * srv_traits_for(const ggml_tensor * cur);
    // supports_op: a MUL_MAT whose weight srv_traits_for takes, with f32 activations of at most SRV_MAXM rows
    bool            supports_op(const ggml_tensor * op);
    // get_tensor_traits: the weight's traits for a supported op, else nullptr
    tensor_traits * get_tensor_traits(const ggml_tensor * op);
    const backend & device() const { return be_; }

  private:
    backend                be_;
    tensor_traits_srv_b200 srv_;
};

// ggml_fa_gqa_small_work_size (patch/srhpm.patch:563-579): the device work bytes of the grouped attention path for
// op = ggml_flash_attn_ext(q = src[0], k = src[1], v = src[2], mask = src[3], sinks = src[4]), or 0 when the path
// does not take it (then ggml's stock path runs). A taken op reports at least 256 bytes, so 0 keeps that meaning.
// The path takes f32 q [256, N, H] with 1 <= N <= 16, q8_0 or f16 k / v [256, L, Hkv] with H a multiple of Hkv,
// an f16 mask or none, f32 sinks or none (the reference's gate, :833-841, takes 2 <= N <= 8 and L >= one tile).
size_t fa_gqa_small_work_size(const backend & be, const ggml_tensor * op, int n_threads);
// ggml_compute_forward_flash_attn_ext_gqa_small behind its gate (patch/srhpm.patch:581-824, :833-841):
// op_params = (scale, max_bias, softcap) as floats (:607-613); dst f32 [256, H, N]. false when the gate refuses
// (the op is not taken, or params->wsize < fa_gqa_small_work_size).
bool   compute_forward_flash_attn_ext_gqa_small(const backend & be, const ggml_compute_params * params,
                                                ggml_tensor * dst);

// common_sampler_sample_and_accept_n with a greedy sampler (upstream) and the reference's relaxed acceptance
// (patch/srhpm.patch:9-35), over device logits f32 [n_vocab, >= n_draft + 1]: returns the emitted ids (the accepted
// drafted tokens and the one after them; n_rollback = draft.size() + 1 - ids.size()). Synchronous on the backend's
// stream; the device buffers are allocated once, for n_vocab and up to 16 drafted tokens.
class common_sampler_b200 {
  public:
    common_sampler_b200(const backend & be, int64_t n_vocab);
    ~common_sampler_b200();
    common_sampler_b200(const common_sampler_b200 &)             = delete;
    common_sampler_b200 & operator=(const common_sampler_b200 &) = delete;
    std::vector<int32_t> sample_and_accept_n(const ggml_tensor * logits, const std::vector<int32_t> & draft,
                                             float relax = 0.0f);

  private:
    backend   be_;
    int64_t   n_vocab_;
    size_t    wsize_ = 0;
    void *    work_  = nullptr;
    int32_t * draft_ = nullptr;  // [16]
    int32_t * ids_   = nullptr;  // [17]
    int32_t * n_     = nullptr;  // [1]
};

}  // namespace srhpm::ggml

#endif
