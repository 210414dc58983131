// Internal declarations shared by the CUDA translation units of libsrhpm_b200 (not part of the C ABI).
#pragma once
#include <cuda_runtime.h>

#include <atomic>
#include <cstdint>
#include <mutex>
#include <unordered_map>

#include "srhpm_b200.h"

struct srhpm_ctx {
    int                  device        = 0;
    int                  q8_0_act_mode = SRHPM_Q8_0_ACT_SIMD;
    int                  num_sms       = 148;
    int32_t *            d_status      = nullptr;  // device status word of the bounded waits
    std::atomic<int64_t> launches{ 0 };
    // arrival counters of the GEMM grids that quantize their own activations (srhpm_mul_mat_fused_quant), one per work
    // buffer in use: kSyncSlots words after the status word, zero at creation; a launch adds exactly 2^20 to its counter
    uint32_t *                            d_sync      = nullptr;
    std::mutex                            sync_mu;
    std::unordered_map<uintptr_t, int>    sync_slots;  // work buffer (aligned base) -> counter index
    int                                   sync_next = 0;
};

namespace srhpm {

constexpr int kSyncSlots = 4096;

void set_last_cuda_error(cudaError_t e);

inline int cuda_status(cudaError_t e) {
    if (e != cudaSuccess) {
        set_last_cuda_error(e);
        return SRHPM_ERR_CUDA;
    }
    return SRHPM_OK;
}

// shape / type facts
bool is_weight_type(int type);
int  weight_block_bytes(int type);

// srv_gemm.cu
size_t gemm_work_size(int wtype, int64_t rows, int64_t K, int64_t N);
// fused_quant: the GEMM grid quantizes its own activations (srhpm_mul_mat_fused_quant)
int    gemm_run(srhpm_ctx * ctx, int wtype, const uint8_t * W, int64_t rows, int64_t K, size_t row_bytes,
                const float * X, int64_t ldx, int64_t N, float * Y, int64_t ldy, void * wdata, size_t wsize,
                int32_t * isum, int32_t * imin, cudaStream_t stream, bool fused_quant = false);
// the product with silu(gate) * up (rows of ld_in floats) as activations, quantized in the GEMM's own prologue (or by
// the SwiGLU record kernel when the grid is too small); the SwiGLU output itself is not stored
int    gemm_run_swiglu(srhpm_ctx * ctx, int wtype, const uint8_t * W, int64_t rows, int64_t K, size_t row_bytes,
                       const float * gate, const float * up, int64_t ld_in, int64_t N, float * Y, int64_t ldy,
                       void * wdata, size_t wsize, cudaStream_t stream);
size_t gemm_work_size_unsplit(int wtype, int64_t rows, int64_t K, int64_t N);
int    gemm_run_prequant(srhpm_ctx * ctx, int wtype, const uint8_t * W, int64_t rows, int64_t K, size_t row_bytes,
                         int64_t N, float * Y, int64_t ldy, void * wdata, size_t wsize, cudaStream_t stream);
// peers != null: the delta is the all-reduce of the ranks' partial rows (srhpm_add_rms_norm_allreduce_quant)
int    norm_quant_run(srhpm_ctx * ctx, int wtype, int64_t rows, int64_t K, int64_t N, float * x, const float * delta,
                      const float * w, float eps, float * y, void * wdata, size_t wsize, cudaStream_t stream,
                      const uint64_t * peers = nullptr, int world = 1, int rank = 0, int slot = 0,
                      uint32_t * epochs = nullptr);
int    swiglu_quant_run(srhpm_ctx * ctx, int wtype, int64_t rows, int64_t K, int64_t N, const float * gate,
                        const float * up, int64_t ld_in, float * h, int64_t ld_out, void * wdata, size_t wsize,
                        cudaStream_t stream);
int    gemm_run_unsplit(srhpm_ctx * ctx, int wtype, const uint8_t * W, int64_t rows, int64_t K, size_t row_bytes,
                        const float * X, int64_t ldx, int64_t N, float * Y, int64_t ldy, void * wdata, size_t wsize,
                        cudaStream_t stream);
int    quantize_q8K_dense(srhpm_ctx * ctx, const float * X, int64_t ldx, int64_t N, int64_t K, int8_t * q, float * d,
                          int16_t * b32, int16_t * b16, cudaStream_t stream);
int    quantize_q8_0_dense(srhpm_ctx * ctx, const float * X, int64_t ldx, int64_t N, int64_t K, void * blocks,
                           cudaStream_t stream);

// static_work.cu
size_t static_work_bytes();
int    gemm_run_static(srhpm_ctx * ctx, int wtype, const uint8_t * W, int64_t rows, int64_t K, size_t row_bytes,
                       const float * X, int64_t ldx, int64_t N, float * Y, int64_t ldy, cudaStream_t stream);

// fa_decode.cu: multi-query attention over a q8_0 or f16 KV cache, DK = DV = 256 (byte strides)
struct FaView {
    const float *   q;
    int64_t         qnb1, qnb2;  // token, head
    int             N, H;
    const uint8_t * k;
    int64_t         knb1, knb2;  // token, KV head
    const uint8_t * v;
    int64_t         vnb1, vnb2;
    int             L, Hkv, kv_type;  // SRHPM_TYPE_Q8_0 or SRHPM_TYPE_F16
    const uint8_t * mask;  // f16 [L..][N..][mne2] or null
    int64_t         mnb1, mnb2;
    int             mne2;
    int64_t         mne0;
    const float *   sinks;  // f32 [H] or null
    float *         dst;    // f32 [DV][H][N]
    int64_t         dnb1, dnb2;
};
size_t fa_work_size(int num_sms, int R, int L, int Hkv);
// rec != null: write this KV range's record set (fa_part_bytes(H, N): float2 {max, sum}[H * N] padded to
// fa_part_ms_bytes(H, N), then f32 [H * N][256] unnormalized outputs; row h * N + t) instead of dst, without sinks
int    fa_run(srhpm_ctx * ctx, const FaView & v, float scale, float max_bias, float softcap, void * wdata,
              size_t wsize, cudaStream_t stream, void * rec = nullptr);
size_t fa_part_ms_bytes(int64_t H, int64_t N);
size_t fa_part_bytes(int64_t H, int64_t N);
// merge of n_parts consecutive record sets (<= 256), then sinks and normalization into dst f32 [256][H][N]
int    fa_merge_run(srhpm_ctx * ctx, const void * parts, int n_parts, int N, int H, const float * sinks, float * dst,
                    int64_t dnb1, int64_t dnb2, cudaStream_t stream);
// the merge of every rank's record set read over peer memory (two flag rounds per row); buffer per rank: the record
// set, then the ready and done flags
size_t fa_peer_buffer_bytes(int64_t H, int64_t N);
int    fa_merge_peers_run(srhpm_ctx * ctx, const uint64_t * peers, int world, int rank, uint32_t * epochs, int N, int H,
                          const float * sinks, float * dst, int64_t dnb1, int64_t dnb2, cudaStream_t stream);

// accept.cu: greedy acceptance (argmax of the target logits, longest accepted prefix)
size_t argmax_work_size(int num_sms, int n_vocab, int n_rows);
int    accept_run(srhpm_ctx * ctx, const uint8_t * logits, int64_t ldb, int n_vocab, int n_rows, const int32_t * draft,
                  int n_draft, float relax, int32_t * out_ids, int32_t * out_n, int64_t vocab_offset,
                  srhpm_argmax_record * out_recs, void * wdata, size_t wsize, cudaStream_t stream);
int    accept_merge_run(srhpm_ctx * ctx, const srhpm_argmax_record * recs, int n_shards, int n_rows,
                        const int32_t * draft, int n_draft, float relax, int32_t * out_ids, int32_t * out_n,
                        cudaStream_t stream);

// decoder_ops.cu
int get_rows_run(srhpm_ctx * ctx, const uint8_t * table, int64_t row_bytes, int is_f16, const int32_t * ids, int n,
                 int64_t d, float * out, cudaStream_t stream);
int add_rms_norm_run(srhpm_ctx * ctx, float * x, const float * delta, const float * w, float eps, float * y, int n,
                     int64_t d, cudaStream_t stream);
int add_rms_norm_ar_run(srhpm_ctx * ctx, float * x, const uint64_t * peers, int world, int rank, int slot,
                        uint32_t * epochs, const float * w, float eps, float * y, int n, int64_t d,
                        cudaStream_t stream);
size_t allreduce_buffer_bytes(int64_t d);
int rope_kv_run(srhpm_ctx * ctx, float * qkv, int64_t ld, int n, int H, int Hkv, int hd, const int32_t * pos,
                float theta_base, uint8_t * kc, int64_t knb1, int64_t knb2, uint8_t * vc, int64_t vnb1, int64_t vnb2,
                int cache_type, cudaStream_t stream);
int swiglu_run(srhpm_ctx * ctx, const float * gate, const float * up, int64_t ld_in, float * out, int64_t ld_out,
               int rows, int64_t cols, cudaStream_t stream);

}  // namespace srhpm
