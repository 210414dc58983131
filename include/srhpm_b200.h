/* srhpm_b200: B200 (sm_100a) kernels for SR-HPM's speculative-verification hot path, behind a plain C ABI.
 *
 * The path verifies 1 + k drafted tokens against a quantized dense decoder in one pass:
 *   - small-batch quantized matmul (ggml_mul_mat with ne[1] = 1..16 on Q4_K / Q5_K / Q6_K / Q3_K / IQ4_XS / Q8_0)
 *   - multi-query attention over an f16 or q8_0 KV cache (ggml_flash_attn_ext with 1..16 query rows)
 *   - greedy longest-prefix acceptance over the target logits
 *
 * Conventions (all entry points):
 *   - tensors are ggml-shaped views (srhpm_tensor: type, ne[4] in elements, nb[4] in bytes, data) of DEVICE memory,
 *     unless an argument says otherwise; the caller owns every buffer, including the work buffer (wdata) whose size
 *     the matching *_work_size call returns.
 *   - calls are asynchronous and ordered on `stream` (a cudaStream_t; NULL = the legacy default stream).
 *   - errors are returned as srhpm_status codes, never by aborting. SRHPM_UNSUPPORTED means "not handled here, run
 *     the stock path", as the reference's compute_forward returning false does.
 *   - one srhpm_ctx per device; a context may be used from several host threads only with external serialisation.
 */
#ifndef SRHPM_B200_H
#define SRHPM_B200_H

#include <stddef.h>
#include <stdint.h>

#ifdef __cplusplus
extern "C" {
#endif

/* ggml_type numbering (GGUF) */
enum srhpm_type {
    SRHPM_TYPE_F32    = 0,
    SRHPM_TYPE_F16    = 1,
    SRHPM_TYPE_Q8_0   = 8,
    SRHPM_TYPE_Q3_K   = 11,
    SRHPM_TYPE_Q4_K   = 12,
    SRHPM_TYPE_Q5_K   = 13,
    SRHPM_TYPE_Q6_K   = 14,
    SRHPM_TYPE_Q8_K   = 15,
    SRHPM_TYPE_IQ4_XS = 23,
    SRHPM_TYPE_I32    = 26,
};

enum srhpm_status {
    SRHPM_OK             = 0,
    SRHPM_UNSUPPORTED    = 1,  /* shape / type outside this path: use the stock path */
    SRHPM_ERR_INVALID    = -1, /* inconsistent arguments */
    SRHPM_ERR_ALIGN      = -2, /* a pointer or stride misses its required alignment */
    SRHPM_ERR_WORKSPACE  = -3, /* wdata missing or smaller than *_work_size */
    SRHPM_ERR_CUDA       = -4, /* a CUDA runtime call failed (srhpm_last_cuda_error has the code) */
    SRHPM_ERR_DEVICE     = -5, /* a kernel reported an error through the context's status word */
    SRHPM_ERR_TOO_LARGE  = -6, /* the product needs more scratch than srhpm_mul_mat_static's fixed buffer holds */
};

/* q8_0 activation quantizer used for Q8_0 weights and for Q against a q8_0 KV cache (the upstream ggml-cpu quantizer
 * is not in the reference; both variants are provided). SIMD: id = 127/amax, round half to even (ggml-cpu's x86
 * path, the default). REF: id = 1/d, roundf (ggml's quantize_row_q8_0_ref). */
enum srhpm_q8_0_act_mode { SRHPM_Q8_0_ACT_SIMD = 0, SRHPM_Q8_0_ACT_REF = 1 };

typedef struct srhpm_tensor {
    int32_t type;   /* enum srhpm_type */
    int64_t ne[4];  /* elements per dimension, ggml order (ne[0] innermost) */
    size_t  nb[4];  /* bytes per step in each dimension */
    void *  data;   /* device pointer */
} srhpm_tensor;

typedef struct srhpm_ctx srhpm_ctx;

/* Context of one device: options, a device status word for bounded-wait errors, launch counters.
 * Replaces dgpu_init (dgpu/dgpu.cu:17-25); srhpm_ctx_destroy has no counterpart there. */
int  srhpm_ctx_create(int device, srhpm_ctx ** out);
int  srhpm_ctx_destroy(srhpm_ctx * ctx);
int  srhpm_ctx_set_q8_0_act_mode(srhpm_ctx * ctx, int mode);
/* kernels this context launched since creation (or the last reset) */
int64_t srhpm_ctx_launch_count(const srhpm_ctx * ctx, int reset);
/* reads (synchronously) and clears the device status word; SRHPM_ERR_DEVICE when a kernel reported an error */
int  srhpm_ctx_check(srhpm_ctx * ctx, int32_t * device_code);
int  srhpm_last_cuda_error(void);
const char * srhpm_status_str(int status);

/* ggml type facts (ggml_blck_size / ggml_type_size / ggml_row_size) */
int    srhpm_blck_size(int type);
size_t srhpm_type_size(int type);
size_t srhpm_row_size(int type, int64_t n);

/* ---- small-batch quantized matmul ------------------------------------------------------------------------------
 * Y = W X in ggml_mul_mat semantics: W = src0 [K, rows] of a quantized type (rows contiguous, nb[1] = row size,
 * data 16-byte aligned), X = src1 f32 [K, N] (any row stride, multiple of 4), Y = dst f32 [rows, N] (any row
 * stride). 1 <= N <= 16, K a multiple of 256. Activations are quantized per row and 256 columns to int8 (bit-identical
 * to the reference's srv_quantize_row, patch/srhpm.patch:5518-5575) or, for Q8_0 weights, to q8_0; each super-block
 * is decoded once for all N rows and reduced with exact int32 sums on the tensor cores.
 * Replaces tensor_traits_srv::work_size / compute_forward (patch/srhpm.patch:6366-6374, :6400-6611) and the dGPU's
 * dgpu_launch + dgpu_collect (dgpu/dgpu.cu:244-312). A row range of W (a view with fewer rows and Y a matching view)
 * is the reference's CPU/GPU row split (patch/srhpm.patch:6497-6529). */
int srhpm_mul_mat_work_size(const srhpm_tensor * W, const srhpm_tensor * X, size_t * size);
int srhpm_mul_mat(srhpm_ctx * ctx, const srhpm_tensor * W, const srhpm_tensor * X, srhpm_tensor * Y, void * wdata,
                  size_t wsize, void * stream);

/* srhpm_mul_mat in ONE kernel launch: the matmul grid quantizes its own activations (every consumer warp of the grid
 * takes a share of the (super-block, row) pairs) and meets at an arrival counter before any CTA loads the records;
 * the same records, so the output is bit-identical to srhpm_mul_mat's. Same work buffer (srhpm_mul_mat_work_size).
 * Faster after a small kernel that leaves the SMs free (attention output -> its projection: the grid is resident
 * early and the activations sit in L2), slower right after another large matmul (the grid becomes resident piecewise
 * as that one drains and the meet waits for its last CTA): measured on a B200, -0.13 ms per 27B-class verify step
 * as the attention output projection, +1.5 us per product in a sweep of back-to-back products. The counter is kept by
 * the context, one per work buffer: calls through one context on several streams need separate work buffers (as
 * their activation records already do). Products whose grid would get more than two quantization jobs per warp
 * fall back to the separate quantizer. No reference counterpart (the reference quantizes on its CPU threads before
 * the barrier, patch/srhpm.patch:6455-6461). */
int srhpm_mul_mat_fused_quant(srhpm_ctx * ctx, const srhpm_tensor * W, const srhpm_tensor * X, srhpm_tensor * Y,
                              void * wdata, size_t wsize, void * stream);

/* The integer part of srhpm_mul_mat, for bit-exact checks: per (token t, row r, block j) the int32 sum of
 * (integer block scale) x (code . activation) over block j (super-block of 256, or the 32-block for Q8_0), written to
 * isum[(t * rows + r) * nblk + j], and for Q4_K / Q5_K the sum of (integer min) x (activation sum) to imin (same
 * layout; may be NULL otherwise). Same kernels and decoders as srhpm_mul_mat. No reference counterpart (test hook). */
int srhpm_mul_mat_isums(srhpm_ctx * ctx, const srhpm_tensor * W, const srhpm_tensor * X, int32_t * isum,
                        int32_t * imin, void * wdata, size_t wsize, void * stream);

/* srhpm_mul_mat without a work buffer, for callers that cannot allocate device memory: a host framework that hands
 * out only the tensors it owns (no scratch per operation), or a latency-critical decode loop where a cudaMalloc
 * would synchronise the device. The scratch is a fixed 1 MiB array inside the library on every device that loads
 * it, kept until the process exits; products are not split along K here. Limit: the activation records and row-block
 * counters of the product must fit 1 MiB (for K up to 32768 and N up to 16 that leaves room for 6 million weight
 * rows); beyond that the call returns SRHPM_ERR_TOO_LARGE and does nothing. The first call on a device looks up the array's device address
 * (make it before any stream capture). All calls share the array: calls whose work overlaps on the GPU race. The
 * context's device must be the calling thread's current device (else SRHPM_ERR_INVALID). Allocates nothing. No
 * counterpart in the reference. */
int srhpm_mul_mat_static(srhpm_ctx * ctx, const srhpm_tensor * W, const srhpm_tensor * X, srhpm_tensor * Y,
                         void * stream);

/* Activation quantizer, row by row: X f32 [K, N] -> q int8 [N][K], d f32 [N][K/256], bsum32 int16 [N][K/32],
 * bsum16 int16 [N][K/16] (dense, device; bsum pointers may be NULL). Bit-identical to srv_quantize_row
 * (patch/srhpm.patch:5518-5575), which equals ggml's quantize_row_q8_K. */
int srhpm_quantize_rows_q8_K(srhpm_ctx * ctx, const srhpm_tensor * X, int8_t * q, float * d, int16_t * bsum32,
                             int16_t * bsum16, void * stream);
/* X f32 [K, N] -> N rows of K/32 q8_0 blocks (34 bytes each, GGUF layout), with the context's q8_0 mode.
 * ggml-cpu from_float of GGML_TYPE_Q8_0 (upstream; used by the reference at patch/srhpm.patch:670-673). */
int srhpm_quantize_rows_q8_0(srhpm_ctx * ctx, const srhpm_tensor * X, void * blocks, void * stream);

/* ---- multi-query attention -------------------------------------------------------------------------------------
 * dst = softmax(scale * Q K^T [softcap] + slope * mask [+ sink]) V in ggml_flash_attn_ext semantics, for the few query
 * tokens of a verification pass: q f32 [DK, N, H] (token stride nb[1], head stride nb[2]), k / v [256, L, Hkv] of type
 * q8_0 or f16 (DK = DV = 256; token stride nb[1] and KV-head stride nb[2] multiples of 16 bytes, data 16-byte aligned, so
 * both the [Hkv][L] layout and llama.cpp's [L][Hkv] cache view are accepted), mask f16 [>= L, >= N, ne2] applied to
 * head h from slice h % ne2 (may be NULL), sinks f32 [H] (may be NULL), dst f32 [DV, H, N] (dst row of head h and
 * token t at h * nb[1] + t * nb[2]). H a multiple of Hkv, 1 <= N <= 16. Q is quantized per row to q8_0 with the
 * context's q8_0 mode and Q.K is the exact q8_0 integer dot product, as the reference's grouped path computes it;
 * with an f16 cache Q stays f32 (split into two f16 parts on the tensor cores). Other types / head sizes:
 * SRHPM_UNSUPPORTED. wdata: srhpm_flash_attn_ext_work_size bytes (0 when the KV range is
 * not split), ordered on `stream` like every call.
 * Replaces ggml_fa_gqa_small_work_size / ggml_compute_forward_flash_attn_ext_gqa_small (patch/srhpm.patch:555-824)
 * behind the gate at patch/srhpm.patch:833-841. */
int srhpm_flash_attn_ext_work_size(const srhpm_ctx * ctx, const srhpm_tensor * q, const srhpm_tensor * k,
                                   const srhpm_tensor * v, size_t * size);
int srhpm_flash_attn_ext(srhpm_ctx * ctx, const srhpm_tensor * q, const srhpm_tensor * k, const srhpm_tensor * v,
                         const srhpm_tensor * mask, const srhpm_tensor * sinks, float scale, float max_bias,
                         float softcap, srhpm_tensor * dst, void * wdata, size_t wsize, void * stream);

/* ---- attention split over the KV range across devices ----------------------------------------------------------
 * Each device holds a range of the cache's tokens: k / v views (and the mask's columns) start at the range's first
 * token and k->ne[1] = its token count (0 for an empty range; no work buffer then). srhpm_flash_attn_ext_partial
 * takes the arguments of srhpm_flash_attn_ext except sinks and dst and writes the range's record set into `part`
 * (srhpm_flash_attn_part_size(H, N) bytes, 16-byte aligned; wdata: srhpm_flash_attn_ext_work_size of the range's
 * views): for row r = h * N + t, float {max, sum} pairs [H * N] (max of the scaled scores in base-2 units; sum = 0 for
 * a range without a finite score), zero-padded to a multiple of 16 bytes, then float acc[H * N][256] (the row's output
 * times its sum, not normalized).
 * srhpm_flash_attn_merge combines n_parts (<= 256) such sets stored one after another (for example gathered from all
 * devices in KV order), adds the sinks (f32 [H] or NULL) and writes dst f32 [256, H, N] as srhpm_flash_attn_ext would
 * for the whole range. The reference splits the KV range into chunks over its CPU threads and merges their
 * (max, sum, acc) records the same way (patch/srhpm.patch:555-579, 779-823); here the devices are the chunks. */
size_t srhpm_flash_attn_part_size(int64_t n_head, int64_t n_tokens);
int    srhpm_flash_attn_ext_partial(srhpm_ctx * ctx, const srhpm_tensor * q, const srhpm_tensor * k,
                                    const srhpm_tensor * v, const srhpm_tensor * mask, float scale, float max_bias,
                                    float softcap, void * part, void * wdata, size_t wsize, void * stream);
int    srhpm_flash_attn_merge(srhpm_ctx * ctx, const void * parts, int n_parts, const srhpm_tensor * sinks,
                              srhpm_tensor * dst, void * stream);
/* The same merge without a collective: every rank's record set sits at the start of its own buffer of
 * srhpm_flash_attn_peer_buffer_size(H, N) bytes, zeroed once and mapped on every rank (peer_buffers[j] = rank j's
 * buffer as this rank addresses it: symmetric memory), written there by srhpm_flash_attn_ext_partial. Per row, the
 * call sends its record row to every rank's buffer as 8-byte (value, epoch) words, waits (bounded: 2 s, then an error
 * status) until every rank's words in its own buffer carry the epoch, merges them in rank order, adds the sinks and
 * writes dst as srhpm_flash_attn_merge does (the same arithmetic, so the same result). epochs: u32 [H * N] on this
 * device, zero at the start, counted per call identically on every rank; two receive slots alternate, so a rank's
 * next call never overwrites words a peer still reads. Every rank must make the same calls in the same order;
 * world <= 8. No counterpart in the reference (one device). */
size_t srhpm_flash_attn_peer_buffer_size(int64_t n_head, int64_t n_tokens);
int    srhpm_flash_attn_merge_peers(srhpm_ctx * ctx, const uint64_t * peer_buffers, int world, int rank,
                                    uint32_t * epochs, const srhpm_tensor * sinks, srhpm_tensor * dst, void * stream);

/* ---- greedy acceptance -----------------------------------------------------------------------------------------
 * Target logits f32 [n_vocab, >= n_draft + 1] (row i scores the token after draft position i; row stride nb[1]) and
 * the drafted ids int32 [n_draft] (device): for i < n_draft, id_i = argmax of row i (the first maximum, as the
 * sequential greedy scan finds it); with relax > 0 a drafted token whose logit is within relax of row i's maximum is
 * taken instead; id_i is emitted and the scan stops at the first id_i != draft[i]; when all n_draft tokens are
 * accepted, the argmax of row n_draft is emitted as well. out_ids int32 [n_draft + 1] and out_n int32 (device) receive
 * the emitted ids and their count (accepted drafted tokens + 1; n_rollback = n_draft + 1 - out_n). 0 <= n_draft <= 16.
 * Replaces common_sampler_sample_and_accept_n with a greedy sampler (upstream) and the reference's relaxed acceptance
 * (patch/srhpm.patch:9-35). wdata: srhpm_verify_accept_work_size bytes. */
int srhpm_verify_accept_work_size(const srhpm_ctx * ctx, const srhpm_tensor * logits, size_t * size);
int srhpm_verify_accept(srhpm_ctx * ctx, const srhpm_tensor * logits, const int32_t * draft, int n_draft, float relax,
                        int32_t * out_ids, int32_t * out_n, void * wdata, size_t wsize, void * stream);

/* Acceptance over a vocabulary sharded across devices: each shard (logits [shard size, n_rows], global ids starting
 * at vocab_offset) writes one record per row with srhpm_argmax_shard; srhpm_accept_merge takes the records of all
 * shards ([n_shards][n_rows], in vocabulary order, gathered to one device) and emits what srhpm_verify_accept would
 * for the whole vocabulary. imax = -1 marks a shard that starts the vocabulary with a NaN logit (argmax 0), -2 a row
 * of the shard without a non-NaN value. No counterpart in the reference (its head is not sharded). */
typedef struct srhpm_argmax_record {
    float   vmax;       /* maximum over the shard's non-NaN logits of the row */
    int32_t imax;       /* its first (global) index */
    float   vdraft;     /* logit of the drafted token of this row, when the shard holds it */
    int32_t has_draft;  /* 1 when it does */
} srhpm_argmax_record;
int srhpm_argmax_shard(srhpm_ctx * ctx, const srhpm_tensor * logits, int64_t vocab_offset, const int32_t * draft,
                       int n_draft, srhpm_argmax_record * out, void * wdata, size_t wsize, void * stream);
int srhpm_accept_merge(srhpm_ctx * ctx, const srhpm_argmax_record * recs, int n_shards, int n_rows,
                       const int32_t * draft, int n_draft, float relax, int32_t * out_ids, int32_t * out_n,
                       void * stream);

/* ---- the element-wise operators of a dense decoder verify step (ggml semantics) ------------------------------------
 * Device pointers, rows of d contiguous values, n <= 16 rows. These surround the verify GEMMs in a full model step
 * (the 27B-class benchmark); the reference runs them as stock ggml operators.
 *   srhpm_get_rows: out[i] = table row ids[i] (f16 or f32 table [d, n_rows] with row stride nb[1]) as f32
 *   srhpm_add_rms_norm: x += delta (delta may be NULL), then y = x / sqrt(mean(x^2) + eps) * w     (x, y [n][d])
 *   srhpm_rope_kv: qkv rows [n][ld] = n_head query heads | n_head_kv key heads | n_head_kv value heads of head_dim;
 *       NeoX rotary embedding (pairs (j, j + head_dim/2), theta_j = pos * theta_base^(-2j/head_dim)) of the query and
 *       key heads in place, then the keys and values are stored into the caches at token pos[t] (views as for
 *       srhpm_flash_attn_ext: [head_dim, capacity, n_head_kv], f16 or q8_0 with the context's q8_0 mode)
 *   srhpm_swiglu: out[t][j] = silu(gate[t][j]) * up[t][j] for n rows of n_ff values (input row stride ld_in, output
 *       ld_out, in floats; gate and up may be the two halves of one fused gate|up GEMM output) */
int srhpm_get_rows(srhpm_ctx * ctx, const srhpm_tensor * table, const int32_t * ids, int n, float * out, void * stream);
int srhpm_add_rms_norm(srhpm_ctx * ctx, float * x, const float * delta, const float * w, float eps, float * y, int n,
                       int64_t d, void * stream);
/* Residual add + RMSNorm fused with the activation quantization of the GEMM that consumes y (a fused GEMM
 * prologue): x += delta (delta may be NULL), y = x / sqrt(mean(x^2) + eps) * w as srhpm_add_rms_norm, and the
 * activation records of y for the product with W_next (its type, rows and K = d: ne = [d, rows]) are written into
 * wdata (sized by srhpm_mul_mat_work_size(W_next, X[d, n])), bit-identical to what srhpm_mul_mat's own quantizer
 * would write; srhpm_mul_mat_prequantized(W_next, X, Y, same wdata) then runs the product on them (X's data is not
 * read, only its shape). K-quant and IQ4_XS weights (Q8_0: SRHPM_UNSUPPORTED, use srhpm_mul_mat). n <= 16,
 * d <= 16384; x, delta, w, y 16-byte aligned. */
int srhpm_add_rms_norm_quant(srhpm_ctx * ctx, float * x, const float * delta, const float * w, float eps, float * y,
                             int n, const srhpm_tensor * W_next, void * wdata, size_t wsize, void * stream);
int srhpm_mul_mat_prequantized(srhpm_ctx * ctx, const srhpm_tensor * W, const srhpm_tensor * X, srhpm_tensor * Y,
                               void * wdata, size_t wsize, void * stream);
/* SwiGLU fused the same way: out = silu(gate) * up as srhpm_swiglu (rows of ld_in / ld_out floats, n_ff = W_next's
 * K columns), and the activation records of out for the product with W_next written into wdata for
 * srhpm_mul_mat_prequantized. */
int srhpm_swiglu_quant(srhpm_ctx * ctx, const float * gate, const float * up, int64_t ld_in, float * out,
                       int64_t ld_out, int n, const srhpm_tensor * W_next, void * wdata, size_t wsize, void * stream);
/* The FFN down projection with the SwiGLU in its own prologue: Y = W . h for h = silu(gate) * up (silu(g) =
 * g / (1 + exp(-g)), as srhpm_swiglu), gate and up f32 views of the same shape and row stride (ne[0] = K, ne[1] = n).
 * The GEMM grid computes h for its activation super-blocks and quantizes it into the records, as
 * srhpm_mul_mat_fused_quant does for X: the work of srhpm_swiglu_quant + srhpm_mul_mat_prequantized in one launch,
 * h itself not stored (when the grid is too small for the prologue, the SwiGLU record kernel runs first). The records
 * are the same bytes, so Y is bit-identical to that pair. K-quant and IQ4_XS W (Q8_0: SRHPM_UNSUPPORTED); wdata of
 * srhpm_mul_mat_work_size(W, gate) bytes. */
int srhpm_mul_mat_swiglu(srhpm_ctx * ctx, const srhpm_tensor * W, const srhpm_tensor * gate, const srhpm_tensor * up,
                         srhpm_tensor * Y, void * wdata, size_t wsize, void * stream);

/* Tensor-parallel residual add + RMSNorm with the all-reduce inside (row-parallel GEMM -> next norm):
 * every rank's row-parallel GEMM (attention output, FFN down) writes its partial sum [n][d] f32 into slot `slot`
 * (0 or 1) of its own symmetric buffer of srhpm_allreduce_buffer_size(d) bytes, zeroed once before first use and
 * mapped on every rank (peer_buffers: a DEVICE array of `world` addresses, this rank's own at [rank]; IPC / symmetric
 * memory set up by the caller). srhpm_add_rms_norm_allreduce then, per row: sends each of its partial values with a
 * per-(slot, row) epoch, as one 8-byte word, into the receive area of every rank's buffer, waits (bounded: 2 s, then
 * SRHPM_ERR_DEVICE through srhpm_ctx_check) until every word it receives carries the epoch, sums the ranks' values in
 * rank order (identical on every rank), adds the sum to x and writes y = x / sqrt(mean(x^2) + eps) * w. epochs: this rank's uint32 [2][16] counters, zeroed once. n <= 16, world <= 8,
 * d a multiple of 4 and <= 16384; x, w, y 16-byte aligned. The two slots alternate (O, down): a slot is rewritten only
 * after the other slot's barrier has passed on every rank. Every rank must make the same sequence of calls. No
 * counterpart in the reference (it runs on one device): the tensor-parallel decoder's all-reduce after O and down. */
size_t srhpm_allreduce_buffer_size(int64_t d);
int srhpm_add_rms_norm_allreduce(srhpm_ctx * ctx, float * x, const uint64_t * peer_buffers, int world, int rank,
                                 int slot, uint32_t * epochs, const float * w, float eps, float * y, int n, int64_t d,
                                 void * stream);
/* srhpm_add_rms_norm_allreduce fused with the activation quantization of the GEMM that consumes y, as
 * srhpm_add_rms_norm_quant is for srhpm_add_rms_norm: the same exchange and rank-order sum of the ranks' slot
 * `slot` rows, the residual add and the norm, and W_next's activation records written into wdata for
 * srhpm_mul_mat_prequantized. One launch instead of the norm plus srhpm_mul_mat's own quantizer; each row is spread
 * over a cluster of 8 CTAs (each sends and sums a share of the columns), with results bit-identical to one CTA per
 * row. Same limits as both (K-quant and IQ4_XS W_next, n <= 16, d <= 16384, world <= 8). No counterpart in the
 * reference (one device). */
int srhpm_add_rms_norm_allreduce_quant(srhpm_ctx * ctx, float * x, const uint64_t * peer_buffers, int world,
                                       int rank, int slot, uint32_t * epochs, const float * w, float eps, float * y,
                                       int n, const srhpm_tensor * W_next, void * wdata, size_t wsize, void * stream);
int srhpm_rope_kv(srhpm_ctx * ctx, float * qkv, int64_t ld, int n, int n_head, int n_head_kv, int head_dim,
                  const int32_t * pos, float theta_base, const srhpm_tensor * k_cache, const srhpm_tensor * v_cache,
                  void * stream);
int srhpm_swiglu(srhpm_ctx * ctx, const float * gate, const float * up, int64_t ld_in, float * out, int64_t ld_out,
                 int n, int64_t n_ff, void * stream);

/* ---- host-side weight quantizer (CPU) -------------------------------------------------------------------------
 * f32 rows -> GGUF blocks of `type` (Q4_K, Q5_K, Q6_K, Q3_K, IQ4_XS, Q8_0, F16). Host pointers. Returns the bytes
 * written. ggml_quantize_chunk's contract (upstream); imatrix is accepted and ignored (uniform importance). */
size_t srhpm_quantize_chunk(int type, const float * src, void * dst, int64_t start, int64_t nrows, int64_t n_per_row,
                            const float * imatrix);

#ifdef __cplusplus
}
#endif
#endif /* SRHPM_B200_H */
