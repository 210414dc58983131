/* TEST INFRASTRUCTURE (oracle): a CPU restatement of the reference's speculative-verification arithmetic, used only
 * by tests/, the smoke check and bench.py's CPU-baseline leg as the checker. Never linked into the product.
 *
 * Parity status: the SRV activation quantizer and the per-type integer dots are pinned against the reference's own
 * kernels compiled from its patch (oracle/_ref, see build_ref.sh) and against the golden fixtures in tests/golden/;
 * block unpacking is also cross-checked against gguf-py's dequantizers. The q8_0 activation quantizer (upstream
 * ggml, absent from the container) is restated in two variants (ORC_Q8_0_SIMD / ORC_Q8_0_REF): parity unpinned.
 * The attention and acceptance restatements are pinned against the reference's FA-GQA function compiled from the
 * patch; greedy acceptance (upstream common_sampler_sample_and_accept_n) is restated: parity unpinned for ties.
 */
#ifndef SRHPM_ORACLE_H
#define SRHPM_ORACLE_H
#include <stdint.h>
#include <stddef.h>

#ifdef __cplusplus
extern "C" {
#endif

enum { ORC_F32 = 0, ORC_F16 = 1, ORC_Q8_0 = 8, ORC_Q3_K = 11, ORC_Q4_K = 12, ORC_Q5_K = 13, ORC_Q6_K = 14,
       ORC_IQ4_XS = 23 };
enum { ORC_Q8_0_SIMD = 0, ORC_Q8_0_REF = 1 };

size_t orc_block_bytes(int type);   /* bytes per block */
int    orc_block_elems(int type);   /* weights per block */

float    orc_fp16_to_fp32(uint16_t h);
uint16_t orc_fp32_to_fp16(float f); /* round to nearest even */

/* patch/srhpm.patch:5518-5575 (srv_quantize_row, Q8_K-identical): per 256 columns int8 q, d = 1/iscale, per-32 and
 * per-16 sums of q (either sum pointer may be NULL) */
void orc_quantize_row_q8K(const float * x, int8_t * q, float * d, int16_t * bsum32, int16_t * bsum16, int64_t K);

/* q8_0 activation quantizer (vec_dot_type of Q8_0 weights and of a q8_0 KV cache). mode: ORC_Q8_0_SIMD / _REF */
void orc_quantize_row_q8_0(const float * x, void * blocks, int64_t K, int mode);

/* ggml dequantize_row_* restated: n weights of `type` -> f32 */
void orc_dequantize(int type, const void * blocks, float * y, int64_t n);

/* Integer sums of one weight row against one quantized activation row.
 * K-quants / IQ4_XS: per super-block sb, main[sb] = sum over the sub-blocks of (integer block scale) x (code dot),
 * mins[sb] = sum_b m_b * bsum32_b (Q4_K / Q5_K; 0 otherwise). Q8_0: per 32-block, main[blk] = code dot, mins unused.
 * xq: int8 activations (Q8_K layout for K-quants/IQ4_XS, or the qs of q8_0 blocks packed densely for Q8_0). */
void orc_row_isums(int type, const void * row, const int8_t * xq, const int16_t * bsum32, int64_t K, int32_t * main_,
                   int32_t * mins);

/* Y[t*rows + r] (double) = sum_k W[r,k] X[t,k] through the exact integer sums above: K-quants / IQ4_XS with the
 * Q8_K activation quantizer, Q8_0 with the q8_0 quantizer of `q8_mode`. Returns -1 for unsupported shapes. */
int orc_mul_mat(int type, const void * W, int64_t rows, int64_t K, const float * X, int64_t N, double * Y, int q8_mode);

/* Stock ggml mul_mat of Q8_0 weights (no SRV kernel exists for Q8_0): activations quantized to q8_0, one
 * vec_dot_q8_0_q8_0 per (row, token) in the lane order of ggml-cpu's x86 path, rows over nth threads. */
int orc_mul_mat_q8_0_f32(const void * W, int64_t rows, int64_t K, const float * X, int64_t N, float * Y, int q8_mode,
                         int nth);

/* Multi-query attention, single pass (no chunking), double precision softmax and accumulation.
 * q f32 [H][N][DK] dense (head-major), k/v of kv_type (ORC_F16 or ORC_Q8_0) laid out [Hkv][L][row] dense,
 * mask f16 [N][L] (NULL = none), sinks f32 [H] (NULL = none), dst f32 [N][H][DV].
 * Q.K follows the reference's arithmetic: for q8_0 K, Q is quantized to q8_0 (q8_mode) and the integer dot scaled
 * by d_k d_q; for f16 K, f32 Q against the f16 values. Scores: scale (divided by softcap when softcap != 0), then
 * softcap*tanh, then + slope*mask (ALiBi slope from max_bias; 1 when max_bias == 0). */
int orc_attention(const float * q, int64_t DK, int64_t N, int64_t H, int kv_type, const void * k, const void * v,
                  int64_t DV, int64_t L, int64_t Hkv, const uint16_t * mask, const float * sinks, float scale,
                  float max_bias, float softcap, int q8_mode, double * dst);

/* The record form of orc_attention for a split of the KV range (the reference's chunked path, whose per-chunk records
 * are written at patch/srhpm.patch:779-784 and merged at :789-823; across devices the ranks are the chunks): over KV
 * tokens [t0, t1) of the same buffers (L tokens per KV head), per row (h, t) the maximum score m (natural-log units,
 * -inf when no score is finite), s = sum exp(score - m) and acc[d] = sum exp(score - m) v[d], unnormalized and
 * without sinks. rec_m, rec_s [H][N], rec_acc [H][N][DV], all double. */
int orc_attention_partial(const float * q, int64_t DK, int64_t N, int64_t H, int kv_type, const void * k,
                          const void * v, int64_t DV, int64_t L, int64_t Hkv, int64_t t0, int64_t t1,
                          const uint16_t * mask, float scale, float max_bias, float softcap, int q8_mode,
                          double * rec_m, double * rec_s, double * rec_acc);

/* Merge of n_parts record sets ([n_parts][H][N] for m and s, [n_parts][H][N][DV] for acc) in part order, then sinks
 * and the division by the sum (patch/srhpm.patch:789-823): parts with s == 0 are skipped. dst f64 [N][H][DV]. */
int orc_attention_merge(int64_t n_parts, int64_t N, int64_t H, int64_t DV, const double * rec_m,
                        const double * rec_s, const double * rec_acc, const float * sinks, double * dst);

/* Greedy longest-prefix acceptance (upstream common_sampler_sample_and_accept_n with greedy sampling, plus the
 * SR-HPM relax of patch/srhpm.patch:9-35). logits f32 [n_draft+1][n_vocab]; out_ids receives the accepted draft
 * tokens followed by one sampled token (at most n_draft+1 ids); returns that count. argmax ties -> lowest id. */
int orc_accept(const float * logits, int64_t n_vocab, const int32_t * draft, int n_draft, float relax,
               int32_t * out_ids);

/* Input generation (not pinned): n f32 weights -> GGUF blocks of `type` by round-to-nearest with per-block scales
 * from each block's range, the inverse of orc_dequantize. Returns the bytes written, -1 for an unsupported type or
 * n not a multiple of the block size. For the CPU reference timings, whose inputs must not come from the product. */
int64_t orc_quantize_rtn(int type, const float * x, void * out, int64_t n);

#ifdef __cplusplus
}
#endif
#endif
