/* srhpm_dgpu: the reference's dGPU library interface (dgpu/dgpu.cu), exported by libsrhpm_dgpu.so on the B200
 * kernels of srhpm_b200.h. ggml-cpu loads the library by name next to itself and binds these functions by name
 * (patch/srhpm.patch:5034-5055; the launcher looks for libsrhpm_dgpu.so on Linux, srhpm/launch.py:124), so it
 * replaces the reference's library without a change on the caller's side.
 *
 * Differences from the reference, both from the B200's design:
 *   - the rows are copied once per key into device memory (HBM) instead of pinned host memory read over PCIe;
 *     max_pinned bounds those copies and dgpu_pinned_bytes reports them;
 *   - the activations are quantized per 256 columns as the CPU's SRV rows are (srv_quantize_row,
 *     patch/srhpm.patch:5518-5575), so the rows a product hands to this library and the rows the CPU computes share
 *     one arithmetic (exact integer sums); the reference's dGPU kernels work on f32 activations.
 * The bandwidth probes of the reference's tools (dgpu_host_alloc, dgpu_dev_ptr, dgpu_read) are not part of the verify
 * path and are not provided. */
#ifndef SRHPM_DGPU_H
#define SRHPM_DGPU_H

#include <stddef.h>
#include <stdint.h>

#ifdef __cplusplus
extern "C" {
#endif

/* dgpu/dgpu.cu:17-25: a context and a stream on the current device; 0, or -1. Idempotent. */
int dgpu_init(void);

/* dgpu/dgpu.cu:241-302: Y = rows . x^T for the first nrows rows of the tensor identified by key (kind 0 = IQ4_XS,
 * 1 = Q3_K; native GGUF rows of K / 256 super-blocks), x = M <= 8 rows of K floats with row stride x_nb bytes.
 * Asynchronous. 0, or -1 bad arguments, -2 the copies would exceed max_pinned bytes, -3 no memory for the copy, -4 no
 * memory for the staging buffers, -5 not initialised or the launch failed, -6 Q3_K rows of an odd number of
 * super-blocks; nothing runs on failure. */
int dgpu_launch(int kind, const void * key, const void * rows, int64_t nrows, int64_t K, int M, const float * x,
                size_t x_nb, size_t max_pinned);

/* dgpu/dgpu.cu:303-312: waits for the last launch and writes y[t][0..nrows) to dst + t * dst_nb (bytes); M and nrows
 * as launched. 0, or -1 (no launch, or another shape), -5 (the launch failed on the device). */
int dgpu_collect(int M, int64_t nrows, char * dst, size_t dst_nb);

/* dgpu/dgpu.cu:235-239: free and total device memory (0, 0 when unavailable). */
void dgpu_mem_info(size_t * free_b, size_t * total_b);

/* dgpu/dgpu.cu:233: bytes of row copies held. */
size_t dgpu_pinned_bytes(void);

#ifdef __cplusplus
}
#endif
#endif
