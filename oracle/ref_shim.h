// TEST INFRASTRUCTURE (oracle). Not part of the product; nothing outside tests/, the smoke check and the
// CPU-baseline leg of bench.py may load what is built from this file.
//
// Minimal stand-ins for the upstream llama.cpp/ggml declarations that the reference's own CPU kernels need, so
// that those kernels compile here from the reference patch itself:
//   - ggml/src/ggml-cpu/srv-kernels.inc            (patch/srhpm.patch:5454-6230)
//   - ggml_compute_forward_flash_attn_ext_gqa_small (patch/srhpm.patch:539-824, from ggml/src/ggml-cpu/ops.cpp)
// The upstream tree (ggml @ d05706b) is not available, so the block layouts below are written from the GGUF
// format facts (sizes cross-checked against gguf-py's GGML_QUANT_SIZES in the tests) and the helper routines
// that the FA-GQA function calls (vec_dot of q8_0, the q8_0 quantizer, simd_gemm, soft_max ...) are restated
// in oracle/ggml_restated.h.
#pragma once
#include <immintrin.h>
#include <stdint.h>
#include <stddef.h>
#include <string.h>
#include <math.h>

#define QK_K 256
#define K_SCALE_SIZE 12
#define QK8_0 32

typedef uint16_t ggml_half;
typedef uint16_t ggml_fp16_t;

// F16C conversions: the same round-to-nearest-even that ggml-cpu uses on x86 hosts
static inline float ref_fp16_to_fp32(ggml_half h) { return _cvtsh_ss(h); }
static inline ggml_half ref_fp32_to_fp16(float f) { return (ggml_half) _cvtss_sh(f, 0); }
#define GGML_CPU_FP16_TO_FP32(x) ref_fp16_to_fp32(x)
#define GGML_CPU_FP32_TO_FP16(x) ref_fp32_to_fp16(x)

// --- block layouts (GGUF) ------------------------------------------------------------------------------------
#define GGML_COMMON_AGGR_U u
#define GGML_COMMON_AGGR_S s

typedef struct {
    union {
        struct { ggml_half d; ggml_half dmin; } s;
        uint32_t dm;
    } u;
    uint8_t scales[K_SCALE_SIZE];
    uint8_t qs[QK_K / 2];
} block_q4_K;  // 144 bytes

typedef struct {
    union {
        struct { ggml_half d; ggml_half dmin; } s;
        uint32_t dm;
    } u;
    uint8_t scales[K_SCALE_SIZE];
    uint8_t qh[QK_K / 8];
    uint8_t qs[QK_K / 2];
} block_q5_K;  // 176 bytes

typedef struct {
    uint8_t   ql[QK_K / 2];
    uint8_t   qh[QK_K / 4];
    int8_t    scales[QK_K / 16];
    ggml_half d;
} block_q6_K;  // 210 bytes

typedef struct {
    uint8_t   hmask[QK_K / 8];
    uint8_t   qs[QK_K / 4];
    uint8_t   scales[12];
    ggml_half d;
} block_q3_K;  // 110 bytes

typedef struct {
    ggml_half d;
    uint16_t  scales_h;
    uint8_t   scales_l[QK_K / 64];
    uint8_t   qs[QK_K / 2];
} block_iq4_xs;  // 136 bytes

typedef struct {
    ggml_half d;
    int8_t    qs[QK8_0];
} block_q8_0;  // 34 bytes

// IQ2/IQ3 layouts: the srv kernels declare decoders for them, none of which the verify path of this build calls
typedef struct { ggml_half d; uint8_t qs[QK_K / 4]; uint8_t qh[QK_K / 32]; uint8_t signs[QK_K / 8]; uint8_t scales[QK_K / 64]; } block_iq3_s;
typedef struct { ggml_half d; uint8_t qs[3 * QK_K / 8]; } block_iq3_xxs;
typedef struct { ggml_half d; uint16_t qs[QK_K / 8]; } block_iq2_xxs;
typedef struct { ggml_half d; uint16_t qs[QK_K / 8]; uint8_t scales[QK_K / 32]; } block_iq2_xs;
typedef struct { ggml_half d; uint8_t qs[QK_K / 4]; uint8_t qh[QK_K / 32]; uint8_t scales[QK_K / 32]; } block_iq2_s;

static_assert(sizeof(block_q4_K) == 144, "q4_K");
static_assert(sizeof(block_q5_K) == 176, "q5_K");
static_assert(sizeof(block_q6_K) == 210, "q6_K");
static_assert(sizeof(block_q3_K) == 110, "q3_K");
static_assert(sizeof(block_iq4_xs) == 136, "iq4_xs");
static_assert(sizeof(block_q8_0) == 34, "q8_0");

// IQ4_NL / IQ4_XS non-linear code book (GGUF format constant; also in the reference at dgpu/dgpu.cu:73)
alignas(16) static const int8_t kvalues_iq4nl[16] = { -127, -104, -83, -65, -49, -35, -22, -10,
                                                        1,   13,   25,  38,  53,  69,  89, 113 };

// grids of the IQ2/IQ3 types: declared only (their decoders are never instantiated here)
extern const uint32_t iq3s_grid[512];
extern const uint32_t iq3xxs_grid[256];
extern const uint8_t  ksigns_iq2xs[128];
extern const uint8_t  kmask_iq2xs[8];
extern const uint64_t iq2xxs_grid[256];
extern const uint64_t iq2xs_grid[512];
extern const uint64_t iq2s_grid[1024];
