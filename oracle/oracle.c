/* TEST INFRASTRUCTURE (oracle): CPU restatement of the reference's verify-path arithmetic. See oracle.h for what is
 * pinned and how. Only tests/, the smoke check and bench.py's CPU-baseline leg load the library built from this file.
 * Build: cc -O2 -ffp-contract=off -shared -fPIC oracle.c -o liboracle.so -lpthread (oracle/Makefile). */
#include "oracle.h"

#include <math.h>
#include <pthread.h>
#include <stdlib.h>
#include <string.h>

#define QK 256
#define QK8 32

static const int8_t kv_iq4nl[16] = { -127, -104, -83, -65, -49, -35, -22, -10, 1, 13, 25, 38, 53, 69, 89, 113 };

size_t orc_block_bytes(int type) {
    switch (type) {
        case ORC_Q4_K: return 144;
        case ORC_Q5_K: return 176;
        case ORC_Q6_K: return 210;
        case ORC_Q3_K: return 110;
        case ORC_IQ4_XS: return 136;
        case ORC_Q8_0: return 34;
        case ORC_F16: return 2;
        case ORC_F32: return 4;
        default: return 0;
    }
}

int orc_block_elems(int type) {
    switch (type) {
        case ORC_Q8_0: return QK8;
        case ORC_F16:
        case ORC_F32: return 1;
        default: return QK;
    }
}

/* IEEE binary16 <-> binary32 from the format definition */
float orc_fp16_to_fp32(uint16_t h) {
    const uint32_t s = (h >> 15) & 1, e = (h >> 10) & 31, m = h & 1023;
    float v;
    if (e == 0) {
        v = ldexpf((float) m, -24);
    } else if (e == 31) {
        v = m ? NAN : INFINITY;
    } else {
        v = ldexpf((float) (m | 1024), (int) e - 25);
    }
    return s ? -v : v;
}

uint16_t orc_fp32_to_fp16(float f) {
    uint32_t x;
    memcpy(&x, &f, 4);
    const uint16_t sign = (uint16_t) ((x >> 16) & 0x8000);
    const uint32_t ax   = x & 0x7fffffffu;
    if (ax >= 0x7f800000u) {
        return sign | (ax > 0x7f800000u ? 0x7e00 : 0x7c00);
    }
    if (ax >= 0x477ff000u) { /* >= 65520: rounds to infinity */
        return sign | 0x7c00;
    }
    if (ax < 0x38800000u) { /* below 2^-14: a binary16 subnormal, value = round(|f| * 2^24) units of 2^-24 */
        float af;
        memcpy(&af, &ax, 4);
        return sign | (uint16_t) nearbyintf(af * 16777216.0f);
    }
    const uint32_t mant = ax & 0x7fffffu;
    uint32_t       h    = ((((ax >> 23) - 127 + 15) & 0x1f) << 10) | (mant >> 13);
    const uint32_t rem  = mant & 0x1fffu;
    if (rem > 0x1000u || (rem == 0x1000u && (h & 1))) {
        h++;
    }
    return sign | (uint16_t) h;
}

static inline float rd16(const uint8_t * p) {
    uint16_t h;
    memcpy(&h, p, 2);
    return orc_fp16_to_fp32(h);
}

void orc_quantize_row_q8K(const float * x, int8_t * q, float * d, int16_t * bsum32, int16_t * bsum16, int64_t K) {
    for (int64_t b = 0; b < K / QK; b++) {
        const float * xb   = x + b * QK;
        int8_t *      qb   = q + b * QK;
        float         amax = 0.0f;
        for (int j = 0; j < QK; j++) {
            const float a = fabsf(xb[j]);
            amax          = a > amax ? a : amax;
        }
        if (amax == 0.0f) {
            memset(qb, 0, QK);
            d[b] = 0.0f;
            continue;
        }
        float mx = 0.0f; /* first element of largest magnitude, with its sign */
        for (int j = 0; j < QK; j++) {
            if (fabsf(xb[j]) == amax) {
                mx = xb[j];
                break;
            }
        }
        const float iscale = -127.0f / mx;
        for (int j = 0; j < QK; j++) {
            long v = lrintf(iscale * xb[j]); /* round half to even */
            qb[j]  = (int8_t) (v > 127 ? 127 : v);
        }
        d[b] = 1.0f / iscale;
    }
    if (bsum32) {
        for (int64_t j = 0; j < K / 32; j++) {
            int s = 0;
            for (int i = 0; i < 32; i++) s += q[32 * j + i];
            bsum32[j] = (int16_t) s;
        }
    }
    if (bsum16) {
        for (int64_t j = 0; j < K / 16; j++) {
            int s = 0;
            for (int i = 0; i < 16; i++) s += q[16 * j + i];
            bsum16[j] = (int16_t) s;
        }
    }
}

void orc_quantize_row_q8_0(const float * x, void * blocks, int64_t K, int mode) {
    uint8_t * y = (uint8_t *) blocks;
    for (int64_t i = 0; i < K / QK8; i++) {
        const float * xb   = x + i * QK8;
        uint8_t *     yb   = y + i * 34;
        float         amax = 0.0f;
        for (int j = 0; j < QK8; j++) {
            const float a = fabsf(xb[j]);
            amax          = a > amax ? a : amax;
        }
        const float    d  = amax / 127.0f;
        const uint16_t dh = orc_fp32_to_fp16(d);
        memcpy(yb, &dh, 2);
        int8_t * qs = (int8_t *) (yb + 2);
        if (mode == ORC_Q8_0_SIMD) {
            const float id = amax != 0.0f ? 127.0f / amax : 0.0f;
            for (int j = 0; j < QK8; j++) qs[j] = (int8_t) lrintf(xb[j] * id);
        } else {
            const float id = d != 0.0f ? 1.0f / d : 0.0f;
            for (int j = 0; j < QK8; j++) qs[j] = (int8_t) roundf(xb[j] * id);
        }
    }
}

/* 6-bit scale / min pair j of a Q4_K / Q5_K super-block (12 packed bytes) */
static void k4_scale_min(int j, const uint8_t * s, int * sc, int * m) {
    if (j < 4) {
        *sc = s[j] & 63;
        *m  = s[j + 4] & 63;
    } else {
        *sc = (s[j + 4] & 0xF) | ((s[j - 4] >> 6) << 4);
        *m  = (s[j + 4] >> 4) | ((s[j] >> 6) << 4);
    }
}

/* the 16 6-bit scales of a Q3_K super-block, minus 32 */
static void q3k_scales(const uint8_t * s, int * sc) {
    for (int i = 0; i < 16; i++) {
        const int lo = i < 8 ? (s[i] & 0xF) : (s[i - 8] >> 4);
        const int hi = (s[8 + (i & 3)] >> (2 * (i >> 2))) & 3;
        sc[i]        = (lo | (hi << 4)) - 32;
    }
}

/* code (integer weight before scaling) of weight i in a super-block, and its integer scale / min */
static int q4k_code(const uint8_t * blk, int i) { return (blk[16 + 32 * (i / 64) + (i % 32)] >> (4 * ((i / 32) & 1))) & 0xF; }
static int q5k_code(const uint8_t * blk, int i) {
    return ((blk[48 + 32 * (i / 64) + (i % 32)] >> (4 * ((i / 32) & 1))) & 0xF) | (((blk[16 + (i % 32)] >> (i / 32)) & 1) << 4);
}
static int q6k_code(const uint8_t * blk, int i) {
    const int b = i / 32, l = i % 32, n = b / 4, g = b % 4;
    const int lo = (blk[64 * n + 32 * (g & 1) + l] >> (4 * (g >> 1))) & 0xF;
    const int hi = (blk[128 + 32 * n + l] >> (2 * g)) & 3;
    return (lo | (hi << 4)) - 32;
}
static int q6k_scale(const uint8_t * blk, int i) {
    const int b = i / 32, l = i % 32, n = b / 4, g = b % 4;
    return (int8_t) blk[192 + 8 * n + 2 * g + (l >= 16)];
}
static int q3k_code(const uint8_t * blk, int i) {
    const int b = i / 32, l = i % 32, n = b / 4, j = b % 4;
    const int q2 = (blk[32 + 32 * n + l] >> (2 * j)) & 3;
    const int hb = (blk[l] >> (4 * n + j)) & 1;
    return q2 - (hb ? 0 : 4);
}
static int iq4xs_scale(const uint8_t * blk, int b) {
    uint16_t sh;
    memcpy(&sh, blk + 2, 2);
    return (((blk[4 + b / 2] >> (4 * (b % 2))) & 0xF) | (((sh >> (2 * b)) & 3) << 4)) - 32;
}
static int iq4xs_code(const uint8_t * blk, int i) {
    const int b = i / 32, l = i % 32;
    const uint8_t v = blk[8 + 16 * b + (l & 15)];
    return kv_iq4nl[l < 16 ? (v & 0xF) : (v >> 4)];
}

void orc_dequantize(int type, const void * blocks, float * y, int64_t n) {
    const uint8_t * p   = (const uint8_t *) blocks;
    const size_t    bs  = orc_block_bytes(type);
    const int       qk  = orc_block_elems(type);
    for (int64_t ib = 0; ib < n / qk; ib++) {
        const uint8_t * blk = p + ib * bs;
        float *         yb  = y + ib * qk;
        switch (type) {
            case ORC_Q8_0: {
                const float d = rd16(blk);
                for (int j = 0; j < QK8; j++) yb[j] = d * (int8_t) blk[2 + j];
            } break;
            case ORC_Q4_K:
            case ORC_Q5_K: {
                const float d = rd16(blk), dmin = rd16(blk + 2);
                for (int i = 0; i < QK; i++) {
                    int sc, m;
                    k4_scale_min(i / 32, blk + 4, &sc, &m);
                    const int q = type == ORC_Q4_K ? q4k_code(blk, i) : q5k_code(blk, i);
                    yb[i]       = d * (float) sc * (float) q - dmin * (float) m;
                }
            } break;
            case ORC_Q6_K: {
                const float d = rd16(blk + 208);
                for (int i = 0; i < QK; i++) yb[i] = d * (float) q6k_scale(blk, i) * (float) q6k_code(blk, i);
            } break;
            case ORC_Q3_K: {
                int sc[16];
                q3k_scales(blk + 96, sc);
                const float d = rd16(blk + 108);
                for (int i = 0; i < QK; i++) yb[i] = d * (float) sc[i / 16] * (float) q3k_code(blk, i);
            } break;
            case ORC_IQ4_XS: {
                const float d = rd16(blk);
                for (int i = 0; i < QK; i++) yb[i] = d * (float) iq4xs_scale(blk, i / 32) * (float) iq4xs_code(blk, i);
            } break;
            case ORC_F16:
                yb[0] = rd16(blk);
                break;
            default:
                break;
        }
    }
}

void orc_row_isums(int type, const void * row, const int8_t * xq, const int16_t * bsum32, int64_t K, int32_t * main_,
                   int32_t * mins) {
    const uint8_t * p  = (const uint8_t *) row;
    const size_t    bs = orc_block_bytes(type);
    if (type == ORC_Q8_0) {
        for (int64_t ib = 0; ib < K / QK8; ib++) {
            const int8_t * w = (const int8_t *) (p + ib * bs + 2);
            int32_t        s = 0;
            for (int j = 0; j < QK8; j++) s += (int32_t) w[j] * xq[ib * QK8 + j];
            main_[ib] = s;
        }
        return;
    }
    for (int64_t sb = 0; sb < K / QK; sb++) {
        const uint8_t * blk = p + sb * bs;
        const int8_t *  x   = xq + sb * QK;
        int32_t         ms = 0, mn = 0;
        switch (type) {
            case ORC_Q4_K:
            case ORC_Q5_K:
                for (int b = 0; b < 8; b++) {
                    int sc, m, dot = 0;
                    k4_scale_min(b, blk + 4, &sc, &m);
                    for (int l = 0; l < 32; l++) {
                        const int i = 32 * b + l;
                        dot += (type == ORC_Q4_K ? q4k_code(blk, i) : q5k_code(blk, i)) * x[i];
                    }
                    ms += sc * dot;
                    mn += m * bsum32[sb * 8 + b];
                }
                break;
            case ORC_Q6_K:
                for (int g = 0; g < 16; g++) {
                    int dot = 0;
                    for (int l = 0; l < 16; l++) dot += q6k_code(blk, 16 * g + l) * x[16 * g + l];
                    ms += q6k_scale(blk, 16 * g) * dot;
                }
                break;
            case ORC_Q3_K: {
                int sc[16];
                q3k_scales(blk + 96, sc);
                for (int g = 0; g < 16; g++) {
                    int dot = 0;
                    for (int l = 0; l < 16; l++) dot += q3k_code(blk, 16 * g + l) * x[16 * g + l];
                    ms += sc[g] * dot;
                }
            } break;
            case ORC_IQ4_XS:
                for (int b = 0; b < 8; b++) {
                    int dot = 0;
                    for (int l = 0; l < 32; l++) dot += iq4xs_code(blk, 32 * b + l) * x[32 * b + l];
                    ms += iq4xs_scale(blk, b) * dot;
                }
                break;
            default:
                break;
        }
        main_[sb] = ms;
        if (mins) {
            mins[sb] = mn;
        }
    }
}

static int supported_weight(int type) {
    return type == ORC_Q4_K || type == ORC_Q5_K || type == ORC_Q6_K || type == ORC_Q3_K || type == ORC_IQ4_XS ||
           type == ORC_Q8_0;
}

int orc_mul_mat(int type, const void * W, int64_t rows, int64_t K, const float * X, int64_t N, double * Y, int q8_mode) {
    if (!supported_weight(type) || K % (type == ORC_Q8_0 ? QK8 : QK) || N < 1) {
        return -1;
    }
    const size_t   bs     = orc_block_bytes(type);
    const int64_t  nblk   = K / orc_block_elems(type);
    const size_t   rowb   = bs * (size_t) nblk;
    int8_t *       xq     = (int8_t *) malloc((size_t) (N * K));
    float *        xd     = (float *) malloc(sizeof(float) * (size_t) (N * nblk));
    int16_t *      bs32   = (int16_t *) malloc(sizeof(int16_t) * (size_t) (N * (K / 32)));
    int32_t *      im     = (int32_t *) malloc(sizeof(int32_t) * (size_t) nblk);
    int32_t *      in     = (int32_t *) malloc(sizeof(int32_t) * (size_t) nblk);
    uint8_t *      qb     = (uint8_t *) malloc((size_t) (K / QK8) * 34);
    for (int64_t t = 0; t < N; t++) {
        if (type == ORC_Q8_0) {
            orc_quantize_row_q8_0(X + t * K, qb, K, q8_mode);
            for (int64_t ib = 0; ib < K / QK8; ib++) {
                memcpy(xq + t * K + ib * QK8, qb + ib * 34 + 2, QK8);
                xd[t * nblk + ib] = rd16(qb + ib * 34);
            }
        } else {
            orc_quantize_row_q8K(X + t * K, xq + t * K, xd + t * nblk, bs32 + t * (K / 32), NULL, K);
        }
    }
    for (int64_t r = 0; r < rows; r++) {
        const uint8_t * row = (const uint8_t *) W + (size_t) r * rowb;
        for (int64_t t = 0; t < N; t++) {
            orc_row_isums(type, row, xq + t * K, bs32 + t * (K / 32), K, im, in);
            double acc = 0.0;
            for (int64_t ib = 0; ib < nblk; ib++) {
                const uint8_t * blk = row + ib * bs;
                const double    xs  = xd[t * nblk + ib];
                double          dw, dmin = 0.0;
                switch (type) {
                    case ORC_Q4_K:
                    case ORC_Q5_K: dw = rd16(blk); dmin = rd16(blk + 2); break;
                    case ORC_Q6_K: dw = rd16(blk + 208); break;
                    case ORC_Q3_K: dw = rd16(blk + 108); break;
                    default: dw = rd16(blk); break; /* IQ4_XS, Q8_0 */
                }
                acc += dw * xs * (double) im[ib];
                if (type == ORC_Q4_K || type == ORC_Q5_K) {
                    acc -= dmin * xs * (double) in[ib];
                }
            }
            Y[t * rows + r] = acc;
        }
    }
    free(xq); free(xd); free(bs32); free(im); free(in); free(qb);
    return 0;
}

struct q80_job {
    const uint8_t *  W;
    const uint8_t *  xqb;
    float *          Y;
    int64_t          rows, nb, N;
    volatile int64_t next;
    pthread_mutex_t  mu;
};

/* rows in dynamic chunks of 16 (the reference's SRV_CHUNK scheduling, patch/srhpm.patch:6301) */
static void * q80_worker(void * arg) {
    struct q80_job * j = (struct q80_job *) arg;
    for (;;) {
        pthread_mutex_lock(&j->mu);
        const int64_t c = j->next++;
        pthread_mutex_unlock(&j->mu);
        const int64_t r0 = c * 16;
        if (r0 >= j->rows) break;
        const int64_t r1 = r0 + 16 < j->rows ? r0 + 16 : j->rows;
        for (int64_t r = r0; r < r1; r++) {
            const uint8_t * w = j->W + (size_t) r * j->nb * 34;
            for (int64_t t = 0; t < j->N; t++) {
                const uint8_t * x      = j->xqb + t * j->nb * 34;
                float           acc[8] = { 0 };
                for (int64_t ib = 0; ib < j->nb; ib++) {
                    const float    d  = rd16(w + ib * 34) * rd16(x + ib * 34);
                    const int8_t * qw = (const int8_t *) (w + ib * 34 + 2);
                    const int8_t * qx = (const int8_t *) (x + ib * 34 + 2);
                    for (int l = 0; l < 8; l++) {
                        const int p = qw[4 * l] * qx[4 * l] + qw[4 * l + 1] * qx[4 * l + 1] +
                                      qw[4 * l + 2] * qx[4 * l + 2] + qw[4 * l + 3] * qx[4 * l + 3];
                        acc[l] = fmaf(d, (float) p, acc[l]);
                    }
                }
                const float s0 = acc[0] + acc[4], s1 = acc[1] + acc[5], s2 = acc[2] + acc[6], s3 = acc[3] + acc[7];
                j->Y[t * j->rows + r] = (s0 + s2) + (s1 + s3);
            }
        }
    }
    return NULL;
}

int orc_mul_mat_q8_0_f32(const void * W, int64_t rows, int64_t K, const float * X, int64_t N, float * Y, int q8_mode,
                         int nth) {
    if (K % QK8 || N < 1 || nth < 1) {
        return -1;
    }
    const int64_t nb  = K / QK8;
    uint8_t *     xqb = (uint8_t *) malloc((size_t) (N * nb * 34));
    for (int64_t t = 0; t < N; t++) orc_quantize_row_q8_0(X + t * K, xqb + t * nb * 34, K, q8_mode);
    struct q80_job job = { (const uint8_t *) W, xqb, Y, rows, nb, N, 0, PTHREAD_MUTEX_INITIALIZER };
    pthread_t *    th  = (pthread_t *) malloc(sizeof(pthread_t) * (size_t) nth);
    for (int i = 1; i < nth; i++) pthread_create(&th[i], NULL, q80_worker, &job);
    q80_worker(&job);
    for (int i = 1; i < nth; i++) pthread_join(th[i], NULL);
    free(th);
    free(xqb);
    return 0;
}

int orc_attention(const float * q, int64_t DK, int64_t N, int64_t H, int kv_type, const void * k, const void * v,
                  int64_t DV, int64_t L, int64_t Hkv, const uint16_t * mask, const float * sinks, float scale,
                  float max_bias, float softcap, int q8_mode, double * dst) {
    if (Hkv <= 0 || H % Hkv || (kv_type != ORC_F16 && kv_type != ORC_Q8_0) ||
        (kv_type == ORC_Q8_0 && (DK % QK8 || DV % QK8))) {
        return -1;
    }
    const int64_t G      = H / Hkv;
    const size_t  krow   = kv_type == ORC_Q8_0 ? (size_t) (DK / QK8) * 34 : (size_t) DK * 2;
    const size_t  vrow   = kv_type == ORC_Q8_0 ? (size_t) (DV / QK8) * 34 : (size_t) DV * 2;
    const float   sc     = softcap != 0.0f ? scale / softcap : scale;
    const uint32_t nhl2  = 1u << (uint32_t) floor(log2((double) H));
    const double  m0     = pow(2.0, -(double) max_bias / nhl2);
    const double  m1     = pow(2.0, -((double) max_bias / 2.0) / nhl2);
    double *      s      = (double *) malloc(sizeof(double) * (size_t) L);
    float *       kf     = (float *) malloc(sizeof(float) * (size_t) (DK > DV ? DK : DV));
    uint8_t *     qq     = (uint8_t *) malloc((size_t) (DK / QK8 + 1) * 34);
    for (int64_t h = 0; h < H; h++) {
        const int64_t g     = h / G;
        const double  slope = max_bias > 0.0f ? (h < (int64_t) nhl2 ? pow(m0, (double) (h + 1))
                                                                      : pow(m1, (double) (2 * (h - nhl2) + 1)))
                                              : 1.0;
        for (int64_t t = 0; t < N; t++) {
            const float * qr = q + (h * N + t) * DK;
            if (kv_type == ORC_Q8_0) {
                orc_quantize_row_q8_0(qr, qq, DK, q8_mode);
            }
            double mx = -INFINITY;
            for (int64_t j = 0; j < L; j++) {
                const uint8_t * kr = (const uint8_t *) k + (size_t) (g * L + j) * krow;
                double          dot = 0.0;
                if (kv_type == ORC_Q8_0) {
                    for (int64_t ib = 0; ib < DK / QK8; ib++) {
                        int32_t isum = 0;
                        for (int l = 0; l < QK8; l++) {
                            isum += (int32_t) (int8_t) kr[ib * 34 + 2 + l] * (int8_t) qq[ib * 34 + 2 + l];
                        }
                        dot += (double) rd16(kr + ib * 34) * (double) rd16(qq + ib * 34) * (double) isum;
                    }
                } else {
                    for (int64_t d = 0; d < DK; d++) dot += (double) qr[d] * (double) rd16(kr + 2 * d);
                }
                double sv = dot * sc;
                if (softcap != 0.0f) {
                    sv = softcap * tanh(sv);
                }
                if (mask) {
                    sv += slope * (double) orc_fp16_to_fp32(mask[t * L + j]);
                }
                s[j] = sv;
                mx   = sv > mx ? sv : mx;
            }
            double * out = dst + (t * H + h) * DV;
            for (int64_t d = 0; d < DV; d++) out[d] = 0.0;
            double sum = 0.0;
            if (mx != -INFINITY) {
                for (int64_t j = 0; j < L; j++) {
                    if (s[j] == -INFINITY) continue;
                    const double p = exp(s[j] - mx);
                    sum += p;
                    orc_dequantize(kv_type, (const uint8_t *) v + (size_t) (g * L + j) * vrow, kf, DV);
                    for (int64_t d = 0; d < DV; d++) out[d] += p * (double) kf[d];
                }
            }
            if (sinks) {
                const double sk = sinks[h];
                if (mx == -INFINITY || sk > mx) {
                    const double r = mx == -INFINITY ? 0.0 : exp(mx - sk);
                    for (int64_t d = 0; d < DV; d++) out[d] *= r;
                    sum = sum * r + 1.0;
                } else {
                    sum += exp(sk - mx);
                }
            }
            const double inv = sum == 0.0 ? 0.0 : 1.0 / sum;
            for (int64_t d = 0; d < DV; d++) out[d] *= inv;
        }
    }
    free(s); free(kf); free(qq);
    return 0;
}

int orc_attention_partial(const float * q, int64_t DK, int64_t N, int64_t H, int kv_type, const void * k,
                          const void * v, int64_t DV, int64_t L, int64_t Hkv, int64_t t0, int64_t t1,
                          const uint16_t * mask, float scale, float max_bias, float softcap, int q8_mode,
                          double * rec_m, double * rec_s, double * rec_acc) {
    if (Hkv <= 0 || H % Hkv || (kv_type != ORC_F16 && kv_type != ORC_Q8_0) ||
        (kv_type == ORC_Q8_0 && (DK % QK8 || DV % QK8)) || t0 < 0 || t1 < t0 || t1 > L) {
        return -1;
    }
    const int64_t  G    = H / Hkv;
    const size_t   krow = kv_type == ORC_Q8_0 ? (size_t) (DK / QK8) * 34 : (size_t) DK * 2;
    const size_t   vrow = kv_type == ORC_Q8_0 ? (size_t) (DV / QK8) * 34 : (size_t) DV * 2;
    const float    sc   = softcap != 0.0f ? scale / softcap : scale;
    const uint32_t nhl2 = 1u << (uint32_t) floor(log2((double) H));
    const double   m0   = pow(2.0, -(double) max_bias / nhl2);
    const double   m1   = pow(2.0, -((double) max_bias / 2.0) / nhl2);
    const int64_t  n    = t1 - t0;
    double *       s    = (double *) malloc(sizeof(double) * (size_t) (n > 0 ? n : 1));
    float *        vf   = (float *) malloc(sizeof(float) * (size_t) (DK > DV ? DK : DV));
    uint8_t *      qq   = (uint8_t *) malloc((size_t) (DK / QK8 + 1) * 34);
    for (int64_t h = 0; h < H; h++) {
        const int64_t g     = h / G;
        const double  slope = max_bias > 0.0f ? (h < (int64_t) nhl2 ? pow(m0, (double) (h + 1))
                                                                      : pow(m1, (double) (2 * (h - nhl2) + 1)))
                                              : 1.0;
        for (int64_t t = 0; t < N; t++) {
            const float * qr = q + (h * N + t) * DK;
            if (kv_type == ORC_Q8_0) {
                orc_quantize_row_q8_0(qr, qq, DK, q8_mode);
            }
            double mx = -INFINITY;
            for (int64_t j = 0; j < n; j++) {
                const uint8_t * kr  = (const uint8_t *) k + (size_t) (g * L + t0 + j) * krow;
                double          dot = 0.0;
                if (kv_type == ORC_Q8_0) {
                    for (int64_t ib = 0; ib < DK / QK8; ib++) {
                        int32_t isum = 0;
                        for (int l = 0; l < QK8; l++) {
                            isum += (int32_t) (int8_t) kr[ib * 34 + 2 + l] * (int8_t) qq[ib * 34 + 2 + l];
                        }
                        dot += (double) rd16(kr + ib * 34) * (double) rd16(qq + ib * 34) * (double) isum;
                    }
                } else {
                    for (int64_t d = 0; d < DK; d++) dot += (double) qr[d] * (double) rd16(kr + 2 * d);
                }
                double sv = dot * sc;
                if (softcap != 0.0f) {
                    sv = softcap * tanh(sv);
                }
                if (mask) {
                    sv += slope * (double) orc_fp16_to_fp32(mask[t * L + t0 + j]);
                }
                s[j] = sv;
                mx   = sv > mx ? sv : mx;
            }
            const int64_t row = h * N + t;
            double *      acc = rec_acc + row * DV;
            for (int64_t d = 0; d < DV; d++) acc[d] = 0.0;
            double sum = 0.0;
            if (mx != -INFINITY) {
                for (int64_t j = 0; j < n; j++) {
                    if (s[j] == -INFINITY) continue;
                    const double p = exp(s[j] - mx);
                    sum += p;
                    orc_dequantize(kv_type, (const uint8_t *) v + (size_t) (g * L + t0 + j) * vrow, vf, DV);
                    for (int64_t d = 0; d < DV; d++) acc[d] += p * (double) vf[d];
                }
            }
            rec_m[row] = mx;
            rec_s[row] = sum;
        }
    }
    free(s); free(vf); free(qq);
    return 0;
}

int orc_attention_merge(int64_t n_parts, int64_t N, int64_t H, int64_t DV, const double * rec_m,
                        const double * rec_s, const double * rec_acc, const float * sinks, double * dst) {
    if (n_parts < 1 || N < 1 || H < 1 || DV < 1) {
        return -1;
    }
    const int64_t rows = H * N;
    for (int64_t h = 0; h < H; h++) {
        for (int64_t t = 0; t < N; t++) {
            const int64_t row = h * N + t;
            double *      out = dst + (t * H + h) * DV;
            double        Mf = -INFINITY, Sf = 0.0;
            for (int64_t d = 0; d < DV; d++) out[d] = 0.0;
            for (int64_t c = 0; c < n_parts; c++) {
                const double sc = rec_s[c * rows + row];
                if (sc == 0.0) continue;
                const double   mc = rec_m[c * rows + row];
                const double   Mn = Mf > mc ? Mf : mc;
                const double   so = Mf == -INFINITY ? 0.0 : exp(Mf - Mn), sn = exp(mc - Mn);
                const double * pa = rec_acc + (c * rows + row) * DV;
                for (int64_t d = 0; d < DV; d++) out[d] = out[d] * so + pa[d] * sn;
                Sf = Sf * so + sc * sn;
                Mf = Mn;
            }
            if (sinks) {
                const double sk = sinks[h];
                if (Mf == -INFINITY || sk > Mf) {
                    const double r = Mf == -INFINITY ? 0.0 : exp(Mf - sk);
                    for (int64_t d = 0; d < DV; d++) out[d] *= r;
                    Sf = Sf * r + 1.0;
                } else {
                    Sf += exp(sk - Mf);
                }
            }
            const double inv = Sf == 0.0 ? 0.0 : 1.0 / Sf;
            for (int64_t d = 0; d < DV; d++) out[d] *= inv;
        }
    }
    return 0;
}

static int32_t argmax_row(const float * lg, int64_t n) {
    int64_t best = 0;
    for (int64_t i = 1; i < n; i++) {
        if (lg[i] > lg[best]) best = i;
    }
    return (int32_t) best;
}

int orc_accept(const float * logits, int64_t n_vocab, const int32_t * draft, int n_draft, float relax,
               int32_t * out_ids) {
    int n = 0, i = 0;
    for (; i < n_draft; i++) {
        const float * lg = logits + (int64_t) i * n_vocab;
        int32_t       id = argmax_row(lg, n_vocab);
        if (relax > 0.0f && draft[i] != id && draft[i] >= 0 && draft[i] < n_vocab) {
            if (lg[id] - lg[draft[i]] <= relax) {
                id = draft[i];
            }
        }
        out_ids[n++] = id;
        if (draft[i] != id) {
            return n;
        }
    }
    out_ids[n++] = argmax_row(logits + (int64_t) i * n_vocab, n_vocab);
    return n;
}

/* ---- input generation: round-to-nearest weight quantizers -------------------------------------------------------
 * The inverse of the block decoders above, with per-block scales from each block's range and no search. They only
 * make valid GGUF blocks of a given f32 matrix for the CPU reference timings (the reference's own quantizers are
 * upstream ggml code, absent here); nothing is pinned to them. */

static uint16_t f16_of(float f, float * back) {
    const uint16_t h = orc_fp32_to_fp16(f);
    *back            = orc_fp16_to_fp32(h);
    return h;
}

static int clampi(long v, int lo, int hi) { return v < lo ? lo : v > hi ? hi : (int) v; }

static void put16(uint8_t * p, uint16_t h) { memcpy(p, &h, 2); }

/* Q4_K / Q5_K: x = d sc q - dmin m per 32 weights, q in 0..nq */
static void rtn_k45(const float * x, uint8_t * blk, int q5) {
    const int nq = q5 ? 31 : 15;
    float     scale[8], mn[8], smax = 0.0f, mmax = 0.0f;
    for (int b = 0; b < 8; b++) {
        float lo = x[32 * b], hi = x[32 * b];
        for (int l = 1; l < 32; l++) {
            lo = x[32 * b + l] < lo ? x[32 * b + l] : lo;
            hi = x[32 * b + l] > hi ? x[32 * b + l] : hi;
        }
        mn[b]    = lo < 0.0f ? -lo : 0.0f;
        scale[b] = (hi + mn[b]) / (float) nq;
        smax     = scale[b] > smax ? scale[b] : smax;
        mmax     = mn[b] > mmax ? mn[b] : mmax;
    }
    float d, dmin;
    put16(blk, f16_of(smax / 63.0f, &d));
    put16(blk + 2, f16_of(mmax / 63.0f, &dmin));
    uint8_t * s = blk + 4;
    memset(s, 0, 12);
    uint8_t * qh = blk + 16;
    uint8_t * qs = blk + (q5 ? 48 : 16);
    if (q5) memset(qh, 0, 32);
    memset(qs, 0, 128);
    for (int b = 0; b < 8; b++) {
        const int sc = d > 0.0f ? clampi(lrintf(scale[b] / d), 0, 63) : 0;
        const int m  = dmin > 0.0f ? clampi(lrintf(mn[b] / dmin), 0, 63) : 0;
        if (b < 4) {
            s[b] |= (uint8_t) sc;
            s[b + 4] |= (uint8_t) m;
        } else {
            s[b + 4] = (uint8_t) ((sc & 0xF) | ((m & 0xF) << 4));
            s[b - 4] |= (uint8_t) ((sc >> 4) << 6);
            s[b] |= (uint8_t) ((m >> 4) << 6);
        }
        const float step = d * (float) sc, off = dmin * (float) m;
        for (int l = 0; l < 32; l++) {
            const int i = 32 * b + l;
            const int q = step > 0.0f ? clampi(lrintf((x[i] + off) / step), 0, nq) : 0;
            qs[32 * (b / 2) + l] |= (uint8_t) ((q & 0xF) << (4 * (b & 1)));
            if (q5) qh[l] |= (uint8_t) (((q >> 4) & 1) << b);
        }
    }
}

/* Q6_K: x = d sc q per 16 weights, q in -32..31, int8 sc */
static void rtn_q6k(const float * x, uint8_t * blk) {
    float scale[16], smax = 0.0f;
    for (int g = 0; g < 16; g++) {
        float a = 0.0f;
        for (int l = 0; l < 16; l++) a = fabsf(x[16 * g + l]) > a ? fabsf(x[16 * g + l]) : a;
        scale[g] = a / 31.0f;
        smax     = scale[g] > smax ? scale[g] : smax;
    }
    float d;
    put16(blk + 208, f16_of(smax / 127.0f, &d));
    memset(blk, 0, 192);
    for (int g = 0; g < 16; g++) {
        const int sc = d > 0.0f ? clampi(lrintf(scale[g] / d), -128, 127) : 0;
        blk[192 + g] = (uint8_t) (int8_t) sc;
        const float step = d * (float) sc;
        for (int l16 = 0; l16 < 16; l16++) {
            const int i = 16 * g + l16, b = i / 32, l = i % 32, n = b / 4, j = b % 4;
            const int q = (step != 0.0f ? clampi(lrintf(x[i] / step), -32, 31) : 0) + 32;
            blk[64 * n + 32 * (j & 1) + l] |= (uint8_t) ((q & 0xF) << (4 * (j >> 1)));
            blk[128 + 32 * n + l] |= (uint8_t) (((q >> 4) & 3) << (2 * j));
        }
    }
}

/* Q3_K: x = d sc q per 16 weights, q in -4..3, sc in -32..31 */
static void rtn_q3k(const float * x, uint8_t * blk) {
    float scale[16], smax = 0.0f;
    for (int g = 0; g < 16; g++) {
        float a = 0.0f;
        for (int l = 0; l < 16; l++) a = fabsf(x[16 * g + l]) > a ? fabsf(x[16 * g + l]) : a;
        scale[g] = a / 4.0f;
        smax     = scale[g] > smax ? scale[g] : smax;
    }
    float d;
    put16(blk + 108, f16_of(smax / 31.0f, &d));
    memset(blk, 0, 108);
    uint8_t * s = blk + 96;
    for (int g = 0; g < 16; g++) {
        const int sc = d > 0.0f ? clampi(lrintf(scale[g] / d), -32, 31) : 0;
        const int u  = sc + 32;
        if (g < 8) {
            s[g] |= (uint8_t) (u & 0xF);
        } else {
            s[g - 8] |= (uint8_t) ((u & 0xF) << 4);
        }
        s[8 + (g & 3)] |= (uint8_t) (((u >> 4) & 3) << (2 * (g >> 2)));
        const float step = d * (float) sc;
        for (int l16 = 0; l16 < 16; l16++) {
            const int i = 16 * g + l16, b = i / 32, l = i % 32, n = b / 4, j = b % 4;
            const int q = step != 0.0f ? clampi(lrintf(x[i] / step), -4, 3) : 0;
            const int hb = q >= 0, q2 = hb ? q : q + 4;
            blk[32 + 32 * n + l] |= (uint8_t) (q2 << (2 * j));
            blk[l] |= (uint8_t) (hb << (4 * n + j));
        }
    }
}

/* IQ4_XS: x = d ls kvalue per 32 weights, ls in -32..31, the nearest of the 16 non-linear values */
static void rtn_iq4xs(const float * x, uint8_t * blk) {
    float scale[8], smax = 0.0f;
    for (int b = 0; b < 8; b++) {
        float a = 0.0f;
        for (int l = 0; l < 32; l++) a = fabsf(x[32 * b + l]) > a ? fabsf(x[32 * b + l]) : a;
        scale[b] = a / 127.0f;
        smax     = scale[b] > smax ? scale[b] : smax;
    }
    float d;
    put16(blk, f16_of(smax / 31.0f, &d));
    memset(blk + 2, 0, 134);
    uint16_t sh = 0;
    for (int b = 0; b < 8; b++) {
        const int ls = d > 0.0f ? clampi(lrintf(scale[b] / d), -32, 31) : 0;
        const int u  = ls + 32;
        blk[4 + b / 2] |= (uint8_t) ((u & 0xF) << (4 * (b % 2)));
        sh |= (uint16_t) (((u >> 4) & 3) << (2 * b));
        const float step = d * (float) ls;
        for (int l = 0; l < 32; l++) {
            const float v = step != 0.0f ? x[32 * b + l] / step : 0.0f;
            int         best = 0;
            for (int k = 1; k < 16; k++) {
                if (fabsf(v - (float) kv_iq4nl[k]) < fabsf(v - (float) kv_iq4nl[best])) best = k;
            }
            blk[8 + 16 * b + (l & 15)] |= (uint8_t) (best << (4 * (l >= 16)));
        }
    }
    put16(blk + 2, sh);
}

int64_t orc_quantize_rtn(int type, const float * x, void * out, int64_t n) {
    const int    qk = orc_block_elems(type);
    const size_t bs = orc_block_bytes(type);
    if (qk <= 1 || n % qk) return -1;
    uint8_t * p = (uint8_t *) out;
    for (int64_t ib = 0; ib < n / qk; ib++) {
        const float * xb  = x + ib * qk;
        uint8_t *     blk = p + ib * bs;
        switch (type) {
            case ORC_Q8_0: orc_quantize_row_q8_0(xb, blk, QK8, ORC_Q8_0_REF); break;
            case ORC_Q4_K: rtn_k45(xb, blk, 0); break;
            case ORC_Q5_K: rtn_k45(xb, blk, 1); break;
            case ORC_Q6_K: rtn_q6k(xb, blk); break;
            case ORC_Q3_K: rtn_q3k(xb, blk); break;
            case ORC_IQ4_XS: rtn_iq4xs(xb, blk); break;
            default: return -1;
        }
    }
    return (int64_t) (n / qk * bs);
}
