// Host-side weight quantizers: f32 rows -> GGUF-packed blocks of Q4_K, Q5_K, Q6_K, Q3_K, IQ4_XS and Q8_0. This is
// the data-format producer that ggml exposes as ggml_quantize_chunk (upstream ggml-quants.c, not vendored by the
// reference); the verify path consumes the packed bytes unchanged. The block layouts are the GGUF ones. The scale
// searches are this library's own (least-squares refinement of a max-based start); they are not bit-identical to
// ggml's quantizers, which parity of the verify path does not need: both the CUDA path and the checker read the
// same packed bytes.
#include "srhpm_b200.h"

#include <algorithm>
#include <cmath>
#include <cstdint>
#include <cstring>
#include <thread>
#include <vector>

#include "fp16_host.h"

namespace {

constexpr int QK  = 256;
constexpr int QK8 = 32;

const int8_t kIq4nl[16] = { -127, -104, -83, -65, -49, -35, -22, -10, 1, 13, 25, 38, 53, 69, 89, 113 };

inline int nearest_int(float v) { return (int) lrintf(v); }

// Fit x ~= scale * L - mn with L in [0, nmax] (mn >= 0) by alternating code assignment and a 2x2 least-squares
// solve, starting from the min/max fit and a few perturbed scales. Returns scale, writes mn and the codes.
float fit_affine(const float * x, int n, int nmax, float * mn_out, uint8_t * L) {
    float lo = x[0], hi = x[0];
    for (int i = 1; i < n; i++) {
        lo = std::min(lo, x[i]);
        hi = std::max(hi, x[i]);
    }
    if (lo > 0) lo = 0;
    if (hi == lo) {
        for (int i = 0; i < n; i++) L[i] = 0;
        *mn_out = -lo;
        return 0.f;
    }
    float best_err = INFINITY, best_s = 0, best_m = 0;
    std::vector<uint8_t> Lt(n);
    for (int step = -6; step <= 6; step++) {
        float s  = (hi - lo) / (nmax + 0.1f * step);
        float mn = -lo;
        for (int iter = 0; iter < 2; iter++) {
            if (s <= 0) break;
            double sl = 0, sll = 0, sx = 0, slx = 0;
            for (int i = 0; i < n; i++) {
                int l = nearest_int((x[i] + mn) / s);
                l     = std::max(0, std::min(nmax, l));
                Lt[i] = (uint8_t) l;
                sl += l; sll += (double) l * l; sx += x[i]; slx += (double) l * x[i];
            }
            const double det = n * sll - sl * sl;
            if (det <= 0) break;
            double ns = (n * slx - sl * sx) / det;
            double nm = (sl * slx - sll * sx) / det;  // x ~= ns*L - nm
            if (nm < 0) {  // min constrained at 0: x ~= ns * L
                nm = 0;
                ns = sll > 0 ? slx / sll : 0;
            }
            s  = (float) ns;
            mn = (float) nm;
        }
        if (s <= 0) continue;
        float err = 0;
        for (int i = 0; i < n; i++) {
            int l = std::max(0, std::min(nmax, nearest_int((x[i] + mn) / s)));
            const float e = s * l - mn - x[i];
            err += e * e;
        }
        if (err < best_err) {
            best_err = err;
            best_s   = s;
            best_m   = mn;
        }
    }
    *mn_out = best_m;
    for (int i = 0; i < n; i++) {
        L[i] = (uint8_t) std::max(0, std::min(nmax, best_s > 0 ? nearest_int((x[i] + best_m) / best_s) : 0));
    }
    return best_s;
}

// Fit x ~= scale * L with L in [-nneg, npos] (signed codes): scale from the signed extreme, refined by least squares.
float fit_symmetric(const float * x, int n, int nneg, int npos) {
    float amax = 0, mx = 0;
    for (int i = 0; i < n; i++) {
        if (fabsf(x[i]) > amax) {
            amax = fabsf(x[i]);
            mx   = x[i];
        }
    }
    if (amax == 0) return 0.f;
    float best_s = 0, best_err = INFINITY;
    for (int step = -4; step <= 4; step++) {
        float s = -mx / (nneg + 0.1f * step);  // the extreme lands on -nneg
        for (int iter = 0; iter < 2; iter++) {
            double sl = 0, sll = 0;
            for (int i = 0; i < n; i++) {
                const int l = std::max(-nneg, std::min(npos, nearest_int(x[i] / s)));
                sl += (double) l * x[i];
                sll += (double) l * l;
            }
            if (sll <= 0) break;
            s = (float) (sl / sll);
        }
        float err = 0;
        for (int i = 0; i < n; i++) {
            const int l = std::max(-nneg, std::min(npos, nearest_int(x[i] / s)));
            const float e = s * l - x[i];
            err += e * e;
        }
        if (err < best_err) {
            best_err = err;
            best_s   = s;
        }
    }
    return best_s;
}

void put16(uint8_t * p, float v) {
    const uint16_t h = srhpm_host_fp32_to_fp16(v);
    memcpy(p, &h, 2);
}
float get16(const uint8_t * p) {
    uint16_t h;
    memcpy(&h, p, 2);
    return srhpm_host_fp16_to_fp32(h);
}

void pack_k4_scales(const int * sc, const int * m, uint8_t * s) {
    for (int j = 0; j < 4; j++) {
        s[j]     = (uint8_t) ((sc[j] & 63) | ((sc[j + 4] >> 4) << 6));
        s[j + 4] = (uint8_t) ((m[j] & 63) | ((m[j + 4] >> 4) << 6));
        s[j + 8] = (uint8_t) ((sc[j + 4] & 0xF) | ((m[j + 4] & 0xF) << 4));
    }
}

// Q4_K (nmax 15) and Q5_K (nmax 31): 8 blocks of 32 with 6-bit (scale, min) under f16 (d, dmin)
void quant_q45k(const float * x, uint8_t * blk, bool q5) {
    const int nmax = q5 ? 31 : 15;
    float     s[8], m[8];
    uint8_t   L[QK];
    for (int b = 0; b < 8; b++) s[b] = fit_affine(x + 32 * b, 32, nmax, &m[b], L + 32 * b);
    float smax = 0, mmax = 0;
    for (int b = 0; b < 8; b++) {
        smax = std::max(smax, s[b]);
        mmax = std::max(mmax, m[b]);
    }
    put16(blk + 0, smax / 63.f);
    put16(blk + 2, mmax / 63.f);
    const float d = get16(blk + 0), dmin = get16(blk + 2);
    int ls[8], lm[8];
    for (int b = 0; b < 8; b++) {
        ls[b] = d > 0 ? std::max(0, std::min(63, nearest_int(s[b] / d))) : 0;
        lm[b] = dmin > 0 ? std::max(0, std::min(63, nearest_int(m[b] / dmin))) : 0;
    }
    pack_k4_scales(ls, lm, blk + 4);
    for (int b = 0; b < 8; b++) {
        const float ds = d * ls[b], dm = dmin * lm[b];
        for (int l = 0; l < 32; l++) {
            L[32 * b + l] = (uint8_t) (ds > 0 ? std::max(0, std::min(nmax, nearest_int((x[32 * b + l] + dm) / ds))) : 0);
        }
    }
    uint8_t * qh = blk + 16;
    uint8_t * qs = blk + (q5 ? 48 : 16);
    if (q5) memset(qh, 0, 32);
    for (int p = 0; p < 4; p++) {
        for (int l = 0; l < 32; l++) {
            const int a = L[64 * p + l], c = L[64 * p + 32 + l];
            qs[32 * p + l] = (uint8_t) ((a & 0xF) | ((c & 0xF) << 4));
            if (q5) {
                qh[l] |= (uint8_t) (((a >> 4) & 1) << (2 * p));
                qh[l] |= (uint8_t) (((c >> 4) & 1) << (2 * p + 1));
            }
        }
    }
}

// Q6_K: 16 groups of 16, signed 6-bit codes (-32..31), int8 group scales under an f16 d
void quant_q6k(const float * x, uint8_t * blk) {
    float s[16], amax = 0, smax = 0;
    for (int g = 0; g < 16; g++) {
        s[g] = fit_symmetric(x + 16 * g, 16, 32, 31);
        if (fabsf(s[g]) > amax) {
            amax = fabsf(s[g]);
            smax = s[g];
        }
    }
    put16(blk + 208, amax > 0 ? -smax / 128.f : 0.f);
    const float d = get16(blk + 208);
    int8_t * sc = (int8_t *) (blk + 192);
    for (int g = 0; g < 16; g++) sc[g] = (int8_t) (d != 0 ? std::max(-128, std::min(127, nearest_int(s[g] / d))) : 0);
    uint8_t L[QK];
    for (int i = 0; i < QK; i++) {
        const float ds = d * sc[i / 16];
        L[i] = (uint8_t) ((ds != 0 ? std::max(-32, std::min(31, nearest_int(x[i] / ds))) : 0) + 32);
    }
    memset(blk, 0, 192);
    for (int n = 0; n < 2; n++) {
        for (int g = 0; g < 4; g++) {
            for (int l = 0; l < 32; l++) {
                const int v = L[128 * n + 32 * g + l];
                blk[64 * n + 32 * (g & 1) + l] |= (uint8_t) ((v & 0xF) << (4 * (g >> 1)));
                blk[128 + 32 * n + l] |= (uint8_t) ((v >> 4) << (2 * g));
            }
        }
    }
}

// Q3_K: 16 groups of 16, codes -4..3 (2 low bits + high bit), 6-bit signed scales under an f16 d
void quant_q3k(const float * x, uint8_t * blk) {
    float s[16], amax = 0, smax = 0;
    for (int g = 0; g < 16; g++) {
        s[g] = fit_symmetric(x + 16 * g, 16, 4, 3);
        if (fabsf(s[g]) > amax) {
            amax = fabsf(s[g]);
            smax = s[g];
        }
    }
    put16(blk + 108, amax > 0 ? -smax / 32.f : 0.f);
    const float d = get16(blk + 108);
    int ls[16];
    for (int g = 0; g < 16; g++) ls[g] = d != 0 ? std::max(-32, std::min(31, nearest_int(s[g] / d))) : 0;
    uint8_t * sc = blk + 96;
    memset(sc, 0, 12);
    for (int i = 0; i < 16; i++) {
        const int v = ls[i] + 32;
        if (i < 8) sc[i] |= (uint8_t) (v & 0xF);
        else       sc[i - 8] |= (uint8_t) ((v & 0xF) << 4);
        sc[8 + (i & 3)] |= (uint8_t) (((v >> 4) & 3) << (2 * (i >> 2)));
    }
    memset(blk, 0, 96);
    for (int i = 0; i < QK; i++) {
        const float ds = d * ls[i / 16];
        const int   l  = (ds != 0 ? std::max(-4, std::min(3, nearest_int(x[i] / ds))) : 0) + 4;
        const int   b = i / 32, ll = i % 32, n = b / 4, j = b % 4;
        blk[32 + 32 * n + ll] |= (uint8_t) ((l & 3) << (2 * j));
        if (l & 4) blk[ll] |= (uint8_t) (1 << (4 * n + j));
    }
}

// nearest code-book entry: the code book is sorted, so count the midpoints below v (binary search)
int iq4_nearest(float v) {
    static const float mid[15] = { -115.5f, -93.5f, -74.0f, -57.0f, -42.0f, -28.5f, -16.0f, -4.5f,
                                   7.0f,    19.0f,  31.5f,  45.5f,  61.0f,  79.0f,  101.0f };
    int lo = 0, hi = 15;  // answer in [lo, hi]
    while (lo < hi) {
        const int m = (lo + hi) >> 1;
        if (v > mid[m]) lo = m + 1;
        else hi = m;
    }
    return lo;
}

// IQ4_XS: 8 blocks of 32 with a non-linear 4-bit code book, 6-bit signed block scales under an f16 d
void quant_iq4xs(const float * x, uint8_t * blk) {
    float s[8], amax = 0, smax = 0;
    for (int b = 0; b < 8; b++) {
        const float * xb = x + 32 * b;
        float bm = 0, bv = 0;
        for (int l = 0; l < 32; l++) {
            if (fabsf(xb[l]) > bm) {
                bm = fabsf(xb[l]);
                bv = xb[l];
            }
        }
        float best_s = 0, best_e = INFINITY;
        for (int step = -8; step <= 8 && bm > 0; step += 4) {
            const float s0 = bv / (kIq4nl[0] + 2.0f * step);  // the extreme on (or near) the -127 code
            double sl = 0, sll = 0;
            for (int l = 0; l < 32; l++) {
                const int q = kIq4nl[iq4_nearest(xb[l] / s0)];
                sl += (double) q * xb[l];
                sll += (double) q * q;
            }
            const float s1 = sll > 0 ? (float) (sl / sll) : s0;
            float e = 0;
            for (int l = 0; l < 32; l++) {
                const float r = s1 * kIq4nl[iq4_nearest(xb[l] / s1)] - xb[l];
                e += r * r;
            }
            if (e < best_e) {
                best_e = e;
                best_s = s1;
            }
        }
        s[b] = best_s;
        if (fabsf(best_s) > amax) {
            amax = fabsf(best_s);
            smax = best_s;
        }
    }
    put16(blk, amax > 0 ? -smax / 32.f : 0.f);
    const float d = get16(blk);
    uint16_t sh = 0;
    memset(blk + 4, 0, 4);
    for (int b = 0; b < 8; b++) {
        const int ls = (d != 0 ? std::max(-32, std::min(31, nearest_int(s[b] / d))) : 0);
        const int v  = ls + 32;
        blk[4 + b / 2] |= (uint8_t) ((v & 0xF) << (4 * (b % 2)));
        sh |= (uint16_t) (((v >> 4) & 3) << (2 * b));
        const float ds = d * ls;
        for (int j = 0; j < 16; j++) {
            const int lo = ds != 0 ? iq4_nearest(x[32 * b + j] / ds) : 8;
            const int hi = ds != 0 ? iq4_nearest(x[32 * b + 16 + j] / ds) : 8;
            blk[8 + 16 * b + j] = (uint8_t) (lo | (hi << 4));
        }
    }
    memcpy(blk + 2, &sh, 2);
}

// Q8_0: d = amax / 127 (f16), q = round(x / d)
void quant_q8_0(const float * x, uint8_t * blk) {
    float amax = 0;
    for (int j = 0; j < QK8; j++) amax = std::max(amax, fabsf(x[j]));
    const float d  = amax / 127.f;
    const float id = d != 0 ? 1.f / d : 0.f;
    put16(blk, d);
    for (int j = 0; j < QK8; j++) blk[2 + j] = (uint8_t) (int8_t) roundf(x[j] * id);
}

}  // namespace

extern "C" size_t srhpm_quantize_chunk(int type, const float * src, void * dst, int64_t start, int64_t nrows,
                                       int64_t n_per_row, const float * imatrix) {
    (void) imatrix;  // uniform importance (the verify-GEMM sweep quantizes IQ4_XS with a uniform matrix)
    const int    qk = srhpm_blck_size(type);
    const size_t bs = srhpm_type_size(type);
    if (qk <= 0 || n_per_row % qk || start % n_per_row || nrows < 0) {
        return 0;
    }
    const int64_t nblk  = nrows * (n_per_row / qk);
    const int64_t blk0  = start / qk;
    uint8_t *     out   = (uint8_t *) dst + (size_t) blk0 * bs;
    const float * in    = src + start;
    const unsigned hw   = std::max(1u, std::min(32u, std::thread::hardware_concurrency()));
    const int64_t per   = (nblk + hw - 1) / hw;
    auto work = [&](int64_t b0, int64_t b1) {
        for (int64_t b = b0; b < b1; b++) {
            const float * xb = in + b * qk;
            uint8_t *     yb = out + (size_t) b * bs;
            switch (type) {
                case SRHPM_TYPE_Q4_K: quant_q45k(xb, yb, false); break;
                case SRHPM_TYPE_Q5_K: quant_q45k(xb, yb, true); break;
                case SRHPM_TYPE_Q6_K: quant_q6k(xb, yb); break;
                case SRHPM_TYPE_Q3_K: quant_q3k(xb, yb); break;
                case SRHPM_TYPE_IQ4_XS: quant_iq4xs(xb, yb); break;
                case SRHPM_TYPE_Q8_0: quant_q8_0(xb, yb); break;
                case SRHPM_TYPE_F16: {
                    const uint16_t h = srhpm_host_fp32_to_fp16(xb[0]);
                    memcpy(yb, &h, 2);
                } break;
                default: break;
            }
        }
    };
    std::vector<std::thread> th;
    for (unsigned i = 0; i < hw; i++) {
        const int64_t b0 = i * per, b1 = std::min(nblk, b0 + per);
        if (b0 < b1) th.emplace_back(work, b0, b1);
    }
    for (auto & t : th) t.join();
    return (size_t) nblk * bs;
}
