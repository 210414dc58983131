// TEST INFRASTRUCTURE (oracle). Builds oracle/_ref/libsrv_ref_*.so: the reference's OWN CPU kernels, compiled
// from the reference patch (extracted by oracle/build_ref.sh into oracle/_ref/), driven the way the reference
// drives them. Used by the tests as the pin for the restated oracle, by tests/golden/make_golden.py to write the
// golden fixtures, and by bench.py's CPU-baseline leg. Never on the product path.
//
//   ref_srv_mul_mat  follows tensor_traits_srv::compute_forward (patch/srhpm.patch:6400-6562): quantize each
//                    activation row with srv_quantize_row (+ per-32 / per-16 sums), permute pairs for IQ4_XS-p,
//                    dynamic chunks of SRV_CHUNK = 16 rows over the threads, tiles of 8 tokens plus the
//                    remainder through srv_row<R, T, OFFP> (patch/srhpm.patch:6119-6226).
//   ref_fa_gqa       runs ggml_compute_forward_flash_attn_ext_gqa_small (patch/srhpm.patch:581-824) on n threads.
#include "ggml_restated.h"

#include <atomic>
#include <thread>
#include <vector>

#include "srv-kernels.inc"  // patch/srhpm.patch:5454-6230, extracted into oracle/_ref/
#include "fa-gqa.inc"       // patch/srhpm.patch:539-824, extracted into oracle/_ref/

using namespace ggml::cpu::repack;

int g_ref_q8_0_mode = 0;

namespace {

constexpr int64_t kSrvChunk = 16;  // SRV_CHUNK, patch/srhpm.patch:6301

template <class R>
struct srv_driver {
    static constexpr bool can_off = srv_off<R>::value > 0;

    template <int T>
    static void tile(const typename R::block * row, int64_t nsb, const int8_t * xq, const float * xs, const int16_t * xb,
                     const int16_t * x16, int64_t K, int64_t m0, float * out, bool off) {
        const int8_t *  xp[T];
        const float *   sp[T];
        const int16_t * bp[T];
        const int16_t * b16[T];
        for (int t = 0; t < T; t++) {
            xp[t]  = xq + (m0 + t) * K;
            sp[t]  = xs + (m0 + t) * (K / QK_K);
            bp[t]  = xb + (m0 + t) * (K / 32);
            b16[t] = x16 + (m0 + t) * (K / 16);
        }
        if constexpr (can_off) {
            if (off) {
                srv_row<R, T, true>(row, nsb, xp, sp, out, bp, b16);
                return;
            }
        }
        srv_row<R, T>(row, nsb, xp, sp, out, bp);
    }

    static void run(const void * W, int64_t rows, int64_t K, const float * X, int64_t M, float * Y, int nth, bool off) {
        const int64_t nsb = K / QK_K;
        std::vector<int8_t>  xq(M * K);
        std::vector<float>   xs(M * nsb);
        std::vector<int16_t> xb(M * (K / 32)), x16(M * (K / 16));
        const bool use_off = can_off && off;
        for (int64_t m = 0; m < M; m++) {
            srv_quantize_row(X + m * K, xq.data() + m * K, xs.data() + m * nsb, K,
                             srv_has_min<R>::value ? xb.data() + m * (K / 32) : nullptr,
                             use_off ? x16.data() + m * (K / 16) : nullptr);
            if constexpr (srv_paired<R>::value) {
                srv_permute_pairs(xq.data() + m * K, K);
            }
        }
        const auto *         base   = (const typename R::block *) W;
        const int64_t        nchunk = (rows + kSrvChunk - 1) / kSrvChunk;
        std::atomic<int64_t> next{ nth };
        auto worker = [&](int ith) {
            float out[8];
            for (int64_t chunk = ith; chunk < nchunk; chunk = next.fetch_add(1)) {
                const int64_t n1 = std::min<int64_t>(rows, (chunk + 1) * kSrvChunk);
                for (int64_t n = chunk * kSrvChunk; n < n1; n++) {
                    const typename R::block * row = base + n * nsb;
                    int64_t                   m0  = 0;
                    auto store = [&](int T) {
                        for (int t = 0; t < T; t++) {
                            Y[(m0 + t) * rows + n] = out[t];
                        }
                    };
                    for (; m0 + 8 <= M; m0 += 8) {
                        tile<8>(row, nsb, xq.data(), xs.data(), xb.data(), x16.data(), K, m0, out, use_off);
                        store(8);
                    }
                    switch (M - m0) {
                        case 7: tile<7>(row, nsb, xq.data(), xs.data(), xb.data(), x16.data(), K, m0, out, use_off); store(7); break;
                        case 6: tile<6>(row, nsb, xq.data(), xs.data(), xb.data(), x16.data(), K, m0, out, use_off); store(6); break;
                        case 5: tile<5>(row, nsb, xq.data(), xs.data(), xb.data(), x16.data(), K, m0, out, use_off); store(5); break;
                        case 4: tile<4>(row, nsb, xq.data(), xs.data(), xb.data(), x16.data(), K, m0, out, use_off); store(4); break;
                        case 3: tile<3>(row, nsb, xq.data(), xs.data(), xb.data(), x16.data(), K, m0, out, use_off); store(3); break;
                        case 2: tile<2>(row, nsb, xq.data(), xs.data(), xb.data(), x16.data(), K, m0, out, use_off); store(2); break;
                        case 1: tile<1>(row, nsb, xq.data(), xs.data(), xb.data(), x16.data(), K, m0, out, use_off); store(1); break;
                        default: break;
                    }
                }
            }
        };
        std::vector<std::thread> th;
        for (int i = 1; i < nth; i++) {
            th.emplace_back(worker, i);
        }
        worker(0);
        for (auto & t : th) {
            t.join();
        }
    }
};

}  // namespace

extern "C" {

// 1 when this build took the AVX-VNNI / AVX512-VNNI path of srv_madd_acc (patch/srhpm.patch:5579-5587)
int ref_srv_vnni(void) {
#if defined(__AVXVNNI__) || (defined(__AVX512VNNI__) && defined(__AVX512VL__))
    return 1;
#else
    return 0;
#endif
}

int ref_srv_quantize_row(const float * x, int8_t * q, float * sx, int64_t K, int16_t * bsum, int16_t * bsum16) {
    if (K % QK_K) {
        return -1;
    }
    srv_quantize_row(x, q, sx, K, bsum, bsum16);
    return 0;
}

// Y[t * rows + r] = sum_k W[r, k] X[t, k] with the reference's SRV kernels. type: ggml_type. off: GGML_SRV_OFF
// (the launcher sets it), paired: GGML_SRV_PAIR for IQ4_XS (default on upstream). Returns -1 for unsupported types.
int ref_srv_mul_mat(int type, const void * W, int64_t rows, int64_t K, const float * X, int64_t M, float * Y, int nth,
                    int off, int paired) {
    if (K % QK_K || M < 1 || M > SRV_MAXM || nth < 1) {
        return -1;
    }
    switch (type) {
        case GGML_TYPE_Q4_K: srv_driver<srv_q45_k<false>>::run(W, rows, K, X, M, Y, nth, off); return 0;
        case GGML_TYPE_Q5_K: srv_driver<srv_q45_k<true>>::run(W, rows, K, X, M, Y, nth, off); return 0;
        case GGML_TYPE_Q6_K: srv_driver<srv_q6_k>::run(W, rows, K, X, M, Y, nth, off); return 0;
        case GGML_TYPE_Q3_K: srv_driver<srv_q3_k>::run(W, rows, K, X, M, Y, nth, off); return 0;
        case GGML_TYPE_IQ4_XS:
            if (paired) {
                srv_driver<srv_iq4_xs_p>::run(W, rows, K, X, M, Y, nth, off);
            } else {
                srv_driver<srv_iq4_xs>::run(W, rows, K, X, M, Y, nth, off);
            }
            return 0;
        default: return -1;
    }
}

void ref_set_q8_0_mode(int mode) { g_ref_q8_0_mode = mode; }

void ref_quantize_row_q8_0_c(const float * x, void * y, int64_t k) { ref_quantize_row_q8_0(x, y, k); }

void ref_vec_dot_q8_0_c(int n, float * s, const void * x, const void * y) { ref_vec_dot_q8_0_q8_0(n, s, 0, x, 0, y, 0, 1); }

// FA-GQA through the reference's own function. Tensors are ggml views: q f32 [DK, N, H] (strides nbq[4]),
// k / v of kv_type (F16 or Q8_0) [DK|DV, L, Hkv] (strides nbk / nbv), mask f16 [L, >=N] (row stride mask_nb1, may
// be null), sinks f32 [H] (may be null), dst f32 [DV, H, N] contiguous. Returns -1 when the grouped path's gate
// (patch/srhpm.patch:833-841) would not take these shapes.
int ref_fa_gqa(const float * q, const size_t * nbq, int64_t DK, int64_t N, int64_t H, int kv_type, const void * k,
               const size_t * nbk, const void * v, const size_t * nbv, int64_t DV, int64_t L, int64_t Hkv,
               const uint16_t * mask, size_t mask_nb1, const float * sinks, float scale, float max_bias, float softcap,
               float * dst, int nth) {
    if (N < 2 || N > FA_GQA_MAX_N || Hkv <= 0 || H % Hkv || L < GGML_FA_TILE_KV || nth < 1) {
        return -1;
    }
    ggml_tensor tq = {}, tk = {}, tv = {}, tm = {}, ts = {}, td = {};
    tq.type = GGML_TYPE_F32;
    tq.ne[0] = DK; tq.ne[1] = N; tq.ne[2] = H; tq.ne[3] = 1;
    for (int i = 0; i < 4; i++) tq.nb[i] = nbq[i];
    tq.data = (void *) q;
    tk.type = (ggml_type) kv_type;
    tk.ne[0] = DK; tk.ne[1] = L; tk.ne[2] = Hkv; tk.ne[3] = 1;
    for (int i = 0; i < 4; i++) tk.nb[i] = nbk[i];
    tk.data = (void *) k;
    tv.type = (ggml_type) kv_type;
    tv.ne[0] = DV; tv.ne[1] = L; tv.ne[2] = Hkv; tv.ne[3] = 1;
    for (int i = 0; i < 4; i++) tv.nb[i] = nbv[i];
    tv.data = (void *) v;
    if (mask) {
        tm.type  = GGML_TYPE_F16;
        tm.ne[0] = L; tm.ne[1] = N; tm.ne[2] = 1; tm.ne[3] = 1;
        tm.nb[0] = 2; tm.nb[1] = mask_nb1; tm.nb[2] = mask_nb1 * N; tm.nb[3] = tm.nb[2];
        tm.data  = (void *) mask;
    }
    if (sinks) {
        ts.type = GGML_TYPE_F32;
        ts.ne[0] = H; ts.ne[1] = ts.ne[2] = ts.ne[3] = 1;
        ts.nb[0] = 4; ts.nb[1] = ts.nb[2] = ts.nb[3] = 4 * H;
        ts.data = (void *) sinks;
    }
    td.type = GGML_TYPE_F32;
    td.ne[0] = DV; td.ne[1] = H; td.ne[2] = N; td.ne[3] = 1;
    td.nb[0] = 4; td.nb[1] = 4 * DV; td.nb[2] = 4 * DV * H; td.nb[3] = 4 * DV * H * N;
    td.data = dst;
    memcpy(&td.op_params[0], &scale, 4);
    memcpy(&td.op_params[1], &max_bias, 4);
    memcpy(&td.op_params[2], &softcap, 4);
    td.src[0] = &tq; td.src[1] = &tk; td.src[2] = &tv;
    td.src[3] = mask ? &tm : nullptr;
    td.src[4] = sinks ? &ts : nullptr;

    const size_t       wsize = ggml_fa_gqa_small_work_size(&td, nth);
    std::vector<float> wdata(wsize / sizeof(float) + 16);
    ggml_threadpool    tp;
    tp.n_threads = nth;
    auto worker = [&](int ith) {
        ggml_compute_params p = { ith, nth, wsize, wdata.data(), &tp, false };
        ggml_compute_forward_flash_attn_ext_gqa_small(&p, &td);
    };
    std::vector<std::thread> th;
    for (int i = 1; i < nth; i++) {
        th.emplace_back(worker, i);
    }
    worker(0);
    for (auto & t : th) {
        t.join();
    }
    return 0;
}

}  // extern "C"
