// Tests of the C++ operator interface (include/srhpm_ggml.hpp), written like the reference's own kernel checks
// (research/tools/srv_bench.cpp: decoders against a scalar restatement; GGML_SRV_CHECK, patch/srhpm.patch:6573-6609:
// compute_forward's rows against ggml's vec_dot), with the oracle's C restatement (oracle/oracle.h) as the checker.
//
//   test_srhpm_ggml cpu        selection (srv_traits_for, supports_op), work_size, the "stock path" answers
//                              (false), and the GGML_ASSERT aborts (in forked children); no CUDA call
//   test_srhpm_ggml cpu-types  with GGML_SRV_TYPES=q4_K,iq4_xs in the environment: only those types are selected
//   test_srhpm_ggml gpu        compute_forward of every SRV type against the oracle (and a row-split view), the
//                              grouped attention behind its gate, greedy acceptance; needs a GPU
// Exit status 0 when every check passes.
#include <cuda_runtime_api.h>
#include <sys/wait.h>
#include <unistd.h>

#include <cmath>
#include <csignal>
#include <cstdio>
#include <cstdlib>
#include <cstring>
#include <functional>
#include <random>
#include <vector>

#include "oracle.h"
#include "srhpm_ggml.hpp"

using namespace srhpm::ggml;

namespace {

int g_fail = 0;

#define CHECK(cond)                                                        \
    do {                                                                   \
        if (!(cond)) {                                                     \
            fprintf(stderr, "FAIL %s:%d: %s\n", __FILE__, __LINE__, #cond); \
            g_fail++;                                                      \
        }                                                                  \
    } while (0)

void * fake_ptr() { return reinterpret_cast<void *>(uintptr_t{ 1 } << 20); }  // never dereferenced

// op = ggml_mul_mat(W, X): W [K, rows] of `wt`, X f32 [K, M], result f32 [rows, M]
struct MulMat {
    ggml_tensor W, X, Y;
    MulMat(ggml_type wt, int64_t K, int64_t rows, int64_t M, void * w = fake_ptr(), void * x = fake_ptr(),
           void * y = fake_ptr()) {
        W      = ggml_tensor_view(wt, K, rows, 1, 1, w);
        X      = ggml_tensor_view(GGML_TYPE_F32, K, M, 1, 1, x);
        Y      = ggml_tensor_view(GGML_TYPE_F32, rows, M, 1, 1, y);
        Y.op   = GGML_OP_MUL_MAT;
        Y.src[0] = &W;
        Y.src[1] = &X;
    }
    MulMat(const MulMat &)             = delete;  // Y.src points into this object
    MulMat & operator=(const MulMat &) = delete;
};

// true when fn() ends the process with SIGABRT (run in a forked child, stderr silenced)
bool aborts(const std::function<void()> & fn) {
    fflush(stdout);
    fflush(stderr);
    const pid_t pid = fork();
    if (pid == 0) {
        if (!freopen("/dev/null", "w", stderr)) _exit(3);
        fn();
        _exit(0);
    }
    int status = 0;
    waitpid(pid, &status, 0);
    return WIFSIGNALED(status) && WTERMSIG(status) == SIGABRT;
}

const ggml_type kSrvTypes[] = { GGML_TYPE_Q3_K, GGML_TYPE_Q4_K, GGML_TYPE_Q5_K,
                                GGML_TYPE_Q6_K, GGML_TYPE_IQ4_XS, GGML_TYPE_Q8_0 };

// ---- CPU ------------------------------------------------------------------------------------------------------------

void test_selection() {
    extra_buffer_type_b200 buf(backend{});
    for (ggml_type t : kSrvTypes) {
        ggml_tensor w = ggml_tensor_view(t, 1024, 64, 1, 1, fake_ptr());
        CHECK(buf.srv_traits_for(&w) != nullptr);
    }
    ggml_tensor f16 = ggml_tensor_view(GGML_TYPE_F16, 1024, 64, 1, 1, fake_ptr());
    CHECK(buf.srv_traits_for(&f16) == nullptr);
    ggml_tensor odd = ggml_tensor_view(GGML_TYPE_Q8_0, 320, 64, 1, 1, fake_ptr());  // K not a multiple of 256
    CHECK(buf.srv_traits_for(&odd) == nullptr);
    ggml_tensor three = ggml_tensor_view(GGML_TYPE_Q4_K, 1024, 64, 2, 1, fake_ptr());
    CHECK(buf.srv_traits_for(&three) == nullptr);

    MulMat ok(GGML_TYPE_Q4_K, 1024, 64, 8);
    CHECK(buf.supports_op(&ok.Y));
    CHECK(buf.get_tensor_traits(&ok.Y) == buf.srv_traits_for(&ok.W));
    MulMat big(GGML_TYPE_Q4_K, 1024, 64, 17);
    CHECK(!buf.supports_op(&big.Y) && buf.get_tensor_traits(&big.Y) == nullptr);
    MulMat half(GGML_TYPE_Q4_K, 1024, 64, 8);
    half.X = ggml_tensor_view(GGML_TYPE_F16, 1024, 8, 1, 1, fake_ptr());
    CHECK(!buf.supports_op(&half.Y));
    MulMat fa(GGML_TYPE_Q4_K, 1024, 64, 8);
    fa.Y.op = GGML_OP_FLASH_ATTN_EXT;
    CHECK(!buf.supports_op(&fa.Y));
}

void test_tensor_helpers() {
    ggml_tensor w = ggml_tensor_view(GGML_TYPE_Q4_K, 1024, 64, 1, 1, fake_ptr());
    CHECK(w.nb[0] == 144 && w.nb[1] == 576 && w.nb[2] == 576 * 64);
    CHECK(ggml_nbytes(&w) == 576u * 64u);
    CHECK(ggml_nrows(&w) == 64);
    ggml_tensor x = ggml_tensor_view(GGML_TYPE_F32, 5120, 8, 1, 1, fake_ptr());
    CHECK(x.nb[1] == 5120 * 4 && ggml_nbytes(&x) == 5120u * 8u * 4u);
}

void test_work_size_and_stock_answers() {
    extra_buffer_type_b200 buf(backend{});
    for (ggml_type t : kSrvTypes) {
        for (int64_t M : { 1, 4, 8, 16 }) {
            MulMat mm(t, 5120, 17408, M);
            tensor_traits * tr = buf.srv_traits_for(&mm.W);
            size_t          s  = 0, want = 0;
            CHECK(tr->work_size(8, &mm.Y, s));
            const srhpm_tensor W = { t, { 5120, 17408, 1, 1 }, { mm.W.nb[0], mm.W.nb[1], mm.W.nb[2], mm.W.nb[3] },
                                     mm.W.data };
            const srhpm_tensor X = { GGML_TYPE_F32, { 5120, M, 1, 1 }, { 4, mm.X.nb[1], mm.X.nb[2], mm.X.nb[3] },
                                     mm.X.data };
            CHECK(srhpm_mul_mat_work_size(&W, &X, &want) == SRHPM_OK && s == want && s > 0);
        }
    }
    MulMat          ok(GGML_TYPE_Q6_K, 1024, 64, 8);
    tensor_traits * tr = buf.srv_traits_for(&ok.W);
    size_t          s  = 0;
    MulMat big(GGML_TYPE_Q6_K, 1024, 64, 17);  // M > SRV_MAXM: the stock path
    CHECK(!tr->work_size(8, &big.Y, s));
    ggml_compute_params p;
    CHECK(!tr->compute_forward(&p, &big.Y));
    MulMat other(GGML_TYPE_Q6_K, 1024, 64, 8);
    other.Y.op = GGML_OP_FLASH_ATTN_EXT;
    CHECK(!tr->work_size(8, &other.Y, s));
    CHECK(!tr->compute_forward(&p, &other.Y));
    // threads other than 0 have nothing to launch on a device backend
    ggml_compute_params p1;
    p1.ith = 1;
    p1.nth = 4;
    CHECK(tr->compute_forward(&p1, &ok.Y));
    // the grouped attention needs the device (its plan depends on the SM count): without one it is not taken
    CHECK(fa_gqa_small_work_size(backend{}, &ok.Y, 8) == 0);
}

void test_asserts() {
    extra_buffer_type_b200 buf(backend{});
    MulMat                 sel(GGML_TYPE_Q4_K, 1024, 64, 8);
    tensor_traits *        tr = buf.srv_traits_for(&sel.W);
    // patch/srhpm.patch:6406-6407: f32 activations, 2-D operands
    CHECK(aborts([&] {
        MulMat mm(GGML_TYPE_Q4_K, 1024, 64, 8);
        mm.X.type = GGML_TYPE_F16;
        ggml_compute_params p;
        tr->compute_forward(&p, &mm.Y);
    }));
    CHECK(aborts([&] {
        MulMat mm(GGML_TYPE_Q4_K, 1024, 64, 4);
        mm.X.ne[2] = 2;
        ggml_compute_params p;
        tr->compute_forward(&p, &mm.Y);
    }));
    // patch/srhpm.patch:6474: the weight rows must be unpadded
    CHECK(aborts([&] {
        MulMat mm(GGML_TYPE_Q4_K, 1024, 64, 4);
        mm.W.nb[1] += 16;
        ggml_compute_params p;
        tr->compute_forward(&p, &mm.Y);
    }));
    // thread 0 of a backend without a device context
    CHECK(aborts([&] {
        MulMat              mm(GGML_TYPE_Q4_K, 1024, 64, 4);
        ggml_compute_params p;
        tr->compute_forward(&p, &mm.Y);
    }));
}

void test_type_filter() {  // run with GGML_SRV_TYPES=q4_K,iq4_xs
    extra_buffer_type_b200 buf(backend{});
    for (ggml_type t : kSrvTypes) {
        ggml_tensor w    = ggml_tensor_view(t, 1024, 64, 1, 1, fake_ptr());
        const bool  want = t == GGML_TYPE_Q4_K || t == GGML_TYPE_IQ4_XS;
        CHECK((buf.srv_traits_for(&w) != nullptr) == want);
    }
}

// ---- GPU ------------------------------------------------------------------------------------------------------------

#define CUDA_OK(call) CHECK((call) == cudaSuccess)

double rel_l2(const float * got, const double * want, size_t n) {
    double e = 0, r = 0;
    for (size_t i = 0; i < n; i++) {
        e += (got[i] - want[i]) * (got[i] - want[i]);
        r += want[i] * want[i];
    }
    return std::sqrt(e / std::max(r, 1e-300));
}

std::vector<float> randn(std::mt19937 & rng, size_t n, float scale) {
    std::normal_distribution<float> d(0.0f, 1.0f);
    std::vector<float>              v(n);
    for (auto & x : v) x = d(rng) * scale;
    return v;
}

// device copy of h, complete on return (the kernels run on a non-blocking stream)
template <class T> T * dev_copy(const std::vector<T> & h) {
    T * p = nullptr;
    CUDA_OK(cudaMalloc(reinterpret_cast<void **>(&p), std::max<size_t>(h.size(), 1) * sizeof(T)));
    if (!h.empty()) CUDA_OK(cudaMemcpy(p, h.data(), h.size() * sizeof(T), cudaMemcpyHostToDevice));
    CUDA_OK(cudaDeviceSynchronize());
    return p;
}

void test_mul_mat_gpu(const backend & be) {
    extra_buffer_type_b200 buf(be);
    std::mt19937           rng(7);
    const int64_t          K = 1024, rows = 520;
    for (ggml_type t : kSrvTypes) {
        const std::vector<float> wf = randn(rng, (size_t) (rows * K), 0.02f);
        std::vector<uint8_t>     wq(srhpm_row_size(t, K) * rows);
        CHECK(srhpm_quantize_chunk(t, wf.data(), wq.data(), 0, rows, K, nullptr) == wq.size());
        for (int64_t M : { 1, 3, 8, 16 }) {
            const std::vector<float> x = randn(rng, (size_t) (M * K), 1.0f);
            void *                   wd = nullptr;
            CUDA_OK(cudaMalloc(&wd, wq.size()));
            float * xd = dev_copy(x);
            float * yd = nullptr;
            CUDA_OK(cudaMalloc(reinterpret_cast<void **>(&yd), (size_t) (rows * M) * sizeof(float)));
            MulMat          mm(t, K, rows, M, wd, xd, yd);
            tensor_traits * tr = buf.get_tensor_traits(&mm.Y);
            CHECK(tr != nullptr);
            if (!tr) continue;
            CHECK(tr->repack(&mm.W, wq.data(), wq.size()) == 0);  // the loader's copy of the native rows
            size_t ws = 0;
            CHECK(tr->work_size(1, &mm.Y, ws));
            void * work = nullptr;
            CUDA_OK(cudaMalloc(&work, std::max<size_t>(ws, 1)));
            ggml_compute_params p;
            p.wsize = ws;
            p.wdata = work;
            CHECK(tr->compute_forward(&p, &mm.Y));
            CUDA_OK(cudaStreamSynchronize(static_cast<cudaStream_t>(be.stream)));
            std::vector<float> y((size_t) (rows * M));
            CUDA_OK(cudaMemcpy(y.data(), yd, y.size() * sizeof(float), cudaMemcpyDeviceToHost));
            std::vector<double> want(y.size());
            CHECK(orc_mul_mat(t, wq.data(), rows, K, x.data(), M, want.data(), ORC_Q8_0_SIMD) == 0);
            const double e = rel_l2(y.data(), want.data(), y.size());
            if (!(e < 1e-5)) fprintf(stderr, "mul_mat type %d M=%lld: rel L2 %.3g\n", (int) t, (long long) M, e);
            CHECK(e < 1e-5);
            if (M == 8) {
                // the reference's row split (patch/srhpm.patch:6497-6529): a view of the first 256 rows and a result
                // view with the full row stride
                CUDA_OK(cudaMemsetAsync(yd, 0, y.size() * sizeof(float), static_cast<cudaStream_t>(be.stream)));
                MulMat part(t, K, 256, M, wd, xd, yd);
                part.Y.nb[1] = (size_t) rows * sizeof(float);
                size_t ws2   = 0;
                CHECK(tr->work_size(1, &part.Y, ws2));
                void * work2 = nullptr;
                CUDA_OK(cudaMalloc(&work2, std::max<size_t>(ws2, 1)));
                ggml_compute_params p2;
                p2.wsize = ws2;
                p2.wdata = work2;
                CHECK(tr->compute_forward(&p2, &part.Y));
                CUDA_OK(cudaStreamSynchronize(static_cast<cudaStream_t>(be.stream)));
                CUDA_OK(cudaMemcpy(y.data(), yd, y.size() * sizeof(float), cudaMemcpyDeviceToHost));
                double e2 = 0, r2 = 0, tail = 0;
                for (int64_t m = 0; m < M; m++) {
                    for (int64_t r = 0; r < rows; r++) {
                        const double g = y[m * rows + r], w = want[m * rows + r];
                        if (r < 256) {
                            e2 += (g - w) * (g - w);
                            r2 += w * w;
                        } else {
                            tail += std::fabs(g);
                        }
                    }
                }
                CHECK(std::sqrt(e2 / r2) < 1e-5);
                CHECK(tail == 0.0);  // rows outside the view untouched
                cudaFree(work2);
            }
            cudaFree(work);
            cudaFree(wd);
            cudaFree(xd);
            cudaFree(yd);
        }
    }
}

uint16_t f16_bits(float v) {
    uint16_t h = 0;
    srhpm_quantize_chunk(GGML_TYPE_F16, &v, &h, 0, 1, 1, nullptr);
    return h;
}

void test_flash_attn_gpu(const backend & be) {
    std::mt19937  rng(11);
    const int64_t H = 8, Hkv = 2, N = 4, L = 700, D = 256;
    for (ggml_type kt : { GGML_TYPE_Q8_0, GGML_TYPE_F16 }) {
        for (int variant = 0; variant < 2; variant++) {
            const float              scale = 1.0f / 16, max_bias = variant ? 8.0f : 0.0f, softcap = variant ? 30.0f : 0.0f;
            const std::vector<float> q     = randn(rng, (size_t) (H * N * D), 1.0f / 16);
            const std::vector<float> kf = randn(rng, (size_t) (Hkv * L * D), 1.0f), vf = randn(rng, (size_t) (Hkv * L * D), 1.0f);
            const size_t             rowb = srhpm_row_size(kt, D);
            std::vector<uint8_t>     kb(rowb * Hkv * L), vb(rowb * Hkv * L);
            srhpm_quantize_chunk(kt, kf.data(), kb.data(), 0, Hkv * L, D, nullptr);
            srhpm_quantize_chunk(kt, vf.data(), vb.data(), 0, Hkv * L, D, nullptr);
            std::vector<uint16_t> mask((size_t) (N * L), 0);
            for (int64_t t = 0; t < N; t++) {
                for (int64_t j = L - N + t + 1; j < L; j++) mask[t * L + j] = 0xFC00;  // -inf
                for (int64_t j = 0; j < 64 && variant; j++) mask[t * L + j] = f16_bits(-0.5f);
            }
            const std::vector<float> sinks = randn(rng, (size_t) H, 1.0f);
            float *                  qd    = dev_copy(q);
            uint8_t *                kd    = dev_copy(kb);
            uint8_t *                vd    = dev_copy(vb);
            uint16_t *               md    = dev_copy(mask);
            float *                  sd    = dev_copy(sinks);
            float *                  od    = nullptr;
            CUDA_OK(cudaMalloc(reinterpret_cast<void **>(&od), (size_t) (N * H * D) * sizeof(float)));
            ggml_tensor tq = ggml_tensor_view(GGML_TYPE_F32, D, N, H, 1, qd);
            ggml_tensor tk = ggml_tensor_view(kt, D, L, Hkv, 1, kd);
            ggml_tensor tv = ggml_tensor_view(kt, D, L, Hkv, 1, vd);
            ggml_tensor tm = ggml_tensor_view(GGML_TYPE_F16, L, N, 1, 1, md);
            ggml_tensor ts = ggml_tensor_view(GGML_TYPE_F32, H, 1, 1, 1, sd);
            ggml_tensor to = ggml_tensor_view(GGML_TYPE_F32, D, H, N, 1, od);
            to.op          = GGML_OP_FLASH_ATTN_EXT;
            to.src[0]      = &tq;
            to.src[1]      = &tk;
            to.src[2]      = &tv;
            to.src[3]      = &tm;
            to.src[4]      = variant ? &ts : nullptr;
            memcpy(&to.op_params[0], &scale, 4);
            memcpy(&to.op_params[1], &max_bias, 4);
            memcpy(&to.op_params[2], &softcap, 4);
            const size_t ws = fa_gqa_small_work_size(be, &to, 1);
            CHECK(ws >= 256);
            void * work = nullptr;
            CUDA_OK(cudaMalloc(&work, ws));
            ggml_compute_params p;
            p.wsize = ws - 1;  // below the gate's size: not taken
            p.wdata = work;
            CHECK(!compute_forward_flash_attn_ext_gqa_small(be, &p, &to));
            p.wsize = ws;
            CHECK(compute_forward_flash_attn_ext_gqa_small(be, &p, &to));
            CUDA_OK(cudaStreamSynchronize(static_cast<cudaStream_t>(be.stream)));
            std::vector<float> out((size_t) (N * H * D));
            CUDA_OK(cudaMemcpy(out.data(), od, out.size() * sizeof(float), cudaMemcpyDeviceToHost));
            std::vector<double> want(out.size());
            CHECK(orc_attention(q.data(), D, N, H, kt, kb.data(), vb.data(), D, L, Hkv, mask.data(),
                                variant ? sinks.data() : nullptr, scale, max_bias, softcap, ORC_Q8_0_SIMD,
                                want.data()) == 0);
            const double e = rel_l2(out.data(), want.data(), out.size());
            if (!(e < 1e-3)) fprintf(stderr, "flash_attn type %d variant %d: rel L2 %.3g\n", (int) kt, variant, e);
            CHECK(e < 1e-3);
            cudaFree(work);
            cudaFree(qd);
            cudaFree(kd);
            cudaFree(vd);
            cudaFree(md);
            cudaFree(sd);
            cudaFree(od);
        }
    }
    // head size 128: the gate does not take it
    ggml_tensor tq = ggml_tensor_view(GGML_TYPE_F32, 128, 4, 8, 1, fake_ptr());
    ggml_tensor tk = ggml_tensor_view(GGML_TYPE_F16, 128, 512, 2, 1, fake_ptr());
    ggml_tensor to = ggml_tensor_view(GGML_TYPE_F32, 128, 8, 4, 1, fake_ptr());
    to.op          = GGML_OP_FLASH_ATTN_EXT;
    to.src[0]      = &tq;
    to.src[1]      = &tk;
    to.src[2]      = &tk;
    CHECK(fa_gqa_small_work_size(be, &to, 1) == 0);
    ggml_compute_params p;
    CHECK(!compute_forward_flash_attn_ext_gqa_small(be, &p, &to));
}

void test_accept_gpu(const backend & be) {
    std::mt19937             rng(5);
    const int64_t            V  = 1000;
    const std::vector<float> lg = randn(rng, (size_t) (5 * V), 1.0f);
    float *                  ld = dev_copy(lg);
    ggml_tensor              tl = ggml_tensor_view(GGML_TYPE_F32, V, 5, 1, 1, ld);
    auto                     argmax = [&](int r) {
        int64_t b = 0;
        for (int64_t i = 1; i < V; i++) {
            if (lg[r * V + i] > lg[r * V + b]) b = i;
        }
        return (int32_t) b;
    };
    common_sampler_b200 smpl(be, V);
    const std::vector<std::vector<int32_t>> drafts = {
        { argmax(0), argmax(1), 7, 9 },                    // two accepted
        { argmax(0), argmax(1), argmax(2), argmax(3) },    // all accepted: the bonus token follows
        { (argmax(0) + 1) % (int32_t) V, 1, 2, 3 },        // none accepted
        {},                                                // no draft: one sampled token
    };
    for (const auto & d : drafts) {
        for (float relax : { 0.0f, 0.5f }) {
            const std::vector<int32_t> got = smpl.sample_and_accept_n(&tl, d, relax);
            std::vector<int32_t>       want(d.size() + 1);
            const int n = orc_accept(lg.data(), V, d.data(), (int) d.size(), relax, want.data());
            want.resize((size_t) n);
            CHECK(got == want);
        }
    }
    cudaFree(ld);
}

}  // namespace

int main(int argc, char ** argv) {
    const char * mode = argc > 1 ? argv[1] : "cpu";
    if (!strcmp(mode, "cpu")) {
        test_tensor_helpers();
        test_selection();
        test_work_size_and_stock_answers();
        test_asserts();
    } else if (!strcmp(mode, "cpu-types")) {
        test_type_filter();
    } else if (!strcmp(mode, "gpu")) {
        backend be;
        if (srhpm_ctx_create(0, &be.ctx) != SRHPM_OK) {
            fprintf(stderr, "FAIL: srhpm_ctx_create\n");
            return 1;
        }
        cudaStream_t s = nullptr;
        CUDA_OK(cudaStreamCreateWithFlags(&s, cudaStreamNonBlocking));
        be.stream = s;
        test_mul_mat_gpu(be);
        test_flash_attn_gpu(be);
        test_accept_gpu(be);
        int32_t code = 0;
        CHECK(srhpm_ctx_check(be.ctx, &code) == SRHPM_OK);
        cudaStreamDestroy(s);
        srhpm_ctx_destroy(be.ctx);
    } else {
        fprintf(stderr, "usage: %s cpu|cpu-types|gpu\n", argv[0]);
        return 2;
    }
    if (g_fail) {
        fprintf(stderr, "%d check(s) failed\n", g_fail);
        return 1;
    }
    printf("%s: all checks passed\n", mode);
    return 0;
}
