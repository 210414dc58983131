// Tests of libsrhpm_dgpu.so, loaded as the reference's ggml-cpu loads its dGPU library: by path, with the four
// entry points bound by name (patch/srhpm.patch:5034-5055) and the signatures of dgpu/dgpu.cu. The checks follow the
// reference's dgpu_test.cpp (the GPU rows against a restatement of the same product), with the oracle as the checker.
//
//   test_srhpm_dgpu <dir> cpu   argument statuses (-1, -6), a launch before dgpu_init (-5), a collect before any
//                               launch (-1); no CUDA call is reached
//   test_srhpm_dgpu <dir> gpu   IQ4_XS and Q3_K rows for M = 1..8 with strided x and dst against the oracle, the
//                               copy kept per key (dgpu_pinned_bytes), the max_pinned budget (-2), collect's shape check
// <dir> holds libsrhpm_dgpu.so. Exit status 0 when every check passes.
#include <dlfcn.h>

#include <cmath>
#include <cstdint>
#include <cstdio>
#include <cstring>
#include <random>
#include <string>
#include <vector>

#include "oracle.h"
#include "srhpm_b200.h"

namespace {

int g_fail = 0;

#define CHECK(cond)                                                        \
    do {                                                                   \
        if (!(cond)) {                                                     \
            fprintf(stderr, "FAIL %s:%d: %s\n", __FILE__, __LINE__, #cond); \
            g_fail++;                                                      \
        }                                                                  \
    } while (0)

// the reference's function types (dgpu/dgpu.cu:17, 235-312)
using init_t     = int (*)();
using launch_t   = int (*)(int, const void *, const void *, int64_t, int64_t, int, const float *, size_t, size_t);
using collect_t  = int (*)(int, int64_t, char *, size_t);
using meminfo_t  = void (*)(size_t *, size_t *);
using pinned_t   = size_t (*)();

struct Dgpu {
    init_t    init    = nullptr;
    launch_t  launch  = nullptr;
    collect_t collect = nullptr;
    meminfo_t mem_info = nullptr;
    pinned_t  pinned  = nullptr;
};

bool load(const std::string & dir, Dgpu & d) {
    void * h = dlopen((dir + "/libsrhpm_dgpu.so").c_str(), RTLD_NOW | RTLD_LOCAL);
    if (!h) {
        fprintf(stderr, "dlopen: %s\n", dlerror());
        return false;
    }
    d.init     = reinterpret_cast<init_t>(dlsym(h, "dgpu_init"));
    d.launch   = reinterpret_cast<launch_t>(dlsym(h, "dgpu_launch"));
    d.collect  = reinterpret_cast<collect_t>(dlsym(h, "dgpu_collect"));
    d.mem_info = reinterpret_cast<meminfo_t>(dlsym(h, "dgpu_mem_info"));
    d.pinned   = reinterpret_cast<pinned_t>(dlsym(h, "dgpu_pinned_bytes"));
    return d.init && d.launch && d.collect && d.mem_info && d.pinned;
}

void test_cpu(const Dgpu & d) {
    std::vector<uint8_t> rows(136 * 4 * 8);
    std::vector<float>   x(1024 * 8);
    const size_t         nb = 1024 * sizeof(float);
    CHECK(d.launch(2, rows.data(), rows.data(), 8, 1024, 1, x.data(), nb, 1 << 30) == -1);    // kind
    CHECK(d.launch(0, rows.data(), rows.data(), 8, 1024, 0, x.data(), nb, 1 << 30) == -1);    // M < 1
    CHECK(d.launch(0, rows.data(), rows.data(), 8, 1024, 9, x.data(), nb, 1 << 30) == -1);    // M > 8
    CHECK(d.launch(0, rows.data(), rows.data(), 8, 1000, 1, x.data(), nb, 1 << 30) == -1);    // K % 256
    CHECK(d.launch(0, rows.data(), rows.data(), 8, 1024, 2, x.data(), nb - 4, 1 << 30) == -1);  // x row stride
    CHECK(d.launch(1, rows.data(), rows.data(), 8, 768, 1, x.data(), 768 * 4, 1 << 30) == -6);  // Q3_K, 3 blocks
    CHECK(d.launch(0, rows.data(), rows.data(), 8, 1024, 1, x.data(), nb, 1 << 30) == -5);    // before dgpu_init
    std::vector<char> dst(64);
    CHECK(d.collect(1, 8, dst.data(), 32) == -1);  // nothing launched
}

std::vector<float> randn(std::mt19937 & rng, size_t n, float scale) {
    std::normal_distribution<float> g(0.0f, 1.0f);
    std::vector<float>              v(n);
    for (auto & x : v) x = g(rng) * scale;
    return v;
}

void test_gpu(const Dgpu & d) {
    CHECK(d.init() == 0);
    CHECK(d.init() == 0);  // idempotent
    size_t fr = 0, tot = 0;
    d.mem_info(&fr, &tot);
    CHECK(tot > 0 && fr <= tot);
    std::mt19937 rng(3);
    const int64_t K = 1024, nrows = 300, xs = K + 8, ys = nrows + 5;  // strided x and dst
    // the library keys its copies by the rows' address, as the reference does: every tensor stays alive (and at its
    // address) until the end, so no two tensors share a key
    std::vector<std::vector<uint8_t>> tensors(2);
    for (int kind : { 0, 1 }) {
        const int                type = kind == 0 ? SRHPM_TYPE_IQ4_XS : SRHPM_TYPE_Q3_K;
        const size_t             rowb = srhpm_row_size(type, K);
        const std::vector<float> wf   = randn(rng, (size_t) (nrows * K), 0.02f);
        std::vector<uint8_t> &   wq   = tensors[kind];
        wq.resize(rowb * nrows);
        CHECK(srhpm_quantize_chunk(type, wf.data(), wq.data(), 0, nrows, K, nullptr) == wq.size());
        const size_t held0 = d.pinned();
        for (int M = 1; M <= 8; M++) {
            const std::vector<float> xv = randn(rng, (size_t) (M * xs), 1.0f);
            CHECK(d.launch(kind, wq.data(), wq.data(), nrows, K, M, xv.data(), xs * sizeof(float), size_t{ 1 } << 30) == 0);
            std::vector<float> y((size_t) (M * ys), -7.0f);
            CHECK(d.collect(M, nrows, reinterpret_cast<char *>(y.data()), ys * sizeof(float)) == 0);
            // the oracle on the same rows and activations (dense x)
            std::vector<float> xd((size_t) (M * K));
            for (int t = 0; t < M; t++) memcpy(&xd[t * K], &xv[t * xs], K * sizeof(float));
            std::vector<double> want((size_t) (M * nrows));
            CHECK(orc_mul_mat(type, wq.data(), nrows, K, xd.data(), M, want.data(), ORC_Q8_0_SIMD) == 0);
            double e = 0, r = 0;
            bool   pad_ok = true;
            for (int t = 0; t < M; t++) {
                for (int64_t i = 0; i < nrows; i++) {
                    const double g = y[t * ys + i], w = want[t * nrows + i];
                    e += (g - w) * (g - w);
                    r += w * w;
                }
                for (int64_t i = nrows; i < ys; i++) pad_ok = pad_ok && y[t * ys + i] == -7.0f;
            }
            const double rel = std::sqrt(e / r);
            if (!(rel < 1e-5)) fprintf(stderr, "kind %d M=%d: rel L2 %.3g\n", kind, M, rel);
            CHECK(rel < 1e-5);
            CHECK(pad_ok);  // bytes between dst rows untouched
        }
        // one copy per key: the eight launches above uploaded the rows once
        CHECK(d.pinned() == held0 + wq.size());
        // fewer rows of the same tensor: the copy is reused
        std::vector<float> x1((size_t) K, 0.5f), y1((size_t) nrows);
        CHECK(d.launch(kind, wq.data(), wq.data(), 100, K, 1, x1.data(), K * sizeof(float), size_t{ 1 } << 30) == 0);
        CHECK(d.pinned() == held0 + wq.size());
        CHECK(d.collect(1, 50, reinterpret_cast<char *>(y1.data()), 100 * sizeof(float)) == -1);  // not its shape
        CHECK(d.collect(1, 100, reinterpret_cast<char *>(y1.data()), 100 * sizeof(float)) == 0);
    }
    // a new key over the budget: refused, nothing held in addition
    std::vector<uint8_t> more(srhpm_row_size(SRHPM_TYPE_IQ4_XS, K) * 64, 0);
    std::vector<float>   x2((size_t) K, 1.0f);
    const size_t         held = d.pinned();
    CHECK(d.launch(0, more.data(), more.data(), 64, K, 1, x2.data(), K * sizeof(float), held + 100) == -2);
    CHECK(d.pinned() == held);
}

}  // namespace

int main(int argc, char ** argv) {
    if (argc < 3) {
        fprintf(stderr, "usage: %s <dir of libsrhpm_dgpu.so> cpu|gpu\n", argv[0]);
        return 2;
    }
    Dgpu d;
    if (!load(argv[1], d)) {
        fprintf(stderr, "FAIL: libsrhpm_dgpu.so or one of its entry points\n");
        return 1;
    }
    if (!strcmp(argv[2], "cpu")) {
        test_cpu(d);
    } else if (!strcmp(argv[2], "gpu")) {
        test_gpu(d);
    } else {
        fprintf(stderr, "unknown mode %s\n", argv[2]);
        return 2;
    }
    if (g_fail) {
        fprintf(stderr, "%d check(s) failed\n", g_fail);
        return 1;
    }
    printf("dgpu %s: all checks passed\n", argv[2]);
    return 0;
}
