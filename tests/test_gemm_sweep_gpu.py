"""The verify-GEMM sweep's own products, every output row, against the reference's kernels and the exact oracle.

The benchmark's workload (the verify-GEMM sweep at k = 2..8): weights [5120x5120], [6144x5120], [17408x5120],
[5120x17408] drawn from N(0, 0.02) and quantized by the library's quantizer to Q4_K, Q5_K, Q6_K, Q8_0 and IQ4_XS,
activations N(0, 1) with N = 2, 4 and 8 rows; the single product Q4_K 17408x5120 at N = 4 on its own. Bars: 1e-3 relative L2
against the reference's f32 kernels (patch/srhpm.patch:6119-6226 via its compute_forward scheduling; Q8_0 through
the restated stock path), 1e-5 against the exact-integer f64 oracle, and no single output off by more than 1e-4 of
the largest exact output (a wrong row or tile would stand out there before it moved the L2 norm)."""
import numpy as np
import pytest
import torch

import oracle as O
import srhpm_b200 as S

pytestmark = pytest.mark.gpu

SHAPES = [(5120, 5120), (6144, 5120), (17408, 5120), (5120, 17408)]
TYPES = [S.Q4_K, S.Q5_K, S.Q6_K, S.Q8_0, S.IQ4_XS]
TOL_REF = 1e-3
TOL_EXACT = 1e-5
TOL_MAX = 1e-4


def rel_l2(a, b):
    a = np.asarray(a, np.float64)
    b = np.asarray(b, np.float64)
    return float(np.linalg.norm(a - b) / max(np.linalg.norm(b), 1e-30))


@pytest.fixture(scope="module")
def packed():
    """Quantized weights by (type, rows, K), made on first use (one f32 matrix per shape, seeded)."""
    cache = {}

    def get(qtype, rows, K):
        key = (qtype, rows, K)
        if key not in cache:
            w = (np.random.default_rng(rows * 7 + K).standard_normal((rows, K), dtype=np.float32)
                 * np.float32(0.02))
            cache[key] = S.quantize_chunk(w, qtype)
        return cache[key]

    return get


def _check(ctx, ref, Wb, qtype, rows, K, N, seed):
    X = np.random.default_rng(seed).standard_normal((N, K), dtype=np.float32)
    W = S.QuantTensor.from_blocks(Wb, qtype, rows, K)
    y = ctx.mul_mat(W, torch.from_numpy(X).cuda()).cpu().numpy()
    ctx.check()
    exact = O.mul_mat(qtype, Wb, rows, K, X)
    assert rel_l2(y, exact) < TOL_EXACT
    assert float(np.abs(y - exact).max()) <= TOL_MAX * float(np.abs(exact).max())
    if qtype == S.Q8_0:
        want = O.mul_mat_q8_0_f32(Wb, rows, K, X, nth=8)
    elif ref is not None:
        want = O.ref_mul_mat(qtype, Wb, rows, K, X, nth=8, off=1, paired=1, lib=ref)
    else:
        want = None
    if want is not None:
        assert rel_l2(y, want) < TOL_REF


def test_single_product_q4K_17408x5120_all_rows(ctx, ref, packed):
    """The single product Q4_K 17408x5120 at N = 4, every row."""
    _check(ctx, ref, packed(S.Q4_K, 17408, 5120), S.Q4_K, 17408, 5120, 4, seed=1)


@pytest.mark.parametrize("shape", SHAPES)
@pytest.mark.parametrize("qtype", TYPES)
def test_sweep_product_all_rows(ctx, ref, packed, qtype, shape):
    rows, K = shape
    Wb = packed(qtype, rows, K)
    for N in (2, 4, 8):
        _check(ctx, ref, Wb, qtype, rows, K, N, seed=100 * N + qtype)
