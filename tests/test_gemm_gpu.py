"""GPU parity of the small-batch quantized matmul (srhpm_mul_mat) against the oracle and the reference's kernels.

Bar: activation quantization and the per-block integer sums bit-exact; outputs within 1e-3 relative L2 of the
reference's f32 kernels (the stated tolerance) and, as a tighter check of the integer path, within 1e-5 of the
exact-integer f64 oracle."""
import ctypes

import numpy as np
import pytest
import torch

import oracle as O
import srhpm_b200 as S
from srhpm_b200 import _lib as L

pytestmark = pytest.mark.gpu

TYPES = [S.Q4_K, S.Q5_K, S.Q6_K, S.Q3_K, S.IQ4_XS, S.Q8_0]
TOL_REF = 1e-3   # relative L2 vs the reference's f32 accumulation
TOL_EXACT = 1e-5  # relative L2 vs the exact-integer f64 oracle


def rel_l2(a, b):
    a = np.asarray(a, np.float64)
    b = np.asarray(b, np.float64)
    return float(np.linalg.norm(a - b) / max(np.linalg.norm(b), 1e-30))


def weights(qtype, rows, K, rng, kind="random"):
    if kind == "random":
        return O.random_blocks(qtype, rows * K // O.BLOCK_ELEMS[qtype], rng).reshape(rows, -1)
    w = (rng.standard_normal((rows, K)) * 0.02).astype(np.float32)
    return S.quantize_chunk(w, qtype)


def test_quantize_rows_q8_K_bit_exact(ctx):
    rng = np.random.default_rng(1)
    K = 2048
    rows = [rng.standard_normal(K), np.zeros(K), np.full(K, -2.5), rng.standard_normal(K) * 1e-30,
            rng.integers(-4, 5, K) * 0.5, rng.standard_normal(K) * 1e6]
    X = np.stack(rows).astype(np.float32)
    X[0, 7], X[0, 100] = -9.0, 9.0
    q, d, b32, b16 = ctx.quantize_rows_q8_K(torch.from_numpy(X).cuda())
    for i in range(X.shape[0]):
        oq, od, ob32, ob16 = O.quantize_row_q8K(X[i])
        assert np.array_equal(q[i].cpu().numpy(), oq)
        assert np.array_equal(d[i].cpu().numpy().view(np.uint32), od.view(np.uint32))
        assert np.array_equal(b32[i].cpu().numpy(), ob32)
        assert np.array_equal(b16[i].cpu().numpy(), ob16)


@pytest.mark.parametrize("mode", [L.Q8_0_ACT_SIMD, L.Q8_0_ACT_REF])
def test_quantize_rows_q8_0_bit_exact(ctx, mode):
    rng = np.random.default_rng(2)
    K = 1024
    X = np.stack([rng.standard_normal(K), rng.integers(-3, 4, K) * 0.25, np.zeros(K),
                  rng.standard_normal(K) * 300]).astype(np.float32)
    ctx.set_q8_0_act_mode(mode)
    try:
        got = ctx.quantize_rows_q8_0(torch.from_numpy(X).cuda()).cpu().numpy()
    finally:
        ctx.set_q8_0_act_mode(L.Q8_0_ACT_SIMD)
    for i in range(X.shape[0]):
        assert np.array_equal(got[i], O.quantize_row_q8_0(X[i], mode))


def _check_isums(ctx, qtype, rows, K, N, rng):
    Wb = weights(qtype, rows, K, rng)
    X = rng.standard_normal((N, K)).astype(np.float32)
    W = S.QuantTensor.from_blocks(Wb, qtype, rows, K)
    isum, imin = ctx.mul_mat_isums(W, torch.from_numpy(X).cuda())
    isum, imin = isum.cpu().numpy(), imin.cpu().numpy()
    for t in range(N):
        if qtype == S.Q8_0:
            qb = O.quantize_row_q8_0(X[t]).reshape(-1, 34)
            xq, b32 = qb[:, 2:].copy().view(np.int8).reshape(-1), None
        else:
            xq, _, b32, _ = O.quantize_row_q8K(X[t])
        for r in range(rows):
            m, mn = O.row_isums(qtype, Wb[r], xq, b32, K)
            assert np.array_equal(isum[t, r], m), (t, r)
            if qtype in (S.Q4_K, S.Q5_K):
                assert np.array_equal(imin[t, r], mn), (t, r)


@pytest.mark.parametrize("qtype", TYPES)
@pytest.mark.parametrize("N", [1, 3, 8, 9, 16])
def test_isums_bit_exact(ctx, qtype, N):
    _check_isums(ctx, qtype, 70, 768, N, np.random.default_rng(10 + N))


@pytest.mark.parametrize("qtype", TYPES)
@pytest.mark.parametrize("N", [1, 2, 3, 4, 5, 7, 8, 9, 12, 16])
def test_mul_mat_vs_oracle_and_reference(ctx, ref, qtype, N):
    rng = np.random.default_rng(1000 * N + qtype)
    rows, K = 133, 1280
    Wb = weights(qtype, rows, K, rng)
    X = rng.standard_normal((N, K)).astype(np.float32)
    W = S.QuantTensor.from_blocks(Wb, qtype, rows, K)
    y = ctx.mul_mat(W, torch.from_numpy(X).cuda()).cpu().numpy()
    assert rel_l2(y, O.mul_mat(qtype, Wb, rows, K, X)) < TOL_EXACT
    if ref is not None and qtype in O.SRV_TYPES:
        assert rel_l2(y, O.ref_mul_mat(qtype, Wb, rows, K, X, nth=4, lib=ref)) < TOL_REF
    elif qtype == S.Q8_0:
        assert rel_l2(y, O.mul_mat_q8_0_f32(Wb, rows, K, X, nth=4)) < TOL_REF


@pytest.mark.parametrize("qtype", TYPES)
def test_mul_mat_quantized_weights(ctx, qtype):
    """Weights from the package's own quantizer (N(0, 0.02) rows, as the benchmark builds them)."""
    rng = np.random.default_rng(7)
    rows, K, N = 300, 2048, 5
    Wb = weights(qtype, rows, K, rng, kind="quantized")
    X = rng.standard_normal((N, K)).astype(np.float32)
    y = ctx.mul_mat(S.QuantTensor.from_blocks(Wb, qtype, rows, K), torch.from_numpy(X).cuda()).cpu().numpy()
    assert rel_l2(y, O.mul_mat(qtype, Wb, rows, K, X)) < TOL_EXACT


@pytest.mark.parametrize("qtype", TYPES)
@pytest.mark.parametrize("shape", [(5120, 5120), (6144, 5120), (17408, 5120), (5120, 17408)])
def test_mul_mat_full_shapes(ctx, ref, qtype, shape):
    """The verify-GEMM sweep shapes at full size; the oracle checks the first and last 96 rows (tile edges)."""
    rows, K = shape
    rng = np.random.default_rng(rows + K + qtype)
    Wb = weights(qtype, rows, K, rng)
    N = 9
    X = rng.standard_normal((N, K)).astype(np.float32)
    y = ctx.mul_mat(S.QuantTensor.from_blocks(Wb, qtype, rows, K), torch.from_numpy(X).cuda()).cpu().numpy()
    for r0, r1 in ((0, 96), (rows - 96, rows)):
        assert rel_l2(y[:, r0:r1], O.mul_mat(qtype, Wb[r0:r1], r1 - r0, K, X)) < TOL_EXACT
    assert np.isfinite(y).all()


def test_mul_mat_views_and_strides(ctx):
    """Row-range view of W (the reference's row split), X and Y with padded row strides."""
    rng = np.random.default_rng(3)
    rows, K, N = 200, 1024, 4
    Wb = weights(S.Q4_K, rows, K, rng)
    W = S.QuantTensor.from_blocks(Wb, S.Q4_K, rows, K)
    Xp = torch.from_numpy(rng.standard_normal((N, K + 64)).astype(np.float32)).cuda()
    X = Xp[:, 16:16 + K]
    Yp = torch.full((N, rows + 37), 7.0, device="cuda")
    r0, r1 = 64, 161
    sub = W.row_slice(r0, r1)
    ctx.mul_mat(sub, X, out=Yp[:, 5:5 + (r1 - r0)])
    want = O.mul_mat(S.Q4_K, Wb[r0:r1], r1 - r0, K, X.cpu().numpy())
    got = Yp.cpu().numpy()
    assert rel_l2(got[:, 5:5 + (r1 - r0)], want) < TOL_EXACT
    assert (got[:, :5] == 7.0).all() and (got[:, 5 + (r1 - r0):] == 7.0).all()


def test_mul_mat_ragged_tail(ctx):
    """A matrix whose byte size is not a multiple of 16 (Q6_K / Q3_K odd rows): the last bytes come in by hand."""
    rng = np.random.default_rng(4)
    for qtype, rows, K in ((S.Q6_K, 65, 256), (S.Q3_K, 1, 256), (S.Q3_K, 67, 768), (S.IQ4_XS, 3, 256)):
        Wb = weights(qtype, rows, K, rng)
        X = rng.standard_normal((6, K)).astype(np.float32)
        y = ctx.mul_mat(S.QuantTensor.from_blocks(Wb, qtype, rows, K), torch.from_numpy(X).cuda()).cpu().numpy()
        assert rel_l2(y, O.mul_mat(qtype, Wb, rows, K, X)) < TOL_EXACT


def test_mul_mat_zero_activations(ctx):
    rng = np.random.default_rng(5)
    rows, K = 64, 512
    Wb = weights(S.Q5_K, rows, K, rng)
    X = np.zeros((3, K), np.float32)
    X[1] = rng.standard_normal(K)
    y = ctx.mul_mat(S.QuantTensor.from_blocks(Wb, S.Q5_K, rows, K), torch.from_numpy(X).cuda()).cpu().numpy()
    assert (y[0] == 0).all() and (y[2] == 0).all()
    assert rel_l2(y[1], O.mul_mat(S.Q5_K, Wb, rows, K, X[1:2])[0]) < TOL_EXACT


def test_mul_mat_status_codes(ctx):
    lib = L.load()
    rng = np.random.default_rng(6)
    rows, K = 64, 512
    W = S.QuantTensor.from_blocks(weights(S.Q4_K, rows, K, rng), S.Q4_K, rows, K)
    X17 = torch.randn(17, K, device="cuda")
    assert ctx.mul_mat_work_size(W, X17)[0] == L.UNSUPPORTED           # > 16 rows: stock path
    X = torch.randn(4, K, device="cuda")
    raw = torch.empty(W.nbytes + 64, dtype=torch.uint8, device="cuda")
    raw[8:8 + W.nbytes].copy_(W.data)
    Wmis = S.QuantTensor(raw[8:8 + W.nbytes], S.Q4_K, rows, K)
    with pytest.raises(S.SrhpmError) as e:
        ctx.mul_mat(Wmis, X)
    assert e.value.status == L.ERR_ALIGN
    Y = torch.empty(4, rows, device="cuda")
    wv, xv, yv = W.view(), S.f32_rows_view(X), S.f32_rows_view(Y)
    small = torch.empty(64, dtype=torch.uint8, device="cuda")
    st = lib.srhpm_mul_mat(ctx.handle, ctypes.byref(wv), ctypes.byref(xv), ctypes.byref(yv),
                           ctypes.c_void_p(small.data_ptr()), small.numel(), None)
    assert st == L.ERR_WORKSPACE
    Wbad = S.QuantTensor(W.data, S.Q4_K, rows, K)
    Wbad.K = 300  # not a multiple of 256
    bad = Wbad.view()
    assert lib.srhpm_mul_mat_work_size(ctypes.byref(bad), ctypes.byref(xv), ctypes.byref(ctypes.c_size_t())) != 0
    ctx.check()


def test_golden_fixtures(ctx):
    """The committed fixtures (outputs of the reference's own kernels) through the CUDA path."""
    import os
    path = os.path.join(os.path.dirname(__file__), "golden", "srv_mul_mat.npz")
    g = np.load(path)
    for key in sorted(k for k in g.files if k.endswith("_W")):
        name = key[:-2]
        qtype, rows, K = (int(v) for v in g[name + "_meta"])
        Wb, X, Yref = g[name + "_W"], g[name + "_X"], g[name + "_Y"]
        y = ctx.mul_mat(S.QuantTensor.from_blocks(Wb, qtype, rows, K), torch.from_numpy(X).cuda()).cpu().numpy()
        assert rel_l2(y, Yref) < TOL_REF, name
