"""srhpm_mul_mat_static: the quantized matmul for callers that cannot allocate device memory (a host framework that
owns every device buffer and offers no scratch per operation, or a decode loop where a cudaMalloc would synchronise
the device). Its scratch is a fixed array inside the library instead of a caller work buffer.

Checked through the C ABI against srhpm_mul_mat (which uses a caller-provided work buffer) on two calls in a row,
within the tolerance of the matmul parity tests, and on three calls issued back to back without synchronisation
against both srhpm_mul_mat and the exact oracle. Collected last (file name) so that a failure here does not stop a
`-x` run before the other tests; it also passes alone in a fresh process, where its first call sets up the array."""
import ctypes

import numpy as np
import pytest
import torch

import oracle as O
import srhpm_b200 as S
from srhpm_b200 import _lib as L

pytestmark = pytest.mark.gpu

TOL = 1e-5  # relative L2, as the matmul parity tests against the exact oracle


def rel_l2(a, b):
    a = np.asarray(a, np.float64)
    b = np.asarray(b, np.float64)
    return float(np.linalg.norm(a - b) / max(np.linalg.norm(b), 1e-30))


def _static(lib, ctx, W, X, Y):
    wv, xv, yv = W.view(), S.f32_rows_view(X), S.f32_rows_view(Y)
    return lib.srhpm_mul_mat_static(ctx.handle, ctypes.byref(wv), ctypes.byref(xv), ctypes.byref(yv),
                                    ctypes.c_void_p(torch.cuda.current_stream().cuda_stream))


def test_static_matches_work_buffer_path_twice():
    lib = L.load()
    ctx = S.Context(0)
    rng = np.random.default_rng(2024)
    cases = [(S.Q4_K, 17408, 5120, 4), (S.Q6_K, 5120, 17408, 9)]  # different shapes, types and N, back to back
    for qtype, rows, K, N in cases:
        blocks = O.random_blocks(qtype, rows * K // O.BLOCK_ELEMS[qtype], rng).reshape(rows, -1)
        W = S.QuantTensor.from_blocks(blocks, qtype, rows, K)
        X = torch.from_numpy(rng.standard_normal((N, K)).astype(np.float32)).cuda()
        want = ctx.mul_mat(W, X)
        got = torch.full((N, rows), float("nan"), device="cuda")
        assert _static(lib, ctx, W, X, got) == L.OK
        torch.cuda.synchronize()
        assert rel_l2(got.cpu().numpy(), want.cpu().numpy()) < TOL
    ctx.check()
    ctx.close()


def test_static_back_to_back_without_sync_matches_oracle():
    """Three calls issued back to back on one stream with no synchronisation between them (the second reuses the
    shared array while the first may still be finishing; the third repeats the first), each into its own output,
    then one synchronisation: every output against srhpm_mul_mat and against the exact oracle."""
    lib = L.load()
    ctx = S.Context(0)
    rng = np.random.default_rng(77)
    cases = [(S.Q4_K, 6144, 5120, 8), (S.Q6_K, 5120, 5120, 3)]
    prepared = []
    for qtype, rows, K, N in cases:
        w = (rng.standard_normal((rows, K)) * 0.02).astype(np.float32)
        blocks = S.quantize_chunk(w, qtype)
        Xh = rng.standard_normal((N, K)).astype(np.float32)
        prepared.append((qtype, rows, K, blocks, S.QuantTensor.from_blocks(blocks, qtype, rows, K),
                         torch.from_numpy(Xh).cuda(), Xh))
    order = [0, 1, 0]
    outs = [torch.full((prepared[i][5].shape[0], prepared[i][1]), float("nan"), device="cuda") for i in order]
    torch.cuda.synchronize()
    for i, y in zip(order, outs):
        assert _static(lib, ctx, prepared[i][4], prepared[i][5], y) == L.OK
    torch.cuda.synchronize()
    for i, y in zip(order, outs):
        qtype, rows, K, blocks, W, X, Xh = prepared[i]
        got = y.cpu().numpy()
        assert rel_l2(got, ctx.mul_mat(W, X).cpu().numpy()) < TOL
        assert rel_l2(got, O.mul_mat(qtype, blocks, rows, K, Xh)) < TOL
    ctx.check()
    ctx.close()


def test_static_rejects_products_beyond_its_buffer():
    lib = L.load()
    ctx = S.Context(0)
    rows, K, N = 64, 65536, 16  # activation records alone exceed the fixed buffer
    W = S.QuantTensor(torch.zeros(rows * lib.srhpm_row_size(S.Q4_K, K), dtype=torch.uint8, device="cuda"), S.Q4_K,
                      rows, K)
    X = torch.zeros(N, K, device="cuda")
    Y = torch.zeros(N, rows, device="cuda")
    assert _static(lib, ctx, W, X, Y) == L.ERR_TOO_LARGE
    ctx.check()
    ctx.close()
