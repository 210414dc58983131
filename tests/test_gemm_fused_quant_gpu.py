"""GPU: srhpm_mul_mat_fused_quant, the matmul that quantizes its own activations (one launch per product), against
srhpm_mul_mat (the same matmul behind a separate quantizer kernel) and against the exact oracle.

The fused form moves the activation quantizer (srv_quantize_row, patch/srhpm.patch:5518-5575) into the GEMM kernel's
prologue: every consumer warp of the grid quantizes a share of the (super-block, token) pairs into the records, and
the grid meets at a counter before any record is loaded. The records are the same bytes either way, so the outputs
must be bit-identical; the grid counter must survive back-to-back launches on one work buffer and CUDA-graph replays
(it advances by a fixed amount per launch)."""
import numpy as np
import pytest
import torch

import oracle as O
import srhpm_b200 as S
from srhpm_b200 import _lib as L

pytestmark = pytest.mark.gpu

TYPES = [S.Q4_K, S.Q5_K, S.Q6_K, S.Q3_K, S.IQ4_XS, S.Q8_0]
TOL_EXACT = 1e-5  # relative L2 vs the exact-integer f64 oracle


def rel_l2(a, b):
    a = np.asarray(a, np.float64)
    b = np.asarray(b, np.float64)
    return float(np.linalg.norm(a - b) / max(np.linalg.norm(b), 1e-30))


def _product(qtype, rows, K, N, seed):
    rng = np.random.default_rng(seed)
    Wb = O.random_blocks(qtype, rows * K // O.BLOCK_ELEMS[qtype], rng).reshape(rows, -1)
    X = rng.standard_normal((N, K)).astype(np.float32)
    return Wb, S.QuantTensor.from_blocks(Wb, qtype, rows, K), torch.from_numpy(X).cuda(), X


def _both(ctx, fn):
    """fn(fused) -> result, through srhpm_mul_mat_fused_quant and srhpm_mul_mat; with the launches of each."""
    ctx.launch_count(reset=True)
    a = fn(True)
    torch.cuda.synchronize()
    la = ctx.launch_count(reset=True)
    b = fn(False)
    torch.cuda.synchronize()
    lb = ctx.launch_count(reset=True)
    ctx.check()
    return a, b, la, lb


@pytest.mark.parametrize("qtype", TYPES)
@pytest.mark.parametrize("N", [1, 2, 4, 8, 9, 16])
@pytest.mark.parametrize("shape", [(133, 1280), (5120, 5120), (17408, 5120), (5120, 17408)])
def test_fused_equals_separate_quantizer(ctx, qtype, N, shape):
    rows, K = shape
    Wb, W, Xd, X = _product(qtype, rows, K, N, rows + K + 10 * N + qtype)
    y1, y0, l1, l0 = _both(ctx, lambda fq: ctx.mul_mat(W, Xd, fused_quant=fq).cpu().numpy())
    assert np.array_equal(y1, y0)
    assert l0 == 2
    if rows >= 5120:  # enough CTAs for at most two quantization jobs per consumer warp: one launch
        assert l1 == 1
    sl = slice(0, 64) if rows > 64 else slice(0, rows)
    assert rel_l2(y1[:, sl], O.mul_mat(qtype, Wb[sl], Wb[sl].shape[0], K, X)) < TOL_EXACT


def test_back_to_back_on_one_work_buffer(ctx):
    """Ten products of different types, shapes and N issued with no synchronisation between them, all on one work
    buffer: each launch rewrites the records the previous one read and meets its own grid at the shared counter."""
    cases = [(S.Q4_K, 5120, 5120, 4), (S.Q8_0, 6144, 5120, 8), (S.Q6_K, 5120, 17408, 2), (S.IQ4_XS, 17408, 5120, 8),
             (S.Q3_K, 6144, 5120, 1), (S.Q5_K, 5120, 5120, 16), (S.Q4_K, 17408, 5120, 4), (S.Q8_0, 5120, 17408, 3),
             (S.Q6_K, 6144, 5120, 9), (S.IQ4_XS, 5120, 5120, 2)]
    prods = [_product(q, r, k, n, 500 + i) for i, (q, r, k, n) in enumerate(cases)]
    sizes = [ctx.mul_mat_work_size(W, Xd)[1] for _, W, Xd, _ in prods]
    work = torch.empty(max(sizes), dtype=torch.uint8, device="cuda")
    want = [ctx.mul_mat(W, Xd).cpu().numpy() for _, W, Xd, _ in prods]
    outs = [torch.empty((Xd.shape[0], W.rows), dtype=torch.float32, device="cuda") for _, W, Xd, _ in prods]
    for _ in range(3):
        for (_, W, Xd, _), o in zip(prods, outs):
            ctx.mul_mat(W, Xd, out=o, work=work, fused_quant=True)
    torch.cuda.synchronize()
    ctx.check()
    for o, w in zip(outs, want):
        assert np.array_equal(o.cpu().numpy(), w)


def test_graph_replays(ctx):
    """Three fused products captured in one CUDA graph and replayed: the grid counter keeps advancing."""
    cases = [(S.Q4_K, 17408, 5120, 4), (S.Q3_K, 5120, 5120, 8), (S.Q8_0, 6144, 5120, 2)]
    prods = [_product(q, r, k, n, 900 + i) for i, (q, r, k, n) in enumerate(cases)]
    work = torch.empty(max(ctx.mul_mat_work_size(W, Xd)[1] for _, W, Xd, _ in prods), dtype=torch.uint8,
                       device="cuda")
    outs = [torch.empty((Xd.shape[0], W.rows), dtype=torch.float32, device="cuda") for _, W, Xd, _ in prods]
    calls = [ctx.prepare_mul_mat(W, Xd, o, work, fused_quant=True) for (_, W, Xd, _), o in zip(prods, outs)]
    s = torch.cuda.Stream()
    s.wait_stream(torch.cuda.current_stream())
    with torch.cuda.stream(s):
        for c in calls:  # first calls outside capture (tensor maps, attributes, the counter slot)
            c()
    torch.cuda.current_stream().wait_stream(s)
    torch.cuda.synchronize()
    g = torch.cuda.CUDAGraph()
    with torch.cuda.graph(g):
        for c in calls:
            c()
    want = [ctx.mul_mat(W, Xd).cpu().numpy() for _, W, Xd, _ in prods]
    for rep in range(5):
        for o in outs:
            o.zero_()
        g.replay()
        torch.cuda.synchronize()
        for o, w in zip(outs, want):
            assert np.array_equal(o.cpu().numpy(), w), rep
    del g
    ctx.check()


SWIGLU_TYPES = [S.Q4_K, S.Q5_K, S.Q6_K, S.Q3_K, S.IQ4_XS]


@pytest.mark.parametrize("qtype", SWIGLU_TYPES)
@pytest.mark.parametrize("N", [1, 4, 9, 16])
@pytest.mark.parametrize("shape", [(133, 1280), (5120, 17408), (2048, 5120)])
def test_swiglu_in_gemm_equals_swiglu_quant(ctx, qtype, N, shape):
    """srhpm_mul_mat_swiglu (the SwiGLU of gate and up computed and quantized in the GEMM grid's prologue) against
    srhpm_swiglu_quant + srhpm_mul_mat_prequantized on the same halves of one gate|up product: bit-identical outputs
    (the same records); one launch when the grid is large enough for the prologue, else the SwiGLU record kernel
    first (two). Against the exact oracle on the SwiGLU rows the separate path stored."""
    import ctypes
    rows, K = shape
    rng = np.random.default_rng(rows + K + N + qtype)
    Wb = O.random_blocks(qtype, rows * K // O.BLOCK_ELEMS[qtype], rng).reshape(rows, -1)
    W = S.QuantTensor.from_blocks(Wb, qtype, rows, K)
    gu = torch.from_numpy(rng.standard_normal((N, 2 * K)).astype(np.float32)).cuda()
    gate, up = gu[:, :K], gu[:, K:]
    lib = L.load()
    h = torch.empty((N, K), dtype=torch.float32, device="cuda")
    y0 = torch.empty((N, rows), dtype=torch.float32, device="cuda")
    st, ws = ctx.mul_mat_work_size(W, h)
    work = torch.empty(ws, dtype=torch.uint8, device="cuda")
    wv, hv, yv = W.view(), S.f32_rows_view(h), S.f32_rows_view(y0)
    ptr = lambda t: ctypes.c_void_p(t.data_ptr())
    ctx.launch_count(reset=True)
    y1 = ctx.mul_mat_swiglu(W, gate, up)
    torch.cuda.synchronize()
    l1 = ctx.launch_count(reset=True)
    L.check(lib.srhpm_swiglu_quant(ctx.handle, ptr(gu), ctypes.c_void_p(gu.data_ptr() + 4 * K), gu.stride(0), ptr(h),
                                   h.stride(0), N, ctypes.byref(wv), ptr(work), work.numel(), None),
            "srhpm_swiglu_quant")
    L.check(lib.srhpm_mul_mat_prequantized(ctx.handle, ctypes.byref(wv), ctypes.byref(hv), ctypes.byref(yv),
                                           ptr(work), work.numel(), None), "srhpm_mul_mat_prequantized")
    torch.cuda.synchronize()
    ctx.check()
    assert torch.equal(y1, y0)
    if rows >= 2048:
        assert l1 == 1
    else:
        assert l1 in (1, 2)
    sl = slice(0, 64)
    assert rel_l2(y1.cpu().numpy()[:, sl], O.mul_mat(qtype, Wb[sl], 64, K, h.cpu().numpy())) < TOL_EXACT


def test_swiglu_in_gemm_graph_replays_and_q8_0(ctx):
    """The SwiGLU prologue under CUDA-graph replays (the grid counter advances), and Q8_0 weights refused."""
    rng = np.random.default_rng(77)
    rows, K, N = 5120, 17408, 9
    W = S.QuantTensor.from_blocks(O.random_blocks(S.Q4_K, rows * K // 256, rng).reshape(rows, -1), S.Q4_K, rows, K)
    gu = torch.from_numpy(rng.standard_normal((N, 2 * K)).astype(np.float32)).cuda()
    want = ctx.mul_mat_swiglu(W, gu[:, :K], gu[:, K:]).clone()
    out = torch.empty_like(want)
    work = torch.empty(ctx.mul_mat_work_size(W, gu[:, :K])[1], dtype=torch.uint8, device="cuda")
    s = torch.cuda.Stream()
    s.wait_stream(torch.cuda.current_stream())
    with torch.cuda.stream(s):
        ctx.mul_mat_swiglu(W, gu[:, :K], gu[:, K:], out=out, work=work, stream=s)
    torch.cuda.current_stream().wait_stream(s)
    torch.cuda.synchronize()
    g = torch.cuda.CUDAGraph()
    with torch.cuda.graph(g):
        ctx.mul_mat_swiglu(W, gu[:, :K], gu[:, K:], out=out, work=work)
    for rep in range(4):
        out.zero_()
        g.replay()
        torch.cuda.synchronize()
        assert torch.equal(out, want), rep
    del g
    ctx.check()
    W8 = S.QuantTensor.from_blocks(O.random_blocks(S.Q8_0, 64 * 1024 // 32, rng).reshape(64, -1), S.Q8_0, 64, 1024)
    gu8 = torch.zeros((2, 2048), device="cuda")
    with pytest.raises(L.SrhpmError) as e:
        ctx.mul_mat_swiglu(W8, gu8[:, :1024], gu8[:, 1024:])
    assert e.value.status == L.UNSUPPORTED
