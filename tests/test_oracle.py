"""CPU tests of the oracle: pinned against the reference's own kernels (compiled from its patch), the committed golden
fixtures, gguf-py's independent block decoders, and the format definitions."""
import numpy as np
import pytest

import oracle as O


def rel_l2(a, b):
    a = np.asarray(a, np.float64)
    b = np.asarray(b, np.float64)
    return float(np.linalg.norm(a - b) / max(np.linalg.norm(b), 1e-30))


def test_fp16_conversion_matches_numpy():
    rng = np.random.default_rng(3)
    x = np.concatenate([rng.standard_normal(4000).astype(np.float32) * 10.0 ** rng.integers(-9, 5, 4000),
                        np.array([0.0, -0.0, 65504.0, 65519.0, 65520.0, 1e-8, 6.0e-8, 2.98e-8, 6.1e-5, 6.09e-5,
                                  np.inf, -np.inf], np.float32)]).astype(np.float32)
    ours = O.fp32_to_fp16_bits(x)
    with np.errstate(over="ignore"):
        want = x.astype(np.float16).view(np.uint16)
    assert np.array_equal(ours, want)


def test_block_sizes_match_gguf():
    gguf = pytest.importorskip("gguf")
    T = gguf.GGMLQuantizationType
    for name, t in [("Q4_K", O.Q4_K), ("Q5_K", O.Q5_K), ("Q6_K", O.Q6_K), ("Q3_K", O.Q3_K), ("IQ4_XS", O.IQ4_XS),
                    ("Q8_0", O.Q8_0)]:
        assert gguf.GGML_QUANT_SIZES[getattr(T, name)] == (O.BLOCK_ELEMS[t], O.BLOCK_BYTES[t])
        assert int(getattr(T, name)) == t


@pytest.mark.parametrize("qtype", [O.Q4_K, O.Q5_K, O.Q6_K, O.Q3_K, O.IQ4_XS, O.Q8_0])
def test_dequantize_matches_gguf(qtype):
    gguf = pytest.importorskip("gguf")
    from gguf import quants
    names = {O.Q4_K: "Q4_K", O.Q5_K: "Q5_K", O.Q6_K: "Q6_K", O.Q3_K: "Q3_K", O.IQ4_XS: "IQ4_XS", O.Q8_0: "Q8_0"}
    rng = np.random.default_rng(11)
    nblk = 64
    blocks = O.random_blocks(qtype, nblk, rng)
    n = nblk * O.BLOCK_ELEMS[qtype]
    ours = O.dequantize(qtype, blocks, n)
    theirs = quants.dequantize(blocks.reshape(1, -1), getattr(gguf.GGMLQuantizationType, names[qtype])).reshape(-1)
    assert np.allclose(ours, theirs, rtol=1e-6, atol=1e-7)


def _edge_rows(K):
    rng = np.random.default_rng(5)
    rows = [rng.standard_normal(K).astype(np.float32),
            np.zeros(K, np.float32),                                     # all zero: q = 0, d = 0
            np.full(K, -2.5, np.float32),                                # every element ties for the max magnitude
            (rng.standard_normal(K) * 1e-30).astype(np.float32),         # tiny values
            (rng.integers(-4, 5, K) * 0.5).astype(np.float32)]           # many exact x.5 products (rounding ties)
    r = rng.standard_normal(K).astype(np.float32)
    r[7], r[100] = -3.0, 3.0                                             # first max is negative
    rows.append(r)
    return rows


def test_q8K_quantizer_bit_exact_vs_reference(ref):
    if ref is None:
        pytest.skip("reference kernels not built (no reference at build time)")
    for x in _edge_rows(1024):
        ours = O.quantize_row_q8K(x)
        theirs = O.ref_quantize_row(x, ref)
        for a, b in zip(ours, theirs):
            assert np.array_equal(a.view(np.uint8), b.view(np.uint8))


@pytest.mark.parametrize("qtype", O.SRV_TYPES)
@pytest.mark.parametrize("N", [1, 2, 3, 4, 5, 8, 9, 16])
def test_oracle_matmul_vs_reference_kernels(ref, qtype, N):
    """The exact-integer oracle against the reference's srv_row kernels (launcher settings: OFF=1, PAIR=1)."""
    if ref is None:
        pytest.skip("reference kernels not built")
    rng = np.random.default_rng(100 + N + qtype)
    K, rows = 768, 37
    W = O.random_blocks(qtype, rows * K // 256, rng)
    X = rng.standard_normal((N, K)).astype(np.float32)
    y_orc = O.mul_mat(qtype, W, rows, K, X)
    y_ref = O.ref_mul_mat(qtype, W, rows, K, X, nth=2, lib=ref)
    assert rel_l2(y_ref, y_orc) < 2e-6


def test_reference_kernel_variants_agree(ref):
    """The reference's own exactness claims: offset path == sign path; paired IQ4_XS ~ plain (1e-7 rel)."""
    if ref is None:
        pytest.skip("reference kernels not built")
    rng = np.random.default_rng(9)
    K, rows = 512, 40
    for qtype in (O.Q3_K, O.Q6_K):
        W = O.random_blocks(qtype, rows * K // 256, rng)
        X = rng.standard_normal((8, K)).astype(np.float32)
        a = O.ref_mul_mat(qtype, W, rows, K, X, off=1, lib=ref)
        b = O.ref_mul_mat(qtype, W, rows, K, X, off=0, lib=ref)
        assert rel_l2(a, b) < 1e-6
    W = O.random_blocks(O.IQ4_XS, rows * K // 256, rng)
    X = rng.standard_normal((8, K)).astype(np.float32)
    assert rel_l2(O.ref_mul_mat(O.IQ4_XS, W, rows, K, X, paired=1, lib=ref),
                  O.ref_mul_mat(O.IQ4_XS, W, rows, K, X, paired=0, lib=ref)) < 1e-6


@pytest.mark.parametrize("qtype", [O.Q4_K, O.Q5_K, O.Q6_K, O.Q3_K, O.IQ4_XS, O.Q8_0])
def test_isums_reconstruct_dequantized_dot(qtype):
    """Integer sums x scales == the f64 dot of dequantized weights and dequantized activations."""
    rng = np.random.default_rng(21)
    K = 512
    W = O.random_blocks(qtype, K // O.BLOCK_ELEMS[qtype], rng)
    x = rng.standard_normal(K).astype(np.float32)
    wf = O.dequantize(qtype, W, K).astype(np.float64)
    if qtype == O.Q8_0:
        qb = O.quantize_row_q8_0(x).reshape(-1, 34)
        xq = qb[:, 2:].copy().view(np.int8).reshape(-1)
        xd = np.repeat(qb[:, :2].copy().view(np.float16).astype(np.float64).reshape(-1), 32)
        m, _ = O.row_isums(qtype, W, xq, None, K)
        dw = W.reshape(-1, 34)[:, :2].copy().view(np.float16).astype(np.float64).reshape(-1)
        got = float(np.sum(dw * xd[::32] * m))
        want = float(np.dot(wf, xq * xd))
    else:
        xq, d, b32, _ = O.quantize_row_q8K(x)
        m, mn = O.row_isums(qtype, W, xq, b32, K)
        bl = W.reshape(-1, O.BLOCK_BYTES[qtype])
        doff = O.D_OFFSET[qtype]
        dw = bl[:, doff[0]:doff[0] + 2].copy().view(np.float16).astype(np.float64).reshape(-1)
        got = float(np.sum(dw * d * m))
        if qtype in (O.Q4_K, O.Q5_K):
            dmin = bl[:, 2:4].copy().view(np.float16).astype(np.float64).reshape(-1)
            got -= float(np.sum(dmin * d * mn))
        want = float(np.dot(wf, xq.astype(np.float64) * np.repeat(d, 256)))
    assert abs(got - want) <= 1e-5 * max(1.0, abs(want))


def test_q8_0_ref_quantizer_matches_gguf():
    """ORC_Q8_0_REF follows ggml's quantize_row_q8_0_ref, which gguf-py's Q8_0 reproduces."""
    gguf = pytest.importorskip("gguf")
    from gguf import quants
    rng = np.random.default_rng(4)
    x = np.concatenate([rng.standard_normal(4096), rng.integers(-3, 4, 1024) * 0.25]).astype(np.float32)
    ours = O.quantize_row_q8_0(x, O.Q8_0_REF)
    theirs = quants.quantize(x.reshape(1, -1), gguf.GGMLQuantizationType.Q8_0).reshape(-1)
    assert np.array_equal(ours, theirs)


def test_q8_0_f32_path_vs_exact():
    rng = np.random.default_rng(6)
    K, rows = 1024, 50
    W = O.random_blocks(O.Q8_0, rows * K // 32, rng)
    X = rng.standard_normal((5, K)).astype(np.float32)
    assert rel_l2(O.mul_mat_q8_0_f32(W, rows, K, X, nth=3), O.mul_mat(O.Q8_0, W, rows, K, X)) < 2e-6


def _fa_inputs(kv_type, rng, H=4, Hkv=2, N=4, D=128, L=160):
    q = (rng.standard_normal((H, N, D)) / 16).astype(np.float32)
    kf = rng.standard_normal((Hkv, L, D)).astype(np.float32)
    vf = rng.standard_normal((Hkv, L, D)).astype(np.float32)
    if kv_type == O.F16:
        k, v = kf.astype(np.float16).view(np.uint8), vf.astype(np.float16).view(np.uint8)
    else:
        k = np.stack([O.quantize_row_q8_0(r, O.Q8_0_REF) for r in kf.reshape(-1, D)])
        v = np.stack([O.quantize_row_q8_0(r, O.Q8_0_REF) for r in vf.reshape(-1, D)])
    mask = np.zeros((N, L), np.float16)
    for t in range(N):  # causal among the draft rows at the end of the cache
        mask[t, L - N + t + 1:] = -np.inf
    return q, k, v, mask.view(np.uint16)


@pytest.mark.parametrize("kv_type", [O.F16, O.Q8_0])
@pytest.mark.parametrize("extras", ["plain", "sinks", "softcap", "alibi"])
def test_oracle_attention_vs_reference_fa_gqa(ref, kv_type, extras):
    if ref is None:
        pytest.skip("reference kernels not built")
    rng = np.random.default_rng(31)
    q, k, v, mask = _fa_inputs(kv_type, rng)
    H, N, D = q.shape
    kw = dict(scale=1.0, max_bias=0.0, softcap=0.0)
    sinks = None
    if extras == "sinks":
        sinks = rng.standard_normal(H).astype(np.float32)
    elif extras == "softcap":
        kw.update(scale=4.0, softcap=20.0)
    elif extras == "alibi":
        kw.update(max_bias=8.0)
    a = O.attention(q, kv_type, k, v, D, 160, 2, mask=mask, sinks=sinks, **kw)
    b = O.ref_fa_gqa(q, kv_type, k, v, D, 160, 2, mask=mask, sinks=sinks, nth=3, lib=ref, **kw)
    assert rel_l2(b, a) < 1e-5


@pytest.mark.parametrize("kv_type", [O.F16, O.Q8_0])
@pytest.mark.parametrize("extras", ["plain", "sinks", "softcap", "alibi"])
def test_oracle_attention_records_and_merge(kv_type, extras):
    """The record form (attention_partial over token ranges + attention_merge, the reference's chunk records and
    merge, patch/srhpm.patch:779-823): one range merged is the pinned single pass bit for bit; any split of the range,
    with empty ranges and a range the mask hides, agrees with it to f64 rounding."""
    rng = np.random.default_rng(37)
    q, k, v, mask = _fa_inputs(kv_type, rng)
    H, N, D = q.shape
    L = 160
    mask = mask.copy()
    mask[:, 40:80] = 0xFC00  # -inf: the range [40, 80) is hidden from every row
    kw = dict(scale=1.0, max_bias=0.0, softcap=0.0)
    sinks = None
    if extras == "sinks":
        sinks = rng.standard_normal(H).astype(np.float32)
    elif extras == "softcap":
        kw.update(scale=4.0, softcap=20.0)
    elif extras == "alibi":
        kw.update(max_bias=8.0)
    whole = O.attention(q, kv_type, k, v, D, L, 2, mask=mask, sinks=sinks, **kw)
    for cuts in ([0, L], [0, 40, 80, L], [0, 0, 33, 128, 128, L], [0, 1, L]):
        recs = [O.attention_partial(q, kv_type, k, v, D, L, 2, a, b, mask=mask, **kw)
                for a, b in zip(cuts[:-1], cuts[1:])]
        got = O.attention_merge(*(np.stack([r[i] for r in recs]) for i in range(3)), sinks=sinks)
        if len(cuts) == 2:
            assert np.array_equal(got, whole)
        else:
            assert np.abs(got - whole).max() <= 1e-12 * np.abs(whole).max()
    # a range with no finite score has sum 0
    m, s_, acc = O.attention_partial(q, kv_type, k, v, D, L, 2, 40, 80, mask=mask, **kw)
    assert np.all(s_ == 0) and np.all(acc == 0) and np.all(np.isneginf(m))


def test_accept_semantics():
    V = 50
    lg = np.zeros((5, V), np.float32)
    for i, tok in enumerate([3, 7, 9, 11, 13]):
        lg[i, tok] = 1.0
    assert O.accept(lg, [3, 7, 9, 11]) == [3, 7, 9, 11, 13]        # all accepted + bonus
    assert O.accept(lg, [3, 8, 9, 11]) == [3, 7]                   # stop at the first mismatch, with the correction
    assert O.accept(lg, [4, 7, 9, 11]) == [3]
    lg[1, 8] = 0.95                                                # within relax of the best
    assert O.accept(lg, [3, 8, 9, 11], relax=0.1) == [3, 8, 9, 11, 13]  # 8 accepted within relax, the rest match
    assert O.accept(lg, [3, 8, 9, 11], relax=0.01) == [3, 7]             # gap 0.05 > relax
    tie = np.zeros((1, V), np.float32)
    tie[0, [5, 2, 40]] = 2.0
    assert O.accept(tie, []) == [2]                                # ties -> lowest id


@pytest.mark.parametrize("qtype", [O.Q4_K, O.Q5_K, O.Q6_K, O.Q3_K, O.IQ4_XS, O.Q8_0])
def test_quantize_rtn_round_trip(qtype):
    """The oracle's round-to-nearest quantizers (input generation for the CPU reference timings) make blocks that
    the oracle's own decoders turn back into the input within the format's resolution."""
    rng = np.random.default_rng(qtype)
    w = (rng.standard_normal((37, 512)) * 0.02).astype(np.float32)
    w[3] = 0.0
    blocks = O.quantize_rtn(qtype, w, nth=3)
    assert blocks.shape == (37, 512 // O.BLOCK_ELEMS[qtype] * O.BLOCK_BYTES[qtype])
    back = O.dequantize(qtype, blocks.reshape(-1), w.size).reshape(w.shape)
    bar = {O.Q3_K: 0.25, O.Q4_K: 0.12, O.IQ4_XS: 0.12, O.Q5_K: 0.06, O.Q6_K: 0.03, O.Q8_0: 0.01}[qtype]
    assert np.linalg.norm(back - w) / np.linalg.norm(w) < bar
    assert not back[3].any()
