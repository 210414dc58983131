"""GPU parity of the multi-query attention (srhpm_flash_attn_ext) against the oracle and the reference's own grouped
FA function (ggml_compute_forward_flash_attn_ext_gqa_small, compiled from its patch into oracle/_ref).

Bar: within 1e-3 relative L2 of the reference's f32 result (the stated tolerance for attention) and of the f64
oracle. The Q.K part is exact integer arithmetic in both; the differences come from P and V entering the tensor cores
as f16 (about 3e-4 relative L2 on random data)."""
import numpy as np
import pytest
import torch

import oracle as O
import srhpm_b200 as S
from srhpm_b200 import _lib as L

pytestmark = pytest.mark.gpu

TOL = 1e-3
D = 256


def rel_l2(a, b):
    a = np.asarray(a, np.float64)
    b = np.asarray(b, np.float64)
    return float(np.linalg.norm(a - b) / max(np.linalg.norm(b), 1e-30))


def q8_rows(x):
    """f32 [..., 256] -> q8_0 bytes [..., 272] (host quantizer of this library; any valid q8_0 bytes do)."""
    shp = x.shape
    b = S.quantize_chunk(np.ascontiguousarray(x.reshape(-1, shp[-1]), np.float32), S.Q8_0)
    return b.reshape(*shp[:-1], -1)


def causal_mask(N, L, width=None):
    m = np.zeros((N, width or L), np.float16)
    for t in range(N):
        m[t, L - N + t + 1:] = -np.inf
    return m


def inputs(rng, H, Hkv, N, L, qscale=1 / 16, kscale=1.0):
    q = (rng.standard_normal((H, N, D)) * qscale).astype(np.float32)
    k = q8_rows((rng.standard_normal((Hkv, L, D)) * kscale).astype(np.float32))
    v = q8_rows(rng.standard_normal((Hkv, L, D)).astype(np.float32))
    return q, k, v


def run(ctx, q, k, v, mask=None, sinks=None, **kw):
    t = lambda a: torch.from_numpy(np.ascontiguousarray(a)).cuda()
    out = ctx.flash_attn_ext(t(q), t(k), t(v), S.Q8_0, mask=t(mask) if mask is not None else None,
                             sinks=t(sinks) if sinks is not None else None, **kw)
    torch.cuda.synchronize()
    ctx.check()
    return out.cpu().numpy()


def oracle(q, k, v, Hkv, mask=None, sinks=None, **kw):
    L = k.shape[1]
    m16 = mask.view(np.uint16) if mask is not None else None
    return O.attention(q, O.Q8_0, k, v, D, L, Hkv, mask=m16, sinks=sinks, **kw)


@pytest.mark.parametrize("H,Hkv,N,L", [(24, 4, 8, 1000), (6, 2, 5, 192), (6, 1, 2, 129), (8, 8, 1, 77),
                                       (12, 2, 16, 300), (4, 1, 3, 5000), (4, 2, 12, 700)])
def test_fa_q8_0_vs_oracle_and_reference(ctx, ref, H, Hkv, N, L):
    rng = np.random.default_rng(H * 1000 + L)
    q, k, v = inputs(rng, H, Hkv, N, L)
    mask = causal_mask(N, L)
    got = run(ctx, q, k, v, mask=mask)
    exp = oracle(q, k, v, Hkv, mask=mask)
    assert rel_l2(got, exp) < TOL
    if ref is not None and 2 <= N <= 8:  # the reference's grouped path takes 2..8 query tokens (P:833-841)
        r = O.ref_fa_gqa(q, O.Q8_0, k, v, D, L, Hkv, mask=mask.view(np.uint16), nth=4, lib=ref)
        assert rel_l2(got, r) < TOL


@pytest.mark.parametrize("extras", ["sinks", "softcap", "alibi", "scale", "nomask"])
def test_fa_q8_0_options(ctx, ref, extras):
    rng = np.random.default_rng(7)
    H, Hkv, N, L = 24, 4, 8, 700
    q, k, v = inputs(rng, H, Hkv, N, L)
    mask, sinks, kw = causal_mask(N, L), None, dict(scale=1.0, max_bias=0.0, softcap=0.0)
    if extras == "sinks":
        sinks = rng.standard_normal(H).astype(np.float32)
    elif extras == "softcap":
        kw.update(scale=4.0, softcap=20.0)
    elif extras == "alibi":
        kw.update(max_bias=8.0)
    elif extras == "scale":
        kw.update(scale=0.0625)
    else:
        mask = None
    got = run(ctx, q, k, v, mask=mask, sinks=sinks, **kw)
    exp = oracle(q, k, v, Hkv, mask=mask, sinks=sinks, **kw)
    assert rel_l2(got, exp) < TOL
    if ref is not None:
        r = O.ref_fa_gqa(q, O.Q8_0, k, v, D, L, Hkv, mask=mask.view(np.uint16) if mask is not None else None,
                         sinks=sinks, nth=4, lib=ref, **kw)
        assert rel_l2(got, r) < TOL


def test_fa_q8_0_peaky_scores(ctx):
    """Large score spread (sharp softmax, the running maximum rises across tiles): the lazy rescale must hold."""
    rng = np.random.default_rng(11)
    H, Hkv, N, L = 12, 2, 4, 2000
    q, k, v = inputs(rng, H, Hkv, N, L, qscale=1.0, kscale=1.0)
    k2 = k.copy()
    got = run(ctx, q, k2, v, scale=0.5)
    exp = oracle(q, k2, v, Hkv, scale=0.5)
    assert rel_l2(got, exp) < TOL


@pytest.mark.parametrize("mode", [L.Q8_0_ACT_SIMD, L.Q8_0_ACT_REF])
def test_fa_q8_0_act_modes(ctx, mode):
    rng = np.random.default_rng(12)
    H, Hkv, N, n_kv = 6, 2, 4, 300
    q, k, v = inputs(rng, H, Hkv, N, n_kv, qscale=0.5)
    ctx.set_q8_0_act_mode(mode)
    try:
        got = run(ctx, q, k, v, mask=causal_mask(N, n_kv))
    finally:
        ctx.set_q8_0_act_mode(L.Q8_0_ACT_SIMD)
    exp = O.attention(q, O.Q8_0, k, v, D, n_kv, Hkv, mask=causal_mask(N, n_kv).view(np.uint16), q8_mode=mode)
    assert rel_l2(got, exp) < TOL


def test_fa_q8_0_llama_cache_layout_and_padded_mask(ctx):
    """KV as llama.cpp's cache view ([L][Hkv][row]: token stride Hkv * 272), mask padded wider and taller."""
    rng = np.random.default_rng(13)
    H, Hkv, N, L = 24, 4, 8, 900
    q, k, v = inputs(rng, H, Hkv, N, L)
    mask = causal_mask(N, L)
    mpad = np.full((16, 1024), -np.inf, np.float16)
    mpad[:N, :L] = mask
    kl = torch.from_numpy(np.ascontiguousarray(k.transpose(1, 0, 2))).cuda().permute(1, 0, 2)
    vl = torch.from_numpy(np.ascontiguousarray(v.transpose(1, 0, 2))).cuda().permute(1, 0, 2)
    out = ctx.flash_attn_ext(torch.from_numpy(q).cuda(), kl, vl, S.Q8_0, mask=torch.from_numpy(mpad).cuda())
    torch.cuda.synchronize()
    exp = oracle(q, k, v, Hkv, mask=mask)
    assert rel_l2(out.cpu().numpy(), exp) < TOL


def test_fa_q8_0_per_head_mask_and_masked_rows(ctx):
    """mask ne2 = H (slice h % ne2 per head); one head's mask hides every token (its rows must come out 0)."""
    rng = np.random.default_rng(14)
    H, Hkv, N, L = 6, 2, 3, 400
    q, k, v = inputs(rng, H, Hkv, N, L)
    m = np.zeros((H, N, L), np.float16)
    for h in range(H):
        m[h, :, rng.integers(0, L, 50)] = -np.inf
    m[4] = -np.inf
    got = run(ctx, q, k, v, mask=m)
    exp = np.zeros_like(got)
    for h in range(H):
        g = h // (H // Hkv)
        exp[:, h] = O.attention(q[h:h + 1], O.Q8_0, k[g:g + 1], v[g:g + 1], D, L, 1,
                                mask=np.ascontiguousarray(m[h]).view(np.uint16))[:, 0]
    assert np.all(got[:, 4] == 0.0)
    assert rel_l2(got, exp) < TOL


def test_fa_q8_0_L131072_full_size(ctx):
    """The verify attention shape at L = 131072 (Q [256, 8, 24], q8_0 K/V [256, L, 4], causal mask among the 8
    draft rows): the kernel runs the whole problem; the f64 oracle checks two of the four KV heads."""
    rng = np.random.default_rng(15)
    H, Hkv, N, L = 24, 4, 8, 131072
    q, k, v = inputs(rng, H, Hkv, N, L)
    mask = causal_mask(N, L)
    got = run(ctx, q, k, v, mask=mask, scale=0.0625)
    G = H // Hkv
    for g in (0, 3):
        exp = O.attention(q[g * G:(g + 1) * G], O.Q8_0, k[g:g + 1], v[g:g + 1], D, L, 1,
                          mask=mask.view(np.uint16), scale=0.0625)
        assert rel_l2(got[:, g * G:(g + 1) * G], exp) < TOL


def test_fa_repeatable(ctx):
    rng = np.random.default_rng(16)
    q, k, v = inputs(rng, 24, 4, 8, 3000)
    a = run(ctx, q, k, v, mask=causal_mask(8, 3000))
    b = run(ctx, q, k, v, mask=causal_mask(8, 3000))
    assert np.array_equal(a, b)


def test_fa_status_codes(ctx):
    rng = np.random.default_rng(17)
    q, k, v = inputs(rng, 6, 2, 4, 256)
    tq, tk, tv = (torch.from_numpy(a).cuda() for a in (q, k, v))
    with pytest.raises(L.SrhpmError) as e:          # head count not a multiple of the KV heads
        ctx.flash_attn_ext(tq[:5], tk, tv, S.Q8_0)
    assert e.value.status == L.ERR_INVALID
    with pytest.raises(L.SrhpmError) as e:          # K and V of different types
        kf = torch.zeros((2, 256, 512), dtype=torch.uint8, device="cuda")
        ctx.flash_attn_ext(tq, kf, tv, S.F16)
    assert e.value.status in (L.UNSUPPORTED, L.ERR_INVALID)
    with pytest.raises(L.SrhpmError) as e:          # head size 128: not this kernel
        k128 = torch.zeros((2, 256, 136), dtype=torch.uint8, device="cuda")
        ctx.flash_attn_ext(tq[:, :, :128].contiguous(), k128, k128, S.Q8_0)
    assert e.value.status in (L.UNSUPPORTED, L.ERR_ALIGN)
    with pytest.raises(L.SrhpmError) as e:          # token stride not a multiple of 16 bytes
        kk = torch.zeros((2, 256, 280), dtype=torch.uint8, device="cuda")[:, :, :272]
        ctx.flash_attn_ext(tq, kk, kk, S.Q8_0)
    assert e.value.status == L.ERR_ALIGN


# ---- f16 KV cache ---------------------------------------------------------------------------------------------------

def f16_inputs(rng, H, Hkv, N, L, qscale=1 / 16, kscale=1.0):
    q = (rng.standard_normal((H, N, D)) * qscale).astype(np.float32)
    k = (rng.standard_normal((Hkv, L, D)) * kscale).astype(np.float16).view(np.uint8)
    v = rng.standard_normal((Hkv, L, D)).astype(np.float16).view(np.uint8)
    return q, k, v


def run16(ctx, q, k, v, mask=None, sinks=None, **kw):
    t = lambda a: torch.from_numpy(np.ascontiguousarray(a)).cuda()
    out = ctx.flash_attn_ext(t(q), t(k), t(v), S.F16, mask=t(mask) if mask is not None else None,
                             sinks=t(sinks) if sinks is not None else None, **kw)
    torch.cuda.synchronize()
    ctx.check()
    return out.cpu().numpy()


@pytest.mark.parametrize("H,Hkv,N,L", [(24, 4, 9, 2057), (24, 4, 8, 1000), (6, 2, 5, 192), (8, 8, 1, 77),
                                       (12, 2, 16, 300), (4, 1, 3, 5000)])
def test_fa_f16_vs_oracle_and_reference(ctx, ref, H, Hkv, N, L):
    rng = np.random.default_rng(H * 1000 + L + 1)
    q, k, v = f16_inputs(rng, H, Hkv, N, L)
    mask = causal_mask(N, L)
    got = run16(ctx, q, k, v, mask=mask)
    exp = O.attention(q, O.F16, k, v, D, L, Hkv, mask=mask.view(np.uint16))
    assert rel_l2(got, exp) < TOL
    if ref is not None and 2 <= N <= 8:
        r = O.ref_fa_gqa(q, O.F16, k, v, D, L, Hkv, mask=mask.view(np.uint16), nth=4, lib=ref)
        assert rel_l2(got, r) < TOL


@pytest.mark.parametrize("extras", ["sinks", "softcap", "alibi", "nomask", "peaky"])
def test_fa_f16_options(ctx, ref, extras):
    rng = np.random.default_rng(21)
    H, Hkv, N, L = 24, 4, 8, 700
    q, k, v = f16_inputs(rng, H, Hkv, N, L, qscale=1.0 if extras == "peaky" else 1 / 16)
    mask, sinks, kw = causal_mask(N, L), None, dict(scale=1.0, max_bias=0.0, softcap=0.0)
    if extras == "sinks":
        sinks = rng.standard_normal(H).astype(np.float32)
    elif extras == "softcap":
        kw.update(scale=4.0, softcap=20.0)
    elif extras == "alibi":
        kw.update(max_bias=8.0)
    elif extras == "peaky":
        kw.update(scale=0.5)
    else:
        mask = None
    got = run16(ctx, q, k, v, mask=mask, sinks=sinks, **kw)
    m16 = mask.view(np.uint16) if mask is not None else None
    exp = O.attention(q, O.F16, k, v, D, L, Hkv, mask=m16, sinks=sinks, **kw)
    assert rel_l2(got, exp) < TOL
    if ref is not None:
        r = O.ref_fa_gqa(q, O.F16, k, v, D, L, Hkv, mask=m16, sinks=sinks, nth=4, lib=ref, **kw)
        assert rel_l2(got, r) < TOL


def test_fa_f16_llama_cache_layout(ctx):
    rng = np.random.default_rng(22)
    H, Hkv, N, L = 24, 4, 9, 2057
    q, k, v = f16_inputs(rng, H, Hkv, N, L)
    mask = causal_mask(N, L)
    kl = torch.from_numpy(np.ascontiguousarray(k.transpose(1, 0, 2))).cuda().permute(1, 0, 2)
    vl = torch.from_numpy(np.ascontiguousarray(v.transpose(1, 0, 2))).cuda().permute(1, 0, 2)
    out = ctx.flash_attn_ext(torch.from_numpy(q).cuda(), kl, vl, S.F16, mask=torch.from_numpy(mask).cuda())
    torch.cuda.synchronize()
    exp = O.attention(q, O.F16, k, v, D, L, Hkv, mask=mask.view(np.uint16))
    assert rel_l2(out.cpu().numpy(), exp) < TOL
