"""KV-cache append of the new tokens (srhpm_rope_kv), byte for byte against the oracle's cache store.

The reference stores K and V rows with ggml_cpy f32 -> the cache type: for a q8_0 cache that is the q8_0 quantizer
of the cache type (patch/srhpm.patch:670-673 is the same from_float on the query side), for f16 a rounding to
nearest even. srhpm_rope_kv turns the keys in place inside the fused QKV rows before storing them, so the stored K
rows are compared with the oracle's store of those rotated rows (bit for bit), the rotation itself with the oracle's
NeoX RoPE (f64 math; within 1e-5 of the largest value), and the V rows with the oracle's store of the untouched input (bit for bit).
Rows of other positions stay as they were; a second append at an earlier position overwrites exactly its rows (the
server's truncate-on-rollback, patch/srhpm.patch:7202, done by writing over the rejected rows)."""
import ctypes

import numpy as np
import pytest
import torch

import oracle as O
import srhpm_b200 as S
from srhpm_b200 import _lib as L
from srhpm_b200.ops import _tensor_view

pytestmark = pytest.mark.gpu

H, HKV, HD = 6, 2, 256


def _append(ctx, qkv, pos, kc, vc, kv_type, base=1e6):
    lib = L.load()
    n = qkv.shape[0]
    tsz = 34 if kv_type == L.Q8_0 else 2
    cap = kc.shape[0]
    kv = _tensor_view(kc, kv_type, [HD, cap, HKV], [tsz, kc.stride(0), kc.stride(1)])
    vv = _tensor_view(vc, kv_type, [HD, cap, HKV], [tsz, vc.stride(0), vc.stride(1)])
    pos_d = torch.tensor(pos, dtype=torch.int32, device="cuda")
    st = lib.srhpm_rope_kv(ctx.handle, ctypes.c_void_p(qkv.data_ptr()), qkv.stride(0), n, H, HKV, HD,
                           ctypes.c_void_p(pos_d.data_ptr()), ctypes.c_float(base), ctypes.byref(kv),
                           ctypes.byref(vv), None)
    assert st == L.OK
    torch.cuda.synchronize()
    ctx.check()


@pytest.mark.parametrize("mode", [L.Q8_0_ACT_SIMD, L.Q8_0_ACT_REF])
@pytest.mark.parametrize("kv_type", [L.F16, L.Q8_0])
def test_kv_append_bytes_exact(ctx, kv_type, mode):
    rng = np.random.default_rng(21 + kv_type + 3 * mode)
    n, cap, p0 = 9, 64, 40
    row = HD // 32 * 34 if kv_type == L.Q8_0 else HD * 2
    x = rng.standard_normal((n, (H + 2 * HKV) * HD)).astype(np.float32)
    x[3, (H + HKV) * HD + 5] = 0.0
    x[4, (H + HKV) * HD:(H + HKV) * HD + 32] = 0.0                      # an all-zero q8_0 block of V
    x[5, H * HD:(H + 1) * HD] *= 1e-30                                  # tiny keys
    x[6, (H + HKV + 1) * HD:] = rng.integers(-3, 4, HD) * 0.5          # ties of the rounding
    kc0 = torch.from_numpy(rng.integers(0, 256, (cap, HKV, row), dtype=np.uint8)).cuda()
    vc0 = torch.from_numpy(rng.integers(0, 256, (cap, HKV, row), dtype=np.uint8)).cuda()
    kc, vc = kc0.clone(), vc0.clone()
    qkv = torch.from_numpy(x).cuda()
    pos = list(range(p0, p0 + n))
    ctx.set_q8_0_act_mode(mode)
    try:
        _append(ctx, qkv, pos, kc, vc, kv_type)
    finally:
        ctx.set_q8_0_act_mode(L.Q8_0_ACT_SIMD)
    turned = qkv.cpu().numpy().reshape(n, H + 2 * HKV, HD)
    want_rot = O.rope_neox(x.reshape(n, H + 2 * HKV, HD)[:, :H + HKV], pos, 1e6)
    assert np.abs(turned[:, :H + HKV] - want_rot).max() <= 1e-5 * np.abs(want_rot).max()
    assert np.array_equal(turned[:, H + HKV:], x.reshape(n, H + 2 * HKV, HD)[:, H + HKV:])  # V untouched
    k_want = O.cache_rows(kv_type, turned[:, H:H + HKV], mode)
    v_want = O.cache_rows(kv_type, x.reshape(n, H + 2 * HKV, HD)[:, H + HKV:], mode)
    kg, vg = kc.cpu().numpy(), vc.cpu().numpy()
    assert np.array_equal(kg[p0:p0 + n], k_want)
    assert np.array_equal(vg[p0:p0 + n], v_want)
    # every other row untouched
    keep = np.r_[0:p0, p0 + n:cap]
    assert np.array_equal(kg[keep], kc0.cpu().numpy()[keep])
    assert np.array_equal(vg[keep], vc0.cpu().numpy()[keep])


@pytest.mark.parametrize("kv_type", [L.F16, L.Q8_0])
def test_kv_append_rollback_overwrites_rejected_rows(ctx, kv_type):
    """Step 1 appends 9 rows at 10..18 and accepts 3 (rows 10..12 stay); step 2 appends at 13.. and must leave
    10..12 as they were and replace 13..21."""
    rng = np.random.default_rng(5)
    cap = 32
    row = HD // 32 * 34 if kv_type == L.Q8_0 else HD * 2
    kc = torch.zeros((cap, HKV, row), dtype=torch.uint8, device="cuda")
    vc = torch.zeros_like(kc)
    x1 = rng.standard_normal((9, (H + 2 * HKV) * HD)).astype(np.float32)
    x2 = rng.standard_normal((9, (H + 2 * HKV) * HD)).astype(np.float32)
    _append(ctx, torch.from_numpy(x1).cuda(), list(range(10, 19)), kc, vc, kv_type)
    first_k, first_v = kc.cpu().numpy().copy(), vc.cpu().numpy().copy()
    _append(ctx, torch.from_numpy(x2).cuda(), list(range(13, 22)), kc, vc, kv_type)
    k2, v2 = kc.cpu().numpy(), vc.cpu().numpy()
    assert np.array_equal(k2[10:13], first_k[10:13]) and np.array_equal(v2[10:13], first_v[10:13])
    v_want = O.cache_rows(kv_type, x2.reshape(9, H + 2 * HKV, HD)[:, H + HKV:])
    assert np.array_equal(v2[13:22], v_want)
    assert not k2[22:].any() and not v2[22:].any() and not k2[:10].any()
