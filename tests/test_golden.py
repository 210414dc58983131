"""CPU: the restated oracle against the committed golden fixtures (outputs of the reference's own kernels), so the
oracle stays pinned even where oracle/_ref cannot be built."""
import os

import numpy as np

import oracle as O

HERE = os.path.join(os.path.dirname(__file__), "golden")


def rel_l2(a, b):
    a = np.asarray(a, np.float64)
    b = np.asarray(b, np.float64)
    return float(np.linalg.norm(a - b) / max(np.linalg.norm(b), 1e-30))


def test_golden_q8K_quantizer():
    g = np.load(os.path.join(HERE, "srv_mul_mat.npz"))
    i = 0
    while f"q8K_{i}_x" in g.files:
        q, d, b32, b16 = O.quantize_row_q8K(g[f"q8K_{i}_x"])
        assert np.array_equal(q, g[f"q8K_{i}_q"])
        assert np.array_equal(d.view(np.uint32), g[f"q8K_{i}_d"].view(np.uint32))
        assert np.array_equal(b32, g[f"q8K_{i}_b32"])
        assert np.array_equal(b16, g[f"q8K_{i}_b16"])
        i += 1
    assert i >= 4


def test_golden_srv_mul_mat():
    g = np.load(os.path.join(HERE, "srv_mul_mat.npz"))
    names = [k[:-5] for k in g.files if k.endswith("_meta")]
    assert len(names) == 5
    for name in names:
        qtype, rows, K = (int(v) for v in g[name + "_meta"])
        y = O.mul_mat(qtype, g[name + "_W"], rows, K, g[name + "_X"])
        assert rel_l2(y, g[name + "_Y"]) < 2e-6, name


def test_golden_fa_gqa():
    g = np.load(os.path.join(HERE, "fa_gqa.npz"))
    for kv in ("f16", "q8_0"):
        kv_type, H, Hkv, N, D, L = (int(v) for v in g[kv + "_meta"])
        q, k, v, mask, sinks = (g[kv + s] for s in ("_q", "_k", "_v", "_mask", "_sinks"))
        for var, kw in (("plain", dict()), ("sinks", dict(sinks=sinks)), ("softcap", dict(scale=4.0, softcap=20.0)),
                        ("alibi", dict(max_bias=8.0))):
            got = O.attention(q, kv_type, k, v, D, L, Hkv, mask=mask, **kw)
            assert rel_l2(got, g[f"{kv}_{var}_dst"]) < 1e-5, (kv, var)
