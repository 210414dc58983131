"""Writes the golden fixtures of tests/golden/ from the reference's OWN kernels, compiled from its patch into
oracle/_ref/ by oracle/build_ref.sh (run `make -C oracle` with the reference available first).

  srv_mul_mat.npz   per type (Q4_K, Q5_K, Q6_K, Q3_K, IQ4_XS): seeded random blocks W, activations X [9, K], and
                    Y = the reference's srv kernels through compute_forward's scheduling (GGML_SRV_OFF=1, paired
                    IQ4_XS: the launcher's settings); plus srv_quantize_row outputs for edge-case rows.
  fa_gqa.npz        ggml_compute_forward_flash_attn_ext_gqa_small outputs for f16 and q8_0 KV caches (causal mask
                    among the draft rows; with sinks / softcap / ALiBi variants).

Usage: python tests/golden/make_golden.py
"""
import os
import sys

import numpy as np

HERE = os.path.dirname(os.path.abspath(__file__))
ROOT = os.path.dirname(os.path.dirname(HERE))
sys.path.insert(0, os.path.join(ROOT, "oracle"))
import oracle as O  # noqa: E402


def srv_fixtures(ref):
    out = {}
    rng = np.random.default_rng(20240601)
    for name, qtype in (("q4_K", O.Q4_K), ("q5_K", O.Q5_K), ("q6_K", O.Q6_K), ("q3_K", O.Q3_K),
                        ("iq4_xs", O.IQ4_XS)):
        rows, K, N = 40, 512, 9
        W = O.random_blocks(qtype, rows * K // 256, rng).reshape(rows, -1)
        X = rng.standard_normal((N, K)).astype(np.float32)
        out[name + "_meta"] = np.array([qtype, rows, K], np.int64)
        out[name + "_W"] = W
        out[name + "_X"] = X
        out[name + "_Y"] = O.ref_mul_mat(qtype, W, rows, K, X, nth=1, off=1, paired=1, lib=ref)
    xs = [rng.standard_normal(512), np.zeros(512), np.full(512, -2.5), rng.integers(-4, 5, 512) * 0.5]
    xs[0][3], xs[0][300] = -7.0, 7.0
    for i, x in enumerate(xs):
        x = x.astype(np.float32)
        q, d, b32, b16 = O.ref_quantize_row(x, ref)
        out[f"q8K_{i}_x"], out[f"q8K_{i}_q"], out[f"q8K_{i}_d"] = x, q, d
        out[f"q8K_{i}_b32"], out[f"q8K_{i}_b16"] = b32, b16
    return out


def fa_fixtures(ref):
    out = {}
    rng = np.random.default_rng(77)
    H, Hkv, N, D, L = 6, 2, 5, 128, 192
    for kvname, kv_type in (("f16", O.F16), ("q8_0", O.Q8_0)):
        q = (rng.standard_normal((H, N, D)) / 16).astype(np.float32)
        kf = rng.standard_normal((Hkv, L, D)).astype(np.float32)
        vf = rng.standard_normal((Hkv, L, D)).astype(np.float32)
        if kv_type == O.F16:
            k = kf.astype(np.float16).view(np.uint8).reshape(Hkv, L, -1)
            v = vf.astype(np.float16).view(np.uint8).reshape(Hkv, L, -1)
        else:
            k = np.stack([O.quantize_row_q8_0(r, O.Q8_0_REF) for r in kf.reshape(-1, D)]).reshape(Hkv, L, -1)
            v = np.stack([O.quantize_row_q8_0(r, O.Q8_0_REF) for r in vf.reshape(-1, D)]).reshape(Hkv, L, -1)
        mask = np.zeros((N, L), np.float16)
        for t in range(N):
            mask[t, L - N + t + 1:] = -np.inf
        mask = mask.view(np.uint16)
        sinks = rng.standard_normal(H).astype(np.float32)
        for var, kw in (("plain", dict()), ("sinks", dict(sinks=sinks)), ("softcap", dict(scale=4.0, softcap=20.0)),
                        ("alibi", dict(max_bias=8.0))):
            key = f"{kvname}_{var}"
            out[key + "_dst"] = O.ref_fa_gqa(q, kv_type, k, v, D, L, Hkv, mask=mask, nth=1, lib=ref, **kw)
        out[kvname + "_q"], out[kvname + "_k"], out[kvname + "_v"] = q, k, v
        out[kvname + "_mask"], out[kvname + "_sinks"] = mask, sinks
        out[kvname + "_meta"] = np.array([kv_type, H, Hkv, N, D, L], np.int64)
    return out


def main():
    ref = O.load_ref("avx2")
    if ref is None:
        raise SystemExit("oracle/_ref is not built: run `make -C oracle` with the reference available")
    np.savez_compressed(os.path.join(HERE, "srv_mul_mat.npz"), **srv_fixtures(ref))
    np.savez_compressed(os.path.join(HERE, "fa_gqa.npz"), **fa_fixtures(ref))
    print("wrote", sorted(f for f in os.listdir(HERE) if f.endswith(".npz")))


if __name__ == "__main__":
    main()
