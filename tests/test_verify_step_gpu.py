"""A whole decoder verify step on the GPU (srhpm_b200.verify_step) against the oracle's restatement (decoder_step):
a small model with the 27B-class step's structure (fused QKV, NEOX RoPE, GQA 2:1, head_dim 256, sliding-window and
full attention layers, SwiGLU, Q4_K / Q3_K / Q6_K weights), f16 and q8_0 KV caches, 1 accepted + 4 drafted tokens.

Bars: the element-wise operators against numpy; the step's logits within 2e-2 relative L2 of the oracle; the KV rows
the step writes; the accepted ids identical wherever the oracle's top-1 margin exceeds 1e-2. The logits bar is looser
than the per-operator 1e-3 because every GEMM re-quantizes its input to int8: once an attention output differs by
~1e-4 (f16 P and V), ~2-3 % of the following activation codes land on the other side of a rounding boundary, and
each such +-1 flip moves the GEMM output by ~0.4 % -- five chained GEMMs per layer, three layers (measured: 5.7e-3)."""
import numpy as np
import pytest
import torch

import oracle as O
import srhpm_b200 as S
from srhpm_b200 import _lib as L
from srhpm_b200 import verify_step as V

pytestmark = pytest.mark.gpu


def rel_l2(a, b):
    a = np.asarray(a, np.float64)
    b = np.asarray(b, np.float64)
    return float(np.linalg.norm(a - b) / max(np.linalg.norm(b), 1e-30))


def test_add_rms_norm_and_swiglu(ctx):
    rng = np.random.default_rng(1)
    x = rng.standard_normal((9, 5120)).astype(np.float32)
    dl = rng.standard_normal((9, 5120)).astype(np.float32)
    w = (1 + 0.1 * rng.standard_normal(5120)).astype(np.float32)
    tx, td, tw = (torch.from_numpy(a).cuda() for a in (x, dl, w))
    ty = torch.empty_like(tx)
    lib = L.load()
    ptr = lambda t: t.data_ptr()
    L.check(lib.srhpm_add_rms_norm(ctx.handle, ptr(tx), ptr(td), ptr(tw), 1e-6, ptr(ty), 9, 5120, None), "norm")
    torch.cuda.synchronize()
    assert np.array_equal(tx.cpu().numpy(), x + dl)
    assert rel_l2(ty.cpu().numpy(), O.rms_norm(x + dl, w, 1e-6)) < 1e-6
    gu = rng.standard_normal((9, 2 * 17408)).astype(np.float32)  # a fused gate | up output
    tgu = torch.from_numpy(gu).cuda()
    to = torch.empty((9, 17408), dtype=torch.float32, device="cuda")
    L.check(lib.srhpm_swiglu(ctx.handle, ptr(tgu), ptr(tgu) + 4 * 17408, 2 * 17408, ptr(to), 17408, 9, 17408, None),
            "swiglu")
    torch.cuda.synchronize()
    assert rel_l2(to.cpu().numpy(), O.swiglu(gu[:, :17408], gu[:, 17408:])) < 1e-6


def small_cfg(kv_type):
    return V.DecoderConfig(n_layer=3, d=512, n_ff=768, H=4, Hkv=2, hd=256, n_vocab=1000, base=1e6, eps=1e-6,
                           window=40, full_every=2, kv_type=kv_type)


@pytest.mark.parametrize("kv_type", [L.F16, L.Q8_0])
def test_verify_step_matches_oracle(ctx, kv_type):
    cfg = small_cfg(kv_type)
    w = V.host_weights(cfg, seed=3)
    rng = np.random.default_rng(4)
    cap, n_past, n = 128, 100, 5
    rowb = 272 if kv_type == L.Q8_0 else 512
    kc = [np.zeros((cap, cfg.Hkv, rowb), np.uint8) for _ in range(cfg.n_layer)]
    vc = [np.zeros((cap, cfg.Hkv, rowb), np.uint8) for _ in range(cfg.n_layer)]
    for l in range(cfg.n_layer):
        kc[l][:n_past] = O.cache_rows(kv_type, rng.standard_normal((n_past, cfg.Hkv, cfg.hd)).astype(np.float32))
        vc[l][:n_past] = O.cache_rows(kv_type, rng.standard_normal((n_past, cfg.Hkv, cfg.hd)).astype(np.float32))
    ids = rng.integers(0, cfg.n_vocab, n)
    dev_w = V.DeviceWeights.from_host(cfg, w)
    dkc = [torch.from_numpy(a).cuda() for a in kc]
    dvc = [torch.from_numpy(a).cuda() for a in vc]
    okc, ovc = [a.copy() for a in kc], [a.copy() for a in vc]
    logits_o, _ = O.decoder_step(cfg.as_dict(), w, okc, ovc, ids, n_past, ids[1:])
    draft = [int(np.argmax(logits_o[i])) for i in range(n - 1)]  # the oracle's own greedy choices: all accepted
    step = V.VerifyStep(ctx, cfg, dev_w, dkc, dvc, n, n_past)
    step.set_tokens(ids, draft)
    step.run()
    torch.cuda.synchronize()
    ctx.check()
    got = step.logits.cpu().numpy()
    assert rel_l2(got, logits_o) < 2e-2, rel_l2(got, logits_o)
    # the KV rows of the new tokens (f16: the same rounding; q8_0: the same quantizer)
    for l in range(cfg.n_layer):
        gk = dkc[l].cpu().numpy()[n_past:n_past + n]
        ok = okc[l][n_past:n_past + n]
        if kv_type == L.F16:
            a, b = gk.view(np.float16).astype(np.float32), ok.view(np.float16).astype(np.float32)
        else:
            a = np.stack([O.dequantize(O.Q8_0, r, cfg.hd) for r in gk.reshape(-1, rowb)])
            b = np.stack([O.dequantize(O.Q8_0, r, cfg.hd) for r in ok.reshape(-1, rowb)])
        assert rel_l2(a, b) < 1e-2, l
    # acceptance: identical where the oracle's top-1 margin is clear
    srt = np.sort(logits_o, axis=1)
    margin = srt[:, -1] - srt[:, -2]
    acc = step.accepted()
    exp = O.accept(logits_o, draft)
    if (margin > 1e-2).all():
        assert acc == exp
    else:
        k = int(np.argmin(margin > 1e-2))
        assert acc[:k] == exp[:k]


def test_verify_step_graph_replay(ctx):
    cfg = small_cfg(L.F16)
    w = V.host_weights(cfg, seed=5)
    cap, n_past, n = 64, 50, 3
    kc = [torch.zeros((cap, cfg.Hkv, 512), dtype=torch.uint8, device="cuda") for _ in range(cfg.n_layer)]
    vc = [torch.zeros((cap, cfg.Hkv, 512), dtype=torch.uint8, device="cuda") for _ in range(cfg.n_layer)]
    step = V.VerifyStep(ctx, cfg, V.DeviceWeights.from_host(cfg, w), kc, vc, n, n_past)
    step.set_tokens([1, 2, 3], [2, 3])
    step.run()
    torch.cuda.synchronize()
    eager = step.logits.clone()
    s = torch.cuda.Stream()
    s.wait_stream(torch.cuda.current_stream())
    g = torch.cuda.CUDAGraph()
    with torch.cuda.stream(s):
        with torch.cuda.graph(g, stream=s):
            step.run(s)
    g.replay()
    g.replay()
    torch.cuda.synchronize()
    ctx.check()
    assert torch.equal(eager, step.logits)
