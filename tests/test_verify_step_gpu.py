"""A whole decoder verify step on the GPU (srhpm_b200.verify_step) against the oracle's restatement (decoder_step):
a small model with the 27B-class step's structure (fused QKV, NEOX RoPE, GQA 2:1, head_dim 256, sliding-window and
full attention layers, SwiGLU, Q4_K / Q3_K / Q6_K weights), f16 and q8_0 KV caches, 1 accepted + 4 drafted tokens.

Bars: the element-wise operators against numpy; the step's logits within 2e-2 relative L2 of the oracle; the KV rows
the step writes; the accepted ids identical wherever the oracle's top-1 margin exceeds 1e-2. The logits bar is looser
than the per-operator 1e-3 because every GEMM re-quantizes its input to int8: once an attention output differs by
~1e-4 (f16 P and V), ~2-3 % of the following activation codes land on the other side of a rounding boundary, and
each such +-1 flip moves the GEMM output by ~0.4 % -- five chained GEMMs per layer, three layers (measured: 5.7e-3)."""
import ctypes

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


def _run_step(ctx, cfg, dev_w, kc, vc, ids, draft, n_past):
    step = V.VerifyStep(ctx, cfg, dev_w, kc, vc, len(ids), n_past)
    step.set_tokens(ids, draft)
    step.run()
    torch.cuda.synchronize()
    ctx.check()
    return step


def _caches(cfg, cap, n_past, rowb, seed):
    rng = np.random.default_rng(seed)
    kc, vc = [], []
    for _ in range(cfg.n_layer):
        for lst in (kc, vc):
            a = np.zeros((cap, cfg.Hkv, rowb), np.uint8)
            a[:n_past] = O.cache_rows(cfg.kv_type, rng.standard_normal((n_past, cfg.Hkv, cfg.hd)).astype(np.float32))
            lst.append(a)
    return kc, vc


def test_step_from_gguf_file_and_unfused_weights(ctx, tmp_path):
    """The GGUF loader uploads the same bytes: the step's logits are identical to those of the same host weights;
    Q / K / V and gate / up as separate GEMMs (the loader's layout when their types differ) agree to 1e-5."""
    pytest.importorskip("gguf")
    from srhpm_b200 import gguf as G
    from test_gguf_loader import write_decoder_gguf
    cfg = small_cfg(L.F16)
    w = V.host_weights(cfg, seed=11)
    path = tmp_path / "m.gguf"
    write_decoder_gguf(path, cfg, w)
    gf = G.GGUFFile(path)
    cfg_f = G.decoder_config(gf, kv_type=L.F16, window=cfg.window, full_every=cfg.full_every)
    dev_f = G.load_decoder(gf, cfg_f, "cuda")
    cap, n_past, ids, draft = 96, 60, [5, 9, 2, 7], [9, 2, 7]
    kc, vc = _caches(cfg, cap, n_past, 512, 12)
    s_host = _run_step(ctx, cfg, V.DeviceWeights.from_host(cfg, w), [torch.from_numpy(a).cuda() for a in kc],
                       [torch.from_numpy(a).cuda() for a in vc], ids, draft, n_past)
    s_file = _run_step(ctx, cfg_f, dev_f, [torch.from_numpy(a).cuda() for a in kc],
                       [torch.from_numpy(a).cuda() for a in vc], ids, draft, n_past)
    assert torch.equal(s_host.logits, s_file.logits)
    assert s_host.accepted() == s_file.accepted()
    # unfused: split each fused matrix back into its parts
    dev_u = V.DeviceWeights.from_host(cfg, w)
    H, Hkv, hd = cfg.H, cfg.Hkv, cfg.hd
    for lay in dev_u.layers:
        qkv, gu = lay.pop("qkv"), lay.pop("gate_up")
        lay["q"], lay["k"], lay["v"] = (qkv.row_slice(a * hd, b * hd) for a, b in
                                        ((0, H), (H, H + Hkv), (H + Hkv, H + 2 * Hkv)))
        lay["gate"], lay["up"] = gu.row_slice(0, cfg.n_ff), gu.row_slice(cfg.n_ff, 2 * cfg.n_ff)
    s_unf = _run_step(ctx, cfg, dev_u, [torch.from_numpy(a).cuda() for a in kc],
                      [torch.from_numpy(a).cuda() for a in vc], ids, draft, n_past)
    assert rel_l2(s_unf.logits.cpu().numpy(), s_host.logits.cpu().numpy()) < 1e-5
    gf.close()


def _tp_worker(rank, world, port, cfg_kw, seed, cap, n_past, ids, draft, q, fused=True):
    import os
    import torch.distributed as dist
    try:
        torch.cuda.set_device(rank)
        os.environ.update(MASTER_ADDR="127.0.0.1", MASTER_PORT=str(port))
        dist.init_process_group("nccl", rank=rank, world_size=world, device_id=torch.device("cuda", rank))
        cfg = V.DecoderConfig(**cfg_kw)
        w = V.host_weights(cfg, seed=seed)
        kc, vc = _caches(cfg, cap, n_past, 512, seed + 1)
        dev_w = V.DeviceWeights.from_host(cfg, w, f"cuda:{rank}", rank=rank, world=world)
        g0, g1 = dev_w.tp["g0"], dev_w.tp["g1"]
        kcr = [torch.from_numpy(np.ascontiguousarray(a[:, g0:g1])).cuda() for a in kc]
        vcr = [torch.from_numpy(np.ascontiguousarray(a[:, g0:g1])).cuda() for a in vc]
        ctx = S.Context(rank)
        tp = V.TensorParallel(rank, world, fused=fused, fused_quant=True)
        step = V.VerifyStep(ctx, cfg, dev_w, kcr, vcr, len(ids), n_past, tp=tp)
        step.set_tokens(ids, draft)
        step.run()
        torch.cuda.synchronize()
        ctx.check()
        # the same step without the fused prologues (separate all-reduce norm and GEMM quantizer): bit-identical
        plain = V.VerifyStep(ctx, cfg, dev_w, [a.clone() for a in kcr], [a.clone() for a in vcr], len(ids), n_past,
                             tp=tp, fuse_prologue=False)
        plain.set_tokens(ids, draft)
        plain.run()
        torch.cuda.synchronize()
        ctx.check()
        same = bool(torch.equal(plain.logits, step.logits))
        parts = [torch.zeros_like(step.logits) for _ in range(world)]
        dist.all_gather(parts, step.logits.contiguous())
        if rank == 0:
            q.put(("ok", torch.cat(parts, dim=1).cpu().numpy(), step.accepted(), same))
        dist.barrier()
        dist.destroy_process_group()
    except BaseException as e:  # report instead of hanging the parent
        q.put(("err", f"rank {rank}: {type(e).__name__}: {e}", None, None))
        raise


@pytest.mark.skipif(torch.cuda.device_count() < 2, reason="needs 2 GPUs")
@pytest.mark.parametrize("Hkv,fused,cap,n_past", [(2, True, 128, 100), (2, False, 128, 100), (1, True, 128, 100),
                                                  (1, True, 512, 400)])
def test_tensor_parallel_step_matches_one_gpu(ctx, Hkv, fused, cap, n_past):
    """Megatron TP over 2 GPUs (column-parallel QKV / gate|up / head, row-parallel O / down, vocabulary-sharded
    acceptance) against the same step on one GPU. The all-reduces run either inside the next RMSNorm over peer memory
    (fused) or as NCCL calls. Hkv = 1 replicates the KV head on both ranks: on the full-attention layer the two
    replicas split its tokens (each attends to its part for all query heads, the records merge over the pair; with
    105 tokens one replica's part is empty, with 405 each gets two tiles). Logits within 2e-2 (the partial sums
    change f32 rounding, re-quantization flips follow, as in the oracle comparison), accepted ids equal where the
    top-1 margin is clear. On each rank the step with the fused prologues (the all-reduce norm writing the next
    GEMM's activation records) gives the same logits bit for bit as the step without them."""
    import socket
    import torch.multiprocessing as mp
    cfg_kw = dict(n_layer=3, d=512, n_ff=768, H=4, Hkv=Hkv, hd=256, n_vocab=1000, base=1e6, eps=1e-6, window=40,
                  full_every=2, kv_type=L.F16)
    cfg = V.DecoderConfig(**cfg_kw)
    seed, ids = 21, [3, 17, 250, 999, 42]
    w = V.host_weights(cfg, seed=seed)
    kc, vc = _caches(cfg, cap, n_past, 512, seed + 1)
    one = _run_step(ctx, cfg, V.DeviceWeights.from_host(cfg, w), [torch.from_numpy(a).cuda() for a in kc],
                    [torch.from_numpy(a).cuda() for a in vc], ids, ids[1:], n_past)
    logits1 = one.logits.cpu().numpy()
    draft = [int(np.argmax(logits1[i])) for i in range(len(ids) - 1)]
    one.set_tokens(ids, draft)
    one.run()
    torch.cuda.synchronize()
    s = socket.socket()
    s.bind(("127.0.0.1", 0))
    port = s.getsockname()[1]
    s.close()
    mpc = mp.get_context("spawn")
    q = mpc.SimpleQueue()
    procs = [mpc.Process(target=_tp_worker, args=(r, 2, port, cfg_kw, seed, cap, n_past, ids, draft, q, fused))
             for r in range(2)]
    for p in procs:
        p.start()
    for p in procs:
        p.join(timeout=300)
    alive = [p for p in procs if p.is_alive()]
    for p in alive:
        p.kill()
    res = []
    while not q.empty():
        res.append(q.get())
    assert not alive, "a rank did not finish"
    errs = [r[1] for r in res if r[0] == "err"]
    assert not errs, errs
    got = [r for r in res if r[0] == "ok"][0]
    assert got[3], "fused and unfused prologues differ"
    assert rel_l2(got[1], logits1) < 2e-2, rel_l2(got[1], logits1)
    srt = np.sort(logits1, axis=1)
    margin = srt[:, -1] - srt[:, -2]
    exp = one.accepted()
    k = len(ids) if (margin > 1e-2).all() else int(np.argmin(margin > 1e-2))
    assert got[2][:k] == exp[:k]


def test_allreduce_norm_one_rank_equals_add_norm(ctx):
    """The fused all-reduce with one rank: the rank sends its partial row to itself as (value, epoch) words and adds
    them, so x + partial and the norm equal srhpm_add_rms_norm with the partial as delta, bit for bit, over two calls
    per slot (the epochs advance)."""
    lib = L.load()
    d, n = 5120, 9
    nbytes = int(lib.srhpm_allreduce_buffer_size(d))
    mine = torch.zeros(nbytes, dtype=torch.uint8, device="cuda")
    peers = torch.tensor([mine.data_ptr()], dtype=torch.int64, device="cuda")
    epochs = torch.zeros(32, dtype=torch.int32, device="cuda")
    w = 1 + 0.1 * torch.randn(d, device="cuda")
    ptr = lambda t: t.data_ptr()
    part = [mine[k * 16 * d * 4:(k + 1) * 16 * d * 4].view(torch.float32).view(16, d) for k in (0, 1)]
    g = torch.Generator(device="cuda")
    g.manual_seed(5)
    for rep in range(4):
        slot = rep % 2
        part[slot][:n] = torch.randn((n, d), device="cuda", generator=g)
        x = torch.randn((n, d), device="cuda", generator=g)
        x2, y, y2 = x.clone(), torch.empty_like(x), torch.empty_like(x)
        L.check(lib.srhpm_add_rms_norm_allreduce(ctx.handle, ptr(x), ptr(peers), 1, 0, slot, ptr(epochs), ptr(w),
                                                 1e-6, ptr(y), n, d, None), "srhpm_add_rms_norm_allreduce")
        delta = part[slot][:n].clone()
        L.check(lib.srhpm_add_rms_norm(ctx.handle, ptr(x2), ptr(delta), ptr(w), ctypes.c_float(1e-6), ptr(y2), n, d,
                                       None), "srhpm_add_rms_norm")
        torch.cuda.synchronize()
        ctx.check()
        assert torch.equal(x, x2) and torch.equal(y, y2), rep
    assert epochs.view(2, 16)[:, :n].tolist() == [[2] * n, [2] * n]


@pytest.mark.parametrize("d,n,qtype", [(5120, 9, S.Q4_K), (5120, 4, S.Q3_K), (1024, 3, S.Q5_K), (16384, 16, S.IQ4_XS)])
def test_allreduce_norm_quant_one_rank_equals_norm_quant(ctx, d, n, qtype):
    """The fused all-reduce + norm + quantization prologue (a cluster of CTAs per row: each sends and sums a share of
    the row's columns, the sum of squares is reduced in the one-CTA kernel's order) with one rank equals
    srhpm_add_rms_norm_quant with the partial rows as delta, bit for bit: x, y, and the GEMM on the records
    (srhpm_mul_mat_prequantized), over two calls per slot (the epochs advance once per call and row)."""
    lib = L.load()
    rows = 192
    nbytes = int(lib.srhpm_allreduce_buffer_size(d))
    mine = torch.zeros(nbytes, dtype=torch.uint8, device="cuda")
    peers = torch.tensor([mine.data_ptr()], dtype=torch.int64, device="cuda")
    epochs = torch.zeros(32, dtype=torch.int32, device="cuda")
    W = S.QuantTensor.from_blocks(O.random_blocks(qtype, rows * d // 256, np.random.default_rng(d + n)), qtype, rows, d)
    wv = W.view()
    w = 1 + 0.1 * torch.randn(d, device="cuda")
    ptr = lambda t: t.data_ptr()
    part = [mine[k * 16 * d * 4:(k + 1) * 16 * d * 4].view(torch.float32).view(16, d) for k in (0, 1)]
    g = torch.Generator(device="cuda")
    g.manual_seed(d + n)
    for rep in range(4):
        slot = rep % 2
        part[slot][:n] = torch.randn((n, d), device="cuda", generator=g)
        x = torch.randn((n, d), device="cuda", generator=g)
        x2, y, y2 = x.clone(), torch.empty_like(x), torch.empty_like(x)
        st, ws = ctx.mul_mat_work_size(W, x)
        work, work2 = (torch.empty(ws, dtype=torch.uint8, device="cuda") for _ in range(2))
        L.check(lib.srhpm_add_rms_norm_allreduce_quant(ctx.handle, ptr(x), ptr(peers), 1, 0, slot, ptr(epochs),
                                                       ptr(w), ctypes.c_float(1e-6), ptr(y), n, ctypes.byref(wv),
                                                       ptr(work), work.numel(), None),
                "srhpm_add_rms_norm_allreduce_quant")
        delta = part[slot][:n].clone()
        L.check(lib.srhpm_add_rms_norm_quant(ctx.handle, ptr(x2), ptr(delta), ptr(w), ctypes.c_float(1e-6), ptr(y2),
                                             n, ctypes.byref(wv), ptr(work2), work2.numel(), None),
                "srhpm_add_rms_norm_quant")
        Y, Y2 = (torch.empty((n, rows), dtype=torch.float32, device="cuda") for _ in range(2))
        for yy, ww_, buf in ((y, Y, work), (y2, Y2, work2)):
            xv, yv = S.f32_rows_view(yy), S.f32_rows_view(ww_)
            L.check(lib.srhpm_mul_mat_prequantized(ctx.handle, ctypes.byref(wv), ctypes.byref(xv), ctypes.byref(yv),
                                                   ptr(buf), buf.numel(), None), "srhpm_mul_mat_prequantized")
        torch.cuda.synchronize()
        ctx.check()
        assert torch.equal(x, x2) and torch.equal(y, y2), rep
        assert torch.equal(Y, Y2), rep
    assert epochs.view(2, 16)[:, :n].tolist() == [[2] * n, [2] * n]
    assert epochs.view(2, 16)[:, n:].abs().sum().item() == 0


def test_allreduce_norm_peer_wait_times_out(ctx):
    """The fused all-reduce's wait is bounded: a second 'rank' that never sends its values (a plain local buffer
    standing in for the peer) ends the wait after ~2 s with an error status read on the host, and the context stays
    usable. No GPU fault and no hang: the kernel gives up and finishes."""
    import time
    lib = L.load()
    d, n = 512, 2
    nbytes = int(lib.srhpm_allreduce_buffer_size(d))
    mine = torch.zeros(nbytes, dtype=torch.uint8, device="cuda")
    fake = torch.zeros(nbytes, dtype=torch.uint8, device="cuda")
    peers = torch.tensor([mine.data_ptr(), fake.data_ptr()], dtype=torch.int64, device="cuda")
    epochs = torch.zeros(32, dtype=torch.int32, device="cuda")
    x = torch.randn((n, d), device="cuda")
    w = torch.ones(d, device="cuda")
    y = torch.empty_like(x)
    ptr = lambda t: t.data_ptr()
    t0 = time.time()
    L.check(lib.srhpm_add_rms_norm_allreduce(ctx.handle, ptr(x), ptr(peers), 2, 0, 0, ptr(epochs), ptr(w), 1e-6,
                                             ptr(y), n, d, None), "srhpm_add_rms_norm_allreduce")
    torch.cuda.synchronize()
    assert time.time() - t0 > 1.5
    with pytest.raises(L.SrhpmError):
        ctx.check()
    ctx.check()  # cleared: the context keeps working
    # this rank sent its (zero) partial values with epoch 1 into both buffers' receive areas (slot 0, rows 0..n-1,
    # source rank 0): 8-byte words, value bits low, epoch high
    off = 2 * 16 * d * 4
    for buf in (mine, fake):
        words = buf[off:].view(torch.int32).view(2, 16, 8, d, 2)
        assert bool((words[0, :n, 0, :, 1] == 1).all()) and bool((words[0, :n, 0, :, 0] == 0).all())
        assert bool((words[0, :n, 1] == 0).all())  # nothing from the stand-in rank


def test_allreduce_norm_quant_peer_wait_times_out(ctx):
    """The fused all-reduce + norm + quantization prologue has the same bounded wait: against a stand-in peer that
    never sends its values it gives up after ~2 s with an error status, and the context stays usable."""
    import time
    lib = L.load()
    d, n, rows = 512, 2, 64
    nbytes = int(lib.srhpm_allreduce_buffer_size(d))
    mine = torch.zeros(nbytes, dtype=torch.uint8, device="cuda")
    fake = torch.zeros(nbytes, dtype=torch.uint8, device="cuda")
    peers = torch.tensor([mine.data_ptr(), fake.data_ptr()], dtype=torch.int64, device="cuda")
    epochs = torch.zeros(32, dtype=torch.int32, device="cuda")
    x = torch.randn((n, d), device="cuda")
    w = torch.ones(d, device="cuda")
    y = torch.empty_like(x)
    W = S.QuantTensor.from_blocks(O.random_blocks(S.Q4_K, rows * d // 256, np.random.default_rng(3)), S.Q4_K, rows, d)
    wv = W.view()
    st, ws = ctx.mul_mat_work_size(W, x)
    work = torch.empty(ws, dtype=torch.uint8, device="cuda")
    ptr = lambda t: t.data_ptr()
    t0 = time.time()
    L.check(lib.srhpm_add_rms_norm_allreduce_quant(ctx.handle, ptr(x), ptr(peers), 2, 0, 0, ptr(epochs), ptr(w),
                                                   1e-6, ptr(y), n, ctypes.byref(wv), ptr(work), work.numel(), None),
            "srhpm_add_rms_norm_allreduce_quant")
    torch.cuda.synchronize()
    assert time.time() - t0 > 1.5
    with pytest.raises(L.SrhpmError):
        ctx.check()
    ctx.check()


def test_fused_norm_quant_prologue_is_exact(ctx):
    """RMSNorm and SwiGLU fused with the next GEMM's activation quantization write the same records as the GEMM's
    own quantizer: the whole step's logits, caches and accepted ids are identical with and without the fusion."""
    cfg = small_cfg(L.F16)
    w = V.host_weights(cfg, seed=31)
    cap, n_past, ids, draft = 128, 70, [4, 8, 15, 16, 23, 42], [8, 15, 16, 23, 42]
    kc, vc = _caches(cfg, cap, n_past, 512, 32)
    dev_w = V.DeviceWeights.from_host(cfg, w)
    outs = []
    for fuse, fq_o, sw in ((False, False, False), (True, False, True), (True, True, True), (True, True, False)):
        # fq_o: GEMMs without a fused prologue (here the attention output projection) quantize their activations in
        # their own grid (one launch instead of 2); sw: the down GEMM computes the SwiGLU in its own grid
        kcd = [torch.from_numpy(a).cuda() for a in kc]
        vcd = [torch.from_numpy(a).cuda() for a in vc]
        step = V.VerifyStep(ctx, cfg, dev_w, kcd, vcd, len(ids), n_past, fuse_prologue=fuse, gemm_fused_quant=fq_o,
                            swiglu_in_gemm=sw)
        step.set_tokens(ids, draft)
        ctx.launch_count(reset=True)
        step.run()
        torch.cuda.synchronize()
        launches = ctx.launch_count(reset=True)
        ctx.check()
        outs.append((step.logits.clone(), [a.clone() for a in kcd], step.accepted(), launches))
    for o in outs[1:]:
        assert torch.equal(outs[0][0], o[0])
        assert all(torch.equal(a, b) for a, b in zip(outs[0][1], o[1]))
        assert outs[0][2] == o[2]
    # kernel launches: the quantizers of the QKV, gate|up, down and head GEMMs are gone (3 per layer + 1), and the
    # SwiGLU kernel too where the down GEMM's grid is large enough to compute it in its prologue (1 more per layer);
    # with the fused output projection the O GEMM's quantizer (1 per layer) when its grid is large enough
    assert outs[0][3] - outs[1][3] in (3 * cfg.n_layer + 1, 4 * cfg.n_layer + 1)
    assert outs[1][3] - outs[2][3] in (0, cfg.n_layer)
    assert outs[3][3] - outs[2][3] == outs[0][3] - outs[1][3] - 3 * cfg.n_layer - 1


@pytest.mark.parametrize("qtype", [S.Q4_K, S.Q5_K, S.Q6_K, S.Q3_K, S.IQ4_XS])
def test_fused_prologues_match_the_gemm_quantizer_every_type(ctx, qtype):
    """srhpm_add_rms_norm_quant and srhpm_swiglu_quant write the activation records in each weight type's byte order
    (natural, Q3_K's and IQ4_XS's permutations): the prequantized GEMM equals srhpm_mul_mat on the same rows bit for
    bit."""
    lib = L.load()
    rng = np.random.default_rng(50 + qtype)
    n, d, rows = 5, 1024, 192
    W = S.QuantTensor.from_blocks(O.random_blocks(qtype, rows * d // 256, rng).reshape(rows, -1), qtype, rows, d)
    wv = W.view()
    x = torch.from_numpy(rng.standard_normal((n, d)).astype(np.float32)).cuda()
    nw = torch.from_numpy((1 + 0.1 * rng.standard_normal(d)).astype(np.float32)).cuda()
    y = torch.empty_like(x)
    st, ws = ctx.mul_mat_work_size(W, x)
    work = torch.empty(ws, dtype=torch.uint8, device="cuda")
    ptr = lambda t: ctypes.c_void_p(t.data_ptr())
    yq = torch.empty((n, rows), device="cuda")
    xv, yqv = S.f32_rows_view(y), S.f32_rows_view(yq)
    xc = x.clone()
    L.check(lib.srhpm_add_rms_norm_quant(ctx.handle, ptr(xc), None, ptr(nw), ctypes.c_float(1e-6), ptr(y), n,
                                         ctypes.byref(wv), ptr(work), work.numel(), None), "srhpm_add_rms_norm_quant")
    L.check(lib.srhpm_mul_mat_prequantized(ctx.handle, ctypes.byref(wv), ctypes.byref(xv), ctypes.byref(yqv),
                                           ptr(work), work.numel(), None), "srhpm_mul_mat_prequantized")
    want = ctx.mul_mat(W, y)
    torch.cuda.synchronize()
    ctx.check()
    assert torch.equal(yq, want)
    # SwiGLU prologue: gate | up halves of one row block
    gu = torch.from_numpy(rng.standard_normal((n, 2 * d)).astype(np.float32)).cuda()
    h = torch.empty((n, d), device="cuda")
    L.check(lib.srhpm_swiglu_quant(ctx.handle, ptr(gu), ctypes.c_void_p(gu.data_ptr() + 4 * d), gu.stride(0), ptr(h),
                                   h.stride(0), n, ctypes.byref(wv), ptr(work), work.numel(), None),
            "srhpm_swiglu_quant")
    hv = S.f32_rows_view(h)
    L.check(lib.srhpm_mul_mat_prequantized(ctx.handle, ctypes.byref(wv), ctypes.byref(hv), ctypes.byref(yqv),
                                           ptr(work), work.numel(), None), "srhpm_mul_mat_prequantized")
    want = ctx.mul_mat(W, h)
    torch.cuda.synchronize()
    ctx.check()
    assert torch.equal(yq, want)


def test_fused_entry_points_status_codes(ctx):
    """The fused prologue / all-reduce entry points return status codes instead of failing: Q8_0 weights have no
    fused prologue (UNSUPPORTED, srhpm_mul_mat quantizes itself), a short workspace, misaligned rows, bad ranks."""
    lib = L.load()
    ptr = lambda t: t.data_ptr()
    d, n = 512, 3
    x = torch.randn((n, d), device="cuda")
    w = torch.ones(d, device="cuda")
    y = torch.empty_like(x)
    Wq8 = S.QuantTensor.quantize(np.random.default_rng(0).standard_normal((64, d)).astype(np.float32) * 0.02, S.Q8_0)
    W4 = S.QuantTensor.quantize(np.random.default_rng(1).standard_normal((64, d)).astype(np.float32) * 0.02, S.Q4_K)
    work = torch.zeros(1 << 20, dtype=torch.uint8, device="cuda")
    v8, v4 = Wq8.view(), W4.view()
    st = lib.srhpm_add_rms_norm_quant(ctx.handle, ptr(x), None, ptr(w), 1e-6, ptr(y), n, ctypes.byref(v8), ptr(work),
                                      work.numel(), None)
    assert st == L.UNSUPPORTED
    st = lib.srhpm_add_rms_norm_quant(ctx.handle, ptr(x), None, ptr(w), 1e-6, ptr(y), n, ctypes.byref(v4), ptr(work),
                                      16, None)
    assert st == L.ERR_WORKSPACE
    st = lib.srhpm_add_rms_norm_quant(ctx.handle, ptr(x) + 4, None, ptr(w), 1e-6, ptr(y), n, ctypes.byref(v4),
                                      ptr(work), work.numel(), None)
    assert st == L.ERR_ALIGN
    st = lib.srhpm_swiglu_quant(ctx.handle, ptr(x), ptr(x), d, ptr(y), d, n, ctypes.byref(v8), ptr(work),
                                work.numel(), None)
    assert st == L.UNSUPPORTED
    peers = torch.zeros(2, dtype=torch.int64, device="cuda")
    epochs = torch.zeros(32, dtype=torch.int32, device="cuda")
    for world, rank, slot in ((9, 0, 0), (2, 2, 0), (2, 0, 2), (0, 0, 0)):
        st = lib.srhpm_add_rms_norm_allreduce(ctx.handle, ptr(x), ptr(peers), world, rank, slot, ptr(epochs),
                                              ptr(w), 1e-6, ptr(y), n, d, None)
        assert st == L.ERR_INVALID, (world, rank, slot)
    torch.cuda.synchronize()
    ctx.check()


def test_verify_step_single_token(ctx):
    """k = 0 (N = 1: only the accepted token, nothing drafted) through the fused prologues: matches the oracle and
    emits exactly the greedy token."""
    cfg = small_cfg(L.F16)
    w = V.host_weights(cfg, seed=41)
    cap, n_past, ids = 64, 30, [123]
    kc, vc = _caches(cfg, cap, n_past, 512, 42)
    okc, ovc = [a.copy() for a in kc], [a.copy() for a in vc]
    logits_o, acc_o = O.decoder_step(cfg.as_dict(), w, okc, ovc, ids, n_past, [])
    step = _run_step(ctx, cfg, V.DeviceWeights.from_host(cfg, w), [torch.from_numpy(a).cuda() for a in kc],
                     [torch.from_numpy(a).cuda() for a in vc], ids, [], n_past)
    assert rel_l2(step.logits.cpu().numpy(), logits_o) < 2e-2
    srt = np.sort(logits_o[0])
    if srt[-1] - srt[-2] > 1e-2:
        assert step.accepted() == acc_o


@pytest.mark.parametrize("kv_type", [L.F16, L.Q8_0])
def test_verify_step_advance_matches_a_step_built_there(ctx, kv_type):
    """Decode-loop bookkeeping: after a step, advance(len(accepted())) moves it to the next cache position (the rows
    written for rejected drafted tokens are hidden, then overwritten: the reference server's truncate-on-rollback).
    The moved step computes exactly what a step built at that position computes on the same cache contents: the same
    logits, accepted ids and cache rows, bit for bit (the same kernels and plans on the same inputs). The sliding
    window's first visible position moves with it (window 40 at position ~100)."""
    cfg = small_cfg(kv_type)
    w = V.host_weights(cfg, seed=51)
    rowb = 272 if kv_type == L.Q8_0 else 512
    cap, n_past, n = 160, 100, 5
    kc, vc = _caches(cfg, cap, n_past, rowb, 52)
    dev_w = V.DeviceWeights.from_host(cfg, w)
    dkc = [torch.from_numpy(a).cuda() for a in kc]
    dvc = [torch.from_numpy(a).cuda() for a in vc]
    rng = np.random.default_rng(53)
    ids = [int(i) for i in rng.integers(0, cfg.n_vocab, n)]
    step = _run_step(ctx, cfg, dev_w, dkc, dvc, ids, ids[1:], n_past)
    emitted = step.accepted()
    kc2, vc2 = [a.clone() for a in dkc], [a.clone() for a in dvc]
    step.advance(len(emitted))
    assert step.n_past == n_past + len(emitted)
    ids2 = [emitted[-1]] + [int(i) for i in rng.integers(0, cfg.n_vocab, n - 1)]
    step.set_tokens(ids2, ids2[1:])
    step.run()
    torch.cuda.synchronize()
    ctx.check()
    fresh = _run_step(ctx, cfg, dev_w, kc2, vc2, ids2, ids2[1:], n_past + len(emitted))
    assert torch.equal(step.logits, fresh.logits)
    assert step.accepted() == fresh.accepted()
    assert all(torch.equal(a, b) for a, b in zip(dkc + dvc, kc2 + vc2))
    with pytest.raises(ValueError):
        step.set_past(cap - n + 1)  # past the end of the cache
    with pytest.raises(ValueError):
        step.advance(0)  # a step emits at least one id
