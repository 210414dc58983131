"""GPU parity of the attention split over the KV range (srhpm_flash_attn_ext_partial + srhpm_flash_attn_merge).

Each rank's range is run on one device, one partial call per range into consecutive record sets, then one merge. This
is what the multi-GPU path computes after its all-gather, without the collective. The result must be within 1e-3
relative L2 of the f64 oracle over the whole range (the attention tolerance) and of srhpm_flash_attn_ext over the
whole range (whose chunks start their running maxima elsewhere, so P meets f16 at other scales). Cases:
- both cache types;
- ranges of one chunk (the kernel writes the record) and of several (the chunk merge writes it);
- empty ranges (more ranks than 128-token tiles);
- a range the mask hides completely;
- sinks, softcap and ALiBi slopes.
The last test runs the same split over 2 GPUs with NCCL when the box has them."""
import numpy as np
import pytest
import torch

import oracle as O
import srhpm_b200 as S
from srhpm_b200 import _lib as L
from srhpm_b200 import shard

pytestmark = pytest.mark.gpu

TOL = 1e-3
D = 256


def rel_l2(a, b):
    a = np.asarray(a, np.float64)
    b = np.asarray(b, np.float64)
    return float(np.linalg.norm(a - b) / max(np.linalg.norm(b), 1e-30))


def make(rng, kv_type, H, Hkv, N, L):
    q = (rng.standard_normal((H, N, D)) / 16).astype(np.float32)
    k = O.cache_rows(kv_type, rng.standard_normal((Hkv, L, D)).astype(np.float32))
    v = O.cache_rows(kv_type, rng.standard_normal((Hkv, L, D)).astype(np.float32))
    mask = np.zeros((N, L), np.float16)
    for t in range(N):
        mask[t, L - N + t + 1:] = -np.inf
    return q, k, v, mask


def split_run(ctx, q, k, v, kv_type, mask, world, sinks=None, **kw):
    """Partial record sets of the world ranges on this device, merged: f32 [N, H, 256]."""
    t = lambda a: torch.from_numpy(np.ascontiguousarray(a)).cuda()
    H, N, _ = q.shape
    L_ = k.shape[1]
    qd, kd, vd, md = t(q), t(k), t(v), t(mask) if mask is not None else None
    pb = ctx.flash_attn_part_size(H, N)
    parts = torch.empty(world * pb, dtype=torch.uint8, device="cuda")
    for r in range(world):
        t0, t1 = shard.kv_range(L_, world, r)
        ctx.flash_attn_ext_partial(qd, kd[:, t0:t1], vd[:, t0:t1], kv_type,
                                   mask=md[:, t0:t1] if md is not None else None,
                                   out=parts[r * pb:(r + 1) * pb], **kw)
    out = ctx.flash_attn_merge(parts, world, H, N, sinks=t(sinks) if sinks is not None else None)
    whole = ctx.flash_attn_ext(qd, kd, vd, kv_type, mask=md, sinks=t(sinks) if sinks is not None else None, **kw)
    torch.cuda.synchronize()
    ctx.check()
    return out.cpu().numpy(), whole.cpu().numpy()


def oracle(q, k, v, kv_type, mask, sinks=None, **kw):
    Hkv, L_ = k.shape[0], k.shape[1]
    return O.attention(q, kv_type, k, v, D, L_, Hkv, mask=mask.view(np.uint16) if mask is not None else None,
                       sinks=sinks, **kw)


@pytest.mark.parametrize("kv_type", [L.Q8_0, L.F16])
@pytest.mark.parametrize("H,Hkv,N,L_,world", [(8, 2, 4, 1000, 2), (8, 2, 8, 4096, 2), (6, 1, 3, 2100, 3),
                                              (24, 4, 8, 8192, 8), (4, 2, 5, 300, 8), (3, 1, 3, 640, 2)])
def test_split_matches_whole_range(ctx, kv_type, H, Hkv, N, L_, world):
    rng = np.random.default_rng(H * 7 + L_ + world)
    q, k, v, mask = make(rng, kv_type, H, Hkv, N, L_)
    got, whole = split_run(ctx, q, k, v, kv_type, mask, world, scale=1 / 16)
    exp = oracle(q, k, v, kv_type, mask, scale=1 / 16)
    assert rel_l2(got, exp) < TOL, rel_l2(got, exp)
    assert rel_l2(got, whole) < TOL, rel_l2(got, whole)


@pytest.mark.parametrize("kv_type", [L.Q8_0, L.F16])
def test_split_sinks_softcap_alibi_and_hidden_range(ctx, kv_type):
    """Sinks are added once, by the merge; the middle range is hidden from every row by the mask (its records have
    sum 0 and are skipped); ALiBi slopes from max_bias scale the mask per head."""
    rng = np.random.default_rng(5)
    H, Hkv, N, L_, world = 8, 2, 4, 1536, 3
    q, k, v, mask = make(rng, kv_type, H, Hkv, N, L_)
    t0, t1 = shard.kv_range(L_, world, 1)
    mask[:, t0:t1] = -np.inf
    mask[:, :t0] += rng.uniform(-1, 0, (N, t0)).astype(np.float16)
    sinks = rng.standard_normal(H).astype(np.float32)
    kw = dict(scale=1 / 8, softcap=30.0, max_bias=8.0)
    got, whole = split_run(ctx, q, k, v, kv_type, mask, world, sinks=sinks, **kw)
    exp = oracle(q, k, v, kv_type, mask, sinks=sinks, **kw)
    assert rel_l2(got, exp) < TOL, rel_l2(got, exp)
    assert rel_l2(got, whole) < TOL, rel_l2(got, whole)


def test_split_all_ranges_empty_or_hidden(ctx):
    """Every score masked: the merge finds no record with a positive sum; the output is 0 (as the whole-range call
    writes), or sink-only (zeros as well, the sink has no value row)."""
    rng = np.random.default_rng(9)
    H, Hkv, N, L_ = 4, 2, 2, 256
    q, k, v, mask = make(rng, L.Q8_0, H, Hkv, N, L_)
    mask[:] = -np.inf
    sinks = rng.standard_normal(H).astype(np.float32)
    got, whole = split_run(ctx, q, k, v, L.Q8_0, mask, 4, sinks=sinks)
    assert np.all(got == 0.0)
    assert np.all(whole == 0.0)


def test_split_part_size_and_errors(ctx):
    assert ctx.flash_attn_part_size(24, 8) == 24 * 8 * (8 + 1024)
    assert ctx.flash_attn_part_size(3, 3) == 80 + 9 * 1024  # {max, sum} pairs padded to 16 bytes
    lib = L.load()
    assert lib.srhpm_flash_attn_part_size(0, 8) == 0
    parts = torch.zeros(ctx.flash_attn_part_size(4, 2) * 257, dtype=torch.uint8, device="cuda")
    with pytest.raises(RuntimeError):
        ctx.flash_attn_merge(parts, 0, 4, 2)
    with pytest.raises(RuntimeError):
        ctx.flash_attn_merge(parts, 257, 4, 2)
    # an empty range writes an empty set: merged alone it gives zeros
    q = torch.zeros((4, 2, D), device="cuda")
    kv = torch.zeros((2, 0, 272), dtype=torch.uint8, device="cuda")
    ctx.flash_attn_ext_partial(q, kv, kv, L.Q8_0, out=parts[:ctx.flash_attn_part_size(4, 2)])
    out = ctx.flash_attn_merge(parts, 1, 4, 2)
    torch.cuda.synchronize()
    ctx.check()
    assert torch.all(out == 0)


def _nccl_worker(rank, world, port, q, k, v, mask, sinks, outdir, resq):
    import os
    import torch.distributed as dist
    from srhpm_b200.split_attn import SplitKAttention
    try:
        torch.cuda.set_device(rank)
        os.environ.update(MASTER_ADDR="127.0.0.1", MASTER_PORT=str(port))
        dist.init_process_group("nccl", rank=rank, world_size=world, device_id=torch.device("cuda", rank))
        ctx = S.Context(rank)
        H, N, _ = q.shape
        dev = lambda a: torch.from_numpy(np.ascontiguousarray(a)).cuda()
        for exchange in ("nccl", "peers"):
            att = SplitKAttention(ctx, rank, world, H, N, torch.device("cuda", rank), exchange=exchange)
            t0, t1 = att.range(k.shape[1])
            for _ in range(3):  # repeated calls reuse the buffers (the epochs count the calls, the slots alternate)
                out = att(dev(q), dev(k[:, t0:t1]), dev(v[:, t0:t1]), L.Q8_0, mask=dev(mask[:, t0:t1]),
                          sinks=dev(sinks), scale=1 / 16)
            torch.cuda.synchronize()
            ctx.check()
            # the output goes through a file: a queue message larger than the pipe's buffer would block until the
            # parent reads it, and the parent reads after joining
            np.save(os.path.join(outdir, f"rank{rank}_{exchange}.npy"), out.cpu().numpy())
        resq.put(("ok", rank, None))
        dist.barrier()
        dist.destroy_process_group()
    except BaseException as e:  # report instead of hanging the parent
        resq.put(("err", rank, f"{type(e).__name__}: {e}"[:2000]))
        raise


@pytest.mark.skipif(torch.cuda.device_count() < 2, reason="needs 2 GPUs")
def test_split_over_two_gpus_nccl(ctx, tmp_path):
    """SplitKAttention over 2 GPUs: each rank holds half the cache's tokens; the record sets are all-gathered with
    NCCL, or exchanged through the ranks' symmetric-memory buffers as (value, epoch) words, and merged on both ranks. Both ranks
    and both exchanges must agree bit for bit and match the oracle over the whole range."""
    import socket
    import torch.multiprocessing as mp
    rng = np.random.default_rng(11)
    H, Hkv, N, L_ = 24, 4, 8, 4096
    q, k, v, mask = make(rng, L.Q8_0, H, Hkv, N, L_)
    sinks = rng.standard_normal(H).astype(np.float32)
    exp = oracle(q, k, v, L.Q8_0, mask, sinks=sinks, scale=1 / 16)
    s = socket.socket()
    s.bind(("127.0.0.1", 0))
    port = s.getsockname()[1]
    s.close()
    mpc = mp.get_context("spawn")
    resq = mpc.SimpleQueue()
    procs = [mpc.Process(target=_nccl_worker, args=(r, 2, port, q, k, v, mask, sinks, str(tmp_path), resq))
             for r in range(2)]
    for p in procs:
        p.start()
    for p in procs:
        p.join(timeout=300)
    alive = [p for p in procs if p.is_alive()]
    for p in alive:
        p.kill()
    res = []
    while not resq.empty():
        res.append(resq.get())
    assert not alive, "a rank did not finish"
    errs = [r[2] for r in res if r[0] == "err"]
    assert not errs, errs
    assert sorted(r[1] for r in res if r[0] == "ok") == [0, 1]
    outs = {(r, x): np.load(tmp_path / f"rank{r}_{x}.npy") for r in (0, 1) for x in ("nccl", "peers")}
    base = outs[(0, "nccl")]
    for key, o in outs.items():
        assert np.array_equal(o, base), key
    assert rel_l2(base, exp) < TOL, rel_l2(base, exp)


def test_merge_peers_single_rank_equals_merge(ctx):
    """srhpm_flash_attn_merge_peers with one rank (its own buffer as the only peer) equals srhpm_flash_attn_merge of
    that record set bit for bit, over repeated calls (the epochs advance each call and the receive slots alternate)."""
    rng = np.random.default_rng(13)
    H, Hkv, N, L_ = 6, 2, 3, 640
    q, k, v, mask = make(rng, L.Q8_0, H, Hkv, N, L_)
    sinks = torch.from_numpy(rng.standard_normal(H).astype(np.float32)).cuda()
    dev = lambda a: torch.from_numpy(np.ascontiguousarray(a)).cuda()
    buf = torch.zeros(ctx.flash_attn_peer_buffer_size(H, N), dtype=torch.uint8, device="cuda")
    peers = torch.tensor([buf.data_ptr()], dtype=torch.int64, device="cuda")
    epochs = torch.zeros(H * N, dtype=torch.int32, device="cuda")
    part = buf[:ctx.flash_attn_part_size(H, N)]
    for _ in range(3):
        ctx.flash_attn_ext_partial(dev(q), dev(k), dev(v), L.Q8_0, mask=dev(mask), scale=1 / 16, out=part)
        got = ctx.flash_attn_merge_peers(peers, 1, 0, epochs, H, N, sinks=sinks).cpu().numpy()
        want = ctx.flash_attn_merge(part.clone(), 1, H, N, sinks=sinks).cpu().numpy()
        ctx.check()
        assert np.array_equal(got, want)
    assert epochs.cpu().tolist() == [3] * (H * N)
    # the record set (16-byte padded), then 2 slots x 8 source ranks x H * N rows x 258 words of 8 bytes
    set16 = (ctx.flash_attn_part_size(H, N) + 15) // 16 * 16
    assert ctx.flash_attn_peer_buffer_size(H, N) == set16 + 2 * 8 * H * N * 258 * 8
