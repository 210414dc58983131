"""Attention split over the KV range across CPU ranks over gloo, with the oracle as every rank's compute.

Each rank takes its tokens from shard.kv_range, the same cut the GPU path uses. It computes the (max, sum, acc) records
of its range (oracle.attention_partial). The ranks all-gather them in rank order, and every rank merges them
(oracle.attention_merge: the reference's record merge, patch/srhpm.patch:789-823). The result must equal the
single-pass oracle over the whole range to f64 rounding. World sizes 2-4, with ranks left without tokens when the
cache has fewer 128-token tiles than ranks.

The last test runs srhpm_b200.split_attn.SplitKAttention itself over gloo. A stand-in context computes each range's
record set with the oracle in the C ABI's byte layout, so the class's buffer slicing, in-place all-gather and merge
call are checked on the CPU."""
import os
import socket

import numpy as np
import pytest
import torch
import torch.distributed as dist
import torch.multiprocessing as mp

import oracle as O
from srhpm_b200 import shard

D = 64


def free_port():
    s = socket.socket()
    s.bind(("127.0.0.1", 0))
    p = s.getsockname()[1]
    s.close()
    return p


def inputs(kv_type, H, Hkv, N, L, seed=1):
    rng = np.random.default_rng(seed)
    q = (rng.standard_normal((H, N, D)) / 4).astype(np.float32)
    k = O.cache_rows(kv_type, rng.standard_normal((Hkv, L, D)).astype(np.float32))
    v = O.cache_rows(kv_type, rng.standard_normal((Hkv, L, D)).astype(np.float32))
    mask = np.zeros((N, L), np.float16)
    for t in range(N):
        mask[t, L - N + t + 1:] = -np.inf
    sinks = rng.standard_normal(H).astype(np.float32)
    return q, k, v, mask.view(np.uint16), sinks


def _worker(rank, world, port, kv_type, H, Hkv, N, L, errq):
    try:
        os.environ.update(MASTER_ADDR="127.0.0.1", MASTER_PORT=str(port))
        dist.init_process_group("gloo", rank=rank, world_size=world)
        q, k, v, mask, sinks = inputs(kv_type, H, Hkv, N, L)
        t0, t1 = shard.kv_range(L, world, rank)
        m, s, acc = O.attention_partial(q, kv_type, k, v, D, L, Hkv, t0, t1, mask=mask, scale=0.125, softcap=20.0)
        got = []
        for a in (m, s, acc):
            mine = torch.from_numpy(np.ascontiguousarray(a))
            parts = [torch.empty_like(mine) for _ in range(world)]
            dist.all_gather(parts, mine)
            got.append(torch.stack(parts).numpy())
        out = O.attention_merge(*got, sinks=sinks)
        exp = O.attention(q, kv_type, k, v, D, L, Hkv, mask=mask, sinks=sinks, scale=0.125, softcap=20.0)
        rel = np.linalg.norm(out - exp) / np.linalg.norm(exp)
        assert rel < 1e-12, rel
        dist.barrier()
        dist.destroy_process_group()
    except BaseException as e:  # report to the parent instead of hanging the others
        errq.put(f"rank {rank}: {type(e).__name__}: {e}")
        raise


@pytest.mark.parametrize("world,kv_type,L", [(2, O.F16, 700), (3, O.Q8_0, 1000), (4, O.Q8_0, 300)])
def test_split_k_attention_equals_whole_range(world, kv_type, L):
    ctx = mp.get_context("spawn")
    errq = ctx.SimpleQueue()
    port = free_port()
    procs = [ctx.Process(target=_worker, args=(r, world, port, kv_type, 6, 2, 4, L, errq)) for r in range(world)]
    for p in procs:
        p.start()
    for p in procs:
        p.join(timeout=300)
    alive = [p for p in procs if p.is_alive()]
    for p in alive:
        p.kill()
    errors = []
    while not errq.empty():
        errors.append(errq.get())
    assert not alive, "a rank did not finish"
    assert not errors, errors
    assert all(p.exitcode == 0 for p in procs)


@pytest.mark.parametrize("L,world", [(8192, 8), (131072, 8), (300, 8), (100, 4), (1000, 3)])
def test_kv_range_tiles_the_cache(L, world):
    rs = [shard.kv_range(L, world, r) for r in range(world)]
    assert rs[0][0] == 0 and rs[-1][1] == L
    assert all(rs[i][1] == rs[i + 1][0] for i in range(world - 1))
    assert all(t0 % shard.KV_TILE == 0 for t0, _ in rs)
    tiles = [-(-(t1 - t0) // shard.KV_TILE) for t0, t1 in rs]
    assert max(tiles) - min(tiles) <= 1


class OracleCtx:
    """Stand-in for srhpm_b200.Context on CPU tensors: the record set of a KV range in the C ABI's byte layout
    ({max, sum} f32 pairs [H * N] padded to 16 bytes, then f32 acc [H * N][D]) computed by the oracle, and the
    merge of such sets. The device kernels behind the same calls are tested on the GPU."""

    def __init__(self, D):
        self.D = D

    def flash_attn_part_size(self, H, N):
        return (H * N * 8 + 15) // 16 * 16 + H * N * self.D * 4

    def _split(self, buf, H, N):
        ms_bytes = (H * N * 8 + 15) // 16 * 16
        ms = buf[:H * N * 8].view(torch.float32).reshape(H, N, 2)
        acc = buf[ms_bytes:ms_bytes + H * N * self.D * 4].view(torch.float32).reshape(H, N, self.D)
        return ms, acc

    def flash_attn_ext_partial(self, q, k, v, kv_type, mask=None, scale=1.0, max_bias=0.0, softcap=0.0, out=None,
                               work=None):
        H, N, D = q.shape
        out.zero_()
        Hkv, Lr = k.shape[0], k.shape[1]
        if Lr > 0:
            m16 = np.ascontiguousarray(mask.numpy()).view(np.uint16) if mask is not None else None
            m, s, acc = O.attention_partial(q.numpy(), kv_type, np.ascontiguousarray(k.numpy()),
                                            np.ascontiguousarray(v.numpy()), D, Lr, Hkv, 0, Lr, mask=m16,
                                            scale=scale, max_bias=max_bias, softcap=softcap)
            ms, a = self._split(out, H, N)
            ms[..., 0] = torch.from_numpy(m.astype(np.float32))
            ms[..., 1] = torch.from_numpy(s.astype(np.float32))
            a.copy_(torch.from_numpy(acc.astype(np.float32)))
        return out

    def flash_attn_merge(self, parts, n_parts, H, N, sinks=None, out=None):
        size = self.flash_attn_part_size(H, N)
        ms, acc = zip(*(self._split(parts[p * size:(p + 1) * size], H, N) for p in range(n_parts)))
        m = np.stack([x[..., 0].numpy() for x in ms]).astype(np.float64)
        s = np.stack([x[..., 1].numpy() for x in ms]).astype(np.float64)
        a = np.stack([x.numpy() for x in acc]).astype(np.float64)
        res = O.attention_merge(m, s, a, sinks=sinks.numpy() if sinks is not None else None)
        out.copy_(torch.from_numpy(res.astype(np.float32)))
        return out


def _class_worker(rank, world, port, kv_type, H, Hkv, N, L, errq):
    from srhpm_b200.split_attn import SplitKAttention
    try:
        os.environ.update(MASTER_ADDR="127.0.0.1", MASTER_PORT=str(port))
        dist.init_process_group("gloo", rank=rank, world_size=world)
        q, k, v, mask, sinks = inputs(kv_type, H, Hkv, N, L, seed=5)
        # the collective exchange (the peer exchange needs device symmetric memory)
        att = SplitKAttention(OracleCtx(D), rank, world, H, N, torch.device("cpu"), exchange="nccl")
        att.out = torch.zeros((N, H, D), dtype=torch.float32)  # the stand-in's head size
        t0, t1 = att.range(L)
        out = att(torch.from_numpy(q), torch.from_numpy(np.ascontiguousarray(k[:, t0:t1])),
                  torch.from_numpy(np.ascontiguousarray(v[:, t0:t1])), kv_type,
                  mask=torch.from_numpy(np.ascontiguousarray(mask[:, t0:t1]).view(np.float16)),
                  sinks=torch.from_numpy(sinks), scale=0.125, softcap=20.0)
        exp = O.attention(q, kv_type, k, v, D, L, Hkv, mask=mask, sinks=sinks, scale=0.125, softcap=20.0)
        rel = np.linalg.norm(out.numpy() - exp) / np.linalg.norm(exp)
        assert rel < 1e-6, rel
        dist.barrier()
        dist.destroy_process_group()
    except BaseException as e:  # report to the parent instead of hanging the others
        errq.put(f"rank {rank}: {type(e).__name__}: {e}")
        raise


@pytest.mark.parametrize("world,kv_type,H,N,L", [(2, O.Q8_0, 6, 4, 700), (3, O.F16, 3, 3, 640), (4, O.Q8_0, 6, 2, 300)])
def test_split_attention_class_over_gloo(world, kv_type, H, N, L):
    """srhpm_b200.split_attn.SplitKAttention itself on gloo ranks: each rank's record set lands in its slot of the
    shared buffer (in-place all_gather_into_tensor), every rank merges all sets; equal to the whole-range oracle.
    H x N = 9 exercises the 16-byte padding of the {max, sum} pairs."""
    ctx = mp.get_context("spawn")
    errq = ctx.SimpleQueue()
    port = free_port()
    procs = [ctx.Process(target=_class_worker, args=(r, world, port, kv_type, H, 2 if H % 2 == 0 else 1, N, L, errq))
             for r in range(world)]
    for p in procs:
        p.start()
    for p in procs:
        p.join(timeout=300)
    alive = [p for p in procs if p.is_alive()]
    for p in alive:
        p.kill()
    errors = []
    while not errq.empty():
        errors.append(errq.get())
    assert not alive, "a rank did not finish"
    assert not errors, errors
    assert all(p.exitcode == 0 for p in procs)
