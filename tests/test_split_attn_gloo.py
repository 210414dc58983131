"""Attention split over the KV range across CPU ranks over gloo, with the oracle as every rank's compute.

Each rank takes its tokens from shard.kv_range, the same cut the GPU path uses. It computes the (max, sum, acc) records
of its range (oracle.attention_partial). The ranks all-gather them in rank order, and every rank merges them
(oracle.attention_merge: the reference's record merge, patch/srhpm.patch:789-823). The result must equal the
single-pass oracle over the whole range to f64 rounding. World sizes 2-4, with ranks left without tokens when the
cache has fewer 128-token tiles than ranks."""
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
