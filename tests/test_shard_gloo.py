"""Host side of the multi-GPU path (srhpm_b200.shard) on CPU ranks over gloo.

Each rank computes its shard with the oracle (the CPU stand-in for its GPU), the collectives run over gloo, and the
gathered / reduced results must equal the unsharded oracle results: row shards bit for bit, K shards within f64
rounding, KV-head shards of attention bit for bit."""
import os
import socket

import numpy as np
import pytest
import torch
import torch.distributed as dist
import torch.multiprocessing as mp

import oracle as O
from srhpm_b200 import shard


def free_port():
    s = socket.socket()
    s.bind(("127.0.0.1", 0))
    p = s.getsockname()[1]
    s.close()
    return p


def test_row_and_vocab_ranges_partition():
    for rows in (1, 7, 5120, 6144, 17408, 151936):
        for world in (1, 2, 3, 4, 8):
            rr = [shard.row_range(rows, world, r) for r in range(world)]
            assert rr[0][0] == 0 and rr[-1][1] == rows
            assert all(rr[i][1] == rr[i + 1][0] for i in range(world - 1))
            sizes = [b - a for a, b in rr]
            assert max(sizes) - min(sizes) <= 1
            assert [shard.vocab_range(rows, world, r) for r in range(world)] == rr


def test_k_range_superblock_boundaries():
    for K in (5120, 17408, 6144):
        for world in (2, 4, 8):
            ks = [shard.k_range(K, world, r) for r in range(world)]
            assert ks[0][0] == 0 and ks[-1][1] == K
            assert all(a % 256 == 0 and b % 256 == 0 for a, b in ks)
            nsb = [(b - a) // 256 for a, b in ks]
            assert max(nsb) - min(nsb) <= 1
    assert [(b - a) // 256 for a, b in (shard.k_range(17408, 8, r) for r in range(8))] == [8, 9, 8, 9, 8, 9, 8, 9]


def test_kv_heads():
    assert [shard.kv_heads(4, 4, r) for r in range(4)] == [(0, 1), (1, 2), (2, 3), (3, 4)]
    with pytest.raises(ValueError):
        shard.kv_heads(4, 8, 0)


def test_packed_slices_roundtrip():
    rng = np.random.default_rng(0)
    shapes = [(2, 5120), (4, 17409), (8, 7), (1, 3)]
    for world in (1, 2, 3, 8):
        pk = shard.PackedSlices(shapes, world)
        full = [rng.standard_normal(s).astype(np.float32) for s in shapes]
        bufs = [np.zeros(pk.size, np.float32) for _ in range(world)]
        for r in range(world):
            for i, (N, rows) in enumerate(shapes):
                r0, r1 = shard.row_range(rows, world, r)
                pk.local_view(bufs[r], i, r)[...] = full[i][:, r0:r1]
        gathered = np.concatenate(bufs)
        for i in range(len(shapes)):
            assert np.array_equal(pk.unpack(gathered, i), full[i])


# ---- multi-process (gloo) -----------------------------------------------------------------------------------------

def _weights(qtype, rows, K, seed):
    return O.random_blocks(qtype, rows * K // O.BLOCK_ELEMS[qtype], np.random.default_rng(seed)).reshape(rows, -1)


def _worker(rank, world, port, case, errq):
    try:
        os.environ.update(MASTER_ADDR="127.0.0.1", MASTER_PORT=str(port))
        dist.init_process_group("gloo", rank=rank, world_size=world)
        rng = np.random.default_rng(5)
        if case == "rows":
            shapes = [(4, 17408, 5120, O.Q4_K), (2, 5120, 5120, O.Q6_K), (8, 6144, 5120, O.IQ4_XS)]
            pk = shard.PackedSlices([(N, rows) for N, rows, K, t in shapes], world)
            local = torch.zeros(pk.size)
            Xs = [rng.standard_normal((N, K)).astype(np.float32) for N, rows, K, t in shapes]
            for i, (N, rows, K, t) in enumerate(shapes):
                W = _weights(t, rows, K, 100 + i)
                r0, r1 = shard.row_range(rows, world, rank)
                pk.local_view(local, i, rank)[...] = torch.from_numpy(O.mul_mat(t, W[r0:r1], r1 - r0, K, Xs[i]))
            parts = [torch.zeros(pk.size) for _ in range(world)]
            dist.all_gather(parts, local)
            gathered = torch.cat(parts)
            if rank == 0:
                for i, (N, rows, K, t) in enumerate(shapes):
                    full = O.mul_mat(t, _weights(t, rows, K, 100 + i), rows, K, Xs[i])
                    assert np.array_equal(pk.unpack(gathered, i).numpy(), full.astype(np.float32)), i
        elif case == "ksplit":
            rows, K, N, t = 512, 17408, 4, O.Q4_K
            W = _weights(t, rows, K, 7)
            X = rng.standard_normal((N, K)).astype(np.float32)
            k0, k1 = shard.k_range(K, world, rank)
            bpr = O.BLOCK_BYTES[t]
            Wk = np.ascontiguousarray(W[:, k0 // 256 * bpr:k1 // 256 * bpr])
            part = torch.from_numpy(O.mul_mat(t, Wk, rows, k1 - k0, np.ascontiguousarray(X[:, k0:k1])))
            dist.all_reduce(part)
            full = O.mul_mat(t, W, rows, K, X)
            rel = np.linalg.norm(part.numpy() - full) / np.linalg.norm(full)
            assert rel < 1e-12, rel
        elif case == "heads":
            H, Hkv, N, D, L = 24, 4, 8, 256, 300
            q = (rng.standard_normal((H, N, D)) / 16).astype(np.float32)
            kv = [np.stack([O.quantize_row_q8_0(r) for r in rng.standard_normal((Hkv * L, D)).astype(np.float32)])
                  .reshape(Hkv, L, -1) for _ in range(2)]
            mask = np.zeros((N, L), np.float16)
            for tq in range(N):
                mask[tq, L - N + tq + 1:] = -np.inf
            g0, g1 = shard.kv_heads(Hkv, world, rank)
            G = H // Hkv
            mine = O.attention(q[g0 * G:g1 * G], O.Q8_0, kv[0][g0:g1], kv[1][g0:g1], D, L, g1 - g0,
                               mask=mask.view(np.uint16))
            parts = [torch.zeros((N, (g1 - g0) * G, D), dtype=torch.float64) for _ in range(world)]
            dist.all_gather(parts, torch.from_numpy(mine))
            if rank == 0:
                got = torch.cat(parts, dim=1).numpy()
                full = O.attention(q, O.Q8_0, kv[0], kv[1], D, L, Hkv, mask=mask.view(np.uint16))
                assert np.array_equal(got, full)
        dist.barrier()
        dist.destroy_process_group()
    except BaseException as e:  # report to the parent instead of hanging the others
        errq.put(f"rank {rank}: {type(e).__name__}: {e}")
        raise


@pytest.mark.parametrize("case,world", [("rows", 2), ("rows", 3), ("ksplit", 2), ("heads", 2), ("heads", 4)])
def test_sharded_path_over_gloo(case, world):
    ctx = mp.get_context("spawn")
    errq = ctx.SimpleQueue()
    port = free_port()
    procs = [ctx.Process(target=_worker, args=(r, world, port, case, errq)) for r in range(world)]
    for p in procs:
        p.start()
    for p in procs:
        p.join(timeout=240)
    alive = [p for p in procs if p.is_alive()]
    for p in alive:
        p.kill()
    errors = []
    while not errq.empty():
        errors.append(errq.get())
    assert not alive, "a rank did not finish"
    assert not errors, errors
    assert all(p.exitcode == 0 for p in procs)
