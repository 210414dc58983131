"""Megatron tensor parallelism of the decoder step on CPU ranks over gloo, with the oracle as every rank's compute.

Each rank takes the slices `shard.tp_layout` and `shard.k_columns` give it (the same cuts the GPU path uploads):
- its query heads and KV heads of QKV, and its caches' KV heads;
- the O columns of its heads;
- its FFN rows of gate / up and the down columns of them;
- its vocabulary rows of the head.

The partial O / down products are all-reduced. Logits are gathered, and the result must equal the oracle's
unsharded `decoder_step`. The oracle sums exact integer block dots in f64, so only f64 rounding separates the two.

World sizes cover what the GPU tests cannot run here: 4 ranks with each KV head replicated on 2 of them, and 4 ranks
with one KV head each; with the replicas of a KV head splitting the full-attention layer's tokens (2 and 4 replicas)
as the GPU step does when there are more ranks than KV heads."""
import os
import socket

import numpy as np
import pytest
import torch
import torch.distributed as dist
import torch.multiprocessing as mp

import oracle as O
from srhpm_b200 import shard

QT = O.Q4_K


def free_port():
    s = socket.socket()
    s.bind(("127.0.0.1", 0))
    p = s.getsockname()[1]
    s.close()
    return p


def make_model(H, Hkv, seed=3):
    cfg = dict(n_layer=2, d=256, n_ff=1024, H=H, Hkv=Hkv, hd=128, n_vocab=300, base=1e6, eps=1e-6, window=24,
               full_every=2, kv_type=O.F16, types={k: QT for k in ("qkv", "o", "gate", "up", "down", "head")})
    rng = np.random.default_rng(seed)

    def q(rows, K):
        return O.random_blocks(QT, rows * K // 256, rng, d_lo=0.002, d_hi=0.004).reshape(rows, -1)

    d, hd, nf = cfg["d"], cfg["hd"], cfg["n_ff"]
    w = {k: [] for k in ("qkv", "o", "gate", "up", "down", "attn_norm", "ffn_norm")}
    for _ in range(cfg["n_layer"]):
        w["qkv"].append(q((H + 2 * Hkv) * hd, d))
        w["o"].append(q(d, H * hd))
        w["gate"].append(q(nf, d))
        w["up"].append(q(nf, d))
        w["down"].append(q(d, nf))
        w["attn_norm"].append((1 + 0.1 * rng.standard_normal(d)).astype(np.float32))
        w["ffn_norm"].append((1 + 0.1 * rng.standard_normal(d)).astype(np.float32))
    w["out_norm"] = (1 + 0.1 * rng.standard_normal(d)).astype(np.float32)
    w["head"] = q(cfg["n_vocab"], d)
    w["emb"] = rng.standard_normal((cfg["n_vocab"], d)).astype(np.float16)
    return cfg, w


def caches(cfg, cap, n_past, seed=4):
    rng = np.random.default_rng(seed)
    kc, vc = [], []
    for _ in range(cfg["n_layer"]):
        for lst in (kc, vc):
            a = np.zeros((cap, cfg["Hkv"], 2 * cfg["hd"]), np.uint8)
            a[:n_past] = O.cache_rows(O.F16, rng.standard_normal((n_past, cfg["Hkv"], cfg["hd"])).astype(np.float32))
            lst.append(a)
    return kc, vc


def tp_step(cfg, w, kc, vc, ids, n_past, rank, world, split=False):
    """The rank's share of O.decoder_step; collectives over the default (gloo) group. split: on full-attention layers
    the r replicas of a KV head (more ranks than KV heads) split its tokens: each computes the records of its part for
    every query head of the KV head, the records are gathered and the replicas' sets merged in replica order."""
    c = cfg
    lay = shard.tp_layout(c["H"], c["Hkv"], c["n_ff"], c["n_vocab"], world, rank)
    h0, h1, g0, g1, f0, f1, v0, v1 = (lay[k] for k in ("h0", "h1", "g0", "g1", "f0", "f1", "v0", "v1"))
    H, Hkv, hd, d = c["H"], c["Hkv"], c["hd"], c["d"]
    nh, ng = h1 - h0, g1 - g0
    n = len(ids)
    pos = np.arange(n_past, n_past + n)
    kcl = [np.ascontiguousarray(a[:, g0:g1]) for a in kc]
    vcl = [np.ascontiguousarray(a[:, g0:g1]) for a in vc]

    def all_reduce(a):
        t = torch.from_numpy(np.ascontiguousarray(a, np.float64))
        dist.all_reduce(t)
        return t.numpy()

    x = w["emb"][np.asarray(ids)].astype(np.float32)
    for l in range(c["n_layer"]):
        y = O.rms_norm(x, w["attn_norm"][l], c["eps"])
        full = w["qkv"][l]
        is_full = c["window"] <= 0 or l % c["full_every"] == c["full_every"] - 1
        split_l = split and lay["r"] > 1 and is_full
        qa, qb = shard.q_heads(lay, split_l)  # this layer's query heads: the rank's, or all of its KV head's
        nq = qb - qa
        wq = np.concatenate([full[qa * hd:qb * hd], full[(H + g0) * hd:(H + g1) * hd],
                             full[(H + Hkv + g0) * hd:(H + Hkv + g1) * hd]])
        qkv = O.mul_mat(QT, wq, (nq + 2 * ng) * hd, d, y).astype(np.float32)
        q = O.rope_neox(qkv[:, :nq * hd].reshape(n, nq, hd), pos, c["base"])
        k = O.rope_neox(qkv[:, nq * hd:(nq + ng) * hd].reshape(n, ng, hd), pos, c["base"])
        v = qkv[:, (nq + ng) * hd:].reshape(n, ng, hd)
        kcl[l][n_past:n_past + n] = O.cache_rows(O.F16, k)
        vcl[l][n_past:n_past + n] = O.cache_rows(O.F16, v)
        start, mask = O.attn_window(l, c["full_every"], c["window"], n_past, n)
        kk = np.ascontiguousarray(kcl[l][start:n_past + n].transpose(1, 0, 2))
        vv = np.ascontiguousarray(vcl[l][start:n_past + n].transpose(1, 0, 2))
        qt = np.ascontiguousarray(q.transpose(1, 0, 2))
        Lv = n_past + n - start
        if split_l:
            t0, t1 = shard.kv_range(Lv, lay["r"], lay["p"])
            m, sm, acc = O.attention_partial(qt, O.F16, kk, vv, hd, Lv, ng, t0, t1, mask=mask.view(np.uint16),
                                             scale=1.0 / np.sqrt(hd))
            rec = torch.from_numpy(np.concatenate([m.ravel(), sm.ravel(), acc.ravel()]))
            recs = [torch.zeros_like(rec) for _ in range(world)]
            dist.all_gather(recs, rec)
            base, hn = rank // lay["r"] * lay["r"], nq * n
            mine = [recs[base + j].numpy() for j in range(lay["r"])]  # the replicas, in replica (= token) order
            merged = O.attention_merge(np.stack([r_[:hn].reshape(nq, n) for r_ in mine]),
                                       np.stack([r_[hn:2 * hn].reshape(nq, n) for r_ in mine]),
                                       np.stack([r_[2 * hn:].reshape(nq, n, hd) for r_ in mine]))
            att = np.ascontiguousarray(merged[:, h0 - qa:h1 - qa])  # [n, own heads, hd]
        else:
            att = O.attention(qt, O.F16, kk, vv, hd, Lv, ng, mask=mask.view(np.uint16), scale=1.0 / np.sqrt(hd))
        wo = shard.k_columns(w["o"][l], 256, 144, h0 * hd, h1 * hd)
        o = all_reduce(O.mul_mat(QT, wo, d, nh * hd, att.astype(np.float32).reshape(n, nh * hd)))
        x = (x + o.astype(np.float32)).astype(np.float32)
        y = O.rms_norm(x, w["ffn_norm"][l], c["eps"])
        g = O.mul_mat(QT, w["gate"][l][f0:f1], f1 - f0, d, y).astype(np.float32)
        u = O.mul_mat(QT, w["up"][l][f0:f1], f1 - f0, d, y).astype(np.float32)
        hh = O.swiglu(g, u)
        wd = shard.k_columns(w["down"][l], 256, 144, f0, f1)
        dn = all_reduce(O.mul_mat(QT, wd, d, f1 - f0, hh))
        x = (x + dn.astype(np.float32)).astype(np.float32)
    y = O.rms_norm(x, w["out_norm"], c["eps"])
    part = O.mul_mat(QT, w["head"][v0:v1], v1 - v0, d, y).astype(np.float32)
    # vocabulary shards differ in size by at most one row: pad to the largest, gather, cut
    width = -(-c["n_vocab"] // world)
    buf = torch.zeros((n, width))
    buf[:, :v1 - v0] = torch.from_numpy(part)
    parts = [torch.zeros((n, width)) for _ in range(world)]
    dist.all_gather(parts, buf)
    cols = [parts[r][:, :shard.vocab_range(c["n_vocab"], world, r)[1] - shard.vocab_range(c["n_vocab"], world, r)[0]]
            for r in range(world)]
    return torch.cat(cols, dim=1).numpy()


def _worker(rank, world, port, H, Hkv, split, errq):
    try:
        os.environ.update(MASTER_ADDR="127.0.0.1", MASTER_PORT=str(port))
        dist.init_process_group("gloo", rank=rank, world_size=world)
        cfg, w = make_model(H, Hkv)
        # 300 past tokens: the full-attention layer's 305 tokens are 3 tiles, so with 4 replicas one part is empty
        cap, n_past, ids = (320, 300, [3, 77, 150, 299, 12]) if split else (64, 40, [3, 77, 150, 299, 12])
        kc, vc = caches(cfg, cap, n_past)
        got = tp_step(cfg, w, kc, vc, ids, n_past, rank, world, split)
        if rank == 0:
            kc1, vc1 = caches(cfg, cap, n_past)
            exp, _ = O.decoder_step(cfg, w, kc1, vc1, ids, n_past, ids[1:])
            rel = np.linalg.norm(got - exp) / np.linalg.norm(exp)
            assert rel < 1e-6, rel
        dist.barrier()
        dist.destroy_process_group()
    except BaseException as e:  # report to the parent instead of hanging the others
        errq.put(f"rank {rank}: {type(e).__name__}: {e}")
        raise


@pytest.mark.parametrize("world,H,Hkv,split", [(2, 4, 2, False), (4, 8, 2, False), (4, 8, 4, False),
                                                (2, 4, 1, True), (4, 8, 2, True), (4, 8, 1, True)])
def test_tensor_parallel_step_equals_unsharded(world, H, Hkv, split):
    """split: the KV head's replicas (2 or 4 of them) split the full-attention layer's tokens and merge their
    records, as the GPU step does with more ranks than KV heads."""
    ctx = mp.get_context("spawn")
    errq = ctx.SimpleQueue()
    port = free_port()
    procs = [ctx.Process(target=_worker, args=(r, world, port, H, Hkv, split, errq)) for r in range(world)]
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
