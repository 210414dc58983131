"""Sharding of the verify path across the GPUs of one box (one process per GPU).

Output rows of a weight matrix are independent, so the verify GEMM shards by rows exactly as the reference splits a
matrix between its CPU and GPU (patch/srhpm.patch:6497-6529): rank j computes rows [rows*j/world, rows*(j+1)/world)
and the slices are all-gathered. Row-parallel layers (attention output, FFN down) shard K on 256-column super-block
boundaries and sum the partial products. The head shards the vocabulary; the acceptance merges per-shard argmax
records (srhpm_argmax_shard / srhpm_accept_merge). Attention shards by KV head, or by KV token range when there
are more ranks than KV heads (each rank's (max, sum, acc) records are all-gathered and merged, as the reference
merges the records of its KV chunks, patch/srhpm.patch:779-823).

This module holds the index arithmetic and the gather layout; the collectives are torch.distributed calls made by the
caller (NCCL on GPUs, gloo in the CPU tests).
"""

QK = 256  # columns per K-quant super-block


def row_range(rows, world, rank):
    """Rows [r0, r1) of `rows` owned by `rank` (balanced; sizes differ by at most one)."""
    return rows * rank // world, rows * (rank + 1) // world


def k_range(K, world, rank):
    """Columns [k0, k1) of a K-split (row-parallel) shard, on super-block boundaries (sizes differ by at most one
    super-block: 68 super-blocks over 8 ranks give 9 or 8)."""
    nsb = K // QK
    return nsb * rank // world * QK, nsb * (rank + 1) // world * QK


def vocab_range(n_vocab, world, rank):
    """Vocabulary ids [v0, v1) of a head shard."""
    return n_vocab * rank // world, n_vocab * (rank + 1) // world


def kv_heads(n_kv, world, rank):
    """KV heads [g0, g1) of an attention shard (world must divide n_kv)."""
    if n_kv % world:
        raise ValueError(f"{n_kv} KV heads do not split over {world} ranks")
    per = n_kv // world
    return per * rank, per * (rank + 1)


KV_TILE = 128  # tokens per attention tile


def kv_range(L, world, rank):
    """KV tokens [t0, t1) of a split-K attention shard: whole 128-token tiles, balanced (tile counts differ by at
    most one), the last range ending at L; a rank gets an empty range when there are fewer tiles than ranks."""
    tiles = -(-L // KV_TILE)
    return min(L, tiles * rank // world * KV_TILE), min(L, tiles * (rank + 1) // world * KV_TILE)


def k_columns(blocks, blk, bpb, k0, k1):
    """Columns [k0, k1) of packed weight rows (numpy uint8 [rows, row bytes], blk values per bpb-byte block; k0, k1 on
    block boundaries) as a contiguous [rows, (k1 - k0) / blk * bpb] array."""
    if k0 % blk or k1 % blk:
        raise ValueError("a column range must start and end on block boundaries")
    import numpy as np
    return np.ascontiguousarray(blocks[:, k0 // blk * bpb:k1 // blk * bpb])


def tp_layout(H, Hkv, n_ff, n_vocab, world, rank):
    """Megatron tensor-parallel slices of rank `rank` of `world` for a GQA decoder (the split of the 27B step):
    query heads [h0, h1); KV heads [g0, g1) (when world > Hkv each KV head is replicated on world / Hkv ranks, the
    ones holding its query heads); FFN rows [f0, f1) on super-block boundaries (the K range of the row-parallel down
    matrix); vocabulary rows [v0, v1) of the head. Column-parallel: QKV, gate, up, head. Row-parallel: O (K = the
    rank's heads), down (K = its FFN rows)."""
    if H % world:
        raise ValueError(f"{H} query heads do not split over {world} ranks")
    hq = H // world
    h0, h1 = rank * hq, (rank + 1) * hq
    if Hkv % world == 0:
        g0, g1 = rank * (Hkv // world), (rank + 1) * (Hkv // world)
    elif world % Hkv == 0:
        g0 = rank // (world // Hkv)
        g1 = g0 + 1
    else:
        raise ValueError(f"{Hkv} KV heads do not map onto {world} ranks")
    G = H // Hkv
    if not (g0 * G <= h0 and h1 <= g1 * G):
        raise ValueError("a rank's query heads must share its KV heads")
    f0, f1 = k_range(n_ff, world, rank)
    v0, v1 = vocab_range(n_vocab, world, rank)
    # KV replicas: r ranks share each KV head (1 when the KV heads split); p is this rank's place among them and
    # [gh0, gh1) the query heads of its KV heads (all r ranks' heads)
    r = world // Hkv if world > Hkv else 1
    return dict(h0=h0, h1=h1, g0=g0, g1=g1, f0=f0, f1=f1, v0=v0, v1=v1, r=r, p=rank % r, gh0=g0 * G, gh1=g1 * G)


def q_heads(lay, split):
    """The query heads [a, b) whose rows of the QKV matrix a rank holds in one layer: its own heads, or, on a layer whose
    attention the KV head's replicas split over the KV range (`split`: lay["r"] > 1), every query head of its KV head
    (each replica computes all of them over its part of the tokens)."""
    return (lay["gh0"], lay["gh1"]) if split and lay["r"] > 1 else (lay["h0"], lay["h1"])


class PackedSlices:
    """Layout of the row slices of several products in one buffer per rank, for one all-gather per step.

    Product i (N_i rows of activations, rows_i output rows) owns N_i * ceil(rows_i / world) floats of every rank's
    buffer (the slice of rank j fills N_i * (r1 - r0) of them, as an [N_i, r1 - r0] row-major block), so that all ranks'
    buffers have one size. After all-gathering into [world][size], `unpack` rebuilds each product's [N_i, rows_i]."""

    def __init__(self, shapes, world):
        self.shapes = list(shapes)  # (N, rows)
        self.world = world
        self.offsets = []
        off = 0
        for N, rows in self.shapes:
            self.offsets.append(off)
            off += N * (-(-rows // world))
        self.size = off

    def local_view(self, buf, i, rank):
        """The [N, r1 - r0] block of product i in rank `rank`'s buffer (a torch view or numpy view)."""
        N, rows = self.shapes[i]
        r0, r1 = row_range(rows, self.world, rank)
        o = self.offsets[i]
        return buf[o:o + N * (r1 - r0)].reshape(N, r1 - r0)

    def unpack(self, gathered, i):
        """Product i as [N, rows] from the gathered buffer ([world * size], ranks in order), concatenated along rows."""
        N, rows = self.shapes[i]
        parts = [self.local_view(gathered[j * self.size:(j + 1) * self.size], i, j) for j in range(self.world)]
        if hasattr(parts[0], "new_empty"):  # torch
            import torch
            return torch.cat(parts, dim=1)
        import numpy as np
        return np.concatenate(parts, axis=1)
