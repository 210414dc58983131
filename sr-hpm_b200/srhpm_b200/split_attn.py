"""Multi-query attention split over the KV range across the GPUs of one box (one process per GPU).

Rank j holds KV tokens shard.kv_range(L, world, j) of every KV head. It runs srhpm_flash_attn_ext_partial over its
range, the ranks' record sets are exchanged, and every rank merges them in rank (= KV) order into the same output
flash_attn_ext gives over the whole range. This is the reference's chunked attention (KV chunks over CPU threads,
records merged per row: patch/srhpm.patch:555-579, 779-823) with the devices as the chunks. Each rank reads 1/world
of the cache; the exchange is H * N * 1032 bytes per rank, sent by every rank straight into the others'
symmetric-memory buffers over NVLink, or through one NCCL all-gather.
"""
import torch
import torch.distributed as dist

from . import shard


class SplitKAttention:
    """Attention of N query tokens and H heads over a KV range split across `world` ranks of `group`.

    __call__(q, k, v, kv_type, mask, ...) takes this rank's slices: k / v uint8 [Hkv, range tokens, row bytes] and
    the mask's columns of the range (f16 [N', range tokens]); q and sinks whole. Returns f32 [N, H, 256] on every
    rank, in the same buffer at every call (copy it to keep it past the next call). Buffers are allocated once, so
    the call can be captured in a CUDA graph. Every rank of the group must make the same calls in the same order.

    exchange="peers" (default): each rank's record set stays in its own symmetric-memory buffer; the merge kernel
    sends every rank its record rows as (value, epoch) words over NVLink and merges what it receives
    (srhpm_flash_attn_merge_peers): no collective launch. exchange="nccl": the record sets are all-gathered with NCCL
    and merged (srhpm_flash_attn_merge). Same result either way."""

    def __init__(self, ctx, rank, world, H, N, device, group=None, exchange="peers"):
        self.ctx, self.rank, self.world, self.H, self.N, self.group = ctx, rank, world, H, N, group
        self.exchange = exchange
        self.part_bytes = ctx.flash_attn_part_size(H, N)
        self.out = torch.empty((N, H, 256), dtype=torch.float32, device=device)
        if exchange == "peers":
            import torch.distributed._symmetric_memory as symm
            nbytes = ctx.flash_attn_peer_buffer_size(H, N)
            buf = symm.empty(nbytes, dtype=torch.uint8, device=device)
            buf.zero_()
            hdl = symm.rendezvous(buf, group if group is not None else dist.group.WORLD)
            self._buf, self._hdl = buf, hdl
            self.peers = torch.tensor([int(p) for p in hdl.buffer_ptrs], dtype=torch.int64, device=device)
            self.epochs = torch.zeros(H * N, dtype=torch.int32, device=device)
            self.mine = buf[:self.part_bytes]
            torch.cuda.synchronize(device)
            dist.barrier(group=group)
        elif exchange == "nccl":
            self.parts = torch.empty(world * self.part_bytes, dtype=torch.uint8, device=device)
            self.mine = self.parts[rank * self.part_bytes:(rank + 1) * self.part_bytes]
        else:
            raise ValueError(f"exchange must be 'nccl' or 'peers', not {exchange!r}")

    def range(self, L):
        return shard.kv_range(L, self.world, self.rank)

    def __call__(self, q, k, v, kv_type, mask=None, sinks=None, scale=1.0, max_bias=0.0, softcap=0.0, work=None):
        self.ctx.flash_attn_ext_partial(q, k, v, kv_type, mask=mask, scale=scale, max_bias=max_bias,
                                        softcap=softcap, out=self.mine, work=work)
        if self.exchange == "peers":
            return self.ctx.flash_attn_merge_peers(self.peers, self.world, self.rank, self.epochs, self.H, self.N,
                                                   sinks=sinks, out=self.out)
        if self.world > 1:
            dist.all_gather_into_tensor(self.parts, self.mine, group=self.group)
        return self.ctx.flash_attn_merge(self.parts, self.world, self.H, self.N, sinks=sinks, out=self.out)
