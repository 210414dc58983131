"""Multi-query attention split over the KV range across the GPUs of one box (one process per GPU).

Rank j holds KV tokens shard.kv_range(L, world, j) of every KV head. It runs srhpm_flash_attn_ext_partial over its
range, the ranks' record sets are all-gathered in rank (= KV) order with one NCCL call, and every rank merges them
with srhpm_flash_attn_merge into the same output flash_attn_ext gives over the whole range. This is the reference's
chunked attention (KV chunks over CPU threads, records merged per row: patch/srhpm.patch:555-579, 779-823) with the
devices as the chunks. Each rank reads 1/world of the cache; the exchange is H * N * 1032 bytes per rank.
"""
import torch
import torch.distributed as dist

from . import shard


class SplitKAttention:
    """Attention of N query tokens and H heads over a KV range split across `world` ranks of `group`.

    __call__(q, k, v, kv_type, mask, ...) takes this rank's slices: k / v uint8 [Hkv, range tokens, row bytes] and
    the mask's columns of the range (f16 [N', range tokens]); q and sinks whole. Returns f32 [N, H, 256] on every
    rank, in the same buffer at every call (copy it to keep it past the next call). Buffers are allocated once, so
    the call can be captured in a CUDA graph. Every rank of the group must make the same calls in the same order."""

    def __init__(self, ctx, rank, world, H, N, device, group=None):
        self.ctx, self.rank, self.world, self.H, self.N, self.group = ctx, rank, world, H, N, group
        self.part_bytes = ctx.flash_attn_part_size(H, N)
        self.parts = torch.empty(world * self.part_bytes, dtype=torch.uint8, device=device)
        self.mine = self.parts[rank * self.part_bytes:(rank + 1) * self.part_bytes]
        self.out = torch.empty((N, H, 256), dtype=torch.float32, device=device)

    def range(self, L):
        return shard.kv_range(L, self.world, self.rank)

    def __call__(self, q, k, v, kv_type, mask=None, sinks=None, scale=1.0, max_bias=0.0, softcap=0.0, work=None):
        self.ctx.flash_attn_ext_partial(q, k, v, kv_type, mask=mask, scale=scale, max_bias=max_bias,
                                        softcap=softcap, out=self.mine, work=work)
        if self.world > 1:
            dist.all_gather_into_tensor(self.parts, self.mine, group=self.group)
        return self.ctx.flash_attn_merge(self.parts, self.world, self.H, self.N, sinks=sinks, out=self.out)
