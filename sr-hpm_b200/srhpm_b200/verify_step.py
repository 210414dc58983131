"""A full verify step of a dense decoder on one GPU, from the library's kernels: token embeddings, per layer RMSNorm,
fused QKV GEMM, NEOX RoPE + KV-cache store, GQA attention over the cache (sliding-window layers see the last `window`
positions), output GEMM, residual, RMSNorm, gate / up GEMMs, SwiGLU, down GEMM, residual; final RMSNorm, output head
GEMM and greedy acceptance of the draft.

This is the measurement harness of the 27B-class step (1 accepted + k drafted tokens scored in one pass); every call it
makes is a C-ABI entry point of libsrhpm_b200 with arguments built once, so a step can be captured in a CUDA graph.
"""
import ctypes
import math

import numpy as np
import torch

from . import _lib as L
from .ops import QuantTensor, _tensor_view, blck_size, f32_rows_view, quantize_chunk, row_size, type_size


class DecoderConfig:
    """Architecture of the synthetic decoder (defaults: the 27B-class model: 64 layers, d 5120, FFN 17408)."""

    def __init__(self, n_layer=64, d=5120, n_ff=17408, H=24, Hkv=4, hd=256, n_vocab=151936, base=1e6, eps=1e-6,
                 window=4096, full_every=4, kv_type=L.F16, types=None):
        self.n_layer, self.d, self.n_ff, self.H, self.Hkv, self.hd = n_layer, d, n_ff, H, Hkv, hd
        self.n_vocab, self.base, self.eps, self.window, self.full_every = n_vocab, base, eps, window, full_every
        self.kv_type = kv_type
        self.types = types or {"qkv": L.Q4_K, "o": L.Q4_K, "gate": L.Q3_K, "up": L.Q3_K, "down": L.Q4_K,
                               "head": L.Q6_K}

    def full_layer(self, li):
        """Layer li attends to the whole cache (else to the last `window` positions)."""
        return self.window <= 0 or li % self.full_every == self.full_every - 1

    def as_dict(self):
        return dict(n_layer=self.n_layer, d=self.d, n_ff=self.n_ff, H=self.H, Hkv=self.Hkv, hd=self.hd,
                    n_vocab=self.n_vocab, base=self.base, eps=self.eps, window=self.window,
                    full_every=self.full_every, kv_type=self.kv_type, types=dict(self.types))

    def shapes(self):
        """(name, type, rows, K) of every weight matrix of one layer."""
        t = self.types
        return [("qkv", t["qkv"], (self.H + 2 * self.Hkv) * self.hd, self.d), ("o", t["o"], self.d, self.H * self.hd),
                ("gate", t["gate"], self.n_ff, self.d), ("up", t["up"], self.n_ff, self.d),
                ("down", t["down"], self.d, self.n_ff)]

    def weight_bytes(self):
        per = sum(rows * row_size(t, K) for _, t, rows, K in self.shapes())
        return self.n_layer * per + self.n_vocab * row_size(self.types["head"], self.d)


def host_weights(cfg, seed=0, std=0.02):
    """Weights drawn from N(0, std) and quantized on the host (srhpm_quantize_chunk): for small models and tests."""
    rng = np.random.default_rng(seed)
    w = {k: [] for k in ("qkv", "o", "gate", "up", "down", "attn_norm", "ffn_norm")}
    for _ in range(cfg.n_layer):
        for name, t, rows, K in cfg.shapes():
            w[name].append(quantize_chunk((rng.standard_normal((rows, K)) * std).astype(np.float32), t))
        w["attn_norm"].append((1.0 + 0.1 * rng.standard_normal(cfg.d)).astype(np.float32))
        w["ffn_norm"].append((1.0 + 0.1 * rng.standard_normal(cfg.d)).astype(np.float32))
    w["out_norm"] = (1.0 + 0.1 * rng.standard_normal(cfg.d)).astype(np.float32)
    w["head"] = quantize_chunk((rng.standard_normal((cfg.n_vocab, cfg.d)) * std).astype(np.float32),
                               cfg.types["head"])
    w["emb"] = rng.standard_normal((cfg.n_vocab, cfg.d)).astype(np.float16)
    return w


# offsets of the f16 super-block scales in each block type (random blocks get sane values there)
_D_OFFSETS = {L.Q4_K: (0, 2), L.Q5_K: (0, 2), L.Q6_K: (208,), L.Q3_K: (108,), L.IQ4_XS: (0,), L.Q8_0: (0,)}


def random_blocks_device(t, rows, K, gen, device, d_lo=1e-4, d_hi=2e-4):
    """Random GGUF blocks of type t on the device: random codes and sub-block scales, f16 super-block scales in
    [d_lo, d_hi] (a random-init quantized matrix; quantizing billions of N(0, 0.02) values on the host would take
    hours, and the kernels stream the same bytes either way)."""
    bpb = type_size(t)
    nblk = rows * K // blck_size(t)
    b = torch.randint(0, 256, (nblk, bpb), dtype=torch.uint8, device=device, generator=gen)
    for off in _D_OFFSETS[t]:
        dv = (torch.rand(nblk, device=device, generator=gen) * (d_hi - d_lo) + d_lo).half()
        b[:, off:off + 2] = dv.view(torch.uint8).view(nblk, 2)
    return QuantTensor(b.view(-1), t, rows, K)


class DeviceWeights:
    """The decoder's weights in device memory; `tp` holds the tensor-parallel slice they are (shard.tp_layout: query
    heads, KV heads, FFN rows, vocabulary rows, rank, world; the whole model when world = 1)."""

    def __init__(self, cfg, device):
        self.cfg, self.device = cfg, device
        self.layers = []
        self.out_norm = self.head = self.emb = None
        self.tp = None

    def _set_tp(self, rank, world, split_kv=True):
        from .shard import tp_layout
        self.tp = dict(tp_layout(self.cfg.H, self.cfg.Hkv, self.cfg.n_ff, self.cfg.n_vocab, world, rank), rank=rank,
                       world=world)
        # split_kv: on full-attention layers the r ranks that share a KV head split its tokens (each attends to its
        # part for every query head of the KV head, the records merge over the r ranks), so their QKV slices hold
        # every query head of the KV head there
        self.tp["split_kv"] = bool(split_kv and self.tp["r"] > 1)
        return self.tp

    def q_heads(self, li):
        """The query heads [a, b) of layer li's QKV rows on this rank (shard.q_heads)."""
        from .shard import q_heads
        return q_heads(self.tp, self.tp["split_kv"] and self.cfg.full_layer(li))

    @classmethod
    def from_host(cls, cfg, w, device="cuda", rank=0, world=1, split_kv=True):
        """From host_weights (packed blocks of the whole model); rank / world cut one tensor-parallel rank's slices:
        QKV rows of its query and KV heads (with split_kv and replicated KV heads, every query head of its KV head on
        full-attention layers), O columns of its heads, gate / up rows and down columns of its FFN rows, head rows of
        its vocabulary range."""
        from .shard import k_columns
        self = cls(cfg, device)
        tp = self._set_tp(rank, world, split_kv)
        hd, H, Hkv = cfg.hd, cfg.H, cfg.Hkv
        h0, h1, g0, g1, f0, f1 = tp["h0"], tp["h1"], tp["g0"], tp["g1"], tp["f0"], tp["f1"]
        t = cfg.types

        def kcols(blocks, qt, k0, k1):
            return k_columns(np.asarray(blocks), blck_size(qt), type_size(qt), k0, k1)

        for l in range(cfg.n_layer):
            lay = {}
            qa, qb = self.q_heads(l)
            qkv = np.asarray(w["qkv"][l]).reshape((H + 2 * Hkv) * hd, -1)
            part = np.concatenate([qkv[qa * hd:qb * hd], qkv[(H + g0) * hd:(H + g1) * hd],
                                   qkv[(H + Hkv + g0) * hd:(H + Hkv + g1) * hd]])
            lay["qkv"] = QuantTensor.from_blocks(part, t["qkv"], (qb - qa + 2 * (g1 - g0)) * hd, cfg.d, device)
            o = np.asarray(w["o"][l]).reshape(cfg.d, -1)
            lay["o"] = QuantTensor.from_blocks(kcols(o, t["o"], h0 * hd, h1 * hd), t["o"], cfg.d, (h1 - h0) * hd, device)
            # gate and up as one matrix (gate rows, then up rows): one GEMM launch, SwiGLU reads the halves
            gu = np.concatenate([np.asarray(w["gate"][l]).reshape(cfg.n_ff, -1)[f0:f1],
                                 np.asarray(w["up"][l]).reshape(cfg.n_ff, -1)[f0:f1]])
            lay["gate_up"] = QuantTensor.from_blocks(gu, t["gate"], 2 * (f1 - f0), cfg.d, device)
            dn = np.asarray(w["down"][l]).reshape(cfg.d, -1)
            lay["down"] = QuantTensor.from_blocks(kcols(dn, t["down"], f0, f1), t["down"], cfg.d, f1 - f0, device)
            lay["attn_norm"] = torch.from_numpy(w["attn_norm"][l]).to(device)
            lay["ffn_norm"] = torch.from_numpy(w["ffn_norm"][l]).to(device)
            self.layers.append(lay)
        self.out_norm = torch.from_numpy(w["out_norm"]).to(device)
        head = np.asarray(w["head"]).reshape(cfg.n_vocab, -1)[tp["v0"]:tp["v1"]]
        self.head = QuantTensor.from_blocks(head, t["head"], tp["v1"] - tp["v0"], cfg.d, device)
        self.emb = torch.from_numpy(w["emb"]).to(device)
        return self

    @classmethod
    def random(cls, cfg, device="cuda", seed=0, rank=0, world=1, split_kv=True):
        """Random GGUF blocks of one tensor-parallel rank's slice shapes (the whole model when world = 1)."""
        self = cls(cfg, device)
        tp = self._set_tp(rank, world, split_kv)
        gen = torch.Generator(device=device)
        gen.manual_seed(seed + 1000 * rank)
        hd, t = cfg.hd, cfg.types
        nh, ng, nf = tp["h1"] - tp["h0"], tp["g1"] - tp["g0"], tp["f1"] - tp["f0"]
        for l in range(cfg.n_layer):
            qa, qb = self.q_heads(l)
            lay = {"qkv": random_blocks_device(t["qkv"], (qb - qa + 2 * ng) * hd, cfg.d, gen, device),
                   "o": random_blocks_device(t["o"], cfg.d, nh * hd, gen, device),
                   "gate_up": random_blocks_device(t["gate"], 2 * nf, cfg.d, gen, device),
                   "down": random_blocks_device(t["down"], cfg.d, nf, gen, device)}
            lay["attn_norm"] = 1.0 + 0.1 * torch.randn(cfg.d, device=device, generator=gen)
            lay["ffn_norm"] = 1.0 + 0.1 * torch.randn(cfg.d, device=device, generator=gen)
            self.layers.append(lay)
        self.out_norm = 1.0 + 0.1 * torch.randn(cfg.d, device=device, generator=gen)
        self.head = random_blocks_device(t["head"], tp["v1"] - tp["v0"], cfg.d, gen, device)
        self.emb = torch.randn((cfg.n_vocab, cfg.d), device=device, generator=gen).half()
        return self

    @classmethod
    def slice_of(cls, full, rank, world, split_kv=True):
        """One tensor-parallel rank's slices cut on the device from the whole model `full` (world = 1 weights, fused
        qkv and gate|up): the same cuts as from_host (QKV rows of the rank's query and KV heads, O columns of its
        heads, gate / up rows and down columns of its FFN rows, head rows of its vocabulary range). Norms and
        embeddings are shared with `full`."""
        cfg = full.cfg
        self = cls(cfg, full.device)
        tp = self._set_tp(rank, world, split_kv)
        hd, H, Hkv = cfg.hd, cfg.H, cfg.Hkv
        h0, h1, g0, g1, f0, f1 = tp["h0"], tp["h1"], tp["g0"], tp["g1"], tp["f0"], tp["f1"]

        def rows2d(qt):
            return qt.data[:qt.rows * qt.row_bytes].view(qt.rows, qt.row_bytes)

        def kcols(qt, k0, k1):
            b, bs = blck_size(qt.qtype), type_size(qt.qtype)
            part = rows2d(qt)[:, k0 // b * bs:k1 // b * bs].contiguous()
            return QuantTensor(part.view(-1), qt.qtype, qt.rows, k1 - k0)

        for l, lay_f in enumerate(full.layers):
            lay = {}
            qa, qb = self.q_heads(l)
            q = rows2d(lay_f["qkv"])
            part = torch.cat([q[qa * hd:qb * hd], q[(H + g0) * hd:(H + g1) * hd],
                              q[(H + Hkv + g0) * hd:(H + Hkv + g1) * hd]])
            lay["qkv"] = QuantTensor(part.reshape(-1), lay_f["qkv"].qtype, part.shape[0], cfg.d)
            lay["o"] = kcols(lay_f["o"], h0 * hd, h1 * hd)
            gu = rows2d(lay_f["gate_up"])
            part = torch.cat([gu[f0:f1], gu[cfg.n_ff + f0:cfg.n_ff + f1]])
            lay["gate_up"] = QuantTensor(part.reshape(-1), lay_f["gate_up"].qtype, part.shape[0], cfg.d)
            lay["down"] = kcols(lay_f["down"], f0, f1)
            lay["attn_norm"], lay["ffn_norm"] = lay_f["attn_norm"], lay_f["ffn_norm"]
            self.layers.append(lay)
        self.out_norm = full.out_norm
        hr = rows2d(full.head)[tp["v0"]:tp["v1"]].contiguous()
        self.head = QuantTensor(hr.view(-1), full.head.qtype, tp["v1"] - tp["v0"], cfg.d)
        self.emb = full.emb
        return self


class TensorParallel:
    """The collectives of a Megatron tensor-parallel step over torch.distributed.

    fused=True (default): the row-parallel O and down GEMMs write their partial sums into a symmetric buffer (torch
    symmetric memory: every rank's buffer mapped on every rank), and the next RMSNorm exchanges the ranks' rows over
    NVLink as (value, epoch) words and sums them itself (srhpm_add_rms_norm_allreduce): no separate collective
    launch.
    fused=False: an NCCL all-reduce after each of those GEMMs (128 per step for 64 layers). The vocabulary shards'
    argmax records are all-gathered with NCCL before the acceptance either way. All of it is captured in the step's
    CUDA graph."""

    def __init__(self, rank, world, group=None, fused=True, fused_quant=True):
        self.rank, self.world, self.group, self.fused = rank, world, group, fused
        # fused_quant: the all-reduce norm also writes the next GEMM's activation records
        # (srhpm_add_rms_norm_allreduce_quant). Measured on two B200s (27B step at k = 8, one process): 6.45 ms,
        # against 6.61 ms with the norm and a separate quantizer kernel per GEMM and 6.64 ms with GEMMs that quantize
        # in their own grid.
        self.fused_quant = fused_quant
        self.part = self.peers = self.epochs = None

    def setup(self, d, device):
        """Symmetric buffer for the fused all-reduce of rows of d values (collective: every rank calls it)."""
        if not self.fused or self.part is not None:
            return
        import torch.distributed as dist
        import torch.distributed._symmetric_memory as symm
        lib = L.load()
        nbytes = int(lib.srhpm_allreduce_buffer_size(d))
        buf = symm.empty(nbytes, dtype=torch.uint8, device=device)
        buf.zero_()
        hdl = symm.rendezvous(buf, self.group if self.group is not None else dist.group.WORLD)
        self._buf, self._hdl = buf, hdl
        self.peers = torch.tensor([int(p) for p in hdl.buffer_ptrs], dtype=torch.int64, device=device)
        self.epochs = torch.zeros(32, dtype=torch.int32, device=device)
        slot = 16 * d * 4
        self.part = [buf[k * slot:(k + 1) * slot].view(torch.float32).view(16, d) for k in (0, 1)]
        torch.cuda.synchronize(device)
        dist.barrier(group=self.group)

    def setup_attention(self, H, N, r, device):
        """Symmetric buffers for the attention split over the r replicas of a KV head (collective: every rank calls
        it): each rank's record set of H heads and N tokens, exchanged with its replicas by
        srhpm_flash_attn_merge_peers; att_peers holds the r replicas' buffers (this rank at rank % r)."""
        if getattr(self, "att_key", None) == (H, N, r):
            return
        import torch.distributed as dist
        import torch.distributed._symmetric_memory as symm
        lib = L.load()
        buf = symm.empty(int(lib.srhpm_flash_attn_peer_buffer_size(H, N)), dtype=torch.uint8, device=device)
        buf.zero_()
        hdl = symm.rendezvous(buf, self.group if self.group is not None else dist.group.WORLD)
        base = self.rank // r * r
        self._att_buf, self._att_hdl = buf, hdl
        self.att_peers = torch.tensor([int(p) for p in hdl.buffer_ptrs[base:base + r]], dtype=torch.int64,
                                      device=device)
        self.att_epochs = torch.zeros(H * N, dtype=torch.int32, device=device)
        self.att_part = buf[:int(lib.srhpm_flash_attn_part_size(H, N))]
        self.att_key = (H, N, r)
        torch.cuda.synchronize(device)
        dist.barrier(group=self.group)

    def all_reduce(self, t):
        import torch.distributed as dist
        dist.all_reduce(t, group=self.group)

    def all_gather(self, out, t):
        import torch.distributed as dist
        dist.all_gather_into_tensor(out, t, group=self.group)


def _py_call(f):
    """A host callable in the step's call list (signature of the C-ABI calls: arguments then the stream, status
    return). It issues on torch's current stream, which `run` makes the step's stream."""
    def call(*args):
        f()
        return L.OK
    return call


class VerifyStep:
    """One verify step of n tokens (1 accepted + k drafted) at cache position n_past, with prebuilt C-ABI calls.

    kcache / vcache: per layer uint8 [capacity, Hkv, row bytes] (f16 or q8_0 rows), the llama.cpp cache layout.
    With tensor parallelism (`tp`, and weights cut by gguf.load_decoder / DeviceWeights.shard) every dimension below
    is this rank's: its query heads, its KV heads (caches hold only those), its FFN rows and its vocabulary rows; the
    residual stream, norms and embeddings are replicated."""

    def __init__(self, ctx, cfg, weights, kcache, vcache, n_tokens, n_past, relax=0.0, tp=None, fuse_prologue=True,
                 gemm_fused_quant=True, swiglu_in_gemm=True):
        self.ctx, self.cfg, self.w = ctx, cfg, weights
        self.fuse_prologue = fuse_prologue  # RMSNorm writes the next GEMM's activation records itself
        # GEMMs without a fused prologue (the attention output projection; under tensor parallelism the QKV and
        # gate|up GEMMs after the all-reduce norm) quantize their activations in their own grid
        # (srhpm_mul_mat_fused_quant: one launch; the small kernel before each leaves the SMs free, so the grid is
        # resident early)
        self.gemm_fused_quant = gemm_fused_quant
        # with fuse_prologue: the FFN down GEMM computes the SwiGLU of its activation super-blocks in its own grid
        # (srhpm_mul_mat_swiglu, one launch) instead of the SwiGLU record kernel + the GEMM on the records
        self.swiglu_in_gemm = swiglu_in_gemm
        self.kcache, self.vcache = kcache, vcache
        self.n, self.n_past, self.relax = n_tokens, n_past, relax
        self.tp = tp if tp is not None and tp.world > 1 else None
        lay = getattr(weights, "tp", None)
        if self.tp is not None and lay is None:
            raise ValueError("tensor parallelism needs the rank's weight slices")
        self.H = lay["h1"] - lay["h0"] if lay else cfg.H
        self.Hkv = lay["g1"] - lay["g0"] if lay else cfg.Hkv
        # KV heads replicated over r ranks with their tokens split on full-attention layers: those layers compute
        # every query head of the KV head (G of them) over this rank's part of the tokens, and the records merge over
        # the r replicas (TensorParallel.setup_attention)
        self.split = bool(self.tp is not None and lay and lay.get("split_kv"))
        self.G = lay["gh1"] - lay["gh0"] if self.split else self.H
        self.n_ff = lay["f1"] - lay["f0"] if lay else cfg.n_ff
        self.vocab_offset = lay["v0"] if lay else 0
        self.V = weights.head.rows
        dev = weights.device
        c, n = cfg, n_tokens
        f32 = dict(dtype=torch.float32, device=dev)
        self.ids = torch.zeros(n, dtype=torch.int32, device=dev)         # input: accepted token + drafted tokens
        self.draft = torch.zeros(max(n - 1, 1), dtype=torch.int32, device=dev)
        self.pos = torch.arange(n_past, n_past + n, dtype=torch.int32, device=dev)
        self.x = torch.zeros((n, c.d), **f32)                              # residual stream
        self.y = torch.zeros((n, c.d), **f32)                              # normed input of a block
        self.qkv = torch.zeros((n, (max(self.H, self.G) + 2 * self.Hkv) * c.hd), **f32)
        self.att = torch.zeros((n, self.H * c.hd), **f32)
        self.att_all = torch.zeros((n, self.G * c.hd), **f32) if self.split else None  # every head of the KV head
        self.o = torch.zeros((n, c.d), **f32)
        self.gu = torch.zeros((n, 2 * self.n_ff), **f32)                   # gate | up
        self.h = torch.zeros((n, self.n_ff), **f32)
        self.logits = torch.zeros((n, self.V), **f32)
        self.out_ids = torch.zeros(n, dtype=torch.int32, device=dev)
        self.out_n = torch.zeros(1, dtype=torch.int32, device=dev)
        if self.tp is not None:
            self.rec = torch.zeros((n, 16), dtype=torch.uint8, device=dev)            # srhpm_argmax_record rows
            self.rec_all = torch.zeros((self.tp.world, n, 16), dtype=torch.uint8, device=dev)
            self.tp.setup(c.d, dev)
            if self.split:
                self.tp.setup_attention(self.G, n, lay["r"], dev)
        self.lib = L.load()
        self._keep = []
        self._calls = []
        self._build()

    # -- argument building -------------------------------------------------------------------------------------------
    def _ptr(self, t):
        return ctypes.c_void_p(t.data_ptr())

    def _mm(self, W, X, Y, fused_quant=None):
        if fused_quant is None:
            fused_quant = self.gemm_fused_quant
        st, ws = self.ctx.mul_mat_work_size(W, X)
        L.check(st, "srhpm_mul_mat_work_size")
        self._ws = max(self._ws, ws)
        wv, xv, yv = W.view(), f32_rows_view(X), f32_rows_view(Y)
        self._keep += [wv, xv, yv]
        if fused_quant:
            return ("mul_mat_fused_quant", self.lib.srhpm_mul_mat_fused_quant,
                    [self.ctx.handle, ctypes.byref(wv), ctypes.byref(xv), ctypes.byref(yv)], True)
        fn = self.lib.srhpm_mul_mat
        return ("mul_mat", fn, [self.ctx.handle, ctypes.byref(wv), ctypes.byref(xv), ctypes.byref(yv)], True)

    def _all_reduce(self, t):
        return ("all_reduce", _py_call(lambda: self.tp.all_reduce(t)), [], False)

    def _fused(self):
        return self.tp is not None and self.tp.fused

    def _rowpar_out(self, slot):
        """Output of a row-parallel GEMM: the rank's partial sums (fused: slot `slot` of the symmetric buffer)."""
        return self.tp.part[slot][:self.n] if self._fused() else self.o

    def _norm_mm(self, delta_slot, wnorm, W, Y):
        """Residual add + RMSNorm of the pending delta, then the GEMM of W on the normed rows into Y: one fused
        norm + activation-quantization launch and the GEMM on its records (srhpm_add_rms_norm_quant, or with the
        tensor-parallel fused all-reduce and TensorParallel.fused_quant srhpm_add_rms_norm_allreduce_quant, +
        srhpm_mul_mat_prequantized), or the separate norm and then the GEMM quantizing its own activations
        (srhpm_mul_mat_fused_quant, or srhpm_mul_mat and its quantizer kernel without gemm_fused_quant)."""
        ar = delta_slot is not None and self._fused()
        if not self.fuse_prologue or W.qtype == L.Q8_0 or (ar and not self.tp.fused_quant):
            return [self._norm(delta_slot, wnorm), self._mm(W, self.y, Y)]
        c, n, lib, h = self.cfg, self.n, self.lib, self.ctx.handle
        st, ws = self.ctx.mul_mat_work_size(W, self.y)
        L.check(st, "srhpm_mul_mat_work_size")
        self._ws = max(self._ws, ws)
        wv, xv, yv = W.view(), f32_rows_view(self.y), f32_rows_view(Y)
        self._keep += [wv, xv, yv]
        if ar:
            tp = self.tp
            norm = ("add_rms_norm_allreduce_quant", lib.srhpm_add_rms_norm_allreduce_quant,
                    [h, self._ptr(self.x), self._ptr(tp.peers), tp.world, tp.rank, delta_slot, self._ptr(tp.epochs),
                     self._ptr(wnorm), ctypes.c_float(c.eps), self._ptr(self.y), n, ctypes.byref(wv)], True)
        else:
            norm = ("add_rms_norm_quant", lib.srhpm_add_rms_norm_quant,
                    [h, self._ptr(self.x), None if delta_slot is None else self._ptr(self.o), self._ptr(wnorm),
                     ctypes.c_float(c.eps), self._ptr(self.y), n, ctypes.byref(wv)], True)
        return [norm, ("mul_mat_prequantized", lib.srhpm_mul_mat_prequantized,
                       [h, ctypes.byref(wv), ctypes.byref(xv), ctypes.byref(yv)], True)]

    def _norm(self, delta_slot, wnorm):
        """Residual add of the pending delta (none for the first block) + RMSNorm into y."""
        c, n, lib, h = self.cfg, self.n, self.lib, self.ctx.handle
        if delta_slot is not None and self._fused():
            tp = self.tp
            return ("add_rms_norm_allreduce", lib.srhpm_add_rms_norm_allreduce,
                    [h, self._ptr(self.x), self._ptr(tp.peers), tp.world, tp.rank, delta_slot, self._ptr(tp.epochs),
                     self._ptr(wnorm), ctypes.c_float(c.eps), self._ptr(self.y), n, c.d], False)
        return ("add_rms_norm", lib.srhpm_add_rms_norm,
                [h, self._ptr(self.x), None if delta_slot is None else self._ptr(self.o), self._ptr(wnorm),
                 ctypes.c_float(c.eps), self._ptr(self.y), n, c.d], False)

    def _cache_view(self, cache, start, length):
        c = self.cfg
        t = cache[start:start + length]
        tsz = 34 if c.kv_type == L.Q8_0 else 2
        # cache [cap, Hkv, row] -> ggml view [hd, length, Hkv] (token stride = stride(0), head stride = stride(1))
        return _tensor_view(t, c.kv_type, [c.hd, length, self.Hkv], [tsz, t.stride(0), t.stride(1)]), t

    def _build(self):
        c, n, lib, h = self.cfg, self.n, self.lib, self.ctx.handle
        H, Hkv, hd = self.H, self.Hkv, c.hd
        self._ws = 0
        calls = []
        # embeddings (the whole table on every rank)
        n_emb = self.w.emb.shape[0]
        emb_t = L.F16 if self.w.emb.dtype == torch.float16 else L.F32
        esz = self.w.emb.element_size()
        emb_v = _tensor_view(self.w.emb, emb_t, [c.d, n_emb], [esz, self.w.emb.stride(0) * esz])
        self._keep.append(emb_v)
        calls.append(("get_rows", lib.srhpm_get_rows,
                      [h, ctypes.byref(emb_v), self._ptr(self.ids), n, self._ptr(self.x)], False))
        L_all = self.n_past + n
        masks = {}
        for li, lay in enumerate(self.w.layers):
            # this layer's query heads: the rank's own, or every head of its KV head on a split layer
            split = self.split and c.full_layer(li)
            Hq = self.G if split else H
            qkv = self.qkv[:, :(Hq + 2 * Hkv) * hd]
            if "qkv" in lay:
                calls += self._norm_mm(None if li == 0 else 1, lay["attn_norm"], lay["qkv"], qkv)
            else:  # Q, K, V of different types: three GEMMs into the column ranges of the qkv rows
                calls.append(self._norm(None if li == 0 else 1, lay["attn_norm"]))
                calls.append(self._mm(lay["q"], self.y, qkv[:, :Hq * hd]))
                calls.append(self._mm(lay["k"], self.y, qkv[:, Hq * hd:(Hq + Hkv) * hd]))
                calls.append(self._mm(lay["v"], self.y, qkv[:, (Hq + Hkv) * hd:]))
            kv_full, kt = self._cache_view(self.kcache[li], 0, self.kcache[li].shape[0])
            vv_full, vt = self._cache_view(self.vcache[li], 0, self.vcache[li].shape[0])
            self._keep += [kv_full, vv_full, kt, vt]
            calls.append(("rope_kv", lib.srhpm_rope_kv,
                          [h, self._ptr(self.qkv), self.qkv.stride(0), n, Hq, Hkv, hd, self._ptr(self.pos),
                           ctypes.c_float(c.base), ctypes.byref(kv_full), ctypes.byref(vv_full)], False))
            # attention over the visible keys (sliding-window layers: the last `window` positions)
            full = c.full_layer(li)
            start = 0 if full else max(0, self.n_past - c.window + 1)
            if (full, start) not in masks:
                masks[(full, start)] = self._mask(full, start)
                self._keep.append(masks[(full, start)])  # the C calls hold raw pointers into it
            mask = masks[(full, start)]
            t0, t1 = start, L_all
            if split:  # this replica's part of the tokens (whole 128-token tiles)
                from .shard import kv_range
                lay_tp = self.w.tp
                a, b = kv_range(L_all, lay_tp["r"], lay_tp["p"])
                t0, t1 = start + a, start + b
            kv, kt2 = self._cache_view(self.kcache[li], t0, t1 - t0)
            vv, vt2 = self._cache_view(self.vcache[li], t0, t1 - t0)
            # q: the rotated query heads inside the qkv rows: ne [hd, n, Hq], token stride = row, head stride = hd
            qv = _tensor_view(self.qkv, L.F32, [hd, n, Hq], [4, self.qkv.stride(0) * 4, hd * 4])
            # the mask's columns of the tokens attended to
            mv = _tensor_view(mask[:, t0 - start:], L.F16, [t1 - t0, mask.shape[0], 1], [2, mask.stride(0) * 2])
            self._keep += [kv, vv, kt2, vt2, qv, mv]
            sz = ctypes.c_size_t()
            if t1 > t0:
                L.check(lib.srhpm_flash_attn_ext_work_size(h, ctypes.byref(qv), ctypes.byref(kv), ctypes.byref(vv),
                                                           ctypes.byref(sz)), "srhpm_flash_attn_ext_work_size")
            self._ws = max(self._ws, sz.value)
            scale = ctypes.c_float(1.0 / math.sqrt(hd))
            if split:
                # the records of this part for every head of the KV head, merged over the replicas: att_all rows
                # [n][G * hd], of which this rank's heads feed its O columns
                tp = self.tp
                ova = _tensor_view(self.att_all, L.F32, [hd, Hq, n], [4, hd * 4, self.att_all.stride(0) * 4])
                self._keep.append(ova)
                calls.append(("flash_attn_ext_partial", lib.srhpm_flash_attn_ext_partial,
                              [h, ctypes.byref(qv), ctypes.byref(kv), ctypes.byref(vv), ctypes.byref(mv), scale,
                               ctypes.c_float(0.0), ctypes.c_float(0.0), self._ptr(tp.att_part)], True))
                calls.append(("flash_attn_merge_peers", lib.srhpm_flash_attn_merge_peers,
                              [h, self._ptr(tp.att_peers), self.w.tp["r"], self.w.tp["p"], self._ptr(tp.att_epochs),
                               None, ctypes.byref(ova)], False))
                o0 = (self.w.tp["h0"] - self.w.tp["gh0"]) * hd
                calls.append(self._mm(lay["o"], self.att_all[:, o0:o0 + H * hd], self._rowpar_out(0)))
            else:
                # dst [hd, H, n]: head stride hd, token stride H * hd -> att rows [n][H * hd]
                ov = _tensor_view(self.att, L.F32, [hd, H, n], [4, hd * 4, self.att.stride(0) * 4])
                self._keep.append(ov)
                calls.append(("flash_attn_ext", lib.srhpm_flash_attn_ext,
                              [h, ctypes.byref(qv), ctypes.byref(kv), ctypes.byref(vv), ctypes.byref(mv), None, scale,
                               ctypes.c_float(0.0), ctypes.c_float(0.0), ctypes.byref(ov)], True))
                calls.append(self._mm(lay["o"], self.att, self._rowpar_out(0)))
            if self.tp is not None and not self._fused():
                calls.append(self._all_reduce(self.o))  # row-parallel O: partial sums over the rank's heads
            if "gate_up" in lay:
                calls += self._norm_mm(0, lay["ffn_norm"], lay["gate_up"], self.gu)
            else:
                calls.append(self._norm(0, lay["ffn_norm"]))
                calls.append(self._mm(lay["gate"], self.y, self.gu[:, :self.n_ff]))
                calls.append(self._mm(lay["up"], self.y, self.gu[:, self.n_ff:]))
            up_ptr = ctypes.c_void_p(self.gu.data_ptr() + 4 * self.n_ff)
            # then the down GEMM: the delta added by the next norm (row-parallel: partial sums over the FFN rows)
            if self.fuse_prologue and lay["down"].qtype != L.Q8_0:
                Wd, Yd = lay["down"], self._rowpar_out(1)
                st, ws = self.ctx.mul_mat_work_size(Wd, self.h)
                L.check(st, "srhpm_mul_mat_work_size")
                self._ws = max(self._ws, ws)
                wv, xv, yv = Wd.view(), f32_rows_view(self.h), f32_rows_view(Yd)
                self._keep += [wv, xv, yv]
                if self.swiglu_in_gemm:
                    gv, uv = f32_rows_view(self.gu[:, :self.n_ff]), f32_rows_view(self.gu[:, self.n_ff:])
                    self._keep += [gv, uv]
                    calls.append(("mul_mat_swiglu", lib.srhpm_mul_mat_swiglu,
                                  [h, ctypes.byref(wv), ctypes.byref(gv), ctypes.byref(uv), ctypes.byref(yv)], True))
                else:
                    calls.append(("swiglu_quant", lib.srhpm_swiglu_quant,
                                  [h, self._ptr(self.gu), up_ptr, self.gu.stride(0), self._ptr(self.h),
                                   self.h.stride(0), n, ctypes.byref(wv)], True))
                    calls.append(("mul_mat_prequantized", lib.srhpm_mul_mat_prequantized,
                                  [h, ctypes.byref(wv), ctypes.byref(xv), ctypes.byref(yv)], True))
            else:
                calls.append(("swiglu", lib.srhpm_swiglu,
                              [h, self._ptr(self.gu), up_ptr, self.gu.stride(0), self._ptr(self.h), self.h.stride(0),
                               n, self.n_ff], False))
                calls.append(self._mm(lay["down"], self.h, self._rowpar_out(1)))
            if self.tp is not None and not self._fused():
                calls.append(self._all_reduce(self.o))
        calls += self._norm_mm(1, self.w.out_norm, self.w.head, self.logits)
        lv = f32_rows_view(self.logits)
        self._keep.append(lv)
        sz = ctypes.c_size_t()
        L.check(lib.srhpm_verify_accept_work_size(h, ctypes.byref(lv), ctypes.byref(sz)),
                "srhpm_verify_accept_work_size")
        self._ws = max(self._ws, sz.value)
        if self.tp is None:
            calls.append(("verify_accept", lib.srhpm_verify_accept,
                          [h, ctypes.byref(lv), self._ptr(self.draft), n - 1, ctypes.c_float(self.relax),
                           self._ptr(self.out_ids), self._ptr(self.out_n)], True))
        else:  # vocabulary-sharded head: per-row (max, first index, draft logit) records, gathered, merged on every rank
            calls.append(("argmax_shard", lib.srhpm_argmax_shard,
                          [h, ctypes.byref(lv), ctypes.c_int64(self.vocab_offset), self._ptr(self.draft), n - 1,
                           self._ptr(self.rec)], True))
            calls.append(("all_gather", _py_call(lambda: self.tp.all_gather(self.rec_all, self.rec)), [], False))
            calls.append(("accept_merge", lib.srhpm_accept_merge,
                          [h, self._ptr(self.rec_all), self.tp.world, n, self._ptr(self.draft), n - 1,
                           ctypes.c_float(self.relax), self._ptr(self.out_ids), self._ptr(self.out_n)], False))
        self.work = torch.empty(max(self._ws, 1 << 16), dtype=torch.uint8, device=self.w.device)
        wargs = [ctypes.c_void_p(self.work.data_ptr()), ctypes.c_size_t(self.work.numel())]
        self._calls = [(name, fn, args + wargs if with_work else args) for name, fn, args, with_work in calls]

    def _mask(self, full, start):
        c, n = self.cfg, self.n
        Lv = self.n_past + n - start
        m = torch.zeros((n, Lv), dtype=torch.float16, device=self.w.device)
        for t in range(n):
            p = self.n_past + t
            a = torch.arange(start, start + Lv, device=self.w.device)
            hide = a > p
            if not full:
                hide |= a <= p - c.window
            m[t][hide] = float("-inf")
        return m

    # -- running ------------------------------------------------------------------------------------------------------
    def launches(self):
        return len(self._calls)

    def run(self, stream=None):
        """Issue the whole step on `stream` (the current stream by default)."""
        st_obj = stream or torch.cuda.current_stream()
        s = ctypes.c_void_p(st_obj.cuda_stream)
        with torch.cuda.stream(st_obj):  # the collectives issue on torch's current stream
            for name, fn, args in self._calls:
                st = fn(*args, s)
                if st != L.OK:
                    raise L.SrhpmError(st, "srhpm_" + name, self.lib)

    def set_past(self, n_past):
        """Move the step to cache position n_past: new positions, masks and attention ranges, the same buffers. The
        prebuilt calls are rebuilt on the host; a CUDA graph captured before must be captured again."""
        cap = self.kcache[0].shape[0]
        if n_past < 0 or n_past + self.n > cap:
            raise ValueError(f"positions {n_past}..{n_past + self.n - 1} do not fit a cache of {cap} tokens")
        torch.cuda.synchronize(self.w.device)  # the previous calls may still read the masks about to be replaced
        self.n_past = n_past
        self.pos.copy_(torch.arange(n_past, n_past + self.n, dtype=torch.int32))
        self._keep = []
        self._build()

    def advance(self, n_emitted):
        """The next step of a decode loop: n_emitted = len(accepted()) of this step (its accepted drafted tokens + 1).
        The cache then holds valid rows up to n_past + n_emitted (this step's first token and the drafted tokens it
        accepted); the rows after them, written for rejected drafted tokens, are hidden by the causal mask and
        overwritten by the next step's KV store. That is the reference server's truncate-on-rollback
        (n_rollback = k + 1 - accepted, patch/srhpm.patch:7202) without a separate pass."""
        if not 1 <= n_emitted <= self.n:
            raise ValueError(f"a step of {self.n} tokens emits 1..{self.n} ids, not {n_emitted}")
        self.set_past(self.n_past + n_emitted)

    def set_tokens(self, ids, draft):
        """Inputs of the step: ids int [n] (accepted token + drafted tokens), draft int [n - 1]."""
        self.ids.copy_(torch.as_tensor(ids, dtype=torch.int32))
        if self.n > 1:
            self.draft.copy_(torch.as_tensor(draft, dtype=torch.int32))

    def accepted(self):
        n = int(self.out_n.item())
        return self.out_ids[:n].cpu().tolist()
