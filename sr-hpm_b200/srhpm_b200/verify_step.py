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
    """Architecture of the synthetic decoder (defaults: the BASELINE 27B-class model)."""

    def __init__(self, n_layer=64, d=5120, n_ff=17408, H=24, Hkv=4, hd=256, n_vocab=151936, base=1e6, eps=1e-6,
                 window=4096, full_every=4, kv_type=L.F16, types=None):
        self.n_layer, self.d, self.n_ff, self.H, self.Hkv, self.hd = n_layer, d, n_ff, H, Hkv, hd
        self.n_vocab, self.base, self.eps, self.window, self.full_every = n_vocab, base, eps, window, full_every
        self.kv_type = kv_type
        self.types = types or {"qkv": L.Q4_K, "o": L.Q4_K, "gate": L.Q3_K, "up": L.Q3_K, "down": L.Q4_K,
                               "head": L.Q6_K}

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
    """The decoder's weights in device memory."""

    def __init__(self, cfg, device):
        self.cfg, self.device = cfg, device
        self.layers = []
        self.out_norm = self.head = self.emb = None

    @classmethod
    def from_host(cls, cfg, w, device="cuda"):
        self = cls(cfg, device)
        for l in range(cfg.n_layer):
            lay = {}
            for name, t, rows, K in cfg.shapes():
                if name not in ("gate", "up"):
                    lay[name] = QuantTensor.from_blocks(w[name][l], t, rows, K, device)
            # gate and up as one matrix (gate rows, then up rows): one GEMM launch, SwiGLU reads the halves
            gu = np.concatenate([np.asarray(w["gate"][l]).reshape(cfg.n_ff, -1),
                                 np.asarray(w["up"][l]).reshape(cfg.n_ff, -1)])
            lay["gate_up"] = QuantTensor.from_blocks(gu, cfg.types["gate"], 2 * cfg.n_ff, cfg.d, device)
            lay["attn_norm"] = torch.from_numpy(w["attn_norm"][l]).to(device)
            lay["ffn_norm"] = torch.from_numpy(w["ffn_norm"][l]).to(device)
            self.layers.append(lay)
        self.out_norm = torch.from_numpy(w["out_norm"]).to(device)
        self.head = QuantTensor.from_blocks(w["head"], cfg.types["head"], cfg.n_vocab, cfg.d, device)
        self.emb = torch.from_numpy(w["emb"]).to(device)
        return self

    @classmethod
    def random(cls, cfg, device="cuda", seed=0):
        self = cls(cfg, device)
        gen = torch.Generator(device=device)
        gen.manual_seed(seed)
        for _ in range(cfg.n_layer):
            lay = {name: random_blocks_device(t, rows, K, gen, device) for name, t, rows, K in cfg.shapes()
                   if name not in ("gate", "up")}
            lay["gate_up"] = random_blocks_device(cfg.types["gate"], 2 * cfg.n_ff, cfg.d, gen, device)
            lay["attn_norm"] = 1.0 + 0.1 * torch.randn(cfg.d, device=device, generator=gen)
            lay["ffn_norm"] = 1.0 + 0.1 * torch.randn(cfg.d, device=device, generator=gen)
            self.layers.append(lay)
        self.out_norm = 1.0 + 0.1 * torch.randn(cfg.d, device=device, generator=gen)
        self.head = random_blocks_device(cfg.types["head"], cfg.n_vocab, cfg.d, gen, device)
        self.emb = torch.randn((cfg.n_vocab, cfg.d), device=device, generator=gen).half()
        return self


class VerifyStep:
    """One verify step of n tokens (1 accepted + k drafted) at cache position n_past, with prebuilt C-ABI calls.

    kcache / vcache: per layer uint8 [capacity, Hkv, row bytes] (f16 or q8_0 rows), the llama.cpp cache layout."""

    def __init__(self, ctx, cfg, weights, kcache, vcache, n_tokens, n_past, relax=0.0):
        self.ctx, self.cfg, self.w = ctx, cfg, weights
        self.kcache, self.vcache = kcache, vcache
        self.n, self.n_past, self.relax = n_tokens, n_past, relax
        dev = weights.device
        c, n = cfg, n_tokens
        f32 = dict(dtype=torch.float32, device=dev)
        self.ids = torch.zeros(n, dtype=torch.int32, device=dev)         # input: accepted token + drafted tokens
        self.draft = torch.zeros(max(n - 1, 1), dtype=torch.int32, device=dev)
        self.pos = torch.arange(n_past, n_past + n, dtype=torch.int32, device=dev)
        self.x = torch.zeros((n, c.d), **f32)                              # residual stream
        self.y = torch.zeros((n, c.d), **f32)                              # normed input of a block
        self.qkv = torch.zeros((n, (c.H + 2 * c.Hkv) * c.hd), **f32)
        self.att = torch.zeros((n, c.H * c.hd), **f32)
        self.o = torch.zeros((n, c.d), **f32)
        self.gu = torch.zeros((n, 2 * c.n_ff), **f32)                      # gate | up
        self.h = torch.zeros((n, c.n_ff), **f32)
        self.logits = torch.zeros((n, c.n_vocab), **f32)
        self.out_ids = torch.zeros(n, dtype=torch.int32, device=dev)
        self.out_n = torch.zeros(1, dtype=torch.int32, device=dev)
        self.lib = L.load()
        self._keep = []
        self._calls = []
        self._build()

    # -- argument building -------------------------------------------------------------------------------------------
    def _ptr(self, t):
        return ctypes.c_void_p(t.data_ptr())

    def _mm(self, W, X, Y):
        st, ws = self.ctx.mul_mat_work_size(W, X)
        L.check(st, "srhpm_mul_mat_work_size")
        self._ws = max(self._ws, ws)
        wv, xv, yv = W.view(), f32_rows_view(X), f32_rows_view(Y)
        self._keep += [wv, xv, yv]
        fn = self.lib.srhpm_mul_mat
        return ("mul_mat", fn, [self.ctx.handle, ctypes.byref(wv), ctypes.byref(xv), ctypes.byref(yv)], True)

    def _cache_view(self, cache, start, length):
        c = self.cfg
        t = cache[start:start + length]
        tsz = 34 if c.kv_type == L.Q8_0 else 2
        blk = 32 if c.kv_type == L.Q8_0 else 1
        # cache [cap, Hkv, row] -> ggml view [hd, length, Hkv] (token stride = stride(0), head stride = stride(1))
        return _tensor_view(t, c.kv_type, [c.hd, length, c.Hkv], [tsz, t.stride(0), t.stride(1)]), t

    def _build(self):
        c, n, lib, h = self.cfg, self.n, self.lib, self.ctx.handle
        self._ws = 0
        calls = []
        # embeddings
        emb_v = _tensor_view(self.w.emb, L.F16, [c.d, c.n_vocab], [2, self.w.emb.stride(0) * 2])
        self._keep.append(emb_v)
        calls.append(("get_rows", lib.srhpm_get_rows,
                      [h, ctypes.byref(emb_v), self._ptr(self.ids), n, self._ptr(self.x)], False))
        L_all = self.n_past + n
        masks = {}
        for li, lay in enumerate(self.w.layers):
            first = li == 0
            calls.append(("add_rms_norm", lib.srhpm_add_rms_norm,
                          [h, self._ptr(self.x), None if first else self._ptr(self.o), self._ptr(lay["attn_norm"]),
                           ctypes.c_float(c.eps), self._ptr(self.y), n, c.d], False))
            calls.append(self._mm(lay["qkv"], self.y, self.qkv))
            kv_full, kt = self._cache_view(self.kcache[li], 0, self.kcache[li].shape[0])
            vv_full, vt = self._cache_view(self.vcache[li], 0, self.vcache[li].shape[0])
            self._keep += [kv_full, vv_full, kt, vt]
            calls.append(("rope_kv", lib.srhpm_rope_kv,
                          [h, self._ptr(self.qkv), self.qkv.stride(0), n, c.H, c.Hkv, c.hd, self._ptr(self.pos),
                           ctypes.c_float(c.base), ctypes.byref(kv_full), ctypes.byref(vv_full)], False))
            # attention over the visible keys (sliding-window layers: the last `window` positions)
            full = c.window <= 0 or li % c.full_every == c.full_every - 1
            start = 0 if full else max(0, self.n_past - c.window + 1)
            if (full, start) not in masks:
                masks[(full, start)] = self._mask(full, start)
                self._keep.append(masks[(full, start)])  # the C calls hold raw pointers into it
            mask = masks[(full, start)]
            kv, kt2 = self._cache_view(self.kcache[li], start, L_all - start)
            vv, vt2 = self._cache_view(self.vcache[li], start, L_all - start)
            # q: the rotated query heads inside the qkv rows: ne [hd, n, H], token stride = row, head stride = hd
            qv = _tensor_view(self.qkv, L.F32, [c.hd, n, c.H], [4, self.qkv.stride(0) * 4, c.hd * 4])
            # dst [hd, H, n]: head stride hd, token stride H * hd -> att rows [n][H * hd]
            ov = _tensor_view(self.att, L.F32, [c.hd, c.H, n], [4, c.hd * 4, self.att.stride(0) * 4])
            mv = _tensor_view(mask, L.F16, [mask.shape[1], mask.shape[0], 1], [2, mask.stride(0) * 2])
            self._keep += [kv, vv, kt2, vt2, qv, ov, mv]
            sz = ctypes.c_size_t()
            L.check(lib.srhpm_flash_attn_ext_work_size(h, ctypes.byref(qv), ctypes.byref(kv), ctypes.byref(vv),
                                                       ctypes.byref(sz)), "srhpm_flash_attn_ext_work_size")
            self._ws = max(self._ws, sz.value)
            calls.append(("flash_attn_ext", lib.srhpm_flash_attn_ext,
                          [h, ctypes.byref(qv), ctypes.byref(kv), ctypes.byref(vv), ctypes.byref(mv), None,
                           ctypes.c_float(1.0 / math.sqrt(c.hd)), ctypes.c_float(0.0), ctypes.c_float(0.0),
                           ctypes.byref(ov)], True))
            calls.append(self._mm(lay["o"], self.att, self.o))
            calls.append(("add_rms_norm", lib.srhpm_add_rms_norm,
                          [h, self._ptr(self.x), self._ptr(self.o), self._ptr(lay["ffn_norm"]), ctypes.c_float(c.eps),
                           self._ptr(self.y), n, c.d], False))
            calls.append(self._mm(lay["gate_up"], self.y, self.gu))
            up_ptr = ctypes.c_void_p(self.gu.data_ptr() + 4 * c.n_ff)
            calls.append(("swiglu", lib.srhpm_swiglu,
                          [h, self._ptr(self.gu), up_ptr, self.gu.stride(0), self._ptr(self.h), self.h.stride(0), n,
                           c.n_ff], False))
            calls.append(self._mm(lay["down"], self.h, self.o))  # o: the delta added by the next add_rms_norm
        calls.append(("add_rms_norm", lib.srhpm_add_rms_norm,
                      [h, self._ptr(self.x), self._ptr(self.o), self._ptr(self.w.out_norm), ctypes.c_float(c.eps),
                       self._ptr(self.y), n, c.d], False))
        calls.append(self._mm(self.w.head, self.y, self.logits))
        lv = f32_rows_view(self.logits)
        self._keep.append(lv)
        sz = ctypes.c_size_t()
        L.check(lib.srhpm_verify_accept_work_size(h, ctypes.byref(lv), ctypes.byref(sz)),
                "srhpm_verify_accept_work_size")
        self._ws = max(self._ws, sz.value)
        calls.append(("verify_accept", lib.srhpm_verify_accept,
                      [h, ctypes.byref(lv), self._ptr(self.draft), n - 1, ctypes.c_float(self.relax),
                       self._ptr(self.out_ids), self._ptr(self.out_n)], True))
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
        s = ctypes.c_void_p((stream or torch.cuda.current_stream()).cuda_stream)
        for name, fn, args in self._calls:
            st = fn(*args, s)
            if st != L.OK:
                raise L.SrhpmError(st, "srhpm_" + name, self.lib)

    def set_tokens(self, ids, draft):
        """Inputs of the step: ids int [n] (accepted token + drafted tokens), draft int [n - 1]."""
        self.ids.copy_(torch.as_tensor(ids, dtype=torch.int32))
        if self.n > 1:
            self.draft.copy_(torch.as_tensor(draft, dtype=torch.int32))

    def accepted(self):
        n = int(self.out_n.item())
        return self.out_ids[:n].cpu().tolist()
