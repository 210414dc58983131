"""Host-side operator layer of the B200 verify path, shaped like the ggml operators it replaces.

    Context.mul_mat(W, X)          ggml_mul_mat(W, X) with ne[1] = N = 1..16 on a GGUF-quantized W
                                   (reference: tensor_traits_srv::compute_forward, patch/srhpm.patch:6400-6611)
    Context.flash_attn_ext(...)    ggml_flash_attn_ext with 1..16 query rows over an f16 / q8_0 KV cache
                                   (reference: ggml_compute_forward_flash_attn_ext_gqa_small, patch/srhpm.patch:581-824)
    Context.flash_attn_ext_partial / flash_attn_merge
                                   the same attention split over KV token ranges: one (max, sum, acc) record set per
                                   range, merged after a gather (reference: its chunk records and their merge,
                                   patch/srhpm.patch:779-823, with devices as the chunks)
    Context.sample_and_accept_n()  greedy longest-prefix acceptance (reference: common_sampler_sample_and_accept_n,
                                   patch/srhpm.patch:1-37)

Tensors are torch tensors in device memory; torch only provides allocation and streams. Every compute call goes to
libsrhpm_b200.so through its C ABI; a missing library raises.
"""
import ctypes
import warnings

import numpy as np
import torch

from . import _lib as L


def _tensor_view(t, type_, ne, nb):
    v = L.SrhpmTensor()
    v.type = type_
    for i in range(4):
        v.ne[i] = ne[i] if i < len(ne) else 1
    last = nb[-1] * (ne[len(nb) - 1] if len(nb) else 1)
    for i in range(4):
        v.nb[i] = nb[i] if i < len(nb) else last
    v.data = t.data_ptr() if t is not None else 0
    return v


def f32_rows_view(x):
    """ggml view of a 2-D f32 tensor [rows, cols] (cols innermost): ne = [cols, rows]."""
    assert x.dtype == torch.float32 and x.dim() == 2 and x.stride(1) == 1
    return _tensor_view(x, L.F32, [x.shape[1], x.shape[0]], [4, x.stride(0) * 4])


def _stream_ptr(stream):
    s = stream if stream is not None else torch.cuda.current_stream()
    return ctypes.c_void_p(s.cuda_stream)


def quantize_chunk(w, qtype):
    """Host weight quantizer: f32 [rows, K] (numpy or CPU torch) -> GGUF-packed bytes (numpy uint8, rows x row_size).
    ggml_quantize_chunk's contract (srhpm_quantize_chunk)."""
    lib = L.load()
    w = np.ascontiguousarray(np.asarray(w, dtype=np.float32))
    rows, K = w.shape
    rs = lib.srhpm_row_size(qtype, K)
    if rs == 0:
        raise ValueError(f"K={K} is not a multiple of the block size of {L.TYPE_NAMES.get(qtype, qtype)}")
    out = np.empty((rows, rs), dtype=np.uint8)
    n = lib.srhpm_quantize_chunk(qtype, w.ctypes.data, out.ctypes.data, 0, rows, K, None)
    if n != rows * rs:
        raise RuntimeError("srhpm_quantize_chunk failed")
    return out


def row_size(qtype, K):
    """Bytes of a row of K values of qtype (ggml_row_size)."""
    return int(L.load().srhpm_row_size(qtype, K))


def type_size(qtype):
    """Bytes of one block of qtype (ggml_type_size)."""
    return int(L.load().srhpm_type_size(qtype))


def blck_size(qtype):
    """Values per block of qtype (ggml_blck_size)."""
    return int(L.load().srhpm_blck_size(qtype))


class QuantTensor:
    """GGUF-packed weight rows in device memory: a ggml tensor of a quantized type with ne = [K, rows]."""

    def __init__(self, data, qtype, rows, K):
        lib = L.load()
        self.qtype, self.rows, self.K = qtype, rows, K
        self.row_bytes = lib.srhpm_row_size(qtype, K)
        if self.row_bytes == 0:
            raise ValueError("K is not a multiple of the block size")
        assert data.dtype == torch.uint8 and data.is_cuda and data.numel() >= rows * self.row_bytes
        self.data = data

    @classmethod
    def from_blocks(cls, blocks, qtype, rows, K, device="cuda"):
        # a read-only map of a GGUF file is fine here: the host tensor is only read by the copy to the device
        with warnings.catch_warnings():
            warnings.filterwarnings("ignore", message="The given NumPy array is not writable")
            t = torch.from_numpy(np.ascontiguousarray(blocks).reshape(-1)).to(device)
        return cls(t, qtype, rows, K)

    @classmethod
    def quantize(cls, w, qtype, device="cuda"):
        w = np.asarray(w, dtype=np.float32)
        return cls.from_blocks(quantize_chunk(w, qtype), qtype, w.shape[0], w.shape[1], device)

    def view(self):
        lib = L.load()
        return _tensor_view(self.data, self.qtype, [self.K, self.rows], [lib.srhpm_type_size(self.qtype),
                                                                         self.row_bytes])

    def row_slice(self, r0, r1):
        """Rows [r0, r1) as their own tensor (a view: the reference's CPU/GPU row split)."""
        sub = self.data[r0 * self.row_bytes:r1 * self.row_bytes]
        return QuantTensor(sub, self.qtype, r1 - r0, self.K)

    @property
    def nbytes(self):
        return self.rows * self.row_bytes


class Context:
    """srhpm_ctx of one device plus a cached work buffer."""

    def __init__(self, device=0):
        self.lib = L.load()
        self.device = torch.device("cuda", device) if isinstance(device, int) else torch.device(device)
        h = ctypes.c_void_p()
        L.check(self.lib.srhpm_ctx_create(self.device.index or 0, ctypes.byref(h)), "srhpm_ctx_create")
        self.handle = h
        self._work = None

    def close(self):
        if self.handle:
            self.lib.srhpm_ctx_destroy(self.handle)
            self.handle = None

    def __del__(self):
        try:
            self.close()
        except Exception:
            pass

    def set_q8_0_act_mode(self, mode):
        L.check(self.lib.srhpm_ctx_set_q8_0_act_mode(self.handle, mode), "set_q8_0_act_mode")

    def launch_count(self, reset=False):
        return int(self.lib.srhpm_ctx_launch_count(self.handle, 1 if reset else 0))

    def check(self):
        code = ctypes.c_int32(0)
        st = self.lib.srhpm_ctx_check(self.handle, ctypes.byref(code))
        if st != L.OK:
            raise L.SrhpmError(st, f"device status {code.value}", self.lib)

    def work(self, nbytes):
        if self._work is None or self._work.numel() < nbytes:
            self._work = torch.empty(max(nbytes, 1 << 16), dtype=torch.uint8, device=self.device)
        return self._work

    # ---- small-batch quantized matmul -------------------------------------------------------------------------
    def mul_mat_work_size(self, W, X):
        wv, xv = W.view(), f32_rows_view(X)
        sz = ctypes.c_size_t()
        st = self.lib.srhpm_mul_mat_work_size(ctypes.byref(wv), ctypes.byref(xv), ctypes.byref(sz))
        return st, sz.value

    def mul_mat(self, W, X, out=None, stream=None, work=None, fused_quant=False):
        """Y[N, rows] = X[N, K] . W[rows, K]^T (ggml_mul_mat(W, X): dst ne = [rows, N]). fused_quant: one launch, the
        matmul grid quantizes its own activations (srhpm_mul_mat_fused_quant; bit-identical output)."""
        X = X if X.stride(-1) == 1 else X.contiguous()
        N = X.shape[0]
        if out is None:
            out = torch.empty((N, W.rows), dtype=torch.float32, device=X.device)
        wv, xv, yv = W.view(), f32_rows_view(X), f32_rows_view(out)
        st, ws = self.mul_mat_work_size(W, X)
        L.check(st, "srhpm_mul_mat_work_size")
        buf = work if work is not None else self.work(ws)
        fn = self.lib.srhpm_mul_mat_fused_quant if fused_quant else self.lib.srhpm_mul_mat
        L.check(fn(self.handle, ctypes.byref(wv), ctypes.byref(xv), ctypes.byref(yv), ctypes.c_void_p(buf.data_ptr()),
                   buf.numel(), _stream_ptr(stream)), "srhpm_mul_mat")
        return out

    def mul_mat_swiglu(self, W, gate, up, out=None, stream=None, work=None):
        """Y[N, rows] = (silu(gate) * up)[N, K] . W[rows, K]^T with the SwiGLU in the matmul grid's own prologue
        (srhpm_mul_mat_swiglu; gate and up of the same shape and row stride, e.g. the two halves of a gate|up
        product)."""
        N = gate.shape[0]
        if out is None:
            out = torch.empty((N, W.rows), dtype=torch.float32, device=gate.device)
        wv, gv, uv, yv = W.view(), f32_rows_view(gate), f32_rows_view(up), f32_rows_view(out)
        st, ws = self.mul_mat_work_size(W, gate)
        L.check(st, "srhpm_mul_mat_work_size")
        buf = work if work is not None else self.work(ws)
        L.check(self.lib.srhpm_mul_mat_swiglu(self.handle, ctypes.byref(wv), ctypes.byref(gv), ctypes.byref(uv),
                                              ctypes.byref(yv), ctypes.c_void_p(buf.data_ptr()), buf.numel(),
                                              _stream_ptr(stream)), "srhpm_mul_mat_swiglu")
        return out

    def prepare_mul_mat(self, W, X, Y, work, fused_quant=False):
        """A zero-argument callable that issues srhpm_mul_mat(W, X) -> Y on the current stream with prebuilt
        arguments (the per-call host cost is one ctypes call); usable under CUDA-graph capture, since the call
        allocates nothing."""
        wv, xv, yv = W.view(), f32_rows_view(X), f32_rows_view(Y)
        st, ws = self.mul_mat_work_size(W, X)
        L.check(st, "srhpm_mul_mat_work_size")
        if work.numel() < ws:
            raise ValueError("work buffer too small")
        fn, lib = (self.lib.srhpm_mul_mat_fused_quant if fused_quant else self.lib.srhpm_mul_mat), self.lib
        args = [self.handle, ctypes.byref(wv), ctypes.byref(xv), ctypes.byref(yv), ctypes.c_void_p(work.data_ptr()),
                work.numel()]
        keep = (wv, xv, yv, W, X, Y, work)

        def run():
            st = fn(*args, ctypes.c_void_p(torch.cuda.current_stream().cuda_stream))
            if st != L.OK:
                raise L.SrhpmError(st, "srhpm_mul_mat", lib)

        run.keep = keep
        return run

    def mul_mat_isums(self, W, X, stream=None):
        """Integer block sums of the matmul: isum, imin int32 [N, rows, nblk] (imin only for Q4_K / Q5_K)."""
        X = X.contiguous()
        N = X.shape[0]
        nblk = W.K // (32 if W.qtype == L.Q8_0 else 256)
        isum = torch.zeros((N, W.rows, nblk), dtype=torch.int32, device=X.device)
        imin = torch.zeros_like(isum)
        wv, xv = W.view(), f32_rows_view(X)
        st, ws = self.mul_mat_work_size(W, X)
        L.check(st, "srhpm_mul_mat_work_size")
        buf = self.work(ws)
        L.check(self.lib.srhpm_mul_mat_isums(self.handle, ctypes.byref(wv), ctypes.byref(xv),
                                             ctypes.c_void_p(isum.data_ptr()), ctypes.c_void_p(imin.data_ptr()),
                                             ctypes.c_void_p(buf.data_ptr()), buf.numel(), _stream_ptr(stream)),
                "srhpm_mul_mat_isums")
        return isum, imin

    # ---- multi-query attention (ggml_flash_attn_ext) -------------------------------------------------------------
    @staticmethod
    def _fa_views(q, k, v, kv_type, mask, sinks, out):
        """ggml views: q f32 [H, N, D] -> ne [D, N, H]; k / v uint8 [Hkv, L, row bytes] (any strides, rows
        contiguous) -> ne [D, L, Hkv]; mask f16 [N', L'] or [ne2, N', L'] -> ne [L', N', ne2]; sinks f32 [H];
        out f32 [N, H, DV] -> ne [DV, H, N]."""
        assert q.dtype == torch.float32 and q.dim() == 3 and q.stride(2) == 1
        H, N, D = q.shape
        tsz, blk = (34, 32) if kv_type == L.Q8_0 else (2, 1)
        views = [_tensor_view(q, L.F32, [D, N, H], [4, q.stride(1) * 4, q.stride(0) * 4])]
        for t in (k, v):
            assert t.dtype == torch.uint8 and t.dim() == 3 and t.stride(2) == 1
            Hkv, Lk, rowb = t.shape
            views.append(_tensor_view(t, kv_type, [rowb // tsz * blk, Lk, Hkv], [tsz, t.stride(1), t.stride(0)]))
        mv = None
        if mask is not None:
            assert mask.dtype == torch.float16 and mask.stride(-1) == 1
            m3 = mask if mask.dim() == 3 else mask.unsqueeze(0)
            mv = _tensor_view(m3, L.F16, [m3.shape[2], m3.shape[1], m3.shape[0]], [2, m3.stride(1) * 2, m3.stride(0) * 2])
        sv = None
        if sinks is not None:
            assert sinks.dtype == torch.float32 and sinks.dim() == 1 and sinks.stride(0) == 1
            sv = _tensor_view(sinks, L.F32, [sinks.shape[0]], [4])
        ov = None
        if out is not None:
            Nn, Hh, DV = out.shape
            ov = _tensor_view(out, L.F32, [DV, Hh, Nn], [4, out.stride(1) * 4, out.stride(0) * 4])
        return views[0], views[1], views[2], mv, sv, ov

    def flash_attn_ext_work_size(self, q, k, v, kv_type):
        qv, kvv, vv, _, _, _ = self._fa_views(q, k, v, kv_type, None, None, None)
        sz = ctypes.c_size_t()
        st = self.lib.srhpm_flash_attn_ext_work_size(self.handle, ctypes.byref(qv), ctypes.byref(kvv),
                                                     ctypes.byref(vv), ctypes.byref(sz))
        return st, sz.value

    def flash_attn_ext(self, q, k, v, kv_type, mask=None, sinks=None, scale=1.0, max_bias=0.0, softcap=0.0,
                       out=None, stream=None, work=None):
        """ggml_flash_attn_ext(q, k, v, mask, scale, max_bias, softcap) + sinks: out f32 [N, H, DV]."""
        H, N, D = q.shape
        DV = v.shape[2] // 34 * 32 if kv_type == L.Q8_0 else v.shape[2] // 2
        if out is None:
            out = torch.empty((N, H, DV), dtype=torch.float32, device=q.device)
        qv, kvv, vv, mv, sv, ov = self._fa_views(q, k, v, kv_type, mask, sinks, out)
        st, ws = self.flash_attn_ext_work_size(q, k, v, kv_type)
        L.check(st, "srhpm_flash_attn_ext_work_size")
        buf = work if work is not None else self.work(ws)
        L.check(self.lib.srhpm_flash_attn_ext(self.handle, ctypes.byref(qv), ctypes.byref(kvv), ctypes.byref(vv),
                                              ctypes.byref(mv) if mv is not None else None,
                                              ctypes.byref(sv) if sv is not None else None, scale, max_bias, softcap,
                                              ctypes.byref(ov), ctypes.c_void_p(buf.data_ptr()), buf.numel(),
                                              _stream_ptr(stream)), "srhpm_flash_attn_ext")
        return out

    # ---- attention split over the KV range across devices ------------------------------------------------------
    def flash_attn_part_size(self, H, N):
        """Bytes of one record set of srhpm_flash_attn_ext_partial for H heads and N query tokens."""
        return int(self.lib.srhpm_flash_attn_part_size(H, N))

    def flash_attn_ext_partial(self, q, k, v, kv_type, mask=None, scale=1.0, max_bias=0.0, softcap=0.0, out=None,
                               stream=None, work=None):
        """The record set of this KV range (k / v uint8 [Hkv, range tokens, row bytes], mask f16 [N', range tokens]
        or [ne2, N', range tokens]; a range of 0 tokens is allowed): uint8 [flash_attn_part_size(H, N)] on the
        device, for flash_attn_merge."""
        H, N, D = q.shape
        nbytes = self.flash_attn_part_size(H, N)
        if out is None:
            out = torch.empty(nbytes, dtype=torch.uint8, device=q.device)
        assert out.dtype == torch.uint8 and out.numel() >= nbytes and out.data_ptr() % 16 == 0
        qv, kvv, vv, mv, _, _ = self._fa_views(q, k, v, kv_type, mask, None, None)
        ws = 0
        if k.shape[1] > 0:
            st, ws = self.flash_attn_ext_work_size(q, k, v, kv_type)
            L.check(st, "srhpm_flash_attn_ext_work_size")
        buf = work if work is not None else self.work(ws)
        L.check(self.lib.srhpm_flash_attn_ext_partial(self.handle, ctypes.byref(qv), ctypes.byref(kvv),
                                                      ctypes.byref(vv), ctypes.byref(mv) if mv is not None else None,
                                                      scale, max_bias, softcap, ctypes.c_void_p(out.data_ptr()),
                                                      ctypes.c_void_p(buf.data_ptr()), buf.numel(),
                                                      _stream_ptr(stream)), "srhpm_flash_attn_ext_partial")
        return out

    def flash_attn_merge(self, parts, n_parts, H, N, sinks=None, out=None, stream=None):
        """Merge n_parts record sets stored one after another in `parts` (uint8, e.g. gathered from all devices in
        KV order), add the sinks and normalize: out f32 [N, H, 256], as flash_attn_ext over the whole range."""
        assert parts.dtype == torch.uint8 and parts.is_contiguous()
        assert parts.numel() >= n_parts * self.flash_attn_part_size(H, N)
        if out is None:
            out = torch.empty((N, H, 256), dtype=torch.float32, device=parts.device)
        ov = _tensor_view(out, L.F32, [out.shape[2], out.shape[1], out.shape[0]],
                          [4, out.stride(1) * 4, out.stride(0) * 4])
        sv = None
        if sinks is not None:
            assert sinks.dtype == torch.float32 and sinks.dim() == 1 and sinks.stride(0) == 1
            sv = _tensor_view(sinks, L.F32, [sinks.shape[0]], [4])
        L.check(self.lib.srhpm_flash_attn_merge(self.handle, ctypes.c_void_p(parts.data_ptr()), n_parts,
                                                ctypes.byref(sv) if sv is not None else None, ctypes.byref(ov),
                                                _stream_ptr(stream)), "srhpm_flash_attn_merge")
        return out

    def flash_attn_peer_buffer_size(self, H, N):
        """Bytes of one rank's buffer for flash_attn_merge_peers: the record set, then its receive area."""
        return int(self.lib.srhpm_flash_attn_peer_buffer_size(H, N))

    def flash_attn_merge_peers(self, peers, world, rank, epochs, H, N, sinks=None, out=None, stream=None):
        """srhpm_flash_attn_merge_peers: every rank's record set at the start of its own peer buffer (peers: int64
        device tensor of the world buffers' addresses on this device), exchanged as (value, epoch) words and merged in
        rank order; epochs: int32 [H * N] device counters, zero at the start. Returns out f32 [N, H, 256]."""
        if out is None:
            out = torch.empty((N, H, 256), dtype=torch.float32, device=peers.device)
        ov = _tensor_view(out, L.F32, [out.shape[2], out.shape[1], out.shape[0]],
                          [4, out.stride(1) * 4, out.stride(0) * 4])
        sv = None
        if sinks is not None:
            assert sinks.dtype == torch.float32 and sinks.dim() == 1 and sinks.stride(0) == 1
            sv = _tensor_view(sinks, L.F32, [sinks.shape[0]], [4])
        assert epochs.numel() >= H * N
        L.check(self.lib.srhpm_flash_attn_merge_peers(self.handle, ctypes.c_void_p(peers.data_ptr()), world, rank,
                                                      ctypes.c_void_p(epochs.data_ptr()),
                                                      ctypes.byref(sv) if sv is not None else None, ctypes.byref(ov),
                                                      _stream_ptr(stream)), "srhpm_flash_attn_merge_peers")
        return out

    # ---- greedy acceptance ------------------------------------------------------------------------------------------
    def sample_and_accept_n(self, logits, draft, relax=0.0, stream=None, work=None):
        """common_sampler_sample_and_accept_n (greedy): logits f32 [>= n_draft + 1, n_vocab] (rows = positions),
        draft int32 [n_draft] on the device -> (ids int32 [n_draft + 1], n int32 [1]) on the device; the emitted ids
        are ids[:n]."""
        assert logits.dtype == torch.float32 and logits.dim() == 2 and logits.stride(1) == 1
        n_draft = int(draft.numel())
        lv = _tensor_view(logits, L.F32, [logits.shape[1], logits.shape[0]], [4, logits.stride(0) * 4])
        sz = ctypes.c_size_t()
        L.check(self.lib.srhpm_verify_accept_work_size(self.handle, ctypes.byref(lv), ctypes.byref(sz)),
                "srhpm_verify_accept_work_size")
        buf = work if work is not None else self.work(sz.value)
        ids = torch.empty(n_draft + 1, dtype=torch.int32, device=logits.device)
        n = torch.empty(1, dtype=torch.int32, device=logits.device)
        d = draft.to(torch.int32).contiguous() if n_draft else None
        L.check(self.lib.srhpm_verify_accept(self.handle, ctypes.byref(lv),
                                             ctypes.c_void_p(d.data_ptr()) if d is not None else None, n_draft,
                                             relax, ctypes.c_void_p(ids.data_ptr()), ctypes.c_void_p(n.data_ptr()),
                                             ctypes.c_void_p(buf.data_ptr()), buf.numel(), _stream_ptr(stream)),
                "srhpm_verify_accept")
        return ids, n

    def argmax_shard(self, logits, vocab_offset, draft=None, stream=None, work=None):
        """Per-row record of a vocabulary shard: uint8 [rows, 16] (srhpm_argmax_record) on the device."""
        assert logits.dtype == torch.float32 and logits.dim() == 2 and logits.stride(1) == 1
        rows = logits.shape[0]
        lv = _tensor_view(logits, L.F32, [logits.shape[1], rows], [4, logits.stride(0) * 4])
        sz = ctypes.c_size_t()
        L.check(self.lib.srhpm_verify_accept_work_size(self.handle, ctypes.byref(lv), ctypes.byref(sz)),
                "srhpm_verify_accept_work_size")
        buf = work if work is not None else self.work(sz.value)
        rec = torch.empty((rows, 16), dtype=torch.uint8, device=logits.device)
        n_draft = int(draft.numel()) if draft is not None else 0
        d = draft.to(torch.int32).contiguous() if n_draft else None
        L.check(self.lib.srhpm_argmax_shard(self.handle, ctypes.byref(lv), vocab_offset,
                                            ctypes.c_void_p(d.data_ptr()) if d is not None else None, n_draft,
                                            ctypes.c_void_p(rec.data_ptr()), ctypes.c_void_p(buf.data_ptr()),
                                            buf.numel(), _stream_ptr(stream)), "srhpm_argmax_shard")
        return rec

    def accept_merge(self, recs, draft, relax=0.0, stream=None):
        """recs uint8 [n_shards, rows, 16] (argmax_shard outputs in vocabulary order) -> (ids, n) as
        sample_and_accept_n."""
        recs = recs.contiguous()
        n_shards, rows = recs.shape[0], recs.shape[1]
        n_draft = int(draft.numel())
        ids = torch.empty(n_draft + 1, dtype=torch.int32, device=recs.device)
        n = torch.empty(1, dtype=torch.int32, device=recs.device)
        d = draft.to(torch.int32).contiguous() if n_draft else None
        L.check(self.lib.srhpm_accept_merge(self.handle, ctypes.c_void_p(recs.data_ptr()), n_shards, rows,
                                            ctypes.c_void_p(d.data_ptr()) if d is not None else None, n_draft, relax,
                                            ctypes.c_void_p(ids.data_ptr()), ctypes.c_void_p(n.data_ptr()),
                                            _stream_ptr(stream)), "srhpm_accept_merge")
        return ids, n

    def quantize_rows_q8_K(self, X, stream=None):
        X = X.contiguous()
        N, K = X.shape
        q = torch.empty((N, K), dtype=torch.int8, device=X.device)
        d = torch.empty((N, K // 256), dtype=torch.float32, device=X.device)
        b32 = torch.empty((N, K // 32), dtype=torch.int16, device=X.device)
        b16 = torch.empty((N, K // 16), dtype=torch.int16, device=X.device)
        xv = f32_rows_view(X)
        L.check(self.lib.srhpm_quantize_rows_q8_K(self.handle, ctypes.byref(xv), ctypes.c_void_p(q.data_ptr()),
                                                  ctypes.c_void_p(d.data_ptr()), ctypes.c_void_p(b32.data_ptr()),
                                                  ctypes.c_void_p(b16.data_ptr()), _stream_ptr(stream)),
                "srhpm_quantize_rows_q8_K")
        return q, d, b32, b16

    def quantize_rows_q8_0(self, X, stream=None):
        X = X.contiguous()
        N, K = X.shape
        out = torch.empty((N, (K // 32) * 34), dtype=torch.uint8, device=X.device)
        xv = f32_rows_view(X)
        L.check(self.lib.srhpm_quantize_rows_q8_0(self.handle, ctypes.byref(xv), ctypes.c_void_p(out.data_ptr()),
                                                  _stream_ptr(stream)), "srhpm_quantize_rows_q8_0")
        return out
