"""GGUF model files -> the verify path's device weights.

The reference leaves this to llama.cpp:
- its launcher reads the metadata with gguf-py's GGUFReader (srhpm/launch.py:45-65);
- llama.cpp uploads the packed blocks unchanged (the SRV buffer type's repack is a memcpy,
  patch/srhpm.patch:6613-6621).

This module does the same for a dense GQA decoder: it reads the file, keeps every quantized matrix in its native
GGUF block layout, and optionally cuts one tensor-parallel rank's slices at load time.

File layout (GGUF v2/v3, little endian):
- magic "GGUF", u32 version, u64 tensor count, u64 key-value count;
- the key-value pairs: string key, u32 value type, value;
- the tensor infos: string name, u32 n_dims, u64 ne[n_dims], u32 ggml type, u64 offset;
- then the data section, starting at the next multiple of `general.alignment` (default 32);
- each tensor at data start + its offset.

A string is a u64 length followed by the bytes.
"""
import mmap
import struct

import numpy as np
import torch

from . import _lib as L

# ggml type -> (values per block, bytes per block)
GGML_BLOCKS = {
    0: (1, 4),      # F32
    1: (1, 2),      # F16
    2: (32, 18),    # Q4_0
    3: (32, 20),    # Q4_1
    6: (32, 22),    # Q5_0
    7: (32, 24),    # Q5_1
    8: (32, 34),    # Q8_0
    9: (32, 36),    # Q8_1
    10: (256, 84),  # Q2_K
    11: (256, 110),  # Q3_K
    12: (256, 144),  # Q4_K
    13: (256, 176),  # Q5_K
    14: (256, 210),  # Q6_K
    15: (256, 292),  # Q8_K
    23: (256, 136),  # IQ4_XS
    30: (1, 2),     # BF16
}

_SCALARS = {0: "<B", 1: "<b", 2: "<H", 3: "<h", 4: "<I", 5: "<i", 6: "<f", 7: "<?", 10: "<Q", 11: "<q", 12: "<d"}


class TensorInfo:
    def __init__(self, name, ne, ggml_type, offset):
        self.name, self.ne, self.type, self.offset = name, list(ne), ggml_type, offset
        blk, bpb = GGML_BLOCKS.get(ggml_type, (0, 0))
        if blk == 0 or ne[0] % blk:
            self.row_bytes = None
            self.nbytes = None
        else:
            self.row_bytes = ne[0] // blk * bpb
            self.nbytes = self.row_bytes * int(np.prod(ne[1:], dtype=np.int64))

    @property
    def rows(self):
        return int(np.prod(self.ne[1:], dtype=np.int64))


class GGUFFile:
    """A parsed GGUF file: `kv` (metadata), `tensors` (name -> TensorInfo); tensor bytes are read through a read-only
    memory map."""

    def __init__(self, path):
        self.path = path
        self._f = open(path, "rb")
        self._mm = mmap.mmap(self._f.fileno(), 0, access=mmap.ACCESS_READ)
        self._pos = 0
        if self._read(4) != b"GGUF":
            raise ValueError(f"{path}: not a GGUF file")
        self.version = self._scalar("<I")
        if self.version not in (2, 3):
            raise ValueError(f"{path}: GGUF version {self.version} is not supported (2, 3)")
        n_tensors, n_kv = self._scalar("<Q"), self._scalar("<Q")
        self.kv = {}
        for _ in range(n_kv):
            key = self._string()
            self.kv[key] = self._value(self._scalar("<I"))
        self.tensors = {}
        for _ in range(n_tensors):
            name = self._string()
            n_dims = self._scalar("<I")
            ne = [self._scalar("<Q") for _ in range(n_dims)]
            ggml_type = self._scalar("<I")
            offset = self._scalar("<Q")
            self.tensors[name] = TensorInfo(name, ne, ggml_type, offset)
        align = int(self.kv.get("general.alignment", 32))
        self.data_start = (self._pos + align - 1) // align * align

    # -- parsing -----------------------------------------------------------------------------------------------------
    def _read(self, n):
        b = self._mm[self._pos:self._pos + n]
        if len(b) != n:
            raise ValueError(f"{self.path}: truncated")
        self._pos += n
        return b

    def _scalar(self, fmt):
        return struct.unpack(fmt, self._read(struct.calcsize(fmt)))[0]

    def _string(self):
        return self._read(self._scalar("<Q")).decode("utf-8")

    def _value(self, vt):
        if vt in _SCALARS:
            return self._scalar(_SCALARS[vt])
        if vt == 8:
            return self._string()
        if vt == 9:
            et, count = self._scalar("<I"), self._scalar("<Q")
            return [self._value(et) for _ in range(count)]
        raise ValueError(f"{self.path}: unknown metadata value type {vt}")

    # -- data --------------------------------------------------------------------------------------------------------
    def data(self, name):
        """The tensor's bytes: numpy uint8 [rows, row_bytes], a view of the memory map."""
        t = self.tensors[name]
        if t.nbytes is None:
            raise ValueError(f"{name}: ggml type {t.type} is not supported")
        start = self.data_start + t.offset
        return np.frombuffer(self._mm, dtype=np.uint8, count=t.nbytes, offset=start).reshape(t.rows, t.row_bytes)

    def close(self):
        """Release the file. Arrays returned by `data` still reference the map; it is then closed when they go."""
        try:
            self._mm.close()
        except BufferError:
            pass
        self._f.close()


# -- a dense decoder ---------------------------------------------------------------------------------------------------

def decoder_config(gf, kv_type=None, window=None, full_every=None):
    """DecoderConfig of a llama / qwen-style dense GQA decoder from its GGUF metadata and tensor shapes. The
    sliding-window pattern is not a standard GGUF key: `window` / `full_every` override `<arch>.attention.
    sliding_window` (0 = full attention in every layer)."""
    from .verify_step import DecoderConfig
    arch = gf.kv["general.architecture"]

    def g(key, default=None):
        return gf.kv.get(f"{arch}.{key}", default)

    n_layer = int(g("block_count"))
    d = int(g("embedding_length"))
    H = int(g("attention.head_count"))
    Hkv = int(g("attention.head_count_kv", H))
    hd = int(g("attention.key_length", d // H))
    n_ff = int(g("feed_forward_length"))
    emb = gf.tensors["token_embd.weight"]
    n_vocab = emb.ne[1]
    win = int(window if window is not None else g("attention.sliding_window", 0) or 0)
    fe = int(full_every if full_every is not None else (1 if win == 0 else 4))
    t = gf.tensors
    head = "output.weight" if "output.weight" in t else "token_embd.weight"
    types = {"qkv": t["blk.0.attn_q.weight"].type, "o": t["blk.0.attn_output.weight"].type,
             "gate": t["blk.0.ffn_gate.weight"].type, "up": t["blk.0.ffn_up.weight"].type,
             "down": t["blk.0.ffn_down.weight"].type, "head": t[head].type}
    return DecoderConfig(n_layer=n_layer, d=d, n_ff=n_ff, H=H, Hkv=Hkv, hd=hd, n_vocab=n_vocab,
                         base=float(g("rope.freq_base", 10000.0)), eps=float(g("attention.layer_norm_rms_epsilon",
                                                                                  1e-6)),
                         window=win, full_every=fe, kv_type=kv_type if kv_type is not None else L.F16, types=types)


def k_columns(blocks, ggml_type, k0, k1):
    """Columns [k0, k1) of packed rows of a ggml type (k0, k1 on block boundaries)."""
    from .shard import k_columns as _kc
    blk, bpb = GGML_BLOCKS[ggml_type]
    return _kc(blocks, blk, bpb, k0, k1)


def load_decoder(gf, cfg, device="cuda", rank=0, world=1, split_kv=True):
    """DeviceWeights of the decoder in `gf` (a GGUFFile), the slices of tensor-parallel rank `rank` of `world` (split_kv:
    as DeviceWeights.from_host).
    Matrices stay in their GGUF block layout; Q, K, V rows become one QKV matrix and gate, up one gate|up matrix
    (per rank: this rank's heads / FFN rows) when their types agree, else they stay separate GEMMs. Token embeddings
    must be F16 or F32 (srhpm_get_rows); norms F32."""
    from .ops import QuantTensor
    from .verify_step import DeviceWeights
    hd = cfg.hd
    w = DeviceWeights(cfg, device)
    lay_tp = w._set_tp(rank, world, split_kv)
    h0, h1, g0, g1 = lay_tp["h0"], lay_tp["h1"], lay_tp["g0"], lay_tp["g1"]
    f0, f1, v0, v1 = lay_tp["f0"], lay_tp["f1"], lay_tp["v0"], lay_tp["v1"]

    def qt(blocks, ggml_type, rows, K):
        return QuantTensor.from_blocks(blocks, ggml_type, rows, K, device)

    def f32(name):
        t = gf.tensors[name]
        if t.type != 0:
            raise ValueError(f"{name}: expected F32")
        return torch.from_numpy(gf.data(name).view(np.float32).reshape(-1).copy()).to(device)

    for l in range(cfg.n_layer):
        p = f"blk.{l}."
        lay = {}
        tq, tk, tv = (gf.tensors[p + f"attn_{x}.weight"] for x in "qkv")
        qa, qb = w.q_heads(l)
        q = gf.data(p + "attn_q.weight")[qa * hd:qb * hd]
        k = gf.data(p + "attn_k.weight")[g0 * hd:g1 * hd]
        v = gf.data(p + "attn_v.weight")[g0 * hd:g1 * hd]
        if tq.type == tk.type == tv.type:
            lay["qkv"] = qt(np.concatenate([q, k, v]), tq.type, (qb - qa + 2 * (g1 - g0)) * hd, cfg.d)
        else:
            lay["q"] = qt(q, tq.type, (qb - qa) * hd, cfg.d)
            lay["k"] = qt(k, tk.type, (g1 - g0) * hd, cfg.d)
            lay["v"] = qt(v, tv.type, (g1 - g0) * hd, cfg.d)
        to = gf.tensors[p + "attn_output.weight"]
        lay["o"] = qt(k_columns(gf.data(p + "attn_output.weight"), to.type, h0 * hd, h1 * hd), to.type, cfg.d,
                      (h1 - h0) * hd)
        tg, tu = gf.tensors[p + "ffn_gate.weight"], gf.tensors[p + "ffn_up.weight"]
        gate = gf.data(p + "ffn_gate.weight")[f0:f1]
        up = gf.data(p + "ffn_up.weight")[f0:f1]
        if tg.type == tu.type:
            lay["gate_up"] = qt(np.concatenate([gate, up]), tg.type, 2 * (f1 - f0), cfg.d)
        else:
            lay["gate"] = qt(gate, tg.type, f1 - f0, cfg.d)
            lay["up"] = qt(up, tu.type, f1 - f0, cfg.d)
        td = gf.tensors[p + "ffn_down.weight"]
        lay["down"] = qt(k_columns(gf.data(p + "ffn_down.weight"), td.type, f0, f1), td.type, cfg.d, f1 - f0)
        lay["attn_norm"] = f32(p + "attn_norm.weight")
        lay["ffn_norm"] = f32(p + "ffn_norm.weight")
        w.layers.append(lay)
    w.out_norm = f32("output_norm.weight")
    head = "output.weight" if "output.weight" in gf.tensors else "token_embd.weight"
    th = gf.tensors[head]
    if th.type not in (L.Q4_K, L.Q5_K, L.Q6_K, L.Q3_K, L.IQ4_XS, L.Q8_0):
        raise ValueError(f"{head}: ggml type {th.type} has no verify GEMM (Q3_K..Q6_K, IQ4_XS, Q8_0)")
    w.head = qt(gf.data(head)[v0:v1], th.type, v1 - v0, cfg.d)
    te = gf.tensors["token_embd.weight"]
    if te.type == 1:
        w.emb = torch.from_numpy(gf.data("token_embd.weight").view(np.float16).reshape(cfg.n_vocab, cfg.d).copy())
    elif te.type == 0:
        w.emb = torch.from_numpy(gf.data("token_embd.weight").view(np.float32).reshape(cfg.n_vocab, cfg.d).copy())
    else:
        raise ValueError("token_embd.weight: only F16 / F32 embeddings are supported")
    w.emb = w.emb.to(device)
    return w
