"""TEST INFRASTRUCTURE (oracle): numpy wrappers over

  - oracle/liboracle.so: the CPU restatement of the reference's verify-path arithmetic (oracle.c), and
  - oracle/_ref/libsrv_ref_{avx2,vnni}.so: the reference's own SRV kernels and FA-GQA function, compiled from its
    patch by build_ref.sh (absent when the reference was not available at build time).

Only tests/, __graft_entry__.smoke() and bench.py's CPU-baseline leg import this module, and only as the checker.
"""
import ctypes
import os

import numpy as np

HERE = os.path.dirname(os.path.abspath(__file__))
ORACLE_PATH = os.path.join(HERE, "liboracle.so")
REF_DIR = os.path.join(HERE, "_ref")

F32, F16, Q8_0, Q3_K, Q4_K, Q5_K, Q6_K, IQ4_XS = 0, 1, 8, 11, 12, 13, 14, 23
BLOCK_BYTES = {Q4_K: 144, Q5_K: 176, Q6_K: 210, Q3_K: 110, IQ4_XS: 136, Q8_0: 34, F16: 2}
BLOCK_ELEMS = {Q4_K: 256, Q5_K: 256, Q6_K: 256, Q3_K: 256, IQ4_XS: 256, Q8_0: 32, F16: 1}
D_OFFSET = {Q4_K: (0, 2), Q5_K: (0, 2), Q6_K: (208,), Q3_K: (108,), IQ4_XS: (0,), Q8_0: (0,)}
SRV_TYPES = (Q4_K, Q5_K, Q6_K, Q3_K, IQ4_XS)  # types with a reference SRV kernel
Q8_0_SIMD, Q8_0_REF = 0, 1

_P = ctypes.c_void_p
_orc = None
_ref = {}


def _ptr(a):
    return ctypes.c_void_p(a.ctypes.data) if a is not None else None


def _u8(a):
    """The bytes of a as a contiguous uint8 vector (no copy when a already is one)."""
    a = np.asarray(a)
    if not a.flags.c_contiguous:
        a = np.ascontiguousarray(a)
    return a.reshape(-1).view(np.uint8)


def load_oracle():
    global _orc
    if _orc is None:
        if not os.path.exists(ORACLE_PATH):
            raise RuntimeError(f"{ORACLE_PATH} is not built: run `make -C oracle`")
        lib = ctypes.CDLL(ORACLE_PATH)
        lib.orc_fp32_to_fp16.restype = ctypes.c_uint16
        lib.orc_fp32_to_fp16.argtypes = [ctypes.c_float]
        lib.orc_fp16_to_fp32.restype = ctypes.c_float
        lib.orc_fp16_to_fp32.argtypes = [ctypes.c_uint16]
        lib.orc_quantize_row_q8K.argtypes = [_P, _P, _P, _P, _P, ctypes.c_int64]
        lib.orc_quantize_row_q8_0.argtypes = [_P, _P, ctypes.c_int64, ctypes.c_int]
        lib.orc_dequantize.argtypes = [ctypes.c_int, _P, _P, ctypes.c_int64]
        lib.orc_row_isums.argtypes = [ctypes.c_int, _P, _P, _P, ctypes.c_int64, _P, _P]
        lib.orc_mul_mat.argtypes = [ctypes.c_int, _P, ctypes.c_int64, ctypes.c_int64, _P, ctypes.c_int64, _P,
                                    ctypes.c_int]
        lib.orc_mul_mat_q8_0_f32.argtypes = [_P, ctypes.c_int64, ctypes.c_int64, _P, ctypes.c_int64, _P, ctypes.c_int,
                                             ctypes.c_int]
        lib.orc_attention.argtypes = [_P, ctypes.c_int64, ctypes.c_int64, ctypes.c_int64, ctypes.c_int, _P, _P,
                                      ctypes.c_int64, ctypes.c_int64, ctypes.c_int64, _P, _P, ctypes.c_float,
                                      ctypes.c_float, ctypes.c_float, ctypes.c_int, _P]
        lib.orc_attention_partial.argtypes = [_P, ctypes.c_int64, ctypes.c_int64, ctypes.c_int64, ctypes.c_int, _P,
                                              _P, ctypes.c_int64, ctypes.c_int64, ctypes.c_int64, ctypes.c_int64,
                                              ctypes.c_int64, _P, ctypes.c_float, ctypes.c_float, ctypes.c_float,
                                              ctypes.c_int, _P, _P, _P]
        lib.orc_attention_merge.argtypes = [ctypes.c_int64, ctypes.c_int64, ctypes.c_int64, ctypes.c_int64, _P, _P,
                                            _P, _P, _P]
        lib.orc_accept.argtypes = [_P, ctypes.c_int64, _P, ctypes.c_int, ctypes.c_float, _P]
        lib.orc_quantize_rtn.restype = ctypes.c_int64
        lib.orc_quantize_rtn.argtypes = [ctypes.c_int, _P, _P, ctypes.c_int64]
        _orc = lib
    return _orc


def _cpu_flags():
    try:
        for line in open("/proc/cpuinfo"):
            if line.startswith("flags"):
                return set(line.split(":", 1)[1].split())
    except OSError:
        pass
    return set()


def ref_variant():
    """'vnni' when this host has AVX-VNNI and that build exists, else 'avx2' (None when neither was built)."""
    flags = _cpu_flags()
    if "avx_vnni" in flags and os.path.exists(os.path.join(REF_DIR, "libsrv_ref_vnni.so")):
        return "vnni"
    if "avx2" in flags and os.path.exists(os.path.join(REF_DIR, "libsrv_ref_avx2.so")):
        return "avx2"
    return None


def load_ref(variant=None):
    """The reference's own kernels, or None when oracle/_ref was not built (no reference at build time)."""
    variant = variant or ref_variant()
    if variant is None:
        return None
    if variant not in _ref:
        lib = ctypes.CDLL(os.path.join(REF_DIR, f"libsrv_ref_{variant}.so"))
        lib.ref_srv_quantize_row.argtypes = [_P, _P, _P, ctypes.c_int64, _P, _P]
        lib.ref_srv_mul_mat.argtypes = [ctypes.c_int, _P, ctypes.c_int64, ctypes.c_int64, _P, ctypes.c_int64, _P,
                                        ctypes.c_int, ctypes.c_int, ctypes.c_int]
        lib.ref_set_q8_0_mode.argtypes = [ctypes.c_int]
        lib.ref_quantize_row_q8_0_c.argtypes = [_P, _P, ctypes.c_int64]
        lib.ref_vec_dot_q8_0_c.argtypes = [ctypes.c_int, _P, _P, _P]
        lib.ref_fa_gqa.argtypes = [_P, _P, ctypes.c_int64, ctypes.c_int64, ctypes.c_int64, ctypes.c_int, _P, _P, _P,
                                   _P, ctypes.c_int64, ctypes.c_int64, ctypes.c_int64, _P, ctypes.c_size_t, _P,
                                   ctypes.c_float, ctypes.c_float, ctypes.c_float, _P, ctypes.c_int]
        _ref[variant] = lib
    return _ref[variant]


# ---- restated oracle ------------------------------------------------------------------------------------------

def fp32_to_fp16_bits(x):
    lib = load_oracle()
    return np.array([lib.orc_fp32_to_fp16(float(v)) for v in np.ravel(x)], dtype=np.uint16)


def quantize_row_q8K(x):
    x = np.ascontiguousarray(x, dtype=np.float32)
    K = x.size
    q = np.empty(K, np.int8)
    d = np.empty(K // 256, np.float32)
    b32 = np.empty(K // 32, np.int16)
    b16 = np.empty(K // 16, np.int16)
    load_oracle().orc_quantize_row_q8K(_ptr(x), _ptr(q), _ptr(d), _ptr(b32), _ptr(b16), K)
    return q, d, b32, b16


def quantize_row_q8_0(x, mode=Q8_0_SIMD):
    x = np.ascontiguousarray(x, dtype=np.float32)
    out = np.empty(x.size // 32 * 34, np.uint8)
    load_oracle().orc_quantize_row_q8_0(_ptr(x), _ptr(out), x.size, mode)
    return out


def dequantize(qtype, blocks, n):
    blocks = _u8(blocks)
    y = np.empty(n, np.float32)
    load_oracle().orc_dequantize(qtype, _ptr(blocks), _ptr(y), n)
    return y


def row_isums(qtype, row, xq, bsum32, K):
    row = _u8(row)
    xq = np.ascontiguousarray(xq, np.int8)
    b32 = np.ascontiguousarray(bsum32, np.int16) if bsum32 is not None else np.zeros(K // 32, np.int16)
    nblk = K // BLOCK_ELEMS[qtype]
    m = np.zeros(nblk, np.int32)
    mn = np.zeros(nblk, np.int32)
    load_oracle().orc_row_isums(qtype, _ptr(row), _ptr(xq), _ptr(b32), K, _ptr(m), _ptr(mn))
    return m, mn


def mul_mat(qtype, W, rows, K, X, q8_mode=Q8_0_SIMD):
    """Exact-integer oracle: double [N, rows]."""
    W = _u8(W)
    X = np.ascontiguousarray(X, np.float32)
    N = X.shape[0]
    Y = np.empty((N, rows), np.float64)
    st = load_oracle().orc_mul_mat(qtype, _ptr(W), rows, K, _ptr(X), N, _ptr(Y), q8_mode)
    assert st == 0, st
    return Y


def mul_mat_q8_0_f32(W, rows, K, X, q8_mode=Q8_0_SIMD, nth=1):
    W = _u8(W)
    X = np.ascontiguousarray(X, np.float32)
    N = X.shape[0]
    Y = np.empty((N, rows), np.float32)
    st = load_oracle().orc_mul_mat_q8_0_f32(_ptr(W), rows, K, _ptr(X), N, _ptr(Y), q8_mode, nth)
    assert st == 0, st
    return Y


def attention(q, kv_type, k, v, DV, L, Hkv, mask=None, sinks=None, scale=1.0, max_bias=0.0, softcap=0.0,
              q8_mode=Q8_0_SIMD):
    """q f32 [H, N, DK]; k, v bytes [Hkv, L, row]; mask f16-bits uint16 [N, L]; returns double [N, H, DV]."""
    q = np.ascontiguousarray(q, np.float32)
    H, N, DK = q.shape
    k = _u8(k)
    v = _u8(v)
    m = np.ascontiguousarray(mask, np.uint16) if mask is not None else None
    s = np.ascontiguousarray(sinks, np.float32) if sinks is not None else None
    dst = np.empty((N, H, DV), np.float64)
    st = load_oracle().orc_attention(_ptr(q), DK, N, H, kv_type, _ptr(k), _ptr(v), DV, L, Hkv, _ptr(m), _ptr(s),
                                     scale, max_bias, softcap, q8_mode, _ptr(dst))
    assert st == 0, st
    return dst


def attention_partial(q, kv_type, k, v, DV, L, Hkv, t0, t1, mask=None, scale=1.0, max_bias=0.0, softcap=0.0,
                      q8_mode=Q8_0_SIMD):
    """Records of KV tokens [t0, t1) (orc_attention_partial): (m [H, N], s [H, N], acc [H, N, DV]), all double;
    m in natural-log units."""
    q = np.ascontiguousarray(q, np.float32)
    H, N, DK = q.shape
    k = _u8(k)
    v = _u8(v)
    msk = np.ascontiguousarray(mask, np.uint16) if mask is not None else None
    m = np.empty((H, N), np.float64)
    s = np.empty((H, N), np.float64)
    acc = np.empty((H, N, DV), np.float64)
    st = load_oracle().orc_attention_partial(_ptr(q), DK, N, H, kv_type, _ptr(k), _ptr(v), DV, L, Hkv, t0, t1,
                                             _ptr(msk), scale, max_bias, softcap, q8_mode, _ptr(m), _ptr(s), _ptr(acc))
    assert st == 0, st
    return m, s, acc


def attention_merge(m, s, acc, sinks=None):
    """Merge record sets stacked on a leading part axis (m, s [P, H, N], acc [P, H, N, DV]) -> double [N, H, DV]."""
    m = np.ascontiguousarray(m, np.float64)
    s = np.ascontiguousarray(s, np.float64)
    acc = np.ascontiguousarray(acc, np.float64)
    P, H, N, DV = acc.shape
    sk = np.ascontiguousarray(sinks, np.float32) if sinks is not None else None
    dst = np.empty((N, H, DV), np.float64)
    st = load_oracle().orc_attention_merge(P, N, H, DV, _ptr(m), _ptr(s), _ptr(acc), _ptr(sk), _ptr(dst))
    assert st == 0, st
    return dst


def accept(logits, draft, relax=0.0):
    logits = np.ascontiguousarray(logits, np.float32)
    draft = np.ascontiguousarray(draft, np.int32)
    n_draft = draft.size
    out = np.empty(n_draft + 1, np.int32)
    n = load_oracle().orc_accept(_ptr(logits), logits.shape[1], _ptr(draft), n_draft, relax, _ptr(out))
    return out[:n].tolist()


# ---- the reference's own kernels ------------------------------------------------------------------------------

def ref_quantize_row(x, lib=None):
    lib = lib or load_ref()
    x = np.ascontiguousarray(x, dtype=np.float32)
    K = x.size
    q = np.empty(K, np.int8)
    d = np.empty(K // 256, np.float32)
    b32 = np.empty(K // 32, np.int16)
    b16 = np.empty(K // 16, np.int16)
    assert lib.ref_srv_quantize_row(_ptr(x), _ptr(q), _ptr(d), K, _ptr(b32), _ptr(b16)) == 0
    return q, d, b32, b16


def ref_mul_mat(qtype, W, rows, K, X, nth=1, off=1, paired=1, lib=None):
    """The reference's SRV kernels (srv_row via compute_forward's scheduling): f32 [N, rows]."""
    lib = lib or load_ref()
    W = _u8(W)
    X = np.ascontiguousarray(X, np.float32)
    N = X.shape[0]
    Y = np.empty((N, rows), np.float32)
    st = lib.ref_srv_mul_mat(qtype, _ptr(W), rows, K, _ptr(X), N, _ptr(Y), nth, off, paired)
    assert st == 0, st
    return Y


def ref_fa_gqa(q, kv_type, k, v, DV, L, Hkv, mask=None, sinks=None, scale=1.0, max_bias=0.0, softcap=0.0, nth=1,
               q8_mode=Q8_0_SIMD, lib=None):
    """The reference's ggml_compute_forward_flash_attn_ext_gqa_small. Same layouts as attention(); f32 [N, H, DV]."""
    lib = lib or load_ref()
    lib.ref_set_q8_0_mode(q8_mode)
    q = np.ascontiguousarray(q, np.float32)
    H, N, DK = q.shape
    k = _u8(k)
    v = _u8(v)
    krow = DK // 32 * 34 if kv_type == Q8_0 else DK * 2
    vrow = DV // 32 * 34 if kv_type == Q8_0 else DV * 2
    nbq = (ctypes.c_size_t * 4)(4, DK * 4, N * DK * 4, H * N * DK * 4)
    nbk = (ctypes.c_size_t * 4)(34 if kv_type == Q8_0 else 2, krow, L * krow, Hkv * L * krow)
    nbv = (ctypes.c_size_t * 4)(34 if kv_type == Q8_0 else 2, vrow, L * vrow, Hkv * L * vrow)
    m = np.ascontiguousarray(mask, np.uint16) if mask is not None else None
    s = np.ascontiguousarray(sinks, np.float32) if sinks is not None else None
    dst = np.zeros((N, H, DV), np.float32)
    st = lib.ref_fa_gqa(_ptr(q), nbq, DK, N, H, kv_type, _ptr(k), nbk, _ptr(v), nbv, DV, L, Hkv, _ptr(m),
                        L * 2, _ptr(s), scale, max_bias, softcap, _ptr(dst), nth)
    assert st == 0, st
    return dst


# ---- inputs -----------------------------------------------------------------------------------------------------

def quantize_rtn(qtype, w, nth=None):
    """f32 [rows, K] -> GGUF blocks uint8 [rows, row_bytes] by the oracle's round-to-nearest quantizers (input
    generation for the CPU reference timings; not pinned to ggml's quantizers). Rows are split over nth threads."""
    from concurrent.futures import ThreadPoolExecutor
    lib = load_oracle()
    w = np.ascontiguousarray(w, dtype=np.float32)
    rows, K = w.shape
    qk = 32 if qtype == Q8_0 else 256
    if K % qk:
        raise ValueError(f"K = {K} is not a multiple of {qk}")
    rb = K // qk * BLOCK_BYTES[qtype]
    out = np.empty((rows, rb), np.uint8)
    nth = nth or os.cpu_count() or 1
    cut = [rows * i // nth for i in range(nth + 1)]

    def part(i):
        r0, r1 = cut[i], cut[i + 1]
        if r1 > r0 and lib.orc_quantize_rtn(qtype, _ptr(w[r0:r1]), _ptr(out[r0:r1]), (r1 - r0) * K) < 0:
            raise RuntimeError("orc_quantize_rtn failed")

    with ThreadPoolExecutor(nth) as ex:
        list(ex.map(part, range(nth)))
    return out


def random_blocks(qtype, nblocks, rng, d_lo=0.005, d_hi=0.02):
    """Random bytes in every field (all bit patterns of codes and scales) with sane f16 block scales, as the
    reference's kernel checks generate them (research/tools/srv_bench.cpp:166-173, dgpu/dgpu_test.cpp:73-77)."""
    bs = BLOCK_BYTES[qtype]
    blocks = rng.integers(0, 256, size=(nblocks, bs), dtype=np.uint8)
    for off in D_OFFSET[qtype]:
        d = rng.uniform(d_lo, d_hi, size=nblocks).astype(np.float16)
        blocks[:, off:off + 2] = d.view(np.uint8).reshape(nblocks, 2)
    return blocks


# ---- a dense decoder verify step, restated -------------------------------------------------------------------------
# The element-wise ggml operators around the verify GEMMs (upstream ggml, not in the reference: rms_norm + mul,
# rope_ext NEOX, swiglu, get_rows, cpy into the KV cache) in numpy, and a whole step composed of them with the exact
# matmul (mul_mat), attention (attention) and acceptance (accept) above.

def rms_norm(x, w, eps):
    """ggml_rms_norm (sum of squares in double, scale 1/sqrtf(mean + eps)) then ggml_mul by w: f32 [n, d]."""
    x = np.asarray(x, np.float32)
    mean = ((x.astype(np.float64) ** 2).sum(axis=-1, keepdims=True) / x.shape[-1]).astype(np.float32)
    scale = (np.float32(1.0) / np.sqrt(mean + np.float32(eps))).astype(np.float32)
    return (x * scale * np.asarray(w, np.float32)).astype(np.float32)


def rope_neox(x, pos, base):
    """ggml_rope_ext, mode NEOX over the whole head: x f32 [n, heads, hd]; pairs (j, j + hd/2) turned by
    pos * base^(-2j/hd). f64 math, f32 result."""
    x = np.asarray(x, np.float32)
    hd = x.shape[-1]
    half = hd // 2
    theta = np.asarray(pos, np.float64)[:, None] * np.power(float(base), -2.0 * np.arange(half) / hd)[None, :]
    c, s = np.cos(theta)[:, None, :], np.sin(theta)[:, None, :]
    x0, x1 = x[..., :half].astype(np.float64), x[..., half:].astype(np.float64)
    return np.concatenate([x0 * c - x1 * s, x0 * s + x1 * c], axis=-1).astype(np.float32)


def swiglu(g, u):
    """ggml_swiglu: silu(g) * u, f32."""
    g64 = np.asarray(g, np.float64)
    return (g64 / (1.0 + np.exp(-g64)) * np.asarray(u, np.float64)).astype(np.float32)


def cache_rows(kv_type, x, q8_mode=Q8_0_SIMD):
    """f32 head rows [..., hd] -> cache bytes [..., row] (ggml_cpy into an f16 or q8_0 cache)."""
    x = np.asarray(x, np.float32)
    if kv_type == F16:
        return x.astype(np.float16).view(np.uint8)
    flat = x.reshape(-1, x.shape[-1])
    return np.stack([quantize_row_q8_0(r, q8_mode) for r in flat]).reshape(*x.shape[:-1], -1)


def attn_window(layer, full_every, window, n_past, n):
    """Keys [start, n_past + n) a layer's new rows attend to and the mask f16 [n, L] (causal; sliding layers also hide
    keys at or beyond `window` positions back): full layers are those with layer % full_every == full_every - 1."""
    L_all = n_past + n
    full = window <= 0 or layer % full_every == full_every - 1
    start = 0 if full else max(0, n_past - window + 1)
    L = L_all - start
    m = np.zeros((n, L), np.float16)
    for t in range(n):
        p = n_past + t
        for j in range(L):
            a = start + j
            if a > p or (not full and a <= p - window):
                m[t, j] = -np.inf
    return start, m


def decoder_step(cfg, w, kcache, vcache, ids, n_past, draft, q8_mode=Q8_0_SIMD, relax=0.0):
    """One verify step of a dense decoder (RMSNorm, fused QKV, NEOX RoPE, GQA attention over the cache, SwiGLU FFN,
    output head, greedy acceptance). cfg: dict n_layer, d, n_ff, H, Hkv, hd, n_vocab, base, eps, window, full_every,
    kv_type, types {'qkv', 'o', 'gate', 'up', 'down', 'head'}. w: dict of host GGUF blocks per layer ('qkv'[l], ...),
    f32 norms ('attn_norm'[l], 'ffn_norm'[l], 'out_norm'), 'head', 'emb' f16 [n_vocab, d]. kcache / vcache: per layer
    uint8 [capacity, Hkv, row] (updated). Returns (logits f32 [n, n_vocab], accepted ids)."""
    c = cfg
    n = len(ids)
    H, Hkv, hd, d = c["H"], c["Hkv"], c["hd"], c["d"]
    ty = c["types"]
    pos = np.arange(n_past, n_past + n)
    x = w["emb"][np.asarray(ids)].astype(np.float32)
    for l in range(c["n_layer"]):
        y = rms_norm(x, w["attn_norm"][l], c["eps"])
        qkv = mul_mat(ty["qkv"], w["qkv"][l], (H + 2 * Hkv) * hd, d, y, q8_mode).astype(np.float32)
        q = rope_neox(qkv[:, :H * hd].reshape(n, H, hd), pos, c["base"])
        k = rope_neox(qkv[:, H * hd:(H + Hkv) * hd].reshape(n, Hkv, hd), pos, c["base"])
        v = qkv[:, (H + Hkv) * hd:].reshape(n, Hkv, hd)
        kcache[l][n_past:n_past + n] = cache_rows(c["kv_type"], k, q8_mode)
        vcache[l][n_past:n_past + n] = cache_rows(c["kv_type"], v, q8_mode)
        start, mask = attn_window(l, c["full_every"], c["window"], n_past, n)
        kk = np.ascontiguousarray(kcache[l][start:n_past + n].transpose(1, 0, 2))
        vv = np.ascontiguousarray(vcache[l][start:n_past + n].transpose(1, 0, 2))
        att = attention(np.ascontiguousarray(q.transpose(1, 0, 2)), c["kv_type"], kk, vv, hd, n_past + n - start, Hkv,
                        mask=mask.view(np.uint16), scale=1.0 / np.sqrt(hd), q8_mode=q8_mode)
        o = mul_mat(ty["o"], w["o"][l], d, H * hd, att.astype(np.float32).reshape(n, H * hd), q8_mode)
        x = (x + o.astype(np.float32)).astype(np.float32)
        y = rms_norm(x, w["ffn_norm"][l], c["eps"])
        g = mul_mat(ty["gate"], w["gate"][l], c["n_ff"], d, y, q8_mode).astype(np.float32)
        u = mul_mat(ty["up"], w["up"][l], c["n_ff"], d, y, q8_mode).astype(np.float32)
        h = swiglu(g, u)
        dn = mul_mat(ty["down"], w["down"][l], d, c["n_ff"], h, q8_mode)
        x = (x + dn.astype(np.float32)).astype(np.float32)
    y = rms_norm(x, w["out_norm"], c["eps"])
    logits = mul_mat(ty["head"], w["head"], c["n_vocab"], d, y, q8_mode).astype(np.float32)
    return logits, accept(logits, draft, relax)
