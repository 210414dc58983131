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
        lib.orc_accept.argtypes = [_P, ctypes.c_int64, _P, ctypes.c_int, ctypes.c_float, _P]
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

def random_blocks(qtype, nblocks, rng, d_lo=0.005, d_hi=0.02):
    """Random bytes in every field (all bit patterns of codes and scales) with sane f16 block scales, as the
    reference's kernel checks generate them (research/tools/srv_bench.cpp:166-173, dgpu/dgpu_test.cpp:73-77)."""
    bs = BLOCK_BYTES[qtype]
    blocks = rng.integers(0, 256, size=(nblocks, bs), dtype=np.uint8)
    for off in D_OFFSET[qtype]:
        d = rng.uniform(d_lo, d_hi, size=nblocks).astype(np.float16)
        blocks[:, off:off + 2] = d.view(np.uint8).reshape(nblocks, 2)
    return blocks
