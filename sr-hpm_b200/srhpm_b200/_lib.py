"""ctypes binding of libsrhpm_b200.so (the C ABI declared in include/srhpm_b200.h).

The library is built in-tree by `make -C sr-hpm_b200` (or __graft_entry__.build()). Loading fails loudly when it is
missing: there is no CPU fallback for any operator of this package.
"""
import ctypes
import os
import re

HERE = os.path.dirname(os.path.abspath(__file__))
LIB_PATH = os.path.join(HERE, "libsrhpm_b200.so")
HEADER_PATH = os.path.abspath(os.path.join(HERE, "..", "..", "include", "srhpm_b200.h"))

# ggml_type numbering
F32, F16, Q8_0, Q3_K, Q4_K, Q5_K, Q6_K, Q8_K, IQ4_XS, I32 = 0, 1, 8, 11, 12, 13, 14, 15, 23, 26
TYPE_NAMES = {F32: "f32", F16: "f16", Q8_0: "q8_0", Q3_K: "q3_K", Q4_K: "q4_K", Q5_K: "q5_K", Q6_K: "q6_K",
              Q8_K: "q8_K", IQ4_XS: "iq4_xs", I32: "i32"}
TYPE_BY_NAME = {v.lower(): k for k, v in TYPE_NAMES.items()}

OK, UNSUPPORTED = 0, 1
ERR_INVALID, ERR_ALIGN, ERR_WORKSPACE, ERR_CUDA, ERR_DEVICE, ERR_TOO_LARGE = -1, -2, -3, -4, -5, -6
Q8_0_ACT_SIMD, Q8_0_ACT_REF = 0, 1


class SrhpmTensor(ctypes.Structure):
    """srhpm_tensor: a ggml-shaped view of device memory."""
    _fields_ = [("type", ctypes.c_int32), ("ne", ctypes.c_int64 * 4), ("nb", ctypes.c_size_t * 4),
                ("data", ctypes.c_void_p)]


class SrhpmError(RuntimeError):
    def __init__(self, status, what, lib=None):
        msg = lib.srhpm_status_str(status).decode() if lib is not None else str(status)
        extra = ""
        if lib is not None and status == ERR_CUDA:
            extra = f" (cudaError {lib.srhpm_last_cuda_error()})"
        super().__init__(f"{what}: status {status}: {msg}{extra}")
        self.status = status


_P = ctypes.c_void_p
_T = ctypes.POINTER(SrhpmTensor)
_SIGNATURES = {
    "srhpm_ctx_create": (ctypes.c_int, [ctypes.c_int, ctypes.POINTER(ctypes.c_void_p)]),
    "srhpm_ctx_destroy": (ctypes.c_int, [_P]),
    "srhpm_ctx_set_q8_0_act_mode": (ctypes.c_int, [_P, ctypes.c_int]),
    "srhpm_ctx_launch_count": (ctypes.c_int64, [_P, ctypes.c_int]),
    "srhpm_ctx_check": (ctypes.c_int, [_P, ctypes.POINTER(ctypes.c_int32)]),
    "srhpm_last_cuda_error": (ctypes.c_int, []),
    "srhpm_status_str": (ctypes.c_char_p, [ctypes.c_int]),
    "srhpm_blck_size": (ctypes.c_int, [ctypes.c_int]),
    "srhpm_type_size": (ctypes.c_size_t, [ctypes.c_int]),
    "srhpm_row_size": (ctypes.c_size_t, [ctypes.c_int, ctypes.c_int64]),
    "srhpm_mul_mat_work_size": (ctypes.c_int, [_T, _T, ctypes.POINTER(ctypes.c_size_t)]),
    "srhpm_mul_mat": (ctypes.c_int, [_P, _T, _T, _T, _P, ctypes.c_size_t, _P]),
    "srhpm_mul_mat_fused_quant": (ctypes.c_int, [_P, _T, _T, _T, _P, ctypes.c_size_t, _P]),
    "srhpm_mul_mat_swiglu": (ctypes.c_int, [_P, _T, _T, _T, _T, _P, ctypes.c_size_t, _P]),
    "srhpm_mul_mat_isums": (ctypes.c_int, [_P, _T, _T, _P, _P, _P, ctypes.c_size_t, _P]),
    "srhpm_mul_mat_static": (ctypes.c_int, [_P, _T, _T, _T, _P]),
    "srhpm_quantize_rows_q8_K": (ctypes.c_int, [_P, _T, _P, _P, _P, _P, _P]),
    "srhpm_quantize_rows_q8_0": (ctypes.c_int, [_P, _T, _P, _P]),
    "srhpm_flash_attn_ext_work_size": (ctypes.c_int, [_P, _T, _T, _T, ctypes.POINTER(ctypes.c_size_t)]),
    "srhpm_flash_attn_ext": (ctypes.c_int, [_P, _T, _T, _T, _T, _T, ctypes.c_float, ctypes.c_float, ctypes.c_float,
                                            _T, _P, ctypes.c_size_t, _P]),
    "srhpm_flash_attn_part_size": (ctypes.c_size_t, [ctypes.c_int64, ctypes.c_int64]),
    "srhpm_flash_attn_ext_partial": (ctypes.c_int, [_P, _T, _T, _T, _T, ctypes.c_float, ctypes.c_float, ctypes.c_float,
                                                    _P, _P, ctypes.c_size_t, _P]),
    "srhpm_flash_attn_merge": (ctypes.c_int, [_P, _P, ctypes.c_int, _T, _T, _P]),
    "srhpm_flash_attn_peer_buffer_size": (ctypes.c_size_t, [ctypes.c_int64, ctypes.c_int64]),
    "srhpm_flash_attn_merge_peers": (ctypes.c_int, [_P, _P, ctypes.c_int, ctypes.c_int, _P, _T, _T, _P]),
    "srhpm_verify_accept_work_size": (ctypes.c_int, [_P, _T, ctypes.POINTER(ctypes.c_size_t)]),
    "srhpm_verify_accept": (ctypes.c_int, [_P, _T, _P, ctypes.c_int, ctypes.c_float, _P, _P, _P, ctypes.c_size_t, _P]),
    "srhpm_argmax_shard": (ctypes.c_int, [_P, _T, ctypes.c_int64, _P, ctypes.c_int, _P, _P, ctypes.c_size_t, _P]),
    "srhpm_accept_merge": (ctypes.c_int, [_P, _P, ctypes.c_int, ctypes.c_int, _P, ctypes.c_int, ctypes.c_float, _P, _P,
                                          _P]),
    "srhpm_get_rows": (ctypes.c_int, [_P, _T, _P, ctypes.c_int, _P, _P]),
    "srhpm_allreduce_buffer_size": (ctypes.c_size_t, [ctypes.c_int64]),
    "srhpm_add_rms_norm_quant": (ctypes.c_int, [_P, _P, _P, _P, ctypes.c_float, _P, ctypes.c_int, _T, _P,
                                                ctypes.c_size_t, _P]),
    "srhpm_mul_mat_prequantized": (ctypes.c_int, [_P, _T, _T, _T, _P, ctypes.c_size_t, _P]),
    "srhpm_swiglu_quant": (ctypes.c_int, [_P, _P, _P, ctypes.c_int64, _P, ctypes.c_int64, ctypes.c_int, _T, _P,
                                          ctypes.c_size_t, _P]),
    "srhpm_add_rms_norm_allreduce": (ctypes.c_int, [_P, _P, _P, ctypes.c_int, ctypes.c_int, ctypes.c_int, _P, _P,
                                                    ctypes.c_float, _P, ctypes.c_int, ctypes.c_int64, _P]),
    "srhpm_add_rms_norm_allreduce_quant": (ctypes.c_int, [_P, _P, _P, ctypes.c_int, ctypes.c_int, ctypes.c_int, _P,
                                                          _P, ctypes.c_float, _P, ctypes.c_int, _T, _P, ctypes.c_size_t,
                                                          _P]),
    "srhpm_add_rms_norm": (ctypes.c_int, [_P, _P, _P, _P, ctypes.c_float, _P, ctypes.c_int, ctypes.c_int64, _P]),
    "srhpm_rope_kv": (ctypes.c_int, [_P, _P, ctypes.c_int64, ctypes.c_int, ctypes.c_int, ctypes.c_int, ctypes.c_int, _P,
                                     ctypes.c_float, _T, _T, _P]),
    "srhpm_swiglu": (ctypes.c_int, [_P, _P, _P, ctypes.c_int64, _P, ctypes.c_int64, ctypes.c_int, ctypes.c_int64,
                                    _P]),
    "srhpm_quantize_chunk": (ctypes.c_size_t, [ctypes.c_int, _P, _P, ctypes.c_int64, ctypes.c_int64, ctypes.c_int64,
                                                _P]),
}

_lib = None


def header_functions(path=HEADER_PATH):
    """Names of every function the C header declares."""
    text = open(path).read()
    text = re.sub(r"/\*.*?\*/", "", text, flags=re.S)
    return sorted(set(re.findall(r"\b(srhpm_[a-z0-9_]+)\s*\(", text)))


def load():
    """Load (once) and return the library with every signature declared."""
    global _lib
    if _lib is not None:
        return _lib
    if not os.path.exists(LIB_PATH):
        raise RuntimeError(f"{LIB_PATH} is not built: run `make -C sr-hpm_b200` (or __graft_entry__.build())")
    lib = ctypes.CDLL(LIB_PATH)
    for name, (res, args) in _SIGNATURES.items():
        fn = getattr(lib, name, None)
        if fn is None:
            continue
        fn.restype = res
        fn.argtypes = args
    _lib = lib
    return lib


def check(status, what):
    if status != OK:
        raise SrhpmError(status, what, _lib)
    return status
