"""srhpm_b200: B200-native kernels for SR-HPM's speculative-verification hot path (quantized small-batch matmul,
multi-query flash-decode attention, greedy prefix acceptance) behind a C ABI, with a ggml-shaped host layer."""
from . import _lib
from ._lib import F16, F32, I32, IQ4_XS, Q3_K, Q4_K, Q5_K, Q6_K, Q8_0, Q8_K, TYPE_BY_NAME, TYPE_NAMES, SrhpmError
from .ops import Context, QuantTensor, f32_rows_view, quantize_chunk

__all__ = ["Context", "QuantTensor", "quantize_chunk", "f32_rows_view", "SrhpmError", "TYPE_NAMES", "TYPE_BY_NAME",
           "F32", "F16", "Q8_0", "Q3_K", "Q4_K", "Q5_K", "Q6_K", "Q8_K", "IQ4_XS", "I32"]
