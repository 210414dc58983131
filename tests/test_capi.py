"""CPU: the C-ABI library loads, exports every function include/srhpm_b200.h declares, and its host-only entry
points behave (no kernel launches here)."""
import ctypes

import numpy as np
import pytest

import oracle as O
import srhpm_b200 as S
from srhpm_b200 import _lib as L


def test_library_exports_every_declared_symbol():
    lib = L.load()
    declared = L.header_functions()
    assert len(declared) >= 15
    missing = [n for n in declared if not hasattr(lib, n)]
    assert not missing, missing


def test_type_facts():
    lib = L.load()
    for t, (qk, bs) in {S.Q4_K: (256, 144), S.Q5_K: (256, 176), S.Q6_K: (256, 210), S.Q3_K: (256, 110),
                        S.IQ4_XS: (256, 136), S.Q8_0: (32, 34), S.F16: (1, 2), S.F32: (1, 4)}.items():
        assert lib.srhpm_blck_size(t) == qk and lib.srhpm_type_size(t) == bs
    assert lib.srhpm_row_size(S.Q4_K, 5120) == 20 * 144
    assert lib.srhpm_row_size(S.Q4_K, 5000) == 0
    assert lib.srhpm_status_str(L.ERR_ALIGN).decode().startswith("misaligned")


@pytest.mark.parametrize("qtype,tol", [(S.Q4_K, 0.12), (S.Q5_K, 0.06), (S.Q6_K, 0.03), (S.Q3_K, 0.25),
                                       (S.IQ4_XS, 0.10), (S.Q8_0, 0.01)])
def test_host_quantizer_round_trip(qtype, tol):
    """srhpm_quantize_chunk produces valid GGUF blocks: dequantized by the oracle they reproduce the input to the
    relative RMS error expected of each format (Q3_K ~ 0.2, Q8_0 ~ 0.005)."""
    rng = np.random.default_rng(8)
    w = (rng.standard_normal((64, 1024)) * 0.02).astype(np.float32)
    blocks = S.quantize_chunk(w, qtype)
    assert blocks.shape == (64, L.load().srhpm_row_size(qtype, 1024))
    back = O.dequantize(qtype, blocks, w.size).reshape(w.shape)
    err = np.sqrt(np.mean((back - w) ** 2)) / np.sqrt(np.mean(w ** 2))
    assert err < tol, err


def test_host_quantizer_rejects_bad_shapes():
    lib = L.load()
    w = np.zeros((2, 300), np.float32)
    out = np.zeros(4096, np.uint8)
    assert lib.srhpm_quantize_chunk(S.Q4_K, w.ctypes.data, out.ctypes.data, 0, 2, 300, None) == 0


def test_ctx_create_reports_errors_without_a_device():
    """Without a usable device the context constructor returns an error code instead of aborting."""
    torch = pytest.importorskip("torch")
    if torch.cuda.is_available():
        pytest.skip("a device is present")
    lib = L.load()
    h = ctypes.c_void_p()
    assert lib.srhpm_ctx_create(0, ctypes.byref(h)) != L.OK
