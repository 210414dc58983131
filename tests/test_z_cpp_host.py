"""The C++ host side through its C++ test programs (tests/cpp), which read like the reference's own kernel checks.

The operator interface (include/srhpm_ggml.hpp, libsrhpm_ggml.so; tests/cpp/test_srhpm_ggml.cpp):
- CPU: srv_traits_for / supports_op selection; work_size; the false answers that send an op to the stock path; the
  GGML_ASSERT aborts (in forked children); the GGML_SRV_TYPES filter;
- GPU: compute_forward of every SRV type and N in {1, 3, 8, 16} within 1e-5 of the oracle's exact sums (and a
  row-split view); the grouped attention behind its gate within 1e-3 of the oracle; greedy acceptance equal to the
  oracle's.

The dGPU library (libsrhpm_dgpu.so; tests/cpp/test_srhpm_dgpu.cpp), loaded by path with its entry points bound by
name as the reference's ggml-cpu binds them:
- CPU: the argument statuses, a launch before dgpu_init, a collect before any launch;
- GPU: IQ4_XS and Q3_K rows for M = 1..8 with strided activations and outputs within 1e-5 of the oracle, one copy per
  key, the max_pinned budget, collect's shape check."""
import os
import subprocess

import pytest

ROOT = os.path.dirname(os.path.dirname(os.path.abspath(__file__)))
CPP = os.path.join(ROOT, "tests", "cpp")
BIN = os.path.join(CPP, "test_srhpm_ggml")
DGPU_BIN = os.path.join(CPP, "test_srhpm_dgpu")
LIBDIR = os.path.join(ROOT, "sr-hpm_b200", "srhpm_b200")


def run(args, env=None):
    # the binaries are built with the libraries (build()); make only rebuilds what a newer source needs
    mk = subprocess.run(["make", "-C", CPP], capture_output=True, text=True)
    assert mk.returncode == 0, mk.stdout + mk.stderr
    r = subprocess.run(args, capture_output=True, text=True, timeout=600, env=env)
    assert r.returncode == 0, r.stdout + r.stderr


def test_cpp_interface_cpu():
    run([BIN, "cpu"])


def test_cpp_interface_type_filter():
    run([BIN, "cpu-types"], env={**os.environ, "GGML_SRV_TYPES": "q4_K,iq4_xs"})


def test_dgpu_library_exports_the_reference_entry_points():
    """Every function include/srhpm_dgpu.h declares (dgpu/dgpu.cu's names, which ggml-cpu binds by name,
    patch/srhpm.patch:5048-5052), and nothing else."""
    import ctypes
    import re
    text = re.sub(r"/\*.*?\*/", "", open(os.path.join(ROOT, "include", "srhpm_dgpu.h")).read(), flags=re.S)
    declared = set(re.findall(r"\b(dgpu_[a-z_]+)\s*\(", text))
    assert {"dgpu_init", "dgpu_launch", "dgpu_collect", "dgpu_mem_info"} <= declared
    lib = ctypes.CDLL(os.path.join(LIBDIR, "libsrhpm_dgpu.so"))
    for name in declared:
        assert hasattr(lib, name), name
    nm = subprocess.run(["nm", "-D", "--defined-only", os.path.join(LIBDIR, "libsrhpm_dgpu.so")],
                        capture_output=True, text=True)
    if nm.returncode == 0:
        exported = {ln.split()[-1] for ln in nm.stdout.splitlines() if " T " in ln}
        assert exported == declared


def test_dgpu_library_cpu():
    run([DGPU_BIN, LIBDIR, "cpu"])


@pytest.mark.gpu
def test_cpp_interface_gpu():
    run([BIN, "gpu"])


@pytest.mark.gpu
def test_dgpu_library_gpu():
    run([DGPU_BIN, LIBDIR, "gpu"])
