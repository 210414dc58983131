"""The C++ operator interface (include/srhpm_ggml.hpp, libsrhpm_ggml.so) through its C++ test program,
tests/cpp/test_srhpm_ggml.cpp, which reads like the reference's own kernel checks:
- CPU: srv_traits_for / supports_op selection; work_size; the false answers that send an op to the stock path; the
  GGML_ASSERT aborts (in forked children); the GGML_SRV_TYPES filter;
- GPU: compute_forward of every SRV type and N in {1, 3, 8, 16} within 1e-5 of the oracle's exact sums (and a
  row-split view); the grouped attention behind its gate within 1e-3 of the oracle; greedy acceptance equal to the
  oracle's."""
import os
import subprocess

import pytest

ROOT = os.path.dirname(os.path.dirname(os.path.abspath(__file__)))
CPP = os.path.join(ROOT, "tests", "cpp")
BIN = os.path.join(CPP, "test_srhpm_ggml")


def run(mode, env=None):
    # the binary is built with the libraries (build()); make only rebuilds it when a source is newer
    mk = subprocess.run(["make", "-C", CPP], capture_output=True, text=True)
    assert mk.returncode == 0, mk.stdout + mk.stderr
    r = subprocess.run([BIN, mode], capture_output=True, text=True, timeout=600, env=env)
    assert r.returncode == 0, r.stdout + r.stderr


def test_cpp_interface_cpu():
    run("cpu")


def test_cpp_interface_type_filter():
    run("cpu-types", env={**os.environ, "GGML_SRV_TYPES": "q4_K,iq4_xs"})


@pytest.mark.gpu
def test_cpp_interface_gpu():
    run("gpu")
