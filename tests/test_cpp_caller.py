"""The C++ drop-in check: tests/cpp/drop_in_caller.cpp is compiled with g++ against the public
headers (include/mxfp6/*.hpp, include/mxfp6_gemm.h) and linked to libmxfp6gemm.so, as a C++
user of the reference library would (reference: include/mxfp6/gemm.hpp:25-64,
tests/test_gemm.cpp:131-201). `host` mode runs without a device; `gpu` mode runs the reference's
quantise -> preprocess -> gemm flow for every output type, a split-K shape and a compact-A shape;
`time` mode times BASELINE config 1 back to back as the reference's harness does.
"""
from __future__ import annotations

import os
import subprocess

import pytest

ROOT = os.path.dirname(os.path.dirname(os.path.abspath(__file__)))
LIB_DIR = os.path.join(ROOT, "mxfp6-gemm_b200", "lib")
SRC = os.path.join(ROOT, "tests", "cpp", "drop_in_caller.cpp")
CUDA_HOME = os.environ.get("CUDA_HOME", "/usr/local/cuda")


@pytest.fixture(scope="module")
def caller(tmp_path_factory, lib):  # `lib` makes sure the library is built and loadable
    exe = str(tmp_path_factory.mktemp("cpp") / "drop_in_caller")
    cmd = ["g++", "-std=c++17", "-O2", "-Wall", "-Wextra", "-Werror",
           "-I", os.path.join(ROOT, "include"), "-I", os.path.join(CUDA_HOME, "include"),
           SRC, "-o", exe,
           "-L", LIB_DIR, "-lmxfp6gemm", f"-Wl,-rpath,{LIB_DIR}",
           "-L", os.path.join(CUDA_HOME, "lib64"), "-lcudart", f"-Wl,-rpath,{os.path.join(CUDA_HOME, 'lib64')}"]
    r = subprocess.run(cmd, capture_output=True, text=True)
    assert r.returncode == 0, r.stderr
    return exe


def _run(exe, mode, timeout):
    r = subprocess.run([exe, mode], capture_output=True, text=True, timeout=timeout)
    assert r.returncode == 0, r.stdout + r.stderr
    return r.stdout


def test_host_mode(caller):
    out = _run(caller, "host", 60)
    assert "host: 0 failure(s)" in out


@pytest.mark.gpu
def test_gpu_mode(caller):
    import torch
    if not torch.cuda.is_available():
        pytest.skip("no CUDA device")
    out = _run(caller, "gpu", 600)
    assert "gpu: 0 failure(s)" in out
    assert out.count("ok   ") == 12, out


@pytest.mark.gpu
def test_time_mode(caller):
    """The C++ timing of BASELINE config 1 runs and reports a per-call time (no threshold: it is a
    measurement, not a check)."""
    import re

    import torch
    if not torch.cuda.is_available():
        pytest.skip("no CUDA device")
    out = _run(caller, "time", 120)
    m = re.search(r"cfg1 back-to-back from C\+\+: ([0-9.]+) us per call", out)
    assert m and float(m.group(1)) > 0, out
    assert "time: 0 failure(s)" in out
