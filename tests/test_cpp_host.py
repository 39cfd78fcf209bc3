"""The C++ face of the ABI (include/gdr.hpp): it compiles against the headers
and library, throws on bunsen's contract violations without a GPU, and on a
GPU its chunked and recurrent forms agree (f32, 1e-4)."""

from __future__ import annotations

import subprocess

import pytest

from bunsen_b200 import _lib
from tests.conftest import ROOT


@pytest.fixture(scope="module")
def exe(tmp_path_factory):
    out = tmp_path_factory.mktemp("cpp") / "rule_cpp"
    lib = _lib.LIB_PATH
    cmd = ["g++", "-std=c++17", "-O1", "-I", str(ROOT / "include"), "-I", "/usr/local/cuda/include",
           str(ROOT / "tests" / "cpp" / "rule_cpp.cpp"), "-o", str(out), str(lib),
           f"-Wl,-rpath,{lib.parent}", "-L/usr/local/cuda/lib64", "-lcudart"]
    subprocess.run(cmd, check=True)
    return out


def test_contracts_throw_like_bunsens_panics(exe):
    res = subprocess.run([str(exe), "contracts"], capture_output=True, text=True)
    assert res.returncode == 0, res.stdout + res.stderr


@pytest.mark.gpu
def test_cpp_chunked_matches_recurrent_on_gpu(exe):
    res = subprocess.run([str(exe), "parity"], capture_output=True, text=True)
    assert res.returncode == 0, res.stdout + res.stderr
