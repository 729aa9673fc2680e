"""The C++ host API (include/b4gemv.hpp), compiled with g++ and linked to
libb4gemv.so, reproduces the reference's quantise()/quantise_nf4() bytes on the
reference benchmark's own glibc inputs.  CPU only."""
from __future__ import annotations

import os
import shutil
import subprocess

import numpy as np
import pytest

ROOT = os.path.dirname(os.path.dirname(os.path.abspath(__file__)))
LIBDIR = os.path.join(ROOT, "int4-gemv_b200", "lib")


@pytest.mark.skipif(shutil.which("g++") is None, reason="no g++")
def test_cpp_header_matches_reference_fixture(tmp_path, golden):
    exe = str(tmp_path / "api_check")
    subprocess.run(["g++", "-std=c++17", "-O2", f"-I{ROOT}/include", "-I/usr/local/cuda/include",
                    os.path.join(ROOT, "tests", "cpp", "api_check.cpp"), f"-L{LIBDIR}", "-lb4gemv",
                    f"-Wl,-rpath,{LIBDIR}", "-o", exe], check=True)
    out = subprocess.run([exe], check=True, capture_output=True, text=True).stdout.splitlines()
    rows = {line.split()[0]: line.split()[1:] for line in out}
    g = golden["kat_glibc"]
    assert [int(v, 16) for v in rows["int4_packed"]] == [int(v) for v in g["int4_packed"].ravel()]
    assert [int(v, 16) for v in rows["int4_scales"]] == [int(v) for v in g["int4_scales"].ravel()]
    assert [int(v, 16) for v in rows["nf4_packed"]] == [int(v) for v in g["nf4_packed"].ravel()]
    assert [int(v, 16) for v in rows["nf4_absmax"]] == [int(v) for v in g["nf4_absmax"].ravel().view(np.uint32)]
    assert rows["median"] == ["3"]
    assert rows["bad_shape"] == ["status", "1"]
