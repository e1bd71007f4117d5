"""The C++ host API (include/smoe.hpp: FfnExec::load / run, Stack) compiled with g++ against libsmoe.so: the
refused arguments on CPU, and on a GPU the same results as the C ABI bit for bit (tests/cpp/ffn_exec_test.cpp)."""
import os
import subprocess
from pathlib import Path

import pytest

from stratametal_b200 import _lib, build

ROOT = Path(__file__).resolve().parents[1]
CUDA = Path(os.environ.get("CUDA_HOME", "/usr/local/cuda"))


@pytest.fixture(scope="module")
def exe(tmp_path_factory):
    build.build()
    out = tmp_path_factory.mktemp("cpp") / "ffn_exec_test"
    so = _lib.lib_path()
    cmd = ["g++", "-std=c++17", "-O2", "-I", str(ROOT / "include"), "-I", str(CUDA / "include"),
           str(ROOT / "tests" / "cpp" / "ffn_exec_test.cpp"), "-o", str(out), str(so),
           f"-Wl,-rpath,{so.parent}", "-L", str(CUDA / "lib64"), "-lcudart"]
    r = subprocess.run(cmd, capture_output=True, text=True)
    assert r.returncode == 0, r.stderr
    return out


def test_cpp_refusals(exe):
    r = subprocess.run([str(exe)], capture_output=True, text=True, timeout=120)
    assert r.returncode == 0, r.stdout + r.stderr
    assert "refusals: ok" in r.stdout


@pytest.mark.gpu
def test_cpp_ffn_exec_and_stack(exe):
    import torch
    if not torch.cuda.is_available():
        pytest.skip("no CUDA device")
    r = subprocess.run([str(exe), "run"], capture_output=True, text=True, timeout=300)
    assert r.returncode == 0, r.stdout + r.stderr
    assert "run: ok" in r.stdout


def test_cpp_residency_rules(tmp_path):
    # host only: the admission rules of the VRAM expert tier (include/smoe_stream.hpp)
    out = tmp_path / "stream_test"
    cmd = ["g++", "-std=c++17", "-O2", "-I", str(ROOT / "include"), "-I", str(CUDA / "include"),
           str(ROOT / "tests" / "cpp" / "stream_test.cpp"), "-o", str(out), "-L", str(CUDA / "lib64"), "-lcudart",
           str(_lib.lib_path()), f"-Wl,-rpath,{_lib.lib_path().parent}"]
    r = subprocess.run(cmd, capture_output=True, text=True)
    assert r.returncode == 0, r.stderr
    r = subprocess.run([str(out)], capture_output=True, text=True, timeout=60)
    assert r.returncode == 0, r.stdout + r.stderr
    assert "residency: ok" in r.stdout
