"""The C++ vocab-sharded step (sixi-asi_b200/host/sixi_sharded.hpp, NCCL C API) and its C++ test.

On CPU the test program is compiled (not linked), which checks the header against the C ABI and
NCCL headers. On a GPU it is linked against libsixi_smp.so, NCCL and cudart and run: one rank per
GPU as threads (S = 1 always, S = 2 with two or more GPUs); every rank's tokens and statuses must
equal the stages composed on one GPU (tests/cpp/test_sharded.cpp).
"""

from __future__ import annotations

import os
import subprocess
from pathlib import Path

import pytest

from conftest import REPO, has_gpu

CUDA = Path(os.environ.get("CUDA_HOME", "/usr/local/cuda"))
SRC = REPO / "tests" / "cpp" / "test_sharded.cpp"
INC = ["-I", str(REPO / "include"), "-I", str(REPO / "sixi-asi_b200" / "host"), "-I", str(CUDA / "include")]
CXX = ["g++", "-std=c++17", "-O2", "-Wall", "-Wextra"]


def test_sharded_step_compiles(tmp_path):
    r = subprocess.run([*CXX, *INC, "-c", str(SRC), "-o", str(tmp_path / "t.o")], capture_output=True, text=True)
    assert r.returncode == 0, r.stderr
    assert "warning" not in r.stderr, r.stderr


@pytest.mark.gpu
def test_sharded_step_over_nccl_on_gpu(tmp_path):
    if not has_gpu():
        pytest.skip("no CUDA device")
    import sixi_smp

    lib = Path(sixi_smp.LIB_PATH)
    assert lib.exists(), "libsixi_smp.so not built"
    exe = tmp_path / "test_sharded"
    cmd = [*CXX, *INC, str(SRC), "-o", str(exe)]
    for d in (lib.parent, CUDA / "lib64"):
        cmd += ["-L", str(d), f"-Wl,-rpath,{d}"]
    cmd += ["-lsixi_smp", "-lnccl", "-lcudart", "-lpthread"]
    r = subprocess.run(cmd, capture_output=True, text=True)
    assert r.returncode == 0, r.stderr
    env = dict(os.environ, NCCL_NVLS_ENABLE="0")
    r = subprocess.run([str(exe)], capture_output=True, text=True, timeout=600, env=env)
    print(r.stdout)
    assert r.returncode == 0, r.stdout + r.stderr
