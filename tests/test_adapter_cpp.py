"""The C++ host adapter (sixi-asi_b200/host/sixi_sampler.hpp) and its C++ parity tests.

On CPU the test programs are compiled (not linked), which checks that the header-only adapter
builds against the C ABI header. On a GPU they are linked and run, and every check must pass:
  tests/cpp/test_adapter.cpp    against the oracle port (liboracle.so)
  tests/cpp/test_spec_step.cpp  verify() against the engine's own SpeculativeDecoder::step, run by
                                the reference build (oracle/_ref/libsixiref.so) with the engine's RNG
"""

from __future__ import annotations

import os
import subprocess
from pathlib import Path

import pytest

from conftest import REPO, has_gpu

CUDA = Path(os.environ.get("CUDA_HOME", "/usr/local/cuda"))
SRC = REPO / "tests" / "cpp" / "test_adapter.cpp"
SRC_STEP = REPO / "tests" / "cpp" / "test_spec_step.cpp"
INC = ["-I", str(REPO / "include"), "-I", str(REPO / "sixi-asi_b200" / "host"), "-I", str(CUDA / "include")]
CXX = ["g++", "-std=c++17", "-O2", "-Wall", "-Wextra"]


@pytest.mark.parametrize("src", [SRC, SRC_STEP], ids=["adapter", "spec_step"])
def test_adapter_compiles(tmp_path, src):
    obj = tmp_path / (src.stem + ".o")
    r = subprocess.run([*CXX, *INC, "-c", str(src), "-o", str(obj)], capture_output=True, text=True)
    assert r.returncode == 0, r.stderr
    assert "warning" not in r.stderr, r.stderr


@pytest.mark.gpu
def test_adapter_parity_on_gpu(tmp_path):
    if not has_gpu():
        pytest.skip("no CUDA device")
    import sixi_smp
    from oracle import binding

    lib = Path(sixi_smp.LIB_PATH)
    assert lib.exists(), "libsixi_smp.so not built"
    binding.port()  # builds liboracle.so when missing
    exe = tmp_path / "test_adapter"
    libdirs = [lib.parent, REPO / "oracle", CUDA / "lib64"]
    cmd = [*CXX, *INC, str(SRC), "-o", str(exe)]
    for d in libdirs:
        cmd += ["-L", str(d), f"-Wl,-rpath,{d}"]
    cmd += ["-lsixi_smp", "-loracle", "-lcudart"]
    r = subprocess.run(cmd, capture_output=True, text=True)
    assert r.returncode == 0, r.stderr
    r = subprocess.run([str(exe)], capture_output=True, text=True, timeout=600)
    print(r.stdout)
    assert r.returncode == 0, r.stdout + r.stderr


@pytest.mark.gpu
def test_adapter_verify_equals_engine_step_on_gpu(tmp_path):
    if not has_gpu():
        pytest.skip("no CUDA device")
    import sixi_smp
    from oracle import binding

    lib = Path(sixi_smp.LIB_PATH)
    assert lib.exists(), "libsixi_smp.so not built"
    ref = binding.REF_PATH
    if not ref.exists():
        pytest.skip("reference build (oracle/_ref) absent")
    exe = tmp_path / "test_spec_step"
    libdirs = [lib.parent, ref.parent, CUDA / "lib64"]
    cmd = [*CXX, *INC, str(SRC_STEP), "-o", str(exe)]
    for d in libdirs:
        cmd += ["-L", str(d), f"-Wl,-rpath,{d}"]
    cmd += ["-lsixi_smp", "-lsixiref", "-lcudart"]
    r = subprocess.run(cmd, capture_output=True, text=True)
    assert r.returncode == 0, r.stderr
    r = subprocess.run([str(exe)], capture_output=True, text=True, timeout=900)
    print(r.stdout)
    assert r.returncode == 0, r.stdout + r.stderr
