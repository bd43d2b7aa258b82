"""The C ABI from C++: tests/abi_driver.cpp built with g++ against include/fvsr_lcsa.h and the in-tree
libfvsr_lcsa.so (the way a Swift or C++ host links it). The CPU mode checks host-side validation and status codes;
the GPU mode runs a small layer (selection with and without a workspace, attention, the streaming forward)."""
from __future__ import annotations

import shutil
import subprocess
from pathlib import Path

import pytest

ROOT = Path(__file__).resolve().parents[1]
CUDA = Path("/usr/local/cuda")


@pytest.fixture(scope="module")
def driver(fvsr, tmp_path_factory):
    gxx = shutil.which("g++")
    if gxx is None or not (CUDA / "include" / "cuda_runtime.h").exists():
        pytest.skip("g++ or the CUDA headers are missing")
    lib_dir = Path(fvsr.LIB_PATH).parent
    exe = tmp_path_factory.mktemp("abi") / "abi_driver"
    cmd = [gxx, "-std=c++17", "-O1", "-Wall", "-I", str(ROOT / "include"), "-I", str(CUDA / "include"),
           str(ROOT / "tests" / "abi_driver.cpp"), "-o", str(exe), "-L", str(lib_dir), "-lfvsr_lcsa",
           f"-Wl,-rpath,{lib_dir}", "-L", str(CUDA / "lib64"), "-lcudart", f"-Wl,-rpath,{CUDA / 'lib64'}"]
    subprocess.run(cmd, check=True, capture_output=True, text=True)
    return exe


def test_abi_driver_host_validation(driver):
    r = subprocess.run([str(driver), "cpu"], capture_output=True, text=True, timeout=120)
    assert r.returncode == 0 and "ok cpu" in r.stdout, r.stdout + r.stderr


@pytest.mark.gpu
def test_abi_driver_small_layer_on_gpu(driver):
    r = subprocess.run([str(driver), "gpu"], capture_output=True, text=True, timeout=300)
    assert r.returncode == 0 and "ok gpu" in r.stdout, r.stdout + r.stderr
