"""The structural:: C++ shim (cove-spmv_b200/include/structural/) compiled
against libcove_b200.so: a compile check on any machine, and the C++ test
program tests/cpp/test_shim.cu run on the GPU."""
import os
import shutil
import subprocess

import pytest

ROOT = os.path.abspath(os.path.join(os.path.dirname(__file__), ".."))
SRC = os.path.join(ROOT, "tests", "cpp", "test_shim.cu")
OUT_DIR = os.path.join(ROOT, "tests", "cpp", "_build")
BIN = os.path.join(OUT_DIR, "test_shim")
LIBDIR = os.path.join(ROOT, "cove-spmv_b200", "cove_b200")


def _build():
    nvcc = shutil.which("nvcc") or "/usr/local/cuda/bin/nvcc"
    os.makedirs(OUT_DIR, exist_ok=True)
    cmd = [nvcc, "-O2", "-std=c++17", "-gencode", "arch=compute_100a,code=sm_100a",
           "-I" + os.path.join(ROOT, "include"), "-I" + os.path.join(ROOT, "cove-spmv_b200", "include"),
           SRC, "-o", BIN, "-L" + LIBDIR, "-lcove_b200", "-Xlinker", "-rpath," + LIBDIR]
    subprocess.run(cmd, check=True, capture_output=True, text=True)


def _stale():
    if not os.path.exists(BIN):
        return True
    t = os.path.getmtime(BIN)
    deps = [SRC, os.path.join(LIBDIR, "libcove_b200.so"),
            os.path.join(ROOT, "tests", "cpp", "codec_golden.inc")]
    inc = os.path.join(ROOT, "cove-spmv_b200", "include", "structural")
    for dp, _, fs in os.walk(inc):
        deps += [os.path.join(dp, f) for f in fs]
    return any(os.path.getmtime(d) > t for d in deps if os.path.exists(d))


@pytest.mark.skipif(not (shutil.which("nvcc") or os.path.exists("/usr/local/cuda/bin/nvcc")),
                    reason="nvcc not available")
def test_shim_compiles_against_the_library():
    if _stale():
        _build()
    assert os.path.exists(BIN)


@pytest.mark.gpu
def test_shim_program_passes_on_gpu():
    if _stale():
        _build()
    r = subprocess.run([BIN], capture_output=True, text=True, timeout=300)
    assert r.returncode == 0, r.stderr + r.stdout
    assert "shim tests passed" in r.stdout
