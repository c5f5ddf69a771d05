"""Every per-codec operator wrapper of the shim (structural/gpu_spmv.cuh)
instantiates for fp64 and fp32 with the reference's parameter lists
(tests/cpp/shim_wrappers_compile.cu, compiled only)."""
import os
import subprocess

ROOT = os.path.abspath(os.path.join(os.path.dirname(__file__), ".."))


def test_operator_wrappers_compile(tmp_path):
    src = os.path.join(ROOT, "tests", "cpp", "shim_wrappers_compile.cu")
    p = subprocess.run(["nvcc", "-c", "-std=c++17", "-gencode", "arch=compute_100a,code=sm_100a",
                        "-I" + os.path.join(ROOT, "cove-spmv_b200", "include"), "-I" + os.path.join(ROOT, "include"),
                        "-o", str(tmp_path / "w.o"), src], capture_output=True, text=True, timeout=600)
    assert p.returncode == 0, p.stderr[-2000:]
