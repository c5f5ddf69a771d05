"""The reference's own tests and drivers built unchanged against this
repository's structural:: shim and libcove_b200 (oracle/Makefile, the
refshim_* programs in oracle/_ref): its option-handling test passes on
CPU, and its CG bench, convert CLI and family runner load the library and
answer without a GPU.  Its GPU converter test, refshim_test_gpu_convert, builds the same
way; it needs a GPU.  These programs exist only where the reference
checkout was present at build time."""
import os
import subprocess

import pytest

ROOT = os.path.abspath(os.path.join(os.path.dirname(__file__), ".."))
REF = os.path.join(ROOT, "oracle", "_ref")
NAMES = ("test_spmv_cli_options", "test_gpu_convert", "bench_cg_solve", "main_gpu_convert", "main_gpu_spmv")

pytestmark = pytest.mark.skipif(not os.path.exists(os.path.join(REF, "libcove_ref.so")),
                                reason="built only where the reference checkout exists")


def _bin(name):
    return os.path.join(REF, "refshim_" + name)


def test_reference_programs_build_on_shim():
    missing = [n for n in NAMES if not os.path.exists(_bin(n))]
    assert not missing, missing


def test_reference_cli_options_test_passes_on_shim():
    p = subprocess.run([_bin("test_spmv_cli_options")], capture_output=True, text=True, timeout=120)
    assert p.returncode == 0, p.stderr
    assert "spmv cli options tests passed" in p.stdout + p.stderr


def test_reference_drivers_load_the_library():
    p = subprocess.run([_bin("bench_cg_solve")], capture_output=True, text=True, timeout=60)
    assert p.returncode == 2 and "usage:" in p.stderr and "synth:N:halfbw:delta" in p.stderr
    p = subprocess.run([_bin("main_gpu_convert")], capture_output=True, text=True, timeout=60)
    assert p.returncode == 2 and "usage:" in p.stderr and "--mode warp_direct" in p.stderr
    # the reference's family runner: its options now go through the shim's parser
    p = subprocess.run([_bin("main_gpu_spmv")], capture_output=True, text=True, timeout=60)
    assert p.returncode == 2 and "usage:" in p.stderr and "global_logkmeans128" in p.stderr
    p = subprocess.run([_bin("main_gpu_spmv"), "m.mtx", "--layout", "sell"], capture_output=True, text=True,
                       timeout=60)
    assert p.returncode != 0 and "layout must be col_bitmap64, col_bitmap64_flag_lb, or cusparse_csr" in p.stderr
