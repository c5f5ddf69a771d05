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


# ---- on a GPU: the reference's own GPU converter test and family runner ----------

@pytest.mark.gpu
def test_reference_gpu_convert_test_passes_on_shim():
    """structural/tests/test_gpu_convert.cu (the GPU converter against the
    CPU converter, the work-item KATs, the family SpMV cases) built against
    the shim: all its checks pass on this library."""
    p = subprocess.run([_bin("test_gpu_convert")], capture_output=True, text=True, timeout=600)
    assert p.returncode == 0, (p.stdout[-2000:], p.stderr[-2000:])
    assert "SKIP" not in p.stderr


@pytest.mark.gpu
@pytest.mark.parametrize("case", __import__("test_family_cli").REF_CASES,
                         ids=[c[0] for c in __import__("test_family_cli").REF_CASES])
def test_reference_family_runner_on_shim(ref_mats, case):
    """The reference's family runner (structural/src/main_gpu_spmv.cu) built
    against the shim answers the reference CLI test's cases
    (structural/tests/test_gpu_spmv_cli.sh) with the same report keys as
    this repository's own struct_gpu_spmv."""
    fam = __import__("test_family_cli")
    cid, mat, args, expected = case
    p = subprocess.run([_bin("main_gpu_spmv"), str(ref_mats[mat]), *args, "--warmup", "0", "--iters", "1",
                        "--verify-cpu"], capture_output=True, text=True, timeout=300)
    assert p.returncode == 0, p.stderr
    d = fam.parse(p.stdout)
    assert d["report_schema"] == "structural_spmv_cli_v3" and d["verify_cpu"].startswith("PASS,")
    assert {k: d.get(k) for k in expected} == expected


from test_family_cli import ref_mats  # noqa: E402,F401  (the reference CLI test's five matrices)
