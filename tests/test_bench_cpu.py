"""bench.py's reference arm (CPU only): the JSON line's keys and the
non-zero-rank behaviour under torchrun.  The timed CPU SpMV is the
reference's own spmv_csr when oracle/_ref is built, else the oracle port."""
import json
import os
import subprocess
import sys

ROOT = os.path.abspath(os.path.join(os.path.dirname(__file__), ".."))


def run_bench(*args, env=None):
    e = dict(os.environ)
    e.update(env or {})
    p = subprocess.run([sys.executable, os.path.join(ROOT, "bench.py"), *args], capture_output=True,
                       text=True, timeout=600, env=e, cwd=ROOT)
    return p.returncode, p.stdout, p.stderr


def test_reference_arm_prints_one_contract_line():
    rc, out, err = run_bench("--impl", "reference", "--workload", "lapl2d_512", "--steps", "2",
                             "--warmup", "3")
    assert rc == 0, err
    lines = [ln for ln in out.splitlines() if ln.strip()]
    assert len(lines) == 1
    d = json.loads(lines[0])
    for k in ("metric", "value", "unit", "n_gpus", "steps", "warmup", "ms_per_step", "higher_is_better",
              "scaling", "vs_baseline", "dtype", "data", "config", "cpu_baseline", "e2e"):
        assert k in d, k
    assert d["impl"] == "reference" and d["metric"] == "spmv_gflops" and d["unit"] == "GFLOP/s"
    assert d["value"] > 0 and d["steps"] == 2 and d["warmup"] == 3 and d["higher_is_better"] is True
    assert d["dtype"] == "f64" and d["config"]["workload"].startswith("lapl2d_512")
    cpu = d["cpu_baseline"]
    assert cpu["kind"] in ("reference", "port") and cpu["cores"] >= 1 and cpu["value"] == d["value"]
    assert d["e2e"] == {"value": d["value"], "unit": "GFLOP/s", "h2d_bytes_per_step": 0,
                        "d2h_bytes_per_step": 0}


def test_reference_arm_other_ranks_exit_quietly():
    rc, out, err = run_bench("--impl", "reference", "--workload", "lapl2d_512", "--steps", "1",
                             env={"RANK": "1", "WORLD_SIZE": "2", "LOCAL_RANK": "1"})
    assert rc == 0, err
    assert out.strip() == ""


def test_reference_arm_for_the_cg_workload_uses_its_metric():
    rc, out, err = run_bench("--impl", "reference", "--workload", "lapl3d_cg", "--grid", "32", "--steps", "1",
                             "--warmup", "3")
    assert rc == 0, err
    d = json.loads(out.strip().splitlines()[-1])
    assert (d["metric"], d["scaling"], d["unit"]) == ("spmv_gflops", "strong", "GFLOP/s")
    assert d["value"] > 0 and d["config"]["workload"].startswith("3D 7-point Laplacian 32^3")
    assert "planes [0, 8)" in d["cpu_baseline"]["sample"]


def test_default_workload_is_the_cg_strong_scaling_config():
    import bench

    args = bench.argparse.Namespace(workload="lapl3d_cg", grid=0, cg_iters=50, bs_n=0)
    cfg = bench.bench_config(args)
    assert cfg["workload"] == ("3D 7-point Laplacian 768^3 (n=452984832, nnz=3167354880), "
                               "50 textbook CG iterations per step")
    assert bench.lapl3d_nnz(768) == 3167354880


def test_reference_arm_never_loads_the_library_and_uses_every_core():
    """The reference arm builds its input with the oracle's generators, so the
    product library is never mapped into its process; OpenMP gets every core
    even when a launcher set OMP_NUM_THREADS=1."""
    code = (
        "import sys, json, argparse; sys.path.insert(0, '.'); import bench;"
        "a = argparse.Namespace(workload='lapl3d_cg', grid=24, cg_iters=50, bs_n=0, steps=1, warmup=1);"
        "bench.run_reference_arm(a);"
        "maps = open('/proc/self/maps').read();"
        "print(json.dumps({'lib': 'libcove_b200' in maps, 'mod': 'cove_b200' in sys.modules}))"
    )
    e = dict(os.environ, OMP_NUM_THREADS="1")
    p = subprocess.run([sys.executable, "-c", code], capture_output=True, text=True, timeout=300, env=e, cwd=ROOT)
    assert p.returncode == 0, p.stderr
    lines = [ln for ln in p.stdout.splitlines() if ln.strip()]
    line, probe = json.loads(lines[0]), json.loads(lines[-1])
    assert probe == {"lib": False, "mod": False}
    if line["cpu_baseline"]["kind"] == "reference":
        assert line["cpu_baseline"]["cores"] == len(os.sched_getaffinity(0))
