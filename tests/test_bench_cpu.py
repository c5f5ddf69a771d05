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
    assert (d["metric"], d["scaling"], d["unit"]) == ("cg_spmv_gflops", "strong", "GFLOP/s")
    assert d["value"] > 0 and "planes [0, 8)" in d["config"]["workload"]
