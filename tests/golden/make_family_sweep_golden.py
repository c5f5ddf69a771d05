"""Writes tests/golden/family_sweep_commands.json: the command lines the
reference's structural/scripts/run_gpu_spmv_family_sweep.py builds for every
operator of its catalog (DEFAULT_OPERATORS), in fp64 and fp32, with the
binary directory and the matrix as placeholders ("BIN/...", "MATRIX").
The script is imported from the reference checkout, as the reference's own
tests/test_gpu_spmv_family_sweep.py does.
Usage: [REF_ROOT=<reference checkout>] python tests/golden/make_family_sweep_golden.py
"""
import importlib.util
import json
import os
from pathlib import Path
from types import SimpleNamespace

ROOT = os.path.abspath(os.path.join(os.path.dirname(__file__), "..", ".."))
REF_ROOT = os.environ.get("REF_ROOT", "/root/reference")  # the reference checkout, as oracle/Makefile
SCRIPT = Path(REF_ROOT) / "structural/scripts/run_gpu_spmv_family_sweep.py"


def main():
    spec = importlib.util.spec_from_file_location("family_sweep", SCRIPT)
    sweep = importlib.util.module_from_spec(spec)
    spec.loader.exec_module(sweep)
    rows = []
    for precision in ("double", "float"):
        args = SimpleNamespace(bin="BIN/struct_gpu_spmv", hybrid_bin=None, precision=precision, warmup=1, iters=2,
                               cusparse_alg="default", verify_cpu=True)
        for op in sweep.DEFAULT_OPERATORS:
            rows.append({"operator": op.name, "precision": precision,
                         "argv": sweep.make_command(args, Path("MATRIX"), op)})
    path = os.path.join(ROOT, "tests", "golden", "family_sweep_commands.json")
    with open(path, "w") as f:
        json.dump(rows, f, indent=1)
        f.write("\n")
    print(f"wrote {path}: {len(rows)} commands")


if __name__ == "__main__":
    main()
