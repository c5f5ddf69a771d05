"""Golden family value-codec payloads from the reference's own builders.

Runs oracle/_ref/ref_codec_golden (oracle/ref_codec_golden.cu, compiled by
oracle/Makefile against the reference headers) and writes its output to
tests/cpp/codec_golden.inc, the expected payloads tests/cpp/test_shim.cu
compares the shim's builders against.

    make -C oracle && python tests/golden/make_codec_golden.py
"""
import os
import subprocess

HERE = os.path.dirname(os.path.abspath(__file__))
ROOT = os.path.join(HERE, "..", "..")


def main():
    out = subprocess.run([os.path.join(ROOT, "oracle", "_ref", "ref_codec_golden")],
                         capture_output=True, text=True, check=True).stdout
    path = os.path.join(ROOT, "tests", "cpp", "codec_golden.inc")
    with open(path, "w") as f:
        f.write(out)
    print(f"wrote {path} ({len(out)} bytes)")


if __name__ == "__main__":
    main()
