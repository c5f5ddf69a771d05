"""Golden MatrixMarket cases from the reference's own loader.

Runs structural::read_matrix_market_with_info (matrix_market.hpp:327-382,
compiled into oracle/_ref/libcove_ref.so by oracle/Makefile) on small
coordinate files and stores the file texts with the CSR it returns, or the
error message it raises, in tests/golden/mm_cases.npz.  Duplicate entries
use values whose sums are exact, so the result does not depend on the order
in which the reference's (unstable) row sort meets them.

    python tests/golden/make_mm_golden.py
"""
import ctypes as C
import os
import tempfile

import numpy as np

HERE = os.path.dirname(os.path.abspath(__file__))
REF = os.path.join(HERE, "..", "..", "oracle", "_ref", "libcove_ref.so")

CASES = {
    "general_real_dups": (8, "%%MatrixMarket matrix coordinate real general\n"
                          "% a comment\n"
                          "5 6 9\n"
                          "1 1 1.5\n"
                          "3 2 -2.25\n"
                          "1 6 0.125\n"
                          "\n"
                          "3 2 0.5\n"
                          "% between entries\n"
                          "5 5 7\n"
                          "3 2 1.0\n"
                          "2 4 3.0e-3\n"
                          "4 1 0.1\n"
                          "4 1 0.2\n"),
    "symmetric_real": (8, "%%MatrixMarket matrix coordinate real symmetric\n"
                       "4 4 5\n"
                       "1 1 4.0\n"
                       "2 1 -1.0\n"
                       "3 2 -1.5\n"
                       "4 4 2.0\n"
                       "4 1 0.3333333333333333\n"),
    "skew_real": (8, "%%MatrixMarket matrix coordinate real skew-symmetric\n"
                  "3 3 2\n"
                  "2 1 1.25\n"
                  "3 1 -0.5\n"),
    "pattern_general": (8, "%%MatrixMarket matrix coordinate pattern general\n"
                        "3 4 4\n"
                        "1 2\n"
                        "3 4\n"
                        "2 1\n"
                        "1 2\n"),
    "pattern_symmetric": (8, "%%MatrixMarket matrix coordinate pattern symmetric\n"
                          "3 3 3\n"
                          "1 1\n"
                          "3 1\n"
                          "2 2\n"),
    "integer_upper_banner": (8, "%%MATRIXMARKET Matrix Coordinate Integer General\n"
                             "2 3 3\n"
                             "1 3 7\n"
                             "2 1 -2\n"
                             "2 2 0\n"),
    "cancel_to_zero": (8, "%%MatrixMarket matrix coordinate real general\n"
                       "2 2 4\n"
                       "1 1 2.5\n"
                       "1 1 -2.5\n"
                       "2 2 1.0\n"
                       "1 2 0.0\n"),
    "crlf_extra_lines": (8, "%%MatrixMarket matrix coordinate real general\r\n"
                         "2 2 2\r\n"
                         "1 2 3.5\r\n"
                         "2 1 -1.0\r\n"
                         "2 2 9.0\r\n"),
    "general_f32": (4, "%%MatrixMarket matrix coordinate real general\n"
                    "3 3 4\n"
                    "1 1 0.1\n"
                    "2 3 3.141592653589793\n"
                    "3 2 1e-40\n"
                    "2 3 1.0\n"),
    "err_out_of_range": (8, "%%MatrixMarket matrix coordinate real general\n"
                         "2 2 1\n"
                         "3 1 1.0\n"),
    "err_short": (8, "%%MatrixMarket matrix coordinate real general\n"
                  "2 2 3\n"
                  "1 1 1.0\n"),
    "err_complex": (8, "%%MatrixMarket matrix coordinate complex general\n"
                    "1 1 1\n"
                    "1 1 1.0 2.0\n"),
    "err_array": (8, "%%MatrixMarket matrix array real general\n"
                  "1 1\n"
                  "1.0\n"),
    "err_missing_value": (8, "%%MatrixMarket matrix coordinate real general\n"
                          "1 1 1\n"
                          "1 1\n"),
}


def main():
    lib = C.CDLL(REF)
    lib.ref_mm_read.restype = C.c_int64
    lib.ref_mm_read.argtypes = [C.c_char_p, C.c_int32, C.c_void_p, C.c_void_p, C.c_void_p,
                                C.c_void_p, C.c_void_p, C.c_void_p]
    lib.ref_last_error.restype = C.c_char_p
    out = {}
    with tempfile.TemporaryDirectory() as d:
        for name, (esz, text) in CASES.items():
            path = os.path.join(d, name + ".mtx")
            with open(path, "w", newline="") as f:
                f.write(text)
            shape = np.zeros(2, np.int32)
            fs = np.zeros(2, np.int32)
            counts = np.zeros(3, np.int64)
            args = [path.encode(), esz, shape.ctypes.data, fs.ctypes.data, counts.ctypes.data]
            nnz = lib.ref_mm_read(*args, None, None, None)
            out[f"{name}/text"] = np.frombuffer(text.encode(), np.uint8)
            out[f"{name}/esz"] = np.array([esz])
            if nnz < 0:
                out[f"{name}/error"] = np.frombuffer(lib.ref_last_error(), np.uint8)
                continue
            rp = np.zeros(shape[0] + 1, np.int32)
            ci = np.zeros(max(nnz, 1), np.int32)
            v = np.zeros(max(nnz, 1), np.float64 if esz == 8 else np.float32)
            lib.ref_mm_read(*args, rp.ctypes.data, ci.ctypes.data, v.ctypes.data)
            out[f"{name}/shape"] = shape
            out[f"{name}/field_symmetry"] = fs
            out[f"{name}/counts"] = counts
            out[f"{name}/row_ptr"] = rp
            out[f"{name}/col_idx"] = ci[:nnz]
            out[f"{name}/values"] = v[:nnz]
    np.savez_compressed(os.path.join(HERE, "mm_cases.npz"), **out)
    print(f"wrote {len(CASES)} cases")


if __name__ == "__main__":
    main()
