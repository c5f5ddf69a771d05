"""The oracle's restatement of the seeded benchmark inputs
(oracle/oracle_workloads.c) gives the same arrays as the library's host
generators (include/cove_synth.h): the reference arm of the benchmark builds
its input from the former, the GPU arm from the latter."""
import numpy as np

import cove_b200 as cb
import oracle as O


def _same(a, b):
    assert len(a) == len(b)
    for u, v in zip(a, b):
        assert u.dtype.kind == v.dtype.kind and np.array_equal(np.asarray(u, v.dtype), v)


def test_lapl3d_rows_match():
    for (nx, ny, nz, rb, re, sh) in ((7, 5, 6, 0, 210, 0), (16, 16, 16, 256, 1280, 0),
                                     (12, 10, 9, 240, 960, 120)):
        rows, n, rp, ci, v = cb.synth_lapl3d(nx, ny, nz, rb, re, sh)
        _same(O.lapl3d_rows(nx, ny, nz, rb, re, sh), (rp, ci, v))


def test_lapl2d_matches():
    rows, n, rp, ci, v = cb.synth_lapl2d(33, 17)
    _same(O.lapl2d(33, 17), (rp, ci, v))


def test_fem27_rows_match():
    nx, ny, nz, dof = 6, 5, 4, 3
    n = nx * ny * nz * dof
    for (rb, re, sh) in ((0, n, 0), (90, 270, 60)):
        rows, _, rp, ci, v = cb.synth_fem27_rows(nx, ny, nz, dof, 1, rb, re, sh)
        _same(O.fem27_rows(nx, ny, nz, dof, 1, rb, re, sh), (rp, ci, v))


def test_vectors_match():
    for kind, seed in (("uniform_pm1", 4), ("uniform01", 2), ("normal", 3)):
        ref = cb.synth_vector(kind, 5000, seed=seed)
        assert np.array_equal(O.vector(kind, seed, 7, 0, 5000), ref)
        assert np.array_equal(O.vector(kind, seed, 7, 1234, 100), ref[1234:1334])


def test_blocksparse_rows_match():
    g = dict(p_block=0.05, p_entry=0.6, outlier_fraction=0.01, seed=11)
    for (n, rb, re) in ((4099, 0, 4099), (4099, 1024, 2048), (4099, 4096, 4099), (1 << 14, 8, 4000)):
        rp, ci, v = cb.synth_blocksparse_rows(n, rb, re, **g)
        _same(O.blocksparse_rows(n, rb, re, **g), (rp, ci, v))
    rows, _, rp, ci, v = cb.synth_blocksparse(1 << 14)  # the bench's default densities, scaled
    _same(O.blocksparse_rows(1 << 14, 0, 1 << 14), (rp, ci, v))


def test_rmat_matches():
    for scale, ef in ((10, 16), (14, 8)):
        _, _, rp, ci, v = cb.synth_rmat(scale, ef, seed=2)
        _same(O.rmat(scale, ef, seed=2), (rp, ci, v))
