"""Pins the CPU oracle (oracle/) to the reference before anything is checked against it.

- The oracle's fp32 triple loop must give the same BITS as the reference's own test oracle
  (tests/reference_gemm.hpp, compiled from the reference sources into oracle/_ref/).
- The reference's production sgemm (AVX2 blocked, src/kernels/gemm.cpp:546) must agree with the
  oracle's fp64 evaluation within the reference's own tolerance (test_kernels.cpp:125-153).
- The committed golden vectors (tests/golden/, made by tests/golden/make_golden.py from the
  reference build) must be reproduced by the oracle; these run even where the reference build
  is absent (the GPU box).
"""
import itertools
import pathlib

import numpy as np
import pytest

from oracle import orc

GOLDEN = pathlib.Path(__file__).resolve().parent / "golden"
SIZES = [1, 7, 33, 257]
ref = orc.ref()
needs_ref = pytest.mark.skipif(ref is None, reason="reference library not built (oracle/_ref)")


def tol_ok(got, want64, mag, rel=1e-5, floor=1e-6):
    """test_kernels.cpp:139-146 with the fp64 result as truth."""
    got = got.astype(np.float64)
    nan_w, nan_g = np.isnan(want64), np.isnan(got)
    inf_w, inf_g = np.isinf(want64), np.isinf(got)
    if not np.array_equal(nan_w, nan_g):
        return False
    fin = ~(nan_w | inf_w | inf_g)
    if not np.array_equal(got[inf_w | inf_g], want64[inf_w | inf_g]):
        return False
    return bool(np.all(np.abs(got[fin] - want64[fin]) <= np.maximum(rel * mag[fin], floor)))


def c_view(p, c):
    return c[: p.m * p.ldc].reshape(p.m, p.ldc)[:, : p.n] if p.m else np.zeros((0, p.n), np.float32)


@needs_ref
def test_f32_loop_matches_reference_oracle_bitwise():
    seed = 1
    for ta, tb, acc in itertools.product((0, 1), repeat=3):
        for m, n, k in itertools.product(SIZES[:3], repeat=3):
            p = orc.Problem(ta, tb, m, n, k, 0, seed)
            seed += 1
            want = p.c.copy()
            ref.ref_reference_sgemm(*p.args(), orc.ptr(want), p.ldc, acc)
            got = orc.sgemm_f32(p, p.c, acc)
            assert got.tobytes() == want.tobytes(), (ta, tb, acc, m, n, k)


@needs_ref
def test_reference_sgemm_within_tolerance_of_fp64_oracle():
    seed = 4000
    for ta, tb, acc in itertools.product((0, 1), repeat=3):
        for m, n, k in [(1, 257, 33), (257, 7, 257), (33, 33, 257), (101, 7, 33), (7, 1029, 261)]:
            p = orc.Problem(ta, tb, m, n, k, 2, seed)
            seed += 1
            got = p.c.copy()
            ref.ref_sgemm(*p.args(), orc.ptr(got), p.ldc, acc)
            want = orc.sgemm_f64(p, p.c, acc)
            mag = orc.magnitude(p, p.c, acc)
            assert tol_ok(c_view(p, got), want, mag), (ta, tb, acc, m, n, k)
            # padding columns untouched
            pad = got[: p.m * p.ldc].reshape(p.m, p.ldc)[:, p.n:]
            assert np.all(pad == orc.SENTINEL)


@needs_ref
def test_inf_nan_problem_matches_reference_oracle_bitwise():
    """test_kernels.cpp:211-231: op(A)(2,0)=Inf, op(B) row 0 cycles 1,-1,0, op(B)(5,3)=NaN."""
    seed = 3000
    for ta, tb, acc in itertools.product((0, 1), repeat=3):
        p = make_inf_nan_problem(ta, tb, seed)
        seed += 1
        want = p.c.copy()
        ref.ref_reference_sgemm(*p.args(), orc.ptr(want), p.ldc, acc)
        got = orc.sgemm_f32(p, p.c, acc)
        assert np.array_equal(np.isnan(got), np.isnan(want))
        fin = ~np.isnan(want)
        assert np.array_equal(got[fin], want[fin])


def make_inf_nan_problem(ta, tb, seed):
    p = orc.Problem(ta, tb, 7, 33, 17, 0, seed)
    p.a[2 if ta else 2 * p.lda] = np.inf
    for j in range(p.n):
        p.b[j * p.ldb if tb else j] = (1.0, -1.0, 0.0)[j % 3]
    p.b[3 * p.ldb + 5 if tb else 5 * p.ldb + 3] = np.nan
    return p


def test_generators_follow_mt19937():
    """std::mt19937(5489) first output 3499211612 (the C++ standard's check value) feeds U[0,1)."""
    u = orc.uniform(5489, 3, 0.0, 1.0)
    assert abs(float(u[0]) - 3499211612 / 2**32) < 1e-7


def test_golden_vectors_reproduced_by_oracle():
    data = np.load(GOLDEN / "gemm_golden.npz")
    cases = data["cases"]
    assert len(cases) >= 8
    for idx, (ta, tb, m, n, k, pad, seed, acc) in enumerate(cases):
        p = orc.Problem(ta, tb, m, n, k, pad, seed)
        # inputs regenerate bit-exactly
        assert p.a.tobytes() == data[f"a{idx}"].tobytes()
        assert p.b.tobytes() == data[f"b{idx}"].tobytes()
        # the reference's triple loop output, bit for bit
        got = orc.sgemm_f32(p, p.c, acc)
        assert got.tobytes() == data[f"loop{idx}"].tobytes()
        # the reference's AVX2 sgemm output, within its own tolerance of the fp64 oracle
        want = orc.sgemm_f64(p, p.c, acc)
        mag = orc.magnitude(p, p.c, acc)
        assert tol_ok(c_view(p, data[f"sgemm{idx}"]), want, mag)
