"""Generates tests/golden/gemm_golden.npz from the reference library itself.

Run in a container that has the reference sources (oracle/Makefile builds oracle/_ref/libnnref.so
from them):  python tests/golden/make_golden.py

For each case (ta, tb, m, n, k, pad, seed, accumulate) it stores the inputs made by the reference
test's problem builder (tests/test_kernels.cpp:68-86), the output of the reference's own
triple-loop oracle (tests/reference_gemm.hpp) and the output of its production sgemm
(src/kernels/gemm.cpp:546). The file is small and committed; the GPU box reads it without the
reference present.
"""
import pathlib
import sys

import numpy as np

ROOT = pathlib.Path(__file__).resolve().parents[2]
sys.path.insert(0, str(ROOT))
from oracle import orc  # noqa: E402

CASES = [
    (0, 0, 7, 33, 17, 0, 11, 0),
    (1, 0, 33, 7, 57, 2, 12, 1),
    (0, 1, 17, 40, 33, 3, 13, 0),
    (1, 1, 9, 9, 129, 1, 14, 1),
    (0, 0, 64, 64, 100, 0, 15, 0),
    (0, 1, 5, 130, 64, 4, 16, 0),
    (1, 0, 101, 3, 31, 0, 17, 1),
    (1, 1, 1, 1, 1, 0, 18, 0),
    (0, 0, 1, 33, 257, 0, 19, 1),
    (0, 1, 40, 24, 8, 1, 20, 0),
]


def main():
    ref = orc.ref()
    if ref is None:
        raise SystemExit("oracle/_ref/libnnref.so not built; run make -C oracle")
    out = {"cases": np.array(CASES, np.int64)}
    for idx, (ta, tb, m, n, k, pad, seed, acc) in enumerate(CASES):
        p = orc.Problem(ta, tb, m, n, k, pad, seed)
        loop = p.c.copy()
        ref.ref_reference_sgemm(*p.args(), orc.ptr(loop), p.ldc, acc)
        sg = p.c.copy()
        ref.ref_sgemm(*p.args(), orc.ptr(sg), p.ldc, acc)
        out[f"a{idx}"], out[f"b{idx}"], out[f"c{idx}"] = p.a, p.b, p.c
        out[f"loop{idx}"], out[f"sgemm{idx}"] = loop, sg
    dst = pathlib.Path(__file__).resolve().parent / "gemm_golden.npz"
    np.savez_compressed(dst, **out)
    print(dst, dst.stat().st_size, "bytes")


if __name__ == "__main__":
    main()
