"""Generates the golden fixtures under tests/golden/ from the reference library itself.

Run in a container that has the reference sources, with REF naming their root (oracle/Makefile
builds oracle/_ref/libnnref.so from them):  REF=<reference root> python tests/golden/make_golden.py

For each case (ta, tb, m, n, k, pad, seed, accumulate) it stores the inputs made by the reference
test's problem builder (tests/test_kernels.cpp:68-86), the output of the reference's own
triple-loop oracle (tests/reference_gemm.hpp) and the output of its production sgemm
(src/kernels/gemm.cpp:546). The file is small and committed; the GPU box reads it without the
reference present.

It also writes two checkpoints with the reference's own writer (src/checkpoint.cpp): the
Sequential{Linear(3, 2)} of tests/test_checkpoint.cpp's golden case saved at step 7 without an
optimizer (linear_step7.nnck), and the same model after one AdamW step on fixed gradients, saved
with the optimizer at step 1 (linear_adamw.nnck).
"""
import os
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
    if not os.environ.get("REF"):
        raise SystemExit("set REF to the reference's source tree (the root holding src/ and tests/)")
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
    checkpoints(ref)


# Sequential{Linear(3, 2)} parameters of the reference's golden checkpoint test, and the gradients and
# AdamW settings of the optimizer-state fixture.
CKPT_W = [0.5, -1.25, 2.0, 3.0, 0.75, -0.5]
CKPT_B = [0.125, -2.0]
CKPT_GW = [0.25, -0.5, 1.5, -2.0, 0.125, 3.0]
CKPT_GB = [-0.75, 0.375]
CKPT_LR, CKPT_WD = 0.01, 0.1


def checkpoints(ref):
    here = pathlib.Path(__file__).resolve().parent
    f32 = lambda v: np.array(v, np.float32)
    w, b, gw, gb = f32(CKPT_W), f32(CKPT_B), f32(CKPT_GW), f32(CKPT_GB)
    plain, adamw = here / "linear_step7.nnck", here / "linear_adamw.nnck"
    if ref.ref_linear_checkpoint_save(str(plain).encode(), orc.ptr(w), orc.ptr(b), None, None, 0.0, 0.0, 7):
        raise SystemExit("reference save failed")
    if ref.ref_linear_checkpoint_save(str(adamw).encode(), orc.ptr(w), orc.ptr(b), orc.ptr(gw), orc.ptr(gb),
                                      CKPT_LR, CKPT_WD, 1):
        raise SystemExit("reference save failed")
    for f in (plain, adamw):
        print(f, f.stat().st_size, "bytes")
    # the reference's own golden file for this model (tests/data/linear_v1.ckpt) pins the writer
    golden = pathlib.Path(os.environ["REF"]) / "tests/data/linear_v1.ckpt"
    if not golden.exists():
        raise SystemExit(f"{golden} not found: REF must name the reference's source tree")
    if golden.read_bytes() != plain.read_bytes():
        raise SystemExit("reference writer disagrees with the reference's golden checkpoint")


if __name__ == "__main__":
    main()
