"""nnb_matmul (batched Tensor matmul, src/tensor.cpp:571-641) against the reference's nn::matmul.

Shapes cover the reference's fold path (batched a times a 2-D b), same-shape batches, numpy-style
broadcast of batch axes in either operand, batch ranks above two, the transpose flags, and the
shape errors the reference throws. Values are checked against the reference build (oracle/_ref)
when present and always against an fp64 evaluation, with the GEMM tests' 3xTF32 bound
|got - want| <= 1e-5 * sum|a*b| (+1e-6).
"""
import numpy as np
import pytest

import nnb
from oracle import orc

pytestmark = pytest.mark.gpu


def op(x, t):
    return np.swapaxes(x, -1, -2) if t else x


CASES = [
    ((3, 4, 5), (5, 6), 0, 0),             # fold
    ((2, 3, 7, 5), (6, 5), 0, 1),          # fold with trans_b
    ((2, 3, 4), (2, 4, 5), 0, 0),
    ((2, 1, 4, 5), (3, 5, 6), 0, 0),       # broadcast both ways
    ((4, 5), (2, 3, 5, 6), 0, 0),          # 2-D a, batched b
    ((2, 2, 3, 4, 5), (2, 1, 5, 6), 0, 0),  # batch rank 3 (host loop over the leading axis)
    ((4, 3, 7), (4, 5, 3), 1, 1),          # both transposed, batched
    ((3, 200, 130), (130, 257), 0, 0),
    ((512, 512), (512, 512), 0, 0),        # config 1 shape
]


@pytest.mark.parametrize("ash,bsh,ta,tb", CASES)
def test_matmul_matches_reference(cuda, ash, bsh, ta, tb):
    torch = cuda
    a = orc.uniform(100, int(np.prod(ash))).reshape(ash)
    b = orc.uniform(101, int(np.prod(bsh))).reshape(bsh)
    got = nnb.matmul(torch.from_numpy(a).cuda(), torch.from_numpy(b).cuda(), ta, tb).cpu().numpy()
    want64 = np.matmul(op(a.astype(np.float64), ta), op(b.astype(np.float64), tb))
    mag = np.matmul(np.abs(op(a.astype(np.float64), ta)), np.abs(op(b.astype(np.float64), tb)))
    assert got.shape == want64.shape
    assert np.all(np.abs(got - want64) <= 1e-5 * mag + 1e-6)
    ref = orc.ref()
    if ref is not None:
        out = np.empty(want64.shape, np.float32)
        ash_c = np.array(ash, np.int64)
        bsh_c = np.array(bsh, np.int64)
        assert ref.ref_matmul_nd(orc.ptr(a), orc.ptr(ash_c), len(ash), orc.ptr(b), orc.ptr(bsh_c), len(bsh), ta, tb,
                                 orc.ptr(out)) == 0
        assert np.all(np.abs(got - out) <= 2e-5 * mag + 1e-6)


@pytest.mark.parametrize("ash,bsh", [((3, 4), (5, 6)), ((2, 3, 4), (3, 4, 5)), ((4,), (4, 4))])
def test_matmul_shape_errors(cuda, ash, bsh):
    torch = cuda
    a = torch.zeros(ash, device="cuda")
    b = torch.zeros(bsh, device="cuda")
    with pytest.raises(nnb.TensorShapeError):
        nnb.matmul(a, b)
    ref = orc.ref()
    if ref is not None:
        an, bn = np.zeros(ash, np.float32), np.zeros(bsh, np.float32)
        out = np.zeros(64, np.float32)
        assert ref.ref_matmul_nd(orc.ptr(an), orc.ptr(np.array(ash, np.int64)), len(ash), orc.ptr(bn),
                                 orc.ptr(np.array(bsh, np.int64)), len(bsh), 0, 0, orc.ptr(out)) == 1
