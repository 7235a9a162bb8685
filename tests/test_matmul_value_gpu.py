"""The autograd matmul ops against the reference build's own nn::matmul / nn::matmul_bt Values
(src/autograd/ops.cpp:683-712, 747-773) and nn::scaled_masked_softmax (ops.cpp:1298-1343).

Shapes cover the folded backward (a 2-D b: one GEMM per gradient, stored or accumulated), the
batched backward with broadcast axes summed away in the reference's order (leading axes first, one
Tensor::sum(0) each, then the size-1 axes), a 2-D a against a batched b, and the accumulate rule
(each operand used twice: the first backward rule stores, the second adds). Products go through
the 3xTF32 tensor-core GEMM, so values agree to the GEMM tests' fp32-grade bound
|got - want| <= 2e-5 * (max|want| + |want|).
"""
import ctypes

import numpy as np
import pytest

import nnb
from oracle import orc

pytestmark = pytest.mark.gpu


def _ref():
    ref = orc.ref()
    if ref is None:
        pytest.skip("reference library not built (oracle/_ref)")
    return ref


def assert_close(got, want, rel=2e-5):
    got, want = np.asarray(got, np.float64), np.asarray(want, np.float64)
    assert got.shape == want.shape, (got.shape, want.shape)
    scale = np.abs(want).max() if want.size else 0.0
    err = np.abs(got - want)
    assert np.all(err <= rel * scale + rel * np.abs(want) + 1e-30), f"max err {err.max():.3e} vs scale {scale:.3e}"


def _out_shape(ash, bsh, bt):
    m, k = ash[-2], ash[-1]
    n = bsh[-2] if bt else bsh[-1]
    if len(bsh) == 2 and len(ash) > 2:
        return tuple(ash[:-1]) + (n,)
    ab, bb = ash[:-2], bsh[:-2]
    r = max(len(ab), len(bb))
    ab = (1,) * (r - len(ab)) + tuple(ab)
    bb = (1,) * (r - len(bb)) + tuple(bb)
    return tuple(max(x, y) for x, y in zip(ab, bb)) + (m, n)


def _reference(ash, bsh, bt, twice, a, b, g):
    ref = _ref()
    y = np.zeros(_out_shape(ash, bsh, bt), np.float32)
    da, db = np.zeros(ash, np.float32), np.zeros(bsh, np.float32)
    A = (ctypes.c_int64 * len(ash))(*ash)
    B = (ctypes.c_int64 * len(bsh))(*bsh)
    rc = ref.ref_matmul_value(orc.ptr(a), A, len(ash), orc.ptr(b), B, len(bsh), int(bt), int(twice), orc.ptr(g),
                              orc.ptr(y), orc.ptr(da), orc.ptr(db))
    assert rc == 0
    return y, da, db


CASES = [
    ((3, 4, 5), (5, 6), False),            # fold: batched a, 2-D b
    ((2, 3, 7, 5), (6, 5), True),          # fold, b stored {n, K}
    ((33, 70), (70, 41), False),           # plain 2-D
    ((40, 64), (48, 64), True),
    ((2, 1, 4, 5), (3, 5, 6), False),      # broadcast both ways: da sums a size-1 axis, db a leading axis
    ((4, 5), (2, 3, 5, 6), False),         # 2-D a, batched b: da sums two leading axes
    ((2, 3, 4, 5), (3, 6, 5), True),       # matmul_bt with a leading axis of a summed for db
    ((1, 3, 8, 16), (2, 1, 12, 16), True),  # size-1 axes on both sides
    ((2, 8, 64, 64), (2, 8, 64, 64), True),  # attention-shaped scores (composed path)
]


@pytest.mark.parametrize("ash,bsh,bt", CASES)
@pytest.mark.parametrize("twice", [False, True])
def test_matmul_value_matches_reference(cuda, ash, bsh, bt, twice):
    torch = cuda
    from nnb import functional as F
    from nnb.autograd import Value

    a = orc.uniform(200, int(np.prod(ash))).reshape(ash)
    b = orc.uniform(201, int(np.prod(bsh))).reshape(bsh)
    osh = _out_shape(ash, bsh, bt)
    g = orc.uniform(202, int(np.prod(osh))).reshape(osh)
    y_r, da_r, db_r = _reference(ash, bsh, bt, twice, a, b, g)

    A = Value.leaf(torch.from_numpy(a).cuda(), True)
    B = Value.leaf(torch.from_numpy(b).cuda(), True)
    op = F.matmul_bt if bt else F.matmul
    Y = op(A, B)
    if twice:
        Y = F.add(Y, op(A, B))
    assert Y.shape == osh
    Y.backward(torch.from_numpy(g).cuda())
    assert_close(Y.data.cpu().numpy(), y_r)
    assert_close(A.grad.cpu().numpy(), da_r)
    assert_close(B.grad.cpu().numpy(), db_r)
    assert nnb.device_error() == 0


def test_matmul_value_shape_errors(cuda):
    torch = cuda
    from nnb import functional as F
    from nnb.autograd import Value

    A = Value.leaf(torch.zeros(3, 4, device="cuda"), True)
    with pytest.raises(nnb.TensorShapeError):
        F.matmul(A, Value.leaf(torch.zeros(5, 6, device="cuda"), True))
    with pytest.raises(nnb.TensorShapeError):
        F.matmul_bt(A, Value.leaf(torch.zeros(6, 5, device="cuda"), True))
    with pytest.raises(nnb.TensorShapeError):
        F.matmul(Value.leaf(torch.zeros(2, 3, 4, device="cuda"), True),
                 Value.leaf(torch.zeros(3, 4, 5, device="cuda"), True))
    ref = _ref()
    a, b = np.zeros((3, 4), np.float32), np.zeros((5, 6), np.float32)
    out = np.zeros(64, np.float32)
    rc = ref.ref_matmul_value(orc.ptr(a), (ctypes.c_int64 * 2)(3, 4), 2, orc.ptr(b), (ctypes.c_int64 * 2)(5, 6), 2, 0,
                              0, orc.ptr(out), orc.ptr(out), orc.ptr(out), orc.ptr(out))
    assert rc == 1                         # the reference throws for the same shapes


SOFTMAX_CASES = [
    (2, 3, 5, 7, False, False),
    (2, 2, 9, 9, True, True),              # causal with key padding
    (1, 4, 4, 6, True, False),             # causal, not square (the reference allows it)
    (3, 8, 64, 64, True, False),
    (2, 1, 33, 130, False, True),          # rows longer than a warp's stride
]


@pytest.mark.parametrize("N,H,Tq,Tk,causal,padded", SOFTMAX_CASES)
def test_scaled_masked_softmax_matches_reference(cuda, N, H, Tq, Tk, causal, padded):
    torch = cuda
    from nnb import functional as F
    from nnb.autograd import Value

    ref = _ref()
    x = orc.normal(210, N * H * Tq * Tk).reshape(N, H, Tq, Tk)
    g = orc.normal(211, x.size).reshape(x.shape)
    pad = None
    if padded:
        pad = np.ones((N, Tk), np.float32)
        pad[:, Tk - 2:] = 0.0
        pad[0, 0] = 0.0
    scale = 0.125
    y_r, dx_r = np.zeros_like(x), np.zeros_like(x)
    ref.ref_scaled_masked_softmax(N, H, Tq, Tk, orc.ptr(x), scale, orc.ptr(pad), int(causal), orc.ptr(g), orc.ptr(y_r),
                                  orc.ptr(dx_r))
    X = Value.leaf(torch.from_numpy(x).cuda(), True)
    pad_d = None if pad is None else torch.from_numpy(pad).cuda()
    Y = F.scaled_masked_softmax(X, scale, pad_d, causal)
    Y.backward(torch.from_numpy(g).cuda())
    assert_close(Y.data.cpu().numpy(), y_r, rel=1e-5)
    assert_close(X.grad.cpu().numpy(), dx_r, rel=1e-5)
    # masked positions: exactly 0 in the stored gradient, untouched when accumulating
    masked = np.zeros(x.shape, bool)
    if causal:
        masked |= np.triu(np.ones((Tq, Tk), bool), 1)[None, None]
    if pad is not None:
        masked |= (pad == 0.0)[:, None, None, :]
    dx = X.grad.cpu().numpy()
    assert np.all(dx[masked] == 0.0) and np.all(dx_r[masked] == 0.0)
    acc = torch.full(x.shape, 7.0, device="cuda")
    s = torch.cuda.current_stream().cuda_stream
    nnb.check(nnb.lib().nnb_scaled_masked_softmax_bwd(s, N, H, Tq, Tk, Y.data.data_ptr(),
                                                      torch.from_numpy(g).cuda().data_ptr(), acc.data_ptr(), 0,
                                                      None if pad_d is None else pad_d.data_ptr(), int(causal),
                                                      ctypes.c_float(scale)))
    got = acc.cpu().numpy()
    assert np.all(got[masked] == 7.0)
    assert_close(got[~masked] - 7.0, dx_r[~masked], rel=1e-5 * 8)


@pytest.mark.parametrize("N,H,T,causal,padded", [(2, 3, 17, True, False), (3, 2, 40, False, True), (2, 8, 64, True, True)])
def test_masked_softmax_rows_in_place(cuda, N, H, T, causal, padded):
    """nnb_masked_softmax_fwd / _bwd, the attention paths' in-place row kernels (masked_softmax_row and
    its backward, ops.cpp:1183-1224), called directly: against the reference's scaled_masked_softmax on
    the same scores (the same row arithmetic: scale, pad -> -1e9, causal -> -2e9 / 0, softmax), and the
    backward turning dL/dP into dL/dS in place with 0 at masked positions."""
    torch = cuda
    ref = _ref()
    x = orc.normal(220, N * H * T * T).reshape(N, H, T, T)
    g = orc.normal(221, x.size).reshape(x.shape)
    pad = None
    if padded:
        pad = np.ones((N, T), np.float32)
        pad[:, T - 3:] = 0.0
    scale = 0.125
    y_r, dx_r = np.zeros_like(x), np.zeros_like(x)
    ref.ref_scaled_masked_softmax(N, H, T, T, orc.ptr(x), scale, orc.ptr(pad), int(causal), orc.ptr(g), orc.ptr(y_r),
                                  orc.ptr(dx_r))
    s = torch.cuda.current_stream().cuda_stream
    scores = torch.from_numpy(x).cuda()
    pad_d = None if pad is None else torch.from_numpy(pad).cuda()
    nnb.check(nnb.lib().nnb_masked_softmax_fwd(s, N, H, T, T, scores.data_ptr(),
                                               None if pad_d is None else pad_d.data_ptr(), int(causal),
                                               ctypes.c_float(scale)))
    assert_close(scores.cpu().numpy(), y_r, rel=1e-5)
    grad = torch.from_numpy(g).cuda()
    nnb.check(nnb.lib().nnb_masked_softmax_bwd(s, N, H, T, T, scores.data_ptr(), grad.data_ptr(),
                                               None if pad_d is None else pad_d.data_ptr(), int(causal),
                                               ctypes.c_float(scale)))
    got = grad.cpu().numpy()
    assert_close(got, dx_r, rel=1e-5)
    if causal:
        assert np.all(got[..., np.triu(np.ones((T, T), bool), 1)] == 0.0)
