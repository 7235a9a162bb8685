"""Ops beyond the configs' paths that the reference's modules use (the next rows of the scope):
conv2d with dilation / groups, avgpool2d, sum / mean over an axis, GlobalAvgPool2d and the
BatchNorm2d module (training mode with its running statistics, evaluation mode), each against the
reference build itself (oracle/_ref) on the same inputs.

Bitwise where the reference's order of operations is reproduced (pooling, reductions, the conv bias
gradient, batchnorm's training-mode outputs and running statistics, its evaluation-mode forward and
input gradient); GEMM-built results to the fp32 bound of the other ops' tests.
"""
import numpy as np
import pytest

import nnb
from oracle import orc

pytestmark = pytest.mark.gpu
P = orc.ptr


def ref():
    r = orc.ref()
    if r is None:
        pytest.skip("reference library not built (oracle/_ref)")
    return r


def S(torch):
    return torch.cuda.current_stream().cuda_stream


def dev(torch, a):
    return torch.from_numpy(np.ascontiguousarray(a)).cuda()


def nrm(seed, *shape):
    return orc.normal(seed, int(np.prod(shape))).reshape(shape)


def assert_close(got, want, rel=2e-5):
    got, want = np.asarray(got, np.float64), np.asarray(want, np.float64)
    assert got.shape == want.shape
    bound = rel * np.abs(want).max() + rel * np.abs(want) + 1e-30
    err = np.abs(got - want)
    assert (err <= bound).all(), f"worst {err.max():.3e} vs scale {np.abs(want).max():.3e}"


def assert_bits(got, want):
    got, want = np.asarray(got, np.float32), np.asarray(want, np.float32)
    assert got.shape == want.shape
    assert got.tobytes() == want.tobytes(), f"max diff {np.abs(got.astype(np.float64) - want).max():.3e}"


@pytest.mark.parametrize("N,Cin,H,W,Cout,k,stride,pad,dil,groups", [
    (2, 4, 11, 9, 6, 3, 1, 2, 2, 2),      # dilation and groups
    (3, 6, 10, 10, 6, 3, 2, 1, 1, 6),     # depthwise, strided
    (2, 8, 12, 13, 4, 2, 1, 0, 3, 4),     # dilation 3, groups 4, no padding
])
def test_conv2d_general_matches_reference(cuda, N, Cin, H, W, Cout, k, stride, pad, dil, groups):
    torch = cuda
    import nnb.functional as F
    from nnb.autograd import Value
    R = ref()
    x, w, b = nrm(201, N, Cin, H, W), nrm(202, Cout, Cin // groups, k, k), nrm(203, Cout)
    ekh = dil * (k - 1) + 1
    ho, wo = (H + 2 * pad - ekh) // stride + 1, (W + 2 * pad - ekh) // stride + 1
    g = nrm(204, N, Cout, ho, wo)
    y_r, dx_r, dw_r, db_r = orc.zeros(N, Cout, ho, wo), orc.zeros(N, Cin, H, W), orc.zeros(*w.shape), orc.zeros(Cout)
    R.ref_conv2d_ex(N, Cin, H, W, Cout, k, k, stride, pad, dil, groups, P(x), P(w), P(b), P(g), P(y_r), P(dx_r),
                    P(dw_r), P(db_r))
    X, Wt, B = (Value.leaf(dev(torch, a), True) for a in (x, w, b))
    Y = F.conv2d(X, Wt, B, stride, pad, dilation=dil, groups=groups)
    Y.backward(dev(torch, g))
    assert_close(Y.data.cpu().numpy(), y_r)
    assert_close(X.grad.cpu().numpy(), dx_r)
    assert_close(Wt.grad.cpu().numpy(), dw_r)
    assert_bits(B.grad.cpu().numpy(), db_r)        # serial over samples then positions, as the reference


@pytest.mark.parametrize("k,stride", [(2, 2), (3, 1), (3, 2)])
def test_avgpool2d_bitwise(cuda, k, stride):
    torch = cuda
    import nnb.functional as F
    from nnb.autograd import Value
    R = ref()
    N, C, H, W = 3, 5, 11, 12
    x = nrm(211, N, C, H, W)
    ho, wo = (H - k) // stride + 1, (W - k) // stride + 1
    g = nrm(212, N, C, ho, wo)
    y_r, dx_r = orc.zeros(N, C, ho, wo), orc.zeros(N, C, H, W)
    R.ref_avgpool2d(N, C, H, W, k, stride, P(x), P(g), P(y_r), P(dx_r))
    X = Value.leaf(dev(torch, x), True)
    Y = F.avgpool2d(X, k, stride)
    Y.backward(dev(torch, g))
    assert_bits(Y.data.cpu().numpy(), y_r)
    assert_bits(X.grad.cpu().numpy(), dx_r)


@pytest.mark.parametrize("axis", [0, 1, 2, 3, -1])
@pytest.mark.parametrize("average", [0, 1])
def test_reduce_axis_bitwise(cuda, axis, average):
    torch = cuda
    import nnb.functional as F
    from nnb.autograd import Value
    R = ref()
    shape = (3, 4, 5, 6)
    x = nrm(221, *shape)
    out_shape = tuple(d for i, d in enumerate(shape) if i != axis % 4)
    g = nrm(222, *out_shape)
    y_r, dx_r = orc.zeros(*out_shape), orc.zeros(*shape)
    R.ref_reduce4(*shape, axis, average, P(x), P(g), P(y_r), P(dx_r))
    X = Value.leaf(dev(torch, x), True)
    Y = (F.mean if average else F.sum)(X, axis)
    assert Y.shape == out_shape
    Y.backward(dev(torch, g))
    assert_bits(Y.data.cpu().numpy(), y_r)
    assert_bits(X.grad.cpu().numpy(), dx_r)


def test_global_avgpool_bitwise(cuda):
    torch = cuda
    from nnb.autograd import Value
    from nnb.nn import GlobalAvgPool2d
    R = ref()
    N, C, H, W = 4, 6, 7, 5
    x, g = nrm(231, N, C, H, W), nrm(232, N, C)
    y_r, dx_r = orc.zeros(N, C), orc.zeros(N, C, H, W)
    R.ref_global_avgpool(N, C, H, W, P(x), P(g), P(y_r), P(dx_r))
    X = Value.leaf(dev(torch, x), True)
    Y = GlobalAvgPool2d()(X)
    Y.backward(dev(torch, g))
    assert_bits(Y.data.cpu().numpy(), y_r)
    assert_bits(X.grad.cpu().numpy(), dx_r)


@pytest.mark.parametrize("evaluate,fuse_relu", [(0, 0), (0, 1), (1, 0), (1, 1)])
@pytest.mark.parametrize("shape", [(6, 5, 7, 9), (1, 3, 1, 300)])
def test_batchnorm2d_module_matches_reference(cuda, evaluate, fuse_relu, shape):
    """Two training-mode steps (running statistics updated with momentum 0.1 and the unbiased
    variance), then, with evaluate, one evaluation-mode forward; output and gradients of the last
    forward, and the running statistics, against the reference's BatchNorm2d with a random weight and
    bias of both signs -- all bit for bit (the evaluation-mode parameter gradients are summed over N,
    then H, then W, as the reference's sum_to_shape does)."""
    torch = cuda
    from nnb.autograd import Value
    from nnb.nn import BatchNorm2d
    R = ref()
    N, C, H, W = shape
    x, g = nrm(241, N, C, H, W), nrm(242, N, C, H, W)
    w, b = orc.uniform(243, C, -1.5, 1.5), orc.uniform(244, C, -1.0, 1.0)
    y_r, dx_r, dw_r, db_r = orc.zeros(N, C, H, W), orc.zeros(N, C, H, W), orc.zeros(C), orc.zeros(C)
    rm_r, rv_r = orc.zeros(C), orc.zeros(C)
    R.ref_bn2d_module_ex(N, C, H, W, 2, evaluate, fuse_relu, P(x), P(g), P(w), P(b), P(y_r), P(dx_r), P(dw_r),
                         P(db_r), P(rm_r), P(rv_r))
    bn = BatchNorm2d(C, torch.device("cuda"))
    bn.weight.data.copy_(dev(torch, w))
    bn.bias.data.copy_(dev(torch, b))
    xd = dev(torch, x)
    for _ in range(2):
        X = Value.leaf(xd, True)
        Y = bn.forward_relu(X) if fuse_relu else bn(X)
    if evaluate:
        bn.eval()
        X = Value.leaf(xd, True)
        Y = bn.forward_relu(X) if fuse_relu else bn(X)
    bn.weight.zero_grad()
    bn.bias.zero_grad()
    Y.backward(dev(torch, g))
    assert_bits(bn.running_mean.cpu().numpy(), rm_r)
    assert_bits(bn.running_var.cpu().numpy(), rv_r)
    assert_bits(Y.data.cpu().numpy(), y_r)
    assert_bits(X.grad.cpu().numpy(), dx_r)
    assert_bits(bn.weight.grad.cpu().numpy(), dw_r)
    assert_bits(bn.bias.grad.cpu().numpy(), db_r)


@pytest.mark.parametrize("shape", [(4, 3, 5, 6), (2, 4, 1, 1), (3, 2, 6, 1), (1, 5, 4, 300)])
@pytest.mark.parametrize("fuse", [0, 1])
def test_batchnorm_eval_op_matches_oracle(cuda, shape, fuse):
    """nnb_batchnorm_eval_fwd / _bwd through the C ABI against the oracle's restatement
    (orc_batchnorm_eval_fwd / _bwd), bit for bit, storing and then accumulating the gradients."""
    torch = cuda
    import ctypes
    N, C, H, W = shape
    x, g = nrm(251, N, C, H, W) * 2.0 + 0.3, nrm(252, N, C, H, W)
    w, b = orc.uniform(253, C, -1.5, 1.5), orc.uniform(254, C, -1.0, 1.0)
    rm, rv = orc.uniform(255, C, -0.5, 0.5), orc.uniform(256, C, 0.5, 2.0)
    y_o, dx_o, dw_o, db_o = orc.zeros(N, C, H, W), orc.zeros(N, C, H, W), orc.zeros(C), orc.zeros(C)
    O = orc.orc
    O.orc_batchnorm_eval_fwd(N, C, H * W, P(x), P(w), P(b), P(rm), P(rv), 1e-5, fuse, P(y_o))
    O.orc_batchnorm_eval_bwd(N, C, H, W, P(g), P(x), P(w), P(b), P(rm), P(rv), 1e-5, fuse, P(dx_o), P(dw_o), P(db_o))
    xd, gd, wd, bd, rmd, rvd = (dev(torch, a) for a in (x, g, w, b, rm, rv))
    y = torch.empty(N, C, H, W, device="cuda")
    alive = torch.empty(N, C, H, W, device="cuda", dtype=torch.uint8) if fuse else None
    s = torch.cuda.current_stream().cuda_stream
    L = nnb.lib()
    eps = ctypes.c_float(1e-5)
    nnb.check(L.nnb_batchnorm_eval_fwd(s, N, C, H * W, xd.data_ptr(), rmd.data_ptr(), rvd.data_ptr(), eps,
                                       wd.data_ptr(), bd.data_ptr(), fuse, y.data_ptr(),
                                       None if alive is None else alive.data_ptr()))
    dx = torch.full((N, C, H, W), 7.0, device="cuda")
    dw, db = torch.full((C,), 7.0, device="cuda"), torch.full((C,), 7.0, device="cuda")
    for first in (1, 0):
        nnb.check(L.nnb_batchnorm_eval_bwd(s, N, C, H, W, gd.data_ptr(), xd.data_ptr(), rmd.data_ptr(),
                                           rvd.data_ptr(), eps, wd.data_ptr(),
                                           None if alive is None else alive.data_ptr(), dx.data_ptr(), first,
                                           dw.data_ptr(), first, db.data_ptr(), first))
        if first:
            assert_bits(y.cpu().numpy(), y_o)
            assert_bits(dx.cpu().numpy(), dx_o)
            assert_bits(dw.cpu().numpy(), dw_o)
            assert_bits(db.cpu().numpy(), db_o)
    assert_bits(dx.cpu().numpy(), dx_o + dx_o)
    assert_bits(dw.cpu().numpy(), dw_o + dw_o)
    assert_bits(db.cpu().numpy(), db_o + db_o)


def test_sequential_folds_relu_like_reference(cuda):
    """Sequential folds ReLU into Conv2d (dilation 1, groups 1) and into BatchNorm2d in training mode
    only (sequential.cpp:16-28, conv2d.hpp:72, batchnorm.hpp:50)."""
    torch = cuda
    from nnb.nn import BatchNorm2d, Conv2d, ReLU, Sequential
    rng = np.random.default_rng(3)
    d = torch.device("cuda")
    conv, convg, bn = Conv2d(4, 4, 3, 1, 1, rng, d), Conv2d(4, 4, 3, 1, 1, rng, d, groups=2), BatchNorm2d(4, d)
    assert conv.can_fuse_relu and not convg.can_fuse_relu
    assert bn.can_fuse_relu
    bn.eval()
    assert not bn.can_fuse_relu
    net = Sequential(conv, ReLU(), bn, ReLU())
    assert [n for n, _ in net.named_buffers()] == ["2.running_mean", "2.running_var"]
