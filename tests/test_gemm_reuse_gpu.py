"""Kept operand packs of the linear layer. The backward's shared output-gradient pack: dX = G W packs
G once (32-wide row panels; once for all depth pieces when dX is cut along its depth) and the weight
gradient dW = G^T X reads that pack MN-major instead of packing G^T again. The kept input pack:
nnb_linear_fwd_ex keeps x's pack from the forward and nnb_linear_bwd_ex's weight gradient reads it
instead of packing X^T.

Neither may change a bit: for every shape (ragged feature counts, several groups, depth-cut weight
and input gradients, shapes that cannot share because a group is not whole 16-row blocks) and both
math modes, the shared paths must give exactly the bits of the same products run without sharing
(separate nnb_sgemm_ex calls; nnb_linear_fwd / nnb_linear_multi_fwd / nnb_linear_gelu_fwd and
nnb_linear_bwd_grouped), non-finite inputs must still come out as the reference's IEEE results, and
a pack written in another math mode must be ignored. The weight gradients are also held to the fp64
bound of the GEMM tests.
"""
import numpy as np
import pytest

import nnb
from oracle import orc

pytestmark = pytest.mark.gpu

MODES = [nnb.MATH_FP32X3, nnb.MATH_TF32]
TOL = {nnb.MATH_FP32X3: 1e-5, nnb.MATH_TF32: 5e-3}


def _dev(torch, a):
    return torch.from_numpy(np.ascontiguousarray(a, np.float32)).cuda()


def _separate(torch, g, x, w, groups, mode):
    """dX and each group's dW through nnb_sgemm_ex, one product per call (no shared pack)."""
    M, n = g.shape
    K = x.shape[1]
    gd, xd, wd = _dev(torch, g), _dev(torch, x), _dev(torch, w)
    dx = torch.zeros(M, K, device="cuda")
    nnb.sgemm(False, False, M, K, n, gd, n, wd, K, dx, K, False, math_mode=mode)
    rg = M // groups
    dws = []
    for z in range(groups):
        dw = torch.zeros(n, K, device="cuda")
        nnb.sgemm(True, False, n, K, rg, gd[z * rg:(z + 1) * rg], n, xd[z * rg:(z + 1) * rg], K, dw, K, False,
                  math_mode=mode)
        dws.append(dw)
    torch.cuda.synchronize()
    return dx.cpu().numpy(), np.stack([d.cpu().numpy() for d in dws])


def _shared(torch, g, x, w, groups, mode):
    M, n = g.shape
    K = x.shape[1]
    gd, xd, wd = _dev(torch, g), _dev(torch, x), _dev(torch, w)
    dx = torch.zeros(M, K, device="cuda")
    dw = torch.zeros(groups, n, K, device="cuda")
    db = torch.zeros(groups, n, device="cuda")
    s = torch.cuda.current_stream().cuda_stream
    old = nnb.get_math_mode()
    nnb.set_math_mode(mode)
    try:
        if groups == 1:
            nnb.check(nnb.lib().nnb_linear_bwd(s, M, K, n, gd.data_ptr(), xd.data_ptr(), wd.data_ptr(), dx.data_ptr(), 1,
                                               dw.data_ptr(), 1, db.data_ptr(), 1))
        else:
            nnb.check(nnb.lib().nnb_linear_bwd_grouped(s, M, K, n, groups, gd.data_ptr(), xd.data_ptr(), wd.data_ptr(),
                                                       dx.data_ptr(), 1, dw.data_ptr(), n * K, 1, db.data_ptr(), n, 1))
        torch.cuda.synchronize()
    finally:
        nnb.set_math_mode(old)
    return dx.cpu().numpy(), dw.cpu().numpy()


def _fp64_bound(g, x, groups, dw, mode):
    M = g.shape[0]
    rg = M // groups
    for z in range(groups):
        gz = g[z * rg:(z + 1) * rg].astype(np.float64)
        xz = x[z * rg:(z + 1) * rg].astype(np.float64)
        exact = gz.T @ xz
        mag = np.abs(gz).T @ np.abs(xz)
        assert np.all(np.abs(dw[z] - exact) <= np.maximum(TOL[mode] * mag, 1e-6))


# (M, K = input features, n = output features, groups): ragged widths (n not a multiple of 32, so the
# shared pack's last 32-wide column is half padding), several groups, a group depth long enough for
# the depth cut (2048 rows >= 2 * max(1024, K)), groups of 24 rows (not whole 16-row blocks: the
# weight gradient packs G^T itself), and input gradients cut along their depth (n >= 2 * max(1024,
# K): G is packed once and every depth piece reads its columns from the pack; 4100 = three 1040-wide
# pieces and a 980-wide last one, which ends inside a 16-column block)
SHAPES = [
    (256, 96, 80, 1),
    (512, 200, 130, 4),
    (4096, 64, 48, 2),
    (96, 40, 24, 4),
    (1024, 512, 512, 8),
    (512, 64, 2048, 2),
    (256, 128, 4100, 1),
]


@pytest.mark.parametrize("mode", MODES)
@pytest.mark.parametrize("shape", SHAPES)
def test_shared_pack_keeps_the_bits_of_separate_products(cuda, shape, mode):
    torch = cuda
    M, K, n, groups = shape
    g = orc.normal(101 + M + n, M * n).reshape(M, n).astype(np.float32)
    x = orc.normal(202 + K, M * K).reshape(M, K).astype(np.float32)
    w = orc.normal(303 + n * K, n * K).reshape(n, K).astype(np.float32)
    dx_s, dw_s = _shared(torch, g, x, w, groups, mode)
    dx_r, dw_r = _separate(torch, g, x, w, groups, mode)
    assert dx_s.tobytes() == dx_r.tobytes()
    assert dw_s.tobytes() == dw_r.tobytes()
    _fp64_bound(g, x, groups, dw_s, mode)


@pytest.mark.parametrize("mode", MODES)
def test_shared_pack_with_non_finite_gradients(cuda, mode):
    """An Inf and a NaN in G: every weight-gradient element whose sum meets them is the IEEE result,
    the others keep their finite bits (the same as the separate products)."""
    torch = cuda
    M, K, n, groups = 512, 72, 96, 2
    g = orc.normal(7, M * n).reshape(M, n).astype(np.float32)
    x = orc.normal(8, M * K).reshape(M, K).astype(np.float32)
    w = orc.normal(9, n * K).reshape(n, K).astype(np.float32)
    g[10, 5] = np.inf
    g[300, 40] = np.nan
    dx_s, dw_s = _shared(torch, g, x, w, groups, mode)
    dx_r, dw_r = _separate(torch, g, x, w, groups, mode)
    assert dx_s.tobytes() == dx_r.tobytes()
    assert dw_s.tobytes() == dw_r.tobytes()
    assert np.isinf(dw_s[0, 5]).any() and np.isnan(dw_s[1, 40]).all()
    assert np.isfinite(dw_s[0, 6]).all() and np.isfinite(dw_s[1, :40]).all()


def _kept(torch, x, w, b, g, groups, mode, fwd_mode=None, count=1, gelu=False):
    """Forward through nnb_linear_fwd_ex keeping x's pack, backward through nnb_linear_bwd_ex reading
    it. count > 1: the multi-weight form (w, b, g stacked), every backward reading the one pack."""
    M, K = x.shape
    n = w.shape[-2]
    lib = nnb.lib()
    s = torch.cuda.current_stream().cuda_stream
    fm = mode if fwd_mode is None else fwd_mode
    old = nnb.get_math_mode()
    try:
        nnb.set_math_mode(fm)
        xd, wd, bd = _dev(torch, x), _dev(torch, w), _dev(torch, b)
        pack = torch.empty(lib.nnb_linear_pack_bytes(M, K, fm), dtype=torch.uint8, device="cuda")
        y = torch.zeros(count, M, n, device="cuda")
        pre = torch.zeros(M, n, device="cuda") if gelu else None
        nnb.check(lib.nnb_linear_fwd_ex(s, count, M, K, n, xd.data_ptr(), wd.data_ptr(), n * K, bd.data_ptr(), n,
                                        y.data_ptr(), M * n, pre.data_ptr() if gelu else None, pack.data_ptr()))
        nnb.set_math_mode(mode)
        outs = []
        for i in range(count):
            gd = _dev(torch, g[i])
            dx = torch.zeros(M, K, device="cuda")
            dw = torch.zeros(groups, n, K, device="cuda")
            db = torch.zeros(groups, n, device="cuda")
            nnb.check(lib.nnb_linear_bwd_ex(s, M, K, n, groups, gd.data_ptr(), xd.data_ptr(), pack.data_ptr(), fm,
                                            wd[i].data_ptr(), dx.data_ptr(), 1, dw.data_ptr(), n * K, 1, db.data_ptr(),
                                            n, 1))
            outs.append((dx.cpu().numpy(), dw.cpu().numpy(), db.cpu().numpy()))
        torch.cuda.synchronize()
    finally:
        nnb.set_math_mode(old)
    return y.cpu().numpy(), (pre.cpu().numpy() if gelu else None), outs


def _plain(torch, x, w, b, g, groups, mode, count=1, gelu=False):
    """The same through nnb_linear_fwd / nnb_linear_gelu_fwd and nnb_linear_bwd_grouped."""
    M, K = x.shape
    n = w.shape[-2]
    lib = nnb.lib()
    s = torch.cuda.current_stream().cuda_stream
    old = nnb.get_math_mode()
    try:
        nnb.set_math_mode(mode)
        xd = _dev(torch, x)
        ys, pres, outs = [], [], []
        for i in range(count):
            wd, bd, gd = _dev(torch, w[i]), _dev(torch, b[i]), _dev(torch, g[i])
            y = torch.zeros(M, n, device="cuda")
            if gelu:
                pre = torch.zeros(M, n, device="cuda")
                nnb.check(lib.nnb_linear_gelu_fwd(s, M, K, n, xd.data_ptr(), wd.data_ptr(), bd.data_ptr(),
                                                  y.data_ptr(), pre.data_ptr()))
                pres.append(pre.cpu().numpy())
            else:
                nnb.check(lib.nnb_linear_fwd(s, M, K, n, xd.data_ptr(), wd.data_ptr(), bd.data_ptr(), y.data_ptr()))
            ys.append(y.cpu().numpy())
            dx = torch.zeros(M, K, device="cuda")
            dw = torch.zeros(groups, n, K, device="cuda")
            db = torch.zeros(groups, n, device="cuda")
            nnb.check(lib.nnb_linear_bwd_grouped(s, M, K, n, groups, gd.data_ptr(), xd.data_ptr(), wd.data_ptr(),
                                                 dx.data_ptr(), 1, dw.data_ptr(), n * K, 1, db.data_ptr(), n, 1))
            outs.append((dx.cpu().numpy(), dw.cpu().numpy(), db.cpu().numpy()))
        torch.cuda.synchronize()
    finally:
        nnb.set_math_mode(old)
    return np.stack(ys), (pres[0] if gelu else None), outs


def _assert_same(kept, plain):
    (yk, pk, ok), (yp, pp, op) = kept, plain
    assert yk.tobytes() == yp.tobytes()
    if pk is not None:
        assert pk.tobytes() == pp.tobytes()
    for a, b in zip(ok, op):
        for u, v in zip(a, b):
            assert u.tobytes() == v.tobytes()


# (M, K, n, groups, count, gelu): one weight, several groups, a depth-cut weight gradient (2048-row
# groups), the q/k/v form (three weights on one input), the GELU form, and 24-row groups (the pack is
# then not readable by the weight gradient and X^T is packed as usual)
KEPT = [
    (256, 96, 80, 1, 1, False),
    (512, 64, 2048, 2, 1, False),
    (512, 200, 130, 4, 1, False),
    (4096, 64, 48, 2, 1, False),
    (1024, 256, 128, 8, 3, False),
    (512, 64, 160, 2, 1, True),
    (96, 40, 24, 4, 1, False),
]


@pytest.mark.parametrize("mode", MODES)
@pytest.mark.parametrize("case", KEPT)
def test_kept_input_pack_keeps_the_bits(cuda, case, mode):
    torch = cuda
    M, K, n, groups, count, gelu = case
    x = orc.normal(11 + M, M * K).reshape(M, K).astype(np.float32)
    w = orc.normal(12 + K, count * n * K).reshape(count, n, K).astype(np.float32)
    b = orc.normal(13 + n, count * n).reshape(count, n).astype(np.float32)
    g = orc.normal(14 + n, count * M * n).reshape(count, M, n).astype(np.float32)
    _assert_same(_kept(torch, x, w, b, g, groups, mode, count=count, gelu=gelu),
                 _plain(torch, x, w, b, g, groups, mode, count=count, gelu=gelu))


def test_kept_input_pack_of_another_math_mode_is_ignored(cuda):
    """A pack written in TF32 mode is not read by a 3xTF32 backward (X is packed again)."""
    torch = cuda
    M, K, n, groups = 256, 64, 96, 2
    x = orc.normal(21, M * K).reshape(M, K).astype(np.float32)
    w = orc.normal(22, n * K).reshape(1, n, K).astype(np.float32)
    b = orc.normal(23, n).reshape(1, n).astype(np.float32)
    g = orc.normal(24, M * n).reshape(1, M, n).astype(np.float32)
    _, _, ok = _kept(torch, x, w, b, g, groups, nnb.MATH_FP32X3, fwd_mode=nnb.MATH_TF32)
    _, _, op = _plain(torch, x, w, b, g, groups, nnb.MATH_FP32X3)
    for u, v in zip(ok[0], op[0]):
        assert u.tobytes() == v.tobytes()


@pytest.mark.parametrize("mode", MODES)
def test_kept_input_pack_with_non_finite_inputs(cuda, mode):
    torch = cuda
    M, K, n, groups = 512, 72, 96, 2
    x = orc.normal(31, M * K).reshape(M, K).astype(np.float32)
    w = orc.normal(32, n * K).reshape(1, n, K).astype(np.float32)
    b = orc.normal(33, n).reshape(1, n).astype(np.float32)
    g = orc.normal(34, M * n).reshape(1, M, n).astype(np.float32)
    x[20, 3] = -np.inf
    x[400, 9] = np.nan
    kept = _kept(torch, x, w, b, g, groups, mode)
    _assert_same(kept, _plain(torch, x, w, b, g, groups, mode))
    dw = kept[2][0][1]
    assert np.isinf(dw[0][:, 3]).all() and np.isnan(dw[1][:, 9]).all() and np.isfinite(dw[0][:, 4]).all()
