"""The linear backward's shared output-gradient pack: dX = G W packs G once (32-wide row panels) and
the weight gradient dW = G^T X reads that pack MN-major instead of packing G^T again.

The shared pack must not change a bit: for every shape (ragged feature counts, several groups, a
depth-cut weight gradient, shapes that cannot share because a group is not whole 16-row blocks)
and both math modes, nnb_linear_bwd / nnb_linear_bwd_grouped must give exactly the bits of the
same products run as separate nnb_sgemm_ex calls (each packing its own operands), and non-finite
gradients must still come out as the reference's IEEE results. The weight gradients are also held
to the fp64 bound of the GEMM tests.
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
# the depth cut (2048 rows >= 2 * max(1024, K)), and groups of 24 rows (not whole 16-row blocks: the
# weight gradient packs G^T itself)
SHAPES = [
    (256, 96, 80, 1),
    (512, 200, 130, 4),
    (4096, 64, 48, 2),
    (96, 40, 24, 4),
    (1024, 512, 512, 8),
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
