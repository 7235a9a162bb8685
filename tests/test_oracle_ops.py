"""Pins the op restatements in oracle/orc_ops.c to the reference build (CPU only).

Every op is run through the reference's own autograd op (oracle/_ref, compiled from the reference
sources; one forward, one backward with a given upstream gradient) and through the oracle's
restatement on the same seeded inputs. Ops without a GEMM must agree bit for bit (same serial
order, same libm calls). Ops built on sgemm use the plain triple loop in the oracle and the AVX2
blocked kernel in the reference, so they agree to the reference test's GEMM tolerance.
"""
import numpy as np
import pytest

from oracle import orc

ref = orc.ref()
pytestmark = pytest.mark.skipif(ref is None, reason="reference library not built (oracle/_ref)")
P = orc.ptr
O = orc.orc


def rnd(seed, *shape, lo=-1.0, hi=1.0):
    return orc.uniform(seed, int(np.prod(shape)), lo, hi).reshape(shape)


def nrm(seed, *shape):
    return orc.normal(seed, int(np.prod(shape))).reshape(shape)


def close(a, b, rel=2e-5, floor=1e-6):
    a, b = np.asarray(a, np.float64), np.asarray(b, np.float64)
    return np.all(np.abs(a - b) <= np.maximum(rel * np.abs(b), floor)), np.abs(a - b).max()


def test_gelu_relu_bitwise():
    x = rnd(1, 5000, lo=-6, hi=6)
    g = rnd(2, 5000)
    y_r, dx_r = orc.zeros(5000), orc.zeros(5000)
    ref.ref_gelu(5000, P(x), P(g), P(y_r), P(dx_r))
    y_o, th, dx_o = orc.zeros(5000), orc.zeros(5000), orc.zeros(5000)
    O.orc_gelu_fwd(5000, P(x), P(y_o), P(th))
    O.orc_gelu_bwd(5000, P(x), P(th), P(g), P(dx_o), 1)
    assert y_o.tobytes() == y_r.tobytes() and dx_o.tobytes() == dx_r.tobytes()
    ref.ref_relu(5000, P(x), P(g), P(y_r), P(dx_r))
    O.orc_relu_fwd(5000, P(x), P(y_o))
    O.orc_relu_bwd(5000, P(x), P(g), P(dx_o), 1)
    assert y_o.tobytes() == y_r.tobytes() and dx_o.tobytes() == dx_r.tobytes()


def test_tanh_restatement_matches_reference_tanh_inplace():
    """The oracle's Cephes tanh gives tanh_inplace's bits (test_kernels.cpp:437-460) and stays
    within 2e-7 of tanh."""
    xs = np.concatenate([np.arange(-12, 12, 0.0037, dtype=np.float32),
                         np.array([0, -0.0, 1e-30, -1e-8, 9, -9, 50, -50, 1e30, -1e30], np.float32)])
    r = xs.copy()
    ref.ref_tanh_inplace(P(r), len(r))
    got = np.array([O.orc_tanh_one(float(x)) for x in xs], np.float32)
    assert got.tobytes() == r.tobytes()
    assert np.all(np.abs(r.astype(np.float64) - np.tanh(xs.astype(np.float64))) <= 2e-7)


def test_linear_matches_reference():
    M, K, n = 37, 65, 23
    x, w, b, g = rnd(3, M, K), rnd(4, n, K), rnd(5, n), rnd(6, M, n)
    out_r = [orc.zeros(M, n), orc.zeros(M, K), orc.zeros(n, K), orc.zeros(n)]
    ref.ref_linear(M, K, n, P(x), P(w), P(b), P(g), *map(P, out_r))
    y, dx, dw, db = orc.zeros(M, n), orc.zeros(M, K), orc.zeros(n, K), orc.zeros(n)
    O.orc_linear_fwd(M, K, n, P(x), P(w), P(b), P(y))
    O.orc_linear_bwd(M, K, n, P(g), P(x), P(w), P(dx), 1, P(dw), 1, P(db), 1)
    for got, want in zip((y, dx, dw), out_r[:3]):
        assert close(got, want)[0]
    assert db.tobytes() == out_r[3].tobytes()          # Tensor::sum(0): same serial order


def test_layernorm_bitwise():
    R, D = 29, 77
    x, gm, bt, g = nrm(7, R, D), rnd(8, D), rnd(9, D), nrm(10, R, D)
    y_r, dx_r, dg_r, db_r = orc.zeros(R, D), orc.zeros(R, D), orc.zeros(D), orc.zeros(D)
    ref.ref_layernorm(R, D, P(x), P(gm), P(bt), 1e-5, P(g), P(y_r), P(dx_r), P(dg_r), P(db_r))
    y, mean, inv = orc.zeros(R, D), orc.zeros(R), orc.zeros(R)
    O.orc_layernorm_fwd(R, D, P(x), P(gm), P(bt), 1e-5, P(y), P(mean), P(inv))
    dx, dg, db = orc.zeros(R, D), orc.zeros(D), orc.zeros(D)
    O.orc_layernorm_bwd(R, D, P(g), P(x), P(gm), P(mean), P(inv), P(dx), 1, P(dg), 1, P(db), 1)
    for got, want in ((y, y_r), (dx, dx_r), (dg, dg_r), (db, db_r)):
        assert got.tobytes() == want.tobytes()


@pytest.mark.parametrize("fuse", [0, 1])
def test_batchnorm_bitwise(fuse):
    N, C, S = 5, 6, 37
    x, w, b, g = nrm(11, N, C, S), rnd(12, C), rnd(13, C), nrm(14, N, C, S)
    y_r, m_r, v_r = orc.zeros(N, C, S), orc.zeros(C), orc.zeros(C)
    dx_r, dw_r, db_r = orc.zeros(N, C, S), orc.zeros(C), orc.zeros(C)
    ref.ref_batchnorm(N, C, S, P(x), P(w), P(b), 1e-5, fuse, P(g), P(y_r), P(m_r), P(v_r), P(dx_r), P(dw_r), P(db_r))
    y, alive, m, v, inv = orc.zeros(N, C, S), np.zeros((N, C, S), np.uint8), orc.zeros(C), orc.zeros(C), orc.zeros(C)
    O.orc_batchnorm_fwd(N, C, S, P(x), P(w), P(b), 1e-5, fuse, P(y), P(alive), P(m), P(v), P(inv))
    dx, dw, db = orc.zeros(N, C, S), orc.zeros(C), orc.zeros(C)
    O.orc_batchnorm_bwd(N, C, S, P(g), P(x), P(w), P(m), P(inv), P(alive) if fuse else None, P(dx), 1, P(dw), 1, P(db), 1)
    for got, want in ((y, y_r), (m, m_r), (v, v_r), (dx, dx_r), (dw, dw_r), (db, db_r)):
        assert got.tobytes() == want.tobytes()


@pytest.mark.parametrize("causal,padded", [(1, 0), (0, 1), (0, 0)])
def test_attention_matches_reference(causal, padded):
    N, T, D, H = 3, 19, 24, 4
    q, k, v, g = nrm(15, N, T, D), nrm(16, N, T, D), nrm(17, N, T, D), nrm(18, N, T, D)
    pad = None
    if padded:
        pad = np.ones((N, T), np.float32)
        pad[1, 15:] = 0.0
        pad[2, 3] = 0.0
    outs_r = [orc.zeros(N, T, D) for _ in range(4)]
    ref.ref_attention(N, T, T, D, H, P(q), P(k), P(v), P(pad), causal, P(g), *map(P, outs_r))
    out, probs = orc.zeros(N, T, D), orc.zeros(N, H, T, T)
    O.orc_attention_fwd(N, T, T, D, H, P(q), P(k), P(v), P(pad), causal, P(out), P(probs))
    dq, dk, dv = orc.zeros(N, T, D), orc.zeros(N, T, D), orc.zeros(N, T, D)
    O.orc_attention_bwd(N, T, T, D, H, P(g), P(q), P(k), P(v), P(probs), P(pad), causal, P(dq), 1, P(dk), 1, P(dv), 1)
    for got, want in zip((out, dq, dk, dv), outs_r):
        ok, err = close(got, want, rel=1e-4, floor=1e-5)
        assert ok, err


@pytest.mark.parametrize("fuse,stride,pad", [(1, 1, 1), (0, 2, 0), (1, 2, 1)])
def test_conv2d_matches_reference(fuse, stride, pad):
    N, Cin, H, W, Cout, kh, kw = 3, 2, 9, 8, 5, 3, 3
    x, w, b = nrm(19, N, Cin, H, W), rnd(20, Cout, Cin, kh, kw), rnd(21, Cout)
    ho, wo = (H + 2 * pad - kh) // stride + 1, (W + 2 * pad - kw) // stride + 1
    g = nrm(22, N, Cout, ho, wo)
    y_r, dx_r, dw_r, db_r = orc.zeros(N, Cout, ho, wo), orc.zeros(N, Cin, H, W), orc.zeros(Cout, Cin, kh, kw), orc.zeros(Cout)
    ref.ref_conv2d(N, Cin, H, W, Cout, kh, kw, stride, pad, P(x), P(w), P(b), fuse, P(g), P(y_r), P(dx_r), P(dw_r), P(db_r))
    y, alive = orc.zeros(N, Cout, ho, wo), np.zeros((N, Cout, ho, wo), np.uint8)
    O.orc_conv2d_fwd(N, Cin, H, W, Cout, kh, kw, stride, pad, P(x), P(w), P(b), fuse, P(y), P(alive))
    dx, dw, db = orc.zeros(N, Cin, H, W), orc.zeros(Cout, Cin, kh, kw), orc.zeros(Cout)
    O.orc_conv2d_bwd(N, Cin, H, W, Cout, kh, kw, stride, pad, P(g), P(x), P(w), P(alive) if fuse else None,
                     P(dx), 1, P(dw), 1, P(db), 1)
    for got, want in ((y, y_r), (dx, dx_r), (dw, dw_r)):
        ok, err = close(got, want, rel=1e-4, floor=1e-5)
        assert ok, err
    if not fuse:
        assert db.tobytes() == db_r.tobytes()


@pytest.mark.parametrize("stride,pad,dil,groups", [(1, 1, 2, 1), (2, 2, 2, 2), (1, 0, 1, 3), (2, 1, 3, 6)])
def test_conv2d_dilated_grouped_matches_reference(stride, pad, dil, groups):
    """conv2d with dilation and groups (ops.cpp:1525-1607): GEMM-built outputs to the reference test's
    GEMM tolerance, the bias gradient (plain loops) bit for bit."""
    N, Cin, H, W, Cout, kh, kw = 2, 6, 11, 10, 6, 3, 3
    x, w, b = nrm(31, N, Cin, H, W), rnd(32, Cout, Cin // groups, kh, kw), rnd(33, Cout)
    ho = (H + 2 * pad - (dil * (kh - 1) + 1)) // stride + 1
    wo = (W + 2 * pad - (dil * (kw - 1) + 1)) // stride + 1
    g = nrm(34, N, Cout, ho, wo)
    y_r, dx_r = orc.zeros(N, Cout, ho, wo), orc.zeros(N, Cin, H, W)
    dw_r, db_r = orc.zeros(Cout, Cin // groups, kh, kw), orc.zeros(Cout)
    ref.ref_conv2d_ex(N, Cin, H, W, Cout, kh, kw, stride, pad, dil, groups, P(x), P(w), P(b), P(g), P(y_r), P(dx_r),
                      P(dw_r), P(db_r))
    y, dx = orc.zeros(N, Cout, ho, wo), orc.zeros(N, Cin, H, W)
    dw, db = orc.zeros(Cout, Cin // groups, kh, kw), orc.zeros(Cout)
    O.orc_conv2d_ex_fwd(N, Cin, H, W, Cout, kh, kw, stride, pad, dil, groups, P(x), P(w), P(b), P(y))
    O.orc_conv2d_ex_bwd(N, Cin, H, W, Cout, kh, kw, stride, pad, dil, groups, P(g), P(x), P(w), P(dx), P(dw), P(db))
    for got, want in ((y, y_r), (dx, dx_r), (dw, dw_r)):
        ok, err = close(got, want, rel=1e-4, floor=1e-5)
        assert ok, err
    assert db.tobytes() == db_r.tobytes()


@pytest.mark.parametrize("fuse", [0, 1])
@pytest.mark.parametrize("steps", [1, 3])
@pytest.mark.parametrize("params", ["default", "random"])
@pytest.mark.parametrize("shape", [(4, 3, 5, 6), (1, 3, 1, 7), (5, 2, 4, 1)])
def test_batchnorm_module_eval_bitwise(fuse, steps, params, shape):
    """BatchNorm2d (batchnorm.cpp:27-60, default eps 1e-5, momentum 0.1): `steps` training forwards
    update the running statistics, then one evaluation-mode forward and its backward, all bit for bit;
    with the default weight 1 and bias 0, and with random weight and bias of both signs (so the fused
    ReLU's decisions move and every w / b term of the restatement counts); shapes with size-1 axes
    check that a reduction is skipped where the reference skips it."""
    N, C, H, W = shape
    x = nrm(35, N, C, H, W) * 2.0 + 0.5
    g = nrm(36, N, C, H, W)
    if params == "default":
        w, b = np.ones(C, np.float32), np.zeros(C, np.float32)
    else:
        w, b = rnd(37, C, lo=-1.5, hi=1.5), rnd(38, C, lo=-1.0, hi=1.0)
    y_r, dx_r, dw_r, db_r = orc.zeros(N, C, H, W), orc.zeros(N, C, H, W), orc.zeros(C), orc.zeros(C)
    rm_r, rv_r = orc.zeros(C), orc.zeros(C)
    ref.ref_bn2d_module_ex(N, C, H, W, steps, 1, fuse, P(x), P(g), P(w), P(b), P(y_r), P(dx_r), P(dw_r), P(db_r),
                           P(rm_r), P(rv_r))
    rm, rv = np.zeros(C, np.float32), np.ones(C, np.float32)
    y_t, alive = orc.zeros(N, C, H, W), np.zeros((N, C, H, W), np.uint8)
    mean, var, inv = orc.zeros(C), orc.zeros(C), orc.zeros(C)
    for _ in range(steps):
        O.orc_batchnorm_fwd(N, C, H * W, P(x), P(w), P(b), 1e-5, fuse, P(y_t), P(alive), P(mean), P(var), P(inv))
        O.orc_bn_running_update(C, N * H * W, 0.1, P(mean), P(var), P(rm), P(rv))
    assert rm.tobytes() == rm_r.tobytes() and rv.tobytes() == rv_r.tobytes()
    y, dx, dw, db = orc.zeros(N, C, H, W), orc.zeros(N, C, H, W), orc.zeros(C), orc.zeros(C)
    O.orc_batchnorm_eval_fwd(N, C, H * W, P(x), P(w), P(b), P(rm), P(rv), 1e-5, fuse, P(y))
    O.orc_batchnorm_eval_bwd(N, C, H, W, P(g), P(x), P(w), P(b), P(rm), P(rv), 1e-5, fuse, P(dx), P(dw), P(db))
    for got, want in ((y, y_r), (dx, dx_r), (dw, dw_r), (db, db_r)):
        assert got.tobytes() == want.tobytes()
    if params == "random" and fuse:
        assert 0 < np.count_nonzero(y) < y.size          # the ReLU is active in both directions


@pytest.mark.parametrize("k,stride", [(2, 2), (3, 1), (3, 2)])
def test_maxpool_bitwise(k, stride):
    N, C, H, W = 2, 3, 9, 10
    x = nrm(23, N, C, H, W)
    x[0, 0, 0, :4] = 0.5                                  # ties: the first maximum wins
    ho, wo = (H - k) // stride + 1, (W - k) // stride + 1
    g = nrm(24, N, C, ho, wo)
    y_r, dx_r = orc.zeros(N, C, ho, wo), orc.zeros(N, C, H, W)
    ref.ref_maxpool2d(N, C, H, W, k, stride, P(x), P(g), P(y_r), P(dx_r))
    y, arg, dx = orc.zeros(N, C, ho, wo), np.zeros((N, C, ho, wo), np.uint32), orc.zeros(N, C, H, W)
    O.orc_maxpool2d_fwd(N, C, H, W, k, stride, P(x), P(y), P(arg))
    O.orc_maxpool2d_bwd(N, C, H, W, k, stride, P(g), P(arg), P(dx), 1)
    assert y.tobytes() == y_r.tobytes() and dx.tobytes() == dx_r.tobytes()


@pytest.mark.parametrize("k,stride", [(2, 2), (3, 1), (3, 2)])
def test_avgpool_bitwise(k, stride):
    """avgpool2d (ops.cpp:1707-1770), overlapping windows included (stride < k)."""
    N, C, H, W = 2, 3, 9, 10
    x = nrm(25, N, C, H, W)
    ho, wo = (H - k) // stride + 1, (W - k) // stride + 1
    g = nrm(26, N, C, ho, wo)
    y_r, dx_r = orc.zeros(N, C, ho, wo), orc.zeros(N, C, H, W)
    ref.ref_avgpool2d(N, C, H, W, k, stride, P(x), P(g), P(y_r), P(dx_r))
    y, dx = orc.zeros(N, C, ho, wo), orc.zeros(N, C, H, W)
    O.orc_avgpool2d_fwd(N, C, H, W, k, stride, P(x), P(y))
    O.orc_avgpool2d_bwd(N, C, H, W, k, stride, P(g), P(dx), 1)
    assert y.tobytes() == y_r.tobytes() and dx.tobytes() == dx_r.tobytes()


@pytest.mark.parametrize("axis", [0, 1, 2, 3, -1])
@pytest.mark.parametrize("average", [0, 1])
def test_reduce_axis_bitwise(axis, average):
    """sum / mean over one axis (ops.cpp:284-327) of a 4-D tensor."""
    shape = (3, 5, 7, 11)
    x = nrm(27, *shape)
    ax = axis % 4
    outer, n, inner = int(np.prod(shape[:ax])), shape[ax], int(np.prod(shape[ax + 1:]))
    g = nrm(28, outer * inner)
    y_r, dx_r = orc.zeros(outer * inner), orc.zeros(*shape)
    ref.ref_reduce4(*shape, axis, average, P(x), P(g), P(y_r), P(dx_r))
    y, dx = orc.zeros(outer * inner), orc.zeros(*shape)
    O.orc_reduce_axis_fwd(outer, n, inner, average, P(x), P(y))
    O.orc_reduce_axis_bwd(outer, n, inner, average, P(g), P(dx), 1)
    assert y.tobytes() == y_r.tobytes() and dx.tobytes() == dx_r.tobytes()


def test_global_avgpool_is_two_axis_means_bitwise():
    """GlobalAvgPool2d (pool2d.cpp:20-23) is mean(mean(x, 3), 2): the axis restatement twice."""
    N, C, H, W = 2, 3, 5, 6
    x = nrm(29, N, C, H, W)
    g = nrm(30, N * C)
    y_r, dx_r = orc.zeros(N * C), orc.zeros(N, C, H, W)
    ref.ref_global_avgpool(N, C, H, W, P(x), P(g), P(y_r), P(dx_r))
    m3, y = orc.zeros(N * C * H), orc.zeros(N * C)
    O.orc_reduce_axis_fwd(N * C * H, W, 1, 1, P(x), P(m3))
    O.orc_reduce_axis_fwd(N * C, H, 1, 1, P(m3), P(y))
    d3, dx = orc.zeros(N * C * H), orc.zeros(N, C, H, W)
    O.orc_reduce_axis_bwd(N * C, H, 1, 1, P(g), P(d3), 1)
    O.orc_reduce_axis_bwd(N * C * H, W, 1, 1, P(d3), P(dx), 1)
    assert y.tobytes() == y_r.tobytes() and dx.tobytes() == dx_r.tobytes()


def test_cross_entropy_bitwise():
    N, C = 33, 10
    logits, t = nrm(25, N, C), orc.integers(26, N, 0, C - 1)
    loss_r, dl_r = orc.zeros(1), orc.zeros(N, C)
    ref.ref_cross_entropy(N, C, P(logits), P(t), 1.0, P(loss_r), P(dl_r))
    sm, loss, dl = orc.zeros(N, C), orc.zeros(1), orc.zeros(N, C)
    O.orc_cross_entropy_fwd(N, C, P(logits), P(t), P(sm), P(loss))
    O.orc_cross_entropy_bwd(N, C, P(sm), P(t), 1.0, P(dl), 1)
    assert loss.tobytes() == loss_r.tobytes() and dl.tobytes() == dl_r.tobytes()


@pytest.mark.parametrize("ls", [0.0, 0.1])
def test_sequence_ce_bitwise(ls):
    N, T, V = 3, 7, 50
    logits, t = nrm(27, N, T, V), orc.integers(28, N * T, 0, V - 1)
    t[4] = -100
    loss_r, dl_r = orc.zeros(1), orc.zeros(N, T, V)
    ref.ref_sequence_ce(N, T, V, P(logits), P(t), -100, ls, 1.0, P(loss_r), P(dl_r))
    sm, loss, dl = orc.zeros(N * T, V), orc.zeros(1), orc.zeros(N, T, V)
    O.orc_sequence_ce_fwd(N * T, V, P(logits), P(t), -100, ls, P(sm), P(loss))
    O.orc_sequence_ce_bwd(N * T, V, P(sm), P(t), -100, ls, 1.0, N * T - 1, P(dl), 1)
    assert loss.tobytes() == loss_r.tobytes() and dl.tobytes() == dl_r.tobytes()


def test_embedding_bitwise():
    V, D, cnt = 17, 12, 60
    w, ids, g = nrm(29, V, D), orc.integers(30, cnt, 0, V - 1), nrm(31, cnt, D)
    out_r, dw_r = orc.zeros(cnt, D), orc.zeros(V, D)
    ref.ref_embedding(V, D, P(w), P(ids), cnt, P(g), P(out_r), P(dw_r))
    out, dw = orc.zeros(cnt, D), orc.zeros(V, D)
    O.orc_embedding_fwd(D, P(w), P(ids), cnt, P(out))
    O.orc_embedding_bwd(D, P(ids), cnt, P(g), P(dw))
    assert out.tobytes() == out_r.tobytes() and dw.tobytes() == dw_r.tobytes()


def test_adamw_bitwise():
    n = 1000
    w0, g = nrm(32, n), nrm(33, n)
    w_r = w0.copy()
    ref.ref_adamw(n, P(w_r), P(g), 3e-4, 0.9, 0.999, 1e-8, 1e-2, 3)
    w, m, v = w0.copy(), orc.zeros(n), orc.zeros(n)
    for step in (1, 2, 3):
        O.orc_adamw_step(n, P(w), P(g), P(m), P(v), 3e-4, 0.9, 0.999, 1e-8, 1e-2, step)
    assert w.tobytes() == w_r.tobytes()
