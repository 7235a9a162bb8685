"""Parity of the B200 op kernels (through the C ABI) with the oracle restatements in oracle/.

The oracle follows the reference's evaluation order and is pinned to the reference build by
tests/test_oracle_ops.py. Ops whose kernels keep that order (relu, gelu, batchnorm, maxpool2d,
embedding, AdamW, column sums over <= 256 rows, conv bias gradient) must match bit for bit; ops
built on the tensor-core GEMM or on warp-tree row sums must match to fp32-grade tolerance:
|got - want| <= 2e-5 * max|want| + 2e-5 * |want| (GEMM, attention, conv) and 1e-5 scaled the same
way (layernorm, softmax / cross entropy).
"""
import ctypes

import numpy as np
import pytest

import nnb
from oracle import orc

pytestmark = pytest.mark.gpu
P = orc.ptr
O = orc.orc
L = None


def lib():
    return nnb.lib()


def dev(torch, a):
    return torch.from_numpy(np.ascontiguousarray(a)).cuda()


def host(t):
    return t.cpu().numpy()


def rnd(seed, *shape, lo=-1.0, hi=1.0):
    return orc.uniform(seed, int(np.prod(shape)), lo, hi).reshape(shape)


def nrm(seed, *shape):
    return orc.normal(seed, int(np.prod(shape))).reshape(shape)


def assert_close(got, want, rel=2e-5):
    got, want = np.asarray(got, np.float64), np.asarray(want, np.float64)
    assert got.shape == want.shape
    scale = np.abs(want).max() if want.size else 0.0
    err = np.abs(got - want)
    bound = rel * scale + rel * np.abs(want) + 1e-30
    assert np.all(err <= bound), f"max err {err.max():.3e} vs scale {scale:.3e}"


def assert_bits(got, want):
    assert np.asarray(got).tobytes() == np.asarray(want).tobytes()


def S(torch):
    return torch.cuda.current_stream().cuda_stream


def ok(st):
    nnb.check(st)


@pytest.mark.parametrize("M,K,n", [(37, 65, 23), (64, 3136, 128), (300, 512, 2048), (1000, 300, 10)])
def test_linear(cuda, M, K, n):
    torch = cuda
    x, w, b, g = rnd(3, M, K), rnd(4, n, K), rnd(5, n), rnd(6, M, n)
    y_o, dx_o, dw_o, db_o = orc.zeros(M, n), orc.zeros(M, K), orc.zeros(n, K), orc.zeros(n)
    O.orc_linear_fwd(M, K, n, P(x), P(w), P(b), P(y_o))
    O.orc_linear_bwd(M, K, n, P(g), P(x), P(w), P(dx_o), 1, P(dw_o), 1, P(db_o), 1)
    dx_, dw_, db_ = dev(torch, x), dev(torch, w), dev(torch, b)
    y = torch.empty(M, n, device="cuda")
    ok(lib().nnb_linear_fwd(S(torch), M, K, n, dx_.data_ptr(), dw_.data_ptr(), db_.data_ptr(), y.data_ptr()))
    gg = dev(torch, g)
    dx = torch.full((M, K), 7.0, device="cuda")
    dw = torch.full((n, K), 7.0, device="cuda")
    db = torch.full((n,), 7.0, device="cuda")
    ok(lib().nnb_linear_bwd(S(torch), M, K, n, gg.data_ptr(), dx_.data_ptr(), dw_.data_ptr(), dx.data_ptr(), 1,
                            dw.data_ptr(), 1, db.data_ptr(), 1))
    assert_close(host(y), y_o)
    assert_close(host(dx), dx_o)
    assert_close(host(dw), dw_o)
    if M <= 256:
        assert_bits(host(db), db_o)
    else:
        assert_close(host(db), db_o, rel=1e-5)
    # accumulate (first = 0) adds to what the buffers hold
    ok(lib().nnb_linear_bwd(S(torch), M, K, n, gg.data_ptr(), dx_.data_ptr(), dw_.data_ptr(), dx.data_ptr(), 0,
                            dw.data_ptr(), 0, db.data_ptr(), 0))
    assert_close(host(dx), 2 * dx_o)
    assert nnb.device_error() == 0


@pytest.mark.parametrize("M,K,n", [(37, 65, 23), (4096, 512, 512), (300, 96, 200)])
def test_linear_multi_matches_separate_linears(cuda, M, K, n):
    """nnb_linear_multi_fwd (one input under three weights, x packed once, one launch) gives each
    output nnb_linear_fwd's bits; the Python linear_multi takes that path for weights at one stride
    (a flat buffer laid out weight, bias, weight, bias, ...) and the per-layer path otherwise, with
    the same outputs and the same gradients either way."""
    torch = cuda
    from nnb import functional as F
    from nnb.autograd import Value
    x = dev(torch, rnd(11, M, K))
    per = n * K + n
    flat = dev(torch, rnd(12, 3 * per))
    ws = [flat[i * per: i * per + n * K].view(n, K) for i in range(3)]
    bs = [flat[i * per + n * K: (i + 1) * per] for i in range(3)]
    want = []
    for w, b in zip(ws, bs):
        y = torch.empty(M, n, device="cuda")
        ok(lib().nnb_linear_fwd(S(torch), M, K, n, x.data_ptr(), w.data_ptr(), b.data_ptr(), y.data_ptr()))
        want.append(host(y))
    y3 = torch.full((3, M, n), 7.0, device="cuda")
    ok(lib().nnb_linear_multi_fwd(S(torch), 3, M, K, n, x.data_ptr(), ws[0].data_ptr(), per, bs[0].data_ptr(), per,
                                  y3.data_ptr(), M * n))
    for i in range(3):
        assert_bits(host(y3[i]), want[i])
    st = lib().nnb_linear_multi_fwd(S(torch), 3, M, K, n, x.data_ptr(), ws[0].data_ptr(), n * K - 1, bs[0].data_ptr(),
                                    per, y3.data_ptr(), M * n)
    assert st == nnb.NNB_ERR_INVALID
    # the Python op: flat parameters (one launch) and separate tensors (per layer), forward and backward
    g = [dev(torch, rnd(20 + i, M, n)) for i in range(3)]
    grads = []
    # copies at uneven gaps (no single stride): the per-layer path
    spread = torch.empty(3 * per + 1024, device="cuda")
    offs = [0, per + 64, 2 * per + 320]
    ws2 = [spread[o: o + n * K].view(n, K) for o in offs]
    bs2 = [spread[o + n * K: o + per] for o in offs]
    for a, b in zip(ws2 + bs2, ws + bs):
        a.copy_(b)
    for batched, params in ((True, [(Value.leaf(w, True), Value.leaf(b, True)) for w, b in zip(ws, bs)]),
                            (False, [(Value.leaf(w, True), Value.leaf(b, True)) for w, b in zip(ws2, bs2)])):
        X = Value.leaf(x, True)
        nnb.trace_reset()
        nnb.trace_enable(True)
        outs = F.linear_multi(X, params)
        nnb.trace_enable(False)
        _, launches = nnb.trace_query(nnb.TRACE_GEMM)
        assert launches == (1 if batched else 3)
        for i, o in enumerate(outs):
            assert_bits(host(o.data), want[i])
        for i, o in enumerate(outs):
            o.backward(g[i])
        grads.append([host(X.grad)] + [host(t.grad) for p in params for t in p])
    for a, b in zip(grads[0], grads[1]):
        assert_bits(a, b)
    assert nnb.device_error() == 0


@pytest.mark.parametrize("R,D", [(29, 77), (4096, 512), (3, 1000)])
def test_layernorm(cuda, R, D):
    torch = cuda
    x, gm, bt, g = nrm(7, R, D), rnd(8, D), rnd(9, D), nrm(10, R, D)
    y_o, m_o, i_o = orc.zeros(R, D), orc.zeros(R), orc.zeros(R)
    O.orc_layernorm_fwd(R, D, P(x), P(gm), P(bt), 1e-5, P(y_o), P(m_o), P(i_o))
    dx_o, dg_o, db_o = orc.zeros(R, D), orc.zeros(D), orc.zeros(D)
    O.orc_layernorm_bwd(R, D, P(g), P(x), P(gm), P(m_o), P(i_o), P(dx_o), 1, P(dg_o), 1, P(db_o), 1)
    tx, tg, tb, tgr = dev(torch, x), dev(torch, gm), dev(torch, bt), dev(torch, g)
    y, m, iv = torch.empty(R, D, device="cuda"), torch.empty(R, device="cuda"), torch.empty(R, device="cuda")
    ok(lib().nnb_layernorm_fwd(S(torch), R, D, tx.data_ptr(), tg.data_ptr(), tb.data_ptr(), 1e-5, y.data_ptr(),
                               m.data_ptr(), iv.data_ptr()))
    dx, dg, db = torch.empty(R, D, device="cuda"), torch.empty(D, device="cuda"), torch.empty(D, device="cuda")
    ok(lib().nnb_layernorm_bwd(S(torch), R, D, tgr.data_ptr(), tx.data_ptr(), tg.data_ptr(), m.data_ptr(),
                               iv.data_ptr(), dx.data_ptr(), 1, dg.data_ptr(), 1, db.data_ptr(), 1))
    assert_close(host(y), y_o, 1e-5)
    assert_close(host(m), m_o, 1e-5)
    assert_close(host(iv), i_o, 1e-5)
    assert_close(host(dx), dx_o, 1e-5)
    assert_close(host(dg), dg_o, 1e-5)
    assert_close(host(db), db_o, 1e-5)


@pytest.mark.parametrize("fuse", [0, 1])
@pytest.mark.parametrize("N,C,S_", [(5, 6, 37), (64, 32, 196)])
def test_batchnorm_bitwise(cuda, fuse, N, C, S_):
    torch = cuda
    x, w, b, g = nrm(11, N, C, S_), rnd(12, C), rnd(13, C), nrm(14, N, C, S_)
    y_o, al_o, m_o, v_o, i_o = (orc.zeros(N, C, S_), np.zeros((N, C, S_), np.uint8), orc.zeros(C), orc.zeros(C),
                                orc.zeros(C))
    O.orc_batchnorm_fwd(N, C, S_, P(x), P(w), P(b), 1e-5, fuse, P(y_o), P(al_o), P(m_o), P(v_o), P(i_o))
    dx_o, dw_o, db_o = orc.zeros(N, C, S_), orc.zeros(C), orc.zeros(C)
    O.orc_batchnorm_bwd(N, C, S_, P(g), P(x), P(w), P(m_o), P(i_o), P(al_o) if fuse else None, P(dx_o), 1, P(dw_o), 1,
                        P(db_o), 1)
    tx, tw, tb, tg = dev(torch, x), dev(torch, w), dev(torch, b), dev(torch, g)
    y = torch.empty(N, C, S_, device="cuda")
    al = torch.empty(N, C, S_, dtype=torch.uint8, device="cuda")
    m, v, iv = (torch.empty(C, device="cuda") for _ in range(3))
    ok(lib().nnb_batchnorm_fwd(S(torch), N, C, S_, tx.data_ptr(), tw.data_ptr(), tb.data_ptr(), 1e-5, fuse,
                               y.data_ptr(), al.data_ptr(), m.data_ptr(), v.data_ptr(), iv.data_ptr()))
    dx, dw, db = torch.empty(N, C, S_, device="cuda"), torch.empty(C, device="cuda"), torch.empty(C, device="cuda")
    ok(lib().nnb_batchnorm_bwd(S(torch), N, C, S_, tg.data_ptr(), tx.data_ptr(), tw.data_ptr(), m.data_ptr(),
                               iv.data_ptr(), al.data_ptr() if fuse else None, dx.data_ptr(), 1, dw.data_ptr(), 1,
                               db.data_ptr(), 1))
    for got, want in ((y, y_o), (m, m_o), (v, v_o), (iv, i_o), (dx, dx_o), (dw, dw_o), (db, db_o)):
        assert_bits(host(got), want)
    if fuse:
        assert_bits(host(al), al_o)


@pytest.mark.parametrize("N,T,D,H,causal,padded", [(3, 19, 24, 4, 1, 0), (3, 19, 24, 4, 0, 1), (2, 70, 64, 2, 0, 0),
                                                    (2, 256, 512, 8, 1, 0)])
def test_attention(cuda, N, T, D, H, causal, padded):
    torch = cuda
    q, k, v, g = nrm(15, N, T, D), nrm(16, N, T, D), nrm(17, N, T, D), nrm(18, N, T, D)
    pad = None
    if padded:
        pad = np.ones((N, T), np.float32)
        pad[1, T - 4:] = 0.0
        pad[2 % N, 3] = 0.0
    out_o, pr_o = orc.zeros(N, T, D), orc.zeros(N, H, T, T)
    O.orc_attention_fwd(N, T, T, D, H, P(q), P(k), P(v), P(pad), causal, P(out_o), P(pr_o))
    dq_o, dk_o, dv_o = orc.zeros(N, T, D), orc.zeros(N, T, D), orc.zeros(N, T, D)
    O.orc_attention_bwd(N, T, T, D, H, P(g), P(q), P(k), P(v), P(pr_o), P(pad), causal, P(dq_o), 1, P(dk_o), 1,
                        P(dv_o), 1)
    tq, tk, tv, tg = dev(torch, q), dev(torch, k), dev(torch, v), dev(torch, g)
    tpad = dev(torch, pad) if padded else None
    out, pr = torch.empty(N, T, D, device="cuda"), torch.empty(N, H, T, T, device="cuda")
    ok(lib().nnb_attention_fwd(S(torch), N, T, T, D, H, tq.data_ptr(), tk.data_ptr(), tv.data_ptr(),
                               tpad.data_ptr() if padded else None, causal, out.data_ptr(), pr.data_ptr()))
    dq, dk, dv = (torch.empty(N, T, D, device="cuda") for _ in range(3))
    ok(lib().nnb_attention_bwd(S(torch), N, T, T, D, H, tg.data_ptr(), tq.data_ptr(), tk.data_ptr(), tv.data_ptr(),
                               pr.data_ptr(), tpad.data_ptr() if padded else None, causal, dq.data_ptr(), 1,
                               dk.data_ptr(), 1, dv.data_ptr(), 1))
    assert_close(host(pr), pr_o, 1e-4)
    assert_close(host(out), out_o, 1e-4)
    for got, want in ((dq, dq_o), (dk, dk_o), (dv, dv_o)):
        assert_close(host(got), want, 1e-4)
    if causal:
        p = host(pr)
        assert np.all(np.triu(p[0, 0], 1) == 0.0)     # causally hidden keys are exactly zero


@pytest.mark.parametrize("N,Cin,H,W,Cout,k,stride,pad,fuse", [(3, 2, 9, 8, 5, 3, 1, 1, 1), (3, 2, 9, 8, 5, 3, 2, 0, 0),
                                                            (64, 1, 28, 28, 32, 3, 1, 1, 1),
                                                            (64, 32, 14, 14, 64, 3, 1, 1, 1)])
def test_conv2d(cuda, N, Cin, H, W, Cout, k, stride, pad, fuse):
    torch = cuda
    x, w, b = nrm(19, N, Cin, H, W), rnd(20, Cout, Cin, k, k), rnd(21, Cout)
    ho, wo = (H + 2 * pad - k) // stride + 1, (W + 2 * pad - k) // stride + 1
    g = nrm(22, N, Cout, ho, wo)
    y_o, al_o = orc.zeros(N, Cout, ho, wo), np.zeros((N, Cout, ho, wo), np.uint8)
    O.orc_conv2d_fwd(N, Cin, H, W, Cout, k, k, stride, pad, P(x), P(w), P(b), fuse, P(y_o), P(al_o))
    dx_o, dw_o, db_o = orc.zeros(N, Cin, H, W), orc.zeros(Cout, Cin, k, k), orc.zeros(Cout)
    O.orc_conv2d_bwd(N, Cin, H, W, Cout, k, k, stride, pad, P(g), P(x), P(w), P(al_o) if fuse else None, P(dx_o), 1,
                     P(dw_o), 1, P(db_o), 1)
    tx, tw, tb, tg = dev(torch, x), dev(torch, w), dev(torch, b), dev(torch, g)
    y = torch.empty(N, Cout, ho, wo, device="cuda")
    al = torch.empty(N, Cout, ho, wo, dtype=torch.uint8, device="cuda")
    ok(lib().nnb_conv2d_fwd(S(torch), N, Cin, H, W, Cout, k, k, stride, pad, tx.data_ptr(), tw.data_ptr(),
                            tb.data_ptr(), fuse, y.data_ptr(), al.data_ptr() if fuse else None))
    assert_close(host(y), y_o)
    # the backward is checked on the oracle's alive mask, so both sides see the same masked gradient
    tal = dev(torch, al_o) if fuse else None
    dx, dw, db = torch.empty(N, Cin, H, W, device="cuda"), torch.empty(Cout, Cin, k, k, device="cuda"), torch.empty(
        Cout, device="cuda")
    ok(lib().nnb_conv2d_bwd(S(torch), N, Cin, H, W, Cout, k, k, stride, pad, tg.data_ptr(), tx.data_ptr(),
                            tw.data_ptr(), tal.data_ptr() if fuse else None, dx.data_ptr(), 1, dw.data_ptr(), 1,
                            db.data_ptr(), 1))
    assert_close(host(dx), dx_o)
    assert_close(host(dw), dw_o)
    assert_bits(host(db), db_o)
    if fuse:   # the mask agrees wherever the output is not within rounding of zero
        near0 = np.abs(y_o) < 1e-4
        assert np.array_equal(host(al)[~near0], al_o[~near0])


@pytest.mark.parametrize("N,Cin,H,W,Cout,k,stride,pad", [(2, 3, 11, 10, 7, 5, 2, 2), (1, 4, 6, 7, 300, 3, 3, 1),
                                                         (5, 130, 5, 5, 3, 1, 1, 0)])
def test_conv2d_implicit_gemm_edges(cuda, N, Cin, H, W, Cout, k, stride, pad):
    """The gathered-operand convolution at shapes the configs do not reach: a 5x5 kernel at stride 2
    (the input gradient's gather skips positions no window reads), more output channels than one
    128-row tile, a 1x1 kernel with 130 input channels (the depth spans several 16-wide stages); then
    accumulation into existing gradients (first = 0) and Inf / NaN inputs propagated as IEEE fp32."""
    torch = cuda
    x, w, b = nrm(23, N, Cin, H, W), rnd(24, Cout, Cin, k, k), rnd(25, Cout)
    ho, wo = (H + 2 * pad - k) // stride + 1, (W + 2 * pad - k) // stride + 1
    g = nrm(26, N, Cout, ho, wo)
    y_o, al_o = orc.zeros(N, Cout, ho, wo), np.zeros((N, Cout, ho, wo), np.uint8)
    O.orc_conv2d_fwd(N, Cin, H, W, Cout, k, k, stride, pad, P(x), P(w), P(b), 0, P(y_o), P(al_o))
    dx_o, dw_o, db_o = orc.zeros(N, Cin, H, W), orc.zeros(Cout, Cin, k, k), orc.zeros(Cout)
    O.orc_conv2d_bwd(N, Cin, H, W, Cout, k, k, stride, pad, P(g), P(x), P(w), None, P(dx_o), 1, P(dw_o), 1, P(db_o), 1)
    tx, tw, tb, tg = dev(torch, x), dev(torch, w), dev(torch, b), dev(torch, g)
    y = torch.empty(N, Cout, ho, wo, device="cuda")
    ok(lib().nnb_conv2d_fwd(S(torch), N, Cin, H, W, Cout, k, k, stride, pad, tx.data_ptr(), tw.data_ptr(),
                            tb.data_ptr(), 0, y.data_ptr(), None))
    assert_close(host(y), y_o)
    dx = torch.full((N, Cin, H, W), 3.0, device="cuda")
    dw = torch.full((Cout, Cin, k, k), 3.0, device="cuda")
    db = torch.full((Cout,), 3.0, device="cuda")
    for first in (1, 0):
        ok(lib().nnb_conv2d_bwd(S(torch), N, Cin, H, W, Cout, k, k, stride, pad, tg.data_ptr(), tx.data_ptr(),
                                tw.data_ptr(), None, dx.data_ptr(), first, dw.data_ptr(), first, db.data_ptr(), first))
        if first:
            assert_close(host(dx), dx_o)
            assert_close(host(dw), dw_o)
            assert_bits(host(db), db_o)
    assert_close(host(dx), 2 * dx_o)
    assert_close(host(dw), 2 * dw_o)
    assert_bits(host(db), db_o + db_o)
    # non-finite inputs
    x[0, 0, 1, 1] = np.inf
    x[N - 1, Cin - 1, H - 1, W - 2] = np.nan
    y_o2, al_o2 = orc.zeros(N, Cout, ho, wo), np.zeros((N, Cout, ho, wo), np.uint8)
    O.orc_conv2d_fwd(N, Cin, H, W, Cout, k, k, stride, pad, P(x), P(w), P(b), 0, P(y_o2), P(al_o2))
    ok(lib().nnb_conv2d_fwd(S(torch), N, Cin, H, W, Cout, k, k, stride, pad, dev(torch, x).data_ptr(), tw.data_ptr(),
                            tb.data_ptr(), 0, y.data_ptr(), None))
    got = host(y)
    assert np.array_equal(np.isnan(got), np.isnan(y_o2))
    inf = np.isinf(y_o2)
    assert np.array_equal(got[inf], y_o2[inf]) and not np.isinf(got[~inf]).any()
    fin = np.isfinite(y_o2)
    assert_close(got[fin], y_o2[fin])
    assert nnb.device_error() == 0


@pytest.mark.parametrize("k,stride,shape", [(2, 2, (64, 32, 28, 28)), (3, 1, (2, 3, 9, 10)), (3, 2, (2, 3, 9, 10))])
def test_maxpool_bitwise(cuda, k, stride, shape):
    torch = cuda
    N, C, H, W = shape
    x = nrm(23, N, C, H, W)
    x[0, 0, 0, :4] = 0.5
    ho, wo = (H - k) // stride + 1, (W - k) // stride + 1
    g = nrm(24, N, C, ho, wo)
    y_o, a_o, dx_o = orc.zeros(N, C, ho, wo), np.zeros((N, C, ho, wo), np.uint32), orc.zeros(N, C, H, W)
    O.orc_maxpool2d_fwd(N, C, H, W, k, stride, P(x), P(y_o), P(a_o))
    O.orc_maxpool2d_bwd(N, C, H, W, k, stride, P(g), P(a_o), P(dx_o), 1)
    tx, tg = dev(torch, x), dev(torch, g)
    y = torch.empty(N, C, ho, wo, device="cuda")
    a = torch.empty(N, C, ho, wo, dtype=torch.int32, device="cuda")
    dx = torch.empty(N, C, H, W, device="cuda")
    ok(lib().nnb_maxpool2d_fwd(S(torch), N, C, H, W, k, stride, tx.data_ptr(), y.data_ptr(), a.data_ptr()))
    ok(lib().nnb_maxpool2d_bwd(S(torch), N, C, H, W, k, stride, tg.data_ptr(), a.data_ptr(), dx.data_ptr(), 1))
    assert_bits(host(y), y_o)
    assert_bits(host(a).view(np.uint32), a_o)
    assert_bits(host(dx), dx_o)


GELU_SPECIALS = [np.nan, np.inf, -np.inf, 0.0, -0.0, 1e-40, -1e-40, 1e-30, -3e-39, 4.4, -4.4, 4.6, -4.6, 9.0,
                 -9.0, 43.6, -43.7, 88.0, 1e30, -1e30, 3.0e38, -3.0e38, 0.5, -0.5]


def assert_bits_or_both_nan(got, want):
    """Bitwise equal, except that a NaN's payload is not compared (the GPU's arithmetic returns its
    canonical NaN where the host's propagates the operand's)."""
    got, want = np.asarray(got, np.float32).ravel(), np.asarray(want, np.float32).ravel()
    nan = np.isnan(want)
    assert np.array_equal(np.isnan(got), nan)
    assert got[~nan].tobytes() == want[~nan].tobytes()


def test_gelu_vector_paths_bitwise(cuda):
    """The four-per-thread GELU kernels (packed fp32 pairs) against the reference's loops bit for bit:
    the backward with the tanh given and recomputed (nnb_gelu_bwd, length a multiple of 4), and the
    forward after linear_gelu's GEMM (its pre-activation set to special values through the bias and a
    zero input) against the scalar nnb_gelu_fwd of the same pre-activation. Specials: NaN, infinities,
    signed zeros, subnormals, values at the tanh clamp and past exp's range."""
    torch = cuda
    n = 100000
    x, g = rnd(41, n, lo=-12, hi=12), rnd(42, n)
    x[:len(GELU_SPECIALS)] = np.array(GELU_SPECIALS, np.float32)
    x[-len(GELU_SPECIALS):] = np.array(GELU_SPECIALS[::-1], np.float32)
    y_o, th_o, dx_o = orc.zeros(n), orc.zeros(n), orc.zeros(n)
    O.orc_gelu_fwd(n, P(x), P(y_o), P(th_o))
    O.orc_gelu_bwd(n, P(x), P(th_o), P(g), P(dx_o), 1)
    tx, tg, tth = dev(torch, x), dev(torch, g), dev(torch, th_o)
    dx = torch.empty(n, device="cuda")
    ok(lib().nnb_gelu_bwd(S(torch), n, tx.data_ptr(), tth.data_ptr(), tg.data_ptr(), dx.data_ptr(), 1))
    assert_bits_or_both_nan(host(dx), dx_o)
    ok(lib().nnb_gelu_bwd(S(torch), n, tx.data_ptr(), None, tg.data_ptr(), dx.data_ptr(), 1))
    assert_bits_or_both_nan(host(dx), dx_o)
    # forward: pre = 0 . w^T + b = b (the epilogue stores acc + 0, then adds the bias)
    M, K, cols = 3, 8, 1024
    b = rnd(43, cols, lo=-12, hi=12)
    b[:len(GELU_SPECIALS)] = np.array(GELU_SPECIALS, np.float32)
    xz, w, tb = torch.zeros(M, K, device="cuda"), dev(torch, rnd(44, cols, K)), dev(torch, b)
    y, pre = torch.empty(M, cols, device="cuda"), torch.empty(M, cols, device="cuda")
    ok(lib().nnb_linear_gelu_fwd(S(torch), M, K, cols, xz.data_ptr(), w.data_ptr(), tb.data_ptr(), y.data_ptr(),
                                 pre.data_ptr()))
    ys, ths = torch.empty(M * cols, device="cuda"), torch.empty(M * cols, device="cuda")
    ok(lib().nnb_gelu_fwd(S(torch), M * cols, pre.data_ptr(), ys.data_ptr(), ths.data_ptr()))
    assert_bits_or_both_nan(host(y), host(ys))
    assert np.isnan(host(y)[0, 0]) and np.isinf(host(pre)[0, 1])
    assert nnb.device_error() == 0


def test_gelu_relu_bitwise(cuda):
    torch = cuda
    n = 100003
    x, g = rnd(1, n, lo=-10, hi=10), rnd(2, n)
    y_o, th_o, dx_o = orc.zeros(n), orc.zeros(n), orc.zeros(n)
    O.orc_gelu_fwd(n, P(x), P(y_o), P(th_o))
    O.orc_gelu_bwd(n, P(x), P(th_o), P(g), P(dx_o), 1)
    tx, tg = dev(torch, x), dev(torch, g)
    y, th, dx = (torch.empty(n, device="cuda") for _ in range(3))
    ok(lib().nnb_gelu_fwd(S(torch), n, tx.data_ptr(), y.data_ptr(), th.data_ptr()))
    ok(lib().nnb_gelu_bwd(S(torch), n, tx.data_ptr(), th.data_ptr(), tg.data_ptr(), dx.data_ptr(), 1))
    assert_bits(host(y), y_o)
    assert_bits(host(th), th_o)
    assert_bits(host(dx), dx_o)
    ok(lib().nnb_gelu_bwd(S(torch), n, tx.data_ptr(), None, tg.data_ptr(), dx.data_ptr(), 1))   # tanh recomputed
    assert_bits(host(dx), dx_o)
    O.orc_relu_fwd(n, P(x), P(y_o))
    O.orc_relu_bwd(n, P(x), P(g), P(dx_o), 1)
    ok(lib().nnb_relu_fwd(S(torch), n, tx.data_ptr(), y.data_ptr()))
    ok(lib().nnb_relu_bwd(S(torch), n, tx.data_ptr(), tg.data_ptr(), dx.data_ptr(), 1))
    assert_bits(host(y), y_o)
    assert_bits(host(dx), dx_o)


def test_gemm_gelu_epilogue_matches_separate_gelu(cuda):
    """A GEMM with the GELU epilogue equals the GEMM followed by the gelu kernel, bit for bit."""
    torch = cuda
    M, K, n = 130, 200, 300
    x, w, b = rnd(40, M, K), rnd(41, n, K), rnd(42, n)
    tx, tw, tb = dev(torch, x), dev(torch, w), dev(torch, b)
    y = torch.empty(M, n, device="cuda")
    ok(lib().nnb_linear_fwd(S(torch), M, K, n, tx.data_ptr(), tw.data_ptr(), tb.data_ptr(), y.data_ptr()))
    yg, th = torch.empty(M, n, device="cuda"), torch.empty(M, n, device="cuda")
    ok(lib().nnb_gelu_fwd(S(torch), M * n, y.data_ptr(), yg.data_ptr(), th.data_ptr()))
    fused, pre = torch.empty(M, n, device="cuda"), torch.empty(M, n, device="cuda")
    ok(lib().nnb_linear_gelu_fwd(S(torch), M, K, n, tx.data_ptr(), tw.data_ptr(), tb.data_ptr(), fused.data_ptr(),
                                 pre.data_ptr()))
    assert torch.equal(pre, y)
    assert torch.equal(fused, yg)


def test_cross_entropy(cuda):
    torch = cuda
    N, C = 64, 10
    logits, t = nrm(25, N, C), orc.integers(26, N, 0, C - 1)
    sm_o, loss_o, dl_o = orc.zeros(N, C), orc.zeros(1), orc.zeros(N, C)
    O.orc_cross_entropy_fwd(N, C, P(logits), P(t), P(sm_o), P(loss_o))
    O.orc_cross_entropy_bwd(N, C, P(sm_o), P(t), 1.0, P(dl_o), 1)
    tl, tt = dev(torch, logits), dev(torch, t)
    sm, loss, norm = torch.empty(N, C, device="cuda"), torch.empty(1, device="cuda"), torch.empty(1, device="cuda")
    ok(lib().nnb_cross_entropy_fwd(S(torch), N, C, tl.data_ptr(), tt.data_ptr(), sm.data_ptr(), loss.data_ptr(),
                                   norm.data_ptr()))
    one = torch.ones(1, device="cuda")
    dl = torch.empty(N, C, device="cuda")
    ok(lib().nnb_cross_entropy_bwd(S(torch), N, C, sm.data_ptr(), tt.data_ptr(), one.data_ptr(), norm.data_ptr(),
                                   dl.data_ptr(), 1))
    assert_close(host(loss), loss_o, 1e-5)
    assert_close(host(sm), sm_o, 1e-5)
    assert_close(host(dl), dl_o, 1e-5)


@pytest.mark.parametrize("ls", [0.0, 0.1])
def test_sequence_ce(cuda, ls):
    torch = cuda
    P_, V = 2048, 4096
    logits, t = nrm(27, P_, V), orc.integers(28, P_, 0, V - 1)
    t[4] = -100
    sm_o, loss_o, dl_o = orc.zeros(P_, V), orc.zeros(1), orc.zeros(P_, V)
    O.orc_sequence_ce_fwd(P_, V, P(logits), P(t), -100, ls, P(sm_o), P(loss_o))
    O.orc_sequence_ce_bwd(P_, V, P(sm_o), P(t), -100, ls, 1.0, P_ - 1, P(dl_o), 1)
    tl, tt = dev(torch, logits), dev(torch, t)
    sm, loss, norm = torch.empty(P_, V, device="cuda"), torch.empty(1, device="cuda"), torch.empty(1, device="cuda")
    ok(lib().nnb_sequence_ce_fwd(S(torch), P_, V, tl.data_ptr(), tt.data_ptr(), -100, ls, sm.data_ptr(),
                                 loss.data_ptr(), norm.data_ptr()))
    one = torch.ones(1, device="cuda")
    dl = torch.empty(P_, V, device="cuda")
    ok(lib().nnb_sequence_ce_bwd(S(torch), P_, V, sm.data_ptr(), tt.data_ptr(), -100, ls, one.data_ptr(),
                                 norm.data_ptr(), dl.data_ptr(), 1))
    assert_close(host(loss), loss_o, 1e-5)
    assert_close(host(dl), dl_o, 1e-5)
    assert np.all(host(dl)[4] == 0.0)


def test_embedding_bitwise(cuda):
    torch = cuda
    V, D, cnt = 4096, 512, 5000
    w, ids, g = nrm(29, V, D), orc.integers(30, cnt, 0, 99), nrm(31, cnt, D)   # many repeats per id
    out_o, dw_o = orc.zeros(cnt, D), nrm(32, V, D)
    dw_init = dw_o.copy()
    O.orc_embedding_fwd(D, P(w), P(ids), cnt, P(out_o))
    O.orc_embedding_bwd(D, P(ids), cnt, P(g), P(dw_o))
    tw, ti, tg = dev(torch, w), dev(torch, ids), dev(torch, g)
    out = torch.empty(cnt, D, device="cuda")
    dw = dev(torch, dw_init)
    ok(lib().nnb_embedding_fwd(S(torch), V, D, tw.data_ptr(), ti.data_ptr(), cnt, out.data_ptr()))
    ok(lib().nnb_embedding_bwd(S(torch), V, D, ti.data_ptr(), cnt, tg.data_ptr(), dw.data_ptr(), 0))
    assert_bits(host(dw), dw_o)
    # first: rows start from zero (ids 100.. get no token, so they become exactly 0)
    dz = orc.zeros(V, D)
    O.orc_embedding_bwd(D, P(ids), cnt, P(g), P(dz))
    ok(lib().nnb_embedding_bwd(S(torch), V, D, ti.data_ptr(), cnt, tg.data_ptr(), dw.data_ptr(), 1))
    assert_bits(host(dw), dz)
    dw = dev(torch, dw_init)
    ok(lib().nnb_embedding_bwd(S(torch), V, D, ti.data_ptr(), cnt, tg.data_ptr(), dw.data_ptr(), 0))
    assert_bits(host(out), out_o)
    assert_bits(host(dw), dw_o)


def test_adamw_bitwise(cuda):
    torch = cuda
    n = 100000
    w0, g = nrm(32, n), nrm(33, n)
    w, m, v = w0.copy(), orc.zeros(n), orc.zeros(n)
    tw, tg, tm, tv = dev(torch, w0), dev(torch, g), torch.zeros(n, device="cuda"), torch.zeros(n, device="cuda")
    for step in (1, 2, 3):
        O.orc_adamw_step(n, P(w), P(g), P(m), P(v), 3e-4, 0.9, 0.999, 1e-8, 1e-2, step)
        ok(lib().nnb_adamw_step(S(torch), n, tw.data_ptr(), tg.data_ptr(), tm.data_ptr(), tv.data_ptr(), 3e-4, 0.9,
                                0.999, 1e-8, 1e-2, step))
    assert_bits(host(tw), w)
    assert_bits(host(tm), m)
    assert_bits(host(tv), v)


def test_adamw_device_scalars_bitwise(cuda):
    """The graph-replayable AdamW (step counter, settings and bias-correction table in device memory)
    gives the host-scalar update's bits, also past the table's end where the corrections saturate."""
    torch = cuda
    n = 50000
    w0, g = nrm(34, n), nrm(35, n)
    table = np.zeros(2 * (1 << 16), np.float32)
    tlen = lib().nnb_adam_bias_table(ctypes.c_float(0.9), ctypes.c_float(0.999), table.ctypes.data, 1 << 16)
    assert 1000 < tlen < (1 << 16) and table[2 * tlen - 2] == 1.0 and table[2 * tlen - 1] == 1.0
    tab = dev(torch, table[: 2 * tlen].copy())
    f = np.float32
    shrink = f(1.0) - f(3e-4) * f(1e-2)
    hyper = dev(torch, np.array([shrink, 3e-4, 0.9, 0.999, 1e-8], np.float32))
    for t in (1, 2, 3, 500, tlen, tlen + 12345):
        a = [dev(torch, w0), dev(torch, g), dev(torch, nrm(36, n) * 0.1), dev(torch, np.abs(nrm(37, n)) * 0.01)]
        b = [x.clone() for x in a]
        ok(lib().nnb_adamw_step(S(torch), n, a[0].data_ptr(), a[1].data_ptr(), a[2].data_ptr(), a[3].data_ptr(), 3e-4,
                                0.9, 0.999, 1e-8, 1e-2, t))
        step = torch.tensor([t - 1], dtype=torch.int64, device="cuda")
        ok(lib().nnb_step_advance(S(torch), step.data_ptr()))
        ok(lib().nnb_adamw_step_device(S(torch), n, b[0].data_ptr(), b[1].data_ptr(), b[2].data_ptr(), b[3].data_ptr(),
                                       hyper.data_ptr(), tab.data_ptr(), tlen, step.data_ptr()))
        assert int(step.item()) == t
        for x, y in zip(a, b):
            assert_bits(host(x), host(y))


def test_shape_errors(cuda):
    torch = cuda
    a = torch.zeros(64, device="cuda")
    with pytest.raises(nnb.TensorShapeError):
        ok(lib().nnb_attention_fwd(S(torch), 1, 4, 4, 6, 4, a.data_ptr(), a.data_ptr(), a.data_ptr(), None, 0,
                                   a.data_ptr(), a.data_ptr()))          # D % heads != 0
    with pytest.raises(nnb.TensorShapeError):
        ok(lib().nnb_attention_fwd(S(torch), 1, 4, 5, 8, 2, a.data_ptr(), a.data_ptr(), a.data_ptr(), None, 1,
                                   a.data_ptr(), a.data_ptr()))          # causal with Tq != Tk
    with pytest.raises(nnb.TensorShapeError):
        ok(lib().nnb_conv2d_fwd(S(torch), 1, 1, 2, 2, 1, 5, 5, 1, 0, a.data_ptr(), a.data_ptr(), a.data_ptr(), 0,
                                a.data_ptr(), None))                     # kernel larger than the input
    with pytest.raises(nnb.TensorShapeError):
        ok(lib().nnb_maxpool2d_fwd(S(torch), 1, 1, 2, 2, 3, 1, a.data_ptr(), a.data_ptr(), a.data_ptr()))
