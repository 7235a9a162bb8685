"""Parity of the sm_100a GEMM (nnb_sgemm*, through the C ABI) with the fp64 oracle.

Re-expresses the reference's kernel tests (tests/test_kernels.cpp) for the GPU build:
sizes {1,7,33,257}^3 x trans flags x accumulate (:157-167), past each CPU block size
(:169-178), zero-size dimensions (:180-201), wide leading dimensions with sentinel padding
(:203-209), Inf/NaN propagation (:211-231) and determinism (:333-341). Tolerances:
3xTF32 |got - want| <= max(1e-5 * sum|a*b|, 1e-6) (the reference test's own bound, tighter than
1e-5*sqrt(K)); TF32 5e-3 * sum|a*b|.
"""
import itertools

import numpy as np
import pytest

import nnb
from oracle import orc

pytestmark = pytest.mark.gpu

SIZES = [1, 7, 33, 257]
MODES = [(nnb.MATH_FP32X3, 1e-5), (nnb.MATH_TF32, 5e-3)]


def run_gpu(torch, p, acc, mode, a=None, b=None, c=None):
    dev = torch.device("cuda")
    da = torch.from_numpy(p.a if a is None else a).to(dev)
    db = torch.from_numpy(p.b if b is None else b).to(dev)
    dc = torch.from_numpy((p.c if c is None else c).copy()).to(dev)
    nnb.sgemm(p.ta, p.tb, p.m, p.n, p.k, da, p.lda, db, p.ldb, dc, p.ldc, acc, math_mode=mode)
    out = dc.cpu().numpy()
    assert nnb.device_error() == 0
    return out


def check(p, got, acc, rel):
    want = orc.sgemm_f64(p, p.c, acc)
    mag = orc.magnitude(p, p.c, acc)
    full = got[: p.m * p.ldc].reshape(p.m, p.ldc) if p.m else np.zeros((0, p.ldc), np.float32)
    # padding columns untouched, no sentinel leaked into the result
    assert np.all(full[:, p.n:] == orc.SENTINEL)
    g = full[:, : p.n].astype(np.float64)
    nan_w, nan_g = np.isnan(want), np.isnan(g)
    assert np.array_equal(nan_w, nan_g), "NaN positions differ"
    inf = np.isinf(want) | np.isinf(g)
    assert np.array_equal(g[inf], want[inf]), "Inf values differ"
    fin = ~(nan_w | inf)
    assert np.all(np.abs(g[fin]) < 1e29)
    err = np.abs(g[fin] - want[fin])
    bound = np.maximum(rel * mag[fin], 1e-6)
    bad = err > bound
    assert not bad.any(), f"{bad.sum()} elements out of tolerance; worst ratio {(err / bound).max():.3g}"


@pytest.mark.parametrize("mode,rel", MODES)
def test_sizes_and_flags(cuda, mode, rel):
    seed = 4000
    for ta, tb, acc in itertools.product((0, 1), repeat=3):
        for m, n, k in itertools.product(SIZES, repeat=3):
            p = orc.Problem(ta, tb, m, n, k, 0, seed)
            seed += 1
            check(p, run_gpu(cuda, p, acc, mode), acc, rel)


@pytest.mark.parametrize("mode,rel", MODES)
def test_past_block_sizes_and_wide_ld(cuda, mode, rel):
    seed = 1000
    cases = [(101, 7, 33), (7, 33, 261), (7, 1029, 33), (7, 1029, 261), (129, 257, 17), (300, 300, 512)]
    for ta, tb, acc in itertools.product((0, 1), repeat=3):
        for m, n, k in cases:
            p = orc.Problem(ta, tb, m, n, k, 0, seed)
            seed += 1
            check(p, run_gpu(cuda, p, acc, mode), acc, rel)
        p = orc.Problem(ta, tb, 7, 33, 33, 3, seed)
        seed += 1
        check(p, run_gpu(cuda, p, acc, mode), acc, rel)


def test_zero_size_dimensions(cuda):
    """test_kernels.cpp:180-201: only the m x n region is written; k == 0 stores 0 or keeps C."""
    torch = cuda
    for m, n, k in [(0, 5, 4), (3, 0, 4), (3, 5, 0)]:
        for acc in (0, 1):
            ldc = 6
            a = torch.ones(16, device="cuda")
            b = torch.ones(32, device="cuda")
            c = torch.full((4 * ldc,), float(orc.SENTINEL), device="cuda")
            cv = c.view(4, ldc)
            cv[:m, :n] = 2.0
            nnb.sgemm(False, False, m, n, k, a, k if k else 1, b, n if n else 1, c, ldc, acc)
            got = c.cpu().numpy().reshape(4, ldc)
            for i in range(4):
                for j in range(ldc):
                    inside = i < m and j < n
                    want = (2.0 if acc else 0.0) if inside else orc.SENTINEL
                    assert got[i, j] == want
                    if inside and not acc:
                        assert not np.signbit(got[i, j])


@pytest.mark.parametrize("mode,rel", MODES)
def test_inf_nan_propagate_like_reference(cuda, mode, rel):
    seed = 3000
    for ta, tb, acc in itertools.product((0, 1), repeat=3):
        p = orc.Problem(ta, tb, 7, 33, 17, 0, seed)
        seed += 1
        p.a[2 if ta else 2 * p.lda] = np.inf
        for j in range(p.n):
            p.b[j * p.ldb if tb else j] = (1.0, -1.0, 0.0)[j % 3]
        p.b[3 * p.ldb + 5 if tb else 5 * p.ldb + 3] = np.nan
        got = run_gpu(cuda, p, acc, mode)
        loop = orc.sgemm_f32(p, p.c, acc)
        assert np.array_equal(np.isnan(got), np.isnan(loop))
        inf = np.isinf(loop)
        assert np.array_equal(got[inf], loop[inf])
        check(p, got, acc, rel)


def test_deterministic(cuda):
    """test_kernels.cpp:333-341: the same call twice gives the same bytes."""
    for acc in (0, 1):
        for mode, _ in MODES:
            p = orc.Problem(0, 1, 101, 75, 300, 2, 5000)
            g1 = run_gpu(cuda, p, acc, mode)
            g2 = run_gpu(cuda, p, acc, mode)
            assert g1.tobytes() == g2.tobytes()


def test_config1_matmul_512(cuda):
    """512^3, A then B from mt19937(0) U[-1,1], against the fp64 oracle."""
    torch = cuda
    n = 512
    ab = orc.uniform(0, 2 * n * n)
    a, b = ab[: n * n], ab[n * n:]
    c = np.zeros(n * n, np.float32)
    da, db = torch.from_numpy(a).cuda(), torch.from_numpy(b).cuda()
    dc = torch.from_numpy(c).cuda()
    nnb.sgemm(False, False, n, n, n, da, n, db, n, dc, n, False)
    got = dc.cpu().numpy().reshape(n, n).astype(np.float64)
    p = orc.Problem(0, 0, 1, 1, 1, 0, 0)   # reuse the oracle entry points on explicit buffers
    p.m = p.n = p.k = n
    p.lda = p.ldb = p.ldc = n
    p.a, p.b, p.c = a, b, c
    want = orc.sgemm_f64(p, c, False)
    mag = orc.magnitude(p, c, False)
    assert np.all(np.abs(got - want) <= 1e-5 * mag)
    # the north-star bound, relative error normalised by sum|a*b|
    assert (np.abs(got - want) / mag).max() <= 1e-5 * np.sqrt(n)


def test_strided_batched_matches_single(cuda):
    torch = cuda
    rng = np.random.default_rng(7)
    for ta, tb in itertools.product((0, 1), repeat=2):
        batch, m, n, k = 5, 70, 90, 130
        a = rng.standard_normal((batch, k, m) if ta else (batch, m, k)).astype(np.float32)
        b = rng.standard_normal((batch, n, k) if tb else (batch, k, n)).astype(np.float32)
        da, db = torch.from_numpy(a).cuda(), torch.from_numpy(b).cuda()
        dc = torch.zeros(batch, m, n, device="cuda")
        lda, ldb = (m if ta else k), (k if tb else n)
        nnb.sgemm_strided_batched(ta, tb, m, n, k, da, lda, a[0].size, db, ldb, b[0].size, dc, n, m * n, batch,
                                  False)
        for i in range(batch):
            one = torch.zeros(m, n, device="cuda")
            nnb.sgemm(ta, tb, m, n, k, da[i], lda, db[i], ldb, one, n, False, math_mode=nnb.MATH_FP32X3)
            assert torch.equal(one, dc[i])
        # broadcast B (stride 0)
        dc2 = torch.zeros(batch, m, n, device="cuda")
        nnb.sgemm_strided_batched(ta, tb, m, n, k, da, lda, a[0].size, db[0], ldb, 0, dc2, n, m * n, batch, False)
        for i in range(batch):
            one = torch.zeros(m, n, device="cuda")
            nnb.sgemm(ta, tb, m, n, k, da[i], lda, db[0], ldb, one, n, False, math_mode=nnb.MATH_FP32X3)
            assert torch.equal(one, dc2[i])


def test_large_sampled(cuda):
    """2048^3 and a ragged 3000 x 2500 x 1800, N(0,1): sampled rows/columns against fp64."""
    torch = cuda
    for (m, n, k), seed in (((2048, 2048, 2048), 41), ((3000, 2500, 1800), 42)):
        a = orc.normal(seed, m * k)
        b = orc.normal(seed + 100, k * n)
        da, db = torch.from_numpy(a).cuda(), torch.from_numpy(b).cuda()
        for mode, rel in MODES:
            dc = torch.zeros(m * n, device="cuda")
            nnb.sgemm(False, False, m, n, k, da, k, db, n, dc, n, False, math_mode=mode)
            got = dc.cpu().numpy().reshape(m, n)
            rows = np.r_[0, m - 1, np.arange(0, m, 97)].repeat(8)
            cols = np.tile(np.r_[0, n - 1, 131, 255, 256, n // 2, n - 2, 1], len(rows) // 8)
            val, mag = orc.sgemm_f64_sample(0, 0, k, a, k, b, n, None, n, 0, rows, cols)
            err = np.abs(got[rows, cols] - val)
            assert np.all(err <= rel * mag), (m, n, k, mode, (err / mag).max())


def test_16384_sampled(cuda):
    """The top of config 4's sweep, 16384^3 (1 GiB operands, 2^24 packed rows per operand): sampled
    rows and columns against fp64, both math modes."""
    torch = cuda
    m = n = k = 16384
    a = orc.normal(51, m * k)
    b = orc.normal(52, k * n)
    da, db = torch.from_numpy(a).cuda(), torch.from_numpy(b).cuda()
    rows = np.r_[0, m - 1, np.arange(0, m, 1021)].repeat(8)
    cols = np.tile(np.r_[0, n - 1, 255, 256, 8191, 8192, n - 2, 4097], len(rows) // 8)
    val, mag = orc.sgemm_f64_sample(0, 0, k, a, k, b, n, None, n, 0, rows, cols)
    for mode, rel in MODES:
        dc = torch.empty(m, n, device="cuda")
        nnb.sgemm(False, False, m, n, k, da, k, db, n, dc, n, False, math_mode=mode)
        got = dc[torch.from_numpy(rows).cuda(), torch.from_numpy(cols).cuda()].cpu().numpy()
        del dc
        err = np.abs(got - val)
        assert np.all(err <= rel * mag), (mode, (err / mag).max())
    assert nnb.device_error() == 0


@pytest.mark.parametrize("mode", [nnb.MATH_FP32X3, nnb.MATH_TF32])
@pytest.mark.parametrize("tb,n", [(0, 8192), (1, 8192), (0, 8000)])
def test_tile_width_does_not_change_bits(cuda, mode, tb, n):
    """A 1024-row band of a wide product runs on 224-wide tiles (296 tiles: two full waves of 148 SMs),
    the 4096-row product it is cut from on 256-wide ones: the band's rows are the same bits."""
    torch = cuda
    m_big, m_band, k = 4096, 1024, 256
    a = torch.from_numpy(orc.normal(71, m_big * k)).cuda().view(m_big, k)
    b = torch.from_numpy(orc.normal(72, k * n)).cuda()
    ldb = k if tb else n
    big = torch.zeros(m_big, n, device="cuda")
    nnb.sgemm(False, bool(tb), m_big, n, k, a, k, b, ldb, big, n, False, math_mode=mode)
    for r0 in (0, 2048):
        band = torch.zeros(m_band, n, device="cuda")
        nnb.sgemm(False, bool(tb), m_band, n, k, a[r0:], k, b, ldb, band, n, False, math_mode=mode)
        assert band.cpu().numpy().tobytes() == big[r0:r0 + m_band].cpu().numpy().tobytes()
    assert nnb.device_error() == 0


@pytest.mark.parametrize("ta,tb,m,n,k", [(0, 0, 4096, 4096, 1024), (1, 1, 4000, 4096, 1100), (0, 1, 3000, 4096, 2048)])
def test_tf32_wide_tiles_same_bits_as_narrow(cuda, ta, tb, m, n, k):
    """TF32 products with at least 148 256 x 256 work items and a depth of 64+ k-blocks run on the wide
    tiles (two 128-row halves sharing each B stage); the 2048-row bands they are cut into here have too
    few such items and run on the 128 x 256 tiles. Each band's rows are the full product's bits, and the
    full product is within the TF32 bound of the fp64 oracle on sampled elements."""
    torch = cuda
    a_h = orc.normal(81, m * k)
    b_h = orc.normal(82, k * n)
    a = torch.from_numpy(a_h).cuda()
    b = torch.from_numpy(b_h).cuda()
    lda, ldb = (m if ta else k), (k if tb else n)
    full = torch.zeros(m, n, device="cuda")
    nnb.sgemm(bool(ta), bool(tb), m, n, k, a, lda, b, ldb, full, n, False, math_mode=nnb.MATH_TF32)
    for r0 in range(0, m, 2048):
        rows = min(2048, m - r0)
        band = torch.zeros(rows, n, device="cuda")
        a_band = a[r0:] if ta else a[r0 * k:]         # op(A) rows r0.. : columns of a stored k x m
        nnb.sgemm(bool(ta), bool(tb), rows, n, k, a_band, lda, b, ldb, band, n, False, math_mode=nnb.MATH_TF32)
        assert band.cpu().numpy().tobytes() == full[r0:r0 + rows].cpu().numpy().tobytes(), r0
    got = full.cpu().numpy()
    rows = np.r_[0, m - 1, np.arange(0, m, 251)].repeat(8)
    cols = np.tile(np.r_[0, n - 1, 255, 256, n // 2, 127, n - 2, 1], len(rows) // 8)
    val, mag = orc.sgemm_f64_sample(ta, tb, k, a_h, lda, b_h, ldb, None, n, 0, rows, cols)
    err = np.abs(got[rows, cols] - val)
    assert np.all(err <= 5e-3 * mag), (err / mag).max()
    assert nnb.device_error() == 0


def test_argument_errors(cuda):
    torch = cuda
    a = torch.zeros(64, device="cuda")
    with pytest.raises(ValueError):
        nnb.sgemm(False, False, 4, 4, 4, a, 3, a, 4, a, 4, False)   # lda < k
    with pytest.raises(ValueError):
        nnb.sgemm(False, False, 4, 4, 4, a, 4, a, 4, a, 3, False)   # ldc < n
    with pytest.raises(ValueError):
        nnb.sgemm(False, False, 4, 4, 4, None, 4, a, 4, a, 4, False)


@pytest.mark.parametrize("mode,rel", MODES)
def test_depth_cut_small_output_long_depth(cuda, mode, rel):
    """Few output tiles and a long depth take the fixed-order depth cut (the reference's
    gemm.cpp:453-485 counterpart): still within tolerance, ragged last piece, accumulate, Inf/NaN."""
    torch = cuda
    for (ta, tb, m, n, k, acc), seed in zip([(1, 0, 64, 96, 4096, 0), (0, 1, 100, 50, 5000, 1), (1, 0, 512, 512, 9000, 0)],
                                            (601, 602, 603)):
        p = orc.Problem(ta, tb, m, n, k, 0, seed)
        check(p, run_gpu(torch, p, acc, mode), acc, rel)
        g1 = run_gpu(torch, p, acc, mode)
        g2 = run_gpu(torch, p, acc, mode)
        assert g1.tobytes() == g2.tobytes()
    p = orc.Problem(0, 0, 7, 33, 4100, 0, 604)
    p.a[2 * p.lda + 4099] = np.inf                    # in the last depth piece
    p.b[1000 * p.ldb + 5] = np.nan
    got = run_gpu(torch, p, 0, mode)
    loop = orc.sgemm_f32(p, p.c, 0)
    assert np.array_equal(np.isnan(got), np.isnan(loop))
    inf = np.isinf(loop)
    assert np.array_equal(got[inf], loop[inf])


@pytest.mark.parametrize("mode", [nnb.MATH_FP32X3, nnb.MATH_TF32])
@pytest.mark.parametrize("ta,tb,m,n,k,pad,acc", [
    (0, 0, 3000, 4100, 300, 0, 0),      # several bands over one packed B, partial last band
    (1, 0, 5000, 2300, 129, 3, 1),      # transposed A (column bands of its storage), strides, accumulate
    (0, 1, 77, 1030, 700, 1, 0),        # one band
    (1, 1, 2100, 64, 2048, 2, 1),       # deep k (depth cut inside the band, B packed per piece)
    (1, 1, 5000, 2048, 4096, 2, 1),     # depth cut in several bands
    (0, 0, 1, 1, 1, 0, 0),              # the reference sweep's smallest sizes
    (1, 0, 7, 33, 257, 1, 1),
    (0, 1, 257, 1, 33, 2, 0),           # one output column
    (0, 0, 300, 40, 0, 0, 0),           # k == 0: C zeroed
    (1, 1, 300, 40, 0, 1, 1),           # k == 0 accumulating: C unchanged
])
def test_sgemm_host_bitwise_equal_to_device(cuda, mode, ta, tb, m, n, k, pad, acc):
    """nnb_sgemm_host (host buffers, banded pipeline of copies and GEMMs) gives the device entry's bits
    on the same operands, padding columns of C untouched."""
    torch = cuda
    p = orc.Problem(ta, tb, m, n, k, pad, 7000 + m)
    want = run_gpu(torch, p, acc, mode)
    c_host = p.c.copy()
    nnb.sgemm_host(ta, tb, m, n, k, p.a, p.lda, p.b, p.ldb, c_host, p.ldc, acc, math_mode=mode)
    assert c_host.tobytes() == want.tobytes()


@pytest.mark.parametrize("mode", [nnb.MATH_FP32X3, nnb.MATH_TF32])
def test_sgemm_host_non_finite_bitwise_equal_to_device(cuda, mode):
    """Infinities and NaNs in A and in the once-packed B reach every band's exact fix-up: the same
    bits as the device entry, and the IEEE pattern of the fp32 loop."""
    torch = cuda
    p = orc.Problem(0, 0, 2000, 4100, 96, 0, 611)
    p.a[1500 * p.lda + 7] = np.inf                    # a row in a later band
    p.b[40 * p.ldb + 4000] = np.nan                   # a column every band reads
    p.b[3 * p.ldb + 17] = -np.inf
    want = run_gpu(torch, p, 0, mode)
    c_host = p.c.copy()
    nnb.sgemm_host(0, 0, p.m, p.n, p.k, p.a, p.lda, p.b, p.ldb, c_host, p.ldc, 0, math_mode=mode)
    assert c_host.tobytes() == want.tobytes()
    loop = orc.sgemm_f32(p, p.c, 0)
    assert np.array_equal(np.isnan(c_host), np.isnan(loop))
    inf = np.isinf(loop)
    assert np.array_equal(c_host[inf], loop[inf])


def test_sgemm_host_release_frees_and_regrows(cuda):
    """nnb_sgemm_host_release frees the kept device buffers; the next call grows them again and gives
    the same bits."""
    torch = cuda
    p = orc.Problem(0, 0, 2048, 2048, 2048, 0, 77)
    c1, c2 = p.c.copy(), p.c.copy()
    nnb.sgemm_host(0, 0, p.m, p.n, p.k, p.a, p.lda, p.b, p.ldb, c1, p.ldc, 0)
    torch.cuda.synchronize()
    free0 = torch.cuda.mem_get_info()[0]
    nnb.sgemm_host_release()
    free1 = torch.cuda.mem_get_info()[0]
    assert free1 - free0 >= 4 * 2048 * 2048 * 4          # at least A, B, C and the packed B
    nnb.sgemm_host(0, 0, p.m, p.n, p.k, p.a, p.lda, p.b, p.ldb, c2, p.ldc, 0)
    assert c1.tobytes() == c2.tobytes()
    assert nnb.device_error() == 0


def test_sgemm_host_pinned_golden(cuda):
    """Pinned torch host tensors, and the reference build's golden case of this module."""
    torch = cuda
    g = np.load(orc.HERE.parent / "tests" / "golden" / "gemm_golden.npz")
    ta, tb, m, n, k, pad, seed, acc = (int(v) for v in g["cases"][1])
    a = torch.from_numpy(g["a1"]).pin_memory()
    b = torch.from_numpy(g["b1"]).pin_memory()
    c = torch.from_numpy(g["c1"].copy()).pin_memory()
    lda = (m if ta else k) + pad
    ldb = (k if tb else n) + pad
    ldc = n + pad
    nnb.sgemm_host(ta, tb, m, n, k, a, lda, b, ldb, c, ldc, acc)
    got = c.numpy().reshape(-1)[: m * ldc].reshape(m, ldc)[:, :n].astype(np.float64)
    ref = g["loop1"].reshape(-1)[: m * ldc].reshape(m, ldc)[:, :n].astype(np.float64)
    assert np.abs(got - ref).max() <= 1e-5 * max(1.0, np.abs(ref).max()) * np.sqrt(k)
