"""nnb_sgemm_noalloc: the GEMM for callers that cannot allocate device memory.

Some hosts of this library cannot call the CUDA allocator on the call path (their own arena
already owns the GPU's memory, or a latency-critical loop must not meet cudaMalloc's device-wide
synchronisation or a pool growth). This entry point keeps the GEMM's scratch in a fixed 32 MiB
device array instead. These tests call it through the C ABI and check, on two calls in a row, that
it gives the allocating entry point's (nnb_sgemm_ex's) bits -- neither shape is cut along its depth
and the tile width does not change an element's arithmetic -- and that both are within the GEMM
tests' fp64-oracle bound; and that the entry point's own error word reads 0 after clean calls.

This file is named to be collected last, so a run that stops at the first failure has run every
other test before it; it also passes alone in a fresh process.
"""
import numpy as np
import pytest

import nnb
from oracle import orc

pytestmark = pytest.mark.gpu

TOL = {nnb.MATH_FP32X3: 1e-5, nnb.MATH_TF32: 5e-3}


def _call_noalloc(torch, p, acc, mode, c_host):
    da = torch.from_numpy(p.a).cuda()
    db = torch.from_numpy(p.b).cuda()
    dc = torch.from_numpy(c_host.copy()).cuda()
    stream = torch.cuda.current_stream().cuda_stream
    st = nnb.lib().nnb_sgemm_noalloc(stream, int(p.ta), int(p.tb), p.m, p.n, p.k, da.data_ptr(), p.lda,
                                     db.data_ptr(), p.ldb, dc.data_ptr(), p.ldc, int(acc), mode)
    assert st == nnb.NNB_OK, nnb.last_error()
    torch.cuda.synchronize()
    return dc.cpu().numpy()


def _call_allocating(torch, p, acc, mode, c_host):
    da = torch.from_numpy(p.a).cuda()
    db = torch.from_numpy(p.b).cuda()
    dc = torch.from_numpy(c_host.copy()).cuda()
    nnb.sgemm(p.ta, p.tb, p.m, p.n, p.k, da, p.lda, db, p.ldb, dc, p.ldc, acc, math_mode=mode)
    torch.cuda.synchronize()
    return dc.cpu().numpy()


def _assert_matches(p, got, want, acc, mode):
    """got (no-alloc) has want's (allocating entry's) bits, and both are within the fp64 bound."""
    g = got[: p.m * p.ldc].reshape(p.m, p.ldc)
    w = want[: p.m * p.ldc].reshape(p.m, p.ldc)
    assert np.all(g[:, p.n:] == orc.SENTINEL)           # padding untouched
    assert g.tobytes() == w.tobytes()
    g = g[:, : p.n].astype(np.float64)
    exact = orc.sgemm_f64(p, p.c, acc)
    assert np.array_equal(np.isnan(g), np.isnan(exact))
    inf = np.isinf(g) | np.isinf(exact)
    assert np.array_equal(g[inf], exact[inf])
    fin = ~(np.isnan(exact) | inf)
    mag = orc.magnitude(p, p.c, acc)
    assert np.all(np.abs(g[fin] - exact[fin]) <= np.maximum(TOL[mode] * mag[fin], 1e-6))


def _error_word(torch, clear=1):
    import ctypes
    word = ctypes.c_int(-1)
    st = nnb.lib().nnb_sgemm_noalloc_error(torch.cuda.current_stream().cuda_stream, ctypes.byref(word), clear)
    assert st == nnb.NNB_OK, nnb.last_error()
    return word.value


@pytest.mark.parametrize("mode", [nnb.MATH_FP32X3, nnb.MATH_TF32])
def test_noalloc_matches_allocating_entry_on_two_calls_in_a_row(cuda, mode):
    torch = cuda
    # First call: a problem with an Inf and a NaN, which sets the non-finite flags in the shared array
    p1 = orc.Problem(1, 0, 300, 257, 129, 2, 9001)
    p1.a[5] = np.inf
    p1.b[7 * p1.ldb + 3] = np.nan
    got1 = _call_noalloc(torch, p1, True, mode, p1.c)
    want1 = _call_allocating(torch, p1, True, mode, p1.c)
    _assert_matches(p1, got1, want1, True, mode)
    # Second call, straight after: finite data of another shape; stale flags or panels from the
    # first call must not leak into it
    p2 = orc.Problem(0, 1, 190, 333, 200, 1, 9002)
    got2 = _call_noalloc(torch, p2, False, mode, p2.c)
    want2 = _call_allocating(torch, p2, False, mode, p2.c)
    _assert_matches(p2, got2, want2, False, mode)
    assert np.all(np.isfinite(got2[: p2.m * p2.ldc].reshape(p2.m, p2.ldc)[:, : p2.n]))
    assert _error_word(torch) == 0


def test_noalloc_rejects_sizes_beyond_its_buffer(cuda):
    torch = cuda
    n = 4096                                  # (4096 + 4096) * 4096 * 2 * 4 bytes = 256 MiB > 32 MiB
    a = torch.zeros(n * n, device="cuda")
    c = torch.full((n * n,), 7.0, device="cuda")
    stream = torch.cuda.current_stream().cuda_stream
    st = nnb.lib().nnb_sgemm_noalloc(stream, 0, 0, n, n, n, a.data_ptr(), n, a.data_ptr(), n, c.data_ptr(), n, 0,
                                     nnb.MATH_FP32X3)
    assert st == nnb.NNB_ERR_UNSUPPORTED
    assert "static buffer" in nnb.last_error()
    torch.cuda.synchronize()
    assert bool((c == 7.0).all())             # nothing was enqueued
