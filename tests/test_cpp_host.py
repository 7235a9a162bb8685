"""The seams as C++17 host code. tests/cpp/sgemm_shim.cpp is the nn::kernels::sgemm
(include/nn/kernels/gemm.hpp:57-59) a maintainer of nn-cpp would add, forwarding to the C ABI's
host-buffer entry: it must compile against include/nnb.h alone, link libnnb.so, reject bad arguments
before any device work (CPU test) and give the device entry's bits from host buffers (GPU test).
tests/cpp/linear_shim.cpp runs the `linear` op (ops.hpp:304) forward and backward through the C ABI
on cudaMalloc'd storage: it must build against the CUDA runtime (CPU test) and give the bits the
Python binding gets from the same entries (GPU test).
"""
import pathlib
import shutil
import subprocess

import numpy as np
import pytest

import nnb
from oracle import orc

HERE = pathlib.Path(__file__).resolve().parent
ROOT = HERE.parent


@pytest.fixture(scope="module")
def shim(tmp_path_factory):
    cxx = shutil.which("g++")
    assert cxx is not None, "g++ is needed to build the C++ host shim"
    exe = tmp_path_factory.mktemp("cpp") / "sgemm_shim"
    lib_dir = str(nnb.LIB_PATH.parent)
    cmd = [cxx, "-std=c++17", "-O2", "-Wall", "-Wextra", "-Werror", "-I", str(ROOT / "include"),
           str(HERE / "cpp" / "sgemm_shim.cpp"), str(ROOT / "nn-cpp_b200" / "host" / "nn_kernels_gemm.cpp"),
           "-L", lib_dir, "-lnnb", f"-Wl,-rpath,{lib_dir}", "-o", str(exe)]
    res = subprocess.run(cmd, capture_output=True, text=True)
    assert res.returncode == 0, res.stderr
    return exe


@pytest.fixture(scope="module")
def linear_shim(tmp_path_factory):
    cxx = shutil.which("g++")
    assert cxx is not None, "g++ is needed to build the C++ host shim"
    exe = tmp_path_factory.mktemp("cpp") / "linear_shim"
    lib_dir = str(nnb.LIB_PATH.parent)
    cuda_home = pathlib.Path("/usr/local/cuda")
    cmd = [cxx, "-std=c++17", "-O2", "-Wall", "-Wextra", "-Werror", "-I", str(ROOT / "include"),
           "-I", str(cuda_home / "include"), str(HERE / "cpp" / "linear_shim.cpp"), "-L", lib_dir, "-lnnb",
           "-L", str(cuda_home / "lib64"), "-lcudart", f"-Wl,-rpath,{lib_dir}", f"-Wl,-rpath,{cuda_home / 'lib64'}",
           "-o", str(exe)]
    res = subprocess.run(cmd, capture_output=True, text=True)
    assert res.returncode == 0, res.stderr
    return exe


def test_cpp_linear_shim_builds(linear_shim):
    assert linear_shim.exists()


def test_cpp_shim_builds_and_rejects_bad_arguments(shim):
    out = subprocess.run([str(shim), "checks"], capture_output=True, text=True, timeout=120)
    assert out.returncode == 0, out.stdout + out.stderr
    assert "checks ok" in out.stdout
    assert out.stdout.count("invalid_argument:") == 3
    assert f"version {nnb.lib().nnb_version().decode()}" in out.stdout


@pytest.mark.gpu
@pytest.mark.parametrize("ta,tb,m,n,k,pad,acc", [
    (0, 0, 257, 300, 129, 0, 0),
    (1, 1, 1000, 4100, 96, 3, 1),        # several bands over one packed B, strided, accumulate
    (0, 1, 33, 7, 2100, 1, 0),           # deep k: the depth cut inside the band
])
def test_cpp_shim_product_equals_device_entry(cuda, shim, tmp_path, ta, tb, m, n, k, pad, acc):
    torch = cuda
    p = orc.Problem(ta, tb, m, n, k, pad, 8100 + m)
    (tmp_path / "in.bin").write_bytes(p.a.tobytes() + p.b.tobytes() + p.c.tobytes())
    args = [str(v) for v in (ta, tb, m, n, k, p.lda, p.ldb, p.ldc, acc)]
    out = subprocess.run([str(shim), "run", *args, str(tmp_path / "in.bin"), str(tmp_path / "out.bin")],
                         capture_output=True, text=True, timeout=300)
    assert out.returncode == 0, out.stdout + out.stderr
    got = np.fromfile(tmp_path / "out.bin", np.float32)
    # the device entry on device copies of the same operands
    da, db = torch.from_numpy(p.a).cuda(), torch.from_numpy(p.b).cuda()
    dc = torch.from_numpy(p.c.copy()).cuda()
    nnb.sgemm(ta, tb, m, n, k, da, p.lda, db, p.ldb, dc, p.ldc, acc)
    assert got.tobytes() == dc.cpu().numpy().tobytes()
    # and the reference test's bound against fp64 (tests/test_kernels.cpp), padding untouched
    full = got[: m * p.ldc].reshape(m, p.ldc)
    assert np.all(full[:, n:] == orc.SENTINEL)
    want = orc.sgemm_f64(p, p.c, acc)
    mag = orc.magnitude(p, p.c, acc)
    assert np.all(np.abs(full[:, :n].astype(np.float64) - want) <= np.maximum(1e-5 * mag, 1e-6))


@pytest.mark.gpu
@pytest.mark.parametrize("M,K,n", [(300, 129, 70), (4096, 512, 1536)])
def test_cpp_linear_shim_equals_python_binding(cuda, linear_shim, tmp_path, M, K, n):
    """linear forward + backward from C++ on device storage: the same bits as the Python binding's
    calls of the same entries, and within the fp32 bound of an fp64 evaluation."""
    torch = cuda
    x, w = orc.normal(901, M * K), orc.normal(902, n * K)
    b, g = orc.normal(903, n), orc.normal(904, M * n)
    (tmp_path / "in.bin").write_bytes(x.tobytes() + w.tobytes() + b.tobytes() + g.tobytes())
    out = subprocess.run([str(linear_shim), str(M), str(K), str(n), str(tmp_path / "in.bin"),
                          str(tmp_path / "out.bin")], capture_output=True, text=True, timeout=300)
    assert out.returncode == 0, out.stdout + out.stderr
    got = np.fromfile(tmp_path / "out.bin", np.float32)
    sizes = [M * n, M * K, n * K, n]
    parts = np.split(got, np.cumsum(sizes)[:-1])
    # the Python binding on the same operands
    L = nnb.lib()
    s = torch.cuda.current_stream().cuda_stream
    xd, wd, bd, gd = (torch.from_numpy(v).cuda() for v in (x, w, b, g))
    y, dx = torch.empty(M * n, device="cuda"), torch.empty(M * K, device="cuda")
    dw, db = torch.empty(n * K, device="cuda"), torch.empty(n, device="cuda")
    nnb.check(L.nnb_linear_fwd(s, M, K, n, xd.data_ptr(), wd.data_ptr(), bd.data_ptr(), y.data_ptr()))
    nnb.check(L.nnb_linear_bwd(s, M, K, n, gd.data_ptr(), xd.data_ptr(), wd.data_ptr(), dx.data_ptr(), 1,
                               dw.data_ptr(), 1, db.data_ptr(), 1))
    for mine, ref in zip(parts, (y, dx, dw, db)):
        assert mine.tobytes() == ref.cpu().numpy().tobytes()
    # fp64 evaluation: y = x w^T + b, dx = g w, dw = g^T x, db = column sums of g
    X, W, G = (v.astype(np.float64) for v in (x.reshape(M, K), w.reshape(n, K), g.reshape(M, n)))
    for mine, want, mag in ((parts[0], X @ W.T + b, np.abs(X) @ np.abs(W).T + np.abs(b)),
                            (parts[1], G @ W, np.abs(G) @ np.abs(W)),
                            (parts[2], G.T @ X, np.abs(G).T @ np.abs(X)),
                            (parts[3], G.sum(0), np.abs(G).sum(0))):
        assert np.all(np.abs(mine.reshape(want.shape) - want) <= 1e-5 * mag + 1e-6)
