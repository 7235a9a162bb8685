"""The reference's own modules, unchanged, on the B200: the reference library rebuilt with its GEMM
translation unit (src/kernels/gemm.cpp) replaced by the drop-in nn-cpp_b200/host/nn_kernels_gemm.cpp
(oracle/_ref/libnnref_nnb.so, built by oracle/Makefile from the reference's other sources as they
are). Every nn::kernels::sgemm the reference's Transformer, MultiHeadAttention, Linear, Conv2d and
Tensor::matmul issue then runs on the GPU through nnb_sgemm_host.

Each workload runs twice through the reference's code -- all-CPU (oracle/_ref/libnnref.so) and with
the GPU drop-in -- on the same inputs; results agree to the 3xTF32 GEMM's fp32-grade tolerance.
"""
import ctypes
import subprocess

import numpy as np
import pytest

import nnb
from oracle import orc


def _libs():
    cpu, gpu = orc.ref(), orc.ref_nnb()
    if cpu is None or gpu is None:
        pytest.skip("reference libraries not built (oracle/_ref)")
    return cpu, gpu


def _close(got, want, rel):
    got, want = np.asarray(got, np.float64), np.asarray(want, np.float64)
    scale = np.abs(want).max()
    err = np.abs(got - want).max()
    assert err <= rel * scale, f"max err {err:.3e} vs scale {scale:.3e}"


def test_dropin_library_has_no_cpu_gemm():
    """libnnref_nnb.so takes nn::kernels::sgemm from the drop-in (libnnb.so is a dependency) and has
    none of the reference's CPU GEMM driver or microkernel."""
    if not orc.REF_NNB_PATH.exists():
        pytest.skip("reference libraries not built (oracle/_ref)")
    syms = subprocess.run(["nm", "-C", str(orc.REF_NNB_PATH)], capture_output=True, text=True).stdout
    assert "T nn::kernels::sgemm(bool, bool," in syms
    assert "micro_avx2" not in syms and "blocked_flat" not in syms
    needed = subprocess.run(["readelf", "-d", str(orc.REF_NNB_PATH)], capture_output=True, text=True).stdout
    assert "libnnb.so" in needed


@pytest.mark.gpu
@pytest.mark.parametrize("dim,heads", [(128, 2), (64, 4)])
def test_reference_transformer_training_on_dropin(cuda, dim, heads):
    """nn::Transformer + nn::AdamW, three steps: losses, first-step gradients and final parameters of
    the reference's code on the GPU GEMM against the same code on its CPU GEMM."""
    cpu, gpu = _libs()
    V, L, T, N, steps, lr, wd = 64, 2, 16, 4, 3, 1e-2, 1e-2
    ids = orc.integers(97, N * (T + 1), 0, V - 1).reshape(N, T + 1)
    x, y = ids[:, :T].copy(), ids[:, 1:].copy()
    from nnb.nn import Transformer, TransformerConfig
    model = Transformer(TransformerConfig(vocab_size=V, dim=dim, heads=heads, layers=L, max_len=T), seed=3)
    init = np.concatenate([p.data.cpu().numpy().ravel() for p in model.parameters()])
    n_params = init.size
    out = {}
    for name, lib in (("cpu", cpu), ("gpu", gpu)):
        losses = np.zeros(steps, np.float32)
        grads, params = np.zeros_like(init), np.zeros_like(init)
        n = lib.ref_transformer_train(V, dim, heads, L, T, N, T, orc.ptr(init), orc.ptr(x), orc.ptr(y), lr, wd, steps,
                                      orc.ptr(losses), orc.ptr(grads), orc.ptr(params))
        assert n == n_params
        out[name] = (losses, grads, params)
    (l_c, g_c, p_c), (l_g, g_g, p_g) = out["cpu"], out["gpu"]
    np.testing.assert_allclose(l_g, l_c, rtol=1e-5)
    _close(g_g, g_c, 1e-4)
    err = np.abs(p_g.astype(np.float64) - p_c)
    assert err.max() <= 2 * lr * steps
    assert (err <= 1e-5 * np.abs(p_c).max()).mean() > 0.995
    assert nnb.device_error() == 0


def _cnn_params():
    """Kaiming-uniform bounds (1/sqrt(fan_in)) and zero biases; the conv weights are rounded to
    multiples of 2^-8 (see test_reference_cnn_on_dropin)."""
    rng = np.random.default_rng(5)
    out = []
    for i, (shape, fan) in enumerate((((32, 1, 3, 3), 9), ((32,), None), ((64, 32, 3, 3), 288), ((64,), None),
                                      ((128, 3136), 3136), ((128,), None), ((10, 128), 128), ((10,), None))):
        if fan is None:
            out.append(np.zeros(shape, np.float32))
        else:
            bound = 1 / np.sqrt(fan)
            w = rng.uniform(-bound, bound, size=shape).astype(np.float32)
            if i in (0, 2):
                w = (np.round(w * 256) / 256).astype(np.float32)
            out.append(w)
    return np.concatenate([p.ravel() for p in out])


@pytest.mark.gpu
def test_reference_cnn_on_dropin(cuda):
    """Config 2's CNN (conv2d_relu, maxpool, linear, cross entropy) composed from the reference's ops,
    one forward and backward, on the GPU GEMM against the CPU GEMM.

    Both runs must take the same decisions (ReLU signs, maxpool's first maximum) for the gradients to
    compare element by element: a flipped decision routes a gradient elsewhere. The images are
    multiples of 1/8 and the conv weights multiples of 2^-8, so every conv output is exact in fp32 on
    both paths (few-bit products, short exact sums; 3xTF32 splits such operands without loss) and the
    conv ReLU and pooling decisions are identical. fc1 (K = 3136) is not exact; the batch (seed 82)
    keeps every fc1 output at least 2.9e-4 of the largest away from 0 -- over ten times the 3xTF32
    product's error there -- and the test asserts that no fc1 decision differs."""
    cpu, gpu = _libs()
    N = 64
    x = (np.round(orc.uniform(82, N * 784, 0.0, 1.0) * 8) / 8).astype(np.float32).reshape(N, 1, 28, 28)
    labels = orc.integers(1082, N, 0, 9)
    params = _cnn_params()
    res = {}
    for name, lib in (("cpu", cpu), ("gpu", gpu)):
        loss, logits = np.zeros(1, np.float32), np.zeros((N, 10), np.float32)
        grads, fc1 = np.zeros_like(params), np.zeros((N, 128), np.float32)
        lib.ref_cnn_fwd_bwd_ex(N, orc.ptr(x), orc.ptr(labels), orc.ptr(params), orc.ptr(loss), orc.ptr(logits),
                               orc.ptr(grads), orc.ptr(fc1))
        res[name] = (loss, logits, grads, fc1)
    (lc, oc, gc, fc), (lg, og, gg, fg) = res["cpu"], res["gpu"]
    assert int(np.count_nonzero((fc > 0) != (fg > 0))) == 0
    _close(fg, fc, 1e-4)
    _close(og, oc, 1e-4)
    np.testing.assert_allclose(lg, lc, rtol=1e-5)
    off = 0
    for shape in ((32, 1, 3, 3), (32,), (64, 32, 3, 3), (64,), (128, 3136), (128,), (10, 128), (10,)):
        n = int(np.prod(shape))
        _close(gg[off:off + n], gc[off:off + n], 1e-4)
        off += n


@pytest.mark.gpu
def test_reference_matmul_on_dropin(cuda):
    """Config 1: nn::matmul (Tensor::matmul) 512^3, and a batched fold, through the drop-in: within the
    3xTF32 bound of the fp64 product."""
    cpu, gpu = _libs()
    for ash, bsh in (((512, 512), (512, 512)), ((3, 40, 70), (70, 33))):
        a = orc.uniform(100, int(np.prod(ash))).reshape(ash)
        b = orc.uniform(101, int(np.prod(bsh))).reshape(bsh)
        out = np.zeros(ash[:-1] + (bsh[-1],), np.float32)
        A = (ctypes.c_int64 * len(ash))(*ash)
        B = (ctypes.c_int64 * len(bsh))(*bsh)
        assert gpu.ref_matmul_nd(orc.ptr(a), A, len(ash), orc.ptr(b), B, len(bsh), 0, 0, orc.ptr(out)) == 0
        exact = np.matmul(a.astype(np.float64), b.astype(np.float64))
        mag = np.matmul(np.abs(a.astype(np.float64)), np.abs(b.astype(np.float64)))
        assert np.all(np.abs(out - exact) <= 1e-5 * mag + 1e-6)
