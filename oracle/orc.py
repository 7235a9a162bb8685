"""ctypes loader for the CPU checkers. TEST INFRASTRUCTURE ONLY.

Only tests/, ``__graft_entry__.smoke()`` and bench.py's cpu_baseline / reference legs import this
module. It exposes:

- :data:`orc` -- ``liborc.so``, this directory's restatement of the reference algorithms
  (orc_gemm.c, orc_ops.c, orc_gen.cpp);
- :func:`ref` -- ``_ref/libnnref.so``, the reference library compiled from its own sources
  (``None`` when it was not built), through ref_shim.cpp's C-ABI.

Helpers return numpy arrays; the problem builders mirror tests/test_kernels.cpp:68-86 of the
reference.
"""
from __future__ import annotations

import ctypes
import pathlib

import numpy as np

HERE = pathlib.Path(__file__).resolve().parent
ORC_PATH = HERE / "liborc.so"
REF_PATH = HERE / "_ref" / "libnnref.so"
SENTINEL = np.float32(1e30)

_c = ctypes
_sz, _p, _i, _u32, _f, _d = _c.c_size_t, _c.c_void_p, _c.c_int, _c.c_uint32, _c.c_float, _c.c_double

_ORC_SIGS = {
    "orc_sgemm_f32": [_i, _i, _sz, _sz, _sz, _p, _sz, _p, _sz, _p, _sz, _i],
    "orc_sgemm_f64": [_i, _i, _sz, _sz, _sz, _p, _sz, _p, _sz, _p, _sz, _i, _p],
    "orc_magnitude": [_i, _i, _sz, _sz, _sz, _p, _sz, _p, _sz, _p, _sz, _i, _p],
    "orc_sgemm_f64_sample": [_i, _i, _sz, _p, _sz, _p, _sz, _p, _sz, _i, _p, _p, _sz, _p, _p],
    "orc_fill_uniform": [_u32, _sz, _f, _f, _p],
    "orc_fill_normal": [_u32, _sz, _f, _f, _p],
    "orc_fill_int": [_u32, _sz, _c.c_int64, _c.c_int64, _p],
    "orc_make_problem": [_i, _i, _sz, _sz, _sz, _sz, _u32, _p, _p, _p],
    "orc_gelu_fwd": [_sz, _p, _p, _p],
    "orc_gelu_bwd": [_sz, _p, _p, _p, _p, _i],
    "orc_relu_fwd": [_sz, _p, _p],
    "orc_relu_bwd": [_sz, _p, _p, _p, _i],
    "orc_colsum": [_sz, _sz, _p, _p, _i],
    "orc_linear_fwd": [_sz, _sz, _sz, _p, _p, _p, _p],
    "orc_linear_bwd": [_sz, _sz, _sz, _p, _p, _p, _p, _i, _p, _i, _p, _i],
    "orc_layernorm_fwd": [_sz, _sz, _p, _p, _p, _f, _p, _p, _p],
    "orc_layernorm_bwd": [_sz, _sz, _p, _p, _p, _p, _p, _p, _i, _p, _i, _p, _i],
    "orc_batchnorm_fwd": [_sz, _sz, _sz, _p, _p, _p, _f, _i, _p, _p, _p, _p, _p],
    "orc_batchnorm_bwd": [_sz, _sz, _sz, _p, _p, _p, _p, _p, _p, _p, _i, _p, _i, _p, _i],
    "orc_attention_fwd": [_sz, _sz, _sz, _sz, _sz, _p, _p, _p, _p, _i, _p, _p],
    "orc_attention_bwd": [_sz, _sz, _sz, _sz, _sz, _p, _p, _p, _p, _p, _p, _i, _p, _i, _p, _i, _p, _i],
    "orc_conv2d_fwd": [_sz, _sz, _sz, _sz, _sz, _sz, _sz, _sz, _sz, _p, _p, _p, _i, _p, _p],
    "orc_conv2d_bwd": [_sz, _sz, _sz, _sz, _sz, _sz, _sz, _sz, _sz, _p, _p, _p, _p, _p, _i, _p, _i, _p, _i],
    "orc_maxpool2d_fwd": [_sz, _sz, _sz, _sz, _sz, _sz, _p, _p, _p],
    "orc_maxpool2d_bwd": [_sz, _sz, _sz, _sz, _sz, _sz, _p, _p, _p, _i],
    "orc_conv2d_ex_fwd": [_sz] * 11 + [_p, _p, _p, _p],
    "orc_conv2d_ex_bwd": [_sz] * 11 + [_p, _p, _p, _p, _p, _p],
    "orc_bn_running_update": [_sz, _sz, _f, _p, _p, _p, _p],
    "orc_batchnorm_eval_fwd": [_sz, _sz, _sz, _p, _p, _p, _p, _p, _f, _i, _p],
    "orc_batchnorm_eval_bwd": [_sz, _sz, _sz, _sz, _p, _p, _p, _p, _p, _p, _f, _i, _p, _p, _p],
    "orc_avgpool2d_fwd": [_sz, _sz, _sz, _sz, _sz, _sz, _p, _p],
    "orc_avgpool2d_bwd": [_sz, _sz, _sz, _sz, _sz, _sz, _p, _p, _i],
    "orc_reduce_axis_fwd": [_sz, _sz, _sz, _i, _p, _p],
    "orc_reduce_axis_bwd": [_sz, _sz, _sz, _i, _p, _p, _i],
    "orc_cross_entropy_fwd": [_sz, _sz, _p, _p, _p, _p],
    "orc_cross_entropy_bwd": [_sz, _sz, _p, _p, _f, _p, _i],
    "orc_sequence_ce_fwd": [_sz, _sz, _p, _p, _c.c_int64, _f, _p, _p],
    "orc_sequence_ce_bwd": [_sz, _sz, _p, _p, _c.c_int64, _f, _f, _sz, _p, _i],
    "orc_embedding_fwd": [_sz, _p, _p, _sz, _p],
    "orc_embedding_bwd": [_sz, _p, _sz, _p, _p],
    "orc_adamw_step": [_sz, _p, _p, _p, _p, _f, _f, _f, _f, _f, _c.c_longlong],
}

_REF_SIGS = {
    "ref_sgemm": ([_i, _i, _sz, _sz, _sz, _p, _sz, _p, _sz, _p, _sz, _i], None),
    "ref_sgemm_portable": ([_i, _i, _sz, _sz, _sz, _p, _sz, _p, _sz, _p, _sz, _i], None),
    "ref_reference_sgemm": ([_i, _i, _sz, _sz, _sz, _p, _sz, _p, _sz, _p, _sz, _i], None),
    "ref_sgemm_uses_avx2": ([], _i),
    "ref_num_threads": ([], _sz),
    "ref_set_threads": ([_sz], None),
    "ref_matmul": ([_sz, _sz, _sz, _sz, _p, _p, _p], None),
    "ref_time_matmul": ([_sz, _sz, _sz, _p, _p, _i], _d),
    "ref_time_sgemm": ([_sz, _sz, _sz, _p, _p, _p, _i], _d),
    "ref_matmul_nd": ([_p, _p, _i, _p, _p, _i, _i, _i, _p], _i),
    "ref_matmul_value": ([_p, _p, _i, _p, _p, _i, _i, _i, _p, _p, _p, _p], _i),
    "ref_scaled_masked_softmax": ([_sz, _sz, _sz, _sz, _p, _f, _p, _i, _p, _p, _p], None),
    "ref_transformer_train": ([_sz, _sz, _sz, _sz, _sz, _sz, _sz, _p, _p, _p, _f, _f, _i, _p, _p, _p],
                              _c.c_longlong),
    "ref_transformer_train_ex": ([_c.c_uint64, _f, _sz, _sz, _sz, _sz, _sz, _sz, _sz, _p, _p, _p, _f, _f, _i, _p, _p,
                                  _p], _c.c_longlong),
    "ref_cnn_fwd_bwd": ([_sz, _p, _p, _p, _p, _p, _p], None),
    "ref_cnn_fwd_bwd_ex": ([_sz, _p, _p, _p, _p, _p, _p, _p], None),
    "ref_linear": ([_sz, _sz, _sz, _p, _p, _p, _p, _p, _p, _p, _p], None),
    "ref_layernorm": ([_sz, _sz, _p, _p, _p, _f, _p, _p, _p, _p, _p], None),
    "ref_batchnorm": ([_sz, _sz, _sz, _p, _p, _p, _f, _i, _p, _p, _p, _p, _p, _p, _p], None),
    "ref_attention": ([_sz, _sz, _sz, _sz, _sz, _p, _p, _p, _p, _i, _p, _p, _p, _p, _p], None),
    "ref_conv2d": ([_sz, _sz, _sz, _sz, _sz, _sz, _sz, _i, _i, _p, _p, _p, _i, _p, _p, _p, _p, _p], None),
    "ref_maxpool2d": ([_sz, _sz, _sz, _sz, _sz, _sz, _p, _p, _p, _p], None),
    "ref_conv2d_ex": ([_sz, _sz, _sz, _sz, _sz, _sz, _sz, _i, _i, _i, _i, _p, _p, _p, _p, _p, _p, _p, _p], None),
    "ref_avgpool2d": ([_sz, _sz, _sz, _sz, _sz, _sz, _p, _p, _p, _p], None),
    "ref_reduce4": ([_sz, _sz, _sz, _sz, _i, _i, _p, _p, _p, _p], None),
    "ref_global_avgpool": ([_sz, _sz, _sz, _sz, _p, _p, _p, _p], None),
    "ref_bn2d_module": ([_sz, _sz, _sz, _sz, _i, _i, _i, _p, _p, _p, _p, _p, _p, _p, _p], None),
    "ref_bn2d_module_ex": ([_sz, _sz, _sz, _sz, _i, _i, _i, _p, _p, _p, _p, _p, _p, _p, _p, _p, _p], None),
    "ref_loader_orders": ([_c.c_uint64, _i, _sz, _sz, _i, _i, _i, _p], _sz),
    "ref_loader_weighted": ([_c.c_uint64, _p, _sz, _sz, _sz, _i, _i, _p], _c.c_longlong),
    "ref_random_split": ([_sz, _p, _i, _c.c_uint64, _p, _p], _i),
    "ref_balanced_weights": ([_p, _sz, _sz, _p], _i),
    "ref_mt19937_outputs": ([_p, _sz, _sz, _p], None),
    "ref_time_loader": ([_sz, _sz, _sz, _sz], _d),
    "ref_time_checkpoint": ([_c.c_char_p, _sz, _sz], _d),
    "ref_derive_outputs": ([_c.c_uint64, _c.c_char_p, _i, _sz, _p], None),
    "ref_dropout_masks": ([_c.c_uint64, _i, _f, _p, _i, _p], None),
    "ref_attention_dropout": ([_c.c_uint64, _sz, _sz, _sz, _sz, _i, _f, _p, _p, _p, _p, _p, _p, _p, _p], None),
    "ref_mha_dropout": ([_c.c_uint64, _sz, _sz, _sz, _sz, _i, _f, _i, _p, _p, _p, _p, _p, _p], None),
    "ref_linear_checkpoint_save": ([_c.c_char_p, _p, _p, _p, _p, _f, _f, _c.c_longlong], _i),
    "ref_linear_checkpoint_load": ([_c.c_char_p, _p, _p], _c.c_longlong),
    "ref_gelu": ([_sz, _p, _p, _p, _p], None),
    "ref_relu": ([_sz, _p, _p, _p, _p], None),
    "ref_tanh_inplace": ([_p, _sz], None),
    "ref_cross_entropy": ([_sz, _sz, _p, _p, _f, _p, _p], None),
    "ref_sequence_ce": ([_sz, _sz, _sz, _p, _p, _i, _f, _f, _p, _p], None),
    "ref_embedding": ([_sz, _sz, _p, _p, _sz, _p, _p, _p], None),
    "ref_adamw": ([_sz, _p, _p, _f, _f, _f, _f, _f, _i], None),
}


def _load(path, sigs):
    L = ctypes.CDLL(str(path))
    for name, spec in sigs.items():
        fn = getattr(L, name, None)
        if fn is None:
            continue
        if isinstance(spec, tuple):
            fn.argtypes, fn.restype = spec
        else:
            fn.argtypes, fn.restype = spec, None
    return L


orc = _load(ORC_PATH, _ORC_SIGS)
orc.orc_tanh_one.argtypes, orc.orc_tanh_one.restype = [_f], _f
orc.orc_exp_one.argtypes, orc.orc_exp_one.restype = [_f], _f
_ref = None


def ref():
    """The reference library built from its sources, or None if oracle/_ref was not built."""
    global _ref
    if _ref is None and REF_PATH.exists():
        _ref = _load(REF_PATH, _REF_SIGS)
    return _ref


REF_NNB_PATH = HERE / "_ref" / "libnnref_nnb.so"
_ref_nnb = None


def ref_nnb():
    """The reference library with its GEMM translation unit (src/kernels/gemm.cpp) replaced by the
    B200 drop-in (nn-cpp_b200/host/nn_kernels_gemm.cpp over libnnb.so): the reference's own modules
    and ops, unchanged, with every sgemm on the GPU. None if it was not built."""
    global _ref_nnb
    if _ref_nnb is None and REF_NNB_PATH.exists():
        _ref_nnb = _load(REF_NNB_PATH, _REF_SIGS)
    return _ref_nnb


def ptr(a) -> int | None:
    """Address of a numpy array's data (None passes through as a NULL pointer)."""
    return None if a is None else a.ctypes.data


def zeros(*shape, dtype=np.float32):
    return np.zeros(shape, dtype)


# ---- generators -------------------------------------------------------------------------------

def uniform(seed: int, n: int, lo: float = -1.0, hi: float = 1.0) -> np.ndarray:
    out = np.empty(n, np.float32)
    orc.orc_fill_uniform(seed, n, lo, hi, ptr(out))
    return out


def normal(seed: int, n: int, mean: float = 0.0, std: float = 1.0) -> np.ndarray:
    out = np.empty(n, np.float32)
    orc.orc_fill_normal(seed, n, mean, std, ptr(out))
    return out


def integers(seed: int, n: int, lo: int, hi: int) -> np.ndarray:
    out = np.empty(n, np.int64)
    orc.orc_fill_int(seed, n, lo, hi, ptr(out))
    return out


class Problem:
    """One GEMM problem laid out like test_kernels.cpp:68-86 (padding = 1e30f)."""

    def __init__(self, ta, tb, m, n, k, pad, seed):
        self.ta, self.tb, self.m, self.n, self.k = bool(ta), bool(tb), m, n, k
        a_rows, a_cols = (k, m) if ta else (m, k)
        b_rows, b_cols = (n, k) if tb else (k, n)
        self.lda, self.ldb, self.ldc = a_cols + pad, b_cols + pad, n + pad
        self.a = np.empty(max(a_rows * self.lda, 1), np.float32)
        self.b = np.empty(max(b_rows * self.ldb, 1), np.float32)
        self.c = np.empty(max(m * self.ldc, 1), np.float32)
        orc.orc_make_problem(int(ta), int(tb), m, n, k, pad, seed, ptr(self.a), ptr(self.b), ptr(self.c))

    def args(self):
        return (int(self.ta), int(self.tb), self.m, self.n, self.k, ptr(self.a), self.lda, ptr(self.b), self.ldb)


# ---- GEMM oracles -----------------------------------------------------------------------------

def sgemm_f32(p: Problem, c: np.ndarray, accumulate: bool) -> np.ndarray:
    """tests/reference_gemm.hpp's fp32 loop (restated in orc_gemm.c) on a copy of c."""
    out = c.copy()
    orc.orc_sgemm_f32(*p.args(), ptr(out), p.ldc, int(accumulate))
    return out


def sgemm_f64(p: Problem, c: np.ndarray, accumulate: bool) -> np.ndarray:
    """fp64 evaluation, m x n."""
    out = np.empty(max(p.m * p.n, 1), np.float64)
    orc.orc_sgemm_f64(*p.args(), ptr(c), p.ldc, int(accumulate), ptr(out))
    return out[: p.m * p.n].reshape(p.m, p.n)


def magnitude(p: Problem, c: np.ndarray, accumulate: bool) -> np.ndarray:
    """test_kernels.cpp:101-109 in fp64, m x n."""
    out = np.empty(max(p.m * p.n, 1), np.float64)
    orc.orc_magnitude(*p.args(), ptr(c), p.ldc, int(accumulate), ptr(out))
    return out[: p.m * p.n].reshape(p.m, p.n)


def sgemm_f64_sample(ta, tb, k, a, lda, b, ldb, c, ldc, accumulate, rows, cols):
    rows = np.ascontiguousarray(rows, np.int64)
    cols = np.ascontiguousarray(cols, np.int64)
    val = np.empty(len(rows), np.float64)
    mag = np.empty(len(rows), np.float64)
    orc.orc_sgemm_f64_sample(int(ta), int(tb), k, ptr(a), lda, ptr(b), ldb, ptr(c) if c is not None else None,
                             ldc, int(accumulate), ptr(rows), ptr(cols), len(rows), ptr(val), ptr(mag))
    return val, mag


# ---- random streams and dropout (src/random.cpp, src/nn/dropout.cpp) -----------------------------

def mt_outputs(state: np.ndarray, n: int):
    """n outputs of the mt19937 whose state is key = state[:624], next index = state[624] (numpy's
    MT19937 bit generator, the published algorithm); returns (outputs uint32[n], new state)."""
    bg = np.random.MT19937()
    bg.state = {"bit_generator": "MT19937", "state": {"key": np.asarray(state[:624], np.uint32), "pos": int(state[624])}}
    out = bg.random_raw(n).astype(np.uint32) if n else np.zeros(0, np.uint32)
    st = bg.state["state"]
    return out, np.concatenate([np.asarray(st["key"], np.uint32), np.array([st["pos"]], np.uint32)])


def dropout_draws(state: np.ndarray, n: int, p: float):
    """Dropout::forward's mask values (src/nn/dropout.cpp:20-31) from an mt19937 state: u = float(x >> 8)
    * 2^-24, 0 when u < p else 1 / (1 - p) in float32; p == 0 or 1 draw nothing. Returns (mask
    float32[n], new state)."""
    p = np.float32(p)
    if p == 0:
        return np.ones(n, np.float32), np.array(state, np.uint32)
    if p == 1:
        return np.zeros(n, np.float32), np.array(state, np.uint32)
    x, new = mt_outputs(state, n)
    u = (x >> 8).astype(np.float32) * np.float32(1.0 / 16777216.0)
    keep = np.float32(1.0) / (np.float32(1.0) - p)
    return np.where(u < p, np.float32(0.0), keep).astype(np.float32), new
