"""Python binding of the B200 C ABI (include/nnb.h), loaded with ctypes.

The library is the in-tree ``libnnb.so`` built by :mod:`nnb._build`. There is no fallback: if the
library is missing, or the process has no sm_100 GPU, every call raises. Device buffers are
``torch`` CUDA tensors (torch is used for allocation and streams only); every compute call goes
through one ``nnb_*`` entry point of the C ABI.

Errors follow the reference's conventions: a shape mismatch raises :class:`TensorShapeError`
(nn::TensorShapeError, include/nn/tensor.hpp:70), a bad argument raises ``ValueError``
(std::invalid_argument), and CUDA or device failures raise :class:`NnbError`.
"""
from __future__ import annotations

import ctypes
import pathlib
import re

_PKG = pathlib.Path(__file__).resolve().parent
LIB_PATH = _PKG / "libnnb.so"
HEADER = _PKG.parent.parent / "include" / "nnb.h"

NNB_OK, NNB_ERR_INVALID, NNB_ERR_CUDA, NNB_ERR_UNSUPPORTED, NNB_ERR_DEVICE, NNB_ERR_SHAPE = range(6)
MATH_FP32X3, MATH_TF32 = 0, 1


class NnbError(RuntimeError):
    """A CUDA, device or support failure reported by the library."""


class TensorShapeError(ValueError):
    """Shapes of the operands do not agree (the reference's nn::TensorShapeError)."""


class TensorIndexError(IndexError):
    """An index outside a tensor or dataset (the reference's nn::TensorIndexError)."""


_lib = None

_c = ctypes
_sz = _c.c_size_t
_p = _c.c_void_p
_i = _c.c_int
_f = _c.c_float

# argument types of every entry point, in header order
_SIGS = {
    "nnb_version": ([], _c.c_char_p),
    "nnb_last_error": ([], _c.c_char_p),
    "nnb_set_math_mode": ([_i], _i),
    "nnb_get_math_mode": ([], _i),
    "nnb_device_error": ([_p], _i),
    "nnb_ipc_export": ([_p, _p, _c.POINTER(_sz)], _i),
    "nnb_ipc_open": ([_p, _sz, _c.POINTER(_p)], _i),
    "nnb_ipc_close": ([_p, _sz], _i),
    "nnb_copy_async": ([_p, _p, _p, _sz], _i),
    "nnb_trace_enable": ([_i], None),
    "nnb_trace_reset": ([], None),
    "nnb_trace_query": ([_i, _c.POINTER(_c.c_double), _c.POINTER(_c.c_longlong)], _i),
    "nnb_launch_count": ([], _c.c_longlong),
    "nnb_sgemm": ([_p, _i, _i, _sz, _sz, _sz, _p, _sz, _p, _sz, _p, _sz, _i], _i),
    "nnb_sgemm_ex": ([_p, _i, _i, _sz, _sz, _sz, _p, _sz, _p, _sz, _p, _sz, _i, _i], _i),
    "nnb_sgemm_host": ([_i, _i, _sz, _sz, _sz, _p, _sz, _p, _sz, _p, _sz, _i], _i),
    "nnb_sgemm_host_async": ([_p, _i, _i, _sz, _sz, _sz, _p, _sz, _p, _sz, _p, _sz, _i, _i], _i),
    "nnb_sgemm_host_release": ([], _i),
    "nnb_sgemm_strided_batched": ([_p, _i, _i, _sz, _sz, _sz, _p, _sz, _sz, _p, _sz, _sz, _p, _sz, _sz,
                                   _sz, _i, _i], _i),
    "nnb_sgemm_noalloc": ([_p, _i, _i, _sz, _sz, _sz, _p, _sz, _p, _sz, _p, _sz, _i, _i], _i),
    "nnb_sgemm_noalloc_error": ([_p, _p, _i], _i),
    "nnb_matmul": ([_p, _p, _p, _i, _p, _p, _i, _i, _i, _p, _p, _p], _i),
    "nnb_linear_fwd": ([_p, _sz, _sz, _sz, _p, _p, _p, _p], _i),
    "nnb_linear_gelu_fwd": ([_p, _sz, _sz, _sz, _p, _p, _p, _p, _p], _i),
    "nnb_linear_bwd": ([_p, _sz, _sz, _sz, _p, _p, _p, _p, _i, _p, _i, _p, _i], _i),
    "nnb_column_sum": ([_p, _sz, _sz, _p, _p, _i], _i),
    "nnb_layernorm_fwd": ([_p, _sz, _sz, _p, _p, _p, _f, _p, _p, _p], _i),
    "nnb_layernorm_bwd": ([_p, _sz, _sz, _p, _p, _p, _p, _p, _p, _i, _p, _i, _p, _i], _i),
    "nnb_batchnorm_fwd": ([_p, _sz, _sz, _sz, _p, _p, _p, _f, _i, _p, _p, _p, _p, _p], _i),
    "nnb_batchnorm_bwd": ([_p, _sz, _sz, _sz, _p, _p, _p, _p, _p, _p, _p, _i, _p, _i, _p, _i], _i),
    "nnb_attention_fwd": ([_p, _sz, _sz, _sz, _sz, _sz, _p, _p, _p, _p, _i, _p, _p], _i),
    "nnb_attention_bwd": ([_p, _sz, _sz, _sz, _sz, _sz, _p, _p, _p, _p, _p, _p, _i, _p, _i, _p, _i, _p, _i], _i),
    "nnb_flash_attention_supported": ([_sz, _sz], _i),
    "nnb_flash_attention_fwd": ([_p, _sz, _sz, _sz, _sz, _sz, _p, _p, _p, _p, _i, _p, _p], _i),
    "nnb_flash_attention_bwd": ([_p, _sz, _sz, _sz, _sz, _sz, _p, _p, _p, _p, _p, _p, _p, _i, _p, _i, _p, _i, _p, _i],
                                _i),
    "nnb_attention_dropout_fwd": ([_p, _sz, _sz, _sz, _sz, _sz, _p, _p, _p, _p, _i, _f, _p, _p, _p, _p], _i),
    "nnb_attention_dropout_bwd": ([_p, _sz, _sz, _sz, _sz, _sz, _p, _p, _p, _p, _p, _p, _f, _p, _p, _i, _p, _i, _p, _i,
                                   _p, _i], _i),
    "nnb_masked_softmax_fwd": ([_p, _sz, _sz, _sz, _sz, _p, _p, _i, _f], _i),
    "nnb_masked_softmax_bwd": ([_p, _sz, _sz, _sz, _sz, _p, _p, _p, _i, _f], _i),
    "nnb_scaled_masked_softmax_fwd": ([_p, _sz, _sz, _sz, _sz, _p, _p, _p, _i, _f], _i),
    "nnb_scaled_masked_softmax_bwd": ([_p, _sz, _sz, _sz, _sz, _p, _p, _p, _i, _p, _i, _f], _i),
    "nnb_conv2d_fwd": ([_p, _sz, _sz, _sz, _sz, _sz, _sz, _sz, _i, _i, _p, _p, _p, _i, _p, _p], _i),
    "nnb_conv2d_bwd": ([_p, _sz, _sz, _sz, _sz, _sz, _sz, _sz, _i, _i, _p, _p, _p, _p, _p, _i, _p, _i, _p, _i], _i),
    "nnb_relu_fwd": ([_p, _sz, _p, _p], _i),
    "nnb_relu_bwd": ([_p, _sz, _p, _p, _p, _i], _i),
    "nnb_gelu_fwd": ([_p, _sz, _p, _p, _p], _i),
    "nnb_gelu_bwd": ([_p, _sz, _p, _p, _p, _p, _i], _i),
    "nnb_fill": ([_p, _sz, _f, _p], _i),
    "nnb_scale": ([_p, _sz, _f, _p, _p], _i),
    "nnb_linear_multi_fwd": ([_p, _sz, _sz, _sz, _sz, _p, _p, _sz, _p, _sz, _p, _sz], _i),
    "nnb_linear_pack_bytes": ([_sz, _sz, _i], _sz),
    "nnb_linear_fwd_ex": ([_p, _sz, _sz, _sz, _sz, _p, _p, _sz, _p, _sz, _p, _sz, _p, _p], _i),
    "nnb_linear_bwd_ex": ([_p, _sz, _sz, _sz, _sz, _p, _p, _p, _i, _p, _p, _i, _p, _sz, _i, _p, _sz, _i], _i),
    "nnb_linear_bwd_grouped": ([_p, _sz, _sz, _sz, _sz, _p, _p, _p, _p, _i, _p, _sz, _i, _p, _sz, _i], _i),
    "nnb_layernorm_bwd_grouped": ([_p, _sz, _sz, _sz, _p, _p, _p, _p, _p, _p, _i, _p, _sz, _i, _p, _sz, _i], _i),
    "nnb_embedding_bwd_grouped": ([_p, _sz, _sz, _sz, _p, _sz, _p, _p, _sz, _i], _i),
    "nnb_add_fwd": ([_p, _sz, _p, _p, _sz, _p], _i),
    "nnb_accumulate": ([_p, _sz, _p, _p, _i, _i], _i),
    "nnb_maxpool2d_fwd": ([_p, _sz, _sz, _sz, _sz, _sz, _sz, _p, _p, _p], _i),
    "nnb_maxpool2d_bwd": ([_p, _sz, _sz, _sz, _sz, _sz, _sz, _p, _p, _p, _i], _i),
    "nnb_avgpool2d_fwd": ([_p, _sz, _sz, _sz, _sz, _sz, _sz, _p, _p], _i),
    "nnb_avgpool2d_bwd": ([_p, _sz, _sz, _sz, _sz, _sz, _sz, _p, _p, _i], _i),
    "nnb_reduce_axis_fwd": ([_p, _sz, _sz, _sz, _p, _i, _p], _i),
    "nnb_reduce_axis_bwd": ([_p, _sz, _sz, _sz, _p, _i, _p, _i], _i),
    "nnb_conv2d_ex_fwd": ([_p, _sz, _sz, _sz, _sz, _sz, _sz, _sz, _i, _i, _i, _i, _p, _p, _p, _p], _i),
    "nnb_conv2d_ex_bwd": ([_p, _sz, _sz, _sz, _sz, _sz, _sz, _sz, _i, _i, _i, _i, _p, _p, _p, _p, _i, _p, _i, _p, _i],
                          _i),
    "nnb_batchnorm_running_update": ([_p, _sz, _sz, _p, _p, _f, _p, _p], _i),
    "nnb_batchnorm_eval_fwd": ([_p, _sz, _sz, _sz, _p, _p, _p, _f, _p, _p, _i, _p, _p], _i),
    "nnb_batchnorm_eval_bwd": ([_p, _sz, _sz, _sz, _sz, _p, _p, _p, _p, _f, _p, _p, _p, _i, _p, _i, _p, _i], _i),
    "nnb_cross_entropy_fwd": ([_p, _sz, _sz, _p, _p, _p, _p, _p], _i),
    "nnb_cross_entropy_bwd": ([_p, _sz, _sz, _p, _p, _p, _p, _p, _i], _i),
    "nnb_sequence_ce_fwd": ([_p, _sz, _sz, _p, _p, _c.c_int64, _f, _p, _p, _p], _i),
    "nnb_sequence_ce_bwd": ([_p, _sz, _sz, _p, _p, _c.c_int64, _f, _p, _p, _p, _i], _i),
    "nnb_embedding_fwd": ([_p, _sz, _sz, _p, _p, _sz, _p], _i),
    "nnb_embedding_bwd": ([_p, _sz, _sz, _p, _sz, _p, _p, _i], _i),
    "nnb_adamw_step": ([_p, _sz, _p, _p, _p, _p, _f, _f, _f, _f, _f, _c.c_longlong], _i),
    "nnb_adam_bias_table": ([_f, _f, _p, _sz], _sz),
    "nnb_step_advance": ([_p, _p], _i),
    "nnb_adamw_step_device": ([_p, _sz, _p, _p, _p, _p, _p, _p, _sz, _p], _i),
    "nnb_manual_seed": ([_c.c_uint64], None),
    "nnb_is_seeded": ([], _i),
    "nnb_seed_epoch": ([], _c.c_uint64),
    "nnb_derive_generator": ([_c.c_char_p, _p], _i),
    "nnb_mt19937_seed_seq": ([_p, _sz, _p], _i),
    "nnb_dropout_mask": ([_p, _p, _sz, _f, _p], _i),
    "nnb_dropout_mask_slice": ([_p, _p, _sz, _sz, _sz, _f, _p], _i),
    "nnb_dropout_apply": ([_p, _sz, _f, _p, _p, _p], _i),
    "nnb_dropout_bwd": ([_p, _sz, _f, _p, _p, _p, _i], _i),
    "nnb_mt19937_seed": ([_c.c_uint32, _p], _i),
    "nnb_mt19937_next": ([_p, _sz, _p], _i),
    "nnb_fnv1a64": ([_c.c_char_p], _c.c_uint64),
    "nnb_splitmix64": ([_c.c_uint64], _c.c_uint64),
    "nnb_portable_shuffle": ([_p, _p, _sz], _i),
    "nnb_weighted_draws": ([_p, _p, _sz, _sz, _p], _i),
    "nnb_gather_rows": ([_p, _p, _sz, _sz, _p, _sz, _p], _i),
    "nnb_gather_windows": ([_p, _p, _sz, _p, _sz, _sz, _p, _p], _i),
}


def header_symbols() -> list[str]:
    """Names of every function declared in include/nnb.h."""
    text = HEADER.read_text()
    return re.findall(r"NNB_API\s+[\w\s\*]*?\b(nnb_\w+)\s*\(", text)


def lib() -> ctypes.CDLL:
    """Loads libnnb.so once; raises if it has not been built."""
    global _lib
    if _lib is None:
        if not LIB_PATH.exists():
            raise NnbError(f"{LIB_PATH} is missing: build it with __graft_entry__.build()")
        L = ctypes.CDLL(str(LIB_PATH))
        for name, (args, res) in _SIGS.items():
            fn = getattr(L, name)
            fn.argtypes = args
            fn.restype = res
        _lib = L
    return _lib


def last_error() -> str:
    return lib().nnb_last_error().decode()


def check(status: int) -> None:
    """Raises the reference-style exception for a non-OK status."""
    if status == NNB_OK:
        return
    msg = last_error()
    if status == NNB_ERR_SHAPE:
        raise TensorShapeError(msg)
    if status == NNB_ERR_INVALID:
        raise ValueError(msg)
    raise NnbError(f"status {status}: {msg}")


def _stream_ptr(stream) -> int | None:
    if stream is None:
        import torch
        return torch.cuda.current_stream().cuda_stream
    if isinstance(stream, int):
        return stream
    return stream.cuda_stream


def _ptr(t) -> int | None:
    if t is None:
        return None
    if isinstance(t, int):
        return t
    return t.data_ptr()


def set_math_mode(mode: int) -> None:
    check(lib().nnb_set_math_mode(mode))


def get_math_mode() -> int:
    return lib().nnb_get_math_mode()


def device_error(stream=None) -> int:
    return lib().nnb_device_error(_stream_ptr(stream))


TRACE_GEMM, TRACE_PACK, TRACE_AUX, TRACE_ROWWISE, TRACE_ATTENTION, TRACE_CONV = range(6)


def trace_enable(on: bool = True) -> None:
    lib().nnb_trace_enable(int(on))


def trace_reset() -> None:
    lib().nnb_trace_reset()


def trace_query(kind: int) -> tuple[float, int]:
    """(total device ms, launches) of one kernel kind since the last reset."""
    ms, n = ctypes.c_double(), ctypes.c_longlong()
    check(lib().nnb_trace_query(kind, ctypes.byref(ms), ctypes.byref(n)))
    return ms.value, n.value


def launch_count() -> int:
    return lib().nnb_launch_count()


def sgemm(trans_a: bool, trans_b: bool, m: int, n: int, k: int, a, lda: int, b, ldb: int, c, ldc: int,
          accumulate: bool, math_mode: int | None = None, stream=None) -> None:
    """nn::kernels::sgemm (include/nn/kernels/gemm.hpp:57) on device buffers through nnb_sgemm[_ex]."""
    s = _stream_ptr(stream)
    if math_mode is None:
        st = lib().nnb_sgemm(s, int(trans_a), int(trans_b), m, n, k, _ptr(a), lda, _ptr(b), ldb, _ptr(c), ldc,
                             int(accumulate))
    else:
        st = lib().nnb_sgemm_ex(s, int(trans_a), int(trans_b), m, n, k, _ptr(a), lda, _ptr(b), ldb, _ptr(c),
                                ldc, int(accumulate), math_mode)
    check(st)


def sgemm_host(trans_a: bool, trans_b: bool, m: int, n: int, k: int, a, lda: int, b, ldb: int, c, ldc: int,
               accumulate: bool, math_mode: int | None = None, stream=None, blocking: bool = True) -> None:
    """nn::kernels::sgemm on host buffers (numpy arrays or CPU torch tensors, page-locked for full
    copy speed) through nnb_sgemm_host[_async]: copies, pipelined GEMM bands and copy-back inside.
    With blocking=False the call is ordered on `stream` (the current one by default) and returns at
    once; the host buffers must stay alive until that stream reaches the end of the call."""
    def addr(x):
        if x is None:
            return None
        if isinstance(x, int):
            return x
        return x.ctypes.data if hasattr(x, "ctypes") else x.data_ptr()
    mode = get_math_mode() if math_mode is None else math_mode
    s = _stream_ptr(stream)
    check(lib().nnb_sgemm_host_async(s, int(trans_a), int(trans_b), m, n, k, addr(a), lda, addr(b), ldb, addr(c), ldc,
                                     int(accumulate), mode))
    if blocking:
        import torch
        torch.cuda.current_stream().synchronize() if stream is None else stream.synchronize()


def sgemm_host_release() -> None:
    """Frees the device buffers nnb_sgemm_host keeps between calls (after waiting for its work)."""
    check(lib().nnb_sgemm_host_release())


def matmul(a, b, trans_a: bool = False, trans_b: bool = False, stream=None):
    """nn::matmul (src/tensor.cpp:571-641) on torch CUDA tensors; returns a new CUDA tensor."""
    import torch
    a, b = a.contiguous(), b.contiguous()
    ash = (ctypes.c_int64 * a.dim())(*a.shape)
    bsh = (ctypes.c_int64 * b.dim())(*b.shape)
    osh = (ctypes.c_int64 * 16)()
    ond = ctypes.c_int()
    s = _stream_ptr(stream)
    check(lib().nnb_matmul(s, a.data_ptr(), ash, a.dim(), b.data_ptr(), bsh, b.dim(), int(trans_a), int(trans_b),
                           None, osh, ctypes.byref(ond)))
    out = torch.empty(tuple(osh[: ond.value]), device=a.device, dtype=torch.float32)
    check(lib().nnb_matmul(s, a.data_ptr(), ash, a.dim(), b.data_ptr(), bsh, b.dim(), int(trans_a), int(trans_b),
                           out.data_ptr(), osh, ctypes.byref(ond)))
    return out


def sgemm_strided_batched(trans_a: bool, trans_b: bool, m: int, n: int, k: int, a, lda: int, stride_a: int,
                          b, ldb: int, stride_b: int, c, ldc: int, stride_c: int, batch: int,
                          accumulate: bool, math_mode: int = MATH_FP32X3, stream=None) -> None:
    check(lib().nnb_sgemm_strided_batched(_stream_ptr(stream), int(trans_a), int(trans_b), m, n, k, _ptr(a), lda,
                                          stride_a, _ptr(b), ldb, stride_b, _ptr(c), ldc, stride_c, batch,
                                          int(accumulate), math_mode))
