"""Differentiable ops over the C ABI, mirroring nn's autograd ops (include/nn/autograd/ops.hpp).

Each function runs the forward kernel(s), returns a Value, and installs a backward rule that
calls the matching backward entry point with the grad_accum `first` flag of every parent that
needs a gradient. Names and argument meaning follow the reference; shape errors raise
nnb.TensorShapeError as the reference throws TensorShapeError.
"""
from __future__ import annotations

import contextlib
import ctypes
import math
import os

import torch

from . import TensorShapeError, check, lib
from .autograd import Value, empty


def _s():
    return torch.cuda.current_stream().cuda_stream


def _p(t):
    return None if t is None else t.data_ptr()


def _need(v: Value) -> bool:
    return v.requires_grad


# Parameter-gradient groups: with n > 1 the rows of every op's batch are n consecutive groups (the
# data-parallel step's virtual shards) and each parameter's gradient buffer is a [n, size] view; the
# ops then write one gradient per group (the *_grouped entry points).
_GROUPS = 1


@contextlib.contextmanager
def param_groups(n: int):
    global _GROUPS
    old, _GROUPS = _GROUPS, n
    try:
        yield
    finally:
        _GROUPS = old


def _gstride(buf, param: Value) -> int:
    """Elements between consecutive groups' gradients in a parameter's gradient buffer."""
    if buf is None:
        return 0
    return buf.stride(0) if buf.dim() == 2 and buf.shape[0] == _GROUPS and _GROUPS > 1 else param.data.numel()


# ---- linear (ops.cpp:714-745) -------------------------------------------------------------------

def linear(x: Value, weight: Value, bias: Value) -> Value:
    xs, ws = x.shape, weight.shape
    if len(xs) < 2 or len(ws) != 2 or xs[-1] != ws[1] or bias.shape != (ws[0],):
        raise TensorShapeError("linear: shapes do not agree")
    n, K = ws
    M = x.data.numel() // K
    y = empty(xs[:-1] + (n,))
    pack, mode = _input_pack(weight, M, K)
    check(lib().nnb_linear_fwd_ex(_s(), 1, M, K, n, _p(x.data), _p(weight.data), 0, _p(bias.data), 0, _p(y), 0, None,
                                  _p(pack)))

    def backward(g):
        _linear_backward(g, x, weight, bias, M, K, n, pack, mode)

    return Value.node(y, (x, weight, bias), backward)


def _input_pack(weight: Value, M: int, K: int):
    """A buffer that keeps the forward GEMM's packed copy of the input x [M, K] for the weight
    gradient G^T x (nnb_linear_fwd_ex / nnb_linear_bwd_ex: x is then packed once per step instead of
    twice, with the same bits), when that gradient will be taken and the tensor core can read the
    pack for it (every parameter-gradient group a whole number of 16-row blocks); else (None, 0)."""
    if not _need(weight) or M % _GROUPS or (M // _GROUPS) % 16:
        return None, 0
    mode = lib().nnb_get_math_mode()
    return empty((lib().nnb_linear_pack_bytes(M, K, mode),), dtype=torch.uint8), mode


def linear_multi(x: Value, layers) -> list[Value]:
    """[linear(x, w_i, b_i) for (w_i, b_i) in layers] (the q, k, v projections of a self-attention,
    src/nn/attention.cpp:34). When the weights (and the biases) sit at one constant stride in memory --
    the data-parallel trainer's flat parameter buffer lays each Linear out as weight then bias -- the
    products run as one launch that packs x once (nnb_linear_multi_fwd); otherwise one linear per
    layer. Either way every output has linear's bits and linear's backward."""
    ws = [w for w, _ in layers]
    bs = [b for _, b in layers]
    if not ws or any(w.shape != ws[0].shape for w in ws) or any(b.shape != (ws[0].shape[0],) for b in bs):
        return [linear(x, w, b) for w, b in layers]
    xs = x.shape
    if len(xs) < 2 or len(ws[0].shape) != 2 or xs[-1] != ws[0].shape[1]:
        raise TensorShapeError("linear: shapes do not agree")
    n, K = ws[0].shape
    M = x.data.numel() // K

    def stride(ts):
        if any(not t.data.is_contiguous() for t in ts):
            return None
        d = [t.data.data_ptr() - ts[0].data.data_ptr() for t in ts]
        if len(ts) == 1:
            return 0
        if d[1] <= 0 or d[1] % 4 or any(d[i] != i * d[1] for i in range(len(ts))):
            return None
        return d[1] // 4

    w_stride, b_stride = stride(ws), stride(bs)
    if len(layers) == 1 or w_stride is None or b_stride is None or w_stride < n * K or b_stride < n:
        return [linear(x, w, b) for w, b in layers]
    y = empty((len(layers),) + xs[:-1] + (n,))
    pack, mode = _input_pack(ws[0], M, K)      # x's pack, shared by every product and its backward
    check(lib().nnb_linear_fwd_ex(_s(), len(layers), M, K, n, _p(x.data), _p(ws[0].data), w_stride,
                                  _p(bs[0].data), b_stride, _p(y), M * n, None, _p(pack)))
    outs = []
    for i, (w, b) in enumerate(layers):
        def backward(g, w=w, b=b):
            _linear_backward(g, x, w, b, M, K, n, pack if _need(w) else None, mode)
        outs.append(Value.node(y[i], (x, w, b), backward))
    return outs


def _linear_backward(g, x, weight, bias, M, K, n, pack=None, mode=0):
    """nnb_linear_bwd_ex: nnb_linear_bwd (one group) or nnb_linear_bwd_grouped, the weight gradient
    reading x's pack from the forward when it was kept."""
    dx, fx = x.grad_accum() if _need(x) else (None, 0)
    dw, fw = weight.grad_accum() if _need(weight) else (None, 0)
    db, fb = bias.grad_accum() if _need(bias) else (None, 0)
    check(lib().nnb_linear_bwd_ex(_s(), M, K, n, _GROUPS, _p(g), _p(x.data), _p(pack), mode, _p(weight.data), _p(dx),
                                  fx, _p(dw), _gstride(dw, weight), fw, _p(db), _gstride(db, bias), fb))


def linear_gelu(x: Value, weight: Value, bias: Value) -> Value:
    """gelu(linear(x, w, b)) as one GEMM with the GELU in its epilogue (same bits as the two ops)."""
    xs, ws = x.shape, weight.shape
    if len(xs) < 2 or len(ws) != 2 or xs[-1] != ws[1] or bias.shape != (ws[0],):
        raise TensorShapeError("linear: shapes do not agree")
    n, K = ws
    M = x.data.numel() // K
    y = empty(xs[:-1] + (n,))
    pre = empty(xs[:-1] + (n,))
    pack, mode = _input_pack(weight, M, K)
    check(lib().nnb_linear_fwd_ex(_s(), 1, M, K, n, _p(x.data), _p(weight.data), 0, _p(bias.data), 0, _p(y), 0,
                                  _p(pre), _p(pack)))

    def backward(g):
        dpre = empty(pre.shape)
        check(lib().nnb_gelu_bwd(_s(), pre.numel(), _p(pre), None, _p(g), _p(dpre), 1))
        _linear_backward(dpre, x, weight, bias, M, K, n, pack, mode)

    return Value.node(y, (x, weight, bias), backward)


# ---- matmul / matmul_bt (ops.cpp:683-712, 747-773) ------------------------------------------------

def _sum_to_shape_into(g: torch.Tensor, target: tuple, dst: torch.Tensor, first: int) -> None:
    """accumulate_grad (ops.cpp:110-117) of a gradient with the broadcast shape g.shape into dst (the
    gradient of a value shaped `target`): the leading axes are summed away one at a time (each a
    Tensor::sum(0), src/tensor.cpp:422-455), then every axis where target has 1 and g does not, in
    axis order (sum_to_shape, ops.cpp:35-53); the result is stored (first) or added into dst."""
    cur = g
    while cur.dim() > len(target):
        red = empty(cur.shape[1:])
        check(lib().nnb_column_sum(_s(), cur.shape[0], red.numel(), _p(cur), _p(red), 1))
        cur = red
    for i, t in enumerate(target):
        if t == 1 and cur.shape[i] != 1:
            sh = list(cur.shape)
            red = empty(sh[:i] + [1] + sh[i + 1:])
            check(lib().nnb_reduce_axis_fwd(_s(), math.prod(sh[:i]), sh[i], math.prod(sh[i + 1:]), _p(cur), 0, _p(red)))
            cur = red
    if tuple(cur.shape) != tuple(target):
        raise TensorShapeError("matmul: gradient does not reduce to the operand's shape")
    check(lib().nnb_accumulate(_s(), cur.numel(), _p(cur), _p(dst), first, 0))


def _accumulate_grad(v: Value, grad: torch.Tensor) -> None:
    dst, first = v.grad_accum()
    if tuple(grad.shape) == v.shape:
        check(lib().nnb_accumulate(_s(), grad.numel(), _p(grad), _p(dst), first, 0))
    else:
        _sum_to_shape_into(grad, v.shape, dst, first)


def _sgemm_into(ta, tb, m, n, k, a, lda, b, ldb, c, ldc, first):
    check(lib().nnb_sgemm(_s(), ta, tb, m, n, k, _p(a), lda, _p(b), ldb, _p(c), ldc, 0 if first else 1))


def _matmul_value(a: Value, b: Value, bt: bool) -> Value:
    from . import matmul as tensor_matmul
    y = tensor_matmul(a.data, b.data, False, bt)

    def backward(g):
        if len(b.shape) == 2 and len(a.shape) >= 2:
            # b a plain matrix: a's leading axes fold into M rows and both gradients come from one
            # GEMM each, stored (first) or accumulated (ops.cpp:686-700, 750-761)
            if bt:
                n, K = b.shape
            else:
                K, n = b.shape
            M = a.data.numel() // K
            if _need(a):
                da, fa = a.grad_accum()
                if bt:
                    _sgemm_into(0, 0, M, K, n, g, n, b.data, K, da, K, fa)
                else:
                    _sgemm_into(0, 1, M, K, n, g, n, b.data, n, da, K, fa)
            if _need(b):
                db, fb = b.grad_accum()
                if bt:
                    _sgemm_into(1, 0, n, K, M, g, n, a.data, K, db, K, fb)
                else:
                    _sgemm_into(1, 0, K, n, M, a.data, K, g, n, db, n, fb)
            return
        # batched b: the batched products, then the broadcast axes summed away (ops.cpp:703-710)
        if _need(a):
            _accumulate_grad(a, tensor_matmul(g, b.data, False, not bt))
        if _need(b):
            _accumulate_grad(b, tensor_matmul(g, a.data, True, False) if bt else tensor_matmul(a.data, g, True, False))

    return Value.node(y, (a, b), backward)


def matmul(a: Value, b: Value) -> Value:
    """a @ b with batch axes broadcast (nn::matmul(const Value&, const Value&), ops.cpp:683)."""
    return _matmul_value(a, b, False)


def matmul_bt(a: Value, b: Value) -> Value:
    """a @ b^T over the last two axes (nn::matmul_bt, ops.cpp:747)."""
    return _matmul_value(a, b, True)


def scaled_masked_softmax(x: Value, scale: float, key_padding_mask: torch.Tensor | None = None,
                          causal: bool = False) -> Value:
    """softmax(masked(x * scale)) over the last axis of x [N, H, Tq, Tk] (ops.cpp:1298-1343): padded
    keys (mask 0) get -1e9 and causally hidden keys (j > i) -2e9 before the softmax."""
    if len(x.shape) != 4 or x.shape[3] == 0:
        raise TensorShapeError("scaled_masked_softmax: x must be [N, H, Tq, Tk]")
    N, H, Tq, Tk = x.shape
    if key_padding_mask is not None and key_padding_mask.numel() and tuple(key_padding_mask.shape) != (N, Tk):
        raise TensorShapeError("scaled_masked_softmax: key_padding_mask must be [N, Tk]")
    pad = key_padding_mask if key_padding_mask is not None and key_padding_mask.numel() else None
    y = empty(x.shape)
    check(lib().nnb_scaled_masked_softmax_fwd(_s(), N, H, Tq, Tk, _p(x.data), _p(y), _p(pad), int(causal),
                                              ctypes.c_float(scale)))

    def backward(g):
        if _need(x):
            dx, f = x.grad_accum()
            check(lib().nnb_scaled_masked_softmax_bwd(_s(), N, H, Tq, Tk, _p(y), _p(g), _p(dx), f, _p(pad), int(causal),
                                                      ctypes.c_float(scale)))

    return Value.node(y, (x,), backward)


# ---- elementwise ------------------------------------------------------------------------------

def add(a: Value, b: Value) -> Value:
    """a + b for equal shapes, or b broadcast over a's leading axes (b's shape a suffix of a's)."""
    if a.shape != b.shape and (len(b.shape) > len(a.shape) or a.shape[len(a.shape) - len(b.shape):] != b.shape):
        raise TensorShapeError("add: shapes do not broadcast")
    y = empty(a.shape)
    check(lib().nnb_add_fwd(_s(), a.data.numel(), _p(a.data), _p(b.data), b.data.numel(), _p(y)))
    same = a.shape == b.shape

    def backward(g):
        if _need(a):
            da, f = a.grad_accum()
            check(lib().nnb_accumulate(_s(), g.numel(), _p(g), _p(da), f, 0))
        if _need(b):
            db, f = b.grad_accum()
            if same:
                check(lib().nnb_accumulate(_s(), g.numel(), _p(g), _p(db), f, 0))
            else:   # sum over the broadcast leading axes (sum_to_shape, ops.cpp:35-53)
                rows = g.numel() // b.data.numel()
                check(lib().nnb_column_sum(_s(), rows, b.data.numel(), _p(g), _p(db), f))

    return Value.node(y, (a, b), backward)


def relu(x: Value) -> Value:
    y = empty(x.shape)
    check(lib().nnb_relu_fwd(_s(), x.data.numel(), _p(x.data), _p(y)))

    def backward(g):
        dx, f = x.grad_accum()
        check(lib().nnb_relu_bwd(_s(), g.numel(), _p(x.data), _p(g), _p(dx), f))

    return Value.node(y, (x,), backward)


def gelu(x: Value) -> Value:
    y, th = empty(x.shape), empty(x.shape)
    check(lib().nnb_gelu_fwd(_s(), x.data.numel(), _p(x.data), _p(y), _p(th)))

    def backward(g):
        dx, f = x.grad_accum()
        check(lib().nnb_gelu_bwd(_s(), g.numel(), _p(x.data), _p(th), _p(g), _p(dx), f))

    return Value.node(y, (x,), backward)


def reshape(x: Value, shape) -> Value:
    shape = tuple(shape)
    n = 1
    for d in shape:
        n *= d
    if n != x.data.numel():
        raise TensorShapeError("reshape: element count differs")
    y = x.data.view(shape)

    def backward(g):
        dx, f = x.grad_accum()
        check(lib().nnb_accumulate(_s(), g.numel(), _p(g), _p(dx), f, 0))

    return Value.node(y, (x,), backward)


# ---- normalisation ------------------------------------------------------------------------------

def layernorm(x: Value, gamma: Value, beta: Value, eps: float) -> Value:
    D = x.shape[-1] if x.shape else 0
    if not x.shape or gamma.shape != (D,) or beta.shape != (D,):
        raise TensorShapeError("layernorm: shapes do not agree")
    R = x.data.numel() // D
    y, mean, inv = empty(x.shape), empty((R,)), empty((R,))
    check(lib().nnb_layernorm_fwd(_s(), R, D, _p(x.data), _p(gamma.data), _p(beta.data), ctypes.c_float(eps), _p(y),
                                  _p(mean), _p(inv)))

    def backward(g):
        dx, fx = x.grad_accum() if _need(x) else (None, 0)
        dg, fg = gamma.grad_accum() if _need(gamma) else (None, 0)
        db, fb = beta.grad_accum() if _need(beta) else (None, 0)
        check(lib().nnb_layernorm_bwd_grouped(_s(), R, D, _GROUPS, _p(g), _p(x.data), _p(gamma.data), _p(mean), _p(inv),
                                              _p(dx), fx, _p(dg), _gstride(dg, gamma), fg, _p(db), _gstride(db, beta),
                                              fb))

    return Value.node(y, (x, gamma, beta), backward)


def batchnorm(x: Value, weight: Value, bias: Value, eps: float, fuse_relu: bool = False,
              mean_out: torch.Tensor | None = None, var_out: torch.Tensor | None = None) -> Value:
    """batchnorm in training mode (ops.cpp:900-1001); mean_out / var_out receive the batch statistics
    (biased variance), as the reference's Tensor* outputs."""
    if len(x.shape) < 2:
        raise TensorShapeError("batchnorm: needs N and C axes")
    N, C = x.shape[0], x.shape[1]
    S = x.data.numel() // max(1, N * C)
    y = empty(x.shape)
    alive = empty(x.shape, dtype=torch.uint8) if fuse_relu else None
    mean = mean_out if mean_out is not None else empty((C,))
    var = var_out if var_out is not None else empty((C,))
    inv = empty((C,))
    check(lib().nnb_batchnorm_fwd(_s(), N, C, S, _p(x.data), _p(weight.data), _p(bias.data), ctypes.c_float(eps),
                                  int(fuse_relu), _p(y), _p(alive), _p(mean), _p(var), _p(inv)))

    def backward(g):
        dx, fx = x.grad_accum() if _need(x) else (None, 0)
        dw, fw = weight.grad_accum() if _need(weight) else (None, 0)
        db, fb = bias.grad_accum() if _need(bias) else (None, 0)
        check(lib().nnb_batchnorm_bwd(_s(), N, C, S, _p(g), _p(x.data), _p(weight.data), _p(mean), _p(inv), _p(alive),
                                      _p(dx), fx, _p(dw), fw, _p(db), fb))

    out = Value.node(y, (x, weight, bias), backward)
    out.name = "batchnorm"
    return out


def batchnorm_eval(x: Value, weight: Value, bias: Value, running_mean: torch.Tensor, running_var: torch.Tensor,
                   eps: float, fuse_relu: bool = False) -> Value:
    """Evaluation-mode batch normalisation from the running statistics (batchnorm.cpp:51-55)."""
    if len(x.shape) < 2:
        raise TensorShapeError("batchnorm: needs N and C axes")
    N, C = x.shape[0], x.shape[1]
    S = x.data.numel() // max(1, N * C)
    if len(x.shape) > 4:
        raise TensorShapeError("batchnorm: at most four axes")
    Hs = x.shape[2] if len(x.shape) > 2 else 1      # the axes the parameter gradients sum over, in order
    Ws = x.shape[3] if len(x.shape) > 3 else 1
    y = empty(x.shape)
    alive = empty(x.shape, dtype=torch.uint8) if fuse_relu else None
    check(lib().nnb_batchnorm_eval_fwd(_s(), N, C, S, _p(x.data), _p(running_mean), _p(running_var),
                                       ctypes.c_float(eps), _p(weight.data), _p(bias.data), int(fuse_relu), _p(y),
                                       _p(alive)))

    def backward(g):
        dx, fx = x.grad_accum() if _need(x) else (None, 0)
        dw, fw = weight.grad_accum() if _need(weight) else (None, 0)
        db, fb = bias.grad_accum() if _need(bias) else (None, 0)
        check(lib().nnb_batchnorm_eval_bwd(_s(), N, C, Hs, Ws, _p(g), _p(x.data), _p(running_mean), _p(running_var),
                                           ctypes.c_float(eps), _p(weight.data), _p(alive), _p(dx), fx, _p(dw), fw,
                                           _p(db), fb))

    return Value.node(y, (x, weight, bias), backward)


# ---- attention (ops.cpp:1226-1296) --------------------------------------------------------------

def attention(q: Value, k: Value, v: Value, heads: int, key_padding_mask: torch.Tensor | None = None,
              causal: bool = False, fused: bool | None = None) -> Value:
    """Multi-head attention (ops.cpp:1226-1296). Head size 64 runs the fused kernels (no
    [N, heads, Tq, Tk] probabilities kept; the backward recomputes them from the row max and sum);
    other head sizes, or fused=False (or NNB_ATTENTION=composed), run the reference's composition:
    head-batched GEMMs around the masked softmax, keeping the probabilities."""
    qs, ks = q.shape, k.shape
    if len(qs) != 3 or len(ks) != 3 or v.shape != ks or qs[0] != ks[0] or qs[2] != ks[2]:
        raise TensorShapeError("attention: shapes do not agree")
    N, Tq, D = qs
    Tk = ks[1]
    if fused is None:
        fused = FUSED_ATTENTION
    if fused and heads > 0 and lib().nnb_flash_attention_supported(D, heads):
        return _flash_attention(q, k, v, heads, key_padding_mask, causal, N, Tq, Tk, D)
    out, probs = empty((N, Tq, D)), empty((N, heads, Tq, Tk))
    check(lib().nnb_attention_fwd(_s(), N, Tq, Tk, D, heads, _p(q.data), _p(k.data), _p(v.data),
                                  _p(key_padding_mask), int(causal), _p(out), _p(probs)))

    def backward(g):
        # fetched in the reference's order (v, q, k: ops.cpp:1273-1275)
        dv, fv = v.grad_accum() if _need(v) else (None, 0)
        dq, fq = q.grad_accum() if _need(q) else (None, 0)
        dk, fk = k.grad_accum() if _need(k) else (None, 0)
        check(lib().nnb_attention_bwd(_s(), N, Tq, Tk, D, heads, _p(g), _p(q.data), _p(k.data), _p(v.data),
                                      _p(probs), _p(key_padding_mask), int(causal), _p(dq), fq, _p(dk), fk, _p(dv),
                                      fv))

    return Value.node(out, (q, k, v), backward)


FUSED_ATTENTION = os.environ.get("NNB_ATTENTION", "fused").lower() != "composed"


def _flash_attention(q, k, v, heads, key_padding_mask, causal, N, Tq, Tk, D) -> Value:
    out, stats = empty((N, Tq, D)), empty((N, heads, Tq, 2))
    check(lib().nnb_flash_attention_fwd(_s(), N, Tq, Tk, D, heads, _p(q.data), _p(k.data), _p(v.data),
                                        _p(key_padding_mask), int(causal), _p(out), _p(stats)))

    def backward(g):
        dv, fv = v.grad_accum() if _need(v) else (None, 0)
        dq, fq = q.grad_accum() if _need(q) else (None, 0)
        dk, fk = k.grad_accum() if _need(k) else (None, 0)
        check(lib().nnb_flash_attention_bwd(_s(), N, Tq, Tk, D, heads, _p(g), _p(q.data), _p(k.data), _p(v.data),
                                            _p(out), _p(stats), _p(key_padding_mask), int(causal), _p(dq), fq, _p(dk),
                                            fk, _p(dv), fv))

    return Value.node(out, (q, k, v), backward)


# ---- dropout (src/nn/dropout.cpp:20-31) and attention with dropout (src/nn/attention.cpp:36-47) ------

# Batch slice of a data-parallel rank: (rows of the whole batch, first row, end row) while a rank runs
# its rows of a batch whose dropout masks the reference draws over all rows at once.
_BATCH_SLICE = None


@contextlib.contextmanager
def batch_slice(total_rows: int, row_lo: int, row_hi: int):
    """Inside, every dropout mask is drawn as this rank's rows [row_lo, row_hi) of the mask the whole
    batch of total_rows rows would draw (dropout.cpp:20-31 draws row-major from one generator), and
    the generator advances past the whole batch's draws: ranks stay in step and every rank's masks are
    the single-process masks' rows."""
    global _BATCH_SLICE
    old = _BATCH_SLICE
    _BATCH_SLICE = None if (row_lo == 0 and row_hi == total_rows) else (total_rows, row_lo, row_hi)
    try:
        yield
    finally:
        _BATCH_SLICE = old


def dropout_mask(state: torch.Tensor, n: int, p: float) -> torch.Tensor:
    """Dropout::forward's n keep / drop decisions drawn from the device generator `state` (advanced
    in place): (n + 31) // 32 words, bit e % 32 of word e // 32 set when element e is kept. Inside
    batch_slice, n covers this rank's rows and the draw is that slice of the whole batch's."""
    keep = empty(((n + 31) // 32,), dtype=torch.int32, device=state.device)
    if _BATCH_SLICE is None:
        check(lib().nnb_dropout_mask(_s(), _p(state), n, ctypes.c_float(p), _p(keep)))
    else:
        total_rows, lo, hi = _BATCH_SLICE
        if hi <= lo or n % (hi - lo):
            raise ValueError("dropout under batch_slice: the tensor's leading axis is not the rank's rows")
        per_row = n // (hi - lo)
        check(lib().nnb_dropout_mask_slice(_s(), _p(state), per_row * total_rows, per_row * lo, n, ctypes.c_float(p),
                                           _p(keep)))
    return keep


def dropout(x: Value, p: float, state: torch.Tensor) -> Value:
    """x * m, m = 0 with probability p else 1 / (1 - p), the mask drawn from `state` in row-major order."""
    n = x.data.numel()
    keep = dropout_mask(state, n, p)
    y = empty(x.shape, device=x.data.device)
    check(lib().nnb_dropout_apply(_s(), n, ctypes.c_float(p), _p(x.data), _p(keep), _p(y)))

    def backward(g):
        if _need(x):
            dx, f = x.grad_accum()
            check(lib().nnb_dropout_bwd(_s(), n, ctypes.c_float(p), _p(g), _p(keep), _p(dx), f))

    return Value.node(y, (x,), backward)


def attention_dropout(q: Value, k: Value, v: Value, heads: int, key_padding_mask: torch.Tensor | None, causal: bool,
                      p: float, state: torch.Tensor) -> Value:
    """MultiHeadAttention's core with its Dropout active: per head scores = q k^T, scaled_masked_softmax
    (ops.cpp:1298-1343), the dropout mask drawn over the [N, heads, Tq, Tk] weights, then weights v.
    The probabilities and the dropped weights are kept for the backward, as the reference's graph
    keeps them."""
    qs, ks = q.shape, k.shape
    if len(qs) != 3 or len(ks) != 3 or v.shape != ks or qs[0] != ks[0] or qs[2] != ks[2]:
        raise TensorShapeError("attention: shapes do not agree")
    N, Tq, D = qs
    Tk = ks[1]
    if heads == 0 or D % heads or (causal and Tq != Tk):
        raise TensorShapeError("attention: bad heads or causal shape")
    if key_padding_mask is not None and tuple(key_padding_mask.shape) != (N, Tk):
        raise TensorShapeError("attention: key padding mask must be [N, Tk]")
    keep = dropout_mask(state, N * heads * Tq * Tk, p)
    out, probs, weights = empty((N, Tq, D)), empty((N, heads, Tq, Tk)), empty((N, heads, Tq, Tk))
    check(lib().nnb_attention_dropout_fwd(_s(), N, Tq, Tk, D, heads, _p(q.data), _p(k.data), _p(v.data),
                                          _p(key_padding_mask), int(causal), ctypes.c_float(p), _p(keep), _p(out),
                                          _p(probs), _p(weights)))

    def backward(g):
        dv, fv = v.grad_accum() if _need(v) else (None, 0)
        dq, fq = q.grad_accum() if _need(q) else (None, 0)
        dk, fk = k.grad_accum() if _need(k) else (None, 0)
        check(lib().nnb_attention_dropout_bwd(_s(), N, Tq, Tk, D, heads, _p(g), _p(q.data), _p(k.data), _p(v.data),
                                              _p(probs), _p(weights), ctypes.c_float(p), _p(keep),
                                              _p(key_padding_mask), int(causal), _p(dq), fq, _p(dk), fk, _p(dv), fv))

    return Value.node(out, (q, k, v), backward)


# ---- convolution and pooling ---------------------------------------------------------------------

def conv2d(x: Value, weight: Value, bias: Value, stride: int, padding: int, fuse_relu: bool = False,
           dilation: int = 1, groups: int = 1) -> Value:
    if dilation != 1 or groups != 1:
        if fuse_relu:
            raise ValueError("conv2d: the folded ReLU needs dilation 1 and groups 1 (conv2d.hpp:72)")
        return _conv2d_general(x, weight, bias, stride, padding, dilation, groups)
    if len(x.shape) != 4 or len(weight.shape) != 4:
        raise TensorShapeError("conv2d: needs 4-D input and weight")
    N, Cin, H, W = x.shape
    Cout, wc, kh, kw = weight.shape
    if wc != Cin or bias.shape != (Cout,):
        raise TensorShapeError("conv2d: channels do not agree")
    if stride <= 0 or padding < 0 or kh > H + 2 * padding or kw > W + 2 * padding:
        raise TensorShapeError("conv2d: bad window")
    ho, wo = (H + 2 * padding - kh) // stride + 1, (W + 2 * padding - kw) // stride + 1
    y = empty((N, Cout, ho, wo))
    alive = empty((N, Cout, ho, wo), dtype=torch.uint8) if fuse_relu else None
    check(lib().nnb_conv2d_fwd(_s(), N, Cin, H, W, Cout, kh, kw, stride, padding, _p(x.data), _p(weight.data),
                               _p(bias.data), int(fuse_relu), _p(y), _p(alive)))

    def backward(g):
        dx, fx = x.grad_accum() if _need(x) else (None, 0)
        dw, fw = weight.grad_accum() if _need(weight) else (None, 0)
        db, fb = bias.grad_accum() if _need(bias) else (None, 0)
        check(lib().nnb_conv2d_bwd(_s(), N, Cin, H, W, Cout, kh, kw, stride, padding, _p(g), _p(x.data),
                                   _p(weight.data), _p(alive), _p(dx), fx, _p(dw), fw, _p(db), fb))

    return Value.node(y, (x, weight, bias), backward)


def _conv2d_general(x: Value, weight: Value, bias: Value, stride: int, padding: int, dilation: int,
                    groups: int) -> Value:
    """conv2d with dilation / groups (ops.cpp:1525-1607): per sample and group, im2col + GEMM."""
    if len(x.shape) != 4 or len(weight.shape) != 4:
        raise TensorShapeError("conv2d: needs 4-D input and weight")
    N, Cin, H, W = x.shape
    Cout, Cg, kh, kw = weight.shape
    if bias.shape != (Cout,) or groups <= 0 or dilation <= 0 or stride <= 0 or padding < 0 or Cin % groups \
            or Cout % groups or Cg != Cin // groups:
        raise TensorShapeError("conv2d: shapes do not agree")
    ekh, ekw = dilation * (kh - 1) + 1, dilation * (kw - 1) + 1
    if ekh > H + 2 * padding or ekw > W + 2 * padding:
        raise TensorShapeError("conv2d: bad window")
    ho, wo = (H + 2 * padding - ekh) // stride + 1, (W + 2 * padding - ekw) // stride + 1
    y = empty((N, Cout, ho, wo))
    check(lib().nnb_conv2d_ex_fwd(_s(), N, Cin, H, W, Cout, kh, kw, stride, padding, dilation, groups, _p(x.data),
                                  _p(weight.data), _p(bias.data), _p(y)))

    def backward(g):
        dx, fx = x.grad_accum() if _need(x) else (None, 0)
        dw, fw = weight.grad_accum() if _need(weight) else (None, 0)
        db, fb = bias.grad_accum() if _need(bias) else (None, 0)
        check(lib().nnb_conv2d_ex_bwd(_s(), N, Cin, H, W, Cout, kh, kw, stride, padding, dilation, groups, _p(g),
                                      _p(x.data), _p(weight.data), _p(dx), fx, _p(dw), fw, _p(db), fb))

    return Value.node(y, (x, weight, bias), backward)


def conv2d_relu(x: Value, weight: Value, bias: Value, stride: int, padding: int) -> Value:
    return conv2d(x, weight, bias, stride, padding, fuse_relu=True)


def maxpool2d(x: Value, kernel_size: int, stride: int) -> Value:
    if len(x.shape) != 4 or kernel_size == 0 or stride == 0:
        raise TensorShapeError("maxpool2d: bad input")
    N, C, H, W = x.shape
    if kernel_size > H or kernel_size > W:
        raise TensorShapeError("maxpool2d: window larger than the input")
    ho, wo = (H - kernel_size) // stride + 1, (W - kernel_size) // stride + 1
    y = empty((N, C, ho, wo))
    arg = empty((N, C, ho, wo), dtype=torch.int32)
    check(lib().nnb_maxpool2d_fwd(_s(), N, C, H, W, kernel_size, stride, _p(x.data), _p(y), _p(arg)))

    def backward(g):
        dx, f = x.grad_accum()
        check(lib().nnb_maxpool2d_bwd(_s(), N, C, H, W, kernel_size, stride, _p(g), _p(arg), _p(dx), f))

    return Value.node(y, (x,), backward)


def avgpool2d(x: Value, kernel_size: int, stride: int) -> Value:
    """avgpool2d (ops.cpp:1707-1772)."""
    if len(x.shape) != 4 or kernel_size == 0 or stride == 0:
        raise TensorShapeError("avgpool2d: bad input")
    N, C, H, W = x.shape
    if kernel_size > H or kernel_size > W:
        raise TensorShapeError("avgpool2d: window larger than the input")
    ho, wo = (H - kernel_size) // stride + 1, (W - kernel_size) // stride + 1
    y = empty((N, C, ho, wo))
    check(lib().nnb_avgpool2d_fwd(_s(), N, C, H, W, kernel_size, stride, _p(x.data), _p(y)))

    def backward(g):
        if _need(x):
            dx, fx = x.grad_accum()
            check(lib().nnb_avgpool2d_bwd(_s(), N, C, H, W, kernel_size, stride, _p(g), _p(dx), fx))

    return Value.node(y, (x,), backward)


def _reduce_axis(x: Value, axis: int, keepdim: bool, average: bool) -> Value:
    """sum / mean over one axis (reduce_axis, ops.cpp:284-376)."""
    shape = list(x.shape)
    nd = len(shape)
    if axis < -nd or axis >= nd:
        raise IndexError("reduce over an axis out of range")     # the reference throws TensorIndexError
    ax = axis + nd if axis < 0 else axis
    n = shape[ax]
    if n == 0:
        raise TensorShapeError("reduce over an empty axis")
    outer = math.prod(shape[:ax])
    inner = math.prod(shape[ax + 1:])
    out_shape = [d for i, d in enumerate(shape) if i != ax] if not keepdim else \
        [1 if i == ax else d for i, d in enumerate(shape)]
    y = empty(tuple(out_shape) if out_shape else (1,))
    check(lib().nnb_reduce_axis_fwd(_s(), outer, n, inner, _p(x.data), int(average), _p(y)))

    def backward(g):
        if _need(x):
            dx, fx = x.grad_accum()
            check(lib().nnb_reduce_axis_bwd(_s(), outer, n, inner, _p(g), int(average), _p(dx), fx))

    return Value.node(y, (x,), backward)


def sum(x: Value, axis: int, keepdim: bool = False) -> Value:      # noqa: A001 - the reference's name
    return _reduce_axis(x, axis, keepdim, False)


def mean(x: Value, axis: int, keepdim: bool = False) -> Value:
    return _reduce_axis(x, axis, keepdim, True)


# ---- embedding and losses -----------------------------------------------------------------------

def embedding(weight: Value, ids: torch.Tensor) -> Value:
    """ids: a CUDA int64 tensor of any shape; returns ids.shape + (D,) (ops.cpp:1991-2015)."""
    if len(weight.shape) != 2:
        raise TensorShapeError("embedding: weight must be 2-D")
    V, D = weight.shape
    cnt = ids.numel()
    out = empty(tuple(ids.shape) + (D,))
    check(lib().nnb_embedding_fwd(_s(), V, D, _p(weight.data), _p(ids), cnt, _p(out)))

    def backward(g):
        dw, f = weight.grad_accum()
        if _GROUPS > 1:
            check(lib().nnb_embedding_bwd_grouped(_s(), V, D, _GROUPS, _p(ids), cnt, _p(g), _p(dw), _gstride(dw, weight),
                                                  f))
        else:
            check(lib().nnb_embedding_bwd(_s(), V, D, _p(ids), cnt, _p(g), _p(dw), f))

    return Value.node(out, (weight,), backward)


def cross_entropy_loss(logits: Value, targets: torch.Tensor) -> Value:
    if len(logits.shape) != 2 or targets.dim() != 1 or targets.numel() != logits.shape[0]:
        raise TensorShapeError("cross_entropy_loss: shapes do not agree")
    N, C = logits.shape
    sm, loss, norm = empty((N, C)), empty((1,)), empty((1,))
    check(lib().nnb_cross_entropy_fwd(_s(), N, C, _p(logits.data), _p(targets), _p(sm), _p(loss), _p(norm)))

    def backward(g):
        dl, f = logits.grad_accum()
        check(lib().nnb_cross_entropy_bwd(_s(), N, C, _p(sm), _p(targets), _p(g), _p(norm), _p(dl), f))

    return Value.node(loss, (logits,), backward)


def sequence_cross_entropy(logits: Value, targets: torch.Tensor, ignore_index: int = -100,
                           label_smoothing: float = 0.0, grad_norm: torch.Tensor | None = None) -> Value:
    """grad_norm: a device scalar used by the backward pass in place of 1/(positions counted here),
    e.g. 1/(positions of the global batch) when this call sees one rank's part of it."""
    if len(logits.shape) != 3 or tuple(targets.shape) != logits.shape[:2]:
        raise TensorShapeError("sequence_cross_entropy: shapes do not agree")
    N, T, V = logits.shape
    P = N * T
    sm, loss, norm = empty((P, V)), empty((1,)), empty((1,))
    check(lib().nnb_sequence_ce_fwd(_s(), P, V, _p(logits.data), _p(targets), ignore_index,
                                    ctypes.c_float(label_smoothing), _p(sm), _p(loss), _p(norm)))

    def backward(g):
        dl, f = logits.grad_accum()
        check(lib().nnb_sequence_ce_bwd(_s(), P, V, _p(sm), _p(targets), ignore_index, ctypes.c_float(label_smoothing),
                                        _p(g), _p(norm if grad_norm is None else grad_norm), _p(dl), f))

    return Value.node(loss, (logits,), backward)
