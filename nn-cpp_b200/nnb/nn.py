"""Modules and the AdamW optimizer on the device, mirroring nn-cpp's nn modules (include/nn/nn/*.hpp)
and optimizer (include/nn/optim/adamw.hpp).

Structure, forward composition, parameter names and their order (named_parameters) follow the
reference, so a checkpoint or a parameter list maps one to one:
  Linear            src/nn/linear.cpp:18-26          weight [out, in], bias [out]
  LayerNorm         src/nn/layernorm.cpp             gamma, beta
  Embedding         src/nn/embedding.cpp             weight [V, D]
  PositionalEncoding (sinusoidal) src/nn/positional.cpp:15-38
  MultiHeadAttention src/nn/attention.cpp:15-48      q., k., v., o. (no active dropout: the fused attention op)
  Dropout           src/nn/dropout.cpp               device mt19937 stream, 1-bit keep masks
  TransformerBlock  src/nn/transformer.cpp:37-55     ln1., attn., ln2., fc1., fc2.  (pre-LN)
  Transformer       src/nn/transformer.cpp:66-90     embed., pos., blocks.<i>., ln_f., head.
  Conv2d / Sequential (folds Conv2d + ReLU into conv2d_relu, src/nn/sequential.cpp:16-28)
Initial values are drawn on the host from a seeded numpy generator with the reference's
distributions (U(+-1/sqrt(fan_in)) weights, zero biases, LayerNorm gamma 1 / beta 0) and uploaded;
to reproduce the reference's own numbers the tests load the same values into both.
"""
from __future__ import annotations

import ctypes
import math
from dataclasses import dataclass

import numpy as np
import torch

from . import TensorShapeError, check, lib
from . import functional as F
from . import random as nnb_random
from .autograd import Value


def _param(array: np.ndarray, device) -> Value:
    return Value.leaf(torch.from_numpy(np.ascontiguousarray(array, np.float32)).to(device), True)


class Module:
    training = True

    def named_parameters(self) -> list[tuple[str, Value]]:
        return []

    def train(self, mode: bool = True):
        """Sets training / evaluation mode here and in every sub-module (Module::train, module.hpp:93)."""
        self.training = mode
        for child in vars(self).values():
            for m in (child if isinstance(child, list) else [child]):
                if isinstance(m, Module):
                    m.train(mode)
        return self

    def eval(self):
        return self.train(False)

    def modules(self):
        """This module and every sub-module, depth first in attribute order."""
        yield self
        for child in vars(self).values():
            for m in (child if isinstance(child, list) else [child]):
                if isinstance(m, Module):
                    yield from m.modules()

    def named_buffers(self) -> list[tuple[str, torch.Tensor]]:
        return []

    def parameters(self) -> list[Value]:
        return [p for _, p in self.named_parameters()]

    def zero_grad(self) -> None:
        for p in self.parameters():
            p.zero_grad()

    def load_parameters(self, arrays) -> None:
        """Copies host arrays (in named_parameters order) into the parameters."""
        params = self.parameters()
        if len(arrays) != len(params):
            raise ValueError("parameter count differs")
        for p, a in zip(params, arrays):
            t = torch.from_numpy(np.ascontiguousarray(a, np.float32).reshape(p.shape))
            p.data.copy_(t, non_blocking=False)

    def __call__(self, x):
        return self.forward(x)


class Linear(Module):
    def __init__(self, in_features: int, out_features: int, rng: np.random.Generator, device):
        lim = 1.0 / math.sqrt(in_features)
        self.weight = _param(rng.uniform(-lim, lim, (out_features, in_features)), device)
        self.bias = _param(np.zeros(out_features), device)

    def forward(self, x: Value) -> Value:
        return F.linear(x, self.weight, self.bias)

    def named_parameters(self):
        return [("weight", self.weight), ("bias", self.bias)]


class LayerNorm(Module):
    def __init__(self, dim: int, device, eps: float = 1e-5):
        self.eps = eps
        self.gamma = _param(np.ones(dim), device)
        self.beta = _param(np.zeros(dim), device)

    def forward(self, x: Value) -> Value:
        return F.layernorm(x, self.gamma, self.beta, self.eps)

    def named_parameters(self):
        return [("gamma", self.gamma), ("beta", self.beta)]


class Embedding(Module):
    def __init__(self, num: int, dim: int, rng: np.random.Generator, device):
        lim = 1.0 / math.sqrt(dim)
        self.weight = _param(rng.uniform(-lim, lim, (num, dim)), device)

    def forward(self, ids: torch.Tensor) -> Value:
        return F.embedding(self.weight, ids)

    def named_parameters(self):
        return [("weight", self.weight)]


def sinusoidal_table(max_len: int, dim: int) -> np.ndarray:
    """positional.cpp:15-24: angle = pos / 10000^((c - c%2)/dim), sin on even c, cos on odd, in double."""
    t = np.zeros((max_len, dim), np.float32)
    for pos in range(max_len):
        for c in range(dim):
            angle = float(pos) / math.pow(10000.0, float(c - c % 2) / float(dim))
            t[pos, c] = math.sin(angle) if c % 2 == 0 else math.cos(angle)
    return t


class PositionalEncoding(Module):
    def __init__(self, max_len: int, dim: int, device):
        self.max_len, self.dim = max_len, dim
        self.pe = Value.leaf(torch.from_numpy(sinusoidal_table(max_len, dim)).to(device), False)

    def forward(self, x: Value) -> Value:
        if len(x.shape) != 3 or x.shape[1] > self.max_len or x.shape[2] != self.dim:
            raise ValueError("PositionalEncoding: bad input shape")
        return F.add(x, Value.leaf(self.pe.data[: x.shape[1]], False))


class Dropout(Module):
    """Inverted dropout (src/nn/dropout.cpp): in training mode each element is zeroed with probability
    p and the rest scaled by 1 / (1 - p); identity in evaluation mode or for p == 0. The layer takes
    the next "dropout" stream at construction (so layers built in the reference's order after the
    same manual_seed draw its masks) and keeps the generator on the device."""

    def __init__(self, p: float = 0.5, device=None):
        if not (0.0 <= p <= 1.0):
            raise ValueError("Dropout: p must be in [0, 1]")
        self.p = p
        self.state = nnb_random.device_generator("dropout", device or torch.device("cuda", torch.cuda.current_device()))

    def active(self) -> bool:
        return self.training and self.p > 0.0

    def forward(self, x: Value) -> Value:
        return F.dropout(x, self.p, self.state) if self.active() else x


class MultiHeadAttention(Module):
    """Multi-head attention (src/nn/attention.cpp). Without active dropout the core is one op (the
    fused kernels for head size 64); with it, the composed path with dropout on the weights."""

    def __init__(self, dim: int, heads: int, causal: bool, rng, device, dropout: float = 0.0):
        if heads == 0 or dim % heads:
            raise ValueError("MultiHeadAttention: dim must be divisible by heads")
        self.dim, self.heads, self.causal = dim, heads, causal
        self.q = Linear(dim, dim, rng, device)
        self.k = Linear(dim, dim, rng, device)
        self.v = Linear(dim, dim, rng, device)
        self.o = Linear(dim, dim, rng, device)
        self.drop = Dropout(dropout, device)

    def forward(self, x: Value) -> Value:
        return self.attend(x, x)

    def attend(self, query: Value, context: Value, key_padding_mask: torch.Tensor | None = None) -> Value:
        """attention.cpp:22-48: queries from `query`, keys and values from `context`."""
        qs, cs = query.shape, context.shape
        if len(qs) != 3 or len(cs) != 3 or qs[2] != self.dim or cs[2] != self.dim or qs[0] != cs[0]:
            raise TensorShapeError("MultiHeadAttention: bad input shapes")
        if query is context:   # self-attention: the three projections share their input
            q, k, v = F.linear_multi(query, [(m.weight, m.bias) for m in (self.q, self.k, self.v)])
        else:
            q, k, v = self.q(query), self.k(context), self.v(context)
        if not self.drop.active():
            return self.o(F.attention(q, k, v, self.heads, key_padding_mask, self.causal))
        return self.o(F.attention_dropout(q, k, v, self.heads, key_padding_mask, self.causal, self.drop.p,
                                          self.drop.state))

    def named_parameters(self):
        out = []
        for name, m in (("q.", self.q), ("k.", self.k), ("v.", self.v), ("o.", self.o)):
            out += [(name + n, p) for n, p in m.named_parameters()]
        return out


class TransformerBlock(Module):
    """x + attn(ln1(x)), then + drop(fc2(gelu(fc1(ln2(.))))) (transformer.cpp:41-44); fc1 + gelu run as
    one GEMM with the GELU in its epilogue. The attention's and the block's Dropout layers are built
    in the reference's member order (attention first), so their streams match its own."""

    def __init__(self, dim: int, heads: int, mlp_ratio: int, causal: bool, rng, device, dropout: float = 0.0):
        self.ln1 = LayerNorm(dim, device)
        self.attn = MultiHeadAttention(dim, heads, causal, rng, device, dropout)
        self.ln2 = LayerNorm(dim, device)
        self.fc1 = Linear(dim, mlp_ratio * dim, rng, device)
        self.fc2 = Linear(mlp_ratio * dim, dim, rng, device)
        self.drop = Dropout(dropout, device)

    def forward(self, x: Value) -> Value:
        h = F.add(x, self.attn(self.ln1(x)))
        return F.add(h, self.drop(self.fc2(F.linear_gelu(self.ln2(h), self.fc1.weight, self.fc1.bias))))

    def named_parameters(self):
        out = []
        for name, m in (("ln1.", self.ln1), ("attn.", self.attn), ("ln2.", self.ln2), ("fc1.", self.fc1),
                        ("fc2.", self.fc2)):
            out += [(name + n, p) for n, p in m.named_parameters()]
        return out


@dataclass
class TransformerConfig:
    """include/nn/nn/transformer.hpp:36-46 (sinusoidal positions)."""
    vocab_size: int
    dim: int
    heads: int
    layers: int
    max_len: int
    mlp_ratio: int = 4
    dropout: float = 0.0
    causal: bool = True


class Transformer(Module):
    def __init__(self, c: TransformerConfig, seed: int = 0, device=None):
        if c.dim == 0 or c.heads == 0 or c.mlp_ratio == 0 or c.dim % c.heads:
            raise ValueError("Transformer: dim must be non-zero and divisible by heads")
        if c.vocab_size == 0 or c.layers == 0 or c.max_len == 0:
            raise ValueError("Transformer: sizes must be non-zero")
        device = device or torch.device("cuda", torch.cuda.current_device())
        rng = np.random.default_rng(seed)
        self.config = c
        self.embed = Embedding(c.vocab_size, c.dim, rng, device)
        self.pos = PositionalEncoding(c.max_len, c.dim, device)
        self.blocks = [TransformerBlock(c.dim, c.heads, c.mlp_ratio, c.causal, rng, device, c.dropout)
                       for _ in range(c.layers)]
        self.ln_f = LayerNorm(c.dim, device)
        self.head = Linear(c.dim, c.vocab_size, rng, device)

    def forward(self, ids: torch.Tensor) -> Value:
        h = self.pos(self.embed(ids))
        for b in self.blocks:
            h = b(h)
        return self.head(self.ln_f(h))

    def named_parameters(self):
        out = [("embed." + n, p) for n, p in self.embed.named_parameters()]
        for i, b in enumerate(self.blocks):
            out += [(f"blocks.{i}." + n, p) for n, p in b.named_parameters()]
        out += [("ln_f." + n, p) for n, p in self.ln_f.named_parameters()]
        out += [("head." + n, p) for n, p in self.head.named_parameters()]
        return out


class Conv2d(Module):
    """conv2d layer (src/nn/conv2d.cpp; conv2d.hpp:37-72): k an int (square) or (kh, kw); weight
    [cout, cin/groups, kh, kw] ~ U(+-1/sqrt(cin/groups * kh * kw)), zero bias."""

    def __init__(self, cin: int, cout: int, k, stride: int, padding: int, rng, device, dilation: int = 1,
                 groups: int = 1):
        kh, kw = (k, k) if isinstance(k, int) else k
        if dilation <= 0 or groups <= 0 or cin % groups or cout % groups:
            raise ValueError("Conv2d: bad dilation / groups")
        lim = 1.0 / math.sqrt((cin // groups) * kh * kw)
        self.stride, self.padding, self.dilation, self.groups = stride, padding, dilation, groups
        self.weight = _param(rng.uniform(-lim, lim, (cout, cin // groups, kh, kw)), device)
        self.bias = _param(np.zeros(cout), device)

    @property
    def can_fuse_relu(self) -> bool:
        return self.dilation == 1 and self.groups == 1               # conv2d.hpp:72

    def forward(self, x: Value) -> Value:
        return F.conv2d(x, self.weight, self.bias, self.stride, self.padding, dilation=self.dilation,
                        groups=self.groups)

    def forward_relu(self, x: Value) -> Value:
        return F.conv2d_relu(x, self.weight, self.bias, self.stride, self.padding)

    def named_parameters(self):
        return [("weight", self.weight), ("bias", self.bias)]


class _BatchNorm(Module):
    """Batch normalisation (src/nn/batchnorm.cpp): training mode normalises with the batch statistics
    and updates running_mean / running_var (momentum, unbiased variance); evaluation mode uses the
    running statistics. A following ReLU folds into the op in training mode only (batchnorm.hpp:50)."""

    rank = 0

    def __init__(self, num_features: int, device, eps: float = 1e-5, momentum: float = 0.1):
        self.num_features, self.eps, self.momentum = num_features, eps, momentum
        self.weight = _param(np.ones(num_features), device)
        self.bias = _param(np.zeros(num_features), device)
        self.running_mean = torch.zeros(num_features, device=device)
        self.running_var = torch.ones(num_features, device=device)
        self.training = True

    def train(self, mode: bool = True):
        self.training = mode
        return self

    def eval(self):
        return self.train(False)

    @property
    def can_fuse_relu(self) -> bool:
        return self.training

    def forward(self, x: Value) -> Value:
        return self._run(x, False)

    def forward_relu(self, x: Value) -> Value:
        return self._run(x, True)

    def _run(self, x: Value, fuse_relu: bool) -> Value:
        if len(x.shape) != self.rank or x.shape[1] != self.num_features:
            raise TensorShapeError("BatchNorm: input shape does not match the layer")
        if self.training:
            C = self.num_features
            mu, var = torch.empty(C, device=x.data.device), torch.empty(C, device=x.data.device)
            out = F.batchnorm(x, self.weight, self.bias, self.eps, fuse_relu, mean_out=mu, var_out=var)
            count = x.data.numel() // C
            check(lib().nnb_batchnorm_running_update(torch.cuda.current_stream().cuda_stream, C, count, mu.data_ptr(),
                                                     var.data_ptr(), ctypes.c_float(self.momentum),
                                                     self.running_mean.data_ptr(), self.running_var.data_ptr()))
            return out
        return F.batchnorm_eval(x, self.weight, self.bias, self.running_mean, self.running_var, self.eps, fuse_relu)

    def named_parameters(self):
        return [("weight", self.weight), ("bias", self.bias)]

    def named_buffers(self):
        return [("running_mean", self.running_mean), ("running_var", self.running_var)]


class BatchNorm1d(_BatchNorm):
    rank = 2


class BatchNorm2d(_BatchNorm):
    rank = 4


class ReLU(Module):
    def forward(self, x):
        return F.relu(x)


class MaxPool2d(Module):
    def __init__(self, k: int, stride: int):
        self.k, self.stride = k, stride

    def forward(self, x):
        return F.maxpool2d(x, self.k, self.stride)


class Flatten(Module):
    def forward(self, x):
        return F.reshape(x, (x.shape[0], int(np.prod(x.shape[1:]))))


class AvgPool2d(Module):
    def __init__(self, k: int, stride: int):
        self.k, self.stride = k, stride

    def forward(self, x):
        return F.avgpool2d(x, self.k, self.stride)


class GlobalAvgPool2d(Module):
    """mean over W then H (pool2d.cpp:20-23): [N, C, H, W] -> [N, C]."""

    def forward(self, x):
        if len(x.shape) != 4:
            raise TensorShapeError("GlobalAvgPool2d: needs a 4-D input")
        return F.mean(F.mean(x, 3), 2)


class Sequential(Module):
    """Runs layers in order; a layer that can fold a following ReLU (Conv2d without dilation / groups,
    BatchNorm in training mode) runs both as one op (sequential.cpp:16-28)."""

    def __init__(self, *layers):
        self.layers = list(layers)

    def forward(self, x):
        i = 0
        while i < len(self.layers):
            layer = self.layers[i]
            if getattr(layer, "can_fuse_relu", False) and i + 1 < len(self.layers) and \
                    isinstance(self.layers[i + 1], ReLU):
                x = layer.forward_relu(x)
                i += 2
                continue
            x = layer(x)
            i += 1
        return x

    def train(self, mode: bool = True):
        for layer in self.layers:
            if hasattr(layer, "train"):
                layer.train(mode)
        return self

    def eval(self):
        return self.train(False)

    def named_parameters(self):
        out = []
        for i, layer in enumerate(self.layers):
            out += [(f"{i}.{n}", p) for n, p in layer.named_parameters()]
        return out

    def named_buffers(self):
        out = []
        for i, layer in enumerate(self.layers):
            if hasattr(layer, "named_buffers"):
                out += [(f"{i}.{n}", b) for n, b in layer.named_buffers()]
        return out


class AdamW:
    """Decoupled weight decay then Adam (src/optim/adamw.cpp:15-24, src/optim/adam.cpp:24-43), one
    fused kernel per parameter; the moment buffers start at zero."""

    def __init__(self, params, lr=1e-3, beta1=0.9, beta2=0.999, eps=1e-8, weight_decay=1e-2):
        self.params = list(params)
        self.lr, self.beta1, self.beta2, self.eps, self.weight_decay = lr, beta1, beta2, eps, weight_decay
        s = torch.cuda.current_stream().cuda_stream
        self.m, self.v = [], []
        for p in self.params:
            for buf in (self.m, self.v):
                t = torch.empty_like(p.data)
                check(lib().nnb_fill(s, t.numel(), 0.0, t.data_ptr()))
                buf.append(t)
        self.t = 0

    def zero_grad(self):
        for p in self.params:
            p.zero_grad()

    # -- checkpoint state (src/optim/adam.cpp:46-71; AdamW has the same entries) -------------------
    def state(self) -> list[tuple[str, torch.Tensor]]:
        dev = self.m[0].device if self.m else torch.device("cpu")
        out = [(n, torch.tensor([v], dtype=torch.float32, device=dev))
               for n, v in (("lr", self.lr), ("beta1", self.beta1), ("beta2", self.beta2), ("eps", self.eps),
                            ("t", float(self.t)))]
        out += [(f"m.{i}", m) for i, m in enumerate(self.m)]
        out += [(f"v.{i}", v) for i, v in enumerate(self.v)]
        return out

    def load_state(self, snapshot) -> None:
        """All or nothing: every entry of state() with its shape, nothing else ("lr" may be absent,
        the current one is kept), as Optimizer::check_state (src/optim/sgd.cpp:27-49)."""
        got = dict(snapshot)
        if len(got) != len(snapshot):
            raise RuntimeError("optimizer state mismatch: duplicate entries")
        if "lr" not in got:
            got["lr"] = np.array([self.lr], np.float32)
        want = self.state()
        problems = ""
        for name, t in want:
            if name not in got:
                problems += " missing:" + name
            elif tuple(np.shape(got[name])) != tuple(t.shape):
                problems += " shape-mismatch:" + name
        names = {n for n, _ in want}
        problems += "".join(" unexpected:" + n for n in got if n not in names)
        if problems:
            raise RuntimeError("optimizer state mismatch:" + problems)
        val = lambda n: float(np.asarray(got[n], np.float32).reshape(-1)[0])
        self.lr, self.beta1, self.beta2, self.eps = val("lr"), val("beta1"), val("beta2"), val("eps")
        self.t = int(val("t"))
        for i, (m, v) in enumerate(zip(self.m, self.v)):
            m.copy_(torch.as_tensor(np.asarray(got[f"m.{i}"], np.float32)).to(m.device))
            v.copy_(torch.as_tensor(np.asarray(got[f"v.{i}"], np.float32)).to(v.device))

    def step(self):
        import ctypes
        self.t += 1
        s = torch.cuda.current_stream().cuda_stream
        for p, m, v in zip(self.params, self.m, self.v):
            if p.grad_fresh:     # nothing reached this parameter: its gradient is all zeros
                check(lib().nnb_fill(s, p.grad.numel(), 0.0, p.grad.data_ptr()))
                p.grad_fresh = False
            check(lib().nnb_adamw_step(s, p.data.numel(), p.data.data_ptr(), p.grad.data_ptr(), m.data_ptr(),
                                       v.data_ptr(), ctypes.c_float(self.lr), ctypes.c_float(self.beta1),
                                       ctypes.c_float(self.beta2), ctypes.c_float(self.eps),
                                       ctypes.c_float(self.weight_decay), self.t))
