"""Device-resident autograd values, mirroring nn::Value (include/nn/autograd/value.hpp:74-228,
src/autograd/value.cpp).

A Value holds its data (a CUDA tensor used as a plain buffer) and a gradient buffer. The
gradient convention is the reference's grad_accum (value.cpp:60-64): a buffer that nothing has
written yet is "fresh", and the first backward rule that reaches it STORES its contribution;
later rules ADD. Every op's backward passes that `first` flag straight to the C ABI, so no
gradient buffer is ever zero-filled. backward() orders the graph with the reference's iterative
post-order DFS (value.cpp:80-132), seeds the root's gradient with 1 and runs the rules in reverse
topological order.

torch provides allocation and streams only; every number is produced by a kernel of libnnb.so.
"""
from __future__ import annotations

from typing import Callable, Sequence

import torch


def empty(shape, dtype=torch.float32, device=None):
    """An uninitialised device buffer (plumbing: no kernel runs)."""
    return torch.empty(tuple(shape), dtype=dtype, device=device or torch.device("cuda", torch.cuda.current_device()))


_ONES: dict = {}


def _one(device) -> torch.Tensor:
    """A device scalar 1.0 (uploaded once per device; the seed of backward())."""
    key = str(device)
    if key not in _ONES:
        _ONES[key] = torch.tensor([1.0], dtype=torch.float32, device=device)
    return _ONES[key]


class Value:
    __slots__ = ("data", "grad", "grad_fresh", "requires_grad", "parents", "backward_fn", "name")

    def __init__(self, data: torch.Tensor, requires_grad: bool = False, parents: Sequence["Value"] = (),
                 backward_fn: Callable[[torch.Tensor], None] | None = None):
        self.data = data
        self.grad: torch.Tensor | None = None
        self.grad_fresh = False
        self.requires_grad = requires_grad
        self.parents = tuple(parents)
        self.backward_fn = backward_fn
        self.name = ""

    # -- construction (value.cpp:26-45) --------------------------------------------------------
    @staticmethod
    def leaf(data: torch.Tensor, requires_grad: bool = False) -> "Value":
        v = Value(data, requires_grad)
        if requires_grad:
            v.grad = torch.empty_like(data)
            v.grad_fresh = True          # stands for zeros until the first write
        return v

    @staticmethod
    def node(data: torch.Tensor, parents: Sequence["Value"], backward_fn) -> "Value":
        if not any(p.requires_grad for p in parents):
            return Value(data, False)
        return Value(data, True, parents, backward_fn)

    # -- gradient access -----------------------------------------------------------------------
    def grad_accum(self) -> tuple[torch.Tensor, int]:
        """The gradient buffer and whether this contribution is the first (store) or not (add).

        A parameter's buffer may be a per-group view set by the data-parallel step (nnb.train); it is
        used as given."""
        if self.grad is None:
            self.grad = torch.empty_like(self.data)
            self.grad_fresh = True
        first = 1 if self.grad_fresh else 0
        self.grad_fresh = False
        return self.grad, first

    def zero_grad(self) -> None:
        """Marks the gradient as all zeros without writing it (value.cpp:69-76)."""
        if self.grad is None or self.grad.shape != self.data.shape:
            self.grad = torch.empty_like(self.data)
        self.grad_fresh = True

    @property
    def shape(self):
        return tuple(self.data.shape)

    # -- backward (value.cpp:80-132) -----------------------------------------------------------
    def backward(self, seed: torch.Tensor | None = None) -> None:
        """Runs the backward rules; the root's gradient is 1, or `seed` (a device tensor with the
        root's element count: an upstream gradient, which lets a non-scalar root be differentiated
        as the reference's tests do with sum(y * g))."""
        if seed is None and self.data.numel() != 1:
            raise ValueError("backward() needs a single-element value (AutogradShapeError)")
        if seed is not None and seed.numel() != self.data.numel():
            raise ValueError("backward(): the seed must have the root's element count")
        topo: list[Value] = []
        expanded, done = set(), set()
        stack = [self]
        while stack:
            v = stack[-1]
            if id(v) in done:
                stack.pop()
                continue
            if id(v) in expanded:
                stack.pop()
                done.add(id(v))
                topo.append(v)
                continue
            expanded.add(id(v))
            for p in v.parents:
                if id(p) not in expanded:
                    stack.append(p)
        for v in topo:
            if v.backward_fn is not None:
                if v.grad is None or v.grad.shape != v.data.shape:
                    v.grad = torch.empty_like(v.data)
                v.grad_fresh = True
        self.grad = (_one(self.data.device) if seed is None else seed).view(self.data.shape)
        self.grad_fresh = False
        for v in reversed(topo):
            if v.backward_fn is not None:
                v.backward_fn(v.grad)
