"""Data-parallel training step whose result does not depend on the number of GPUs.

The global batch is cut into a fixed number of virtual shards S (8 for the 64-sequence config).
Each rank runs ONE forward and backward over the sequences of the shards it owns, with every
parameter-gradient op writing one gradient per shard (the *_grouped entry points: per-shard weight
gradients as one batched GEMM, per-shard bias / LayerNorm / embedding sums). The [S_local, P]
shard gradients are all-gathered (NCCL over NVLink, one collective per step) into [S, P], and every
rank sums the S rows in shard order 0, 1, ..., S-1 with one kernel (a serial sum from +0 per
element) before the identical AdamW step.

Every shard's arithmetic is independent of how many GPUs there are (a row's result never depends on
how many rows a kernel processes, and the per-shard sums run over the shard's own rows), and so is
the order of the final sum: the weights after a step are bitwise identical at 1, 2, 4 or 8 GPUs.
The reference has no distributed training; its guarantee is the same independence from the thread
count (tests/test_transformer.cpp:525).

The loss gradient is normalised by the global number of positions (grad_norm), so the update is
the one of the mean loss over the global batch.
"""
from __future__ import annotations

import torch

from . import check, lib
from . import functional as F
from .autograd import empty


class ShardedTrainer:
    def __init__(self, model, optimizer, shards: int = 8, world: int = 1, rank: int = 0, group=None):
        if shards % world:
            raise ValueError("the virtual shard count must be a multiple of the number of ranks")
        self.model, self.opt = model, optimizer
        self.shards, self.world, self.rank, self.group = shards, world, rank, group
        self.owned = list(range(rank * shards // world, (rank + 1) * shards // world))
        self.params = model.parameters()
        self.sizes = [p.data.numel() for p in self.params]
        self.total = sum(self.sizes)
        dev = self.params[0].data.device
        self.shard_grads = empty((len(self.owned), self.total), device=dev)
        self.all_grads = self.shard_grads if world == 1 else empty((shards, self.total), device=dev)
        self.reduced = empty((self.total,), device=dev)
        self.grad_norm = None
        self.local_loss = empty((1,), device=dev)
        self.all_loss = self.local_loss if world == 1 else empty((world,), device=dev)
        self.loss = empty((1,), device=dev)

    def _point_grads(self, flat: torch.Tensor) -> None:
        """Parameter gradients as views of `flat` ([P] or per-shard [S_local, P])."""
        off = 0
        for p, n in zip(self.params, self.sizes):
            p.grad = flat[..., off: off + n] if flat.dim() == 2 else flat[off: off + n].view(p.data.shape)
            p.grad_fresh = True
            off += n

    def step(self, ids: torch.Tensor, targets: torch.Tensor) -> torch.Tensor:
        """One step on the global batch ids/targets [B, T] (device int64); returns the mean loss
        over the global batch (a device scalar)."""
        B, T = ids.shape
        per = B // self.shards
        lo, hi = self.owned[0] * per, (self.owned[-1] + 1) * per
        s = torch.cuda.current_stream().cuda_stream
        if self.grad_norm is None:
            self.grad_norm = torch.tensor([1.0 / (B * T)], dtype=torch.float32, device=ids.device)
        self._point_grads(self.shard_grads)
        groups = len(self.owned)
        with F.param_groups(groups):
            logits = self.model(ids[lo:hi])
            loss = F.sequence_cross_entropy(logits, targets[lo:hi], grad_norm=self.grad_norm)
            loss.backward()
        if any(p.grad_fresh for p in self.params):
            raise RuntimeError("a parameter received no gradient")
        check(lib().nnb_accumulate(s, 1, loss.data.data_ptr(), self.local_loss.data_ptr(), 1, 0))
        if self.world > 1:
            import torch.distributed as dist
            dist.all_gather_into_tensor(self.all_grads, self.shard_grads, group=self.group)
            dist.all_gather_into_tensor(self.all_loss, self.local_loss, group=self.group)
        check(lib().nnb_column_sum(s, self.shards, self.total, self.all_grads.data_ptr(), self.reduced.data_ptr(), 1))
        self._point_grads(self.reduced)
        for p in self.params:
            p.grad_fresh = False
        self.opt.step()
        # mean loss over ranks (each rank's loss is the mean over its equal share of positions)
        check(lib().nnb_column_sum(s, self.world, 1, self.all_loss.data_ptr(), self.loss.data_ptr(), 1))
        check(lib().nnb_scale(s, 1, 1.0 / self.world, self.loss.data_ptr(), self.loss.data_ptr()))
        return self.loss
