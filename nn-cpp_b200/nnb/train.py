"""Data-parallel training step whose result does not depend on the number of GPUs.

The global batch is cut into a fixed number of virtual shards (8 for the 64-sequence config). Each
rank owns a contiguous range of shards and runs forward + backward once per owned shard, writing
that shard's gradients into a buffer of its own (the parameters' gradient views point into it, and
every parameter is STORED, never accumulated, by the shard's backward). The shard gradients are
then all-gathered (NCCL over NVLink, one collective per step) and every rank sums them in shard
order 0, 1, ..., S-1 with one kernel (nnb_column_sum over S rows: a serial sum from +0 in row order)
before the identical AdamW step. Every shard's arithmetic is the same whatever the number of GPUs,
and so is the order of the final sum, hence the weights after a step are bitwise identical at 1, 2,
4 or 8 GPUs. (The reference has no distributed training; its guarantee is the same independence
from the thread count, tests/test_transformer.cpp:525.)

Each shard's loss is seeded with 1/S, so the update equals that of the mean loss over the global
batch.
"""
from __future__ import annotations

import ctypes

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
        self.seed = torch.tensor([1.0 / shards], dtype=torch.float32, device=dev)
        self.shard_loss = empty((len(self.owned),), device=dev)
        self.all_loss = self.shard_loss if world == 1 else empty((shards,), device=dev)
        self.loss = empty((1,), device=dev)

    def _point_grads(self, flat: torch.Tensor) -> None:
        off = 0
        for p, n in zip(self.params, self.sizes):
            p.grad = flat[off: off + n].view(p.data.shape)
            p.grad_fresh = True
            off += n

    def step(self, ids: torch.Tensor, targets: torch.Tensor) -> torch.Tensor:
        """One step on the global batch ids/targets [B, T] (device int64); returns the mean loss
        (a device scalar)."""
        B = ids.shape[0]
        per = B // self.shards
        s = torch.cuda.current_stream().cuda_stream
        for j, sh in enumerate(self.owned):
            self._point_grads(self.shard_grads[j])
            rows = slice(sh * per, (sh + 1) * per)
            logits = self.model(ids[rows])
            loss = F.sequence_cross_entropy(logits, targets[rows])
            loss.backward(self.seed)
            check(lib().nnb_accumulate(s, 1, loss.data.data_ptr(), self.shard_loss[j:j + 1].data_ptr(), 1, 0))
            for p in self.params:
                if p.grad_fresh:      # a parameter no rule reached has a zero gradient
                    check(lib().nnb_fill(s, p.grad.numel(), 0.0, p.grad.data_ptr()))
                    p.grad_fresh = False
        if self.world > 1:
            import torch.distributed as dist
            dist.all_gather_into_tensor(self.all_grads, self.shard_grads, group=self.group)
            dist.all_gather_into_tensor(self.all_loss, self.shard_loss, group=self.group)
        check(lib().nnb_column_sum(s, self.shards, self.total, self.all_grads.data_ptr(), self.reduced.data_ptr(), 1))
        self._point_grads(self.reduced)
        for p in self.params:
            p.grad_fresh = False
        self.opt.step()
        # mean loss: sum of the shard losses (in shard order) times 1/S
        check(lib().nnb_column_sum(s, self.shards, 1, self.all_loss.data_ptr(), self.loss.data_ptr(), 1))
        return self.loss
