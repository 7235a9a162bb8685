"""Data-parallel training step whose result does not depend on the number of GPUs.

The global batch is cut into a fixed number of virtual shards S (8 for the 64-sequence config).
Each rank runs ONE forward and backward over the sequences of the shards it owns, with every
parameter-gradient op writing one gradient per shard (the *_grouped entry points: per-shard weight
gradients as one batched GEMM, per-shard bias / LayerNorm / embedding sums), into [S_local, P].

The parameters live in one flat buffer (each parameter a view of it), cut into `world` equal
slices. One NCCL all-to-all gives every rank the S shard gradients of its own slice, in shard order
([S, P/world]); the rank sums those S rows in shard order 0, 1, ..., S-1 (a serial sum from +0 per
element), runs AdamW on its slice (one launch: AdamW is elementwise and its settings are shared by
all parameters), and an in-place all-gather returns the updated slices to every rank. Per step a
rank receives (world-1)/world of S_local x P gradients plus (world-1)/world of P weights, instead of
every shard's full gradient.

Every shard's arithmetic is independent of how many GPUs there are (a row's result never depends on
how many rows a kernel processes, and the per-shard sums run over the shard's own rows), and so are
the order of the final sum and the elementwise update: the weights after a step are bitwise
identical at 1, 2, 4 or 8 GPUs. The reference has no distributed training; its guarantee is the same
independence from the thread count (tests/test_transformer.cpp:525).

The loss gradient is normalised by the global number of positions (grad_norm), so the update is
the one of the mean loss over the global batch. The trainer takes the optimizer's settings and step
counter and performs its update itself (AdamW's per-parameter moment buffers are not used). The step
counter, the settings and Adam's bias corrections (a table computed on the host with the reference's
own formula) live in device memory, so a whole step -- forward, backward, the collectives and the
update -- can be captured once into a CUDA graph and replayed (capture()): no per-launch host work.
"""
from __future__ import annotations

import ctypes

import numpy as np
import torch

from . import check, lib
from . import functional as F
from .autograd import empty


def shard_owners(shards: int, world: int, rank: int) -> list[int]:
    """The virtual shards rank `rank` owns: a contiguous run, equal for every rank, in shard order."""
    if shards % world:
        raise ValueError("the virtual shard count must be a multiple of the number of ranks")
    return list(range(rank * shards // world, (rank + 1) * shards // world))


def exchange_shard_gradients(shard_grads: torch.Tensor, send: torch.Tensor, recv: torch.Tensor, chunk: int,
                             world: int, group=None) -> None:
    """The data-parallel step's one gradient exchange.

    shard_grads [S_local, P]: this rank's per-shard gradients. The flat parameters are cut into
    `world` slices of `chunk` elements (the last one padded). send [world, S_local, chunk] receives
    slice d of every local shard in send[d] (padding left as it is: zero), and one all-to-all leaves in
    recv [S, chunk] every rank's shards of THIS rank's slice, source ranks in order -- which is shard
    order, since each rank owns a contiguous run of shards. Plain tensor copies and one collective:
    it runs on CUDA tensors over NCCL and on CPU tensors over gloo alike."""
    import torch.distributed as dist
    total = shard_grads.shape[1]
    for d in range(world):
        d_lo, d_hi = d * chunk, min(total, (d + 1) * chunk)
        if d_hi > d_lo:
            send[d, :, : d_hi - d_lo].copy_(shard_grads[:, d_lo:d_hi])
    dist.all_to_all_single(recv, send.view(world * shard_grads.shape[0], chunk), group=group)


def gather_weight_slices(flat_w: torch.Tensor, chunk: int, rank: int, group=None) -> None:
    """Every rank's updated slice of the flat parameters back to every rank, in place."""
    import torch.distributed as dist
    dist.all_gather_into_tensor(flat_w, flat_w[rank * chunk:(rank + 1) * chunk], group=group)


class ShardedTrainer:
    def __init__(self, model, optimizer, shards: int = 8, world: int = 1, rank: int = 0, group=None):
        if shards % world:
            raise ValueError("the virtual shard count must be a multiple of the number of ranks")
        self.model, self.opt = model, optimizer
        self.shards, self.world, self.rank, self.group = shards, world, rank, group
        self.owned = shard_owners(shards, world, rank)
        self.params = model.parameters()
        self.sizes = [p.data.numel() for p in self.params]
        self.total = sum(self.sizes)
        dev = self.params[0].data.device
        s = torch.cuda.current_stream(dev).cuda_stream
        # flat parameter storage, padded to `world` equal slices; parameters become views of it
        self.chunk = -(-self.total // world)
        self.flat_w = empty((self.chunk * world,), device=dev)
        check(lib().nnb_fill(s, self.flat_w.numel(), 0.0, self.flat_w.data_ptr()))
        off = 0
        for p, n in zip(self.params, self.sizes):
            view = self.flat_w[off: off + n].view(p.data.shape)
            view.copy_(p.data)
            p.data = view
            off += n
        self.lo = rank * self.chunk
        self.hi = min(self.total, self.lo + self.chunk)
        self.m, self.v = empty((self.chunk,), device=dev), empty((self.chunk,), device=dev)
        for t in (self.m, self.v):
            check(lib().nnb_fill(s, t.numel(), 0.0, t.data_ptr()))
        self.shard_grads = empty((len(self.owned), self.total), device=dev)
        if world > 1:
            self.send = empty((world, len(self.owned), self.chunk), device=dev)
            check(lib().nnb_fill(s, self.send.numel(), 0.0, self.send.data_ptr()))    # padding stays zero
            self.recv = empty((shards, self.chunk), device=dev)
            self.reduced = empty((self.chunk,), device=dev)
        else:
            self.reduced = empty((self.total,), device=dev)
        self.grad_norm = None
        # step counter, settings and bias corrections on the device (graph-replayable update)
        self.step_dev = torch.tensor([int(optimizer.t)], dtype=torch.int64, device=dev)
        self.hyper_dev = empty((5,), device=dev)
        self._hyper_key, self._betas, self.table_dev, self.table_len = None, None, None, 0
        self._refresh_hyper()
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

    def optimizer_to_params(self) -> None:
        """Copies the trainer's moment buffers into the optimizer's per-parameter ones (e.g. before
        a checkpoint is saved); with several ranks every rank gathers the full buffers."""
        self._moments(to_opt=True)

    def optimizer_from_params(self) -> None:
        """The reverse of optimizer_to_params (e.g. after a checkpoint was loaded into the optimizer)."""
        self._moments(to_opt=False)
        self.step_dev.fill_(int(self.opt.t))
        self._refresh_hyper()

    def _refresh_hyper(self) -> None:
        """Copies the optimizer's settings to the device when they changed (outside a captured graph),
        and rebuilds the bias-correction table when the betas changed."""
        o = self.opt
        f = np.float32
        key = (f(o.lr), f(o.beta1), f(o.beta2), f(o.eps), f(o.weight_decay))
        if key == self._hyper_key:
            return
        lr, b1, b2, eps, wd = key
        shrink = f(1.0) - lr * wd                      # float arithmetic, as AdamW::step (adamw.cpp:16)
        self.hyper_dev.copy_(torch.from_numpy(np.array([shrink, lr, b1, b2, eps], np.float32)))
        if (b1, b2) != self._betas:
            for cap in (1 << 16, 1 << 20, 1 << 24):
                table = np.zeros(2 * cap, np.float32)
                n = lib().nnb_adam_bias_table(ctypes.c_float(b1), ctypes.c_float(b2), table.ctypes.data, cap)
                if n < cap or (table[2 * n - 2] == 1.0 and table[2 * n - 1] == 1.0):
                    break
            self.table_dev = torch.from_numpy(table[: 2 * n].copy()).to(self.hyper_dev.device)
            self.table_len, self._betas = n, (b1, b2)
        self._hyper_key = key

    def _moments(self, to_opt: bool) -> None:
        dev = self.m.device
        for mine, theirs in ((self.m, self.opt.m), (self.v, self.opt.v)):
            full = torch.zeros(self.chunk * self.world, device=dev)
            if to_opt:
                if self.world > 1:
                    import torch.distributed as dist
                    dist.all_gather_into_tensor(full, mine, group=self.group)
                else:
                    full[: self.chunk].copy_(mine)
                off = 0
                for t, n in zip(theirs, self.sizes):
                    t.view(-1).copy_(full[off: off + n])
                    off += n
            else:
                off = 0
                for t, n in zip(theirs, self.sizes):
                    full[off: off + n].copy_(t.view(-1))
                    off += n
                mine.copy_(full[self.lo: self.lo + self.chunk])

    def _adamw(self, s, n: int, w_ptr: int, g_ptr: int) -> None:
        check(lib().nnb_adamw_step_device(s, n, w_ptr, g_ptr, self.m.data_ptr(), self.v.data_ptr(),
                                          self.hyper_dev.data_ptr(), self.table_dev.data_ptr(), self.table_len,
                                          self.step_dev.data_ptr()))

    def step(self, ids: torch.Tensor, targets: torch.Tensor) -> torch.Tensor:
        """One step on the global batch ids/targets [B, T] (device int64); returns the mean loss
        over the global batch (a device scalar)."""
        self._refresh_hyper()
        B, T = ids.shape
        per = B // self.shards
        lo, hi = self.owned[0] * per, (self.owned[-1] + 1) * per
        s = torch.cuda.current_stream().cuda_stream
        if self.grad_norm is None:
            self.grad_norm = torch.tensor([1.0 / (B * T)], dtype=torch.float32, device=ids.device)
        self._point_grads(self.shard_grads)
        groups = len(self.owned)
        # with several ranks each dropout mask is this rank's rows of the whole batch's draw
        with F.param_groups(groups), F.batch_slice(B, lo, hi):
            logits = self.model(ids[lo:hi])
            loss = F.sequence_cross_entropy(logits, targets[lo:hi], grad_norm=self.grad_norm)
            loss.backward()
        if any(p.grad_fresh for p in self.params):
            raise RuntimeError("a parameter received no gradient")
        for p in self.params:
            p.grad_fresh = False
        check(lib().nnb_accumulate(s, 1, loss.data.data_ptr(), self.local_loss.data_ptr(), 1, 0))
        self.opt.t += 1
        check(lib().nnb_step_advance(s, self.step_dev.data_ptr()))
        if self.world == 1:
            check(lib().nnb_column_sum(s, self.shards, self.total, self.shard_grads.data_ptr(),
                                       self.reduced.data_ptr(), 1))
            self._adamw(s, self.total, self.flat_w.data_ptr(), self.reduced.data_ptr())
        else:
            import torch.distributed as dist
            exchange_shard_gradients(self.shard_grads, self.send, self.recv, self.chunk, self.world, self.group)
            dist.all_gather_into_tensor(self.all_loss, self.local_loss, group=self.group)
            check(lib().nnb_column_sum(s, self.shards, self.chunk, self.recv.data_ptr(), self.reduced.data_ptr(), 1))
            self._adamw(s, self.hi - self.lo, self.flat_w[self.lo:].data_ptr(), self.reduced.data_ptr())
            gather_weight_slices(self.flat_w, self.chunk, self.rank, self.group)
        # mean loss over ranks (each rank's loss is the mean over its equal share of positions)
        check(lib().nnb_column_sum(s, self.world, 1, self.all_loss.data_ptr(), self.loss.data_ptr(), 1))
        check(lib().nnb_scale(s, 1, 1.0 / self.world, self.loss.data_ptr(), self.loss.data_ptr()))
        return self.loss

    def capture(self, ids: torch.Tensor, targets: torch.Tensor, warmup: int = 2) -> "GraphedTrainStep":
        """Runs `warmup` ordinary steps on (ids, targets), then captures one step into a CUDA graph
        (see GraphedTrainStep). The warm-up steps are real training steps."""
        return GraphedTrainStep(self, ids, targets, warmup)


class GraphedTrainStep:
    """One ShardedTrainer step captured into a CUDA graph, collectives included.

    Calling it copies the batch into the graph's fixed input buffers (when given), refreshes the
    optimizer's settings on the device if they changed, replays the graph and returns the loss
    buffer (a device scalar, valid once the stream reaches it). Every replay is exactly one step: the
    device step counter advances inside the graph and the host mirror (optimizer.t) here.
    """

    def __init__(self, trainer: ShardedTrainer, ids: torch.Tensor, targets: torch.Tensor, warmup: int = 2):
        self.trainer = trainer
        self.ids, self.targets = ids.clone(), targets.clone()
        side = torch.cuda.Stream()
        side.wait_stream(torch.cuda.current_stream())
        with torch.cuda.stream(side):
            for _ in range(max(1, warmup)):
                trainer.step(self.ids, self.targets)
        torch.cuda.current_stream().wait_stream(side)
        torch.cuda.synchronize()
        lib().nnb_trace_enable(0)                 # no event records inside the graph
        t_host = trainer.opt.t
        self.graph = torch.cuda.CUDAGraph()
        with torch.cuda.graph(self.graph, capture_error_mode="thread_local"):
            self.loss = trainer.step(self.ids, self.targets)
        trainer.opt.t = t_host                    # capturing ran nothing
        torch.cuda.synchronize()

    def __call__(self, ids: torch.Tensor | None = None, targets: torch.Tensor | None = None) -> torch.Tensor:
        if ids is not None:
            self.ids.copy_(ids, non_blocking=True)
        if targets is not None:
            self.targets.copy_(targets, non_blocking=True)
        self.trainer._refresh_hyper()
        self.graph.replay()
        self.trainer.opt.t += 1
        return self.loss

    def release(self) -> None:
        """Drops the graph (needed before the process group is destroyed when it holds collectives)."""
        self.graph = None
