"""Datasets and the DataLoader (include/nn/data/dataloader.hpp, dataset.hpp, tensor_dataset.hpp,
subset.hpp, text.hpp; src/data/*.cpp).

The sample ORDER is the reference's, drawn on the host by libnnb exactly as the reference draws it:
each DataLoader takes the next "dataloader" stream at construction (nnb.random), reshuffles with the
portable Fisher-Yates of src/data/shuffle.hpp or redraws a weighted epoch (dataloader.cpp:58-73) in
reset_epoch(), and random_split seeds its own mt19937 from the folded 64-bit seed. So after the same
manual_seed the loaders visit the same samples in the same batches.

Batch ASSEMBLY is B200-side:
- TensorDataset and SequenceDataset (and Subsets of them) are uploaded to HBM once; the epoch's order
  is uploaded once per epoch; each get_batch is one gather launch (nnb_gather_rows /
  nnb_gather_windows) on the current stream: no per-batch host work or host-to-device copy.
- Any other Dataset (a Python object with size() / get(i)) is stacked on the host into one of two
  pinned buffers and copied asynchronously on a separate copy stream; iterating over the loader
  stages batch b + 1 while batch b is being consumed (double buffering), and the consumer's stream
  waits on an event before using a batch.

Batches: get_batch(b) returns (x, y) on the device, x wrapped as a leaf Value (requires_grad False)
like the reference. A SequenceDataset's batches are int64 token ids [B, block] (what nnb's Embedding
takes) where the reference returns float ids.
"""
from __future__ import annotations

import math

import numpy as np
import torch

from . import TensorIndexError, TensorShapeError, check, lib
from . import random as nnb_random
from .autograd import Value


# ---- datasets ------------------------------------------------------------------------------------

class Dataset:
    """size() samples; get(i) -> (input, target) as numpy arrays (dataset.hpp)."""

    def size(self) -> int:
        raise NotImplementedError

    def get(self, index: int):
        raise NotImplementedError

    def __len__(self) -> int:
        return self.size()


class TensorDataset(Dataset):
    """Rows of two arrays with the same leading size (tensor_dataset.hpp); any numpy dtype."""

    def __init__(self, inputs, targets):
        self.inputs, self.targets = np.ascontiguousarray(inputs), np.ascontiguousarray(targets)
        if self.inputs.ndim == 0 or self.targets.ndim == 0 or self.inputs.shape[0] != self.targets.shape[0]:
            raise TensorShapeError("TensorDataset: inputs and targets need the same first dimension")
        self._dev = {}

    def size(self) -> int:
        return self.inputs.shape[0]

    def get(self, index: int):
        if not 0 <= index < self.size():
            raise TensorIndexError("TensorDataset: index out of range")
        return self.inputs[index], self.targets[index]

    def resident(self, device):
        """The two arrays in HBM on `device` (uploaded on first use)."""
        key = str(device)
        if key not in self._dev:
            self._dev[key] = tuple(torch.from_numpy(a).to(device) for a in (self.inputs, self.targets))
        return self._dev[key]


class SequenceDataset(Dataset):
    """Next-token windows over a token stream (text.hpp, text.cpp:48-70): sample i is
    (tokens[i : i + block], tokens[i + 1 : i + 1 + block]); size = len(tokens) - block."""

    def __init__(self, tokens, block_size: int):
        t = np.asarray(tokens)
        if block_size == 0 or t.ndim != 1 or t.size <= block_size:
            raise ValueError("SequenceDataset: need block_size >= 1 and tokens.size() > block_size")
        ids = t.astype(np.int64)
        if (ids != t).any() or ids.min() < 0 or ids.max() >= 2 ** 31:
            raise ValueError("SequenceDataset: tokens must be non-negative integer ids below 2^31")
        self.tokens, self.block_size = ids.astype(np.int32), block_size
        self._dev = {}

    def size(self) -> int:
        return self.tokens.size - self.block_size

    def get(self, index: int):
        if not 0 <= index < self.size():
            raise TensorIndexError("SequenceDataset: index out of range")
        b = self.block_size
        return (self.tokens[index: index + b].astype(np.float32), self.tokens[index + 1: index + 1 + b].astype(np.float32))

    def resident(self, device):
        key = str(device)
        if key not in self._dev:
            self._dev[key] = torch.from_numpy(self.tokens).to(device)
        return self._dev[key]


class CharVocab:
    """Byte-level vocabulary of a text (text.cpp:12-45): ids are the distinct bytes in increasing order."""

    def __init__(self, text: str | bytes):
        data = text.encode("latin-1") if isinstance(text, str) else bytes(text)
        self.chars = bytes(sorted(set(data)))
        self._ids = {c: i for i, c in enumerate(self.chars)}

    def size(self) -> int:
        return len(self.chars)

    def encode(self, s: str | bytes) -> np.ndarray:
        data = s.encode("latin-1") if isinstance(s, str) else bytes(s)
        try:
            return np.array([self._ids[c] for c in data], np.float32)
        except KeyError:
            raise ValueError("CharVocab::encode: character not in vocabulary") from None

    def decode(self, ids) -> str:
        out = bytearray()
        for f in np.asarray(ids, np.float32).ravel():
            if not (0.0 <= f < len(self.chars)) or f != np.floor(f):
                raise ValueError("CharVocab::decode: invalid id")
            out.append(self.chars[int(f)])
        return out.decode("latin-1")


class Subset(Dataset):
    """The samples of `dataset` at `indices`, in that order (subset.hpp, subset.cpp:12-26)."""

    def __init__(self, dataset: Dataset, indices):
        self.dataset = dataset
        self.indices = np.asarray(indices, np.int64).reshape(-1)
        if self.indices.size and (self.indices.min() < 0 or self.indices.max() >= dataset.size()):
            raise TensorIndexError("Subset: index out of range")

    def size(self) -> int:
        return int(self.indices.size)

    def get(self, index: int):
        if not 0 <= index < self.size():
            raise TensorIndexError("Subset: index out of range")
        return self.dataset.get(int(self.indices[index]))


def _mt19937_seeded(seed32: int) -> np.ndarray:
    state = np.zeros(nnb_random.STATE_WORDS, np.uint32)
    check(lib().nnb_mt19937_seed(seed32 & 0xFFFFFFFF, state.ctypes.data))
    return state


def _shuffle(state: np.ndarray, v: np.ndarray) -> None:
    """portable_shuffle (shuffle.hpp:45-49) in place on a uint64 array."""
    check(lib().nnb_portable_shuffle(state.ctypes.data, v.ctypes.data, v.size))


def random_split(dataset: Dataset, fractions, seed: int) -> list[Subset]:
    """subset.cpp:28-82: sizes floor(f * n) with the remainder on the last non-empty split, order from a
    portable shuffle seeded by (seed & 0xffffffff) ^ (seed >> 32)."""
    fractions = list(fractions)
    if not fractions:
        raise ValueError("random_split: no fractions given")
    total = 0.0
    for f in fractions:
        if not f > 0.0:
            raise ValueError("random_split: fractions must be positive")
        total += f
    if abs(total - 1.0) > 1e-9:
        raise ValueError("random_split: fractions must sum to 1")
    n = dataset.size()
    sizes = [int(math.floor(f * float(n))) for f in fractions]
    assigned = sum(sizes)
    if assigned > n:
        raise ValueError("random_split: fractions exceed the dataset size")
    last = len(sizes) - 1
    while last > 0 and sizes[last] == 0:
        last -= 1
    sizes[last] += n - assigned
    if any(s == 0 for s in sizes):
        raise ValueError("random_split: a split would be empty")
    order = np.arange(n, dtype=np.uint64)
    seed &= 0xFFFFFFFFFFFFFFFF
    _shuffle(_mt19937_seeded((seed & 0xFFFFFFFF) ^ (seed >> 32)), order)
    out, pos = [], 0
    for s in sizes:
        out.append(Subset(dataset, order[pos: pos + s].astype(np.int64)))
        pos += s
    return out


def balanced_sample_weights(labels, num_classes: int) -> np.ndarray:
    """Weight 1 / count(class) per sample (dataloader.cpp:98-106)."""
    labels = np.asarray(labels, np.int64).reshape(-1)
    if labels.size and (labels.min() < 0 or labels.max() >= num_classes):
        raise ValueError("balanced_sample_weights: label out of range")
    counts = np.bincount(labels, minlength=num_classes)
    return 1.0 / counts[labels].astype(np.float64)


# ---- the loader ----------------------------------------------------------------------------------

def _resident_base(dataset: Dataset):
    """(base dataset held in HBM, index map or None) for TensorDataset / SequenceDataset and Subsets of
    them; None for any other dataset."""
    index_map = None
    while isinstance(dataset, Subset):
        index_map = dataset.indices if index_map is None else dataset.indices[index_map]
        dataset = dataset.dataset
    if isinstance(dataset, (TensorDataset, SequenceDataset)):
        return dataset, index_map
    return None


class _Staged:
    __slots__ = ("x", "y", "event")

    def __init__(self, x, y, event):
        self.x, self.y, self.event = x, y, event


class DataLoader:
    """Batches over a Dataset (dataloader.hpp / dataloader.cpp).

    DataLoader(dataset, batch_size, shuffle=False, drop_last=False), or the weighted form
    DataLoader(dataset, batch_size, sample_weights=w, num_samples=0, drop_last=False): each epoch
    draws num_samples (0: the dataset size) samples with replacement in proportion to w.
    """

    def __init__(self, dataset: Dataset, batch_size: int, shuffle: bool = False, drop_last: bool = False, *,
                 sample_weights=None, num_samples: int = 0, device=None):
        if isinstance(num_samples, bool):
            raise TypeError("DataLoader: num_samples is a count, not a flag")
        if batch_size == 0:
            raise TensorShapeError("DataLoader: batch_size must be positive")
        self.dataset, self.batch_size, self.drop_last = dataset, int(batch_size), bool(drop_last)
        self.device = device or torch.device("cuda", torch.cuda.current_device())
        self.state = nnb_random.derive_generator("dataloader")
        n = dataset.size()
        self.cumulative = None
        if sample_weights is not None:
            w = np.asarray(sample_weights, np.float64).reshape(-1)
            if w.size != n:
                raise ValueError("DataLoader: need one sample weight per dataset sample")
            if not np.isfinite(w).all() or (w < 0).any():
                raise ValueError("DataLoader: sample weights must be finite and non-negative")
            self.cumulative = np.cumsum(w)         # running sums in sample order, in double
            if not self.cumulative[-1] > 0.0:
                raise ValueError("DataLoader: sample weights sum to zero")
            self.shuffle, self.num_samples = False, int(num_samples) if num_samples else n
        else:
            self.shuffle, self.num_samples = bool(shuffle), n
        self.indices = np.arange(n, dtype=np.uint64)
        self._resident = _resident_base(dataset)
        self._dev_indices = None
        self._copy_stream, self._pinned, self._events = None, [None, None], [None, None]
        self.reset_epoch()

    def num_batches(self) -> int:
        b = self.batch_size
        return self.num_samples // b if self.drop_last else (self.num_samples + b - 1) // b

    def __len__(self) -> int:
        return self.num_batches()

    def reset_epoch(self) -> None:
        """Reshuffle, or redraw a weighted epoch (dataloader.cpp:58-74); nothing for a plain loader."""
        if self.cumulative is not None:
            self.indices = np.zeros(self.num_samples, np.uint64)
            check(lib().nnb_weighted_draws(self.state.ctypes.data, self.cumulative.ctypes.data, self.cumulative.size,
                                           self.num_samples, self.indices.ctypes.data))
        elif self.shuffle:
            _shuffle(self.state, self.indices)
        self._dev_indices = None

    def epoch_indices(self) -> np.ndarray:
        """This epoch's sample order (host copy)."""
        return self.indices.astype(np.int64)

    def _range(self, b: int):
        if not 0 <= b < self.num_batches():
            raise TensorIndexError("DataLoader: batch index out of range")
        start = b * self.batch_size
        return start, min(start + self.batch_size, self.indices.size)

    def get_batch(self, b: int):
        start, end = self._range(b)
        if self._resident is not None:
            return self._gather(start, end)
        staged = self._stage(b, 0)
        torch.cuda.current_stream().wait_event(staged.event)
        return staged.x, staged.y

    def __iter__(self):
        nb = self.num_batches()
        if self._resident is not None:
            for b in range(nb):
                yield self._gather(*self._range(b))
            return
        nxt = self._stage(0, 0) if nb else None
        for b in range(nb):
            cur = nxt
            if b + 1 < nb:
                nxt = self._stage(b + 1, (b + 1) & 1)     # its copy overlaps the consumer's work on batch b
            torch.cuda.current_stream().wait_event(cur.event)
            yield cur.x, cur.y

    # -- HBM-resident datasets: one gather launch per tensor ----------------------------------------
    def _gather(self, start: int, end: int):
        base, index_map = self._resident
        if self._dev_indices is None:
            idx = self.indices.astype(np.int64)
            if index_map is not None:
                idx = index_map[idx]
            self._dev_indices = torch.from_numpy(idx).to(self.device)          # one upload per epoch
        idx = self._dev_indices[start:end]
        count = end - start
        s = torch.cuda.current_stream().cuda_stream
        if isinstance(base, SequenceDataset):
            tokens = base.resident(self.device)
            x = torch.empty((count, base.block_size), dtype=torch.int64, device=self.device)
            y = torch.empty_like(x)
            check(lib().nnb_gather_windows(s, tokens.data_ptr(), tokens.numel(), idx.data_ptr(), count, base.block_size,
                                           x.data_ptr(), y.data_ptr()))
            return x, y
        inputs, targets = base.resident(self.device)
        out = []
        for src in (inputs, targets):
            dst = torch.empty((count,) + tuple(src.shape[1:]), dtype=src.dtype, device=self.device)
            row_bytes = src[0].numel() * src.element_size() if src.shape[0] else 0
            check(lib().nnb_gather_rows(s, src.data_ptr(), row_bytes, src.shape[0], idx.data_ptr(), count,
                                        dst.data_ptr()))
            out.append(dst)
        return Value.leaf(out[0], False), out[1]

    # -- any other dataset: host stacking into pinned memory, copies on a side stream ---------------
    def _stage(self, b: int, slot: int) -> _Staged:
        start, end = self._range(b)
        xs, ys = zip(*(self.dataset.get(int(i)) for i in self.indices[start:end]))
        x_np, y_np = np.stack([np.asarray(v) for v in xs]), np.stack([np.asarray(v) for v in ys])
        if self._copy_stream is None:
            self._copy_stream = torch.cuda.Stream(self.device)
        if self._events[slot] is not None:
            self._events[slot].synchronize()         # the previous copy out of this slot has finished
        need = x_np.nbytes + y_np.nbytes
        buf = self._pinned[slot]
        if buf is None or buf.numel() < need:
            buf = self._pinned[slot] = torch.empty(max(need, 1), dtype=torch.uint8, pin_memory=True)
        host = buf.numpy()
        hx = host[: x_np.nbytes].view(x_np.dtype).reshape(x_np.shape)
        hy = host[x_np.nbytes: need].view(y_np.dtype).reshape(y_np.shape)
        np.copyto(hx, x_np)
        np.copyto(hy, y_np)
        consumer = torch.cuda.current_stream(self.device)
        with torch.cuda.stream(self._copy_stream):
            xd = torch.from_numpy(hx).to(self.device, non_blocking=True)
            yd = torch.from_numpy(hy).to(self.device, non_blocking=True)
            ev = torch.cuda.Event()
            ev.record(self._copy_stream)
        xd.record_stream(consumer)
        yd.record_stream(consumer)
        self._events[slot] = ev
        return _Staged(Value.leaf(xd, False), yd, ev)
