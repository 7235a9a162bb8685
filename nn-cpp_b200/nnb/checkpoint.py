"""Checkpoints of a model's parameters / buffers and an optimizer's state, in the reference's
portable binary format (src/checkpoint.cpp; include/nn/checkpoint.hpp), so that files move both
ways between the reference and this build.

Format (little-endian): "NNCK", uint32 version 1, uint32 entry count, then per entry: uint32 name
length, the name bytes, one kind byte (1 = int64 value, 0 = float32 tensor), then the int64 value,
or uint32 rank, rank x uint64 dims and the float32 data. Entries: "model.<name>" for every named
parameter then every named buffer, "optim.<name>" for every optimizer state entry, and "step".
A save goes to path + ".tmp" and is renamed over path; a load validates the whole file against the
model (and optimizer) before it modifies anything.
"""
from __future__ import annotations

import os
import struct

import numpy as np
import torch

MAGIC = b"NNCK"
VERSION = 1
MAX_NAME = 4096
MAX_NDIM = 8


class CheckpointError(RuntimeError):
    """The reference throws std::runtime_error for the same conditions."""


def _encode(entries) -> bytes:
    out = bytearray(MAGIC)
    out += struct.pack("<II", VERSION, len(entries))
    for name, value in entries:
        nb = name.encode()
        out += struct.pack("<I", len(nb)) + nb
        if isinstance(value, int):
            out += b"\x01" + struct.pack("<q", value)
            continue
        arr = np.ascontiguousarray(value, dtype="<f4")
        out += b"\x00" + struct.pack("<I", arr.ndim)
        out += b"".join(struct.pack("<Q", d) for d in arr.shape)
        out += arr.tobytes()
    return bytes(out)


def _decode(data: bytes):
    pos = 0

    def take(n: int) -> bytes:
        nonlocal pos
        if n > len(data) - pos:
            raise CheckpointError("load_checkpoint: unexpected end of file")
        chunk = data[pos:pos + n]
        pos += n
        return chunk

    if take(4) != MAGIC:
        raise CheckpointError("load_checkpoint: not a checkpoint file")
    if struct.unpack("<I", take(4))[0] != VERSION:
        raise CheckpointError("load_checkpoint: unsupported checkpoint version")
    count = struct.unpack("<I", take(4))[0]
    entries, seen = [], set()
    for _ in range(count):
        name_len = struct.unpack("<I", take(4))[0]
        if name_len > MAX_NAME or name_len > len(data) - pos:
            raise CheckpointError("load_checkpoint: bad entry name length")
        name = take(name_len).decode("utf-8", "surrogateescape")     # names are raw bytes in the format
        if name in seen:
            raise CheckpointError("load_checkpoint: duplicate entry " + name)
        seen.add(name)
        kind = take(1)[0]
        if kind == 1:
            entries.append((name, struct.unpack("<q", take(8))[0]))
        elif kind == 0:
            ndim = struct.unpack("<I", take(4))[0]
            if ndim > MAX_NDIM:
                raise CheckpointError("load_checkpoint: bad rank for " + name)
            shape, elems = [], 1
            for _ in range(ndim):
                dim = struct.unpack("<Q", take(8))[0]
                # every element takes 4 file bytes, so the bytes left bound any honest element count
                if dim != 0 and elems > (len(data) - pos) // 4 // dim:
                    raise CheckpointError("load_checkpoint: bad shape for " + name)
                elems *= dim
                shape.append(dim)
            if elems > (len(data) - pos) // 4:
                raise CheckpointError("load_checkpoint: unexpected end of file")
            arr = np.frombuffer(take(elems * 4), dtype="<f4").reshape(shape).astype(np.float32)
            entries.append((name, arr))
        else:
            raise CheckpointError("load_checkpoint: bad entry kind for " + name)
    if pos != len(data):
        raise CheckpointError("load_checkpoint: trailing bytes after last entry")
    return entries


def _buffers(model):
    buffers = model.named_buffers() if hasattr(model, "named_buffers") else []
    names = {n for n, _ in model.named_parameters()}
    for n, _ in buffers:
        if n in names:
            raise CheckpointError("checkpoint: buffer name collides: " + n)
        names.add(n)
    return buffers


def _host(t: torch.Tensor) -> np.ndarray:
    return t.detach().to("cpu", torch.float32).contiguous().numpy()


def save_checkpoint(path: str, model, optimizer=None, step: int = 0) -> None:
    """save_checkpoint (checkpoint.hpp:17-31)."""
    entries = [("model." + n, _host(p.data)) for n, p in model.named_parameters()]
    entries += [("model." + n, _host(b)) for n, b in _buffers(model)]
    if optimizer is not None:
        entries += [("optim." + n, _host(t)) for n, t in optimizer.state()]
    entries.append(("step", int(step)))
    data = _encode(entries)
    tmp = path + ".tmp"
    try:
        with open(tmp, "wb") as f:
            f.write(data)
    except OSError as e:
        _discard(tmp)
        raise CheckpointError("save_checkpoint: cannot write " + tmp) from e
    try:
        os.replace(tmp, path)
    except OSError as e:
        _discard(tmp)
        raise CheckpointError(f"save_checkpoint: cannot replace {path}: {e.strerror}") from e


def _discard(tmp: str) -> None:
    """Removes a partly written temporary file (never a directory that squats on its name)."""
    if os.path.isfile(tmp):
        try:
            os.remove(tmp)
        except OSError:
            pass


def load_checkpoint(path: str, model, optimizer=None) -> int:
    """load_checkpoint (checkpoint.hpp:33-47): returns the stored step."""
    try:
        with open(path, "rb") as f:
            data = f.read()
    except OSError as e:
        raise CheckpointError("load_checkpoint: cannot open " + path) from e
    entries = _decode(data)
    by_name = dict(entries)
    params = model.named_parameters()
    buffers = _buffers(model)
    expected = {"model." + n for n, _ in params} | {"model." + n for n, _ in buffers}
    problems = ""
    step, has_step = 0, False
    optim_state = []
    for name, value in entries:
        if name == "step" and isinstance(value, int):
            step, has_step = value, True
        elif name.startswith("optim."):
            if isinstance(value, int):
                problems += " bad-kind:" + name
            else:
                optim_state.append((name[6:], value))
        elif name not in expected:
            problems += " unexpected:" + name
    if not has_step:
        problems += " missing:step"
    targets = [(n, p.data) for n, p in params] + list(buffers)
    for n, t in targets:
        v = by_name.get("model." + n)
        if v is None or isinstance(v, int):
            problems += " missing:model." + n
        elif tuple(v.shape) != tuple(t.shape):
            problems += " shape-mismatch:model." + n
    if problems:
        raise CheckpointError("load_checkpoint: checkpoint does not match model:" + problems)
    if optimizer is not None:
        if not optim_state:
            raise CheckpointError("load_checkpoint: checkpoint has no optimizer state")
        optimizer.load_state(optim_state)
    for n, t in targets:
        t.copy_(torch.from_numpy(by_name["model." + n]).to(t.device))
    return step
