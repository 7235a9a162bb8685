"""Library-wide seeding and per-component random streams (include/nn/random.hpp, src/random.cpp).

The registry lives in libnnb (host C++): ``manual_seed(seed)`` fixes the base and resets the
per-name counters, and the k-th ``derive_generator(name)`` after it hands out the same mt19937 the
reference's k-th derive_generator(name) does, so components built in the same order after the
same seed (e.g. every Dropout layer, in construction order) draw the reference's numbers. A
generator is returned as its 625-word state (624 untempered words + the next-word index) in host
memory; :func:`device_generator` puts one on the GPU, where nnb_dropout_mask advances it in place.
"""
from __future__ import annotations

import numpy as np
import torch

from . import check, lib

STATE_WORDS = 625


def manual_seed(seed: int) -> None:
    """Seeds the library and resets every stream counter (random.hpp:25)."""
    lib().nnb_manual_seed(int(seed) & 0xFFFFFFFFFFFFFFFF)


def is_seeded() -> bool:
    return bool(lib().nnb_is_seeded())


def seed_epoch() -> int:
    """Counts manual_seed calls, so a component that caches a generator can notice a re-seed."""
    return int(lib().nnb_seed_epoch())


def derive_generator(stream: str) -> np.ndarray:
    """The next generator of the named stream, as its host state (uint32[625])."""
    state = np.zeros(STATE_WORDS, np.uint32)
    check(lib().nnb_derive_generator(stream.encode(), state.ctypes.data))
    return state


def device_generator(stream: str, device) -> torch.Tensor:
    """derive_generator(stream) copied to `device` (int32[625] holding the uint32 words)."""
    return torch.from_numpy(derive_generator(stream).view(np.int32)).to(device)
