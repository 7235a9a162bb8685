"""Random streams and dropout masks on the host (no GPU): the library's seeding registry
(nnb_manual_seed / nnb_derive_generator, host C++ in libnnb) against the reference's own
src/random.cpp and std::mt19937 / std::seed_seq (through oracle/_ref), and the oracle's dropout
draws (oracle/orc.py dropout_draws) against the reference's Dropout layer.

The GPU draws (the device generator) are checked against the same reference calls in
tests/test_dropout_gpu.py.
"""
import numpy as np
import pytest

import nnb
import nnb.random as nr
from oracle import orc


def ref():
    r = orc.ref()
    if r is None:
        pytest.skip("reference library not built (oracle/_ref)")
    return r


@pytest.mark.parametrize("seeds", [[], [0], [5, 7], [1, 2, 3, 4, 5], [0xFFFFFFFF, 0x80000000]])
def test_seed_seq_state_matches_std(seeds):
    R = ref()
    s = np.array(seeds, np.uint32)
    state = np.zeros(625, np.uint32)
    nnb.check(nnb.lib().nnb_mt19937_seed_seq(s.ctypes.data if len(s) else None, len(s), state.ctypes.data))
    assert state[624] == 624
    n = 2000
    mine, _ = orc.mt_outputs(state, n)
    want = np.zeros(n, np.uint32)
    R.ref_mt19937_outputs(s.ctypes.data if len(s) else None, len(s), n, want.ctypes.data)
    assert (mine == want).all()


@pytest.mark.parametrize("seed,stream,skip", [(0, "dropout", 0), (42, "dropout", 3), (2**64 - 1, "dataloader", 1),
                                              (7, "", 0), (123456789, "a much longer stream name", 2)])
def test_derive_generator_matches_reference(seed, stream, skip):
    R = ref()
    nr.manual_seed(seed)
    for _ in range(skip):
        nr.derive_generator(stream)
    state = nr.derive_generator(stream)
    n = 1500
    mine, _ = orc.mt_outputs(state, n)
    want = np.zeros(n, np.uint32)
    R.ref_derive_outputs(seed, stream.encode(), skip, n, want.ctypes.data)
    assert (mine == want).all()


def test_registry_counters_epoch_and_independent_streams():
    nr.manual_seed(9)
    e = nr.seed_epoch()
    assert nr.is_seeded()
    a0 = nr.derive_generator("a")
    nr.derive_generator("b")                    # another name does not move "a"'s counter
    a1 = nr.derive_generator("a")
    nr.manual_seed(9)
    assert nr.seed_epoch() == e + 1
    assert (nr.derive_generator("a") == a0).all()
    nr.derive_generator("a")
    assert not (a0 == a1).all()


SIZES = [1, 31, 32, 593, 624, 625, 1248, 1000, 64, 5000, 3]


@pytest.mark.parametrize("p", [0.1, 0.5, 0.95, 0.0, 1.0])
@pytest.mark.parametrize("skip", [0, 2])
def test_oracle_dropout_draws_match_reference(p, skip):
    """The oracle's mask values from the stream nnb derives are the reference Dropout's masks, call
    after call (the stream continues across calls; p 0 and 1 draw nothing)."""
    R = ref()
    sizes = np.array(SIZES, np.uintp)
    want = np.zeros(int(sizes.sum()), np.float32)
    R.ref_dropout_masks(11, skip, p, sizes.ctypes.data, len(sizes), want.ctypes.data)
    nr.manual_seed(11)
    for _ in range(skip):
        nr.derive_generator("dropout")
    state = nr.derive_generator("dropout")
    got = []
    for n in SIZES:
        m, state = orc.dropout_draws(state, n, p)
        got.append(m)
    assert np.concatenate(got).tobytes() == want.tobytes()


def test_dropout_host_checks():
    L = nnb.lib()
    assert L.nnb_dropout_apply(None, 4, 1.5, None, None, None) == nnb.NNB_ERR_INVALID
    assert L.nnb_dropout_mask(None, None, 0, 0.5, None) == nnb.NNB_OK          # nothing to draw
    assert L.nnb_dropout_mask(None, None, 0, -0.1, None) == nnb.NNB_ERR_INVALID
    assert L.nnb_derive_generator(None, None) == nnb.NNB_ERR_INVALID
