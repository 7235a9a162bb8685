"""The data pipeline's host side (no GPU): sample orders, splits and weights.

Pinned against the reference's own known answers (tests/test_dataloader.cpp:142-180, 766-785;
tests/test_random.cpp:89-97) and, through oracle/_ref, against the reference's DataLoader,
random_split and balanced_sample_weights on many configurations: the loaders visit the same samples
in the same batches, epoch after epoch. Batch assembly on the device is in tests/test_data_gpu.py.
"""
import numpy as np
import pytest

import nnb
import nnb.random as nr
from nnb.data import (CharVocab, DataLoader, SequenceDataset, Subset, TensorDataset, balanced_sample_weights,
                      random_split)
from oracle import orc

CPU = "cpu"


def ref():
    r = orc.ref()
    if r is None:
        pytest.skip("reference library not built (oracle/_ref)")
    return r


def index_dataset(n):
    v = np.arange(n, dtype=np.float32).reshape(n, 1)
    return TensorDataset(v, v.copy())


def loader(*args, **kw):
    kw.setdefault("device", CPU)        # sample order only: nothing reaches a device
    return DataLoader(*args, **kw)


def batches_of(ld):
    idx = ld.epoch_indices()
    return [idx[b * ld.batch_size: (b + 1) * ld.batch_size] for b in range(ld.num_batches())]


# -- known answers of the reference's tests ---------------------------------------------------------

def test_stream_hashing_pins():
    L = nnb.lib()
    assert L.nnb_fnv1a64(b"a") == 0xaf63dc4c8601ec8c
    assert L.nnb_fnv1a64(b"dataloader") == 9636703306727871938
    assert L.nnb_splitmix64(0) == 16294208416658607535
    assert L.nnb_splitmix64(12345) == 2454886589211414944
    nr.manual_seed(7)
    st = nr.derive_generator("a")
    out = np.zeros(1, np.uint32)
    nnb.check(L.nnb_mt19937_next(st.ctypes.data, 1, out.ctypes.data))
    assert out[0] == 2730421840


def test_seeded_loader_epoch_order_pin():
    nr.manual_seed(42)
    ld = loader(index_dataset(10), 10, True)
    assert ld.epoch_indices().tolist() == [1, 2, 3, 7, 6, 8, 0, 5, 9, 4]


def test_random_split_permutation_pin():
    parts = random_split(index_dataset(10), [0.5, 0.5], 42)
    assert np.concatenate([p.indices for p in parts]).tolist() == [1, 3, 9, 7, 6, 0, 8, 4, 5, 2]
    first = lambda seed: random_split(index_dataset(10), [0.5, 0.5], seed)[0].indices.tolist()
    assert first(5) != first(5 + (1 << 32))
    assert first(5) == first(5 << 32)               # the halves fold to the same engine seed


def test_weighted_draws_pin():
    nr.manual_seed(1)
    ld = loader(index_dataset(5), 8, sample_weights=[1, 2, 3, 0, 4], num_samples=8)
    assert ld.epoch_indices().tolist() == [2, 1, 0, 0, 1, 4, 2, 2]


def test_trailing_zero_weight_never_drawn():
    nr.manual_seed(3)
    ld = loader(index_dataset(2), 100, sample_weights=[1, 0], num_samples=1000)
    assert ld.num_batches() == 10 and (ld.epoch_indices() == 0).all()


# -- against the reference's loader -----------------------------------------------------------------

@pytest.mark.parametrize("n,batch,shuffle,drop_last,skip", [
    (10, 10, 1, 0, 0), (1, 4, 1, 0, 0), (7, 3, 1, 0, 1), (100, 32, 1, 1, 0), (1000, 64, 1, 0, 2), (13, 5, 0, 0, 0),
    (13, 5, 0, 1, 0), (4097, 100, 1, 0, 0)])
def test_loader_orders_match_reference(n, batch, shuffle, drop_last, skip):
    R = ref()
    epochs = 3
    want = np.zeros(n * epochs, np.float32)
    got_n = R.ref_loader_orders(11, skip, n, batch, shuffle, drop_last, epochs, want.ctypes.data)
    nr.manual_seed(11)
    for _ in range(skip):
        loader(index_dataset(n), batch, bool(shuffle))
    ld = loader(index_dataset(n), batch, bool(shuffle), bool(drop_last))
    got = []
    for e in range(epochs):
        if e:
            ld.reset_epoch()
        got += [np.asarray(b) for b in batches_of(ld)]
    got = np.concatenate(got).astype(np.float32) if got else np.zeros(0, np.float32)
    assert got.size == got_n and (got == want[:got_n]).all()


@pytest.mark.parametrize("n,batch,num_samples,drop_last", [(5, 8, 8, 0), (50, 7, 0, 0), (300, 64, 1000, 1), (1, 3, 5, 0)])
def test_weighted_loader_matches_reference(n, batch, num_samples, drop_last):
    R = ref()
    rng = np.random.default_rng(n)
    w = rng.uniform(0, 3, n)
    w[rng.integers(0, n, n // 5)] = 0.0
    if w.sum() == 0:
        w[0] = 1.0
    epochs = 2
    want = np.zeros((num_samples or n) * epochs, np.float32)
    got_n = R.ref_loader_weighted(4, w.ctypes.data, n, batch, num_samples, drop_last, epochs, want.ctypes.data)
    nr.manual_seed(4)
    ld = loader(index_dataset(n), batch, drop_last=bool(drop_last), sample_weights=w, num_samples=num_samples)
    got = []
    for e in range(epochs):
        if e:
            ld.reset_epoch()
        got += [np.asarray(b) for b in batches_of(ld)]
    got = np.concatenate(got).astype(np.float32)
    assert got.size == got_n and (got == want[:got_n]).all()
    assert not (w[got.astype(np.int64)] == 0).any()


@pytest.mark.parametrize("n,fractions,seed", [(10, [0.5, 0.5], 42), (101, [0.7, 0.2, 0.1], 7), (3, [0.34, 0.33, 0.33], 1),
                                              (9, [0.34, 0.33, 0.33], 5),
                                              (1000, [0.25] * 4, 2 ** 40 + 9)])
def test_random_split_matches_reference(n, fractions, seed):
    R = ref()
    fr = np.array(fractions, np.float64)
    sizes = np.zeros(len(fractions), np.uintp)
    want = np.zeros(n, np.float32)
    if R.ref_random_split(n, fr.ctypes.data, len(fractions), seed, sizes.ctypes.data, want.ctypes.data):
        with pytest.raises(ValueError):           # the reference threw: so must we
            random_split(index_dataset(n), fractions, seed)
        return
    parts = random_split(index_dataset(n), fractions, seed)
    assert [p.size() for p in parts] == sizes.tolist()
    assert np.concatenate([p.indices for p in parts]).astype(np.float32).tolist() == want.tolist()


def test_balanced_sample_weights_match_reference():
    R = ref()
    labels = np.random.default_rng(0).integers(0, 7, 500).astype(np.uintp)
    want = np.zeros(500, np.float64)
    assert R.ref_balanced_weights(labels.ctypes.data, 500, 7, want.ctypes.data) == 0
    assert balanced_sample_weights(labels, 7).tobytes() == want.tobytes()
    with pytest.raises(ValueError):
        balanced_sample_weights([0, 7], 7)


# -- checks and host semantics ----------------------------------------------------------------------

def test_loader_rejects_bad_arguments():
    ds = index_dataset(4)
    with pytest.raises(nnb.TensorShapeError):
        loader(ds, 0)
    for w in ([1, 2, 3], [1, -1, 1, 1], [1, np.nan, 1, 1], [0, 0, 0, 0]):
        with pytest.raises(ValueError):
            loader(ds, 2, sample_weights=w)
    with pytest.raises(TypeError):
        loader(ds, 2, sample_weights=[1, 1, 1, 1], num_samples=True)
    ld = loader(ds, 3)
    assert ld.num_batches() == 2
    with pytest.raises(nnb.TensorIndexError):
        ld.get_batch(2)
    assert loader(ds, 3, drop_last=True).num_batches() == 1


def test_random_split_rejects_bad_fractions():
    ds = index_dataset(4)
    for fr in ([], [0.5, 0.6], [1.0, 0.0], [0.9, 0.05, 0.05]):
        with pytest.raises(ValueError):
            random_split(ds, fr, 1)


def test_subset_and_datasets():
    ds = index_dataset(6)
    s = Subset(ds, [5, 0, 3])
    assert s.size() == 3 and s.get(0)[0][0] == 5
    with pytest.raises(nnb.TensorIndexError):
        Subset(ds, [6])
    with pytest.raises(nnb.TensorShapeError):
        TensorDataset(np.zeros((3, 2)), np.zeros((4,)))
    seq = SequenceDataset([3, 1, 4, 1, 5, 9, 2], 3)
    assert seq.size() == 4
    x, y = seq.get(1)
    assert x.tolist() == [1, 4, 1] and y.tolist() == [4, 1, 5]
    with pytest.raises(ValueError):
        SequenceDataset([1, 2], 2)
    with pytest.raises(nnb.TensorIndexError):
        seq.get(4)


def test_char_vocab():
    v = CharVocab("hello world")
    assert v.size() == 8 and v.chars == b" dehlorw"
    ids = v.encode("hold")
    assert ids.dtype == np.float32 and v.decode(ids) == "hold"
    with pytest.raises(ValueError):
        v.encode("z")
    with pytest.raises(ValueError):
        v.decode([8.0])
    with pytest.raises(ValueError):
        v.decode([1.5])
