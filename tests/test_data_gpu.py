"""DataLoader batch assembly on the GPU.

- HBM-resident TensorDataset: every batch of three epochs (shuffled, plain, weighted, drop_last) is
  the stack of the dataset's rows in the epoch's order, bit for bit, for row sizes taking the 16-,
  4- and 1-byte gather paths; with the index dataset the batches are the reference loader's own.
- SequenceDataset windows, Subsets of resident datasets, the host (pinned, double-buffered) path of
  a plain Python Dataset against the resident path, and a bad index (zero row + device error word).
"""
import numpy as np
import pytest

from oracle import orc

pytestmark = pytest.mark.gpu


def _epochs(ld, epochs):
    out = []
    for e in range(epochs):
        if e:
            ld.reset_epoch()
        out.append([(x.data if hasattr(x, "data") else x, y) for x, y in ld])
    return out


@pytest.mark.parametrize("row_shape,dtype", [((3, 5), np.float32), ((3,), np.float32), ((7,), np.uint8),
                                             ((1, 28, 28), np.float32)])
@pytest.mark.parametrize("mode", ["shuffle", "plain", "weighted", "drop_last"])
def test_resident_tensor_dataset_batches(cuda, row_shape, dtype, mode):
    torch = cuda
    import nnb.random as nr
    from nnb.data import DataLoader, TensorDataset
    n, batch = 203, 32
    rng = np.random.default_rng(1)
    inputs = (rng.standard_normal((n,) + row_shape) * 50).astype(dtype)
    targets = rng.integers(0, 7, n).astype(np.int64)
    nr.manual_seed(8)
    kw = {"shuffle": mode == "shuffle", "drop_last": mode == "drop_last"}
    if mode == "weighted":
        kw = {"sample_weights": rng.uniform(0, 1, n), "num_samples": 150}
    ld = DataLoader(TensorDataset(inputs, targets), batch, **kw)
    for e in range(3):
        if e:
            ld.reset_epoch()
        order = ld.epoch_indices()
        for b in range(ld.num_batches()):
            x, y = ld.get_batch(b)
            sel = order[b * batch: (b + 1) * batch]
            assert not x.requires_grad
            assert x.data.cpu().numpy().tobytes() == inputs[sel].tobytes()
            assert y.cpu().numpy().tobytes() == targets[sel].tobytes()
    assert ld.num_batches() == {"drop_last": n // batch, "weighted": 5}.get(mode, -(-n // batch))


def test_resident_batches_are_the_reference_loaders(cuda):
    import nnb.random as nr
    from nnb.data import DataLoader, TensorDataset
    R = orc.ref()
    if R is None:
        pytest.skip("reference library not built (oracle/_ref)")
    n, batch, epochs = 1000, 64, 3
    want = np.zeros(n * epochs, np.float32)
    got_n = R.ref_loader_orders(19, 0, n, batch, 1, 0, epochs, want.ctypes.data)
    v = np.arange(n, dtype=np.float32).reshape(n, 1)
    nr.manual_seed(19)
    ld = DataLoader(TensorDataset(v, v.copy()), batch, True)
    got = np.concatenate([x.cpu().numpy().ravel() for ep in _epochs(ld, epochs) for x, _ in ep])
    assert got.size == got_n and got.tobytes() == want[:got_n].tobytes()


def test_sequence_dataset_windows(cuda):
    import nnb.random as nr
    from nnb.data import DataLoader, SequenceDataset
    tokens = np.random.default_rng(2).integers(0, 500, 10_000)
    ds = SequenceDataset(tokens, 64)
    nr.manual_seed(3)
    ld = DataLoader(ds, 48, True)
    order = ld.epoch_indices()
    for b in (0, 7, ld.num_batches() - 1):
        x, y = ld.get_batch(b)
        sel = order[b * 48: (b + 1) * 48]
        assert x.dtype == y.dtype and str(x.dtype) == "torch.int64"
        want_x = np.stack([tokens[s: s + 64] for s in sel])
        want_y = np.stack([tokens[s + 1: s + 65] for s in sel])
        assert (x.cpu().numpy() == want_x).all() and (y.cpu().numpy() == want_y).all()


def test_subset_of_resident_dataset(cuda):
    import nnb.random as nr
    from nnb.data import DataLoader, TensorDataset, random_split
    n = 97
    inputs = np.random.default_rng(4).standard_normal((n, 6)).astype(np.float32)
    targets = np.arange(n, dtype=np.int64)
    train, val = random_split(TensorDataset(inputs, targets), [0.8, 0.2], 11)
    nr.manual_seed(5)
    ld = DataLoader(train, 16, True)
    order = train.indices[ld.epoch_indices()]
    seen = []
    for b, (x, y) in enumerate(ld):
        sel = order[b * 16: (b + 1) * 16]
        assert x.data.cpu().numpy().tobytes() == inputs[sel].tobytes()
        seen += y.cpu().numpy().tolist()
    assert sorted(seen) == sorted(train.indices.tolist())


class _PlainDataset:
    """A user dataset with only size() / get(i): the loader stacks it on the host."""

    def __init__(self, inputs, targets):
        self.inputs, self.targets = inputs, targets

    def size(self):
        return len(self.inputs)

    def get(self, i):
        return self.inputs[i], self.targets[i]


def test_host_path_double_buffered_matches_resident(cuda):
    import nnb.random as nr
    from nnb.data import DataLoader, TensorDataset
    n = 300
    rng = np.random.default_rng(6)
    inputs = rng.standard_normal((n, 2, 9)).astype(np.float32)
    targets = rng.integers(0, 10, n).astype(np.int64)
    nr.manual_seed(21)
    plain = DataLoader(_PlainDataset(inputs, targets), 40, True)
    nr.manual_seed(21)
    resident = DataLoader(TensorDataset(inputs, targets), 40, True)
    for e in range(2):
        if e:
            plain.reset_epoch()
            resident.reset_epoch()
        a = [(x.data.cpu().numpy(), y.cpu().numpy()) for x, y in plain]
        b = [(x.data.cpu().numpy(), y.cpu().numpy()) for x, y in resident]
        assert len(a) == len(b) == 8
        for (xa, ya), (xb, yb) in zip(a, b):
            assert xa.tobytes() == xb.tobytes() and ya.tobytes() == yb.tobytes()
    x, y = plain.get_batch(3)
    assert x.data.cpu().numpy().tobytes() == inputs[plain.epoch_indices()[120:160]].tobytes()


def test_bad_index_writes_zero_row_and_sets_device_error(cuda):
    torch = cuda
    import nnb
    src = torch.arange(12, dtype=torch.float32, device="cuda").view(4, 3)
    idx = torch.tensor([1, 9, 3], dtype=torch.int64, device="cuda")
    dst = torch.full((3, 3), 5.0, device="cuda")
    s = torch.cuda.current_stream().cuda_stream
    nnb.check(nnb.lib().nnb_gather_rows(s, src.data_ptr(), 12, 4, idx.data_ptr(), 3, dst.data_ptr()))
    assert dst.cpu().numpy().tolist() == [[3, 4, 5], [0, 0, 0], [9, 10, 11]]
    assert nnb.lib().nnb_device_error(s) == 17
    assert nnb.lib().nnb_device_error(s) == 0
