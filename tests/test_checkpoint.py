"""Checkpoints in the reference's NNCK v1 format (src/checkpoint.cpp, tests/test_checkpoint.cpp).

The fixtures under tests/golden/ were written by the reference's own save_checkpoint
(tests/golden/make_golden.py); linear_step7.nnck is byte-identical to the reference's golden file
tests/data/linear_v1.ckpt. CPU tests: our writer reproduces the fixtures byte for byte, our reader
restores them, malformed and mismatching files are rejected with the model untouched (the
reference test's cases), and our reader accepts or rejects exactly the files the reference's reader
does (every truncation and seeded byte mutations, through oracle/_ref). GPU tests: AdamW's state
after one step saves to the reference's bytes, loads back, and a data-parallel run resumed from a
checkpoint continues bit for bit like the uninterrupted run.
"""
import os
import pathlib
import struct

import numpy as np
import pytest
import torch

from nnb.checkpoint import CheckpointError, load_checkpoint, save_checkpoint
from nnb.nn import Linear, ReLU, Sequential
from oracle import orc

GOLDEN = pathlib.Path(__file__).resolve().parent / "golden"
W = [0.5, -1.25, 2.0, 3.0, 0.75, -0.5]           # tests/test_checkpoint.cpp's golden Linear(3, 2)
B = [0.125, -2.0]
GW = [0.25, -0.5, 1.5, -2.0, 0.125, 3.0]         # gradients and settings of linear_adamw.nnck
GB = [-0.75, 0.375]
LR, WD = 0.01, 0.1
CPU = torch.device("cpu")


def linear32(device=CPU, w=W, b=B):
    m = Sequential(Linear(3, 2, np.random.default_rng(0), device))
    p = m.named_parameters()
    p[0][1].data.copy_(torch.tensor(w, dtype=torch.float32).view(2, 3))
    p[1][1].data.copy_(torch.tensor(b, dtype=torch.float32))
    return m


def mlp(hidden=3, seed=0, device=CPU):
    rng = np.random.default_rng(seed)
    return Sequential(Linear(2, hidden, rng, device), ReLU(), Linear(hidden, 1, rng, device))


def snapshot(m):
    return [p.data.cpu().numpy().copy() for p in m.parameters()]


def same(a, b):
    return len(a) == len(b) and all(x.shape == y.shape and x.tobytes() == y.tobytes() for x, y in zip(a, b))


def header(count):
    return b"NNCK" + struct.pack("<II", 1, count)


def rejected(tmp_path, data, model=None):
    """Loading `data` must raise CheckpointError and leave the model's parameters as they were."""
    path = str(tmp_path / "bad.nnck")
    pathlib.Path(path).write_bytes(data)
    m = model or mlp()
    before = snapshot(m)
    with pytest.raises(CheckpointError):
        load_checkpoint(path, m)
    assert same(snapshot(m), before)


# -- the writer and reader against the reference's bytes ------------------------------------------

def test_writer_matches_reference_golden(tmp_path):
    path = str(tmp_path / "a.nnck")
    save_checkpoint(path, linear32(), step=7)
    assert pathlib.Path(path).read_bytes() == (GOLDEN / "linear_step7.nnck").read_bytes()


def test_reader_restores_reference_golden():
    m = linear32(w=[0.0] * 6, b=[0.0, 0.0])
    assert load_checkpoint(str(GOLDEN / "linear_step7.nnck"), m) == 7
    assert same(snapshot(m), [np.array(W, np.float32).reshape(2, 3), np.array(B, np.float32)])


def test_bytes_match_documented_format(tmp_path):
    """tests/test_checkpoint.cpp:112-128, written out by hand."""
    m = Sequential(Linear(1, 1, np.random.default_rng(0), CPU))
    m.named_parameters()[0][1].data.fill_(1.0)
    m.named_parameters()[1][1].data.fill_(2.0)
    path = str(tmp_path / "a.nnck")
    save_checkpoint(path, m)
    want = header(3)
    want += struct.pack("<I", 14) + b"model.0.weight" + b"\0" + struct.pack("<IQQI", 2, 1, 1, 0x3F800000)
    want += struct.pack("<I", 12) + b"model.0.bias" + b"\0" + struct.pack("<IQI", 1, 1, 0x40000000)
    want += struct.pack("<I", 4) + b"step" + b"\1" + struct.pack("<q", 0)
    assert pathlib.Path(path).read_bytes() == want


def test_round_trip_restores_weights_and_step(tmp_path):
    a, b = mlp(seed=1), mlp(seed=2)
    path = str(tmp_path / "a.nnck")
    save_checkpoint(path, a, step=42)
    assert load_checkpoint(path, b) == 42
    assert same(snapshot(a), snapshot(b))
    assert not os.path.exists(path + ".tmp")


def test_zero_parameter_model_round_trips(tmp_path):
    path = str(tmp_path / "a.nnck")
    save_checkpoint(path, Sequential(ReLU()), step=7)
    assert load_checkpoint(path, Sequential(ReLU())) == 7


def test_nan_inf_negative_zero_bit_exact(tmp_path):
    a, b = Sequential(Linear(2, 2, np.random.default_rng(0), CPU)), Sequential(Linear(2, 2, np.random.default_rng(1), CPU))
    bits = np.array([0x7FC00001, 0x7F800000, 0xFF800000, 0x80000000], np.uint32)     # NaN with payload
    a.parameters()[0].data.copy_(torch.from_numpy(bits.view(np.float32).reshape(2, 2)))
    path = str(tmp_path / "a.nnck")
    save_checkpoint(path, a)
    load_checkpoint(path, b)
    assert b.parameters()[0].data.numpy().view(np.uint32).reshape(-1).tolist() == bits.tolist()


# -- rejection cases of tests/test_checkpoint.cpp ---------------------------------------------------

def test_every_truncation_rejected(tmp_path):
    path = str(tmp_path / "a.nnck")
    save_checkpoint(path, mlp(seed=5))
    data = pathlib.Path(path).read_bytes()
    for n in range(len(data)):
        rejected(tmp_path, data[:n])


def test_bad_magic_version_duplicates_and_trailing_bytes(tmp_path):
    path = str(tmp_path / "a.nnck")
    save_checkpoint(path, mlp(seed=5))
    data = pathlib.Path(path).read_bytes()
    rejected(tmp_path, b"X" + data[1:])
    rejected(tmp_path, data[:4] + b"\2" + data[5:])
    rejected(tmp_path, data + b"\0")
    dup = header(2) + 2 * (struct.pack("<I", 4) + b"step" + b"\1" + struct.pack("<q", 0))
    rejected(tmp_path, dup)
    bad_kind = header(1) + struct.pack("<I", 4) + b"step" + b"\2" + struct.pack("<q", 0)
    rejected(tmp_path, bad_kind)


def test_absurd_headers_rejected_without_allocating(tmp_path):
    rejected(tmp_path, header(1) + struct.pack("<I", 0x7FFFFFFF))
    name = struct.pack("<I", 14) + b"model.0.weight" + b"\0"
    rejected(tmp_path, header(1) + name + struct.pack("<I", 255))
    rejected(tmp_path, header(1) + name + struct.pack("<IQQ", 2, 1 << 40, 1 << 40))
    rejected(tmp_path, header(0xFFFFFFFF))
    (tmp_path / "shape.nnck").write_bytes(header(1) + name + struct.pack("<IQQ", 2, 1 << 40, 1 << 40))
    with pytest.raises(CheckpointError, match="bad shape"):
        load_checkpoint(str(tmp_path / "shape.nnck"), mlp())


def test_extra_or_missing_layers_rejected_with_entry_name(tmp_path):
    small, big = Sequential(Linear(2, 3, np.random.default_rng(0), CPU)), mlp()
    path = str(tmp_path / "a.nnck")
    save_checkpoint(path, big)
    before = snapshot(small)
    with pytest.raises(CheckpointError, match=r"model\.2\.weight"):
        load_checkpoint(path, small)
    assert same(snapshot(small), before)
    save_checkpoint(path, small)
    before = snapshot(big)
    with pytest.raises(CheckpointError, match=r"model\.2\.weight"):
        load_checkpoint(path, big)
    assert same(snapshot(big), before)


def test_wrong_shape_rejected_with_entry_name(tmp_path):
    a, b = mlp(3), mlp(4)
    path = str(tmp_path / "a.nnck")
    save_checkpoint(path, a)
    before = snapshot(b)
    with pytest.raises(CheckpointError, match=r"shape-mismatch:model\.0\.weight"):
        load_checkpoint(path, b)
    assert same(snapshot(b), before)


def test_failed_save_keeps_previous_checkpoint(tmp_path):
    a, b = mlp(seed=1), mlp(seed=2)
    path = str(tmp_path / "a.nnck")
    save_checkpoint(path, a, step=5)
    original = pathlib.Path(path).read_bytes()
    os.mkdir(path + ".tmp")                        # a directory squats on the temporary name
    with pytest.raises(CheckpointError):
        save_checkpoint(path, b, step=9)
    assert pathlib.Path(path).read_bytes() == original
    assert load_checkpoint(path, b) == 5


class _StubOptimizer:
    """The optimizer side of the protocol (state() / load_state()) without device buffers."""

    def __init__(self):
        self.loaded = None

    def state(self):
        return [("lr", torch.tensor([0.1]))]

    def load_state(self, snapshot):
        self.loaded = snapshot


def test_optimizer_requested_from_model_only_file(tmp_path):
    a, b = mlp(seed=1), mlp(seed=2)
    path = str(tmp_path / "a.nnck")
    save_checkpoint(path, a)
    before = snapshot(b)
    opt = _StubOptimizer()
    with pytest.raises(CheckpointError, match="optim"):
        load_checkpoint(path, b, opt)
    assert same(snapshot(b), before) and opt.loaded is None


def test_inference_load_ignores_optimizer_entries(tmp_path):
    a, b = mlp(seed=1), mlp(seed=2)
    path = str(tmp_path / "a.nnck")
    save_checkpoint(path, a, _StubOptimizer(), step=3)
    assert load_checkpoint(path, b) == 3
    assert same(snapshot(a), snapshot(b))
    opt = _StubOptimizer()
    load_checkpoint(path, b, opt)
    assert [n for n, _ in opt.loaded] == ["lr"]


def test_int_optimizer_entry_rejected(tmp_path):
    a = Sequential(ReLU())
    data = header(2) + struct.pack("<I", 8) + b"optim.lr" + b"\1" + struct.pack("<q", 1)
    data += struct.pack("<I", 4) + b"step" + b"\1" + struct.pack("<q", 0)
    (tmp_path / "a.nnck").write_bytes(data)
    with pytest.raises(CheckpointError, match="bad-kind:optim.lr"):
        load_checkpoint(str(tmp_path / "a.nnck"), a)


# -- our reader and writer against the reference's own (oracle/_ref, CPU) --------------------------

def ref():
    r = orc.ref()
    if r is None:
        pytest.skip("reference library not built (oracle/_ref)")
    return r


def ours_load(path):
    """(step, w, b) from our reader into Sequential{Linear(3, 2)}, or None when it rejects the file."""
    m = linear32(w=[9.0] * 6, b=[9.0, 9.0])
    try:
        step = load_checkpoint(path, m)
    except CheckpointError:
        return None
    w, b = snapshot(m)
    return step, w.reshape(-1), b


def ref_load(R, path):
    w, b = np.full(6, 9.0, np.float32), np.full(2, 9.0, np.float32)
    step = R.ref_linear_checkpoint_load(path.encode(), orc.ptr(w), orc.ptr(b))
    return None if step == -1 else (step, w, b)


def agree(got, want):
    if got is None or want is None:
        return got is None and want is None
    return got[0] == want[0] and got[1].tobytes() == want[1].tobytes() and got[2].tobytes() == want[2].tobytes()


def test_reader_accepts_exactly_what_reference_accepts(tmp_path):
    R = ref()
    rng = np.random.default_rng(7)
    path = str(tmp_path / "m.nnck")
    n_accept = 0
    for fixture in ("linear_step7.nnck", "linear_adamw.nnck"):
        data = (GOLDEN / fixture).read_bytes()
        cases = [data[:n] for n in range(0, len(data), 3)] + [data]
        for _ in range(300):
            mutated = bytearray(data)
            for pos in rng.integers(0, len(data), rng.integers(1, 3)):
                mutated[pos] = rng.integers(0, 256)
            cases.append(bytes(mutated))
        for case in cases:
            pathlib.Path(path).write_bytes(case)
            want = ref_load(R, path)
            if want is not None and want[0] == -1:
                continue        # a stored step of -1 reads as the shim's rejection code
            got = ours_load(path)
            assert agree(got, want), f"disagree on {case.hex()}"
            n_accept += want is not None
    assert n_accept > 50        # the mutations also hit the float payloads that both readers accept


def test_writer_matches_reference_writer(tmp_path):
    R = ref()
    rng = np.random.default_rng(8)
    for step in (0, 1, -5, 1 << 40, -(1 << 62)):
        w, b = rng.standard_normal(6).astype(np.float32), rng.standard_normal(2).astype(np.float32)
        mine, theirs = str(tmp_path / "mine.nnck"), str(tmp_path / "theirs.nnck")
        save_checkpoint(mine, linear32(w=w.tolist(), b=b.tolist()), step=step)
        assert R.ref_linear_checkpoint_save(theirs.encode(), orc.ptr(w), orc.ptr(b), None, None, 0.0, 0.0, step) == 0
        assert pathlib.Path(mine).read_bytes() == pathlib.Path(theirs).read_bytes()


# -- optimizer state on the GPU ---------------------------------------------------------------------

def _adamw_after_one_step(torch_mod):
    from nnb.nn import AdamW
    dev = torch_mod.device("cuda")
    m = linear32(dev)
    opt = AdamW(m.parameters(), lr=LR, weight_decay=WD)
    for p, g in zip(m.parameters(), (GW, GB)):
        p.grad.copy_(torch_mod.tensor(g, dtype=torch_mod.float32, device=dev).view(p.data.shape))
        p.grad_fresh = False
    opt.step()
    return m, opt


@pytest.mark.gpu
def test_adamw_state_saves_reference_bytes(cuda, tmp_path):
    """One AdamW step (the fused kernel) then a save with the optimizer: the reference's bytes."""
    m, opt = _adamw_after_one_step(cuda)
    path = str(tmp_path / "a.nnck")
    save_checkpoint(path, m, opt, step=1)
    assert pathlib.Path(path).read_bytes() == (GOLDEN / "linear_adamw.nnck").read_bytes()


@pytest.mark.gpu
def test_adamw_state_loads_and_resumes(cuda, tmp_path):
    """The reference's file loads into a fresh model and an AdamW with other settings; the next step
    then matches the uninterrupted optimizer's bit for bit (tests/test_checkpoint.cpp:292-305)."""
    torch_mod = cuda
    from nnb.nn import AdamW
    dev = torch_mod.device("cuda")
    a, opt_a = _adamw_after_one_step(torch_mod)
    b = linear32(dev, w=[0.0] * 6, b=[0.0, 0.0])
    opt_b = AdamW(b.parameters(), lr=0.5, beta1=0.5, weight_decay=WD)
    assert load_checkpoint(str(GOLDEN / "linear_adamw.nnck"), b, opt_b) == 1
    assert same(snapshot(a), snapshot(b))
    assert (opt_b.lr, opt_b.beta1, opt_b.t) == (np.float32(LR), np.float32(0.9), 1)
    for x, y in zip(opt_a.m + opt_a.v, opt_b.m + opt_b.v):
        assert x.cpu().numpy().tobytes() == y.cpu().numpy().tobytes()
    for m, opt in ((a, opt_a), (b, opt_b)):
        for p, g in zip(m.parameters(), (GB * 3, GW[:2])):
            p.grad.copy_(torch_mod.tensor(g, dtype=torch_mod.float32, device=dev).view(p.data.shape))
            p.grad_fresh = False
        opt.step()
    assert same(snapshot(a), snapshot(b))


@pytest.mark.gpu
def test_reference_reads_our_optimizer_file(cuda, tmp_path):
    R = ref()
    m, opt = _adamw_after_one_step(cuda)
    path = str(tmp_path / "a.nnck")
    save_checkpoint(path, m, opt, step=11)
    got = ref_load(R, path)
    assert got is not None and got[0] == 11
    w, b = snapshot(m)
    assert got[1].tobytes() == w.reshape(-1).tobytes() and got[2].tobytes() == b.tobytes()


@pytest.mark.gpu
def test_batchnorm_running_statistics_round_trip(cuda, tmp_path):
    torch_mod = cuda
    from nnb.autograd import Value
    from nnb.nn import BatchNorm2d
    dev = torch_mod.device("cuda")
    a, b = Sequential(BatchNorm2d(3, dev)), Sequential(BatchNorm2d(3, dev))
    x = torch_mod.from_numpy(orc.normal(5, 2 * 3 * 4 * 4).reshape(2, 3, 4, 4)).to(dev)
    a(Value.leaf(x, True))
    path = str(tmp_path / "bn.nnck")
    save_checkpoint(path, a, step=2)
    assert load_checkpoint(path, b) == 2
    for (na, ta), (nb, tb) in zip(a.named_buffers(), b.named_buffers()):
        assert na == nb and ta.cpu().numpy().tobytes() == tb.cpu().numpy().tobytes()
    assert [n for n, _ in a.named_buffers()] == ["0.running_mean", "0.running_var"]


@pytest.mark.gpu
def test_sharded_trainer_resumes_bitwise(cuda, tmp_path):
    """Two data-parallel steps, a checkpoint (model, optimizer, step), two more steps; a fresh model
    and trainer loaded from the checkpoint reach the same weights bit for bit after its two steps."""
    torch_mod = cuda
    from nnb.nn import AdamW, Transformer, TransformerConfig
    from nnb.train import ShardedTrainer
    cfg = TransformerConfig(vocab_size=64, dim=64, heads=1, layers=1, max_len=32)
    g = torch_mod.Generator().manual_seed(9)
    ids = torch_mod.randint(0, 64, (8, 33), generator=g)
    x, y = ids[:, :-1].contiguous().cuda(), ids[:, 1:].contiguous().cuda()
    a = Transformer(cfg, seed=4)
    tr_a = ShardedTrainer(a, AdamW(a.parameters(), lr=3e-3), shards=8)
    for _ in range(2):
        tr_a.step(x, y)
    tr_a.optimizer_to_params()
    path = str(tmp_path / "t.nnck")
    save_checkpoint(path, a, tr_a.opt, step=2)
    for _ in range(2):
        tr_a.step(x, y)
    b = Transformer(cfg, seed=5)
    opt_b = AdamW(b.parameters(), lr=1.0)
    assert load_checkpoint(path, b, opt_b) == 2
    tr_b = ShardedTrainer(b, opt_b, shards=8)
    tr_b.optimizer_from_params()
    for _ in range(2):
        tr_b.step(x, y)
    assert same(snapshot(a), snapshot(b))
