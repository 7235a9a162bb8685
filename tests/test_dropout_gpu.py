"""Dropout and attention with dropout on the GPU, against the reference build (oracle/_ref).

- The device generator's masks are the reference Dropout layer's masks bit for bit, call after call
  (sizes straddling the 624-word blocks), for several p, after other layers took earlier streams;
  the backward multiplies by the same mask; p 0 / 1 and evaluation mode.
- A large draw (3M elements) against the oracle's draws from the same state.
- MultiHeadAttention with dropout active (the composed path: head GEMMs around the masked softmax
  and the dropped weights), two forward + backward calls, against the reference's module: outputs
  and gradients to the fp32 bound of the other attention tests (the masks are identical, the
  products are tensor-core 3xTF32).
- A Transformer with dropout trained for three steps against the reference's.
"""
import numpy as np
import pytest

from oracle import orc

pytestmark = pytest.mark.gpu
SIZES = [1, 31, 32, 593, 624, 625, 1248, 1000, 64, 5000, 3, 40000]


def ref():
    r = orc.ref()
    if r is None:
        pytest.skip("reference library not built (oracle/_ref)")
    return r


def _close(got, want, rel):
    got, want = np.asarray(got, np.float64), np.asarray(want, np.float64)
    scale = np.abs(want).max()
    err = np.abs(got - want).max()
    assert err <= rel * scale, f"max err {err:.3e} vs scale {scale:.3e}"


@pytest.mark.parametrize("p", [0.1, 0.5, 0.95, 1.0, 0.0])
@pytest.mark.parametrize("skip", [0, 3])
def test_dropout_layer_masks_bitwise(cuda, p, skip):
    torch = cuda
    import nnb.random as nr
    from nnb.autograd import Value
    from nnb.nn import Dropout
    R = ref()
    sizes = np.array(SIZES, np.uintp)
    want = np.zeros(int(sizes.sum()), np.float32)
    R.ref_dropout_masks(5, skip, p, sizes.ctypes.data, len(sizes), want.ctypes.data)
    nr.manual_seed(5)
    for _ in range(skip):
        Dropout(p)
    d = Dropout(p)
    off = 0
    for n in SIZES:
        x = Value.leaf(torch.ones(n, device="cuda"), True)
        y = d(x)
        m = want[off: off + n]
        assert y.data.cpu().numpy().tobytes() == m.tobytes(), f"mask of the call of size {n}"
        if p > 0:                                  # p == 0 returns the input itself, as the reference
            g = torch.arange(n, dtype=torch.float32, device="cuda") - 7.5
            y.backward(g)
            assert x.grad.cpu().numpy().tobytes() == (g.cpu().numpy() * m + np.float32(0)).tobytes()
        off += n


def test_dropout_large_draw_matches_oracle(cuda):
    torch = cuda
    import nnb.functional as F
    import nnb.random as nr
    nr.manual_seed(77)
    host = nr.derive_generator("dropout")
    state = torch.from_numpy(host.view(np.int32)).cuda()
    n, p = 3_000_017, 0.3
    mine = []
    for size in (n, 1000):                         # the second call continues the stream
        keep = F.dropout_mask(state, size, p).cpu().numpy().view(np.uint32)
        bits = ((keep[:, None] >> np.arange(32, dtype=np.uint32)) & 1).reshape(-1)[:size]
        mine.append(bits)
    s = host
    for size, bits in zip((n, 1000), mine):
        m, s = orc.dropout_draws(s, size, p)
        assert (bits == (m != 0)).all()
    assert state.cpu().numpy().view(np.uint32).tobytes() == s.tobytes()      # the device state advanced alike


def test_dropout_eval_mode_is_identity(cuda):
    torch = cuda
    from nnb.autograd import Value
    from nnb.nn import Dropout
    d = Dropout(0.5).eval()
    x = Value.leaf(torch.randn(100, device="cuda"), True)
    assert d(x) is x


@pytest.mark.parametrize("N,T,D,H,causal,p", [(2, 33, 64, 2, 1, 0.3), (3, 17, 48, 4, 0, 0.1), (1, 130, 64, 1, 1, 0.5)])
def test_attention_dropout_op_matches_reference(cuda, N, T, D, H, causal, p):
    """The attention core with dropout (nnb_dropout_mask + nnb_attention_dropout_fwd/bwd) against the
    reference's own composition (split heads, matmul_bt, scaled_masked_softmax, Dropout, matmul):
    identical masks, products to the fp32 bound."""
    torch = cuda
    import nnb.functional as F
    import nnb.random as nr
    from nnb.autograd import Value
    R = ref()
    q, k, v, g = (orc.normal(400 + i, N * T * D) for i in range(4))
    o_r, dq_r, dk_r, dv_r = (orc.zeros(N * T * D) for _ in range(4))
    R.ref_attention_dropout(12, N, T, D, H, causal, p, *(orc.ptr(a) for a in (q, k, v, g, o_r, dq_r, dk_r, dv_r)))
    nr.manual_seed(12)
    state = nr.device_generator("dropout", torch.device("cuda"))
    Q, K, V = (Value.leaf(torch.from_numpy(a.reshape(N, T, D)).cuda(), True) for a in (q, k, v))
    Y = F.attention_dropout(Q, K, V, H, None, bool(causal), p, state)
    Y.backward(torch.from_numpy(g.reshape(N, T, D)).cuda())
    _close(Y.data.cpu().numpy().ravel(), o_r, 2e-5)
    for got, want in ((Q.grad, dq_r), (K.grad, dk_r), (V.grad, dv_r)):
        _close(got.cpu().numpy().ravel(), want, 2e-5)


def _mha_params(D, seed):
    ws = []
    for i in range(4):
        ws.append(orc.uniform(seed + 2 * i, D * D, -0.3, 0.3))
        ws.append(orc.uniform(seed + 2 * i + 1, D, -0.1, 0.1))
    return ws


@pytest.mark.parametrize("D,heads,causal,p", [(32, 4, 1, 0.2), (64, 1, 0, 0.5), (48, 3, 1, 1.0)])
def test_mha_with_dropout_matches_reference(cuda, D, heads, causal, p):
    torch = cuda
    import nnb.random as nr
    from nnb.autograd import Value
    from nnb.nn import MultiHeadAttention
    R = ref()
    N, T, calls = 2, 19, 2
    params = _mha_params(D, 300)
    flat = np.concatenate(params)
    x, g = orc.normal(310, N * T * D), orc.normal(311, N * T * D)
    y_r, dx_r, dp_r = orc.zeros(N * T * D), orc.zeros(N * T * D), np.zeros_like(flat)
    R.ref_mha_dropout(21, N, T, D, heads, causal, p, calls, orc.ptr(flat), orc.ptr(x), orc.ptr(g), orc.ptr(y_r),
                      orc.ptr(dx_r), orc.ptr(dp_r))
    nr.manual_seed(21)
    mha = MultiHeadAttention(D, heads, bool(causal), np.random.default_rng(0), torch.device("cuda"), dropout=p)
    for (name, prm), w in zip(mha.named_parameters(), params):
        prm.data.copy_(torch.from_numpy(w.reshape(prm.data.shape)))
    for _ in range(calls):
        for prm in mha.parameters():
            prm.zero_grad()
        X = Value.leaf(torch.from_numpy(x.reshape(N, T, D)).cuda(), True)
        Y = mha(X)
        Y.backward(torch.from_numpy(g.reshape(N, T, D)).cuda())
    _close(Y.data.cpu().numpy().ravel(), y_r, 2e-5)
    _close(X.grad.cpu().numpy().ravel(), dx_r, 2e-5)
    got = np.concatenate([prm.grad.cpu().numpy().ravel() for prm in mha.parameters()]).astype(np.float64)
    # per parameter against its own scale; k.bias's gradient is zero in exact arithmetic (softmax
    # backward rows sum to zero), so both programs hold rounding noise there: bounded by the
    # gradients' overall scale instead
    floor = 2e-2 * np.abs(dp_r).max()
    off = 0
    for w in params:
        seg_g, seg_r = got[off: off + w.size], dp_r[off: off + w.size].astype(np.float64)
        assert np.abs(seg_g - seg_r).max() <= 5e-5 * max(np.abs(seg_r).max(), floor)
        off += w.size


def test_transformer_with_dropout_trains_like_reference(cuda):
    torch = cuda
    import nnb.random as nr
    from nnb.nn import AdamW, Transformer, TransformerConfig
    from nnb.train import ShardedTrainer
    R = ref()
    vocab, dim, heads, layers, T, N, steps, lr, wd, p = 64, 32, 4, 2, 16, 4, 3, 1e-2, 1e-2, 0.1
    cfg = TransformerConfig(vocab_size=vocab, dim=dim, heads=heads, layers=layers, max_len=T, dropout=p)
    ids = orc.integers(95, N * (T + 1), 0, vocab - 1).reshape(N, T + 1)
    x, y = ids[:, :T].copy(), ids[:, 1:].copy()
    nr.manual_seed(33)
    model = Transformer(cfg, seed=3)
    init = np.concatenate([q.data.cpu().numpy().ravel() for q in model.parameters()])
    tr = ShardedTrainer(model, AdamW(model.parameters(), lr=lr, weight_decay=wd), shards=2)
    losses = [float(tr.step(torch.from_numpy(x).cuda(), torch.from_numpy(y).cuda()).cpu()[0]) for _ in range(steps)]
    r_losses, r_grads, r_params = np.zeros(steps, np.float32), np.zeros_like(init), np.zeros_like(init)
    n = R.ref_transformer_train_ex(33, p, vocab, dim, heads, layers, T, N, T, orc.ptr(init), orc.ptr(x), orc.ptr(y),
                                   lr, wd, steps, orc.ptr(r_losses), orc.ptr(r_grads), orc.ptr(r_params))
    assert n == init.size
    np.testing.assert_allclose(losses, r_losses, rtol=1e-5)
    got = np.concatenate([q.data.cpu().numpy().ravel() for q in model.parameters()]).astype(np.float64)
    err = np.abs(got - r_params)
    assert err.max() <= 2 * lr * steps
    assert (err <= 1e-5 * np.abs(r_params).max()).mean() > 0.995


def test_dropout_mask_slice_is_the_rows_of_the_whole_draw(cuda):
    """nnb_dropout_mask_slice: a rank's slice of a draw has the bits of the same outputs of the whole
    draw, and the generator ends where the whole draw leaves it -- for slices inside one 2^24-output
    chunk, across a chunk boundary, at the end, and empty."""
    torch = cuda
    import ctypes
    import nnb
    import nnb.random as nr
    nr.manual_seed(71)
    state0 = nr.device_generator("dropout", torch.device("cuda"))
    total, p = (1 << 24) + 3 * 4096 + 96, 0.3
    s = torch.cuda.current_stream().cuda_stream
    full_state = state0.clone()
    full = torch.empty((total + 31) // 32, dtype=torch.int32, device="cuda")
    nnb.check(nnb.lib().nnb_dropout_mask(s, full_state.data_ptr(), total, ctypes.c_float(p), full.data_ptr()))
    bits = np.unpackbits(full.cpu().numpy().view(np.uint8), bitorder="little")[:total]
    for offset, count in ((0, 4096), (4096 * 7, 12288 + 5), ((1 << 24) - 4096, 8192), (total - 96, 96), (64, 0)):
        st = state0.clone()
        keep = torch.zeros(max(1, (count + 31) // 32), dtype=torch.int32, device="cuda")
        nnb.check(nnb.lib().nnb_dropout_mask_slice(s, st.data_ptr(), total, offset, count, ctypes.c_float(p),
                                                   keep.data_ptr()))
        got = np.unpackbits(keep.cpu().numpy().view(np.uint8), bitorder="little")[:count]
        assert np.array_equal(got, bits[offset:offset + count]), (offset, count)
        assert torch.equal(st, full_state), (offset, count)
    with pytest.raises(nnb.NnbError):
        nnb.check(nnb.lib().nnb_dropout_mask_slice(s, state0.clone().data_ptr(), total, 5, 10, ctypes.c_float(p),
                                                   full.data_ptr()))


def test_data_parallel_dropout_ranks_emulated(cuda):
    """The data-parallel step with dropout, each rank's pass run one after another on one GPU (the
    generators reset to the step's start state for every rank, as separate GPUs hold their own copies):
    every rank's rows draw their part of the whole batch's masks, so the gathered shard gradients
    equal the one-rank step's bit for bit, the loss agrees, and every rank's generators end in the same
    state."""
    torch = cuda
    import nnb
    import nnb.random as nr
    from nnb import functional as F
    from nnb.nn import AdamW, Dropout, Transformer, TransformerConfig
    from nnb.train import ShardedTrainer
    cfg = TransformerConfig(vocab_size=48, dim=64, heads=1, layers=2, max_len=32, dropout=0.1)  # head size 64
    ids = orc.integers(96, 8 * 33, 0, 47).reshape(8, 33)
    x_d, y_d = torch.from_numpy(ids[:, :32].copy()).cuda(), torch.from_numpy(ids[:, 1:].copy()).cuda()
    nr.manual_seed(5)
    m1 = Transformer(cfg, seed=3)
    tr1 = ShardedTrainer(m1, AdamW(m1.parameters(), lr=1e-3), shards=8)
    drops1 = [mod for mod in m1.modules() if isinstance(mod, Dropout)]
    start = [d.state.clone() for d in drops1]
    loss1 = tr1.step(x_d, y_d).clone()
    g1 = tr1.reduced.clone()
    end1 = [d.state.clone() for d in drops1]
    # the same step as 4 ranks of 2 shards each
    nr.manual_seed(5)
    m4 = Transformer(cfg, seed=3)
    drops4 = [mod for mod in m4.modules() if isinstance(mod, Dropout)]
    opt = AdamW(m4.parameters(), lr=1e-3)
    trs = [ShardedTrainer(m4, opt, shards=8, world=4, rank=r) for r in range(4)]
    norm = torch.tensor([1.0 / x_d.numel()], device="cuda")
    gathered = torch.empty(8, trs[0].total, device="cuda")
    losses = []
    for r, tr in enumerate(trs):
        for d, s0 in zip(drops4, start):
            d.state.copy_(s0)
        tr._point_grads(tr.shard_grads)
        with F.param_groups(2), F.batch_slice(8, 2 * r, 2 * r + 2):
            logits = m4(x_d[2 * r:2 * r + 2])
            loss = F.sequence_cross_entropy(logits, y_d[2 * r:2 * r + 2], grad_norm=norm)
            loss.backward()
        losses.append(loss.data.clone())
        gathered[2 * r:2 * r + 2].copy_(tr.shard_grads)
        for d, e in zip(drops4, end1):
            assert torch.equal(d.state, e)
    reduced = torch.empty(trs[0].total, device="cuda")
    s = torch.cuda.current_stream().cuda_stream
    nnb.check(nnb.lib().nnb_column_sum(s, 8, trs[0].total, gathered.data_ptr(), reduced.data_ptr(), 1))
    assert torch.equal(reduced, g1)
    # the loss is each rank's mean, averaged over ranks: the same value, summed in another order
    np.testing.assert_allclose(float(torch.cat(losses).mean()), float(loss1[0]), rtol=1e-6)
