"""End-to-end training steps on the GPU against the reference's own modules.

- Transformer (config 5's architecture at a small size): nnb's Transformer + AdamW and the
  reference's nn::Transformer + nn::AdamW (oracle/_ref) start from the same parameters and train on
  the same batch; losses, first-step gradients and the parameters after three steps agree to fp32
  tolerance. Training twice gives the same bits (tests/test_transformer.cpp:464), and the
  virtual-shard data-parallel step gives the same bits whatever the shard placement.
- CNN (config 2, full size): the Sequential conv/pool/linear stack and cross entropy, one forward and
  backward, against the reference's ops composed the same way.
"""
import numpy as np
import pytest

from oracle import orc

pytestmark = pytest.mark.gpu


def _flat(model):
    return np.concatenate([p.data.cpu().numpy().ravel() for p in model.parameters()])


def _flat_grads(model):
    return np.concatenate([p.grad.cpu().numpy().ravel() for p in model.parameters()])


def _close(got, want, rel):
    got, want = np.asarray(got, np.float64), np.asarray(want, np.float64)
    scale = np.abs(want).max()
    err = np.abs(got - want).max()
    assert err <= rel * scale, f"max err {err:.3e} vs scale {scale:.3e}"


def _batch(torch, vocab, N, T, seed):
    ids = orc.integers(seed, N * (T + 1), 0, vocab - 1).reshape(N, T + 1)
    x, y = ids[:, :T].copy(), ids[:, 1:].copy()          # next-token targets
    return x, y, torch.from_numpy(x).cuda(), torch.from_numpy(y).cuda()


def _train(torch, cfg, x_d, y_d, steps, lr, wd, shards=1, seed=3):
    from nnb.nn import AdamW, Transformer
    from nnb.train import ShardedTrainer

    model = Transformer(cfg, seed=seed)
    opt = AdamW(model.parameters(), lr=lr, weight_decay=wd)
    tr = ShardedTrainer(model, opt, shards=shards)
    losses, grads = [], None
    for s in range(steps):
        loss = tr.step(x_d, y_d)
        losses.append(float(loss.cpu()[0]))
        if s == 0:
            grads = tr.reduced.cpu().numpy().copy()
    return model, losses, grads


@pytest.mark.parametrize("dim,heads", [(32, 4), (128, 2)])     # head size 8: composed attention; 64: fused
def test_transformer_training_matches_reference(cuda, dim, heads):
    torch = cuda
    ref = orc.ref()
    if ref is None:
        pytest.skip("reference library not built (oracle/_ref)")
    from nnb.nn import Transformer, TransformerConfig

    cfg = TransformerConfig(vocab_size=64, dim=dim, heads=heads, layers=2, max_len=16)
    N, T, steps, lr, wd = 4, 16, 3, 1e-2, 1e-2
    x, y, x_d, y_d = _batch(torch, 64, N, T, 90)
    init = _flat(Transformer(cfg, seed=3))
    model, losses, grads = _train(torch, cfg, x_d, y_d, steps, lr, wd, shards=1, seed=3)

    r_losses = np.zeros(steps, np.float32)
    r_grads = np.zeros_like(init)
    r_params = np.zeros_like(init)
    n = ref.ref_transformer_train(64, dim, heads, 2, 16, N, T, orc.ptr(init), orc.ptr(x), orc.ptr(y), lr, wd, steps,
                                  orc.ptr(r_losses), orc.ptr(r_grads), orc.ptr(r_params))
    assert n == init.size
    np.testing.assert_allclose(losses, r_losses, rtol=1e-5)
    _close(grads, r_grads, 1e-4)
    # Adam moves an element whose gradient is rounding noise by about +-lr per step whatever the
    # noise's size, so the parameters after the steps are compared as: all within the Adam step
    # bound (2 lr per step), and all but a sliver (elements with near-zero gradients) to 1e-5.
    got = _flat(model).astype(np.float64)
    err = np.abs(got - r_params)
    assert err.max() <= 2 * lr * steps
    tight = err <= 1e-5 * np.abs(r_params).max()
    assert tight.mean() > 0.995, tight.mean()
    assert losses[-1] < losses[0]


@pytest.mark.parametrize("dim,heads", [(64, 4), (128, 2)])      # head size 16: composed attention; 64: fused
def test_transformer_training_deterministic_and_shard_invariant(cuda, dim, heads):
    torch = cuda
    import nnb
    from nnb import functional as F
    from nnb.nn import AdamW, Transformer, TransformerConfig
    from nnb.train import ShardedTrainer

    cfg = TransformerConfig(vocab_size=96, dim=dim, heads=heads, layers=2, max_len=32)
    _, _, x_d, y_d = _batch(torch, 96, 8, 32, 91)
    m1, l1, g1 = _train(torch, cfg, x_d, y_d, 2, 3e-3, 1e-2, shards=8)
    m2, l2, _ = _train(torch, cfg, x_d, y_d, 2, 3e-3, 1e-2, shards=8)
    assert _flat(m1).tobytes() == _flat(m2).tobytes()
    assert l1 == l2
    # The first step's reduced gradient, recomputed as 4 ranks of 2 shards each would (each "rank"
    # runs its own rows with 2 parameter-gradient groups), gathered and summed in shard order: the
    # same bits as the single-rank step (this is the data-parallel step at 4 GPUs, one rank at a time)
    m3 = Transformer(cfg, seed=3)
    opt = AdamW(m3.parameters(), lr=3e-3, weight_decay=1e-2)
    trs = [ShardedTrainer(m3, opt, shards=8, world=4, rank=r) for r in range(4)]
    norm = torch.tensor([1.0 / x_d.numel()], device="cuda")
    gathered = torch.empty(8, trs[0].total, device="cuda")
    for r, tr in enumerate(trs):
        tr._point_grads(tr.shard_grads)
        with F.param_groups(2):
            logits = m3(x_d[2 * r:2 * r + 2])
            loss = F.sequence_cross_entropy(logits, y_d[2 * r:2 * r + 2], grad_norm=norm)
            loss.backward()
        gathered[2 * r:2 * r + 2].copy_(tr.shard_grads)
    reduced = torch.empty(trs[0].total, device="cuda")
    s = torch.cuda.current_stream().cuda_stream
    nnb.check(nnb.lib().nnb_column_sum(s, 8, trs[0].total, gathered.data_ptr(), reduced.data_ptr(), 1))
    assert reduced.cpu().numpy().tobytes() == g1.tobytes()
    # and as 8 ranks of one shard each (the ungrouped path)
    m4 = Transformer(cfg, seed=3)
    tr8 = [ShardedTrainer(m4, AdamW(m4.parameters()), shards=8, world=8, rank=r) for r in range(8)]
    for r, tr in enumerate(tr8):
        tr._point_grads(tr.shard_grads)
        logits = m4(x_d[r:r + 1])
        loss = F.sequence_cross_entropy(logits, y_d[r:r + 1], grad_norm=norm)
        loss.backward()
        gathered[r:r + 1].copy_(tr.shard_grads)
    nnb.check(nnb.lib().nnb_column_sum(s, 8, trs[0].total, gathered.data_ptr(), reduced.data_ptr(), 1))
    assert reduced.cpu().numpy().tobytes() == g1.tobytes()


@pytest.mark.parametrize("dim,heads,dropout", [(64, 1, 0.0), (32, 4, 0.1)])
def test_graphed_training_step_bitwise_equal_to_eager(cuda, dim, heads, dropout):
    """The trainer's step captured into a CUDA graph (warm-up steps, capture, replays) gives the eager
    steps' weights, losses and optimizer step count bit for bit -- with dropout too (the generator
    state advances inside the graph)."""
    torch = cuda
    import nnb.random as nr
    from nnb.nn import AdamW, Transformer, TransformerConfig
    from nnb.train import ShardedTrainer

    cfg = TransformerConfig(vocab_size=96, dim=dim, heads=heads, layers=2, max_len=32, dropout=dropout)
    _, _, x_d, y_d = _batch(torch, 96, 8, 32, 92)
    runs = []
    for graphed in (False, True):
        nr.manual_seed(4)
        model = Transformer(cfg, seed=3)
        tr = ShardedTrainer(model, AdamW(model.parameters(), lr=3e-3, weight_decay=1e-2), shards=8)
        losses = []
        if graphed:
            step = tr.capture(x_d, y_d, warmup=2)
            losses += [None, None]
            for _ in range(3):
                losses.append(float(step().cpu()[0]))
            step.release()
        else:
            for _ in range(5):
                losses.append(float(tr.step(x_d, y_d).cpu()[0]))
            losses[:2] = [None, None]
        runs.append((_flat(model), losses, tr.opt.t))
    (w_e, l_e, t_e), (w_g, l_g, t_g) = runs
    assert t_e == t_g == 5
    assert l_e == l_g
    assert w_e.tobytes() == w_g.tobytes()


def test_cnn_forward_backward_matches_reference(cuda):
    torch = cuda
    ref = orc.ref()
    if ref is None:
        pytest.skip("reference library not built (oracle/_ref)")
    import nnb.functional as F
    from nnb.autograd import Value
    from nnb.nn import Conv2d, Flatten, Linear, MaxPool2d, ReLU, Sequential

    rng = np.random.default_rng(5)
    dev = torch.device("cuda")
    conv1, conv2 = Conv2d(1, 32, 3, 1, 1, rng, dev), Conv2d(32, 64, 3, 1, 1, rng, dev)
    fc1, fc2 = Linear(3136, 128, rng, dev), Linear(128, 10, rng, dev)
    front = Sequential(conv1, ReLU(), MaxPool2d(2, 2), conv2, ReLU(), MaxPool2d(2, 2), Flatten(), fc1)
    params_l = list(front.parameters()) + list(fc2.parameters())
    # Decisions must match for the gradients to compare element by element (a flipped ReLU or a
    # different first maximum in a pooling window routes a gradient elsewhere). Images that are
    # multiples of 1/8 and conv weights that are multiples of 2^-8 make every conv output exact in
    # fp32 on both sides (few-bit products, short exact sums; 3xTF32 splits such operands without
    # loss), so the conv ReLU and pooling decisions are identical; fc1's are shared below.
    for conv in (conv1, conv2):
        conv.weight.data.copy_(torch.round(conv.weight.data * 256) / 256)
    N = 64
    x = (np.round(orc.uniform(50, N * 784, 0.0, 1.0) * 8) / 8).astype(np.float32).reshape(N, 1, 28, 28)
    labels = orc.integers(51, N, 0, 9)
    params = np.concatenate([p.data.cpu().numpy().ravel() for p in params_l])

    r_loss, r_logits, r_grads = np.zeros(1, np.float32), np.zeros((N, 10), np.float32), np.zeros_like(params)
    r_fc1 = np.zeros((N, 128), np.float32)
    ref.ref_cnn_fwd_bwd_ex(N, orc.ptr(x), orc.ptr(labels), orc.ptr(params), orc.ptr(r_loss), orc.ptr(r_logits),
                           orc.ptr(r_grads), orc.ptr(r_fc1))

    for p in params_l:
        p.zero_grad()
    h = front(Value.leaf(torch.from_numpy(x).cuda(), False))
    fc1_gpu = h.data.cpu().numpy()
    _close(fc1_gpu, r_fc1, 1e-4)
    # fc1's ReLU decisions: the 3xTF32 product's error at K = 3136 (about 2e-5 of fc1's output) can
    # move a decision that sits within ~5e-6 of zero. Each moved decision routes a gradient g instead
    # of 0 into everything upstream, so the backward below runs on the reference's own pre-activation
    # (its decisions); every gradient then agrees element by element to fp32 GEMM accuracy.
    flipped = int(np.count_nonzero((fc1_gpu > 0) != (r_fc1 > 0)))
    assert flipped <= 8, flipped
    near = np.abs(r_fc1[(fc1_gpu > 0) != (r_fc1 > 0)])
    assert near.size == 0 or near.max() <= 1e-4 * np.abs(r_fc1).max()
    h.data.copy_(torch.from_numpy(r_fc1))
    logits = fc2(F.relu(h))
    loss = F.cross_entropy_loss(logits, torch.from_numpy(labels).cuda())
    loss.backward()
    grads = np.concatenate([p.grad.cpu().numpy().ravel() for p in params_l])
    _close(logits.data.cpu().numpy(), r_logits, 1e-4)     # logits are small sums of larger terms
    np.testing.assert_allclose(float(loss.data.cpu()[0]), float(r_loss[0]), rtol=1e-5)
    off = 0
    names = ["conv1.w", "conv1.b", "conv2.w", "conv2.b", "fc1.w", "fc1.b", "fc2.w", "fc2.b"]
    for name, p in zip(names, params_l):
        n = p.data.numel()
        g, r = grads[off:off + n], r_grads[off:off + n]
        off += n
        _close(g, r, 1e-4)


def test_transformer_config5_shape_matches_reference(cuda):
    """Config 5's model (vocab 4096, d 512, 8 heads, 4 layers, T 512) on two sequences: loss, the first
    step's gradients and the parameters after two AdamW steps against the reference's Transformer."""
    torch = cuda
    ref = orc.ref()
    if ref is None:
        pytest.skip("reference library not built (oracle/_ref)")
    from nnb.nn import Transformer, TransformerConfig

    V, D, H, Lyr, T, N = 4096, 512, 8, 4, 512, 2
    cfg = TransformerConfig(vocab_size=V, dim=D, heads=H, layers=Lyr, max_len=T)
    steps, lr, wd = 2, 3e-4, 1e-2
    x, y, x_d, y_d = _batch(torch, V, N, T, 95)
    init = _flat(Transformer(cfg, seed=3))
    model, losses, grads = _train(torch, cfg, x_d, y_d, steps, lr, wd, shards=1, seed=3)

    r_losses = np.zeros(steps, np.float32)
    r_grads = np.zeros_like(init)
    r_params = np.zeros_like(init)
    n = ref.ref_transformer_train(V, D, H, Lyr, T, N, T, orc.ptr(init), orc.ptr(x), orc.ptr(y), lr, wd, steps,
                                  orc.ptr(r_losses), orc.ptr(r_grads), orc.ptr(r_params))
    assert n == init.size == 16808960
    np.testing.assert_allclose(losses, r_losses, rtol=1e-5)
    _close(grads, r_grads, 1e-4)
    # per parameter tensor too, so a small tensor's error is not hidden by the embedding's scale; a
    # tensor whose true gradient is zero (the attention key biases: a bias added to every key shifts a
    # softmax row by a constant) holds rounding noise only and is held to the global scale
    off = 0
    floor = 1e-3 * np.abs(r_grads).max()
    for name, p in model.named_parameters():
        k = p.data.numel()
        got, want = grads[off:off + k].astype(np.float64), r_grads[off:off + k].astype(np.float64)
        scale = max(np.abs(want).max(), floor)
        assert np.abs(got - want).max() <= 2e-4 * scale, name
        off += k
    got = _flat(model).astype(np.float64)
    err = np.abs(got - r_params)
    assert err.max() <= 2 * lr * steps
    tight = err <= 1e-5 * np.abs(r_params).max()
    assert tight.mean() > 0.995, tight.mean()


def test_graphed_cnn_step_matches_eager(cuda):
    """A CUDA-graph replay of the CNN step (nnb.graph) gives the eager step's bits."""
    torch = cuda
    import nnb.functional as F
    from nnb.autograd import Value
    from nnb.graph import GraphedStep
    from nnb.nn import Conv2d, Flatten, Linear, MaxPool2d, ReLU, Sequential

    rng = np.random.default_rng(8)
    dev = torch.device("cuda")
    net = Sequential(Conv2d(1, 8, 3, 1, 1, rng, dev), ReLU(), MaxPool2d(2, 2), Flatten(), Linear(8 * 14 * 14, 10, rng, dev))
    x = torch.from_numpy(orc.uniform(52, 16 * 784, 0.0, 1.0).reshape(16, 1, 28, 28)).cuda()
    y = torch.from_numpy(orc.integers(53, 16, 0, 9)).cuda()

    def step():
        net.zero_grad()
        loss = F.cross_entropy_loss(net(Value.leaf(x, False)), y)
        loss.backward()
        return loss

    eager_loss = step().data.clone()
    eager_grads = [p.grad.clone() for p in net.parameters()]
    g = GraphedStep(step)
    x.copy_(torch.from_numpy(orc.uniform(52, 16 * 784, 0.0, 1.0).reshape(16, 1, 28, 28)))
    out = g()
    torch.cuda.synchronize()
    assert torch.equal(out.data, eager_loss)
    for p, e in zip(net.parameters(), eager_grads):
        assert torch.equal(p.grad, e)
