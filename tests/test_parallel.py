"""Host logic of the sharded GEMM: band partition and gather (CPU, gloo, world size 2), and on two or
more GPUs (NCCL) the bitwise identity of the sharded product with the single-GPU one.

The reference's analogue is thread-count invariance (tests/test_kernels.cpp:343-380): here the
number of GPUs plays the role of the thread count.
"""
import os
import socket

import numpy as np
import pytest
import torch.multiprocessing as mp

from nnb.parallel import row_bands


def test_row_bands_cover_rows_in_whole_tiles():
    for m in (1, 127, 128, 1000, 8192, 16384):
        for world in (1, 2, 3, 4, 8):
            bands = row_bands(m, world)
            assert len(bands) == world
            assert bands[0][0] == 0 and bands[-1][1] == m
            for (s0, e0), (s1, _) in zip(bands, bands[1:]):
                assert e0 == s1
            nonempty = [(s, e) for s, e in bands if e > s]
            for s, e in nonempty:
                assert s % 128 == 0
            for s, e in nonempty[:-1]:
                assert (e - s) % 128 == 0
    assert row_bands(8192, 8) == [(i * 1024, (i + 1) * 1024) for i in range(8)]


def _free_port():
    with socket.socket() as s:
        s.bind(("127.0.0.1", 0))
        return s.getsockname()[1]


def _gloo_worker(rank, world, port, m, n, k, out_dir):
    import torch
    import torch.distributed as dist

    from nnb.parallel import gather_rows, row_bands
    from oracle import orc

    os.environ.update(MASTER_ADDR="127.0.0.1", MASTER_PORT=str(port))
    dist.init_process_group("gloo", rank=rank, world_size=world)
    try:
        a = orc.uniform(7, m * k).reshape(m, k)
        b = orc.uniform(8, k * n).reshape(k, n)
        bands = row_bands(m, world)
        s, e = bands[rank]
        band = np.zeros((e - s, n), np.float32)
        if e > s:
            orc.orc.orc_sgemm_f32(0, 0, e - s, n, k, orc.ptr(np.ascontiguousarray(a[s:e])), k, orc.ptr(b), n,
                                  orc.ptr(band), n, 0)
        full = gather_rows(torch.from_numpy(band), bands)
        if rank == 0:
            np.save(os.path.join(out_dir, "gathered.npy"), full.numpy())
    finally:
        dist.destroy_process_group()


def test_gather_rows_gloo_world2(tmp_path):
    """Two CPU ranks each compute a band with the oracle's fp32 loop; the gathered matrix is bitwise
    the single-process product."""
    from oracle import orc

    m, n, k = 300, 40, 33                       # bands of 256 and 44 rows: unequal heights
    mp.start_processes(_gloo_worker, args=(2, _free_port(), m, n, k, str(tmp_path)), nprocs=2, join=True,
                       start_method="spawn")
    got = np.load(tmp_path / "gathered.npy")
    a = orc.uniform(7, m * k).reshape(m, k)
    b = orc.uniform(8, k * n).reshape(k, n)
    want = np.zeros((m, n), np.float32)
    orc.orc.orc_sgemm_f32(0, 0, m, n, k, orc.ptr(a), k, orc.ptr(b), n, orc.ptr(want), n, 0)
    assert got.tobytes() == want.tobytes()


def _nccl_worker(rank, world, port, m, n, k, mode, gather, out_dir):
    import datetime

    import torch
    import torch.distributed as dist

    import nnb
    from nnb.parallel import PeerBuffer, gather_rows, row_bands

    os.environ.update(MASTER_ADDR="127.0.0.1", MASTER_PORT=str(port))
    torch.cuda.set_device(rank)
    dist.init_process_group("nccl", rank=rank, world_size=world, device_id=torch.device("cuda", rank),
                            timeout=datetime.timedelta(seconds=60))
    try:
        g = torch.Generator(device="cuda").manual_seed(5)
        a = torch.randn(m, k, device="cuda", generator=g)
        b = torch.randn(k, n, device="cuda", generator=g)
        bands = row_bands(m, world)
        s, e = bands[rank]
        if gather == "peer":
            # the GEMM's epilogue stores this rank's tiles straight into rank 0's C over NVLink
            peer = PeerBuffer((m, n), owner=0)
            if e > s:
                nnb.sgemm(False, False, e - s, n, k, a[s:e], k, b, n, peer.ptr + s * n * 4, n, False, math_mode=mode)
            torch.cuda.synchronize()
            dist.barrier(device_ids=[rank])
            full = peer.tensor
        else:
            band = torch.empty(e - s, n, device="cuda")
            nnb.sgemm(False, False, e - s, n, k, a[s:e], k, b, n, band, n, False, math_mode=mode)
            full = gather_rows(band, bands)
        if rank == 0:
            single = torch.empty(m, n, device="cuda")
            nnb.sgemm(False, False, m, n, k, a, k, b, n, single, n, False, math_mode=mode)
            np.save(os.path.join(out_dir, f"eq_{mode}_{gather}.npy"), np.array([bool(torch.equal(full, single))]))
        dist.barrier(device_ids=[rank])
        if gather == "peer":
            peer.close()
    finally:
        dist.destroy_process_group()


@pytest.mark.gpu
@pytest.mark.parametrize("gather", ["nccl", "peer"])
@pytest.mark.parametrize("mode", [0, 1])
@pytest.mark.parametrize("m,n,k", [(1000, 700, 900), (4096, 8192, 128)])
def test_sharded_gemm_bitwise_equal_to_single_gpu(cuda, tmp_path, mode, gather, m, n, k):
    """Bands computed on every GPU of the box (2-8) and gathered on GPU 0 (by an NCCL gather after the GEMM, or by the
    GEMM's own epilogue storing into GPU 0's C through peer memory) equal the one-GPU product bit for
    bit. In the wide case the bands run on 224-wide tiles and the one-GPU product on 256-wide ones."""
    torch = cuda
    world = torch.cuda.device_count()
    if world < 2:
        pytest.skip("needs two or more GPUs")
    mp.start_processes(_nccl_worker, args=(world, _free_port(), m, n, k, mode, gather, str(tmp_path)), nprocs=world,
                       join=True, start_method="spawn")
    assert bool(np.load(tmp_path / f"eq_{mode}_{gather}.npy")[0])


def _dp_worker(rank, world, port, out_dir, dropout=0.0):
    import torch
    import torch.distributed as dist

    import nnb.random as nr
    from nnb.nn import AdamW, Transformer, TransformerConfig
    from nnb.train import ShardedTrainer

    os.environ.update(MASTER_ADDR="127.0.0.1", MASTER_PORT=str(port))
    torch.cuda.set_device(rank)
    dist.init_process_group("nccl", rank=rank, world_size=world, device_id=torch.device("cuda", rank))
    try:
        nr.manual_seed(9)
        # head size 64: fused attention without dropout, the composed path with it
        cfg = TransformerConfig(vocab_size=128, dim=128, heads=2, layers=2, max_len=64, dropout=dropout)
        g = torch.Generator().manual_seed(3)
        ids = torch.randint(0, 128, (8, 65), generator=g)
        x, y = ids[:, :-1].contiguous().cuda(), ids[:, 1:].contiguous().cuda()
        model = Transformer(cfg, seed=4)
        tr = ShardedTrainer(model, AdamW(model.parameters(), lr=3e-3), shards=8, world=world, rank=rank)
        for _ in range(2):
            tr.step(x, y)
        flat = torch.cat([p.data.reshape(-1) for p in model.parameters()])
        # the same two steps with the second one captured into a CUDA graph (all-to-all and all-gather
        # inside the graph) and replayed
        nr.manual_seed(9)
        gmodel = Transformer(cfg, seed=4)
        gtr = ShardedTrainer(gmodel, AdamW(gmodel.parameters(), lr=3e-3), shards=8, world=world, rank=rank)
        step = gtr.capture(x, y, warmup=1)
        step()
        torch.cuda.synchronize()
        gflat = torch.cat([p.data.reshape(-1) for p in gmodel.parameters()])
        step.release()
        if rank == 0:
            nr.manual_seed(9)
            ref_model = Transformer(cfg, seed=4)
            ref_tr = ShardedTrainer(ref_model, AdamW(ref_model.parameters(), lr=3e-3), shards=8)
            for _ in range(2):
                ref_tr.step(x, y)
            ref_flat = torch.cat([p.data.reshape(-1) for p in ref_model.parameters()])
            np.save(os.path.join(out_dir, f"dp_eq_{dropout}.npy"), np.array([bool(torch.equal(flat, ref_flat)),
                                                                             bool(torch.equal(gflat, ref_flat))]))
        dist.barrier(device_ids=[rank])
    finally:
        dist.destroy_process_group()


@pytest.mark.gpu
@pytest.mark.parametrize("dropout", [0.0, 0.1])
def test_data_parallel_step_bitwise_equal_to_single_gpu(cuda, tmp_path, dropout):
    """Two training steps of the virtual-shard data-parallel step on every GPU of the box (2, 4 or 8;
    the largest divisor of 8 otherwise) give the same weights, bit for bit, as on one GPU -- with
    dropout too (each rank draws its rows of the whole batch's masks)."""
    torch = cuda
    world = torch.cuda.device_count()
    if world < 2:
        pytest.skip("needs two or more GPUs")
    while 8 % world:               # the 8 virtual shards need a world that divides them
        world -= 1
    mp.start_processes(_dp_worker, args=(world, _free_port(), str(tmp_path), dropout), nprocs=world, join=True,
                       start_method="spawn")
    eq = np.load(tmp_path / f"dp_eq_{dropout}.npy")
    assert bool(eq[0]), "eager data-parallel steps differ from one GPU"
    assert bool(eq[1]), "graph-replayed data-parallel step differs from one GPU"


def _attn_worker(rank, world, port, out_dir):
    import datetime

    import torch
    import torch.distributed as dist

    import nnb
    from nnb.parallel import ShardedAttention

    os.environ.update(MASTER_ADDR="127.0.0.1", MASTER_PORT=str(port))
    torch.cuda.set_device(rank)
    dist.init_process_group("nccl", rank=rank, world_size=world, device_id=torch.device("cuda", rank),
                            timeout=datetime.timedelta(seconds=60))
    try:
        B, T, D, H = 11, 130, 128, 2                 # 11 samples over 2-8 ranks: unequal shares
        g = torch.Generator(device="cuda").manual_seed(21)
        q, k, v, go = (torch.randn(B, T, D, device="cuda", generator=g) for _ in range(4))
        sa = ShardedAttention(B, T, D, H, causal=True)
        n0, n1 = sa.n0, sa.n1
        sa.step(q[n0:n1].contiguous(), k[n0:n1].contiguous(), v[n0:n1].contiguous(), go[n0:n1].contiguous())
        torch.cuda.synchronize()
        dist.barrier(device_ids=[rank])
        if rank == 0:
            L, s = nnb.lib(), torch.cuda.current_stream().cuda_stream
            o = torch.empty(B, T, D, device="cuda")
            st = torch.empty(B, H, T, 2, device="cuda")
            dq, dk, dv = (torch.empty(B, T, D, device="cuda") for _ in range(3))
            nnb.check(L.nnb_flash_attention_fwd(s, B, T, T, D, H, q.data_ptr(), k.data_ptr(), v.data_ptr(), None, 1,
                                                o.data_ptr(), st.data_ptr()))
            nnb.check(L.nnb_flash_attention_bwd(s, B, T, T, D, H, go.data_ptr(), q.data_ptr(), k.data_ptr(),
                                                v.data_ptr(), o.data_ptr(), st.data_ptr(), None, 1, dq.data_ptr(), 1,
                                                dk.data_ptr(), 1, dv.data_ptr(), 1))
            torch.cuda.synchronize()
            eq = [bool(torch.equal(a.tensor, b)) for a, b in ((sa.out, o), (sa.dq, dq), (sa.dk, dk), (sa.dv, dv))]
            np.save(os.path.join(out_dir, "attn_eq.npy"), np.array(eq))
        dist.barrier(device_ids=[rank])
        sa.close()
    finally:
        dist.destroy_process_group()


@pytest.mark.gpu
def test_sharded_attention_bitwise_equal_to_single_gpu(cuda, tmp_path):
    """Attention forward + backward split by samples over every GPU of the box (2-8), O / dQ / dK / dV gathered on GPU 0
    (dQ / dK / dV stored there by the backward kernels through peer memory, O by a peer copy): the
    one-GPU results, bit for bit."""
    torch = cuda
    world = torch.cuda.device_count()
    if world < 2:
        pytest.skip("needs two or more GPUs")
    mp.start_processes(_attn_worker, args=(world, _free_port(), str(tmp_path)), nprocs=world, join=True,
                       start_method="spawn")
    assert np.load(tmp_path / "attn_eq.npy").all()


# ---- host logic of the data-parallel exchange and of the attention shares (gloo, CPU) ----------

def _dp_exchange_worker(rank, world, port, shards, total, out_dir):
    import torch
    import torch.distributed as dist

    from nnb.train import exchange_shard_gradients, gather_weight_slices, shard_owners
    from oracle import orc

    os.environ.update(MASTER_ADDR="127.0.0.1", MASTER_PORT=str(port))
    dist.init_process_group("gloo", rank=rank, world_size=world)
    try:
        owned = shard_owners(shards, world, rank)
        # shard i's gradient is a fixed function of i alone, wherever it is computed
        shard_grads = torch.from_numpy(np.stack([orc.normal(300 + i, total) for i in owned]))
        chunk = -(-total // world)
        send = torch.zeros(world, len(owned), chunk)
        recv = torch.empty(shards, chunk)
        exchange_shard_gradients(shard_grads, send, recv, chunk, world)
        reduced = np.zeros(chunk, np.float32)
        orc.orc.orc_colsum(shards, chunk, orc.ptr(recv.numpy()), orc.ptr(reduced), 1)
        flat_w = torch.zeros(chunk * world)
        lo = rank * chunk
        n = min(total, lo + chunk) - lo
        flat_w[lo:lo + n] = torch.from_numpy(reduced[:n])      # stands in for AdamW on this rank's slice
        gather_weight_slices(flat_w, chunk, rank)
        np.save(os.path.join(out_dir, f"flat_{rank}.npy"), flat_w[:total].numpy())
    finally:
        dist.destroy_process_group()


@pytest.mark.parametrize("world,total", [(2, 1001), (4, 37)])
def test_data_parallel_exchange_gloo(tmp_path, world, total):
    """The data-parallel step's exchange on CPU ranks: slicing into the send buffer, the all-to-all,
    the shard-order sum of the received rows (the oracle's Tensor::sum(0)) and the in-place all-gather
    of the slices leave on EVERY rank the single-process shard-order sum of all 8 shards, bit for
    bit (an uneven last slice included)."""
    from oracle import orc

    shards = 8
    mp.start_processes(_dp_exchange_worker, args=(world, _free_port(), shards, total, str(tmp_path)), nprocs=world,
                       join=True, start_method="spawn")
    allg = np.stack([orc.normal(300 + i, total) for i in range(shards)])
    want = np.zeros(total, np.float32)
    orc.orc.orc_colsum(shards, total, orc.ptr(allg), orc.ptr(want), 1)
    for r in range(world):
        assert np.load(tmp_path / f"flat_{r}.npy").tobytes() == want.tobytes()


def test_shard_owners():
    from nnb.train import shard_owners
    for world in (1, 2, 4, 8):
        runs = [shard_owners(8, world, r) for r in range(world)]
        assert sum(runs, []) == list(range(8))
        assert all(len(r) == 8 // world for r in runs)
    with pytest.raises(ValueError):
        shard_owners(8, 3, 0)


def _attn_share_worker(rank, world, port, B, T, D, H, path):
    import torch.distributed as dist

    from nnb.parallel import sample_shares, share_offset_bytes
    from oracle import orc

    os.environ.update(MASTER_ADDR="127.0.0.1", MASTER_PORT=str(port))
    dist.init_process_group("gloo", rank=rank, world_size=world)
    try:
        shares = sample_shares(B, world)
        n0, n1 = shares[rank]
        q, k, v = (orc.normal(310 + j, B * T * D).reshape(B, T, D) for j in range(3))
        # the owner's full-size O buffer, shared by the ranks as the peer buffer is on the GPUs
        owner = np.memmap(path, dtype=np.float32, mode="r+", shape=(B, T, D))
        if n1 > n0:
            o = np.zeros((n1 - n0, T, D), np.float32)
            p = np.zeros((n1 - n0, H, T, T), np.float32)
            orc.orc.orc_attention_fwd(n1 - n0, T, T, D, H, orc.ptr(np.ascontiguousarray(q[n0:n1])),
                                      orc.ptr(np.ascontiguousarray(k[n0:n1])), orc.ptr(np.ascontiguousarray(v[n0:n1])),
                                      None, 1, orc.ptr(o), orc.ptr(p))
            raw = owner.view(np.uint8).reshape(-1)
            off = share_offset_bytes(n0, T, D)
            raw[off: off + o.nbytes] = o.view(np.uint8).reshape(-1)
            owner.flush()
        dist.barrier()
    finally:
        dist.destroy_process_group()


@pytest.mark.parametrize("world,B", [(2, 5), (3, 7)])
def test_sharded_attention_shares_gloo(tmp_path, world, B):
    """ShardedAttention's partition on CPU ranks: every rank computes the attention of its samples
    (the oracle standing in for the fused kernels) and stores it at its share's byte offset in the
    owner's full-size buffer; the assembled output is the whole-batch result bit for bit (the shares
    tile the batch with no gap or overlap, and samples are independent)."""
    from nnb.parallel import sample_shares
    from oracle import orc

    T, D, H = 9, 8, 2
    shares = sample_shares(B, world)
    assert shares[0][0] == 0 and shares[-1][1] == B
    assert all(a[1] == b[0] for a, b in zip(shares, shares[1:]))
    assert max(e - s for s, e in shares) - min(e - s for s, e in shares) <= 1
    path = tmp_path / "owner_o.bin"
    np.zeros((B, T, D), np.float32).tofile(path)
    mp.start_processes(_attn_share_worker, args=(world, _free_port(), B, T, D, H, str(path)), nprocs=world, join=True,
                       start_method="spawn")
    got = np.fromfile(path, np.float32).reshape(B, T, D)
    q, k, v = (orc.normal(310 + j, B * T * D).reshape(B, T, D) for j in range(3))
    want = np.zeros((B, T, D), np.float32)
    probs = np.zeros((B, H, T, T), np.float32)
    orc.orc.orc_attention_fwd(B, T, T, D, H, orc.ptr(q), orc.ptr(k), orc.ptr(v), None, 1, orc.ptr(want), orc.ptr(probs))
    assert got.tobytes() == want.tobytes()
