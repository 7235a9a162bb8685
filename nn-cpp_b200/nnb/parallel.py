"""Multi-GPU plumbing for the sharded GEMM (one process per GPU, torch.distributed).

The reference has no distributed code; its only parallelism is the thread pool, whose results do
not depend on the thread count (tests/test_kernels.cpp:343-380). The B200 build keeps that
guarantee across GPU counts: a large GEMM is split into contiguous bands of whole 128-row tiles of
C (and A); every rank holds all of B and computes its band with the same tile sequence and k order
as the single-GPU kernel, so the bands are bitwise the rows the single-GPU product would hold.
Bands reach the gathering rank in one of two ways:
- fused: the gathering rank's full C is exported as CUDA IPC memory (PeerBuffer) and every rank runs
  its GEMM with C pointing into it, so the kernel's epilogue stores each finished tile straight into
  that GPU's memory over NVLink while the next tiles are computed -- the transfer overlaps the math
  tile by tile and no collective moves data;
- collective: gather_rows, an NCCL gather after the GEMM (gloo on CPU in the tests).
"""
from __future__ import annotations

TILE_ROWS = 128


def row_bands(m: int, world: int, align: int = TILE_ROWS) -> list[tuple[int, int]]:
    """Contiguous [start, stop) row bands, one per rank, in whole `align`-row tiles where possible.

    Tiles are dealt out as evenly as possible (earlier ranks take the extra tile); the last band
    ends at m. Ranks beyond the tile count get empty bands.
    """
    if world < 1:
        raise ValueError("world must be at least 1")
    tiles = (m + align - 1) // align
    base, extra = divmod(tiles, world)
    bands, start = [], 0
    for r in range(world):
        count = base + (1 if r < extra else 0)
        stop = min(m, start + count * align)
        bands.append((start, stop))
        start = stop
    return bands


def gather_rows(band, bands, dst: int = 0, group=None):
    """Gathers each rank's band of rows into the full matrix on rank `dst` (None elsewhere).

    `band` is this rank's [rows, cols] tensor; every rank takes part. Bands of unequal height are
    padded to the tallest band for the collective and trimmed again on `dst`.
    """
    import torch
    import torch.distributed as dist

    rank, world = dist.get_rank(group), dist.get_world_size(group)
    cols = band.shape[1]
    tallest = max(stop - start for start, stop in bands)
    send = band
    if band.shape[0] != tallest:
        send = torch.zeros(tallest, cols, dtype=band.dtype, device=band.device)
        send[: band.shape[0]] = band
    recv = [torch.empty(tallest, cols, dtype=band.dtype, device=band.device) for _ in range(world)] if rank == dst else None
    dist.gather(send.contiguous(), recv, dst=dst, group=group)
    if rank != dst:
        return None
    return torch.cat([recv[r][: stop - start] for r, (start, stop) in enumerate(bands)], dim=0)


class PeerBuffer:
    """A float32 buffer of `shape` on rank `owner` that every rank of the group can store into.

    The owner allocates it (``tensor``) and exports a CUDA IPC handle (nnb_ipc_export); the handle is
    broadcast over the process group and the other ranks map it (nnb_ipc_open). ``ptr`` is the
    buffer's address on this rank: the owner's own pointer, or the mapped peer pointer. ``close()``
    unmaps on every rank and then synchronises the group, after which the owner may free the tensor.
    """

    def __init__(self, shape, owner: int = 0, group=None, device=None):
        import ctypes

        import torch
        import torch.distributed as dist

        from . import check, lib

        self.group, self.owner = group, owner
        self.rank = dist.get_rank(group)
        device = device or torch.device("cuda", torch.cuda.current_device())
        self.tensor = torch.empty(tuple(shape), dtype=torch.float32, device=device) if self.rank == owner else None
        msg = torch.zeros(72, dtype=torch.uint8, device=device)
        if self.rank == owner:
            handle = (ctypes.c_ubyte * 64)()
            offset = ctypes.c_size_t()
            check(lib().nnb_ipc_export(self.tensor.data_ptr(), handle, ctypes.byref(offset)))
            msg[:64] = torch.tensor(list(handle), dtype=torch.uint8)
            msg[64:] = torch.tensor(list(offset.value.to_bytes(8, "little")), dtype=torch.uint8)
        dist.broadcast(msg, src=owner, group=group)
        raw = bytes(msg.cpu().tolist())
        self.offset = int.from_bytes(raw[64:], "little")
        if self.rank == owner:
            self.ptr, self._mapped = self.tensor.data_ptr(), False
        else:
            handle = (ctypes.c_ubyte * 64).from_buffer_copy(raw[:64])
            out = ctypes.c_void_p()
            check(lib().nnb_ipc_open(handle, self.offset, ctypes.byref(out)))
            self.ptr, self._mapped = out.value, True

    def close(self) -> None:
        import torch
        import torch.distributed as dist

        from . import check, lib

        torch.cuda.synchronize()
        if self._mapped:
            check(lib().nnb_ipc_close(self.ptr, self.offset))
            self._mapped = False
        dist.barrier(group=self.group, device_ids=[torch.cuda.current_device()])


def sample_shares(batch: int, world: int) -> list[tuple[int, int]]:
    """The attention workload's partition: rank r holds samples [n0, n1) of the global batch, contiguous
    runs as equal as possible in rank order (all heads of a sample stay on one rank)."""
    return row_bands(batch, world, align=1)


def share_offset_bytes(n0: int, T: int, D: int) -> int:
    """Byte offset of sample n0 in a [batch, T, D] fp32 buffer: where a rank's share of O / dQ / dK /
    dV lands in the owner's full-size buffers."""
    return n0 * T * D * 4


class ShardedAttention:
    """Multi-head attention forward + backward of a batch split by samples over the ranks, with O, dQ,
    dK and dV gathered on rank `owner` (the batch x head partition of the attention workload).

    Each rank holds q, k, v and the upstream gradient for its samples [n0, n1) of the global batch of
    `batch` samples. The owner's full-size O, dQ, dK and dV are PeerBuffers: the backward kernels'
    epilogues store this rank's dQ / dK / dV tiles straight into them over NVLink, and O (written
    locally, since the backward reads it) is copied to the owner by a peer copy that overlaps the
    backward. Every (sample, head) is computed exactly as on one GPU, so the gathered results are
    bitwise the one-GPU ones. Head size 64 runs the fused kernels.
    """

    def __init__(self, batch: int, T: int, D: int, heads: int, causal: bool = True, owner: int = 0, group=None,
                 device=None):
        import torch
        import torch.distributed as dist

        from . import lib

        if not lib().nnb_flash_attention_supported(D, heads):
            raise ValueError("ShardedAttention: the fused kernels need head size 64")
        self.rank, self.world = dist.get_rank(group), dist.get_world_size(group)
        self.batch, self.T, self.D, self.heads, self.causal = batch, T, D, heads, causal
        self.device = device or torch.device("cuda", torch.cuda.current_device())
        self.bands = sample_shares(batch, self.world)
        self.n0, self.n1 = self.bands[self.rank]
        self.local = self.n1 - self.n0
        self.out, self.dq, self.dk, self.dv = (PeerBuffer((batch, T, D), owner, group, self.device) for _ in range(4))
        self.o_local = torch.empty(max(self.local, 1), T, D, device=self.device)
        self.stats = torch.empty(max(self.local, 1), heads, T, 2, device=self.device)
        self.copy_stream = torch.cuda.Stream(self.device)
        self.group = group

    def _at(self, buf: "PeerBuffer") -> int:
        return buf.ptr + share_offset_bytes(self.n0, self.T, self.D)

    def step(self, q, k, v, go) -> None:
        """Forward and backward of this rank's samples (q, k, v, go: [local, T, D] on this device),
        enqueued on the current stream; the owner's buffers hold them once every rank's stream has
        passed this point (synchronise and barrier before reading)."""
        import torch

        from . import check, lib

        if self.local == 0:
            return
        L, s = lib(), torch.cuda.current_stream(self.device)
        N, T, D, H = self.local, self.T, self.D, self.heads
        check(L.nnb_flash_attention_fwd(s.cuda_stream, N, T, T, D, H, q.data_ptr(), k.data_ptr(), v.data_ptr(), None,
                                        int(self.causal), self.o_local.data_ptr(), self.stats.data_ptr()))
        # O to the owner on the copy stream (a copy-engine peer copy) while the backward runs
        self.copy_stream.wait_stream(s)
        check(L.nnb_copy_async(self.copy_stream.cuda_stream, self._at(self.out), self.o_local.data_ptr(), N * T * D * 4))
        check(L.nnb_flash_attention_bwd(s.cuda_stream, N, T, T, D, H, go.data_ptr(), q.data_ptr(), k.data_ptr(),
                                        v.data_ptr(), self.o_local.data_ptr(), self.stats.data_ptr(), None,
                                        int(self.causal), self._at(self.dq), 1, self._at(self.dk), 1,
                                        self._at(self.dv), 1))
        s.wait_stream(self.copy_stream)

    def close(self) -> None:
        for b in (self.out, self.dq, self.dk, self.dv):
            b.close()
