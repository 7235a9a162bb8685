"""Multi-GPU plumbing for the sharded GEMM (one process per GPU, torch.distributed).

The reference has no distributed code; its only parallelism is the thread pool, whose results do
not depend on the thread count (tests/test_kernels.cpp:343-380). The B200 build keeps that
guarantee across GPU counts: a large GEMM is split into contiguous bands of whole 128-row tiles of
C (and A); every rank holds all of B and computes its band with the same tile sequence and k order
as the single-GPU kernel, so the bands are bitwise the rows the single-GPU product would hold.
Bands are gathered to one rank with a collective of the process group (NCCL over NVLink on GPUs,
gloo on CPU in the tests).
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
