"""Host logic of the depth-sharded decode, without a GPU: the slab partition
and the torch.distributed communicator (halo exchange, statistics all-reduce)
on gloo ranks over CPU tensors."""

from __future__ import annotations

import socket

import pytest
import torch
import torch.multiprocessing as mp

from lesiondiffusion_mlx_b200.sharded_decode import LocalDepthComm, partition_depth


def test_partition_depth_is_contiguous_and_balanced():
    for depth, parts in [(62, 8), (62, 1), (8, 8), (31, 4), (10, 3)]:
        slabs = partition_depth(depth, parts)
        assert slabs[0][0] == 0 and slabs[-1][1] == depth
        assert all(a[1] == b[0] for a, b in zip(slabs, slabs[1:]))
        sizes = [b - a for a, b in slabs]
        assert max(sizes) - min(sizes) <= 1 and min(sizes) >= 1
    with pytest.raises(ValueError):
        partition_depth(3, 4)


def test_partition_depth_gives_leftover_slices_to_the_end_slabs():
    """An end slab exchanges one halo per conv, an inner slab two: the slices
    left after an even split go to the end slabs first, then inwards."""
    sizes = lambda depth, parts: [b - a for a, b in partition_depth(depth, parts)]  # noqa: E731
    assert sizes(62, 4) == [16, 15, 15, 16]
    assert sizes(62, 8) == [8, 8, 8, 7, 7, 8, 8, 8]
    assert sizes(10, 3) == [4, 3, 3]
    assert sizes(11, 3) == [4, 3, 4]
    assert sizes(9, 3) == [3, 3, 3]


def _volume(depth: int) -> torch.Tensor:
    # (1, depth, 3, 2, 8) with every slice distinct
    return torch.arange(depth * 3 * 2 * 8, dtype=torch.float32).reshape(1, depth, 3, 2, 8)


def _padded(vol: torch.Tensor, start: int, stop: int) -> torch.Tensor:
    buf = torch.zeros((1, stop - start + 2, *vol.shape[2:]), dtype=vol.dtype)
    buf[:, 1:-1] = vol[:, start:stop]
    return buf


def _expected(vol: torch.Tensor, start: int, stop: int) -> torch.Tensor:
    want = torch.zeros((1, stop - start + 2, *vol.shape[2:]), dtype=vol.dtype)
    lo, hi = max(start - 1, 0), min(stop + 1, vol.shape[1])
    want[:, lo - (start - 1): hi - (start - 1)] = vol[:, lo:hi]
    return want


def test_local_exchange_fills_inner_halos_only():
    vol = _volume(10)
    slabs = partition_depth(10, 3)
    bufs = [_padded(vol, a, b) for a, b in slabs]
    LocalDepthComm().exchange(bufs)
    for (a, b), buf in zip(slabs, bufs):
        assert torch.equal(buf, _expected(vol, a, b))
    stats = [torch.full((1, 4, 2), float(i + 1), dtype=torch.float64) for i in range(3)]
    LocalDepthComm().all_reduce(stats)
    assert all(torch.equal(s, torch.full((1, 4, 2), 6.0, dtype=torch.float64)) for s in stats)


def _free_port() -> int:
    with socket.socket() as s:
        s.bind(("127.0.0.1", 0))
        return s.getsockname()[1]


def _dist_worker(rank: int, world: int, port: int, depth: int, errors) -> None:
    import torch.distributed as dist

    from lesiondiffusion_mlx_b200.sharded_decode import DistDepthComm

    try:
        dist.init_process_group("gloo", init_method=f"tcp://127.0.0.1:{port}", rank=rank, world_size=world)
        vol = _volume(depth)
        start, stop = partition_depth(depth, world)[rank]
        buf = _padded(vol, start, stop)
        comm = DistDepthComm()
        comm.exchange([buf])
        assert torch.equal(buf, _expected(vol, start, stop)), f"rank {rank} halo mismatch"
        stats = torch.full((1, 4, 2), float(rank + 1), dtype=torch.float64)
        comm.all_reduce([stats])
        assert torch.equal(stats, torch.full((1, 4, 2), world * (world + 1) / 2, dtype=torch.float64))
        dist.barrier()
        dist.destroy_process_group()
    except Exception as exc:  # reported to the parent
        errors.put(f"rank {rank}: {exc!r}")
        raise


@pytest.mark.parametrize("world,depth", [(2, 7), (3, 10)])
def test_dist_exchange_and_all_reduce_on_gloo_ranks(world, depth):
    ctx = mp.get_context("spawn")
    errors = ctx.SimpleQueue()
    mp.start_processes(_dist_worker, args=(world, _free_port(), depth, errors), nprocs=world, join=True,
                       start_method="spawn")
    assert errors.empty()
