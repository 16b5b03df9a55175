"""Depth-sharded VQ decode on the GPU: the decode over depth slabs (halo
exchange before every 3x3x3 / upsampling conv, GroupNorm statistics summed
over all slabs) against the unsharded decode and the CPU oracle.

On one GPU the ranks are emulated in one process (``LocalDepthComm``); with
two or more GPUs the NCCL communicator runs one process per GPU."""

from __future__ import annotations

import socket
import tempfile
from pathlib import Path

import numpy as np
import pytest
import torch
import torch.multiprocessing as mp

from oracle.networks import OracleVq, torch_weights
from tests.golden.fixture_weights import vq_fixture_weights

pytestmark = pytest.mark.gpu


def rel_l2(a, b) -> float:
    a = np.asarray(a, np.float64)
    b = np.asarray(b, np.float64)
    return float(np.linalg.norm(a - b) / max(np.linalg.norm(b), 1e-30))


def _decoder(device, scaled: bool = False):
    from lesiondiffusion_mlx_b200.networks import VqDecoderB200

    raw = vq_fixture_weights(7)
    dec = VqDecoderB200(torch_weights({k: v for k, v in raw.items() if not k.startswith("encoder")}, torch.float16),
                        device=device, scaled=scaled)
    return dec, raw


def _latent(depth: int, seed: int = 5) -> np.ndarray:
    return np.random.default_rng(seed).standard_normal((1, 4, depth, 6, 5)).astype(np.float32)


def _ndhwc(z: np.ndarray, device) -> torch.Tensor:
    t = torch.from_numpy(z).permute(0, 2, 3, 4, 1).to(torch.float16)
    buf = torch.zeros((*t.shape[:-1], 8), dtype=torch.float16)
    buf[..., :4] = t
    return buf.to(device)[..., :4]


@pytest.mark.parametrize("scaled", [False, True])
@pytest.mark.parametrize("parts", [1, 2, 3])
def test_emulated_slabs_match_unsharded_decode(cuda_device, parts, scaled):
    from lesiondiffusion_mlx_b200.sharded_decode import LocalDepthComm, ShardedVqDecoder, partition_depth

    dec, raw = _decoder(cuda_device, scaled)
    depth = 9
    z = _latent(depth)
    zd = _ndhwc(z, cuda_device)
    whole = dec.decode(zd).float()
    slabs = [zd[:, a:b] for a, b in partition_depth(depth, parts)]
    outs = ShardedVqDecoder(dec, LocalDepthComm()).decode(slabs, depth)
    torch.cuda.synchronize()
    got = torch.cat([o.float() for o in outs], dim=1)
    assert got.shape == whole.shape
    assert rel_l2(got.cpu().numpy(), whole.cpu().numpy()) <= 2e-3
    oracle = OracleVq(torch_weights(raw, torch.float16), scaled=scaled)
    ref = oracle.decode(torch.from_numpy(z).to(torch.float16)).float().numpy()
    assert rel_l2(got.permute(0, 4, 1, 2, 3).cpu().numpy(), ref) <= 1e-2


def _free_port() -> int:
    with socket.socket() as s:
        s.bind(("127.0.0.1", 0))
        return s.getsockname()[1]


def _nccl_worker(rank: int, world: int, port: int, depth: int, out_dir: str) -> None:
    import datetime

    import torch.distributed as dist

    from lesiondiffusion_mlx_b200.sharded_decode import DistDepthComm, ShardedVqDecoder, partition_depth

    torch.cuda.set_device(rank)
    dist.init_process_group("nccl", init_method=f"tcp://127.0.0.1:{port}", rank=rank, world_size=world,
                            timeout=datetime.timedelta(seconds=120), device_id=torch.device("cuda", rank))
    device = torch.device("cuda", rank)
    dec, _ = _decoder(device)
    a, b = partition_depth(depth, world)[rank]
    zd = _ndhwc(_latent(depth), device)[:, a:b]
    (out,) = ShardedVqDecoder(dec, DistDepthComm()).decode([zd], depth)
    torch.cuda.synchronize()
    torch.save(out.float().cpu(), Path(out_dir) / f"slab{rank}.pt")
    dist.barrier()
    dist.destroy_process_group()


def test_nccl_slabs_match_unsharded_decode(cuda_device):
    world = min(torch.cuda.device_count(), 4)
    if world < 2:
        pytest.skip("needs two or more GPUs (the one-GPU emulation is covered above)")
    from lesiondiffusion_mlx_b200.sharded_decode import partition_depth

    depth = 9
    with tempfile.TemporaryDirectory() as tmp:
        mp.start_processes(_nccl_worker, args=(world, _free_port(), depth, tmp), nprocs=world, join=True,
                           start_method="spawn")
        got = torch.cat([torch.load(Path(tmp) / f"slab{r}.pt") for r in range(world)], dim=1)
    dec, _ = _decoder(cuda_device)
    whole = dec.decode(_ndhwc(_latent(depth), cuda_device)).float().cpu()
    assert len(partition_depth(depth, world)) == world
    assert rel_l2(got.numpy(), whole.numpy()) <= 2e-3
