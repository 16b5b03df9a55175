"""End-to-end generation throughput (config 5): seeds -> denoising trajectory
-> VQ decode -> HU volume, as volumes per minute.

    python -m lesiondiffusion_mlx_b200.e2e_bench [--seeds 8] [--batch 1] [--sampler ddim|dpm]
    torchrun --nproc-per-node N -m lesiondiffusion_mlx_b200.e2e_bench --seeds 64 --batch 8

Each rank takes every N-th seed (no collective on the data path).  A batch of
seeds runs the config-3 UNet with the fused sampler step as one CUDA graph
per step (DDIM 200 steps with injected per-step noise, or DPM++-2M 50
steps), then the config-4 decoder turns the final latent (the 7 denoised
channels plus the mask channel, 8 channels as the decoder expects) into a
1 x 128 x 160 x 160 HU volume.  Random-init weights (UNet seed 100, decoder
seed 200), seeded inputs; the known latent is smoothed N(0, 1) (seed 300)
and the mask the 8 x 8 x 5 box of the config-3 inputs.  The schedule is the
real LINet ``alphas_cumprod`` (f16).  The whole run is timed with CUDA
events, max over ranks.
"""

from __future__ import annotations

import argparse
import datetime
import json
import os
from pathlib import Path

import numpy as np
import torch

from . import ops, workloads
from .networks import LdmUnetB200, VqDecoderB200
from .sampling import DdimSampler, Dpmpp2mSampler, PreparedSampler


GOLDEN = Path(__file__).resolve().parents[1] / "tests" / "golden" / "reference_fixtures.npz"


def _alphas() -> np.ndarray:
    """The real LINet ``alphas_cumprod`` (1000 entries, f16) from the reference's
    DPM++ recording, the schedule config 5 names."""
    with np.load(GOLDEN, allow_pickle=False) as archive:
        return archive["dpmpp_2m/linet_4.alphas_cumprod"]


def main() -> None:
    ap = argparse.ArgumentParser()
    ap.add_argument("--seeds", type=int, default=8)
    ap.add_argument("--batch", type=int, default=1)
    ap.add_argument("--sampler", choices=("ddim", "dpm"), default="ddim")
    ap.add_argument("--no-decode", action="store_true")
    a = ap.parse_args()

    world = int(os.environ.get("WORLD_SIZE", "1"))
    rank = int(os.environ.get("RANK", "0"))
    local = int(os.environ.get("LOCAL_RANK", "0"))
    torch.cuda.set_device(local)
    device = torch.device("cuda", local)
    dist = None
    if world > 1:
        import torch.distributed as dist

        dist.init_process_group("nccl", timeout=datetime.timedelta(seconds=600), device_id=device)

    cfg = workloads.CONFIG3
    raw = workloads.unet_weights(cfg, 8, 8, 768, seed=100)
    unet = LdmUnetB200({k: torch.from_numpy(v) for k, v in raw.items()}, cfg, device=device)
    dec = None
    if not a.no_decode:
        dec = VqDecoderB200({k: torch.from_numpy(v) for k, v in workloads.config4_decoder_weights().items()},
                            device=device, groups=32)
    inp = workloads.config3_inputs(seed=101, batch=a.batch)
    cache = unet.prepare_context(torch.from_numpy(inp["context"]).to(device))
    steps = 200 if a.sampler == "ddim" else 50
    sampler = DdimSampler(_alphas(), steps) if a.sampler == "ddim" else Dpmpp2mSampler(_alphas(), steps)
    _, c, d, h, w = workloads.CONFIG3_LATENT
    image = torch.from_numpy(workloads.source_latent((a.batch, c - 1, d, h, w), seed=300)).permute(0, 2, 3, 4, 1)
    mask = torch.from_numpy(inp["mask"][:, 0])
    prepared = PreparedSampler(sampler, unet, cache, image.to(device), mask.to(device), graph=True)
    mine = list(range(rank, a.seeds, world))
    batches = [mine[i: i + a.batch] for i in range(0, len(mine), a.batch)]
    zlat = torch.zeros((a.batch, d, h, w, 8), dtype=torch.float16, device=device)
    mask_d = mask.to(device, torch.float16)

    def run_batch(seeds: list[int]) -> torch.Tensor | None:
        gen = torch.Generator(device=device).manual_seed(1000 + seeds[0])
        init = torch.randn(prepared.state.x.shape, generator=gen, device=device)
        noise = torch.randn(prepared.state.noise.shape, generator=gen, device=device) \
            if a.sampler == "ddim" else None
        x = prepared.run(init, noise)
        if dec is None:
            return None
        zlat[..., : c - 1].copy_(x)
        zlat[..., c - 1].copy_(mask_d)
        return ops.hu_map(dec.decode(zlat, quantize=False))

    run_batch(batches[0] if batches else [rank])  # warm-up: graph capture, first-use packing
    torch.cuda.synchronize()
    if dist is not None:
        dist.barrier()
    start = torch.cuda.Event(enable_timing=True)
    end = torch.cuda.Event(enable_timing=True)
    start.record()
    out = None
    for seeds in batches:
        out = run_batch(seeds)
    end.record()
    torch.cuda.synchronize()
    ms = start.elapsed_time(end)
    if dist is not None:
        t = torch.tensor([ms], device=device)
        dist.all_reduce(t, op=dist.ReduceOp.MAX)
        ms = float(t.item())
    volumes = len(range(0, a.seeds)) if world > 1 else len(mine)
    if rank == 0:
        print(json.dumps({
            "metric": "volumes/min", "value": volumes / (ms / 1e3) * 60.0, "n_gpus": world, "seeds": a.seeds,
            "batch_per_gpu": a.batch, "sampler": a.sampler, "steps": steps, "decode": dec is not None,
            "ms_total": ms, "ms_per_volume_per_gpu": ms / max(1, len(mine)),
            "output": [1, 1, 128, 160, 160] if dec is not None else None,
            "finite": bool(out is None or torch.isfinite(out).all().item()),
            "data": "synthetic (random-init UNet seed 100, decoder seed 200, seeded noise)",
        }), flush=True)
    if dist is not None:
        dist.barrier()
        dist.destroy_process_group()


if __name__ == "__main__":
    main()
