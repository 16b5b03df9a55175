"""LMNet FP32 stage throughput: the mask-generation UNet (LMNET_CONFIG,
mlx_model.py:69) on the 64 x 152 x 152 crop (mlx_pipeline.py:20) in FP32,
sampled with DDIM or DPM++-2M as the reference's _run_lmnet does
(medmlx.py:1168-1257).  One JSON line.

    python -m lesiondiffusion_mlx_b200.lmnet_bench [--steps 200] [--sampler ddim|dpm]

Random-init He-normal FP32 weights (seed 400); the conditioning channels are
synthetic (anatomy labels / 104, an ellipsoidal organ, a box inside it); the
condition is 8 context vectors of width 768 ~ N(0, 1).  The whole trajectory
runs as graph replays of one captured step (UNet + fused sampler update) and
is timed with CUDA events; a second capture of one step with event pairs
around every conv / attention launch gives the per-kind breakdown.
"""

from __future__ import annotations

import argparse
import json

import numpy as np
import torch

from . import _lib, instrument, workloads
from .networks import LdmUnetB200, UnetConfig
from .sampling import DdimSampler, Dpmpp2mSampler, PreparedSampler

LMNET_CONFIG = UnetConfig(16, 1, (4,), (1, 2, 4), 32, False)
LMNET_CROP = (64, 152, 152)


def conditioning(shape: tuple[int, int, int], seed: int = 401) -> np.ndarray:
    """(1, D, H, W, 3) f32: anatomy label id / 104, organ mask, box mask."""
    rng = np.random.default_rng(seed)
    d, h, w = shape
    zz, yy, xx = np.meshgrid(np.linspace(-1, 1, d), np.linspace(-1, 1, h), np.linspace(-1, 1, w), indexing="ij")
    organ = (zz ** 2 / 0.6 + yy ** 2 / 0.5 + xx ** 2 / 0.5) < 1.0
    labels = rng.integers(0, 105, size=(d // 8 + 1, h // 8 + 1, w // 8 + 1))
    labels = np.repeat(np.repeat(np.repeat(labels, 8, 0), 8, 1), 8, 2)[:d, :h, :w]
    box = np.zeros(shape, dtype=bool)
    box[d // 2 - 6: d // 2 + 6, h // 2 - 12: h // 2 + 12, w // 2 - 12: w // 2 + 12] = True
    out = np.stack([labels / 104.0, organ, box & organ], axis=-1).astype(np.float32)
    return out[None]


def main() -> None:
    ap = argparse.ArgumentParser()
    ap.add_argument("--steps", type=int, default=200)
    ap.add_argument("--sampler", choices=("ddim", "dpm"), default="ddim")
    a = ap.parse_args()
    device = torch.device("cuda", 0)
    torch.cuda.set_device(device)
    raw = workloads.unet_weights(LMNET_CONFIG, 4, 1, 768, seed=400)
    unet = LdmUnetB200({k: torch.from_numpy(v) for k, v in raw.items()}, LMNET_CONFIG, device=device,
                       dtype=torch.float32)
    ctx = torch.from_numpy(np.random.default_rng(402).standard_normal((1, 8, 768)).astype(np.float32))
    cache = unet.prepare_context(ctx.to(device))
    betas = np.linspace(0.00085 ** 0.5, 0.012 ** 0.5, 1000, dtype=np.float64) ** 2
    alphas = np.cumprod(1.0 - betas).astype(np.float32)  # LMNet keeps its schedule in FP32
    sampler = DdimSampler(alphas, a.steps) if a.sampler == "ddim" else Dpmpp2mSampler(alphas, a.steps)
    cond = torch.from_numpy(conditioning(LMNET_CROP)).to(device)
    prepared = PreparedSampler(sampler, unet, cache, cond, None, graph=True)
    gen = torch.Generator(device=device).manual_seed(403)
    init = torch.randn(prepared.state.x.shape, generator=gen, device=device)
    noise = torch.randn(prepared.state.noise.shape, generator=gen, device=device)

    prepared.begin(init, noise)
    launches0 = _lib.launch_count()
    prepared.capture()
    launches = _lib.launch_count() - launches0  # the warm-up step + the captured step
    out = prepared.run(init, noise)  # warm-up trajectory (graph already captured)
    torch.cuda.synchronize()
    start = torch.cuda.Event(enable_timing=True)
    end = torch.cuda.Event(enable_timing=True)
    start.record()
    out = prepared.run(init, noise)
    end.record()
    torch.cuda.synchronize()
    ms = start.elapsed_time(end)

    timer = instrument.KernelTimer()
    graph = torch.cuda.CUDAGraph()
    prepared.begin(init, noise)
    with instrument.timing(timer), torch.cuda.graph(graph):
        prepared._step()
    prepared.begin(init, noise)
    graph.replay()
    torch.cuda.synchronize()
    kinds = {k: {"launches": v["launches"], "ms": round(v["ms"], 4),
                 "tflops": round(v["flops"] / max(v["ms"], 1e-9) / 1e9, 1)} for k, v in timer.summary().items()}
    flops = sum(v["flops"] for v in timer.summary().values())
    print(json.dumps({
        "metric": "LMNet FP32 trajectory seconds", "value": ms / 1e3, "unit": "s", "sampler": a.sampler,
        "steps": a.steps, "ms_per_step": ms / a.steps, "crop": list(LMNET_CROP), "dtype": "f32 (split-f16 tensor cores)",
        "gpu_launches_per_step": launches // 2, "step_gflop": flops / 1e9,
        "kernel_ms_per_step_instrumented": kinds, "finite": bool(torch.isfinite(out).all().item()),
        "data": "synthetic (random-init LMNet weights seed 400, synthetic conditioning and context)",
    }), flush=True)


if __name__ == "__main__":
    main()
