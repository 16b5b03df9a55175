"""Per-kernel micro-benchmarks of the hot-path shapes (also the target of the
``ncu`` captures summarised under ``profiles/``).

    python -m lesiondiffusion_mlx_b200.kernel_cases [conv|attention|norm|all] [--case NAME] [--iters N]
    python -m lesiondiffusion_mlx_b200.kernel_cases step [--eager N]   # config-3 step launch table

Each case runs on seeded random inputs and prints one JSON line per case with
the CUDA-event time per launch (back-to-back launches replayed from a CUDA
graph, L2 warm) and the achieved TFLOP/s or GB/s of its algorithmic work.  Conv cases are the distinct 3x3x3 / strided / folded-up
layer shapes of the config-3 UNet (1 x 32 x 40 x 40 latent) plus BASELINE
config 1 (the FP32 conv op); attention cases are BASELINE config 2.
"""

from __future__ import annotations

import argparse
import json

import torch

from . import ops
from .conv import conv3d_ndhwc, pack_upsample_weight, pack_weight

# name: (D, H, W, Cin, Cout, kind) with kind conv / s2 / up / pw / exact
CONV_CASES = {
    "l0_128": (32, 40, 40, 128, 128, "conv"),
    "l0_in8": (32, 40, 40, 8, 128, "conv"),
    "l0_cat256": (32, 40, 40, 256, 128, "conv"),
    "down0": (32, 40, 40, 128, 128, "s2"),
    "l1_256": (16, 20, 20, 256, 256, "conv"),
    "l1_cat512": (16, 20, 20, 512, 256, "conv"),
    "down1": (16, 20, 20, 256, 256, "s2"),
    "l2_512": (8, 10, 10, 512, 512, "conv"),
    "l2_cat1024": (8, 10, 10, 1024, 512, "conv"),
    "up2": (8, 10, 10, 512, 512, "up"),
    "up1": (16, 20, 20, 256, 256, "up"),
    "out8": (32, 40, 40, 128, 8, "conv"),
    "ff1_512": (8, 10, 10, 512, 1024, "pw"),
    "qkv_256": (16, 20, 20, 256, 768, "pw"),
    "cfg1_fp32": (32, 40, 40, 128, 128, "exact"),
}

ATTN_CASES = {
    "self_6400_bf16": (1, 6400, 6400, 8, 64, torch.bfloat16),
    "cross_6400x77_bf16": (1, 6400, 77, 8, 64, torch.bfloat16),
    "self_6400_h4": (1, 6400, 6400, 4, 64, torch.float16),
    "self_800_h8": (1, 800, 800, 8, 64, torch.float16),
    "lmnet_self_23104_f32": (1, 23104, 23104, 2, 32, torch.float32),  # LMNet's FP32 level (16 x 38 x 38)
}


def _time(fn, iters: int) -> float:
    """Mean milliseconds per call: ``iters`` back-to-back calls captured in one
    CUDA graph and timed with CUDA events (no host launch overhead inside the
    timed region; L2 is warm across calls)."""
    for _ in range(3):
        fn()
    torch.cuda.synchronize()
    graph = torch.cuda.CUDAGraph()
    with torch.cuda.graph(graph):
        for _ in range(iters):
            fn()
    graph.replay()
    torch.cuda.synchronize()
    s = torch.cuda.Event(enable_timing=True)
    e = torch.cuda.Event(enable_timing=True)
    s.record()
    graph.replay()
    e.record()
    torch.cuda.synchronize()
    return s.elapsed_time(e) / iters


def conv_case(name: str, iters: int, stats: bool = False) -> dict:
    d, h, w, cin, cout, kind = CONV_CASES[name]
    g = torch.Generator(device="cuda").manual_seed(0)
    exact = kind == "exact"
    wt = torch.randn((cout, cin, *((1, 1, 1) if kind == "pw" else (3, 3, 3))), generator=g, device="cuda")
    wt = wt * (cin * wt[0, 0].numel()) ** -0.5
    bias = torch.randn(cout, generator=g, device="cuda") * 0.02
    if exact:
        x32 = torch.randn((1, d, h, w, cin), generator=g, device="cuda")
        x = ops.prepare_input(x32, split=True)
        packed = pack_weight(wt.float())
    else:
        x = torch.randn((1, d, h, w, cin), generator=g, device="cuda").to(torch.float16)
        packed = pack_upsample_weight(wt.half()) if kind == "up" else pack_weight(wt.half(), stride=2 if kind == "s2" else 1)
    stride = 2 if kind == "s2" else 1
    st = torch.zeros((1, cout, 2), dtype=torch.float64, device="cuda") if stats else None
    fn = lambda: conv3d_ndhwc(x, packed, bias, stride=stride, in_channels=cin, stats=st)  # noqa: E731
    ms = _time(fn, iters)
    out_vox = {"s2": ((d + 1) // 2) * ((h + 1) // 2) * ((w + 1) // 2), "up": 8 * d * h * w}.get(kind, d * h * w)
    taps = {"pw": 1, "up": 8}.get(kind, 27)
    flops = 2.0 * out_vox * cout * taps * cin
    return {"kernel": "conv3d+stats" if stats else "conv3d", "case": name, "shape": [d, h, w, cin, cout],
            "kind": kind, "ms": ms,
            "tflops": flops / ms / 1e9, "gflop": flops / 1e9}


def attn_case(name: str, iters: int) -> dict:
    b, lq, lk, heads, dim, dtype = ATTN_CASES[name]
    g = torch.Generator(device="cuda").manual_seed(1)
    q = torch.randn((b, lq, heads * dim), generator=g, device="cuda").to(dtype)
    k = torch.randn((b, lk, heads * dim), generator=g, device="cuda").to(dtype)
    v = torch.randn((b, lk, heads * dim), generator=g, device="cuda").to(dtype)
    fn = lambda: ops.flash_attention(q, k, v, heads=heads, scale=dim ** -0.5)  # noqa: E731
    ms = _time(fn, iters)
    flops = 4.0 * b * heads * lq * lk * dim
    nbytes = 2.0 * b * (lq + 2 * lk + lq) * heads * dim
    return {"kernel": "attention", "case": name, "ms": ms, "tflops": flops / ms / 1e9, "gbs": nbytes / ms / 1e6}


def norm_case(iters: int) -> list[dict]:
    out = []
    for d, h, w, c in ((32, 40, 40, 128), (16, 20, 20, 512), (8, 10, 10, 1024)):
        x = torch.randn((1, d, h, w, c), device="cuda").to(torch.float16)
        gam = torch.ones(c, device="cuda")
        ms_gn = _time(lambda: ops.group_norm_affine(x, gam, gam, groups=32, eps=1e-5), iters)
        aff = ops.group_norm_affine(x, gam, gam, groups=32, eps=1e-5)
        ms_pr = _time(lambda: ops.prepare_input(x, affine=aff, silu=True), iters)
        xs = x.double().reshape(1, -1, c)
        st = torch.stack([xs.sum(1), (xs * xs).sum(1)], dim=-1).contiguous()
        ms_af = _time(lambda: ops.group_norm_affine_from_stats(st, gam, gam, voxels=d * h * w, groups=32, eps=1e-5),
                      iters)
        nbytes = x.numel() * 2
        out.append({"kernel": "group_norm_stats", "shape": [d, h, w, c], "ms": ms_gn, "gbs": nbytes / ms_gn / 1e6})
        out.append({"kernel": "prepare", "shape": [d, h, w, c], "ms": ms_pr, "gbs": 2 * nbytes / ms_pr / 1e6})
        out.append({"kernel": "group_norm_affine_from_stats", "shape": [d, h, w, c], "ms": ms_af})
    return out


def _config3_step():
    """The config-3 denoise step of ``bench.py``: UNet (seed 100) + fused DDIM update, prepared."""
    from pathlib import Path

    import numpy as np

    from . import workloads
    from .networks import LdmUnetB200
    from .sampling import DdimSampler, PreparedSampler

    golden = Path(__file__).resolve().parents[1] / "tests" / "golden" / "reference_fixtures.npz"
    with np.load(golden, allow_pickle=False) as archive:
        alphas = archive["dpmpp_2m/linet_4.alphas_cumprod"]
    dev = torch.device("cuda", torch.cuda.current_device())
    cfg = workloads.CONFIG3
    raw = workloads.unet_weights(cfg, 8, 8, 768, seed=100)
    unet = LdmUnetB200({k: torch.from_numpy(v).half() for k, v in raw.items()}, cfg, device=dev)
    inp = workloads.config3_inputs(seed=101)
    cache = unet.prepare_context(torch.from_numpy(inp["context"]).to(dev))
    image = torch.from_numpy(workloads.source_latent((1, 7, 32, 40, 40), seed=300)).permute(0, 2, 3, 4, 1)
    prepared = PreparedSampler(DdimSampler(alphas, 200), unet, cache, image.to(dev),
                               torch.from_numpy(inp["mask"][:, 0]).to(dev), graph=False)
    g = torch.Generator(device=dev).manual_seed(1000)
    prepared.begin(torch.randn(prepared.state.x.shape, generator=g, device=dev),
                   torch.randn(prepared.state.noise.shape, generator=g, device=dev))
    return prepared


def step_case(eager: int, iters: int) -> list[dict]:
    """``eager`` > 0: that many eager config-3 steps (every launch separate, for
    ncu).  Otherwise: the step as a CUDA graph, its mean time over ``iters``
    replays, and one row per launch kind and shape from the device-clock
    timer (conv and attention launches time themselves; the rest have event
    pairs, which add gaps)."""
    from . import instrument

    prepared = _config3_step()
    # every step below advances the schedule's device step counter: stay inside its tables
    executed = eager if eager > 0 else iters + 7
    if executed > prepared.sampler.steps:
        raise ValueError(f"{executed} steps exceed the {prepared.sampler.steps}-step schedule")
    if eager > 0:
        for _ in range(eager):
            prepared._step()
        torch.cuda.synchronize()
        return [{"kernel": "config3_step", "eager_steps": eager}]
    timer = instrument.KernelTimer(device_clock=True)
    timer.arm(prepared.state.x.device)
    prepared._step()
    torch.cuda.synchronize()
    timed = torch.cuda.CUDAGraph()
    with instrument.timing(timer), torch.cuda.graph(timed):
        prepared._step()
    ms = _time(prepared._step, iters)
    for _ in range(3):
        timer.reset()
        timed.replay()
    torch.cuda.synchronize()
    rows: dict[tuple[str, str], list[float]] = {}
    for kind, label, flops, t in timer.launches():
        r = rows.setdefault((kind, label), [0, 0.0, 0.0])
        r[0] += 1
        r[1] += t
        r[2] += flops
    out = [{"kernel": "config3_step", "ms_per_step": ms}]
    for (kind, label), (n, t, flops) in sorted(rows.items(), key=lambda kv: -kv[1][1]):
        out.append({"kernel": kind, "shape": label, "launches": n, "ms": t, "us_per_launch": 1e3 * t / n,
                    "tflops": flops / t / 1e9 if t and flops else None})
    return out


def main() -> None:
    ap = argparse.ArgumentParser()
    ap.add_argument("what", nargs="?", default="all", choices=("conv", "attention", "norm", "step", "all"))
    ap.add_argument("--case", default=None)
    ap.add_argument("--iters", type=int, default=10)
    ap.add_argument("--stats", action="store_true", help="conv cases also accumulate GroupNorm statistics")
    ap.add_argument("--eager", type=int, default=0, help="step: run this many eager steps (for ncu) and exit")
    a = ap.parse_args()
    if a.what == "step":
        for r in step_case(a.eager, a.iters):
            print(json.dumps(r), flush=True)
        return
    if a.what in ("conv", "all"):
        for name in ([a.case] if a.case else CONV_CASES):
            print(json.dumps(conv_case(name, a.iters, stats=a.stats)), flush=True)
    if a.what in ("attention", "all"):
        for name in ([a.case] if a.case and a.what == "attention" else ATTN_CASES):
            print(json.dumps(attn_case(name, a.iters)), flush=True)
    if a.what in ("norm", "all"):
        for r in norm_case(a.iters):
            print(json.dumps(r), flush=True)


if __name__ == "__main__":
    main()
