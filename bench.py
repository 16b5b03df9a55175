#!/usr/bin/env python
"""Denoise-step benchmark of the B200 hot path (prints one JSON line).

Workload (the metric's "denoise steps/s at a 40x40x32
latent"): one conditioned-mode denoise step = the LINet-shaped 3-D UNet
forward (model channels 128, multipliers 1/2/4, 2 residual blocks, 64-wide
attention heads at 16x20x20 and 8x10x10, cross-attention to 77 x 768) on a
1 x 8 x 32 x 40 x 40 f16 latent (7 channels + mask) plus the fused DDIM
update (200-step schedule on the real LINet alphas), captured as one CUDA
graph and replayed.  Random-init weights (seed 100), synthetic inputs.

Multi-GPU: one process per GPU (torchrun); every rank runs its own
trajectory replica (seeds are data-parallel, no collective on the data
path), timing is the max over ranks, ``value`` is the steps/s of all ranks.

Besides the timed K steps the line carries: ``trajectory`` (one full
200-step DDIM trajectory plus the config-4a decode to HU, the north star's
"generation under 10 s" unit), ``decode_4b`` (the config-4b VQ decode:
unsharded at N = 1, depth-sharded over the N ranks with NCCL halo exchange
and GroupNorm all-reduces at N > 1), the conv ``roofline`` against the
measured burst bf16 peak (the step is milliseconds long), and at N = 1 the
CPU baseline.  Clocks are sampled from the start of the timed steps to the
end of the trajectory.

``--impl reference`` times the CPU restatement of the reference arithmetic
(``oracle/``, the reference itself is MLX/Metal-only) on the host cores, on
the same workload ``config``.
"""

from __future__ import annotations

import argparse
import json
import os
import statistics
import subprocess
import sys
import threading
import time
from pathlib import Path

import numpy as np
import torch

ROOT = Path(__file__).resolve().parent
sys.path.insert(0, str(ROOT))

METRIC = "denoise steps/s (config-3 UNet step + DDIM update, 1x8x32x40x40 latent)"
UNIT = "steps/s"
GOLDEN = ROOT / "tests" / "golden" / "reference_fixtures.npz"


def parse() -> argparse.Namespace:
    ap = argparse.ArgumentParser(description=__doc__)
    ap.add_argument("--gpus", type=int, default=1)
    ap.add_argument("--steps", type=int, default=40)
    ap.add_argument("--warmup", type=int, default=5)
    ap.add_argument("--impl", choices=("b200", "reference"), default="b200")
    ap.add_argument("--no-cpu-baseline", action="store_true", help="skip the CPU oracle timing (profiling runs)")
    return ap.parse_args()


def linet_alphas() -> np.ndarray:
    with np.load(GOLDEN, allow_pickle=False) as archive:
        return archive["dpmpp_2m/linet_4.alphas_cumprod"]  # the real LINet schedule, f16


class ClockSampler:
    """Sample nvidia-smi SM clocks and throttle reasons every 100 ms in a thread."""

    FIELDS = ("clocks.sm,clocks.max.sm,power.draw,clocks_event_reasons.active,clocks_event_reasons.hw_slowdown,"
              "clocks_event_reasons.hw_thermal_slowdown,clocks_event_reasons.sw_thermal_slowdown,"
              "clocks_event_reasons.sw_power_cap")

    def __init__(self, index: int):
        self.index = index
        self.proc = None
        self.lines: list[str] = []

    def start(self) -> None:
        try:
            self.proc = subprocess.Popen(
                ["nvidia-smi", "-i", str(self.index), f"--query-gpu={self.FIELDS}", "--format=csv,noheader,nounits",
                 "-lms", "100"], stdout=subprocess.PIPE, stderr=subprocess.DEVNULL, text=True)
            self.thread = threading.Thread(target=self._read, daemon=True)
            self.thread.start()
        except (OSError, ValueError):
            self.proc = None

    def _read(self) -> None:
        assert self.proc is not None and self.proc.stdout is not None
        for line in self.proc.stdout:
            self.lines.append(line.strip())

    def stop(self) -> dict:
        if self.proc is None:
            return {"sm_mhz": None, "sm_max_mhz": None, "reasons": ["nvidia-smi unavailable"]}
        self.proc.terminate()
        try:
            self.proc.wait(timeout=5)
        except subprocess.TimeoutExpired:
            self.proc.kill()
        sm, mx, reasons = [], [], set()
        names = ("active", "hw_slowdown", "hw_thermal_slowdown", "sw_thermal_slowdown", "sw_power_cap")
        for line in self.lines:
            parts = [p.strip() for p in line.split(",")]
            if len(parts) < 8:
                continue
            try:
                sm.append(float(parts[0]))
                mx.append(float(parts[1]))
            except ValueError:
                continue
            for name, val in zip(names[1:], parts[4:8]):
                if val.lower() == "active":
                    reasons.add(name)
        return {"sm_mhz": statistics.median(sm) if sm else None, "sm_max_mhz": max(mx) if mx else None,
                "reasons": sorted(reasons), "samples": len(sm)}


def dist_setup(n: int):
    if n <= 1 and int(os.environ.get("WORLD_SIZE", "1")) <= 1:
        return 0, 1, 0
    import datetime

    import torch.distributed as dist

    rank = int(os.environ["RANK"])
    world = int(os.environ["WORLD_SIZE"])
    local = int(os.environ.get("LOCAL_RANK", rank))
    torch.cuda.set_device(local)
    dist.init_process_group("nccl", timeout=datetime.timedelta(seconds=120), device_id=torch.device("cuda", local))
    return rank, world, local


_ORACLE: dict = {}


def config3_param_bytes() -> int:
    """f16 bytes of the config-3 UNet's weights."""
    from lesiondiffusion_mlx_b200 import workloads

    raw = workloads.unet_weights(workloads.CONFIG3, 8, 8, 768, seed=0, shapes_only=True)
    return int(sum(v.size * 2 for v in raw.values()))


def workload_config(world: int) -> dict:
    """The workload both arms report (identical dicts, so the two lines compare)."""
    return {
        "workload": "config3-unet-ddim-step", "latent": [1, 8, 32, 40, 40], "context": [1, 77, 768],
        "global_batch": world, "parallelism": f"replicas x{world} (independent seeds)",
        "l2": f"per-step working set > L2: {config3_param_bytes() / 1e6:.0f} MB of weights streamed every step",
        "graph": "one CUDA graph per step (UNet forward + fused DDIM update)",
        "schedule": "DDIM 200 steps, eta 1, real LINet alphas_cumprod",
    }


def cpu_step_time(depth: int, threads: int) -> tuple[float, dict]:
    """Seconds per oracle (CPU, FP32) config-3 UNet step + DDIM update on a depth-cropped latent."""
    from lesiondiffusion_mlx_b200 import workloads
    from oracle import samplers as osamp
    from oracle.networks import OracleUnet, UnetConfig, torch_weights

    torch.set_num_threads(threads)
    if "model" not in _ORACLE:
        cfg = workloads.CONFIG3
        raw = workloads.unet_weights(cfg, 8, 8, 768, seed=100)
        model = OracleUnet(torch_weights(raw, torch.float16),
                           UnetConfig(cfg.model_channels, cfg.num_res_blocks, cfg.attention_resolutions,
                                      cfg.channel_mult, cfg.num_head_channels, cfg.skip_context),
                           compute=torch.float32)
        inp = workloads.config3_inputs()
        _ORACLE["model"] = model
        _ORACLE["inp"] = inp
        _ORACLE["coeffs"] = osamp.ddim_coefficients(linet_alphas(), 200)
        _ORACLE["kv"] = model.project_context(torch.from_numpy(inp["context"]), torch.float16)
    model, inp, coeffs = _ORACLE["model"], _ORACLE["inp"], _ORACLE["coeffs"]
    projected, cache = _ORACLE["kv"]
    x = torch.from_numpy(np.ascontiguousarray(inp["x"][:, :, :depth]))
    t = torch.from_numpy(inp["timesteps"])
    t0 = time.perf_counter()
    eps = model.forward(x, t, projected, cache)
    state = np.ascontiguousarray(inp["x"][:, :7, :depth])
    osamp.ddim_update(state, eps.float().numpy()[:, :7], coeffs["alphas"][-1], coeffs["previous"][-1],
                      coeffs["sigmas"][-1], coeffs["sqrt_one_minus"][-1], np.zeros_like(state))
    return time.perf_counter() - t0, {"depth": depth}


def cpu_baseline(budget_s: float = 25.0) -> dict:
    """Time the oracle step on the host cores on a bounded sample (depth crop), scaled to the full latent."""
    threads = len(os.sched_getaffinity(0))
    full_depth = 32
    t4, _ = cpu_step_time(4, threads)  # calibration (also warms up)
    depth = int(max(4, min(full_depth, (budget_s / max(t4, 1e-3)) * 4)) // 4 * 4)
    t, _ = cpu_step_time(depth, threads)
    full = t * full_depth / depth
    return {
        "value": 1.0 / full, "unit": UNIT, "cores": threads, "kind": "port",
        "sample": f"one UNet step + DDIM update on a 1x8x{depth}x40x40 depth crop ({t:.2f} s), "
                  f"scaled by {full_depth}/{depth} to the 32-deep latent",
    }


def run_reference(args, rank: int) -> None:
    if rank != 0:
        return
    threads = len(os.sched_getaffinity(0))
    total = args.steps + args.warmup
    t4, _ = cpu_step_time(4, threads)
    budget = 150.0 / max(total, 1)
    depth = int(max(4, min(32, budget / max(t4, 1e-3) * 4)) // 4 * 4)
    for _ in range(args.warmup):
        cpu_step_time(depth, threads)
    times = [cpu_step_time(depth, threads)[0] for _ in range(args.steps)]
    per_step_full = sum(times) / len(times) * 32 / depth
    value = 1.0 / per_step_full
    world = int(os.environ.get("WORLD_SIZE", "1"))
    line = {
        "metric": METRIC, "value": value, "unit": UNIT, "n_gpus": args.gpus, "steps": args.steps,
        "warmup": args.warmup, "ms_per_step": per_step_full * 1e3, "higher_is_better": True, "scaling": "weak",
        "vs_baseline": None, "dtype": "f16 (storage; FP32/FP64 CPU arithmetic)", "data": "synthetic",
        "impl": "reference",
        "config": workload_config(max(world, args.gpus)),
        "execution": f"one replica on {threads} host cores (rank 0 only)",
        "cpu_baseline": {"value": value, "unit": UNIT, "cores": threads, "kind": "port",
                         "sample": f"each step: one oracle UNet step + DDIM update on a 1x8x{depth}x40x40 depth "
                                   f"crop, scaled by 32/{depth}; the reference is MLX/Metal-only and cannot run here"},
        "e2e": {"value": value, "unit": UNIT, "h2d_bytes_per_step": 0, "d2h_bytes_per_step": 0},
    }
    print(json.dumps(line), flush=True)


def _max_over_ranks(value: float, world: int, device) -> float:
    if world <= 1:
        return value
    import torch.distributed as dist

    t = torch.tensor([value], dtype=torch.float64, device=device)
    dist.all_reduce(t, op=dist.ReduceOp.MAX)
    return float(t.item())


def main() -> None:
    args = parse()
    rank, world, local = dist_setup(args.gpus)
    if args.impl == "reference":
        run_reference(args, rank)
        if world > 1:
            import torch.distributed as dist

            dist.destroy_process_group()
        return

    from lesiondiffusion_mlx_b200 import _lib, instrument, ops, vq_bench, workloads
    from lesiondiffusion_mlx_b200.networks import LdmUnetB200, VqDecoderB200
    from lesiondiffusion_mlx_b200.sampling import DdimSampler, HostStreamedSteps, PreparedSampler

    dist = None
    if world > 1:
        import torch.distributed as dist
    device = torch.device("cuda", local)
    torch.cuda.set_device(device)
    cfg = workloads.CONFIG3
    raw = workloads.unet_weights(cfg, 8, 8, 768, seed=100)
    weights = {k: torch.from_numpy(v).to(torch.float16) for k, v in raw.items()}
    unet = LdmUnetB200(weights, cfg, device=device)
    inp = workloads.config3_inputs(seed=101 + rank)
    cache = unet.prepare_context(torch.from_numpy(inp["context"]).to(device))
    sampler = DdimSampler(linet_alphas(), 200)
    image = torch.from_numpy(workloads.source_latent((1, 7, 32, 40, 40), seed=300)).permute(0, 2, 3, 4, 1)
    mask = torch.from_numpy(inp["mask"][:, 0])
    prepared = PreparedSampler(sampler, unet, cache, image.to(device), mask.to(device), graph=False)
    gen = torch.Generator(device=device).manual_seed(1000 + rank)
    init = torch.randn(prepared.state.x.shape, generator=gen, device=device)
    noise = torch.randn(prepared.state.noise.shape, generator=gen, device=device)
    prepared.begin(init, noise)
    decoder = VqDecoderB200({k: torch.from_numpy(v) for k, v in workloads.config4_decoder_weights().items()},
                            device=device, groups=32)
    latent = torch.zeros((1, 32, 40, 40, 8), dtype=torch.float16, device=device)

    # Capture one step (UNet + DDIM update + step advance) twice: a plain graph
    # for the timed region, and a copy replayed afterwards for the per-kernel
    # breakdown.  In the copy every conv and attention launch times itself from
    # the device clock (its first CTA past the dependency wait to its last CTA
    # or split-K reduce finishing; no node is added to its path), and the other
    # kernels have CUDA event pairs around them (whose nodes add gaps).
    timer = instrument.KernelTimer(device_clock=True)
    timer.arm(device)
    prepared._step()  # eager warm-up (first-use setup outside capture)
    torch.cuda.synchronize()
    launches0 = _lib.launch_count()
    graph = torch.cuda.CUDAGraph()
    with torch.cuda.graph(graph):
        prepared._step()
    launches_per_step = _lib.launch_count() - launches0
    timed_graph = torch.cuda.CUDAGraph()
    with instrument.timing(timer), torch.cuda.graph(timed_graph):
        prepared._step()
    prepared.begin(init, noise)

    stream = torch.cuda.current_stream(device)
    done = 0
    for _ in range(args.warmup):
        if done and done % sampler.steps == 0:
            prepared.begin(init, noise)
        graph.replay()
        done += 1
    decoder.decode(latent, quantize=False)  # warm-up of the decoder (first-use packing)
    torch.cuda.synchronize()
    prepared.begin(init, noise)
    done = 0

    if dist is not None:
        dist.barrier()
    clocks = ClockSampler(device.index)
    clocks.start()
    time.sleep(0.3)
    torch.cuda.synchronize()
    start = torch.cuda.Event(enable_timing=True)
    end = torch.cuda.Event(enable_timing=True)
    start.record(stream)
    for _ in range(args.steps):
        if done and done % sampler.steps == 0:
            # a full 200-step trajectory finished: restart from the initial state (device copies only)
            prepared.begin(init, noise)
        graph.replay()
        done += 1
    end.record(stream)
    torch.cuda.synchronize()
    elapsed_ms = start.elapsed_time(end)

    # One whole generation, the north star's unit: a 200-step DDIM trajectory
    # from the initial state, then the config-4a decode of [latent | mask] to
    # HU (1 x 128 x 160 x 160).  Same clocks record.
    prepared.begin(init, noise)
    t_start = torch.cuda.Event(enable_timing=True)
    t_mid = torch.cuda.Event(enable_timing=True)
    t_end = torch.cuda.Event(enable_timing=True)
    t_start.record(stream)
    for _ in range(sampler.steps):
        graph.replay()
    t_mid.record(stream)
    latent[..., :7].copy_(prepared.state.x)
    latent[..., 7].copy_(prepared.state.mask)
    hu = ops.hu_map(decoder.decode(latent, quantize=False))
    t_end.record(stream)
    torch.cuda.synchronize()
    clock_info = clocks.stop()
    trajectory_ms = t_start.elapsed_time(t_mid)
    decode_ms = t_mid.elapsed_time(t_end)
    hu_finite = bool(torch.isfinite(hu).all().item())
    del hu

    prepared.begin(init, noise)
    for _ in range(3):
        timer.reset()
        timed_graph.replay()
    torch.cuda.synchronize()
    kernel = timer.summary()
    # the conv launches by kind: 3x3x3 (strided and folded-up included) and pointwise / dense
    conv_kinds: dict[str, list[float]] = {}
    for kind, label, flops, ms in timer.launches():
        if kind == "conv3d":
            entry = conv_kinds.setdefault("pointwise" if label.startswith("mode3 ") else "3x3x3", [0, 0.0, 0.0])
            entry[0] += 1
            entry[1] += ms
            entry[2] += flops
    elapsed_ms = _max_over_ranks(elapsed_ms, world, device)
    trajectory_ms = _max_over_ranks(trajectory_ms, world, device)
    decode_ms = _max_over_ranks(decode_ms, world, device)
    if dist is not None:
        dist.barrier()
    ms_per_step = elapsed_ms / args.steps
    value = world * args.steps / (elapsed_ms / 1e3)

    # End to end through the public step API with host buffers: every step
    # the step's noise comes from pinned host memory and the updated latent is
    # read back to pinned host memory (HostStreamedSteps: the copies run on a
    # copy stream beside the neighbouring steps' compute).
    host_noise = noise[0].cpu().pin_memory()
    host_out = torch.empty(prepared.state.x.shape, dtype=torch.float32).pin_memory()
    prepared.begin(init, noise)
    streamer = HostStreamedSteps(prepared, step=graph.replay)
    if dist is not None:
        dist.barrier()
    torch.cuda.synchronize()
    e_start = torch.cuda.Event(enable_timing=True)
    e_end = torch.cuda.Event(enable_timing=True)
    e_steps = args.steps
    e_start.record(stream)
    streamer.start(host_noise)
    for i in range(e_steps):
        if i and i % sampler.steps == 0:
            prepared.begin(init)  # a trajectory finished: restart its state (the noise slots stay the stream's)
        streamer.step(host_noise if i + 1 < e_steps else None, host_out)
    streamer.finish()
    e_end.record(stream)
    torch.cuda.synchronize()
    e_ms = _max_over_ranks(e_start.elapsed_time(e_end), world, device)
    e_value = world * e_steps / (e_ms / 1e3)
    status = _lib.device_status(reset=True)
    del graph, timed_graph, prepared, unet, decoder, latent
    torch.cuda.empty_cache()

    # Config 4b: unsharded on one GPU, depth-sharded over all ranks at N > 1
    # (every rank takes part; collectives in the same order on every rank).
    decode_4b = vq_bench.measure("4b", device, steps=2, warmup=1, dist=dist)

    if rank == 0:
        peaks = {}
        peaks_file = ROOT / "MEASURED_PEAKS.json"
        if peaks_file.exists():
            peaks = json.loads(peaks_file.read_text())
        conv = kernel.get("conv3d", {"ms": float("nan"), "flops": 0.0, "launches": 0})
        attn = kernel.get("attention", {"ms": float("nan"), "flops": 0.0, "launches": 0})
        conv_tflops = conv["flops"] / (conv["ms"] * 1e-3) / 1e12 if conv["ms"] else None
        attn_tflops = attn["flops"] / (attn["ms"] * 1e-3) / 1e12 if attn["ms"] else None
        # The step is a few milliseconds and the timed region well under a second,
        # so kernels run at burst clocks: the burst peak is the denominator.
        peak_burst = peaks.get("bf16_tflops", 1590.0)
        peak_sustained = peaks.get("bf16_tflops_sustained", 1400.0)
        peak_kind = "measured burst bf16 (MEASURED_PEAKS.json)" if peaks else "fallback burst (1.59 PFLOP/s)"
        traffic_file = ROOT / "profiles" / "conv3d_traffic.json"
        traffic = None
        if traffic_file.exists():
            traffic = json.loads(traffic_file.read_text()).get("bytes_per_step")
        device_clocked = {"conv3d", "attention"}
        decode_4b["frac_of_burst_per_gpu"] = decode_4b["tflops_per_gpu"] / peak_burst
        line = {
            "metric": METRIC, "value": value, "unit": UNIT, "n_gpus": world, "steps": args.steps,
            "warmup": args.warmup, "ms_per_step": ms_per_step, "higher_is_better": True, "scaling": "weak",
            "vs_baseline": None, "dtype": "f16", "data": "synthetic (random-init weights, seeded inputs)",
            "config": workload_config(world),
            "roofline": {
                "kernel": "conv3d (tcgen05 implicit GEMM)", "bound": "tensor",
                "achieved": conv_tflops, "peak": peak_burst, "unit": "TFLOP/s",
                "frac": (conv_tflops / peak_burst) if conv_tflops else None, "peak_kind": peak_kind,
                "frac_of_sustained": (conv_tflops / peak_sustained) if conv_tflops else None,
                "traffic": traffic,
                "flops_per_step": conv["flops"], "launches_per_step": conv["launches"], "ms_per_step": conv["ms"],
                "by_kind": {
                    name: {"launches": n, "ms_per_step": round(ms, 4),
                           "achieved": flops / (ms * 1e-3) / 1e12 if ms else None,
                           "frac": flops / (ms * 1e-3) / 1e12 / peak_burst if ms else None}
                    for name, (n, ms, flops) in sorted(conv_kinds.items())
                },
            },
            "attention": {"achieved_tflops": attn_tflops, "frac": (attn_tflops / peak_burst) if attn_tflops else None,
                          "flops_per_step": attn["flops"], "ms_per_step": attn["ms"], "launches": attn["launches"]},
            "e2e": {"value": e_value, "unit": UNIT, "h2d_bytes_per_step": int(host_noise.numel() * 4),
                    "d2h_bytes_per_step": int(host_out.numel() * 4)},
            "trajectory": {
                "ddim200_s": trajectory_ms / 1e3, "decode_4a_to_hu_s": decode_ms / 1e3,
                "generation_s": (trajectory_ms + decode_ms) / 1e3, "target_s": 10.0, "hu_finite": hu_finite,
                "what": "200 DDIM steps from the initial state (graph replays) + config-4a decode of "
                        "[7 latent channels | mask] to a 1x128x160x160 HU volume, per rank, max over ranks",
            },
            "decode_4b": decode_4b,
            "kernel_ms_per_step": {
                "device_clock": {k: round(v["ms"], 4) for k, v in sorted(kernel.items()) if k in device_clocked},
                "cuda_events": {k: round(v["ms"], 4) for k, v in sorted(kernel.items()) if k not in device_clocked},
                "note": "device_clock spans are exact per launch; cuda_events spans include the event nodes' gaps",
            },
            "gpu_launches": int(launches_per_step * args.steps),
            "launches_per_step": int(launches_per_step),
            "clocks": clock_info,
            "device_status": status,
        }
        if world == 1 and not args.no_cpu_baseline:
            line["cpu_baseline"] = cpu_baseline()
        print(json.dumps(line), flush=True)
    if dist is not None:
        dist.barrier()
        dist.destroy_process_group()


if __name__ == "__main__":
    main()
