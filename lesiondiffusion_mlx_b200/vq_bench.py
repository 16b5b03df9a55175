"""VQ-decode throughput (config 4): one JSON line per run.

    python -m lesiondiffusion_mlx_b200.vq_bench --config 4a
    torchrun --nproc-per-node N -m lesiondiffusion_mlx_b200.vq_bench --config 4b

4a decodes the 1x8x32x40x40 latent to 1x1x128x160x160 on one GPU with the
unsharded decoder; 4b decodes 1x8x62x110x110 to 1x1x248x440x440 sharded
along depth over the ranks (halo exchange over NCCL, GroupNorm statistics
all-reduced), or unsharded on one GPU.  Random-init weights (seed 200),
seeded N(0, 1) latent, f16, decode without quantization (the 8-channel
latent has no 4-wide codebook).  Each timed decode is bracketed by a
barrier and CUDA events; the time is the max over ranks.  FLOPs are the
algorithmic conv FLOPs of the decode (2 * out_voxels * Cout * taps * Cin,
8 taps for the folded upsampling conv), counted by the conv wrapper.
"""

from __future__ import annotations

import argparse
import datetime
import json
import os

import numpy as np
import torch

from . import instrument, workloads
from .networks import VqDecoderB200


def _weights(device) -> dict[str, torch.Tensor]:
    raw = workloads.config4_decoder_weights()
    return {k: torch.from_numpy(v) for k, v in raw.items()}


def measure(config: str, device: torch.device, *, steps: int = 3, warmup: int = 1, groups: int = 32,
            dist=None, halo_sms: int = 8) -> dict:
    """Time the config-4 decode (``"4a"`` / ``"4b"``) on this rank and return its record.

    With ``dist`` (an initialised ``torch.distributed`` with more than one
    rank) the latent is split along depth over the ranks; otherwise the
    unsharded decoder runs on ``device``.  Each timed decode is bracketed by
    a barrier and CUDA events, and the time is the max over ranks.  Collective
    calls are made in the same order on every rank."""
    world = dist.get_world_size() if dist is not None else 1
    rank = dist.get_rank() if dist is not None else 0
    dec = VqDecoderB200(_weights(device), device=device, groups=groups)
    shape = workloads.CONFIG4_LATENTS[config]
    z = np.random.default_rng(201).standard_normal(shape).astype(np.float32)
    zt = torch.from_numpy(z).permute(0, 2, 3, 4, 1).to(device, torch.float16)
    zbuf = torch.zeros((*zt.shape[:-1], 8), dtype=torch.float16, device=device)
    zbuf[..., : zt.shape[-1]] = zt
    depth = shape[2]
    comm = None
    if world > 1:
        from .sharded_decode import DistDepthComm, ShardedVqDecoder, partition_depth

        start, stop = partition_depth(depth, world)[rank]
        comm = DistDepthComm(timed=True)
        sharded = ShardedVqDecoder(dec, comm, halo_sms=halo_sms)

        def run():
            return sharded.decode([zbuf[:, start:stop]], depth, quantize=False)[0]
    else:
        def run():
            return dec.decode(zbuf, quantize=False)

    # FLOPs of one decode (whole volume: each rank counts its slab, summed below).
    timer = instrument.KernelTimer()
    with instrument.timing(timer):
        out = run()
    torch.cuda.synchronize()
    flops = sum(v["flops"] for v in timer.summary().values())
    if dist is not None:
        t = torch.tensor([flops], dtype=torch.float64, device=device)
        dist.all_reduce(t)
        flops = float(t.item())
    for _ in range(warmup):
        run()
    if comm is not None:
        comm.comm_ms(reset=True)
    times, comm_times = [], []
    for _ in range(steps):
        if dist is not None:
            dist.barrier()
        torch.cuda.synchronize()
        s = torch.cuda.Event(enable_timing=True)
        e = torch.cuda.Event(enable_timing=True)
        s.record()
        out = run()
        e.record()
        torch.cuda.synchronize()
        ms = s.elapsed_time(e)
        if comm is not None:
            comm_times.append(comm.comm_ms(reset=True))
        if dist is not None:
            t = torch.tensor([ms], device=device)
            dist.all_reduce(t, op=dist.ReduceOp.MAX)
            ms = float(t.item())
        times.append(ms)
    ms = float(np.median(times))
    finite = bool(torch.isfinite(out.float()).all().item())
    record = {
        "config": config, "latent": list(shape), "output": [1, 1, depth * 4, shape[3] * 4, shape[4] * 4],
        "n_gpus": world, "parallelism": f"depth-sharded x{world}" if world > 1 else "one GPU, unsharded",
        "ms_per_decode": ms, "decode_tflop": flops / 1e12, "tflops_total": flops / ms / 1e9,
        "tflops_per_gpu": flops / ms / 1e9 / world, "steps": steps, "warmup": warmup, "dtype": "f16",
        "data": "synthetic (random-init weights seed 200, N(0,1) latent seed 201)", "finite": finite,
    }
    if comm_times:
        # this rank's median time waiting on halo exchanges / statistics all-reduces per decode,
        # and the max of that over ranks
        local = {k: float(np.median([c[k] for c in comm_times])) for k in ("exchange", "all_reduce")}
        t = torch.tensor([local["exchange"], local["all_reduce"]], device=device)
        dist.all_reduce(t, op=dist.ReduceOp.MAX)
        record["halo_sms"] = halo_sms
        record["halo_exchange_ms"] = float(t[0].item())
        record["gn_all_reduce_ms"] = float(t[1].item())
        record["halo_exchanges"] = int(comm_times[0]["exchange_calls"])
        record["gn_all_reduces"] = int(comm_times[0]["all_reduce_calls"])
    del dec, out
    torch.cuda.empty_cache()
    return record


def main() -> None:
    ap = argparse.ArgumentParser()
    ap.add_argument("--config", choices=("4a", "4b"), default="4a")
    ap.add_argument("--steps", type=int, default=3)
    ap.add_argument("--warmup", type=int, default=1)
    ap.add_argument("--groups", type=int, default=32)
    ap.add_argument("--halo-sms", type=int, default=8, help="SMs the slab-interior conv leaves to the halo exchange")
    a = ap.parse_args()

    world = int(os.environ.get("WORLD_SIZE", "1"))
    rank = int(os.environ.get("RANK", "0"))
    local = int(os.environ.get("LOCAL_RANK", "0"))
    torch.cuda.set_device(local)
    device = torch.device("cuda", local)
    dist = None
    if world > 1:
        import torch.distributed as dist

        dist.init_process_group("nccl", timeout=datetime.timedelta(seconds=300), device_id=device)
    record = measure(a.config, device, steps=a.steps, warmup=a.warmup, groups=a.groups, dist=dist,
                     halo_sms=a.halo_sms)
    if rank == 0:
        print(json.dumps({"metric": "VQ decode TFLOP/s", **record}), flush=True)
    if dist is not None:
        dist.barrier()
        dist.destroy_process_group()


if __name__ == "__main__":
    main()
