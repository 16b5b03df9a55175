"""The host-streamed sampler stepping (``sampling.HostStreamedSteps``): each
step's noise copied in from pinned host memory and each step's latent copied
out on a copy stream, overlapped with the neighbouring steps, gives exactly
the latents of plain device stepping (GPU).

The step here is the fused DDIM update with a fixed prediction instead of the
network (the network's GroupNorm statistics are summed by atomics, so two
runs of it agree only to the last bits), which makes both runs bit-exact; the
device noise slots are filled with 1e3 before the streamed run, so a step
that read a slot before its copy-in landed would be far off."""

from __future__ import annotations

import numpy as np
import pytest
import torch

pytestmark = pytest.mark.gpu


@pytest.mark.parametrize("steps", [1, 2, 6])
def test_host_streamed_steps_match_device_steps(cuda_device, steps):
    from lesiondiffusion_mlx_b200 import ops, workloads
    from lesiondiffusion_mlx_b200.networks import LdmUnetB200, UnetConfig
    from lesiondiffusion_mlx_b200.sampling import DdimSampler, HostStreamedSteps, PreparedSampler

    config = UnetConfig(32, 1, (2,), (1, 2), 32, False)
    raw = workloads.unet_weights(config, 5, 4, 32, seed=21)
    unet = LdmUnetB200({k: torch.from_numpy(v).half() for k, v in raw.items()}, config, device=cuda_device)
    rng = np.random.default_rng(5 + steps)
    shape = (1, 4, 8, 8)
    image = torch.from_numpy(rng.standard_normal((*shape, 4)).astype(np.float32)).to(cuda_device)
    mask = torch.zeros(shape, dtype=torch.float32)
    mask[:, 1:3, 2:6, 2:6] = 1.0
    alphas = np.linspace(0.9999, 0.02, 1000).astype(np.float32)
    sampler = DdimSampler(alphas, steps)
    steps = sampler.steps  # steps the schedule executes (noise slots)
    prepared = PreparedSampler(sampler, unet, {}, image, mask.to(cuda_device), graph=False)
    s = prepared.state
    eps = torch.from_numpy(rng.standard_normal(tuple(s.x.shape)).astype(np.float32)).half().to(cuda_device)

    def det_step():
        ops.sampler_step(sampler.kind, s.x, eps=eps, prev=s.prev, noise=s.noise,
                         noise_step_stride=int(s.noise[0].numel()), mask=s.mask, image=s.image, net_in=s.net_in,
                         coeff=s.coeff, step=s.step)
        ops.step_advance(s.step)

    rounds = 2 * steps + 1  # over two trajectory restarts: every noise slot is refilled
    init = torch.from_numpy(rng.standard_normal(tuple(s.x.shape)).astype(np.float32))
    noise = torch.from_numpy(rng.standard_normal((rounds, *s.x.shape)).astype(np.float32))

    want = []
    for i in range(rounds):
        if i % steps == 0:
            prepared.begin(init.to(cuda_device))
        s.noise[i % steps].copy_(noise[i].to(cuda_device))
        det_step()
        want.append(s.x.clone())
    torch.cuda.synchronize()

    prepared.begin(init.to(cuda_device), torch.full((steps, *s.x.shape), 1e3).to(cuda_device))
    host_noise = [n.pin_memory() for n in noise]
    host_out = [torch.empty(tuple(s.x.shape), dtype=torch.float32).pin_memory() for _ in range(rounds)]
    streamer = HostStreamedSteps(prepared, step=det_step)
    streamer.start(host_noise[0])
    for i in range(rounds):
        if i and i % steps == 0:
            prepared.begin(init.to(cuda_device))
        streamer.step(host_noise[i + 1] if i + 1 < rounds else None, host_out[i])
    streamer.finish()
    torch.cuda.synchronize()
    for i in range(rounds):
        assert torch.equal(host_out[i], want[i].cpu()), f"step {i}"


def test_step_counter_past_the_tables_touches_nothing(cuda_device):
    """A step graph replayed past the end of its schedule: with the device
    step counter at the tables' row count, the sampler step and the timestep
    embedding read and write nothing and set status bit 1 instead."""
    from lesiondiffusion_mlx_b200 import _lib, ops

    _lib.device_status(reset=True)
    g = torch.Generator(device=cuda_device).manual_seed(3)
    rows, shape = 3, (1, 4, 6, 6, 4)
    x = torch.randn(shape, generator=g, device=cuda_device)
    eps = torch.randn(shape, generator=g, device=cuda_device).half()
    noise = torch.randn((rows, *shape), generator=g, device=cuda_device)
    coeff = torch.tensor([[0.5, 0.6, 0.1, 0.7, 0.0]] * rows, device=cuda_device)
    table = torch.arange(2 * rows, dtype=torch.int32, device=cuda_device).view(rows, 2)
    emb = torch.full((2, 32), 7.0, device=cuda_device)
    step = torch.tensor([rows - 1], dtype=torch.int32, device=cuda_device)
    before = x.clone()
    ops.sampler_step(1, x, eps=eps, noise=noise, noise_step_stride=int(noise[0].numel()), coeff=coeff, step=step)
    ops.timestep_embedding(table, 32, step=step, out=emb)
    torch.cuda.synchronize()
    assert _lib.device_status(reset=False) == 0
    assert not torch.equal(x, before) and not torch.equal(emb, torch.full_like(emb, 7.0))
    step.fill_(rows)  # one past the last row
    moved, emb_before = x.clone(), emb.clone()
    ops.sampler_step(1, x, eps=eps, noise=noise, noise_step_stride=int(noise[0].numel()), coeff=coeff, step=step)
    ops.timestep_embedding(table, 32, step=step, out=emb)
    torch.cuda.synchronize()
    assert torch.equal(x, moved) and torch.equal(emb, emb_before)
    assert _lib.device_status(reset=True) & 2
    assert _lib.device_status(reset=False) == 0

