"""The host-streamed sampler stepping (``sampling.HostStreamedSteps``): each
step's noise copied in from pinned host memory and each step's latent copied
out on a copy stream, overlapped with the neighbouring steps, gives the
latents of plain device stepping (GPU).  Two runs of the network agree to the
last bits only up to the order of the GroupNorm statistics' atomic adds, so
the latents are compared at 1e-3; a step that read another step's noise (or
the 1e3 placeholder left in the device slots) would be off by ~0.1 or more."""

from __future__ import annotations

import numpy as np
import pytest
import torch

pytestmark = pytest.mark.gpu


@pytest.mark.parametrize("graph", [False, True])
def test_host_streamed_steps_match_device_steps(cuda_device, graph):
    from lesiondiffusion_mlx_b200 import workloads
    from lesiondiffusion_mlx_b200.networks import LdmUnetB200, UnetConfig
    from lesiondiffusion_mlx_b200.sampling import DdimSampler, HostStreamedSteps, PreparedSampler

    config = UnetConfig(32, 1, (2,), (1, 2), 32, False)
    raw = workloads.unet_weights(config, 5, 4, 32, seed=21)
    unet = LdmUnetB200({k: torch.from_numpy(v).half() for k, v in raw.items()}, config, device=cuda_device)
    rng = np.random.default_rng(5)
    context = torch.from_numpy(rng.standard_normal((1, 3, 32)).astype(np.float32)).to(cuda_device)
    cache = unet.prepare_context(context)
    shape = (1, 4, 8, 8)
    image = torch.from_numpy(rng.standard_normal((*shape, 4)).astype(np.float32)).to(cuda_device)
    mask = torch.zeros(shape, dtype=torch.float32)
    mask[:, 1:3, 2:6, 2:6] = 1.0
    alphas = np.linspace(0.9999, 0.02, 1000).astype(np.float32)
    steps = 5
    prepared = PreparedSampler(DdimSampler(alphas, steps), unet, cache, image, mask.to(cuda_device), graph=graph)
    init = torch.from_numpy(rng.standard_normal((1, *shape[1:], 4)).astype(np.float32))
    noise = torch.from_numpy(rng.standard_normal((steps, 1, *shape[1:], 4)).astype(np.float32))

    # plain device stepping
    prepared.begin(init.to(cuda_device), noise.to(cuda_device))
    if graph:
        prepared.capture()
    want = []
    for _ in range(steps):
        prepared.step()
        want.append(prepared.state.x.clone())
    torch.cuda.synchronize()

    # host-streamed stepping: the device noise slots hold garbage until each step's copy-in
    prepared.begin(init.to(cuda_device), torch.full_like(noise, 1e3).to(cuda_device))
    host_noise = [n.pin_memory() for n in noise]
    host_out = [torch.empty(want[0].shape, dtype=torch.float32).pin_memory() for _ in range(steps)]
    streamer = HostStreamedSteps(prepared)
    streamer.start(host_noise[0])
    for i in range(steps):
        streamer.step(host_noise[i + 1] if i + 1 < steps else None, host_out[i])
    streamer.finish()
    torch.cuda.synchronize()
    for i in range(steps):
        torch.testing.assert_close(host_out[i], want[i].cpu(), rtol=1e-3, atol=1e-3, msg=f"step {i}")
