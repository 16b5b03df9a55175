"""The reference's binding API on the B200 sampler: ``unet.prepare_denoiser(context)``
and ``sampler.prepare(denoiser, image, mask=)`` (mlx_model.py:570-597,
mlx_sampling.py:138-200, _dpm.py:82-100) against a ``PreparedSampler`` run on
the same seeded noise (GPU)."""

from __future__ import annotations

import numpy as np
import pytest
import torch

pytestmark = pytest.mark.gpu


def _rel_l2(a: torch.Tensor, b: torch.Tensor) -> float:
    a, b = a.double(), b.double()
    return float((a - b).norm() / b.norm().clamp_min(1e-30))


@pytest.mark.parametrize("kind", ["ddim", "dpmpp_2m"])
def test_prepare_binds_a_denoiser_like_the_reference(cuda_device, kind):
    """``unet.prepare_denoiser(context)`` + ``sampler.prepare(denoiser, image,
    mask=)`` (the reference's mlx_model.py:570-597 and mlx_sampling.py:138-200 /
    _dpm.py:82-100): ``sample()`` gives the trajectory of a ``PreparedSampler``
    run on the same seeded noise, in NCDHW, with the known region exactly the
    conditioning image, and fresh noise on the next call."""
    from lesiondiffusion_mlx_b200 import workloads
    from lesiondiffusion_mlx_b200.networks import LdmUnetB200, UnetConfig
    from lesiondiffusion_mlx_b200.sampling import DdimSampler, Dpmpp2mSampler, PreparedSampler

    config = UnetConfig(32, 1, (2,), (1, 2), 32, False)
    raw = workloads.unet_weights(config, 5, 4, 32, seed=23)
    unet = LdmUnetB200({k: torch.from_numpy(v).half() for k, v in raw.items()}, config, device=cuda_device)
    rng = np.random.default_rng(31)
    context = torch.from_numpy(rng.standard_normal((1, 6, 32)).astype(np.float32))
    image = torch.from_numpy(rng.standard_normal((1, 4, 4, 8, 8)).astype(np.float32))
    mask = torch.zeros((1, 1, 4, 8, 8))
    mask[:, :, 1:3, 2:6, 2:6] = 1.0
    alphas = np.linspace(0.9999, 0.02, 1000).astype(np.float32)
    sampler = DdimSampler(alphas, 4) if kind == "ddim" else Dpmpp2mSampler(alphas, 4)

    denoise = unet.prepare_denoiser(context)
    # the network input's channel stride is padded to 8 (as the sampler writes it)
    x = torch.zeros((1, 4, 8, 8, 8), dtype=torch.float16, device=cuda_device)[..., :5]
    x.copy_(torch.from_numpy(rng.standard_normal((1, 4, 8, 8, 5)).astype(np.float32)).half())
    t = torch.tensor([500], dtype=torch.int32, device=cuda_device)
    assert _rel_l2(denoise(x, t), unet(x, t, context)) <= 1e-2

    sample = sampler.prepare(denoise, image, mask=mask, generator=torch.Generator(device=cuda_device).manual_seed(5))
    got = sample()
    again = sample()
    g = torch.Generator(device=cuda_device).manual_seed(5)
    prepared = PreparedSampler(sampler, unet, denoise.cache, image.permute(0, 2, 3, 4, 1).to(cuda_device),
                               mask[:, 0].to(cuda_device), graph=True)
    initial = torch.randn(tuple(prepared.state.x.shape), generator=g, device=cuda_device)
    noise = torch.randn(tuple(prepared.state.noise.shape), generator=g, device=cuda_device) if kind == "ddim" else None
    want = prepared.run(initial, noise).permute(0, 4, 1, 2, 3)
    torch.cuda.synchronize()
    assert tuple(got.shape) == tuple(image.shape) and got.dtype == torch.float32
    # the GroupNorm statistics are summed by atomics, so two runs agree to the last bits of the f16
    # network outputs, not bit for bit, and the trajectory amplifies an early one-ulp difference: the
    # trajectory bar of the other sampler tests (relative L2 <= 1e-2) applies
    assert _rel_l2(got, want) <= 1e-2
    known = (mask.expand_as(image) == 0).to(cuda_device)
    assert torch.equal(got[known], image.to(cuda_device)[known])
    assert not torch.allclose(got, again)
