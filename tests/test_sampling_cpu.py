"""Host-side checks of the samplers' ``prepare`` binding (no device work):
what it accepts as a denoiser and as a mask, as the reference's
``Sampler.prepare(denoiser, conditioning_image, mask=)`` (mlx_sampling.py:138)."""

from __future__ import annotations

from types import SimpleNamespace

import numpy as np
import pytest
import torch


def _sampler():
    from lesiondiffusion_mlx_b200.sampling import DdimSampler

    return DdimSampler(np.linspace(0.9999, 0.02, 1000).astype(np.float32), 4)


def test_prepare_takes_only_a_bound_denoiser():
    image = torch.zeros((1, 4, 2, 4, 4))
    with pytest.raises(TypeError, match="prepare_denoiser"):
        _sampler().prepare(lambda x, t: x, image)


def test_prepare_checks_image_and_mask_layouts():
    bound = SimpleNamespace(unet=SimpleNamespace(device=torch.device("cpu")), cache={})
    with pytest.raises(ValueError, match="NCDHW"):
        _sampler().prepare(bound, torch.zeros((4, 2, 4, 4)))
    with pytest.raises(ValueError, match="mask must be"):
        _sampler().prepare(bound, torch.zeros((1, 4, 2, 4, 4)), mask=torch.zeros((1, 2, 4, 4)))


def test_prepare_converts_the_reference_layouts():
    """The NCDHW conditioning image and (B, 1, D, H, W) mask reach the prepared
    sampler as its NDHWC image and (B, D, H, W) mask (constructed on the CPU:
    the sampler allocates its buffers there and launches nothing until a draw)."""
    unet = SimpleNamespace(device=torch.device("cpu"), in_channels=5, exact=False)
    bound = SimpleNamespace(unet=unet, cache={})
    image = torch.arange(1 * 4 * 2 * 3 * 5, dtype=torch.float32).reshape(1, 4, 2, 3, 5)
    mask = (torch.arange(2 * 3 * 5).reshape(1, 1, 2, 3, 5) % 2).float()
    sample = _sampler().prepare(bound, image, mask=mask)
    state = sample.prepared.state
    assert torch.equal(state.image, image.permute(0, 2, 3, 4, 1))
    assert torch.equal(state.mask, mask[:, 0])
    assert tuple(state.x.shape) == (1, 2, 3, 5, 4) and tuple(state.noise.shape) == (4, 1, 2, 3, 5, 4)
