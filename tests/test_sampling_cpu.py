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
