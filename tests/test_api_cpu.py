"""The drop-in operator layer's argument checks, which need no GPU.

``api.nax_conv3d`` raises ``ValueError`` where the reference does
(_nax_conv.py:506-510: packed rows that do not fit x's channels and dtype;
:553-554: a residual whose shape is not the output's) and for the stride /
upsample combinations it does not take; the eligibility helpers answer as
the reference's (_nax_conv.py:321-328, _attention.py:283-299).  All checks
run before any device work, so CPU tensors exercise them.
"""

from __future__ import annotations

import pytest
import torch

from lesiondiffusion_mlx_b200 import api


def _weight(cout: int, cin: int, dtype=torch.float16, k: int = 3) -> torch.Tensor:
    return torch.zeros((cout, cin, k, k, k), dtype=dtype)


def test_nax_conv3d_rejects_weights_packed_for_other_channels():
    packed = api.pack_weight(_weight(16, 32))
    x = torch.zeros((1, 24, 4, 4, 4), dtype=torch.float16)
    with pytest.raises(ValueError, match="do not fit 24 input channels"):
        api.nax_conv3d(x, packed, torch.zeros(16))


def test_nax_conv3d_rejects_weights_packed_for_the_other_dtype():
    packed = api.pack_weight(_weight(16, 32))  # f16 packing
    x = torch.zeros((1, 32, 4, 4, 4), dtype=torch.float32)
    with pytest.raises(ValueError, match="float32"):
        api.nax_conv3d(x, packed, torch.zeros(16))
    packed32 = api.pack_weight(_weight(16, 32, torch.float32))
    with pytest.raises(ValueError, match="float16"):
        api.nax_conv3d(x.half(), packed32, torch.zeros(16))


def test_nax_conv3d_rejects_a_residual_of_another_shape():
    packed = api.pack_weight(_weight(16, 32))
    x = torch.zeros((1, 32, 4, 6, 8), dtype=torch.float16)
    with pytest.raises(ValueError, match="residual shape"):
        api.nax_conv3d(x, packed, torch.zeros(16), residual=torch.zeros((1, 16, 4, 6, 7), dtype=torch.float16))
    # stride 2 halves the grid (rounding up): a full-size residual is wrong
    packed2 = api.pack_weight(_weight(16, 32), stride=2)
    with pytest.raises(ValueError, match=r"!= output \(1, 16, 2, 3, 4\)"):
        api.nax_conv3d(x, packed2, torch.zeros(16), stride=2,
                       residual=torch.zeros((1, 16, 4, 6, 8), dtype=torch.float16))
    up = api.pack_upsample_weight(_weight(16, 32))
    with pytest.raises(ValueError, match=r"!= output \(1, 16, 8, 12, 16\)"):
        api.nax_conv3d(x, up, torch.zeros(16), upsample=True,
                       residual=torch.zeros((1, 16, 4, 6, 8), dtype=torch.float16))


def test_nax_conv3d_rejects_mismatched_upsample_and_stride():
    x = torch.zeros((1, 32, 4, 4, 4), dtype=torch.float16)
    plain = api.pack_weight(_weight(16, 32))
    up = api.pack_upsample_weight(_weight(16, 32))
    with pytest.raises(ValueError, match="pack_upsample_weight"):
        api.nax_conv3d(x, plain, torch.zeros(16), upsample=True)
    with pytest.raises(ValueError, match="pack_upsample_weight"):
        api.nax_conv3d(x, up, torch.zeros(16))
    with pytest.raises(ValueError, match="stride"):
        api.nax_conv3d(x, plain, torch.zeros(16), stride=3)
    with pytest.raises(ValueError, match="NCDHW"):
        api.nax_conv3d(x[0], plain, torch.zeros(16))


def test_packing_geometry_and_eligibility():
    plain = api.pack_weight(_weight(40, 24))
    up = api.pack_upsample_weight(_weight(40, 24))
    exact = api.pack_weight(_weight(40, 24, torch.float32))
    assert (plain.ndim, up.ndim) == (2, 3)
    assert plain.dtype == torch.float16 and exact.dtype == torch.float32
    # K: 27 taps x 24 channels padded to 32 (x2 planes in exact mode); rows padded to the column tile
    assert plain.tensor.shape[1] == 27 * 32 and exact.tensor.shape[1] == 2 * 27 * 32
    assert up.tensor.shape[1] == 8 * 32 and up.tensor.shape[0] == 8 * plain.tensor.shape[0]
    assert api.nax_eligible(_weight(8, 8)) and not api.nax_eligible(_weight(8, 8, k=1))
    with pytest.raises(ValueError):
        api.pack_upsample_weight(_weight(8, 8, k=1))


def test_attention_eligibility():
    q = torch.zeros((1, 10, 256), dtype=torch.float16)
    assert api.flash_eligible(q, q, 4)  # 64-wide heads
    assert api.flash_eligible(q, q, 8)  # 32-wide
    assert not api.flash_eligible(q, q, 2)  # 128-wide heads: not a kernel head width
    assert not api.flash_eligible(q, q.float(), 4)
    assert not api.flash_eligible(q.float(), q.float(), 4)
    assert not api.flash_eligible(q, torch.zeros((1, 10, 128), dtype=torch.float16), 4)
    with pytest.raises(ValueError, match="float16 projections"):
        api.flash_attention_half(q.to(torch.bfloat16), q.to(torch.bfloat16), q.to(torch.bfloat16), heads=8, scale=0.2)


def test_other_operator_argument_errors():
    with pytest.raises(ValueError, match=r"\(positions, 4\)"):
        api.nearest_codebook4(torch.zeros((10, 3)), torch.zeros((5, 3)))
    with pytest.raises(ValueError, match="three spatial axes"):
        api.resize_nearest(torch.zeros((1, 1, 2, 2, 2)), (4, 4))
    with pytest.raises(ValueError, match="CUDA"):
        api.piecewise_ct(torch.zeros(3), inverse=False)  # device kernels take device tensors only


def test_native_group_norm_eligibility():
    """The predicate the reference tests before its native GroupNorm, answered
    with the limits of the GroupNorm kernels here."""
    x = torch.zeros((1, 64, 2, 2, 2), dtype=torch.float16)
    assert api.native_group_norm_eligible(x, 32)
    assert api.native_group_norm_eligible(x.float(), 16)
    assert not api.native_group_norm_eligible(x.to(torch.bfloat16), 32)  # f16 / f32 only
    assert not api.native_group_norm_eligible(x, 24)  # groups must divide the channels
    assert not api.native_group_norm_eligible(torch.zeros((1, 12, 2, 2, 2), dtype=torch.float16), 12)  # 12 % 8
    assert not api.native_group_norm_eligible(torch.zeros((1, 2048, 1, 1, 1), dtype=torch.float16), 1)  # > 1024 per group
    assert not api.native_group_norm_eligible(torch.zeros((1, 64, 4), dtype=torch.float16), 32)  # not NCDHW
