"""GroupNorm statistics fused into the convolution epilogue, and the
normalize pass that derives the affine from them.

The reference computes GroupNorm statistics in a separate call on the conv
output (medmlx-core group_norm_affine, lesiondiffusion_mlx/mlx_model.py:
328-358).  Here the conv that produces a tensor also adds each channel's sum
and sum of squares of the values it stores (``conv3d_ndhwc(stats=...)``) and
``group_norm_affine_from_stats`` turns them into the per-group affine without
reading the tensor.  The tests check (1) the statistics against FP64 sums of
the conv's own stored output, on every epilogue path (plain, split-K reduce,
folded upsampling parities, stride 2, FP32 exact, residual + shift), and (2)
the affine and the normalized output against the oracle's GroupNorm.
"""

from __future__ import annotations

import numpy as np
import pytest
import torch

from oracle import ops as oracle_ops

pytestmark = pytest.mark.gpu

SUM_TOL = 1e-5  # relative to the sum of |x| (sums) or of x^2 (sums of squares)


def ndhwc(x: torch.Tensor) -> torch.Tensor:
    return x.permute(0, 2, 3, 4, 1).contiguous()


def ncdhw(x: torch.Tensor) -> torch.Tensor:
    return x.permute(0, 4, 1, 2, 3).contiguous()


CASES = [
    # (input NCDHW shape, out channels, kind, residual+shift)
    ((1, 32, 24, 24, 40), 64, "conv", False),  # 180 tiles: TMEM epilogue
    ((1, 32, 24, 24, 40), 64, "conv", True),
    ((2, 256, 5, 6, 7), 128, "conv", True),  # few tiles: split-K reduce kernel
    ((1, 32, 16, 20, 24), 48, "up", False),  # folded upsampling, 8 output parities
    ((1, 64, 8, 10, 12), 64, "up", False),  # ... with split-K
    ((1, 64, 16, 20, 24), 64, "s2", False),  # stride 2 (split-K)
    ((1, 32, 24, 24, 40), 32, "exact", False),  # FP32 exact mode, f32 staging
]


@pytest.mark.parametrize("shape,cout,kind,extra", CASES)
def test_conv_epilogue_statistics_match_stored_output(cuda_device, shape, cout, kind, extra):
    from lesiondiffusion_mlx_b200 import ops
    from lesiondiffusion_mlx_b200.conv import conv3d_ndhwc, pack_upsample_weight, pack_weight

    rng = np.random.default_rng(sum(shape) + cout)
    b, cin = shape[0], shape[1]
    x = torch.from_numpy(rng.normal(size=shape).astype(np.float32) + 0.5)
    w = torch.from_numpy((rng.normal(size=(cout, cin, 3, 3, 3)) * (cin * 27) ** -0.5).astype(np.float32))
    bias = torch.from_numpy(rng.normal(size=cout).astype(np.float32) * 0.1).to(cuda_device)
    xd = ndhwc(x).to(cuda_device)
    if kind == "exact":
        xin = ops.prepare_input(xd, split=True)
        packed = pack_weight(w.to(cuda_device))
    else:
        xin = xd.half()
        wd = w.half().to(cuda_device)
        packed = pack_upsample_weight(wd) if kind == "up" else pack_weight(wd, stride=2 if kind == "s2" else 1)
    shift = residual = None
    if extra:
        probe = conv3d_ndhwc(xin, packed, bias, in_channels=cin)
        shift = torch.from_numpy(rng.normal(size=(b, cout)).astype(np.float32)).to(cuda_device)
        residual = torch.from_numpy(rng.normal(size=tuple(probe.shape)).astype(np.float32)).to(probe.dtype)
        residual = residual.to(cuda_device)
    stats = torch.zeros((b, cout, 2), dtype=torch.float64, device=cuda_device)
    out = conv3d_ndhwc(xin, packed, bias, stride=2 if kind == "s2" else 1, shift=shift, residual=residual,
                       stats=stats, in_channels=cin)
    torch.cuda.synchronize()
    vals = out.double().reshape(b, -1, cout)
    want_sum = vals.sum(1)
    want_sq = (vals * vals).sum(1)
    got = stats.cpu()
    assert torch.all((got[..., 0] - want_sum.cpu()).abs() <= SUM_TOL * vals.abs().sum(1).cpu() + 1e-9)
    assert torch.all((got[..., 1] - want_sq.cpu()).abs() <= SUM_TOL * want_sq.cpu() + 1e-9)


@pytest.mark.parametrize("dtype", [torch.float16, torch.float32])
@pytest.mark.parametrize("shape,groups,split", [((2, 64, 3, 5, 7), 32, None), ((1, 768, 2, 4, 5), 32, 512),
                                                ((1, 8, 4, 4, 4), 8, None), ((1, 96, 3, 4, 5), 32, 40)])
def test_affine_from_stats_matches_oracle_group_norm(cuda_device, dtype, shape, groups, split):
    from lesiondiffusion_mlx_b200 import ops

    rng = np.random.default_rng(sum(shape) + 7)
    x = torch.from_numpy((rng.normal(size=shape) * 3 + 1.5).astype(np.float32)).to(dtype)
    gamma = torch.from_numpy(rng.normal(size=shape[1]).astype(np.float32))
    beta = torch.from_numpy(rng.normal(size=shape[1]).astype(np.float32))
    expected = oracle_ops.group_norm_affine(x, gamma, beta, groups=groups, eps=1e-5)
    xd = ndhwc(x).to(cuda_device)
    voxels = shape[2] * shape[3] * shape[4]

    def sums(t: torch.Tensor) -> torch.Tensor:
        v = t.double().reshape(t.shape[0], -1, t.shape[-1])
        return torch.stack([v.sum(1), (v * v).sum(1)], dim=-1).contiguous()

    g, bt = gamma.to(cuda_device), beta.to(cuda_device)
    if split:
        x1 = xd[..., :split].contiguous()
        x2 = xd[..., split:].contiguous()
        affine = ops.group_norm_affine_from_stats(sums(x1), g, bt, voxels=voxels, groups=groups, eps=1e-5,
                                                  stats2=sums(x2))
        prepared = ops.prepare_input(x1, affine=affine, silu=True, x2=x2)
    else:
        affine = ops.group_norm_affine_from_stats(sums(xd), g, bt, voxels=voxels, groups=groups, eps=1e-5)
        prepared = ops.prepare_input(xd, affine=affine, silu=True)
    torch.cuda.synchronize()
    np.testing.assert_allclose(affine.cpu().numpy(), expected.numpy(), rtol=2e-5, atol=2e-5)
    want = oracle_ops.apply_affine(x, expected, silu=True).to(torch.float16).float()
    got = ncdhw(prepared.float().cpu())
    ulp = np.spacing(np.abs(want.numpy()).astype(np.float16)).astype(np.float32)
    assert np.all(np.abs(got.numpy() - want.numpy()) <= 2 * ulp + 1e-6)


@pytest.mark.parametrize("dtype", [torch.float16, torch.float32])
@pytest.mark.parametrize("shape,groups,split,exact", [((2, 64, 3, 5, 7), 32, None, False),
                                                      ((1, 768, 2, 4, 5), 32, 512, False),
                                                      ((3, 96, 3, 4, 5), 32, 40, True),
                                                      ((1, 128, 8, 9, 10), 16, None, True)])
def test_prepare_from_stats_equals_affine_then_prepare(cuda_device, dtype, shape, groups, split, exact):
    """The one-launch normalize pass gives the same bits as the affine kernel
    followed by the plain normalize pass (both sources, f16 rounding and the
    FP32 hi/lo split, several batch items)."""
    from lesiondiffusion_mlx_b200 import ops

    rng = np.random.default_rng(sum(shape) + 11)
    x = torch.from_numpy((rng.normal(size=shape) * 2 - 0.7).astype(np.float32)).to(dtype)
    gamma = torch.from_numpy(rng.normal(size=shape[1]).astype(np.float32)).to(cuda_device)
    beta = torch.from_numpy(rng.normal(size=shape[1]).astype(np.float32)).to(cuda_device)
    xd = ndhwc(x).to(cuda_device)
    voxels = shape[2] * shape[3] * shape[4]

    def sums(t: torch.Tensor) -> torch.Tensor:
        v = t.double().reshape(t.shape[0], -1, t.shape[-1])
        return torch.stack([v.sum(1), (v * v).sum(1)], dim=-1).contiguous()

    x1, x2 = (xd[..., :split].contiguous(), xd[..., split:].contiguous()) if split else (xd, None)
    s1, s2 = sums(x1), (None if x2 is None else sums(x2))
    affine = ops.group_norm_affine_from_stats(s1, gamma, beta, voxels=voxels, groups=groups, eps=1e-5, stats2=s2)
    want = ops.prepare_input(x1, affine=affine, silu=True, split=exact, x2=x2)
    got = ops.prepare_input_from_stats(x1, s1, gamma, beta, groups=groups, eps=1e-5, silu=True, split=exact, x2=x2,
                                       stats2=s2)
    torch.cuda.synchronize()
    assert torch.equal(got, want)
    # statistics of a larger volume (one slab of a sharded decode): the voxel count is the volume's
    affine = ops.group_norm_affine_from_stats(s1, gamma, beta, voxels=3 * voxels, groups=groups, eps=1e-5,
                                              stats2=s2)
    want = ops.prepare_input(x1, affine=affine, silu=True, split=exact, x2=x2)
    got = ops.prepare_input_from_stats(x1, s1, gamma, beta, groups=groups, eps=1e-5, silu=True, split=exact, x2=x2,
                                       stats2=s2, voxels=3 * voxels)
    torch.cuda.synchronize()
    assert torch.equal(got, want)


def test_fused_statistics_feed_group_norm(cuda_device):
    """conv (with statistics) -> affine from statistics equals the statistics
    pass over the same conv output."""
    from lesiondiffusion_mlx_b200 import ops
    from lesiondiffusion_mlx_b200.conv import conv3d_ndhwc, pack_weight

    rng = np.random.default_rng(3)
    x = torch.from_numpy(rng.normal(size=(1, 32, 24, 24, 40)).astype(np.float16)).to(cuda_device)
    w = torch.from_numpy((rng.normal(size=(128, 32, 3, 3, 3)) * (32 * 27) ** -0.5).astype(np.float16))
    bias = torch.from_numpy(rng.normal(size=128).astype(np.float32) * 0.5).to(cuda_device)
    stats = torch.zeros((1, 128, 2), dtype=torch.float64, device=cuda_device)
    out = conv3d_ndhwc(ndhwc(x), pack_weight(w.to(cuda_device)), bias, stats=stats)
    gamma = torch.from_numpy(rng.normal(size=128).astype(np.float32)).to(cuda_device)
    beta = torch.from_numpy(rng.normal(size=128).astype(np.float32)).to(cuda_device)
    fused = ops.group_norm_affine_from_stats(stats, gamma, beta, voxels=24 * 24 * 40, groups=32, eps=1e-5)
    two_pass = ops.group_norm_affine(out, gamma, beta, groups=32, eps=1e-5)
    torch.cuda.synchronize()
    np.testing.assert_allclose(fused.cpu().numpy(), two_pass.cpu().numpy(), rtol=2e-5, atol=2e-5)


def test_device_status_clean(cuda_device):
    from lesiondiffusion_mlx_b200 import _lib

    assert _lib.device_status(reset=True) == 0
