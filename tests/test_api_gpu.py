"""The drop-in operator layer (``lesiondiffusion_mlx_b200.api``) against the
oracle on the reference's own layouts (GPU).

Every function keeps the reference signature it replaces: ``nax_conv3d``
(_nax_conv.py:451-463), ``flash_attention`` / ``flash_eligible``
(_attention.py:283-375), ``nearest_codebook4`` (_vq.py:64),
``upsample_nearest2`` / ``resize_nearest`` (_spatial.py:41-69),
``piecewise_ct`` (mlx_pipeline.py:72-96) and medmlx-core's
``group_norm_affine`` / ``native_group_norm`` (called at mlx_model.py:328-358),
on NCDHW (volumes) and ``(B, L, heads * d)`` (projections) CUDA tensors.
Tolerances: rel-L2 <= 1e-2 for f16 / bf16 results and <= 1e-4 for FP32,
exact equality for the index and copy operators.
"""

from __future__ import annotations

import numpy as np
import pytest
import torch

from oracle import ops as oops

pytestmark = pytest.mark.gpu


def rel_l2(a, b) -> float:
    a = np.asarray(a, dtype=np.float64)
    b = np.asarray(b, dtype=np.float64)
    return float(np.linalg.norm(a - b) / max(np.linalg.norm(b), 1e-30))


def _case(shape, cout, seed, dtype=torch.float16, k=3):
    rng = np.random.default_rng(seed)
    c = shape[1]
    x = torch.from_numpy((rng.normal(size=shape) * 1.5 + 0.3).astype(np.float32)).to(dtype)
    w = torch.from_numpy((rng.normal(size=(cout, c, k, k, k)) * (c * k ** 3) ** -0.5).astype(np.float32)).to(dtype)
    b = torch.from_numpy((rng.normal(size=cout) * 0.1).astype(np.float32))
    g = torch.from_numpy((1 + 0.2 * rng.normal(size=c)).astype(np.float32))
    beta = torch.from_numpy((0.2 * rng.normal(size=c)).astype(np.float32))
    return x, w, b, g, beta


def test_nax_conv3d_affine_silu_residual(cuda_device):
    """``residual + conv(SiLU(x * scale + offset)) + bias`` with the affine of
    ``group_norm_affine`` (the norm_silu_conv call at mlx_model.py:328-342)."""
    from lesiondiffusion_mlx_b200 import api

    x, w, b, g, beta = _case((2, 64, 5, 6, 7), 48, seed=1)
    res = torch.from_numpy(np.random.default_rng(2).normal(size=(2, 48, 5, 6, 7)).astype(np.float16))
    dev = lambda t: t.to(cuda_device)  # noqa: E731
    affine = api.group_norm_affine(dev(x), dev(g), dev(beta), groups=32, eps=1e-5, mx=None)
    assert affine.dtype == torch.float32 and tuple(affine.shape) == (2 * 64 * 2,)
    packed = api.pack_weight(dev(w), None)
    out = api.nax_conv3d(dev(x), packed, dev(b), affine=affine, silu=True, residual=dev(res), mx=None)
    torch.cuda.synchronize()
    assert out.dtype == torch.float16 and tuple(out.shape) == (2, 48, 5, 6, 7) and out.is_contiguous()
    want_affine = oops.group_norm_affine(x, g, beta, groups=32, eps=1e-5)
    np.testing.assert_allclose(affine.cpu().numpy().reshape(2, 64, 2), want_affine.numpy(), rtol=2e-5, atol=2e-5)
    prepared = oops.apply_affine(x, want_affine, silu=True).to(torch.float16)
    want = oops.conv3d(prepared, w, b, residual=res, dtype=torch.float16)
    assert rel_l2(out.float().cpu().numpy(), want.float().numpy()) <= 1e-2


@pytest.mark.parametrize("stride", [1, 2])
def test_nax_conv3d_per_batch_bias_and_output_scale(cuda_device, stride):
    """A ``(B, O)`` bias (one bias per batch item) and ``output_scale`` (bias
    scaled with the conv, the residual not)."""
    from lesiondiffusion_mlx_b200 import api

    x, w, _, _, _ = _case((2, 32, 6, 7, 5), 40, seed=3)
    bias2 = torch.from_numpy(np.random.default_rng(4).normal(size=(2, 40)).astype(np.float32) * 0.1)
    out_grid = tuple((n - 1) // stride + 1 for n in (6, 7, 5))
    res = torch.from_numpy(np.random.default_rng(5).normal(size=(2, 40, *out_grid)).astype(np.float16))
    packed = api.pack_weight(w.to(cuda_device), stride=stride)
    out = api.nax_conv3d(x.to(cuda_device), packed, bias2.to(cuda_device), stride=stride, output_scale=0.25,
                         residual=res.to(cuda_device))
    torch.cuda.synchronize()
    want = oops.conv3d(x, w, None, stride=stride, shift=bias2, output_scale=0.25, residual=res, dtype=torch.float16)
    assert tuple(out.shape) == tuple(want.shape)
    assert rel_l2(out.float().cpu().numpy(), want.float().numpy()) <= 1e-2


def test_nax_conv3d_upsample(cuda_device):
    """``upsample=True`` with ``pack_upsample_weight``: the conv of the nearest
    2x upsampling via the eight folded parity filters (_nax_conv.py:367-405)."""
    from lesiondiffusion_mlx_b200 import api

    x, w, b, _, _ = _case((1, 32, 4, 5, 3), 24, seed=6)
    packed = api.pack_upsample_weight(w.to(cuda_device))
    assert packed.ndim == 3
    out = api.nax_conv3d(x.to(cuda_device), packed, b.to(cuda_device), upsample=True)
    torch.cuda.synchronize()
    want = oops.upsample_conv(x, w, b, dtype=torch.float16)
    assert tuple(out.shape) == (1, 24, 8, 10, 6)
    assert rel_l2(out.float().cpu().numpy(), want.float().numpy()) <= 1e-2
    # the fold equals the conv of the materialized nearest upsampling up to the folded weights' rounding
    plain = oops.conv3d(oops.upsample_nearest2(x), w, b, dtype=torch.float16)
    assert rel_l2(out.float().cpu().numpy(), plain.float().numpy()) <= 1e-2


def test_nax_conv3d_fp32_exact_mode_with_affine(cuda_device):
    """Float32 ``x`` and weights: the split-f16 exact mode returns float32 at
    the FP32 tolerance, with the affine + SiLU applied in FP32."""
    from lesiondiffusion_mlx_b200 import api

    x, w, b, g, beta = _case((1, 48, 6, 5, 7), 32, seed=7, dtype=torch.float32)
    affine = api.group_norm_affine(x.to(cuda_device), g.to(cuda_device), beta.to(cuda_device), groups=16, eps=1e-6)
    packed = api.pack_weight(w.to(cuda_device))
    out = api.nax_conv3d(x.to(cuda_device), packed, b.to(cuda_device), affine=affine, silu=True)
    torch.cuda.synchronize()
    assert out.dtype == torch.float32
    want_affine = oops.group_norm_affine(x, g, beta, groups=16, eps=1e-6)
    prepared = oops.apply_affine(x, want_affine, silu=True)
    want = oops.conv3d(prepared, w, b, dtype=torch.float32)
    assert rel_l2(out.cpu().numpy(), want.numpy()) <= 1e-4


@pytest.mark.parametrize("dtype", [torch.float16, torch.float32])
@pytest.mark.parametrize("silu", [False, True])
def test_native_group_norm(cuda_device, dtype, silu):
    """GroupNorm (+ SiLU) in FP32 with one rounding to x's dtype (mlx_model.py:348-358)."""
    from lesiondiffusion_mlx_b200 import api

    x, _, _, g, beta = _case((2, 96, 3, 4, 5), 8, seed=8, dtype=dtype)
    out = api.native_group_norm(x.to(cuda_device), g.to(cuda_device), beta.to(cuda_device), groups=32, eps=1e-6,
                                silu=silu)
    torch.cuda.synchronize()
    want = oops.native_group_norm(x, g, beta, groups=32, eps=1e-6, silu=silu)
    assert out.dtype == dtype and tuple(out.shape) == tuple(x.shape)
    tol = 1e-2 if dtype == torch.float16 else 1e-4
    assert rel_l2(out.float().cpu().numpy(), want.float().numpy()) <= tol
    if dtype == torch.float16:
        ulp = np.spacing(np.abs(want.float().numpy()).astype(np.float16)).astype(np.float32)
        assert np.all(np.abs(out.float().cpu().numpy() - want.float().numpy()) <= 2 * ulp + 1e-6)


@pytest.mark.parametrize("dtype", [torch.float16, torch.bfloat16])
@pytest.mark.parametrize("lq,lk", [(700, 700), (640, 77)])
def test_flash_attention(cuda_device, dtype, lq, lk):
    """Head-interleaved projections ``(B, L, heads * 64)``: self-attention and
    cross-attention to 77 keys against float64 softmax attention."""
    from lesiondiffusion_mlx_b200 import api

    rng = np.random.default_rng(lq + lk)
    q, k, v = (torch.from_numpy(rng.normal(size=(1, n, 4 * 64)).astype(np.float32)).to(dtype)
               for n in (lq, lk, lk))
    assert api.flash_eligible(q, k, 4)
    out = api.flash_attention(q.to(cuda_device), k.to(cuda_device), v.to(cuda_device), heads=4, scale=0.125, mx=None)
    torch.cuda.synchronize()
    want = oops.attention(q, k, v, heads=4, scale=0.125)
    assert out.dtype == dtype
    assert rel_l2(out.float().cpu().numpy(), want.float().numpy()) <= 1e-2


@pytest.mark.parametrize("length", [256, 300])
def test_flash_attention_half(cuda_device, length):
    """The FP16 entry point on the reference kernel's case (32-wide heads, equal
    query and key lengths; 300 is not a multiple of 32, which the reference
    leaves to its caller) against the oracle's restatement of the reference's
    FP16 flash contract."""
    from lesiondiffusion_mlx_b200 import api

    rng = np.random.default_rng(length)
    q, k, v = (torch.from_numpy(rng.normal(size=(2, length, 8 * 32)).astype(np.float32)).half() for _ in range(3))
    out = api.flash_attention_half(q.to(cuda_device), k.to(cuda_device), v.to(cuda_device), heads=8,
                                   scale=32 ** -0.5, mx=None)
    torch.cuda.synchronize()
    want = oops.attention(q, k, v, heads=8, scale=32 ** -0.5)
    assert out.dtype == torch.float16 and tuple(out.shape) == tuple(q.shape)
    assert rel_l2(out.float().cpu().numpy(), want.float().numpy()) <= 1e-2


@pytest.mark.parametrize("dtype", [torch.float16, torch.float32])
def test_nearest_codebook4(cuda_device, dtype):
    """int32 indices, bit-exact with the oracle's rounding order, ties to the first index."""
    from lesiondiffusion_mlx_b200 import api

    rng = np.random.default_rng(9)
    codebook = rng.normal(size=(300, 4)).astype(np.float32)
    z = np.concatenate([rng.normal(size=(997, 4)).astype(np.float32), codebook[:5], codebook[:5]])
    z_t, cb_t = (torch.from_numpy(a).to(dtype) for a in (z, codebook))
    idx = api.nearest_codebook4(z_t.to(cuda_device), cb_t.to(cuda_device), None, mx=None)
    torch.cuda.synchronize()
    assert idx.dtype == torch.int32 and tuple(idx.shape) == (z.shape[0],)
    npd = np.float16 if dtype == torch.float16 else np.float32
    want = oops.nearest_codebook4(z_t.numpy().astype(npd), cb_t.numpy().astype(npd))
    np.testing.assert_array_equal(idx.cpu().numpy(), want)


def test_upsample_nearest2_and_resize_nearest(cuda_device):
    from lesiondiffusion_mlx_b200 import api

    rng = np.random.default_rng(10)
    x = torch.from_numpy(rng.normal(size=(2, 5, 3, 4, 6)).astype(np.float16))
    up = api.upsample_nearest2(x.to(cuda_device), mx=None)
    resized = api.resize_nearest(x.to(cuda_device), (7, 3, 11))
    xf = torch.from_numpy(rng.normal(size=(1, 2, 9, 5, 4)).astype(np.float32))
    down = api.resize_nearest(xf.to(cuda_device), (4, 5, 3))
    torch.cuda.synchronize()
    assert torch.equal(up.cpu(), oops.upsample_nearest2(x))
    assert torch.equal(resized.cpu(), oops.resize_nearest(x, (7, 3, 11)))
    assert torch.equal(down.cpu(), oops.resize_nearest(xf, (4, 5, 3)))


def test_piecewise_ct_both_directions(cuda_device):
    """Normalized -> HU and HU -> normalized, knots and clipping included, as the
    oracle's restatement of mlx_pipeline.py:72-96 (FP32 arithmetic: exact up to
    the last bit of the slope product)."""
    from lesiondiffusion_mlx_b200 import api

    values = np.concatenate([np.linspace(-0.5, 1.5, 4001), [0.0, 0.2, 0.8, 1.0]]).astype(np.float32)
    x = torch.from_numpy(values.reshape(1, 1, 5, 1, 801))
    hu = api.piecewise_ct(x.to(cuda_device), None, inverse=True)
    torch.cuda.synchronize()
    want = oops.piecewise_ct(x, inverse=True)
    assert hu.dtype == torch.float32 and tuple(hu.shape) == tuple(x.shape)
    np.testing.assert_allclose(hu.cpu().numpy(), want.numpy(), rtol=0, atol=1e-3)
    hu_in = np.concatenate([np.linspace(-1500, 1500, 6001), [-1000, -200, 200, 1000]]).astype(np.float32)
    h = torch.from_numpy(hu_in.reshape(5, 1201))
    norm = api.piecewise_ct(h.to(cuda_device), None)
    torch.cuda.synchronize()
    assert norm.dtype == torch.float32 and tuple(norm.shape) == tuple(h.shape)
    np.testing.assert_allclose(norm.cpu().numpy(), oops.piecewise_ct(h).numpy(), rtol=0, atol=1e-7)


def test_nax_available_on_the_gpu_box(cuda_device):
    from lesiondiffusion_mlx_b200 import api

    assert api.nax_available(None)
