"""Op-level CPU restatement of the reference hot-path arithmetic (test only).

Tensors are NCDHW ``torch`` CPU tensors like the reference's.  ``dtype`` is
the storage dtype of the layer (float16 for LINet/decoder, float32 for the
FP32 networks); arithmetic runs in ``compute`` (float64 by default, float32
for large cases) and rounds to ``dtype`` exactly where the reference's native
(conditioned-mode) path rounds.  Paths are relative to
``src/lesiondiffusion_mlx/`` of lesiondiffusion-mlx 0.3.0.
"""

from __future__ import annotations

import math

import numpy as np
import torch
import torch.nn.functional as F

DEFAULT_COMPUTE = torch.float64


def conv3d(
    x: torch.Tensor,
    weight: torch.Tensor,
    bias: torch.Tensor | None = None,
    *,
    stride: int = 1,
    padding: int = 1,
    shift: torch.Tensor | None = None,
    residual: torch.Tensor | None = None,
    output_scale: float = 1.0,
    dtype: torch.dtype,
    compute: torch.dtype = DEFAULT_COMPUTE,
) -> torch.Tensor:
    """3-D convolution rounded once: ``(conv + bias + shift) * scale + residual``.

    Follows ``nax_conv3d``'s contract (_nax_conv.py:451-499 and the epilogue
    at :239-274): operands are the stored values, products accumulate at high
    precision, bias (plus the per-batch shift, summed in FP32 first as at
    mlx_model.py:340-341) is added before scaling, the residual after, and
    the result is rounded to ``dtype`` once.
    """
    y = F.conv3d(x.to(compute), weight.to(compute), None, stride=stride, padding=padding)
    add = None
    if bias is not None:
        add = bias.to(torch.float32)
    if shift is not None:
        add = shift.to(torch.float32) if add is None else add[None] + shift.to(torch.float32)
    if add is not None:
        y = y + (add.to(compute)[:, :, None, None, None] if add.ndim == 2 else add.to(compute)[:, None, None, None])
    y = y * output_scale
    if residual is not None:
        y = y + residual.to(compute)
    return y.to(dtype)


def upsample_conv_weight(weight: torch.Tensor) -> torch.Tensor:
    """Fold a 3x3x3 weight into eight 2x2x2 parity filters (_nax_conv.py:367-405).

    Returns float32 ``(8, O, C, 2, 2, 2)``; parity ``pd*4 + ph*2 + pw``.  The
    per-axis fold is (k0, k1 + k2) for parity 0 and (k0 + k1, k2) for
    parity 1, applied depth, height, width in order with FP32 sums.
    """
    w = weight.to(torch.float32)

    def fold(t: torch.Tensor, dim: int) -> torch.Tensor:
        k0, k1, k2 = t.unbind(dim)
        return torch.stack([torch.stack([k0, k1 + k2], dim), torch.stack([k0 + k1, k2], dim)], dim)

    f = fold(fold(fold(w, 2), 4), 6)  # (O, C, pd, td, ph, th, pw, tw)
    f = f.permute(2, 4, 6, 0, 1, 3, 5, 7)  # (pd, ph, pw, O, C, td, th, tw)
    return f.reshape(8, *w.shape[:2], 2, 2, 2)


def upsample_conv(
    x: torch.Tensor, weight: torch.Tensor, bias: torch.Tensor | None, *, dtype: torch.dtype,
    output_scale: float = 1.0, compute: torch.dtype = DEFAULT_COMPUTE,
) -> torch.Tensor:
    """Conv of a nearest 2x upsampling via folded parity filters (mlx_model.py:272-288).

    F16 networks round each merged tap once to f16 (_nax_conv.py:376-379);
    FP32 networks keep the FP32 sums.
    """
    folded = upsample_conv_weight(weight)
    if dtype == torch.float16:
        folded = folded.to(torch.float16)
    b, _, d, h, w = x.shape
    out = torch.empty((b, weight.shape[0], 2 * d, 2 * h, 2 * w), dtype=compute)
    xp = F.pad(x.to(compute), (1, 1, 1, 1, 1, 1))
    for par in range(8):
        pd, ph, pw = par >> 2, (par >> 1) & 1, par & 1
        # parity p, tap t reads source m + p + t - 1 = padded m + p + t.
        window = xp[:, :, pd : pd + d + 1, ph : ph + h + 1, pw : pw + w + 1]
        out[:, :, pd::2, ph::2, pw::2] = F.conv3d(window, folded[par].to(compute))
    if bias is not None:
        out = out + bias.to(torch.float32).to(compute)[:, None, None, None]
    return (out * output_scale).to(dtype)


def pointwise_conv(
    x: torch.Tensor, weight: torch.Tensor, bias: torch.Tensor | None, *, dtype: torch.dtype,
    compute: torch.dtype = DEFAULT_COMPUTE,
) -> torch.Tensor:
    """1x1x1 conv as ``W @ x`` (mlx_model.py:183-194): the f16 product rounds before the bias add."""
    w2 = weight.reshape(weight.shape[0], weight.shape[1]).to(compute)
    y = torch.einsum("oc,bcdhw->bodhw", w2, x.to(compute)).to(dtype)
    if bias is not None:
        y = (y.to(compute) + bias.to(compute)[:, None, None, None]).to(dtype)
    return y


def dense(
    x: torch.Tensor, weight: torch.Tensor, bias: torch.Tensor | None, *, dtype: torch.dtype,
    compute: torch.dtype = DEFAULT_COMPUTE,
) -> torch.Tensor:
    """Linear layer on the last axis, bias added before one rounding (mlx_model.py:204-220)."""
    y = x.to(compute) @ weight.to(compute).T
    if bias is not None:
        y = y + bias.to(compute)
    return y.to(dtype)


def group_norm_affine(
    x: torch.Tensor, gamma: torch.Tensor, beta: torch.Tensor, *, groups: int, eps: float
) -> torch.Tensor:
    """Per-(batch, channel) FP32 ``(scale, offset)`` of a GroupNorm (B, C, 2).

    Restates medmlx-core's ``group_norm_affine`` from its call sites
    (mlx_model.py:328-335, _scaled_vq.py:93-100): biased variance over each
    group's channels and voxels, ``scale = gamma * rsqrt(var + eps)`` and
    ``offset = beta - mean * scale``.  Statistics are taken in float64.
    """
    b, c = x.shape[:2]
    g = x.to(torch.float64).reshape(b, groups, -1)
    mean = g.mean(dim=2)
    var = g.var(dim=2, unbiased=False)
    rstd = torch.rsqrt(var + eps)
    per = c // groups
    mean_c = mean.repeat_interleave(per, dim=1)
    rstd_c = rstd.repeat_interleave(per, dim=1)
    scale = gamma.to(torch.float64)[None] * rstd_c
    offset = beta.to(torch.float64)[None] - mean_c * scale
    return torch.stack([scale, offset], dim=2).to(torch.float32)


def apply_affine(x: torch.Tensor, affine: torch.Tensor, *, silu: bool) -> torch.Tensor:
    """FP32 ``x * scale + offset`` then optional SiLU (_nax_conv.py:126-135)."""
    y = x.to(torch.float32) * affine[:, :, 0, None, None, None] + affine[:, :, 1, None, None, None]
    if silu:
        y = y / (1.0 + torch.exp(-y))
    return y


def native_group_norm(
    x: torch.Tensor, gamma: torch.Tensor, beta: torch.Tensor, *, groups: int, eps: float, silu: bool,
) -> torch.Tensor:
    """GroupNorm (+ fused SiLU) computed in FP32 and rounded once (mlx_model.py:262-270, :348-358)."""
    affine = group_norm_affine(x, gamma, beta, groups=groups, eps=eps)
    return apply_affine(x, affine, silu=silu).to(x.dtype)


def norm_silu_conv(
    x: torch.Tensor, gamma: torch.Tensor, beta: torch.Tensor, weight: torch.Tensor, bias: torch.Tensor | None,
    *, groups: int, eps: float, shift: torch.Tensor | None = None, residual: torch.Tensor | None = None,
    output_scale: float = 1.0, compute: torch.dtype = DEFAULT_COMPUTE,
) -> torch.Tensor:
    """``residual + conv(SiLU(GN(x))) + shift`` on the native path (mlx_model.py:290-342).

    The normalize-SiLU result is rounded once to f16 as the conv's prepared
    input (_nax_conv.py:136-138); FP32 networks keep it in FP32 (exact mode).
    """
    affine = group_norm_affine(x, gamma, beta, groups=groups, eps=eps)
    prepared = apply_affine(x, affine, silu=True)
    if x.dtype == torch.float16:
        prepared = prepared.to(torch.float16)
    return conv3d(
        prepared, weight, bias, shift=shift, residual=residual, output_scale=output_scale, dtype=x.dtype,
        compute=compute,
    )


def layer_norm(x: torch.Tensor, gamma: torch.Tensor, beta: torch.Tensor, eps: float = 1e-5) -> torch.Tensor:
    """Last-axis LayerNorm in FP32, returned in x's dtype (mlx_model.py:360-367)."""
    y = F.layer_norm(x.to(torch.float32), (x.shape[-1],), gamma.to(torch.float32), beta.to(torch.float32), eps)
    return y.to(x.dtype)


def gelu(x: torch.Tensor) -> torch.Tensor:
    """Exact erf GELU in FP32, returned in x's dtype (mlx_model.py:369-374)."""
    y = x.to(torch.float32)
    return (y * (1 + torch.erf(y / math.sqrt(2))) * 0.5).to(x.dtype)


def silu(x: torch.Tensor) -> torch.Tensor:
    """UNet SiLU: FP32 then one rounding (mlx_model.py:409-413)."""
    y = x.to(torch.float32)
    return (y / (1 + torch.exp(-y))).to(x.dtype)


def attention(
    q: torch.Tensor, k: torch.Tensor, v: torch.Tensor, *, heads: int, scale: float,
    compute: torch.dtype = DEFAULT_COMPUTE,
) -> torch.Tensor:
    """``softmax(q k^T * scale) v`` on projection-layout ``(B, L, heads*d)`` tensors.

    Half inputs follow the flash contract of _attention_half.py:58-113: FP32
    scores and running sums, probabilities rounded to f16 for the PV product,
    output divided by the FP32 sum and rounded once.  FP32 inputs use an
    exact softmax rounded once.
    """
    b, lq, width = q.shape
    d = width // heads
    qh = q.to(compute).reshape(b, lq, heads, d).transpose(1, 2)
    kh = k.to(compute).reshape(b, k.shape[1], heads, d).transpose(1, 2)
    vh = v.to(compute).reshape(b, v.shape[1], heads, d).transpose(1, 2)
    s = (qh @ kh.transpose(-1, -2)) * scale
    p = torch.exp(s - s.amax(dim=-1, keepdim=True))
    total = p.sum(dim=-1, keepdim=True)
    if q.dtype in (torch.float16, torch.bfloat16):
        p = p.to(q.dtype).to(compute)
    o = (p @ vh) / total
    return o.transpose(1, 2).reshape(b, lq, width).to(q.dtype)


def timestep_embedding(timesteps: torch.Tensor, channels: int) -> torch.Tensor:
    """Sinusoidal ``[cos, sin]`` embedding in FP32 (mlx_model.py:609-612)."""
    half = channels // 2
    frequency = torch.exp(-math.log(10000) * torch.arange(half, dtype=torch.float32) / half)
    phase = timesteps[:, None].to(torch.float32) * frequency[None]
    return torch.cat([torch.cos(phase), torch.sin(phase)], dim=1)


def upsample_nearest2(x: torch.Tensor) -> torch.Tensor:
    """Duplicate every voxel along each spatial axis (_spatial.py:41-57)."""
    return x.repeat_interleave(2, 2).repeat_interleave(2, 3).repeat_interleave(2, 4)


def resize_nearest(x: torch.Tensor, shape: tuple[int, int, int]) -> torch.Tensor:
    """Resize with source index ``floor(i * in / out)`` per axis (_spatial.py:60-69)."""
    for axis, target in enumerate(shape, start=2):
        ratio = torch.tensor(x.shape[axis] / target, dtype=torch.float32)
        idx = torch.floor(torch.arange(target, dtype=torch.float32) * ratio).to(torch.int64)
        x = x.index_select(axis, idx)
    return x


def piecewise_ct(array: torch.Tensor, *, inverse: bool = False) -> torch.Tensor:
    """Four-knot HU <-> normalized map with clipping (mlx_pipeline.py:72-96)."""
    inputs, outputs = (
        ((0.0, 0.2, 0.8, 1.0), (-1000.0, -200.0, 200.0, 1000.0))
        if inverse
        else ((-1000.0, -200.0, 200.0, 1000.0), (0.0, 0.2, 0.8, 1.0))
    )
    a = array.to(torch.float32)
    result = torch.full(a.shape, outputs[0], dtype=torch.float32)
    for i in range(3):
        slope = (outputs[i + 1] - outputs[i]) / (inputs[i + 1] - inputs[i])
        inside = (a >= inputs[i]) & (a < inputs[i + 1])
        result = torch.where(inside, np.float32(slope) * (a - np.float32(inputs[i])) + np.float32(outputs[i]), result)
    return torch.where(a >= inputs[-1], torch.tensor(outputs[-1], dtype=torch.float32), result)


# ---------------------------------------------------------------- VQ search


def _f32(v: np.ndarray) -> np.ndarray:
    return v.astype(np.float32)


def codebook_norm(codebook: np.ndarray) -> np.ndarray:
    """Rounded squares summed in FP32, cast to the codebook dtype (mlx_model.py:763-767)."""
    sq = (codebook * codebook).astype(codebook.dtype).astype(np.float32)
    total = ((sq[:, 0] + sq[:, 1]) + sq[:, 2]) + sq[:, 3]
    return total.astype(codebook.dtype)


def nearest_codebook4(z: np.ndarray, codebook: np.ndarray, cb_norm: np.ndarray | None = None) -> np.ndarray:
    """Index of the nearest code for each ``(P, 4)`` vector (_vq.py:12-49, :64-82).

    Distance ``T(T(|z|^2 + |e|^2) - T(2 * T(dot)))`` in the storage dtype T,
    with the dot product as an FMA chain in FP32; smallest index on ties;
    NaN distances take priority in first-index order, as MLX argmin.
    """
    dtype = z.dtype
    if cb_norm is None:
        cb_norm = codebook_norm(codebook)
    z_norm = codebook_norm(z)
    zf = z.astype(np.float64)
    cf = codebook.astype(np.float64)
    # FMA chain: d = f32(z0 c0); d = f32(z_i c_i + d) with one rounding each
    # (float64 holds each exact product and the sum to well past f32 width).
    dot = _f32(zf[:, None, 0] * cf[None, :, 0])
    for i in range(1, 4):
        dot = _f32(zf[:, None, i] * cf[None, :, i] + dot.astype(np.float64))
    summed = (z_norm[:, None].astype(np.float32) + cb_norm[None, :].astype(np.float32)).astype(dtype)
    doubled = (np.asarray(2, dtype) * dot.astype(dtype)).astype(dtype)
    distance = (summed.astype(np.float32) - doubled.astype(np.float32)).astype(dtype)
    nan = np.isnan(distance)
    index = np.where(nan.any(axis=1), nan.argmax(axis=1), np.nanargmin(np.where(nan, np.inf, distance), axis=1))
    return index.astype(np.int32)


def quantize(z: torch.Tensor, codebook: torch.Tensor) -> torch.Tensor:
    """Straight-through ``z + (e - z)`` in the dtype (mlx_model.py:742-803)."""
    shape = z.shape
    flat = z.permute(0, 2, 3, 4, 1).reshape(-1, shape[1])
    idx = nearest_codebook4(flat.numpy(), codebook.numpy())
    selected = codebook[torch.from_numpy(idx).long()]
    quantized = flat + (selected - flat)
    return quantized.reshape(shape[0], *shape[2:], shape[1]).permute(0, 4, 1, 2, 3).contiguous()
