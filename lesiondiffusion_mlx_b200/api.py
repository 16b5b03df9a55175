"""Drop-in operator API with the reference's names, arguments and errors.

These functions mirror lesiondiffusion_mlx's native-kernel operators
(``_nax_conv.py``, ``_attention.py``, ``_vq.py``, ``_spatial.py``,
``mlx_pipeline.piecewise_ct``) and medmlx-core's group-norm helpers on
``torch`` CUDA tensors in the reference's NCDHW / projection layouts.  Each
call converts to NDHWC where needed and runs the B200 kernels through the C
ABI; there is no other compute path.  The trailing ``mx`` keyword of the
reference signatures is accepted and ignored, so call sites port unchanged.
"""

from __future__ import annotations

import torch

from . import _lib, ops
from .conv import PackedWeight, conv3d_ndhwc
from .conv import pack_upsample_weight as _pack_upsample
from .conv import pack_weight as _pack

__all__ = [
    "nax_available", "nax_eligible", "pack_weight", "pack_upsample_weight", "nax_conv3d", "flash_eligible",
    "flash_attention", "flash_attention_half", "group_norm_affine", "native_group_norm",
    "native_group_norm_eligible", "nearest_codebook4", "upsample_nearest2",
    "resize_nearest", "piecewise_ct",
]


def _to_ndhwc(x: torch.Tensor, pad_to: int = 8) -> torch.Tensor:
    """NCDHW -> NDHWC f16/f32 view whose channel stride is a multiple of ``pad_to``."""
    b, c, d, h, w = x.shape
    width = (c + pad_to - 1) // pad_to * pad_to
    buf = torch.empty((b, d, h, w, width), dtype=x.dtype, device=x.device)
    if width > c:
        buf[..., c:].zero_()
    buf[..., :c].copy_(x.permute(0, 2, 3, 4, 1))
    return buf[..., :c]


def _to_ncdhw(x: torch.Tensor) -> torch.Tensor:
    return x.permute(0, 4, 1, 2, 3).contiguous()


def nax_available(mx=None) -> bool:
    """Whether the B200 kernels can run: a CUDA device and the built C library (_nax_conv.py:301-312)."""
    if not torch.cuda.is_available():
        return False
    try:
        _lib.library()
    except ImportError:
        return False
    major, _ = torch.cuda.get_device_capability()
    return major >= 10


def nax_eligible(weight: torch.Tensor) -> bool:
    """A Torch-layout ``(O, C, 3, 3, 3)`` weight fits the conv kernel (_nax_conv.py:321-328)."""
    return weight.ndim == 5 and tuple(weight.shape[2:]) == (3, 3, 3)


def pack_weight(weight: torch.Tensor, mx=None, *, stride: int = 1) -> PackedWeight:
    """Pack ``(O, C, 3, 3, 3)`` (f16, or f32 for exact mode) for ``nax_conv3d`` (_nax_conv.py:350-364)."""
    return _pack(weight, stride=stride)


def pack_upsample_weight(weight: torch.Tensor, mx=None) -> PackedWeight:
    """Fold ``(O, C, 3, 3, 3)`` into eight 2x2x2 parity filters (_nax_conv.py:367-405)."""
    return _pack_upsample(weight)


def nax_conv3d(
    x: torch.Tensor, packed: PackedWeight, bias: torch.Tensor, *, affine: torch.Tensor | None = None,
    silu: bool = False, stride: int = 1, upsample: bool = False, output_scale: float = 1.0,
    residual: torch.Tensor | None = None, mx=None,
) -> torch.Tensor:
    """Padding-1 3x3x3 convolution of NCDHW ``x`` in its dtype (_nax_conv.py:451-619).

    f16 ``x``: the prepared input (optional per-(b, c) affine, then SiLU) is
    rounded to f16 once, products accumulate in FP32, bias (``(O,)`` or per
    batch ``(B, O)``) is added before ``output_scale``, the residual after,
    and the result rounds once.  f32 ``x`` runs the split-f16 exact mode and
    returns float32.  Raises ``ValueError`` when ``packed`` does not match
    ``x``'s channels and dtype or ``residual`` does not have the output's shape.
    """
    if x.ndim != 5:
        raise ValueError("nax_conv3d expects NCDHW input")
    exact = x.dtype == torch.float32
    if packed.exact != exact:
        raise ValueError(f"packed weight rows do not fit {int(x.shape[1])} {'float32' if exact else 'float16'} "
                         "input channels")
    if int(x.shape[1]) != packed.in_channels:
        raise ValueError(f"packed weight rows do not fit {int(x.shape[1])} input channels")
    if upsample != (packed.kind == "up"):
        raise ValueError("upsample=True needs pack_upsample_weight weights (and only those)")
    if stride not in (1, 2) or (upsample and stride != 1):
        raise ValueError("stride must be 1 or 2 (1 with upsample)")
    batch = int(x.shape[0])
    grid = tuple(int(n) for n in x.shape[2:])
    if upsample:
        out_grid = tuple(2 * n for n in grid)
    elif stride == 2:
        out_grid = tuple((n - 1) // 2 + 1 for n in grid)
    else:
        out_grid = grid
    cout = packed.out_channels
    if residual is not None and tuple(residual.shape) != (batch, cout, *out_grid):
        raise ValueError(f"residual shape {tuple(residual.shape)} != output {(batch, cout, *out_grid)}")
    xl = _to_ndhwc(x)
    if affine is not None:
        affine = affine.reshape(batch, int(x.shape[1]), 2).to(torch.float32).contiguous()
    if exact or affine is not None or silu:
        prepared = ops.prepare_input(xl, affine=affine, silu=silu, split=exact)
    else:
        prepared = xl
    bias32 = bias.to(torch.float32)
    shift = None
    if bias32.ndim == 2:
        shift, bias32 = bias32.contiguous(), None
    else:
        bias32 = bias32.contiguous()
    res = None if residual is None else _to_ndhwc(residual)
    out = conv3d_ndhwc(prepared, packed, bias32, stride=stride, shift=shift, residual=res,
                       output_scale=output_scale, in_channels=int(x.shape[1]))
    return _to_ncdhw(out)


def flash_eligible(q: torch.Tensor, k: torch.Tensor, heads: int, mx=None) -> bool:
    """Projections ``(B, L, heads * d)`` the attention kernel takes: d in {16, 32, 64}, f16/bf16."""
    if q.dtype != k.dtype or q.dtype not in (torch.float16, torch.bfloat16) or q.ndim != 3 or k.ndim != 3:
        return False
    width = int(q.shape[-1])
    return width % heads == 0 and width // heads in (16, 32, 64) and int(k.shape[-1]) == width


def flash_attention(q: torch.Tensor, k: torch.Tensor, v: torch.Tensor, *, heads: int, scale: float,
                    mx=None) -> torch.Tensor:
    """Multi-head attention on head-interleaved projections (_attention.py:331-375)."""
    return ops.flash_attention(q.contiguous(), k.contiguous(), v.contiguous(), heads=heads, scale=scale)


def flash_attention_half(q: torch.Tensor, k: torch.Tensor, v: torch.Tensor, *, heads: int, scale: float,
                         mx=None) -> torch.Tensor:
    """FP16 attention on head-interleaved projections, returning q's shape in
    float16 (_attention_half.py:129-147).  The reference's kernel takes 32-wide
    heads over equal query / key lengths that are multiples of 32 and leaves that
    dispatch to the caller; the tcgen05 kernel here also takes 16- and 64-wide
    heads and any lengths, with the same result where both apply."""
    if not (q.dtype == k.dtype == v.dtype == torch.float16):
        raise ValueError(f"flash_attention_half takes float16 projections, got {q.dtype}, {k.dtype}, {v.dtype}")
    return flash_attention(q, k, v, heads=heads, scale=scale)


def group_norm_affine(x: torch.Tensor, weight: torch.Tensor, bias: torch.Tensor, *, groups: int, eps: float,
                      mx=None) -> torch.Tensor:
    """Flat ``(B * C * 2)`` FP32 ``(scale, offset)`` pairs of GroupNorm on NCDHW ``x``."""
    affine = ops.group_norm_affine(_to_ndhwc(x), weight, bias, groups=groups, eps=eps)
    return affine.reshape(-1)


def native_group_norm_eligible(x: torch.Tensor, groups: int, mx=None) -> bool:
    """Whether ``group_norm_affine`` / ``native_group_norm`` take ``x`` with ``groups``
    groups: the predicate the reference's layers test before their native
    GroupNorm (medmlx-core, called at mlx_model.py:240, :268, :321).  Here: a
    5-D NCDHW float16 / float32 tensor whose channels are a multiple of 8 that
    ``groups`` divides, at most 1024 channels per group and 8192 in all."""
    if x.ndim != 5 or x.dtype not in (torch.float16, torch.float32) or groups <= 0:
        return False
    c = int(x.shape[1])
    return c % 8 == 0 and c % groups == 0 and c // groups <= 1024 and c <= 8192


def native_group_norm(x: torch.Tensor, weight: torch.Tensor, bias: torch.Tensor, *, groups: int, eps: float,
                      silu: bool = False, mx=None) -> torch.Tensor:
    """GroupNorm (+ SiLU) in FP32 with one rounding to ``x``'s dtype, NCDHW."""
    xl = _to_ndhwc(x)
    affine = ops.group_norm_affine(xl, weight, bias, groups=groups, eps=eps)
    if x.dtype == torch.float16:
        return _to_ncdhw(ops.prepare_input(xl, affine=affine, silu=silu))
    split = ops.prepare_input(xl, affine=affine, silu=silu, split=True)
    c = int(x.shape[1])
    cpad = split.shape[-1] // 2
    value = split[..., :c].float() + split[..., cpad : cpad + c].float() / 2048.0
    return _to_ncdhw(value)


def nearest_codebook4(z: torch.Tensor, codebook: torch.Tensor, codebook_norm: torch.Tensor | None = None,
                      mx=None) -> torch.Tensor:
    """int32 nearest-code indices of ``(P, 4)`` vectors (_vq.py:64-82)."""
    if z.ndim != 2 or z.shape[1] != 4:
        raise ValueError("nearest_codebook4 expects (positions, 4) vectors")
    return ops.vq_nearest4(z.contiguous()[None], codebook.contiguous())[0]


def upsample_nearest2(x: torch.Tensor, *, mx=None) -> torch.Tensor:
    """Nearest 2x upsampling of NCDHW ``x`` (_spatial.py:41-57)."""
    return resize_nearest(x, tuple(2 * int(s) for s in x.shape[2:]))


def resize_nearest(x: torch.Tensor, shape: tuple[int, ...], *, mx=None) -> torch.Tensor:
    """NCDHW nearest resize with source index floor(i * in / out) (_spatial.py:60-69)."""
    if len(shape) != 3:
        raise ValueError("LesionDiffusion nearest resizing needs three spatial axes")
    if x.ndim != 5:
        raise ValueError("resize_nearest expects NCDHW input")
    # rows are copied whole, so resize the channel-padded buffer (rows a
    # multiple of 8 bytes) and drop the padding afterwards
    c = int(x.shape[1])
    padded = _to_ndhwc(x, max(1, 8 // x.element_size()))
    full = padded.as_strided((*padded.shape[:-1], padded.stride(-2)), padded.stride())
    out = ops.resize_nearest(full, tuple(int(s) for s in shape))
    return _to_ncdhw(out[..., :c])


def piecewise_ct(array: torch.Tensor, mx=None, *, inverse: bool = False) -> torch.Tensor:
    """Four-knot CT map on the device (mlx_pipeline.py:72-96): HU -> normalized,
    or normalized -> HU with ``inverse=True``; float32 result of ``array``'s shape."""
    if inverse:
        flat = array.reshape(1, -1, 1)
        return ops.hu_map(flat).reshape(array.shape)
    flat = array.to(torch.float32).contiguous().reshape(1, -1)
    return ops.ct_normalize(flat, out_dtype=torch.float32, pad_to=1).reshape(array.shape)
