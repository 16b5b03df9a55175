"""Convolution operators over the C ABI: weight packing and the NDHWC conv.

This is the B200 counterpart of ``lesiondiffusion_mlx/_nax_conv.py``: the
reference packs Torch-layout ``(O, C, 3, 3, 3)`` weights once and runs an
implicit-GEMM convolution with bias / per-batch shift / residual / output
scale fused before a single rounding.  Here activations stay NDHWC on the
device, weights are packed K-major per output channel
(``[parity][O'][tap][C']``) for the tcgen05 kernel, and every call goes
through ``ldb_conv3d_fwd``.
"""

from __future__ import annotations

import ctypes
from dataclasses import dataclass

import torch

from . import _lib, instrument

MODE_CONV, MODE_STRIDE2, MODE_UP2, MODE_POINTWISE, MODE_STRIDE2_PAD01 = (
    _lib.LDB_CONV_3X3X3,
    _lib.LDB_CONV_3X3X3_S2,
    _lib.LDB_CONV_UP2,
    _lib.LDB_CONV_1X1,
    _lib.LDB_CONV_3X3X3_S2_PAD01,
)


@dataclass
class PackedWeight:
    """A weight packed for ``ldb_conv3d_fwd``.

    ``tensor`` is f16 ``(parities * rows, k_total)``; ``kind`` is ``"conv"``
    (27 taps, stride 1 or 2), ``"up"`` (8 parities x 8 folded taps) or
    ``"pointwise"`` (one tap).  ``exact`` weights hold the f16 hi plane then
    the 2^11-scaled lo plane of an FP32 weight along K.
    """

    tensor: torch.Tensor
    kind: str
    in_channels: int
    out_channels: int
    exact: bool

    @property
    def ndim(self) -> int:
        """2 for plain packing, 3 for folded upsampling (the reference's shapes)."""
        return 3 if self.kind == "up" else 2

    @property
    def dtype(self) -> torch.dtype:
        return torch.float32 if self.exact else torch.float16


def _geometry(in_channels: int, out_channels: int, mode: int, exact: bool) -> tuple[int, int]:
    desc = _lib.ConvDesc(
        batch=1, depth=1, height=1, width=1, in_channels=in_channels,
        x_ld=max(8, ((2 * ((in_channels + 15) // 16) * 16) if exact else in_channels + 7) // 8 * 8),
        out_channels=out_channels, out_ld=out_channels, res_ld=out_channels, mode=mode,
        exact=int(exact), out_dtype=_lib.LDB_F16, act=0, output_scale=1.0,
    )
    rows = ctypes.c_int(0)
    k_total = ctypes.c_int(0)
    _lib.call("ldb_conv3d_weight_rows", ctypes.byref(desc), ctypes.byref(rows), ctypes.byref(k_total))
    return rows.value, k_total.value


def _split_planes(taps: torch.Tensor) -> torch.Tensor:
    """FP32 ``(..., K)`` as f16 ``(..., 2K)``: hi then 2^11-scaled lo (_nax_conv.py:343-347)."""
    hi = taps.to(torch.float16)
    lo = ((taps - hi.to(torch.float32)) * 2048.0).to(torch.float16)
    return torch.cat([hi, lo], dim=-1)


def _pack_rows(taps: torch.Tensor, rows: int, exact: bool) -> torch.Tensor:
    """``taps`` is f32 ``(P, O, T, C')``; pad O to ``rows`` and flatten K."""
    parities, out_channels, ntaps, cpad = taps.shape
    taps = torch.nn.functional.pad(taps, (0, 0, 0, 0, 0, rows - out_channels))
    flat = taps.reshape(parities, rows, ntaps * cpad)
    packed = _split_planes(flat) if exact else flat.to(torch.float16)
    return packed.reshape(parities * rows, -1).contiguous()


def pack_weight(weight: torch.Tensor, *, stride: int = 1) -> PackedWeight:
    """Pack a Torch ``(O, C, k, k, k)`` weight (k = 3 or 1) for the conv kernel.

    Mirrors ``pack_weight`` (_nax_conv.py:350-364): input channels are
    zero-padded to a multiple of 16; an FP32 weight packs for exact mode.
    """
    if weight.ndim != 5 or weight.shape[2] != weight.shape[3] or weight.shape[3] != weight.shape[4]:
        raise ValueError(f"expected an (O, C, k, k, k) weight, got {tuple(weight.shape)}")
    exact = weight.dtype == torch.float32
    out_channels, in_channels, k = (int(s) for s in weight.shape[:3])
    if k not in (1, 3):
        raise ValueError("only 1x1x1 and 3x3x3 weights are supported")
    kind = "pointwise" if k == 1 else "conv"
    mode = MODE_POINTWISE if k == 1 else (MODE_STRIDE2 if stride == 2 else MODE_CONV)
    rows, _ = _geometry(in_channels, out_channels, mode, exact)
    cpad = (in_channels + 15) // 16 * 16
    w = weight.detach().to(torch.float32)
    taps = w.permute(0, 2, 3, 4, 1).reshape(out_channels, k ** 3, in_channels)
    taps = torch.nn.functional.pad(taps, (0, cpad - in_channels))
    return PackedWeight(_pack_rows(taps[None], rows, exact), kind, in_channels, out_channels, exact)


def pack_dense_weight(weight: torch.Tensor) -> PackedWeight:
    """Pack a ``(O, C)`` dense/linear weight as a pointwise conv."""
    if weight.ndim != 2:
        raise ValueError(f"expected an (O, C) weight, got {tuple(weight.shape)}")
    return pack_weight(weight[:, :, None, None, None])


def pack_upsample_weight(weight: torch.Tensor) -> PackedWeight:
    """Fold a ``(O, C, 3, 3, 3)`` weight into eight 2x2x2 parity filters.

    Same fold as ``pack_upsample_weight`` (_nax_conv.py:367-405): per axis,
    parity 0 uses taps (k0, k1 + k2) on source offsets (m - 1, m) and parity 1
    uses (k0 + k1, k2) on (m, m + 1).  Sums are FP32, folded axis by axis, and
    rounded to f16 once (FP32 weights keep the sums and split into planes).
    """
    if weight.ndim != 5 or tuple(weight.shape[2:]) != (3, 3, 3):
        raise ValueError(f"expected an (O, C, 3, 3, 3) weight, got {tuple(weight.shape)}")
    exact = weight.dtype == torch.float32
    out_channels, in_channels = int(weight.shape[0]), int(weight.shape[1])
    rows, _ = _geometry(in_channels, out_channels, MODE_UP2, exact)
    cpad = (in_channels + 15) // 16 * 16
    w = weight.detach().to(torch.float32)

    def fold(t: torch.Tensor, dim: int) -> torch.Tensor:
        k0, k1, k2 = t.unbind(dim)
        return torch.stack([torch.stack([k0, k1 + k2], dim), torch.stack([k0 + k1, k2], dim)], dim)

    f = fold(w, 2)        # (O, C, pd, td, kh, kw)
    f = fold(f, 4)        # (O, C, pd, td, ph, th, kw)
    f = fold(f, 6)        # (O, C, pd, td, ph, th, pw, tw)
    f = f.permute(2, 4, 6, 0, 3, 5, 7, 1)  # (pd, ph, pw, O, td, th, tw, C)
    f = f.reshape(8, out_channels, 8, in_channels)
    f = torch.nn.functional.pad(f, (0, cpad - in_channels))
    return PackedWeight(_pack_rows(f, rows, exact), "up", in_channels, out_channels, exact)


def _ptr(t: torch.Tensor | None) -> int | None:
    return None if t is None else t.data_ptr()


def _dense_ld(shape, strides, what: str) -> int:
    """Channel stride of an NDHWC layout that is dense over voxels (only the
    channel stride may exceed C)."""
    if len(shape) != 5 or (strides[4] != 1 and shape[4] != 1):
        raise ValueError(f"{what} must be (B, D, H, W, C) with unit channel stride")
    ld = int(strides[3])
    expect = ld
    for dim in (3, 2, 1, 0):
        if int(shape[dim]) != 1 and int(strides[dim]) != expect:
            raise ValueError(f"{what} must be dense over voxels (only the channel stride may exceed C)")
        expect *= int(shape[dim])
    return ld


def conv_geometry(x_shape, x_strides, packed: PackedWeight, *, stride: int = 1,
                  in_channels: int | None = None, depth_halo: int = 0,
                  pad01: bool = False) -> tuple[int, tuple[int, int, int], int, int]:
    """Validate an NDHWC input layout for ``packed``; return (mode, output grid, x_ld, cin).

    With ``depth_halo`` = 1 the first and last depth slices of x are halo
    slices read by the taps and the output covers the interior slices.  With
    ``pad01`` a stride-2 conv pads with zeros only after each axis (the VQ
    encoder's downsample, mlx_model.py:735-736).
    Pure host logic (no device access), shared by ``conv3d_ndhwc`` and the CPU tests.
    """
    x_ld = _dense_ld(x_shape, x_strides, "x")
    if depth_halo not in (0, 1):
        raise ValueError("depth_halo must be 0 or 1")
    depth, height, width = (int(s) for s in x_shape[1:4])
    depth -= 2 * depth_halo
    if depth <= 0:
        raise ValueError("x has no interior depth slice")
    if depth_halo and stride != 1:
        raise ValueError("a depth halo needs stride 1")
    cin = packed.in_channels if in_channels is None else in_channels
    if packed.kind == "up":
        if stride != 1:
            raise ValueError("upsampling convolution has stride 1")
        return MODE_UP2, (2 * depth, 2 * height, 2 * width), x_ld, cin
    if packed.kind == "pointwise":
        if stride != 1:
            raise ValueError("pointwise convolution has stride 1")
        return MODE_POINTWISE, (depth, height, width), x_ld, cin
    if stride == 2 and pad01:
        if min(depth, height, width) < 2:
            raise ValueError("padding (0, 1) with stride 2 needs extents >= 2")
        return MODE_STRIDE2_PAD01, tuple((n - 2) // 2 + 1 for n in (depth, height, width)), x_ld, cin
    if pad01:
        raise ValueError("pad01 applies to stride-2 convolutions")
    if stride == 2:
        return MODE_STRIDE2, tuple((n - 1) // 2 + 1 for n in (depth, height, width)), x_ld, cin
    if stride != 1:
        raise ValueError("stride must be 1 or 2")
    return MODE_CONV, (depth, height, width), x_ld, cin


def conv3d_ndhwc(
    x: torch.Tensor,
    packed: PackedWeight,
    bias: torch.Tensor | None = None,
    *,
    stride: int = 1,
    shift: torch.Tensor | None = None,
    residual: torch.Tensor | None = None,
    output_scale: float = 1.0,
    act: int = _lib.LDB_ACT_NONE,
    out: torch.Tensor | None = None,
    out_dtype: torch.dtype | None = None,
    in_channels: int | None = None,
    stats: torch.Tensor | None = None,
    depth_halo: int = 0,
    pad01: bool = False,
    max_ctas: int = 0,
) -> torch.Tensor:
    """Convolve NDHWC ``x`` ``(B, D, H, W, C)`` (channel stride = ``x.stride(3)``).

    ``x`` is f16 (or, for exact weights, the split hi/lo f16 planes from
    ``prepare_input``).  ``bias`` is f32 ``(O,)``; ``shift`` f32 ``(B, O)``;
    ``residual`` has the output's dtype and shape.  The output is NDHWC with
    ``O`` channels; a new output has its channel stride padded to 8 so it can
    feed the next convolution.  Stride applies only to ``kind == "conv"``.
    With ``stats`` (float64 ``(B, O, 2)``, zero on entry) the kernel also adds
    each channel's sum and sum of squares of the stored output: the GroupNorm
    statistics that ``ops.group_norm_affine_from_stats`` consumes.  With
    ``depth_halo`` = 1, x's first and last depth slices are a neighbour's
    slices (depth-sharded volumes) and the output covers the interior.
    """
    if x.device.type != "cuda":
        raise ValueError("conv3d_ndhwc needs CUDA tensors")
    if x.dtype != torch.float16:
        raise ValueError(f"conv input must be float16 (split planes for FP32), got {x.dtype}")
    mode, grid, x_ld, cin = conv_geometry(tuple(x.shape), tuple(x.stride()), packed, stride=stride,
                                          in_channels=in_channels, depth_halo=depth_halo, pad01=pad01)
    batch = int(x.shape[0])
    cout = packed.out_channels
    if out_dtype is None:
        out_dtype = torch.float32 if packed.exact else torch.float16
    if out is None:
        out_ld = (cout + 7) // 8 * 8
        out = torch.empty((batch, *grid, out_ld), device=x.device, dtype=out_dtype)[..., :cout]
    if out.dtype != out_dtype or tuple(out.shape) != (batch, *grid, cout):
        raise ValueError(f"out must be {(batch, *grid, cout)} {out_dtype}")
    out_ld = _dense_ld(tuple(out.shape), tuple(out.stride()), "out")
    res_ld = cout
    if residual is not None:
        if tuple(residual.shape) != (batch, *grid, cout) or residual.dtype != out_dtype:
            raise ValueError(f"residual shape {tuple(residual.shape)} {residual.dtype} != output "
                             f"{(batch, *grid, cout)} {out_dtype}")
        res_ld = _dense_ld(tuple(residual.shape), tuple(residual.stride()), "residual")
    if bias is not None and (bias.dtype != torch.float32 or bias.numel() != cout or not bias.is_contiguous()):
        raise ValueError("bias must be a contiguous float32 (O,) tensor")
    if shift is not None and (shift.dtype != torch.float32 or tuple(shift.shape) != (batch, cout)
                              or not shift.is_contiguous()):
        raise ValueError("shift must be a contiguous float32 (B, O) tensor")
    depth, height, width = (int(s) for s in x.shape[1:4])
    desc = _lib.ConvDesc(
        batch=batch, depth=depth, height=height, width=width, in_channels=cin, x_ld=x_ld,
        out_channels=cout, out_ld=out_ld, res_ld=res_ld, mode=mode, exact=int(packed.exact),
        out_dtype=_lib.LDB_F32 if out_dtype == torch.float32 else _lib.LDB_F16, act=act,
        output_scale=float(output_scale), depth_halo=depth_halo, max_ctas=int(max_ctas),
    )
    ws_bytes = ctypes.c_size_t(0)
    _lib.call("ldb_conv3d_workspace_size", ctypes.byref(desc), ctypes.byref(ws_bytes))
    workspace = None
    if ws_bytes.value:
        workspace = torch.empty(ws_bytes.value, dtype=torch.uint8, device=x.device)
    stream = torch.cuda.current_stream(x.device).cuda_stream
    taps = {MODE_POINTWISE: 1, MODE_UP2: 8}.get(mode, 27)
    flops = 2.0 * batch * grid[0] * grid[1] * grid[2] * cout * taps * cin
    if stats is not None and (stats.dtype != torch.float64 or tuple(stats.shape) != (batch, cout, 2)
                              or not stats.is_contiguous()):
        raise ValueError(f"stats must be a contiguous float64 {(batch, cout, 2)} tensor")
    label = f"mode{mode} B{batch} {grid[0]}x{grid[1]}x{grid[2]} {cin}->{cout}{' exact' if packed.exact else ''}"
    desc.clock = instrument.device_clock("conv3d", flops, x.device, label)
    with instrument.maybe_time("conv3d", flops, device_clocked=desc.clock is not None):
        if stats is None:
            _lib.call(
                "ldb_conv3d_fwd", stream, ctypes.byref(desc), x.data_ptr(), packed.tensor.data_ptr(), _ptr(bias),
                _ptr(shift), _ptr(residual), out.data_ptr(), _ptr(workspace), ws_bytes.value,
            )
        else:
            _lib.call(
                "ldb_conv3d_fwd_gn_stats", stream, ctypes.byref(desc), x.data_ptr(), packed.tensor.data_ptr(),
                _ptr(bias), _ptr(shift), _ptr(residual), out.data_ptr(), stats.data_ptr(), _ptr(workspace),
                ws_bytes.value,
            )
    return out
