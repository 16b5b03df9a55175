"""NDHWC device operators over the C ABI (everything except the conv, which
lives in ``conv.py``).

Activations are channels-last ``torch`` CUDA tensors: volumes ``(B, D, H, W,
C)`` and token matrices ``(B, L, C)``.  A tensor may be a channel slice of a
wider buffer (its channel stride is ``stride(-2)``).  Each function checks
shapes, dtypes and alignment, then launches on the current stream.
"""

from __future__ import annotations

import ctypes

import torch

from . import _lib, instrument

_DT = {torch.float16: _lib.LDB_F16, torch.float32: _lib.LDB_F32, torch.bfloat16: _lib.LDB_BF16}


def _stream(t: torch.Tensor) -> int:
    return torch.cuda.current_stream(t.device).cuda_stream


def _ptr(t: torch.Tensor | None) -> int | None:
    return None if t is None else t.data_ptr()


def _rows(t: torch.Tensor) -> tuple[int, int, int]:
    """(voxels per batch item, channels, channel stride) of a channels-last tensor."""
    if t.stride(-1) != 1 and t.shape[-1] != 1:
        raise ValueError("channel axis must have unit stride")
    ld = int(t.stride(-2)) if t.ndim >= 2 else int(t.shape[-1])
    per = 1
    for s in t.shape[1:-1]:
        per *= int(s)
    # dense over voxels: stride of dim i == ld * prod(shape[i+1:-1])
    expect = ld
    for i in range(t.ndim - 2, 0, -1):
        if int(t.stride(i)) != expect and int(t.shape[i]) != 1:
            raise ValueError("tensor must be dense over voxels (only the channel stride may exceed C)")
        expect *= int(t.shape[i])
    return per, int(t.shape[-1]), ld


def group_norm_affine(
    x: torch.Tensor, gamma: torch.Tensor | None, beta: torch.Tensor | None, *, groups: int, eps: float,
    x2: torch.Tensor | None = None,
) -> torch.Tensor:
    """Per-(batch, channel) FP32 GroupNorm affine ``(B, C, 2)`` of ``[x | x2]``."""
    voxels, c1, ld1 = _rows(x)
    c2, ld2 = 0, 0
    if x2 is not None:
        v2, c2, ld2 = _rows(x2)
        if v2 != voxels or x2.shape[0] != x.shape[0] or x2.dtype != x.dtype:
            raise ValueError("concatenated sources must share batch, voxels and dtype")
    batch = int(x.shape[0])
    channels = c1 + c2
    ws = ctypes.c_size_t(0)
    _lib.call("ldb_group_norm_workspace_size", batch, voxels, channels, ctypes.byref(ws))
    workspace = torch.empty(ws.value, dtype=torch.uint8, device=x.device)
    affine = torch.empty((batch, channels, 2), dtype=torch.float32, device=x.device)
    g = None if gamma is None else gamma.to(torch.float32).contiguous()
    b = None if beta is None else beta.to(torch.float32).contiguous()
    with instrument.maybe_time("group_norm", 0.0):
        _lib.call(
            "ldb_group_norm_affine", _stream(x), x.data_ptr(), c1, ld1, _ptr(x2), c2, ld2, _DT[x.dtype], batch,
            voxels, groups, _ptr(g), _ptr(b), float(eps), affine.data_ptr(), workspace.data_ptr(), ws.value,
        )
    return affine


def prepare_input(
    x: torch.Tensor, *, affine: torch.Tensor | None = None, silu: bool = False, split: bool = False,
    x2: torch.Tensor | None = None, out: torch.Tensor | None = None,
) -> torch.Tensor:
    """``f16(silu?(x * scale + offset))`` over ``[x | x2]``, or the split hi/lo planes.

    Without ``split`` the output has ``C`` channels padded to a multiple of 8
    (returned as a ``C``-channel view); with ``split`` it holds the hi plane
    then the 2^11-scaled lo plane, each padded to 16 channels.
    """
    voxels, c1, ld1 = _rows(x)
    c2, ld2 = 0, 0
    if x2 is not None:
        _, c2, ld2 = _rows(x2)
    channels = c1 + c2
    if affine is not None and (affine.dtype != torch.float32 or tuple(affine.shape) != (x.shape[0], channels, 2)):
        raise ValueError("affine must be float32 (B, C, 2)")
    cpad = (channels + 15) // 16 * 16 if split else (channels + 7) // 8 * 8
    width = 2 * cpad if split else cpad
    lead = tuple(int(s) for s in x.shape[:-1])
    if out is None:
        out = torch.empty((*lead, width), dtype=torch.float16, device=x.device)
    _, _, out_ld = _rows(out)
    with instrument.maybe_time("prepare", 0.0):
        _lib.call(
            "ldb_prepare_input", _stream(x), x.data_ptr(), c1, ld1, _ptr(x2), c2, ld2, _DT[x.dtype],
            int(x.shape[0]), voxels, _ptr(affine), int(silu), int(split), out.data_ptr(), out_ld,
        )
    return out if split else out[..., :channels]


def group_norm_affine_from_stats(
    stats: torch.Tensor, gamma: torch.Tensor | None, beta: torch.Tensor | None, *, voxels: int, groups: int,
    eps: float, stats2: torch.Tensor | None = None,
) -> torch.Tensor:
    """``group_norm_affine`` from producer statistics: float64 ``(B, C, 2)`` sums
    and sums of squares per source (as ``conv3d_ndhwc(..., stats=...)``
    accumulates them) over ``voxels`` voxels per batch item."""
    if stats.dtype != torch.float64 or stats.ndim != 3 or stats.shape[2] != 2 or not stats.is_contiguous():
        raise ValueError("stats must be a contiguous float64 (B, C, 2) tensor")
    batch, c1 = int(stats.shape[0]), int(stats.shape[1])
    c2 = 0
    if stats2 is not None:
        if stats2.dtype != torch.float64 or stats2.shape[0] != batch or not stats2.is_contiguous():
            raise ValueError("stats2 must be a contiguous float64 (B, C2, 2) tensor")
        c2 = int(stats2.shape[1])
    affine = torch.empty((batch, c1 + c2, 2), dtype=torch.float32, device=stats.device)
    g = None if gamma is None else gamma.to(torch.float32).contiguous()
    b = None if beta is None else beta.to(torch.float32).contiguous()
    with instrument.maybe_time("group_norm", 0.0):
        _lib.call("ldb_group_norm_affine_from_stats", torch.cuda.current_stream(stats.device).cuda_stream,
                  stats.data_ptr(), c1, _ptr(stats2), c2, batch, int(voxels), groups, _ptr(g), _ptr(b), float(eps),
                  affine.data_ptr())
    return affine


def prepare_input_from_stats(
    x: torch.Tensor, stats: torch.Tensor, gamma: torch.Tensor | None, beta: torch.Tensor | None, *, groups: int,
    eps: float, silu: bool = False, split: bool = False, x2: torch.Tensor | None = None,
    stats2: torch.Tensor | None = None, out: torch.Tensor | None = None, voxels: int | None = None,
) -> torch.Tensor:
    """``prepare_input(x, affine=group_norm_affine_from_stats(stats, ...))`` in
    one launch.  ``voxels`` is the count per batch item the statistics cover
    (default: those of ``x``; larger for one slab of a sharded volume)."""
    per_batch, c1, ld1 = _rows(x)
    batch = int(x.shape[0])
    c2, ld2 = 0, 0
    if x2 is not None:
        _, c2, ld2 = _rows(x2)
    for s, c in ((stats, c1), (stats2, c2)):
        if s is None and c == 0:
            continue
        if (s is None or s.dtype != torch.float64 or tuple(s.shape) != (batch, c, 2) or not s.is_contiguous()):
            raise ValueError(f"stats must be contiguous float64 {(batch, c, 2)} tensors, one per source")
    channels = c1 + c2
    cpad = (channels + 15) // 16 * 16 if split else (channels + 7) // 8 * 8
    width = 2 * cpad if split else cpad
    lead = tuple(int(s) for s in x.shape[:-1])
    if out is None:
        out = torch.empty((*lead, width), dtype=torch.float16, device=x.device)
    _, _, out_ld = _rows(out)
    g = None if gamma is None else gamma.to(torch.float32).contiguous()
    b = None if beta is None else beta.to(torch.float32).contiguous()
    with instrument.maybe_time("prepare", 0.0):
        _lib.call(
            "ldb_prepare_input_from_stats", _stream(x), x.data_ptr(), c1, ld1, _ptr(x2), c2, ld2, _DT[x.dtype],
            batch, per_batch, int(voxels or 0), stats.data_ptr(), _ptr(stats2), groups, _ptr(g), _ptr(b), float(eps), int(silu),
            int(split), out.data_ptr(), out_ld,
        )
    return out if split else out[..., :channels]


def layer_norm(x: torch.Tensor, gamma: torch.Tensor, beta: torch.Tensor, eps: float = 1e-5,
               out: torch.Tensor | None = None, split: bool = False) -> torch.Tensor:
    """Last-axis LayerNorm of f16 or f32 rows in FP32; ``gamma``/``beta`` f32.

    The output is f16; with ``split`` it holds the hi plane then the
    2^11-scaled low plane (each padded to 16 channels), the input format of
    the FP32-exact conv."""
    if x.dtype not in (torch.float16, torch.float32):
        raise ValueError("layer_norm expects float16 or float32")
    voxels, c, ld = _rows(x)
    rows = int(x.shape[0]) * voxels
    cpad = (c + 15) // 16 * 16
    if out is None:
        out = torch.empty((*x.shape[:-1], 2 * cpad if split else c), dtype=torch.float16, device=x.device)
    _, _, out_ld = _rows(out)
    with instrument.maybe_time("layer_norm", 0.0):
        _lib.call("ldb_layer_norm_ex", _stream(x), x.data_ptr(), _DT[x.dtype], ld, gamma.data_ptr(), beta.data_ptr(),
                  float(eps), out.data_ptr(), out_ld, rows, c, int(split))
    return out


def flash_attention(q: torch.Tensor, k: torch.Tensor, v: torch.Tensor, *, heads: int, scale: float,
                    out: torch.Tensor | None = None) -> torch.Tensor:
    """``softmax(q k^T * scale) v`` per head on projection-layout ``(B, L, H*D)`` tensors.

    float16 / bfloat16 inputs run the tcgen05 flash kernel directly; float32
    inputs (16-, 32- or 64-wide heads; the reference's FP32 kernel, _attention.py:148-375)
    run it in the split-f16 form and return float32."""
    if q.ndim != 3 or k.ndim != 3 or v.ndim != 3:
        raise ValueError("attention inputs are (B, L, heads * head_dim)")
    if q.dtype == torch.float32 and k.dtype == q.dtype and v.dtype == q.dtype:
        return _flash_attention_f32(q, k, v, heads=heads, scale=scale, out=out)
    if q.dtype not in (torch.float16, torch.bfloat16) or k.dtype != q.dtype or v.dtype != q.dtype:
        raise ValueError("attention inputs must share dtype float16, bfloat16 or float32")
    batch, lq, width = (int(s) for s in q.shape)
    lk = int(k.shape[1])
    if width % heads:
        raise ValueError("projection width must divide evenly into heads")
    if k.stride(1) != v.stride(1) or k.stride(0) != v.stride(0):
        raise ValueError("k and v must share strides")
    for t in (q, k, v):
        if t.stride(2) != 1 or t.stride(0) != t.shape[1] * t.stride(1):
            raise ValueError("attention inputs must be row-major with unit column stride")
    if out is None:
        out = torch.empty((batch, lq, width), dtype=q.dtype, device=q.device)
    ws_bytes = ctypes.c_size_t(0)
    _lib.call("ldb_flash_attention_workspace_size", batch, lq, lk, heads, width // heads, ctypes.byref(ws_bytes))
    ws = torch.empty(ws_bytes.value, dtype=torch.uint8, device=q.device) if ws_bytes.value else None
    flops = 4.0 * batch * lq * lk * width
    clock = instrument.device_clock("attention", flops, q.device, f"B{batch} {lq}x{lk} h{heads}x{width // heads}")
    with instrument.maybe_time("attention", flops, device_clocked=clock is not None):
        _lib.call(
            "ldb_flash_attention_timed", _stream(q), q.data_ptr(), int(q.stride(1)), k.data_ptr(), v.data_ptr(),
            int(k.stride(1)), out.data_ptr(), int(out.stride(1)), batch, lq, lk, heads, width // heads,
            float(scale), _DT[q.dtype], _ptr(ws), ws_bytes.value, clock,
        )
    return out


def _flash_attention_f32(q: torch.Tensor, k: torch.Tensor, v: torch.Tensor, *, heads: int, scale: float,
                         out: torch.Tensor | None) -> torch.Tensor:
    batch, lq, width = (int(s) for s in q.shape)
    lk = int(k.shape[1])
    if width % heads or width // heads not in (16, 32, 64):
        raise ValueError("FP32 attention takes heads 16, 32 or 64 wide")
    d = width // heads
    if k.stride(1) != v.stride(1) or k.stride(0) != v.stride(0):
        raise ValueError("k and v must share strides")
    for t in (q, k, v):
        if t.stride(2) != 1 or t.stride(0) != t.shape[1] * t.stride(1):
            raise ValueError("attention inputs must be row-major with unit column stride")
    if out is None:
        out = torch.empty((batch, lq, width), dtype=torch.float32, device=q.device)
    ws_bytes = ctypes.c_size_t(0)
    _lib.call("ldb_flash_attention_f32_workspace_size", batch, lq, lk, heads, d, ctypes.byref(ws_bytes))
    ws = torch.empty(ws_bytes.value, dtype=torch.uint8, device=q.device)
    with instrument.maybe_time("attention", 4.0 * batch * lq * lk * width):
        _lib.call(
            "ldb_flash_attention_f32", _stream(q), q.data_ptr(), int(q.stride(1)), k.data_ptr(), v.data_ptr(),
            int(k.stride(1)), out.data_ptr(), int(out.stride(1)), batch, lq, lk, heads, d, float(scale),
            ws.data_ptr(), ws_bytes.value,
        )
    return out


def timestep_embedding(timesteps: torch.Tensor, channels: int, *, step: torch.Tensor | None = None,
                       out_dtype: torch.dtype = torch.float32, out: torch.Tensor | None = None) -> torch.Tensor:
    """[cos, sin] embedding of int32 ``timesteps`` ``(B,)`` (or row ``*step`` of a ``(S, B)`` table;
    a step outside the table writes nothing and sets the device status, ``ldb_device_status``)."""
    if timesteps.dtype != torch.int32:
        raise ValueError("timesteps must be int32")
    batch = int(timesteps.shape[-1])
    steps = int(timesteps.numel() // max(batch, 1))
    if out is None:
        out = torch.empty((batch, channels), dtype=out_dtype, device=timesteps.device)
    _lib.call("ldb_timestep_embedding", _stream(timesteps), timesteps.data_ptr(), _ptr(step), steps, batch,
              channels, out.data_ptr(), _DT[out.dtype])
    return out


def dense_small(x: torch.Tensor, weight: torch.Tensor, bias: torch.Tensor | None, *, in_silu: bool = False,
                out_silu: bool = False, out_dtype: torch.dtype = torch.float16, round_f16: bool = False,
                out: torch.Tensor | None = None) -> torch.Tensor:
    """Dense layer for 1..16 rows: ``silu?(silu?(x) @ weight^T + bias)``."""
    if x.dtype != torch.float16 or weight.dtype != torch.float16:
        raise ValueError("dense_small expects float16 x and weight")
    rows, k = int(x.shape[0]), int(x.shape[1])
    n = int(weight.shape[0])
    if out is None:
        out = torch.empty((rows, n), dtype=out_dtype, device=x.device)
    with instrument.maybe_time("dense_small", 0.0):
        _lib.call(
            "ldb_dense_small", _stream(x), x.data_ptr(), int(x.stride(0)), weight.data_ptr(), _ptr(bias),
            out.data_ptr(), int(out.stride(0)), rows, n, k, int(in_silu), int(out_silu), _DT[out.dtype],
            int(round_f16),
        )
    return out


def sampler_step(
    kind: int, x: torch.Tensor, *, eps: torch.Tensor | None = None, prev: torch.Tensor | None = None,
    noise: torch.Tensor | None = None, noise_step_stride: int = 0, mask: torch.Tensor | None = None,
    image: torch.Tensor | None = None, net_in: torch.Tensor | None = None, coeff: torch.Tensor | None = None,
    step: torch.Tensor | None = None, net_split: bool = False,
) -> None:
    """One fused sampler step over the f32 state ``x`` (B, V..., C) (see ldb_sampler_step_ex).

    ``eps`` is the f16 or f32 prediction; with ``net_split`` the next network
    input is written in the FP32-exact split format (hi plane, then 2^11-scaled
    low plane, each padded to 16 channels).  With ``step`` the coefficient and
    noise tables are read at ``*step``; a step past either table writes
    nothing and sets the device status (``ldb_device_status``)."""
    voxels, channels, _ = _rows(x)
    steps = 2 ** 31 - 1  # rows of the step tables (the smaller of the two)
    if coeff is not None:
        steps = min(steps, int(coeff.numel() // 5))
    if noise is not None and noise_step_stride > 0:
        steps = min(steps, int(noise.numel() // noise_step_stride))
    batch = int(x.shape[0])
    eps_ld = 0
    if eps is not None:
        _, _, eps_ld = _rows(eps)
    image_c = 0
    if image is not None:
        _, image_c, _ = _rows(image)
    in_ld = 0
    if net_in is not None:
        _, _, in_ld = _rows(net_in)
    with instrument.maybe_time("sampler_step", 0.0):
        _lib.call(
            "ldb_sampler_step_ex", _stream(x), kind, x.data_ptr(), _ptr(prev), _ptr(eps),
            _DT[eps.dtype] if eps is not None else _lib.LDB_F16, eps_ld, _ptr(noise), int(noise_step_stride),
            _ptr(mask), _ptr(image), image_c, _ptr(net_in), in_ld, int(net_split), batch, voxels, channels,
            _ptr(coeff), _ptr(step), steps,
        )


def vq_nearest4(z: torch.Tensor, codebook: torch.Tensor, *, quantized: torch.Tensor | None = None) -> torch.Tensor:
    """Nearest-code indices (int32) of 4-channel rows of ``z``; optionally writes ``z + (e - z)``."""
    positions_per, c, z_ld = _rows(z)
    if c != 4 or codebook.shape[-1] != 4 or codebook.dtype != z.dtype:
        raise ValueError("vq_nearest4 needs 4-channel z and a (E, 4) codebook of the same dtype")
    positions = positions_per * int(z.shape[0])
    indices = torch.empty(tuple(int(s) for s in z.shape[:-1]), dtype=torch.int32, device=z.device)
    out_ld = 4
    if quantized is not None:
        _, _, out_ld = _rows(quantized)
    _lib.call(
        "ldb_vq_nearest4", _stream(z), z.data_ptr(), z_ld, positions, codebook.contiguous().data_ptr(),
        int(codebook.shape[0]), _DT[z.dtype], indices.data_ptr(), _ptr(quantized), out_ld,
    )
    return indices


def resize_nearest(x: torch.Tensor, shape: tuple[int, int, int]) -> torch.Tensor:
    """Nearest resize of an NDHWC volume to spatial ``shape`` (floor(i * in / out) per axis)."""
    if x.ndim != 5:
        raise ValueError("resize_nearest expects (B, D, H, W, C)")
    _, c, ld = _rows(x)
    esz = x.element_size()
    if (c * esz) % 8:
        raise ValueError("rows must be a multiple of 8 bytes")
    out = torch.empty((x.shape[0], *shape, c), dtype=x.dtype, device=x.device)
    _lib.call(
        "ldb_resize_nearest", _stream(x), x.data_ptr(), int(x.shape[0]), int(x.shape[1]), int(x.shape[2]),
        int(x.shape[3]), c * esz, ld * esz, out.data_ptr(), shape[0], shape[1], shape[2], c * esz,
    )
    return out


def hu_map(x: torch.Tensor) -> torch.Tensor:
    """Inverse CT map to HU of channel 0 of a channels-last volume (f32 result without the channel axis)."""
    voxels, _, ld = _rows(x)
    n = voxels * int(x.shape[0])
    out = torch.empty(tuple(int(s) for s in x.shape[:-1]), dtype=torch.float32, device=x.device)
    _lib.call("ldb_hu_map", _stream(x), x.data_ptr(), _DT[x.dtype], ld, n, out.data_ptr())
    return out


def ct_normalize(hu: torch.Tensor, *, out_dtype: torch.dtype = torch.float16, pad_to: int = 8) -> torch.Tensor:
    """HU volume ``(B, D, H, W)`` (f32, contiguous) -> normalized NDHWC ``(B, D, H, W, 1)``
    in ``out_dtype`` whose channel stride is ``pad_to`` (a conv input), padding zero."""
    if hu.device.type != "cuda" or hu.dtype != torch.float32 or not hu.is_contiguous():
        raise ValueError("ct_normalize expects a contiguous float32 CUDA HU tensor")
    buf = torch.zeros((*hu.shape, pad_to), dtype=out_dtype, device=hu.device)
    _lib.call("ldb_ct_normalize", _stream(hu), hu.data_ptr(), hu.numel(), buf.data_ptr(), _DT[out_dtype], pad_to)
    return buf[..., :1]


def step_advance(step: torch.Tensor) -> None:
    """Increment the device step counter (int32 scalar tensor)."""
    _lib.call("ldb_step_advance", _stream(step), step.data_ptr())
