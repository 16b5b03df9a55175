"""tcgen05 implicit-GEMM convolution vs float64 references (GPU).

Bounds follow the reference's error model (tests/test_native_kernels.py:1-10
and :37-39 of lesiondiffusion-mlx): each f16 rounding of the output adds at
most half an f16 spacing, FP32 accumulation adds a small multiple of 2^-23
times the sum of absolute products, folded f16 upsampling weights add 2^-11
times that sum, and the FP32 exact mode adds a multiple of 2^-22.  The
single-op tolerance of the build (relative L2 <= 1e-2 for f16, <= 1e-4 for
FP32) is checked as well.
"""

from __future__ import annotations

import numpy as np
import pytest
import torch
import torch.nn.functional as F

pytestmark = pytest.mark.gpu

ACCUMULATION_EPS = 8 * 2.0**-23
OPERAND_ROUNDING = 2.0**-11
SPLIT_ERROR = 4 * 2.0**-22


def half_spacing(values: np.ndarray) -> np.ndarray:
    return np.spacing(np.abs(values).astype(np.float16)).astype(np.float64) / 2


def to_ndhwc(x: torch.Tensor, ld: int | None = None) -> torch.Tensor:
    """NCDHW -> NDHWC with an optional padded channel stride (view of a wider buffer)."""
    b, c, d, h, w = x.shape
    ld = c if ld is None else ld
    buf = torch.zeros((b, d, h, w, ld), dtype=x.dtype, device=x.device)
    buf[..., :c] = x.permute(0, 2, 3, 4, 1)
    return buf[..., :c]


def reference(x64: torch.Tensor, w64: torch.Tensor, bias64: torch.Tensor | None, stride: int, padding: int):
    out = F.conv3d(x64, w64, None, stride=stride, padding=padding)
    mag = F.conv3d(x64.abs(), w64.abs(), None, stride=stride, padding=padding)
    if bias64 is not None:
        out = out + bias64[:, None, None, None]
        mag = mag + bias64.abs()[:, None, None, None]
    return out.numpy(), mag.numpy()


def rel_l2(actual: np.ndarray, expected: np.ndarray) -> float:
    return float(np.linalg.norm(actual - expected) / max(np.linalg.norm(expected), 1e-30))


def f16_case(shape, out_channels, kernel, seed):
    rng = np.random.default_rng(seed)
    channels = shape[1]
    x = rng.normal(size=shape).astype(np.float16)
    w = (rng.normal(size=(out_channels, channels, kernel, kernel, kernel)) * (channels * kernel**3) ** -0.5).astype(np.float16)
    b = (rng.normal(size=(out_channels,)) * 0.1).astype(np.float16)
    return torch.from_numpy(x), torch.from_numpy(w), torch.from_numpy(b)


@pytest.mark.parametrize(
    ("shape", "out_channels", "stride"),
    [
        ((1, 16, 5, 7, 9), 32, 1),  # odd extents, partial bricks
        ((2, 32, 4, 6, 3), 128, 1),  # batched
        ((1, 48, 9, 3, 5), 64, 1),  # three 16-channel K blocks per tap
        ((1, 5, 6, 4, 7), 4, 1),  # zero-padded input and output channels
        ((2, 24, 7, 6, 9), 40, 2),  # stride 2, odd and even extents
        ((1, 512, 4, 4, 4), 128, 1),  # few tiles, large C: split-K
        ((1, 128, 8, 10, 10), 256, 1),  # 256-column tiles
        ((1, 64, 3, 4, 5), 16, 2),  # stride 2, 16-column tiles
    ],
)
def test_conv_f16_accumulates_in_fp32_and_rounds_once(cuda_device, shape, out_channels, stride):
    from lesiondiffusion_mlx_b200.conv import conv3d_ndhwc, pack_weight

    x, w, b = f16_case(shape, out_channels, 3, seed=sum(shape))
    ld = (shape[1] + 7) // 8 * 8
    xd = to_ndhwc(x.to(cuda_device), ld)
    packed = pack_weight(w.to(cuda_device), stride=stride)
    out = conv3d_ndhwc(xd, packed, b.to(cuda_device).float(), stride=stride)
    torch.cuda.synchronize()
    actual = out.permute(0, 4, 1, 2, 3).double().cpu().numpy()
    expected, mag = reference(x.double(), w.double(), b.double(), stride, 1)
    assert actual.shape == expected.shape
    error = np.abs(actual - expected)
    bound = half_spacing(expected) + ACCUMULATION_EPS * mag
    assert np.all(error <= bound), f"max excess {(error - bound).max()}"
    assert rel_l2(actual, expected) <= 1e-2


@pytest.mark.parametrize("split", [False, True])
@pytest.mark.parametrize("output_scale", [1.0, 0.25])
def test_conv_adds_shift_and_residual_before_rounding(cuda_device, split, output_scale):
    from lesiondiffusion_mlx_b200.conv import conv3d_ndhwc, pack_weight

    channels = 512 if split else 32
    x, w, _ = f16_case((2, channels, 4, 4, 4), 64, 3, seed=channels)
    rng = np.random.default_rng(1)
    shift = torch.from_numpy(rng.normal(size=(2, 64)).astype(np.float32))
    residual = torch.from_numpy(rng.normal(size=(2, 64, 4, 4, 4)).astype(np.float16))
    out = conv3d_ndhwc(
        to_ndhwc(x.to(cuda_device)), pack_weight(w.to(cuda_device)), None, shift=shift.to(cuda_device),
        residual=to_ndhwc(residual.to(cuda_device)).contiguous(), output_scale=output_scale,
    )
    torch.cuda.synchronize()
    actual = out.permute(0, 4, 1, 2, 3).double().cpu().numpy()
    products, mag = reference(x.double(), w.double(), None, 1, 1)
    expected = (products + shift.double().numpy()[:, :, None, None, None]) * output_scale + residual.double().numpy()
    error = np.abs(actual - expected)
    assert np.all(error <= half_spacing(expected) + ACCUMULATION_EPS * mag * output_scale)


def test_upsample_conv_matches_conv_of_nearest_upsampling(cuda_device):
    from lesiondiffusion_mlx_b200.conv import conv3d_ndhwc, pack_upsample_weight

    x, w, b = f16_case((2, 32, 3, 5, 4), 64, 3, seed=21)
    out = conv3d_ndhwc(to_ndhwc(x.to(cuda_device)), pack_upsample_weight(w.to(cuda_device)), b.to(cuda_device).float())
    torch.cuda.synchronize()
    actual = out.permute(0, 4, 1, 2, 3).double().cpu().numpy()
    up = x.double().repeat_interleave(2, 2).repeat_interleave(2, 3).repeat_interleave(2, 4)
    expected, mag = reference(up, w.double(), b.double(), 1, 1)
    assert actual.shape == expected.shape
    error = np.abs(actual - expected)
    assert np.all(error <= half_spacing(expected) + (ACCUMULATION_EPS + OPERAND_ROUNDING) * mag)


@pytest.mark.parametrize(
    ("shape", "out_channels", "kind"),
    [
        ((1, 256, 5, 7, 6), 256, "up"),  # folded upsampling: a pair holds two bricks of one output parity
        ((1, 256, 8, 10, 10), 512, "conv"),  # two 256-column tiles, split over K
        ((2, 256, 6, 9, 5), 256, "s2"),  # stride 2, batch 2
        ((1, 128, 3, 9, 14), 256, "conv"),  # three bricks: the second pair's second brick is a placeholder
    ],
)
def test_paired_cta_tiles(cuda_device, shape, out_channels, kind):
    """256-column f16 3x3x3 convs run as CTA pairs (one M = 256 product of two
    bricks per K step, each CTA staging half of the weight rows): outputs with
    per-batch shift and residual within the analytic bound, and the GroupNorm
    statistics the epilogue adds equal to the sums of the stored output."""
    from lesiondiffusion_mlx_b200.conv import conv3d_ndhwc, pack_upsample_weight, pack_weight

    x, w, b = f16_case(shape, out_channels, 3, seed=sum(shape) + out_channels)
    batch = shape[0]
    stride = 2 if kind == "s2" else 1
    if kind == "up":
        out_grid = tuple(2 * n for n in shape[2:])
        packed = pack_upsample_weight(w.to(cuda_device))
    else:
        out_grid = tuple((n - 1) // stride + 1 for n in shape[2:])
        packed = pack_weight(w.to(cuda_device), stride=stride)
    rng = np.random.default_rng(7)
    shift = torch.from_numpy(rng.normal(size=(batch, out_channels)).astype(np.float32) * 0.1)
    residual = torch.from_numpy(rng.normal(size=(batch, out_channels, *out_grid)).astype(np.float16))
    stats = torch.zeros((batch, out_channels, 2), dtype=torch.float64, device=cuda_device)
    out = conv3d_ndhwc(to_ndhwc(x.to(cuda_device)), packed, b.to(cuda_device).float(), stride=stride,
                       shift=shift.to(cuda_device), residual=to_ndhwc(residual.to(cuda_device)).contiguous(),
                       stats=stats)
    torch.cuda.synchronize()
    actual = out.permute(0, 4, 1, 2, 3).double().cpu().numpy()
    xin = x.double()
    rounding = ACCUMULATION_EPS
    if kind == "up":
        xin = xin.repeat_interleave(2, 2).repeat_interleave(2, 3).repeat_interleave(2, 4)
        rounding += OPERAND_ROUNDING
    products, mag = reference(xin, w.double(), b.double(), stride, 1)
    expected = products + shift.double().numpy()[:, :, None, None, None] + residual.double().numpy()
    assert actual.shape == expected.shape
    error = np.abs(actual - expected)
    bound = half_spacing(expected) + rounding * mag
    assert np.all(error <= bound), f"max excess {(error - bound).max()}"
    sums = actual.reshape(batch, out_channels, -1)
    want = np.stack([sums.sum(-1), (sums * sums).sum(-1)], axis=-1)
    np.testing.assert_allclose(stats.cpu().numpy(), want, rtol=1e-5, atol=1e-3)


@pytest.mark.parametrize("shape,out_channels", [((2, 48, 3, 5, 7), 40), ((1, 256, 2, 4, 100), 512)])
def test_pointwise_conv_and_gelu(cuda_device, shape, out_channels):
    from lesiondiffusion_mlx_b200 import _lib
    from lesiondiffusion_mlx_b200.conv import conv3d_ndhwc, pack_weight

    x, w, b = f16_case(shape, out_channels, 1, seed=11)
    xd = to_ndhwc(x.to(cuda_device))
    packed = pack_weight(w.to(cuda_device))
    out = conv3d_ndhwc(xd, packed, b.to(cuda_device).float())
    gelu = conv3d_ndhwc(xd, packed, b.to(cuda_device).float(), act=_lib.LDB_ACT_GELU)
    torch.cuda.synchronize()
    actual = out.permute(0, 4, 1, 2, 3).double().cpu().numpy()
    expected, mag = reference(x.double(), w.double(), b.double(), 1, 0)
    assert np.all(np.abs(actual - expected) <= half_spacing(expected) + ACCUMULATION_EPS * mag)
    rounded = torch.from_numpy(actual.astype(np.float16).astype(np.float64))
    gelu_expected = (rounded * 0.5 * (1 + torch.erf(rounded / np.sqrt(2)))).numpy()
    gelu_actual = gelu.permute(0, 4, 1, 2, 3).double().cpu().numpy()
    assert np.all(np.abs(gelu_actual - gelu_expected) <= 2 * half_spacing(gelu_expected) + 1e-6)


@pytest.mark.parametrize("shape,out_channels", [((2, 96, 3, 5, 7), 256), ((1, 64, 4, 9, 10), 128),
                                                ((2, 32, 1, 1, 200), 48)])
def test_pointwise_conv_over_flat_voxel_rows(cuda_device, shape, out_channels):
    """Pointwise convs are planned over each volume's voxels as one row (tiles
    of 128 consecutive voxels, the last one partial): per-batch shift,
    residual and the GroupNorm statistics of the stored output stay exact."""
    from lesiondiffusion_mlx_b200.conv import conv3d_ndhwc, pack_weight

    x, w, b = f16_case(shape, out_channels, 1, seed=sum(shape) + 3 * out_channels)
    batch = shape[0]
    rng = np.random.default_rng(17)
    shift = torch.from_numpy(rng.normal(size=(batch, out_channels)).astype(np.float32) * 0.1)
    residual = torch.from_numpy(rng.normal(size=(batch, out_channels, *shape[2:])).astype(np.float16))
    stats = torch.zeros((batch, out_channels, 2), dtype=torch.float64, device=cuda_device)
    out = conv3d_ndhwc(to_ndhwc(x.to(cuda_device)), pack_weight(w.to(cuda_device)), b.to(cuda_device).float(),
                       shift=shift.to(cuda_device), residual=to_ndhwc(residual.to(cuda_device)).contiguous(),
                       stats=stats)
    torch.cuda.synchronize()
    actual = out.permute(0, 4, 1, 2, 3).double().cpu().numpy()
    products, mag = reference(x.double(), w.double(), b.double(), 1, 0)
    expected = products + shift.double().numpy()[:, :, None, None, None] + residual.double().numpy()
    error = np.abs(actual - expected)
    assert np.all(error <= half_spacing(expected) + ACCUMULATION_EPS * mag), f"max excess {error.max()}"
    sums = actual.reshape(batch, out_channels, -1)
    want = np.stack([sums.sum(-1), (sums * sums).sum(-1)], axis=-1)
    np.testing.assert_allclose(stats.cpu().numpy(), want, rtol=1e-5, atol=1e-3)


@pytest.mark.parametrize(
    ("shape", "out_channels", "kind", "extra"),
    [
        ((1, 32, 24, 24, 40), 128, "conv", False),  # whole 8 x 8 planes
        ((1, 64, 45, 21, 27), 128, "conv", True),  # ragged planes and depth; shift + residual + scale
        ((1, 96, 41, 24, 24), 64, "conv", True),  # 64 output channels (weight rows past 64 read as zero)
        ((1, 32, 12, 16, 16), 128, "up", False),  # folded upsampling, 8 output parities
        ((1, 256, 30, 24, 40), 128, "pw", False),  # pointwise: planned voxel-major (the path it runs on)
    ],
)
def test_channel_major_tile(cuda_device, shape, out_channels, kind, extra):
    """Convs with 64 / 128 output channels on grids that need no split-K run as
    channel-major tiles (out^T = W x^T, transposed epilogue)."""
    from lesiondiffusion_mlx_b200.conv import conv3d_ndhwc, pack_upsample_weight, pack_weight

    k = 1 if kind == "pw" else 3
    x, w, b = f16_case(shape, out_channels, k, seed=sum(shape) + out_channels)
    wd = w.to(cuda_device)
    packed = pack_upsample_weight(wd) if kind == "up" else pack_weight(wd)
    xd = to_ndhwc(x.to(cuda_device))
    batch = shape[0]
    if kind == "up":
        up = x.double().repeat_interleave(2, 2).repeat_interleave(2, 3).repeat_interleave(2, 4)
        expected, mag = reference(up, w.double(), b.double(), 1, 1)
        tol_mag = ACCUMULATION_EPS + OPERAND_ROUNDING
    else:
        expected, mag = reference(x.double(), w.double(), b.double(), 1, 1 if k == 3 else 0)
        tol_mag = ACCUMULATION_EPS
    shift = residual = None
    scale = 1.0
    if extra:
        rng = np.random.default_rng(9)
        shift_np = rng.normal(size=(batch, out_channels)).astype(np.float32)
        res_np = rng.normal(size=expected.shape).astype(np.float16)
        shift = torch.from_numpy(shift_np).to(cuda_device)
        residual = to_ndhwc(torch.from_numpy(res_np).to(cuda_device)).contiguous()
        scale = 0.5
        expected = (expected + shift_np.astype(np.float64)[:, :, None, None, None]) * scale + res_np.astype(np.float64)
        mag = mag * scale
    out = conv3d_ndhwc(xd, packed, b.to(cuda_device).float(), shift=shift, residual=residual, output_scale=scale)
    torch.cuda.synchronize()
    actual = out.permute(0, 4, 1, 2, 3).double().cpu().numpy()
    assert actual.shape == expected.shape
    error = np.abs(actual - expected)
    bound = half_spacing(expected) + tol_mag * mag
    assert np.all(error <= bound), f"max excess {(error - bound).max()}"


def test_channel_major_tile_gelu(cuda_device):
    """GELU in the channel-major epilogue: the conv output rounded to f16,
    then the FP32 erf GELU, rounded once more (as the voxel-major tile)."""
    from lesiondiffusion_mlx_b200 import _lib
    from lesiondiffusion_mlx_b200.conv import conv3d_ndhwc, pack_weight

    x, w, b = f16_case((1, 64, 19, 21, 17), 128, 3, seed=77)
    xd = to_ndhwc(x.to(cuda_device))
    packed = pack_weight(w.to(cuda_device))
    plain = conv3d_ndhwc(xd, packed, b.to(cuda_device).float())
    gelu = conv3d_ndhwc(xd, packed, b.to(cuda_device).float(), act=_lib.LDB_ACT_GELU)
    torch.cuda.synchronize()
    rounded = plain.permute(0, 4, 1, 2, 3).double().cpu()
    expected = (rounded * 0.5 * (1 + torch.erf(rounded / np.sqrt(2)))).numpy()
    actual = gelu.permute(0, 4, 1, 2, 3).double().cpu().numpy()
    assert np.all(np.abs(actual - expected) <= 2 * half_spacing(expected) + 1e-6)


@pytest.mark.parametrize("shape,out_channels", [((1, 16, 8, 8, 8), 16), ((2, 32, 7, 9, 6), 48),
                                                ((1, 64, 24, 20, 30), 64)])
def test_stride2_conv_padded_after_only(cuda_device, shape, out_channels):
    """Stride 2 with zero padding (0, 1) per axis: the VQ encoder's downsample
    (mlx_model.py:735-736: pad after, then a stride-2 valid conv)."""
    from lesiondiffusion_mlx_b200.conv import conv3d_ndhwc, pack_weight

    x, w, b = f16_case(shape, out_channels, 3, seed=sum(shape) + 3)
    out = conv3d_ndhwc(to_ndhwc(x.to(cuda_device), (shape[1] + 7) // 8 * 8), pack_weight(w.to(cuda_device), stride=2),
                       b.to(cuda_device).float(), stride=2, pad01=True)
    torch.cuda.synchronize()
    actual = out.permute(0, 4, 1, 2, 3).double().cpu().numpy()
    xp = F.pad(x.double(), (0, 1, 0, 1, 0, 1))
    expected, mag = reference(xp, w.double(), b.double(), 2, 0)
    assert actual.shape == expected.shape
    error = np.abs(actual - expected)
    bound = half_spacing(expected) + ACCUMULATION_EPS * mag
    assert np.all(error <= bound), f"max excess {(error - bound).max()}"


def fp32_case(shape, out_channels, seed):
    rng = np.random.default_rng(seed)
    scales = np.exp(rng.normal(size=(1, shape[1], 1, 1, 1)) * 2)
    x = (rng.normal(size=shape) * scales).astype(np.float32)
    w = (rng.normal(size=(out_channels, shape[1], 3, 3, 3)) * (27 * shape[1]) ** -0.5).astype(np.float32)
    b = (rng.normal(size=(out_channels,)) * 0.1).astype(np.float32)
    return torch.from_numpy(x), torch.from_numpy(w), torch.from_numpy(b)


def split_input(x_ndhwc: torch.Tensor, cpad: int) -> torch.Tensor:
    """f32 NDHWC -> f16 [hi | 2^11-scaled lo] planes, each padded to cpad channels."""
    *lead, c = x_ndhwc.shape
    hi = x_ndhwc.to(torch.float16)
    lo = ((x_ndhwc - hi.float()) * 2048.0).to(torch.float16)
    out = torch.zeros((*lead, 2 * cpad), dtype=torch.float16, device=x_ndhwc.device)
    out[..., :c] = hi
    out[..., cpad : cpad + c] = lo
    return out


@pytest.mark.parametrize(
    ("shape", "out_channels", "stride"),
    [
        ((1, 4, 5, 7, 9), 16, 1),
        ((1, 16, 6, 5, 4), 1, 1),
        ((2, 24, 7, 6, 9), 40, 2),
        ((1, 64, 4, 6, 5), 128, 1),
        ((1, 512, 4, 4, 4), 64, 1),
    ],
)
def test_conv_fp32_exact_mode(cuda_device, shape, out_channels, stride):
    from lesiondiffusion_mlx_b200.conv import conv3d_ndhwc, pack_weight

    x, w, b = fp32_case(shape, out_channels, seed=sum(shape) + out_channels)
    cpad = (shape[1] + 15) // 16 * 16
    xs = split_input(to_ndhwc(x.to(cuda_device)).contiguous(), cpad)
    packed = pack_weight(w.to(cuda_device), stride=stride)
    assert packed.exact
    out = conv3d_ndhwc(xs, packed, b.to(cuda_device), stride=stride, in_channels=shape[1])
    torch.cuda.synchronize()
    actual = out.permute(0, 4, 1, 2, 3).double().cpu().numpy()
    expected, mag = reference(x.double(), w.double(), b.double(), stride, 1)
    bound = (ACCUMULATION_EPS + SPLIT_ERROR) * mag + 2.0**-23 * np.abs(expected)
    assert np.all(np.abs(actual - expected) <= bound), f"max excess {(np.abs(actual - expected) - bound).max()}"
    assert rel_l2(actual, expected) <= 1e-4


@pytest.mark.parametrize("shape,cout", [((1, 128, 8, 10, 12), 128), ((1, 512, 4, 5, 6), 512)])
def test_device_clock_records_each_launch(cuda_device, shape, cout):
    """The device-clock timing of a conv launch (plain, and split-K with its
    reduce) and of an attention launch: end after start, within the event
    time of the launch, results unchanged."""
    from lesiondiffusion_mlx_b200 import instrument, ops
    from lesiondiffusion_mlx_b200.conv import conv3d_ndhwc, pack_weight

    g = torch.Generator(device=cuda_device).manual_seed(5)
    x = torch.randn((shape[0], *shape[2:], shape[1]), generator=g, device=cuda_device).half()
    w = (torch.randn((cout, shape[1], 3, 3, 3), generator=g, device=cuda_device) * 0.02).half()
    packed = pack_weight(w)
    q = torch.randn((1, 700, 128), generator=g, device=cuda_device).half()
    want = conv3d_ndhwc(x, packed)
    want_attn = ops.flash_attention(q, q, q, heads=2, scale=0.125)
    timer = instrument.KernelTimer(device_clock=True)
    timer.arm(x.device)
    s = torch.cuda.Event(enable_timing=True)
    e = torch.cuda.Event(enable_timing=True)
    s.record()
    with instrument.timing(timer):
        got = conv3d_ndhwc(x, packed)
        got_attn = ops.flash_attention(q, q, q, heads=2, scale=0.125)
    e.record()
    torch.cuda.synchronize()
    summary = timer.summary()
    assert torch.equal(got, want) and torch.equal(got_attn, want_attn)
    for kind in ("conv3d", "attention"):
        assert summary[kind]["launches"] == 1
        assert 0 < summary[kind]["ms"] <= s.elapsed_time(e)


def test_device_status_clean(cuda_device):
    from lesiondiffusion_mlx_b200 import _lib

    assert _lib.device_status(reset=True) == 0
