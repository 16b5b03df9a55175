"""GPU operators vs the CPU oracle and the reference's golden vectors.

Each test calls the C ABI through ``lesiondiffusion_mlx_b200.ops`` and
compares with ``oracle`` (a restatement of the reference arithmetic) on the
same seeded inputs; sampler and VQ tests also replay the reference's own
recordings (tests/golden/reference_fixtures.npz).
"""

from __future__ import annotations

from pathlib import Path

import numpy as np
import pytest
import torch

from oracle import ops as oracle_ops
from oracle import samplers as oracle_samplers

pytestmark = pytest.mark.gpu

GOLDEN = Path(__file__).parent / "golden" / "reference_fixtures.npz"


def golden(name: str) -> dict[str, np.ndarray]:
    with np.load(GOLDEN, allow_pickle=False) as archive:
        return {k.split("/", 1)[1]: archive[k] for k in archive.files if k.startswith(name + "/")}


def ndhwc(x: torch.Tensor) -> torch.Tensor:
    return x.permute(0, 2, 3, 4, 1).contiguous()


def ncdhw(x: torch.Tensor) -> torch.Tensor:
    return x.permute(0, 4, 1, 2, 3).contiguous()


def rel_l2(a, b) -> float:
    a = np.asarray(a, dtype=np.float64)
    b = np.asarray(b, dtype=np.float64)
    return float(np.linalg.norm(a - b) / max(np.linalg.norm(b), 1e-30))


@pytest.mark.parametrize("dtype", [torch.float16, torch.float32])
@pytest.mark.parametrize("shape,groups,split", [((2, 64, 3, 5, 7), 32, None), ((1, 768, 2, 4, 5), 32, 512),
                                                  ((1, 96, 4, 6, 8), 16, None)])
def test_group_norm_affine_and_prepare(cuda_device, dtype, shape, groups, split):
    from lesiondiffusion_mlx_b200 import ops

    rng = np.random.default_rng(sum(shape))
    x = torch.from_numpy((rng.normal(size=shape) * 3 + 1.5).astype(np.float32)).to(dtype)
    gamma = torch.from_numpy(rng.normal(size=shape[1]).astype(np.float32))
    beta = torch.from_numpy(rng.normal(size=shape[1]).astype(np.float32))
    expected = oracle_ops.group_norm_affine(x, gamma, beta, groups=groups, eps=1e-5)
    xd = ndhwc(x).to(cuda_device)
    if split:
        x1 = xd[..., :split].contiguous()
        x2 = xd[..., split:].contiguous()
        affine = ops.group_norm_affine(x1, gamma.to(cuda_device), beta.to(cuda_device), groups=groups, eps=1e-5, x2=x2)
        prepared = ops.prepare_input(x1, affine=affine, silu=True, x2=x2)
    else:
        affine = ops.group_norm_affine(xd, gamma.to(cuda_device), beta.to(cuda_device), groups=groups, eps=1e-5)
        prepared = ops.prepare_input(xd, affine=affine, silu=True)
    torch.cuda.synchronize()
    np.testing.assert_allclose(affine.cpu().numpy(), expected.numpy(), rtol=2e-5, atol=2e-5)
    want = oracle_ops.apply_affine(x, expected, silu=True).to(torch.float16).float()
    got = ncdhw(prepared.float().cpu())
    ulp = np.spacing(np.abs(want.numpy()).astype(np.float16)).astype(np.float32)
    assert np.all(np.abs(got.numpy() - want.numpy()) <= 2 * ulp + 1e-6)


def test_prepare_split_planes(cuda_device):
    from lesiondiffusion_mlx_b200 import ops

    rng = np.random.default_rng(5)
    x = torch.from_numpy(rng.normal(size=(1, 3, 4, 5, 24)).astype(np.float32) * 100)
    out = ops.prepare_input(x.to(cuda_device), split=True)
    torch.cuda.synchronize()
    o = out.cpu()
    assert o.shape[-1] == 64
    hi = o[..., :24].float()
    lo = o[..., 32:56].float()
    assert torch.all(o[..., 24:32] == 0) and torch.all(o[..., 56:] == 0)
    recon = hi.double() + lo.double() / 2048
    assert torch.allclose(recon, x.double(), rtol=2 ** -21, atol=0)


def test_layer_norm(cuda_device):
    from lesiondiffusion_mlx_b200 import ops

    rng = np.random.default_rng(7)
    x = torch.from_numpy(rng.normal(size=(2, 33, 512)).astype(np.float16))
    g = torch.from_numpy(rng.normal(size=512).astype(np.float32))
    b = torch.from_numpy(rng.normal(size=512).astype(np.float32))
    got = ops.layer_norm(x.to(cuda_device), g.to(cuda_device), b.to(cuda_device), 1e-5).cpu().float()
    want = oracle_ops.layer_norm(x, g, b, 1e-5).float()
    ulp = np.spacing(np.abs(want.numpy()).astype(np.float16)).astype(np.float32)
    assert np.all(np.abs(got.numpy() - want.numpy()) <= ulp + 1e-6)


@pytest.mark.parametrize(
    "batch,lq,lk,heads,qscale,d",
    [
        (1, 96, 96, 2, 2.0, 16),
        (1, 96, 96, 2, 2.0, 32),
        (2, 520, 300, 2, 2.0, 64),
        (2, 300, 200, 2, 2.0, 32),  # partial query and key tiles
        (1, 640, 77, 2, 2.0, 32),  # cross-attention, one partial key block
        (1, 2048, 2048, 4, 6.0, 32),  # peaked softmax: the running maximum moves
        (1, 23104, 23104, 2, 1.0, 32),  # LMNet's 16 x 38 x 38 level, 2 heads of 32 (stream-K)
        (1, 4000, 1000, 16, 2.0, 32),  # stream-K with up to 3 segments per CTA, partial tiles
    ],
)
def test_flash_attention_f32(cuda_device, batch, lq, lk, heads, qscale, d):
    """FP32 attention (split-f16 tensor-core products) against float64 softmax
    attention at the FP32 tolerance (rel-L2 <= 1e-4; measured ~1e-6)."""
    from lesiondiffusion_mlx_b200 import ops

    rng = np.random.default_rng(lq + 3 * lk)
    q = (rng.normal(size=(batch, lq, heads * d)) * qscale).astype(np.float32)
    k = rng.normal(size=(batch, lk, heads * d)).astype(np.float32)
    v = rng.normal(size=(batch, lk, heads * d)).astype(np.float32)
    scale = d ** -0.5
    got = ops.flash_attention(*(torch.from_numpy(a).to(cuda_device) for a in (q, k, v)), heads=heads, scale=scale)
    torch.cuda.synchronize()
    assert got.dtype == torch.float32
    got = got.cpu().numpy()
    rows = np.arange(lq)
    if lq > 1024:
        rows = np.unique(np.concatenate([np.arange(200), np.arange(lq - 150, lq), np.arange(0, lq, 211)]))
    exact = oracle_ops.attention(torch.from_numpy(q[:, rows]).double(), torch.from_numpy(k).double(),
                                 torch.from_numpy(v).double(), heads=heads, scale=scale).numpy()
    assert np.all(np.isfinite(got))
    err = rel_l2(got[:, rows], exact)
    assert err <= 1e-4, err
    np.testing.assert_allclose(got[:, rows], exact, rtol=1e-4, atol=1e-5)


@pytest.mark.parametrize(
    "batch,lq,lk,heads,d,dtype,ties",
    [
        (1, 96, 96, 2, 32, torch.float16, False),
        (2, 32, 32, 1, 32, torch.float16, False),
        (1, 1056, 1056, 2, 32, torch.float16, False),  # partial final query tile
        (1, 512, 512, 4, 32, torch.float16, True),  # equal logits across key tiles
        (1, 640, 640, 8, 64, torch.float16, False),
        (1, 640, 77, 8, 64, torch.float16, False),  # cross-attention, one partial key block
        (2, 300, 200, 4, 64, torch.bfloat16, False),
        (1, 6400, 6400, 8, 64, torch.bfloat16, False),  # config-2 self-attention
        (1, 6400, 77, 8, 64, torch.bfloat16, False),  # config-2 cross-attention: 200 units, persistent grid
        (3, 2000, 100, 12, 64, torch.float16, False),  # short keys, persistent grid across batches and heads
        (1, 6400, 6400, 4, 64, torch.float16, False),  # stream-K: 100 pairs on all SMs, 2 segments per CTA
        (1, 4000, 1000, 16, 64, torch.float16, False),  # stream-K, up to 3 segments per CTA, partial tiles
    ],
)
def test_flash_attention(cuda_device, batch, lq, lk, heads, d, dtype, ties):
    from lesiondiffusion_mlx_b200 import ops

    rng = np.random.default_rng(lq + lk + d)
    q = rng.normal(size=(batch, lq, heads * d)) * 2.0
    k = rng.normal(size=(batch, lk, heads * d)) * 2.0
    v = rng.normal(size=(batch, lk, heads * d))
    if ties:
        q = np.zeros_like(q)
    qt, kt, vt = (torch.from_numpy(a.astype(np.float32)).to(dtype) for a in (q, k, v))
    scale = d ** -0.5
    got = ops.flash_attention(qt.to(cuda_device), kt.to(cuda_device), vt.to(cuda_device), heads=heads, scale=scale)
    torch.cuda.synchronize()
    got = got.float().cpu().numpy()
    # Query rows are independent: long sequences are checked on a subset of
    # rows (first and last tiles plus a stride) so the oracle stays fast.
    rows = np.arange(lq)
    if lq > 1024:
        rows = np.unique(np.concatenate([np.arange(256), np.arange(lq - 200, lq), np.arange(0, lq, 97)]))
    got = got[:, rows]
    qs = qt[:, torch.from_numpy(rows)]
    # flash-contract reference (probabilities rounded to the input type) and exact softmax, both float64
    want = oracle_ops.attention(qs, kt, vt, heads=heads, scale=scale).float().numpy()
    exact = oracle_ops.attention(qs.double(), kt.double(), vt.double(), heads=heads, scale=scale).numpy()
    assert np.all(np.isfinite(got))
    if dtype == torch.float16:
        np.testing.assert_allclose(got, exact, rtol=2e-3, atol=2e-3)
    assert rel_l2(got, exact) <= 1e-2
    assert rel_l2(got, want) <= 1e-2


def test_timestep_embedding_and_dense_small(cuda_device):
    from lesiondiffusion_mlx_b200 import ops

    t = torch.tensor([0, 17, 999], dtype=torch.int32)
    got = ops.timestep_embedding(t.to(cuda_device), 128).cpu()
    want = oracle_ops.timestep_embedding(t, 128)
    # cos/sin of phases up to ~1000 rad: a few FP32 ulps of the phase
    np.testing.assert_allclose(got.numpy(), want.numpy(), atol=3e-5, rtol=0)
    rng = np.random.default_rng(3)
    x = torch.from_numpy(rng.normal(size=(3, 128)).astype(np.float16))
    w = torch.from_numpy((rng.normal(size=(512, 128)) / 11).astype(np.float16))
    b = torch.from_numpy(rng.normal(size=512).astype(np.float16)).float()
    y = ops.dense_small(x.to(cuda_device), w.to(cuda_device), b.to(cuda_device), in_silu=True).cpu().float()
    ref = oracle_ops.dense(oracle_ops.silu(x), w, b.to(torch.float16), dtype=torch.float16).float()
    ulp = np.spacing(np.abs(ref.numpy()).astype(np.float16)).astype(np.float32)
    assert np.all(np.abs(y.numpy() - ref.numpy()) <= ulp + 1e-3)


def _ddim_on_gpu(device, f, toy, eps_dtype=torch.float16):
    """Replay a reference DDIM recording with the fused GPU sampler step."""
    from lesiondiffusion_mlx_b200 import ops

    coeffs = oracle_samplers.ddim_coefficients(f["alphas"], int(f["steps"]))
    n = len(coeffs["timesteps"])
    table = np.stack([coeffs["alphas"], coeffs["previous"], coeffs["sigmas"], coeffs["sqrt_one_minus"],
                      np.zeros(n, np.float32)], axis=1)[::-1].copy()  # in execution order
    mask = f.get("mask")
    image = f["image"]
    x = torch.from_numpy(f["initial"]).to(device)
    x = ndhwc(x)
    img = ndhwc(torch.from_numpy(image)).to(device)
    noise = torch.stack([ndhwc(torch.from_numpy(a)) for a in f["noise"]]).to(device).contiguous()
    coeff = torch.from_numpy(table).to(device)
    step = torch.zeros((), dtype=torch.int32, device=device)
    channels = x.shape[-1]
    extra = 1 if mask is not None else image.shape[1]
    net_in = torch.zeros((*x.shape[:-1], (channels + extra + 7) // 8 * 8), dtype=torch.float16, device=device)
    m = None if mask is None else torch.from_numpy(mask[:, 0]).to(device).contiguous()
    ops.sampler_step(0, x, mask=m, image=img, net_in=net_in[..., : channels + extra])
    for i in range(n):
        t = int(coeffs["timesteps"][n - 1 - i])
        # network input as the reference builds it (f32 concat), then the toy denoiser
        net32 = torch.cat([x, m[..., None] if m is not None else img], dim=-1)
        eps = toy(ncdhw(net32).cpu().numpy(), np.array([t], np.int32), f["condition"])
        eps_d = ndhwc(torch.from_numpy(np.asarray(eps, np.float32))).to(eps_dtype).to(device)
        ops.sampler_step(1, x, eps=eps_d, noise=noise, noise_step_stride=int(noise[0].numel()), mask=m,
                         image=img, net_in=net_in[..., : channels + extra], coeff=coeff, step=step)
        ops.step_advance(step)
    torch.cuda.synchronize()
    return ncdhw(x).cpu().numpy()


@pytest.mark.parametrize("name", ["ddim_mask", "ddim_inpainting"])
def test_fused_ddim_step_replays_reference_trajectory(cuda_device, name):
    from tests.golden.fixture_weights import sampling_toy_denoiser

    f = golden(name)
    got = _ddim_on_gpu(cuda_device, f, sampling_toy_denoiser)
    # the GPU step takes the prediction in f16 (the LINet output dtype); the
    # toy denoiser's FP32 prediction rounds to f16 on the way in, so the
    # trajectory matches the recording to f16 input precision.
    np.testing.assert_allclose(got, f["output"], rtol=2e-3, atol=2e-3)


def test_fused_ddim_step_fp32_prediction_replays_lmnet_trajectory(cuda_device):
    """LMNet's sampler (no mask, [x | conditioning] input) with the FP32
    network's f32 prediction: the recording at the reference's FP32
    tolerance, and the next network input written in the split format."""
    from lesiondiffusion_mlx_b200 import ops
    from tests.golden.fixture_weights import sampling_toy_denoiser

    f = golden("ddim_mask")
    assert f.get("mask") is None
    got = _ddim_on_gpu(cuda_device, f, sampling_toy_denoiser, eps_dtype=torch.float32)
    np.testing.assert_allclose(got, f["output"], rtol=2e-5, atol=2e-6)
    # split network input: hi + lo / 2048 reproduces [x | image] in FP32
    x = ndhwc(torch.from_numpy(f["output"])).to(cuda_device).contiguous()
    img = ndhwc(torch.from_numpy(f["image"])).to(cuda_device).contiguous()
    c = int(x.shape[-1]) + int(img.shape[-1])
    cpad = (c + 15) // 16 * 16
    net = torch.full((*x.shape[:-1], 2 * cpad), 7.0, dtype=torch.float16, device=cuda_device)
    ops.sampler_step(0, x, image=img, net_in=net, net_split=True)
    torch.cuda.synchronize()
    back = net[..., :cpad].float() + net[..., cpad:].float() / 2048.0
    want = torch.cat([x, img], dim=-1)
    assert torch.allclose(back[..., :c], want, rtol=1e-6, atol=1e-7)
    assert torch.all(net[..., c:cpad] == 0) and torch.all(net[..., cpad + c:] == 0)


@pytest.mark.parametrize("steps", [4, 8, 25])
def test_fused_dpm_step_replays_diffusers_trajectory(cuda_device, steps):
    from lesiondiffusion_mlx_b200 import ops

    f = golden("dpmpp_2m")
    d = {k.split(".", 1)[1]: v for k, v in f.items() if k.startswith(f"linet_{steps}.")}
    ts, coeffs = oracle_samplers.dpm_coefficients(d["alphas_cumprod"], steps)
    dev = cuda_device
    x = ndhwc(torch.from_numpy(d["initial_noise"])).to(dev)
    prev = x.clone()
    img = ndhwc(torch.from_numpy(d["conditioning_image"])).to(dev)
    m = torch.from_numpy(d["mask"][:, 0]).to(dev).contiguous()
    coeff = torch.from_numpy(coeffs).to(dev)
    step = torch.zeros((), dtype=torch.int32, device=dev)
    net_in = torch.zeros((*x.shape[:-1], 8), dtype=torch.float16, device=dev)
    ops.sampler_step(0, x, mask=m, image=img, net_in=net_in[..., :5])
    observed = []
    for i in range(steps):
        observed.append(ncdhw(x).cpu().numpy())
        eps = ndhwc(torch.from_numpy(d["predictions"][i])).to(dev)  # recorded f16 predictions
        ops.sampler_step(2, x, eps=eps, prev=prev, mask=m, image=img, net_in=net_in[..., :5], coeff=coeff, step=step)
        ops.step_advance(step)
    torch.cuda.synchronize()
    out = ncdhw(x).cpu().numpy()
    np.testing.assert_allclose(out, d["output"], rtol=2e-5, atol=2e-6)
    np.testing.assert_allclose(np.stack(observed), d["projected_inputs"], rtol=2e-5, atol=2e-6)
    outside = np.broadcast_to(d["mask"] == 0, out.shape)
    np.testing.assert_array_equal(out[outside], d["conditioning_image"][outside])


@pytest.mark.parametrize("dtype", [np.float32, np.float16])
@pytest.mark.parametrize("positions,entries", [(1, 2048), (2, 33), (3, 1), (31, 2), (32, 32), (33, 31), (5000, 2048)])
def test_vq_nearest4_exact(cuda_device, dtype, positions, entries):
    from lesiondiffusion_mlx_b200 import ops

    rng = np.random.default_rng(317)
    cb = rng.normal(size=(entries, 4)).astype(np.float32)
    if entries > 3:
        cb[-1] = cb[0]
        cb[3] = -cb[2]
    pts = np.concatenate([(cb[:-1] + cb[1:]) / 2, cb, np.zeros((1, 4))]).astype(np.float32)
    pts = np.tile(pts, (positions // len(pts) + 1, 1))[:positions]
    if positions > 100:
        pts = rng.normal(size=(positions, 4)).astype(np.float32)
    for z in (pts, np.array([[np.nan, 0, 0, 0], [300, 1, -2, 3]], np.float32)):
        zt = z.astype(dtype)
        cbt = cb.astype(dtype)
        want = oracle_ops.nearest_codebook4(zt, cbt)
        tz = torch.from_numpy(zt).to(cuda_device)[None]
        q = torch.empty_like(tz)
        idx = ops.vq_nearest4(tz, torch.from_numpy(cbt).to(cuda_device), quantized=q)
        torch.cuda.synchronize()
        np.testing.assert_array_equal(idx.cpu().numpy()[0], want)
        e = cbt[want]
        expect_q = (zt + (e - zt).astype(dtype)).astype(dtype)
        np.testing.assert_array_equal(q.cpu().numpy()[0], expect_q)


@pytest.mark.parametrize("dtype_name", ["float32", "float16"])
def test_vq_quantize_matches_reference_recording(cuda_device, dtype_name):
    from lesiondiffusion_mlx_b200 import ops
    from tests.golden.fixture_weights import vq_fixture_weights

    f = golden("vq_" + dtype_name)
    dtype = getattr(torch, dtype_name)
    cb = torch.from_numpy(vq_fixture_weights(int(f["weight_seed"]))["quantize.embedding.weight"]).to(dtype)
    z = ndhwc(torch.from_numpy(f["z"]).to(dtype)).to(cuda_device)
    q = torch.empty_like(z)
    ops.vq_nearest4(z, cb.to(cuda_device), quantized=q)
    torch.cuda.synchronize()
    np.testing.assert_array_equal(ncdhw(q.cpu()).numpy(), f["quantized"])


def test_resize_nearest_and_hu_map(cuda_device):
    from lesiondiffusion_mlx_b200 import ops

    rng = np.random.default_rng(9)
    x = torch.from_numpy(rng.normal(size=(1, 4, 5, 7, 3)).astype(np.float32))
    for shape in ((8, 10, 14), (3, 3, 5), (5, 7, 3)):
        got = ops.resize_nearest(ndhwc(x).to(cuda_device), shape).cpu()
        want = oracle_ops.resize_nearest(x, shape)
        np.testing.assert_array_equal(ncdhw(got).numpy(), want.numpy())
    f = golden("pipeline")
    norm = torch.from_numpy(f["normalized"]).reshape(1, -1, 1).to(cuda_device)
    hu = ops.hu_map(norm).cpu().numpy().reshape(-1)
    np.testing.assert_allclose(hu, f["inverse_output"], atol=4 * np.spacing(np.float32(1000)), rtol=0)
    vals = torch.from_numpy(rng.uniform(-0.3, 1.3, size=(1, 4096, 1)).astype(np.float32))
    got = ops.hu_map(vals.to(cuda_device)).cpu().numpy().reshape(-1)
    want = oracle_ops.piecewise_ct(vals.reshape(-1), inverse=True).numpy()
    np.testing.assert_allclose(got, want, atol=4 * np.spacing(np.float32(1000)), rtol=0)


def test_device_status_clean(cuda_device):
    from lesiondiffusion_mlx_b200 import _lib

    assert _lib.device_status(reset=True) == 0
