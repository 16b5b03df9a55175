"""Parity at the BASELINE configurations' own shapes (GPU).

Each benchmarked configuration is checked at the shape it is measured on, so
a defect that only large grids reach (tile or brick planning, split-K
choice, 32-bit index arithmetic) cannot pass the suite:

* config 1: the FP32-exact conv 1 x 32 x 40 x 40 x 128 -> 128 against a
  float64 conv, with the reference's analytic bound (tests/test_native_kernels.py
  of lesiondiffusion-mlx) and relative L2 <= 1e-4;
* config 3: the full benchmarked step -- the model-channels-128, two-block
  UNet on the 1 x 8 x 32 x 40 x 40 latent with the 77 x 768 context plus the
  fused DDIM update, replayed from the same CUDA graph ``bench.py`` times --
  against the oracle (relative L2 <= 1e-2 on the prediction);
* config 4a: the 512/256/128/64 decoder (GroupNorm 32, two nearest 2x
  upsamplings) on a depth crop of the 32 x 40 x 40 latent against the oracle
  (relative L2 <= 1e-2), and the full 128 x 160 x 160 decode against the same
  decode over depth slabs (a size-independent property);
* the north star's full-pipeline bound: injected initial and per-step noise
  -> 4 DDIM steps of the config-3 UNet -> the config-4 decoder -> HU, mean
  absolute error <= 1 HU against the oracle's composition of the same steps
  (lesiondiffusion-mlx: mlx_sampling.py:66-69 noise hooks, medmlx.py:1438-1455
  decode to HU).

Inputs are seeded synthetic data with the BASELINE shapes and distributions;
weights are random He-normal (no checkpoints are available).
"""

from __future__ import annotations

import os
from pathlib import Path

import numpy as np
import pytest
import torch
import torch.nn.functional as F

from oracle import ops as oops
from oracle import samplers as osamp
from oracle.networks import OracleUnet, OracleVq, UnetConfig as OracleConfig, torch_weights

pytestmark = pytest.mark.gpu

GOLDEN = Path(__file__).parent / "golden" / "reference_fixtures.npz"
ACCUMULATION_EPS = 8 * 2.0**-23
SPLIT_ERROR = 4 * 2.0**-22


def rel_l2(a, b) -> float:
    a = np.asarray(a, np.float64)
    b = np.asarray(b, np.float64)
    return float(np.linalg.norm(a - b) / max(np.linalg.norm(b), 1e-30))


def _threads() -> None:
    torch.set_num_threads(max(1, len(os.sched_getaffinity(0))))


def _linet_alphas() -> np.ndarray:
    with np.load(GOLDEN, allow_pickle=False) as archive:
        return archive["dpmpp_2m/linet_4.alphas_cumprod"]


def _oracle_unet(raw: dict, cfg) -> OracleUnet:
    return OracleUnet(torch_weights(raw, torch.float16),
                      OracleConfig(cfg.model_channels, cfg.num_res_blocks, cfg.attention_resolutions,
                                   cfg.channel_mult, cfg.num_head_channels, cfg.skip_context),
                      compute=torch.float32)


# ----------------------------------------------------------------- config 1


def test_config1_fp32_conv_at_its_shape(cuda_device):
    """Config 1: x ~ N(0, 1) (seed 0), w ~ N(0, 1/sqrt(27 * 128)) (seed 1),
    bias ~ N(0, 0.02) (seed 2), NDHWC FP32, through the split-f16 exact mode."""
    from lesiondiffusion_mlx_b200 import ops
    from lesiondiffusion_mlx_b200.conv import conv3d_ndhwc, pack_weight

    _threads()
    x = torch.randn((1, 32, 40, 40, 128), generator=torch.Generator().manual_seed(0))
    w = torch.randn((128, 128, 3, 3, 3), generator=torch.Generator().manual_seed(1)) / np.sqrt(27 * 128)
    b = torch.randn((128,), generator=torch.Generator().manual_seed(2)) * 0.02
    xs = ops.prepare_input(x.to(cuda_device), split=True)
    packed = pack_weight(w.to(cuda_device))
    assert packed.exact
    out = conv3d_ndhwc(xs, packed, b.to(cuda_device), in_channels=128)
    torch.cuda.synchronize()
    assert out.dtype == torch.float32 and tuple(out.shape) == (1, 32, 40, 40, 128)
    actual = out.permute(0, 4, 1, 2, 3).double().cpu().numpy()
    x64 = x.permute(0, 4, 1, 2, 3).double()
    w64 = w.double()
    expected = (F.conv3d(x64, w64, None, padding=1) + b.double()[:, None, None, None]).numpy()
    mag = (F.conv3d(x64.abs(), w64.abs(), None, padding=1) + b.double().abs()[:, None, None, None]).numpy()
    bound = (ACCUMULATION_EPS + SPLIT_ERROR) * mag + 2.0**-23 * np.abs(expected)
    assert np.all(np.abs(actual - expected) <= bound), f"max excess {(np.abs(actual - expected) - bound).max()}"
    assert rel_l2(actual, expected) <= 1e-4


# ----------------------------------------------------------------- config 3


def test_config3_benchmarked_step_matches_oracle(cuda_device):
    """The step ``bench.py`` times (same weights, inputs, schedule and graph)
    against the oracle's UNet forward and DDIM update."""
    from lesiondiffusion_mlx_b200 import workloads
    from lesiondiffusion_mlx_b200.networks import LdmUnetB200
    from lesiondiffusion_mlx_b200.sampling import DdimSampler, PreparedSampler

    _threads()
    cfg = workloads.CONFIG3
    raw = workloads.unet_weights(cfg, 8, 8, 768, seed=100)
    unet = LdmUnetB200({k: torch.from_numpy(v).to(torch.float16) for k, v in raw.items()}, cfg, device=cuda_device)
    inp = workloads.config3_inputs(seed=101)
    cache = unet.prepare_context(torch.from_numpy(inp["context"]).to(cuda_device))
    alphas = _linet_alphas()
    sampler = DdimSampler(alphas, 200)
    image = workloads.source_latent((1, 7, 32, 40, 40), seed=300)
    mask = inp["mask"]
    prepared = PreparedSampler(sampler, unet, cache, torch.from_numpy(image).permute(0, 2, 3, 4, 1).to(cuda_device),
                               torch.from_numpy(mask[:, 0]).to(cuda_device), graph=True)
    gen = np.random.default_rng(1000)
    init = gen.standard_normal((1, 7, 32, 40, 40)).astype(np.float32)
    noise = gen.standard_normal((200, 1, 7, 32, 40, 40), dtype=np.float32)
    to_dev = lambda a: torch.from_numpy(np.ascontiguousarray(np.moveaxis(a, -4, -1))).to(cuda_device)  # noqa: E731
    prepared.begin(to_dev(init), to_dev(noise))
    prepared.capture()
    prepared.step()
    torch.cuda.synchronize()
    eps_gpu = prepared.eps.permute(0, 4, 1, 2, 3).float().cpu().numpy()
    x_gpu = prepared.state.x.permute(0, 4, 1, 2, 3).cpu().numpy()

    coeffs = osamp.ddim_coefficients(alphas, 200)
    index = len(coeffs["timesteps"]) - 1  # the first step runs the largest timestep
    composed = (init * mask + (np.float32(1) - mask) * image).astype(np.float32)
    net_in = np.concatenate([composed, mask], axis=1)
    oracle = _oracle_unet(raw, cfg)
    projected, kv = oracle.project_context(torch.from_numpy(inp["context"]), torch.float16)
    t = torch.full((1,), int(coeffs["timesteps"][index]), dtype=torch.int32)
    eps_ref = oracle.forward(torch.from_numpy(net_in).to(torch.float16), t, projected, kv).float().numpy()
    assert eps_gpu.shape == eps_ref.shape == (1, 8, 32, 40, 40)
    assert np.all(np.isfinite(eps_gpu))
    assert rel_l2(eps_gpu, eps_ref) <= 1e-2
    x_ref = osamp.ddim_update(composed, eps_ref[:, :7], coeffs["alphas"][index], coeffs["previous"][index],
                              coeffs["sigmas"][index], coeffs["sqrt_one_minus"][index], noise[0])
    x_ref = (x_ref * mask + (np.float32(1) - mask) * image).astype(np.float32)
    # the update is FP32 arithmetic on the f16 prediction, so the state carries
    # the prediction's error (scaled by the update's eps coefficient)
    assert rel_l2(x_gpu, x_ref) <= 1e-2


# ----------------------------------------------------------------- config 4a


def _config4_decoder(device):
    from lesiondiffusion_mlx_b200 import workloads
    from lesiondiffusion_mlx_b200.networks import VqDecoderB200

    raw = workloads.config4_decoder_weights(seed=200)
    dec = VqDecoderB200({k: torch.from_numpy(v) for k, v in raw.items()}, device=device, groups=32)
    return dec, raw


def _ndhwc_f16(z: np.ndarray, device) -> torch.Tensor:
    return torch.from_numpy(np.ascontiguousarray(np.moveaxis(z, 1, -1))).to(device, torch.float16)


def test_config4a_decoder_depth_crop_matches_oracle(cuda_device):
    """Widths 512/256/128/64, GroupNorm 32, two 2x upsamplings: a 4-slice depth
    crop of the 32 x 40 x 40 latent -> 1 x 1 x 16 x 160 x 160 (every level at its
    full config-4a height and width)."""
    _threads()
    dec, raw = _config4_decoder(cuda_device)
    z = np.random.default_rng(201).standard_normal((1, 8, 4, 40, 40)).astype(np.float32)
    out = dec.decode(_ndhwc_f16(z, cuda_device), quantize=False)
    torch.cuda.synchronize()
    got = out.permute(0, 4, 1, 2, 3).float().cpu().numpy()
    assert got.shape == (1, 1, 16, 160, 160)
    oracle = OracleVq(torch_weights(raw, torch.float16), groups=32, compute=torch.float32)
    ref = oracle.decode(torch.from_numpy(z).to(torch.float16), quantize=False).float().numpy()
    assert np.all(np.isfinite(got))
    assert rel_l2(got, ref) <= 1e-2


def test_config4a_full_decode_equals_decode_over_depth_slabs(cuda_device):
    """The whole 32 x 40 x 40 -> 128 x 160 x 160 decode against the same decode
    run over four depth slabs (halo exchange, statistics summed over slabs)."""
    from lesiondiffusion_mlx_b200.sharded_decode import LocalDepthComm, ShardedVqDecoder, partition_depth

    dec, _ = _config4_decoder(cuda_device)
    z = np.random.default_rng(202).standard_normal((1, 8, 32, 40, 40)).astype(np.float32)
    zd = _ndhwc_f16(z, cuda_device)
    whole = dec.decode(zd, quantize=False)
    sharded = ShardedVqDecoder(dec, LocalDepthComm())
    slabs = sharded.decode([zd[:, a:b] for a, b in partition_depth(32, 4)], 32, quantize=False)
    torch.cuda.synchronize()
    assert tuple(whole.shape) == (1, 128, 160, 160, 1)
    joined = torch.cat(slabs, dim=1)
    assert torch.isfinite(whole).all()
    assert rel_l2(joined.float().cpu().numpy(), whole.float().cpu().numpy()) <= 2e-3


# ----------------------------------------------------------- full pipeline


def test_full_pipeline_decoded_volume_within_one_hu(cuda_device):
    """identical injected noise -> 4 DDIM steps of the
    config-3 UNet (latent crop 8 x 20 x 20, mask box, smoothed source latent,
    real LINet alphas) -> config-4 decoder on [7 denoised channels | mask] ->
    HU; mean absolute HU error <= 1 against the oracle's composition."""
    from lesiondiffusion_mlx_b200 import ops, workloads
    from lesiondiffusion_mlx_b200.networks import LdmUnetB200
    from lesiondiffusion_mlx_b200.sampling import DdimSampler, PreparedSampler

    _threads()
    d, h, w = 8, 20, 20
    cfg = workloads.CONFIG3
    raw = workloads.unet_weights(cfg, 8, 8, 768, seed=100)
    unet = LdmUnetB200({k: torch.from_numpy(v).to(torch.float16) for k, v in raw.items()}, cfg, device=cuda_device)
    dec, draw = _config4_decoder(cuda_device)
    context = workloads.config3_inputs(seed=101)["context"]
    mask = np.zeros((1, 1, d, h, w), np.float32)
    mask[:, :, 2:7, 6:14, 6:14] = 1
    image = workloads.source_latent((1, 7, d, h, w), seed=300)
    rng = np.random.default_rng(5)
    init = rng.standard_normal((1, 7, d, h, w)).astype(np.float32)
    noise = rng.standard_normal((4, 1, 7, d, h, w)).astype(np.float32)
    alphas = _linet_alphas()

    to_dev = lambda a: torch.from_numpy(np.ascontiguousarray(np.moveaxis(a, -4, -1))).to(cuda_device)  # noqa: E731
    cache = unet.prepare_context(torch.from_numpy(context).to(cuda_device))
    prepared = PreparedSampler(DdimSampler(alphas, 4), unet, cache, to_dev(image),
                               torch.from_numpy(mask[:, 0]).to(cuda_device), graph=True)
    x = prepared.run(to_dev(init), to_dev(noise))
    z = torch.zeros((1, d, h, w, 8), dtype=torch.float16, device=cuda_device)
    z[..., :7] = x
    z[..., 7] = torch.from_numpy(mask[0, 0]).to(cuda_device)
    hu = ops.hu_map(dec.decode(z, quantize=False))
    torch.cuda.synchronize()
    hu_gpu = hu.cpu().numpy()[0]

    oracle = _oracle_unet(raw, cfg)
    projected, kv = oracle.project_context(torch.from_numpy(context), torch.float16)

    def denoise(net_in, t, _condition):
        return oracle.forward(torch.from_numpy(net_in).to(torch.float16), torch.from_numpy(t), projected, kv).float()

    coeffs = osamp.ddim_coefficients(alphas, 4)
    x_ref = osamp.ddim_sample(denoise, None, image, coeffs, initial_noise=init, step_noise=noise, mask=mask)
    z_ref = np.concatenate([x_ref, mask], axis=1)
    dec_ref = OracleVq(torch_weights(draw, torch.float16), groups=32, compute=torch.float32)
    out_ref = dec_ref.decode(torch.from_numpy(z_ref).to(torch.float16), quantize=False)
    hu_ref = oops.piecewise_ct(out_ref, inverse=True).numpy()[0, 0]
    assert hu_gpu.shape == hu_ref.shape == (4 * d, 4 * h, 4 * w)
    assert np.all(np.isfinite(hu_gpu))
    mae = float(np.mean(np.abs(hu_gpu.astype(np.float64) - hu_ref)))
    assert mae <= 1.0, f"decoded-volume MAE {mae:.3f} HU"
