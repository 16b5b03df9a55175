"""B200 UNet and VQ decoder vs the reference recordings and the CPU oracle (GPU).

The reference's Torch-CPU recordings of the pinned upstream model are the
golden vectors (f16 tolerance 2e-3 absolute / relative, as in the
reference's tests/test_equivalence.py:62-73); larger BASELINE-shaped
networks are checked against the oracle at the build's f16 bound
(relative L2 <= 1e-2).
"""

from __future__ import annotations

import json
from pathlib import Path

import numpy as np
import pytest
import torch

from oracle.networks import OracleUnet, OracleVq, UnetConfig as OracleConfig, torch_weights
from tests.golden.fixture_weights import unet_fixture_weights, vq_fixture_weights

pytestmark = pytest.mark.gpu

GOLDEN = Path(__file__).parent / "golden" / "reference_fixtures.npz"


def golden(name: str) -> dict[str, np.ndarray]:
    with np.load(GOLDEN, allow_pickle=False) as archive:
        return {k.split("/", 1)[1]: archive[k] for k in archive.files if k.startswith(name + "/")}


def to_input(x: np.ndarray, device) -> torch.Tensor:
    """NCDHW float -> NDHWC f16 view with the channel stride padded to 8."""
    t = torch.from_numpy(x).permute(0, 2, 3, 4, 1)
    c = t.shape[-1]
    buf = torch.zeros((*t.shape[:-1], (c + 7) // 8 * 8), dtype=torch.float16)
    buf[..., :c] = t.to(torch.float16)
    return buf.to(device)[..., :c]


def rel_l2(a, b) -> float:
    a = np.asarray(a, np.float64)
    b = np.asarray(b, np.float64)
    return float(np.linalg.norm(a - b) / max(np.linalg.norm(b), 1e-30))


def test_unet_matches_reference_recording(cuda_device):
    from lesiondiffusion_mlx_b200.networks import LdmUnetB200, UnetConfig

    f = golden("unet_inpainting")
    cfg = json.loads(f["config"].item())
    config = UnetConfig(cfg["model_channels"], cfg["num_res_blocks"], tuple(cfg["attention_resolutions"]),
                        tuple(cfg["channel_mult"]), cfg["num_head_channels"], cfg["skip_context"])
    raw = unet_fixture_weights(int(f["weight_seed"]), skip_context=config.skip_context)
    model = LdmUnetB200(torch_weights(raw, torch.float16), config, device=cuda_device)
    x = to_input(f["x"], cuda_device)
    t = torch.from_numpy(f["timesteps"].astype(np.int32)).to(cuda_device)
    out = model(x, t, torch.from_numpy(f["context"]))
    torch.cuda.synchronize()
    got = out.permute(0, 4, 1, 2, 3).float().cpu().numpy()
    np.testing.assert_allclose(got, f["output"].astype(np.float32), rtol=2e-3, atol=2e-3)
    oracle = OracleUnet(torch_weights(raw, torch.float16), OracleConfig(**{k: getattr(config, k) for k in (
        "model_channels", "num_res_blocks", "attention_resolutions", "channel_mult", "num_head_channels",
        "skip_context")}))
    ref = oracle(torch.from_numpy(f["x"]), torch.from_numpy(f["timesteps"]), torch.from_numpy(f["context"]))
    assert rel_l2(got, ref.float().numpy()) <= 1e-2


def random_unet_weights(config, in_ch, out_ch, ctx_dim, seed):
    """He-normal random weights with the reference's state-dict names."""
    rng = np.random.default_rng(seed)
    w: dict[str, np.ndarray] = {}

    def conv(key, i, o, k=3):
        w[key + ".weight"] = (rng.normal(size=(o, i, k, k, k)) * np.sqrt(2.0 / (i * k ** 3))).astype(np.float32)
        w[key + ".bias"] = (rng.normal(size=o) * 0.02).astype(np.float32)

    def lin(key, i, o, bias=True):
        w[key + ".weight"] = (rng.normal(size=(o, i)) * np.sqrt(1.0 / i)).astype(np.float32)
        if bias:
            w[key + ".bias"] = (rng.normal(size=o) * 0.02).astype(np.float32)

    def norm(key, c):
        w[key + ".weight"] = (1 + 0.1 * rng.normal(size=c)).astype(np.float32)
        w[key + ".bias"] = (0.1 * rng.normal(size=c)).astype(np.float32)

    mc = config.model_channels
    emb = 4 * mc
    lin("time_embed.0", mc, emb)
    lin("time_embed.2", emb, emb)
    if not config.skip_context:
        lin("context_linear_projection", ctx_dim, ctx_dim, bias=False)

    def res(key, i, o):
        norm(key + ".in_layers.0", i)
        conv(key + ".in_layers.2", i, o)
        lin(key + ".emb_layers.1", emb, o)
        norm(key + ".out_layers.0", o)
        conv(key + ".out_layers.3", o, o)
        if i != o:
            conv(key + ".skip_connection", i, o, 1)

    def tr(key, c):
        norm(key + ".norm", c)
        conv(key + ".proj_in", c, c, 1)
        conv(key + ".proj_out", c, c, 1)
        b = key + ".transformer_blocks.0"
        for n in ("norm1", "norm2", "norm3"):
            norm(f"{b}.{n}", c)
        for a in ("attn1", "attn2"):
            cd = c if a == "attn1" or config.skip_context else ctx_dim
            lin(f"{b}.{a}.to_q", c, c, bias=False)
            lin(f"{b}.{a}.to_k", cd, c, bias=False)
            lin(f"{b}.{a}.to_v", cd, c, bias=False)
            lin(f"{b}.{a}.to_out.0", c, c)
        lin(b + ".ff.net.0.0", c, 2 * c)
        lin(b + ".ff.net.2", 2 * c, c)

    conv("input_blocks.0.0", in_ch, mc)
    chans = [mc]
    ch = mc
    block, res_ = 1, 1
    for level, mult in enumerate(config.channel_mult):
        for _ in range(config.num_res_blocks):
            res(f"input_blocks.{block}.0", ch, mult * mc)
            ch = mult * mc
            if res_ in config.attention_resolutions:
                tr(f"input_blocks.{block}.1", ch)
            chans.append(ch)
            block += 1
        if level < len(config.channel_mult) - 1:
            conv(f"input_blocks.{block}.0.op", ch, ch)
            chans.append(ch)
            block += 1
            res_ *= 2
    res("middle_block.0", ch, ch)
    tr("middle_block.1", ch)
    res("middle_block.2", ch, ch)
    block = 0
    for level in reversed(range(len(config.channel_mult))):
        mult = config.channel_mult[level]
        for i in range(config.num_res_blocks + 1):
            skip = chans.pop()
            res(f"output_blocks.{block}.0", ch + skip, mult * mc)
            ch = mult * mc
            has_attn = res_ in config.attention_resolutions
            if has_attn:
                tr(f"output_blocks.{block}.1", ch)
            if level and i == config.num_res_blocks:
                conv(f"output_blocks.{block}.{2 if has_attn else 1}.conv", ch, ch)
                res_ //= 2
            block += 1
    norm("out.0", ch)
    conv("out.2", ch, out_ch)
    return w


@pytest.mark.parametrize("skip_context", [False, True])
def test_unet_baseline_shape_matches_oracle(cuda_device, skip_context):
    from lesiondiffusion_mlx_b200.networks import LdmUnetB200, UnetConfig

    config = UnetConfig(64, 1, (2, 4), (1, 2, 4), 64, skip_context)
    raw = random_unet_weights(config, 8, 8, 96, seed=100)
    model = LdmUnetB200(torch_weights(raw, torch.float16), config, device=cuda_device)
    rng = np.random.default_rng(101)
    x = rng.normal(size=(2, 8, 8, 12, 12)).astype(np.float32)
    t = np.array([17, 640], np.int32)
    ctx = rng.normal(size=(2, 77, 96)).astype(np.float32)
    out = model(to_input(x, cuda_device), torch.from_numpy(t).to(cuda_device), torch.from_numpy(ctx))
    torch.cuda.synchronize()
    got = out.permute(0, 4, 1, 2, 3).float().cpu().numpy()
    ocfg = OracleConfig(64, 1, (2, 4), (1, 2, 4), 64, skip_context)
    oracle = OracleUnet(torch_weights(raw, torch.float16), ocfg, compute=torch.float32)
    ref = oracle(torch.from_numpy(x), torch.from_numpy(t), torch.from_numpy(ctx)).float().numpy()
    assert np.all(np.isfinite(got))
    assert rel_l2(got, ref) <= 1e-2


def test_fp32_unet_matches_reference_recording(cuda_device):
    """The FP32 network (LMNet's arithmetic: split-f16 convs, dense layers and
    attention) against the reference's FP32 Torch-CPU recording."""
    from lesiondiffusion_mlx_b200.networks import LdmUnetB200, UnetConfig

    f = golden("unet_mask")
    assert f["dtype"].item() == "float32"
    cfg = json.loads(f["config"].item())
    config = UnetConfig(cfg["model_channels"], cfg["num_res_blocks"], tuple(cfg["attention_resolutions"]),
                        tuple(cfg["channel_mult"]), cfg["num_head_channels"], cfg["skip_context"])
    raw = unet_fixture_weights(int(f["weight_seed"]), skip_context=config.skip_context)
    model = LdmUnetB200(torch_weights(raw, torch.float32), config, device=cuda_device, dtype=torch.float32)
    x = torch.from_numpy(f["x"]).permute(0, 2, 3, 4, 1).contiguous().to(cuda_device)
    t = torch.from_numpy(f["timesteps"].astype(np.int32)).to(cuda_device)
    out = model(x, t, torch.from_numpy(f["context"]))
    torch.cuda.synchronize()
    assert out.dtype == torch.float32
    got = out.permute(0, 4, 1, 2, 3).cpu().numpy()
    want = f["output"].astype(np.float64)
    assert rel_l2(got, want) <= 1e-4
    np.testing.assert_allclose(got, want, rtol=1e-4, atol=1e-5)


def test_fp32_unet_lmnet_shape_matches_oracle(cuda_device):
    """LMNet's topology (16 channels, one residual block per level, attention
    at the 4x level and the middle, 32-wide heads, context) at a small crop,
    FP32, against the oracle's FP32 network (rel-L2 <= 1e-4)."""
    from lesiondiffusion_mlx_b200.networks import LdmUnetB200, UnetConfig

    config = UnetConfig(16, 1, (4,), (1, 2, 4), 32, False)
    raw = random_unet_weights(config, 4, 1, 768, seed=300)
    model = LdmUnetB200(torch_weights(raw, torch.float32), config, device=cuda_device, dtype=torch.float32)
    rng = np.random.default_rng(301)
    x = rng.normal(size=(1, 4, 16, 24, 24)).astype(np.float32)
    t = np.array([531], np.int32)
    ctx = rng.normal(size=(1, 8, 768)).astype(np.float32)
    xin = model.split_input(torch.from_numpy(x).permute(0, 2, 3, 4, 1).contiguous().to(cuda_device))
    out = model(xin, torch.from_numpy(t).to(cuda_device), torch.from_numpy(ctx))
    torch.cuda.synchronize()
    got = out.permute(0, 4, 1, 2, 3).cpu().numpy()
    oracle = OracleUnet(torch_weights(raw, torch.float32), OracleConfig(16, 1, (4,), (1, 2, 4), 32, False))
    ref = oracle(torch.from_numpy(x), torch.from_numpy(t), torch.from_numpy(ctx)).double().numpy()
    assert np.all(np.isfinite(got))
    assert rel_l2(got, ref) <= 1e-4


def test_fp32_lmnet_sampler_matches_oracle_trajectory(cuda_device):
    """Four DDIM steps of the FP32 LMNet-shaped network through the prepared
    sampler (CUDA-graph replay, split network input) against the oracle's
    trajectory with the oracle's FP32 network and the same injected noise."""
    from lesiondiffusion_mlx_b200.networks import LdmUnetB200, UnetConfig
    from lesiondiffusion_mlx_b200.sampling import DdimSampler, PreparedSampler
    from oracle import samplers as oracle_samplers

    config = UnetConfig(16, 1, (4,), (1, 2, 4), 32, False)
    raw = random_unet_weights(config, 4, 1, 768, seed=310)
    model = LdmUnetB200(torch_weights(raw, torch.float32), config, device=cuda_device, dtype=torch.float32)
    rng = np.random.default_rng(311)
    cond = rng.random(size=(1, 3, 8, 16, 16)).astype(np.float32)
    ctx = rng.normal(size=(1, 8, 768)).astype(np.float32)
    init = rng.normal(size=(1, 1, 8, 16, 16)).astype(np.float32)
    betas = np.linspace(0.00085 ** 0.5, 0.012 ** 0.5, 1000, dtype=np.float64) ** 2
    alphas = np.cumprod(1.0 - betas).astype(np.float32)
    steps = 4
    noise = rng.normal(size=(steps, 1, 1, 8, 16, 16)).astype(np.float32)
    sampler = DdimSampler(alphas, steps)
    cache = model.prepare_context(torch.from_numpy(ctx).to(cuda_device))
    prepared = PreparedSampler(sampler, model, cache, torch.from_numpy(cond).permute(0, 2, 3, 4, 1).to(cuda_device),
                               None, graph=True)
    to_ndhwc = lambda a: torch.from_numpy(a).permute(0, 2, 3, 4, 1)  # noqa: E731
    out = prepared.run(to_ndhwc(init).to(cuda_device),
                       torch.stack([to_ndhwc(n) for n in noise]).to(cuda_device))
    torch.cuda.synchronize()
    got = out.permute(0, 4, 1, 2, 3).cpu().numpy()
    oracle = OracleUnet(torch_weights(raw, torch.float32), OracleConfig(16, 1, (4,), (1, 2, 4), 32, False))

    def denoise(net_in, t, condition):
        return oracle(torch.from_numpy(net_in), torch.from_numpy(t), torch.from_numpy(condition)).float().numpy()

    coeffs = oracle_samplers.ddim_coefficients(alphas, steps)
    want = oracle_samplers.ddim_sample(denoise, ctx, cond, coeffs, initial_noise=init, step_noise=list(noise))
    assert np.all(np.isfinite(got))
    assert rel_l2(got, want) <= 1e-4


@pytest.mark.parametrize("quantize", [True, False])
def test_vq_decoder_matches_reference_recording(cuda_device, quantize):
    from lesiondiffusion_mlx_b200.networks import VqDecoderB200

    f = golden("vq_float16")
    raw = vq_fixture_weights(int(f["weight_seed"]))
    dec = VqDecoderB200(torch_weights({k: v for k, v in raw.items() if not k.startswith("encoder")}, torch.float16),
                        device=cuda_device)
    z = to_input(f["z"], cuda_device)
    out = dec.decode(z, quantize=quantize)
    torch.cuda.synchronize()
    got = out.permute(0, 4, 1, 2, 3).float().cpu().numpy()
    want = f["decoded" if quantize else "decoded_unquantized"].astype(np.float32)
    np.testing.assert_allclose(got, want, rtol=2e-3, atol=2e-3)
    oracle = OracleVq(torch_weights(raw, torch.float16))
    ref = oracle.decode(torch.from_numpy(f["z"]).to(torch.float16), quantize=quantize).float().numpy()
    assert rel_l2(got, ref) <= 1e-2


def test_vq_encoder_matches_oracle(cuda_device):
    """VQ encoder (mlx_model.py:729-740), including the stride-2 downsample padded
    only after each axis, against the oracle on the reference fixture weights."""
    from lesiondiffusion_mlx_b200.networks import VqEncoderB200

    raw = vq_fixture_weights(7)
    enc = VqEncoderB200(torch_weights(raw, torch.float16), device=cuda_device)
    x = np.random.default_rng(4).standard_normal((1, 1, 10, 8, 12)).astype(np.float32)
    z = enc.encode(to_input(x, cuda_device))
    torch.cuda.synchronize()
    got = z.permute(0, 4, 1, 2, 3).float().cpu().numpy()
    ref = OracleVq(torch_weights(raw, torch.float16)).encode(torch.from_numpy(x).to(torch.float16)).float().numpy()
    assert got.shape == ref.shape
    assert np.all(np.isfinite(got))
    assert rel_l2(got, ref) <= 1e-2


def test_bundle_loaders_build_the_same_networks(cuda_device, tmp_path):
    """Networks built from the stage-prefixed safetensors bundle (medmlx.py:1585-1602)
    decode and encode like networks built from the same state dict cast to f16
    (the stage loader casts every array, as the reference's does); GroupNorm
    statistics are summed with atomics, so runs agree to rounding, not bits."""
    from lesiondiffusion_mlx_b200.networks import VqDecoderB200, VqEncoderB200
    from lesiondiffusion_mlx_b200.weights import load_vq_decoder, load_vq_encoder, write_safetensors

    raw = vq_fixture_weights(7)
    write_safetensors(tmp_path / "model.safetensors", {"vq." + k: v for k, v in raw.items()})
    tw = {k: torch.from_numpy(np.asarray(v)).to(torch.float16) for k, v in raw.items()}
    z = to_input(np.random.default_rng(2).standard_normal((1, 4, 3, 4, 5)).astype(np.float32), cuda_device)
    a = VqDecoderB200({k: v for k, v in tw.items() if not k.startswith("encoder")}, device=cuda_device).decode(z)
    b = load_vq_decoder(tmp_path, device=cuda_device).decode(z)
    x = to_input(np.random.default_rng(3).standard_normal((1, 1, 6, 8, 8)).astype(np.float32), cuda_device)
    c = VqEncoderB200(tw, device=cuda_device).encode(x)
    d = load_vq_encoder(tmp_path, device=cuda_device).encode(x)
    torch.cuda.synchronize()
    assert rel_l2(a.float().cpu().numpy(), b.float().cpu().numpy()) <= 2e-3
    assert rel_l2(c.float().cpu().numpy(), d.float().cpu().numpy()) <= 2e-3
