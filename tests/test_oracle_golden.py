"""Pin the CPU oracle against the reference's golden vectors (CPU only).

The vectors are the reference's Torch-CPU recordings of the pinned upstream
model (copied by tests/golden/make_golden.py).  Tolerances are the
reference's own (tests/test_equivalence.py:62-73 of lesiondiffusion-mlx):
f16 atol = rtol = 2e-3, FP32 atol 2e-6 / rtol 2e-5; quantization and
timestep schedules are bit-exact.
"""

from __future__ import annotations

import json
from pathlib import Path

import numpy as np
import pytest
import torch

from oracle import ops, samplers
from oracle.networks import OracleUnet, OracleVq, UnetConfig, torch_weights
from tests.golden.fixture_weights import sampling_toy_denoiser, unet_fixture_weights, vq_fixture_weights

GOLDEN = Path(__file__).parent / "golden" / "reference_fixtures.npz"


@pytest.fixture(scope="module")
def golden() -> dict[str, np.ndarray]:
    with np.load(GOLDEN, allow_pickle=False) as archive:
        return {k: archive[k] for k in archive.files}


def fixture(golden: dict, name: str) -> dict[str, np.ndarray]:
    prefix = name + "/"
    return {k[len(prefix):]: v for k, v in golden.items() if k.startswith(prefix)}


def assert_numerical(actual: np.ndarray, expected: np.ndarray) -> None:
    assert actual.dtype == expected.dtype
    atol, rtol = (2e-3, 2e-3) if expected.dtype == np.float16 else (2e-6, 2e-5)
    np.testing.assert_allclose(actual.astype(np.float64), expected.astype(np.float64), atol=atol, rtol=rtol)


@pytest.mark.parametrize("name", ["unet_mask", "unet_inpainting"])
def test_oracle_unet_matches_reference_recording(golden, name):
    f = fixture(golden, name)
    cfg = json.loads(f["config"].item())
    config = UnetConfig(
        cfg["model_channels"], cfg["num_res_blocks"], tuple(cfg["attention_resolutions"]),
        tuple(cfg["channel_mult"]), cfg["num_head_channels"], cfg["skip_context"],
    )
    dtype = torch.float16 if f["dtype"].item() == "float16" else torch.float32
    weights = torch_weights(unet_fixture_weights(int(f["weight_seed"]), skip_context=config.skip_context), dtype)
    model = OracleUnet(weights, config)
    out = model(torch.from_numpy(f["x"]), torch.from_numpy(f["timesteps"]), torch.from_numpy(f["context"]))
    assert_numerical(out.numpy(), f["output"])


@pytest.mark.parametrize("dtype_name", ["float32", "float16"])
def test_oracle_vq_matches_reference_recording(golden, dtype_name):
    f = fixture(golden, "vq_" + dtype_name)
    dtype = getattr(torch, dtype_name)
    model = OracleVq(torch_weights(vq_fixture_weights(int(f["weight_seed"])), dtype))
    z = torch.from_numpy(f["z"]).to(dtype)
    quantized = model.quantize(z).numpy()
    assert quantized.dtype == f["quantized"].dtype
    np.testing.assert_array_equal(quantized, f["quantized"])
    assert_numerical(model.decode(z).numpy(), f["decoded"])
    assert_numerical(model.decode(z, quantize=False).numpy(), f["decoded_unquantized"])


@pytest.mark.parametrize("name", ["ddim_mask", "ddim_inpainting"])
def test_oracle_ddim_matches_reference_recording(golden, name):
    f = fixture(golden, name)
    coeffs = samplers.ddim_coefficients(f["alphas"], int(f["steps"]))
    np.testing.assert_array_equal(coeffs["timesteps"], f["timesteps"])
    for ours, theirs in (("alphas", "alphas_selected"), ("previous", "previous"),
                         ("sqrt_one_minus", "sqrt_one_minus"), ("sigmas", "sigmas")):
        assert_numerical(coeffs[ours], f[theirs])
    mask = f.get("mask")
    out = samplers.ddim_sample(
        sampling_toy_denoiser, f["condition"], f["image"], coeffs, initial_noise=f["initial"],
        step_noise=f["noise"], mask=mask,
    )
    assert_numerical(out, f["output"])


@pytest.mark.parametrize("stage", ["lmnet", "linet"])
@pytest.mark.parametrize("steps", [4, 8, 25])
def test_oracle_dpm_matches_diffusers_trajectory(golden, stage, steps):
    f = fixture(golden, "dpmpp_2m")
    d = {k.split(".", 1)[1]: v for k, v in f.items() if k.startswith(f"{stage}_{steps}.")}
    ts, coeffs = samplers.dpm_coefficients(d["alphas_cumprod"], steps)
    np.testing.assert_array_equal(np.array(ts), d["timesteps"])
    image = d["conditioning_image"]
    mask = d.get("mask")
    observed: list[np.ndarray] = []
    predictions = d["predictions"]

    def denoiser(x, timestep):
        i = len(observed) - 1
        np.testing.assert_array_equal(timestep, d["timesteps"][i : i + 1].astype(np.int32))
        return predictions[i]

    out = samplers.dpm_sample(denoiser, image, ts, coeffs, initial_noise=d["initial_noise"], mask=mask,
                              observer=lambda x: observed.append(x[:, : image.shape[1]].copy()))
    assert_numerical(out, d["output"])
    assert_numerical(np.stack(observed), d["projected_inputs"])
    if mask is not None:
        outside = np.broadcast_to(mask == 0, out.shape)
        np.testing.assert_array_equal(out[outside], image[outside])


@pytest.mark.parametrize("name", ["silu", "softmax"])
def test_oracle_half_activations(golden, name):
    f = fixture(golden, "unet_activations")
    x = torch.from_numpy(f[name + "_input"])
    if name == "silu":
        actual = ops.silu(x).numpy()
    else:
        y = torch.softmax(x.to(torch.float32), dim=-1)
        actual = y.to(torch.float16).numpy()
    expected = f[name + "_output"]
    ulps = np.abs(actual.astype(np.float32) - expected.astype(np.float32)) / np.abs(np.spacing(expected)).astype(np.float32)
    assert float(ulps.max()) <= 1
    assert float(np.sqrt(np.mean(ulps ** 2))) <= 0.1


def test_oracle_piecewise_ct(golden):
    f = fixture(golden, "pipeline")
    forward = ops.piecewise_ct(torch.from_numpy(f["ct"])).numpy()
    assert_numerical(forward, f["ct_output"])
    inverse = ops.piecewise_ct(torch.from_numpy(f["normalized"]), inverse=True).numpy()
    np.testing.assert_allclose(inverse, f["inverse_output"], atol=4 * np.spacing(np.float32(1000)), rtol=0)
