"""The LINet stage runner (``runner.run_linet``, the reference's ``_run_linet``,
medmlx.py:1260-1435) end to end from a weight bundle, and the FP32 decoder it
uses by default (GPU).

The bundle is written with the reference's stage-prefixed safetensors names:
the golden VQ autoencoder (encoder, codebook, decoder; rescaled to He-normal
magnitudes so the decode is sensitive to its input) and a small LINet-shaped
UNet (4 latent channels + mask in, 32 model channels, attention at the
lower level, cross-attention to a 3 x 32 context) with the real LINet
``alphas_cumprod``.  The oracle composes the same draw from its restatements:
CT map -> encoder -> nearest mask resize -> window -> DDIM with injected noise
-> write-back -> FP32 quantize + decode -> HU.  As in the reference's own
end-to-end test (tests/test_medmlx.py:420-459: "nearest-code switches make a
uniform HU bound invalid for independently computed latents"), generation and
decoding are checked apart: the encoder's latent and the sampled window against
the oracle's at the f16 bound (relative L2 <= 1e-2), and the decode of the
runner's own latent to HU against the oracle's decode of that latent at the
north star's bound (mean absolute error <= 1 HU), generated and reconstructed.
"""

from __future__ import annotations

from pathlib import Path

import numpy as np
import pytest
import torch

from oracle import ops as oops
from oracle import samplers as osamp
from oracle.networks import OracleUnet, OracleVq, UnetConfig as OracleConfig, torch_weights
from tests.golden.fixture_weights import vq_fixture_weights

pytestmark = pytest.mark.gpu

GOLDEN = Path(__file__).parent / "golden" / "reference_fixtures.npz"


def golden(name: str) -> dict[str, np.ndarray]:
    with np.load(GOLDEN, allow_pickle=False) as archive:
        return {k.split("/", 1)[1]: archive[k] for k in archive.files if k.startswith(name + "/")}


def rel_l2(a, b) -> float:
    a = np.asarray(a, np.float64)
    b = np.asarray(b, np.float64)
    return float(np.linalg.norm(a - b) / max(np.linalg.norm(b), 1e-30))


def test_fp32_decoder_matches_reference_recording(cuda_device):
    """The FP32 decode (``decoder_mode="reference"``) against the reference's
    FP32 recording of the golden VQ: quantized codes bit-exact, decode at the
    reference's FP32 tolerance (2e-6 absolute + 2e-5 relative)."""
    from lesiondiffusion_mlx_b200.networks import VqDecoderB200

    f = golden("vq_float32")
    raw = vq_fixture_weights(int(f["weight_seed"]))
    dec = VqDecoderB200(torch_weights({k: v for k, v in raw.items() if not k.startswith("encoder")}, torch.float32),
                        device=cuda_device, dtype=torch.float32)
    z = torch.from_numpy(f["z"]).permute(0, 2, 3, 4, 1).contiguous().to(cuda_device)
    out = dec.decode(z).permute(0, 4, 1, 2, 3).cpu().numpy()
    q = dec.quantize(z).permute(0, 4, 1, 2, 3).cpu().numpy()
    assert out.dtype == np.float32
    np.testing.assert_array_equal(q, f["quantized"])
    np.testing.assert_allclose(out, f["decoded"], rtol=2e-5, atol=2e-6)


def _he_vq(seed: int) -> dict[str, np.ndarray]:
    """The golden VQ weights rescaled to He-normal magnitudes (codebook to unit scale)."""
    out = {}
    for k, v in vq_fixture_weights(seed).items():
        if k.endswith(".weight") and v.ndim == 5:
            v = v * np.float32(np.sqrt(2.0 / (v.shape[1] * v[0, 0].size)) / 0.02)
        elif k == "quantize.embedding.weight":
            v = v * np.float32(50.0)
        out[k] = v
    return out


@pytest.fixture(scope="module")
def bundle(tmp_path_factory):
    from lesiondiffusion_mlx_b200 import workloads
    from lesiondiffusion_mlx_b200.networks import UnetConfig
    from lesiondiffusion_mlx_b200.weights import write_safetensors

    config = UnetConfig(32, 1, (2,), (1, 2), 32, False)
    unet = workloads.unet_weights(config, 5, 4, 32, seed=41)
    vq = _he_vq(7)
    alphas = golden("dpmpp_2m")["linet_4.alphas_cumprod"]
    tensors = {f"linet.{k}": v for k, v in unet.items()}
    tensors["linet.alphas_cumprod"] = alphas
    tensors.update({f"vq.{k}": v for k, v in vq.items()})
    path = tmp_path_factory.mktemp("bundle") / "model.safetensors"
    write_safetensors(path, tensors)
    return path, config, unet, vq, alphas


def _volume(shape=(16, 24, 24), seed=3) -> tuple[np.ndarray, np.ndarray]:
    """A CT-like volume in HU (smoothed noise around soft tissue, air and bone
    extremes clipped by the map) and a box lesion."""
    from lesiondiffusion_mlx_b200 import workloads

    smooth = workloads.source_latent((1, 1, *shape), seed=seed, sigma=1.5)[0, 0]
    image = (40.0 + 900.0 * smooth / np.abs(smooth).max()).astype(np.float32)
    lesion = np.zeros(shape, bool)
    lesion[6:11, 9:15, 8:14] = True
    return image, lesion


@pytest.mark.parametrize("sampler,decoder_mode", [("ddim", "reference"), ("ddim", "scaled_fp16"),
                                                   ("dpmpp_2m", "reference")])
def test_run_linet_matches_oracle_composition(cuda_device, bundle, sampler, decoder_mode):
    from lesiondiffusion_mlx_b200 import runner

    path, config, unet_w, vq_w, alphas = bundle
    image, lesion = _volume()
    crop = (8, 16, 16)
    nets = runner.LinetNetworks.from_bundle(path, config=config, decoder_mode=decoder_mode, device=cuda_device)
    window = runner.linet_latent_window(lesion, crop)
    wshape = tuple(s.stop - s.start for s in window)
    rng = np.random.default_rng(11)
    context = rng.standard_normal((1, 3, 32)).astype(np.float32)
    init = rng.standard_normal((1, 4, *wshape)).astype(np.float32)
    noise = rng.standard_normal((4, 1, 4, *wshape)).astype(np.float32)
    to_dev = lambda a: torch.from_numpy(np.ascontiguousarray(np.moveaxis(a, -4, -1))).to(cuda_device)  # noqa: E731
    gen_hu, recon_hu, facts = runner.run_linet(image, lesion, nets, context=torch.from_numpy(context), steps=4,
                                               sampler=sampler, crop=crop, initial_noise=to_dev(init),
                                               step_noise=to_dev(noise) if sampler == "ddim" else None,
                                               output_region="lesion", keep_latent=True)
    ncdhw = lambda t: t.permute(0, 4, 1, 2, 3).contiguous().cpu()  # noqa: E731
    encoded_gpu, latent_gpu = ncdhw(facts["encoded"]), ncdhw(facts["latent"])
    gen = gen_hu.cpu().numpy()
    recon = recon_hu.cpu().numpy()
    assert gen.shape == recon.shape == image.shape and facts["window"] == [[s.start, s.stop] for s in window]
    assert np.all(np.isfinite(gen)) and np.all(np.isfinite(recon))

    # oracle composition of the same draw
    norm = oops.piecewise_ct(torch.from_numpy(image)[None, None]).to(torch.float16)
    enc = OracleVq(torch_weights(vq_w, torch.float16), compute=torch.float32).encode(norm)
    mask = oops.resize_nearest(torch.from_numpy(lesion)[None, None].to(torch.float16), tuple(enc.shape[2:]))
    sel = (slice(None), slice(None), *window)
    image_w = enc[sel].float().numpy()
    mask_w = (mask[sel].float().numpy() > 0.5).astype(np.float32)
    oracle = OracleUnet(torch_weights(unet_w, torch.float16), OracleConfig(32, 1, (2,), (1, 2), 32, False),
                        compute=torch.float32)
    projected, kv = oracle.project_context(torch.from_numpy(context), torch.float16)

    def denoise(net_in, t, _condition):
        return oracle.forward(torch.from_numpy(net_in).to(torch.float16), torch.from_numpy(t), projected, kv).float()

    if sampler == "ddim":
        x = osamp.ddim_sample(denoise, None, image_w, osamp.ddim_coefficients(alphas, 4), initial_noise=init,
                              step_noise=noise, mask=mask_w)
    else:
        ts, coeffs = osamp.dpm_coefficients(alphas, 4)
        x = osamp.dpm_sample(lambda net_in, t: denoise(net_in, t, None), image_w, ts, coeffs, initial_noise=init,
                             mask=mask_w)
    # generation: encoder latent and sampled window at the f16 bound
    assert rel_l2(encoded_gpu.float().numpy(), enc.float().numpy()) <= 1e-2
    assert rel_l2(latent_gpu[sel].float().numpy(), x) <= 1e-2
    assert torch.equal(latent_gpu[:, :, :window[0].start], encoded_gpu[:, :, :window[0].start])  # outside the window

    def decode(z16):
        if decoder_mode == "reference":
            model = OracleVq(torch_weights(vq_w, torch.float32), compute=torch.float64)
            return model.decode(z16.float())
        model = OracleVq(torch_weights(vq_w, torch.float16), scaled=True, compute=torch.float32)
        return model.decode(z16)

    # decoding: the oracle decodes the runner's own latents (the same codes)
    want = oops.piecewise_ct(decode(latent_gpu), inverse=True).numpy()[0, 0]
    want_recon = oops.piecewise_ct(decode(encoded_gpu), inverse=True).numpy()[0, 0]
    mae = float(np.mean(np.abs(gen.astype(np.float64) - want)))
    mae_recon = float(np.mean(np.abs(recon.astype(np.float64) - want_recon)))
    assert mae <= 1.0, f"generated volume MAE {mae:.3f} HU"
    assert mae_recon <= 1.0, f"reconstruction MAE {mae_recon:.3f} HU"
    # the draw changed the lesion window and only the decode's reach around it
    assert np.abs(gen - recon).max() > 1.0
