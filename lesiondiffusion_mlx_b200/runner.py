"""LINet generation stage on the B200 kernels: the ``_run_linet`` path of the
reference runner (lesiondiffusion_mlx/medmlx.py:1260-1435) from a weight
bundle or prebuilt networks.

One draw:

1. the source CT (HU, source axis order) is mapped to the normalized range
   and rounded to f16 (``piecewise_ct``, medmlx.py:1289-1291) and encoded to
   the VQ latent (``encode_source``, mlx_pipeline.py:99-109);
2. the lesion mask is nearest-resized to the latent grid (medmlx.py:1306-1312;
   a 0/1 mask stays 0/1, so the reference's ``> 0.5`` keeps it as is);
3. LINet's sampling window is the latent image of the fixed-size crop
   centred on the lesion's bounding box (``source_crop`` and
   ``_linet_latent_window``, mlx_pipeline.py:38-69, medmlx.py:1458-1470);
4. the context-bound denoiser samples that window with the fused DDIM or
   DPM++-2M sampler (one CUDA graph per step), and the result is written
   back into the latent rounded to f16 (medmlx.py:1340-1349);
5. the decoder quantizes and decodes the latent to HU (``_decode_ct``,
   medmlx.py:1438-1455): the FP32 decode of ``decoder_mode="reference"`` or
   the scaled f16 decode of ``"scaled_fp16"``; with
   ``output_region="lesion"`` the unmodified latent is decoded too
   (medmlx.py:1381-1390), for the lesion-change compositing.

The text encoder runs once per request and is not on this path: the caller
passes its output (the conditioning sequence) as ``context``.  Volumes stay in
the source axis order; the RAS reorientation is geometry, outside this path.
"""

from __future__ import annotations

import time
from dataclasses import dataclass

import numpy as np
import torch

from . import ops
from .networks import LdmUnetB200, UnetConfig, VqDecoderB200, VqEncoderB200
from .sampling import DdimSampler, Dpmpp2mSampler, PreparedSampler

LINET_CROP = (128, 128, 128)  # image-resolution crop LINet samples (mlx_pipeline.py:21)
# The reference LINet topology (mlx_model.py:72) in conditioned mode (context used).
LINET_CONFIG = UnetConfig(128, 2, (4, 8), (1, 2, 4), 32, False)


def source_crop(mask: np.ndarray, shape: tuple[int, int, int]) -> tuple[slice, slice, slice]:
    """Fixed-size crop centred on the mask's bounding box (mlx_pipeline.py:38-69):
    per axis the centre is the floor midpoint of the extent and the crop is
    shifted to stay inside the volume."""
    points = np.argwhere(mask)
    if points.size == 0:
        raise ValueError("LesionDiffusion cannot crop an empty lesion mask")
    slices = []
    for axis, requested in enumerate(shape):
        length = int(mask.shape[axis])
        if length < requested:
            raise ValueError(f"Pinned LesionDiffusion crop requires source axis {axis} >= {requested}; got {length}")
        center = int((points[:, axis].min() + points[:, axis].max()) // 2)
        start = min(max(center - requested // 2, 0), length - requested)
        slices.append(slice(start, start + requested))
    return slices[0], slices[1], slices[2]


def linet_latent_window(lesion: np.ndarray, crop: tuple[int, int, int] = LINET_CROP) -> tuple[slice, slice, slice]:
    """LINet's window on the half-resolution latent: the crop bounds halved,
    rounding down (medmlx.py:1458-1470)."""
    return tuple(slice(s.start // 2, s.stop // 2) for s in source_crop(lesion, crop))  # type: ignore[return-value]


@dataclass
class LinetNetworks:
    """The networks of one LINet stage: VQ encoder, denoiser (with its
    ``alphas_cumprod``) and the quantizer + decoder."""

    encoder: VqEncoderB200
    unet: LdmUnetB200
    alphas_cumprod: np.ndarray
    decoder: VqDecoderB200

    @classmethod
    def from_bundle(cls, path, *, config: UnetConfig = LINET_CONFIG, decoder_mode: str = "reference",
                    device: torch.device | str = "cuda", groups: int = 16) -> "LinetNetworks":
        """Load the stages from the reference's weight bundle (medmlx.py:1285-1379)."""
        from .weights import load_linet, load_stage, load_vq_encoder

        if decoder_mode not in ("reference", "scaled_fp16"):
            raise ValueError("LesionDiffusion decoder_mode must be reference or scaled_fp16")
        encoder = load_vq_encoder(path, device=device, groups=groups)
        unet, alphas = load_linet(path, config, device=device)
        if alphas is None:
            raise ValueError("the linet stage of the bundle has no alphas_cumprod")
        dtype = torch.float32 if decoder_mode == "reference" else torch.float16
        w = load_stage(path, "vq", dtype=dtype, prefixes=("quantize.", "post_quant_conv.", "decoder."))
        decoder = VqDecoderB200(w, device=device, dtype=dtype, groups=groups, scaled=decoder_mode == "scaled_fp16")
        return cls(encoder, unet, np.asarray(alphas), decoder)


def _decode_hu(decoder: VqDecoderB200, latent: torch.Tensor) -> torch.Tensor:
    """Quantize + decode an f16 latent in the decoder's dtype and map to HU (medmlx.py:1438-1455)."""
    z = latent if latent.dtype == decoder.p.dtype else latent.to(decoder.p.dtype)
    out = decoder.decode(z, quantize=True)
    if not bool(torch.isfinite(out).all()):
        raise FloatingPointError("the VQ decoder produced non-finite voxels before CT remapping")
    hu = ops.hu_map(out)
    return hu[0]


def run_linet(image_hu, lesion: np.ndarray, nets: LinetNetworks, *, context: torch.Tensor | None,
              sampler: str = "ddim", steps: int = 200, crop: tuple[int, int, int] = LINET_CROP,
              initial_noise: torch.Tensor | None = None, step_noise: torch.Tensor | None = None,
              generator: torch.Generator | None = None, output_region: str = "box", graph: bool = True,
              keep_latent: bool = False) -> tuple[torch.Tensor, torch.Tensor | None, dict]:
    """One LINet draw on an even-sized source volume.

    ``image_hu`` is the (D, H, W) float32 CT in HU (NumPy or a CUDA tensor),
    ``lesion`` the boolean (D, H, W) mask on the host, ``context`` the
    conditioning sequence (1, N, C) or None.  ``initial_noise`` / ``step_noise``
    inject the sampler's noise in the window's NDHWC layout (the reference's
    hooks, mlx_sampling.py:66-69); otherwise it is drawn from ``generator`` on
    the device.  Returns the generated CT in HU (D, H, W), the decode of the
    unmodified latent for ``output_region="lesion"`` (else None), and stage facts
    (with ``keep_latent`` also the encoded latent and the latent after the
    write-back, f16 NDHWC, as ``"encoded"`` and ``"latent"``).
    """
    if sampler not in ("ddim", "dpmpp_2m"):
        raise ValueError("LesionDiffusion sampler must be ddim or dpmpp_2m")
    if output_region not in ("box", "lesion"):
        raise ValueError("LesionDiffusion output_region must be box or lesion")
    lesion = np.asarray(lesion).astype(bool)
    device = nets.unet.device
    hu = torch.as_tensor(image_hu, dtype=torch.float32).to(device).contiguous()
    if hu.ndim != 3 or tuple(hu.shape) != lesion.shape:
        raise ValueError("image and lesion must be (D, H, W) volumes of one shape")
    if any(int(n) % 2 for n in hu.shape):
        raise ValueError("the LINet stage takes even extents (the runner pads to them first)")
    window = linet_latent_window(lesion, crop)
    started = time.perf_counter()

    # 1. normalize + encode
    latent = nets.encoder.encode(ops.ct_normalize(hu[None]))
    if not bool(torch.isfinite(latent).all()):
        raise FloatingPointError("the VQ encoder produced non-finite latents")
    _, d, h, w, c = (int(v) for v in latent.shape)
    latent = latent.contiguous()
    # 2. mask on the latent grid
    mask_full = torch.zeros((1, *lesion.shape, 4), dtype=torch.float16, device=device)
    mask_full[..., 0] = torch.from_numpy(lesion).to(device, torch.float16)
    mask = ops.resize_nearest(mask_full, (d, h, w))[..., 0]  # (1, d, h, w) of 0/1
    # 3.-4. sample the window and write it back
    sel = (slice(None), *window)
    input_window = latent[sel].float().contiguous()  # (1, wd, wh, ww, c)
    mask_window = mask[sel].float().contiguous()
    alphas = nets.alphas_cumprod
    smp = DdimSampler(alphas, steps) if sampler == "ddim" else Dpmpp2mSampler(alphas, steps)
    cache = nets.unet.prepare_context(None if context is None else context.to(device))
    prepared = PreparedSampler(smp, nets.unet, cache, input_window, mask_window, graph=graph)
    if initial_noise is None:
        initial_noise = torch.randn(prepared.state.x.shape, generator=generator, device=device)
        if sampler == "ddim":
            step_noise = torch.randn(prepared.state.noise.shape, generator=generator, device=device)
    generated = prepared.run(initial_noise, step_noise)
    encoded = latent.clone() if keep_latent else None
    latent[sel] = generated.to(torch.float16)
    if not bool(torch.isfinite(latent).all()):
        raise FloatingPointError("LINet produced non-finite latents before quantization")
    torch.cuda.synchronize(device)
    sampled = time.perf_counter()
    # 5. decode to HU
    written = latent.clone() if keep_latent else None
    generated_hu = _decode_hu(nets.decoder, latent)
    reconstruction_hu = None
    if output_region == "lesion":
        latent[sel] = input_window.to(torch.float16)
        reconstruction_hu = _decode_hu(nets.decoder, latent)
    torch.cuda.synchronize(device)
    facts = {
        "status": "completed", "device": str(device), "dtype": "float16",
        "decode_dtype": "float32" if nets.decoder.p.dtype == torch.float32 else "float16",
        "latent_shape": [1, c, d, h, w], "window": [[s.start, s.stop] for s in window],
        "output_shape": list(hu.shape), "diffusion_steps": smp.steps, "sampler": sampler,
        "input_reconstruction_decoded": reconstruction_hu is not None, "finite": True,
        "encode_and_sampling_s": sampled - started, "decode_s": time.perf_counter() - sampled,
    }
    if keep_latent:
        facts["encoded"], facts["latent"] = encoded, written
    return generated_hu, reconstruction_hu, facts
