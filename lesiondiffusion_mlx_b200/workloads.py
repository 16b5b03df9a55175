"""Synthetic workloads of the benchmark configurations (random-init weights
with the reference's state-dict names, seeded inputs).

There is no network access for checkpoints or datasets, so every network is
random-initialized (He-normal convolutions and dense layers, unit-ish norm
scales) from a seed, with the layer names and shapes of the reference's
LINet-style UNet (mlx_model.py:384-654) and VQ decoder (:657-819).

* Config 3 (the headline step): UNet with model channels 128, channel
  multipliers (1, 2, 4), two residual blocks per level, spatial transformers
  with 64-wide heads at the two lowest resolutions (16x20x20 and 8x10x10 for
  a 32x40x40 latent), cross-attention to a 77 x 768 context, 8 input
  channels (7 latent channels plus the binary mask channel) and 8 outputs.
* Config 4 (VQ decode): widths 512 / 256 / 128 / 64 at 32x40x40 /
  64x80x80 / 128x160x160 / 128x160x160 (2x nearest upsampling before the
  second and third stage), GroupNorm(32), one output channel.
"""

from __future__ import annotations

import numpy as np

from .networks import UnetConfig

CONFIG3 = UnetConfig(model_channels=128, num_res_blocks=2, attention_resolutions=(2, 4), channel_mult=(1, 2, 4),
                     num_head_channels=64, skip_context=False)
CONFIG3_LATENT = (1, 8, 32, 40, 40)  # (B, C, D, H, W): 7 latent channels + mask
CONFIG3_CONTEXT = (1, 77, 768)


class _ShapeOnly:
    """A stand-in generator whose draws are zero-stride arrays: the weight
    dictionary keeps every name and shape without drawing (or storing) values."""

    def standard_normal(self, shape, dtype=np.float32):
        return np.broadcast_to(np.zeros((), dtype=dtype), shape)


def unet_weights(config: UnetConfig, in_channels: int, out_channels: int, context_dim: int, seed: int,
                 *, shapes_only: bool = False) -> dict[str, np.ndarray]:
    """He-normal float32 weights for a UNet of ``config`` (reference state-dict names).

    ``shapes_only`` returns read-only zero-stride arrays of the right shapes
    (for counting parameters without drawing them)."""
    rng = _ShapeOnly() if shapes_only else np.random.default_rng(seed)
    w: dict[str, np.ndarray] = {}

    def conv(key: str, i: int, o: int, k: int = 3) -> None:
        w[key + ".weight"] = (rng.standard_normal((o, i, k, k, k), dtype=np.float32)
                              * np.float32(np.sqrt(2.0 / (i * k ** 3))))
        w[key + ".bias"] = rng.standard_normal(o, dtype=np.float32) * np.float32(0.02)

    def lin(key: str, i: int, o: int, bias: bool = True) -> None:
        w[key + ".weight"] = rng.standard_normal((o, i), dtype=np.float32) * np.float32(np.sqrt(1.0 / i))
        if bias:
            w[key + ".bias"] = rng.standard_normal(o, dtype=np.float32) * np.float32(0.02)

    def norm(key: str, c: int) -> None:
        w[key + ".weight"] = 1 + np.float32(0.1) * rng.standard_normal(c, dtype=np.float32)
        w[key + ".bias"] = np.float32(0.1) * rng.standard_normal(c, dtype=np.float32)

    mc = config.model_channels
    emb = 4 * mc
    lin("time_embed.0", mc, emb)
    lin("time_embed.2", emb, emb)
    if not config.skip_context:
        lin("context_linear_projection", context_dim, context_dim, bias=False)

    def resblock(key: str, i: int, o: int) -> None:
        norm(key + ".in_layers.0", i)
        conv(key + ".in_layers.2", i, o)
        lin(key + ".emb_layers.1", emb, o)
        norm(key + ".out_layers.0", o)
        conv(key + ".out_layers.3", o, o)
        if i != o:
            conv(key + ".skip_connection", i, o, 1)

    def transformer(key: str, c: int) -> None:
        norm(key + ".norm", c)
        conv(key + ".proj_in", c, c, 1)
        conv(key + ".proj_out", c, c, 1)
        blk = key + ".transformer_blocks.0"
        for n in ("norm1", "norm2", "norm3"):
            norm(f"{blk}.{n}", c)
        for attn in ("attn1", "attn2"):
            kv_in = c if attn == "attn1" or config.skip_context else context_dim
            lin(f"{blk}.{attn}.to_q", c, c, bias=False)
            lin(f"{blk}.{attn}.to_k", kv_in, c, bias=False)
            lin(f"{blk}.{attn}.to_v", kv_in, c, bias=False)
            lin(f"{blk}.{attn}.to_out.0", c, c)
        lin(blk + ".ff.net.0.0", c, 2 * c)
        lin(blk + ".ff.net.2", 2 * c, c)

    conv("input_blocks.0.0", in_channels, mc)
    skip_channels = [mc]
    ch = mc
    block, resolution = 1, 1
    for level, mult in enumerate(config.channel_mult):
        for _ in range(config.num_res_blocks):
            resblock(f"input_blocks.{block}.0", ch, mult * mc)
            ch = mult * mc
            if resolution in config.attention_resolutions:
                transformer(f"input_blocks.{block}.1", ch)
            skip_channels.append(ch)
            block += 1
        if level < len(config.channel_mult) - 1:
            conv(f"input_blocks.{block}.0.op", ch, ch)
            skip_channels.append(ch)
            block += 1
            resolution *= 2
    resblock("middle_block.0", ch, ch)
    transformer("middle_block.1", ch)
    resblock("middle_block.2", ch, ch)
    block = 0
    for level in reversed(range(len(config.channel_mult))):
        mult = config.channel_mult[level]
        for i in range(config.num_res_blocks + 1):
            resblock(f"output_blocks.{block}.0", ch + skip_channels.pop(), mult * mc)
            ch = mult * mc
            has_attention = resolution in config.attention_resolutions
            if has_attention:
                transformer(f"output_blocks.{block}.1", ch)
            if level and i == config.num_res_blocks:
                conv(f"output_blocks.{block}.{2 if has_attention else 1}.conv", ch, ch)
                resolution //= 2
            block += 1
    norm("out.0", ch)
    conv("out.2", ch, out_channels)
    return w


def vq_decoder_weights(widths: tuple[int, ...], upsample_after: tuple[int, ...], latent_channels: int,
                       out_channels: int, codebook_size: int, seed: int) -> dict[str, np.ndarray]:
    """Random decoder weights: ``widths`` per level in execution order (top first);
    level ``len(widths) - 1 - i`` upsamples after its blocks when ``i`` is in ``upsample_after``."""
    rng = np.random.default_rng(seed)
    w: dict[str, np.ndarray] = {}

    def conv(key: str, i: int, o: int, k: int = 3) -> None:
        w[key + ".weight"] = (rng.standard_normal((o, i, k, k, k), dtype=np.float32)
                              * np.float32(np.sqrt(2.0 / (i * k ** 3))))
        w[key + ".bias"] = rng.standard_normal(o, dtype=np.float32) * np.float32(0.02)

    def norm(key: str, c: int) -> None:
        w[key + ".weight"] = 1 + np.float32(0.1) * rng.standard_normal(c, dtype=np.float32)
        w[key + ".bias"] = np.float32(0.1) * rng.standard_normal(c, dtype=np.float32)

    def resblock(key: str, i: int, o: int) -> None:
        norm(key + ".norm1", i)
        conv(key + ".conv1", i, o)
        norm(key + ".norm2", o)
        conv(key + ".conv2", o, o)
        if i != o:
            conv(key + ".nin_shortcut", i, o, 1)

    w["quantize.embedding.weight"] = rng.standard_normal((codebook_size, latent_channels), dtype=np.float32)
    conv("post_quant_conv", latent_channels, latent_channels, 1)
    top = widths[0]
    conv("decoder.conv_in", latent_channels, top)
    resblock("decoder.mid.block_1", top, top)
    resblock("decoder.mid.block_2", top, top)
    ch = top
    n = len(widths)
    for i, width in enumerate(widths):
        level = n - 1 - i
        resblock(f"decoder.up.{level}.block.0", ch, width)
        resblock(f"decoder.up.{level}.block.1", width, width)
        ch = width
        if i in upsample_after:
            conv(f"decoder.up.{level}.upsample.conv", ch, ch)
    norm("decoder.norm_out", ch)
    conv("decoder.conv_out", ch, out_channels)
    return w


# Config 4 (VQ decode): decoder widths 512 / 256 / 128 / 64 in execution order
# with a 2x nearest upsample after the first two levels, 8-channel latent, one
# output channel; 4a is the 32x40x40 latent on one GPU, 4b the 62x110x110
# latent sharded along depth.  GroupNorm groups 32 (BASELINE) for these shapes.
CONFIG4_WIDTHS = (512, 256, 128, 64)
CONFIG4_UPSAMPLE_AFTER = (0, 1)
CONFIG4_LATENTS = {"4a": (1, 8, 32, 40, 40), "4b": (1, 8, 62, 110, 110)}


def config4_decoder_weights(seed: int = 200) -> dict[str, np.ndarray]:
    return vq_decoder_weights(CONFIG4_WIDTHS, CONFIG4_UPSAMPLE_AFTER, latent_channels=8, out_channels=1,
                              codebook_size=512, seed=seed)


def config3_inputs(seed: int = 101, batch: int = 1) -> dict[str, np.ndarray]:
    """Seeded config-3 inputs: noise latent with the mask channel last, context, timesteps.

    The mask is a binary box of 8 x 8 x 5 latent voxels (x, y, z) centred in the
    32 x 40 x 40 latent; channels 0-6 are N(0, 1) noise.
    """
    rng = np.random.default_rng(seed)
    _, c, d, h, w = CONFIG3_LATENT
    x = rng.standard_normal((batch, c, d, h, w), dtype=np.float32)
    mask = np.zeros((batch, 1, d, h, w), dtype=np.float32)
    d0, h0, w0 = d // 2 - 2, h // 2 - 4, w // 2 - 4
    mask[:, :, d0 : d0 + 5, h0 : h0 + 8, w0 : w0 + 8] = 1
    x[:, c - 1 :] = mask
    context = rng.standard_normal((batch, *CONFIG3_CONTEXT[1:]), dtype=np.float32)
    timesteps = rng.integers(0, 1000, size=batch).astype(np.int32)
    return {"x": x, "mask": mask, "context": context, "timesteps": timesteps}


def source_latent(shape: tuple[int, ...], seed: int = 300, sigma: float = 2.0) -> np.ndarray:
    """CT-like source latent: N(0, 1) smoothed by a Gaussian of ``sigma`` voxels per spatial axis."""
    rng = np.random.default_rng(seed)
    z = rng.standard_normal(shape, dtype=np.float32)
    radius = int(3 * sigma)
    taps = np.exp(-0.5 * (np.arange(-radius, radius + 1) / sigma) ** 2)
    taps = (taps / taps.sum()).astype(np.float32)
    for axis in range(2, z.ndim):
        z = np.apply_along_axis(lambda v: np.convolve(np.pad(v, radius, mode="reflect"), taps, mode="valid"), axis, z)
    return z.astype(np.float32)
