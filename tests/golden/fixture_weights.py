"""Seeded synthetic weights of the reference's golden-vector models.

The reference's recordings were made with weights drawn from NumPy's
``default_rng(seed)``: every tensor is ``standard_normal(shape) * 0.02`` (+1
for norm scales) in float32, drawn in a fixed key order (lesiondiffusion-mlx
tests/_fixture_models.py:31-157).  Reproducing the recordings requires the
same draws in the same order, so the key sequence below necessarily matches
that module; the code itself is written independently.
"""

from __future__ import annotations

import numpy as np


class _Draws:
    def __init__(self, seed: int):
        self.rng = np.random.default_rng(seed)
        self.out: dict[str, np.ndarray] = {}

    def tensor(self, key: str, shape: tuple[int, ...], offset: float = 0.0) -> None:
        self.out[key] = self.rng.standard_normal(shape).astype(np.float32) * np.float32(0.02) + offset

    def linear(self, key: str, n_in: int, n_out: int, bias: bool = True) -> None:
        self.tensor(key + ".weight", (n_out, n_in))
        if bias:
            self.tensor(key + ".bias", (n_out,))

    def conv(self, key: str, n_in: int, n_out: int, k: int = 3) -> None:
        self.tensor(key + ".weight", (n_out, n_in, k, k, k))
        self.tensor(key + ".bias", (n_out,))

    def norm(self, key: str, channels: int) -> None:
        self.tensor(key + ".weight", (channels,), offset=1.0)
        self.tensor(key + ".bias", (channels,))


def unet_fixture_weights(seed: int, *, skip_context: bool) -> dict[str, np.ndarray]:
    """Weights of the golden UNet (mc 32, mult (1, 2), 1 res block, attention at 1 and 2)."""
    r = _Draws(seed)
    r.linear("time_embed.0", 32, 128)
    r.linear("time_embed.2", 128, 128)
    if not skip_context:
        r.linear("context_linear_projection", 6, 6, bias=False)

    def resblock(key: str, n_in: int, n_out: int) -> None:
        r.norm(key + ".in_layers.0", n_in)
        r.conv(key + ".in_layers.2", n_in, n_out)
        r.linear(key + ".emb_layers.1", 128, n_out)
        r.norm(key + ".out_layers.0", n_out)
        r.conv(key + ".out_layers.3", n_out, n_out)
        if n_in != n_out:
            r.conv(key + ".skip_connection", n_in, n_out, 1)

    def spatial_transformer(key: str, ch: int) -> None:
        r.norm(key + ".norm", ch)
        r.conv(key + ".proj_in", ch, ch, 1)
        r.conv(key + ".proj_out", ch, ch, 1)
        blk = key + ".transformer_blocks.0"
        for n in ("norm1", "norm2", "norm3"):
            r.norm(f"{blk}.{n}", ch)
        for attn in ("attn1", "attn2"):
            ctx = ch if attn == "attn1" or skip_context else 6
            r.linear(f"{blk}.{attn}.to_q", ch, ch, bias=False)
            r.linear(f"{blk}.{attn}.to_k", ctx, ch, bias=False)
            r.linear(f"{blk}.{attn}.to_v", ctx, ch, bias=False)
            r.linear(f"{blk}.{attn}.to_out.0", ch, ch)
        r.linear(blk + ".ff.net.0.0", ch, 2 * ch)
        r.linear(blk + ".ff.net.2", 2 * ch, ch)

    r.conv("input_blocks.0.0", 5 if skip_context else 4, 32)
    resblock("input_blocks.1.0", 32, 32)
    spatial_transformer("input_blocks.1.1", 32)
    r.conv("input_blocks.2.0.op", 32, 32)
    resblock("input_blocks.3.0", 32, 64)
    spatial_transformer("input_blocks.3.1", 64)
    resblock("middle_block.0", 64, 64)
    spatial_transformer("middle_block.1", 64)
    resblock("middle_block.2", 64, 64)
    for i, n_in, n_out in ((0, 128, 64), (1, 96, 64), (2, 96, 32), (3, 64, 32)):
        resblock(f"output_blocks.{i}.0", n_in, n_out)
        spatial_transformer(f"output_blocks.{i}.1", n_out)
    r.conv("output_blocks.1.2.conv", 64, 64)
    r.norm("out.0", 32)
    r.conv("out.2", 32, 5 if skip_context else 1)
    return r.out


def vq_fixture_weights(seed: int) -> dict[str, np.ndarray]:
    """Weights of the golden VQ autoencoder (4-channel latent, codebook of 8)."""
    r = _Draws(seed)

    def resblock(key: str, n_in: int, n_out: int) -> None:
        r.norm(key + ".norm1", n_in)
        r.conv(key + ".conv1", n_in, n_out)
        r.norm(key + ".norm2", n_out)
        r.conv(key + ".conv2", n_out, n_out)
        if n_in != n_out:
            r.conv(key + ".nin_shortcut", n_in, n_out, 1)

    r.conv("encoder.conv_in", 1, 16)
    resblock("encoder.down.0.block.0", 16, 16)
    r.conv("encoder.down.0.downsample.conv", 16, 16)
    resblock("encoder.down.1.block.0", 16, 32)
    resblock("encoder.down.2.block.0", 32, 32)
    for name in ("block_1", "block_2"):
        resblock("encoder.mid." + name, 32, 32)
        resblock("decoder.mid." + name, 32, 32)
    r.norm("encoder.norm_out", 32)
    r.conv("encoder.conv_out", 32, 4)
    r.conv("quant_conv", 4, 4, 1)
    r.tensor("quantize.embedding.weight", (8, 4))
    r.conv("post_quant_conv", 4, 4, 1)
    r.conv("decoder.conv_in", 4, 32)
    for level, n_in, n_out in ((2, 32, 32), (1, 32, 32), (0, 32, 16)):
        resblock(f"decoder.up.{level}.block.0", n_in, n_out)
        resblock(f"decoder.up.{level}.block.1", n_out, n_out)
    r.conv("decoder.up.1.upsample.conv", 32, 32)
    r.norm("decoder.norm_out", 16)
    r.conv("decoder.conv_out", 16, 1)
    return r.out


def sampling_toy_denoiser(x, timestep, condition):
    """Deterministic toy noise predictor used by the DDIM recordings.

    ``x * 0.125 + t * 0.001 + sum(condition) * 0.01`` on the first channel of
    a 4-channel input (tests/_fixture_models.py:200-211 of the reference).
    Works on NumPy or torch arrays.
    """
    x = x[:, :1] if x.shape[1] == 4 else x
    return x * 0.125 + timestep.reshape(-1, 1, 1, 1, 1).astype("float32") * 0.001 + condition.sum() * 0.01
