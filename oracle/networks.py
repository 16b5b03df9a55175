"""CPU restatement of the reference networks: the 3-D LDM UNet and the VQ
autoencoder (mlx_model.py:384-819), on the native (conditioned-mode)
arithmetic contract.  Test infrastructure only.

``weights`` map upstream state-dict names to torch CPU tensors in the
network dtype.  ``source_rounding=True`` adds the extra roundings of the
reference's per-op (source) arithmetic: SiLU/GN rounded separately from the
conv input, and the conv output rounded before the shift and the residual
are added (mlx_model.py:323-326).
"""

from __future__ import annotations

import math
import re
from dataclasses import dataclass

import torch

from . import ops

UPSAMPLE_CONV = re.compile(r"(?:^output_blocks\.\d+\.\d+|\.upsample)\.conv$")


@dataclass(frozen=True)
class UnetConfig:
    """Architecture of one UNet (mlx_model.py:45-72)."""

    model_channels: int
    num_res_blocks: int
    attention_resolutions: tuple[int, ...]
    channel_mult: tuple[int, ...] = (1, 2, 4)
    num_head_channels: int = 32
    skip_context: bool = False


class _ComputeCache(dict):
    """The weight dict, plus cached compute-dtype copies of every tensor.

    Lookups return the stored tensors unchanged; ``ops`` converts operands
    with ``.to(compute)``, which is free for tensors already in that dtype, so
    conversions are done once here instead of on every call.
    """

    def __init__(self, weights: dict[str, torch.Tensor], compute: torch.dtype):
        super().__init__(weights)
        self.compute = compute
        self.converted: dict[str, torch.Tensor] = {}

    def as_compute(self, key: str) -> torch.Tensor:
        t = self.converted.get(key)
        if t is None:
            t = self[key].to(self.compute)
            self.converted[key] = t
        return t


class OracleLayers:
    def __init__(self, weights: dict[str, torch.Tensor], *, source_rounding: bool = False,
                 compute: torch.dtype = ops.DEFAULT_COMPUTE):
        self.w = _ComputeCache(weights, compute)
        self.source_rounding = source_rounding
        self.compute = compute

    def _bias(self, key: str) -> torch.Tensor | None:
        return self.w.get(key + ".bias")

    def conv(self, x: torch.Tensor, key: str, *, padding: int = 1, stride: int = 1) -> torch.Tensor:
        """mlx_model.py:159-202: 3x3x3 rounds once; 1x1x1 rounds the product then the bias add."""
        weight = self.w.as_compute(key + ".weight")
        if weight.shape[2:] == (1, 1, 1) and padding == 0:
            return ops.pointwise_conv(x, weight, self._bias(key), dtype=x.dtype, compute=self.compute)
        return ops.conv3d(x, weight, self._bias(key), stride=stride, padding=padding, dtype=x.dtype,
                          compute=self.compute)

    def dense(self, x: torch.Tensor, key: str) -> torch.Tensor:
        return ops.dense(x, self.w.as_compute(key + ".weight"), self._bias(key), dtype=x.dtype,
                         compute=self.compute)

    def norm(self, x: torch.Tensor, key: str, *, groups: int, eps: float, silu: bool = False) -> torch.Tensor:
        return ops.native_group_norm(x, self.w[key + ".weight"], self.w[key + ".bias"], groups=groups, eps=eps,
                                     silu=silu)

    def norm_silu_conv(self, x, norm_key, conv_key, *, groups, eps, shift=None, residual=None,
                       output_scale: float = 1.0):
        """mlx_model.py:290-342."""
        if self.source_rounding:
            h = ops.silu(self.norm(x, norm_key, groups=groups, eps=eps))
            y = self.conv(h, conv_key)
            if shift is not None:
                y = (y.to(torch.float32) + shift.to(torch.float32)[:, :, None, None, None]).to(x.dtype)
            if residual is not None:
                y = (residual.to(torch.float32) + y.to(torch.float32)).to(x.dtype)
            return y
        return ops.norm_silu_conv(
            x, self.w[norm_key + ".weight"], self.w[norm_key + ".bias"], self.w.as_compute(conv_key + ".weight"),
            self._bias(conv_key), groups=groups, eps=eps, shift=shift, residual=residual,
            output_scale=output_scale, compute=self.compute,
        )

    def upsample_conv(self, x: torch.Tensor, key: str, *, output_scale: float = 1.0) -> torch.Tensor:
        """mlx_model.py:272-288 (folded nearest-2x conv)."""
        return ops.upsample_conv(x, self.w[key + ".weight"], self._bias(key), dtype=x.dtype,
                                 output_scale=output_scale, compute=self.compute)


def _add(a: torch.Tensor, b: torch.Tensor) -> torch.Tensor:
    """Elementwise add rounded to the operands' dtype."""
    return (a.to(torch.float32) + b.to(torch.float32)).to(a.dtype)


class OracleUnet(OracleLayers):
    """LdmUnet (mlx_model.py:384-654) on CPU."""

    def __init__(self, weights, config: UnetConfig, **kw):
        super().__init__(weights, **kw)
        self.config = config

    def residual(self, x: torch.Tensor, emb: torch.Tensor, key: str) -> torch.Tensor:
        """mlx_model.py:420-441."""
        channels = x.shape[1]
        groups = 32 if channels % 32 == 0 else channels
        shift = self.dense(ops.silu(emb), key + ".emb_layers.1")
        h = self.norm_silu_conv(x, key + ".in_layers.0", key + ".in_layers.2", groups=groups, eps=1e-5,
                                shift=shift)
        groups = 32 if h.shape[1] % 32 == 0 else h.shape[1]
        if key + ".skip_connection.weight" in self.w:
            x = self.conv(x, key + ".skip_connection", padding=0)
        return self.norm_silu_conv(h, key + ".out_layers.0", key + ".out_layers.3", groups=groups, eps=1e-5,
                                   residual=x)

    def attention(self, x, context, key, heads, projected_kv=None):
        """mlx_model.py:443-493 with the flash contract for every head width."""
        context = x if context is None else context
        q = self.dense(x, key + ".to_q")
        if projected_kv is None:
            k, v = self.dense(context, key + ".to_k"), self.dense(context, key + ".to_v")
        else:
            k, v = projected_kv
        depth = q.shape[-1] // heads
        result = ops.attention(q, k, v, heads=heads, scale=depth ** -0.5, compute=self.compute)
        return self.dense(result, key + ".to_out.0")

    def transformer(self, x, context, key, projected_kv=None):
        """mlx_model.py:522-552."""
        residual = x
        x = self.conv(self.norm(x, key + ".norm", groups=32, eps=1e-6), key + ".proj_in", padding=0)
        shape = x.shape
        x = x.permute(0, 2, 3, 4, 1).reshape(shape[0], -1, shape[1])
        heads = shape[1] // self.config.num_head_channels
        blk = key + ".transformer_blocks.0"
        ln = lambda t, n: ops.layer_norm(t, self.w[f"{blk}.{n}.weight"], self.w[f"{blk}.{n}.bias"])  # noqa: E731
        x = _add(x, self.attention(ln(x, "norm1"), None, blk + ".attn1", heads))
        kv = None if projected_kv is None else projected_kv.get(blk + ".attn2")
        x = _add(x, self.attention(ln(x, "norm2"), context, blk + ".attn2", heads, kv))
        ff = ops.gelu(self.dense(ln(x, "norm3"), blk + ".ff.net.0.0"))
        x = _add(x, self.dense(ff, blk + ".ff.net.2"))
        x = x.reshape(shape[0], *shape[2:], shape[1]).permute(0, 4, 1, 2, 3)
        return _add(residual, self.conv(x, key + ".proj_out", padding=0))

    def time_embedding(self, timesteps: torch.Tensor, dtype: torch.dtype) -> torch.Tensor:
        """mlx_model.py:609-614."""
        emb = ops.timestep_embedding(timesteps, self.config.model_channels).to(dtype)
        return self.dense(ops.silu(self.dense(emb, "time_embed.0")), "time_embed.2")

    def project_context(self, context: torch.Tensor | None, dtype: torch.dtype):
        """Context projection and every attn2 K/V, once per binding (mlx_model.py:570-597)."""
        if context is None or self.config.skip_context:
            return None, {}
        projected = self.dense(context.to(dtype), "context_linear_projection")
        cache = {}
        for name in self.w:
            if name.endswith(".attn2.to_k.weight"):
                key = name.removesuffix(".to_k.weight")
                cache[key] = (self.dense(projected, key + ".to_k"), self.dense(projected, key + ".to_v"))
        return projected, cache

    def __call__(self, x: torch.Tensor, timesteps: torch.Tensor, context: torch.Tensor | None) -> torch.Tensor:
        dtype = self.w["time_embed.0.weight"].dtype
        projected, cache = self.project_context(context, dtype)
        return self.forward(x, timesteps, projected, cache)

    def forward(self, x, timesteps, projected, cache):
        """mlx_model.py:599-654."""
        cfg = self.config
        dtype = self.w["time_embed.0.weight"].dtype
        emb = self.time_embedding(timesteps, dtype)
        x = self.conv(x.to(dtype), "input_blocks.0.0")
        skips = [x]
        block, resolution = 1, 1
        for level in range(len(cfg.channel_mult)):
            for _ in range(cfg.num_res_blocks):
                key = f"input_blocks.{block}"
                x = self.residual(x, emb, key + ".0")
                if resolution in cfg.attention_resolutions:
                    x = self.transformer(x, projected, key + ".1", cache)
                skips.append(x)
                block += 1
            if level < len(cfg.channel_mult) - 1:
                x = self.conv(x, f"input_blocks.{block}.0.op", stride=2)
                skips.append(x)
                block += 1
                resolution *= 2
        x = self.residual(x, emb, "middle_block.0")
        x = self.transformer(x, projected, "middle_block.1", cache)
        x = self.residual(x, emb, "middle_block.2")
        block = 0
        for level in reversed(range(len(cfg.channel_mult))):
            for i in range(cfg.num_res_blocks + 1):
                key = f"output_blocks.{block}"
                x = self.residual(torch.cat([x, skips.pop()], dim=1), emb, key + ".0")
                has_attention = resolution in cfg.attention_resolutions
                if has_attention:
                    x = self.transformer(x, projected, key + ".1", cache)
                if level and i == cfg.num_res_blocks:
                    x = self.upsample_conv(x, key + f".{2 if has_attention else 1}.conv")
                    resolution //= 2
                block += 1
        groups = 32 if x.shape[1] % 32 == 0 else x.shape[1]
        return self.norm_silu_conv(x, "out.0", "out.2", groups=groups, eps=1e-5)


class OracleVq(OracleLayers):
    """VqAutoencoder (mlx_model.py:657-819) on CPU; ``scaled`` follows ScaledVqDecoder
    (_scaled_vq.py:27-118) for the scaled-f16 decode."""

    SCALE = 0.25

    def __init__(self, weights, *, scaled: bool = False, groups: int = 16, **kw):
        super().__init__(weights, **kw)
        self.scaled = scaled
        self.groups = groups
        names = list(weights)
        # Decoder levels run from the highest index down (mlx_model.py:813-817); the
        # reference checkpoint has levels 2, 1, 0 with one upsample after level 1.
        self.levels = sorted({int(n.split(".")[2]) for n in names if n.startswith("decoder.up.")}, reverse=True)
        self.blocks = {lvl: sorted({int(n.split(".")[4]) for n in names
                                    if n.startswith(f"decoder.up.{lvl}.block.")}) for lvl in self.levels}

    def residual(self, x: torch.Tensor, key: str, *, scaled: bool = False) -> torch.Tensor:
        """mlx_model.py:720-727 (ScaledVqDecoder.norm_silu_conv for the scaled variant:
        blocks after the upsample take eps * s^2 and scale their output, _scaled_vq.py:75-118)."""
        eps1 = 1e-6 * (self.SCALE ** 2 if scaled else 1.0)
        h = self.norm_silu_conv(x, key + ".norm1", key + ".conv1", groups=self.groups, eps=eps1)
        if key + ".nin_shortcut.weight" in self.w:
            x = self.conv(x, key + ".nin_shortcut", padding=0)
        scale = self.SCALE if scaled else 1.0
        return self.norm_silu_conv(h, key + ".norm2", key + ".conv2", groups=self.groups, eps=1e-6, residual=x,
                                   output_scale=scale)

    def encode(self, x: torch.Tensor) -> torch.Tensor:
        """mlx_model.py:729-740."""
        x = self.conv(x, "encoder.conv_in")
        for level in range(3):
            x = self.residual(x, f"encoder.down.{level}.block.0")
            if level == 0:
                x = torch.nn.functional.pad(x, (0, 1, 0, 1, 0, 1))
                x = self.conv(x, "encoder.down.0.downsample.conv", padding=0, stride=2)
        x = self.residual(x, "encoder.mid.block_1")
        x = self.residual(x, "encoder.mid.block_2")
        x = self.norm_silu_conv(x, "encoder.norm_out", "encoder.conv_out", groups=16, eps=1e-6)
        return self.conv(x, "quant_conv", padding=0)

    def quantize(self, z: torch.Tensor) -> torch.Tensor:
        return ops.quantize(z, self.w["quantize.embedding.weight"])

    def decode(self, z: torch.Tensor, *, quantize: bool = True) -> torch.Tensor:
        """mlx_model.py:805-819."""
        x = self.conv(self.quantize(z) if quantize else z, "post_quant_conv", padding=0)
        x = self.conv(x, "decoder.conv_in")
        x = self.residual(x, "decoder.mid.block_1")
        x = self.residual(x, "decoder.mid.block_2")
        upsampled = False
        for level in self.levels:
            for block in self.blocks[level]:
                x = self.residual(x, f"decoder.up.{level}.block.{block}", scaled=self.scaled and upsampled)
            if f"decoder.up.{level}.upsample.conv.weight" in self.w:
                scale = self.SCALE if self.scaled else 1.0
                x = self.upsample_conv(x, f"decoder.up.{level}.upsample.conv", output_scale=scale)
                upsampled = True
        eps = 1e-6 * (self.SCALE ** 2 if self.scaled else 1.0)
        return self.norm_silu_conv(x, "decoder.norm_out", "decoder.conv_out", groups=self.groups, eps=eps)


def torch_weights(arrays: dict, dtype: torch.dtype) -> dict[str, torch.Tensor]:
    """NumPy float32 weights -> torch tensors of the network dtype."""
    return {k: torch.from_numpy(v).to(dtype) for k, v in arrays.items()}


def conv_flops(weight_shape, out_voxels: int, taps: int | None = None) -> float:
    """2 * M * N * K for a convolution (folded up-convs count their 8 taps)."""
    o, c = weight_shape[:2]
    k = taps if taps is not None else math.prod(weight_shape[2:])
    return 2.0 * out_voxels * o * c * k
