"""B200 networks of the hot path: the 3-D LDM UNet denoiser and the VQ
decoder, composed from the sm_100a operators.

These mirror ``LdmUnet`` and ``VqAutoencoder`` of lesiondiffusion_mlx
(mlx_model.py:384-819) on the native (conditioned-mode) arithmetic, but keep
every activation NDHWC on the device:

* ``norm_silu_conv`` = GroupNorm statistics -> one prepare pass (affine +
  SiLU, f16 rounding; also fuses the skip concatenation) -> tcgen05 conv
  with bias, per-batch shift and residual in its epilogue.
* Transformer tokens are the NDHWC voxels themselves (no transposes); Q, K
  and V come from one fused projection GEMM; residual adds and GELU live in
  the GEMM epilogues; attention is the tcgen05 flash kernel.
* The time-embedding MLP and every residual block's embedding projection
  are skinny GEMMs (rows = batch).

Weights use the reference's state-dict names and are packed once at
construction.  Forward passes allocate through PyTorch's caching allocator,
so a whole step can be captured in a CUDA graph.
"""

from __future__ import annotations

import re
from dataclasses import dataclass

import torch

from . import _lib, ops
from .conv import PackedWeight, conv3d_ndhwc, pack_upsample_weight, pack_weight

UPSAMPLE_CONV = re.compile(r"(?:^output_blocks\.\d+\.\d+|\.upsample)\.conv$")


@dataclass(frozen=True)
class UnetConfig:
    """UNet architecture (mlx_model.py:45-72)."""

    model_channels: int
    num_res_blocks: int
    attention_resolutions: tuple[int, ...]
    channel_mult: tuple[int, ...] = (1, 2, 4)
    num_head_channels: int = 32
    skip_context: bool = False


class _Params:
    """Device copies of a reference-named state dict, packed on first use."""

    def __init__(self, weights: dict[str, torch.Tensor], device: torch.device, dtype: torch.dtype):
        self.raw = weights
        self.device = device
        self.dtype = dtype
        self._cache: dict[tuple[str, str], object] = {}

    def has(self, name: str) -> bool:
        return name in self.raw

    def _get(self, kind: str, key: str, build):
        k = (kind, key)
        if k not in self._cache:
            self._cache[k] = build()
        return self._cache[k]

    def f32(self, name: str) -> torch.Tensor | None:
        if name not in self.raw:
            return None
        return self._get("f32", name, lambda: self.raw[name].to(self.device, torch.float32).contiguous())

    def f16(self, name: str) -> torch.Tensor:
        return self._get("f16", name, lambda: self.raw[name].to(self.device, torch.float16).contiguous())

    def conv(self, key: str, stride: int = 1) -> PackedWeight:
        def build():
            w = self.raw[key + ".weight"].to(self.device, self.dtype)
            if UPSAMPLE_CONV.search(key):
                return pack_upsample_weight(w)
            return pack_weight(w, stride=stride)

        return self._get(f"conv{stride}", key, build)

    def dense_packed(self, *keys: str) -> PackedWeight:
        """Pointwise-packed dense weight; several keys are stacked along outputs (fused Q/K/V)."""

        def build():
            ws = [self.raw[k + ".weight"] for k in keys]
            w = torch.cat([t.reshape(t.shape[0], -1) for t in ws], 0).to(self.device, self.dtype)
            return pack_weight(w[:, :, None, None, None])

        return self._get("dense", "|".join(keys), build)

    def dense_bias(self, *keys: str) -> torch.Tensor | None:
        def build():
            parts = []
            for k in keys:
                b = self.raw.get(k + ".bias")
                if b is None:
                    n = self.raw[k + ".weight"].shape[0]
                    b = torch.zeros(n, dtype=self.dtype)
                parts.append(b.to(self.dtype))
            if all(self.raw.get(k + ".bias") is None for k in keys):
                return None
            return torch.cat(parts).to(self.device, torch.float32).contiguous()

        return self._get("dbias", "|".join(keys), build)


def _voxels(x: torch.Tensor) -> tuple[int, int, int]:
    return int(x.shape[1]), int(x.shape[2]), int(x.shape[3])


_GN_STATS = "_ldb_gn_stats"  # attribute of a conv output that carries its GroupNorm statistics
# Attribute of a tensor in the FP32-exact conv input format (f16 hi plane then
# 2^11-scaled low plane, each padded to 16 channels): its channel count.
_SPLIT_C = "_ldb_split_c"


def _mark_split(t: torch.Tensor, channels: int) -> torch.Tensor:
    setattr(t, _SPLIT_C, channels)
    return t


class _Layers:
    """Layer helpers shared by the networks.  With float32 weights (``exact``)
    every conv and dense layer runs the FP32-exact split-f16 conv, activations
    are f32, and the inputs of those layers are written in the split format
    (by the norm pass, the LayerNorm, or an explicit split pass)."""

    def __init__(self, params: _Params):
        self.p = params
        self.exact = params.dtype == torch.float32
        # Float64 arena that conv outputs feeding a GroupNorm take their
        # statistics slices from: allocated once per (batch, device) and
        # cleared by a memset at the start of every forward (a memset node in
        # a captured step, no kernel).
        self._arena: torch.Tensor | None = None
        self._arenas: dict[tuple[int, torch.device], torch.Tensor] = {}
        self._arena_pos = 0
        self._stats_channels = sum(int(w.shape[0]) for w in params.raw.values() if w.ndim == 5)

    def _begin_stats(self, batch: int, device: torch.device) -> None:
        key = (batch, device)
        arena = self._arenas.get(key)
        if arena is None:
            arena = torch.empty(batch * self._stats_channels * 2, dtype=torch.float64, device=device)
            self._arenas[key] = arena
        _lib.call("ldb_clear_async", torch.cuda.current_stream(device).cuda_stream, arena.data_ptr(),
                  arena.numel() * arena.element_size())
        self._arena = arena
        self._arena_pos = 0

    def _take_stats(self, batch: int, channels: int) -> torch.Tensor | None:
        n = batch * channels * 2
        if self._arena is None or self._arena_pos + n > self._arena.numel():
            return None
        t = self._arena[self._arena_pos : self._arena_pos + n].view(batch, channels, 2)
        self._arena_pos += n
        return t

    def conv(self, x: torch.Tensor, key: str, *, stride: int = 1, residual: torch.Tensor | None = None,
             shift: torch.Tensor | None = None, output_scale: float = 1.0, stats: bool = False,
             pad01: bool = False) -> torch.Tensor:
        """3x3x3 (stride 1/2, or folded up-2x) or pointwise conv of NDHWC f16 x.

        With ``stats`` the output also carries its GroupNorm statistics,
        accumulated by the conv epilogue, for the GroupNorm that reads it;
        ``pad01`` pads a stride-2 conv with zeros only after each axis."""
        packed = self.p.conv(key, stride)
        st = self._take_stats(int(x.shape[0]), packed.out_channels) if stats else None
        x, cin = self._conv_input(x)
        out = conv3d_ndhwc(x, packed, self.p.f32(key + ".bias"), stride=stride, residual=residual, shift=shift,
                           output_scale=output_scale, stats=st, pad01=pad01, in_channels=cin)
        if st is not None:
            setattr(out, _GN_STATS, st)
        return out

    def _conv_input(self, x: torch.Tensor) -> tuple[torch.Tensor, int | None]:
        """(conv input, its channel count for the split format) of an activation."""
        if not self.exact:
            return x, None
        c = getattr(x, _SPLIT_C, None)
        if c is None:
            c = int(x.shape[-1])
            if c % 8:  # the split pass reads 8-channel groups: zero-pad the rows
                x = torch.nn.functional.pad(x, (0, 8 - c % 8))
            x = ops.prepare_input(x, split=True)
        return x, c

    def group_norm_input(self, x: torch.Tensor, norm_key: str, *, groups: int, eps: float, silu: bool,
                         x2: torch.Tensor | None = None) -> torch.Tensor:
        """``f16(silu?(GN([x | x2])))``: one normalize pass that derives the affine
        from the producers' statistics when both sources carry them, else a
        statistics pass and then the normalize pass."""
        gamma, beta = self.p.f32(norm_key + ".weight"), self.p.f32(norm_key + ".bias")
        st1 = getattr(x, _GN_STATS, None)
        st2 = None if x2 is None else getattr(x2, _GN_STATS, None)
        channels = int(x.shape[-1]) + (0 if x2 is None else int(x2.shape[-1]))
        if st1 is not None and (x2 is None or st2 is not None):
            out = ops.prepare_input_from_stats(x, st1, gamma, beta, groups=groups, eps=eps, silu=silu, x2=x2,
                                               stats2=st2, split=self.exact)
        else:
            affine = ops.group_norm_affine(x, gamma, beta, groups=groups, eps=eps, x2=x2)
            out = ops.prepare_input(x, affine=affine, silu=silu, x2=x2, split=self.exact)
        return _mark_split(out, channels) if self.exact else out

    def norm_silu_conv(self, x: torch.Tensor, norm_key: str, conv_key: str, *, groups: int, eps: float,
                       shift: torch.Tensor | None = None, residual: torch.Tensor | None = None,
                       x2: torch.Tensor | None = None, output_scale: float = 1.0, stats: bool = False
                       ) -> torch.Tensor:
        """``residual + conv(SiLU(GN([x | x2]))) + shift`` (mlx_model.py:290-342)."""
        prepared = self.group_norm_input(x, norm_key, groups=groups, eps=eps, silu=True, x2=x2)
        return self.conv(prepared, conv_key, residual=residual, shift=shift, output_scale=output_scale, stats=stats)

    def dense(self, x: torch.Tensor, *keys: str, residual: torch.Tensor | None = None,
              act: int = _lib.LDB_ACT_NONE) -> torch.Tensor:
        """Linear layer(s) on token rows (B, L, C) via the pointwise tensor-core conv."""
        packed = self.p.dense_packed(*keys)
        bias = self.p.dense_bias(*keys)
        x, cin = self._conv_input(x)
        b, length = int(x.shape[0]), int(x.shape[1])
        x5 = x.unsqueeze(1).unsqueeze(1)
        res5 = None if residual is None else residual.unsqueeze(1).unsqueeze(1)
        out = conv3d_ndhwc(x5, packed, bias, residual=res5, act=act, in_channels=cin)
        return out.view(b, length, packed.out_channels)


class LdmUnetB200(_Layers):
    """The LDM UNet (mlx_model.py:384-654) on B200 kernels, NDHWC.

    float16 is the LINet arithmetic; float32 is LMNet's FP32 stage
    (medmlx.py:1168-1257): FP32-exact split-f16 convs and dense layers, FP32
    split-f16 attention, f32 activations.  The float32 network takes its
    input in the split format (``split_input``), as the sampler writes it."""

    def __init__(self, weights: dict[str, torch.Tensor], config: UnetConfig, *, device: torch.device | str = "cuda",
                 dtype: torch.dtype = torch.float16):
        if dtype not in (torch.float16, torch.float32):
            raise ValueError("the B200 UNet runs in float16 (LINet) or float32 (LMNet)")
        super().__init__(_Params(weights, torch.device(device), dtype))
        self.config = config
        self.device = torch.device(device)
        self._side_streams: dict[torch.device, torch.cuda.Stream] = {}
        self.in_channels = int(weights["input_blocks.0.0.weight"].shape[1])
        self.out_channels = int(weights["out.2.weight"].shape[0])
        self._pack_all()
        self._stack_embedding_projections()
        self._pack_dense()

    def _stack_embedding_projections(self) -> None:
        """Stack every residual block's ``emb_layers.1`` so one skinny GEMM per step
        produces all per-block shifts (they all read the same ``silu(emb)``)."""
        keys = sorted(n[: -len(".emb_layers.1.weight")] for n in self.p.raw if n.endswith(".emb_layers.1.weight"))
        self._emb_keys = tuple(k + ".emb_layers.1" for k in keys)
        offsets: dict[str, tuple[int, int]] = {}
        weights, biases, start = [], [], 0
        for key in keys:
            w = self.p.raw[key + ".emb_layers.1.weight"]
            n = int(w.shape[0])
            offsets[key] = (start, start + n)
            weights.append(w.to(torch.float16))
            biases.append(self.p.raw[key + ".emb_layers.1.bias"].to(torch.float16).to(torch.float32))
            start += n
        self._emb_offsets = offsets
        self._emb_weight = torch.cat(weights).to(self.device).contiguous()
        self._emb_bias = torch.cat(biases).to(self.device).contiguous()

    def _pack_all(self) -> None:
        """Pack every weight now so a captured step holds no packing work."""
        for name in self.p.raw:
            if not name.endswith(".weight"):
                continue
            key = name[: -len(".weight")]
            w = self.p.raw[name]
            if w.ndim == 5 and w.shape[2:] == (3, 3, 3):
                self.p.conv(key, 2 if key.endswith(".op") else 1)
            elif w.ndim == 5:
                self.p.conv(key)
            self.p.f32(key + ".bias")
        for name in self.p.raw:
            if name.endswith(".norm.weight") or re.search(r"(in_layers\.0|out_layers\.0|norm[123]|out\.0)\.weight$", name):
                self.p.f32(name)
                self.p.f32(name[: -len("weight")] + "bias")

    def _pack_dense(self) -> None:
        """Pack the dense layers the forward pass uses (fused Q/K/V, Q alone when
        a context gives K/V, the output and feed-forward projections, the time
        and block embeddings), so that no step, eager or captured, packs."""
        groups: list[tuple[str, ...]] = []
        if self.exact:
            groups += [("time_embed.0",), ("time_embed.2",), self._emb_keys]
        else:
            for key in ("time_embed.0", "time_embed.2"):
                self.p.f16(key + ".weight")
                self.p.f32(key + ".bias")
        for name in self.p.raw:
            if not name.endswith(".attn1.to_q.weight"):
                continue
            blk = name[: -len(".attn1.to_q.weight")]
            for attn in (blk + ".attn1", blk + ".attn2"):
                groups += [(attn + ".to_q", attn + ".to_k", attn + ".to_v"), (attn + ".to_q",), (attn + ".to_out.0",)]
            groups += [(blk + ".ff.net.0.0",), (blk + ".ff.net.2",)]
        for keys in groups:
            if not keys or not all(k + ".weight" in self.p.raw for k in keys):
                continue
            if len({tuple(self.p.raw[k + ".weight"].shape[1:]) for k in keys}) != 1:
                continue  # (cross-attention K/V read the context width: never fused with Q)
            self.p.dense_packed(*keys)
            self.p.dense_bias(*keys)

    # ------------------------------------------------------------- blocks

    def split_input(self, x: torch.Tensor) -> torch.Tensor:
        """The network input in the format ``forward`` takes: f16 as is; for the
        float32 network the split planes of f32 ``x``."""
        if not self.exact:
            return x
        split, c = self._conv_input(x)
        return _mark_split(split, c)

    def _rows_dense(self, x: torch.Tensor, *keys: str, silu: bool = False) -> torch.Tensor:
        """FP32 dense layer on (B, C) rows (``silu`` applied to the input first)."""
        c = int(x.shape[-1])
        xs = ops.prepare_input(x, silu=silu, split=True).view(int(x.shape[0]), 1, 1, 1, -1)
        out = conv3d_ndhwc(xs, self.p.dense_packed(*keys), self.p.dense_bias(*keys), in_channels=c)
        return out.view(int(x.shape[0]), -1)

    def time_embedding(self, timesteps: torch.Tensor, step: torch.Tensor | None = None) -> torch.Tensor:
        """mlx_model.py:609-614; ``timesteps`` int32 (B,) or a (steps, B) table read at ``*step``."""
        if self.exact:
            emb = ops.timestep_embedding(timesteps, self.config.model_channels, step=step, out_dtype=torch.float32)
            h = self._rows_dense(emb, "time_embed.0")
            return self._rows_dense(h, "time_embed.2", silu=True)
        emb = ops.timestep_embedding(timesteps, self.config.model_channels, step=step, out_dtype=torch.float16)
        h = ops.dense_small(emb, self.p.f16("time_embed.0.weight"), self.p.f32("time_embed.0.bias"))
        return ops.dense_small(h, self.p.f16("time_embed.2.weight"), self.p.f32("time_embed.2.bias"), in_silu=True)

    def block_shifts(self, emb: torch.Tensor) -> torch.Tensor:
        """All residual blocks' ``dense(silu(emb), emb_layers.1)`` in one launch, f16-rounded f32."""
        if self.exact:
            return self._rows_dense(emb, *self._emb_keys, silu=True)
        return ops.dense_small(emb, self._emb_weight, self._emb_bias, in_silu=True, out_dtype=torch.float32,
                               round_f16=True)

    def residual(self, x: torch.Tensor, emb: torch.Tensor, key: str, x2: torch.Tensor | None = None) -> torch.Tensor:
        """mlx_model.py:420-441 (with the skip concatenation [x | x2] fused into the norm pass).

        ``emb`` is the stacked per-block shift table from ``block_shifts``."""
        if not self.exact and self.p.has(key + ".skip_connection.weight"):
            return self._residual_with_skip_branch(x, emb, key, x2)
        channels = int(x.shape[-1]) + (0 if x2 is None else int(x2.shape[-1]))
        groups = 32 if channels % 32 == 0 else channels
        lo, hi = self._emb_offsets[key]
        shift = emb[:, lo:hi].contiguous()
        h = self.norm_silu_conv(x, key + ".in_layers.0", key + ".in_layers.2", groups=groups, eps=1e-5,
                                shift=shift, x2=x2, stats=True)
        out_c = int(h.shape[-1])
        groups = 32 if out_c % 32 == 0 else out_c
        if self.p.has(key + ".skip_connection.weight"):
            cat = x
            if x2 is not None:
                cat = ops.prepare_input(x, x2=x2, split=self.exact)
                if self.exact:
                    _mark_split(cat, int(x.shape[-1]) + int(x2.shape[-1]))
            skip = self.conv(cat, key + ".skip_connection")
        else:
            skip = x
        return self.norm_silu_conv(h, key + ".out_layers.0", key + ".out_layers.3", groups=groups, eps=1e-5,
                                   residual=skip, stats=True)

    def _side_stream(self, device: torch.device) -> torch.cuda.Stream:
        stream = self._side_streams.get(device)
        if stream is None:
            stream = torch.cuda.Stream(device)
            self._side_streams[device] = stream
        return stream

    def _residual_with_skip_branch(self, x: torch.Tensor, emb: torch.Tensor, key: str,
                                   x2: torch.Tensor | None) -> torch.Tensor:
        """``residual`` for f16 blocks with a 1x1 skip projection: the skip branch
        (the [x | x2] copy and the projection) runs on a side stream while the
        main stream normalizes and convolves, and joins before the second conv
        adds it.  Its buffers are allocated on the main stream first, so the
        allocator never frees memory one stream still uses."""
        main = torch.cuda.current_stream(x.device)
        side = self._side_stream(x.device)
        packed = self.p.conv(key + ".skip_connection")
        b, d, hh, ww, c1 = (int(v) for v in x.shape)
        cin = c1 + (0 if x2 is None else int(x2.shape[-1]))
        cat = None
        if x2 is not None:
            cat = torch.empty((b, d, hh, ww, (cin + 7) // 8 * 8), dtype=torch.float16, device=x.device)
        cout = packed.out_channels
        skip = torch.empty((b, d, hh, ww, (cout + 7) // 8 * 8), dtype=torch.float16, device=x.device)[..., :cout]
        side.wait_stream(main)
        with torch.cuda.stream(side):
            src = x if cat is None else ops.prepare_input(x, x2=x2, out=cat)
            conv3d_ndhwc(src, packed, self.p.f32(key + ".skip_connection.bias"), out=skip, in_channels=cin)
        channels = cin
        groups = 32 if channels % 32 == 0 else channels
        lo, hi = self._emb_offsets[key]
        shift = emb[:, lo:hi].contiguous()
        h = self.norm_silu_conv(x, key + ".in_layers.0", key + ".in_layers.2", groups=groups, eps=1e-5,
                                shift=shift, x2=x2, stats=True)
        out_c = int(h.shape[-1])
        groups = 32 if out_c % 32 == 0 else out_c
        main.wait_stream(side)
        return self.norm_silu_conv(h, key + ".out_layers.0", key + ".out_layers.3", groups=groups, eps=1e-5,
                                   residual=skip, stats=True)

    def attention(self, x: torch.Tensor, key: str, heads: int, kv: tuple[torch.Tensor, torch.Tensor] | None,
                  residual: torch.Tensor) -> torch.Tensor:
        """``residual + to_out(attention(x, context))`` (mlx_model.py:443-493)."""
        c = getattr(x, _SPLIT_C, None) or int(x.shape[-1])
        if kv is None:
            qkv = self.dense(x, key + ".to_q", key + ".to_k", key + ".to_v")
            q, k, v = qkv[..., :c], qkv[..., c : 2 * c], qkv[..., 2 * c :]
        else:
            q = self.dense(x, key + ".to_q")
            k, v = kv
        depth = c // heads
        attn = ops.flash_attention(q, k, v, heads=heads, scale=depth ** -0.5)
        return self.dense(attn, key + ".to_out.0", residual=residual)

    def transformer(self, x: torch.Tensor, key: str, cache: dict) -> torch.Tensor:
        """mlx_model.py:522-552 on NDHWC tokens."""
        b = int(x.shape[0])
        c = int(x.shape[-1])
        normed = self.group_norm_input(x, key + ".norm", groups=32, eps=1e-6, silu=False)
        t = self.conv(normed, key + ".proj_in")
        tokens = t.view(b, -1, c)
        heads = c // self.config.num_head_channels
        blk = key + ".transformer_blocks.0"

        def ln(t_: torch.Tensor, n: str) -> torch.Tensor:
            out = ops.layer_norm(t_, self.p.f32(f"{blk}.{n}.weight"), self.p.f32(f"{blk}.{n}.bias"), 1e-5,
                                 split=self.exact)
            return _mark_split(out, c) if self.exact else out

        tokens = self.attention(ln(tokens, "norm1"), blk + ".attn1", heads, None, tokens)
        tokens = self.attention(ln(tokens, "norm2"), blk + ".attn2", heads, cache.get(blk + ".attn2"), tokens)
        ff = self.dense(ln(tokens, "norm3"), blk + ".ff.net.0.0", act=_lib.LDB_ACT_GELU)
        tokens = self.dense(ff, blk + ".ff.net.2", residual=tokens)
        return self.conv(tokens.view(t.shape), key + ".proj_out", residual=x, stats=True)

    def prepare_context(self, context: torch.Tensor | None) -> dict:
        """Project the context and every attn2 K/V once per binding (mlx_model.py:570-597)."""
        if context is None or self.config.skip_context:
            return {}
        ctx = context.to(self.device, torch.float32 if self.exact else torch.float16).contiguous()
        width = int(context.shape[-1])
        if width % 8:
            ctx = torch.nn.functional.pad(ctx, (0, 8 - width % 8))
            # f16: a channel view of the zero-padded rows; FP32: split planes of
            # the padded rows (the zero channels meet zero weight rows)
            ctx = _mark_split(ops.prepare_input(ctx, split=True), width) if self.exact else ctx[..., :width]
        projected = self.dense(ctx, "context_linear_projection")
        cache = {}
        for name in self.p.raw:
            if name.endswith(".attn2.to_k.weight"):
                key = name[: -len(".to_k.weight")]
                c = int(self.p.raw[key + ".to_k.weight"].shape[0])
                kv = self.dense(projected, key + ".to_k", key + ".to_v")
                cache[key] = (kv[..., :c], kv[..., c:])
        return cache

    def forward(self, x: torch.Tensor, timesteps: torch.Tensor, cache: dict, step: torch.Tensor | None = None
                ) -> torch.Tensor:
        """Noise prediction for NDHWC f16 ``x`` (B, D, H, W, C_in) (mlx_model.py:599-654)."""
        cfg = self.config
        emb = self.block_shifts(self.time_embedding(timesteps, step))
        self._begin_stats(int(x.shape[0]), x.device)
        h = self.conv(x, "input_blocks.0.0", stats=True)
        skips = [h]
        block, resolution = 1, 1
        for level in range(len(cfg.channel_mult)):
            for _ in range(cfg.num_res_blocks):
                key = f"input_blocks.{block}"
                h = self.residual(h, emb, key + ".0")
                if resolution in cfg.attention_resolutions:
                    h = self.transformer(h, key + ".1", cache)
                skips.append(h)
                block += 1
            if level < len(cfg.channel_mult) - 1:
                h = self.conv(h, f"input_blocks.{block}.0.op", stride=2, stats=True)
                skips.append(h)
                block += 1
                resolution *= 2
        h = self.residual(h, emb, "middle_block.0")
        h = self.transformer(h, "middle_block.1", cache)
        h = self.residual(h, emb, "middle_block.2")
        block = 0
        for level in reversed(range(len(cfg.channel_mult))):
            for i in range(cfg.num_res_blocks + 1):
                key = f"output_blocks.{block}"
                h = self.residual(h, emb, key + ".0", x2=skips.pop())
                has_attention = resolution in cfg.attention_resolutions
                if has_attention:
                    h = self.transformer(h, key + ".1", cache)
                if level and i == cfg.num_res_blocks:
                    h = self.conv(h, key + f".{2 if has_attention else 1}.conv", stats=True)
                    resolution //= 2
                block += 1
        groups = 32 if h.shape[-1] % 32 == 0 else int(h.shape[-1])
        out = self.norm_silu_conv(h, "out.0", "out.2", groups=groups, eps=1e-5)
        self._arena = None
        return out

    def __call__(self, x: torch.Tensor, timesteps: torch.Tensor, context: torch.Tensor | None) -> torch.Tensor:
        return self.forward(x, timesteps, self.prepare_context(context))

    def prepare_denoiser(self, context: torch.Tensor | None) -> "BoundDenoiser":
        """Bind ``context`` and project its cross-attention keys / values once
        (mlx_model.py:570-597): the result is ``denoise(x, timesteps)``, and the
        samplers' ``prepare`` takes it.  Its projections belong to this binding."""
        return BoundDenoiser(self, self.prepare_context(context))


class BoundDenoiser:
    """A UNet bound to one context (``LdmUnetB200.prepare_denoiser``).

    ``denoise(x, timesteps)`` predicts the noise of the network input ``x``
    (NDHWC, the layout of ``LdmUnetB200.forward``; the reference's callable
    takes NCDHW MLX arrays) with the binding's precomputed cross-attention
    keys and values."""

    def __init__(self, unet: LdmUnetB200, cache: dict):
        self.unet = unet
        self.cache = cache

    def __call__(self, x: torch.Tensor, timesteps: torch.Tensor) -> torch.Tensor:
        return self.unet.forward(x, timesteps, self.cache)


class VqDecoderB200(_Layers):
    """VQ quantize + decode (mlx_model.py:742-819) on B200 kernels, NDHWC.

    ``levels`` lists decoder levels from the top (first run) down with
    ``(blocks, upsample_after)``; the reference's LINet VQ is 3 levels with
    one upsample after level 1 (the default).  ``scaled`` selects the
    scaled-f16 decode of ScaledVqDecoder (_scaled_vq.py:27-118).  float32
    weights run the reference's FP32 conditioned decode (medmlx.py:1374-1379,
    ``decoder_mode="reference"``): FP32 quantize, FP32-exact split-f16 convs,
    f32 activations.
    """

    SCALE = 0.25

    def __init__(self, weights: dict[str, torch.Tensor], *, device: torch.device | str = "cuda",
                 dtype: torch.dtype = torch.float16, groups: int = 16, scaled: bool = False):
        if dtype not in (torch.float16, torch.float32):
            raise ValueError("the B200 decoder runs in float16 or float32")
        if scaled and dtype != torch.float16:
            raise ValueError("the scaled decoder is the float16 one")
        super().__init__(_Params(weights, torch.device(device), dtype))
        self.device = torch.device(device)
        self.groups = groups
        self.scaled = scaled
        names = set(weights)
        self.levels = sorted({int(m.group(1)) for n in names if (m := re.match(r"decoder\.up\.(\d+)\.", n))},
                             reverse=True)
        self.blocks = {lvl: sorted({int(m.group(1)) for n in names
                                    if (m := re.match(rf"decoder\.up\.{lvl}\.block\.(\d+)\.", n))})
                       for lvl in self.levels}
        self.codebook = weights["quantize.embedding.weight"].to(self.device, dtype).contiguous()
        for name in names:
            if name.endswith(".weight") and weights[name].ndim == 5:
                self.p.conv(name[: -len(".weight")])

    def residual(self, x: torch.Tensor, key: str, scaled_in: bool = False, scaled_out: bool = False) -> torch.Tensor:
        """mlx_model.py:720-727 (+ _scaled_vq.py:75-118 scaling)."""
        eps1 = 1e-6 * (self.SCALE ** 2 if scaled_in else 1.0)
        h = self.norm_silu_conv(x, key + ".norm1", key + ".conv1", groups=self.groups, eps=eps1, stats=True)
        skip = self.conv(x, key + ".nin_shortcut") if self.p.has(key + ".nin_shortcut.weight") else x
        return self.norm_silu_conv(h, key + ".norm2", key + ".conv2", groups=self.groups, eps=1e-6, residual=skip,
                                   output_scale=self.SCALE if scaled_out else 1.0, stats=True)

    def quantize(self, z: torch.Tensor) -> torch.Tensor:
        """Nearest code + straight-through value (mlx_model.py:742-803)."""
        c = int(z.shape[-1])
        buf = torch.zeros((*z.shape[:-1], (c + 7) // 8 * 8), dtype=z.dtype, device=z.device)
        q = buf[..., :c]
        ops.vq_nearest4(z, self.codebook, quantized=q)
        return q

    def decode(self, z: torch.Tensor, *, quantize: bool = True, to_hu: bool = False) -> torch.Tensor:
        """Decode NDHWC latent ``z`` (B, d, h, w, C) in the decoder's dtype to (B, 2d, 2h, 2w, C_out)
        (mlx_model.py:805-819)."""
        if z.dtype != self.p.dtype:
            raise ValueError(f"latent dtype {z.dtype} != decoder dtype {self.p.dtype}")
        x = self.quantize(z) if quantize else z
        self._begin_stats(int(z.shape[0]), z.device)
        x = self.conv(x, "post_quant_conv")
        x = self.conv(x, "decoder.conv_in", stats=True)
        x = self.residual(x, "decoder.mid.block_1")
        x = self.residual(x, "decoder.mid.block_2")
        upsampled = False
        for level in self.levels:
            for block in self.blocks[level]:
                key = f"decoder.up.{level}.block.{block}"
                x = self.residual(x, key, scaled_in=self.scaled and upsampled, scaled_out=self.scaled and upsampled)
            if self.p.has(f"decoder.up.{level}.upsample.conv.weight"):
                x = self.conv(x, f"decoder.up.{level}.upsample.conv",
                              output_scale=self.SCALE if self.scaled else 1.0, stats=True)
                upsampled = True
        eps = 1e-6 * (self.SCALE ** 2 if self.scaled else 1.0)
        out = self.norm_silu_conv(x, "decoder.norm_out", "decoder.conv_out", groups=self.groups, eps=eps)
        self._arena = None
        return ops.hu_map(out) if to_hu else out


class VqEncoderB200(_Layers):
    """VQ encoder (mlx_model.py:729-740) on B200 kernels, NDHWC f16.

    conv_in; per level its residual blocks (mlx_model.py:720-727) and, where
    the weights have one, a stride-2 downsample conv padded with zeros only
    after each axis (mlx_model.py:735-736); two mid blocks; GroupNorm + SiLU
    + conv_out; the 1x1 quant_conv.  Levels and blocks follow the weights.
    """

    def __init__(self, weights: dict[str, torch.Tensor], *, device: torch.device | str = "cuda",
                 dtype: torch.dtype = torch.float16, groups: int = 16):
        if dtype != torch.float16:
            raise ValueError("the B200 encoder runs in float16")
        super().__init__(_Params(weights, torch.device(device), dtype))
        self.device = torch.device(device)
        self.groups = groups
        names = set(weights)
        self.levels = sorted({int(m.group(1)) for n in names if (m := re.match(r"encoder\.down\.(\d+)\.", n))})
        self.blocks = {lvl: sorted({int(m.group(1)) for n in names
                                    if (m := re.match(rf"encoder\.down\.{lvl}\.block\.(\d+)\.", n))})
                       for lvl in self.levels}
        for name in names:
            if name.startswith(("encoder.", "quant_conv")) and name.endswith(".weight") and weights[name].ndim == 5:
                key = name[: -len(".weight")]
                self.p.conv(key, 2 if key.endswith("downsample.conv") else 1)

    def residual(self, x: torch.Tensor, key: str) -> torch.Tensor:
        h = self.norm_silu_conv(x, key + ".norm1", key + ".conv1", groups=self.groups, eps=1e-6, stats=True)
        skip = self.conv(x, key + ".nin_shortcut") if self.p.has(key + ".nin_shortcut.weight") else x
        return self.norm_silu_conv(h, key + ".norm2", key + ".conv2", groups=self.groups, eps=1e-6, residual=skip,
                                   stats=True)

    def encode(self, x: torch.Tensor) -> torch.Tensor:
        """Encode an NDHWC f16 volume (B, D, H, W, C_in) to the latent (B, d, h, w, C_latent)."""
        self._begin_stats(int(x.shape[0]), x.device)
        x = self.conv(x, "encoder.conv_in", stats=True)
        for level in self.levels:
            for block in self.blocks[level]:
                x = self.residual(x, f"encoder.down.{level}.block.{block}")
            if self.p.has(f"encoder.down.{level}.downsample.conv.weight"):
                x = self.conv(x, f"encoder.down.{level}.downsample.conv", stride=2, pad01=True, stats=True)
        x = self.residual(x, "encoder.mid.block_1")
        x = self.residual(x, "encoder.mid.block_2")
        x = self.norm_silu_conv(x, "encoder.norm_out", "encoder.conv_out", groups=self.groups, eps=1e-6)
        self._arena = None
        return self.conv(x, "quant_conv")
