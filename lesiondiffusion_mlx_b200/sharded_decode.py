"""Depth-sharded VQ decode (the large-volume decode spread over several GPUs).

The decoder of ``networks.VqDecoderB200`` (reference: mlx_model.py:720-727,
:805-819) is split along depth: every GPU holds a contiguous slab of the
latent depth and produces the matching slab of the output.  Two things cross
slab boundaries:

* every 3x3x3 convolution (and the folded 2x upsampling conv) reads one depth
  slice beyond each end of its slab.  Activations live in buffers with one
  halo slice on each side; before such a conv the boundary slices are sent to
  the neighbours (grouped NCCL send/recv), and the conv reads the halo through
  ``depth_halo = 1`` instead of zero padding.  At the two ends of the volume
  the halo stays zero, which is the zero padding of the unsharded conv;
* every GroupNorm normalizes over the whole volume (medmlx.py:87-88): each
  producing conv accumulates its slab's per-channel sums (``stats``), the
  slabs' sums are all-reduced, and the affine uses the global voxel count.

Quantization and the HU map are per voxel and need no exchange.

The decode runs over a *list* of slabs with a communicator, so the same code
serves one slab per process (``DistDepthComm`` over torch.distributed, NCCL
on GPUs, gloo on CPU) and all slabs in one process (``LocalDepthComm``, which
emulates the ranks on one GPU so the sharding can be checked against the
unsharded decode).  Batch size 1 (one volume).
"""

from __future__ import annotations

import torch

from . import ops
from .conv import conv3d_ndhwc
from .networks import VqDecoderB200


def partition_depth(depth: int, parts: int) -> list[tuple[int, int]]:
    """Contiguous [start, stop) slabs of ``depth`` slices, sizes differing by at most one.

    The slices left over after an even split go to the end slabs first (slab
    0, the last slab, then 1, the second to last, ...): an end slab exchanges
    one halo per conv, an inner slab two, so the end slabs can take the extra
    slice without becoming the slowest."""
    if parts <= 0 or depth < parts:
        raise ValueError(f"cannot split {depth} slices into {parts} non-empty slabs")
    base, extra = divmod(depth, parts)
    order = [i for pair in zip(range(parts), reversed(range(parts))) for i in pair]
    bigger = set()
    for i in order:
        if len(bigger) == extra:
            break
        bigger.add(i)
    out, start = [], 0
    for i in range(parts):
        stop = start + base + (1 if i in bigger else 0)
        out.append((start, stop))
        start = stop
    return out


class LocalDepthComm:
    """All slabs in this process: halo exchange by copies, statistics summed."""

    def exchange_begin(self, bufs: list[torch.Tensor]):
        """Start the halo exchange (here: done at once by stream-ordered copies)."""
        self.exchange(bufs)
        return None

    def exchange_end(self, handle) -> None:
        """Wait for the exchange begun by ``exchange_begin``."""

    def exchange(self, bufs: list[torch.Tensor]) -> None:
        """``bufs[i]`` (1, d_i + 2, H, W, ld): fill the halo slices from the neighbours."""
        for i, buf in enumerate(bufs):
            if i > 0:
                buf[:, 0].copy_(bufs[i - 1][:, -2])
            if i + 1 < len(bufs):
                buf[:, -1].copy_(bufs[i + 1][:, 1])

    def all_reduce(self, stats: list[torch.Tensor]) -> None:
        total = stats[0].clone()
        for s in stats[1:]:
            total += s
        for s in stats:
            s.copy_(total)


class DistDepthComm:
    """One slab per process, neighbours are ranks r - 1 and r + 1 of ``group``.

    With ``timed = True`` every exchange and all-reduce is bracketed by CUDA
    events on the current stream (the time the decode waits for it);
    ``comm_ms()`` sums the spans recorded so far."""

    def __init__(self, group=None, timed: bool = False):
        import torch.distributed as dist

        self.dist = dist
        self.group = group
        self.rank = dist.get_rank(group)
        self.world = dist.get_world_size(group)
        self.timed = timed
        self._spans: dict[str, list] = {"exchange": [], "all_reduce": []}

    def _span(self, kind: str):
        if not self.timed:
            return None
        start, end = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
        start.record()
        self._spans[kind].append((start, end))
        return end

    def comm_ms(self, reset: bool = True) -> dict[str, float]:
        """Milliseconds the decode spent in exchanges and all-reduces (synchronizes)."""
        torch.cuda.synchronize()
        out = {k: float(sum(s.elapsed_time(e) for s, e in v)) for k, v in self._spans.items()}
        out.update({k + "_calls": len(v) for k, v in self._spans.items()})
        if reset:
            self._spans = {"exchange": [], "all_reduce": []}
        return out

    def _peer(self, r: int) -> int:
        return self.dist.get_global_rank(self.group, r) if self.group is not None else r

    def exchange(self, bufs: list[torch.Tensor]) -> None:
        self.exchange_end(self.exchange_begin(bufs))

    def exchange_begin(self, bufs: list[torch.Tensor]):
        """Post the grouped sends and receives of the halo slices and return
        their requests: NCCL runs them on its own stream after the work already
        on the current stream, so kernels launched before ``exchange_end``
        overlap them (they must not read the halo slices or write the
        boundary slices)."""
        (buf,) = bufs
        dist = self.dist
        p2p = []
        # Same order on every rank: towards rank - 1 first, then towards rank + 1.
        # A depth slice of a batch-1 slab buffer is contiguous (whole channel
        # stride included), so the sends read and the receives write the slab
        # buffer in place.
        if self.rank > 0:
            p2p.append(dist.P2POp(dist.isend, _slice(buf, 1), self._peer(self.rank - 1), self.group))
            p2p.append(dist.P2POp(dist.irecv, _slice(buf, 0), self._peer(self.rank - 1), self.group))
        if self.rank + 1 < self.world:
            last = int(buf.shape[1]) - 1
            p2p.append(dist.P2POp(dist.isend, _slice(buf, last - 1), self._peer(self.rank + 1), self.group))
            p2p.append(dist.P2POp(dist.irecv, _slice(buf, last), self._peer(self.rank + 1), self.group))
        return dist.batch_isend_irecv(p2p) if p2p else []

    def exchange_end(self, handle) -> None:
        """Make the current stream wait for the posted exchange (the span the
        decode waits is what ``comm_ms`` reports as exchange time)."""
        end = self._span("exchange")
        for req in handle:
            req.wait()
        if end is not None:
            end.record()

    def all_reduce(self, stats: list[torch.Tensor]) -> None:
        (s,) = stats
        end = self._span("all_reduce")
        self.dist.all_reduce(s, group=self.group)
        if end is not None:
            end.record()


def _slice(buf: torch.Tensor, index: int) -> torch.Tensor:
    """Depth slice ``index`` of a (1, D, H, W, ld) slab buffer, as a contiguous tensor view."""
    view = buf[:, index]
    if not view.is_contiguous():
        raise ValueError("slab buffers must be batch-1 and dense, so that a depth slice is contiguous")
    return view


class _Slab:
    """An activation slab: (1, d + 2, H, W, ld) buffer with zero halo slices.
    ``x`` is the interior, ``full`` the whole buffer (halo included),
    ``stats`` the GroupNorm sums of the interior when its producer made them."""

    def __init__(self, depth: int, height: int, width: int, channels: int, dtype, device):
        ld = (channels + 7) // 8 * 8
        self.buf = torch.zeros((1, depth + 2, height, width, ld), dtype=dtype, device=device)
        self.channels = channels
        self.stats: torch.Tensor | None = None

    @property
    def full(self) -> torch.Tensor:
        return self.buf[..., : self.channels]

    @property
    def x(self) -> torch.Tensor:
        return self.buf[:, 1:-1, ..., : self.channels]


class ShardedVqDecoder:
    """``VqDecoderB200.decode`` over depth slabs (see the module docstring).

    ``decode`` takes the slabs this process holds (one per rank with
    ``DistDepthComm``, all of them with ``LocalDepthComm``) and the latent
    depth of the whole volume, and returns the output slabs.
    """

    def __init__(self, decoder: VqDecoderB200, comm, *, halo_sms: int = 8):
        self.dec = decoder
        self.p = decoder.p
        self.comm = comm
        # SMs the slab-interior conv leaves free, while an exchange is in
        # flight, for the exchange's communication kernels, which otherwise
        # wait for the conv's persistent grid to finish (0: none)
        self.halo_sms = int(halo_sms)

    # ------------------------------------------------------------ primitives

    def _new(self, like: list[_Slab], channels: int, scale: int = 1) -> list[_Slab]:
        return [_Slab(scale * s.x.shape[1], scale * s.x.shape[2], scale * s.x.shape[3], channels, s.buf.dtype,
                      s.buf.device) for s in like]

    def _conv(self, src: list[_Slab], key: str, *, halo: bool, residual: list[_Slab] | None = None,
              output_scale: float = 1.0, stats: bool = True) -> list[_Slab]:
        """Conv ``key`` of every slab into new slabs; 3x3x3 / up convs read the halo.

        With a halo the exchange runs under the slab's interior: output slices
        1 .. d - 2 read only the slab's own slices, so that conv is launched
        while the boundary slices travel; after the exchange the two boundary
        output slices (which read a halo slice each) follow.  Slabs of fewer
        than three slices wait for the exchange and run one conv."""
        packed = self.p.conv(key)
        up = 2 if packed.kind == "up" else 1
        bias = self.p.f32(key + ".bias")
        out = self._new(src, packed.out_channels, up)
        for o in out:
            if stats:
                o.stats = torch.zeros((1, packed.out_channels, 2), dtype=torch.float64, device=o.buf.device)
        res = [None] * len(src) if residual is None else [r.x for r in residual]

        def run(s: _Slab, o: _Slab, r, first: int, last: int, max_ctas: int = 0) -> None:
            """Output slices [first, last) of the slab from input slices [first, last + 2) of its halo buffer."""
            conv3d_ndhwc(s.full[:, first:last + 2], packed, bias, out=o.x[:, up * first:up * last],
                          residual=None if r is None else r[:, up * first:up * last], output_scale=output_scale,
                          stats=o.stats, depth_halo=1, max_ctas=max_ctas)

        if not halo:
            for s, o, r in zip(src, out, res):
                conv3d_ndhwc(s.x, packed, bias, out=o.x, residual=r, output_scale=output_scale, stats=o.stats)
            return out
        handle = self.comm.exchange_begin([s.buf for s in src])
        split = all(int(s.x.shape[1]) >= 3 for s in src)
        if split:
            interior_ctas = 0
            if self.halo_sms > 0 and handle is not None:
                sms = torch.cuda.get_device_properties(src[0].buf.device).multi_processor_count
                interior_ctas = max(2, sms - self.halo_sms)
            for s, o, r in zip(src, out, res):
                run(s, o, r, 1, int(s.x.shape[1]) - 1, interior_ctas)
        self.comm.exchange_end(handle)
        for s, o, r in zip(src, out, res):
            d = int(s.x.shape[1])
            if split:
                run(s, o, r, 0, 1)
                run(s, o, r, d - 1, d)
            else:
                run(s, o, r, 0, d)
        return out

    def _norm(self, src: list[_Slab], key: str, *, eps: float, voxels: int) -> list[_Slab]:
        """GroupNorm + SiLU of every slab over the whole volume into new slabs."""
        self.comm.all_reduce([s.stats for s in src])
        gamma, beta = self.p.f32(key + ".weight"), self.p.f32(key + ".bias")
        out = self._new(src, src[0].channels)
        for s, o in zip(src, out):
            ops.prepare_input_from_stats(s.x, s.stats, gamma, beta, groups=self.dec.groups, eps=eps, silu=True,
                                         out=o.x, voxels=voxels)
        return out

    def _residual(self, x: list[_Slab], key: str, voxels: int, scaled_in: bool, scaled_out: bool) -> list[_Slab]:
        s = self.dec.SCALE
        h = self._norm(x, key + ".norm1", eps=1e-6 * (s * s if scaled_in else 1.0), voxels=voxels)
        h = self._conv(h, key + ".conv1", halo=True)
        skip = self._conv(x, key + ".nin_shortcut", halo=False, stats=False) \
            if self.p.has(key + ".nin_shortcut.weight") else x
        h = self._norm(h, key + ".norm2", eps=1e-6, voxels=voxels)
        return self._conv(h, key + ".conv2", halo=True, residual=skip, output_scale=s if scaled_out else 1.0)

    # ------------------------------------------------------------ decode

    def decode(self, z_slabs: list[torch.Tensor], latent_depth: int, *, quantize: bool = True,
               to_hu: bool = False) -> list[torch.Tensor]:
        """Decode NDHWC f16 latent slabs (1, d_i, h, w, C) of a volume with
        ``latent_depth`` slices; returns the output slabs (1, s * d_i, ...)."""
        dec = self.dec
        if any(int(z.shape[0]) != 1 for z in z_slabs):
            raise ValueError("the sharded decode handles one volume (batch 1)")
        _, _, hh, ww, c = (int(v) for v in z_slabs[0].shape)
        voxels = latent_depth * hh * ww
        x = []
        for z in z_slabs:
            s = _Slab(int(z.shape[1]), hh, ww, c, torch.float16, z.device)
            s.x.copy_(dec.quantize(z) if quantize else z)
            x.append(s)
        x = self._conv(x, "post_quant_conv", halo=False, stats=False)
        x = self._conv(x, "decoder.conv_in", halo=True)
        x = self._residual(x, "decoder.mid.block_1", voxels, False, False)
        x = self._residual(x, "decoder.mid.block_2", voxels, False, False)
        upsampled = False
        for level in dec.levels:
            for block in dec.blocks[level]:
                scaled = dec.scaled and upsampled
                x = self._residual(x, f"decoder.up.{level}.block.{block}", voxels, scaled, scaled)
            if self.p.has(f"decoder.up.{level}.upsample.conv.weight"):
                x = self._conv(x, f"decoder.up.{level}.upsample.conv", halo=True,
                               output_scale=dec.SCALE if dec.scaled else 1.0)
                voxels *= 8
                upsampled = True
        eps = 1e-6 * (dec.SCALE ** 2 if dec.scaled else 1.0)
        h = self._norm(x, "decoder.norm_out", eps=eps, voxels=voxels)
        out = self._conv(h, "decoder.conv_out", halo=True, stats=False)
        return [ops.hu_map(o.x) if to_hu else o.x for o in out]
