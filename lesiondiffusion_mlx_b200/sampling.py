"""DDIM and DPM++-2M samplers on the B200 path.

Host side (once per sampler): the reference's schedules and per-step
coefficients, with the checkpoint dtype's rounding boundaries kept
(mlx_sampling.py:27-60, _dpm.py:30-62, _schedules.py:11-55).  Device side
(every step): the UNet forward plus one fused ``ldb_sampler_step`` kernel
that applies the update, re-imposes the known region and writes the next
network input.  Per-step inputs (timesteps, coefficients, noise) live in
device tables indexed by a device step counter, so one step is captured as
a CUDA graph and replayed for every step of the trajectory.
"""

from __future__ import annotations

from dataclasses import dataclass

import numpy as np
import torch

from . import ops

KIND_COMPOSE, KIND_DDIM, KIND_DPM = 0, 1, 2


def lesion_diffusion_timesteps(steps: int, total: int = 1000) -> tuple[int, ...]:
    """Uniform DDIM indices ``value + 1`` for ``value in range(0, total, total // steps)`` (_schedules.py:11-39)."""
    if not isinstance(steps, int) or isinstance(steps, bool) or steps < 1:
        raise ValueError("LesionDiffusion DDIM steps must be a positive integer")
    if not isinstance(total, int) or isinstance(total, bool) or total < steps:
        raise ValueError("LesionDiffusion DDIM schedule must contain at least as many timesteps")
    timesteps = tuple(v + 1 for v in range(0, total, total // steps))
    if timesteps[-1] >= total:
        raise ValueError(f"LesionDiffusion DDIM steps {steps} produce out-of-bounds indices for a "
                         f"{total}-timestep schedule; choose another diffusion_steps value")
    return timesteps


def dpm_solver_timesteps(steps: int, total: int = 1000) -> tuple[int, ...]:
    """Descending linspace schedule with nearest-even rounding (_schedules.py:42-55)."""
    if not isinstance(steps, int) or isinstance(steps, bool) or steps < 1:
        raise ValueError("DPM-Solver++ steps must be a positive integer")
    if not isinstance(total, int) or total < 2 or steps >= total:
        raise ValueError("DPM-Solver++ steps must be smaller than the training schedule")
    return tuple(int(v) for v in np.linspace(0, total - 1, steps + 1).round()[::-1][:-1])


def _host(alphas_cumprod) -> np.ndarray:
    if isinstance(alphas_cumprod, torch.Tensor):
        return alphas_cumprod.detach().cpu().numpy()
    return np.asarray(alphas_cumprod)


class DdimSampler:
    """Stochastic DDIM with eta (mlx_sampling.py:17-200) on the B200 path.

    ``coefficients`` is an f32 ``(steps, 5)`` table in execution order (largest
    timestep first): ``(alpha, previous, sigma, sqrt(1 - alpha), 0)``.
    """

    kind = KIND_DDIM

    def __init__(self, alphas_cumprod, steps: int, *, eta: float = 1.0):
        acp = _host(alphas_cumprod)
        dtype = acp.dtype.type
        self.timesteps = lesion_diffusion_timesteps(steps, int(acp.shape[0]))
        alphas = acp[np.array(self.timesteps)]
        previous = np.concatenate([acp[:1], alphas[:-1]])
        one = dtype(1)
        one_minus = (one - alphas).astype(dtype)
        sqrt_one_minus = np.sqrt(one_minus).astype(dtype).astype(np.float32)
        inverse_variance = (one / one_minus).astype(dtype).astype(np.float32)
        a32 = alphas.astype(np.float32)
        p32 = previous.astype(np.float32)
        f = np.float32
        sigmas = (f(eta) * np.sqrt(((f(1) - p32) * inverse_variance).astype(f) * (f(1) - (a32 / p32).astype(f)))).astype(f)
        self.alphas, self.previous, self.sigmas, self.sqrt_one_minus = a32, p32, sigmas, sqrt_one_minus
        table = np.stack([a32, p32, sigmas, sqrt_one_minus, np.zeros_like(a32)], axis=1)
        # a copy, not ascontiguousarray: a one-row reversed view counts as contiguous with a negative stride
        self.coefficients = table[::-1].copy()
        self.execution_timesteps = tuple(reversed(self.timesteps))

    @property
    def steps(self) -> int:
        return len(self.timesteps)

    def prepare(self, denoiser, conditioning_image: torch.Tensor, *, mask: torch.Tensor | None = None,
                generator: torch.Generator | None = None):
        """``sample()`` for a context-bound denoiser (``prepare_sample``)."""
        return prepare_sample(self, denoiser, conditioning_image, mask=mask, generator=generator)


class Dpmpp2mSampler:
    """Deterministic DPM-Solver++ 2M, Diffusers-0.42.1 midpoint (_dpm.py:21-153).

    ``coefficients`` is f32 ``(steps, 5)``: ``(alpha, sigma, ratio, clean, history)``.
    """

    kind = KIND_DPM

    def __init__(self, alphas_cumprod, steps: int):
        acp = _host(alphas_cumprod)
        self.timesteps = dpm_solver_timesteps(steps, int(acp.shape[0]))
        f = np.float32
        abar = acp[np.array(self.timesteps)].astype(f)
        ratios = np.sqrt(((f(1) - abar) / abar).astype(f)).astype(f)
        alpha = (f(1) / np.sqrt((ratios ** 2 + f(1)).astype(f))).astype(f)
        sigma = (ratios * alpha).astype(f)
        log_snr = (np.log(alpha) - np.log(sigma)).astype(f)
        if not np.all(np.isfinite(log_snr)):
            raise ValueError("DPM-Solver++ needs finite sampled alphas strictly between zero and one")
        table = np.zeros((len(self.timesteps), 5), dtype=f)
        for i in range(len(self.timesteps)):
            if i == len(self.timesteps) - 1:
                ratio, clean, history = f(0), f(1), f(0)
            else:
                h = f(log_snr[i + 1] - log_snr[i])
                ratio = f(sigma[i + 1] / sigma[i])
                clean = f(-alpha[i + 1] * f(np.expm1(f(-h))))
                history = f(0) if i == 0 else f(f(f(0.5) * clean) * h / f(log_snr[i] - log_snr[i - 1]))
            table[i] = (alpha[i], sigma[i], ratio, clean, history)
        self.coefficients = table
        self.execution_timesteps = tuple(self.timesteps)

    @property
    def steps(self) -> int:
        return len(self.timesteps)

    def prepare(self, denoiser, conditioning_image: torch.Tensor, *, mask: torch.Tensor | None = None,
                generator: torch.Generator | None = None):
        """``sample()`` for a context-bound denoiser (``prepare_sample``)."""
        return prepare_sample(self, denoiser, conditioning_image, mask=mask, generator=generator)


def prepare_sample(sampler, denoiser, conditioning_image: torch.Tensor, *, mask: torch.Tensor | None = None,
                   generator: torch.Generator | None = None, graph: bool = True):
    """The reference's ``Sampler.prepare(denoiser, conditioning_image, mask=)``
    (mlx_sampling.py:138-200, _dpm.py:82-100) on the B200 step.

    ``denoiser`` is what ``LdmUnetB200.prepare_denoiser`` returns;
    ``conditioning_image`` is NCDHW (the known latent with a mask, the
    concatenated image without one) and ``mask`` ``(B, 1, D, H, W)``, as in the
    reference.  The returned ``sample()`` draws a fresh initial noise (and, for
    DDIM, one noise tensor per step) from ``generator`` on the device, runs the
    whole trajectory (one captured CUDA graph per step with ``graph``) and
    returns the NCDHW float32 sample, the known region re-imposed.  The draws
    come from torch's generator, not MLX's, so the noise itself differs from
    the reference's."""
    if not (hasattr(denoiser, "unet") and hasattr(denoiser, "cache")):
        raise TypeError("prepare takes the denoiser that LdmUnetB200.prepare_denoiser returns")
    if conditioning_image.ndim != 5:
        raise ValueError(f"conditioning_image must be NCDHW, got shape {tuple(conditioning_image.shape)}")
    dev = denoiser.unet.device
    image = conditioning_image.to(dev, torch.float32).permute(0, 2, 3, 4, 1).contiguous()
    m = None
    if mask is not None:
        b, _, d, h, w = conditioning_image.shape
        if tuple(mask.shape) != (b, 1, d, h, w):
            raise ValueError(f"mask must be {(b, 1, d, h, w)}, got {tuple(mask.shape)}")
        m = mask.to(dev, torch.float32)[:, 0].contiguous()
    prepared = PreparedSampler(sampler, denoiser.unet, denoiser.cache, image, m, graph=graph)

    def sample() -> torch.Tensor:
        s = prepared.state
        initial = torch.randn(tuple(s.x.shape), generator=generator, device=dev)
        step_noise = torch.randn(tuple(s.noise.shape), generator=generator, device=dev) \
            if sampler.kind == KIND_DDIM else None
        return prepared.run(initial, step_noise).permute(0, 4, 1, 2, 3).clone()

    sample.prepared = prepared
    return sample


@dataclass
class SamplerState:
    """Device buffers of one prepared trajectory (all NDHWC)."""

    x: torch.Tensor          # (B, D, H, W, C) f32 composed state
    prev: torch.Tensor       # DPM history
    net_in: torch.Tensor     # (B, D, H, W, C + extra) f16 view (channel stride padded to 8)
    noise: torch.Tensor      # (steps, B, D, H, W, C) f32
    coeff: torch.Tensor      # (steps, 5) f32
    timesteps: torch.Tensor  # (steps, B) int32
    step: torch.Tensor       # () int32 device step counter
    mask: torch.Tensor | None
    image: torch.Tensor


class PreparedSampler:
    """A sampler bound to a UNet, its context cache, the known latent and mask.

    ``run(initial_noise, step_noise)`` executes the whole trajectory on the
    device (replaying a captured CUDA graph of one step when ``graph=True``)
    and returns the final NDHWC f32 latent.  ``step_noise`` follows the
    reference's injection hooks (mlx_sampling.py:66-69): one tensor per step
    in execution order; DPM++ ignores it.
    """

    def __init__(self, sampler, unet, cache: dict, image: torch.Tensor, mask: torch.Tensor | None, *,
                 graph: bool = True):
        self.sampler = sampler
        self.unet = unet
        self.cache = cache
        self.graph_enabled = graph
        dev = unet.device
        b, d, h, w, ci = (int(s) for s in image.shape)
        # Inpainting (mask given): the state has the image's channels and the
        # network reads [x | mask]; generation (no mask, LMNet): a one-channel
        # state and [x | conditioning image] (mlx_sampling.py:105-110).
        c = ci if mask is not None else 1
        extra = 1 if mask is not None else ci
        steps = sampler.steps
        # The FP32 network (LMNet) takes its input as split hi / low planes.
        self.net_split = bool(getattr(unet, "exact", False))
        if self.net_split:
            net_in = torch.zeros((b, d, h, w, 2 * ((c + extra + 15) // 16 * 16)), dtype=torch.float16, device=dev)
            setattr(net_in, "_ldb_split_c", c + extra)
        else:
            width = (c + extra + 7) // 8 * 8
            net_in = torch.zeros((b, d, h, w, width), dtype=torch.float16, device=dev)[..., : c + extra]
        self.state = SamplerState(
            x=torch.zeros((b, d, h, w, c), dtype=torch.float32, device=dev),
            prev=torch.zeros((b, d, h, w, c), dtype=torch.float32, device=dev),
            net_in=net_in,
            noise=torch.zeros((steps, b, d, h, w, c), dtype=torch.float32, device=dev),
            coeff=torch.from_numpy(np.array(sampler.coefficients, dtype=np.float32)).to(dev),
            timesteps=torch.tensor([[t] * b for t in sampler.execution_timesteps], dtype=torch.int32, device=dev),
            step=torch.zeros((), dtype=torch.int32, device=dev),
            mask=None if mask is None else mask.to(dev, torch.float32).reshape(b, d, h, w).contiguous(),
            image=image.to(dev, torch.float32).contiguous(),
        )
        if unet.in_channels != c + extra:
            raise ValueError(f"UNet takes {unet.in_channels} channels, sampler provides {c + extra}")
        self._graph: torch.cuda.CUDAGraph | None = None
        self.eps: torch.Tensor | None = None

    def _step(self) -> None:
        s = self.state
        self.eps = self.unet.forward(s.net_in, s.timesteps, self.cache, step=s.step)
        ops.sampler_step(
            self.sampler.kind, s.x, eps=self.eps, prev=s.prev, noise=s.noise,
            noise_step_stride=int(s.noise[0].numel()), mask=s.mask, image=s.image, net_in=s.net_in,
            coeff=s.coeff, step=s.step, net_split=self.net_split,
        )
        ops.step_advance(s.step)

    def begin(self, initial_noise: torch.Tensor, step_noise: torch.Tensor | None = None) -> None:
        """Load the initial state and noise, reset the step counter, compose the first input."""
        s = self.state
        s.x.copy_(initial_noise.to(s.x.device, torch.float32))
        s.prev.copy_(s.x)
        if step_noise is not None and self.sampler.kind == KIND_DDIM:
            s.noise.copy_(step_noise.to(s.noise.device, torch.float32))
        s.step.zero_()
        ops.sampler_step(KIND_COMPOSE, s.x, mask=s.mask, image=s.image, net_in=s.net_in, net_split=self.net_split)

    def capture(self) -> None:
        """Capture one denoise step as a CUDA graph (after one eager warm-up step)."""
        s = self.state
        saved = (s.x.clone(), s.prev.clone(), s.net_in.clone(), s.step.clone())
        self._step()  # warm-up: first-use setup happens outside the capture
        torch.cuda.synchronize()
        graph = torch.cuda.CUDAGraph()
        with torch.cuda.graph(graph):
            self._step()
        s.x.copy_(saved[0])
        s.prev.copy_(saved[1])
        s.net_in.copy_(saved[2])
        s.step.copy_(saved[3])
        self._graph = graph

    def step(self) -> None:
        """Advance one step (graph replay when captured)."""
        if self._graph is not None:
            self._graph.replay()
        else:
            self._step()

    def run(self, initial_noise: torch.Tensor, step_noise: torch.Tensor | None = None) -> torch.Tensor:
        self.begin(initial_noise, step_noise)
        if self.graph_enabled and self._graph is None:
            self.capture()
        for _ in range(self.sampler.steps):
            self.step()
        return self.state.x


class HostStreamedSteps:
    """Steps a prepared sampler with host I/O every step: step i's noise is
    copied in from pinned host memory and its updated latent copied out to
    pinned host memory, both on a copy stream, so the copy-in of step i + 1
    and the copy-out of step i - 1 run while step i computes.

    Step i's noise goes to noise slot i mod steps (the slot the sampler reads
    at step i of a trajectory that restarts every ``steps`` steps); a slot is
    refilled only after the step that last read it has run.  The latent is
    first copied into one of two device staging buffers (a device-to-device
    copy on the compute stream) so that the next step can update it while
    the host copy is in flight.  ``finish()`` makes the compute stream wait
    for every copy; call it before ``PreparedSampler.begin`` with step noise,
    which rewrites the noise slots.
    """

    def __init__(self, prepared: PreparedSampler, step=None):
        self.prepared = prepared
        self._run_step = step if step is not None else prepared.step  # e.g. a captured graph's replay
        s = prepared.state
        self.device = s.x.device
        self.compute = torch.cuda.current_stream(self.device)
        self.copy = torch.cuda.Stream(self.device)
        self.stage = [torch.empty_like(s.x), torch.empty_like(s.x)]
        self._in_done: dict[int, torch.cuda.Event] = {}
        self._step_done: dict[int, torch.cuda.Event] = {}
        self._out_done: list[torch.cuda.Event | None] = [None, None]
        self._count = 0

    def _copy_in(self, i: int, host_noise: torch.Tensor) -> None:
        steps = self.prepared.sampler.steps
        last_reader = self._step_done.pop(i - steps, None)  # the step that last read this slot
        with torch.cuda.stream(self.copy):
            if last_reader is not None:
                self.copy.wait_event(last_reader)
            self.prepared.state.noise[i % steps].copy_(host_noise, non_blocking=True)
            ev = torch.cuda.Event()
            ev.record(self.copy)
        self._in_done[i] = ev

    def start(self, host_noise: torch.Tensor) -> None:
        """Begin the copy-in of the first step's noise (the sampler at step 0),
        after all work already queued on the compute stream."""
        self._count = 0
        self._step_done.clear()
        self.copy.wait_stream(self.compute)
        self._copy_in(0, host_noise)

    def step(self, next_host_noise: torch.Tensor | None, host_out: torch.Tensor) -> None:
        """Run the next step (its noise copy already started), start the copy-in
        of the following step's noise when given, and the copy-out of this
        step's latent into ``host_out``."""
        i = self._count
        s = self.prepared.state
        self.compute.wait_event(self._in_done.pop(i))
        self._run_step()
        done = torch.cuda.Event()
        done.record(self.compute)
        self._step_done[i] = done
        if next_host_noise is not None:
            self._copy_in(i + 1, next_host_noise)
        buf = i & 1
        if self._out_done[buf] is not None:
            self.compute.wait_event(self._out_done[buf])  # the copy-out two steps back has read the buffer
        self.stage[buf].copy_(s.x)
        ready = torch.cuda.Event()
        ready.record(self.compute)
        with torch.cuda.stream(self.copy):
            self.copy.wait_event(ready)
            host_out.copy_(self.stage[buf], non_blocking=True)
            out_done = torch.cuda.Event()
            out_done.record(self.copy)
        self._out_done[buf] = out_done
        self._count = i + 1

    def finish(self) -> None:
        """Make the compute stream wait for every copy issued so far."""
        for ev in self._out_done:
            if ev is not None:
                self.compute.wait_event(ev)
        for ev in self._in_done.values():
            self.compute.wait_event(ev)
        self._in_done.clear()
