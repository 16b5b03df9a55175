"""CPU restatement of the reference samplers (test only): uniform DDIM with
eta and injected noise (mlx_sampling.py:17-136) and the Diffusers-0.42.1
midpoint DPM-Solver++ 2M (_dpm.py:21-153), plus their timestep schedules
(_schedules.py:11-55).  Arrays are NumPy; each op is rounded to the dtype the
reference computes it in.
"""

from __future__ import annotations

import numpy as np


def ddim_timesteps(steps: int, total: int = 1000) -> tuple[int, ...]:
    """``value + 1`` for value in ``range(0, total, total // steps)`` (_schedules.py:11-39)."""
    if not isinstance(steps, int) or isinstance(steps, bool) or steps < 1:
        raise ValueError("DDIM steps must be a positive integer")
    if not isinstance(total, int) or total < steps:
        raise ValueError("DDIM schedule must contain at least as many timesteps")
    ts = tuple(v + 1 for v in range(0, total, total // steps))
    if ts[-1] >= total:
        raise ValueError(f"DDIM steps {steps} produce out-of-bounds indices for a {total}-step schedule")
    return ts


def dpm_timesteps(steps: int, total: int = 1000) -> tuple[int, ...]:
    """Descending linspace with nearest-even rounding (_schedules.py:42-55)."""
    if not isinstance(steps, int) or isinstance(steps, bool) or steps < 1:
        raise ValueError("DPM-Solver++ steps must be a positive integer")
    if total < 2 or steps >= total:
        raise ValueError("DPM-Solver++ steps must be smaller than the training schedule")
    return tuple(int(v) for v in np.linspace(0, total - 1, steps + 1).round()[::-1][:-1])


def ddim_coefficients(alphas_cumprod: np.ndarray, steps: int, eta: float = 1.0) -> dict[str, np.ndarray]:
    """Per-step DDIM coefficients (mlx_sampling.py:27-60).

    Selected alphas keep the checkpoint dtype (f16 for LINet): ``1 - a``, its
    square root and its reciprocal are evaluated in that dtype before FP32
    promotion; the sigma product is FP32.
    """
    dtype = alphas_cumprod.dtype
    ts = ddim_timesteps(steps, int(alphas_cumprod.shape[0]))
    alphas = alphas_cumprod[np.array(ts)]
    previous = np.concatenate([alphas_cumprod[:1], alphas[:-1]])
    one = np.asarray(1, dtype)
    one_minus = (one - alphas).astype(dtype)
    sqrt_one_minus = np.sqrt(one_minus).astype(dtype).astype(np.float32)
    inverse_variance = (one / one_minus).astype(dtype).astype(np.float32)
    a32 = alphas.astype(np.float32)
    p32 = previous.astype(np.float32)
    sigmas = (np.float32(eta) * np.sqrt(
        ((np.float32(1) - p32) * inverse_variance).astype(np.float32)
        * (np.float32(1) - (a32 / p32).astype(np.float32))
    )).astype(np.float32)
    return {
        "timesteps": np.array(ts, dtype=np.int64),
        "alphas": a32,
        "previous": p32,
        "sqrt_one_minus": sqrt_one_minus,
        "sigmas": sigmas,
    }


def ddim_update(x, eps, alpha, previous, sigma, sqrt_one_minus, noise):
    """One DDIM update in FP32 (mlx_sampling.py:128-132)."""
    f = np.float32
    predicted = ((x - f(sqrt_one_minus) * eps).astype(f) / np.sqrt(f(alpha))).astype(f)
    direction = (np.sqrt(f(1) - f(previous) - f(sigma) ** 2).astype(f) * eps).astype(f)
    return (np.sqrt(f(previous)) * predicted + direction + f(sigma) * noise).astype(f)


def ddim_sample(denoiser, condition, image, coeffs, *, initial_noise, step_noise, mask=None):
    """Full DDIM trajectory with injected noise (mlx_sampling.py:105-136)."""
    x = initial_noise.astype(np.float32)
    n = len(coeffs["timesteps"])
    for iteration, index in enumerate(reversed(range(n))):
        timestep = np.full((x.shape[0],), coeffs["timesteps"][index], dtype=np.int32)
        if mask is not None:
            x = (x * mask + (np.float32(1) - mask) * image).astype(np.float32)
            net_in = np.concatenate([x, mask.astype(np.float32)], axis=1)
        else:
            net_in = np.concatenate([x, image], axis=1)
        eps = np.asarray(denoiser(net_in, timestep, condition))
        if mask is not None:
            eps = eps[:, : image.shape[1]]
        eps = eps.astype(np.float32)
        x = ddim_update(x, eps, coeffs["alphas"][index], coeffs["previous"][index], coeffs["sigmas"][index],
                        coeffs["sqrt_one_minus"][index], step_noise[iteration])
    if mask is not None:
        x = (x * mask + (np.float32(1) - mask) * image).astype(np.float32)
    return x


def dpm_coefficients(alphas_cumprod: np.ndarray, steps: int) -> tuple[tuple[int, ...], np.ndarray]:
    """Midpoint 2M coefficients ``(alpha, sigma, ratio, clean, history)`` per step (_dpm.py:30-62)."""
    ts = dpm_timesteps(steps, int(alphas_cumprod.shape[0]))
    f = np.float32
    abar = alphas_cumprod[np.array(ts)].astype(f)
    ratios = np.sqrt(((f(1) - abar) / abar).astype(f)).astype(f)
    alpha = (f(1) / np.sqrt((ratios ** 2 + f(1)).astype(f))).astype(f)
    sigma = (ratios * alpha).astype(f)
    log_snr = (np.log(alpha) - np.log(sigma)).astype(f)
    if not np.all(np.isfinite(log_snr)):
        raise ValueError("DPM-Solver++ needs finite sampled alphas strictly between zero and one")
    coeffs = np.zeros((len(ts), 5), dtype=f)
    for i in range(len(ts)):
        if i == len(ts) - 1:
            ratio, clean, history = f(0), f(1), f(0)
        else:
            h = f(log_snr[i + 1] - log_snr[i])
            ratio = f(sigma[i + 1] / sigma[i])
            clean = f(-alpha[i + 1] * f(np.expm1(f(-h))))
            history = f(0) if i == 0 else f(f(f(0.5) * clean) * h / f(log_snr[i] - log_snr[i - 1]))
        coeffs[i] = (alpha[i], sigma[i], ratio, clean, history)
    return ts, coeffs


def dpm_update(x, previous, eps, coeff):
    """One 2M step: returns (updated, predicted) (_dpm.py:129-133)."""
    f = np.float32
    predicted = ((x - coeff[1] * eps).astype(f) / coeff[0]).astype(f)
    updated = (coeff[2] * x + coeff[3] * predicted + coeff[4] * (predicted - previous)).astype(f)
    return updated, predicted


def dpm_sample(denoiser, image, ts, coeffs, *, initial_noise, mask=None, observer=None):
    """Full DPM++-2M trajectory (_dpm.py:102-153)."""
    x = initial_noise.astype(np.float32)
    previous = x
    for i, t in enumerate(ts):
        timestep = np.full((x.shape[0],), t, dtype=np.int32)
        if mask is not None:
            x = (x * mask + (np.float32(1) - mask) * image).astype(np.float32)
            net_in = np.concatenate([x, mask.astype(np.float32)], axis=1)
        else:
            net_in = np.concatenate([x, image], axis=1)
        if observer is not None:
            observer(net_in)
        eps = np.asarray(denoiser(net_in, timestep))
        if mask is not None:
            eps = eps[:, : image.shape[1]]
        x, previous = dpm_update(x, previous, eps.astype(np.float32), coeffs[i])
    if mask is not None:
        x = (x * mask + (np.float32(1) - mask) * image).astype(np.float32)
    return x
