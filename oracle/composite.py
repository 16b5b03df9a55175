"""CPU restatement of the output-region compositing (TEST INFRASTRUCTURE ONLY,
see the package docstring): ``localize_output`` and ``apply_lesion_change``
of lesiondiffusion_mlx/medmlx.py:2531-2690, in NumPy (FP64 weights and
blend, f32 results, SciPy's cubic maximum filter as the reference uses).
The reference's own test of the lesion mode (tests/test_medmlx.py:78-141)
reads a CT that is not distributed; its analytic expectations are mirrored
on a synthetic volume in ``tests/test_composite_gpu.py``.
"""

from __future__ import annotations

import numpy as np


def localize_output(original: np.ndarray, generated: np.ndarray, bbox: tuple[slice, slice, slice],
                    spacing_mm: tuple[float, float, float], margin_mm: float = 6.0) -> tuple[np.ndarray, int]:
    """(localized f32 volume, weighted voxel count), medmlx.py:2531-2614."""
    spacing = np.asarray(spacing_mm, dtype=np.float64)
    radius = np.ceil(margin_mm / spacing).astype(int)
    start = np.array([s.start for s in bbox])
    stop = np.array([s.stop for s in bbox])
    low = np.maximum(0, start - radius)
    high = np.minimum(np.array(original.shape[:3]), stop + radius)
    # squared distance in mm from the box, accumulated over the axes in order
    sq = np.zeros(tuple(high - low), dtype=np.float64)
    for axis in range(3):
        idx = np.arange(low[axis], high[axis])
        off = np.where(idx < start[axis], start[axis] - idx, np.where(idx >= stop[axis], idx - (stop[axis] - 1), 0))
        mm = off * spacing[axis]
        view = [1, 1, 1]
        view[axis] = mm.size
        sq = sq + (mm ** 2).reshape(view)
    dist = np.sqrt(sq)
    near = dist < margin_mm
    weight = np.zeros_like(dist)
    weight[near] = 0.5 * (1.0 + np.cos(np.pi * dist[near] / margin_mm))
    out = np.asarray(original, dtype=np.float32).copy()
    region = tuple(slice(int(a), int(b)) for a, b in zip(low, high))
    win = out[region]
    raw = np.asarray(generated[region], dtype=np.float32)
    blend = (weight > 0) & (weight < 1)
    win[blend] = (raw[blend] * weight[blend] + win[blend] * (1.0 - weight[blend])).astype(np.float32)
    out[bbox] = generated[bbox]
    return out, int(np.count_nonzero(near))


def apply_lesion_change(original: np.ndarray, generated: np.ndarray, reconstruction: np.ndarray, lesion: np.ndarray,
                        reach_voxels: int = 33) -> tuple[np.ndarray, int, float | None]:
    """(localized f32 volume, reached voxel count, offset HU or None),
    medmlx.py:2617-2690."""
    from scipy.ndimage import maximum_filter

    pts = np.argwhere(lesion)
    if pts.size == 0:
        raise ValueError("empty lesion")
    low = np.maximum(pts.min(axis=0) - reach_voxels, 0)
    high = np.minimum(pts.max(axis=0) + reach_voxels + 1, np.array(original.shape[:3]))
    region = tuple(slice(int(a), int(b)) for a, b in zip(low, high))
    reached = maximum_filter(lesion[region].astype(np.uint8), size=2 * reach_voxels + 1) > 0
    change = np.asarray(generated[region], dtype=np.float32) - np.asarray(reconstruction[region], dtype=np.float32)
    out = np.asarray(original, dtype=np.float32).copy()
    win = out[region]
    win[reached] += change[reached]
    inp = np.asarray(original[region], dtype=np.float64)
    around = reached & ~lesion[region] & (np.abs(inp) < 1000)
    offset = np.asarray(reconstruction[region], dtype=np.float64)[around] - inp[around]
    return out, int(np.count_nonzero(reached)), (round(float(offset.mean()), 3) if offset.size else None)
