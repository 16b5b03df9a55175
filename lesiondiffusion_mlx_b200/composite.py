"""Output-region compositing on the GPU: the reference's ``localize_output``
(``output_region="box"``) and ``apply_lesion_change`` (``output_region=
"lesion"``), lesiondiffusion_mlx/medmlx.py:2531-2690, with the same names,
keyword arguments, results and errors.

Volumes are CUDA tensors (or arrays, copied to the current device) of shape
``(n0, n1, n2)`` in the reference's axis order; ``original`` is taken as
float32 (the reference's output is its float32 cast outside the composited
region).  Each function returns ``(localized float32 tensor, facts)``.
"""

from __future__ import annotations

import ctypes
import math

import numpy as np
import torch

from . import _lib

LOCALIZATION_MARGIN_MM = 6.0  # medmlx.py:82
DECODER_REACH_VOXELS = 33  # medmlx.py:90


class ModelExecutionError(RuntimeError):
    """Raised where the reference raises its ``ModelExecutionError``."""


def _volume(x, device: torch.device, dtype: torch.dtype = torch.float32) -> torch.Tensor:
    t = x if isinstance(x, torch.Tensor) else torch.from_numpy(np.ascontiguousarray(x))
    return t.to(device=device, dtype=dtype).contiguous()


def _device(*xs) -> torch.device:
    for x in xs:
        if isinstance(x, torch.Tensor) and x.is_cuda:
            return x.device
    return torch.device("cuda", torch.cuda.current_device())


def _stream(device: torch.device) -> int:
    return torch.cuda.current_stream(device).cuda_stream


def localize_output(*, original, generated, bbox: tuple[slice, slice, slice], spacing_mm: tuple[float, float, float],
                    margin_mm: float = LOCALIZATION_MARGIN_MM) -> tuple[torch.Tensor, dict[str, object]]:
    """Keep the generated CT inside ``bbox`` and feather it into the original
    over ``margin_mm`` (cosine weight of the Euclidean distance in mm)."""
    if tuple(original.shape) != tuple(generated.shape):
        raise ModelExecutionError("LesionDiffusion raw output shape does not match the original CT")
    device = _device(original, generated)
    orig = _volume(original, device)
    gen = _volume(generated, device)
    n = tuple(int(s) for s in orig.shape[:3])
    start = [int(s.start) for s in bbox]
    stop = [int(s.stop) for s in bbox]
    out = torch.empty_like(orig)
    weighted = torch.zeros(1, dtype=torch.int64, device=device)
    c_start = (ctypes.c_int * 3)(*start)
    c_stop = (ctypes.c_int * 3)(*stop)
    c_spacing = (ctypes.c_double * 3)(*(float(s) for s in spacing_mm))
    _lib.call("ldb_localize_box", _stream(device), orig.data_ptr(), gen.data_ptr(), out.data_ptr(), *n,
              ctypes.addressof(c_start), ctypes.addressof(c_stop), ctypes.addressof(c_spacing), float(margin_mm),
              weighted.data_ptr())
    radius = [math.ceil(margin_mm / float(s)) for s in spacing_mm]
    low = [max(0, a - r) for a, r in zip(start, radius)]
    high = [min(size, b + r) for size, b, r in zip(n, stop, radius)]
    return out, {
        "policy": "bbox_generated_cosine_feather_to_original_ct",
        "margin_mm": margin_mm,
        "blend_weight": "0.5 * (1 + cos(pi * distance_mm / margin_mm))",
        "distance_metric": "euclidean_voxel_center_distance_in_physical_mm",
        "bounding_box": {"start_voxel": start, "stop_voxel_exclusive": stop},
        "affected_region": {"start_voxel": low, "stop_voxel_exclusive": high,
                            "weighted_voxel_count": int(weighted.item())},
        "outside_affected_region": "original_ct_cast_float32",
    }


def apply_lesion_change(*, original, generated, reconstruction, lesion,
                        reach_voxels: int = DECODER_REACH_VOXELS) -> tuple[torch.Tensor, dict[str, object]]:
    """Add ``generated - reconstruction`` to the original within ``reach_voxels``
    of a lesion voxel along every axis; report the reconstruction offset."""
    if not tuple(original.shape) == tuple(generated.shape) == tuple(reconstruction.shape) == tuple(lesion.shape):
        raise ModelExecutionError("LesionDiffusion lesion change arrays differ in shape")
    device = _device(original, generated, reconstruction, lesion)
    orig = _volume(original, device)
    gen = _volume(generated, device)
    rec = _volume(reconstruction, device)
    les = _volume(lesion, device, torch.bool).view(torch.uint8)
    n = tuple(int(s) for s in orig.shape[:3])
    stream = _stream(device)
    extent = torch.empty(7, dtype=torch.int32, device=device)
    _lib.call("ldb_lesion_extent", stream, les.data_ptr(), *n, extent.data_ptr())
    ext = extent.cpu().tolist()
    if ext[0] == 0:
        raise ModelExecutionError("LesionDiffusion lesion change needs a non-empty lesion")
    out = torch.empty_like(orig)
    workspace = torch.empty(2 * orig.numel(), dtype=torch.uint8, device=device)
    stats = torch.empty(3, dtype=torch.float64, device=device)
    _lib.call("ldb_apply_lesion_change", stream, orig.data_ptr(), gen.data_ptr(), rec.data_ptr(), les.data_ptr(),
              out.data_ptr(), *n, int(reach_voxels), workspace.data_ptr(), workspace.numel(), stats.data_ptr())
    total, count, reached = stats.cpu().tolist()
    low = [max(ext[1 + a] - reach_voxels, 0) for a in range(3)]
    high = [min(ext[4 + a] + reach_voxels + 1, n[a]) for a in range(3)]
    return out, {
        "policy": "original_plus_generated_minus_input_reconstruction",
        "reach_voxels": reach_voxels,
        "reach_metric": "per_axis_voxel_distance_from_nearest_lesion_voxel",
        "changed_region": {"start_voxel": low, "stop_voxel_exclusive": high, "voxel_count": int(reached)},
        "input_reconstruction_offset_hu": round(total / count, 3) if count else None,
        "outside_changed_region": "original_ct_cast_float32",
    }
