"""ctypes binding of ``libldb200.so``, the C ABI declared in ``include/ldb200.h``.

The library is the only compute path: there is no Python or PyTorch fallback.
Loading fails loudly when the shared object has not been built, and every
call that returns a negative status raises ``LdbError`` carrying the
library's own message.
"""

from __future__ import annotations

import ctypes
import threading
from pathlib import Path

LIBRARY_PATH = Path(__file__).resolve().parent / "libldb200.so"

LDB_OK = 0
LDB_F16, LDB_F32, LDB_BF16 = 0, 1, 2
LDB_CONV_3X3X3, LDB_CONV_3X3X3_S2, LDB_CONV_UP2, LDB_CONV_1X1, LDB_CONV_3X3X3_S2_PAD01 = 0, 1, 2, 3, 4
LDB_ACT_NONE, LDB_ACT_GELU = 0, 1


class LdbError(RuntimeError):
    """A C-ABI call returned a negative status."""

    def __init__(self, name: str, code: int, message: str):
        super().__init__(f"{name} failed ({code}): {message}")
        self.code = code


class ConvDesc(ctypes.Structure):
    """Mirror of ``ldb_conv_desc``; ``struct_size`` is filled in on construction."""

    _fields_ = [
        ("struct_size", ctypes.c_int),
        ("batch", ctypes.c_int),
        ("depth", ctypes.c_int),
        ("height", ctypes.c_int),
        ("width", ctypes.c_int),
        ("in_channels", ctypes.c_int),
        ("x_ld", ctypes.c_int),
        ("out_channels", ctypes.c_int),
        ("out_ld", ctypes.c_int),
        ("res_ld", ctypes.c_int),
        ("mode", ctypes.c_int),
        ("exact", ctypes.c_int),
        ("out_dtype", ctypes.c_int),
        ("act", ctypes.c_int),
        ("output_scale", ctypes.c_float),
        ("depth_halo", ctypes.c_int),
        ("max_ctas", ctypes.c_int),
        ("clock", ctypes.c_void_p),
    ]

    def __init__(self, *args, **kwargs):
        super().__init__(*args, **kwargs)
        self.struct_size = ctypes.sizeof(ConvDesc)


_P = ctypes.c_void_p
_I = ctypes.c_int
_F = ctypes.c_float
_SZ = ctypes.c_size_t

# name -> (argtypes); every function returns int unless listed in _RESTYPES.
SIGNATURES: dict[str, list] = {
    "ldb_version": [],
    "ldb_launch_count": [],
    "ldb_last_error": [],
    "ldb_clear_async": [_P, _P, _SZ],
    "ldb_device_status": [ctypes.POINTER(ctypes.c_uint), _I],
    "ldb_conv3d_workspace_size": [ctypes.POINTER(ConvDesc), ctypes.POINTER(_SZ)],
    "ldb_conv3d_weight_rows": [ctypes.POINTER(ConvDesc), ctypes.POINTER(_I), ctypes.POINTER(_I)],
    "ldb_conv3d_fwd": [_P, ctypes.POINTER(ConvDesc), _P, _P, _P, _P, _P, _P, _P, _SZ],
    "ldb_conv3d_fwd_gn_stats": [_P, ctypes.POINTER(ConvDesc), _P, _P, _P, _P, _P, _P, _P, _P, _SZ],
    "ldb_group_norm_workspace_size": [_I, _I, _I, ctypes.POINTER(_SZ)],
    "ldb_group_norm_affine": [_P, _P, _I, _I, _P, _I, _I, _I, _I, _I, _I, _P, _P, _F, _P, _P, _SZ],
    "ldb_group_norm_affine_noalloc": [_P, _P, _I, _I, _P, _I, _I, _I, _I, _I, _I, _P, _P, _F, _P],
    "ldb_prepare_input": [_P, _P, _I, _I, _P, _I, _I, _I, _I, _I, _P, _I, _I, _P, _I],
    "ldb_group_norm_affine_from_stats": [_P, _P, _I, _P, _I, _I, _I, _I, _P, _P, _F, _P],
    "ldb_prepare_input_from_stats": [_P, _P, _I, _I, _P, _I, _I, _I, _I, _I, _I, _P, _P, _I, _P, _P, _F, _I, _I, _P, _I],
    "ldb_layer_norm_ex": [_P, _P, _I, _I, _P, _P, _F, _P, _I, _I, _I, _I],
    "ldb_layer_norm": [_P, _P, _I, _P, _P, _F, _P, _I, _I, _I],
    "ldb_flash_attention": [_P, _P, _I, _P, _P, _I, _P, _I, _I, _I, _I, _I, _I, _F, _I],
    "ldb_flash_attention_workspace_size": [_I, _I, _I, _I, _I, ctypes.POINTER(_SZ)],
    "ldb_flash_attention_f32_workspace_size": [_I, _I, _I, _I, _I, ctypes.POINTER(_SZ)],
    "ldb_flash_attention_f32": [_P, _P, _I, _P, _P, _I, _P, _I, _I, _I, _I, _I, _I, _F, _P, _SZ],
    "ldb_flash_attention_timed": [_P, _P, _I, _P, _P, _I, _P, _I, _I, _I, _I, _I, _I, _F, _I, _P, _SZ, _P],
    "ldb_flash_attention_ws": [_P, _P, _I, _P, _P, _I, _P, _I, _I, _I, _I, _I, _I, _F, _I, _P, _SZ],
    "ldb_step_advance": [_P, _P],
    "ldb_timestep_embedding": [_P, _P, _P, _I, _I, _I, _P, _I],
    "ldb_dense_small": [_P, _P, _I, _P, _P, _P, _I, _I, _I, _I, _I, _I, _I, _I],
    "ldb_sampler_step_ex": [_P, _I, _P, _P, _P, _I, _I, _P, ctypes.c_longlong, _P, _P, _I, _P, _I, _I, _I, _I, _I, _P, _P,
                            _I],
    "ldb_sampler_step": [_P, _I, _P, _P, _P, _I, _P, ctypes.c_longlong, _P, _P, _I, _P, _I, _I, _I, _I, _P, _P, _I],
    "ldb_vq_nearest4": [_P, _P, _I, ctypes.c_longlong, _P, _I, _I, _P, _P, _I],
    "ldb_resize_nearest": [_P, _P, _I, _I, _I, _I, _I, _I, _P, _I, _I, _I, _I],
    "ldb_localize_box": [_P, _P, _P, _P, _I, _I, _I, _P, _P, _P, ctypes.c_double, _P],
    "ldb_lesion_extent": [_P, _P, _I, _I, _I, _P],
    "ldb_apply_lesion_change": [_P, _P, _P, _P, _P, _P, _I, _I, _I, _I, _P, _SZ, _P],
    "ldb_hu_map": [_P, _P, _I, _I, ctypes.c_longlong, _P],
    "ldb_ct_normalize": [_P, _P, ctypes.c_longlong, _P, _I, _I],
}
_RESTYPES = {"ldb_last_error": ctypes.c_char_p, "ldb_launch_count": ctypes.c_ulonglong}

_lock = threading.Lock()
_lib: ctypes.CDLL | None = None


def library() -> ctypes.CDLL:
    """Load (once) and return the C library with typed signatures."""
    global _lib
    with _lock:
        if _lib is None:
            if not LIBRARY_PATH.exists():
                raise ImportError(
                    f"{LIBRARY_PATH} is missing: build it with "
                    "`python -m lesiondiffusion_mlx_b200.build` (there is no fallback path)"
                )
            lib = ctypes.CDLL(str(LIBRARY_PATH))
            for name, argtypes in SIGNATURES.items():
                fn = getattr(lib, name)
                fn.argtypes = argtypes
                fn.restype = _RESTYPES.get(name, ctypes.c_int)
            _lib = lib
        return _lib


def call(name: str, *args) -> int:
    """Invoke ``name`` and raise ``LdbError`` on a negative status."""
    lib = library()
    rc = getattr(lib, name)(*args)
    if rc < 0:
        raise LdbError(name, rc, lib.ldb_last_error().decode(errors="replace"))
    return rc


def launch_count() -> int:
    """Kernels launched (or captured) by the library so far in this process."""
    return int(library().ldb_launch_count())


def device_status(reset: bool = True) -> int:
    """Read (and by default clear) the current device's status word."""
    value = ctypes.c_uint(0)
    call("ldb_device_status", ctypes.byref(value), int(reset))
    return int(value.value)
