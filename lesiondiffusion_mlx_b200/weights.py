"""The reference's weight bundle: one ``model.safetensors`` whose tensor names
carry a stage prefix (``linet.``, ``vq.``, ``lmnet.``, ``linet_text.``, ...),
read without the ``safetensors`` package, and loaders that build the B200
networks from it.

``load_stage`` mirrors the reference's (lesiondiffusion_mlx/medmlx.py:
1585-1602): the ``<stage>.`` prefix is removed, ``prefixes`` keeps only the
named components of the stage, and every array is cast to ``dtype``.

The safetensors layout: an 8-byte little-endian header length, a JSON header
``{name: {"dtype", "shape", "data_offsets": [begin, end]}, "__metadata__": {...}}``
and the raw little-endian tensor bytes, offsets relative to the end of the
header.
"""

from __future__ import annotations

import json
import struct
from pathlib import Path

import numpy as np
import torch

_NP = {
    "F64": np.float64, "F32": np.float32, "F16": np.float16, "I64": np.int64, "I32": np.int32,
    "I16": np.int16, "I8": np.int8, "U8": np.uint8, "BOOL": np.bool_,
}
_CODE = {np.dtype(v): k for k, v in _NP.items()}


def read_safetensors(path: str | Path) -> dict[str, np.ndarray]:
    """All tensors of a safetensors file as NumPy arrays (bfloat16 widened to float32)."""
    data = Path(path).read_bytes()
    if len(data) < 8:
        raise ValueError(f"{path}: not a safetensors file")
    (n,) = struct.unpack("<Q", data[:8])
    if 8 + n > len(data):
        raise ValueError(f"{path}: header length {n} exceeds the file")
    header = json.loads(data[8: 8 + n].decode("utf-8"))
    body = memoryview(data)[8 + n:]
    out: dict[str, np.ndarray] = {}
    for name, info in header.items():
        if name == "__metadata__":
            continue
        begin, end = (int(v) for v in info["data_offsets"])
        shape = tuple(int(s) for s in info["shape"])
        if not 0 <= begin <= end <= len(body):
            raise ValueError(f"{path}: {name} data offsets [{begin}, {end}) lie outside the {len(body)}-byte body")
        if any(s < 0 for s in shape):
            raise ValueError(f"{path}: {name} has a negative extent in shape {shape}")
        itemsize = 2 if info["dtype"] == "BF16" else (np.dtype(_NP[info["dtype"]]).itemsize if info["dtype"] in _NP
                                                        else 0)
        count = int(np.prod(shape)) if shape else 1
        if itemsize and end - begin != count * itemsize:
            raise ValueError(f"{path}: {name} holds {end - begin} bytes, shape {shape} of {info['dtype']} needs "
                             f"{count * itemsize}")
        raw = body[begin:end]
        if info["dtype"] == "BF16":
            bits = np.frombuffer(raw, dtype="<u2").astype(np.uint32) << 16
            arr = bits.view(np.float32)
        elif info["dtype"] in _NP:
            arr = np.frombuffer(raw, dtype=np.dtype(_NP[info["dtype"]]).newbyteorder("<"))
        else:
            raise ValueError(f"{path}: unsupported dtype {info['dtype']} for {name}")
        out[name] = arr.reshape(shape).copy()
    return out


def write_safetensors(path: str | Path, tensors: dict[str, np.ndarray], metadata: dict[str, str] | None = None) -> None:
    """Write NumPy arrays as a safetensors file (little-endian, 8-byte aligned header)."""
    header: dict[str, object] = {}
    chunks, offset = [], 0
    for name, arr in tensors.items():
        a = np.ascontiguousarray(arr)
        if a.dtype not in _CODE:
            raise ValueError(f"unsupported dtype {a.dtype} for {name}")
        b = a.astype(a.dtype.newbyteorder("<"), copy=False).tobytes()
        header[name] = {"dtype": _CODE[a.dtype], "shape": list(a.shape), "data_offsets": [offset, offset + len(b)]}
        chunks.append(b)
        offset += len(b)
    if metadata:
        header["__metadata__"] = dict(metadata)
    text = json.dumps(header, separators=(",", ":")).encode("utf-8")
    text += b" " * (-len(text) % 8)
    with open(path, "wb") as f:
        f.write(struct.pack("<Q", len(text)))
        f.write(text)
        for b in chunks:
            f.write(b)


def _bundle(path: str | Path) -> Path:
    p = Path(path)
    return p / "model.safetensors" if p.is_dir() else p


def load_stage(path: str | Path, name: str, *, dtype: torch.dtype = torch.float16,
               prefixes: tuple[str, ...] | None = None) -> dict[str, torch.Tensor]:
    """One stage of the bundle (a directory holding ``model.safetensors``, or the file).

    Removes the ``<stage>.`` prefix, keeps the names starting with one of
    ``prefixes`` when given, and casts to ``dtype``."""
    tensors = read_safetensors(_bundle(path))
    prefix = name + "."
    out = {}
    for key, arr in tensors.items():
        if not key.startswith(prefix):
            continue
        short = key[len(prefix):]
        if prefixes is not None and not short.startswith(prefixes):
            continue
        out[short] = torch.from_numpy(arr).to(dtype)
    if not out:
        raise KeyError(f"{_bundle(path)} has no tensors for stage {name!r}")
    return out


def load_linet(path: str | Path, config, *, device: torch.device | str = "cuda"):
    """The LINet denoiser of the bundle on B200 kernels and its ``alphas_cumprod``."""
    from .networks import LdmUnetB200

    w = load_stage(path, "linet", dtype=torch.float16)
    alphas = w.pop("alphas_cumprod", None)
    return LdmUnetB200(w, config, device=device), (None if alphas is None else alphas.numpy())


def load_vq_decoder(path: str | Path, *, device: torch.device | str = "cuda", scaled: bool = False,
                    groups: int = 16):
    """The VQ quantizer + decoder of the bundle (``quantize.``, ``post_quant_conv.``, ``decoder.``)."""
    from .networks import VqDecoderB200

    w = load_stage(path, "vq", dtype=torch.float16, prefixes=("quantize.", "post_quant_conv.", "decoder."))
    return VqDecoderB200(w, device=device, scaled=scaled, groups=groups)


def load_vq_encoder(path: str | Path, *, device: torch.device | str = "cuda", groups: int = 16):
    """The VQ encoder of the bundle (``encoder.``, ``quant_conv.``), as the reference loads it (medmlx.py:1287)."""
    from .networks import VqEncoderB200

    w = load_stage(path, "vq", dtype=torch.float16, prefixes=("encoder.", "quant_conv."))
    return VqEncoderB200(w, device=device, groups=groups)
