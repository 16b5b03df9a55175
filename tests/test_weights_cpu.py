"""The stage-prefixed safetensors bundle (reference: medmlx.py:1585-1602) and the
standalone reader / writer, on CPU."""

from __future__ import annotations

import json
import struct

import numpy as np
import pytest
import torch

from lesiondiffusion_mlx_b200.weights import load_stage, read_safetensors, write_safetensors


def _bundle(tmp_path):
    rng = np.random.default_rng(0)
    tensors = {
        "linet.input_blocks.0.0.weight": rng.standard_normal((4, 2, 3, 3, 3)).astype(np.float32),
        "linet.alphas_cumprod": np.linspace(0.99, 0.01, 10).astype(np.float16),
        "vq.encoder.conv_in.weight": rng.standard_normal((2, 1, 3, 3, 3)).astype(np.float16),
        "vq.quant_conv.bias": np.arange(3, dtype=np.float32),
        "vq.decoder.conv_out.bias": np.ones(1, dtype=np.float32),
        "lmnet.steps": np.arange(5, dtype=np.int32),
    }
    (tmp_path / "model.safetensors").parent.mkdir(parents=True, exist_ok=True)
    write_safetensors(tmp_path / "model.safetensors", tensors, metadata={"format": "pt"})
    return tensors


def test_round_trip_keeps_names_shapes_dtypes_and_values(tmp_path):
    tensors = _bundle(tmp_path)
    back = read_safetensors(tmp_path / "model.safetensors")
    assert set(back) == set(tensors)
    for k, v in tensors.items():
        assert back[k].dtype == v.dtype and back[k].shape == v.shape
        assert np.array_equal(back[k], v)


def test_load_stage_strips_prefix_filters_components_and_casts(tmp_path):
    tensors = _bundle(tmp_path)
    linet = load_stage(tmp_path, "linet", dtype=torch.float16)
    assert set(linet) == {"input_blocks.0.0.weight", "alphas_cumprod"}
    assert all(t.dtype == torch.float16 for t in linet.values())
    np.testing.assert_array_equal(linet["input_blocks.0.0.weight"].numpy(),
                                  tensors["linet.input_blocks.0.0.weight"].astype(np.float16))
    enc = load_stage(tmp_path / "model.safetensors", "vq", dtype=torch.float32, prefixes=("encoder.", "quant_conv."))
    assert set(enc) == {"encoder.conv_in.weight", "quant_conv.bias"}
    assert enc["quant_conv.bias"].dtype == torch.float32
    with pytest.raises(KeyError):
        load_stage(tmp_path, "linet_text")


def test_bfloat16_tensors_widen_to_float32(tmp_path):
    values = np.array([1.0, -2.5, 3.140625, 65280.0], dtype=np.float32)  # exact in bfloat16
    bits = (values.view(np.uint32) >> 16).astype("<u2")
    header = json.dumps({"x": {"dtype": "BF16", "shape": [2, 2], "data_offsets": [0, 8]}}).encode()
    header += b" " * (-len(header) % 8)
    path = tmp_path / "bf16.safetensors"
    path.write_bytes(struct.pack("<Q", len(header)) + header + bits.tobytes())
    x = read_safetensors(path)["x"]
    assert x.dtype == np.float32 and x.shape == (2, 2)
    np.testing.assert_array_equal(x.ravel(), values)


def test_truncated_file_is_rejected(tmp_path):
    _bundle(tmp_path)
    data = (tmp_path / "model.safetensors").read_bytes()
    (tmp_path / "bad.safetensors").write_bytes(data[:-10])
    with pytest.raises(ValueError):
        read_safetensors(tmp_path / "bad.safetensors")


@pytest.mark.parametrize("offsets,shape,message", [
    ([-8, 8], [2], "outside"),          # a negative start would slice from the end of the body
    ([8, 4], [1], "outside"),           # end before begin
    ([0, 24], [2], "outside"),          # past the 16-byte body
    ([0, 12], [2], "holds 12 bytes"),   # not the shape's byte count
    ([0, 8], [-2], "negative extent"),
])
def test_tensor_records_outside_or_inconsistent_with_the_body_are_rejected(tmp_path, offsets, shape, message):
    """Each tensor's data offsets must lie inside the body and span exactly its
    shape's bytes; anything else is a ValueError, never a silent misread."""
    header = json.dumps({"x": {"dtype": "F32", "shape": shape, "data_offsets": offsets}}).encode()
    header += b" " * (-len(header) % 8)
    path = tmp_path / "bad.safetensors"
    path.write_bytes(struct.pack("<Q", len(header)) + header + np.arange(4, dtype="<f4").tobytes())
    with pytest.raises(ValueError, match=message):
        read_safetensors(path)
