"""Extract the reference's golden vectors into ``tests/golden/reference_fixtures.npz``.

The reference (lesiondiffusion-mlx 0.3.0) commits Torch-CPU recordings of
its pinned upstream model under ``tests/fixtures/darwin-arm64/``.  This
script copies the arrays the oracle pins against (UNet, VQ, DDIM, DPM++-2M,
activation and CT-map recordings) into one small archive so that tests never
read the reference checkout at run time.  Keys are ``<fixture>/<array>``.

Run from the repository root with the reference checkout available:

    python tests/golden/make_golden.py /path/to/lesiondiffusion-mlx
"""

from __future__ import annotations

import json
import sys
from pathlib import Path

import numpy as np

FIXTURES = {
    "unet_mask": None,
    "unet_inpainting": None,
    "vq_float16": None,
    "vq_float32": None,
    "ddim_mask": None,
    "ddim_inpainting": None,
    "dpmpp_2m": None,
    "unet_activations": None,
    "pipeline": ("ct", "normalized", "ct_output", "inverse_output"),
}
METADATA = ("schema_version", "upstream_revision", "text_revision", "backend", "recording_platform",
            "torch_version", "numpy_version", "transformers_version")


def main(reference_root: str) -> None:
    src = Path(reference_root) / "tests" / "fixtures" / "darwin-arm64"
    out: dict[str, np.ndarray] = {}
    for name, keys in FIXTURES.items():
        with np.load(src / f"{name}.npz", allow_pickle=False) as fixture:
            for key in fixture.files if keys is None else keys:
                if key in METADATA:
                    continue
                out[f"{name}/{key}"] = fixture[key]
    meta = json.loads((src / "dpmpp_2m.json").read_text())
    out["dpmpp_2m/json"] = np.array(json.dumps(meta))
    target = Path(__file__).resolve().parent / "reference_fixtures.npz"
    np.savez_compressed(target, **out)
    print(f"wrote {len(out)} arrays to {target}")


if __name__ == "__main__":
    if len(sys.argv) != 2:
        sys.exit("usage: python tests/golden/make_golden.py /path/to/lesiondiffusion-mlx")
    main(sys.argv[1])
