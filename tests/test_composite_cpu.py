"""Pins the compositing oracle (oracle/composite.py) on the CPU: the
reference's analytic lesion-mode test (tests/test_medmlx.py:78-141) on a
synthetic CT, and hand-computed box-mode weights."""

from __future__ import annotations

import math

import numpy as np
import pytest

from oracle import composite


@pytest.mark.parametrize("reach", [3, 33])
def test_oracle_lesion_change_analytic(reach):
    shift = reach - 3
    shape = tuple(size + 2 * shift for size in (24, 20, 18))
    original = (np.random.default_rng(7).normal(size=shape) * 300.0).astype(np.float32)
    original[8 + shift, 6 + shift, 5 + shift] = 1350.0
    lesion = np.zeros(shape, dtype=bool)
    lesion[10 + shift: 13 + shift, 8 + shift: 11 + shift, 7 + shift: 10 + shift] = True
    reconstruction = np.clip(original, -1000, 1000) - 9.0
    generated = reconstruction + np.float32(0.25)
    shell = np.zeros(shape, dtype=bool)
    shell[9 + shift: 14 + shift, 7 + shift: 12 + shift, 6 + shift: 11 + shift] = True
    generated[shell] -= 2.25
    generated[lesion] -= 28.0
    out, count, offset = composite.apply_lesion_change(original, generated, reconstruction, lesion, reach)
    reached = np.zeros(shape, dtype=bool)
    reached[7: 16 + 2 * shift, 5: 14 + 2 * shift, 4: 13 + 2 * shift] = True
    np.testing.assert_array_equal(out[~reached], original[~reached])
    np.testing.assert_array_equal(out[reached & ~shell], original[reached & ~shell] + np.float32(0.25))
    np.testing.assert_allclose(out[lesion], original[lesion] - 30.0, atol=1e-4)
    assert offset == pytest.approx(-9.0)
    assert count == int(reached.sum())


def test_oracle_box_weights_by_hand():
    shape = (9, 9, 9)
    original = np.zeros(shape, np.float32)
    generated = np.full(shape, 100.0, np.float32)
    bbox = (slice(4, 5), slice(4, 5), slice(4, 5))
    out, weighted = composite.localize_output(original, generated, bbox, (1.0, 2.0, 1.0), margin_mm=3.0)
    assert out[4, 4, 4] == 100.0
    # one voxel along axis 0: d = 1 mm; along axis 1: d = 2 mm; diagonal (1, 0, 1): d = sqrt(2)
    for idx, d in (((5, 4, 4), 1.0), ((4, 5, 4), 2.0), ((5, 4, 5), math.sqrt(2.0))):
        w = 0.5 * (1.0 + math.cos(math.pi * d / 3.0))
        assert out[idx] == np.float32(100.0 * w)
    assert out[4, 6, 4] == 0.0  # d = 4 mm > margin
    assert out[7, 4, 4] == 0.0  # d = 3 mm: not < margin
    # voxels with d < 3 mm: |i| <= 2 along axes 0/2 with i0^2 + (2 i1)^2 + i2^2 < 9
    want = sum(1 for a in range(-2, 3) for b in range(-1, 2) for c in range(-2, 3) if a * a + 4 * b * b + c * c < 9)
    assert weighted == want
