"""Output-region compositing on the GPU (``output_region="box"`` and
``"lesion"``, lesiondiffusion_mlx/medmlx.py:2531-2690) against the oracle
restatement, plus the reference's own analytic lesion-mode test
(tests/test_medmlx.py:78-141) on a synthetic CT."""

from __future__ import annotations

import numpy as np
import pytest
import torch

from oracle import composite as oracle_composite

pytestmark = pytest.mark.gpu


def _ct(shape, seed):
    rng = np.random.default_rng(seed)
    return (rng.normal(size=shape) * 300.0).astype(np.float32)


@pytest.mark.parametrize("shape,bbox,spacing,margin", [
    ((40, 36, 30), (slice(10, 20), slice(8, 15), slice(12, 18)), (0.8, 0.7, 2.5), 6.0),
    ((33, 29, 17), (slice(0, 5), slice(20, 29), slice(3, 16)), (1.0, 1.0, 1.0), 6.0),  # box at the edges
    ((24, 24, 24), (slice(11, 12), slice(11, 12), slice(11, 12)), (1.5, 0.9, 1.2), 4.3),  # one-voxel box
])
def test_localize_box_matches_oracle(cuda_device, shape, bbox, spacing, margin):
    from lesiondiffusion_mlx_b200.composite import localize_output

    original = _ct(shape, 1)
    generated = _ct(shape, 2) + 40.0
    want, weighted = oracle_composite.localize_output(original, generated, bbox, spacing, margin)
    got, facts = localize_output(original=torch.from_numpy(original).to(cuda_device), generated=generated, bbox=bbox,
                                 spacing_mm=spacing, margin_mm=margin)
    got = got.cpu().numpy()
    assert facts["affected_region"]["weighted_voxel_count"] == weighted
    # FP64 weights with one f32 rounding: the device cos may differ from the
    # host's in the last FP64 bit, which can move the f32 result by one ulp.
    ulp = np.spacing(np.abs(want)).astype(np.float32)
    assert np.all(np.abs(got - want) <= ulp)
    assert np.array_equal(got[bbox], generated[bbox])
    far = np.ones(shape, dtype=bool)
    far[tuple(slice(max(0, s.start - 8), s.stop + 8) for s in bbox)] = False
    assert np.array_equal(got[far], original[far])


def test_localize_box_rejects_shape_mismatch(cuda_device):
    from lesiondiffusion_mlx_b200.composite import ModelExecutionError, localize_output

    with pytest.raises(ModelExecutionError):
        localize_output(original=np.zeros((4, 4, 4), np.float32), generated=np.zeros((4, 4, 5), np.float32),
                        bbox=(slice(0, 1),) * 3, spacing_mm=(1.0, 1.0, 1.0))


@pytest.mark.parametrize("reach", [3, 33])
def test_lesion_change_cancels_reconstruction_offset_and_keeps_distant_input(cuda_device, reach):
    """The reference's analytic lesion-mode test, on a synthetic CT in place of
    the HCC-TACE crop it reads."""
    from lesiondiffusion_mlx_b200.composite import apply_lesion_change

    shift = reach - 3
    shape = tuple(size + 2 * shift for size in (24, 20, 18))
    original = _ct(shape, 7)
    original[8 + shift, 6 + shift, 5 + shift] = 1350.0  # bone above the decoder's 1000 HU clip
    lesion = np.zeros(shape, dtype=bool)
    lesion[10 + shift: 13 + shift, 8 + shift: 11 + shift, 7 + shift: 10 + shift] = True
    reconstruction = np.clip(original, -1000, 1000) - 9.0
    generated = reconstruction + np.float32(0.25)
    shell = np.zeros(shape, dtype=bool)
    shell[9 + shift: 14 + shift, 7 + shift: 12 + shift, 6 + shift: 11 + shift] = True
    generated[shell] -= 2.25
    generated[lesion] -= 28.0
    got, facts = apply_lesion_change(original=original, generated=generated, reconstruction=reconstruction,
                                     lesion=lesion, reach_voxels=reach)
    got = got.cpu().numpy()
    reached = np.zeros(shape, dtype=bool)
    reached[7: 16 + 2 * shift, 5: 14 + 2 * shift, 4: 13 + 2 * shift] = True
    np.testing.assert_array_equal(got[~reached], original[~reached])
    assert got[8 + shift, 6 + shift, 5 + shift] == original[8 + shift, 6 + shift, 5 + shift] + 0.25
    np.testing.assert_array_equal(got[reached & ~shell], original[reached & ~shell] + np.float32(0.25))
    np.testing.assert_allclose(got[lesion], original[lesion] - 30.0, atol=1e-4)
    np.testing.assert_allclose(got[shell & ~lesion], original[shell & ~lesion] - 2.0, atol=1e-4)
    assert facts["input_reconstruction_offset_hu"] == pytest.approx(-9.0)
    assert facts["changed_region"]["voxel_count"] == int(reached.sum())


@pytest.mark.parametrize("shape,reach,seed", [((30, 26, 22), 4, 0), ((40, 17, 35), 9, 1), ((12, 50, 9), 33, 2)])
def test_lesion_change_matches_oracle(cuda_device, shape, reach, seed):
    """Random blobs (some touching the volume's faces): bit-exact volume,
    same reached count and offset."""
    from lesiondiffusion_mlx_b200.composite import apply_lesion_change

    rng = np.random.default_rng(seed)
    original = _ct(shape, 10 + seed)
    original[rng.random(shape) < 0.02] = 1500.0
    reconstruction = np.clip(original, -1000, 1000) + rng.normal(size=shape).astype(np.float32)
    generated = reconstruction + rng.normal(size=shape).astype(np.float32) * 5
    lesion = rng.random(shape) < 0.002
    lesion[0, 0, 0] = True
    want, count, offset = oracle_composite.apply_lesion_change(original, generated, reconstruction, lesion, reach)
    got, facts = apply_lesion_change(original=original, generated=generated, reconstruction=reconstruction,
                                     lesion=lesion, reach_voxels=reach)
    assert np.array_equal(got.cpu().numpy(), want)
    assert facts["changed_region"]["voxel_count"] == count
    assert facts["input_reconstruction_offset_hu"] == pytest.approx(offset, abs=1.5e-3)


def test_lesion_change_rejects_empty_lesion(cuda_device):
    from lesiondiffusion_mlx_b200.composite import ModelExecutionError, apply_lesion_change

    z = np.zeros((6, 6, 6), np.float32)
    with pytest.raises(ModelExecutionError):
        apply_lesion_change(original=z, generated=z, reconstruction=z, lesion=np.zeros((6, 6, 6), bool))


def test_lesion_change_reach_beyond_the_volume(cuda_device):
    """A reach longer than every axis (here 2^30 voxels) changes exactly what a
    reach of the longest axis changes: the whole volume."""
    from lesiondiffusion_mlx_b200.composite import apply_lesion_change

    shape = (12, 20, 9)
    rng = np.random.default_rng(7)
    original = _ct(shape, 17)
    reconstruction = original + rng.normal(size=shape).astype(np.float32)
    generated = reconstruction + 3.0
    lesion = np.zeros(shape, bool)
    lesion[3, 15, 2] = True
    far, far_facts = apply_lesion_change(original=original, generated=generated, reconstruction=reconstruction,
                                         lesion=lesion, reach_voxels=2 ** 30)
    axis, axis_facts = apply_lesion_change(original=original, generated=generated, reconstruction=reconstruction,
                                           lesion=lesion, reach_voxels=max(shape))
    assert np.array_equal(far.cpu().numpy(), axis.cpu().numpy())
    assert far_facts["changed_region"]["voxel_count"] == axis_facts["changed_region"]["voxel_count"] == int(
        np.prod(shape))
