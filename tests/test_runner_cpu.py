"""Host logic of the LINet stage runner: the crop centred on the lesion and
LINet's latent window (mlx_pipeline.py:38-69 ``source_crop``, medmlx.py:1458-1470
``_linet_latent_window``), worked by hand."""

from __future__ import annotations

import numpy as np
import pytest

from lesiondiffusion_mlx_b200 import runner


def _mask(shape, box):
    m = np.zeros(shape, bool)
    m[tuple(slice(a, b) for a, b in box)] = True
    return m


def test_crop_is_centred_on_the_bounding_box_and_kept_inside():
    m = _mask((40, 50, 60), ((10, 15), (20, 31), (0, 3)))
    # centres: (10 + 14) // 2 = 12, (20 + 30) // 2 = 25, (0 + 2) // 2 = 1
    crops = runner.source_crop(m, (8, 10, 12))
    assert crops == (slice(8, 16), slice(20, 30), slice(0, 12))  # axis 2 shifted to start at 0
    m2 = _mask((40, 50, 60), ((36, 40), (0, 1), (55, 60)))
    assert runner.source_crop(m2, (8, 10, 12)) == (slice(32, 40), slice(0, 10), slice(48, 60))


def test_latent_window_halves_the_crop_rounding_down():
    m = _mask((40, 50, 60), ((11, 16), (20, 31), (7, 9)))
    crop = runner.source_crop(m, (9, 10, 13))  # centres 13, 25, (7 + 8) // 2 = 7 -> starts 9, 20, 1
    assert crop == (slice(9, 18), slice(20, 30), slice(1, 14))
    assert runner.linet_latent_window(m, (9, 10, 13)) == (slice(4, 9), slice(10, 15), slice(0, 7))


def test_crop_errors():
    with pytest.raises(ValueError, match="empty lesion"):
        runner.source_crop(np.zeros((8, 8, 8), bool), (4, 4, 4))
    with pytest.raises(ValueError, match="axis 1 >= 9"):
        runner.source_crop(_mask((8, 8, 8), ((1, 2), (1, 2), (1, 2))), (4, 9, 4))
