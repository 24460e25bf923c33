"""Segmenter mask areas on the GPU (shipk_mask_area) against the reference's own kernel and the
oracle.

Bar: bit-exact areas. The reference's mask_area_into (ops.cu:196-255,418-458) is compiled from
its source into oracle/_ref/libshipref.so and run on the same device inputs; the oracle
restates it on the CPU. Shapes: the shipped segmenter's (300 candidates, 6 + 32 columns, 32
planes of 160 x 160) and odd ones (cells not a multiple of 4, 17 channels, one candidate).
"""

from __future__ import annotations

import ctypes
from pathlib import Path

import numpy as np
import pytest

from shipinfer_b200 import ValidationError
from shipinfer_b200.masks import mask_area_device

pytestmark = pytest.mark.gpu

REF_LIB = Path(__file__).resolve().parents[1] / "oracle" / "_ref" / "libshipref.so"


def _inputs(crops: int, candidates: int, prefix: int, channels: int, cells_hw: tuple[int, int], seed: int):
    rng = np.random.default_rng(seed)
    rows = rng.standard_normal((crops, candidates, prefix + channels)).astype(np.float32)
    rows[:, :, 4] = rng.uniform(0.0, 1.0, (crops, candidates)).astype(np.float32)
    rows[0, :, 4] = 0.1                          # below the threshold: area 0
    rows[1 % crops, 3:9, 4] = 0.95               # ties: the first one is chosen
    if crops > 2:
        rows[2, 0, 4] = np.nan                   # a NaN in row 0 is never displaced
    if crops > 3:
        rows[3, 5:40, 4] = np.nan                # NaNs elsewhere never win
    protos = rng.standard_normal((crops, channels, *cells_hw)).astype(np.float32) * 2
    return rows, protos


CASES = [
    pytest.param(16, 300, 6, 32, (160, 160), id="shipped-shapes"),
    pytest.param(5, 300, 6, 32, (37, 41), id="cells-not-multiple-of-4"),
    pytest.param(4, 1, 6, 17, (20, 20), id="one-candidate-17-channels"),
    pytest.param(9, 64, 8, 3, (7, 9), id="fewer-cells-than-the-cluster-slices"),
]


@pytest.mark.parametrize(("crops", "candidates", "prefix", "channels", "cells_hw"), CASES)
@pytest.mark.parametrize("mask_threshold", [0.5, 0.3, 0.81])
def test_matches_reference_kernel_and_oracle(cuda, orc, crops, candidates, prefix, channels, cells_hw,
                                             mask_threshold):
    rows, protos = _inputs(crops, candidates, prefix, channels, cells_hw, seed=crops + channels)
    t_rows, t_protos = cuda.from_numpy(rows).cuda(), cuda.from_numpy(protos).cuda()
    got = mask_area_device(t_rows, t_protos, prefix=prefix, score_threshold=0.25,
                           mask_threshold=mask_threshold, crop_hw=(256, 128)).cpu().numpy()
    want = orc.mask_area(rows, protos, prefix=prefix, score_threshold=0.25, mask_threshold=mask_threshold,
                         crop_hw=(256, 128))
    assert np.array_equal(got.view(np.uint32), want.view(np.uint32)), (got, want)
    assert got[0] == 0.0 and (got[1:] > 0).any()
    if REF_LIB.exists():
        ref = ctypes.CDLL(str(REF_LIB))
        out = cuda.empty(crops, dtype=cuda.float32, device="cuda")
        cells = cells_hw[0] * cells_hw[1]
        rc = ref.ref_mask_area(ctypes.c_void_p(t_rows.data_ptr()), candidates, prefix + channels, prefix,
                               ctypes.c_void_p(t_protos.data_ptr()), channels, cells, crops, ctypes.c_float(0.25),
                               ctypes.c_float(mask_threshold), 256, 128, ctypes.c_void_p(out.data_ptr()), None)
        assert rc == 0
        cuda.cuda.synchronize()
        assert np.array_equal(out.cpu().numpy().view(np.uint32), got.view(np.uint32))


def test_refusals_match_the_reference(cuda):
    rows = cuda.zeros((2, 10, 38), device="cuda")
    protos = cuda.zeros((2, 32, 16), device="cuda")
    with pytest.raises(ValidationError):  # 32 coefficients against 31 planes
        mask_area_device(rows, protos[:, :31].contiguous(), prefix=6, score_threshold=0.25, mask_threshold=0.5,
                         crop_hw=(8, 8))
    for bad in (0.0, 1.0, float("nan")):
        with pytest.raises(ValidationError):
            mask_area_device(rows, protos, prefix=6, score_threshold=0.25, mask_threshold=bad, crop_hw=(8, 8))
    empty = mask_area_device(rows[:0], protos[:0], prefix=6, score_threshold=0.25, mask_threshold=0.5,
                             crop_hw=(8, 8))
    assert empty.numel() == 0
