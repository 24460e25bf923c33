"""The kernels' fast normalisation against IEEE-754 division, for every input it can meet.

The letterbox, crop and NV12 kernels compute (v - mean) / std with a correctly rounded
division built from RN(1/std) and fused multiply-adds (Markstein's method) instead of a divide.
shipk_normalise_check evaluates that and __fdiv_rn for every single-precision v in [0, 256)
(1.13e9 inputs: every value normalisation can receive, since blended and converted pixels are
clamped to [0, 255]) and counts results that differ in any bit. Bar: zero, for the constants
the reference ships (ImageNet mean/std on the 0..255 scale, /255) and a spread of others.
"""

from __future__ import annotations

import ctypes

import pytest

from _data import IMAGENET_MEAN, IMAGENET_STD
from shipinfer_b200 import _native

pytestmark = pytest.mark.gpu

CONSTANTS = [(0.0, 255.0), (0.0, 1.0), (0.0, 127.5), (127.5, 127.5), (128.0, 3.0), (0.0, 7.0),
             (0.485, 0.229), (0.5, 0.5), (16.0, 219.0), (1e-3, 1e3), (-3.25, 0.1)]
CONSTANTS += list(zip(IMAGENET_MEAN, IMAGENET_STD))


@pytest.mark.parametrize("mean,std", CONSTANTS, ids=[f"{m:g}/{s:g}" for m, s in CONSTANTS])
def test_fast_division_matches_ieee_division_on_all_of_0_to_256(cuda, mean, std):
    result = cuda.tensor([0, -1], dtype=cuda.int64, device="cuda")  # {0, UINT64_MAX}
    lib = _native.lib()
    rc = lib.shipk_normalise_check(float(mean), float(std), ctypes.c_void_p(result.data_ptr()), None)
    _native.check(rc)
    cuda.cuda.synchronize()
    count, first = result.cpu().tolist()
    assert count == 0, f"{count} inputs differ, first v bits {first & 0xffffffff:#010x}"


def test_constants_outside_the_fast_range_are_refused(cuda):
    result = cuda.tensor([0, -1], dtype=cuda.int64, device="cuda")
    rc = _native.lib().shipk_normalise_check(0.0, 1e-9, ctypes.c_void_p(result.data_ptr()), None)
    assert rc == _native.ERANGE
