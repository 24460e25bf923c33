"""The NV12 conversion constants, derived rather than trusted.

The limited-range YCbCr -> R'G'B' matrix follows from the standard's luma weights: with
Kg = 1 - Kr - Kb, luma scale 255/219 and chroma scale 255/224,

    ys  = 255/219 (written 1.164383)      cbu = 2 (1 - Kb) 255/224
    cgu = 2 Kb (1 - Kb) / Kg * 255/224    cgv = 2 Kr (1 - Kr) / Kg * 255/224
    crv = 2 (1 - Kr) 255/224

(ITU-R BT.601: Kr 0.299, Kb 0.114; ITU-R BT.709: Kr 0.2126, Kb 0.0722). The reference's
nv12_to_bgr writes the BT.601 chroma terms rounded to six decimals and the luma scale
255/219 = 1.16438356... as 1.164383 (csrc/shipinfer/runtime/ops.cu:159-166); BT.709 has no
reference, so this build uses the same construction and the same luma literal. Here the kernels'
constants (shipinfer_b200/csrc/common.cuh) and the oracle's (oracle/oracle.c) must both be the
float32 roundings of those six-decimal values, derived in float64 — and, where the reference
tree is present, the BT.601 ones must be the numbers its own source writes.
"""

from __future__ import annotations

import os
import re
from pathlib import Path

import numpy as np
import pytest

from _data import yuv_constants

ROOT = Path(__file__).resolve().parents[1]
REFERENCE_OPS = Path(os.environ.get("SHIPK_REFERENCE", "/root/reference")) / "csrc/shipinfer/runtime/ops.cu"


def _matrix_block(text: str, matrix: int) -> dict[str, float]:
    """The constants a source file assigns for one matrix (the `if (matrix == 709)` branch or
    its else), plus the shared luma scale."""
    ys = float(re.search(r"ys\s*=\s*([0-9.]+)f", text).group(1))
    branch = re.search(r"matrix == 709\)\s*\{(.*?)\}\s*else\s*\{(.*?)\}", text, re.S)
    body = branch.group(1) if matrix == 709 else branch.group(2)
    vals = {k: float(v) for k, v in re.findall(r"(cbu|cgu|cgv|crv)\s*=\s*([0-9.]+)f", body)}
    vals["ys"] = ys
    return vals


@pytest.mark.parametrize("path", ["shipinfer_b200/csrc/common.cuh", "oracle/oracle.c"])
@pytest.mark.parametrize("matrix", [601, 709])
def test_constants_are_the_derived_matrix(path, matrix):
    text = (ROOT / path).read_text()
    got = _matrix_block(text, matrix)
    want = dict(zip(("ys", "cbu", "cgu", "cgv", "crv"), yuv_constants(matrix)))
    assert set(got) == set(want)
    for name, value in want.items():
        assert np.float32(got[name]) == np.float32(value), (path, matrix, name, got[name], value)
    # the luma literal is 255/219 to within a unit of the sixth decimal
    assert abs(want["ys"] - 255.0 / 219.0) < 1e-6


def test_bt709_differs_from_bt601_where_the_standards_differ():
    a, b = yuv_constants(601), yuv_constants(709)
    assert a[0] == b[0]  # the luma scale is range-only
    assert all(x != y for x, y in zip(a[1:], b[1:]))
    assert yuv_constants(709) == (1.164383, 2.112402, 0.213249, 0.532909, 1.792741)


@pytest.mark.skipif(not REFERENCE_OPS.exists(), reason="the reference source tree is not present")
def test_bt601_constants_are_the_reference_sources():
    """The reference's nv12_to_bgr literals, read from its source as text."""
    text = REFERENCE_OPS.read_text()
    literals = [float(v) for v in re.findall(r"\b([0-2]\.\d{6})f\b", text)]
    for value in yuv_constants(601):
        assert value in literals, value
