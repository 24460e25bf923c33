"""NV12 letterbox on the GPU, through the C ABI.

* BT.601 + nearest is the reference's own NV12 kernel (csrc/shipinfer/runtime/ops.cu:148-194):
  bit-exact against the oracle, and — when oracle/_ref/libshipref.so (the reference's kernels
  compiled from its sources) is present — bit-exact against the reference kernel itself.
* BT.709 + bilinear (config 5) has no reference implementation: bit-exact against the
  oracle's restatement, which is this build's definition (parity unpinned by the reference).
"""

from __future__ import annotations

import ctypes
from pathlib import Path

import numpy as np
import pytest

from _data import nv12_frames
from shipinfer_b200 import NormalizeParams, Nv12Frame, ValidationError

pytestmark = pytest.mark.gpu

REF_LIB = Path(__file__).resolve().parents[1] / "oracle" / "_ref" / "libshipref.so"


def exact(a: np.ndarray, b: np.ndarray) -> bool:
    return a.shape == b.shape and a.dtype == b.dtype and np.array_equal(a.view(np.uint8), b.view(np.uint8))


def run(torch, ops, planes, dst, dtype, matrix, sampling, params=NormalizeParams(), pad=114):
    frames = [Nv12Frame(torch.from_numpy(buf).cuda(), h, w, pitch, uv) for buf, h, w, pitch, uv in planes]
    out = torch.empty((len(planes), 3, *dst), dtype=dtype, device="cuda")
    ops.letterbox_nv12_device(frames, out, params, pad_value=pad, matrix=matrix, sampling=sampling)
    torch.cuda.synchronize()
    return out.cpu().numpy()


CASES = [
    pytest.param((90, 160), 160, 90, (64, 64), id="tight-90x160"),
    pytest.param((90, 160), 192, 96, (64, 64), id="padded-nvdec-surface"),
    pytest.param((1080, 1920), 2048, 1088, (640, 640), id="1080p-padded"),
    pytest.param((37, 51), 64, 40, (50, 50), id="odd-sizes"),
    # ratio RN(1/3): tap weights of 2^-26 next to conversions as small as 2^-26, so the kernel
    # keeps its tiny-numerator test on for the default zero-mean constants
    pytest.param((40, 60), 64, 40, (120, 180), id="3x-upscale-tiny-weights"),
]


@pytest.mark.parametrize(("hw", "pitch", "coded_h", "dst"), CASES)
@pytest.mark.parametrize(("matrix", "sampling"), [(601, "nearest"), (709, "bilinear"), (601, "bilinear"),
                                                  (709, "nearest")])
def test_matches_oracle(cuda, ops, orc, hw, pitch, coded_h, dst, matrix, sampling):
    planes = nv12_frames(2, hw, seed=hw[0], pitch=pitch, coded_h=coded_h)
    want = orc.letterbox_nv12(planes, dst, matrix=matrix, sampling=0 if sampling == "nearest" else 1)
    got = run(cuda, ops, planes, dst, cuda.float32, matrix, sampling)
    assert exact(got, want), f"max |d| {np.abs(got - want).max()}"
    got16 = run(cuda, ops, planes, dst, cuda.float16, matrix, sampling)
    assert exact(got16, want.astype(np.float16))


def test_config5_4k_bilinear_709_fp16(cuda, ops, orc):
    """Config 5 shape (batch reduced to 2 for test time): 3840x2160 NV12 -> 1280x1280 fp16."""
    planes = nv12_frames(2, (2160, 3840), seed=0)
    want = orc.letterbox_nv12(planes, (1280, 1280), matrix=709, sampling=1)
    got = run(cuda, ops, planes, (1280, 1280), cuda.float16, 709, "bilinear")
    assert exact(got, want.astype(np.float16))


@pytest.mark.skipif(not REF_LIB.exists(), reason="oracle/_ref/libshipref.so not built")
@pytest.mark.parametrize(("hw", "pitch", "coded_h", "dst"), CASES)
def test_nearest_601_matches_the_reference_kernel(cuda, ops, hw, pitch, coded_h, dst):
    """The reference's nv12_letterbox_into, compiled from its own source, on the same surface."""
    ref = ctypes.CDLL(str(REF_LIB))
    ref.ref_nv12_letterbox.argtypes = [ctypes.c_void_p, ctypes.c_int, ctypes.c_int, ctypes.c_int,
                                       ctypes.c_ulonglong, ctypes.c_void_p, ctypes.c_int, ctypes.c_int,
                                       ctypes.c_int, ctypes.c_float, ctypes.c_void_p, ctypes.c_void_p]
    (buf, h, w, p, uv), = nv12_frames(1, hw, seed=5, pitch=pitch, coded_h=coded_h)
    dev = cuda.from_numpy(buf).cuda()
    theirs = cuda.empty((1, 3, *dst), dtype=cuda.float32, device="cuda")
    pad = np.float32(114) / np.float32(255)
    rc = ref.ref_nv12_letterbox(dev.data_ptr(), h, w, p, uv, theirs.data_ptr(), dst[0], dst[1], 1,
                                float(pad), None, None)
    assert rc == 0
    mine = run(cuda, ops, [(buf, h, w, p, uv)], dst, cuda.float32, 601, "nearest")
    cuda.cuda.synchronize()
    assert exact(mine, theirs.cpu().numpy())


def test_layout_refusals_match_the_reference(cuda, ops):
    buf = cuda.zeros(192 * 96 * 2, dtype=cuda.uint8, device="cuda")
    out = cuda.empty((1, 3, 64, 64), device="cuda")
    with pytest.raises(ValidationError, match="inside the luma plane"):
        ops.letterbox_nv12_device([Nv12Frame(buf, 90, 160, 192, 192 * 80)], out, NormalizeParams())
    with pytest.raises(ValidationError, match="narrower than the width"):
        ops.letterbox_nv12_device([Nv12Frame(buf, 90, 160, 100, 100 * 90)], out, NormalizeParams())
