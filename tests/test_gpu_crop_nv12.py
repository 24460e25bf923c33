"""Crops straight from NV12 surfaces on the GPU (shipk_crop_nv12) against the reference's own
kernel and the oracle.

Bar: bit-exact. The reference's nv12_crop_resize_into (ops.cu:260-318, one frame per call) is
compiled from its source into oracle/_ref/libshipref.so and run per frame on the same device
surfaces; the oracle restates it on the CPU. The kernel here takes every box of every frame in
one launch.
"""

from __future__ import annotations

import ctypes
from pathlib import Path

import numpy as np
import pytest

from _data import nv12_frames
from shipinfer_b200 import Nv12Frame, ValidationError

pytestmark = pytest.mark.gpu

REF_LIB = Path(__file__).resolve().parents[1] / "oracle" / "_ref" / "libshipref.so"


def _boxes(n: int, h: int, w: int, seed: int) -> np.ndarray:
    rng = np.random.default_rng(seed)
    bw = np.exp(rng.uniform(np.log(4.0), np.log(w * 0.8), n))
    bh = np.exp(rng.uniform(np.log(4.0), np.log(h * 0.8), n))
    x = rng.uniform(-10.0, w - bw + 10)
    y = rng.uniform(-10.0, h - bh + 10)
    boxes = np.stack([x, y, x + bw, y + bh], axis=1).astype(np.float32)
    boxes[0] = [5.5, 7.25, 5.5, 40]  # zero width: a crop of zeros
    boxes[1] = [-50, -50, 1e9, 1e9]  # the whole frame
    return boxes


@pytest.mark.parametrize(("hw", "pitch", "dst"), [((270, 480), None, (64, 32)), ((181, 323), 384, (37, 29)),
                                                  ((720, 1280), None, (256, 128))],
                         ids=["tight", "odd-with-pitch", "720p-embedder"])
@pytest.mark.parametrize("swap_rb", [True, False])
def test_matches_reference_kernel_and_oracle(cuda, ops, orc, hw, pitch, dst, swap_rb):
    planes = nv12_frames(3, hw, seed=hw[0], pitch=pitch)
    boxes = np.concatenate([_boxes(12, hw[0], hw[1], seed=k) for k in range(3)])
    frame_of = np.repeat(np.arange(3, dtype=np.int32), 12)
    dev_bufs = [cuda.from_numpy(p[0]).cuda() for p in planes]
    frames = [Nv12Frame(b, p[1], p[2], p[3], p[4]) for b, p in zip(dev_bufs, planes)]
    t_boxes = cuda.from_numpy(boxes).cuda()
    out = cuda.empty((len(boxes), 3, *dst), dtype=cuda.float32, device="cuda")
    ops.crop_nv12_device(frames, t_boxes, out, swap_rb=swap_rb, box_frame=cuda.from_numpy(frame_of).cuda())
    got = out.cpu().numpy()
    want = orc.crop_nv12(planes, boxes, dst, frame_of, swap_rb)
    assert np.array_equal(got.view(np.uint32), want.view(np.uint32)), np.argwhere(got != want)[:5]
    assert (got[0] == 0).all() and got[1].any()
    if REF_LIB.exists():
        ref = ctypes.CDLL(str(REF_LIB))
        for f in range(3):
            sel = frame_of == f
            sub = cuda.from_numpy(np.ascontiguousarray(boxes[sel])).cuda()
            rout = cuda.empty((int(sel.sum()), 3, *dst), dtype=cuda.float32, device="cuda")
            _, h, w, p, uvo = planes[f]
            rc = ref.ref_nv12_crop(ctypes.c_void_p(dev_bufs[f].data_ptr()), h, w, p, ctypes.c_ulonglong(uvo),
                                   ctypes.c_void_p(sub.data_ptr()), int(sel.sum()), ctypes.c_void_p(rout.data_ptr()),
                                   dst[0], dst[1], int(swap_rb), None)
            assert rc == 0
            cuda.cuda.synchronize()
            r = rout.cpu().numpy()
            assert np.array_equal(r.view(np.uint32), got[sel].view(np.uint32)), (f, np.argwhere(r != got[sel])[:5])
    out16 = cuda.empty((len(boxes), 3, *dst), dtype=cuda.float16, device="cuda")
    ops.crop_nv12_device(frames, t_boxes, out16, swap_rb=swap_rb, box_frame=cuda.from_numpy(frame_of).cuda())
    assert np.array_equal(out16.cpu().numpy(), want.astype(np.float16))


def test_layout_refusals(cuda, ops):
    buf = cuda.zeros(64 * 48 * 3 // 2, dtype=cuda.uint8, device="cuda")
    out = cuda.empty((1, 3, 8, 8), device="cuda")
    boxes = cuda.tensor([[0.0, 0.0, 10.0, 10.0]], device="cuda")
    with pytest.raises(ValidationError):  # stride narrower than the width
        ops.crop_nv12_device([Nv12Frame(buf, 48, 64, 32, 64 * 48)], boxes, out)
    with pytest.raises(ValidationError):  # chroma inside the luma plane
        ops.crop_nv12_device([Nv12Frame(buf, 48, 64, 64, 64 * 40)], boxes, out)
