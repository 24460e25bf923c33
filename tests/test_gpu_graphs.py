"""A detector step's device work captured once in a CUDA graph and replayed on new inputs.

The production path (reference base.py:100-141 and its ADR-007): frames already on
the device are letterboxed straight into the engine's input binding (a caller-owned tensor with
a stable address), crops go into the embedder's binding, and the detector heads are suppressed
into preallocated outputs; the whole step is one graph replay. Each entry point allocates
nothing, synchronises nothing and takes torch's current stream, so it captures; after each
replay on new frame and head contents (written into the same buffers), every output equals the
oracle's on those contents bit for bit.
"""

from __future__ import annotations

import numpy as np
import pytest

from _data import IMAGENET_MEAN, IMAGENET_STD, crop_boxes, frames_u8, nms_heads
from shipinfer_b200 import NormalizeParams

pytestmark = pytest.mark.gpu

UNIT = NormalizeParams()
IMAGENET = NormalizeParams(mean=IMAGENET_MEAN, std=IMAGENET_STD)
HW = (720, 1280)


def exact(a: np.ndarray, b: np.ndarray) -> bool:
    return a.shape == b.shape and a.dtype == b.dtype and np.array_equal(a.view(np.uint8), b.view(np.uint8))


@pytest.mark.parametrize("mode", ["global", "relaxed"])
def test_preprocess_crop_and_nms_replay_from_one_graph(cuda, ops, orc, mode):
    torch = cuda
    frames = [torch.from_numpy(f).cuda() for f in frames_u8(4, HW, seed=31)]
    binding = torch.empty((4, 3, 640, 640), dtype=torch.float16, device="cuda")  # the detector's input
    boxes_h, idx_h = crop_boxes(4, 16, hw=HW, seed=3)
    boxes, idx = torch.from_numpy(boxes_h).cuda(), torch.from_numpy(idx_h).cuda()
    crops = torch.empty((64, 3, 256, 128), dtype=torch.float16, device="cuda")  # the embedder's input
    b, s, c = (torch.from_numpy(x).cuda() for x in nms_heads(4, 8400, 2, seed=41))
    keep = torch.empty((4, 300), dtype=torch.int64, device="cuda")
    counts = torch.empty((4,), dtype=torch.int32, device="cuda")

    def step():
        ops.letterbox_device(frames, binding, UNIT)
        ops.crop_device(frames, boxes, crops, IMAGENET, box_frame=idx)
        ops.nms_device(b, s, c, iou_threshold=0.45, score_threshold=0.25, max_det=300, num_classes=2,
                       class_aware=True, keep=keep, counts=counts)

    # first launches outside capture (kernel attributes, the NMS workspace), then capture
    side = torch.cuda.Stream()
    side.wait_stream(torch.cuda.current_stream())
    with torch.cuda.stream(side):
        step()
    torch.cuda.current_stream().wait_stream(side)
    torch.cuda.synchronize()
    graph = torch.cuda.CUDAGraph()
    with torch.cuda.graph(graph, capture_error_mode=mode):
        step()

    for k in range(2):
        new_frames = frames_u8(4, HW, seed=100 + k)
        for dst, src in zip(frames, new_frames):
            dst.copy_(torch.from_numpy(src))
        nb, ns, nc = nms_heads(4, 8400, 2, seed=200 + k)
        b.copy_(torch.from_numpy(nb))
        s.copy_(torch.from_numpy(ns))
        c.copy_(torch.from_numpy(nc))
        graph.replay()
        torch.cuda.synchronize()
        want = orc.letterbox(new_frames, (640, 640), UNIT.mean, UNIT.std, UNIT.swap_rb, 114).astype(np.float16)
        assert exact(binding.cpu().numpy(), want)
        want_c = orc.crop(new_frames, boxes_h, (256, 128), idx_h, IMAGENET.mean, IMAGENET.std, True)
        assert exact(crops.cpu().numpy(), want_c.astype(np.float16))
        want_k, want_n = orc.nms_batched(nb, ns, nc, 0.45, 0.25, 300, num_classes=2)
        assert np.array_equal(counts.cpu().numpy(), np.asarray(want_n, np.int32))
        assert np.array_equal(keep.cpu().numpy(), np.asarray(want_k, np.int64))
