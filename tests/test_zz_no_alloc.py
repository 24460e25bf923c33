"""The allocation-free NMS entry point (shipk_nms_static) against the workspace one (shipk_nms).

shipk_nms_static keeps its scratch in a static device array inside libshipk.so instead of a
caller-provided workspace. Both entry points are called here through the C ABI on the same
device inputs, twice in a row (the second call must see the scratch its first call left
behind and still agree), for config 2's class-aware batch and a class-agnostic batch, and
every result is also compared with the CPU oracle (the reference's NumpyImageOps.nms
restated, per class and merged), since the static path lays out its scratch and resets its
arrival counters on its own; a request larger than the static scratch must be refused with
SHIPK_ERANGE. This file sorts last so that it also runs after every other GPU test in one
session.
"""

from __future__ import annotations

import ctypes

import numpy as np
import pytest

from _data import nms_heads
from shipinfer_b200 import _native

pytestmark = pytest.mark.gpu


def _ptr(t) -> ctypes.c_void_p:
    return ctypes.c_void_p(t.data_ptr())


def _run_both(torch, boxes, scores, classes, num_classes, class_aware, max_det):
    lib = _native.lib()
    b, n = scores.shape
    dev = "cuda"
    tb = torch.from_numpy(boxes).to(dev)
    ts = torch.from_numpy(scores).to(dev)
    tc = torch.from_numpy(classes).to(dev)
    ws_bytes = lib.shipk_nms_workspace_bytes(b, n, num_classes, int(class_aware), max_det)
    ws = torch.empty(max(int(ws_bytes), 1), dtype=torch.uint8, device=dev)
    results = []
    for entry in ("shipk_nms", "shipk_nms_static", "shipk_nms_static", "shipk_nms"):
        keep = torch.full((b, max_det), 7, dtype=torch.int64, device=dev)  # junk: every slot is written
        counts = torch.full((b,), -5, dtype=torch.int32, device=dev)
        if entry == "shipk_nms":
            rc = lib.shipk_nms(_ptr(tb), _ptr(ts), _ptr(tc), b, n, num_classes, int(class_aware), 0.45, 0.25,
                               max_det, _ptr(keep), _ptr(counts), _ptr(ws), ctypes.c_size_t(ws.numel()), None)
        else:
            rc = lib.shipk_nms_static(_ptr(tb), _ptr(ts), _ptr(tc), b, n, num_classes, int(class_aware), 0.45,
                                      0.25, max_det, _ptr(keep), _ptr(counts), None)
        _native.check(rc)
        torch.cuda.synchronize()
        results.append((entry, keep.cpu().numpy(), counts.cpu().numpy()))
    return results


@pytest.mark.parametrize("class_aware", [True, False], ids=["class-aware", "class-agnostic"])
def test_static_scratch_matches_the_workspace_entry_twice_in_a_row(cuda, orc, class_aware):
    boxes, scores, classes = nms_heads(batch=16, n=8400, classes=2, seed=3)
    results = _run_both(cuda, boxes, scores, classes, 2, class_aware, 300)
    _, want_keep, want_counts = results[0]
    assert want_counts.min() > 0
    for entry, keep, counts in results[1:]:
        assert np.array_equal(counts, want_counts), entry
        assert np.array_equal(keep, want_keep), entry
    orc_keep, orc_counts = orc.nms_batched(boxes, scores, classes, 0.45, 0.25, 300, num_classes=2,
                                           class_aware=class_aware)
    for entry, keep, counts in results:
        assert np.array_equal(counts, orc_counts), entry
        assert np.array_equal(keep, orc_keep), entry


def test_a_request_beyond_the_static_scratch_is_refused(cuda):
    lib = _native.lib()
    b, n, classes, max_det = 64, 16, 64, 4096  # 64 x 64 x 4096 x 4 bytes: far above 1 MiB
    keep = cuda.empty((b, max_det), dtype=cuda.int64, device="cuda")
    counts = cuda.empty((b,), dtype=cuda.int32, device="cuda")
    boxes = cuda.zeros((b, n, 4), dtype=cuda.float32, device="cuda")
    scores = cuda.zeros((b, n), dtype=cuda.float32, device="cuda")
    cls = cuda.zeros((b, n), dtype=cuda.int32, device="cuda")
    rc = lib.shipk_nms_static(_ptr(boxes), _ptr(scores), _ptr(cls), b, n, classes, 1, 0.45, 0.25, max_det,
                              _ptr(keep), _ptr(counts), None)
    assert rc == _native.ERANGE
    assert "static scratch" in _native.last_error()
