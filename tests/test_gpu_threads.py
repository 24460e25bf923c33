"""Worker threads sharing one ThreadLocalImageOps on the B200: each thread gets its own
NativeImageOps (its own staging context) and the threads run host-frame letterboxes, crops and
NMS at the same time; every result is bit-exact to the oracle. This is the reference's
multi-GPU preprocessing arrangement (thread_local.py:77-192) on one device."""

from __future__ import annotations

import threading

import numpy as np
import pytest

from _data import IMAGENET_MEAN, IMAGENET_STD, frames_u8, nms_heads
from shipinfer_b200 import NormalizeParams
from shipinfer_b200.thread_local import ThreadLocalImageOps

pytestmark = pytest.mark.gpu


def test_threads_each_get_their_own_ops_and_exact_results(cuda, orc):
    tl = ThreadLocalImageOps(devices=[0])
    params = NormalizeParams(mean=IMAGENET_MEAN, std=IMAGENET_STD, swap_rb=True)
    n_threads, rounds = 4, 3
    work = []
    for t in range(n_threads):
        frames = frames_u8(2, [(720, 1280), (1080, 1920), (480, 640), (300, 500)][t], seed=40 + t)
        boxes = np.array([[10, 20, 200, 150], [5.5, 7.25, 60, 90], [0, 0, 300, 250]], np.float32)
        b, s, _ = nms_heads(1, 2000, 1, seed=50 + t)
        work.append((frames, boxes, b[0], s[0]))
    results = [[] for _ in range(n_threads)]
    errors = []
    start = threading.Barrier(n_threads)

    def worker(t):
        try:
            frames, boxes, b, s = work[t]
            start.wait()
            for _ in range(rounds):
                lb = tl.letterbox_batch(frames, (640, 640), params)
                crops = tl.crop_batch(frames[0], boxes, (256, 128), params)
                kept = tl.nms(b, s, 0.45, 0.25, 300)
                results[t].append((lb.tensor, crops, kept, id(tl.delegate())))
        except Exception as exc:  # pragma: no cover - reported below
            errors.append(exc)

    threads = [threading.Thread(target=worker, args=(t,)) for t in range(n_threads)]
    for th in threads:
        th.start()
    for th in threads:
        th.join()
    assert not errors, errors
    assert tl.assignments() == {0: n_threads}
    assert len({r[0][3] for r in results}) == n_threads  # one delegate per thread
    for t in range(n_threads):
        frames, boxes, b, s = work[t]
        want_lb = orc.letterbox(frames, (640, 640), params.mean, params.std, params.swap_rb, 114)
        want_crop = orc.crop([frames[0]], boxes, (256, 128), None, params.mean, params.std, params.swap_rb)
        want_keep = orc.nms(b, s, 0.45, 0.25, 300)
        for lb, crops, kept, _ in results[t]:
            assert np.array_equal(lb.view(np.uint32), want_lb.view(np.uint32))
            assert np.array_equal(crops.view(np.uint32), want_crop.view(np.uint32))
            assert kept.tolist() == list(want_keep)
