"""ThreadLocalImageOps host logic on the CPU, with a recording stand-in for the GPU ops.

Pins the reference's per-thread contract (``thread_local.py:77-192``, tested there by
``tests/runtime/test_thread_local_ops.py``): one delegate per thread, built lazily on that
thread; devices handed out in rotation; a failed build still consumes its device slot;
``assignments()`` counts only delegates that exist.
"""

from __future__ import annotations

import threading

import numpy as np
import pytest

from shipinfer_b200 import NormalizeParams
from shipinfer_b200.thread_local import ThreadLocalImageOps


class Recorder:
    """Stands in for NativeImageOps: records the thread that built it and the calls it gets."""

    on_device = True

    def __init__(self, device: int) -> None:
        self.device = device
        self.built_on = threading.get_ident()
        self.calls: list[tuple] = []

    def letterbox_batch(self, images, dst_size, params, *, pad_value=114):
        self.calls.append(("letterbox_batch", len(images), dst_size, pad_value))
        return "lb"

    def letterbox_to_device(self, images, out, params, *, pad_value=114):
        self.calls.append(("letterbox_to_device", len(images), out, pad_value))
        return "ltd"

    def crop_batch(self, image, boxes, dst_size, params):
        self.calls.append(("crop_batch", boxes.shape, dst_size))
        return "crop"

    def nms(self, boxes, scores, iou_threshold, score_threshold, max_output):
        self.calls.append(("nms", iou_threshold, score_threshold, max_output))
        return "nms"

    def crop_device(self, *args):
        self.calls.append(("crop_device",) + args)
        return "crop_device"


def run_threads(n, fn):
    out, errs = [None] * n, []

    def body(i):
        try:
            out[i] = fn(i)
        except Exception as exc:  # pragma: no cover - reported below
            errs.append(exc)

    threads = [threading.Thread(target=body, args=(i,)) for i in range(n)]
    for t in threads:
        t.start()
    for t in threads:
        t.join()
    assert not errs, errs
    return out


def test_one_delegate_per_thread_built_on_that_thread():
    tl = ThreadLocalImageOps(Recorder, devices=[0, 1, 2, 3])
    got = run_threads(8, lambda i: (tl.delegate(), tl.delegate(), threading.get_ident()))
    delegates = [d for d, again, _ in got]
    assert all(d is again for d, again, _ in got)           # stable within a thread
    assert len({id(d) for d in delegates}) == 8            # distinct across threads
    assert all(d.built_on == tid for d, _, tid in got)     # built by the thread that uses it
    assert tl.assignments() == {0: 2, 1: 2, 2: 2, 3: 2}    # round-robin spread


def test_devices_rotate_in_first_call_order():
    tl = ThreadLocalImageOps(Recorder, devices=[5, 7])
    order = []
    gate = threading.Lock()

    def first_call(i):
        with gate:  # serialise first calls so the rotation order is observable
            d = tl.delegate().device
            order.append(d)
        return tl.device_of_this_thread()

    got = run_threads(5, first_call)
    assert order == [5, 7, 5, 7, 5]
    assert sorted(got) == sorted(order)
    assert tl.device_of_this_thread() is None  # the main thread never called


def test_a_failed_build_consumes_its_slot_and_is_not_counted():
    attempts = []

    def factory(device):
        attempts.append(device)
        if len(attempts) == 1:
            raise RuntimeError("no context on this device")
        return Recorder(device)

    tl = ThreadLocalImageOps(factory, devices=[0, 1])
    with pytest.raises(RuntimeError):
        tl.delegate()
    assert tl.assignments() == {}
    ops = tl.delegate()                     # the same thread retries on the next device
    assert ops.device == 1 and attempts == [0, 1]
    assert tl.assignments() == {1: 1}


def test_calls_reach_the_threads_delegate_unchanged():
    tl = ThreadLocalImageOps(Recorder, devices=[])  # empty: device 0
    params = NormalizeParams()
    frames = [np.zeros((4, 4, 3), np.uint8)] * 3
    boxes = np.zeros((2, 4), np.float32)
    assert tl.letterbox_batch(frames, (8, 8), params, pad_value=0) == "lb"
    assert tl.letterbox_to_device(frames, "out", params) == "ltd"
    assert tl.crop_batch(frames[0], boxes, (4, 2), params) == "crop"
    assert tl.nms(boxes, np.zeros(2, np.float32), 0.45, 0.25, 300) == "nms"
    assert tl.crop_device(1, 2) == "crop_device"   # the device-resident API passes through
    assert tl.on_device is True
    d = tl.delegate()
    assert d.device == 0
    assert d.calls == [("letterbox_batch", 3, (8, 8), 0), ("letterbox_to_device", 3, "out", 114),
                       ("crop_batch", (2, 4), (4, 2)), ("nms", 0.45, 0.25, 300), ("crop_device", 1, 2)]
    with pytest.raises(AttributeError):
        tl._private_thing
