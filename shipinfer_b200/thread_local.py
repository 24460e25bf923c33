"""Per-thread image ops spread over the GPUs, for pipelines whose worker threads share one seam.

Mirrors the reference's ``ThreadLocalImageOps`` (``src/shipinfer/runtime/ops/thread_local.py:
77-192``), its mechanism for multi-GPU preprocessing: a stage holds ONE ops object, but every
worker thread that calls it gets its own delegate, because a :class:`NativeImageOps` keeps a
staging context that two threads must not share. Each thread's delegate is bound, on its first
call, to the next device of ``devices`` in rotation, and stays on it for the thread's life, so
preprocessing spreads over the GPUs instead of landing on device 0 (a frame stays on the GPU
that letterboxes it).

Same behaviour as the reference at its edges: construction is lazy and happens on the calling
thread, outside the lock (a slow build does not hold up other threads' first calls); a factory
that raises still consumes its device slot, so that thread's retry moves on to the next device;
:meth:`assignments` counts only delegates that were built.
"""

from __future__ import annotations

import threading
from collections.abc import Callable, Sequence
from typing import Any

import numpy as np

from shipinfer_b200.types import LetterboxResult, NormalizeParams

__all__ = ["ThreadLocalImageOps"]


class ThreadLocalImageOps:
    """Delegates each call to the calling thread's own ops instance.

    Args:
        factory: ``device_index -> ops`` (``NativeImageOps`` by default).
        devices: the device indices handed to threads in rotation; ``(0,)`` when empty.
    """

    name = "thread_local"

    def __init__(self, factory: Callable[[int], Any] | None = None, devices: Sequence[int] = (0,)) -> None:
        if factory is None:
            from shipinfer_b200.ops import NativeImageOps

            factory = NativeImageOps
        self._factory = factory
        self._devices = tuple(int(d) for d in devices) or (0,)
        self._local = threading.local()
        self._lock = threading.Lock()
        self._handed_out = 0                 # device slots given to threads, failed builds included
        self._built: dict[int, int] = {}     # device -> delegates that exist

    def delegate(self) -> Any:
        """The calling thread's ops instance, built (and bound to its device) on first use."""
        ops = getattr(self._local, "ops", None)
        if ops is not None:
            return ops
        with self._lock:
            device = self._devices[self._handed_out % len(self._devices)]
            self._handed_out += 1
        ops = self._factory(device)  # outside the lock: it creates a CUDA context and staging
        with self._lock:
            self._built[device] = self._built.get(device, 0) + 1
        self._local.ops = ops
        self._local.device = device
        return ops

    def device_of_this_thread(self) -> int | None:
        """The device the calling thread's delegate is bound to, or None before its first call."""
        return getattr(self._local, "device", None)

    def assignments(self) -> dict[int, int]:
        """``device -> delegates built``: how many threads preprocess on each GPU."""
        with self._lock:
            return dict(self._built)

    @property
    def on_device(self) -> bool:
        return bool(getattr(self.delegate(), "on_device", False))

    # ---- the reference seam (``ImageOps``), delegated ----

    def letterbox_batch(
        self, images: Sequence[np.ndarray], dst_size: tuple[int, int], params: NormalizeParams, *, pad_value: int = 114
    ) -> LetterboxResult:
        return self.delegate().letterbox_batch(images, dst_size, params, pad_value=pad_value)

    def letterbox_to_device(
        self, images: Sequence[np.ndarray], out: Any, params: NormalizeParams, *, pad_value: int = 114
    ) -> tuple[np.ndarray, np.ndarray]:
        return self.delegate().letterbox_to_device(images, out, params, pad_value=pad_value)

    def crop_batch(
        self, image: np.ndarray, boxes: np.ndarray, dst_size: tuple[int, int], params: NormalizeParams
    ) -> np.ndarray:
        return self.delegate().crop_batch(image, boxes, dst_size, params)

    def nms(
        self, boxes: np.ndarray, scores: np.ndarray, iou_threshold: float, score_threshold: float, max_output: int
    ) -> np.ndarray:
        return self.delegate().nms(boxes, scores, iou_threshold, score_threshold, max_output)

    def describe(self) -> str:
        return f"thread_local over devices {list(self._devices)}"

    def __getattr__(self, attr: str) -> Any:
        # the device-resident API (letterbox_device, crop_device, nms_device, ...) of the
        # calling thread's delegate
        if attr.startswith("_"):
            raise AttributeError(attr)
        return getattr(self.delegate(), attr)
