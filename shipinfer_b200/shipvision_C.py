"""A drop-in for the ``shipvision._C`` extension module, backed by ``libshipk.so``.

The reference loads its fused kernels as ``shipvision._C`` (``src/shipinfer/runtime/native.py:
47-93``) and reads this surface off it; ``tests/runtime/test_native_reachable.py`` pins it:

* ``cuda_available()`` -> bool — the probe ``native_module()`` and ``NativeImageOps`` require;
* ``__version__`` (str attribute), ``platform`` (str attribute, not callable),
  ``device_count()`` -> int;
* ``ImageOps(device_index)`` with ``letterbox_into`` (3 return values), ``letterbox_batch``
  (4), ``crop_batch`` and ``nms`` with the argument lists ``native_ops.py:158-232`` passes.

Registering this module under that name (``sys.modules["shipvision._C"] = this``, or a
``shipvision/_C.py`` that star-imports it) makes the reference's ``NativeImageOps`` and
``execution.provider=native`` run on the B200 kernels with no change on the reference side.
"""

from __future__ import annotations

import sys
from collections.abc import Sequence
from types import ModuleType
from typing import Any

import numpy as np

from shipinfer_b200 import _native
from shipinfer_b200.ops import NativeImageOps
from shipinfer_b200.types import NormalizeParams

__all__ = ["ImageOps", "cuda_available", "device_count", "install", "platform"]

__version__: str = _native.lib().shipk_version().decode()
platform: str = "cuda"


def install(name: str = "shipvision._C") -> ModuleType:
    """Register this module as ``name`` (and its parent package, if it has none) in
    ``sys.modules``, so ``importlib.import_module("shipvision._C")`` — what the reference's
    ``native_module()`` does (``runtime/native.py:67``) — returns it."""
    module = sys.modules[__name__]
    parent, _, child = name.rpartition(".")
    if parent and parent not in sys.modules:
        package = ModuleType(parent)
        package.__path__ = []  # a namespace-like package: submodules come from sys.modules
        sys.modules[parent] = package
    sys.modules[name] = module
    if parent:
        setattr(sys.modules[parent], child, module)
    return module


def cuda_available() -> bool:
    """True when the sm_100a kernels have a device to run on."""
    return bool(_native.lib().shipk_cuda_available())


def device_count() -> int:
    return int(_native.lib().shipk_device_count())


def _params(mean: Sequence[float], std: Sequence[float], swap_rb: bool) -> NormalizeParams:
    return NormalizeParams(mean=tuple(float(m) for m in mean), std=tuple(float(s) for s in std),
                           swap_rb=bool(swap_rb))


class ImageOps:
    """``shipvision._C.ImageOps``: one per thread, bound to one device."""

    def __init__(self, device_index: int) -> None:
        self._ops = NativeImageOps(device_index=device_index, stream=0)
        self._device_index = int(device_index)

    def letterbox_into(
        self,
        images: Sequence[np.ndarray],
        out_ptr: int,
        out_nbytes: int,
        dst_h: int,
        dst_w: int,
        mean: Sequence[float],
        std: Sequence[float],
        swap_rb: bool,
        pad: int,
        stream: int,
    ) -> tuple[np.ndarray, np.ndarray, np.ndarray]:
        """Host frames into float32 NCHW at ``out_ptr``; ``(scales, pads, extents)``."""
        import ctypes

        ops = self._ops
        if not images:
            raise ValueError("letterbox needs at least one image")
        frames, _keep = ops._host_frames(images)
        n = len(images)
        maps = (_native.LetterboxMap * n)()
        p = _params(mean, std, swap_rb)
        lib = _native.lib()
        import torch

        with torch.cuda.device(self._device_index):
            _native.check(
                lib.shipk_ctx_letterbox_host(
                    ops._ctx, frames, n, int(out_ptr), _native.DTYPE_F32, int(out_nbytes), int(dst_h),
                    int(dst_w), _native.floats3(p.mean), _native.floats3(p.std), int(p.swap_rb),
                    float(pad), maps, ctypes.c_void_p(int(stream)) if stream else None,
                )
            )
        return ops._maps(maps, n)

    def letterbox_batch(
        self,
        images: Sequence[np.ndarray],
        dst_h: int,
        dst_w: int,
        mean: Sequence[float],
        std: Sequence[float],
        swap_rb: bool,
        pad: int,
        stream: int,
    ) -> tuple[np.ndarray, np.ndarray, np.ndarray, np.ndarray]:
        r = self._with_stream(stream).letterbox_batch(
            list(images), (int(dst_h), int(dst_w)), _params(mean, std, swap_rb), pad_value=pad
        )
        return r.tensor, r.scales, r.pads, r.extents

    def crop_batch(
        self,
        image: np.ndarray,
        boxes: np.ndarray,
        dst_h: int,
        dst_w: int,
        mean: Sequence[float],
        std: Sequence[float],
        swap_rb: bool,
        stream: int,
    ) -> np.ndarray:
        return self._with_stream(stream).crop_batch(
            image, boxes, (int(dst_h), int(dst_w)), _params(mean, std, swap_rb)
        )

    def nms(
        self,
        boxes: np.ndarray,
        scores: np.ndarray,
        iou_threshold: float,
        score_threshold: float,
        max_output: int,
        stream: int,
    ) -> np.ndarray:
        return self._with_stream(stream).nms(boxes, scores, iou_threshold, score_threshold, max_output)

    def _with_stream(self, stream: int) -> Any:
        self._ops._stream = int(stream)
        return self._ops
