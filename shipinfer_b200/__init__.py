"""shipinfer_b200 — B200-native (sm_100a) data-plane image kernels for ShipInfer.

The hot path of ShipInfer's image-ops seam — fused letterbox (BGR or NV12), batched ROI
crop-resize, and device NMS — as hand-written CUDA behind the C ABI in ``include/shipk.h``.

* :class:`NativeImageOps` — the reference's ``ImageOps`` seam (``letterbox_batch``,
  ``letterbox_to_device``, ``crop_batch``, ``nms``) plus the device-resident batched API.
* :class:`ThreadLocalImageOps` — one ``NativeImageOps`` per worker thread, threads spread
  over the GPUs in rotation (the reference's multi-GPU preprocessing wrapper).
* :mod:`shipinfer_b200.shipvision_C` — the ``shipvision._C`` surface the reference's loader
  probes, for a drop-in under ``execution.provider=native``.

Build the library with ``python -m shipinfer_b200.build``. Nothing here falls back to the CPU.
"""

from shipinfer_b200.errors import ConfigurationError, NativeError, ValidationError
from shipinfer_b200.ops import NativeImageOps, Nv12Frame, check_device_output, nms_workspace_bytes
from shipinfer_b200.thread_local import ThreadLocalImageOps
from shipinfer_b200.types import LetterboxResult, NormalizeParams

__all__ = [
    "ConfigurationError",
    "LetterboxResult",
    "NativeError",
    "NativeImageOps",
    "NormalizeParams",
    "Nv12Frame",
    "ThreadLocalImageOps",
    "ValidationError",
    "check_device_output",
    "nms_workspace_bytes",
]

__version__ = "0.1.0"
