"""TEST INFRASTRUCTURE ONLY: numpy-facing wrapper of the C oracle (``oracle.c``).

Only ``tests/``, ``__graft_entry__.smoke()`` and ``bench.py``'s CPU-baseline arm import this
module, and only as the checker or as the timed CPU baseline. The product package
(``shipinfer_b200``) never imports it and has no CPU fallback.

Every function restates one reference formulation (file:line cited in ``oracle.c``):

* :func:`letterbox_fit` — ``torch_ops.py:373-379``;
* :func:`letterbox` — ``TorchImageOps._letterbox`` (``torch_ops.py:349-403``) with
  ``F.interpolate`` in its CUDA formulation;
* :func:`crop` — ``TorchImageOps.crop_batch`` + ``_bilinear_axis``
  (``torch_ops.py:405-507,574-614``), batched over frames;
* :func:`nms` / :func:`nms_batched` — ``NumpyImageOps.nms`` (``numpy_ops.py:120-155``), plus
  the per-class merge for class-aware suppression;
* :func:`letterbox_nv12` — ``nv12_letterbox_kernel`` (``csrc/shipinfer/runtime/ops.cu:148-194``)
  for BT.601/nearest, and this build's BT.709/bilinear definition (parity unpinned).
"""

from __future__ import annotations

import ctypes
import os
import subprocess
from collections.abc import Sequence
from pathlib import Path

import numpy as np

_HERE = Path(__file__).resolve().parent
_LIB_PATH = _HERE / "_build" / "liborc.so"
_lib: ctypes.CDLL | None = None


class _Fit(ctypes.Structure):
    _fields_ = [
        ("scale", ctypes.c_float),
        ("pad_x", ctypes.c_int),
        ("pad_y", ctypes.c_int),
        ("new_w", ctypes.c_int),
        ("new_h", ctypes.c_int),
    ]


class _Frame(ctypes.Structure):
    _fields_ = [
        ("data", ctypes.c_void_p),
        ("h", ctypes.c_int),
        ("w", ctypes.c_int),
        ("pitch", ctypes.c_int64),
    ]


class _Nv12(ctypes.Structure):
    _fields_ = [
        ("data", ctypes.c_void_p),
        ("h", ctypes.c_int),
        ("w", ctypes.c_int),
        ("pitch", ctypes.c_int64),
        ("uv_offset", ctypes.c_int64),
    ]


def build() -> Path:
    """Compile the oracle with its Makefile (a no-op when it is up to date)."""
    subprocess.run(["make", "-s", "-C", str(_HERE)], check=True)
    return _LIB_PATH


def lib() -> ctypes.CDLL:
    global _lib
    if _lib is None:
        if not _LIB_PATH.exists():
            build()
        _lib = ctypes.CDLL(str(_LIB_PATH))
        _lib.orc_letterbox_fit.restype = _Fit
        _lib.orc_letterbox_fit.argtypes = [ctypes.c_int] * 4
        _lib.orc_letterbox_fit_f32.restype = _Fit
        _lib.orc_letterbox_fit_f32.argtypes = [ctypes.c_int] * 4
        _lib.orc_nms.restype = ctypes.c_int
    return _lib


def _fptr(a: np.ndarray):
    return a.ctypes.data_as(ctypes.c_void_p)


def _floats3(values: Sequence[float]) -> ctypes.Array:
    return (ctypes.c_float * 3)(*[float(np.float32(v)) for v in values])


def letterbox_fit(src_h: int, src_w: int, dst_h: int, dst_w: int) -> tuple[float, int, int, int, int]:
    """``(scale, pad_x, pad_y, new_w, new_h)`` as the reference places a frame."""
    f = lib().orc_letterbox_fit(src_h, src_w, dst_h, dst_w)
    return f.scale, f.pad_x, f.pad_y, f.new_w, f.new_h


def letterbox_fit_f32(src_h: int, src_w: int, dst_h: int, dst_w: int) -> tuple[float, int, int, int, int]:
    """``(scale, pad_x, pad_y, new_w, new_h)`` as the reference's C++ data plane places a frame
    (``csrc/shipinfer/runtime/ops.cu:341-356``, float32 arithmetic)."""
    f = lib().orc_letterbox_fit_f32(src_h, src_w, dst_h, dst_w)
    return f.scale, f.pad_x, f.pad_y, f.new_w, f.new_h


def _frames(images: Sequence[np.ndarray]) -> tuple[ctypes.Array, list[np.ndarray]]:
    keep = []
    arr = (_Frame * len(images))()
    for i, img in enumerate(images):
        if img.ndim != 3 or img.shape[2] != 3 or img.dtype != np.uint8:
            raise ValueError(f"image {i}: expected (H, W, 3) uint8, got {img.shape} {img.dtype}")
        if img.strides[1] != 3 or img.strides[2] != 1:
            img = np.ascontiguousarray(img)
        keep.append(img)
        arr[i] = _Frame(img.ctypes.data, img.shape[0], img.shape[1], img.strides[0])
    return arr, keep


def _threads(threads: int | None) -> int:
    # Default: every CPU this process may run on, explicitly, so that an OMP_NUM_THREADS a
    # launcher set for its workers (torchrun sets 1) does not shrink the CPU baseline.
    return cpu_threads() if threads is None else int(threads)


def letterbox(
    images: Sequence[np.ndarray],
    dst_size: tuple[int, int],
    mean: Sequence[float] = (0.0, 0.0, 0.0),
    std: Sequence[float] = (255.0, 255.0, 255.0),
    swap_rb: bool = True,
    pad_value: float = 114.0,
    threads: int | None = None,
    cpp_fit: bool = False,
) -> np.ndarray:
    """float32 ``(n, 3, H, W)``: the reference letterbox on uint8 BGR frames. ``cpp_fit``
    places frames with the C++ data plane's float32 rule instead of the Python plane's."""
    dst_h, dst_w = dst_size
    frames, _keep = _frames(images)
    out = np.empty((len(images), 3, dst_h, dst_w), dtype=np.float32)
    lib().orc_letterbox_u8_fit(
        frames, ctypes.c_int(len(images)), ctypes.c_int(dst_h), ctypes.c_int(dst_w),
        _floats3(mean), _floats3(std), ctypes.c_int(int(swap_rb)),
        ctypes.c_float(pad_value), ctypes.c_int(int(cpp_fit)), _fptr(out), ctypes.c_int(_threads(threads)),
    )
    return out


def crop(
    images: Sequence[np.ndarray],
    boxes: np.ndarray,
    dst_size: tuple[int, int],
    frame_index: np.ndarray | None = None,
    mean: Sequence[float] = (0.0, 0.0, 0.0),
    std: Sequence[float] = (255.0, 255.0, 255.0),
    swap_rb: bool = True,
    threads: int | None = None,
) -> np.ndarray:
    """float32 ``(N, 3, h, w)``: the reference crop of box ``i`` from ``images[frame_index[i]]``."""
    dst_h, dst_w = dst_size
    boxes = np.ascontiguousarray(boxes, dtype=np.float32).reshape(-1, 4)
    n = boxes.shape[0]
    frames, _keep = _frames(images)
    idx = None
    if frame_index is not None:
        idx = np.ascontiguousarray(frame_index, dtype=np.int32)
    out = np.empty((n, 3, dst_h, dst_w), dtype=np.float32)
    if n == 0:
        return out
    lib().orc_crop_u8(
        frames, ctypes.c_int(len(images)), _fptr(boxes),
        None if idx is None else _fptr(idx), ctypes.c_int(n), ctypes.c_int(dst_h),
        ctypes.c_int(dst_w), _floats3(mean), _floats3(std), ctypes.c_int(int(swap_rb)),
        _fptr(out), ctypes.c_int(_threads(threads)),
    )
    return out


def nms(
    boxes: np.ndarray, scores: np.ndarray, iou_threshold: float, score_threshold: float,
    max_output: int,
) -> np.ndarray:
    """int64 kept indices, class-agnostic, exactly as ``NumpyImageOps.nms``."""
    boxes = np.ascontiguousarray(boxes, dtype=np.float32).reshape(-1, 4)
    scores = np.ascontiguousarray(scores, dtype=np.float32).reshape(-1)
    keep = np.empty(max(int(max_output), 1), dtype=np.int64)
    k = lib().orc_nms(
        _fptr(boxes), _fptr(scores), ctypes.c_int(boxes.shape[0]),
        ctypes.c_float(iou_threshold), ctypes.c_float(score_threshold),
        ctypes.c_int(int(max_output)), _fptr(keep),
    )
    return keep[:k].copy()


def nms_batched(
    boxes: np.ndarray,
    scores: np.ndarray,
    classes: np.ndarray | None,
    iou_threshold: float,
    score_threshold: float,
    max_output: int,
    num_classes: int = 1,
    class_aware: bool = True,
    threads: int | None = None,
) -> tuple[np.ndarray, np.ndarray]:
    """``(keep int64 [B, max_output] -1 padded, counts int32 [B])``."""
    boxes = np.ascontiguousarray(boxes, dtype=np.float32)
    B, n = boxes.shape[0], boxes.shape[1]
    scores = np.ascontiguousarray(scores, dtype=np.float32).reshape(B, n)
    if classes is None:
        classes = np.zeros((B, n), dtype=np.int32)
        class_aware = False
    classes = np.ascontiguousarray(classes, dtype=np.int32).reshape(B, n)
    keep = np.empty((B, max(int(max_output), 0)), dtype=np.int64)
    counts = np.empty(B, dtype=np.int32)
    lib().orc_nms_batched(
        _fptr(boxes), _fptr(scores), _fptr(classes), ctypes.c_int(B), ctypes.c_int(n),
        ctypes.c_int(num_classes), ctypes.c_int(int(class_aware)),
        ctypes.c_float(iou_threshold), ctypes.c_float(score_threshold),
        ctypes.c_int(int(max_output)), _fptr(keep), _fptr(counts),
        ctypes.c_int(_threads(threads)),
    )
    return keep, counts


def crop_nv12(
    planes: Sequence[tuple[np.ndarray, int, int, int, int]],
    boxes: np.ndarray,
    dst_size: tuple[int, int],
    box_frame: np.ndarray | None = None,
    swap_rb: bool = True,
    threads: int | None = None,
) -> np.ndarray:
    """float32 [n, 3, dst_h, dst_w] crops from NV12 surfaces ``(buffer, h, w, pitch,
    uv_offset)``, as the reference's nv12_crop_resize_kernel."""
    arr = (_Nv12 * len(planes))()
    keep = []
    for i, (buf, h, w, pitch, uv_offset) in enumerate(planes):
        buf = np.ascontiguousarray(buf, dtype=np.uint8)
        keep.append(buf)
        arr[i] = _Nv12(buf.ctypes.data, h, w, pitch, uv_offset)
    boxes = np.ascontiguousarray(boxes, dtype=np.float32).reshape(-1, 4)
    n = boxes.shape[0]
    bf = None if box_frame is None else np.ascontiguousarray(box_frame, dtype=np.int32)
    out = np.empty((n, 3, dst_size[0], dst_size[1]), np.float32)
    lib().orc_crop_nv12(
        arr, ctypes.c_int(len(planes)), _fptr(boxes), None if bf is None else _fptr(bf), ctypes.c_int(n),
        ctypes.c_int(dst_size[0]), ctypes.c_int(dst_size[1]), ctypes.c_int(int(swap_rb)), _fptr(out),
        ctypes.c_int(_threads(threads)),
    )
    return out


def decode(
    rows: np.ndarray,
    *,
    score_threshold: float,
    max_detections: int,
    scale: float = 1.0,
    pad: tuple[float, float] = (0.0, 0.0),
    frame_hw: tuple[int, int] | None = None,
    count: int | None = None,
) -> tuple[np.ndarray, np.ndarray, np.ndarray, int]:
    """``(boxes f32 [k,4], scores f32 [k], class_ids int32 [k], discarded)`` as the reference's
    ``decode_detections`` returns them for one frame."""
    rows = np.ascontiguousarray(rows, dtype=np.float32).reshape(-1, 6)
    R = rows.shape[0]
    cap = max(0, min(int(max_detections), R))
    boxes = np.empty((max(cap, 1), 4), np.float32)
    scores = np.empty(max(cap, 1), np.float32)
    classes = np.empty(max(cap, 1), np.int32)
    discarded = ctypes.c_int(0)
    h, w = frame_hw if frame_hw is not None else (-1, -1)
    m = lib().orc_decode(
        _fptr(rows), ctypes.c_int(R), ctypes.c_int(-1 if count is None else int(count)),
        ctypes.c_float(scale), ctypes.c_float(pad[0]), ctypes.c_float(pad[1]), ctypes.c_int(h),
        ctypes.c_int(w), ctypes.c_float(score_threshold), ctypes.c_int(int(max_detections)),
        _fptr(boxes), _fptr(scores), _fptr(classes), ctypes.byref(discarded),
    )
    return boxes[:m].copy(), scores[:m].copy(), classes[:m].copy(), int(discarded.value)


def mask_area(
    rows: np.ndarray,
    protos: np.ndarray,
    *,
    prefix: int,
    score_threshold: float,
    mask_threshold: float,
    crop_hw: tuple[int, int],
    threads: int | None = None,
) -> np.ndarray:
    """float32 areas [crops] as the reference's mask_area_into computes them. rows:
    [crops, candidates, stride]; protos: [crops, channels, cells] (any trailing shape)."""
    rows = np.ascontiguousarray(rows, dtype=np.float32)
    crops, candidates, stride = rows.shape
    protos = np.ascontiguousarray(protos, dtype=np.float32).reshape(crops, -1)
    channels = stride - prefix
    cells = protos.shape[1] // channels
    areas = np.empty(crops, np.float32)
    lib().orc_mask_area(
        _fptr(rows), ctypes.c_int(crops), ctypes.c_int(candidates), ctypes.c_int(stride), ctypes.c_int(prefix),
        _fptr(protos), ctypes.c_int(channels), ctypes.c_int(cells), ctypes.c_float(score_threshold),
        ctypes.c_float(mask_threshold), ctypes.c_int(crop_hw[0]), ctypes.c_int(crop_hw[1]), _fptr(areas),
        ctypes.c_int(_threads(threads)),
    )
    return areas


def decode_batched(
    rows: np.ndarray,
    *,
    score_threshold: float,
    max_detections: int,
    scales: np.ndarray,
    pads: np.ndarray,
    frame_hw: np.ndarray | None = None,
    counts: np.ndarray | None = None,
    threads: int | None = None,
) -> tuple[np.ndarray, np.ndarray, np.ndarray, np.ndarray, np.ndarray]:
    """:func:`decode` over a batch ``rows [B, R, 6]`` on the host cores: ``(boxes [B,cap,4],
    scores [B,cap], class_ids [B,cap], counts [B], discarded [B])``, valid up to counts[b]."""
    rows = np.ascontiguousarray(rows, dtype=np.float32)
    B, R = rows.shape[0], rows.shape[1]
    cap = max(int(max_detections), 0)
    boxes = np.zeros((B, max(cap, 1), 4), np.float32)
    scores = np.zeros((B, max(cap, 1)), np.float32)
    classes = np.zeros((B, max(cap, 1)), np.int32)
    out_counts = np.zeros(B, np.int32)
    discarded = np.zeros(B, np.int32)
    scales = np.ascontiguousarray(scales, dtype=np.float32)
    pads = np.ascontiguousarray(pads, dtype=np.float32)
    hw = None if frame_hw is None else np.ascontiguousarray(frame_hw, dtype=np.int32)
    cnt = None if counts is None else np.ascontiguousarray(counts, dtype=np.int32)
    lib().orc_decode_batched(
        _fptr(rows), ctypes.c_int(B), ctypes.c_int(R), None if cnt is None else _fptr(cnt), _fptr(scales),
        _fptr(pads), None if hw is None else _fptr(hw), ctypes.c_float(score_threshold), ctypes.c_int(int(max_detections)),
        _fptr(boxes), _fptr(scores), _fptr(classes), _fptr(out_counts), _fptr(discarded), ctypes.c_int(_threads(threads)),
    )
    return boxes[:, :cap], scores[:, :cap], classes[:, :cap], out_counts, discarded


def letterbox_nv12(
    planes: Sequence[tuple[np.ndarray, int, int, int, int]],
    dst_size: tuple[int, int],
    mean: Sequence[float] = (0.0, 0.0, 0.0),
    std: Sequence[float] = (255.0, 255.0, 255.0),
    swap_rb: bool = True,
    pad_value: float = 114.0,
    matrix: int = 709,
    sampling: int = 1,
    threads: int | None = None,
    cpp_fit: bool = False,
) -> np.ndarray:
    """NV12 frames given as ``(buffer uint8 1-D, h, w, pitch, uv_offset)``; ``cpp_fit`` as in
    :func:`letterbox`."""
    dst_h, dst_w = dst_size
    arr = (_Nv12 * len(planes))()
    keep = []
    for i, (buf, h, w, pitch, uv_offset) in enumerate(planes):
        buf = np.ascontiguousarray(buf, dtype=np.uint8)
        keep.append(buf)
        arr[i] = _Nv12(buf.ctypes.data, h, w, pitch, uv_offset)
    out = np.empty((len(planes), 3, dst_h, dst_w), dtype=np.float32)
    lib().orc_letterbox_nv12_fit(
        arr, ctypes.c_int(len(planes)), ctypes.c_int(dst_h), ctypes.c_int(dst_w),
        _floats3(mean), _floats3(std), ctypes.c_int(int(swap_rb)), ctypes.c_float(pad_value),
        ctypes.c_int(matrix), ctypes.c_int(sampling), ctypes.c_int(int(cpp_fit)), _fptr(out),
        ctypes.c_int(_threads(threads)),
    )
    return out


def cpu_threads() -> int:
    """Host threads the oracle's OpenMP loops use by default: the process's CPU affinity."""
    try:
        return len(os.sched_getaffinity(0))
    except AttributeError:  # pragma: no cover - non-Linux
        return os.cpu_count() or 1
