"""Detector decode on the device: detector rows -> source-frame detections.

Mirrors the reference's ``decode_detections`` (``src/shipinfer/topology/elements/detections.py:
423-515``) — same arguments, same ``DecodeParams`` defaults, same results bit for bit — with the
work done by ``shipk_decode_detections`` (truncate to the detector's count, score threshold,
cap by score, un-letterbox with the placement the preprocess reported, clip to the frame).

* :func:`decode_detections` — one frame from host rows, the reference's signature; returns
  :class:`Detections`.
* :func:`decode_detections_device` — a batch of frames as device tensors, one launch, results
  left on the device (for a pipeline that crops next without a host round trip).
"""

from __future__ import annotations

import ctypes
from collections.abc import Mapping
from dataclasses import dataclass, field
from typing import Any

import numpy as np

from shipinfer_b200 import _native
from shipinfer_b200.errors import ValidationError

__all__ = ["UNKNOWN_LABEL", "DecodeParams", "Detections", "decode_detections", "decode_detections_device"]

#: Label of a class id the label map does not name (reference detections.py:48).
UNKNOWN_LABEL = "unknown"
_ROW_WIDTH = 6


@dataclass(frozen=True)
class DecodeParams:
    """How a detector's raw rows become detections (reference detections.py:229-241)."""

    class_labels: Mapping[int, str] = field(default_factory=lambda: {0: "person", 8: "ship"})
    score_threshold: float = 0.25
    max_detections: int = 100


@dataclass(frozen=True)
class Detections:
    """One frame's detections in source pixels (reference detections.py:68-110)."""

    boxes: np.ndarray
    scores: np.ndarray
    class_ids: np.ndarray
    labels: tuple[str, ...] = ()
    discarded: int = 0

    def __post_init__(self) -> None:
        n = self.boxes.shape[0]
        if self.boxes.ndim != 2 or self.boxes.shape[1] != 4:
            raise ValidationError(f"detection boxes must be (N, 4), got {self.boxes.shape}")
        if self.scores.shape != (n,) or self.class_ids.shape != (n,):
            raise ValidationError(
                f"detection arrays disagree: boxes={self.boxes.shape} "
                f"scores={self.scores.shape} class_ids={self.class_ids.shape}"
            )
        if len(self.labels) != n:
            raise ValidationError(f"got {len(self.labels)} labels for {n} detections")

    @classmethod
    def empty(cls) -> Detections:
        return cls(boxes=np.zeros((0, 4), np.float32), scores=np.zeros((0,), np.float32),
                   class_ids=np.zeros((0,), np.int32), labels=())

    def __len__(self) -> int:
        return int(self.boxes.shape[0])


def _torch():
    import torch

    return torch


def _ptr(t: Any) -> int | None:
    return int(t.data_ptr()) if t is not None and t.numel() else None


def decode_detections_device(
    rows: Any,
    scales: Any,
    pads: Any,
    *,
    score_threshold: float = 0.25,
    max_detections: int = 100,
    frame_hw: Any = None,
    counts: Any = None,
    stream: int | None = None,
) -> tuple[Any, Any, Any, Any, Any]:
    """Decode a batch on the device.

    Args:
        rows: CUDA float32 ``[B, R, 6]`` — ``[x1, y1, x2, y2, score, class]`` in letterboxed pixels.
        scales: CUDA float32 ``[B]``; pads: CUDA float32 ``[B, 2]`` (x, y) — the placement the
            letterbox reported for each frame.
        frame_hw: CUDA int32 ``[B, 2]`` source (height, width) to clip to, or ``None``.
        counts: CUDA int32 ``[B]`` rows the detector filled, or ``None``.
        stream: CUDA stream handle; torch's current stream when ``None``.

    Returns:
        ``(boxes [B, max_det, 4], scores [B, max_det], class_ids int32 [B, max_det],
        counts int32 [B], discarded int32 [B])`` on the device; slots past a frame's count hold
        zeros and class -1.
    """
    torch = _torch()
    if rows.dim() != 3 or int(rows.shape[2]) != _ROW_WIDTH or rows.dtype != torch.float32 or not rows.is_contiguous():
        raise ValidationError(f"rows must be a contiguous float32 [B, R, {_ROW_WIDTH}] CUDA tensor")
    B, R = int(rows.shape[0]), int(rows.shape[1])
    if tuple(scales.shape) != (B,) or scales.dtype != torch.float32 or not scales.is_contiguous():
        raise ValidationError("scales must be a contiguous float32 [B] CUDA tensor")
    if tuple(pads.shape) != (B, 2) or pads.dtype != torch.float32 or not pads.is_contiguous():
        raise ValidationError("pads must be a contiguous float32 [B, 2] CUDA tensor")
    if frame_hw is not None and (tuple(frame_hw.shape) != (B, 2) or frame_hw.dtype != torch.int32
                                 or not frame_hw.is_contiguous()):
        raise ValidationError("frame_hw must be a contiguous int32 [B, 2] CUDA tensor")
    if counts is not None and (tuple(counts.shape) != (B,) or counts.dtype != torch.int32 or not counts.is_contiguous()):
        raise ValidationError("counts must be a contiguous int32 [B] CUDA tensor")
    cap = int(max_detections)
    dev = rows.device
    boxes = torch.empty((B, max(cap, 0), 4), dtype=torch.float32, device=dev)
    out_scores = torch.empty((B, max(cap, 0)), dtype=torch.float32, device=dev)
    class_ids = torch.empty((B, max(cap, 0)), dtype=torch.int32, device=dev)
    out_counts = torch.empty((B,), dtype=torch.int32, device=dev)
    discarded = torch.empty((B,), dtype=torch.int32, device=dev)
    handle = torch.cuda.current_stream(dev).cuda_stream if stream is None else int(stream)
    with torch.cuda.device(dev):
        _native.check(
            _native.lib().shipk_decode_detections(
                _ptr(rows), B, R, _ptr(counts), _ptr(scales), _ptr(pads), _ptr(frame_hw),
                float(score_threshold), cap, _ptr(boxes), _ptr(out_scores), _ptr(class_ids),
                int(out_counts.data_ptr()), int(discarded.data_ptr()), ctypes.c_void_p(handle),
            )
        )
    return boxes, out_scores, class_ids, out_counts, discarded


def decode_detections(
    rows: np.ndarray,
    *,
    params: DecodeParams,
    scale: float = 1.0,
    pad: tuple[float, float] = (0.0, 0.0),
    frame_hw: tuple[int, int] | None = None,
    count: int | None = None,
    device_index: int = 0,
) -> Detections:
    """One frame's detector output -> source-frame detections, as the reference's
    ``decode_detections`` (same arguments, same results), computed on device ``device_index``.
    ``scale`` is used as the float32 the letterbox reports (``LetterboxResult.scales``), which
    is what the reference's callers pass.

    Raises:
        ValidationError: the output is not ``(R, 6)``.
    """
    array = np.asarray(rows)
    if array.ndim != 2 or array.shape[1] != _ROW_WIDTH:
        raise ValidationError(
            f"detector output must be (rows, {_ROW_WIDTH}) [x1,y1,x2,y2,score,class], got {array.shape}"
        )
    total = array.shape[0] if count is None else max(0, min(int(count), array.shape[0]))
    if total == 0:
        return Detections.empty()
    torch = _torch()
    dev = torch.device("cuda", device_index)
    t_rows = torch.from_numpy(np.ascontiguousarray(array, dtype=np.float32)).reshape(1, -1, _ROW_WIDTH).to(dev)
    t_scale = torch.tensor([float(np.float32(scale))], dtype=torch.float32, device=dev)
    t_pad = torch.tensor([[float(pad[0]), float(pad[1])]], dtype=torch.float32, device=dev)
    t_hw = None if frame_hw is None else torch.tensor([[int(frame_hw[0]), int(frame_hw[1])]], dtype=torch.int32, device=dev)
    t_count = None if count is None else torch.tensor([int(count)], dtype=torch.int32, device=dev)
    boxes, scores, class_ids, counts, discarded = decode_detections_device(
        t_rows, t_scale, t_pad, score_threshold=params.score_threshold, max_detections=params.max_detections,
        frame_hw=t_hw, counts=t_count,
    )
    n = int(counts.cpu()[0])
    ids = class_ids[0, :n].cpu().numpy()
    return Detections(
        boxes=boxes[0, :n].cpu().numpy(),
        scores=scores[0, :n].cpu().numpy(),
        class_ids=ids,
        labels=tuple(params.class_labels.get(int(c), UNKNOWN_LABEL) for c in ids),
        discarded=int(discarded.cpu()[0]),
    )
