"""Segmenter mask areas on the device: one area per crop.

Mirrors the reference's ``mask_area_into`` (``csrc/shipinfer/runtime/ops.h:117-120``,
``ops.cu:196-255,418-458``) — same arguments, same refusals, same results — on
``shipk_mask_area``: a cluster of CTAs per crop reads the prototype bank once with 16-byte
loads and meets in distributed shared memory.
"""

from __future__ import annotations

import ctypes
from typing import Any

from shipinfer_b200 import _native
from shipinfer_b200.errors import ValidationError

__all__ = ["mask_area_device"]


def mask_area_device(
    rows: Any,
    protos: Any,
    *,
    prefix: int,
    score_threshold: float,
    mask_threshold: float,
    crop_hw: tuple[int, int],
    areas: Any = None,
    stream: int | None = None,
) -> Any:
    """Areas of the segmenter's strongest instance per crop.

    Args:
        rows: CUDA float32 ``[crops, candidates, stride]`` — score in column 4, mask
            coefficients in ``[prefix, stride)``.
        protos: CUDA float32 ``[crops, channels, ...]`` prototype planes, ``channels`` equal to
            ``stride - prefix``.
        prefix: the column where the coefficients start.
        score_threshold: a strongest score below it gives area 0.
        mask_threshold: the probability a cell must reach, in (0, 1).
        crop_hw: the crop size the segmenter was fed; a cell count times
            ``h * w / cells`` is the area in crop pixels.
        areas: optional CUDA float32 ``[crops]`` to fill.
        stream: CUDA stream handle; torch's current stream when ``None``.

    Returns:
        CUDA float32 ``[crops]`` areas.
    """
    import torch

    if rows.dim() != 3 or rows.dtype != torch.float32 or not rows.is_contiguous():
        raise ValidationError("rows must be a contiguous float32 [crops, candidates, stride] CUDA tensor")
    crops, candidates, stride = (int(x) for x in rows.shape)
    if protos.dtype != torch.float32 or not protos.is_contiguous() or int(protos.shape[0]) != crops or protos.dim() < 2:
        raise ValidationError("protos must be a contiguous float32 [crops, channels, ...] CUDA tensor")
    channels = int(protos.shape[1])
    cells = int(protos[0, 0].numel()) if crops else 0
    if areas is None:
        areas = torch.empty((crops,), dtype=torch.float32, device=rows.device)
    handle = torch.cuda.current_stream(rows.device).cuda_stream if stream is None else int(stream)
    with torch.cuda.device(rows.device):
        _native.check(
            _native.lib().shipk_mask_area(
                int(rows.data_ptr()) if rows.numel() else None, candidates, stride, int(prefix),
                int(protos.data_ptr()) if protos.numel() else None, channels, cells, crops,
                float(score_threshold), float(mask_threshold), int(crop_hw[0]), int(crop_hw[1]),
                int(areas.data_ptr()) if areas.numel() else None, ctypes.c_void_p(handle),
            )
        )
    return areas
