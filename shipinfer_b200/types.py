"""Value types of the image-ops seam, mirroring the reference's ``runtime/ops/base.py:32-68``."""

from __future__ import annotations

from dataclasses import dataclass

import numpy as np

__all__ = ["LetterboxResult", "NormalizeParams"]


@dataclass(frozen=True, slots=True)
class NormalizeParams:
    """Mean/std normalisation in the source pixel scale (0-255), and the channel order.

    Output value = ``(pixel - mean[c]) / std[c]`` per output channel; ``swap_rb`` turns the
    BGR source into RGB. Same fields, defaults and validation as the reference's
    ``NormalizeParams`` (``base.py:32-44``).
    """

    mean: tuple[float, float, float] = (0.0, 0.0, 0.0)
    std: tuple[float, float, float] = (255.0, 255.0, 255.0)
    swap_rb: bool = True

    def __post_init__(self) -> None:
        if any(s == 0 for s in self.std):
            raise ValueError("normalisation std must be non-zero")


@dataclass(frozen=True, slots=True)
class LetterboxResult:
    """A batched letterbox plus the placement needed to undo it (``base.py:46-68``).

    ``tensor`` is ``(N, C, H, W)``; ``scales`` float32 ``(N,)``; ``pads`` float32 ``(N, 2)`` as
    ``(pad_x, pad_y)``; ``extents`` int32 ``(N, 2)`` as ``(new_h, new_w)``.
    """

    tensor: object
    scales: np.ndarray
    pads: np.ndarray
    extents: np.ndarray
