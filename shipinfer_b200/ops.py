"""The image-ops seam on the shipk kernels.

:class:`NativeImageOps` mirrors the reference's ``NativeImageOps``
(``src/shipinfer/runtime/ops/native_ops.py:75-235``): same constructor, same methods
(``letterbox_batch``, ``letterbox_to_device``, ``crop_batch``, ``nms``), same arguments, same
exceptions (``ValidationError`` for an output tensor it cannot legally write, and
``ConfigurationError`` for a missing or unusable build). Host numpy frames go through the
library's per-instance staging context, which uploads only the source rows the resize reads.

It also carries the device-resident API the batched kernels allow and the reference's seam
cannot express: ``letterbox_device`` / ``letterbox_nv12_device`` (frames already on the GPU,
written into a caller-owned fp32 or fp16 tensor), ``crop_device`` (every box of every frame in
one launch) and ``nms_device`` (batched, optionally class-aware, results left on the device).

One instance per thread, as the reference requires (``thread_local.py:14-24``): the staging
context is reused across calls and is not safe to share.
"""

from __future__ import annotations

import ctypes
from collections.abc import Sequence
from dataclasses import dataclass
from typing import Any

import numpy as np

from shipinfer_b200 import _native
from shipinfer_b200.errors import ConfigurationError, ValidationError
from shipinfer_b200.types import LetterboxResult, NormalizeParams

__all__ = ["NativeImageOps", "Nv12Frame", "check_device_output", "nms_workspace_bytes"]

#: Bytes per chunk of a staged device-to-host copy (NativeImageOps._to_host).
STAGE_BYTES = 8 << 20


def _torch():
    try:
        import torch
    except ImportError as exc:  # pragma: no cover - torch is a hard dependency here
        raise ConfigurationError("shipinfer_b200 needs torch for device tensors") from exc
    return torch


def check_device_output(
    out: Any,
    *,
    device_index: int,
    rows: int,
    caller: str,
    dtypes: tuple[str, ...] = ("float32",),
) -> None:
    """Reject an output tensor the kernels cannot legally write into.

    The checks and messages of the reference's ``check_device_output``
    (``native_ops.py:22-72``): CUDA, the bound device, the dtype, rank 4 with C=3, contiguous,
    at least ``rows`` rows. ``dtypes`` widens the dtype rule to fp16 where the call writes it.
    """
    torch = _torch()
    if not getattr(out, "is_cuda", False):
        raise ValidationError(
            f"{caller} needs a CUDA tensor; got one on {getattr(out, 'device', 'the host')}"
        )
    index = out.device.index
    if index != device_index:
        raise ValidationError(
            f"{caller} was given a tensor on cuda:{index} but these ops are bound to "
            f"cuda:{device_index}; a cross-device write is refused"
        )
    allowed = [getattr(torch, d) for d in dtypes]
    if out.dtype not in allowed:
        names = " or ".join(dtypes)
        raise ValidationError(f"{caller} writes {names}; the output tensor is {out.dtype}")
    if out.dim() != 4 or int(out.shape[1]) != 3:
        raise ValidationError(
            f"{caller} needs an (N, 3, H, W) output tensor; got {tuple(out.shape)}"
        )
    if not out.is_contiguous():
        raise ValidationError(
            f"{caller} writes contiguous NCHW; the output tensor is not contiguous "
            f"(shape {tuple(out.shape)}, strides {tuple(out.stride())}) — a channels-last "
            "or sliced tensor would be filled as though it were NCHW"
        )
    if int(out.shape[0]) < rows:
        raise ValidationError(
            f"{caller} output holds {int(out.shape[0])} rows but the batch has {rows}"
        )


def _dtype_code(out: Any) -> int:
    torch = _torch()
    return _native.DTYPE_F32 if out.dtype == torch.float32 else _native.DTYPE_F16


def _nbytes(t: Any) -> int:
    return int(t.numel() * t.element_size())


@dataclass(frozen=True)
class Nv12Frame:
    """An NV12 surface on the device: ``buffer`` (uint8 CUDA tensor) holds the luma plane at
    offset 0 and the interleaved chroma plane at ``uv_offset``; both use ``pitch`` bytes per
    row (NVDEC's padded surfaces included)."""

    buffer: Any
    height: int
    width: int
    pitch: int
    uv_offset: int

    @classmethod
    def tight(cls, buffer: Any, height: int, width: int) -> Nv12Frame:
        return cls(buffer, height, width, width, width * height)


def nms_workspace_bytes(batch: int, n: int, num_classes: int, class_aware: bool, max_det: int) -> int:
    return int(
        _native.lib().shipk_nms_workspace_bytes(batch, n, num_classes, int(class_aware), max_det)
    )


class NativeImageOps:
    """Fused sm_100a kernels behind the reference's ``ImageOps`` interface."""

    name = "native"
    on_device = True

    def __init__(self, device_index: int = 0, stream: int | None = None) -> None:
        """Bind to the library and one device, or say precisely why that is impossible.

        Raises:
            ConfigurationError: the library is not built, or no device can run its sm_100a
                kernels — a missing build and an unusable one are one operational event, as
                in the reference (``native_ops.py:96-127``).
        """
        self._lib = _native.lib()
        if not self._lib.shipk_cuda_available():
            raise ConfigurationError(
                "shipk is built but reports no usable GPU kernels — it needs an sm_100 (B200) "
                "device visible to this process"
            )
        if not 0 <= device_index < self._lib.shipk_device_count():
            raise ConfigurationError(f"cuda:{device_index} is not a visible device")
        self._device_index = int(device_index)
        self._stream = stream
        handle = ctypes.c_void_p()
        _native.check(self._lib.shipk_ctx_create(self._device_index, ctypes.byref(handle)))
        self._ctx = handle
        self._nms_ws: Any = None
        self._nms_key: tuple[int, ...] | None = None
        self._stage: Any = None  # two pinned chunk buffers and their events, made on first use

    def __del__(self) -> None:  # pragma: no cover - interpreter shutdown order varies
        ctx = getattr(self, "_ctx", None)
        if ctx:
            try:
                self._lib.shipk_ctx_destroy(ctx)
            except Exception:
                pass
            self._ctx = None

    # -- helpers --------------------------------------------------------------------------

    @property
    def device_index(self) -> int:
        return self._device_index

    def _stream_handle(self) -> int:
        if self._stream is not None:
            return int(self._stream)
        torch = _torch()
        return int(torch.cuda.current_stream(self._device_index).cuda_stream)

    def _device_guard(self):
        return _torch().cuda.device(self._device_index)

    def _torch_stream(self) -> Any:
        """The stream this instance launches on, as a torch stream object."""
        torch = _torch()
        handle = self._stream_handle()
        if handle == 0:
            return torch.cuda.default_stream(self._device_index)
        return torch.cuda.ExternalStream(handle, device=torch.device("cuda", self._device_index))

    def _to_host(self, t: Any) -> np.ndarray:
        """``t`` (a contiguous CUDA tensor this instance wrote on its stream) as a fresh host array
        the caller owns. Results above STAGE_BYTES cross PCIe in chunks through two pinned
        buffers, each chunk's DMA in flight while the host copies the one before out of the other
        (the reference's ping-pong staging, torch_ops.py:187-296): a copy into pageable memory
        goes through the driver's own bounce buffer at a fraction of the link's speed. Smaller
        results are copied directly, as the reference does for a single span."""
        torch = _torch()
        host = torch.empty(tuple(t.shape), dtype=t.dtype)
        nbytes = t.numel() * t.element_size()
        stream = self._torch_stream()
        with torch.cuda.device(self._device_index), torch.cuda.stream(stream):
            if nbytes <= STAGE_BYTES:
                host.copy_(t)
                return host.numpy()
            if self._stage is None:
                self._stage = ([torch.empty(STAGE_BYTES, dtype=torch.uint8).pin_memory() for _ in range(2)],
                               [torch.cuda.Event() for _ in range(2)])
            bufs, events = self._stage
            src = t.reshape(-1).view(torch.uint8)
            dst = host.reshape(-1).view(torch.uint8)
            spans = [(lo, min(lo + STAGE_BYTES, nbytes)) for lo in range(0, nbytes, STAGE_BYTES)]
            for k, (lo, hi) in enumerate(spans):
                bufs[k % 2][: hi - lo].copy_(src[lo:hi], non_blocking=True)
                events[k % 2].record(stream)
                if k:
                    # drain the previous chunk while this one's DMA runs; a buffer is refilled two
                    # chunks on, after its host copy has finished (host order)
                    plo, phi = spans[k - 1]
                    events[(k - 1) % 2].synchronize()
                    dst[plo:phi].copy_(bufs[(k - 1) % 2][: phi - plo])
            lo, hi = spans[-1]
            events[(len(spans) - 1) % 2].synchronize()
            dst[lo:hi].copy_(bufs[(len(spans) - 1) % 2][: hi - lo])
        return host.numpy()

    @staticmethod
    def _host_frames(images: Sequence[np.ndarray]) -> tuple[ctypes.Array, list[np.ndarray]]:
        keep = []
        arr = (_native.HostFrameU8 * len(images))()
        for i, img in enumerate(images):
            img = np.asarray(img)
            if img.ndim != 3 or img.shape[2] != 3:
                raise ValueError(f"image {i}: expected (H, W, 3), got {img.shape}")
            if img.dtype != np.uint8:
                raise ValidationError(f"image {i}: expected uint8 pixels, got {img.dtype}")
            if img.strides[1] != 3 or img.strides[2] != 1 or img.strides[0] < 3 * img.shape[1]:
                img = np.ascontiguousarray(img)
            keep.append(img)
            arr[i] = _native.HostFrameU8(img.ctypes.data, img.shape[0], img.shape[1], img.strides[0])
        return arr, keep

    @staticmethod
    def _device_frames(frames: Sequence[Any], device_index: int) -> ctypes.Array:
        torch = _torch()
        arr = (_native.FrameU8 * len(frames))()
        for i, f in enumerate(frames):
            if not getattr(f, "is_cuda", False) or f.device.index != device_index:
                raise ValidationError(f"frame {i} must be a uint8 tensor on cuda:{device_index}")
            if f.dtype != torch.uint8 or f.dim() != 3 or int(f.shape[2]) != 3:
                raise ValidationError(
                    f"frame {i}: expected a (H, W, 3) uint8 tensor, got {tuple(f.shape)} {f.dtype}"
                )
            if int(f.stride(2)) != 1 or int(f.stride(1)) != 3:
                raise ValidationError(f"frame {i}: pixels must be packed BGR (strides (pitch, 3, 1))")
            arr[i] = _native.FrameU8(int(f.data_ptr()), int(f.shape[0]), int(f.shape[1]), int(f.stride(0)))
        return arr

    @staticmethod
    def _maps(maps: ctypes.Array, n: int) -> tuple[np.ndarray, np.ndarray, np.ndarray]:
        scales = np.array([maps[i].scale for i in range(n)], dtype=np.float32)
        pads = np.array([(maps[i].pad_x, maps[i].pad_y) for i in range(n)], dtype=np.float32).reshape(n, 2)
        extents = np.array([(maps[i].new_h, maps[i].new_w) for i in range(n)], dtype=np.int32).reshape(n, 2)
        return scales, pads, extents

    # -- the reference seam ---------------------------------------------------------------

    def letterbox_to_device(
        self,
        images: Sequence[np.ndarray],
        out: Any,
        params: NormalizeParams,
        *,
        pad_value: int = 114,
    ) -> tuple[np.ndarray, np.ndarray]:
        """Host frames straight into a caller-owned float32 CUDA tensor (the fast path).

        Raises:
            ValidationError: if ``out`` violates the contract (see :func:`check_device_output`).
        """
        scales, pads, _extents = self._letterbox_host(
            images, out, params, pad_value, caller="letterbox_to_device"
        )
        return scales, pads

    def _letterbox_host(self, images, out, params, pad_value, *, caller, dtypes=("float32",)):
        if not images:
            raise ValueError("letterbox needs at least one image")
        check_device_output(out, device_index=self._device_index, rows=len(images), caller=caller, dtypes=dtypes)
        frames, _keep = self._host_frames(images)
        n = len(images)
        maps = (_native.LetterboxMap * n)()
        with self._device_guard():
            _native.check(
                self._lib.shipk_ctx_letterbox_host(
                    self._ctx, frames, n, int(out.data_ptr()), _dtype_code(out), _nbytes(out),
                    int(out.shape[2]), int(out.shape[3]), _native.floats3(params.mean),
                    _native.floats3(params.std), int(bool(params.swap_rb)), float(pad_value),
                    maps, self._stream_handle(),
                )
            )
        return self._maps(maps, n)

    def letterbox_batch(
        self,
        images: Sequence[np.ndarray],
        dst_size: tuple[int, int],
        params: NormalizeParams,
        *,
        pad_value: int = 114,
    ) -> LetterboxResult:
        """Fused preprocess returned as numpy (correct, and not the production path)."""
        torch = _torch()
        dst_h, dst_w = dst_size
        out = torch.empty((len(images), 3, dst_h, dst_w), dtype=torch.float32, device=f"cuda:{self._device_index}")
        scales, pads, extents = self._letterbox_host(images, out, params, pad_value, caller="letterbox_batch")
        return LetterboxResult(tensor=self._to_host(out), scales=scales, pads=pads, extents=extents)

    def crop_batch(
        self,
        image: np.ndarray,
        boxes: np.ndarray,
        dst_size: tuple[int, int],
        params: NormalizeParams,
    ) -> np.ndarray:
        """N boxes of one host frame into one float32 ``(N, 3, h, w)`` host array."""
        torch = _torch()
        dst_h, dst_w = dst_size
        boxes = np.ascontiguousarray(boxes, dtype=np.float32).reshape(-1, 4)
        n = boxes.shape[0]
        if n == 0:
            return np.empty((0, 3, dst_h, dst_w), dtype=np.float32)
        frames, _keep = self._host_frames([image])
        out = torch.empty((n, 3, dst_h, dst_w), dtype=torch.float32, device=f"cuda:{self._device_index}")
        with self._device_guard():
            _native.check(
                self._lib.shipk_ctx_crop_host(
                    self._ctx, frames, boxes.ctypes.data, n, int(out.data_ptr()), _native.DTYPE_F32,
                    _nbytes(out), dst_h, dst_w, _native.floats3(params.mean),
                    _native.floats3(params.std), int(bool(params.swap_rb)), self._stream_handle(),
                )
            )
        return self._to_host(out)

    def nms(
        self,
        boxes: np.ndarray,
        scores: np.ndarray,
        iou_threshold: float,
        score_threshold: float,
        max_output: int,
    ) -> np.ndarray:
        """Class-agnostic NMS of host arrays; int64 kept indices, exactly the numpy oracle's."""
        keep, counts = self._nms_host(
            np.asarray(boxes, dtype=np.float32).reshape(1, -1, 4),
            np.asarray(scores, dtype=np.float32).reshape(1, -1),
            None, iou_threshold, score_threshold, max_output, 1, False,
        )
        return keep[0, : int(counts[0])].copy()

    def nms_batched(
        self,
        boxes: np.ndarray,
        scores: np.ndarray,
        classes: np.ndarray | None,
        iou_threshold: float,
        score_threshold: float,
        max_det: int,
        *,
        num_classes: int | None = None,
        class_aware: bool | None = None,
    ) -> tuple[np.ndarray, np.ndarray]:
        """Host arrays ``[B, N, 4]`` / ``[B, N]`` / ``[B, N]`` -> ``(keep [B, max_det], counts [B])``."""
        boxes = np.asarray(boxes, dtype=np.float32)
        scores = np.asarray(scores, dtype=np.float32)
        if class_aware is None:
            class_aware = classes is not None
        if class_aware and num_classes is None:
            num_classes = int(np.max(classes)) + 1 if np.size(classes) else 1
        return self._nms_host(boxes, scores, classes, iou_threshold, score_threshold, max_det,
                              int(num_classes or 1), bool(class_aware))

    def _nms_host(self, boxes, scores, classes, iou, score, max_det, num_classes, class_aware):
        if boxes.ndim != 3 or boxes.shape[2] != 4:
            raise ValidationError(f"boxes must be (B, N, 4); got {boxes.shape}")
        B, n = boxes.shape[:2]
        boxes = np.ascontiguousarray(boxes, dtype=np.float32)
        scores = np.ascontiguousarray(scores, dtype=np.float32).reshape(B, n)
        cls = None
        if class_aware:
            if classes is None:
                raise ValidationError("class-aware NMS needs classes")
            cls = np.ascontiguousarray(classes, dtype=np.int32).reshape(B, n)
        max_det = int(max_det)
        keep = np.empty((B, max(max_det, 0)), dtype=np.int64)
        counts = np.empty(B, dtype=np.int32)
        with self._device_guard():
            _native.check(
                self._lib.shipk_ctx_nms_host(
                    self._ctx, boxes.ctypes.data, scores.ctypes.data,
                    None if cls is None else cls.ctypes.data, B, n, num_classes, int(class_aware),
                    float(iou), float(score), max_det, keep.ctypes.data if keep.size else None,
                    counts.ctypes.data, self._stream_handle(),
                )
            )
        return keep, counts

    def describe(self) -> str:
        return f"shipk sm_100a kernels on cuda:{self._device_index}"

    def __repr__(self) -> str:
        return f"<NativeImageOps cuda:{self._device_index}>"

    # -- device-resident API --------------------------------------------------------------

    def letterbox_device(
        self,
        frames: Sequence[Any],
        out: Any,
        params: NormalizeParams,
        *,
        pad_value: float = 114,
    ) -> tuple[np.ndarray, np.ndarray, np.ndarray]:
        """Device uint8 ``(H, W, 3)`` BGR frames into ``out`` (float32 or float16 NCHW).

        One launch for the whole batch. Returns ``(scales, pads, extents)`` computed on the
        host; nothing is synchronised.
        """
        if len(frames) == 0:
            raise ValueError("letterbox needs at least one image")
        check_device_output(out, device_index=self._device_index, rows=len(frames),
                            caller="letterbox_device", dtypes=("float32", "float16"))
        arr = self._device_frames(frames, self._device_index)
        n = len(frames)
        maps = (_native.LetterboxMap * n)()
        with self._device_guard():
            _native.check(
                self._lib.shipk_letterbox_u8(
                    arr, n, int(out.data_ptr()), _dtype_code(out), _nbytes(out), int(out.shape[2]),
                    int(out.shape[3]), _native.floats3(params.mean), _native.floats3(params.std),
                    int(bool(params.swap_rb)), float(pad_value), maps, self._stream_handle(),
                )
            )
        return self._maps(maps, n)

    def letterbox_nv12_device(
        self,
        frames: Sequence[Nv12Frame],
        out: Any,
        params: NormalizeParams,
        *,
        pad_value: float = 114,
        matrix: int = 709,
        sampling: str = "bilinear",
    ) -> tuple[np.ndarray, np.ndarray, np.ndarray]:
        """NV12 surfaces on the device into ``out``; ``matrix`` 601 or 709 (limited range);
        ``sampling`` "bilinear" or "nearest" (the reference NV12 kernel's parity mode)."""
        torch = _torch()
        if len(frames) == 0:
            raise ValueError("letterbox needs at least one image")
        if sampling not in ("bilinear", "nearest"):
            raise ValidationError(f"sampling must be 'bilinear' or 'nearest', got {sampling!r}")
        check_device_output(out, device_index=self._device_index, rows=len(frames),
                            caller="letterbox_nv12_device", dtypes=("float32", "float16"))
        n = len(frames)
        arr = (_native.FrameNv12 * n)()
        for i, f in enumerate(frames):
            buf = f.buffer
            if not getattr(buf, "is_cuda", False) or buf.device.index != self._device_index or buf.dtype != torch.uint8:
                raise ValidationError(f"NV12 frame {i} must be a uint8 tensor on cuda:{self._device_index}")
            need = int(f.uv_offset) + int(f.pitch) * ((int(f.height) + 1) // 2)
            if _nbytes(buf) < need:
                raise ValidationError(f"NV12 frame {i}: buffer holds {_nbytes(buf)} bytes, its planes need {need}")
            arr[i] = _native.FrameNv12(int(buf.data_ptr()), int(f.height), int(f.width), int(f.pitch), int(f.uv_offset))
        maps = (_native.LetterboxMap * n)()
        with self._device_guard():
            _native.check(
                self._lib.shipk_letterbox_nv12(
                    arr, n, int(out.data_ptr()), _dtype_code(out), _nbytes(out), int(out.shape[2]),
                    int(out.shape[3]), _native.floats3(params.mean), _native.floats3(params.std),
                    int(bool(params.swap_rb)), float(pad_value), int(matrix),
                    0 if sampling == "nearest" else 1, maps, self._stream_handle(),
                )
            )
        return self._maps(maps, n)

    def crop_nv12_device(
        self,
        frames: Sequence[Nv12Frame],
        boxes: Any,
        out: Any,
        *,
        swap_rb: bool = True,
        box_frame: Any = None,
    ) -> Any:
        """Crops straight from NV12 surfaces on the device into ``out`` ``[N, 3, h, w]``
        (float32 or float16): the reference's ``nv12_crop_resize_into`` (ops.cu:260-318) for
        every box of every frame in one launch; ``box_frame`` (CUDA int32 ``[N]``) names each
        box's frame (default: all frame 0). Values are BGR (RGB with ``swap_rb``) / 255."""
        torch = _torch()
        if len(frames) == 0:
            raise ValueError("crop needs at least one frame")
        if boxes.dim() != 2 or int(boxes.shape[1]) != 4 or boxes.dtype != torch.float32 or not boxes.is_contiguous():
            raise ValidationError("boxes must be a contiguous float32 [N, 4] CUDA tensor")
        n_boxes = int(boxes.shape[0])
        check_device_output(out, device_index=self._device_index, rows=n_boxes, caller="crop_nv12_device",
                            dtypes=("float32", "float16"))
        if box_frame is not None and (box_frame.dtype != torch.int32 or tuple(box_frame.shape) != (n_boxes,)):
            raise ValidationError("box_frame must be an int32 [N] CUDA tensor")
        arr = (_native.FrameNv12 * len(frames))()
        for i, f in enumerate(frames):
            buf = f.buffer
            if not getattr(buf, "is_cuda", False) or buf.device.index != self._device_index or buf.dtype != torch.uint8:
                raise ValidationError(f"NV12 frame {i} must be a uint8 tensor on cuda:{self._device_index}")
            need = int(f.uv_offset) + int(f.pitch) * ((int(f.height) + 1) // 2)
            if _nbytes(buf) < need:
                raise ValidationError(f"NV12 frame {i}: buffer holds {_nbytes(buf)} bytes, its planes need {need}")
            arr[i] = _native.FrameNv12(int(buf.data_ptr()), int(f.height), int(f.width), int(f.pitch), int(f.uv_offset))
        with self._device_guard():
            _native.check(
                self._lib.shipk_crop_nv12(
                    arr, len(frames), int(boxes.data_ptr()) if n_boxes else None,
                    int(box_frame.data_ptr()) if box_frame is not None and n_boxes else None, n_boxes,
                    int(out.data_ptr()) if out.numel() else None, _dtype_code(out), _nbytes(out),
                    int(out.shape[2]), int(out.shape[3]), int(bool(swap_rb)), self._stream_handle(),
                )
            )
        return out

    def crop_device(
        self,
        frames: Sequence[Any],
        boxes: Any,
        out: Any,
        params: NormalizeParams,
        *,
        box_frame: Any = None,
    ) -> None:
        """Every box of every device frame in one launch: ``boxes`` float32 ``[N, 4]`` and
        ``box_frame`` int32 ``[N]`` (or None: all on ``frames[0]``) on the device; ``out``
        float32/float16 ``[N, 3, h, w]``."""
        torch = _torch()
        n = int(boxes.shape[0]) if boxes is not None else 0
        check_device_output(out, device_index=self._device_index, rows=n, caller="crop_device",
                            dtypes=("float32", "float16"))
        if boxes.dtype != torch.float32 or boxes.dim() != 2 or int(boxes.shape[1]) != 4 or not boxes.is_contiguous():
            raise ValidationError("boxes must be a contiguous float32 [N, 4] CUDA tensor")
        if box_frame is not None and (box_frame.dtype != torch.int32 or not box_frame.is_contiguous()
                                      or int(box_frame.numel()) != n):
            raise ValidationError("box_frame must be a contiguous int32 [N] CUDA tensor")
        arr = self._device_frames(frames, self._device_index)
        with self._device_guard():
            _native.check(
                self._lib.shipk_crop_u8(
                    arr, len(frames), int(boxes.data_ptr()) if n else None,
                    int(box_frame.data_ptr()) if box_frame is not None and n else None, n,
                    int(out.data_ptr()), _dtype_code(out), _nbytes(out), int(out.shape[2]),
                    int(out.shape[3]), _native.floats3(params.mean), _native.floats3(params.std),
                    int(bool(params.swap_rb)), self._stream_handle(),
                )
            )

    def nms_device(
        self,
        boxes: Any,
        scores: Any,
        classes: Any = None,
        *,
        iou_threshold: float,
        score_threshold: float,
        max_det: int,
        num_classes: int = 1,
        class_aware: bool | None = None,
        keep: Any = None,
        counts: Any = None,
    ) -> tuple[Any, Any]:
        """Batched NMS on device tensors ``[B, N, 4]``, ``[B, N]``, ``[B, N]`` int32.

        Returns ``(keep int64 [B, max_det] -1 padded, counts int32 [B])`` on the device; one
        launch, no synchronisation.
        """
        torch = _torch()
        if class_aware is None:
            class_aware = classes is not None
        if boxes.dim() != 3 or int(boxes.shape[2]) != 4 or boxes.dtype != torch.float32 or not boxes.is_contiguous():
            raise ValidationError("boxes must be a contiguous float32 [B, N, 4] CUDA tensor")
        B, n = int(boxes.shape[0]), int(boxes.shape[1])
        if scores.dtype != torch.float32 or tuple(scores.shape) != (B, n) or not scores.is_contiguous():
            raise ValidationError("scores must be a contiguous float32 [B, N] CUDA tensor")
        if class_aware and (classes is None or classes.dtype != torch.int32 or tuple(classes.shape) != (B, n)
                            or not classes.is_contiguous()):
            raise ValidationError("class-aware NMS needs contiguous int32 [B, N] classes")
        dev = f"cuda:{self._device_index}"
        if keep is None:
            keep = torch.empty((B, max(max_det, 0)), dtype=torch.int64, device=dev)
        if counts is None:
            counts = torch.empty((B,), dtype=torch.int32, device=dev)
        key = (B, n, num_classes, int(class_aware), max_det)
        need = nms_workspace_bytes(B, n, num_classes, bool(class_aware), max_det)
        if self._nms_ws is None or _nbytes(self._nms_ws) < need:
            self._nms_ws = torch.empty((max(need, 1),), dtype=torch.uint8, device=dev)
        self._nms_key = key
        with self._device_guard():
            _native.check(
                self._lib.shipk_nms(
                    int(boxes.data_ptr()), int(scores.data_ptr()),
                    int(classes.data_ptr()) if class_aware else None, B, n, int(num_classes),
                    int(bool(class_aware)), float(iou_threshold), float(score_threshold), int(max_det),
                    int(keep.data_ptr()) if keep.numel() else None, int(counts.data_ptr()),
                    int(self._nms_ws.data_ptr()), _nbytes(self._nms_ws), self._stream_handle(),
                )
            )
        return keep, counts
