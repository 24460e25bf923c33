"""ctypes binding of ``libshipk.so`` (the C ABI in ``include/shipk.h``).

The library is required: if it is missing or cannot be loaded this module raises
:class:`~shipinfer_b200.errors.ConfigurationError` naming the build command. There is no
CPU fallback anywhere in this package.
"""

from __future__ import annotations

import ctypes
import os
import threading
from pathlib import Path

from shipinfer_b200.errors import ConfigurationError, NativeError, ValidationError

__all__ = [
    "DTYPE_F16",
    "DTYPE_F32",
    "FrameNv12",
    "FrameU8",
    "HostFrameU8",
    "LetterboxMap",
    "check",
    "lib",
    "library_path",
]

_PKG = Path(__file__).resolve().parent
LIB_PATH = Path(os.environ.get("SHIPK_LIBRARY", str(_PKG / "_lib" / "libshipk.so")))

OK, EINVAL, EDEVICE, ECUDA, ERANGE, ENOMEM = 0, 1, 2, 3, 4, 5
DTYPE_F32, DTYPE_F16 = 0, 1


class FrameU8(ctypes.Structure):
    _fields_ = [
        ("data", ctypes.c_void_p),
        ("height", ctypes.c_int32),
        ("width", ctypes.c_int32),
        ("pitch", ctypes.c_int64),
    ]


HostFrameU8 = FrameU8  # same layout: shipk_host_frame_u8


class FrameNv12(ctypes.Structure):
    _fields_ = [
        ("luma", ctypes.c_void_p),
        ("height", ctypes.c_int32),
        ("width", ctypes.c_int32),
        ("pitch", ctypes.c_int64),
        ("uv_offset", ctypes.c_int64),
    ]


class LetterboxMap(ctypes.Structure):
    _fields_ = [
        ("scale", ctypes.c_float),
        ("pad_x", ctypes.c_int32),
        ("pad_y", ctypes.c_int32),
        ("new_w", ctypes.c_int32),
        ("new_h", ctypes.c_int32),
    ]


_F3 = ctypes.c_float * 3
_VP = ctypes.c_void_p
_I = ctypes.c_int
_SZ = ctypes.c_size_t
_F = ctypes.c_float

#: name -> (restype, argtypes); every symbol include/shipk.h declares.
SIGNATURES: dict[str, tuple[object, list[object]]] = {
    "shipk_version": (ctypes.c_char_p, []),
    "shipk_cuda_available": (_I, []),
    "shipk_device_count": (_I, []),
    "shipk_last_error": (_SZ, [ctypes.c_char_p, _SZ]),
    "shipk_letterbox_fit": (_I, [_I, _I, _I, _I, ctypes.POINTER(LetterboxMap)]),
    "shipk_letterbox_u8": (
        _I,
        [ctypes.POINTER(FrameU8), _I, _VP, _I, _SZ, _I, _I, _F3, _F3, _I, _F,
         ctypes.POINTER(LetterboxMap), _VP],
    ),
    "shipk_letterbox_nv12": (
        _I,
        [ctypes.POINTER(FrameNv12), _I, _VP, _I, _SZ, _I, _I, _F3, _F3, _I, _F, _I, _I,
         ctypes.POINTER(LetterboxMap), _VP],
    ),
    "shipk_crop_u8": (
        _I,
        [ctypes.POINTER(FrameU8), _I, _VP, _VP, _I, _VP, _I, _SZ, _I, _I, _F3, _F3, _I, _VP],
    ),
    "shipk_crop_nv12": (
        _I,
        [ctypes.POINTER(FrameNv12), _I, _VP, _VP, _I, _VP, _I, _SZ, _I, _I, _I, _VP],
    ),
    "shipk_nms_workspace_bytes": (_SZ, [_I, _I, _I, _I, _I]),
    "shipk_nms_launch_shape": (_I, [_I, _I, _I, _I, _I, ctypes.POINTER(ctypes.c_int), ctypes.POINTER(ctypes.c_int)]),
    "shipk_nms": (
        _I,
        [_VP, _VP, _VP, _I, _I, _I, _I, _F, _F, _I, _VP, _VP, _VP, _SZ, _VP],
    ),
    "shipk_nms_static": (
        _I,
        [_VP, _VP, _VP, _I, _I, _I, _I, _F, _F, _I, _VP, _VP, _VP],
    ),
    "shipk_decode_detections": (
        _I,
        [_VP, _I, _I, _VP, _VP, _VP, _VP, _F, _I, _VP, _VP, _VP, _VP, _VP, _VP],
    ),
    "shipk_mask_area": (
        _I,
        [_VP, _I, _I, _I, _VP, _I, _I, _I, _F, _F, _I, _I, _VP, _VP],
    ),
    "shipk_normalise_check": (_I, [_F, _F, _VP, _VP]),
    "shipk_dp_letterbox_fit": (_I, [_I, _I, _I, _I, ctypes.POINTER(LetterboxMap)]),
    "shipk_dp_letterbox_into": (_I, [_VP, _I, _I, _VP, _I, _I, _I, _F, ctypes.POINTER(LetterboxMap), _VP]),
    "shipk_dp_crop_resize_into": (_I, [_VP, _I, _I, _VP, _I, _VP, _I, _I, _I, _VP]),
    "shipk_dp_nv12_letterbox_into": (
        _I,
        [_VP, _I, _I, _I, _SZ, _VP, _I, _I, _I, _F, ctypes.POINTER(LetterboxMap), _VP],
    ),
    "shipk_dp_nv12_crop_resize_into": (_I, [_VP, _I, _I, _I, _SZ, _VP, _I, _VP, _I, _I, _I, _VP]),
    "shipk_ctx_create": (_I, [_I, ctypes.POINTER(_VP)]),
    "shipk_ctx_destroy": (None, [_VP]),
    "shipk_ctx_letterbox_host": (
        _I,
        [_VP, ctypes.POINTER(FrameU8), _I, _VP, _I, _SZ, _I, _I, _F3, _F3, _I, _F,
         ctypes.POINTER(LetterboxMap), _VP],
    ),
    "shipk_ctx_crop_host": (
        _I,
        [_VP, ctypes.POINTER(FrameU8), _VP, _I, _VP, _I, _SZ, _I, _I, _F3, _F3, _I, _VP],
    ),
    "shipk_ctx_nms_host": (
        _I,
        [_VP, _VP, _VP, _VP, _I, _I, _I, _I, _F, _F, _I, _VP, _VP, _VP],
    ),
}

_lock = threading.Lock()
_lib: ctypes.CDLL | None = None


def library_path() -> Path:
    return LIB_PATH


def lib() -> ctypes.CDLL:
    """The loaded library, with every signature declared. Raises ConfigurationError."""
    global _lib
    if _lib is not None:
        return _lib
    with _lock:
        if _lib is not None:
            return _lib
        if not LIB_PATH.exists():
            raise ConfigurationError(
                f"the shipk kernels are not built ({LIB_PATH} is missing). Build them with\n"
                "    python -m shipinfer_b200.build\n"
                "(needs the CUDA toolkit with sm_100a support). There is no CPU fallback."
            )
        try:
            handle = ctypes.CDLL(str(LIB_PATH))
        except OSError as exc:
            raise ConfigurationError(f"cannot load {LIB_PATH}: {exc}") from exc
        for name, (restype, argtypes) in SIGNATURES.items():
            fn = getattr(handle, name)
            fn.restype = restype
            fn.argtypes = argtypes
        _lib = handle
        return handle


def last_error() -> str:
    buf = ctypes.create_string_buffer(1024)
    lib().shipk_last_error(buf, len(buf))
    return buf.value.decode("utf-8", "replace")


def check(rc: int) -> None:
    """Raise the Python exception for a non-zero status code."""
    if rc == OK:
        return
    message = last_error()
    if rc in (EINVAL, EDEVICE, ENOMEM):
        raise ValidationError(message)
    if rc == ERANGE:
        raise ConfigurationError(message)
    raise NativeError(message)


def floats3(values) -> ctypes.Array:
    return _F3(*[float(v) for v in values])
