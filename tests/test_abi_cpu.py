"""The C ABI without a GPU: the library loads, exports every declared symbol, and refuses bad
arguments with the documented status codes and messages before touching a device."""

from __future__ import annotations

import ctypes
import re
import subprocess
import sys
import threading
from pathlib import Path

import numpy as np
import pytest

from shipinfer_b200 import _native

ROOT = Path(__file__).resolve().parents[1]
HEADER = ROOT / "include" / "shipk.h"


def declared_symbols() -> set[str]:
    text = HEADER.read_text()
    return set(re.findall(r"SHIPK_API\s+[\w\s\*]+?\b(shipk_\w+)\s*\(", text))


@pytest.fixture(scope="module")
def lib():
    return _native.lib()


def test_every_declared_symbol_is_exported(lib):
    names = declared_symbols()
    assert len(names) >= 15
    out = subprocess.run(["nm", "-D", "--defined-only", str(_native.library_path())], capture_output=True,
                         text=True, check=True).stdout
    exported = {line.split()[-1] for line in out.splitlines() if line.strip()}
    missing = names - exported
    assert not missing, f"declared in include/shipk.h but not exported: {missing}"
    # and nothing else leaks: internal C++ symbols stay hidden
    assert {n for n in exported if n.startswith("shipk_")} == names


def test_binding_declares_the_same_surface():
    assert set(_native.SIGNATURES) == declared_symbols()


def test_probes_without_a_device(lib):
    import torch

    assert lib.shipk_version().decode().startswith("0.")
    if not torch.cuda.is_available():
        assert lib.shipk_cuda_available() == 0
        assert lib.shipk_device_count() == 0


def test_letterbox_fit_is_pythons_placement(lib):
    m = _native.LetterboxMap()
    assert lib.shipk_letterbox_fit(1080, 1920, 640, 640, ctypes.byref(m)) == 0
    assert (m.new_w, m.new_h, m.pad_x, m.pad_y) == (640, 360, 0, 140)
    assert np.float32(m.scale) == np.float32(640 / 1920)
    assert lib.shipk_letterbox_fit(251, 500, 250, 250, ctypes.byref(m)) == 0 and m.new_h == 126
    assert lib.shipk_letterbox_fit(0, 10, 10, 10, ctypes.byref(m)) == _native.EINVAL


def _fit_f32(sh: int, sw: int, dh: int, dw: int) -> tuple[int, int, int, int]:
    """The C++ data plane's placement (reference ops.cu:341-356) in numpy float32."""
    f = np.float32
    s = min(f(dw) / f(sw), f(dh) / f(sh))
    nw, nh = max(1, int(np.rint(f(sw) * s))), max(1, int(np.rint(f(sh) * s)))
    return (dw - nw) // 2, (dh - nh) // 2, nw, nh


REF_LIB = ROOT / "oracle" / "_ref" / "libshipref.so"
FIT_SIZES = [(sh, sw, dh, dw) for sh in (1, 2, 90, 180, 251, 340, 479, 660, 720, 1080, 1081, 2160)
             for sw in (1, 3, 160, 500, 1280, 1919, 1920, 3840) for dh, dw in ((224, 224), (640, 640), (100, 37))]


def test_dp_letterbox_fit_is_the_cpp_planes_placement(lib):
    """shipk_dp_letterbox_fit follows the data plane's float32 rule; shipk_letterbox_fit the
    Python plane's double one. 180x1280 -> 224x224 is where they part (32 rows against 31)."""
    m = _native.LetterboxMap()
    assert lib.shipk_dp_letterbox_fit(180, 1280, 224, 224, ctypes.byref(m)) == 0
    assert (m.new_w, m.new_h, m.pad_x, m.pad_y) == (224, 32, 0, 96)
    assert lib.shipk_letterbox_fit(180, 1280, 224, 224, ctypes.byref(m)) == 0 and m.new_h == 31
    for sh, sw, dh, dw in FIT_SIZES:
        assert lib.shipk_dp_letterbox_fit(sh, sw, dh, dw, ctypes.byref(m)) == 0
        assert (m.pad_x, m.pad_y, m.new_w, m.new_h) == _fit_f32(sh, sw, dh, dw), (sh, sw, dh, dw)
    assert lib.shipk_dp_letterbox_fit(0, 10, 10, 10, ctypes.byref(m)) == _native.EINVAL


@pytest.mark.skipif(not REF_LIB.exists(), reason="oracle/_ref/libshipref.so not built")
def test_dp_letterbox_fit_equals_the_reference_build():
    """Pinned to the reference's own letterbox_fit, compiled from its ops.cu (host code)."""
    ref = ctypes.CDLL(str(REF_LIB))
    got = (ctypes.c_int * 4)()
    for sh, sw, dh, dw in FIT_SIZES:
        ref.ref_letterbox_fit(sh, sw, dh, dw, got)
        assert tuple(got) == _fit_f32(sh, sw, dh, dw), (sh, sw, dh, dw)


def err() -> str:
    return _native.last_error()


F3 = _native.floats3


def test_letterbox_refusals(lib):
    frames = (_native.FrameU8 * 1)(_native.FrameU8(0x1000, 10, 10, 30))
    assert lib.shipk_letterbox_u8(frames, 0, None, 0, 0, 8, 8, F3([0] * 3), F3([255] * 3), 1, 114.0, None, None) \
        == _native.EINVAL and "at least one frame" in err()
    assert lib.shipk_letterbox_u8(frames, 1, None, 7, 0, 8, 8, F3([0] * 3), F3([255] * 3), 1, 114.0, None, None) \
        == _native.EINVAL and "out_dtype" in err()
    assert lib.shipk_letterbox_u8(frames, 1, None, 0, 0, 8, 8, F3([0] * 3), F3([1, 0, 1]), 1, 114.0, None, None) \
        == _native.EINVAL and "std must be non-zero" in err()
    assert lib.shipk_letterbox_u8(frames, 1, None, 0, 100, 8, 8, F3([0] * 3), F3([255] * 3), 1, 114.0, None, None) \
        == _native.ENOMEM and "needs 768" in err()
    assert lib.shipk_letterbox_u8(None, 1, None, 0, 768, 8, 8, F3([0] * 3), F3([255] * 3), 1, 114.0, None, None) \
        == _native.EINVAL and "frames is null" in err()
    assert lib.shipk_letterbox_u8(frames, 1, None, 0, 768, 0, 8, F3([0] * 3), F3([255] * 3), 1, 114.0, None, None) \
        == _native.EINVAL and "outside 1..32768" in err()


def test_nv12_refusals(lib):
    frames = (_native.FrameNv12 * 1)(_native.FrameNv12(0x1000, 90, 160, 192, 192 * 90))
    args = (frames, 1, None, 0, 1 << 20, 64, 64, F3([0] * 3), F3([255] * 3), 1, 114.0)
    assert lib.shipk_letterbox_nv12(*args, 123, 1, None, None) == _native.EINVAL and "601 nor 709" in err()
    assert lib.shipk_letterbox_nv12(*args, 709, 5, None, None) == _native.EINVAL and "sampling" in err()


def test_crop_and_nms_refusals(lib):
    frames = (_native.FrameU8 * 65)()
    assert lib.shipk_crop_u8(frames, 65, None, None, 1, None, 0, 0, 8, 8, F3([0] * 3), F3([255] * 3), 1, None) \
        == _native.ERANGE and "at most 64" in err()
    assert lib.shipk_crop_u8(frames, 1, None, None, -1, None, 0, 0, 8, 8, F3([0] * 3), F3([255] * 3), 1, None) \
        == _native.EINVAL and "negative" in err()
    assert lib.shipk_crop_u8(frames, 1, None, None, 0, None, 0, 0, 8, 8, F3([0] * 3), F3([255] * 3), 1, None) == 0
    assert lib.shipk_nms(None, None, None, -1, 10, 1, 0, 0.5, 0.2, 10, None, None, None, 0, None) == _native.EINVAL
    assert lib.shipk_nms(None, None, None, 1, 10, 0, 1, 0.5, 0.2, 10, None, None, None, 0, None) == _native.EINVAL \
        and "num_classes" in err()
    assert lib.shipk_nms(None, None, None, 1, 10, 1, 0, 0.5, 0.2, 5000, None, None, None, 0, None) \
        == _native.ERANGE and "4096" in err()
    assert lib.shipk_nms(None, None, None, 0, 10, 1, 0, 0.5, 0.2, 10, None, None, None, 0, None) == 0


def test_nms_launch_shape_refusals_and_empty_shapes(lib):
    ctas, cluster = ctypes.c_int(-5), ctypes.c_int(-5)
    shape = lambda *a: lib.shipk_nms_launch_shape(*a, ctypes.byref(ctas), ctypes.byref(cluster))
    assert shape(1, 10, 1, 0, 5000) == _native.ERANGE and "4096" in err()
    assert shape(1, 10, 0, 1, 10) == _native.EINVAL and "num_classes" in err()
    assert lib.shipk_nms_launch_shape(1, 10, 1, 0, 10, None, None) == _native.EINVAL and "NULL" in err()
    # nothing to launch: no device needed
    assert shape(4, 0, 2, 1, 300) == 0 and (ctas.value, cluster.value) == (0, 1)
    assert shape(0, 8400, 2, 1, 300) == 0 and (ctas.value, cluster.value) == (0, 1)


def test_workspace_size_is_monotonic(lib):
    a = lib.shipk_nms_workspace_bytes(16, 8400, 2, 1, 300)
    b = lib.shipk_nms_workspace_bytes(32, 8400, 2, 1, 300)
    c = lib.shipk_nms_workspace_bytes(16, 8400, 80, 1, 300)
    assert 0 < a < b and a < c
    assert lib.shipk_nms_workspace_bytes(16, 8400, 2, 0, 300) < a


def test_ctx_refuses_a_missing_device(lib):
    handle = ctypes.c_void_p()
    rc = lib.shipk_ctx_create(lib.shipk_device_count() + 3, ctypes.byref(handle))
    assert rc == _native.EINVAL and "not one of" in err() and not handle.value
    assert lib.shipk_ctx_letterbox_host(None, None, 1, None, 0, 0, 8, 8, F3([0] * 3), F3([255] * 3), 1, 114.0,
                                        None, None) == _native.EINVAL and "ctx is null" in err()


def test_last_error_is_per_thread_and_truncates(lib):
    lib.shipk_nms(None, None, None, -1, 0, 1, 0, 0.5, 0.2, 10, None, None, None, 0, None)
    mine = err()
    seen = []

    def other():
        m = _native.LetterboxMap()
        lib.shipk_letterbox_fit(-1, 1, 1, 1, ctypes.byref(m))
        seen.append(_native.last_error())

    t = threading.Thread(target=other)
    t.start()
    t.join()
    assert "shipk_nms" in mine and "shipk_letterbox_fit" in seen[0]
    assert err() == mine, "another thread's failure must not overwrite this thread's message"
    buf = ctypes.create_string_buffer(6)
    full = lib.shipk_last_error(buf, 6)
    assert full == len(mine) and buf.value == mine[:5].encode()


def test_status_codes_map_to_python_exceptions():
    from shipinfer_b200.errors import ConfigurationError, NativeError, ValidationError

    lib = _native.lib()
    lib.shipk_nms(None, None, None, -1, 0, 1, 0, 0.5, 0.2, 10, None, None, None, 0, None)
    with pytest.raises(ValidationError):
        _native.check(_native.EINVAL)
    with pytest.raises(ConfigurationError):
        _native.check(_native.ERANGE)
    with pytest.raises(NativeError):
        _native.check(_native.ECUDA)


def test_a_missing_library_is_a_configuration_error(tmp_path):
    code = (
        "import os; os.environ['SHIPK_LIBRARY'] = %r\n"
        "from shipinfer_b200 import _native\n"
        "from shipinfer_b200.errors import ConfigurationError\n"
        "try:\n    _native.lib()\nexcept ConfigurationError as e:\n    print('refused:', e)\n"
    ) % str(tmp_path / "nope.so")
    out = subprocess.run([sys.executable, "-c", code], cwd=ROOT, capture_output=True, text=True, check=True).stdout
    assert out.startswith("refused:") and "python -m shipinfer_b200.build" in out
