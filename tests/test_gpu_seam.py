"""The ``shipvision._C`` surface, called exactly as the reference's NativeImageOps calls it
(src/shipinfer/runtime/ops/native_ops.py:112-232), on a B200."""

from __future__ import annotations

import numpy as np
import pytest

from _data import frames_u8

pytestmark = pytest.mark.gpu


@pytest.fixture(scope="module")
def C(cuda):
    from shipinfer_b200 import shipvision_C

    assert shipvision_C.cuda_available() is True
    assert shipvision_C.device_count() >= 1
    assert isinstance(shipvision_C.__version__, str) and isinstance(shipvision_C.platform, str)
    return shipvision_C


def test_letterbox_into_returns_three_values(C, cuda, orc):
    ops = C.ImageOps(0)
    frames = frames_u8(2, (480, 640), seed=1)
    out = cuda.empty((2, 3, 256, 256), dtype=cuda.float32, device="cuda:0")
    scales, pads, extents = ops.letterbox_into(
        [np.ascontiguousarray(f) for f in frames], int(out.data_ptr()), int(out.numel() * out.element_size()),
        256, 256, [0.0, 0.0, 0.0], [255.0, 255.0, 255.0], True, 114, 0,
    )
    cuda.cuda.synchronize()
    assert scales.tolist() == [np.float32(0.4)] * 2
    assert pads.tolist() == [[0.0, 32.0]] * 2 and extents.tolist() == [[192, 256]] * 2
    assert np.array_equal(out.cpu().numpy(), orc.letterbox(frames, (256, 256)))


def test_letterbox_batch_returns_four_values(C, orc):
    ops = C.ImageOps(0)
    frames = frames_u8(1, (720, 1280), seed=2)
    tensor, scales, pads, extents = ops.letterbox_batch(frames, 640, 640, [0, 0, 0], [255, 255, 255], True, 114, 0)
    assert tensor.shape == (1, 3, 640, 640) and extents.tolist() == [[360, 640]]
    assert np.array_equal(tensor, orc.letterbox(frames, (640, 640)))


def test_crop_batch_and_nms(C, orc):
    ops = C.ImageOps(0)
    frame = frames_u8(1, (480, 640), seed=7)[0]
    boxes = np.array([[10, 10, 200, 200], [300, 100, 500, 400]], dtype=np.float32)
    got = ops.crop_batch(frame, boxes, 64, 64, [0, 0, 0], [255, 255, 255], True, 0)
    assert np.array_equal(got, orc.crop([frame], boxes, (64, 64)))
    b = np.array([[10, 10, 100, 100], [15, 15, 105, 105], [300, 300, 400, 400], [305, 305, 405, 405],
                  [500, 500, 520, 520]], np.float32)
    s = np.array([0.90, 0.80, 0.95, 0.70, 0.60], np.float32)
    kept = ops.nms(b, s, 0.5, 0.1, 10, 0)
    assert kept.dtype == np.int64 and kept.tolist() == [2, 0, 4]


@pytest.mark.parametrize("side_stream", [False, True], ids=["default-stream", "side-stream"])
def test_a_large_host_result_is_staged_bit_exactly(cuda, orc, side_stream):
    """8 x 1080p -> [8, 3, 640, 640] float32 (39 MB) comes home through the two pinned chunk
    buffers; twice in a row (the second call refills the same buffers), on the default stream and
    on a stream the instance was given, both bit-exact to the oracle."""
    from shipinfer_b200 import NativeImageOps, NormalizeParams
    from shipinfer_b200 import ops as ops_module

    stream = cuda.cuda.Stream() if side_stream else None
    ops = NativeImageOps(device_index=0, stream=stream.cuda_stream if stream else None)
    for seed in (3, 4):
        frames = frames_u8(8, (1080, 1920), seed=seed)
        r = ops.letterbox_batch(frames, (640, 640), NormalizeParams())
        assert r.tensor.nbytes > 2 * ops_module.STAGE_BYTES
        assert np.array_equal(r.tensor.view(np.uint32), orc.letterbox(frames, (640, 640)).view(np.uint32))

