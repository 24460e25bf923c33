"""Batched ROI crop-resize on the GPU, through the C ABI, against the oracle and torch CUDA.

Bar: bit-exact. Geometry cases are the reference's own (tests/runtime/test_torch_crop_batch.py
CASES: plain, clipped, degenerate among valid, reversed, one-pixel box, upsampled,
downsampled-hard, one-pixel output, float, far-edge, twenty random, one-pixel frame).
"""

from __future__ import annotations

import numpy as np
import pytest

from _data import IMAGENET_MEAN, IMAGENET_STD, crop_boxes, frames_u8
from shipinfer_b200 import NormalizeParams, ValidationError

pytestmark = pytest.mark.gpu


def gradient_frame(height: int, width: int) -> np.ndarray:
    ys, xs = np.mgrid[0:height, 0:width]
    return np.stack([xs % 256, ys % 256, (xs * 7 + ys * 13) % 256], axis=-1).astype(np.uint8)


def random_boxes(count: int, shape, seed: int = 7) -> np.ndarray:
    rng = np.random.default_rng(seed)
    height, width = shape[:2]
    xs = rng.uniform(-10.0, width + 10.0, size=(count, 2))
    ys = rng.uniform(-10.0, height + 10.0, size=(count, 2))
    return np.stack([xs.min(axis=1), ys.min(axis=1), xs.max(axis=1), ys.max(axis=1)], axis=1).astype(np.float32)


FRAME = gradient_frame(48, 64)
NOISE = np.random.default_rng(20260826).integers(0, 256, (97, 131, 3), dtype=np.uint8)
PIXEL = np.full((1, 1, 3), 200, dtype=np.uint8)
CASES = [
    pytest.param(FRAME, [[8, 6, 40, 30]], (16, 16), id="plain-box"),
    pytest.param(FRAME, [[-30, -20, 200, 400]], (12, 20), id="clipped"),
    pytest.param(FRAME, [[0, 0, 16, 16], [10, 10, 10, 10], [4, 4, 20, 30], [7, 9, 7, 40]], (8, 8),
                 id="degenerate-among-valid"),
    pytest.param(FRAME, [[40, 30, 8, 6]], (8, 8), id="reversed"),
    pytest.param(FRAME, [[5, 5, 6, 6]], (6, 6), id="one-pixel-box"),
    pytest.param(FRAME, [[3, 4, 5, 7]], (16, 32), id="upsampled"),
    pytest.param(NOISE, [[0, 0, 130, 96]], (4, 5), id="downsampled-hard"),
    pytest.param(FRAME, [[2, 3, 33, 41]], (1, 1), id="one-pixel-output"),
    pytest.param(FRAME, [[1.5, 2.5, 30.25, 20.75]], (9, 11), id="float"),
    pytest.param(FRAME, [[60, 44, 64, 48]], (7, 7), id="far-edge"),
    pytest.param(NOISE, random_boxes(20, NOISE.shape), (14, 10), id="twenty-random"),
    pytest.param(PIXEL, [[0, 0, 1, 1]], (4, 4), id="one-pixel-frame"),
]
IMAGENET = NormalizeParams(mean=(103.5, 116.3, 123.7), std=(57.4, 57.1, 58.4))
PARAM_SETS = [
    pytest.param(NormalizeParams(swap_rb=True), id="unit-rgb"),
    pytest.param(NormalizeParams(swap_rb=False), id="unit-bgr"),
    pytest.param(IMAGENET, id="imagenet-rgb"),
    pytest.param(NormalizeParams(mean=IMAGENET.mean, std=IMAGENET.std, swap_rb=False), id="imagenet-bgr"),
]


def exact(a: np.ndarray, b: np.ndarray) -> bool:
    return a.shape == b.shape and a.dtype == b.dtype and np.array_equal(a.view(np.uint8), b.view(np.uint8))


def crop_on_device(torch, ops, frames, boxes, dst, params, dtype=None, frame_index=None):
    dtype = dtype or torch.float32
    boxes = np.asarray(boxes, np.float32).reshape(-1, 4)
    dev_frames = [torch.from_numpy(f).cuda() for f in frames]
    out = torch.empty((len(boxes), 3, *dst), dtype=dtype, device="cuda")
    bidx = None if frame_index is None else torch.from_numpy(np.asarray(frame_index, np.int32)).cuda()
    ops.crop_device(dev_frames, torch.from_numpy(boxes).cuda(), out, params, box_frame=bidx)
    torch.cuda.synchronize()
    return out.cpu().numpy()


def torch_reference_crop(torch, image, boxes, dst, params):
    """TorchImageOps.crop_batch (torch_ops.py:405-507) on torch CUDA, step for step."""
    dst_h, dst_w = dst
    boxes = np.asarray(boxes, np.float32).reshape(-1, 4)
    src_h, src_w = image.shape[:2]
    planes = torch.from_numpy(np.ascontiguousarray(image)).to("cuda").permute(2, 0, 1)
    clipped = np.empty_like(boxes, dtype=np.int64)
    clipped[:, [0, 2]] = np.clip(boxes[:, [0, 2]], 0, src_w - 1)
    clipped[:, [1, 3]] = np.clip(boxes[:, [1, 3]], 0, src_h - 1)
    widths = clipped[:, 2] - clipped[:, 0]
    heights = clipped[:, 3] - clipped[:, 1]

    def axis(origin, extent, dst_n):
        extent_safe = np.maximum(extent, 1).astype(np.int64)
        scale = extent_safe.astype(np.float32) / np.float32(dst_n)
        centres = np.arange(dst_n, dtype=np.float32) + np.float32(0.5)
        src = scale[:, None] * centres[None, :] - np.float32(0.5)
        np.maximum(src, np.float32(0.0), out=src)
        last = (extent_safe - 1)[:, None]
        i0 = np.minimum(src.astype(np.int64), last)
        w1 = (src - i0.astype(np.float32)).astype(np.float32)
        i1 = np.minimum(i0 + 1, last)
        return origin[:, None] + i0, origin[:, None] + i1, w1

    col0, col1, wx = axis(clipped[:, 0], widths, dst_w)
    row0, row1, wy = axis(clipped[:, 1], heights, dst_h)
    columns = torch.from_numpy(np.stack((col0, col1))).cuda()
    rows = torch.from_numpy(np.stack((row0, row1))).cuda()
    across = torch.from_numpy(wx).cuda()
    down = torch.from_numpy(wy).cuda()
    count = boxes.shape[0]
    out = torch.empty((3, count, dst_h, dst_w), dtype=torch.float32, device="cuda")
    column = columns.unsqueeze(2)
    weight = across.unsqueeze(1)

    def sample(r):
        pair = planes[:, r.unsqueeze(2), column].float()
        return torch.lerp(pair[:, 0], pair[:, 1], weight)

    torch.lerp(sample(rows[0]), sample(rows[1]), down.unsqueeze(2), out=out)
    degenerate = np.nonzero((widths <= 0) | (heights <= 0))[0]
    if degenerate.size:
        out[:, torch.from_numpy(degenerate).cuda()] = 0.0
    order = torch.tensor([2, 1, 0] if params.swap_rb else [0, 1, 2], device="cuda")
    result = out.permute(1, 0, 2, 3)[:, order]
    mean = torch.tensor(params.mean, dtype=torch.float32, device="cuda").view(1, 3, 1, 1)
    std = torch.tensor(params.std, dtype=torch.float32, device="cuda").view(1, 3, 1, 1)
    result.sub_(mean).div_(std)
    torch.cuda.synchronize()
    return result.cpu().numpy()


@pytest.mark.parametrize(("image", "boxes", "dst"), CASES)
@pytest.mark.parametrize("params", PARAM_SETS)
def test_reference_cases_match_oracle_bit_exact(cuda, ops, orc, image, boxes, dst, params):
    boxes = np.asarray(boxes, np.float32)
    want = orc.crop([image], boxes, dst, None, params.mean, params.std, params.swap_rb)
    got = crop_on_device(cuda, ops, [image], boxes, dst, params)
    assert exact(got, want), f"max |d| {np.abs(got - want).max()}"
    got16 = crop_on_device(cuda, ops, [image], boxes, dst, params, dtype=cuda.float16)
    assert exact(got16, want.astype(np.float16))


@pytest.mark.parametrize(("image", "boxes", "dst"), CASES)
def test_reference_cases_match_torch_cuda(cuda, ops, image, boxes, dst):
    for params in (NormalizeParams(), IMAGENET):
        want = torch_reference_crop(cuda, image, boxes, dst, params)
        got = crop_on_device(cuda, ops, [image], boxes, dst, params)
        bad = np.argwhere(got.view(np.uint32) != want.view(np.uint32))
        assert bad.size == 0, f"{len(bad)} elements differ from torch CUDA, first {bad[:3].tolist()}"


def test_config3_batch_fp16_bit_exact(cuda, ops, orc):
    """Config 3: 8 x 1080p, 64 boxes each -> [512,3,256,128] fp16, ImageNet mean/std."""
    frames = frames_u8(8, seed=0)
    boxes, idx = crop_boxes(8, 64)
    params = NormalizeParams(mean=IMAGENET_MEAN, std=IMAGENET_STD)
    want = orc.crop(frames, boxes, (256, 128), idx, params.mean, params.std, True)
    got = crop_on_device(cuda, ops, frames, boxes, (256, 128), params, cuda.float16, idx)
    assert got.shape == (512, 3, 256, 128)
    assert exact(got, want.astype(np.float16))


def test_frame_index_out_of_range_is_a_black_crop(cuda, ops, orc):
    frames = frames_u8(2, (64, 96), seed=3)
    boxes = np.array([[4, 4, 40, 30], [4, 4, 40, 30], [1, 2, 50, 60]], np.float32)
    idx = np.array([1, 7, -1], np.int32)
    params = NormalizeParams(mean=IMAGENET.mean, std=IMAGENET.std)
    got = crop_on_device(cuda, ops, frames, boxes, (16, 8), params, frame_index=idx)
    want = orc.crop(frames, boxes, (16, 8), idx, params.mean, params.std, True)
    assert exact(got, want)
    black = ((0.0 - np.asarray(params.mean, np.float32)) / np.asarray(params.std, np.float32)).astype(np.float32)
    assert np.array_equal(got[1], np.broadcast_to(black[[0, 1, 2]][:, None, None], got[1].shape))


def test_large_boxes_fall_back_to_cached_reads(cuda, ops, orc):
    """Boxes spanning most of a 4K frame: strips wider than the kernel's prefetch window, read
    through the cache alone; same bits either way."""
    frame = frames_u8(1, (2160, 3840), seed=8)
    boxes = np.array([[0, 0, 3839, 2159], [10.5, 20.25, 3800, 400], [3000, 5, 3839, 2100]], np.float32)
    want = orc.crop(frame, boxes, (64, 256))
    got = crop_on_device(cuda, ops, frame, boxes, (64, 256), NormalizeParams())
    assert exact(got, want)


@pytest.mark.parametrize("dst", [(20, 300), (9, 301), (5, 130), (3, 66)], ids=["w300", "w301", "w130", "w66"])
@pytest.mark.parametrize("offset", [0, 1, 2], ids=["aligned", "offset1", "offset2"])
@pytest.mark.parametrize("dtype", ["float32", "float16"])
def test_output_widths_strips_and_alignment(cuda, ops, orc, dst, offset, dtype):
    """Several column strips per box, odd and even widths, and outputs that start 1 or 2
    elements past an aligned address: each picks a different store width; same bits."""
    frame = frames_u8(1, (480, 640), seed=21)
    boxes = np.array([[3.5, 7.25, 630, 470], [100, 50, 140, 70], [0, 0, 639, 1], [20, 30, 21, 300]],
                     np.float32)
    torch_dtype = getattr(cuda, dtype)
    n = len(boxes) * 3 * dst[0] * dst[1]
    flat = cuda.empty((n + offset,), dtype=torch_dtype, device="cuda")
    out = flat[offset:].view(len(boxes), 3, *dst)
    ops.crop_device([cuda.from_numpy(frame[0]).cuda()], cuda.from_numpy(boxes).cuda(), out, IMAGENET)
    cuda.cuda.synchronize()
    want = orc.crop(frame, boxes, dst, None, IMAGENET.mean, IMAGENET.std, True).astype(dtype)
    assert exact(out.cpu().numpy(), want)


def test_constants_outside_the_fast_division_range(cuda, ops, orc):
    """std below 2^-20: the kernel divides with IEEE division instead of Markstein's; same bits."""
    frame = frames_u8(1, (64, 96), seed=4)
    boxes = np.array([[4, 4, 40, 30], [1, 2, 90, 60]], np.float32)
    params = NormalizeParams(mean=(0.0, 1e-3, 200.0), std=(1e-7, 3e-7, 2e-7), swap_rb=True)
    got = crop_on_device(cuda, ops, frame, boxes, (12, 20), params)
    assert exact(got, orc.crop(frame, boxes, (12, 20), None, params.mean, params.std, True))


def test_crop_batch_host_path(cuda, ops, orc):
    """crop_batch: host frame and boxes (row-subset upload), numpy float32 out."""
    frame = frames_u8(1, (1080, 1920), seed=12)[0]
    boxes, _ = crop_boxes(1, 15, seed=13)
    got = ops.crop_batch(frame, boxes, (256, 128), IMAGENET)
    assert got.dtype == np.float32 and got.shape == (15, 3, 256, 128)
    assert exact(got, orc.crop([frame], boxes, (256, 128), None, IMAGENET.mean, IMAGENET.std, True))
    empty = ops.crop_batch(frame, np.zeros((0, 4), np.float32), (256, 128), IMAGENET)
    assert empty.shape == (0, 3, 256, 128)


def test_crop_refusals(cuda, ops):
    frame = cuda.zeros((32, 32, 3), dtype=cuda.uint8, device="cuda")
    boxes = cuda.zeros((2, 4), dtype=cuda.float32, device="cuda")
    with pytest.raises(ValidationError):
        ops.crop_device([frame], boxes, cuda.empty((1, 3, 8, 8), device="cuda"), NormalizeParams())
    with pytest.raises(ValidationError):
        ops.crop_device([frame], boxes.double(), cuda.empty((2, 3, 8, 8), device="cuda"), NormalizeParams())


def test_frames_at_unaligned_addresses_and_pitches(cuda, ops, orc):
    """Frame views whose rows start at every byte offset modulo 4 (odd base, odd pitch) and an
    aligned view of the same pixels: the same crops, bit for bit."""
    base = np.random.default_rng(13).integers(0, 256, (300, 401, 3), dtype=np.uint8)
    dev = cuda.from_numpy(base).cuda()
    boxes = np.array([[3, 5, 150, 120], [0.5, 0.5, 300, 250], [100, 40, 140, 290], [7, 9, 15, 12]], np.float32)
    for y0, x0 in [(0, 0), (1, 1), (2, 3), (5, 2)]:
        view = dev[y0:y0 + 280, x0:x0 + 390]          # pitch 1203 bytes, base offset 3 * x0 + 1203 * y0
        host = np.ascontiguousarray(base[y0:y0 + 280, x0:x0 + 390])
        want = orc.crop([host], boxes, (64, 48), None, IMAGENET_MEAN, IMAGENET_STD, True)
        out = cuda.empty((4, 3, 64, 48), dtype=cuda.float32, device="cuda")
        ops.crop_device([view], cuda.from_numpy(boxes).cuda(), out, NormalizeParams(IMAGENET_MEAN, IMAGENET_STD))
        cuda.cuda.synchronize()
        assert np.array_equal(out.cpu().numpy().view(np.uint32), want.view(np.uint32))
