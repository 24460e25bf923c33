"""Fused letterbox on the GPU, through the C ABI, against the oracle and against torch CUDA.

Bar: bit-exact. The oracle restates TorchImageOps._letterbox (torch_ops.py:349-403) with
F.interpolate in its CUDA formulation; ``torch_reference_letterbox`` below runs the
reference's own call sequence on torch CUDA (fill, interpolate, paste, flip, sub, div).
"""

from __future__ import annotations

import numpy as np
import pytest

from _data import IMAGENET_MEAN, IMAGENET_STD, frames_u8
from shipinfer_b200 import NormalizeParams, ValidationError

pytestmark = pytest.mark.gpu

UNIT = NormalizeParams()
IMAGENET_BGR = NormalizeParams(mean=IMAGENET_MEAN, std=IMAGENET_STD, swap_rb=False)

GEOMETRIES = [
    pytest.param((1080, 1920), (640, 640), id="1080p-640"),
    pytest.param((720, 1280), (640, 640), id="720p-640"),
    pytest.param((480, 640), (256, 256), id="vga-256"),
    pytest.param((300, 300), (256, 256), id="square-upscale"),
    pytest.param((251, 500), (250, 250), id="half-even-extent"),
    pytest.param((90, 160), (64, 64), id="90x160-64"),
    pytest.param((640, 200), (320, 320), id="portrait"),
    pytest.param((33, 77), (100, 37), id="odd-everything"),
    pytest.param((1, 1), (8, 8), id="one-pixel"),
    pytest.param((97, 131), (13, 640), id="wide-canvas"),
    # ratio RN(1/3): row and column 1 get the tap weight 2^-26, so blends can be tiny and the
    # kernel keeps its tiny-numerator test on for the unit (zero-mean) constants
    pytest.param((120, 160), (360, 480), id="3x-upscale-tiny-weights"),
    # exact 2:1 reductions (every weight 1/2): the integer-sum path; with an odd source height
    # the rows' ratio is not 2 and only the columns are half-weight pairs
    pytest.param((720, 1280), (360, 640), id="2to1-no-bars"),
    pytest.param((721, 1280), (640, 640), id="2to1-across-odd-rows"),
    pytest.param((1280, 720), (640, 640), id="2to1-portrait-bars"),
    pytest.param((90, 96), (45, 48), id="2to1-small"),
]


def exact(a: np.ndarray, b: np.ndarray) -> bool:
    """Bitwise equality (distinguishes -0.0 and NaN payloads)."""
    return a.shape == b.shape and a.dtype == b.dtype and np.array_equal(
        a.view(np.uint8), b.view(np.uint8)
    )


def run_device(torch, ops, frames, dst, params, dtype, pad=114):
    dev = [torch.from_numpy(f).cuda() for f in frames]
    out = torch.empty((len(frames), 3, *dst), dtype=dtype, device="cuda")
    maps = ops.letterbox_device(dev, out, params, pad_value=pad)
    torch.cuda.synchronize()
    return out.cpu().numpy(), maps


def torch_reference_letterbox(torch, frames, dst, params, pad=114):
    """TorchImageOps._letterbox (torch_ops.py:349-403) on torch CUDA, step for step."""
    dst_h, dst_w = dst
    n = len(frames)
    canvas = torch.empty((n, 3, dst_h, dst_w), dtype=torch.float32, device="cuda")
    canvas.fill_(float(pad))
    for i, image in enumerate(frames):
        src_h, src_w = image.shape[:2]
        scale = min(dst_h / src_h, dst_w / src_w)
        new_h = max(1, round(src_h * scale))
        new_w = max(1, round(src_w * scale))
        pad_y = (dst_h - new_h) // 2
        pad_x = (dst_w - new_w) // 2
        src = torch.from_numpy(np.ascontiguousarray(image)).to("cuda").permute(2, 0, 1).unsqueeze(0).float()
        resized = torch.nn.functional.interpolate(src, size=(new_h, new_w), mode="bilinear", align_corners=False)
        canvas[i, :, pad_y : pad_y + new_h, pad_x : pad_x + new_w] = resized[0]
    if params.swap_rb:
        canvas[:n] = canvas[:n].flip(1)
    mean = torch.tensor(params.mean, dtype=torch.float32, device="cuda").view(1, 3, 1, 1)
    std = torch.tensor(params.std, dtype=torch.float32, device="cuda").view(1, 3, 1, 1)
    canvas[:n].sub_(mean).div_(std)
    torch.cuda.synchronize()
    return canvas.cpu().numpy()


@pytest.mark.parametrize(("src", "dst"), GEOMETRIES)
@pytest.mark.parametrize("params", [UNIT, IMAGENET_BGR], ids=["unit-rgb", "imagenet-bgr"])
def test_matches_oracle_bit_exact(cuda, ops, orc, src, dst, params):
    frames = frames_u8(2, src, seed=hash((src, dst)) % 1000)
    want = orc.letterbox(frames, dst, params.mean, params.std, params.swap_rb, 114)
    got32, maps = run_device(cuda, ops, frames, dst, params, cuda.float32)
    assert exact(got32, want), f"fp32 differs at {np.argwhere(got32 != want)[:5].tolist()}"
    got16, _ = run_device(cuda, ops, frames, dst, params, cuda.float16)
    assert exact(got16, want.astype(np.float16))
    scale, pad_x, pad_y, new_w, new_h = orc.letterbox_fit(*src, *dst)
    assert maps[0][0] == np.float32(scale)
    assert maps[1][0].tolist() == [pad_x, pad_y]
    assert maps[2][0].tolist() == [new_h, new_w]


@pytest.mark.parametrize(("src", "dst"), GEOMETRIES)
def test_matches_torch_cuda_formulation(cuda, ops, src, dst):
    """The reference's own torch path run on CUDA: bit-exact."""
    frames = frames_u8(2, src, seed=7)
    for params in (UNIT, IMAGENET_BGR):
        want = torch_reference_letterbox(cuda, frames, dst, params)
        got, _ = run_device(cuda, ops, frames, dst, params, cuda.float32)
        bad = np.argwhere(got.view(np.uint32) != want.view(np.uint32))
        assert bad.size == 0, f"{len(bad)} elements differ from torch CUDA, first {bad[:3].tolist()}"


def test_config1_batch_bit_exact(cuda, ops, orc):
    """Config 1: 8 x 1080p -> [8,3,640,640] fp32, pad 114, /255, BGR->RGB."""
    frames = frames_u8(8, (1080, 1920), seed=0)
    want = orc.letterbox(frames, (640, 640))
    got, maps = run_device(cuda, ops, frames, (640, 640), UNIT, cuda.float32)
    assert exact(got, want)
    # p[3y+1][3x+1] / 255 exactly, and the bars are 114/255
    assert got[0, 0, 0, 0] == np.float32(114) / np.float32(255)
    assert got[3, 0, 140, 5] == np.float32(frames[3][1, 16, 2]) / np.float32(255)
    assert maps[2].tolist() == [[360, 640]] * 8


@pytest.mark.parametrize(
    "params",
    [
        pytest.param(NormalizeParams(mean=(0.0, 0.0, 0.0), std=(1e-7, 3e-7, 7e-7)), id="std-below-fast-range"),
        # 1/std is subnormal and so are the quotients: the table path for exact taps
        pytest.param(NormalizeParams(mean=(0.0, 0.0, 0.0), std=(1e38, 255.0, 255.0)), id="subnormal-quotients"),
        pytest.param(NormalizeParams(mean=(1e-30, 0.5, 3e7), std=(255.0, 1.0, 255.0)), id="mean-outside-fast-range"),
    ],
)
@pytest.mark.parametrize(("src", "dst"), [((1080, 1920), (640, 640)), ((33, 77), (100, 37)), ((720, 1280), (640, 640))],
                         ids=["exact-taps", "blended", "half-weights"])
def test_constants_outside_the_fast_division_range(cuda, ops, orc, params, src, dst):
    """Normalisation constants the division-free path does not take: the table of normalise(k)
    (exact taps) and IEEE division (blended pixels) give the oracle's bits."""
    frames = frames_u8(2, src, seed=11)
    want = orc.letterbox(frames, dst, params.mean, params.std, params.swap_rb)
    for dtype in (cuda.float32, cuda.float16):
        got, _ = run_device(cuda, ops, frames, dst, params, dtype)
        with np.errstate(over="ignore"):  # quotients beyond fp16's range round to inf, as on the device
            ref = want if dtype == cuda.float32 else want.astype(np.float16)
        assert exact(got, ref)


@pytest.mark.parametrize("swap_rb", [True, False], ids=["rgb", "bgr"])
@pytest.mark.parametrize("mean", [(0.0, 0.0, 0.0), (0.25, -3.5, 64.0), (123.675, 116.28, 103.53)],
                         ids=["zero-mean", "quarter-means", "imagenet-means"])
def test_half_weight_rows_every_sum(cuda, ops, orc, swap_rb, mean):
    """720p -> 640: every value is (p00 + p01 + p10 + p11) / 4 normalised. Frames whose 2x2
    blocks cover every sum 0..1020 in every channel, with means that 2^21 + mean represents
    exactly (one fma) and that it does not."""
    rng = np.random.default_rng(21)
    frame = rng.integers(0, 256, (720, 1280, 3), dtype=np.uint8)
    # the image's first two output rows (source rows 0-3) hold every sum k = 0..1020 per channel,
    # split over the four taps of each 2x2 block
    k = np.arange(1021)
    for c in range(3):
        ks = np.roll(k, 337 * c)
        ks = np.concatenate([ks, ks[:259]]).reshape(2, 640)
        taps = [np.minimum(ks, 255), np.clip(ks - 255, 0, 255), np.clip(ks - 510, 0, 255), np.clip(ks - 765, 0, 255)]
        for j, (dy, dx) in enumerate([(0, 0), (0, 1), (1, 0), (1, 1)]):
            for r in range(2):
                frame[2 * r + dy, dx::2, c] = taps[j][r]
    params = NormalizeParams(mean=mean, std=(255.0, 57.12, 0.75), swap_rb=swap_rb)
    frames = [frame, np.ascontiguousarray(frame[::-1])]
    want = orc.letterbox(frames, (640, 640), params.mean, params.std, params.swap_rb)
    for dtype in (cuda.float32, cuda.float16):
        got, _ = run_device(cuda, ops, frames, (640, 640), params, dtype)
        assert exact(got, want if dtype == cuda.float32 else want.astype(np.float16))


def test_half_weight_rows_at_every_row_alignment(cuda, ops, orc):
    """720p views whose rows start at every offset modulo 16: rows that the word loads can read
    take the integer-sum path, the others the per-tap path, with the same bits."""
    rng = np.random.default_rng(23)
    base = rng.integers(0, 256, (730, 1300, 3), dtype=np.uint8)
    dev = cuda.from_numpy(base).cuda()
    for x0 in (0, 16, 1, 5):
        view = dev[5:725, x0:x0 + 1280]  # pitch 3900 bytes: the row start moves by 12 mod 16 per row
        host = np.ascontiguousarray(base[5:725, x0:x0 + 1280])
        want = orc.letterbox([host], (640, 640))
        for dtype in (cuda.float32, cuda.float16):
            out = cuda.empty((1, 3, 640, 640), dtype=dtype, device="cuda")
            ops.letterbox_device([view], out, UNIT)
            cuda.cuda.synchronize()
            assert exact(out.cpu().numpy(), want if dtype == cuda.float32 else want.astype(np.float16))


def test_ragged_batch_in_one_call(cuda, ops, orc):
    """50 cameras do not agree on resolution: one launch, mixed sizes."""
    rng = np.random.default_rng(3)
    frames = [rng.integers(0, 256, hw + (3,), dtype=np.uint8)
              for hw in [(1080, 1920), (720, 1280), (480, 640), (300, 300), (1, 1), (640, 200)]]
    want = orc.letterbox(frames, (640, 640))
    got, _ = run_device(cuda, ops, frames, (640, 640), UNIT, cuda.float16)
    assert exact(got, want.astype(np.float16))


def test_batch_larger_than_one_launch(cuda, ops, orc):
    frames = frames_u8(70, (36, 64), seed=5)
    want = orc.letterbox(frames, (32, 32))
    got, _ = run_device(cuda, ops, frames, (32, 32), UNIT, cuda.float32)
    assert exact(got, want)


def test_strided_and_unaligned_frames(cuda, ops, orc):
    """Row pitch wider than the pixels, and a frame starting at an odd byte address."""
    base = np.random.default_rng(11).integers(0, 256, (200, 333, 3), dtype=np.uint8)
    dev_full = cuda.from_numpy(base).cuda()
    view = dev_full[7:150, 5:300]              # pitch 999 bytes, start offset not 16-aligned
    host_view = np.ascontiguousarray(base[7:150, 5:300])
    want = orc.letterbox([host_view], (96, 128))
    out = cuda.empty((1, 3, 96, 128), dtype=cuda.float32, device="cuda")
    ops.letterbox_device([view], out, UNIT)
    cuda.cuda.synchronize()
    assert exact(out.cpu().numpy(), want)


def test_output_row_not_vector_aligned(cuda, ops, orc):
    frames = frames_u8(1, (120, 90), seed=2)
    for dst in [(50, 51), (7, 3)]:
        want = orc.letterbox(frames, dst)
        for dtype in (cuda.float32, cuda.float16):
            got, _ = run_device(cuda, ops, frames, dst, UNIT, dtype)
            ref = want if dtype == cuda.float32 else want.astype(np.float16)
            assert exact(got, ref)


def test_host_frames_upload_only_needed_rows_and_agree(cuda, ops, orc):
    """letterbox_to_device (host frames, row-subset upload) equals the device-frame path."""
    frames = frames_u8(3, (1080, 1920), seed=9) + frames_u8(2, (720, 1280), seed=10)
    out = cuda.empty((5, 3, 640, 640), dtype=cuda.float32, device="cuda")
    scales, pads = ops.letterbox_to_device(frames, out, UNIT)
    cuda.cuda.synchronize()
    assert exact(out.cpu().numpy(), orc.letterbox(frames, (640, 640)))
    assert scales.dtype == np.float32 and pads.shape == (5, 2)


def test_letterbox_batch_returns_host_result(cuda, ops, orc):
    frames = frames_u8(2, (480, 640), seed=4)
    r = ops.letterbox_batch(frames, (256, 256), IMAGENET_BGR, pad_value=0)
    assert isinstance(r.tensor, np.ndarray) and r.tensor.dtype == np.float32
    want = orc.letterbox(frames, (256, 256), IMAGENET_BGR.mean, IMAGENET_BGR.std, False, 0)
    assert exact(r.tensor, want)
    assert r.extents.tolist() == [[192, 256]] * 2 and r.pads.tolist() == [[0, 32]] * 2


def test_refusals_are_validation_errors(cuda, ops):
    frames = frames_u8(2, (64, 64))
    with pytest.raises(ValidationError, match="float32"):
        ops.letterbox_to_device(frames, cuda.empty((2, 3, 32, 32), dtype=cuda.float64, device="cuda"), UNIT)
    with pytest.raises(ValidationError, match="contiguous"):
        ops.letterbox_to_device(
            frames, cuda.empty((2, 32, 32, 3), dtype=cuda.float32, device="cuda").permute(0, 3, 1, 2), UNIT
        )
    with pytest.raises(ValidationError, match="rows"):
        ops.letterbox_to_device(frames, cuda.empty((1, 3, 32, 32), dtype=cuda.float32, device="cuda"), UNIT)
    with pytest.raises(ValidationError, match="CUDA tensor"):
        ops.letterbox_to_device(frames, cuda.empty((2, 3, 32, 32)), UNIT)
    with pytest.raises(ValueError):
        ops.letterbox_to_device([], cuda.empty((2, 3, 32, 32), device="cuda"), UNIT)
