"""NV12 letterbox on the GPU, through the C ABI.

* BT.601 + nearest is the reference's own NV12 kernel (csrc/shipinfer/runtime/ops.cu:148-194):
  bit-exact against the oracle, and — when oracle/_ref/libshipref.so (the reference's kernels
  compiled from its sources) is present — bit-exact against the reference kernel itself.
* BT.709 + bilinear (config 5) has no reference implementation. It is pinned twice: bit-exact
  against the oracle's C restatement, and bit-exact against an independent composition of torch
  CUDA ops (``torch_nv12_letterbox``): the whole frame converted to RGB by the limited-range
  matrix built from Kr/Kb, then ``F.interpolate(bilinear, align_corners=False)``, pasted on the
  pad canvas, flipped, ``sub_``/``div_`` — the reference's own letterbox sequence
  (torch_ops.py:349-403) run on the converted frame. Bilinear after conversion is the same
  definition as converting each tap and blending, because the blend is linear in its taps.
"""

from __future__ import annotations

import ctypes
from pathlib import Path

import numpy as np
import pytest

from _data import nv12_frames, yuv_constants
from shipinfer_b200 import NormalizeParams, Nv12Frame, ValidationError

pytestmark = pytest.mark.gpu

REF_LIB = Path(__file__).resolve().parents[1] / "oracle" / "_ref" / "libshipref.so"


def exact(a: np.ndarray, b: np.ndarray) -> bool:
    return a.shape == b.shape and a.dtype == b.dtype and np.array_equal(a.view(np.uint8), b.view(np.uint8))


def run(torch, ops, planes, dst, dtype, matrix, sampling, params=NormalizeParams(), pad=114):
    frames = [Nv12Frame(torch.from_numpy(buf).cuda(), h, w, pitch, uv) for buf, h, w, pitch, uv in planes]
    out = torch.empty((len(planes), 3, *dst), dtype=dtype, device="cuda")
    ops.letterbox_nv12_device(frames, out, params, pad_value=pad, matrix=matrix, sampling=sampling)
    torch.cuda.synchronize()
    return out.cpu().numpy()


CASES = [
    pytest.param((90, 160), 160, 90, (64, 64), id="tight-90x160"),
    pytest.param((90, 160), 192, 96, (64, 64), id="padded-nvdec-surface"),
    pytest.param((1080, 1920), 2048, 1088, (640, 640), id="1080p-padded"),
    pytest.param((37, 51), 64, 40, (50, 50), id="odd-sizes"),
    # ratio RN(1/3): tap weights of 2^-26 next to conversions as small as 2^-26, so the kernel
    # keeps its tiny-numerator test on for the default zero-mean constants
    pytest.param((40, 60), 64, 40, (120, 180), id="3x-upscale-tiny-weights"),
]


@pytest.mark.parametrize(("hw", "pitch", "coded_h", "dst"), CASES)
@pytest.mark.parametrize(("matrix", "sampling"), [(601, "nearest"), (709, "bilinear"), (601, "bilinear"),
                                                  (709, "nearest")])
def test_matches_oracle(cuda, ops, orc, hw, pitch, coded_h, dst, matrix, sampling):
    planes = nv12_frames(2, hw, seed=hw[0], pitch=pitch, coded_h=coded_h)
    want = orc.letterbox_nv12(planes, dst, matrix=matrix, sampling=0 if sampling == "nearest" else 1)
    got = run(cuda, ops, planes, dst, cuda.float32, matrix, sampling)
    assert exact(got, want), f"max |d| {np.abs(got - want).max()}"
    got16 = run(cuda, ops, planes, dst, cuda.float16, matrix, sampling)
    assert exact(got16, want.astype(np.float16))


def torch_nv12_letterbox(torch, planes, dst, matrix, sampling_bilinear=True, mean=(0.0, 0.0, 0.0),
                         std=(255.0, 255.0, 255.0), pad=114.0, swap_rb=True):
    """The NV12 letterbox composed of torch CUDA ops, sharing no code with the kernel or the
    oracle. Conversion per pixel (chroma co-sited: column 2*(x//2), row y//2, as nv12_to_bgr):
    Y' = float32((Y - 16) * ys); B = Y' + cbu*U; G = (Y' - cgu*U) - cgv*V; R = Y' + crv*V, each
    sum computed in float64 and rounded once to float32 — the value of the fused multiply-add
    nvcc makes of each, since every product and sum here is exact in float64 (at most 36
    significant bits) — then clamped to [0, 255]. Then F.interpolate(bilinear,
    align_corners=False) to the placement's extent, the pad canvas, flip, sub_, div_
    (torch_ops.py:349-403)."""
    import torch.nn.functional as F

    ys, cbu, cgu, cgv, crv = (float(np.float32(v)) for v in yuv_constants(matrix))
    dh, dw = dst
    out = torch.empty((len(planes), 3, dh, dw), dtype=torch.float32, device="cuda")
    for i, (buf, h, w, pitch, uv) in enumerate(planes):
        d = torch.from_numpy(buf).cuda()
        luma = d[: pitch * h].view(h, pitch)[:, :w].float()
        ch = (h + 1) // 2
        chroma = d[uv: uv + pitch * ch].view(ch, pitch)[:, : ((w + 1) // 2) * 2].view(ch, -1, 2)
        u = chroma[:, :, 0].repeat_interleave(2, 0).repeat_interleave(2, 1)[:h, :w].double() - 128.0
        v = chroma[:, :, 1].repeat_interleave(2, 0).repeat_interleave(2, 1)[:h, :w].double() - 128.0
        yp = ((luma - 16.0) * torch.tensor(ys, dtype=torch.float32, device="cuda")).double()
        b = (yp + cbu * u).float()
        g = ((yp - cgu * u).float().double() - cgv * v).float()
        r = (yp + crv * v).float()
        bgr = torch.stack([b, g, r]).clamp_(0.0, 255.0)[None]
        s = min(dh / h, dw / w)  # torch_ops.py:374-378, Python floats
        nh, nw = max(1, round(h * s)), max(1, round(w * s))
        py, px = (dh - nh) // 2, (dw - nw) // 2
        mode = "bilinear" if sampling_bilinear else "nearest"
        kw = {"align_corners": False} if sampling_bilinear else {}
        resized = F.interpolate(bgr, size=(nh, nw), mode=mode, **kw)
        canvas = torch.full((1, 3, dh, dw), float(pad), dtype=torch.float32, device="cuda")
        canvas[:, :, py: py + nh, px: px + nw] = resized
        if swap_rb:
            canvas = canvas.flip(1)
        m = torch.tensor(mean, dtype=torch.float32, device="cuda").view(1, 3, 1, 1)
        sd = torch.tensor(std, dtype=torch.float32, device="cuda").view(1, 3, 1, 1)
        out[i] = canvas.sub_(m).div_(sd)[0]
    torch.cuda.synchronize()
    return out.cpu().numpy()


TORCH_CASES = [
    pytest.param((2160, 3840), 3840, 2160, (1280, 1280), id="config5-4k"),
    pytest.param((90, 160), 192, 96, (64, 64), id="padded-surface-downscale"),
    pytest.param((37, 51), 64, 40, (50, 50), id="odd-sizes-upscale"),
    pytest.param((1080, 1920), 2048, 1088, (640, 640), id="1080p-exact-taps"),
    pytest.param((720, 1280), 1280, 720, (416, 416), id="720p-non-dyadic"),
    pytest.param((40, 60), 64, 40, (120, 180), id="3x-upscale-tiny-weights"),
]


@pytest.mark.parametrize(("hw", "pitch", "coded_h", "dst"), TORCH_CASES)
@pytest.mark.parametrize("params", [NormalizeParams(),
                                    NormalizeParams(mean=(123.7, 116.3, 103.5), std=(58.4, 57.1, 57.4))],
                         ids=["unit", "imagenet"])
def test_709_bilinear_matches_a_torch_composition(cuda, ops, hw, pitch, coded_h, dst, params):
    """Config 5's definition pinned independently of this build's oracle: bit-exact in fp32 and
    after the fp16 rounding."""
    planes = nv12_frames(2 if hw[0] >= 1080 else 3, hw, seed=hw[1], pitch=pitch, coded_h=coded_h)
    want = torch_nv12_letterbox(cuda, planes, dst, 709, mean=params.mean, std=params.std, swap_rb=params.swap_rb)
    got = run(cuda, ops, planes, dst, cuda.float32, 709, "bilinear", params)
    assert exact(got, want), f"{np.count_nonzero(got != want)} values differ, max |d| {np.abs(got - want).max()}"
    got16 = run(cuda, ops, planes, dst, cuda.float16, 709, "bilinear", params)
    assert exact(got16, want.astype(np.float16))


def test_config5_4k_bilinear_709_fp16(cuda, ops, orc):
    """Config 5 shape (batch reduced to 2 for test time): 3840x2160 NV12 -> 1280x1280 fp16."""
    planes = nv12_frames(2, (2160, 3840), seed=0)
    want = orc.letterbox_nv12(planes, (1280, 1280), matrix=709, sampling=1)
    got = run(cuda, ops, planes, (1280, 1280), cuda.float16, 709, "bilinear")
    assert exact(got, want.astype(np.float16))


@pytest.mark.skipif(not REF_LIB.exists(), reason="oracle/_ref/libshipref.so not built")
@pytest.mark.parametrize(("hw", "pitch", "coded_h", "dst"), CASES)
def test_nearest_601_matches_the_reference_kernel(cuda, ops, hw, pitch, coded_h, dst):
    """The reference's nv12_letterbox_into, compiled from its own source, on the same surface."""
    ref = ctypes.CDLL(str(REF_LIB))
    ref.ref_nv12_letterbox.argtypes = [ctypes.c_void_p, ctypes.c_int, ctypes.c_int, ctypes.c_int,
                                       ctypes.c_ulonglong, ctypes.c_void_p, ctypes.c_int, ctypes.c_int,
                                       ctypes.c_int, ctypes.c_float, ctypes.c_void_p, ctypes.c_void_p]
    (buf, h, w, p, uv), = nv12_frames(1, hw, seed=5, pitch=pitch, coded_h=coded_h)
    dev = cuda.from_numpy(buf).cuda()
    theirs = cuda.empty((1, 3, *dst), dtype=cuda.float32, device="cuda")
    pad = np.float32(114) / np.float32(255)
    rc = ref.ref_nv12_letterbox(dev.data_ptr(), h, w, p, uv, theirs.data_ptr(), dst[0], dst[1], 1,
                                float(pad), None, None)
    assert rc == 0
    mine = run(cuda, ops, [(buf, h, w, p, uv)], dst, cuda.float32, 601, "nearest")
    cuda.cuda.synchronize()
    assert exact(mine, theirs.cpu().numpy())


def test_layout_refusals_match_the_reference(cuda, ops):
    buf = cuda.zeros(192 * 96 * 2, dtype=cuda.uint8, device="cuda")
    out = cuda.empty((1, 3, 64, 64), device="cuda")
    with pytest.raises(ValidationError, match="inside the luma plane"):
        ops.letterbox_nv12_device([Nv12Frame(buf, 90, 160, 192, 192 * 80)], out, NormalizeParams())
    with pytest.raises(ValidationError, match="narrower than the width"):
        ops.letterbox_nv12_device([Nv12Frame(buf, 90, 160, 100, 100 * 90)], out, NormalizeParams())
