"""The kernels against the reference's own CUDA path, by hash.

``tests/golden/cuda_hashes.json`` holds SHA-256s of ``TorchImageOps(device_index=0)`` outputs —
the reference's letterbox (``torch_ops.py:349-403``) and crop (``torch_ops.py:405-507``) run by
the reference's own code on a B200 — written by ``tests/golden/make_cuda_golden.py``. Here the
sm_100a kernels compute the same outputs from the same seeded inputs, through the C ABI, and
their bytes must hash the same: bit-exact to the reference's CUDA formulation, including the
non-dyadic letterbox geometries where torch's CPU and CUDA blends part, config 1, config 3 and
the reference's 12 crop geometry cases under its 4 normalisations.
"""

from __future__ import annotations

import hashlib
import json
import sys
from pathlib import Path

import numpy as np
import pytest

from _data import IMAGENET_MEAN, IMAGENET_STD, crop_boxes, frames_u8, kernels_bench_inputs
from shipinfer_b200 import NormalizeParams

pytestmark = pytest.mark.gpu

GOLDEN = Path(__file__).resolve().parent / "golden"
HASHES = GOLDEN / "cuda_hashes.json"
sys.path.insert(0, str(GOLDEN))

from make_cuda_golden import LETTERBOX_CASES, letterbox_inputs  # noqa: E402

NORMS = {
    "unit": NormalizeParams(),
    "imagenet": NormalizeParams(mean=IMAGENET_MEAN, std=IMAGENET_STD),
    "imagenet-bgr": NormalizeParams(mean=IMAGENET_MEAN, std=IMAGENET_STD, swap_rb=False),
}


def sha(a: np.ndarray) -> str:
    return hashlib.sha256(np.ascontiguousarray(a).tobytes()).hexdigest()


@pytest.fixture(scope="module")
def hashes():
    if not HASHES.exists():
        pytest.fail("tests/golden/cuda_hashes.json is missing: run tests/golden/make_cuda_golden.py on a B200")
    return json.loads(HASHES.read_text())


@pytest.mark.parametrize("case", LETTERBOX_CASES, ids=[c[0] for c in LETTERBOX_CASES])
@pytest.mark.parametrize("dtype", ["f32", "f16"])
def test_letterbox_hashes_equal_the_reference_cuda_path(cuda, ops, hashes, case, dtype):
    name, shapes, seed, dst, norm, pad = case
    frames = frames_u8(8, shapes[0], seed=0) if name == "config1" else letterbox_inputs(shapes, seed)
    dev = [cuda.from_numpy(f).cuda() for f in frames]
    out = cuda.empty((len(frames), 3, *dst), dtype=cuda.float32 if dtype == "f32" else cuda.float16, device="cuda")
    ops.letterbox_device(dev, out, NORMS[norm], pad_value=pad)
    cuda.cuda.synchronize()
    assert sha(out.cpu().numpy()) == hashes[f"letterbox/{name}/{dtype}"]


def _crop(torch, ops, frames, boxes, dst, params, dtype, frame_index=None):
    dev = [torch.from_numpy(np.ascontiguousarray(f)).cuda() for f in frames]
    out = torch.empty((len(boxes), 3, *dst), dtype=dtype, device="cuda")
    bidx = None if frame_index is None else torch.from_numpy(np.asarray(frame_index, np.int32)).cuda()
    ops.crop_device(dev, torch.from_numpy(np.asarray(boxes, np.float32)).cuda(), out, params, box_frame=bidx)
    torch.cuda.synchronize()
    return out.cpu().numpy()


@pytest.mark.parametrize("dtype", ["f32", "f16"])
def test_config3_crops_hash_equal_the_reference_cuda_path(cuda, ops, hashes, dtype):
    frames = frames_u8(8, (1080, 1920), seed=0)
    boxes, idx = crop_boxes(8, 64)
    got = _crop(cuda, ops, frames, boxes, (256, 128), NORMS["imagenet"],
                cuda.float32 if dtype == "f32" else cuda.float16, idx)
    assert sha(got) == hashes[f"crop/config3/{dtype}"]


def test_reference_crop_cases_hash_equal_the_reference_cuda_path(cuda, ops, hashes):
    table = np.load(GOLDEN / "crop.npz")
    params = {pid: NormalizeParams(mean=tuple(row[:3]), std=tuple(row[3:6]), swap_rb=bool(row[6]))
              for pid, row in zip(table["param_ids"], table["params"])}
    cases = sorted({k.split("/")[0] for k in table.files if k.endswith("/image")})
    assert len(cases) == 12
    for cid in cases:
        image, boxes = table[f"{cid}/image"], table[f"{cid}/boxes"]
        dst = tuple(int(v) for v in table[f"{cid}/dst"])
        for pid, p in params.items():
            if len(boxes) == 0:
                got = np.zeros((0, 3, *dst), np.float32)
            else:
                got = _crop(cuda, ops, [image], boxes, dst, p, cuda.float32)
            assert sha(got) == hashes[f"crop/case/{cid}/{pid}"], (cid, pid)
    frame, kb, _, _ = kernels_bench_inputs(0)
    assert sha(_crop(cuda, ops, [frame], kb, (256, 128), NormalizeParams(), cuda.float32)) == \
        hashes["crop/kernels_bench/f32"]
