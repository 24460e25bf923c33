"""The CPU oracle against golden vectors produced by the reference itself (CPU tier).

tests/golden/make_golden.py ran the reference's TorchImageOps / NumpyImageOps / plan_shards
on seeded inputs; these tests check the C oracle (oracle/oracle.c) against those outputs, so
every GPU parity test downstream inherits a checker pinned to the reference.

Tolerances, stated per case:
* crop, NMS, geometry, and letterbox geometries with exact ratios: bit-exact;
* letterbox at a non-dyadic ratio with fractional taps (33x77 -> 100x37): the oracle follows
  torch's CUDA bilinear formulation, the reference CPU path blends in another order, so the
  two differ by at most 2 ulp of the unnormalised value (0-255 scale).
"""

from __future__ import annotations

import hashlib
import json
from pathlib import Path

import numpy as np
import pytest

from _data import IMAGENET_MEAN, IMAGENET_STD, camera_mix, crop_boxes, frames_u8, kernels_bench_inputs, nms_heads

GOLDEN = Path(__file__).resolve().parent / "golden"


def sha(a: np.ndarray) -> str:
    return hashlib.sha256(np.ascontiguousarray(a).tobytes()).hexdigest()


@pytest.fixture(scope="module")
def orc():
    from oracle import oracle

    oracle.build()
    return oracle


def test_letterbox_geometry(orc):
    for case in json.loads((GOLDEN / "geometry.json").read_text()):
        scale, pad_x, pad_y, new_w, new_h = orc.letterbox_fit(*case["src"], *case["dst"])
        assert np.float32(scale) == np.float32(case["scale"]), case
        assert [pad_x, pad_y] == case["pad"] and [new_h, new_w] == case["extent"], case


def test_known_geometry_answers(orc):
    """test_ops_parity.py:44-48 and test_dataplane.cpp:297-306,345-346."""
    assert orc.letterbox_fit(720, 1280, 256, 256)[:3] == (np.float32(0.2), 0, 56)
    assert orc.letterbox_fit(1080, 1920, 640, 640)[1:] == (0, 140, 640, 360)
    assert orc.letterbox_fit(251, 500, 250, 250)[4] == 126  # 125.5 rounds half to even
    assert orc.letterbox_fit(90, 160, 64, 64)[1:] == (0, 14, 64, 36)


LETTERBOX = np.load(GOLDEN / "letterbox.npz")
LB_CASES = sorted({k.split("/")[0] for k in LETTERBOX.files})


@pytest.mark.parametrize("name", LB_CASES)
def test_letterbox_against_reference_cpu(orc, name):
    seed, dh, dw, pad, swap = LETTERBOX[f"{name}/meta"].tolist()
    shapes = [tuple(s) for s in LETTERBOX[f"{name}/shapes"].tolist()]
    norm = LETTERBOX[f"{name}/norm"]
    rng = np.random.default_rng(seed)
    frames = [rng.integers(0, 256, (*hw, 3), dtype=np.uint8) for hw in shapes]
    got = orc.letterbox(frames, (dh, dw), norm[:3], norm[3:], bool(swap), pad)
    want = LETTERBOX[f"{name}/out"]
    assert got.shape == want.shape and got.dtype == want.dtype
    if name in EXACT_TAPS:
        assert np.array_equal(got.view(np.uint32), want.view(np.uint32)), f"max |d| {np.abs(got - want).max()}"
    else:
        # Fractional taps at a non-dyadic ratio: torch's CPU bilinear blends in another order
        # than its CUDA kernel (which the oracle and the kernels follow bit for bit), so the
        # pixel value may differ by up to 3 ulp of the 0-255 scale (3 * 2^-16 * 2) before
        # normalisation; afterwards that is 3 * 2^-15 / std, plus one ulp of the output.
        std = np.asarray(norm[3:], np.float32)[None, :, None, None]
        tol = 3 * 2.0**-15 / std + np.spacing(np.abs(want).astype(np.float32))
        assert (np.abs(got - want) <= tol).all(), f"max |d| {np.abs(got - want).max()}"


#: Cases whose resize ratios make every tap weight exact (dyadic ratios): bit-exact to the CPU.
EXACT_TAPS = {"90x160-64-unit", "61x45-32x48-imagenet-pad0", "1x1-8"}


def test_letterbox_config1_hash(orc):
    hashes = json.loads((GOLDEN / "hashes.json").read_text())
    frames = frames_u8(8, (1080, 1920), seed=0)
    assert sha(orc.letterbox(frames, (640, 640))) == hashes["config1_letterbox_f32"]


CROP = np.load(GOLDEN / "crop.npz")
CROP_CASES = sorted({k.split("/")[0] for k in CROP.files if "/" in k and not k.startswith("kernels_bench")})


@pytest.mark.parametrize("case", CROP_CASES)
def test_crop_cases_against_reference_cpu(orc, case):
    image, boxes = CROP[f"{case}/image"], CROP[f"{case}/boxes"]
    dst = tuple(CROP[f"{case}/dst"].tolist())
    for pid, row in zip(CROP["param_ids"].tolist(), CROP["params"]):
        got = orc.crop([image], boxes, dst, None, row[:3], row[3:6], bool(row[6]))
        want = CROP[f"{case}/{pid}"]
        assert np.array_equal(got.view(np.uint32), want.view(np.uint32)), f"{case}/{pid}"


def test_crop_kernel_benchmark_boxes(orc):
    frame, boxes, _, _ = kernels_bench_inputs(0)
    assert np.array_equal(boxes, CROP["kernels_bench/boxes"])
    got = orc.crop([frame], boxes, (256, 128))
    assert sha(got) == str(CROP["kernels_bench/out_sha256"])


def test_crop_config3_hash(orc):
    hashes = json.loads((GOLDEN / "hashes.json").read_text())
    frames = frames_u8(8, (1080, 1920), seed=0)
    boxes, idx = crop_boxes(8, 64)
    got = orc.crop(frames, boxes, (256, 128), idx, IMAGENET_MEAN, IMAGENET_STD, True)
    assert sha(got.astype(np.float16)) == hashes["config3_crop_f16"]


NMS = np.load(GOLDEN / "nms.npz")


def test_nms_known_answers(orc):
    b, s = NMS["known/boxes"], NMS["known/scores"]
    assert orc.nms(b, s, 0.5, 0.1, 10).tolist() == NMS["known/a"].tolist() == [2, 0, 4]
    assert orc.nms(b, s, 0.5, 0.85, 10).tolist() == NMS["known/b"].tolist() == [2, 0]
    assert orc.nms(b, s, 0.5, 0.0, 1).tolist() == NMS["known/c"].tolist() == [2]
    assert orc.nms(np.empty((0, 4), np.float32), np.empty(0, np.float32), 0.5, 0.1, 10).size == 0


def test_nms_hundred_fleets(orc):
    for trial in range(100):
        iou, floor, count = NMS[f"fleet{trial}/args"].tolist()
        got = orc.nms(NMS[f"fleet{trial}/boxes"], NMS[f"fleet{trial}/scores"], iou, floor, int(count))
        assert got.tolist() == NMS[f"fleet{trial}/kept"].tolist(), trial


def test_nms_kernel_benchmark_case(orc):
    _, _, b, s = kernels_bench_inputs(0)
    assert orc.nms(b, s, 0.45, 0.25, 300).tolist() == NMS["kernels_bench/kept"].tolist()


def test_nms_config2_class_aware(orc):
    b, s, c = nms_heads(16, 8400, 2, seed=0)
    keep, counts = orc.nms_batched(b, s, c, 0.45, 0.25, 300, num_classes=2)
    assert np.array_equal(keep, NMS["config2/keep"]) and np.array_equal(counts, NMS["config2/counts"])


def test_camera_partition_matches_plan_shards():
    from shipinfer_b200.shard import plan_cameras

    fps, _ = camera_mix()
    load = {f"cam{c:02d}": f for c, f in fps.items()}
    for g, shards in json.loads((GOLDEN / "shards.json").read_text()).items():
        assert [list(s) for s in plan_cameras(load, list(range(int(g))))] == shards


def _decode_cases():
    data = np.load(GOLDEN / "decode.npz")
    n = len([k for k in data.files if k.startswith("rows_")])
    return data, n


def test_decode_against_reference(orc):
    """The C restatement of decode_detections against the reference's own outputs
    (topology/elements/detections.py:423-515), bit for bit."""
    data, n = _decode_cases()
    assert n == 24
    for i in range(n):
        count, scale, pad_x, pad_y, fh, fw, thr, cap = data[f"args_{i}"].tolist()
        boxes, scores, classes, discarded = orc.decode(
            data[f"rows_{i}"], score_threshold=thr, max_detections=int(cap), scale=scale, pad=(pad_x, pad_y),
            frame_hw=None if fh < 0 else (int(fh), int(fw)), count=None if count < 0 else int(count))
        assert np.array_equal(boxes.view(np.uint32), data[f"boxes_{i}"].view(np.uint32)), i
        assert np.array_equal(scores.view(np.uint32), data[f"scores_{i}"].view(np.uint32)), i
        assert np.array_equal(classes, data[f"classes_{i}"]), i
        assert discarded == int(data[f"discarded_{i}"][0]), i


@pytest.mark.parametrize(("mean", "std"), [((0.0, 0.0, 0.0), (255.0, 255.0, 255.0)), (IMAGENET_MEAN, IMAGENET_STD)],
                         ids=["unit", "imagenet"])
def test_two_to_one_reduction_is_the_quarter_sum(orc, mean, std):
    """At an exact 2:1 reduction every tap weight is 1/2, so the bilinear value is exactly the
    four taps' sum over 4 and the output is normalise(S / 4) — the premise of the GPU kernel's
    integer-sum path, checked here on the oracle (itself pinned to the reference above)."""
    frame = frames_u8(1, (90, 160), seed=31)[0]
    got = orc.letterbox([frame], (45, 80), mean, std, True, 114)[0]
    p = frame.astype(np.int64)
    s = p[0::2, 0::2] + p[0::2, 1::2] + p[1::2, 0::2] + p[1::2, 1::2]  # [45, 80, 3] BGR sums
    v = (s.astype(np.float32) * np.float32(0.25))[..., ::-1]          # exact; channels to RGB
    want = ((v - np.float32(mean)) / np.float32(std)).astype(np.float32).transpose(2, 0, 1)
    assert np.array_equal(got.view(np.uint32), want.view(np.uint32))
