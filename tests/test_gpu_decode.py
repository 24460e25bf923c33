"""Detector decode on the GPU (shipk_decode_detections) against the reference and the oracle.

Bar: bit-exact boxes, scores, class ids, counts and discarded counts. The golden cases are the
reference's own ``decode_detections`` outputs (tests/golden/decode.npz, written by
tests/golden/make_golden.py); the batched cases compare with the oracle's restatement.
"""

from __future__ import annotations

from pathlib import Path

import numpy as np
import pytest

from shipinfer_b200 import ConfigurationError, ValidationError
from shipinfer_b200.decode import DecodeParams, decode_detections, decode_detections_device

pytestmark = pytest.mark.gpu

GOLDEN = Path(__file__).resolve().parent / "golden" / "decode.npz"


def bits(a: np.ndarray) -> np.ndarray:
    return np.ascontiguousarray(a).view(np.uint32)


def test_reference_cases_bit_exact(cuda):
    data = np.load(GOLDEN)
    for i in range(24):
        count, scale, pad_x, pad_y, fh, fw, thr, cap = data[f"args_{i}"].tolist()
        d = decode_detections(
            data[f"rows_{i}"], params=DecodeParams(score_threshold=thr, max_detections=int(cap)), scale=scale,
            pad=(pad_x, pad_y), frame_hw=None if fh < 0 else (int(fh), int(fw)),
            count=None if count < 0 else int(count))
        assert np.array_equal(bits(d.boxes), bits(data[f"boxes_{i}"])), i
        assert np.array_equal(bits(d.scores), bits(data[f"scores_{i}"])), i
        assert np.array_equal(d.class_ids, data[f"classes_{i}"]), i
        assert d.discarded == int(data[f"discarded_{i}"][0]), i
        assert len(d.labels) == len(d)


def _batch(B: int, R: int, seed: int):
    rng = np.random.default_rng(seed)
    rows = np.empty((B, R, 6), np.float32)
    rows[..., :4] = rng.uniform(-30.0, 700.0, (B, R, 4))
    rows[..., 4] = rng.uniform(0.0, 1.0, (B, R))
    rows[::2, :, 4] = np.round(rows[::2, :, 4] * 16) / 16  # ties in every other frame
    rows[..., 5] = rng.uniform(0.0, 80.0, (B, R))
    rows[1, :7, 0] = np.nan
    rows[1, 7:9, 4] = np.nan
    rows[1, 9:12, 1] = np.inf
    rows[1, 12:14, 2] = -np.inf
    rows[1, 14, 3] = np.float32(-np.nan)  # a NaN with the sign bit set keeps it
    scales = np.array([np.float32(1 / 3), 0.5, 1.0, np.float32(0.29999998)] * (B // 4), np.float32)[:B]
    pads = rng.integers(0, 300, (B, 2)).astype(np.float32)
    hw = np.stack([rng.integers(200, 2200, B), rng.integers(200, 4000, B)], axis=1).astype(np.int32)
    counts = rng.integers(-5, R + 50, B).astype(np.int32)
    return rows, scales, pads, hw, counts


@pytest.mark.parametrize(("thr", "cap"), [(0.25, 300), (0.0, 4096), (0.5, 1), (0.9, 100), (0.3, 0)])
@pytest.mark.parametrize("with_counts", [False, True])
def test_batched_matches_oracle(cuda, orc, thr, cap, with_counts):
    B, R = 8, 8400
    rows, scales, pads, hw, counts = _batch(B, R, seed=int(thr * 100) + cap)
    t = lambda a: cuda.from_numpy(a).cuda()  # noqa: E731
    boxes, scores, classes, n, discarded = decode_detections_device(
        t(rows), t(scales), t(pads), score_threshold=thr, max_detections=cap, frame_hw=t(hw),
        counts=t(counts) if with_counts else None)
    cuda.cuda.synchronize()
    boxes, scores, classes, n, discarded = (x.cpu().numpy() for x in (boxes, scores, classes, n, discarded))
    for b in range(B):
        wb, ws, wc, wd = orc.decode(rows[b], score_threshold=thr, max_detections=cap, scale=float(scales[b]),
                                    pad=(float(pads[b, 0]), float(pads[b, 1])), frame_hw=(int(hw[b, 0]), int(hw[b, 1])),
                                    count=int(counts[b]) if with_counts else None)
        k = len(ws)
        assert n[b] == k and discarded[b] == wd, b
        assert np.array_equal(bits(boxes[b, :k]), bits(wb)), b
        assert np.array_equal(bits(scores[b, :k]), bits(ws)), b
        assert np.array_equal(classes[b, :k], wc), b
        assert (classes[b, k:] == -1).all() and (scores[b, k:] == 0).all()


@pytest.mark.parametrize("spread", ["equal", "low_byte", "two_low_bytes", "unstaged"])
def test_narrow_score_spreads(cuda, orc, spread):
    """The radix select starts at the first byte of the order bits in which the passing rows'
    scores differ: none (every passing score equal, so only row bits separate the keys), the
    lowest byte, the two lowest bytes; and a frame too long to stage its scores in shared
    memory (read from global memory on every pass)."""
    B, R = 4, 20000 if spread == "unstaged" else 8400
    rows, scales, pads, hw, _ = _batch(B, R, seed=11)
    rng = np.random.default_rng(12)
    if spread != "unstaged":
        base = np.float32(0.7).view(np.uint32) & np.uint32(0xFFFF0000)  # about 0.6992
        width = {"equal": 1, "low_byte": 256, "two_low_bytes": 65536}[spread]
        passing = rng.random((B, R)) < 0.8
        s = (base + rng.integers(0, width, (B, R)).astype(np.uint32)).view(np.float32)
        rows[..., 4] = np.where(passing, s, np.float32(0.1))
    t = lambda a: cuda.from_numpy(a).cuda()  # noqa: E731
    for cap in (100, 1):
        boxes, scores, classes, n, discarded = decode_detections_device(
            t(rows), t(scales), t(pads), score_threshold=0.25, max_detections=cap, frame_hw=t(hw))
        cuda.cuda.synchronize()
        boxes, scores, classes, n, discarded = (x.cpu().numpy() for x in (boxes, scores, classes, n, discarded))
        for b in range(B):
            wb, ws, wc, wd = orc.decode(rows[b], score_threshold=0.25, max_detections=cap, scale=float(scales[b]),
                                        pad=(float(pads[b, 0]), float(pads[b, 1])),
                                        frame_hw=(int(hw[b, 0]), int(hw[b, 1])))
            k = len(ws)
            assert n[b] == k == cap and discarded[b] == wd, (spread, cap, b)
            assert np.array_equal(bits(boxes[b, :k]), bits(wb)), (spread, cap, b)
            assert np.array_equal(bits(scores[b, :k]), bits(ws)), (spread, cap, b)
            assert np.array_equal(classes[b, :k], wc), (spread, cap, b)


def test_without_clip_and_empty_frames(cuda, orc):
    rows, scales, pads, _, _ = _batch(4, 257, seed=3)
    t = lambda a: cuda.from_numpy(a).cuda()  # noqa: E731
    boxes, scores, classes, n, discarded = decode_detections_device(
        t(rows), t(scales), t(pads), score_threshold=0.2, max_detections=50,
        counts=t(np.array([0, 257, 1, 300], np.int32)))
    cuda.cuda.synchronize()
    for b, count in enumerate([0, 257, 1, 300]):
        wb, ws, wc, wd = orc.decode(rows[b], score_threshold=0.2, max_detections=50, scale=float(scales[b]),
                                    pad=(float(pads[b, 0]), float(pads[b, 1])), count=count)
        k = len(ws)
        assert int(n[b]) == k and int(discarded[b]) == wd
        assert np.array_equal(bits(boxes[b, :k].cpu().numpy()), bits(wb))


def test_refusals(cuda):
    rows = cuda.zeros((2, 10, 6), dtype=cuda.float32, device="cuda")
    s, p = cuda.ones(2, device="cuda"), cuda.zeros((2, 2), device="cuda")
    with pytest.raises(ConfigurationError):
        decode_detections_device(rows, s, p, max_detections=5000)
    with pytest.raises(ValidationError):
        decode_detections_device(rows[:, :, :5].contiguous(), s, p)
    with pytest.raises(ValidationError):
        decode_detections(np.zeros((4, 5), np.float32), params=DecodeParams())
