"""Generate the golden fixtures by running the REFERENCE's own CPU implementations.

Run where the reference source tree is available (it is imported, never copied):

    python tests/golden/make_golden.py [--reference /path/to/shipinfer]

It imports ``shipinfer.runtime.ops`` from ``<reference>/src`` and records, for seeded inputs:

* ``geometry.json`` — letterbox placements (scale, pads, extents) from
  ``TorchImageOps._letterbox`` (``torch_ops.py:373-394``);
* ``letterbox.npz`` — ``TorchImageOps().letterbox_batch`` outputs on CPU for small frames;
* ``crop.npz`` — ``TorchImageOps().crop_batch`` for the reference's 12 crop geometry cases
  (``tests/runtime/test_torch_crop_batch.py``) x 4 normalisations, plus 15 kernel-benchmark
  boxes (``benchmarks/kernels.py:298-320``);
* ``nms.npz`` — ``NumpyImageOps().nms``: the known answers, 100 random fleets, the kernel
  benchmark's 25 000-candidate case, and config 2 (16 x 8400, per class + merge);
* ``hashes.json`` — SHA-256 of full-size reference outputs (config 1 letterbox fp32, config 3
  crops fp16) that are too large to commit, with the seeds that regenerate their inputs;
* ``shards.json`` — ``plan_shards`` on config 4's 50-camera fleet for 1, 2, 4 and 8 GPUs;
* ``decode.npz`` — ``decode_detections`` (``topology/elements/detections.py:423-515``) on 24
  seeded detector outputs: ties, NaN and infinite values, signed zeros, counts, caps, a zero
  scale and frames without a clamp.

The tests in ``tests/test_oracle_golden.py`` check the C oracle against these files, so the
oracle is pinned to the reference itself.
"""

from __future__ import annotations

import argparse
import hashlib
import json
import sys
from pathlib import Path

import numpy as np

HERE = Path(__file__).resolve().parent
sys.path.insert(0, str(HERE.parent))

from _data import (  # noqa: E402
    IMAGENET_MEAN, IMAGENET_STD, camera_mix, crop_boxes, frames_u8, kernels_bench_inputs, nms_heads,
)


def sha(a: np.ndarray) -> str:
    return hashlib.sha256(np.ascontiguousarray(a).tobytes()).hexdigest()


def reference_crop_cases(ref_tests: Path):
    sys.path.insert(0, str(ref_tests))
    import test_torch_crop_batch as T  # the reference's own case table

    cases = [(c.id, c.values[0], np.asarray(c.values[1], np.float32), tuple(c.values[2])) for c in T.CASES]
    params = [(p.id, p.values[0]) for p in T.PARAM_SETS]
    return cases, params


def main() -> None:
    ap = argparse.ArgumentParser()
    ap.add_argument("--reference", default="/root/reference")
    args = ap.parse_args()
    ref = Path(args.reference)
    sys.path.insert(0, str(ref / "src"))
    from shipinfer.runtime.ops import NormalizeParams, NumpyImageOps, TorchImageOps
    from shipinfer.scheduling.sharding import plan_shards

    torch_ops, numpy_ops = TorchImageOps(), NumpyImageOps()

    # ---- geometry
    shapes = [(1080, 1920, 640, 640), (720, 1280, 640, 640), (2160, 3840, 1280, 1280), (480, 640, 256, 256),
              (1280, 720, 256, 256), (720, 1280, 256, 256), (251, 500, 250, 250), (90, 160, 64, 64),
              (300, 300, 256, 256), (640, 200, 320, 320), (33, 77, 100, 37), (1, 1, 8, 8), (97, 131, 13, 640),
              (1000, 1, 64, 64), (3, 1001, 640, 640), (1079, 1921, 640, 640)]
    geometry = []
    for h, w, dh, dw in shapes:
        r = numpy_ops.letterbox_batch([np.zeros((h, w, 3), np.uint8)], (dh, dw), NormalizeParams())
        geometry.append({"src": [h, w], "dst": [dh, dw], "scale": float(r.scales[0]),
                         "pad": [float(v) for v in r.pads[0]], "extent": [int(v) for v in r.extents[0]]})
    (HERE / "geometry.json").write_text(json.dumps(geometry, indent=1))

    # ---- small letterbox outputs (inputs regenerated from the seeds)
    imagenet_bgr = NormalizeParams(mean=(103.5, 116.3, 123.7), std=(57.4, 57.1, 58.4), swap_rb=False)
    lb_cases = [
        ("90x160-64-unit", [(90, 160)], (64, 64), NormalizeParams(), 114, 11),
        ("48x64-40-imagenet-bgr", [(48, 64)], (40, 40), imagenet_bgr, 114, 12),
        ("33x77-100x37-unit", [(33, 77)], (100, 37), NormalizeParams(), 114, 13),
        ("61x45-32x48-imagenet-pad0", [(61, 45)], (32, 48), NormalizeParams(mean=(103.5, 116.3, 123.7),
                                                                               std=(57.4, 57.1, 58.4)), 0, 14),
        ("1x1-8", [(1, 1)], (8, 8), NormalizeParams(), 114, 15),
        ("ragged-48", [(90, 160), (48, 64), (20, 20)], (48, 48), NormalizeParams(), 114, 16),
        ("251x500-50-unit", [(251, 500)], (50, 50), NormalizeParams(), 114, 17),
    ]
    lb = {}
    for name, shapes_, dst, p, pad, seed in lb_cases:
        rng = np.random.default_rng(seed)
        frames = [rng.integers(0, 256, (*hw, 3), dtype=np.uint8) for hw in shapes_]
        r = torch_ops.letterbox_batch(frames, dst, p, pad_value=pad)
        lb[f"{name}/out"] = r.tensor
        lb[f"{name}/meta"] = np.array([seed, dst[0], dst[1], pad, int(p.swap_rb)], np.int64)
        lb[f"{name}/shapes"] = np.array(shapes_, np.int64)
        lb[f"{name}/norm"] = np.array([*p.mean, *p.std], np.float64)
    np.savez_compressed(HERE / "letterbox.npz", **lb)

    # ---- crops: the reference's own case table x normalisations, and the kernel-bench boxes
    cases, params = reference_crop_cases(ref / "tests" / "runtime")
    crop = {}
    for cid, image, boxes, dst in cases:
        crop[f"{cid}/image"] = image
        crop[f"{cid}/boxes"] = boxes
        crop[f"{cid}/dst"] = np.array(dst, np.int64)
        for pid, p in params:
            crop[f"{cid}/{pid}"] = torch_ops.crop_batch(image, boxes, dst, p)
    crop["params"] = np.array([[*p.mean, *p.std, float(p.swap_rb)] for _, p in params], np.float64)
    crop["param_ids"] = np.array([pid for pid, _ in params])
    frame, kb, nms_b, nms_s = kernels_bench_inputs(0)  # benchmarks/kernels.py:_inputs(seed=0)
    crop["kernels_bench/boxes"] = kb
    crop["kernels_bench/out_sha256"] = np.array(sha(torch_ops.crop_batch(frame, kb, (256, 128), NormalizeParams())))
    np.savez_compressed(HERE / "crop.npz", **crop)

    # ---- NMS
    nms = {}
    ka_boxes = np.array([[10, 10, 100, 100], [15, 15, 105, 105], [300, 300, 400, 400], [305, 305, 405, 405],
                         [500, 500, 520, 520]], np.float32)
    ka_scores = np.array([0.90, 0.80, 0.95, 0.70, 0.60], np.float32)
    nms["known/boxes"], nms["known/scores"] = ka_boxes, ka_scores
    nms["known/a"] = numpy_ops.nms(ka_boxes, ka_scores, 0.5, 0.1, 10)
    nms["known/b"] = numpy_ops.nms(ka_boxes, ka_scores, 0.5, 0.85, 10)
    nms["known/c"] = numpy_ops.nms(ka_boxes, ka_scores, 0.5, 0.0, 1)
    rng = np.random.default_rng(7)  # tests/runtime/test_ops_vs_shipvision.py:174-186's fleets
    fleets = []
    for trial in range(100):
        count = int(rng.integers(1, 80))
        corner = rng.random((count, 2)).astype(np.float32) * 100
        extent = rng.random((count, 2)).astype(np.float32) * 40 + 1
        boxes = np.concatenate([corner, corner + extent], axis=1).astype(np.float32)
        scores = rng.random(count).astype(np.float32)
        iou, floor = float(rng.choice([0.3, 0.5, 0.7])), float(rng.choice([0.0, 0.25]))
        kept = numpy_ops.nms(boxes, scores, iou, floor, count)
        nms[f"fleet{trial}/boxes"], nms[f"fleet{trial}/scores"] = boxes, scores
        nms[f"fleet{trial}/args"] = np.array([iou, floor, count], np.float64)
        nms[f"fleet{trial}/kept"] = kept
        fleets.append(trial)
    nms["kernels_bench/kept"] = numpy_ops.nms(nms_b, nms_s, 0.45, 0.25, 300)
    b, s, c = nms_heads(16, 8400, 2, seed=0)
    keep = np.full((16, 300), -1, np.int64)
    counts = np.zeros(16, np.int32)
    for i in range(16):
        merged = []
        for cls in range(2):
            idx = np.nonzero(c[i] == cls)[0]
            kept = idx[numpy_ops.nms(b[i][idx], s[i][idx], 0.45, 0.25, 300)]
            merged.extend(kept.tolist())
        merged.sort(key=lambda j: (-float(s[i][j]), j))
        merged = merged[:300]
        keep[i, : len(merged)] = merged
        counts[i] = len(merged)
    nms["config2/keep"], nms["config2/counts"] = keep, counts
    np.savez_compressed(HERE / "nms.npz", **nms)

    # ---- full-size hashes
    hashes = {}
    frames = frames_u8(8, (1080, 1920), seed=0)
    hashes["config1_letterbox_f32"] = sha(torch_ops.letterbox_batch(frames, (640, 640), NormalizeParams()).tensor)
    boxes, idx = crop_boxes(8, 64)
    p3 = NormalizeParams(mean=IMAGENET_MEAN, std=IMAGENET_STD)
    crops = np.concatenate([torch_ops.crop_batch(frames[f], boxes[idx == f], (256, 128), p3) for f in range(8)])
    hashes["config3_crop_f16"] = sha(crops.astype(np.float16))
    hashes["note"] = ("inputs: tests/_data.py frames_u8(8, (1080,1920), seed=0); crop_boxes(8, 64) (seed 1); "
                      "reference outputs from TorchImageOps on CPU")
    (HERE / "hashes.json").write_text(json.dumps(hashes, indent=1))

    # ---- detector decode (topology/elements/detections.py:423-515), one frame per case
    from shipinfer.topology.elements.detections import DecodeParams, decode_detections

    dec = {}
    rng = np.random.default_rng(11)
    geoms = [((1080, 1920), float(np.float32(1 / 3)), (0.0, 140.0)), ((720, 1280), 0.5, (0.0, 140.0)),
             ((2160, 3840), float(np.float32(1 / 3)), (0.0, 280.0)), ((480, 640), 1.0, (0.0, 80.0))]
    cases = []
    for k in range(24):
        R = 8400 if k == 1 else [300, 2000, 1, 17, 1000][k % 5]
        rows = np.empty((R, 6), np.float32)
        rows[:, :4] = rng.uniform(-20.0, 660.0, (R, 4)).astype(np.float32)
        rows[:, 4] = rng.uniform(0.0, 1.0, R).astype(np.float32)
        if k % 3 == 0:
            rows[:, 4] = np.round(rows[:, 4] * 8) / 8  # ties everywhere
        rows[:, 5] = rng.uniform(-1.0, 80.0, R).astype(np.float32)
        if k % 4 == 1:  # non-finite values and signed zeros
            rows[rng.integers(0, R, 3), rng.integers(0, 4, 3)] = np.nan
            rows[rng.integers(0, R, 2), 4] = np.nan
            rows[rng.integers(0, R, 2), 5] = np.inf
            rows[rng.integers(0, R, 2), 0] = -0.0
            rows[rng.integers(0, R, 2), 4] = -0.0
        hw, scale, pad = geoms[k % 4]
        count = [None, R // 2, 0, R + 5, None, 3][k % 6]
        thr = [0.25, 0.5, 0.0, 0.9][k % 4]
        cap = [100, 300, 5, 0, 4096, 1][k % 6]
        frame = None if k % 7 == 3 else hw
        sc = 0.0 if k == 13 else scale  # a zero scale leaves coordinates unscaled
        cases.append((rows, count, sc, pad, frame, thr, cap))
    for i, (rows, count, sc, pad, frame, thr, cap) in enumerate(cases):
        d = decode_detections(rows, params=DecodeParams(score_threshold=thr, max_detections=cap), scale=sc,
                              pad=pad, frame_hw=frame, count=count)
        dec[f"rows_{i}"] = rows
        dec[f"args_{i}"] = np.array([-1 if count is None else count, sc, pad[0], pad[1],
                                     -1 if frame is None else frame[0], -1 if frame is None else frame[1], thr, cap],
                                    np.float64)
        dec[f"boxes_{i}"] = np.asarray(d.boxes, np.float32).reshape(-1, 4)
        dec[f"scores_{i}"] = np.asarray(d.scores, np.float32)
        dec[f"classes_{i}"] = np.asarray(d.class_ids, np.int32)
        dec[f"discarded_{i}"] = np.array([d.discarded], np.int64)
    np.savez_compressed(HERE / "decode.npz", **dec)

    # ---- config 4's camera partition
    fps, _sizes = camera_mix()
    load = {f"cam{c:02d}": f for c, f in fps.items()}
    shards = {}
    for g in (1, 2, 4, 8):
        plan = plan_shards(load, shards=g, gpus=list(range(g)))
        shards[str(g)] = [list(sh.cameras) for sh in plan.shards]
    (HERE / "shards.json").write_text(json.dumps(shards, indent=1))
    print("golden fixtures written to", HERE)


if __name__ == "__main__":
    main()
