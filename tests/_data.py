"""Seeded synthetic inputs with the benchmark configs' shapes and value distributions.

No public dataset is involved on this path; these generators stand in for camera frames and
detector heads (uniform random pixels, YOLO-640-shaped candidate sets).
"""

from __future__ import annotations

import numpy as np

FRAME_1080 = (1080, 1920)
FRAME_720 = (720, 1280)
IMAGENET_MEAN = tuple(255.0 * m for m in (0.485, 0.456, 0.406))
IMAGENET_STD = tuple(255.0 * s for s in (0.229, 0.224, 0.225))


def frames_u8(count: int, hw: tuple[int, int] = FRAME_1080, seed: int = 0) -> list[np.ndarray]:
    """``count`` uint8 BGR frames, pixels uniform in [0, 255]."""
    rng = np.random.default_rng(seed)
    return [rng.integers(0, 256, (*hw, 3), dtype=np.uint8) for _ in range(count)]


def nms_heads(batch: int = 16, n: int = 8400, classes: int = 2, seed: int = 0, size: float = 640.0):
    """``(boxes [B,n,4] f32 xyxy, scores [B,n] f32, classes [B,n] int32)`` for config 2:
    centres uniform in [0, size], width/height log-uniform in [8, 320], clipped to the image;
    scores uniform in (0, 1); classes uniform."""
    rng = np.random.default_rng(seed)
    boxes = np.empty((batch, n, 4), np.float32)
    scores = np.empty((batch, n), np.float32)
    cls = np.empty((batch, n), np.int32)
    for b in range(batch):
        c = rng.uniform(0.0, size, (n, 2))
        wh = np.exp(rng.uniform(np.log(8.0), np.log(320.0), (n, 2)))
        xy1 = np.clip(c - wh / 2, 0.0, size)
        xy2 = np.clip(c + wh / 2, 0.0, size)
        boxes[b] = np.concatenate([xy1, xy2], axis=1).astype(np.float32)
        scores[b] = rng.uniform(0.0, 1.0, n).astype(np.float32)
        cls[b] = rng.integers(0, classes, n).astype(np.int32)
    return boxes, scores, cls


def crop_boxes(frames: int = 8, per_frame: int = 64, hw: tuple[int, int] = FRAME_1080, seed: int = 1):
    """Config 3's boxes: ``(boxes [frames*per_frame, 4] f32, frame_index [..] int32)``; width
    and height log-uniform in [16, 400], each box fully inside its frame."""
    rng = np.random.default_rng(seed)
    H, W = hw
    out = []
    idx = []
    for f in range(frames):
        w = np.exp(rng.uniform(np.log(16.0), np.log(400.0), per_frame))
        h = np.exp(rng.uniform(np.log(16.0), np.log(400.0), per_frame))
        x = rng.uniform(0.0, W - w)
        y = rng.uniform(0.0, H - h)
        out.append(np.stack([x, y, x + w, y + h], axis=1))
        idx.append(np.full(per_frame, f, np.int32))
    return np.concatenate(out).astype(np.float32), np.concatenate(idx)


def nv12_frames(count: int, hw: tuple[int, int] = (2160, 3840), seed: int = 0, pitch: int | None = None,
                coded_h: int | None = None) -> list[tuple[np.ndarray, int, int, int, int]]:
    """NV12 surfaces ``(buffer, h, w, pitch, uv_offset)``: luma uniform in [16, 235], chroma
    in [16, 240]; ``pitch`` / ``coded_h`` pad the surface as a decoder would."""
    rng = np.random.default_rng(seed)
    H, W = hw
    pitch = pitch or W
    coded_h = coded_h or H
    uv_offset = pitch * coded_h
    out = []
    for _ in range(count):
        buf = np.zeros(uv_offset + pitch * ((H + 1) // 2), np.uint8)
        luma = buf[: pitch * H].reshape(H, pitch)
        luma[:, :W] = rng.integers(16, 236, (H, W), dtype=np.uint8)
        chroma = buf[uv_offset:].reshape((H + 1) // 2, pitch)
        cw = ((W + 1) // 2) * 2
        chroma[:, :cw] = rng.integers(16, 241, ((H + 1) // 2, cw), dtype=np.uint8)
        out.append((buf, H, W, pitch, uv_offset))
    return out


def camera_mix(seed: int = 0):
    """Config 4's 50 cameras: ids 0..34 send 1080p, 35..49 send 720p; camera 0 at 8x fps."""
    fps = {cam: 20.0 for cam in range(50)}
    fps[0] = 160.0
    sizes = {cam: (FRAME_1080 if cam < 35 else FRAME_720) for cam in range(50)}
    return fps, sizes


def kernels_bench_inputs(seed: int = 0):
    """The reference kernel benchmark's inputs (benchmarks/kernels.py:298-320 ``_inputs``):
    ``(frame 1080p uint8, 15 boxes f32, 25 000 NMS boxes f32, 25 000 scores f32)``."""
    rng = np.random.default_rng(seed)
    frame = rng.integers(0, 255, (1080, 1920, 3), dtype=np.uint8)
    boxes = np.stack([rng.uniform(0, 1920 - 64, 15), rng.uniform(0, 1080 - 64, 15),
                      rng.uniform(64, 1920, 15), rng.uniform(64, 1080, 15)], axis=1).astype(np.float32)
    nms_boxes = np.stack([rng.uniform(0, 1000, 25000), rng.uniform(0, 1000, 25000),
                          rng.uniform(1000, 2000, 25000), rng.uniform(1000, 2000, 25000)], axis=1).astype(np.float32)
    nms_scores = rng.uniform(0, 1, 25000).astype(np.float32)
    return frame, boxes, nms_boxes, nms_scores


def yuv_constants(matrix: int) -> tuple[float, float, float, float, float]:
    """(ys, cbu, cgu, cgv, crv) of the limited-range YCbCr -> R'G'B' matrix built from the
    standard's Kr and Kb (ITU-R BT.601: 0.299, 0.114; BT.709: 0.2126, 0.0722) in float64, with
    Kg = 1 - Kr - Kb, chroma scale 255/224: cbu = 2(1-Kb)·c, cgu = 2Kb(1-Kb)/Kg·c,
    cgv = 2Kr(1-Kr)/Kg·c, crv = 2(1-Kr)·c, each rounded to six decimals as the reference's
    nv12_to_bgr writes its BT.601 constants (csrc/shipinfer/runtime/ops.cu:159-166). The luma
    scale 255/219 = 1.16438356... is range-only (the same in both standards); the reference
    writes it 1.164383, cut rather than rounded at the sixth decimal, and that literal is kept."""
    kr, kb = (0.2126, 0.0722) if matrix == 709 else (0.299, 0.114)
    kg = 1.0 - kr - kb
    c = 255.0 / 224.0
    ys = np.floor(255.0 / 219.0 * 1e6) / 1e6
    return (float(ys), round(2 * (1 - kb) * c, 6), round(2 * kb * (1 - kb) / kg * c, 6),
            round(2 * kr * (1 - kr) / kg * c, 6), round(2 * (1 - kr) * c, 6))
