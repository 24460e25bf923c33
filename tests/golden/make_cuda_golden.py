"""Record SHA-256s of the reference's CUDA formulation: its own ``TorchImageOps(device_index=0)``.

Run on a B200 with the reference importable. Its offline install under ``baseline/_ref``
(``pip install --no-index --no-deps --target baseline/_ref <reference>``) is the default;
``--reference-site`` points elsewhere (a ``src/`` tree works too):

    python tests/golden/make_cuda_golden.py [--reference-site baseline/_ref] [--out FILE]

For the seeded inputs of ``tests/_data.py`` and the reference's own crop case table (kept in
``tests/golden/crop.npz`` by ``make_golden.py``) it writes ``cuda_hashes.json``: the SHA-256 of
each output array's bytes, together with the GPU, torch and CUDA versions it ran on. The
kernels' GPU test (``tests/test_gpu_reference_cuda.py``) recomputes the same outputs with the
sm_100a kernels and compares the hashes, so the kernels are pinned to the reference's CUDA
path itself and not only to a restatement of it.
"""

from __future__ import annotations

import argparse
import hashlib
import json
import sys
from pathlib import Path

import numpy as np

HERE = Path(__file__).resolve().parent
ROOT = HERE.parents[1]
sys.path.insert(0, str(HERE.parent))

from _data import IMAGENET_MEAN, IMAGENET_STD, crop_boxes, frames_u8, kernels_bench_inputs  # noqa: E402

# (name, frame shapes, seed, dst, normalisation, pad): letterbox cases beyond config 1. The
# non-dyadic ones are where torch's CPU and CUDA blends part, so they pin the CUDA order.
LETTERBOX_CASES = [
    ("config1", [(1080, 1920)] * 8, 0, (640, 640), "unit", 114),
    ("720p-2to1", [(720, 1280)] * 4, 1, (640, 640), "unit", 114),
    ("non-dyadic-imagenet", [(1000, 1500), (777, 1333), (1080, 1920)], 2, (640, 640), "imagenet", 114),
    ("upscale-unit-pad0", [(90, 160), (33, 77)], 3, (416, 416), "unit", 0),
    ("portrait-imagenet-bgr", [(1280, 720)], 4, (384, 640), "imagenet-bgr", 114),
]


def sha(a: np.ndarray) -> str:
    return hashlib.sha256(np.ascontiguousarray(a).tobytes()).hexdigest()


def normalisations(NormalizeParams):
    return {
        "unit": NormalizeParams(),
        "imagenet": NormalizeParams(mean=IMAGENET_MEAN, std=IMAGENET_STD),
        "imagenet-bgr": NormalizeParams(mean=IMAGENET_MEAN, std=IMAGENET_STD, swap_rb=False),
    }


def letterbox_inputs(shapes, seed):
    rng = np.random.default_rng(seed)
    return [rng.integers(0, 256, (*hw, 3), dtype=np.uint8) for hw in shapes]


def main() -> None:
    ap = argparse.ArgumentParser()
    ap.add_argument("--reference-site", default=str(ROOT / "baseline" / "_ref"))
    ap.add_argument("--out", default=str(HERE / "cuda_hashes.json"))
    args = ap.parse_args()
    sys.path.insert(0, args.reference_site)
    import torch

    from shipinfer.runtime.ops import NormalizeParams, TorchImageOps

    assert torch.cuda.is_available(), "the CUDA formulation needs a GPU"
    ops = TorchImageOps(device_index=0)
    norms = normalisations(NormalizeParams)
    out = {"provenance": {"gpu": torch.cuda.get_device_name(0), "torch": torch.__version__,
                          "cuda": torch.version.cuda,
                          "what": "SHA-256 of TorchImageOps(device_index=0) outputs (the reference's CUDA path)"}}

    for name, shapes, seed, dst, norm, pad in LETTERBOX_CASES:
        frames = frames_u8(8, shapes[0], seed=0) if name == "config1" else letterbox_inputs(shapes, seed)
        r = ops.letterbox_batch(frames, dst, norms[norm], pad_value=pad)
        out[f"letterbox/{name}/f32"] = sha(np.asarray(r.tensor, np.float32))
        out[f"letterbox/{name}/f16"] = sha(np.asarray(r.tensor, np.float32).astype(np.float16))

    frames = frames_u8(8, (1080, 1920), seed=0)
    boxes, idx = crop_boxes(8, 64)
    p3 = norms["imagenet"]
    crops = np.concatenate([ops.crop_batch(frames[f], boxes[idx == f], (256, 128), p3) for f in range(8)])
    out["crop/config3/f32"] = sha(crops.astype(np.float32))
    out["crop/config3/f16"] = sha(crops.astype(np.float16))

    table = np.load(HERE / "crop.npz")
    params = {pid: NormalizeParams(mean=tuple(row[:3]), std=tuple(row[3:6]), swap_rb=bool(row[6]))
              for pid, row in zip(table["param_ids"], table["params"])}
    cases = sorted({k.split("/")[0] for k in table.files if k.endswith("/image")})
    for cid in cases:
        image, cboxes, cdst = table[f"{cid}/image"], table[f"{cid}/boxes"], tuple(int(v) for v in table[f"{cid}/dst"])
        for pid, p in params.items():
            out[f"crop/case/{cid}/{pid}"] = sha(np.asarray(ops.crop_batch(image, cboxes, cdst, p), np.float32))

    frame, kb, _, _ = kernels_bench_inputs(0)
    out["crop/kernels_bench/f32"] = sha(np.asarray(ops.crop_batch(frame, kb, (256, 128), NormalizeParams()), np.float32))

    Path(args.out).write_text(json.dumps(out, indent=1) + "\n")
    print(f"{len(out) - 1} hashes written to {args.out}")


if __name__ == "__main__":
    main()
