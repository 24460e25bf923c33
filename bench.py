#!/usr/bin/env python
"""Benchmark of the shipk hot path on B200; prints ONE JSON line (rank 0).

Default workload (config 1, the one the headline metric is quoted on): fused letterbox of a
batch of 8 x 1920x1080 uint8 BGR frames to [8, 3, 640, 640] float32 (pad 114, /255, BGR->RGB).
One step = one batch through the hot path. The same run also measures the other configs of
the metric and reports them under ``extras``: ``nms`` (config 2, the metric's "NMS imgs/s"),
``crop`` (config 3), ``nv12`` (config 5), ``stream`` (config 4, cameras sharded over the GPUs
by the reference's plan_shards rule) and ``seam`` (the reference's kernel-benchmark cases and
pageable host frames through the Python seam). ``--config`` makes any workload the headline
(``mask``, ``decode`` and ``nv12crop`` are the rows next to the path); ``--no-extras`` skips
the rest.

* ``value``: whole-job throughput with inputs resident in HBM. The K timed steps are captured
  into CUDA graphs (uploaded before timing); that K-step replay is timed with CUDA events on
  its stream, back to back, until at least ``--min-seconds`` of device time has elapsed
  (barrier + synchronize around the set), and the median window is the measurement; the time
  is the max over ranks of each rank's median. Inputs cycle through a ring of distinct
  batches larger than L2, so every step reads its frames from HBM.
* ``e2e``: the same metric through the host-frame C-ABI call (``shipk_ctx_letterbox_host``,
  the reference's ``letterbox_to_device`` path) from pinned host frames, with the H2D copies
  and a D2H read of the step's result inside the timed region.
* ``roofline``: algorithmic bytes per launch / median launch duration against the measured
  HBM copy bandwidth; ``traffic`` = DRAM bytes per launch from the committed ncu summary of
  the same kernel (steady state: consecutive launches, no cache flush between them).
* ``cpu_baseline``: the CPU oracle (the reference's formulation restated in C, OpenMP over all
  host cores) on a bounded sample, rank 0 at N=1; ``cpu_baseline_reference``: the reference's
  own ``TorchImageOps()`` on the host cores (configs 1 and 3), when its offline install is
  present under ``baseline/_ref``.

``--impl reference`` times the CPU implementation alone, for the driver's reference arm.
Multi-GPU (torchrun): frames are sharded by camera, one replica per GPU, no collectives on
the data path (``scaling: weak``); the barrier and the max over ranks run on a gloo group of
CPU tensors, so NCCL is never initialised.
"""

from __future__ import annotations

import argparse
import ctypes
import datetime
import json
import math
import os
import statistics
import sys
import threading
import time
from pathlib import Path

import numpy as np

ROOT = Path(__file__).resolve().parent
sys.path.insert(0, str(ROOT))
sys.path.insert(0, str(ROOT / "tests"))

L2_BYTES = 126 * 1024 * 1024
FALLBACK_HBM_GBS = 6650.0


def parse_args() -> argparse.Namespace:
    p = argparse.ArgumentParser(description=__doc__.split("\n")[0])
    p.add_argument("--gpus", type=int, default=1)
    p.add_argument("--steps", type=int, default=1000)
    p.add_argument("--warmup", type=int, default=20)
    p.add_argument("--impl", choices=["shipk", "reference"], default="shipk")
    p.add_argument("--config", choices=["letterbox", "nms", "crop", "nv12", "stream", "mask", "decode", "nv12crop"],
                   default="letterbox")
    p.add_argument("--no-cpu-baseline", action="store_true")
    p.add_argument("--no-e2e", action="store_true")
    p.add_argument("--no-extras", action="store_true", help="measure the headline workload only")
    p.add_argument("--cpu-seconds", type=float, default=10.0, help="CPU sample of the headline workload")
    p.add_argument("--extra-cpu-seconds", type=float, default=5.0, help="CPU sample of each extra workload")
    p.add_argument("--min-seconds", type=float, default=0.5,
                   help="repeat the K-step replay until this much device time has elapsed")
    return p.parse_args()


# ---------------------------------------------------------------------------------------------
# peaks, clocks, profiles


def hbm_peak() -> tuple[float, str]:
    path = ROOT / "MEASURED_PEAKS.json"
    try:
        return float(json.loads(path.read_text())["hbm_gbs"]), "measured"
    except Exception:
        return FALLBACK_HBM_GBS, "fallback"


def ncu_traffic(name: str) -> float | None:
    """DRAM bytes per launch from the committed ncu summary (profiles/<name>.txt), if any."""
    path = ROOT / "profiles" / f"{name}.txt"
    if not path.exists():
        return None
    for line in path.read_text().splitlines():
        if line.startswith("traffic_bytes_per_launch:"):
            try:
                return float(line.split(":", 1)[1].split()[0])
            except ValueError:
                return None
    return None


class ClockSampler:
    """Polls NVML for the SM clock and clock-event reasons while the benchmark runs."""

    REASONS = {
        0x0000000000000004: "sw_power_cap",
        0x0000000000000008: "hw_slowdown",
        0x0000000000000020: "sw_thermal_slowdown",
        0x0000000000000040: "hw_thermal_slowdown",
        0x0000000000000080: "hw_power_brake_slowdown",
    }

    def __init__(self, device: int) -> None:
        self.samples: list[tuple[float, int, int]] = []
        self.max_mhz = None
        self._stop = threading.Event()
        self._thread = None
        try:
            import pynvml

            pynvml.nvmlInit()
            visible = os.environ.get("CUDA_VISIBLE_DEVICES")
            index = int(visible.split(",")[device]) if visible else device
            self._h = pynvml.nvmlDeviceGetHandleByIndex(index)
            self._nvml = pynvml
            self.max_mhz = pynvml.nvmlDeviceGetMaxClockInfo(self._h, pynvml.NVML_CLOCK_SM)
        except Exception:
            self._nvml = None

    def start(self) -> None:
        if self._nvml is None:
            return
        self._thread = threading.Thread(target=self._run, daemon=True)
        self._thread.start()

    def _run(self) -> None:
        nv = self._nvml
        get_reasons = getattr(nv, "nvmlDeviceGetCurrentClocksEventReasons", None) or getattr(
            nv, "nvmlDeviceGetCurrentClocksThrottleReasons"
        )
        while not self._stop.is_set():
            try:
                sm = nv.nvmlDeviceGetClockInfo(self._h, nv.NVML_CLOCK_SM)
                reasons = get_reasons(self._h)
                self.samples.append((time.perf_counter(), sm, reasons))
            except Exception:
                return
            time.sleep(0.002)

    def stop(self) -> None:
        self._stop.set()
        if self._thread:
            self._thread.join(timeout=2)

    def summary(self, t0: float, t1: float) -> dict:
        if self._nvml is None:
            return {"sm_mhz": None, "sm_max_mhz": None, "reasons": [], "note": "NVML unavailable"}
        window = [s for s in self.samples if t0 <= s[0] <= t1]
        note = f"{len(window)} NVML samples inside the timed window"
        if not window:  # the window was shorter than the poll period: nearest samples around it
            window = sorted(self.samples, key=lambda s: min(abs(s[0] - t0), abs(s[0] - t1)))[:3]
            note = "timed window shorter than the NVML poll period; nearest samples"
        reasons = sorted({name for s in window for bit, name in self.REASONS.items() if s[2] & bit})
        return {
            "sm_mhz": statistics.median(s[1] for s in window) if window else None,
            "sm_max_mhz": self.max_mhz,
            "reasons": reasons,
            "samples": len(window),
            "note": note,
        }


# ---------------------------------------------------------------------------------------------
# distributed plumbing (barrier and max-over-ranks only; the data path has no collective)


class Dist:
    """Barrier, max over ranks and a gather of one number per rank, on a gloo process group of
    CPU tensors. The data path has no collective, and NCCL is never initialised."""

    def __init__(self) -> None:
        self.world = int(os.environ.get("WORLD_SIZE", "1"))
        self.rank = int(os.environ.get("RANK", "0"))
        self.local = int(os.environ.get("LOCAL_RANK", "0"))
        self.pg = None

    def init(self) -> None:
        if self.world > 1:
            import torch.distributed as dist

            os.environ.setdefault("MASTER_ADDR", "127.0.0.1")
            dist.init_process_group("gloo", timeout=datetime.timedelta(seconds=120))
            self.pg = dist

    def barrier(self) -> None:
        if self.pg:
            self.pg.barrier()

    def max(self, value: float) -> float:
        if not self.pg:
            return value
        import torch

        t = torch.tensor([value], dtype=torch.float64)
        self.pg.all_reduce(t, op=self.pg.ReduceOp.MAX)
        return float(t.item())

    def gather(self, value: float) -> list[float]:
        if not self.pg:
            return [value]
        import torch

        parts = [torch.zeros(1, dtype=torch.float64) for _ in range(self.world)]
        self.pg.all_gather(parts, torch.tensor([value], dtype=torch.float64))
        return [float(t.item()) for t in parts]

    def close(self) -> None:
        if self.pg:
            self.pg.destroy_process_group()


# ---------------------------------------------------------------------------------------------
# graph capture of K steps


def cudart():
    return ctypes.CDLL("libcudart.so.12")


def capture_steps(torch, launch, steps: int, ring: int, chunk: int = 512):
    """CUDA graphs that together run exactly `steps` launches: a chunk graph replayed
    floor(steps/chunk) times and a tail graph. `launch(i, stream)` issues step i."""
    chunk = max(ring, (min(chunk, steps) // ring) * ring) if steps >= ring else steps
    graphs = []
    rt = cudart()
    stream = torch.cuda.Stream()

    def build(count):
        g = torch.cuda.CUDAGraph()
        with torch.cuda.graph(g, stream=stream, capture_error_mode="relaxed"):
            handle = torch.cuda.current_stream().cuda_stream
            for i in range(count):
                launch(i, handle)
        rc = rt.cudaGraphUpload(ctypes.c_void_p(g.raw_cuda_graph_exec()), ctypes.c_void_p(stream.cuda_stream))
        if rc != 0:
            raise RuntimeError(f"cudaGraphUpload failed ({rc})")
        return g

    full, tail = divmod(steps, chunk) if chunk else (0, 0)
    main = build(chunk) if full else None
    tail_g = build(tail) if tail else None
    torch.cuda.synchronize()

    def replay():
        for _ in range(full):
            main.replay()
        if tail_g is not None:
            tail_g.replay()

    return replay, stream, [g for g in (main, tail_g) if g is not None]


# ---------------------------------------------------------------------------------------------
# workloads


class Letterbox:
    """Config 1: 8 x 1080p BGR -> [8, 3, 640, 640] fp32."""

    name = "letterbox"
    metric = "preprocess img/s (1080p->640x640 fused letterbox, config 1)"
    unit = "img/s"
    dtype = "f32"
    profile = "letterbox_u8_config1"
    workload = "fused letterbox, 8 x 1920x1080 uint8 BGR -> [8,3,640,640] fp32 (config 1)"
    batch = 8
    hw = (1080, 1920)
    dst = (640, 640)

    def __init__(self, torch, lib, native, device: int):
        from _data import frames_u8

        self.torch, self.lib, self.native = torch, lib, native
        self.ring = self.input_ring()
        host = frames_u8(self.batch, self.hw, seed=0)
        base = torch.from_numpy(np.stack(host)).to(f"cuda:{device}")
        # distinct bytes in every ring slot: each slot is the seed batch rolled by its index
        self.inputs = torch.stack([torch.roll(base, shifts=k * 7919, dims=2) for k in range(self.ring)])
        # outputs also cycle through more than L2 (4 x 39 MB), so no step's writes are absorbed by
        # lines a previous step left in L2
        self.nout = 4
        self.outputs = torch.empty((self.nout, self.batch, 3, *self.dst), dtype=torch.float32, device=f"cuda:{device}")
        self.host_frames = host
        self.frames = []
        for k in range(self.ring):
            arr = (native.FrameU8 * self.batch)()
            for i in range(self.batch):
                f = self.inputs[k, i]
                arr[i] = native.FrameU8(f.data_ptr(), self.hw[0], self.hw[1], f.stride(0))
            self.frames.append(arr)
        self.mean = native.floats3([0, 0, 0])
        self.std = native.floats3([255, 255, 255])
        self.out_nbytes = self.outputs[0].numel() * 4
        self.device = device

    @classmethod
    def touched_bytes(cls) -> int:
        """Source bytes one step reads: the contributing rows, 360 of 1080 at 1080p -> 640."""
        return cls.batch * 360 * cls.hw[1] * 3

    @classmethod
    def input_ring(cls) -> int:
        """Distinct input batches cycled per step: enough that the bytes the kernel reads over
        the ring are 1.5 x L2 (so no step finds its rows still in L2), an even count."""
        ring = max(2, -(-int(1.5 * L2_BYTES) // cls.touched_bytes()))
        return ring + ring % 2

    @classmethod
    def static_config(cls) -> dict:
        """The config, computed without a GPU (the reference arm prints the same one)."""
        ring, nout = cls.input_ring(), 4
        out_nbytes = cls.batch * 3 * cls.dst[0] * cls.dst[1] * 4
        return {
            "workload": cls.workload,
            "batch": cls.batch,
            "src": "1920x1080x3 uint8 BGR, uniform random",
            "dst": "640x640 NCHW fp32, pad 114, /255, BGR->RGB",
            "l2": f"inputs larger than L2: ring of {ring} distinct batches "
                  f"({ring * cls.batch * cls.hw[0] * cls.hw[1] * 3 / 1e6:.0f} MB of frames, of which the kernel "
                  f"reads {ring * cls.touched_bytes() / 1e6:.0f} MB) cycled per step, "
                  f"outputs a ring of {nout} ({nout * out_nbytes / 1e6:.0f} MB)",
            "parallelism": "camera-sharded replicas, one per GPU",
        }

    def config(self) -> dict:
        return self.static_config()

    def algorithmic_bytes(self) -> int:
        # per image: output 3*640*640*4 + the 360 contributing source rows (scale 3, weight 1)
        return self.batch * (3 * 640 * 640 * 4 + 360 * 1920 * 3)

    def launch(self, i: int, stream: int) -> None:
        rc = self.lib.shipk_letterbox_u8(
            self.frames[i % self.ring], self.batch, self.outputs[i % self.nout].data_ptr(), self.native.DTYPE_F32,
            self.out_nbytes, self.dst[0], self.dst[1], self.mean, self.std, 1, 114.0, None, stream,
        )
        if rc:
            self.native.check(rc)

    # e2e: pinned host frames through the host-frame entry point, D2H of the result rows
    def e2e_setup(self):
        torch = self.torch
        self.pinned = [torch.from_numpy(np.stack(self.host_frames)).pin_memory() for _ in range(2)]
        self.pinned[1].copy_(torch.roll(self.pinned[1], shifts=7919, dims=2))
        ctx = ctypes.c_void_p()
        self.native.check(self.lib.shipk_ctx_create(self.device, ctypes.byref(ctx)))
        self.ctx = ctx
        self.host_arrays = []
        for k in range(2):
            arr = (self.native.FrameU8 * self.batch)()
            for i in range(self.batch):
                f = self.pinned[k][i]
                arr[i] = self.native.FrameU8(f.data_ptr(), self.hw[0], self.hw[1], f.stride(0))
            self.host_arrays.append(arr)
        self.readback = torch.empty((self.batch, 3, self.dst[1]), dtype=torch.float32).pin_memory()
        # bytes each step moves: the contributing rows, the row maps, and the result rows
        self.h2d = self.batch * (360 * 1920 * 3 + 1080 * 4)
        self.d2h = self.readback.numel() * 4

    def e2e_step(self, i: int, stream) -> None:
        rc = self.lib.shipk_ctx_letterbox_host(
            self.ctx, self.host_arrays[i % 2], self.batch, self.outputs[i % 2].data_ptr(), self.native.DTYPE_F32,
            self.out_nbytes, self.dst[0], self.dst[1], self.mean, self.std, 1, 114.0, None, stream.cuda_stream,
        )
        if rc:
            self.native.check(rc)
        # the first letterboxed row of every image comes home: the step's result is on the host
        self.readback.copy_(self.outputs[i % 2][:, :, 140, :], non_blocking=True)

    def e2e_close(self):
        self.lib.shipk_ctx_destroy(self.ctx)

    def cpu_sample(self):
        from oracle import oracle

        frames = self.host_frames
        return (lambda: oracle.letterbox(frames, self.dst)), self.batch, "one batch of 8 x 1080p frames per call"


class Nms:
    """Config 2: 16 images x 8400 candidates, 2 classes, class-aware, score 0.25, IoU 0.45."""

    name = "nms"
    workload = "class-aware NMS, 16 x 8400 boxes, 2 classes, score 0.25, IoU 0.45, max_det 300 (config 2)"
    metric = "NMS imgs/s (16 x 8400 candidates, class-aware, config 2)"
    unit = "img/s"
    dtype = "f32"
    profile = "nms_config2"
    batch = 16
    bound = "latency"
    bound_note = ("3.3 MB of input fits L2: the kernel is bound by the per-segment greedy walk's latency, so "
                  "the HBM fraction is not its limit")

    def __init__(self, torch, lib, native, device: int):
        from _data import nms_heads

        self.torch, self.lib, self.native = torch, lib, native
        b, s, c = nms_heads(16, 8400, 2, seed=0)
        self.host = (b, s, c)
        dev = f"cuda:{device}"
        self.ring = 2
        self.boxes = [torch.from_numpy(np.roll(b, k, axis=1)).to(dev) for k in range(self.ring)]
        self.scores = [torch.from_numpy(np.roll(s, k, axis=1)).to(dev) for k in range(self.ring)]
        self.classes = [torch.from_numpy(np.roll(c, k, axis=1)).to(dev) for k in range(self.ring)]
        self.keep = torch.empty((16, 300), dtype=torch.int64, device=dev)
        self.counts = torch.empty((16,), dtype=torch.int32, device=dev)
        ws = lib.shipk_nms_workspace_bytes(16, 8400, 2, 1, 300)
        self.ws = torch.empty((ws,), dtype=torch.uint8, device=dev)
        self.device = device

    def config(self) -> dict:
        return {"workload": self.workload,
                "batch": 16, "l2": "inputs (3.2 MB) fit in L2; NMS is latency-bound, not HBM-bound",
                "parallelism": "camera-sharded replicas, one per GPU"}

    def launch_shape(self) -> dict:
        ctas, cluster = ctypes.c_int(), ctypes.c_int()
        self.native.check(self.lib.shipk_nms_launch_shape(16, 8400, 2, 1, 300, ctypes.byref(ctas), ctypes.byref(cluster)))
        return {"ctas": ctas.value, "threads_per_cta": 1024, "cluster": cluster.value,
                "note": "an image x class segment per CTA, joined by helper CTAs in its thread-block cluster"}

    def algorithmic_bytes(self) -> int:
        return 16 * 8400 * (16 + 4 + 4) + 16 * 300 * 8 + 16 * 4

    def launch(self, i: int, stream: int) -> None:
        k = i % self.ring
        rc = self.lib.shipk_nms(self.boxes[k].data_ptr(), self.scores[k].data_ptr(), self.classes[k].data_ptr(),
                                16, 8400, 2, 1, 0.45, 0.25, 300, self.keep.data_ptr(), self.counts.data_ptr(),
                                self.ws.data_ptr(), self.ws.numel(), stream)
        if rc:
            self.native.check(rc)

    def cpu_sample(self):
        from oracle import oracle

        b, s, c = self.host
        return (lambda: oracle.nms_batched(b, s, c, 0.45, 0.25, 300, num_classes=2)), 16, "16 images x 8400 per call"


class Crop:
    """Config 3: 8 x 1080p frames x 64 boxes -> [512, 3, 256, 128] fp16, ImageNet normalisation."""

    name = "crop"
    workload = "batched crop-resize, 8 x 1080p x 64 boxes -> [512,3,256,128] fp16 (config 3)"
    metric = "crop-resize boxes/s (8 x 64 boxes -> 256x128 fp16, config 3)"
    unit = "boxes/s"
    dtype = "f32"
    profile = "crop_config3"
    batch = 512

    def __init__(self, torch, lib, native, device: int):
        from _data import IMAGENET_MEAN, IMAGENET_STD, crop_boxes, frames_u8

        self.torch, self.lib, self.native = torch, lib, native
        dev = f"cuda:{device}"
        self.host_frames = frames_u8(8, seed=0)
        boxes, idx = crop_boxes(8, 64)
        w = (np.clip(boxes[:, 2], 0, 1919).astype(np.int64) - np.clip(boxes[:, 0], 0, 1919).astype(np.int64))
        h = (np.clip(boxes[:, 3], 0, 1079).astype(np.int64) - np.clip(boxes[:, 1], 0, 1079).astype(np.int64))
        self.src_bytes = int((w * h * 3).sum())
        # enough frame batches that the box pixels read over the ring are 1.5 x L2
        self.ring = max(2, -(-int(1.5 * L2_BYTES) // self.src_bytes))
        base = torch.from_numpy(np.stack(self.host_frames)).to(dev)
        self.inputs = torch.stack([torch.roll(base, shifts=k * 7919, dims=2) for k in range(self.ring)])
        self.host_boxes, self.host_idx = boxes, idx
        self.boxes = torch.from_numpy(boxes).to(dev)
        self.idx = torch.from_numpy(idx).to(dev)
        self.outputs = torch.empty((2, 512, 3, 256, 128), dtype=torch.float16, device=dev)
        self.frames = []
        for k in range(self.ring):
            arr = (native.FrameU8 * 8)()
            for i in range(8):
                f = self.inputs[k, i]
                arr[i] = native.FrameU8(f.data_ptr(), 1080, 1920, f.stride(0))
            self.frames.append(arr)
        self.mean = native.floats3(IMAGENET_MEAN)
        self.std = native.floats3(IMAGENET_STD)
        self.mean_t, self.std_t = IMAGENET_MEAN, IMAGENET_STD

    def config(self) -> dict:
        return {"workload": self.workload,
                "batch": 512, "l2": f"inputs larger than L2: ring of {self.ring} frame batches (the boxes' "
                                    f"{self.ring * self.src_bytes / 1e6:.0f} MB of pixels), outputs a ring of 2",
                "parallelism": "camera-sharded replicas, one per GPU"}

    def algorithmic_bytes(self) -> int:
        return 512 * 3 * 256 * 128 * 2 + self.src_bytes

    def launch(self, i: int, stream: int) -> None:
        rc = self.lib.shipk_crop_u8(self.frames[i % self.ring], 8, self.boxes.data_ptr(), self.idx.data_ptr(), 512,
                                    self.outputs[i % 2].data_ptr(), self.native.DTYPE_F16, self.outputs[0].numel() * 2,
                                    256, 128, self.mean, self.std, 1, stream)
        if rc:
            self.native.check(rc)

    def cpu_sample(self):
        from oracle import oracle

        frames, boxes, idx = self.host_frames, self.host_boxes[:64], self.host_idx[:64]
        return (lambda: oracle.crop(frames, boxes, (256, 128), idx, self.mean_t, self.std_t, True)), 64, \
            "64 boxes of one frame per call"


class Nv12:
    """Config 5: 32 x 3840x2160 NV12 -> [32, 3, 1280, 1280] fp16, BT.709 limited, bilinear."""

    name = "nv12"
    workload = "NV12 BT.709 bilinear letterbox, 32 x 3840x2160 -> [32,3,1280,1280] fp16 (config 5)"
    metric = "4K NV12 letterbox img/s (32 x 2160p -> 1280x1280 fp16, config 5)"
    unit = "img/s"
    dtype = "f32"
    profile = "letterbox_nv12_config5"
    batch = 32

    def __init__(self, torch, lib, native, device: int):
        from _data import nv12_frames

        self.torch, self.lib, self.native = torch, lib, native
        dev = f"cuda:{device}"
        planes = nv12_frames(4, (2160, 3840), seed=0)
        self.host_planes = planes
        bufs = [torch.from_numpy(p[0]).to(dev) for p in planes]
        self.inputs = [bufs[i % 4].roll(i * 31) for i in range(self.batch)]  # 32 distinct surfaces (398 MB)
        self.ring = 1
        self.outputs = torch.empty((2, self.batch, 3, 1280, 1280), dtype=torch.float16, device=dev)
        self.arr = (native.FrameNv12 * self.batch)()
        for i, b in enumerate(self.inputs):
            self.arr[i] = native.FrameNv12(b.data_ptr(), 2160, 3840, 3840, 3840 * 2160)
        self.mean = native.floats3([0, 0, 0])
        self.std = native.floats3([255, 255, 255])

    def config(self) -> dict:
        return {"workload": self.workload,
                "batch": 32, "l2": "inputs larger than L2: 32 distinct 12.4 MB surfaces per step",
                "parallelism": "camera-sharded replicas, one per GPU"}

    def algorithmic_bytes(self) -> int:
        return self.batch * (3 * 1280 * 1280 * 2 + 720 * 3840 + 720 * 3840)

    def launch(self, i: int, stream: int) -> None:
        rc = self.lib.shipk_letterbox_nv12(self.arr, self.batch, self.outputs[i % 2].data_ptr(), self.native.DTYPE_F16,
                                           self.outputs[0].numel() * 2, 1280, 1280, self.mean, self.std, 1, 114.0,
                                           709, 1, None, stream)
        if rc:
            self.native.check(rc)

    def cpu_sample(self):
        from oracle import oracle

        planes = self.host_planes[:1]
        return (lambda: oracle.letterbox_nv12(planes, (1280, 1280), matrix=709, sampling=1)), 1, "one 4K frame per call"


class Nv12Crop:
    """NV12 crops (the C++ data plane's embedder input): 8 x 1080p NVDEC surfaces (pitch 2048,
    1088 coded rows) x 64 boxes -> [512, 3, 256, 128] fp16, BT.601, value / 255."""

    name = "nv12crop"
    workload = "NV12 crop-resize, 8 x 1080p NV12 surfaces x 64 boxes -> [512,3,256,128] fp16, BT.601, /255"
    metric = "NV12 crop-resize boxes/s (8 x 1080p NV12 x 64 boxes -> 256x128 fp16)"
    unit = "boxes/s"
    dtype = "f32"
    profile = "crop_nv12_embedder"
    batch = 512

    def __init__(self, torch, lib, native, device: int):
        from _data import crop_boxes, nv12_frames

        self.torch, self.lib, self.native = torch, lib, native
        dev = f"cuda:{device}"
        self.host_planes = nv12_frames(8, (1080, 1920), seed=0, pitch=2048, coded_h=1088)
        boxes, idx = crop_boxes(8, 64)
        # luma and chroma bytes of each clipped box
        x1 = np.clip(boxes[:, 0], 0, 1919).astype(np.int64)
        x2 = np.clip(boxes[:, 2], 0, 1919).astype(np.int64)
        y1 = np.clip(boxes[:, 1], 0, 1079).astype(np.int64)
        y2 = np.clip(boxes[:, 3], 0, 1079).astype(np.int64)
        w, h = np.maximum(x2 - x1, 0), np.maximum(y2 - y1, 0)
        self.src_bytes = int((w * h + w * ((h + 1) // 2)).sum())
        # enough surface batches that the box bytes read over the ring are 1.5 x L2
        self.ring = max(2, -(-int(1.5 * L2_BYTES) // self.src_bytes))
        base = [torch.from_numpy(p[0]).to(dev) for p in self.host_planes]
        self.inputs = [[b.roll(k * 7919) for b in base] for k in range(self.ring)]
        self.host_boxes, self.host_idx = boxes, idx
        self.boxes = torch.from_numpy(boxes).to(dev)
        self.idx = torch.from_numpy(idx).to(dev)
        self.outputs = torch.empty((2, 512, 3, 256, 128), dtype=torch.float16, device=dev)
        self.frames = []
        for k in range(self.ring):
            arr = (native.FrameNv12 * 8)()
            for i, (_, h, w, pitch, uv) in enumerate(self.host_planes):
                arr[i] = native.FrameNv12(self.inputs[k][i].data_ptr(), h, w, pitch, uv)
            self.frames.append(arr)

    def config(self) -> dict:
        return {"workload": self.workload,
                "batch": 512, "l2": f"inputs larger than L2: ring of {self.ring} surface batches (the boxes' "
                                    f"{self.ring * self.src_bytes / 1e6:.0f} MB of luma and chroma), two outputs",
                "parallelism": "camera-sharded replicas, one per GPU"}

    def algorithmic_bytes(self) -> int:
        return 512 * 3 * 256 * 128 * 2 + self.src_bytes

    def launch(self, i: int, stream: int) -> None:
        rc = self.lib.shipk_crop_nv12(self.frames[i % self.ring], 8, self.boxes.data_ptr(), self.idx.data_ptr(), 512,
                                      self.outputs[i % 2].data_ptr(), self.native.DTYPE_F16,
                                      self.outputs[0].numel() * 2, 256, 128, 1, stream)
        if rc:
            self.native.check(rc)

    def cpu_sample(self):
        return _nv12crop_cpu_sample(self.host_planes, self.host_boxes, self.host_idx)


def _nv12crop_cpu_sample(planes, boxes, idx):
    from oracle import oracle

    return (lambda: oracle.crop_nv12(planes, boxes[:64], (256, 128), idx[:64], True)), 64, \
        "64 boxes of one frame per call (C oracle)"


class Stream:
    """Config 4: 50 cameras (35 x 1080p, 15 x 720p, camera 0 at 8x the rate) sharded by camera;
    per GPU, batches of 32 frames letterboxed to [32,3,640,640] fp16, and class-aware NMS of the
    detector heads. A step's NMS does not read its letterbox's output (it works on detections
    of frames already through the detector, as the data plane's postprocess runs beside the next
    batch's preprocess), so each step forks it onto a second stream and joins it before the step
    ends: the two kernels overlap where the GPU has room for both."""

    name = "stream"
    workload = ("50-camera stream: letterbox mixed 1080p/720p -> [32,3,640,640] fp16, then class-aware "
                "NMS 32 x 8400 (config 4)")
    metric = "50-camera stream frames/s (letterbox fp16 + class-aware NMS per frame, config 4)"
    unit = "img/s"
    dtype = "f32"
    profile = "letterbox_stream_config4"
    batch = 32
    launches_per_step = 2  # the letterbox kernel and the NMS kernel
    cycle = 4              # distinct batches; every slot of the cycle is its own frame

    def __init__(self, torch, lib, native, device: int):
        from _data import camera_mix, nms_heads

        from shipinfer_b200.shard import shard_of

        self.torch, self.lib, self.native = torch, lib, native
        rank, world = int(os.environ.get("RANK", "0")), int(os.environ.get("WORLD_SIZE", "1"))
        fps, sizes = camera_mix()
        load = {f"cam{c:02d}": f for c, f in fps.items()}
        self.cameras = [int(n[3:]) for n in shard_of(load, list(range(world)), rank)]
        # smooth weighted round-robin over this GPU's cameras, weights = offered fps
        credit = {c: 0.0 for c in self.cameras}
        total = sum(fps[c] for c in self.cameras)
        slots = []
        for _ in range(self.cycle * self.batch):
            for c in self.cameras:
                credit[c] += fps[c]
            pick = max(self.cameras, key=lambda c: (credit[c], -c))
            credit[pick] -= total
            slots.append(pick)
        self.slots = slots
        dev = f"cuda:{device}"
        gen = torch.Generator(device=dev)
        gen.manual_seed(1000 + rank)
        self.frames, self.arrays, self.src_bytes = [], [], []
        for k in range(self.cycle):
            arr = (native.FrameU8 * self.batch)()
            nbytes = 0
            for j in range(self.batch):
                h, w = sizes[slots[k * self.batch + j]]
                f = torch.randint(0, 256, (h, w, 3), dtype=torch.uint8, device=dev, generator=gen)
                self.frames.append(f)
                arr[j] = native.FrameU8(f.data_ptr(), h, w, f.stride(0))
                # compulsory bytes: 640x640x3 fp16 out + the rows the resize reads (1080p: 360 of
                # 1080 at scale 3; 720p: every row at scale 2)
                nbytes += 3 * 640 * 640 * 2 + (360 * 1920 * 3 if h == 1080 else h * w * 3)
            self.arrays.append(arr)
            self.src_bytes.append(nbytes)
        self.nout = 4
        self.outputs = torch.empty((self.nout, self.batch, 3, 640, 640), dtype=torch.float16, device=dev)
        self.out_nbytes = self.outputs[0].numel() * 2
        b, sc, c = nms_heads(self.batch, 8400, 2, seed=0)
        self.ring = self.cycle
        self.heads = [(torch.from_numpy(np.roll(b, k, axis=1)).to(dev), torch.from_numpy(np.roll(sc, k, axis=1)).to(dev),
                       torch.from_numpy(np.roll(c, k, axis=1)).to(dev)) for k in range(2)]
        self.keep = torch.empty((self.batch, 300), dtype=torch.int64, device=dev)
        self.counts = torch.empty((self.batch,), dtype=torch.int32, device=dev)
        ws = lib.shipk_nms_workspace_bytes(self.batch, 8400, 2, 1, 300)
        self.ws = torch.empty((ws,), dtype=torch.uint8, device=dev)
        self.mean = native.floats3([0, 0, 0])
        self.std = native.floats3([255, 255, 255])
        self.device = device
        self.side = torch.cuda.Stream(device=dev)
        rt = cudart()
        self.events = []
        for _ in range(2):  # fork and join markers (no timing)
            e = ctypes.c_void_p()
            if rt.cudaEventCreateWithFlags(ctypes.byref(e), 2) != 0:
                raise RuntimeError("cudaEventCreateWithFlags failed")
            self.events.append(e)

    def config(self) -> dict:
        n1080 = sum(1 for c in self.slots if c < 35)
        return {"workload": self.workload,
                "batch": self.batch, "cameras_on_rank0": len(self.cameras),
                "frames_1080p_share": round(n1080 / len(self.slots), 3),
                "l2": f"inputs larger than L2: {len(self.frames)} distinct frames "
                      f"({sum(f.numel() for f in self.frames) / 1e6:.0f} MB) per GPU, outputs a ring of {self.nout}",
                "parallelism": "cameras sharded over GPUs by offered fps (plan_shards), one process per GPU"}

    def algorithmic_bytes(self) -> int:
        """Bytes of the letterbox launch (the dominant kernel), averaged over the cycle."""
        return sum(self.src_bytes) // len(self.src_bytes)

    def launch_shape(self) -> dict:
        ctas, cluster = ctypes.c_int(), ctypes.c_int()
        self.native.check(self.lib.shipk_nms_launch_shape(self.batch, 8400, 2, 1, 300, ctypes.byref(ctas),
                                                          ctypes.byref(cluster)))
        return {"nms": {"ctas": ctas.value, "threads_per_cta": 1024, "cluster": cluster.value}}

    def letterbox(self, i: int, stream: int) -> None:
        rc = self.lib.shipk_letterbox_u8(
            self.arrays[i % self.cycle], self.batch, self.outputs[i % self.nout].data_ptr(), self.native.DTYPE_F16,
            self.out_nbytes, 640, 640, self.mean, self.std, 1, 114.0, None, stream)
        if rc:
            self.native.check(rc)

    # e2e: the cycle's first batch as pinned host frames through the host-frame letterbox entry
    # point; beside it, on the second stream, the step's detector heads uploaded from pinned
    # host memory, NMS, and the kept indices and counts read back; plus each image's first
    # letterboxed row read back, as the headline's e2e does
    e2e_path = ("per step: shipk_ctx_letterbox_host from 32 pinned host frames (only the source rows the "
                "resize reads cross PCIe) and a D2H read of each image's first letterboxed row; beside it "
                "on a second stream an H2D copy of the step's detector heads, shipk_nms, and a D2H read of "
                "the kept indices and counts")

    def e2e_setup(self):
        torch = self.torch
        frames = self.frames[: self.batch]
        self.pinned = [f.cpu().pin_memory() for f in frames]
        arr = (self.native.HostFrameU8 * self.batch)()
        for j, f in enumerate(self.pinned):
            arr[j] = self.native.HostFrameU8(f.data_ptr(), f.shape[0], f.shape[1], f.stride(0))
        self.host_array = arr
        ctx = ctypes.c_void_p()
        self.native.check(self.lib.shipk_ctx_create(self.device, ctypes.byref(ctx)))
        self.ctx = ctx
        self.host_heads = [tuple(t.cpu().pin_memory() for t in h) for h in self.heads]
        self.dev_heads = [torch.empty_like(t) for t in self.heads[0]]
        self.rb_rows = torch.empty((self.batch, 3, 640), dtype=torch.float16).pin_memory()
        self.rb_keep = torch.empty((self.batch, 300), dtype=torch.int64).pin_memory()
        self.rb_counts = torch.empty((self.batch,), dtype=torch.int32).pin_memory()
        self.e2e_events = (torch.cuda.Event(), torch.cuda.Event())
        # bytes each step moves: each frame's rows the resize reads and its row map, the heads;
        # home: the letterboxed rows, the kept indices and the counts
        self.h2d = sum((360 * 1920 * 3 if f.shape[0] == 1080 else f.shape[0] * f.shape[1] * 3) + f.shape[0] * 4
                       for f in frames) + sum(t.numel() * t.element_size() for t in self.heads[0])
        self.d2h = sum(t.numel() * t.element_size() for t in (self.rb_rows, self.rb_keep, self.rb_counts))

    def e2e_step(self, i: int, stream) -> None:
        torch = self.torch
        fork, join = self.e2e_events
        fork.record(stream)
        self.side.wait_event(fork)
        out = self.outputs[i % self.nout]
        rc = self.lib.shipk_ctx_letterbox_host(
            self.ctx, self.host_array, self.batch, out.data_ptr(), self.native.DTYPE_F16, self.out_nbytes, 640, 640,
            self.mean, self.std, 1, 114.0, None, stream.cuda_stream)
        if rc:
            self.native.check(rc)
        self.rb_rows.copy_(out[:, :, 140, :], non_blocking=True)
        with torch.cuda.stream(self.side):
            for d, h in zip(self.dev_heads, self.host_heads[i % 2]):
                d.copy_(h, non_blocking=True)
            b, sc, c = self.dev_heads
            rc = self.lib.shipk_nms(b.data_ptr(), sc.data_ptr(), c.data_ptr(), self.batch, 8400, 2, 1, 0.45, 0.25,
                                    300, self.keep.data_ptr(), self.counts.data_ptr(), self.ws.data_ptr(),
                                    self.ws.numel(), self.side.cuda_stream)
            if rc:
                self.native.check(rc)
            self.rb_keep.copy_(self.keep, non_blocking=True)
            self.rb_counts.copy_(self.counts, non_blocking=True)
        join.record(self.side)
        stream.wait_event(join)

    def e2e_close(self):
        self.lib.shipk_ctx_destroy(self.ctx)

    def launch(self, i: int, stream: int) -> None:
        rt = cudart()
        fork, join = self.events
        main, side = ctypes.c_void_p(stream), ctypes.c_void_p(self.side.cuda_stream)
        if rt.cudaEventRecord(fork, main) or rt.cudaStreamWaitEvent(side, fork, 0):
            raise RuntimeError("stream fork failed")
        self.letterbox(i, stream)
        b, sc, c = self.heads[i % 2]
        rc = self.lib.shipk_nms(b.data_ptr(), sc.data_ptr(), c.data_ptr(), self.batch, 8400, 2, 1, 0.45, 0.25, 300,
                                self.keep.data_ptr(), self.counts.data_ptr(), self.ws.data_ptr(), self.ws.numel(),
                                side.value)
        if rc:
            self.native.check(rc)
        if rt.cudaEventRecord(join, side) or rt.cudaStreamWaitEvent(main, join, 0):
            raise RuntimeError("stream join failed")

    dominant = letterbox

    def cpu_sample(self):
        return _stream_cpu_sample()


def _stream_cpu_sample():
    """Eight frames of the camera mix (six 1080p, two 720p) letterboxed to fp16 and their heads
    suppressed, on the host cores."""
    from oracle import oracle

    from _data import FRAME_720, frames_u8, nms_heads

    frames = frames_u8(6, (1080, 1920), seed=0) + frames_u8(2, FRAME_720, seed=1)
    b, s, c = nms_heads(8, 8400, 2, seed=0)

    def step():
        oracle.letterbox(frames, (640, 640)).astype(np.float16)
        oracle.nms_batched(b, s, c, 0.45, 0.25, 300, num_classes=2)

    return step, 8, "8 frames (6 x 1080p, 2 x 720p) letterboxed to fp16 plus NMS on their 8 x 8400 heads"


class Mask:
    """Segmenter mask areas: a batch of 64 crops at the shipped segmenter's shapes (300
    candidates x 38 columns, 32 prototype planes of 160 x 160), one area per crop."""

    name = "mask"
    workload = ("mask area, 64 crops: rows [64,300,38], prototypes [64,32,160,160] fp32, score 0.25, "
                "mask threshold 0.5, crop 256x128")
    metric = "mask-area crops/s (64 crops x 32 x 160 x 160 prototypes)"
    unit = "crops/s"
    dtype = "f32"
    profile = "mask_area_segmenter"
    batch = 64

    def __init__(self, torch, lib, native, device: int):
        self.torch, self.lib, self.native = torch, lib, native
        dev = f"cuda:{device}"
        gen = torch.Generator(device=dev)
        gen.manual_seed(5)
        self.rows = torch.randn((self.batch, 300, 38), device=dev, generator=gen)
        self.rows[:, :, 4].uniform_(0.0, 1.0, generator=gen)
        # two distinct banks (420 MB) cycled, so every step reads its planes from HBM
        self.ring = 2
        self.protos = [torch.randn((self.batch, 32, 160, 160), device=dev, generator=gen) for _ in range(self.ring)]
        self.areas = torch.empty((self.batch,), dtype=torch.float32, device=dev)

    def config(self) -> dict:
        return {"workload": self.workload,
                "batch": self.batch, "l2": "inputs larger than L2: two 210 MB prototype banks cycled",
                "parallelism": "camera-sharded replicas, one per GPU"}

    def algorithmic_bytes(self) -> int:
        # the prototype bank, the score column, the chosen row and the area, per crop
        return self.batch * (32 * 160 * 160 * 4 + 300 * 4 + 38 * 4 + 4)

    def launch(self, i: int, stream: int) -> None:
        rc = self.lib.shipk_mask_area(self.rows.data_ptr(), 300, 38, 6, self.protos[i % self.ring].data_ptr(), 32,
                                      160 * 160, self.batch, 0.25, 0.5, 256, 128, self.areas.data_ptr(), stream)
        if rc:
            self.native.check(rc)

    def cpu_sample(self):
        return _mask_cpu_sample()


def _mask_cpu_sample():
    from oracle import oracle

    rng = np.random.default_rng(5)
    rows = rng.standard_normal((4, 300, 38)).astype(np.float32)
    rows[:, :, 4] = rng.uniform(0.0, 1.0, (4, 300))
    protos = rng.standard_normal((4, 32, 160, 160)).astype(np.float32)
    return (lambda: oracle.mask_area(rows, protos, prefix=6, score_threshold=0.25, mask_threshold=0.5,
                                     crop_hw=(256, 128))), 4, "4 crops of 32 x 160 x 160 per call (C oracle, OpenMP)"


class Decode:
    """Detector decode: 32 frames x 8400 raw detector rows -> at most 100 detections each
    (score 0.25), un-letterboxed and clipped to 1080p."""

    name = "decode"
    workload = ("decode_detections on the device: 32 frames x 8400 rows [x1,y1,x2,y2,score,class], "
                "score 0.25, cap 100, scale 1/3, pad (0,140), clip 1080p")
    metric = "detector decode frames/s (32 x 8400 rows, cap 100)"
    unit = "img/s"
    dtype = "f32"
    profile = "decode_detections"
    batch = 32

    def __init__(self, torch, lib, native, device: int):
        self.torch, self.lib, self.native = torch, lib, native
        dev = f"cuda:{device}"
        gen = torch.Generator(device=dev)
        gen.manual_seed(7)
        self.ring = 2
        self.rows = []
        for _ in range(self.ring):
            r = torch.rand((self.batch, 8400, 6), device=dev, generator=gen) * 640
            r[:, :, 4] = torch.rand((self.batch, 8400), device=dev, generator=gen)
            self.rows.append(r.contiguous())
        self.scales = torch.full((self.batch,), float(np.float32(1 / 3)), device=dev)
        self.pads = torch.tensor([[0.0, 140.0]] * self.batch, device=dev)
        self.hw = torch.tensor([[1080, 1920]] * self.batch, dtype=torch.int32, device=dev)
        self.boxes = torch.empty((self.batch, 100, 4), device=dev)
        self.scores = torch.empty((self.batch, 100), device=dev)
        self.classes = torch.empty((self.batch, 100), dtype=torch.int32, device=dev)
        self.counts = torch.empty((self.batch,), dtype=torch.int32, device=dev)
        self.discarded = torch.empty((self.batch,), dtype=torch.int32, device=dev)

    def config(self) -> dict:
        return {"workload": self.workload,
                "batch": self.batch, "l2": "inputs (6.5 MB a step) fit in L2; the kernel is latency-bound",
                "parallelism": "camera-sharded replicas, one per GPU"}

    def algorithmic_bytes(self) -> int:
        return self.batch * (8400 * 6 * 4 + 100 * (16 + 4 + 4) + 8)

    def launch(self, i: int, stream: int) -> None:
        rc = self.lib.shipk_decode_detections(
            self.rows[i % self.ring].data_ptr(), self.batch, 8400, None, self.scales.data_ptr(), self.pads.data_ptr(),
            self.hw.data_ptr(), 0.25, 100, self.boxes.data_ptr(), self.scores.data_ptr(), self.classes.data_ptr(),
            self.counts.data_ptr(), self.discarded.data_ptr(), stream)
        if rc:
            self.native.check(rc)

    def cpu_sample(self):
        return _decode_cpu_sample()


def _decode_cpu_sample():
    from oracle import oracle

    rng = np.random.default_rng(7)
    rows = (rng.uniform(0, 640, (32, 8400, 6))).astype(np.float32)
    rows[:, :, 4] = rng.uniform(0, 1, (32, 8400))

    scales = np.full(32, np.float32(1 / 3), np.float32)
    pads = np.tile(np.array([0.0, 140.0], np.float32), (32, 1))
    hw = np.tile(np.array([1080, 1920], np.int32), (32, 1))
    return (lambda: oracle.decode_batched(rows, score_threshold=0.25, max_detections=100, scales=scales, pads=pads,
                                          frame_hw=hw)), 32, "32 frames x 8400 rows per call (C oracle, OpenMP)"


WORKLOADS = {"letterbox": Letterbox, "nms": Nms, "crop": Crop, "nv12": Nv12, "stream": Stream, "mask": Mask,
             "decode": Decode, "nv12crop": Nv12Crop}


# ---------------------------------------------------------------------------------------------


def cpu_rate(sample, seconds: float) -> tuple[float, float, int]:
    """Units per second of the CPU sample, run repeatedly for about `seconds`."""
    fn, units, _ = sample
    fn()  # warm (builds the oracle if needed, faults in pages)
    done, t0 = 0, time.perf_counter()
    while True:
        fn()
        done += units
        elapsed = time.perf_counter() - t0
        if elapsed >= seconds:
            return done / elapsed, elapsed, done


def cpu_threads() -> int:
    try:
        return len(os.sched_getaffinity(0))
    except AttributeError:
        return os.cpu_count() or 1


# ---------------------------------------------------------------------------------------------
# the reference's own CPU path (TorchImageOps on the host), when its offline install is present

REFERENCE_SITE = ROOT / "baseline" / "_ref"


def reference_ops_module():
    """``shipinfer.runtime.ops`` from the reference's offline install under baseline/_ref, or
    None (with the reason) when it is absent. The reference is run unmodified through its own
    public API."""
    if not (REFERENCE_SITE / "shipinfer").exists():
        return None, "the reference's offline install (baseline/_ref) is absent"
    if str(REFERENCE_SITE) not in sys.path:
        sys.path.append(str(REFERENCE_SITE))
    try:
        import shipinfer.runtime.ops as ref_ops

        return ref_ops, None
    except Exception as exc:  # the reason goes into the line
        return None, f"importing the reference failed: {type(exc).__name__}: {exc}"


def reference_cpu_sample(name: str):
    """``((fn, units, description), None)``: a bounded sample of the workload through the
    reference's TorchImageOps() on the host cores (torch CPU threads = every CPU of the
    affinity), for configs 1 and 3; ``(None, why)`` where there is none."""
    ref, why = reference_ops_module()
    if ref is None:
        return None, why
    import torch

    torch.set_num_threads(cpu_threads())
    from _data import IMAGENET_MEAN, IMAGENET_STD, crop_boxes, frames_u8

    ops = ref.TorchImageOps()
    if name == "letterbox":
        frames = frames_u8(8, (1080, 1920), seed=0)
        p = ref.NormalizeParams()
        return ((lambda: ops.letterbox_batch(frames, (640, 640), p)), 8,
                "TorchImageOps().letterbox_batch of one batch of 8 x 1080p frames per call"), None
    if name == "crop":
        frames = frames_u8(1, (1080, 1920), seed=0)
        boxes, _ = crop_boxes(1, 64)
        p = ref.NormalizeParams(mean=IMAGENET_MEAN, std=IMAGENET_STD)
        return ((lambda: ops.crop_batch(frames[0], boxes, (256, 128), p).astype(np.float16)), 64,
                "TorchImageOps().crop_batch of 64 boxes of one frame per call, then fp16"), None
    return None, "the reference has no CPU path for this workload"


def reference_cpu_entry(name: str, seconds: float, unit: str) -> dict | None:
    sample, why = reference_cpu_sample(name)
    if sample is None:
        return {"unavailable": why} if why else None
    rate, secs, done = cpu_rate(sample, seconds)
    return {"value": rate, "unit": unit, "cores": cpu_threads(), "kind": "reference",
            "sample": f"{sample[2]}, repeated {done // sample[1]} times over {secs:.1f} s "
                      f"(the reference's own code from baseline/_ref, torch CPU threads {cpu_threads()})"}


# ---------------------------------------------------------------------------------------------
# the reference arm


def run_reference(args, dist: Dist) -> None:
    """The reference arm: the reference's CPU formulation (the C oracle port) on host cores,
    the headline workload and, unless --no-extras, the extras' workloads."""
    if dist.rank != 0:
        return
    cls = WORKLOADS[args.config]

    def time_cpu(c):
        fn, units, desc = _cpu_only_sample(c)
        for _ in range(max(args.warmup, 0)):
            fn()
        t0 = time.perf_counter()
        for _ in range(args.steps):
            fn()
        elapsed = time.perf_counter() - t0
        return units * args.steps / elapsed, elapsed / args.steps * 1e3, desc

    value, ms, desc = time_cpu(cls)
    line = {
        "impl": "reference",
        "metric": cls.metric,
        "value": value,
        "unit": cls.unit,
        "n_gpus": args.gpus,
        "steps": args.steps,
        "warmup": args.warmup,
        "ms_per_step": ms,
        "higher_is_better": True,
        "scaling": "weak",
        "vs_baseline": None,
        "dtype": cls.dtype,
        "data": "synthetic",
        # the GPU arm's config where it is computable without a GPU, else its workload
        "config": cls.static_config() if hasattr(cls, "static_config") else {"workload": cls.workload},
        "cpu_baseline": {"value": value, "unit": cls.unit, "cores": cpu_threads(), "kind": "port",
                         "sample": f"{args.steps} steps, each {desc} (C oracle, OpenMP)"},
        "e2e": {"value": value, "unit": cls.unit, "h2d_bytes_per_step": 0, "d2h_bytes_per_step": 0},
    }
    if not args.no_extras and args.config == "letterbox":
        line["cpu_baseline_reference"] = reference_cpu_entry("letterbox", args.extra_cpu_seconds, cls.unit)
        extras = {}
        for key in EXTRAS:
            c = WORKLOADS[key]
            v, m, d = time_cpu(c)
            extras[key] = {"metric": c.metric, "value": v, "unit": c.unit, "ms_per_step": m, "kind": "port",
                           "cores": cpu_threads(), "sample": f"{args.steps} steps, each {d}"}
        ref_crop = reference_cpu_entry("crop", args.extra_cpu_seconds, Crop.unit)
        if ref_crop is not None:
            extras["crop"]["cpu_baseline_reference"] = ref_crop
        line["extras"] = extras
    print(json.dumps(line), flush=True)


def _cpu_only_sample(cls):
    from oracle import oracle

    from _data import IMAGENET_MEAN, IMAGENET_STD, crop_boxes, frames_u8, nms_heads, nv12_frames

    if cls is Letterbox:
        frames = frames_u8(8, (1080, 1920), seed=0)
        return (lambda: oracle.letterbox(frames, (640, 640))), 8, "one batch of 8 x 1080p frames"
    if cls is Nms:
        b, s, c = nms_heads(16, 8400, 2, seed=0)
        return (lambda: oracle.nms_batched(b, s, c, 0.45, 0.25, 300, num_classes=2)), 16, "16 images x 8400"
    if cls is Crop:
        frames = frames_u8(8, seed=0)
        boxes, idx = crop_boxes(8, 64)
        return (lambda: oracle.crop(frames, boxes[:64], (256, 128), idx[:64], IMAGENET_MEAN, IMAGENET_STD, True)), \
            64, "64 boxes of one frame"
    if cls is Stream:
        return _stream_cpu_sample()
    if cls is Mask:
        return _mask_cpu_sample()
    if cls is Decode:
        return _decode_cpu_sample()
    if cls is Nv12Crop:
        boxes, idx = crop_boxes(8, 64)
        planes = nv12_frames(8, (1080, 1920), seed=0, pitch=2048, coded_h=1088)
        return _nv12crop_cpu_sample(planes, boxes, idx)
    planes = nv12_frames(1, (2160, 3840), seed=0)
    return (lambda: oracle.letterbox_nv12(planes, (1280, 1280), matrix=709, sampling=1)), 1, "one 4K frame"


# ---------------------------------------------------------------------------------------------
# device timing


MAX_REPEATS = 20000


def time_replays(torch, dist: Dist, launch, steps: int, ring: int, min_seconds: float) -> dict:
    """Capture `steps` launches into CUDA graphs, then time that K-step replay back to back
    with CUDA events on the replay stream until at least `min_seconds` of device time has
    elapsed. Barrier + synchronize before and after the set; every rank replays the same
    number of times (from a calibration replay's max over ranks). Returns the rank-max of the
    per-rank median window (ms), the repeat count, the per-rank medians and the host clock
    around the set."""
    replay, stream, graphs = capture_steps(torch, launch, steps, ring)
    cal_start, cal_end = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
    dist.barrier()
    torch.cuda.synchronize()
    with torch.cuda.stream(stream):
        cal_start.record(stream)
        replay()
        cal_end.record(stream)
    torch.cuda.synchronize()
    cal_ms = dist.max(cal_start.elapsed_time(cal_end))
    repeats = int(min(MAX_REPEATS, max(5, math.ceil(min_seconds * 1e3 / max(cal_ms, 1e-3)))))
    events = [(torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)) for _ in range(repeats)]
    dist.barrier()
    torch.cuda.synchronize()
    t0 = time.perf_counter()
    with torch.cuda.stream(stream):
        for start, end in events:
            start.record(stream)
            replay()
            end.record(stream)
    torch.cuda.synchronize()
    t1 = time.perf_counter()
    dist.barrier()
    windows = sorted(start.elapsed_time(end) for start, end in events)
    median = statistics.median(windows)
    per_rank = dist.gather(median)
    del graphs
    return {"window_ms": max(per_rank), "repeats": repeats, "per_rank_ms": per_rank, "t0": t0, "t1": t1,
            "spread": (windows[-1] - windows[0]) / median if median > 0 else 0.0}


def per_rank_summary(per_rank: list[float], steps: int) -> dict:
    per_step = sorted(v / steps for v in per_rank)
    return {"min": per_step[0], "median": statistics.median(per_step), "max": per_step[-1],
            "ranks": [v / steps for v in per_rank]}


def measure_workload(torch, dist: Dist, w, args, peak: float, peak_kind: str) -> dict:
    """Warm-up, the timed replays, and the dominant kernel alone where a step runs two."""
    stream = torch.cuda.Stream()
    with torch.cuda.stream(stream):
        for i in range(args.warmup):
            w.launch(i, stream.cuda_stream)
    torch.cuda.synchronize()
    ring = math.lcm(w.ring, getattr(w, "nout", 2))
    t = time_replays(torch, dist, w.launch, args.steps, ring, args.min_seconds)
    ms_per_step = t["window_ms"] / args.steps
    kernel_ms = ms_per_step
    if hasattr(w, "dominant"):
        k = time_replays(torch, dist, w.dominant, args.steps, ring, args.min_seconds)
        kernel_ms = k["window_ms"] / args.steps
    achieved = w.algorithmic_bytes() / (kernel_ms / 1e3) / 1e9
    bound = getattr(w, "bound", "hbm")
    entry = {
        "metric": w.metric,
        "value": w.batch * dist.world / (ms_per_step / 1e3),
        "unit": w.unit,
        "ms_per_step": ms_per_step,
        "timing": {"steps": args.steps, "repeats": t["repeats"], "statistic": "median window, max over ranks",
                   "spread": t["spread"]},
        "config": w.config(),
        "roofline": {
            "bound": bound,
            "achieved": achieved,
            "peak": peak,
            "unit": "GB/s",
            "frac": achieved / peak,
            "peak_kind": f"{peak_kind} (MEASURED_PEAKS.json hbm_gbs)" if peak_kind == "measured" else "fallback",
            "algorithmic_bytes_per_launch": w.algorithmic_bytes(),
            "kernel_ms": kernel_ms,
            "traffic": ncu_traffic(w.profile),
        },
        # every launch of the timed set: K steps per window, `repeats` windows
        "gpu_launches": args.steps * t["repeats"] * getattr(w, "launches_per_step", 1),
        "_t": (t["t0"], t["t1"]),
    }
    if bound != "hbm":
        entry["roofline"]["note"] = getattr(w, "bound_note", "")
    if hasattr(w, "launch_shape"):
        entry["launch"] = w.launch_shape()
    if dist.world > 1:
        entry["per_rank_ms"] = per_rank_summary(t["per_rank_ms"], args.steps)
    return entry


def e2e_pinned(torch, dist: Dist, w, args) -> dict:
    """A workload's e2e through the host-frame C ABI, from pinned host frames: the headline's,
    and the stream extra's (config 4 with its host-to-device copies)."""
    w.e2e_setup()
    es = torch.cuda.Stream()
    with torch.cuda.stream(es):
        for i in range(max(args.warmup, 3)):
            w.e2e_step(i, es)
    torch.cuda.synchronize()
    e_start, e_end = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
    dist.barrier()
    torch.cuda.synchronize()
    with torch.cuda.stream(es):
        e_start.record(es)
        for i in range(args.steps):
            w.e2e_step(i, es)
        e_end.record(es)
    torch.cuda.synchronize()
    dist.barrier()
    own = e_start.elapsed_time(e_end)
    e_ms = dist.max(own)
    w.e2e_close()
    out = {"value": w.batch * args.steps * dist.world / (e_ms / 1e3), "unit": w.unit,
           "h2d_bytes_per_step": w.h2d, "d2h_bytes_per_step": w.d2h,
           "ms_per_step": e_ms / args.steps,
           "path": getattr(w, "e2e_path", "shipk_ctx_letterbox_host from pinned host frames (only the source "
                                          "rows the resize reads cross PCIe), then a D2H read of each image's "
                                          "first letterboxed row")}
    if dist.world > 1:
        out["per_rank_ms"] = per_rank_summary(dist.gather(own), args.steps)
    return out


# ---------------------------------------------------------------------------------------------
# the seam: the reference's kernel-benchmark cases and pageable frames through the Python API


def _host_time(torch, device: int, call, iterations: int = 20, repeat: int = 7, warmup: int = 3) -> float:
    """Median per-call seconds over `repeat` batches of `iterations` synchronised calls, as the
    reference's kernel benchmark times a call (benchmarks/kernels.py:115-168): host clock
    around the batch, a device synchronize after each call."""
    def synced():
        call()
        torch.cuda.synchronize(device)

    for _ in range(warmup):
        synced()
    batches = []
    for _ in range(repeat):
        t0 = time.perf_counter()
        for _ in range(iterations):
            synced()
        batches.append((time.perf_counter() - t0) / iterations)
    return statistics.median(batches)


def _kernel_cases(torch, ops, device: int, NormalizeParams) -> dict:
    """The reference kernel benchmark's three cases (benchmarks/kernels.py:323-343) on its own
    inputs: letterbox_to_device of one 1080p frame, crop_batch of 15 boxes, nms of 25 000."""
    from _data import kernels_bench_inputs

    frame, boxes, nms_boxes, nms_scores = kernels_bench_inputs(0)
    params = NormalizeParams()
    out = torch.empty((1, 3, 640, 640), dtype=torch.float32, device=f"cuda:{device}")
    return {
        "letterbox_to_device_1x1080p": lambda: ops.letterbox_to_device([frame], out, params),
        "crop_batch_15_boxes": lambda: ops.crop_batch(frame, boxes, (256, 128), params),
        "nms_25000_candidates": lambda: ops.nms(nms_boxes, nms_scores, 0.45, 0.25, 300),
    }


# the reference's published figures for the same calls (RTX A5000; .claude/TASKS.md:1171-1176)
PUBLISHED_US = {"letterbox_to_device_1x1080p": 657.0, "crop_batch_15_boxes": 1303.0,
                "nms_25000_candidates": 33300.0}


def measure_seam(torch, dist: Dist, device: int) -> dict:
    """Through the reference-facing Python API (NativeImageOps and the shipvision._C surface)
    with pageable numpy frames, as callers use it; timed with the host clock around each
    synchronised call (it includes the host-side staging). Beside it, when the reference's
    offline install is present, the same calls through the reference's own
    TorchImageOps(device_index) on this GPU."""
    from _data import frames_u8

    from shipinfer_b200 import NativeImageOps, NormalizeParams, shipvision_C

    ops = NativeImageOps(device_index=device)
    out = {"timing": "median of 7 batches of 20 calls, host clock, device synchronize after each call "
                     "(benchmarks/kernels.py:115-168)"}
    cases = {}
    for name, call in _kernel_cases(torch, ops, device, NormalizeParams).items():
        sec = dist.max(_host_time(torch, device, call))
        cases[name] = {"us_per_call": sec * 1e6, "reference_published_us_a5000": PUBLISHED_US[name]}
    # config 1 from pageable host frames: letterbox_to_device (device tensor out, one row read
    # back), the shipvision._C letterbox_into (raw pointer out) and letterbox_batch (numpy out)
    frames = frames_u8(8, (1080, 1920), seed=0)
    params = NormalizeParams()
    dev_out = torch.empty((8, 3, 640, 640), dtype=torch.float32, device=f"cuda:{device}")
    row = torch.empty((8, 3, 640), dtype=torch.float32).pin_memory()

    def to_device():
        ops.letterbox_to_device(frames, dev_out, params)
        row.copy_(dev_out[:, :, 140, :])

    c_ops = shipvision_C.ImageOps(device)

    def into():
        c_ops.letterbox_into(frames, dev_out.data_ptr(), dev_out.numel() * 4, 640, 640, [0, 0, 0],
                             [255, 255, 255], True, 114, torch.cuda.current_stream(device).cuda_stream)

    config1 = {}
    for name, call, iters in (("letterbox_to_device_pageable", to_device, 10),
                              ("shipvision_C_letterbox_into_pageable", into, 10),
                              ("letterbox_batch_numpy_out", lambda: ops.letterbox_batch(frames, (640, 640), params),
                               5)):
        sec = dist.max(_host_time(torch, device, call, iterations=iters, repeat=5))
        config1[name] = {"img_per_s": 8 * dist.world / sec, "ms_per_batch": sec * 1e3}
    out["kernel_cases"] = cases
    out["config1_pageable"] = config1
    ref, why = reference_ops_module()
    if ref is None:
        out["reference_torch_cuda"] = {"unavailable": why}
    else:
        rops = ref.TorchImageOps(device_index=device)
        rc = {}
        for name, call in _kernel_cases(torch, rops, device, ref.NormalizeParams).items():
            sec = dist.max(_host_time(torch, device, call))
            rc[name] = {"us_per_call": sec * 1e6}
        rout = torch.empty((8, 3, 640, 640), dtype=torch.float32, device=f"cuda:{device}")
        rparams = ref.NormalizeParams()

        def ref_to_device():
            rops.letterbox_to_device(frames, rout, rparams)
            row.copy_(rout[:, :, 140, :])

        sec = dist.max(_host_time(torch, device, ref_to_device, iterations=10, repeat=5))
        rc["config1_letterbox_to_device_pageable"] = {"img_per_s": 8 * dist.world / sec, "ms_per_batch": sec * 1e3}
        sec = dist.max(_host_time(torch, device, lambda: rops.letterbox_batch(frames, (640, 640), rparams),
                                  iterations=5, repeat=5))
        rc["config1_letterbox_batch_numpy_out"] = {"img_per_s": 8 * dist.world / sec, "ms_per_batch": sec * 1e3}
        out["reference_torch_cuda"] = {"what": "the reference's TorchImageOps(device_index) on this GPU, "
                                               "same calls and inputs (its own code from baseline/_ref)", **rc}
    return out


EXTRAS = ("nms", "crop", "nv12", "stream")


def main() -> None:
    args = parse_args()
    dist = Dist()
    if args.impl == "reference":
        run_reference(args, dist)
        return

    import torch

    from shipinfer_b200 import _native

    dist.init()
    device = dist.local
    torch.cuda.set_device(device)
    lib = _native.lib()
    peak, peak_kind = hbm_peak()
    clocks = ClockSampler(device)
    clocks.start()

    w = WORKLOADS[args.config](torch, lib, _native, device)
    head = measure_workload(torch, dist, w, args, peak, peak_kind)
    clocks_summary = clocks.summary(*head.pop("_t"))

    e2e = None
    if not args.no_e2e and hasattr(w, "e2e_setup"):
        e2e = e2e_pinned(torch, dist, w, args)
    cpu = cpu_ref = None
    if dist.rank == 0 and dist.world == 1 and not args.no_cpu_baseline:
        sample = w.cpu_sample()
        rate, secs, done = cpu_rate(sample, args.cpu_seconds)
        cpu = {"value": rate, "unit": w.unit, "cores": cpu_threads(), "kind": "port",
               "sample": f"{sample[2]}, repeated {done // sample[1]} times over {secs:.1f} s (C oracle, OpenMP)"}
        if args.config in ("letterbox", "crop"):
            cpu_ref = reference_cpu_entry(args.config, args.extra_cpu_seconds, w.unit)
    del w
    torch.cuda.empty_cache()

    extras = None
    if not args.no_extras and args.config == "letterbox":
        extras = {}
        for key in EXTRAS:
            x = WORKLOADS[key](torch, lib, _native, device)
            entry = measure_workload(torch, dist, x, args, peak, peak_kind)
            entry["clocks"] = clocks.summary(*entry.pop("_t"))
            if not args.no_e2e and hasattr(x, "e2e_setup"):
                entry["e2e"] = e2e_pinned(torch, dist, x, args)
            if dist.rank == 0 and dist.world == 1 and not args.no_cpu_baseline:
                sample = x.cpu_sample()
                rate, secs, done = cpu_rate(sample, args.extra_cpu_seconds)
                entry["cpu_baseline"] = {"value": rate, "unit": x.unit, "cores": cpu_threads(), "kind": "port",
                                         "sample": f"{sample[2]}, repeated {done // sample[1]} times over "
                                                   f"{secs:.1f} s (C oracle, OpenMP)"}
                if key == "crop":
                    entry["cpu_baseline_reference"] = reference_cpu_entry("crop", args.extra_cpu_seconds, x.unit)
            extras[key] = entry
            del x
            torch.cuda.empty_cache()
        extras["seam"] = measure_seam(torch, dist, device)
    clocks.stop()

    if dist.rank == 0:
        line = {
            "metric": head["metric"],
            "value": head["value"],
            "unit": head["unit"],
            "n_gpus": dist.world,
            "steps": args.steps,
            "warmup": args.warmup,
            "ms_per_step": head["ms_per_step"],
            "higher_is_better": True,
            "scaling": "weak",
            "vs_baseline": None,
            "dtype": WORKLOADS[args.config].dtype,
            "data": "synthetic",
            "config": head["config"],
            "timing": head["timing"],
            "roofline": head["roofline"],
            "cpu_baseline": cpu,
            "e2e": e2e,
            "gpu_launches": head["gpu_launches"],
            "clocks": clocks_summary,
        }
        if cpu_ref is not None:
            line["cpu_baseline_reference"] = cpu_ref
        if "per_rank_ms" in head:
            line["per_rank_ms"] = head["per_rank_ms"]
        if extras is not None:
            line["extras"] = extras
        print(json.dumps(line), flush=True)
    dist.close()


if __name__ == "__main__":
    main()
