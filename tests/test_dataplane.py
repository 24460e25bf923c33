"""The C++ data plane's pixel calls (reference csrc/shipinfer/runtime/ops.h) on libshipk.

shipinfer_b200/dataplane/ops_shipk.cpp implements ops.h's functions (letterbox_fit,
letterbox_into, crop_resize_into, nv12_letterbox_into, nv12_crop_resize_into, mask_area_into)
on the C ABI, as a drop-in for ops.cu. Here:

* it compiles against the reference tree's own headers (when the reference is present), which is
  what makes it a drop-in, and against the restated headers beside it;
* a harness (tests/dataplane_harness.cpp) compiled with it exposes the C++ calls to ctypes:
  host-side geometry and refusals run on the CPU; on a B200 every call is checked against the
  oracle bit for bit, the NV12 and mask calls being the reference kernels' own arithmetic;
* shipinfer_b200/dataplane/crop_batch.cpp, the reference's CropStage (stages.cpp:195-245) over
  a batch of frames: its row selection on the CPU, and on a B200 its one-upload, one-launch-per-
  set-and-representation, one-synchronise run against the per-frame calls and the oracle.
"""

from __future__ import annotations

import ctypes
import os
import shutil
import subprocess
from pathlib import Path

import numpy as np
import pytest

ROOT = Path(__file__).resolve().parents[1]
DP = ROOT / "shipinfer_b200" / "dataplane"
LIBDIR = ROOT / "shipinfer_b200" / "_lib"
REFERENCE = Path(os.environ.get("SHIPK_REFERENCE", "/root/reference")) / "csrc"  # the reference tree, if present
CUDA_INCLUDE = Path(os.environ.get("CUDA_HOME", "/usr/local/cuda")) / "include"
PAD = float(np.float32(114) / np.float32(255))  # the bars' output value: what 114 normalises to


def _cxx() -> str:
    cxx = shutil.which("g++") or shutil.which("c++")
    if cxx is None:
        pytest.skip("no C++ compiler")
    return cxx


@pytest.fixture(scope="module")
def harness(tmp_path_factory):
    """ops_shipk.cpp + the harness, linked against the in-tree libshipk.so."""
    if not (LIBDIR / "libshipk.so").exists():
        pytest.skip("libshipk.so is not built")
    out = tmp_path_factory.mktemp("dataplane") / "libdp_harness.so"
    cuda_lib = CUDA_INCLUDE.parent / "lib64"
    cmd = [_cxx(), "-std=c++17", "-O2", "-shared", "-fPIC", f"-I{DP / 'include'}", f"-I{DP}", f"-I{ROOT / 'include'}",
           f"-I{CUDA_INCLUDE}", str(DP / "ops_shipk.cpp"), str(DP / "crop_batch.cpp"),
           str(ROOT / "tests" / "dataplane_harness.cpp"), f"-L{LIBDIR}", "-lshipk", f"-L{cuda_lib}", "-lcudart",
           f"-Wl,-rpath,{LIBDIR}", f"-Wl,-rpath,{cuda_lib}", "-o", str(out)]
    subprocess.run(cmd, check=True, capture_output=True, text=True)
    lib = ctypes.CDLL(str(out))
    vp, i, f, fp, cp = ctypes.c_void_p, ctypes.c_int, ctypes.c_float, ctypes.POINTER(ctypes.c_float), ctypes.c_char_p
    u64 = ctypes.c_ulonglong
    lib.h_letterbox_fit.argtypes = [i, i, i, i, fp, cp, i]
    lib.h_letterbox_into.argtypes = [vp, i, i, vp, i, i, i, f, fp, vp, cp, i]
    lib.h_crop_resize_into.argtypes = [vp, i, i, vp, i, vp, i, i, i, vp, cp, i]
    lib.h_nv12_letterbox_into.argtypes = [vp, i, i, i, u64, vp, i, i, i, f, fp, vp, cp, i]
    lib.h_nv12_crop_resize_into.argtypes = [vp, i, i, i, u64, vp, i, vp, i, i, i, vp, cp, i]
    lib.h_mask_area_into.argtypes = [vp, i, i, i, vp, i, i, i, f, f, i, i, vp, vp, cp, i]
    ip = ctypes.POINTER(ctypes.c_int)
    lib.h_batched_crop.argtypes = [i, vp, vp, ip, ip, ip, ctypes.POINTER(u64), ip, fp, ip, ip, i, ip, ip, ip, vp, i,
                                   i, vp, ip, ip, ip, ip, cp, i]
    return lib


def _err():
    return ctypes.create_string_buffer(512)


def _map():
    return (ctypes.c_float * 5)()


def test_drop_in_compiles_against_the_reference_headers():
    """ops_shipk.cpp in place of ops.cu, with the reference tree's own ops.h / platform.h /
    types.h on the include path."""
    if not (REFERENCE / "shipinfer" / "runtime" / "ops.h").exists():
        pytest.skip("the reference source tree is not present on this machine")
    for src in ("ops_shipk.cpp", "crop_batch.cpp"):
        cmd = [_cxx(), "-std=c++17", "-fsyntax-only", f"-I{REFERENCE}", f"-I{ROOT / 'include'}", f"-I{DP}",
               f"-I{CUDA_INCLUDE}", str(DP / src)]
        res = subprocess.run(cmd, capture_output=True, text=True)
        assert res.returncode == 0, res.stderr


@pytest.mark.parametrize(("src", "dst", "want"), [
    ((1080, 1920), (640, 640), (np.float32(1 / 3), 0, 140, 640, 360)),
    ((720, 1280), (640, 640), (0.5, 0, 140, 640, 360)),
    ((2160, 3840), (1280, 1280), (np.float32(1 / 3), 0, 280, 1280, 720)),
    ((251, 500), (250, 250), (0.5, 0, 62, 250, 126)),  # round half to even: 125.5 -> 126
    ((90, 160), (64, 64), (0.4, 0, 14, 64, 36)),
])
def test_letterbox_fit_known_answers(harness, src, dst, want):
    m, e = _map(), _err()
    assert harness.h_letterbox_fit(src[0], src[1], dst[0], dst[1], m, e, 512) == 0, e.value
    assert m[0] == pytest.approx(float(np.float32(want[0])), abs=0) and tuple(int(v) for v in m[1:]) == want[1:]


def test_letterbox_fit_is_the_planes_float32_rule(harness, orc):
    """The plane's letterbox_fit is ops.cu's float32 rule, not the Python plane's double one:
    they part at 180x1280 -> 224x224 (32 rows against 31)."""
    m, e = _map(), _err()
    for src in ((180, 1280), (340, 1280), (660, 1280), (1080, 1920)):
        assert harness.h_letterbox_fit(src[0], src[1], 224, 224, m, e, 512) == 0, e.value
        scale, px, py, nw, nh = orc.letterbox_fit_f32(src[0], src[1], 224, 224)
        assert (m[0], int(m[1]), int(m[2]), int(m[3]), int(m[4])) == (scale, px, py, nw, nh)
    assert harness.h_letterbox_fit(180, 1280, 224, 224, m, e, 512) == 0 and int(m[4]) == 32
    assert orc.letterbox_fit(180, 1280, 224, 224)[4] == 31


def test_nv12_layout_refusals_are_config_errors(harness):
    e = _err()
    # stride narrower than the width: refused before any pointer is looked at
    rc = harness.h_nv12_letterbox_into(None, 64, 96, 80, 80 * 64, None, 32, 32, 1, PAD, _map(), None, e, 512)
    assert rc == 1 and b"is narrower than the width" in e.value
    rc = harness.h_nv12_crop_resize_into(None, 64, 96, 96, 96 * 10, None, 3, None, 16, 16, 1, None, e, 512)
    assert rc == 1 and b"inside the luma plane" in e.value


def test_empty_calls_are_no_ops(harness):
    e = _err()
    assert harness.h_crop_resize_into(None, 64, 96, None, 0, None, 16, 16, 1, None, e, 512) == 0
    assert harness.h_nv12_crop_resize_into(None, 64, 96, 10, 0, None, 0, None, 16, 16, 1, None, e, 512) == 0
    assert harness.h_mask_area_into(None, 0, 0, 0, None, 0, 0, 0, 0.25, 0.5, 1, 1, None, None, e, 512) == 0


def test_mask_row_refusal_is_a_config_error(harness):
    e = _err()
    rc = harness.h_mask_area_into(None, 300, 6, 6, None, 32, 100, 4, 0.25, 0.5, 256, 128, None, None, e, 512)
    assert rc == 1 and b"stride must exceed the prefix" in e.value


# ---- on the device --------------------------------------------------------------------------


def _stream(torch):
    return ctypes.c_void_p(torch.cuda.current_stream().cuda_stream)


@pytest.mark.gpu
@pytest.mark.parametrize(("src", "dst"), [((1080, 1920), (640, 640)), ((720, 1280), (640, 640)),
                                          ((33, 77), (100, 37)), ((180, 1280), (224, 224))])
@pytest.mark.parametrize("swap_rb", [True, False])
def test_letterbox_into_matches_oracle(cuda, harness, orc, src, dst, swap_rb):
    from _data import frames_u8

    frame = frames_u8(1, src, seed=src[0])[0]
    d_src = cuda.from_numpy(frame).cuda()
    out = cuda.empty((3, *dst), dtype=cuda.float32, device="cuda")
    m, e = _map(), _err()
    rc = harness.h_letterbox_into(d_src.data_ptr(), src[0], src[1], out.data_ptr(), dst[0], dst[1], int(swap_rb), PAD,
                                  m, _stream(cuda), e, 512)
    assert rc == 0, e.value
    cuda.cuda.synchronize()
    want = orc.letterbox([frame], dst, swap_rb=swap_rb, pad_value=114.0, cpp_fit=True)[0]
    assert np.array_equal(out.cpu().numpy().view(np.uint32), want.view(np.uint32))


@pytest.mark.gpu
def test_crop_resize_into_matches_oracle(cuda, harness, orc):
    from _data import crop_boxes, frames_u8

    frame = frames_u8(1, seed=3)[0]
    boxes, _ = crop_boxes(1, 40, seed=5)
    boxes[0] = [10.5, 20.0, 10.5, 400.0]  # zero width: black
    d_src, d_boxes = cuda.from_numpy(frame).cuda(), cuda.from_numpy(boxes).cuda()
    out = cuda.empty((len(boxes), 3, 256, 128), dtype=cuda.float32, device="cuda")
    e = _err()
    rc = harness.h_crop_resize_into(d_src.data_ptr(), 1080, 1920, d_boxes.data_ptr(), len(boxes), out.data_ptr(),
                                    256, 128, 1, _stream(cuda), e, 512)
    assert rc == 0, e.value
    cuda.cuda.synchronize()
    want = orc.crop([frame], boxes, (256, 128), None, (0.0, 0.0, 0.0), (255.0, 255.0, 255.0), True)
    got = out.cpu().numpy()
    assert np.array_equal(got.view(np.uint32), want.view(np.uint32))
    assert not got[0].any()


@pytest.mark.gpu
@pytest.mark.parametrize("swap_rb", [True, False])
def test_nv12_calls_match_oracle(cuda, harness, orc, swap_rb):
    from _data import crop_boxes, nv12_frames

    buf, h, w, pitch, uv = nv12_frames(1, (1080, 1920), seed=9, pitch=2048, coded_h=1088)[0]
    d = cuda.from_numpy(buf).cuda()
    out = cuda.empty((3, 640, 640), dtype=cuda.float32, device="cuda")
    m, e = _map(), _err()
    rc = harness.h_nv12_letterbox_into(d.data_ptr(), h, w, pitch, uv, out.data_ptr(), 640, 640, int(swap_rb), PAD, m,
                                       _stream(cuda), e, 512)
    assert rc == 0, e.value
    boxes, _ = crop_boxes(1, 24, seed=6)
    d_boxes = cuda.from_numpy(boxes).cuda()
    crops = cuda.empty((len(boxes), 3, 256, 128), dtype=cuda.float32, device="cuda")
    rc = harness.h_nv12_crop_resize_into(d.data_ptr(), h, w, pitch, uv, d_boxes.data_ptr(), len(boxes),
                                         crops.data_ptr(), 256, 128, int(swap_rb), _stream(cuda), e, 512)
    assert rc == 0, e.value
    cuda.cuda.synchronize()
    planes = [(buf, h, w, pitch, uv)]
    want = orc.letterbox_nv12(planes, (640, 640), swap_rb=swap_rb, pad_value=114.0, matrix=601, sampling=0,
                              cpp_fit=True)[0]
    assert np.array_equal(out.cpu().numpy().view(np.uint32), want.view(np.uint32))
    want_c = orc.crop_nv12(planes, boxes, (256, 128), None, swap_rb)
    assert np.array_equal(crops.cpu().numpy().view(np.uint32), want_c.view(np.uint32))
    assert (m[0], m[2], m[4]) == (float(np.float32(1 / 3)), 140.0, 360.0)


REF_LIB = ROOT / "oracle" / "_ref" / "libshipref.so"


@pytest.mark.gpu
@pytest.mark.parametrize(("src", "surface"), [((180, 1280), (1280, 184)), ((340, 1280), (1280, 340)),
                                              ((660, 1280), (1344, 672)), ((1080, 1920), (2048, 1088))])
def test_nv12_letterbox_into_places_as_the_reference_kernel(cuda, harness, orc, src, surface):
    """At the sizes where the two placement rules part, the plane's nv12_letterbox_into equals
    the reference's own nv12_letterbox_into (compiled from its ops.cu into oracle/_ref) and the
    oracle with the float32 placement, bit for bit, and returns the same map."""
    from _data import nv12_frames

    if not REF_LIB.exists():
        pytest.skip("oracle/_ref/libshipref.so not built")
    ref = ctypes.CDLL(str(REF_LIB))
    ref.ref_nv12_letterbox.argtypes = [ctypes.c_void_p, ctypes.c_int, ctypes.c_int, ctypes.c_int, ctypes.c_ulonglong,
                                       ctypes.c_void_p, ctypes.c_int, ctypes.c_int, ctypes.c_int, ctypes.c_float,
                                       ctypes.c_void_p, ctypes.c_void_p]
    (buf, h, w, pitch, uv), = nv12_frames(1, src, seed=src[0], pitch=surface[0], coded_h=surface[1])
    d = cuda.from_numpy(buf).cuda()
    mine = cuda.full((3, 224, 224), -1.0, dtype=cuda.float32, device="cuda")
    theirs = cuda.full((3, 224, 224), -2.0, dtype=cuda.float32, device="cuda")
    m, e = _map(), _err()
    rc = harness.h_nv12_letterbox_into(d.data_ptr(), h, w, pitch, uv, mine.data_ptr(), 224, 224, 1, PAD, m,
                                       _stream(cuda), e, 512)
    assert rc == 0, e.value
    ref_map = (ctypes.c_int * 4)()
    assert ref.ref_nv12_letterbox(d.data_ptr(), h, w, pitch, uv, theirs.data_ptr(), 224, 224, 1, PAD,
                                  ctypes.c_void_p(cuda.cuda.current_stream().cuda_stream), ref_map) == 0
    cuda.cuda.synchronize()
    assert (int(m[1]), int(m[2]), int(m[3]), int(m[4])) == tuple(ref_map)
    assert np.array_equal(mine.cpu().numpy().view(np.uint32), theirs.cpu().numpy().view(np.uint32))
    want = orc.letterbox_nv12([(buf, h, w, pitch, uv)], (224, 224), pad_value=114.0, matrix=601, sampling=0,
                              cpp_fit=True)[0]
    assert np.array_equal(mine.cpu().numpy().view(np.uint32), want.view(np.uint32))


@pytest.mark.gpu
def test_mask_area_into_matches_oracle(cuda, harness, orc):
    rng = np.random.default_rng(12)
    rows = rng.standard_normal((6, 300, 38)).astype(np.float32)
    rows[:, :, 4] = rng.uniform(0.0, 1.0, (6, 300))
    rows[2, :, 4] = 0.1  # below the score threshold: area 0
    protos = rng.standard_normal((6, 32, 160, 160)).astype(np.float32)
    d_rows, d_protos = cuda.from_numpy(rows).cuda(), cuda.from_numpy(protos).cuda()
    areas = cuda.empty((6,), dtype=cuda.float32, device="cuda")
    e = _err()
    rc = harness.h_mask_area_into(d_rows.data_ptr(), 300, 38, 6, d_protos.data_ptr(), 32, 160 * 160, 6, 0.25, 0.5,
                                  256, 128, areas.data_ptr(), _stream(cuda), e, 512)
    assert rc == 0, e.value
    cuda.cuda.synchronize()
    want = orc.mask_area(rows, protos, prefix=6, score_threshold=0.25, mask_threshold=0.5, crop_hw=(256, 128))
    assert np.array_equal(areas.cpu().numpy().view(np.uint32), np.asarray(want, np.float32).view(np.uint32))
    assert areas[2].item() == 0.0


# ---- crops for a batch of frames (crop_batch.cpp) ---------------------------------------------

ANY, NONE = -1, -2  # CropSpec::kAnyClass, CropSpec::kNoClass


def _arr(ctype, values):
    return (ctype * max(len(values), 1))(*values)


def _batched(harness, frames, sets, *, select_only, stream=None):
    """frames: dicts with bgr / nv12 (device pointer or None), h, w, stride, uv, dets (list of
    (x1, y1, x2, y2, class, index)); sets: (class_id, h, w, dst pointer or None)."""
    dets = [d for fr in frames for d in fr["dets"]]
    total = sum(len(fr["dets"]) for fr in frames) * len(sets) + 1
    rows, fo, oi, launches, e = _arr(ctypes.c_int, [0] * len(sets)), (ctypes.c_int * total)(), \
        (ctypes.c_int * total)(), ctypes.c_int(0), _err()
    rc = harness.h_batched_crop(
        len(frames), _arr(ctypes.c_void_p, [fr.get("bgr") for fr in frames]),
        _arr(ctypes.c_void_p, [fr.get("nv12") for fr in frames]), _arr(ctypes.c_int, [fr["h"] for fr in frames]),
        _arr(ctypes.c_int, [fr["w"] for fr in frames]), _arr(ctypes.c_int, [fr.get("stride", 0) for fr in frames]),
        _arr(ctypes.c_ulonglong, [fr.get("uv", 0) for fr in frames]),
        _arr(ctypes.c_int, [len(fr["dets"]) for fr in frames]),
        _arr(ctypes.c_float, [v for d in dets for v in d[:4]]), _arr(ctypes.c_int, [d[4] for d in dets]),
        _arr(ctypes.c_int, [d[5] for d in dets]), len(sets), _arr(ctypes.c_int, [s[0] for s in sets]),
        _arr(ctypes.c_int, [s[1] for s in sets]), _arr(ctypes.c_int, [s[2] for s in sets]),
        _arr(ctypes.c_void_p, [s[3] for s in sets]), int(select_only), 0, stream, rows, fo, oi,
        ctypes.byref(launches), e, 512)
    assert rc == 0, e.value
    out, k = [], 0
    for s_i in range(len(sets)):
        n = rows[s_i]
        out.append((list(fo[k:k + n]), list(oi[k:k + n])))
        k += n
    return out, launches.value


def test_batched_crop_selects_rows_as_crop_stage(harness):
    """Per set, a row per detection of the set's class (every row for kAnyClass, none for
    kNoClass); BGR frames' rows first, then NV12 frames', each frame's in detection order."""
    fake = 0x1000  # a pointer the selection never dereferences
    frames = [
        {"bgr": fake, "h": 1080, "w": 1920, "dets": [(0, 0, 9, 9, 1, 0), (1, 1, 8, 8, 0, 1), (2, 2, 7, 7, 1, 2)]},
        {"nv12": fake, "h": 1080, "w": 1920, "stride": 2048, "uv": 2048 * 1088,
         "dets": [(0, 0, 5, 5, 0, 0), (3, 3, 9, 9, 1, 1)]},
        {"bgr": fake, "h": 720, "w": 1280, "dets": []},
        {"bgr": fake, "h": 720, "w": 1280, "dets": [(4, 4, 9, 9, 1, 7)]},
    ]
    (c1, any_, none), launches = _batched(harness, frames, [(1, 32, 32, None), (ANY, 16, 16, None),
                                                            (NONE, 8, 8, None)], select_only=True)
    assert c1 == ([0, 0, 3, 1], [0, 2, 7, 1])
    assert any_ == ([0, 0, 0, 3, 1, 1], [0, 1, 2, 7, 0, 1])
    assert none == ([], []) and launches == 0


def test_batched_crop_refuses_a_frame_with_two_representations(harness):
    fake = 0x1000
    rows, fo, oi, launches, e = (ctypes.c_int * 1)(), (ctypes.c_int * 1)(), (ctypes.c_int * 1)(), ctypes.c_int(0), \
        _err()
    rc = harness.h_batched_crop(1, _arr(ctypes.c_void_p, [fake]), _arr(ctypes.c_void_p, [fake]),
                                _arr(ctypes.c_int, [10]), _arr(ctypes.c_int, [10]), _arr(ctypes.c_int, [10]),
                                _arr(ctypes.c_ulonglong, [100]), _arr(ctypes.c_int, [0]), _arr(ctypes.c_float, []),
                                _arr(ctypes.c_int, []), _arr(ctypes.c_int, []), 1, _arr(ctypes.c_int, [ANY]),
                                _arr(ctypes.c_int, [8]), _arr(ctypes.c_int, [8]), None, 1, 0, None, rows, fo, oi,
                                ctypes.byref(launches), e, 512)
    assert rc == 1 and b"exactly one of" in e.value


@pytest.mark.gpu
def test_batched_crop_equals_the_per_frame_calls(cuda, harness, orc):
    """Six frames (four BGR, two NV12 surfaces) with class 0/1 detections and three crop sets:
    one upload, one launch per set and representation, one synchronise — and every row equal, bit
    for bit, to the reference-shaped per-frame call (crop_resize_into / nv12_crop_resize_into) and
    to the oracle."""
    from _data import crop_boxes, frames_u8, nv12_frames

    rng = np.random.default_rng(21)
    bgr_host = frames_u8(4, (1080, 1920), seed=31)
    nv12_host = nv12_frames(2, (1080, 1920), seed=32, pitch=2048, coded_h=1088)
    keep = []
    frames = []
    for k in range(6):
        boxes, _ = crop_boxes(1, 12 + 3 * k, seed=40 + k)
        if k == 2:
            boxes[0] = [50.0, 60.0, 50.0, 300.0]  # zero width: a black crop
        classes = rng.integers(0, 2, len(boxes))
        dets = [(*map(float, b), int(c), 10 * k + j) for j, (b, c) in enumerate(zip(boxes, classes))]
        if k < 4:
            d = cuda.from_numpy(bgr_host[k]).cuda()
            frames.append({"bgr": d.data_ptr(), "h": 1080, "w": 1920, "dets": dets})
        else:
            buf, h, w, pitch, uv = nv12_host[k - 4]
            d = cuda.from_numpy(buf).cuda()
            frames.append({"nv12": d.data_ptr(), "h": h, "w": w, "stride": pitch, "uv": uv, "dets": dets})
        keep.append(d)
    sizes = [(0, 256, 128), (ANY, 64, 48), (NONE, 32, 32)]
    totals = [sum(1 for fr in frames for d in fr["dets"] if c == ANY or d[4] == c) for c, _, _ in sizes]
    dsts = [cuda.full((max(n, 1), 3, h, w), -7.0, dtype=cuda.float32, device="cuda")
            for n, (_, h, w) in zip(totals, sizes)]
    sets = [(c, h, w, t.data_ptr()) for (c, h, w), t in zip(sizes, dsts)]
    stream = cuda.cuda.Stream()
    out, launches = _batched(harness, frames, sets, select_only=False, stream=ctypes.c_void_p(stream.cuda_stream))
    assert launches == 4  # two non-empty sets x (BGR, NV12)
    for (c, h, w), (fo, oi), dst, n in zip(sizes, out, dsts, totals):
        assert len(fo) == n
        got = dst.cpu().numpy()[:n]
        for f in range(6):
            rows = [r for r in range(n) if fo[r] == f]
            if not rows:
                continue
            assert rows == list(range(rows[0], rows[-1] + 1))  # a frame's rows are contiguous
            sel = [d for d in frames[f]["dets"] if c == ANY or d[4] == c]
            assert [d[5] for d in sel] == [oi[r] for r in rows]
            bx = np.array([d[:4] for d in sel], np.float32)
            d_boxes = cuda.from_numpy(bx).cuda()
            one = cuda.empty((len(sel), 3, h, w), dtype=cuda.float32, device="cuda")
            e = _err()
            fr = frames[f]
            if "bgr" in fr:
                rc = harness.h_crop_resize_into(fr["bgr"], 1080, 1920, d_boxes.data_ptr(), len(sel), one.data_ptr(),
                                                h, w, 1, _stream(cuda), e, 512)
                want = orc.crop([bgr_host[f]], bx, (h, w), None, (0.0, 0.0, 0.0), (255.0, 255.0, 255.0), True)
            else:
                rc = harness.h_nv12_crop_resize_into(fr["nv12"], fr["h"], fr["w"], fr["stride"], fr["uv"],
                                                     d_boxes.data_ptr(), len(sel), one.data_ptr(), h, w, 1,
                                                     _stream(cuda), e, 512)
                want = orc.crop_nv12([nv12_host[f - 4]], bx, (h, w), None, True)
            assert rc == 0, e.value
            cuda.cuda.synchronize()
            mine = got[rows[0]:rows[-1] + 1]
            assert np.array_equal(mine.view(np.uint32), one.cpu().numpy().view(np.uint32)), (c, f)
            assert np.array_equal(mine.view(np.uint32), want.view(np.uint32)), (c, f)
    assert totals[2] == 0 and out[2] == ([], [])

