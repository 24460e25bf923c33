"""Device NMS, through the C ABI, against the oracle (NumpyImageOps.nms semantics).

Bar: kept indices bit-exact (same indices, same order, same counts).
"""

from __future__ import annotations

import numpy as np
import pytest

from _data import nms_heads

pytestmark = pytest.mark.gpu


def device_nms(torch, ops, boxes, scores, classes, iou, score, max_det, num_classes=1, class_aware=None):
    b = torch.from_numpy(np.ascontiguousarray(boxes, np.float32)).cuda()
    s = torch.from_numpy(np.ascontiguousarray(scores, np.float32)).cuda()
    c = None if classes is None else torch.from_numpy(np.ascontiguousarray(classes, np.int32)).cuda()
    keep, counts = ops.nms_device(b, s, c, iou_threshold=iou, score_threshold=score, max_det=max_det,
                                  num_classes=num_classes, class_aware=class_aware)
    torch.cuda.synchronize()
    return keep.cpu().numpy(), counts.cpu().numpy()


KA_BOXES = np.array(
    [[10, 10, 100, 100], [15, 15, 105, 105], [300, 300, 400, 400], [305, 305, 405, 405], [500, 500, 520, 520]],
    dtype=np.float32,
)
KA_SCORES = np.array([0.90, 0.80, 0.95, 0.70, 0.60], dtype=np.float32)


def test_known_answer(cuda, ops):
    """The reference's known answers, tests/runtime/test_ops_parity.py:128-164."""
    assert ops.nms(KA_BOXES, KA_SCORES, 0.5, 0.1, 10).tolist() == [2, 0, 4]
    assert ops.nms(KA_BOXES, KA_SCORES, 0.5, 0.85, 10).tolist() == [2, 0]
    assert ops.nms(KA_BOXES, KA_SCORES, 0.5, 0.0, 1).tolist() == [2]
    assert ops.nms(np.empty((0, 4), np.float32), np.empty(0, np.float32), 0.5, 0.1, 10).size == 0


def test_random_fleets_match_oracle(cuda, ops, orc):
    """100 random fleets with ties (test_ops_vs_shipvision.py:169-190's generator, plus ties)."""
    rng = np.random.default_rng(7)
    for trial in range(100):
        count = int(rng.integers(1, 200))
        corner = rng.random((count, 2)).astype(np.float32) * 100
        extent = rng.random((count, 2)).astype(np.float32) * 40 + 1
        boxes = np.concatenate([corner, corner + extent], axis=1).astype(np.float32)
        scores = rng.random(count).astype(np.float32)
        scores[rng.integers(0, count, count // 4)] = scores[0]
        iou, floor = float(rng.choice([0.3, 0.45, 0.5, 0.7])), float(rng.choice([0.0, 0.1, 0.25]))
        max_out = int(rng.integers(1, count + 5))
        want = orc.nms(boxes, scores, iou, floor, max_out)
        got = ops.nms(boxes, scores, iou, floor, max_out)
        assert got.tolist() == want.tolist(), f"trial {trial}"


def test_config2_class_aware_bit_exact(cuda, ops, orc):
    """Config 2: 16 x 8400 candidates, 2 classes, score 0.25, IoU 0.45, max_det 300."""
    boxes, scores, classes = nms_heads(16, 8400, 2, seed=0)
    want_keep, want_counts = orc.nms_batched(boxes, scores, classes, 0.45, 0.25, 300, num_classes=2)
    keep, counts = device_nms(cuda, ops, boxes, scores, classes, 0.45, 0.25, 300, num_classes=2)
    assert counts.tolist() == want_counts.tolist()
    assert np.array_equal(keep, want_keep)
    assert (counts == 300).all()


def test_class_agnostic_batched(cuda, ops, orc):
    boxes, scores, _ = nms_heads(4, 8400, 1, seed=1)
    want_keep, want_counts = orc.nms_batched(boxes, scores, None, 0.5, 0.25, 300, class_aware=False)
    keep, counts = device_nms(cuda, ops, boxes, scores, None, 0.5, 0.25, 300, class_aware=False)
    assert counts.tolist() == want_counts.tolist() and np.array_equal(keep, want_keep)


def test_segment_larger_than_one_sort_chunk(cuda, ops, orc):
    """25 000 candidates (the reference benchmark's count) and a low threshold: the segment is
    sorted in radix-selected chunks, and dense overlap forces the walk past the first one."""
    rng = np.random.default_rng(5)
    n = 25000
    c = rng.uniform(0, 200, (n, 2))
    wh = rng.uniform(20, 60, (n, 2))
    boxes = np.concatenate([c - wh / 2, c + wh / 2], 1).astype(np.float32)[None]
    scores = rng.random(n).astype(np.float32)[None]
    for iou, max_det in [(0.05, 4096), (0.45, 300)]:
        want_keep, want_counts = orc.nms_batched(boxes, scores, None, iou, 0.0, max_det, class_aware=False)
        keep, counts = device_nms(cuda, ops, boxes, scores, None, iou, 0.0, max_det, class_aware=False)
        assert counts.tolist() == want_counts.tolist() and np.array_equal(keep, want_keep)


def test_many_classes_and_out_of_range_ids(cuda, ops, orc):
    boxes, scores, _ = nms_heads(3, 3000, 1, seed=2)
    rng = np.random.default_rng(9)
    classes = rng.integers(-2, 83, (3, 3000)).astype(np.int32)  # ids outside [0, 80) are ignored
    want_keep, want_counts = orc.nms_batched(boxes, scores, classes, 0.45, 0.1, 300, num_classes=80)
    keep, counts = device_nms(cuda, ops, boxes, scores, classes, 0.45, 0.1, 300, num_classes=80)
    assert counts.tolist() == want_counts.tolist() and np.array_equal(keep, want_keep)


def test_edge_cases(cuda, ops, orc):
    boxes, scores, classes = nms_heads(2, 500, 2, seed=4)
    # ties everywhere, -0.0 and +0.0 scores, max_det above the candidate count
    scores = np.round(scores * 4) / 4
    scores[:, :5] = -0.0
    scores[:, 5:10] = 0.0
    for max_det in (0, 1, 7, 1000):
        want = orc.nms_batched(boxes, scores.astype(np.float32), classes, 0.45, 0.0, max_det, num_classes=2)
        got = device_nms(cuda, ops, boxes, scores, classes, 0.45, 0.0, max_det, num_classes=2)
        assert got[1].tolist() == want[1].tolist() and np.array_equal(got[0], want[0]), max_det
    # no candidate passes the threshold
    keep, counts = device_nms(cuda, ops, boxes, scores, classes, 0.45, 2.0, 300, num_classes=2)
    assert counts.tolist() == [0, 0] and (keep == -1).all()


def test_non_finite_boxes_follow_numpy(cuda, ops, orc):
    rng = np.random.default_rng(12)
    boxes, scores, _ = nms_heads(1, 400, 1, seed=6)
    boxes[0, rng.integers(0, 400, 10), rng.integers(0, 4, 10)] = np.nan
    boxes[0, rng.integers(0, 400, 5), 2] = np.inf
    scores[0, rng.integers(0, 400, 5)] = np.nan
    want = orc.nms_batched(boxes, scores, None, 0.45, 0.1, 300, class_aware=False)
    got = device_nms(cuda, ops, boxes, scores, None, 0.45, 0.1, 300, class_aware=False)
    assert got[1].tolist() == want[1].tolist() and np.array_equal(got[0], want[0])


def test_host_batched_entry(cuda, ops, orc):
    boxes, scores, classes = nms_heads(2, 2000, 3, seed=8)
    keep, counts = ops.nms_batched(boxes, scores, classes, 0.5, 0.2, 100, num_classes=3)
    want_keep, want_counts = orc.nms_batched(boxes, scores, classes, 0.5, 0.2, 100, num_classes=3)
    assert counts.tolist() == want_counts.tolist() and np.array_equal(keep, want_keep)


def _near_threshold_pairs(thr: float, count: int, seed: int) -> np.ndarray:
    """Two-box images whose float32 IoU is RN(w / W) for integers W in [2^22, 2^24) and
    w = floor(thr * W) + d, d in [-4, 4]: boxes [x0, y0, x0+W, y0+1] and [x0, y0, x0+w, y0+1]
    intersect in exactly w and unite in exactly W, so every IoU lies a few ulps from thr, on
    both sides of it."""
    rng = np.random.default_rng(seed)
    W = rng.integers(1 << 22, 1 << 24, count).astype(np.int64)
    d = rng.integers(-4, 5, count)
    w = (np.floor(np.float64(np.float32(thr)) * W).astype(np.int64) + d).clip(1, None)
    x0 = rng.integers(0, 64, count)
    y0 = rng.integers(0, 64, count)
    a = np.stack([x0, y0, x0 + W, y0 + 1], axis=1)
    b = np.stack([x0, y0, x0 + w, y0 + 1], axis=1)
    return np.stack([a, b], axis=1).astype(np.float32)  # every coordinate is an exact float


@pytest.mark.parametrize("thr", [0.45, 0.5, 0.3, 0.7, 0.25])
def test_iou_threshold_boundaries(cuda, ops, orc, thr):
    """Pairs whose IoU rounds to the threshold or to its neighbours: the kernel's division-free
    survivor test must decide every one as numpy's float32 division does."""
    pairs = _near_threshold_pairs(thr, 4096, seed=int(thr * 1000))
    n = len(pairs)
    boxes = pairs.reshape(n, 2, 4)
    scores = np.tile(np.array([0.9, 0.8], np.float32), (n, 1))
    want = orc.nms_batched(boxes, scores, None, thr, 0.1, 2, class_aware=False)
    got = device_nms(cuda, ops, boxes, scores, None, thr, 0.1, 2, class_aware=False)
    assert got[1].tolist() == want[1].tolist() and np.array_equal(got[0], want[0])
    # the set holds both outcomes
    assert 0 < int((want[1] == 1).sum()) < n


@pytest.mark.parametrize(("num_classes", "max_det"), [(2, 300), (8, 300), (8, 1024), (9, 300), (2, 4096), (3, 4096)],
                         ids=["2x300-cluster", "8x300-cluster", "8x1024-cluster", "9x300-counter",
                              "2x4096-cluster", "3x4096-counter"])
def test_class_merge_paths_twice_in_a_row(cuda, ops, orc, num_classes, max_det):
    """Both ways the classes of an image meet: one thread-block cluster (2..8 classes with
    classes x max_det <= 8192) or the workspace's arrival counters (more classes, or more
    survivors); each twice in a row on the instance's cached workspace, against the oracle."""
    boxes, scores, classes = nms_heads(6, 4000, num_classes, seed=20 + num_classes)
    want_keep, want_counts = orc.nms_batched(boxes, scores, classes, 0.45, 0.05, max_det, num_classes=num_classes)
    for _ in range(2):
        keep, counts = device_nms(cuda, ops, boxes, scores, classes, 0.45, 0.05, max_det, num_classes=num_classes)
        assert counts.tolist() == want_counts.tolist()
        assert np.array_equal(keep, want_keep)


@pytest.mark.parametrize("kind", ["signs", "all-equal", "few-values", "narrow"])
def test_radix_select_key_spreads(cuda, ops, orc, kind):
    """More candidates than one sorted round (512), with key sets whose highest differing bit
    sits anywhere: scores of both signs (the sign bit), one score for all (only the index bits
    differ), a few distinct values, and a narrow band of nearby floats. The radix selects start
    below the bits every key shares."""
    rng = np.random.default_rng({"signs": 1, "all-equal": 2, "few-values": 3, "narrow": 4}[kind])
    n = 6000
    boxes, _, _ = nms_heads(2, n, 1, seed=31)
    if kind == "signs":
        scores = rng.uniform(-1.0, 1.0, (2, n)).astype(np.float32)
        scores[:, :7] = -0.0
        scores[:, 7:13] = 0.0
    elif kind == "all-equal":
        scores = np.full((2, n), 0.75, np.float32)
    elif kind == "few-values":
        scores = rng.choice(np.array([-0.5, 0.0, 0.25, 0.5, 0.9], np.float32), (2, n))
    else:
        scores = (np.float32(0.6) + rng.integers(0, 4096, (2, n)) * np.float32(2.0 ** -30)).astype(np.float32)
    for max_det, iou in [(300, 0.45), (1000, 0.45), (600, 0.1)]:
        want = orc.nms_batched(boxes, scores, None, iou, -2.0, max_det, class_aware=False)
        got = device_nms(cuda, ops, boxes, scores, None, iou, -2.0, max_det, class_aware=False)
        assert got[1].tolist() == want[1].tolist() and np.array_equal(got[0], want[0]), (kind, max_det, iou)


def test_launch_shape(cuda, ops, orc):
    """shipk_nms_launch_shape reports the launch shipk_nms makes: a CTA per segment, times the
    helper CTAs that share a first round's pair tests, in clusters that hold an image's classes
    (up to 8 classes) or one segment; and the results with that shape are the oracle's."""
    import ctypes

    from shipinfer_b200 import _native

    lib = _native.lib()
    ctas, cluster = ctypes.c_int(), ctypes.c_int()

    def shape(*a):
        _native.check(lib.shipk_nms_launch_shape(*a, ctypes.byref(ctas), ctypes.byref(cluster)))
        return ctas.value, cluster.value

    c, k = shape(16, 8400, 2, 1, 300)  # config 2: two classes merge in one cluster
    split = c // 32
    assert c == 32 * split and 1 <= split <= 4 and k == 2 * split
    c, k = shape(4, 8400, 1, 0, 300)  # class-agnostic: a cluster per segment
    assert c % 4 == 0 and k == c // 4 and 1 <= k <= 8
    c, k = shape(3, 3000, 80, 1, 300)  # 240 segments: no room for helpers, arrival-counter merge
    assert (c, k) == (240, 1)
    c, k = shape(2, 8400, 2, 1, 4096)  # no block resolve at this max_det: the class cluster only
    assert (c, k) == (4, 2)
    for b in (1, 2, 5, 16, 37):
        c, k = shape(b, 4000, 2, 1, 300)
        assert c % (2 * b) == 0 and k == 2 * (c // (2 * b)) and c <= max(2 * b, 148)
        boxes, scores, classes = nms_heads(b, 4000, 2, seed=40 + b)
        want = orc.nms_batched(boxes, scores, classes, 0.45, 0.25, 300, num_classes=2)
        got = device_nms(cuda, ops, boxes, scores, classes, 0.45, 0.25, 300, num_classes=2)
        assert got[1].tolist() == want[1].tolist() and np.array_equal(got[0], want[0]), b


@pytest.mark.parametrize(("iou", "max_det"), [(0.45, 300), (0.45, 1000), (0.7, 300), (0.3, 4096), (0.45, 50)])
def test_dense_pools_with_kept_box_filter(cuda, ops, orc, iou, max_det):
    """The reference kernel benchmark's 25 000 boxes (benchmarks/kernels.py:298-320), which all
    share one point: few boxes survive, so the kernel visits every eligible candidate, over
    several shared-memory pools, and drops from each pool what the boxes kept so far remove.
    Class-agnostic (one segment and its helpers) and class-aware over two classes."""
    from _data import kernels_bench_inputs

    _, _, b, s = kernels_bench_inputs(0)
    boxes, scores = b[None], s[None]
    want = orc.nms_batched(boxes, scores, None, iou, 0.25, max_det, class_aware=False)
    got = device_nms(cuda, ops, boxes, scores, None, iou, 0.25, max_det, class_aware=False)
    assert got[1].tolist() == want[1].tolist() and np.array_equal(got[0], want[0])
    classes = (np.arange(b.shape[0]) % 2).astype(np.int32)[None]
    want = orc.nms_batched(boxes, scores, classes, iou, 0.25, max_det, num_classes=2)
    got = device_nms(cuda, ops, boxes, scores, classes, iou, 0.25, max_det, num_classes=2)
    assert got[1].tolist() == want[1].tolist() and np.array_equal(got[0], want[0])


def test_replicas_with_an_empty_image_and_non_finite_boxes(cuda, ops, orc):
    """Class-agnostic batches run each image on a cluster of replicas (the leader and helpers
    taking the same steps). One image with no eligible candidate (its replicas only pass the
    block's barriers at the end), dense images whose pools are filtered across the replicas,
    and boxes with NaN or infinite coordinates among them (the filter's general survivor test)."""
    from _data import kernels_bench_inputs

    _, _, b, s = kernels_bench_inputs(3)
    rng = np.random.default_rng(17)
    n = 8000
    boxes = np.stack([b[:n], b[n:2 * n], b[2 * n:3 * n]]).astype(np.float32)
    scores = np.stack([s[:n], s[n:2 * n], s[2 * n:3 * n]]).astype(np.float32)
    scores[1] = 0.1  # nothing reaches the threshold in image 1
    bad = rng.integers(0, n, 40)
    boxes[2, bad[:20], rng.integers(0, 4, 20)] = np.nan
    boxes[2, bad[20:], 2] = np.inf
    for iou, max_det in [(0.45, 300), (0.3, 100)]:
        want = orc.nms_batched(boxes, scores, None, iou, 0.25, max_det, class_aware=False)
        got = device_nms(cuda, ops, boxes, scores, None, iou, 0.25, max_det, class_aware=False)
        assert got[1].tolist() == want[1].tolist() and np.array_equal(got[0], want[0]), (iou, max_det)
        assert want[1][1] == 0
