"""GPU parity of the YOLOv8 Detect tail and the detection post-processing
against the CPU oracle (through the C ABI): the tail's f32 output bit-identical,
the detections identical in value and order (decode + class-aware / agnostic
NMS + the reference's swap_remove order), the reference's own KATs run through
the device API, and the edge cases (no candidate, every anchor a candidate,
ties, one class, NaN scores, zero-area boxes, the anchor limit)."""
import json
import os

import numpy as np
import pytest

import dragonwing_edge_rs_b200 as dw
from dragonwing_edge_rs_b200 import ops
from dragonwing_edge_rs_b200.backend import BackendError
from oracle import dwref

pytestmark = pytest.mark.gpu

KATS = json.load(open(os.path.join(os.path.dirname(__file__), "golden", "reference_kats.json")))
V8_GRIDS = [(80, 80), (40, 40), (20, 20)]
V8_STRIDES = [8.0, 16.0, 32.0]


@pytest.fixture(scope="module")
def be():
    b = dw.CudaBackend(0)
    yield b
    b.close()


def run_detect(be, boxes, clss, strides, bs, cs):
    n, nc = boxes[0].shape[0], clss[0].shape[3]
    desc = ops.YoloDetectDesc(n, nc, [b.shape[1:3] for b in boxes], strides, bs, cs)
    tables = ops.prepare_yolo_detect(be, desc)
    db = [be.upload_array(b) for b in boxes]
    dc = [be.upload_array(c) for c in clss]
    out = be.alloc(n * (4 + nc) * desc.anchors * 4)
    ops.yolo_detect_i8(be, desc, tables, db, dc, out)
    res = be.download_array(out, np.float32, (n, 4 + nc, desc.anchors))
    for b in db + dc + [out, tables]:
        b.free()
    return res


@pytest.mark.parametrize("n,nc,grids,seed", [
    (2, 80, V8_GRIDS, 1),                        # the YOLOv8n head at 640x640
    (1, 5, [(7, 9)], 2),                         # one level, nc not a multiple of 16 (byte loads)
    (3, 16, [(13, 11), (7, 6), (4, 3), (2, 2)], 3),  # four levels
])
def test_detect_tail_bit_exact(be, n, nc, grids, seed):
    rng = np.random.default_rng(seed)
    boxes = [rng.integers(-128, 128, (n, h, w, 64), dtype=np.int8) for h, w in grids]
    clss = [rng.integers(-128, 128, (n, h, w, nc), dtype=np.int8) for h, w in grids]
    strides = [8.0 * 2 ** i for i in range(len(grids))]
    bs = [float(np.float32(rng.uniform(0.01, 0.1))) for _ in grids]
    cs = [float(np.float32(rng.uniform(0.01, 0.1))) for _ in grids]
    got = run_detect(be, boxes, clss, strides, bs, cs)
    ref = dwref.yolo_detect_i8(boxes, clss, strides, bs, cs)
    assert np.array_equal(got, ref)


def test_detect_tail_extreme_levels(be):
    """Saturated and constant bins (softmax of equal terms, of one dominant
    term) and the class-score extremes."""
    n, nc = 1, 16
    grids = [(4, 4)]
    boxes = np.zeros((n, 4, 4, 64), np.int8)
    boxes[0, 0, 0] = 127
    boxes[0, 0, 1] = -128
    boxes[0, 1, 0, ::16] = 127
    boxes[0, 1, 0, 1::16] = -128
    boxes[0, 2] = np.arange(64, dtype=np.int64).astype(np.int8)
    clss = np.tile(np.array([-128, 127, 0, -1, 1, 64, -64, 100, -100, 5, 6, 7, 8, 9, 10, 11], np.int8),
                   (n, 4, 4, 1))
    for bs in (1.0, 0.5, 1e-3):
        got = run_detect(be, [boxes], [clss], [8.0], [bs], [0.25])
        ref = dwref.yolo_detect_i8([boxes], [clss], [8.0], [bs], [0.25])
        assert np.array_equal(got, ref)


def random_raw(rng, n, nc, A, grid=16, conf_levels=40):
    raw = np.zeros((n, 4 + nc, A), np.float32)
    raw[:, 0] = rng.integers(0, grid, (n, A)) * (640 / grid) + rng.normal(0, 8, (n, A))
    raw[:, 1] = rng.integers(0, grid, (n, A)) * (640 / grid) + rng.normal(0, 8, (n, A))
    raw[:, 2] = rng.uniform(10, 200, (n, A))
    raw[:, 3] = rng.uniform(10, 200, (n, A))
    raw[:, 4:] = rng.integers(0, conf_levels, (n, nc, A)) / conf_levels
    return raw


def run_post(be, raw, nc, A, iw, ih, thr, iou, flags=0):
    n = raw.shape[0]
    d_raw = be.upload_array(np.ascontiguousarray(raw, np.float32))
    try:
        return ops.postprocess_yolo(be, d_raw, n, nc, A, iw, ih, thr, iou, flags)
    finally:
        d_raw.free()


def assert_same_detections(got, raw, nc, A, iw, ih, thr, iou, flags=0):
    for i in range(raw.shape[0]):
        ref = dwref.postprocess_yolo(raw[i], nc, A, iw, ih, thr, iou, flags)
        assert len(got[i]) == len(ref), (i, len(got[i]), len(ref))
        assert np.array_equal(got[i]["bbox"], ref["bbox"])
        assert np.array_equal(got[i]["class_id"], ref["class_id"])
        assert np.array_equal(got[i]["confidence"], ref["confidence"])


@pytest.mark.parametrize("flags", [0, dw.ops.YOLO_ANCHOR_ROWS, dw.ops.YOLO_NMS_AGNOSTIC, dw.ops.YOLO_NO_NMS])
def test_postprocess_matches_oracle(be, flags):
    rng = np.random.default_rng(11 + flags)
    n, nc, A = 3, 80, 8400
    raw = random_raw(rng, n, nc, A)
    if flags & dw.ops.YOLO_ANCHOR_ROWS:
        raw = np.ascontiguousarray(raw.transpose(0, 2, 1))
    thr = 0.9 if flags & dw.ops.YOLO_NMS_AGNOSTIC else 0.5
    got = run_post(be, raw, nc, A, 1280, 720, thr, 0.45, flags)
    assert_same_detections(got, raw, nc, A, 1280, 720, thr, 0.45, flags)
    assert sum(len(g) for g in got) > 0


@pytest.mark.parametrize("A,nc,thr,seed", [
    (1, 3, 0.0, 1), (2, 1, 0.0, 2), (31, 2, 0.1, 3), (257, 7, 0.2, 4), (1000, 1, 0.0, 5),  # one class: one segment
    (4097, 80, 0.0, 6), (16384, 80, 0.5, 7),                                             # every anchor / the limit
])
def test_postprocess_sizes_and_thresholds(be, A, nc, thr, seed):
    rng = np.random.default_rng(seed)
    raw = random_raw(rng, 2, nc, A, grid=4)
    got = run_post(be, raw, nc, A, 640, 640, thr, 0.5)
    assert_same_detections(got, raw, nc, A, 640, 640, thr, 0.5)


def test_postprocess_no_candidates_and_nan_scores(be):
    rng = np.random.default_rng(21)
    raw = random_raw(rng, 2, 10, 500)
    got = run_post(be, raw, 10, 500, 640, 480, 2.0, 0.5)
    assert all(len(g) == 0 for g in got)
    raw[0, 4:, ::3] = np.nan          # NaN never wins the strict '>' (class 0 / next best)
    raw[1, 2:4, ::5] = 0.0            # zero-area boxes: union 0 -> IoU 0
    raw[1, 4:, ::7] = 1.0             # ties at the top confidence: anchor order
    got = run_post(be, raw, 10, 500, 640, 480, 0.2, 0.3)
    assert_same_detections(got, raw, 10, 500, 640, 480, 0.2, 0.3)


def test_postprocess_reference_kats_through_device(be):
    """nms_basic and nms_different_classes (postprocess.rs:369-395) fed through
    decode: 640x640 image (scale 1), boxes given as centre/size."""
    def raw_for(dets, nc):
        A = len(dets)
        raw = np.zeros((1, 4 + nc, A), np.float32)
        for a, (b, c, f) in enumerate(dets):
            raw[0, 0, a], raw[0, 1, a] = (b[0] + b[2]) / 2, (b[1] + b[3]) / 2
            raw[0, 2, a], raw[0, 3, a] = b[2] - b[0], b[3] - b[1]
            raw[0, 4 + c, a] = f
        return raw
    k = KATS["nms_basic"]
    raw = raw_for(k["dets"], 1)
    got = run_post(be, raw, 1, 3, 640, 640, 0.25, k["iou_threshold"])[0]
    assert len(got) == k["expected_len"]
    assert abs(got[0]["confidence"] - k["expected_first_confidence"]) < k["tolerance"]
    assert np.array_equal(got["bbox"][0], np.array(k["dets"][0][0], np.float32))
    k = KATS["nms_different_classes"]
    raw = raw_for(k["dets"], 2)
    got = run_post(be, raw, 2, 2, 640, 640, 0.25, k["iou_threshold"])[0]
    assert len(got) == k["expected_len"]


def test_postprocess_on_detect_output(be):
    """The tail's output straight into the post-processing (the graph's path)."""
    rng = np.random.default_rng(31)
    n, nc = 2, 80
    boxes = [rng.integers(-128, 128, (n, h, w, 64), dtype=np.int8) for h, w in V8_GRIDS]
    clss = [rng.integers(-128, 60, (n, h, w, nc), dtype=np.int8) for h, w in V8_GRIDS]
    raw = run_detect(be, boxes, clss, V8_STRIDES, [0.05, 0.06, 0.07], [0.04, 0.05, 0.06])
    got = run_post(be, raw, nc, 8400, 640, 640, 0.25, 0.45)
    assert_same_detections(got, raw, nc, 8400, 640, 640, 0.25, 0.45)


def test_postprocess_errors(be):
    raw = be.alloc(4 * 84 * 16385)
    counts = be.alloc(4)
    dets = be.alloc(24 * 16385)
    with pytest.raises(BackendError) as e:
        ops.postprocess_yolo_device(be, raw, 1, 80, 16385, 640, 640, 0.25, 0.45, 0, None, dets, counts)
    assert e.value.status == dw._lib.DW_ERR_UNSUPPORTED
    with pytest.raises(BackendError) as e:
        ops.postprocess_yolo_device(be, raw, 1, 80, 8400, 640, 640, 0.25, 0.45, 0, None, dets, counts)
    assert e.value.status == dw._lib.DW_ERR_SIZE_MISMATCH
    # zero anchors: every count is 0
    c2 = be.alloc(8)
    assert [len(d) for d in ops.postprocess_yolo(be, raw, 2, 0, 0, 640, 640, 0.25, 0.45)] == [0, 0]
    for b in (raw, counts, dets, c2):
        b.free()
