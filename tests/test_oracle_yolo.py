"""CPU checks of the YOLO post-processing oracle (oracle/dwref.c):

* the reference's own known-answer tests (postprocess.rs:346-407, ops.rs sigmoid
  and softmax tests), transcribed in tests/golden/reference_kats.json;
* the oracle's decode + NMS against a line-by-line Python transcription of
  postprocess.rs on small random cases (float32 arithmetic, output order
  included);
* the two rules the device post-processing uses in place of the reference's
  sequential loops: the output order of its swap_remove deletion (positions
  filled by following p -> L_p - 1 until a kept rank, L_p = kept + removed
  ranks <= p), on random and exhaustive keep patterns; and the batched greedy
  NMS (32 candidates resolved in order, then the rest filtered by the batch's
  kept boxes), against the greedy loop on random boxes.
"""
import json
import os

import numpy as np
import pytest

from oracle import dwref

KATS = json.load(open(os.path.join(os.path.dirname(__file__), "golden", "reference_kats.json")))
F = np.float32


def det(bbox, cls=0, conf=0.9):
    return dwref.detections([(bbox, cls, conf)])[0]


def test_iou_kats():
    k = KATS["iou_no_overlap"]
    assert dwref.iou(det(k["a"]), det(k["b"], conf=0.8)) == k["expected"]
    k = KATS["iou_full_overlap"]
    assert abs(dwref.iou(det(k["a"]), det(k["b"], conf=0.8)) - k["expected"]) < k["tolerance"]
    k = KATS["iou_partial_overlap"]
    num, den = k["expected"]
    assert abs(dwref.iou(det(k["a"]), det(k["b"], conf=0.8)) - num / den) < k["tolerance"]


def test_area_kat():
    k = KATS["detection_area"]
    assert abs(dwref.det_area(det(k["bbox"])) - k["expected"]) < k["tolerance"]


def test_nms_kats():
    k = KATS["nms_basic"]
    out = dwref.nms(dwref.detections(k["dets"]), k["iou_threshold"])
    assert len(out) == k["expected_len"]
    assert abs(out[0]["confidence"] - k["expected_first_confidence"]) < k["tolerance"]
    k = KATS["nms_different_classes"]
    assert len(dwref.nms(dwref.detections(k["dets"]), k["iou_threshold"])) == k["expected_len"]


def test_decode_empty_kat():
    k = KATS["decode_empty"]
    out = dwref.decode_detections_v8(np.zeros(0, np.float32), k["num_classes"], k["num_detections"],
                                     k["img_width"], k["img_height"], k["conf_threshold"])
    assert len(out) == k["expected_len"]


def test_sigmoid_softmax_kats():
    k = KATS["sigmoid_f32_basic"]
    y = dwref.sigmoid_f32(k["x"])
    assert np.all(np.abs(y - np.array(k["expected"], np.float32)) < k["tolerance"])
    k = KATS["softmax_basic"]
    y = dwref.softmax_f32(k["x"], len(k["x"]))
    assert abs(float(y.sum()) - 1.0) < k["sum_tolerance"]
    assert y[0] < y[1] < y[2] and np.all(y > 0)


# ---- line-by-line Python transcription of postprocess.rs (float32) ----

def py_decode(raw, nc, A, iw, ih, thr, alt=False):
    """decode_detections_v8 (:78-146) / _alt (:151-208)."""
    raw = raw.reshape(-1)
    if raw.size < (4 + nc) * A:
        return []
    sx, sy = F(iw) / F(640.0), F(ih) / F(640.0)
    out = []
    for a in range(A):
        at = (lambda ch: raw[a * (4 + nc) + ch]) if alt else (lambda ch: raw[ch * A + a])
        cx, cy, w, h = at(0), at(1), at(2), at(3)
        bc, best = 0, F(0.0)
        for c in range(nc):
            v = at(4 + c)
            if v > best:
                best, bc = v, c
        if best < F(thr):
            continue
        x1 = (cx - w / F(2.0)) * sx
        y1 = (cy - h / F(2.0)) * sy
        x2 = (cx + w / F(2.0)) * sx
        y2 = (cy + h / F(2.0)) * sy
        clamp = lambda v, hi: min(max(v, F(0.0)), F(hi))  # noqa: E731
        out.append(([clamp(x1, iw), clamp(y1, ih), clamp(x2, iw), clamp(y2, ih)], bc, best))
    return out


def py_iou(a, b):
    """iou (:36-55)."""
    x1, y1 = max(a[0][0], b[0][0]), max(a[0][1], b[0][1])
    x2, y2 = min(a[0][2], b[0][2]), min(a[0][3], b[0][3])
    inter = max(x2 - x1, F(0.0)) * max(y2 - y1, F(0.0))
    area = lambda d: max(d[0][2] - d[0][0], F(0.0)) * max(d[0][3] - d[0][1], F(0.0))  # noqa: E731
    uni = area(a) + area(b) - inter
    return inter / uni if uni > F(0.0) else F(0.0)


def py_nms(dets, thr, agnostic=False):
    """nms (:227-265) / nms_agnostic (:270-300), with the swap_remove deletion."""
    d = sorted(dets, key=lambda t: -t[2])  # stable, like Vec::sort_by
    keep = [True] * len(d)
    for i in range(len(d)):
        if not keep[i]:
            continue
        for j in range(i + 1, len(d)):
            if not keep[j]:
                continue
            if not agnostic and d[i][1] != d[j][1]:
                continue
            if py_iou(d[i], d[j]) > F(thr):
                keep[j] = False
    for i in range(len(d) - 1, -1, -1):
        if not keep[i]:
            d[i] = d[-1]
            d.pop()
    return d


def as_rows(arr):
    return [([F(v) for v in r["bbox"]], int(r["class_id"]), F(r["confidence"])) for r in arr]


def random_raw(rng, nc, A, grid=8):
    """Boxes clustered on a coarse grid (so NMS has work), scores with ties."""
    raw = np.zeros((4 + nc, A), np.float32)
    raw[0] = rng.integers(0, grid, A) * (640 / grid) + rng.normal(0, 8, A)
    raw[1] = rng.integers(0, grid, A) * (640 / grid) + rng.normal(0, 8, A)
    raw[2] = rng.uniform(20, 160, A)
    raw[3] = rng.uniform(20, 160, A)
    raw[4:] = rng.integers(0, 40, (nc, A)) / 40.0  # quantised: many equal confidences
    return raw.astype(np.float32)


@pytest.mark.parametrize("seed,nc,A,flags", [(0, 3, 60, 0), (1, 1, 90, 0), (2, 5, 120, 2), (3, 4, 75, 1),
                                             (4, 2, 64, 4), (5, 6, 200, 0)])
def test_oracle_postprocess_matches_python_transcription(seed, nc, A, flags):
    rng = np.random.default_rng(seed)
    raw = random_raw(rng, nc, A)
    if flags & 1:
        raw = np.ascontiguousarray(raw.T)
    iw, ih, thr, iou_thr = 800, 600, 0.3, 0.45
    got = as_rows(dwref.postprocess_yolo(raw, nc, A, iw, ih, thr, iou_thr, flags))
    want = py_decode(raw, nc, A, iw, ih, thr, alt=bool(flags & 1))
    if not flags & 4:
        want = py_nms(want, iou_thr, agnostic=bool(flags & 2))
    assert len(got) == len(want)
    for g, w in zip(got, want):
        assert g[1] == w[1] and g[2] == w[2] and all(a == b for a, b in zip(g[0], w[0]))


def swap_remove_order(keep):
    """The reference's deletion loop (postprocess.rs:257-264) on ranks."""
    v = list(range(len(keep)))
    for i in range(len(keep) - 1, -1, -1):
        if not keep[i]:
            v[i] = v[-1]
            v.pop()
    return v


def pointer_jumping_order(keep):
    """The device rule: K kept; L_r = K + (removed ranks <= r); a removed rank r
    links to L_r - 1, a kept rank to itself; position p < K ends with the kept
    rank its chain reaches (found by pointer doubling)."""
    keep = np.asarray(keep, bool)
    c = keep.size
    rem = np.cumsum(~keep)
    K = c - (int(rem[-1]) if c else 0)
    nxt = np.where(keep, np.arange(c), K + rem - 1)
    for _ in range(16):
        nn = nxt[nxt]
        if np.array_equal(nn, nxt):
            break
        nxt = nn
    return nxt[:K].tolist()


@pytest.mark.parametrize("p_keep", [0.05, 0.3, 0.5, 0.8, 0.97])
def test_device_order_rule_equals_swap_remove(p_keep):
    rng = np.random.default_rng(int(p_keep * 100))
    for c in list(range(1, 12)) + [37, 100, 513, 4000]:
        for _ in range(20 if c < 100 else 3):
            keep = rng.random(c) < p_keep
            keep[0] = True  # the top-ranked candidate is never suppressed
            assert pointer_jumping_order(keep) == swap_remove_order(list(keep))


def test_device_order_rule_exhaustive_small():
    for c in range(1, 11):
        for bits in range(1 << (c - 1)):
            keep = [True] + [bool(bits >> i & 1) for i in range(c - 1)]
            assert pointer_jumping_order(keep) == swap_remove_order(keep)


def test_detect_tail_oracle_formula():
    """dwref_yolo_detect_i8 against a float32 numpy restatement (exp from numpy,
    so compared with a tolerance: only the formula is checked here)."""
    rng = np.random.default_rng(7)
    n, nc = 2, 5
    grids, strides = [(4, 5), (2, 3)], [8.0, 16.0]
    bs, cs = [0.05, 0.07], [0.03, 0.09]
    boxes = [rng.integers(-128, 128, (n, h, w, 64), dtype=np.int8) for h, w in grids]
    clss = [rng.integers(-128, 128, (n, h, w, nc), dtype=np.int8) for h, w in grids]
    out = dwref.yolo_detect_i8(boxes, clss, strides, bs, cs)
    A = sum(h * w for h, w in grids)
    assert out.shape == (n, 4 + nc, A)
    off = 0
    for l, (h, w) in enumerate(grids):
        x = boxes[l].astype(np.float32).reshape(n, h * w, 4, 16) * F(bs[l])
        e = np.exp(x - x.max(-1, keepdims=True))
        p = e / e.sum(-1, keepdims=True)
        dist = (p * np.arange(16, dtype=np.float32)).sum(-1)
        gy, gx = np.divmod(np.arange(h * w), w)
        ax, ay = gx + 0.5, gy + 0.5
        x1, y1, x2, y2 = ax - dist[..., 0], ay - dist[..., 1], ax + dist[..., 2], ay + dist[..., 3]
        ref = np.stack([(x1 + x2) / 2, (y1 + y2) / 2, x2 - x1, y2 - y1], 1) * strides[l]
        np.testing.assert_allclose(out[:, :4, off:off + h * w], ref, rtol=1e-5, atol=1e-4)
        sg = 1 / (1 + np.exp(-(clss[l].astype(np.float32) * F(cs[l]))))
        np.testing.assert_allclose(out[:, 4:, off:off + h * w], sg.reshape(n, h * w, nc).transpose(0, 2, 1),
                                   rtol=1e-6, atol=1e-7)
        off += h * w


def batched_nms_keep(dets, thr, batch=32):
    """The device NMS rule on one class's candidates in rank order: the first
    `batch` entries of the live list are resolved in order (kept unless an
    earlier kept entry of the batch overlaps by IoU > thr), then the rest of the
    list keeps only entries no kept batch box overlaps; repeat."""
    keep = [False] * len(dets)
    live = list(range(len(dets)))
    while live:
        head, rest = live[:batch], live[batch:]
        kept = []
        for q in head:
            if all(not py_iou(dets[k], dets[q]) > F(thr) for k in kept):
                kept.append(q)
                keep[q] = True
        live = [j for j in rest if all(not py_iou(dets[k], dets[j]) > F(thr) for k in kept)]
    return keep


def greedy_keep(dets, thr):
    """The reference's loop (postprocess.rs:233-255) on one class, in rank order."""
    keep = [True] * len(dets)
    for i in range(len(dets)):
        if not keep[i]:
            continue
        for j in range(i + 1, len(dets)):
            if keep[j] and py_iou(dets[i], dets[j]) > F(thr):
                keep[j] = False
    return keep


@pytest.mark.parametrize("seed,n,batch,thr", [(0, 10, 32, 0.45), (1, 200, 32, 0.45), (2, 300, 4, 0.3), (6, 400, 64, 0.45), (7, 600, 128, 0.45),
                                              (3, 150, 32, 0.7), (4, 64, 1, 0.45), (5, 257, 32, 0.0)])
def test_device_batched_nms_rule_equals_greedy(seed, n, batch, thr):
    rng = np.random.default_rng(seed)
    raw = random_raw(rng, 1, n, grid=6)
    dets = py_decode(raw, 1, n, 640, 640, 0.0)
    dets = sorted(dets, key=lambda t: -t[2])
    assert batched_nms_keep(dets, thr, batch) == greedy_keep(dets, thr)


def iou_gt_rule(inter, uni, t):
    """The device's division-free test of RN(inter / uni) > t (exact in double)."""
    t = np.float32(t)
    tp = np.nextafter(t, np.float32(np.inf))
    mid = (float(t) + float(tp)) * 0.5
    tie_up = (int(tp.view(np.uint32)) & 1) == 0
    if not uni > 0:
        return bool(np.float32(0.0) > t)
    lhs, rhs = float(inter), mid * float(uni)
    return lhs > rhs or (lhs == rhs and tie_up)


def test_division_free_iou_threshold_rule():
    rng = np.random.default_rng(3)
    ts = [0.45, 0.5, 0.3, 0.0, -0.0, 1.0, 0.7, -0.25, 1e-40, 3e-45, np.inf, np.nan,
          float(np.nextafter(np.float32(0.45), np.float32(1)))]
    for t in ts:
        t32 = np.float32(t)
        uni = rng.uniform(1e-3, 1e5, 4000).astype(np.float32)
        frac = rng.uniform(0, 1.2, 4000).astype(np.float32)
        inter = (uni * frac).astype(np.float32)
        # quotients right at t and its neighbours
        inter[:500] = (uni[:500] * t32).astype(np.float32) if np.isfinite(t32) else inter[:500]
        for i, u in zip(inter, uni):
            q = np.float32(i) / np.float32(u)
            assert iou_gt_rule(i, u, t) == bool(q > t32), (i, u, t)
        assert iou_gt_rule(np.float32(0), np.float32(0), t) == bool(np.float32(0) > t32)
    # exact ties exist only for subnormal thresholds: q == midpoint of (t, next(t))
    for k in range(1, 60):
        t = np.uint32(k).view(np.float32)
        tp = np.nextafter(t, np.float32(1))
        for e in range(0, 40):
            uni = np.float32(2.0 ** e)
            inter = np.float32((float(t) + float(tp)) * 0.5 * float(uni))
            if float(inter) == (float(t) + float(tp)) * 0.5 * float(uni):  # representable: an exact tie
                q = np.float32(inter) / uni
                assert iou_gt_rule(inter, uni, t) == bool(q > t)
