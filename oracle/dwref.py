"""ctypes/numpy wrapper over the CPU oracle ``oracle/libdwref.so``.

TEST INFRASTRUCTURE ONLY: imported by ``tests/``, ``__graft_entry__.smoke()`` and
``bench.py``'s CPU-baseline leg, as the checker.  The product package
(``dragonwing_edge_rs_b200``) never imports this module.

Each wrapper mirrors the reference function named in its docstring
(paths relative to the reference repository root).
"""
from __future__ import annotations

import ctypes
import os
import subprocess

import numpy as np

_HERE = os.path.dirname(os.path.abspath(__file__))
_LIB_PATH = os.path.join(_HERE, "libdwref.so")

EPI_NONE, EPI_RELU, EPI_RELU6, EPI_SILU = 0, 1, 2, 3


class ConvDesc(ctypes.Structure):
    """Same field meaning as ``dw_conv_desc`` in include/dw_cuda.h."""

    _fields_ = [(n, ctypes.c_int32) for n in (
        "n", "h", "w", "c_in", "c_out", "k_h", "k_w", "stride_h", "stride_w",
        "pad_t", "pad_l", "pad_b", "pad_r", "group", "epilogue", "q6")] + [("inv_s_out", ctypes.c_float)]


class YoloDesc(ctypes.Structure):
    """Same field meaning as ``dw_yolo_detect_desc`` in include/dw_cuda.h."""

    _fields_ = [("n", ctypes.c_int32), ("num_classes", ctypes.c_int32), ("reg_max", ctypes.c_int32),
                ("num_levels", ctypes.c_int32), ("h", ctypes.c_int32 * 4), ("w", ctypes.c_int32 * 4),
                ("stride", ctypes.c_float * 4), ("box_scale", ctypes.c_float * 4), ("cls_scale", ctypes.c_float * 4)]


# Detection (crates/dragonwing-onnx/src/postprocess.rs:12-19)
DETECTION_DTYPE = np.dtype([("bbox", "<f4", (4,)), ("class_id", "<u4"), ("confidence", "<f4")])


def build() -> str:
    """Compile the oracle with its Makefile (gcc only; seconds)."""
    subprocess.run(["make", "-s", "-C", _HERE], check=True)
    return _LIB_PATH


_lib = None


def lib() -> ctypes.CDLL:
    global _lib
    if _lib is None:
        if not os.path.exists(_LIB_PATH):
            build()
        _lib = ctypes.CDLL(_LIB_PATH)
        _declare(_lib)
    return _lib


def _p(a):
    return a.ctypes.data_as(ctypes.c_void_p) if a is not None else None


def _declare(L):
    vp, sz, f32, i32 = ctypes.c_void_p, ctypes.c_size_t, ctypes.c_float, ctypes.c_int
    sig = {
        "dwref_gemm_i8": [vp, vp, vp, sz, sz, sz],
        "dwref_conv2d_i8_nhwc": [vp, vp, vp] + [sz] * 11,
        "dwref_requantize_i32_to_i8": [vp, vp, sz, f32],
        "dwref_relu_i8": [vp, vp, sz],
        "dwref_add_i8": [vp, vp, vp, sz, f32, f32],
        "dwref_quantize_f32_to_i8": [vp, vp, sz, f32],
        "dwref_dequantize_i8_to_f32": [vp, vp, sz, f32],
        "dwref_quantize_u8_to_i8": [vp, vp, sz, f32],
        "dwref_per_channel_scales": [vp, vp, sz, sz],
        "dwref_per_channel_quantize": [vp, vp, vp, sz, sz],
        "dwref_conv2d_fused_i8": [vp, vp, vp, vp, vp, vp, ctypes.POINTER(ConvDesc), i32],
        "dwref_conv2d_acc_i32": [vp, vp, vp, ctypes.POINTER(ConvDesc), i32],
        "dwref_qgemm_i8": [vp, vp, vp, vp, vp, sz, sz, sz, i32, ctypes.c_int32, i32],
        "dwref_maxpool_i8_nhwc": [vp, vp] + [sz] * 12,
        "dwref_concat_c_i8": [vp, vp, vp, ctypes.c_int32, sz],
        "dwref_resize_nearest_i8": [vp, vp] + [sz] * 6,
        "dwref_conv2d_f16_nhwc": [vp, vp, vp, vp, i32] + [sz] * 11 + [i32],
        "dwref_dwconv_f16_nhwc": [vp, vp, vp, vp, i32] + [sz] * 11 + [i32],
        "dwref_bias_relu_f16": [vp, vp, i32, sz, sz],
        "dwref_f16_from_f32_array": [vp, vp, sz],
        "dwref_f16_to_f32_array": [vp, vp, sz],
        "dwref_gemm_f16": [vp, vp, vp, sz, sz, sz, i32],
        "dwref_add_f16": [vp, vp, vp, sz],
        "dwref_relu_f16": [vp, vp, sz],
        "dwref_gap_f16": [vp, vp, sz, sz, sz, sz],
        "dwref_maxpool_f16_nhwc": [vp, vp] + [sz] * 12,
    }
    sig["dwref_yolo_detect_i8"] = [vp, vp, vp, ctypes.POINTER(YoloDesc)]
    sig["dwref_sigmoid_f32"] = [vp, vp, sz]
    sig["dwref_softmax_f32"] = [vp, vp, sz, sz]
    for name, args in sig.items():
        fn = getattr(L, name)
        fn.argtypes = args
        fn.restype = None
    for name in ("dwref_conv2d_fused_i8", "dwref_conv2d_acc_i32"):
        getattr(L, name).restype = ctypes.c_int
    L.dwref_f32_to_i8.argtypes = [f32]
    L.dwref_f32_to_i8.restype = ctypes.c_int8
    L.dwref_quantscale_quantize.argtypes = [f32, f32]
    L.dwref_quantscale_quantize.restype = ctypes.c_int8
    L.dwref_requant_scale.argtypes = [f32, f32, f32]
    L.dwref_requant_scale.restype = f32
    L.dwref_expf.argtypes = [f32]
    L.dwref_expf.restype = f32
    L.dwref_silu_f32.argtypes = [f32]
    L.dwref_silu_f32.restype = f32
    L.dwref_set_silu_exp_libm.argtypes = [ctypes.c_int]
    L.dwref_set_silu_exp_libm.restype = None
    L.dwref_silu_epilogue_f32.argtypes = [f32]
    L.dwref_silu_epilogue_f32.restype = f32
    L.dwref_f16_from_f32.argtypes = [f32]
    L.dwref_f16_from_f32.restype = ctypes.c_uint16
    L.dwref_f16_to_f32.argtypes = [ctypes.c_uint16]
    L.dwref_f16_to_f32.restype = f32
    L.dwref_det_area.argtypes = [vp]
    L.dwref_det_area.restype = f32
    L.dwref_iou.argtypes = [vp, vp]
    L.dwref_iou.restype = f32
    L.dwref_decode_detections_v8.argtypes = [vp, vp, sz, sz, sz, ctypes.c_uint32, ctypes.c_uint32, f32, i32]
    L.dwref_decode_detections_v8.restype = sz
    L.dwref_nms.argtypes = [vp, sz, f32, i32]
    L.dwref_nms.restype = sz
    L.dwref_postprocess_yolo.argtypes = [vp, vp, sz, sz, sz, ctypes.c_uint32, ctypes.c_uint32, f32, f32, i32]
    L.dwref_postprocess_yolo.restype = sz
    L.dwref_num_cpus.argtypes = []
    L.dwref_num_cpus.restype = ctypes.c_int


def _c(a, dtype):
    return np.ascontiguousarray(a, dtype=dtype)


def num_cpus() -> int:
    return lib().dwref_num_cpus()


# ---- reference scalar ops (crates/dragonwing-cpu/src/ops.rs) ----

def gemm_i8(a, b, m, n, k):
    """ops.rs:2981-2995 gemm_i8_scalar."""
    a, b = _c(a, np.int8), _c(b, np.int8)
    c = np.empty(m * n, np.int32)
    lib().dwref_gemm_i8(_p(c), _p(a), _p(b), m, n, k)
    return c


def conv2d_i8_nhwc(x, w, n, h, wd, c_in, c_out, k_h, k_w, s_h, s_w, p_h, p_w):
    """ops.rs:3086-3142 conv2d_i8_nhwc (i32 output)."""
    x, w = _c(x, np.int8), _c(w, np.int8)
    ho = (h + 2 * p_h - k_h) // s_h + 1
    wo = (wd + 2 * p_w - k_w) // s_w + 1
    out = np.empty(n * ho * wo * c_out, np.int32)
    lib().dwref_conv2d_i8_nhwc(_p(out), _p(x), _p(w), n, h, wd, c_in, c_out, k_h, k_w, s_h, s_w, p_h, p_w)
    return out


def requantize_i32_to_i8(acc, scale):
    """ops.rs:3380-3386."""
    acc = _c(acc, np.int32)
    out = np.empty(acc.size, np.int8)
    lib().dwref_requantize_i32_to_i8(_p(out), _p(acc), acc.size, scale)
    return out


def relu_i8(x):
    """ops.rs:3315-3319."""
    x = _c(x, np.int8)
    out = np.empty(x.size, np.int8)
    lib().dwref_relu_i8(_p(out), _p(x), x.size)
    return out


def add_i8(a, b, ra, rb):
    """ops.rs:3197-3209."""
    a, b = _c(a, np.int8), _c(b, np.int8)
    out = np.empty(a.size, np.int8)
    lib().dwref_add_i8(_p(out), _p(a), _p(b), a.size, ra, rb)
    return out


def quantize_f32_to_i8(x, scale):
    """ops.rs:3503-3525."""
    x = _c(x, np.float32)
    out = np.empty(x.size, np.int8)
    lib().dwref_quantize_f32_to_i8(_p(out), _p(x), x.size, scale)
    return out


def quantize_u8_to_i8(x, scale):
    """u8 * (1/255) then quantize_f32_to_i8 (ops.rs:3503-3525)."""
    x = _c(x, np.uint8)
    out = np.empty(x.size, np.int8)
    lib().dwref_quantize_u8_to_i8(_p(out), _p(x), x.size, scale)
    return out


def dequantize_i8_to_f32(x, scale):
    """ops.rs:3453-3457."""
    x = _c(x, np.int8)
    out = np.empty(x.size, np.float32)
    lib().dwref_dequantize_i8_to_f32(_p(out), _p(x), x.size, scale)
    return out


def quantscale_quantize(scale, value):
    """crates/dragonwing-core/src/quantization.rs:94-99."""
    return int(lib().dwref_quantscale_quantize(scale, value))


def per_channel_scales(weights, num_channels):
    """quantization.rs:154-171."""
    w = _c(weights, np.float32)
    s = np.empty(num_channels, np.float32)
    lib().dwref_per_channel_scales(_p(s), _p(w), w.size, num_channels)
    return s


def per_channel_quantize(weights, scales):
    """quantization.rs:178-195."""
    w, s = _c(weights, np.float32), _c(scales, np.float32)
    out = np.empty(w.size, np.int8)
    lib().dwref_per_channel_quantize(_p(out), _p(w), _p(s), w.size, s.size)
    return out


def requant_scale(s_in, s_w, s_out):
    """crates/dragonwing-onnx/src/quantize.rs:245."""
    return float(lib().dwref_requant_scale(s_in, s_w, s_out))


# ---- fused op contract ----

def conv_desc(n, h, w, c_in, c_out, k_h, k_w, s_h=1, s_w=1, pads=(0, 0, 0, 0), group=1,
              epilogue=EPI_NONE, q6=127, inv_s_out=0.0) -> ConvDesc:
    pt, pl, pb, pr = pads
    return ConvDesc(n, h, w, c_in, c_out, k_h, k_w, s_h, s_w, pt, pl, pb, pr, group, epilogue, q6,
                    inv_s_out)


def out_hw(d: ConvDesc):
    return ((d.h + d.pad_t + d.pad_b - d.k_h) // d.stride_h + 1,
            (d.w + d.pad_l + d.pad_r - d.k_w) // d.stride_w + 1)


def conv2d_fused_i8(x, w_hwio, bias, M, D, d: ConvDesc, threads=1):
    """Fused-op contract: conv -> +bias -> per-channel requant -> epilogue."""
    ho, wo = out_hw(d)
    x, w = _c(x, np.int8), _c(w_hwio, np.int8)
    bias = None if bias is None else _c(bias, np.int32)
    M = None if M is None else _c(M, np.float32)
    D = None if D is None else _c(D, np.float32)
    y = np.empty(d.n * ho * wo * d.c_out, np.int8)
    rc = lib().dwref_conv2d_fused_i8(_p(y), _p(x), _p(w), _p(bias), _p(M), _p(D), ctypes.byref(d), threads)
    if rc != 0:
        raise ValueError("dwref_conv2d_fused_i8: invalid descriptor")
    return y


def conv2d_acc_i32(x, w_hwio, d: ConvDesc, threads=1):
    ho, wo = out_hw(d)
    x, w = _c(x, np.int8), _c(w_hwio, np.int8)
    acc = np.empty(d.n * ho * wo * d.c_out, np.int32)
    rc = lib().dwref_conv2d_acc_i32(_p(acc), _p(x), _p(w), ctypes.byref(d), threads)
    if rc != 0:
        raise ValueError("dwref_conv2d_acc_i32: invalid descriptor")
    return acc


def qgemm_i8(a, b, bias, M, m, n, k, epilogue=EPI_NONE, q6=127, threads=1):
    """gemm_i8_scalar + per-column epilogue of the contract."""
    a, b = _c(a, np.int8), _c(b, np.int8)
    bias = None if bias is None else _c(bias, np.int32)
    M = _c(M, np.float32)
    y = np.empty(m * n, np.int8)
    lib().dwref_qgemm_i8(_p(y), _p(a), _p(b), _p(bias), _p(M), m, n, k, epilogue, q6, threads)
    return y


def expf(x: float) -> float:
    return float(lib().dwref_expf(x))


def set_silu_exp_libm(on: bool) -> None:
    """Measurement switch: the SiLU epilogue uses the host libm's expf (the
    reference's f32::exp, ops.rs:1865-1870) instead of the shared exp."""
    lib().dwref_set_silu_exp_libm(1 if on else 0)


def silu_epilogue_f32(y: float) -> float:
    """The float SiLU the int8 epilogue uses under the current exp switch."""
    return lib().dwref_silu_epilogue_f32(y)


def silu_f32(x: float) -> float:
    return float(lib().dwref_silu_f32(x))


# ---- glue ----

def maxpool_i8(x, n, h, w, c, k_h, k_w, s_h, s_w, pads=(0, 0, 0, 0)):
    pt, pl, pb, pr = pads
    ho = (h + pt + pb - k_h) // s_h + 1
    wo = (w + pl + pr - k_w) // s_w + 1
    x = _c(x, np.int8)
    y = np.empty(n * ho * wo * c, np.int8)
    lib().dwref_maxpool_i8_nhwc(_p(y), _p(x), n, h, w, c, k_h, k_w, s_h, s_w, pt, pl, pb, pr)
    return y


def concat_c_i8(xs, cs, pixels):
    xs = [_c(x, np.int8) for x in xs]
    ptrs = (ctypes.c_void_p * len(xs))(*[x.ctypes.data for x in xs])
    cs_arr = np.asarray(cs, np.int32)
    y = np.empty(pixels * int(cs_arr.sum()), np.int8)
    lib().dwref_concat_c_i8(_p(y), ctypes.cast(ptrs, ctypes.c_void_p), _p(cs_arr), len(xs), pixels)
    return y


def resize_nearest_i8(x, n, h_in, w_in, h_out, w_out, c):
    x = _c(x, np.int8)
    y = np.empty(n * h_out * w_out * c, np.int8)
    lib().dwref_resize_nearest_i8(_p(y), _p(x), n, h_in, w_in, h_out, w_out, c)
    return y


# ---- fp16 ----

def f16_from_f32(v: float) -> int:
    return int(lib().dwref_f16_from_f32(v))


def f16_to_f32(h: int) -> float:
    return float(lib().dwref_f16_to_f32(h))


def conv2d_f16(x, w_hwio, bias, relu, n, h, w, c_in, c_out, k_h, k_w, s_h, s_w, p_h, p_w, threads=1):
    """ops.rs:1442-1511 (+ runtime.rs:1483-1497 bias, ops.rs:345 relu); uint16 bit patterns."""
    x, wt = _c(x, np.uint16), _c(w_hwio, np.uint16)
    b = None if bias is None else _c(bias, np.uint16)
    ho = (h + 2 * p_h - k_h) // s_h + 1
    wo = (w + 2 * p_w - k_w) // s_w + 1
    y = np.empty(n * ho * wo * c_out, np.uint16)
    lib().dwref_conv2d_f16_nhwc(_p(y), _p(x), _p(wt), _p(b), int(relu), n, h, w, c_in, c_out, k_h, k_w,
                                s_h, s_w, p_h, p_w, threads)
    return y


def dwconv_f16(x, w, relu, n, h, wd, c, mult, k_h, k_w, s_h, s_w, p_h, p_w, threads=1, bias=None):
    """ops.rs:2819-2937 depthwise fp16 (+ runtime.rs:1483-1497 bias, relu)."""
    x, wt = _c(x, np.uint16), _c(w, np.uint16)
    b = None if bias is None else _c(bias, np.uint16)
    ho = (h + 2 * p_h - k_h) // s_h + 1
    wo = (wd + 2 * p_w - k_w) // s_w + 1
    y = np.empty(n * ho * wo * c * mult, np.uint16)
    lib().dwref_dwconv_f16_nhwc(_p(y), _p(x), _p(wt), _p(b), int(relu), n, h, wd, c, mult, k_h, k_w, s_h, s_w,
                                p_h, p_w, threads)
    return y


def bias_relu_f16(y, bias, relu, rows, c):
    """runtime.rs:1264-1275 / 1483-1497 bias step (+ Relu), on a copy of y."""
    y = np.array(_c(y, np.uint16), copy=True)
    b = None if bias is None else _c(bias, np.uint16)
    lib().dwref_bias_relu_f16(_p(y), _p(b), int(relu), rows, c)
    return y


def f16_from_f32_array(x):
    x = _c(x, np.float32)
    y = np.empty(x.size, np.uint16)
    lib().dwref_f16_from_f32_array(_p(y), _p(x), x.size)
    return y


def f16_to_f32_array(x):
    x = _c(x, np.uint16)
    y = np.empty(x.size, np.float32)
    lib().dwref_f16_to_f32_array(_p(y), _p(x), x.size)
    return y


def gemm_f16(a, b, m, n, k, threads=1):
    a, b = _c(a, np.uint16), _c(b, np.uint16)
    c = np.empty(m * n, np.uint16)
    lib().dwref_gemm_f16(_p(c), _p(a), _p(b), m, n, k, threads)
    return c


def add_f16(a, b):
    a, b = _c(a, np.uint16), _c(b, np.uint16)
    y = np.empty(a.size, np.uint16)
    lib().dwref_add_f16(_p(y), _p(a), _p(b), a.size)
    return y


def relu_f16(x):
    x = _c(x, np.uint16)
    y = np.empty(x.size, np.uint16)
    lib().dwref_relu_f16(_p(y), _p(x), x.size)
    return y


def gap_f16(x, n, h, w, c):
    x = _c(x, np.uint16)
    y = np.empty(n * c, np.uint16)
    lib().dwref_gap_f16(_p(y), _p(x), n, h, w, c)
    return y


def maxpool_f16(x, n, h, w, c, k_h, k_w, s_h, s_w, pads=(0, 0, 0, 0)):
    pt, pl, pb, pr = pads
    ho = (h + pt + pb - k_h) // s_h + 1
    wo = (w + pl + pr - k_w) // s_w + 1
    x = _c(x, np.uint16)
    y = np.empty(n * ho * wo * c, np.uint16)
    lib().dwref_maxpool_f16_nhwc(_p(y), _p(x), n, h, w, c, k_h, k_w, s_h, s_w, pt, pl, pb, pr)
    return y


# ---- YOLOv8 Detect tail and post-processing (crates/dragonwing-onnx/src/postprocess.rs) ----

def sigmoid_f32(x):
    """sigmoid_f32_scalar (crates/dragonwing-cpu/src/ops.rs:1865-1870)."""
    x = _c(x, np.float32)
    y = np.empty_like(x)
    lib().dwref_sigmoid_f32(_p(y), _p(x), x.size)
    return y


def softmax_f32(x, n):
    """softmax_f32 (ops.rs:1609-1640) along rows of n."""
    x = _c(x, np.float32)
    y = np.empty_like(x)
    lib().dwref_softmax_f32(_p(y), _p(x), x.size, n)
    return y


def yolo_detect_i8(boxes, clss, strides, box_scales, cls_scales, reg_max=16):
    """The Detect head's f32 tail on int8 head outputs (dwref_yolo_detect_i8):
    boxes[l] int8 [n, h, w, 4*reg_max], clss[l] int8 [n, h, w, nc] -> f32 [n, 4 + nc, A]."""
    boxes = [_c(b, np.int8) for b in boxes]
    clss = [_c(c, np.int8) for c in clss]
    n, nc = boxes[0].shape[0], clss[0].shape[3]
    d = YoloDesc()
    d.n, d.num_classes, d.reg_max, d.num_levels = n, nc, reg_max, len(boxes)
    A = 0
    for i, b in enumerate(boxes):
        d.h[i], d.w[i] = b.shape[1], b.shape[2]
        d.stride[i], d.box_scale[i], d.cls_scale[i] = strides[i], box_scales[i], cls_scales[i]
        A += b.shape[1] * b.shape[2]
    out = np.empty((n, 4 + nc, A), np.float32)
    bp = (ctypes.c_void_p * len(boxes))(*[b.ctypes.data for b in boxes])
    cp = (ctypes.c_void_p * len(clss))(*[c.ctypes.data for c in clss])
    lib().dwref_yolo_detect_i8(_p(out), ctypes.cast(bp, ctypes.c_void_p), ctypes.cast(cp, ctypes.c_void_p),
                               ctypes.byref(d))
    return out


def detections(rows) -> np.ndarray:
    """[(bbox4, class_id, confidence), ...] -> DETECTION_DTYPE array."""
    return np.array([(tuple(b), c, f) for b, c, f in rows], DETECTION_DTYPE)


def det_area(det) -> float:
    """Detection::area (postprocess.rs:28-32)."""
    d = np.ascontiguousarray(np.array(det, DETECTION_DTYPE).reshape(1))
    return float(lib().dwref_det_area(_p(d)))


def iou(a, b) -> float:
    """iou (postprocess.rs:36-55)."""
    da = np.ascontiguousarray(np.array(a, DETECTION_DTYPE).reshape(1))
    db = np.ascontiguousarray(np.array(b, DETECTION_DTYPE).reshape(1))
    return float(lib().dwref_iou(_p(da), _p(db)))


def decode_detections_v8(raw, num_classes, num_detections, img_width, img_height, conf_threshold, alt=False):
    """decode_detections_v8 (postprocess.rs:78-146) / _alt (:151-208) on one image."""
    raw = _c(raw, np.float32).reshape(-1)
    out = np.zeros(max(1, num_detections), DETECTION_DTYPE)
    k = lib().dwref_decode_detections_v8(_p(out), _p(raw), raw.size, num_classes, num_detections, img_width,
                                         img_height, conf_threshold, 1 if alt else 0)
    return out[:k].copy()


def nms(dets, iou_threshold, agnostic=False):
    """nms (postprocess.rs:227-265) / nms_agnostic (:270-300): returns the kept list in the reference's order."""
    d = np.ascontiguousarray(np.array(dets, DETECTION_DTYPE).reshape(-1)).copy()
    k = lib().dwref_nms(_p(d), d.size, iou_threshold, 1 if agnostic else 0)
    return d[:k].copy()


def postprocess_yolo(raw, num_classes, num_detections, img_width, img_height, conf_threshold, iou_threshold,
                     flags=0):
    """postprocess_yolo (postprocess.rs:319-340) on one image (flags: 1 alt layout, 2 agnostic, 4 no NMS)."""
    raw = _c(raw, np.float32).reshape(-1)
    out = np.zeros(max(1, num_detections), DETECTION_DTYPE)
    k = lib().dwref_postprocess_yolo(_p(out), _p(raw), raw.size, num_classes, num_detections, img_width,
                                     img_height, conf_threshold, iou_threshold, flags)
    return out[:k].copy()
