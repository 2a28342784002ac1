"""Op free functions of the B200 backend.

The names, argument order and argument meaning follow the reference's op
functions (``dragonwing_vulkan::ops`` in crates/dragonwing-vulkan/src/ops.rs and
``dragonwing_cpu::ops`` in crates/dragonwing-cpu/src/ops.rs): free functions
taking the backend, input buffers, the output buffer and the NHWC dims.  Every
function enqueues device work on the backend's stream and raises
``BackendError`` on any argument or size problem.  The ``*_i8`` functions
without a reference counterpart implement the build's superset contract of
the fused op (int32 bias, per-channel requant, ReLU6/SiLU, depthwise).
"""
from __future__ import annotations

import ctypes
from dataclasses import dataclass

import numpy as np

from . import _lib as L
from .backend import CudaBackend, CudaBuffer

EPI_NONE, EPI_RELU, EPI_RELU6, EPI_SILU = L.EPI_NONE, L.EPI_RELU, L.EPI_RELU6, L.EPI_SILU


def _h(buf):
    return None if buf is None else buf.handle


# ---------------------------------------------------------------------------
# Reference op signatures (crates/dragonwing-vulkan/src/ops.rs)
# ---------------------------------------------------------------------------

def conv2d_requant_relu_i8_packed(backend: CudaBackend, input_packed: CudaBuffer, kernel_packed: CudaBuffer,
                                  output_packed: CudaBuffer, n, h_in, w_in, c_in, c_out, k_h, k_w,
                                  stride_h, stride_w, pad_h, pad_w, requant_scale: float, do_relu: bool):
    """ops.rs:2294-2417: fused int8 conv -> requant(scalar) -> optional ReLU.

    Kernel layout is HWIO (the graph's layout after convert_nchw_to_nhwc)."""
    backend._check(L.load().dw_conv2d_requant_relu_i8(
        backend.handle, input_packed.handle, kernel_packed.handle, output_packed.handle,
        n, h_in, w_in, c_in, c_out, k_h, k_w, stride_h, stride_w, pad_h, pad_w, float(requant_scale),
        1 if do_relu else 0))


def conv2d_i8_nhwc_packed(backend, input_packed, kernel_packed, output_i32, n, h_in, w_in, c_in, c_out,
                          k_h, k_w, stride_h, stride_w, pad_h, pad_w):
    """ops.rs:1822: int8 conv to int32 accumulators (HWIO kernel)."""
    backend._check(L.load().dw_conv2d_i8_nhwc(
        backend.handle, input_packed.handle, kernel_packed.handle, output_i32.handle,
        n, h_in, w_in, c_in, c_out, k_h, k_w, stride_h, stride_w, pad_h, pad_w))


def gemm_i8_packed(backend, a_packed, b_packed, c_i32, m, n, k):
    """ops.rs:1723: C_i32[m,n] = A[m,k] @ B[k,n] (row-major int8)."""
    backend._check(L.load().dw_gemm_i8(backend.handle, a_packed.handle, b_packed.handle, c_i32.handle, m, n, k))


def requantize_i32_to_i8_packed(backend, input_i32, output_packed, requant_scale: float):
    """ops.rs:1998 (cpu ops.rs:3366-3386)."""
    backend._check(L.load().dw_requantize_i32_to_i8(backend.handle, input_i32.handle, output_packed.handle,
                                                    float(requant_scale)))


def add_i8_packed(backend, a_packed, b_packed, output_packed, scale_a_over_y: float, scale_b_over_y: float):
    """ops.rs:2105 (cpu ops.rs:3176-3209)."""
    backend._check(L.load().dw_add_i8(backend.handle, a_packed.handle, b_packed.handle, output_packed.handle,
                                      float(scale_a_over_y), float(scale_b_over_y)))


def relu_i8_packed(backend, input_packed, output_packed):
    """ops.rs:2179 (cpu ops.rs:3301-3319)."""
    backend._check(L.load().dw_relu_i8(backend.handle, input_packed.handle, output_packed.handle))


def quantize_f32_to_i8_packed(backend, input_f32, output_packed, scale: float):
    """ops.rs:2032 (cpu ops.rs:3503-3525)."""
    backend._check(L.load().dw_quantize_f32_to_i8(backend.handle, input_f32.handle, output_packed.handle,
                                                  float(scale)))


def dequantize_i8_packed_to_f32(backend, input_packed, output_f32, scale: float):
    """ops.rs:2069 (cpu ops.rs:3439-3457)."""
    backend._check(L.load().dw_dequantize_i8_to_f32(backend.handle, input_packed.handle, output_f32.handle,
                                                    float(scale)))


# ---------------------------------------------------------------------------
# The fused op contract
# ---------------------------------------------------------------------------

@dataclass
class ConvDesc:
    """OpParams::Conv2dRequantReluI8Nhwc (crates/dragonwing-onnx/src/builder.rs:345-360)
    plus NHWC dims, bias/per-channel requant and the extended epilogues."""

    n: int
    h: int
    w: int
    c_in: int
    c_out: int
    k_h: int = 3
    k_w: int = 3
    stride_h: int = 1
    stride_w: int = 1
    pads: tuple = (0, 0, 0, 0)  # [top, left, bottom, right]
    group: int = 1
    epilogue: int = EPI_NONE
    q6: int = 127
    inv_s_out: float = 0.0

    def out_hw(self):
        pt, pl, pb, pr = self.pads
        return ((self.h + pt + pb - self.k_h) // self.stride_h + 1,
                (self.w + pl + pr - self.k_w) // self.stride_w + 1)

    def to_c(self) -> L.DwConvDesc:
        pt, pl, pb, pr = self.pads
        return L.DwConvDesc(self.n, self.h, self.w, self.c_in, self.c_out, self.k_h, self.k_w, self.stride_h,
                            self.stride_w, pt, pl, pb, pr, self.group, self.epilogue, self.q6, self.inv_s_out)


def prepare_weights_i8(backend: CudaBackend, desc: ConvDesc, w_hwio: CudaBuffer) -> CudaBuffer:
    """HWIO (or depthwise [kh,kw,C,mult]) int8 kernel -> the kernels' layout (once)."""
    out = ctypes.c_void_p()
    d = desc.to_c()
    backend._check(L.load().dw_prepare_weights_i8(backend.handle, ctypes.byref(d), w_hwio.handle, ctypes.byref(out)))
    return CudaBuffer(backend, out, L.load().dw_buf_len(out))


def conv2d_i8(backend: CudaBackend, desc: ConvDesc, x: CudaBuffer, w_prep: CudaBuffer, bias, M, D, y: CudaBuffer):
    """Fused conv: y = epilogue(requant(conv(x, w) + bias)) (contract in include/dw_cuda.h)."""
    d = desc.to_c()
    backend._check(L.load().dw_conv2d_i8(backend.handle, ctypes.byref(d), x.handle, w_prep.handle, _h(bias), _h(M),
                                         _h(D), y.handle))


def prepare_gemm_b_i8(backend: CudaBackend, b_kn: CudaBuffer, k: int, n: int) -> CudaBuffer:
    out = ctypes.c_void_p()
    backend._check(L.load().dw_prepare_gemm_b_i8(backend.handle, b_kn.handle, k, n, ctypes.byref(out)))
    return CudaBuffer(backend, out, k * n)


def qgemm_i8(backend: CudaBackend, a, b_prep, bias, M, y, m, n, k, epilogue=EPI_NONE, q6=127):
    """QGemm with int32 bias and per-column requant to int8."""
    backend._check(L.load().dw_qgemm_i8(backend.handle, a.handle, b_prep.handle, _h(bias), M.handle, y.handle,
                                        m, n, k, epilogue, q6))


def quantize_u8_to_i8(backend, input_u8, output_i8, scale: float):
    backend._check(L.load().dw_quantize_u8_to_i8(backend.handle, input_u8.handle, output_i8.handle, float(scale)))


def maxpool_i8(backend, x, y, n, h, w, c, k_h, k_w, s_h, s_w, pads=(0, 0, 0, 0)):
    pt, pl, pb, pr = pads
    backend._check(L.load().dw_maxpool_i8(backend.handle, x.handle, y.handle, n, h, w, c, k_h, k_w, s_h, s_w,
                                          pt, pl, pb, pr))


def _view(v):
    """(CudaBuffer, byte offset, pitch) -> dw_view."""
    buf, off, pitch = v
    return L.DwView(buf.handle.value, off, pitch)


def conv2d_i8_view(backend: CudaBackend, desc: ConvDesc, x, w_prep: CudaBuffer, bias, M, D, y):
    """conv2d_i8 with the input and output given as (buffer, byte offset, pixel pitch) channel-range views."""
    d, xv, yv = desc.to_c(), _view(x), _view(y)
    backend._check(L.load().dw_conv2d_i8_view(backend.handle, ctypes.byref(d), ctypes.byref(xv), w_prep.handle,
                                              _h(bias), _h(M), _h(D), ctypes.byref(yv)))


def conv2d_add_i8_view(backend: CudaBackend, desc: ConvDesc, x, w_prep: CudaBuffer, bias, M, D, residual, ra, rb, y):
    """y = add_i8(residual, conv(x)) fused (ratios ra for the residual, rb for the conv's result); the
    tensors as (buffer, byte offset, pixel pitch) views."""
    d, xv, rv, yv = desc.to_c(), _view(x), _view(residual), _view(y)
    backend._check(L.load().dw_conv2d_add_i8_view(backend.handle, ctypes.byref(d), ctypes.byref(xv), w_prep.handle,
                                                  _h(bias), _h(M), _h(D), ctypes.byref(rv), float(ra), float(rb),
                                                  ctypes.byref(yv)))


def add_i8_view(backend, a, b, out, pixels, c, ra, rb):
    av, bv, ov = _view(a), _view(b), _view(out)
    backend._check(L.load().dw_add_i8_view(backend.handle, ctypes.byref(av), ctypes.byref(bv), ctypes.byref(ov),
                                           pixels, c, float(ra), float(rb)))


def maxpool_chain_i8_view(backend, x, ys, n, h, w, c, k):
    """len(ys) chained k x k stride-1 maxpools with k/2 padding: ys[0] = pool(x), ys[i] = pool(ys[i-1]); the
    tensors as (buffer, byte offset, pixel pitch) views."""
    xv = _view(x)
    arr = (L.DwView * len(ys))(*[_view(v) for v in ys])
    backend._check(L.load().dw_maxpool_chain_i8_view(backend.handle, ctypes.byref(xv), arr, len(ys), n, h, w, c, k))


def maxpool_i8_view(backend, x, y, n, h, w, c, k_h, k_w, s_h, s_w, pads):
    xv, yv = _view(x), _view(y)
    pt, pl, pb, pr = pads
    backend._check(L.load().dw_maxpool_i8_view(backend.handle, ctypes.byref(xv), ctypes.byref(yv), n, h, w, c, k_h,
                                               k_w, s_h, s_w, pt, pl, pb, pr))


def concat_i8(backend, xs, channels, pixels, y):
    arr = (ctypes.c_void_p * len(xs))(*[b.handle.value for b in xs])
    cs = (ctypes.c_int32 * len(channels))(*channels)
    backend._check(L.load().dw_concat_i8(backend.handle, ctypes.cast(arr, L.PVP), cs, len(xs), pixels, y.handle))


def slice_c_i8(backend, x, y, pixels, c_total, c0, c_len):
    backend._check(L.load().dw_slice_c_i8(backend.handle, x.handle, y.handle, pixels, c_total, c0, c_len))


def resize_nearest_i8(backend, x, y, n, h_in, w_in, h_out, w_out, c):
    backend._check(L.load().dw_resize_nearest_i8(backend.handle, x.handle, y.handle, n, h_in, w_in, h_out, w_out, c))


# ---------------------------------------------------------------------------
# fp16 path (binary16 buffers; conversions as F16::from_f32 / F16::to_f32,
# crates/dragonwing-core/src/dtype.rs:164-263)
# ---------------------------------------------------------------------------

def conv2d_fp16_nhwc(backend, input, kernel, output, n, h_in, w_in, c_in, c_out, k_h, k_w, stride_h, stride_w,
                     pad_h, pad_w):
    """crates/dragonwing-vulkan/src/ops.rs:1385: fp16 conv, f32 accumulation, HWIO kernel."""
    backend._check(L.load().dw_conv2d_fp16_nhwc(backend.handle, input.handle, kernel.handle, output.handle,
                                                n, h_in, w_in, c_in, c_out, k_h, k_w, stride_h, stride_w, pad_h, pad_w))


def gemm_fp16(backend, a, b, c, m, n, k):
    """crates/dragonwing-vulkan/src/ops.rs:1184: C[m,n] = A[m,k] @ B[k,n] in fp16, f32 accumulation."""
    backend._check(L.load().dw_gemm_f16(backend.handle, a.handle, b.handle, c.handle, m, n, k))


def add_fp16(backend, a, b, y):
    """crates/dragonwing-vulkan/src/ops.rs:933: y = a + b (fp16)."""
    backend._check(L.load().dw_add_f16(backend.handle, a.handle, b.handle, y.handle))


def relu_fp16(backend, x):
    """crates/dragonwing-vulkan/src/ops.rs:856: in-place ReLU (fp16)."""
    backend._check(L.load().dw_relu_f16(backend.handle, x.handle))


def add_relu_fp16(backend, a, b, y):
    """add_fp16 then relu_fp16 in one pass."""
    backend._check(L.load().dw_add_relu_f16(backend.handle, a.handle, b.handle, y.handle))


def prepare_weights_f16(backend: CudaBackend, desc: ConvDesc, w_hwio: CudaBuffer) -> CudaBuffer:
    """HWIO (or depthwise [kh,kw,C,mult]) fp16 kernel -> the kernels' layout (once)."""
    out = ctypes.c_void_p()
    d = desc.to_c()
    backend._check(L.load().dw_prepare_weights_f16(backend.handle, ctypes.byref(d), w_hwio.handle, ctypes.byref(out)))
    return CudaBuffer(backend, out, L.load().dw_buf_len(out))


def conv2d_f16(backend: CudaBackend, desc: ConvDesc, x: CudaBuffer, w_prep: CudaBuffer, bias, y: CudaBuffer):
    """fp16 conv + f16 bias (rounded as the CPU runtime does) + optional ReLU
    (desc.epilogue EPI_NONE or EPI_RELU)."""
    d = desc.to_c()
    backend._check(L.load().dw_conv2d_f16(backend.handle, ctypes.byref(d), x.handle, w_prep.handle, _h(bias),
                                          y.handle))


def conv2d_add_f16(backend: CudaBackend, desc: ConvDesc, x: CudaBuffer, w_prep: CudaBuffer, bias, residual,
                   y: CudaBuffer):
    """fp16 conv + bias, then + residual (add_fp16), then ReLU if desc.epilogue
    is EPI_RELU: the Conv -> Add -> Relu of a residual block in one op."""
    d = desc.to_c()
    backend._check(L.load().dw_conv2d_add_f16(backend.handle, ctypes.byref(d), x.handle, w_prep.handle, _h(bias),
                                              residual.handle, y.handle))


def prepare_gemm_b_f16(backend: CudaBackend, b_kn: CudaBuffer, k: int, n: int) -> CudaBuffer:
    out = ctypes.c_void_p()
    backend._check(L.load().dw_prepare_gemm_b_f16(backend.handle, b_kn.handle, k, n, ctypes.byref(out)))
    return CudaBuffer(backend, out, 2 * k * n)


def gemm_f16_bias(backend: CudaBackend, a, b_prep, bias, y, m, n, k, relu=False):
    """Gemm F16 + bias as the CPU runtime runs it (runtime.rs:1247-1275)."""
    backend._check(L.load().dw_gemm_f16_bias(backend.handle, a.handle, b_prep.handle, _h(bias), y.handle, m, n, k,
                                             1 if relu else 0))


def maxpool_f16(backend, x, y, n, h, w, c, k_h, k_w, s_h, s_w, pads=(0, 0, 0, 0)):
    pt, pl, pb, pr = pads
    backend._check(L.load().dw_maxpool_f16(backend.handle, x.handle, y.handle, n, h, w, c, k_h, k_w, s_h, s_w,
                                           pt, pl, pb, pr))


def global_avgpool_f16(backend, x, y, n, h, w, c):
    backend._check(L.load().dw_global_avgpool_f16(backend.handle, x.handle, y.handle, n, h, w, c))


def cast_f32_to_f16(backend, x, y, pixels, c_src, c_dst=None):
    backend._check(L.load().dw_cast_f32_to_f16(backend.handle, x.handle, y.handle, pixels, c_src,
                                               c_src if c_dst is None else c_dst))


def cast_f16_to_f32(backend, x, y):
    backend._check(L.load().dw_cast_f16_to_f32(backend.handle, x.handle, y.handle))


def unfold_w_f32_to_f16(backend, x, y, n, h, w, c, k_w, stride_w, pad_l, w_out, c_dst):
    """Horizontal unfold + F16 conversion of a few-channel f32 image (the
    first conv's input layout for the tensor cores; contract in include/dw_cuda.h)."""
    backend._check(L.load().dw_unfold_w_f32_to_f16(backend.handle, x.handle, y.handle, n, h, w, c, k_w, stride_w,
                                                   pad_l, w_out, c_dst))


def conv2d_stem_u8_i8(backend: CudaBackend, desc: ConvDesc, x_u8: CudaBuffer, in_scale: float, w_hwio: CudaBuffer,
                      bias, M, D, y: CudaBuffer):
    """The input stem in one pass: the uint8 image's quantisation and the fused
    3x3 conv on its 3 channels (contract in include/dw_cuda.h)."""
    d = desc.to_c()
    backend._check(L.load().dw_conv2d_stem_u8_i8(backend.handle, ctypes.byref(d), x_u8.handle, float(in_scale),
                                                 w_hwio.handle, _h(bias), _h(M), _h(D), y.handle))


def im2col_u8_to_i8(backend, x, y, n, h, w, c, k_h, k_w, s_h, s_w, p_t, p_l, h_out, w_out, c_dst, scale):
    """im2col of a uint8 image fused with its quantisation (contract in include/dw_cuda.h)."""
    backend._check(L.load().dw_im2col_u8_to_i8(backend.handle, x.handle, y.handle, n, h, w, c, k_h, k_w, s_h, s_w,
                                               p_t, p_l, h_out, w_out, c_dst, float(scale)))


# ---------------------------------------------------------------------------
# YOLOv8 Detect tail and detection post-processing
# (crates/dragonwing-onnx/src/postprocess.rs)
# ---------------------------------------------------------------------------

YOLO_ANCHOR_ROWS, YOLO_NMS_AGNOSTIC, YOLO_NO_NMS = L.YOLO_ANCHOR_ROWS, L.YOLO_NMS_AGNOSTIC, L.YOLO_NO_NMS

# Detection (postprocess.rs:12-19): bbox [x1, y1, x2, y2], class_id, confidence.
DETECTION_DTYPE = np.dtype([("bbox", "<f4", (4,)), ("class_id", "<u4"), ("confidence", "<f4")])


@dataclass
class YoloDetectDesc:
    """The Detect head after its last convolutions: per level the (h, w) grid,
    the stride and the dequantisation scales of the int8 box tensor
    [n, h, w, 4*reg_max] and class tensor [n, h, w, num_classes]."""

    n: int
    num_classes: int
    grids: list
    strides: list
    box_scales: list
    cls_scales: list
    reg_max: int = 16

    @property
    def anchors(self) -> int:
        return sum(h * w for h, w in self.grids)

    def to_c(self) -> L.DwYoloDetectDesc:
        d = L.DwYoloDetectDesc()
        d.n, d.num_classes, d.reg_max, d.num_levels = self.n, self.num_classes, self.reg_max, len(self.grids)
        for i, (h, w) in enumerate(self.grids):
            d.h[i], d.w[i] = h, w
            d.stride[i], d.box_scale[i], d.cls_scale[i] = self.strides[i], self.box_scales[i], self.cls_scales[i]
        return d


def prepare_yolo_detect(backend: CudaBackend, desc: YoloDetectDesc) -> CudaBuffer:
    """The sigmoid and softmax tables of the head (once per model)."""
    out = ctypes.c_void_p()
    d = desc.to_c()
    backend._check(L.load().dw_prepare_yolo_detect(backend.handle, ctypes.byref(d), ctypes.byref(out)))
    return CudaBuffer(backend, out, L.load().dw_buf_len(out))


def yolo_detect_i8(backend: CudaBackend, desc: YoloDetectDesc, tables: CudaBuffer, boxes, clss, out: CudaBuffer):
    """int8 box/class head outputs -> the model output f32 [n, 4 + nc, anchors]."""
    d = desc.to_c()
    nb = len(boxes)
    bx = (ctypes.c_void_p * nb)(*[b.handle.value for b in boxes])
    cx = (ctypes.c_void_p * nb)(*[b.handle.value for b in clss])
    backend._check(L.load().dw_yolo_detect_i8(backend.handle, ctypes.byref(d), tables.handle,
                                              ctypes.cast(bx, L.PVP), ctypes.cast(cx, L.PVP), out.handle))


def postprocess_yolo_workspace(n: int, num_detections: int) -> int:
    return int(L.load().dw_postprocess_yolo_workspace(n, num_detections))


def postprocess_yolo_device(backend: CudaBackend, raw: CudaBuffer, n: int, num_classes: int, num_detections: int,
                            img_width: int, img_height: int, conf_threshold: float, iou_threshold: float,
                            flags: int, workspace, dets: CudaBuffer, counts: CudaBuffer):
    """postprocess_yolo for n images, results left on the device: image i's
    detections are dets[i*num_detections : i*num_detections + counts[i]]."""
    backend._check(L.load().dw_postprocess_yolo(backend.handle, raw.handle, n, num_classes, num_detections,
                                                img_width, img_height, float(conf_threshold),
                                                float(iou_threshold), flags, _h(workspace), _h(dets),
                                                counts.handle))


def detections_from_host(dets: np.ndarray, counts: np.ndarray, num_detections: int) -> list:
    """Splits the device layout (read back) into one Detection array per image."""
    recs = np.frombuffer(np.ascontiguousarray(dets).tobytes(), DETECTION_DTYPE)
    return [recs[i * num_detections:i * num_detections + int(c)].copy() for i, c in enumerate(counts)]


def postprocess_yolo(backend: CudaBackend, raw: CudaBuffer, n: int, num_classes: int, num_detections: int,
                     img_width: int, img_height: int, conf_threshold: float, iou_threshold: float,
                     flags: int = 0) -> list:
    """postprocess_yolo (postprocess.rs:319-340) on a device-resident model
    output: returns, per image, its detections as a DETECTION_DTYPE array in
    the reference's order."""
    counts = backend.alloc(4 * n)
    dets = backend.alloc(n * num_detections * DETECTION_DTYPE.itemsize) if num_detections else None
    try:
        postprocess_yolo_device(backend, raw, n, num_classes, num_detections, img_width, img_height,
                                conf_threshold, iou_threshold, flags, None, dets, counts)
        cnt = backend.download_array(counts, np.int32)
        raw_d = backend.download_array(dets, np.uint8) if dets is not None else np.zeros(0, np.uint8)
    finally:
        counts.free()
        if dets is not None:
            dets.free()
    return detections_from_host(raw_d, cnt, num_detections)
