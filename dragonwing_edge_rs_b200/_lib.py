"""ctypes binding of libdragonwing_cuda.so (include/dw_cuda.h).

The library is built in-tree (``python -m dragonwing_edge_rs_b200.build``).
Loading fails loudly when it is missing: there is no CPU fallback.
"""
from __future__ import annotations

import ctypes
import os

PKG = os.path.dirname(os.path.abspath(__file__))
LIB_PATH = os.path.join(PKG, "libdragonwing_cuda.so")

# dw_status
DW_OK = 0
DW_ERR_INVALID_ARG = 1
DW_ERR_SIZE_MISMATCH = 2
DW_ERR_UNSUPPORTED = 3
DW_ERR_OOM = 4
DW_ERR_TIMEOUT = 5
DW_ERR_DEVICE = 6
DW_ERR_KERNEL_WAIT_EXPIRED = 7
STATUS_NAMES = {
    0: "DW_OK", 1: "DW_ERR_INVALID_ARG", 2: "DW_ERR_SIZE_MISMATCH", 3: "DW_ERR_UNSUPPORTED", 4: "DW_ERR_OOM",
    5: "DW_ERR_TIMEOUT", 6: "DW_ERR_DEVICE", 7: "DW_ERR_KERNEL_WAIT_EXPIRED",
}

# dw_epilogue
EPI_NONE, EPI_RELU, EPI_RELU6, EPI_SILU = 0, 1, 2, 3
# dw_conv_path
PATH_AUTO, PATH_DIRECT, PATH_UMMA = 0, 1, 2
# dw_dw_variant
DWV_AUTO, DWV_SLAB, DWV_STREAM2, DWV_STREAM2X2, DWV_STREAM4 = 0, 1, 2, 3, 4


class DwConfig(ctypes.Structure):
    _fields_ = [("wait_cap_ms", ctypes.c_uint32), ("trace", ctypes.c_int32), ("conv_path", ctypes.c_int32),
                ("dw_variant", ctypes.c_int32), ("reserved", ctypes.c_int32 * 4)]


class DwConvDesc(ctypes.Structure):
    _fields_ = [(n, ctypes.c_int32) for n in (
        "n", "h", "w", "c_in", "c_out", "k_h", "k_w", "stride_h", "stride_w",
        "pad_t", "pad_l", "pad_b", "pad_r", "group", "epilogue", "q6")] + [("inv_s_out", ctypes.c_float)]


# dw_yolo_flags
YOLO_ANCHOR_ROWS, YOLO_NMS_AGNOSTIC, YOLO_NO_NMS = 1, 2, 4
YOLO_MAX_LEVELS = 4


class DwYoloDetectDesc(ctypes.Structure):
    _fields_ = [("n", ctypes.c_int32), ("num_classes", ctypes.c_int32), ("reg_max", ctypes.c_int32),
                ("num_levels", ctypes.c_int32), ("h", ctypes.c_int32 * YOLO_MAX_LEVELS),
                ("w", ctypes.c_int32 * YOLO_MAX_LEVELS), ("stride", ctypes.c_float * YOLO_MAX_LEVELS),
                ("box_scale", ctypes.c_float * YOLO_MAX_LEVELS), ("cls_scale", ctypes.c_float * YOLO_MAX_LEVELS)]


class DwView(ctypes.Structure):
    """dw_view: a channel range (byte offset, pixel pitch) of a wider NHWC int8 tensor."""
    _fields_ = [("buf", ctypes.c_void_p), ("offset", ctypes.c_size_t), ("pitch", ctypes.c_int32)]


# Every exported function with its argument types (restype is dw_status unless listed).
vp, sz, i32, u32, f32 = ctypes.c_void_p, ctypes.c_size_t, ctypes.c_int, ctypes.c_uint32, ctypes.c_float
PDESC = ctypes.POINTER(DwConvDesc)
PVP = ctypes.POINTER(ctypes.c_void_p)
SIGNATURES = {
    "dw_name": ([], ctypes.c_char_p),
    "dw_version": ([], ctypes.c_char_p),
    "dw_create": ([i32, ctypes.POINTER(DwConfig), PVP], i32),
    "dw_destroy": ([vp], None),
    "dw_last_error": ([vp], ctypes.c_char_p),
    "dw_alloc": ([vp, sz, PVP], i32),
    "dw_buf_wrap": ([vp, vp, sz, PVP], i32),
    "dw_free": ([vp, vp], i32),
    "dw_buf_len": ([vp], sz),
    "dw_buf_device_ptr": ([vp], vp),
    "dw_upload": ([vp, vp, vp, sz], i32),
    "dw_download": ([vp, vp, vp, sz], i32),
    "dw_upload_async": ([vp, vp, sz, vp, sz], i32),
    "dw_download_async": ([vp, vp, sz, vp, sz], i32),
    "dw_synchronize": ([vp, u32], i32),
    "dw_host_alloc": ([vp, sz, PVP], i32),
    "dw_host_free": ([vp, vp], i32),
    "dw_stream": ([vp], vp),
    "dw_sm_count": ([vp], i32),
    "dw_launch_count": ([vp], ctypes.c_uint64),
    "dw_scratch_bytes": ([vp], ctypes.c_size_t),
    "dw_debug_expire_wait": ([vp, u32], i32),
    "dw_capture_begin": ([vp], i32),
    "dw_capture_end": ([vp, PVP], i32),
    "dw_graph_launch": ([vp, vp], i32),
    "dw_graph_destroy": ([vp], None),
    "dw_prepare_weights_i8": ([vp, PDESC, vp, PVP], i32),
    "dw_conv2d_i8": ([vp, PDESC, vp, vp, vp, vp, vp, vp], i32),
    "dw_conv2d_requant_relu_i8": ([vp, vp, vp, vp] + [sz] * 11 + [f32, i32], i32),
    "dw_conv2d_requant_relu_i8_noalloc": ([vp, vp, vp, vp] + [sz] * 11 + [f32, i32], i32),
    "dw_conv2d_i8_nhwc": ([vp, vp, vp, vp] + [sz] * 11, i32),
    "dw_gemm_i8": ([vp, vp, vp, vp, sz, sz, sz], i32),
    "dw_prepare_gemm_b_i8": ([vp, vp, sz, sz, PVP], i32),
    "dw_qgemm_i8": ([vp, vp, vp, vp, vp, vp, sz, sz, sz, i32, i32], i32),
    "dw_requantize_i32_to_i8": ([vp, vp, vp, f32], i32),
    "dw_relu_i8": ([vp, vp, vp], i32),
    "dw_add_i8": ([vp, vp, vp, vp, f32, f32], i32),
    "dw_quantize_f32_to_i8": ([vp, vp, vp, f32], i32),
    "dw_quantize_u8_to_i8": ([vp, vp, vp, f32], i32),
    "dw_dequantize_i8_to_f32": ([vp, vp, vp, f32], i32),
    "dw_maxpool_i8": ([vp, vp, vp] + [sz] * 12, i32),
    "dw_concat_i8": ([vp, PVP, ctypes.POINTER(ctypes.c_int32), ctypes.c_int32, sz, vp], i32),
    "dw_slice_c_i8": ([vp, vp, vp, sz, sz, sz, sz], i32),
    "dw_resize_nearest_i8": ([vp, vp, vp] + [sz] * 6, i32),
    "dw_copy_async": ([vp, vp, sz, vp, sz, sz], i32),
    "dw_event_create": ([vp, PVP], i32),
    "dw_event_destroy": ([vp], None),
    "dw_event_record": ([vp, vp], i32),
    "dw_stream_wait_event": ([vp, vp], i32),
    # fp16 path
    "dw_prepare_weights_f16": ([vp, ctypes.POINTER(DwConvDesc), vp, PVP], i32),
    "dw_conv2d_f16": ([vp, ctypes.POINTER(DwConvDesc), vp, vp, vp, vp], i32),
    "dw_conv2d_add_f16": ([vp, ctypes.POINTER(DwConvDesc), vp, vp, vp, vp, vp], i32),
    "dw_conv2d_fp16_nhwc": ([vp, vp, vp, vp] + [sz] * 11, i32),
    "dw_gemm_f16": ([vp, vp, vp, vp, sz, sz, sz], i32),
    "dw_prepare_gemm_b_f16": ([vp, vp, sz, sz, PVP], i32),
    "dw_gemm_f16_bias": ([vp, vp, vp, vp, vp, sz, sz, sz, i32], i32),
    "dw_add_f16": ([vp, vp, vp, vp], i32),
    "dw_add_relu_f16": ([vp, vp, vp, vp], i32),
    "dw_relu_f16": ([vp, vp], i32),
    "dw_maxpool_f16": ([vp, vp, vp] + [sz] * 12, i32),
    "dw_global_avgpool_f16": ([vp, vp, vp] + [sz] * 4, i32),
    "dw_cast_f32_to_f16": ([vp, vp, vp, sz, sz, sz], i32),
    "dw_cast_f16_to_f32": ([vp, vp, vp], i32),
    "dw_unfold_w_f32_to_f16": ([vp, vp, vp] + [sz] * 9, i32),
    "dw_im2col_u8_to_i8": ([vp, vp, vp] + [sz] * 13 + [f32], i32),
    "dw_conv2d_stem_u8_i8": ([vp, PDESC, vp, f32, vp, vp, vp, vp, vp], i32),
    # channel-range views
    "dw_conv2d_i8_view": ([vp, PDESC, ctypes.POINTER(DwView), vp, vp, vp, vp, ctypes.POINTER(DwView)], i32),
    "dw_conv2d_add_i8_view": ([vp, PDESC, ctypes.POINTER(DwView), vp, vp, vp, vp, ctypes.POINTER(DwView), f32, f32,
                               ctypes.POINTER(DwView)], i32),
    "dw_add_i8_view": ([vp, ctypes.POINTER(DwView), ctypes.POINTER(DwView), ctypes.POINTER(DwView), sz, sz, f32, f32],
                       i32),
    "dw_maxpool_i8_view": ([vp, ctypes.POINTER(DwView), ctypes.POINTER(DwView)] + [sz] * 12, i32),
    "dw_maxpool_chain_i8_view": ([vp, ctypes.POINTER(DwView), ctypes.POINTER(DwView), i32] + [sz] * 5, i32),
    # YOLOv8 Detect tail and post-processing
    "dw_prepare_yolo_detect": ([vp, ctypes.POINTER(DwYoloDetectDesc), PVP], i32),
    "dw_yolo_detect_i8": ([vp, ctypes.POINTER(DwYoloDetectDesc), vp, PVP, PVP, vp], i32),
    "dw_postprocess_yolo_workspace": ([sz, sz], sz),
    "dw_postprocess_yolo": ([vp, vp, sz, sz, sz, u32, u32, f32, f32, ctypes.c_int32, vp, vp, vp], i32),
}

_lib = None


def load() -> ctypes.CDLL:
    """Loads the in-tree library (raises if it has not been built)."""
    global _lib
    if _lib is None:
        if not os.path.exists(LIB_PATH):
            raise RuntimeError(
                f"{LIB_PATH} is missing: build it with `python -m dragonwing_edge_rs_b200.build` "
                "(the B200 backend has no CPU fallback)")
        lib = ctypes.CDLL(LIB_PATH)
        for name, (args, res) in SIGNATURES.items():
            fn = getattr(lib, name)
            fn.argtypes = args
            fn.restype = res
        _lib = lib
    return _lib
