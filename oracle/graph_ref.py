"""CPU execution of a fused-INT8 graph with the oracle ops.

TEST INFRASTRUCTURE ONLY: the checker for CudaGraphRuntime and the timed CPU
baseline of bench.py.  Each op maps to the oracle restatement of the
reference op it stands for: the fused conv to the contract composition of
conv2d_i8_nhwc / requantize / relu (crates/dragonwing-cpu/src/ops.rs:3086-3142,
3366-3386, 3301-3319), AddQuantized to add_i8 (ops.rs:3176-3209), MaxPool to
maxpool2d (ops.rs:1513-1551), Concat/Split to concat_f32/split_f32 on int8
bytes (ops.rs:2141-2246, 2407), Resize to resize_f32 Nearest (ops.rs:2320-2348),
QuantizeU8 to u8*(1/255) -> quantize_f32_to_i8 (ops.rs:3503-3525),
YoloDetect to the exported Detect tail's f32 ops (softmax_f32, the DFL conv,
Sub/Add/Div/Mul, sigmoid_f32_scalar; dwref_yolo_detect_i8), YoloPostprocess to
postprocess_yolo (crates/dragonwing-onnx/src/postprocess.rs:319-340).
The unfused int8 ops the reference's quantizer emits (quantize.rs:176-249) run
as themselves: Conv to conv2d_i8_nhwc's int32 accumulators (+ the bias),
Requantize to requantize_i32_to_i8 per channel, Relu to relu_i8, Clip to the
int8 bounds quantize(min) / quantize(max), DequantizeLinear / Sigmoid / Mul /
QuantizeLinear to the f32 SiLU chain (sigmoid_f32_scalar with the host libm's
expf, ops.rs:1865-1870; quantize_f32_to_i8).

UnfoldF32ToF16 (a device lowering of the input conv, see
dragonwing_edge_rs_b200.graph.lower_unfold_stem_f16) is the input conversion
laid out as a horizontal unfold.  fp16 graphs follow the reference's F16 CPU
runtime: CastF32ToF16 is the input
conversion (runtime.rs:842-851), Conv2dF16 is conv2d_fp16_nhwc (ops.rs:1442-1511)
plus the runtime's bias and Relu steps (runtime.rs:1483-1497, 967-971),
AddF16 is add_fp16 (ops.rs:434-446) + Relu, MaxPoolF16 and
GlobalAveragePoolF16 are runtime.rs:1545-1563 and 1155-1170, GemmF16 is
gemm_fp16 (ops.rs:461-481) + the bias step (runtime.rs:1264-1275).  fp16
tensors are held as uint16 bit patterns.  """
from __future__ import annotations

import numpy as np

from dragonwing_edge_rs_b200 import quantization as Q
from dragonwing_edge_rs_b200.graph import conv_desc_of
from oracle import dwref


def run_graph(graph, feeds: dict, threads: int = 1, batch_slice=None, return_all: bool = False) -> dict:
    """Runs `graph` on the CPU.  `feeds` maps input names to arrays.  With
    `batch_slice` = (b0, b1), only images b0..b1-1 are computed (every op is
    per-image), which bounds the CPU time of large-batch graphs.  `return_all`
    returns every tensor, not only the graph outputs."""
    b0, b1 = batch_slice if batch_slice else (0, None)
    vals = {}
    for name in graph.inputs:
        t = graph.tensors[name]
        arr = np.asarray(feeds[name]).reshape(t.shape)
        vals[name] = np.ascontiguousarray(arr[b0:b1])

    def shape_of(name):
        t = graph.tensors[name]
        n = vals[graph.inputs[0]].shape[0]
        return (n,) + tuple(t.shape[1:])

    for op in graph.ops:
        t = op.op_type
        if t in ("Conv2dRequantReluI8Nhwc", "Conv2dStemU8I8"):
            d = op.params["desc"]
            x = vals[op.inputs[0]]
            if t == "Conv2dStemU8I8":  # device lowering of QuantizeU8 + the input conv: the same two steps
                x = dwref.quantize_u8_to_i8(x, op.params["in_scale"]).reshape(x.shape)
            n = x.shape[0]
            od = dwref.conv_desc(n, d.h, d.w, d.c_in, d.c_out, d.k_h, d.k_w, d.stride_h, d.stride_w, d.pads,
                                 d.group, d.epilogue, d.q6, d.inv_s_out)
            w = graph.initializers[op.inputs[1]]
            bias = graph.initializers[op.inputs[2]]
            M = graph.initializers[op.inputs[3]]
            D = graph.initializers[op.inputs[4]]
            y = dwref.conv2d_fused_i8(x, w, bias, M, D if d.epilogue == dwref.EPI_SILU else None, od, threads)
            vals[op.outputs[0]] = y.reshape(shape_of(op.outputs[0]))
        elif t == "Conv":
            # the unfused int8 conv: conv2d_i8_nhwc (ops.rs:3086-3142) to int32
            # accumulators, plus the int32 bias with wrapping adds
            d = conv_desc_of(graph, op)
            x = vals[op.inputs[0]]
            n = x.shape[0]
            od = dwref.conv_desc(n, d.h, d.w, d.c_in, d.c_out, d.k_h, d.k_w, d.stride_h, d.stride_w, d.pads,
                                 d.group, 0, 127, 0.0)
            acc = dwref.conv2d_acc_i32(x, graph.initializers[op.inputs[1]], od, threads)
            if len(op.inputs) > 2 and op.inputs[2]:
                bias = np.asarray(graph.initializers[op.inputs[2]], np.int32)
                acc = (acc.reshape(-1, d.c_out).astype(np.int64) + bias).astype(np.uint32).view(np.int32)
            vals[op.outputs[0]] = acc.reshape(shape_of(op.outputs[0]))
        elif t == "Requantize":
            # requantize_i32_to_i8_scalar (ops.rs:3380-3386) per output channel:
            # (i8) roundf(clamp((f32)acc * M[c], -128, 127))
            acc = vals[op.inputs[0]]
            c = acc.shape[-1]
            if len(op.inputs) > 1:
                M = np.asarray(graph.initializers[op.inputs[1]], np.float32)
            else:
                M = np.full(c, np.float32(op.params["scale"]), np.float32)
            f = acc.astype(np.float32) * M
            q = Q.roundf_away(np.clip(f, np.float32(-128.0), np.float32(127.0)))
            vals[op.outputs[0]] = q.astype(np.int8)
        elif t == "Relu":
            x = vals[op.inputs[0]]
            vals[op.outputs[0]] = dwref.relu_i8(x).reshape(x.shape)
        elif t == "Clip":
            # Clip on an int8 tensor of scale s: bounds quantised with
            # quantize_f32_to_i8 (ops.rs:3503-3525)
            x = vals[op.inputs[0]]
            s = graph.tensors[op.inputs[0]].scale
            lo = int(dwref.quantize_f32_to_i8(np.array([op.params["min"]], np.float32), s)[0])
            hi = int(dwref.quantize_f32_to_i8(np.array([op.params["max"]], np.float32), s)[0])
            vals[op.outputs[0]] = np.minimum(np.maximum(x, np.int8(lo)), np.int8(hi)).astype(np.int8)
        elif t == "DequantizeLinear":
            # int32 accumulators (bias included) to f32 with the per-channel D = s_in * s_w[c]
            acc = vals[op.inputs[0]]
            D = np.asarray(graph.initializers[op.inputs[1]], np.float32)
            vals[op.outputs[0]] = acc.astype(np.float32) * D
        elif t == "Sigmoid":
            x = vals[op.inputs[0]]
            vals[op.outputs[0]] = dwref.sigmoid_f32(x).reshape(x.shape)
        elif t == "Mul":
            vals[op.outputs[0]] = vals[op.inputs[0]] * vals[op.inputs[1]]
        elif t == "SiLU":
            # x * sigmoid(x): the fused form of Mul(x, Sigmoid(x)), same two roundings
            x = vals[op.inputs[0]]
            vals[op.outputs[0]] = x * dwref.sigmoid_f32(x).reshape(x.shape)
        elif t == "QuantizeLinear":
            x = vals[op.inputs[0]]
            vals[op.outputs[0]] = dwref.quantize_f32_to_i8(x, op.params["scale"]).reshape(x.shape)
        elif t == "Conv2dAddI8":  # device fusion of Conv2dRequantReluI8Nhwc -> AddQuantized(residual, conv)
            d = op.params["desc"]
            x = vals[op.inputs[0]]
            n = x.shape[0]
            od = dwref.conv_desc(n, d.h, d.w, d.c_in, d.c_out, d.k_h, d.k_w, d.stride_h, d.stride_w, d.pads,
                                 d.group, d.epilogue, d.q6, d.inv_s_out)
            y = dwref.conv2d_fused_i8(x, graph.initializers[op.inputs[1]], graph.initializers[op.inputs[2]],
                                      graph.initializers[op.inputs[3]], graph.initializers[op.inputs[4]]
                                      if d.epilogue == dwref.EPI_SILU else None, od, threads)
            res = vals[op.inputs[5]]
            z = dwref.add_i8(res, y.reshape(res.shape), op.params["ra"], op.params["rb"])
            vals[op.outputs[0]] = z.reshape(shape_of(op.outputs[0]))
        elif t == "AddQuantized":
            a, b = vals[op.inputs[0]], vals[op.inputs[1]]
            y = dwref.add_i8(a, b, op.params["scale_a_over_out"], op.params["scale_b_over_out"])
            vals[op.outputs[0]] = y.reshape(a.shape)
        elif t == "MaxPoolChainI8":  # device fusion of chained stride-1 MaxPools (SPPF)
            x = vals[op.inputs[0]]
            n, h, w, c = x.shape
            k = op.params["k"]
            p = k // 2
            for o in op.outputs:
                x = dwref.maxpool_i8(x, n, h, w, c, k, k, 1, 1, (p, p, p, p)).reshape(n, h, w, c)
                vals[o] = x
        elif t == "MaxPool":
            x = vals[op.inputs[0]]
            n, h, w, c = x.shape
            k, s, p = op.params["k"], op.params["s"], op.params["pad"]
            vals[op.outputs[0]] = dwref.maxpool_i8(x, n, h, w, c, k, k, s, s, (p, p, p, p)).reshape(shape_of(op.outputs[0]))
        elif t == "Concat":
            xs = [vals[i] for i in op.inputs]
            n, h, w, _ = xs[0].shape
            vals[op.outputs[0]] = dwref.concat_c_i8(xs, op.params["channels"], n * h * w).reshape(shape_of(op.outputs[0]))
        elif t == "Split":
            x = vals[op.inputs[0]]
            c0, cl = op.params["c0"], op.params["c_len"]
            vals[op.outputs[0]] = np.ascontiguousarray(x[..., c0:c0 + cl])
        elif t == "Resize":
            x = vals[op.inputs[0]]
            n, h, w, c = x.shape
            _, ho, wo, _ = shape_of(op.outputs[0])
            vals[op.outputs[0]] = dwref.resize_nearest_i8(x, n, h, w, ho, wo, c).reshape(n, ho, wo, c)
        elif t == "Im2colU8ToI8":  # device lowering of QuantizeU8 + the input conv (same integers)
            vals[op.outputs[0]] = im2col_u8_op(op, vals[op.inputs[0]])
        elif t == "QuantizeU8":
            x = vals[op.inputs[0]]
            vals[op.outputs[0]] = dwref.quantize_u8_to_i8(x, op.params["scale"]).reshape(x.shape)
        elif t == "Dequantize":
            x = vals[op.inputs[0]]
            vals[op.outputs[0]] = dwref.dequantize_i8_to_f32(x, op.params["scale"]).reshape(x.shape)
        elif t == "YoloDetect":
            pr = op.params
            boxes, clss = [vals[x] for x in op.inputs[0::2]], [vals[x] for x in op.inputs[1::2]]
            vals[op.outputs[0]] = dwref.yolo_detect_i8(boxes, clss, pr["strides"], pr["box_scales"],
                                                       pr["cls_scales"], pr["reg_max"])
        elif t == "YoloPostprocess":
            vals[op.outputs[0]], vals[op.outputs[1]] = postprocess_op(op, vals[op.inputs[0]])
        elif t == "CastF32ToF16":
            x = vals[op.inputs[0]]
            vals[op.outputs[0]] = dwref.f16_from_f32_array(x).reshape(x.shape)
        elif t == "UnfoldF32ToF16":
            vals[op.outputs[0]] = unfold_f16_op(op, vals[op.inputs[0]])
        elif t == "Conv2dF16":
            vals[op.outputs[0]] = conv_f16_op(graph, op, vals[op.inputs[0]], threads)
        elif t == "Conv2dAddF16":  # Conv2dF16 (no ReLU) -> AddF16 (ReLU per desc), fused on the device
            y = conv_f16_op(graph, op, vals[op.inputs[0]], threads, relu=False)
            y = dwref.add_f16(y, vals[op.inputs[3]])
            if op.params["desc"].epilogue == dwref.EPI_RELU:
                y = dwref.relu_f16(y)
            vals[op.outputs[0]] = y.reshape(shape_of(op.outputs[0]))
        elif t == "AddF16":
            a, b = vals[op.inputs[0]], vals[op.inputs[1]]
            y = dwref.add_f16(a, b)
            if op.params.get("relu"):
                y = dwref.relu_f16(y)
            vals[op.outputs[0]] = y.reshape(a.shape)
        elif t == "MaxPoolF16":
            x = vals[op.inputs[0]]
            n, h, w, c = x.shape
            k, s, p = op.params["k"], op.params["s"], op.params["pad"]
            y = dwref.maxpool_f16(x, n, h, w, c, k, k, s, s, (p, p, p, p))
            vals[op.outputs[0]] = y.reshape(shape_of(op.outputs[0]))
        elif t == "GlobalAveragePoolF16":
            x = vals[op.inputs[0]]
            n, h, w, c = x.shape
            vals[op.outputs[0]] = dwref.gap_f16(x, n, h, w, c).reshape(n, c)
        elif t == "GemmF16":
            vals[op.outputs[0]] = gemm_f16_op(graph, op, vals[op.inputs[0]], threads)
        elif t == "CastF16ToF32":
            x = vals[op.inputs[0]]
            vals[op.outputs[0]] = dwref.f16_to_f32_array(x).reshape(x.shape)
        else:
            raise ValueError(f"unsupported op {t}")
    if return_all:
        return vals
    return {name: vals[name] for name in graph.outputs}


def postprocess_op(op, raw):
    """YoloPostprocess: postprocess_yolo per image, laid out as the device op
    leaves it (records [n, A]; the first counts[i] of image i are its
    detections, the rest zero)."""
    pr = op.params
    n, A = raw.shape[0], pr["num_detections"]
    dets = np.zeros((n, A), dwref.DETECTION_DTYPE)
    cnt = np.zeros(n, np.int32)
    for i in range(n):
        d = dwref.postprocess_yolo(raw[i], pr["nc"], A, pr["img_width"], pr["img_height"], pr["conf_threshold"],
                                   pr["iou_threshold"], pr["flags"])
        dets[i, :len(d)] = d
        cnt[i] = len(d)
    return dets.view(np.uint8).reshape(n, A, dwref.DETECTION_DTYPE.itemsize), cnt


def conv_f16_op(graph, op, x, threads=1, relu=None):
    """One Conv2dF16 op on uint16 NHWC input `x` (its real channels only);
    `relu` overrides the descriptor's epilogue."""
    d = op.params["desc"]
    n, h, w, c_in = x.shape
    wt = graph.initializers[op.inputs[1]].view(np.uint16)
    bias = graph.initializers[op.inputs[2]].view(np.uint16)
    pt, pl, pb, pr = d.pads
    assert pt == pb and pl == pr, "the CPU conv takes symmetric pads"
    if relu is None:
        relu = d.epilogue == dwref.EPI_RELU
    ho, wo = d.out_hw()
    if d.group == 1:
        y = dwref.conv2d_f16(x, wt, bias, relu, n, h, w, c_in, d.c_out, d.k_h, d.k_w, d.stride_h, d.stride_w,
                             pt, pl, threads)
    else:
        y = dwref.dwconv_f16(x, wt, relu, n, h, w, c_in, d.c_out // c_in, d.k_h, d.k_w, d.stride_h, d.stride_w,
                             pt, pl, threads, bias=bias)
    return y.reshape(n, ho, wo, d.c_out)


def gemm_f16_op(graph, op, x, threads=1):
    """One GemmF16 op: gemm_fp16 then the runtime's bias step."""
    m = x.shape[0]
    n, k = op.params["n"], op.params["k"]
    wt = graph.initializers[op.inputs[1]].view(np.uint16)
    bias = graph.initializers[op.inputs[2]].view(np.uint16)
    y = dwref.gemm_f16(x, wt, m, n, k, threads)
    return dwref.bias_relu_f16(y, bias, False, m, n).reshape(m, n)


def unfold_f16_op(op, x):
    """UnfoldF32ToF16 on an f32 NHWC array: y[n,r,j,q*c+ch] = from_f32(x[n,r,j*sw+q-pl,ch])."""
    pr = op.params
    n, h, w, c = x.shape
    kw, sw, pl, wo, cd = pr["k_w"], pr["stride_w"], pr["pad_l"], pr["w_out"], pr["c_dst"]
    xp = np.zeros((n, h, w + kw + sw * wo, c), np.float32)
    xp[:, :, pl:pl + w, :] = x
    y = np.zeros((n, h, wo, cd), np.uint16)
    for q in range(kw):
        cols = xp[:, :, q:q + sw * wo:sw, :][:, :, :wo, :]
        y[..., q * c:(q + 1) * c] = dwref.f16_from_f32_array(cols).reshape(n, h, wo, c)
    return y


def im2col_u8_op(op, x):
    """Im2colU8ToI8 on a uint8 NHWC image: quantize_u8_to_i8 then the im2col gather."""
    pr = op.params
    n, h, w, c = x.shape
    q = dwref.quantize_u8_to_i8(x, pr["scale"]).reshape(n, h, w, c)
    kh, kw, sh, sw, pt, pl = pr["k_h"], pr["k_w"], pr["s_h"], pr["s_w"], pr["p_t"], pr["p_l"]
    ho, wo, cd = pr["h_out"], pr["w_out"], pr["c_dst"]
    qp = np.zeros((n, h + kh + sh * ho, w + kw + sw * wo, c), np.int8)
    qp[:, pt:pt + h, pl:pl + w, :] = q
    y = np.zeros((n, ho, wo, cd), np.int8)
    for a in range(kh):
        for b_ in range(kw):
            k0 = (a * kw + b_) * c
            y[..., k0:k0 + c] = qp[:, a:a + sh * ho:sh, b_:b_ + sw * wo:sw, :][:, :ho, :wo, :]
    return y
