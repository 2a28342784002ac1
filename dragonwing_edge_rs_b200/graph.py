"""Graph IR and CUDA graph runtime for fused-INT8 and fp16 networks.

The IR mirrors the reference's compiled op list: ``CompiledOp`` with
``op_type`` / ``inputs`` / ``outputs`` / ``params``
(crates/dragonwing-onnx/src/builder.rs:204-361), where the fused conv is
``OpParams::Conv2dRequantReluI8Nhwc`` extended with bias, per-channel
requantisation, ReLU6/SiLU and depthwise groups.  ``CudaGraphRuntime`` mirrors
``VulkanGraphRuntime`` (crates/dragonwing-onnx/src/vulkan_runtime.rs:72-419):
it owns one device buffer per tensor, uploads initializers once at
construction, dispatches ops in order from ``run()``, and can record the whole
op list once as a CUDA graph (the reference's single-command-buffer
``OpsRecorder`` batching) so a forward pass is one launch.

All tensors are NHWC.  int8 tensors carry a per-tensor scale (symmetric, zero
point 0, crates/dragonwing-core/src/quantization.rs:1-30).
"""
from __future__ import annotations

import ctypes
from dataclasses import dataclass, field

import numpy as np

from . import _lib as L
from . import ops
from . import quantization as Q
from .backend import BackendError, CudaBackend, CudaBuffer
from .ops import ConvDesc

_NP = {"i8": np.int8, "u8": np.uint8, "f32": np.float32, "i32": np.int32, "f16": np.float16}


@dataclass
class TensorInfo:
    name: str
    shape: tuple
    dtype: str = "i8"
    scale: float | None = None

    @property
    def nbytes(self) -> int:
        return int(np.prod(self.shape)) * np.dtype(_NP[self.dtype]).itemsize


@dataclass
class CompiledOp:
    """builder.rs:204 CompiledOp.  op_type values used here:
    Conv2dRequantReluI8Nhwc (fused conv), AddQuantized, MaxPool, Concat, Split,
    Resize, QuantizeU8, Dequantize, YoloDetect (the Detect head's tail),
    YoloPostprocess (postprocess_yolo), and the fp16 ops."""

    name: str
    op_type: str
    inputs: list
    outputs: list
    params: dict = field(default_factory=dict)


@dataclass
class Graph:
    tensors: dict
    ops: list
    initializers: dict
    inputs: list
    outputs: list
    views: dict = field(default_factory=dict)  # tensor -> (parent tensor, channel offset): see lower_concat_views_i8

    def add_tensor(self, name, shape, dtype="i8", scale=None):
        self.tensors[name] = TensorInfo(name, tuple(int(s) for s in shape), dtype, scale)
        return name

    # ---- work accounting (algorithmic ops = 2*MACs, padding taps included;
    # a conv whose input channels were zero-padded counts its real channels) ----
    def conv_ops(self):
        total = 0
        for op in self.ops:
            if op.op_type in ("Conv2dRequantReluI8Nhwc", "Conv2dAddI8", "Conv2dF16", "Conv2dAddF16"):
                d: ConvDesc = op.params["desc"]
                ho, wo = d.out_hw()
                c_in = op.params.get("c_in_real", d.c_in)  # a lowered conv counts its real channels
                per = d.k_h * d.k_w * (c_in if d.group == 1 else 1)
                total += 2 * d.n * ho * wo * d.c_out * per
            elif op.op_type == "Conv":  # the reference's unfused int8 conv (int32 accumulators)
                d = conv_desc_of(self, op)
                ho, wo = d.out_hw()
                total += 2 * d.n * ho * wo * d.c_out * d.k_h * d.k_w * (d.c_in if d.group == 1 else 1)
            elif op.op_type == "GemmF16":
                total += 2 * op.params["m"] * op.params["n"] * op.params["k"]
        return total


# ---------------------------------------------------------------------------
# builder helpers
# ---------------------------------------------------------------------------

class GraphBuilder:
    """Builds a fused INT8 graph with seeded random weights.

    Float weights are He-normal, folded BN is represented by an int32 bias,
    weights are quantised per output channel with the reference's symmetric
    scheme (quantization.rs:154-195), activation scales are drawn uniformly
    from ``act_scale_range``, and M / D / q6 are derived with the reference
    formulas (quantize.rs:245, ops.rs:3503-3525)."""

    def __init__(self, seed: int, act_scale_range=(0.01, 0.05), unfused: bool = False):
        self.rng = np.random.default_rng(seed)
        self.lo, self.hi = act_scale_range
        self.g = Graph({}, [], {}, [], [])
        self._n = 0
        # unfused: every conv in the form the reference's QuantizedGraphCompiler
        # emits (quantize.rs:176-191, 218-249) -- a Conv writing int32
        # accumulators, then Requantize (+ Relu / Clip) or, for SiLU, the f32
        # chain DequantizeLinear -> Sigmoid -> Mul -> QuantizeLinear -- for the
        # fusion passes (apply_fusion_passes) to collapse.  The same seed draws
        # the same weights and scales in both modes.
        self.unfused = unfused

    def _name(self, base):
        self._n += 1
        return f"{base}_{self._n}"

    def act_scale(self) -> float:
        return float(np.float32(self.rng.uniform(self.lo, self.hi)))

    def input(self, name, shape, dtype="i8", scale=None):
        self.g.add_tensor(name, shape, dtype, scale)
        self.g.inputs.append(name)
        return name

    def conv(self, x, c_out, k=3, s=1, pad=None, group=1, act="relu", out_scale=None, name=None):
        g = self.g
        xi = g.tensors[x]
        n, h, w, c_in = xi.shape
        p = k // 2 if pad is None else pad
        pads = p if isinstance(p, tuple) else (p, p, p, p)
        name = name or self._name("conv")
        dw = group != 1
        if dw:
            assert group == c_in and c_out % c_in == 0
            mult = c_out // c_in
            fan_in = k * k
            wf = self.rng.normal(0.0, np.sqrt(2.0 / fan_in), (c_out, k * k)).astype(np.float32)
        else:
            fan_in = k * k * c_in
            wf = self.rng.normal(0.0, np.sqrt(2.0 / fan_in), (c_out, k, k, c_in)).astype(np.float32)
        wq, s_w = Q.per_channel_symmetric(wf)
        if dw:  # [c_out, k*k] -> [k, k, c_in, mult]
            w_layout = wq.reshape(c_in, mult, k, k).transpose(2, 3, 0, 1).copy()
        else:   # OHWI -> HWIO (the graph layout after convert_nchw_to_nhwc, graph.rs:261-275)
            w_layout = wq.transpose(1, 2, 3, 0).copy()
        s_in = xi.scale
        s_out = out_scale if out_scale is not None else self.act_scale()
        bias = self.rng.integers(-1000, 1001, c_out).astype(np.int32)
        epi = {"none": L.EPI_NONE, "relu": L.EPI_RELU, "relu6": L.EPI_RELU6, "silu": L.EPI_SILU}[act]
        desc = ConvDesc(n, h, w, c_in, c_out, k, k, s, s, pads, group, epi)
        desc.q6 = Q.relu6_ceiling(s_out)
        desc.inv_s_out = float(np.float32(1.0) / np.float32(s_out))
        ho, wo = desc.out_hw()
        y = g.add_tensor(name + "_out", (n, ho, wo, c_out), "i8", s_out)
        if self.unfused:
            return self._conv_unfused(name, x, y, w_layout, bias, s_in, s_w, s_out, desc, act)
        for suffix, arr in (("_w", w_layout), ("_b", bias), ("_M", Q.requant_scales(s_in, s_w, s_out)),
                            ("_D", Q.dequant_scales(s_in, s_w))):
            g.initializers[name + suffix] = arr
        g.ops.append(CompiledOp(name, "Conv2dRequantReluI8Nhwc", [x, name + "_w", name + "_b", name + "_M", name + "_D"],
                                [y], {"desc": desc}))
        return y

    def _conv_unfused(self, name, x, y, w_layout, bias, s_in, s_w, s_out, desc, act):
        """The conv as the reference's quantizer leaves it, with its defects fixed:
        the int32 accumulator is a tensor of its own (`{y}_i32`, shaped), the bias
        is a Conv input, and the requantisation is per output channel (an
        initializer M), not the average of the channel scales."""
        g = self.g
        shape = g.tensors[y].shape
        g.initializers[name + "_w"] = w_layout
        g.initializers[name + "_b"] = bias
        acc = g.add_tensor(y + "_i32", shape, "i32")
        g.ops.append(CompiledOp(name, "Conv", [x, name + "_w", name + "_b"], [acc],
                                {"kernel_shape": (desc.k_h, desc.k_w), "strides": (desc.stride_h, desc.stride_w),
                                 "pads": tuple(desc.pads), "dilations": (1, 1), "group": desc.group}))
        if act == "silu":
            g.initializers[name + "_D"] = Q.dequant_scales(s_in, s_w)
            yf = g.add_tensor(name + "_deq", shape, "f32")
            sig = g.add_tensor(name + "_sig", shape, "f32")
            z = g.add_tensor(name + "_silu", shape, "f32")
            g.ops.append(CompiledOp(name + "_dequant", "DequantizeLinear", [acc, name + "_D"], [yf], {}))
            g.ops.append(CompiledOp(name + "_sigmoid", "Sigmoid", [yf], [sig], {}))
            g.ops.append(CompiledOp(name + "_mul", "Mul", [yf, sig], [z], {}))
            g.ops.append(CompiledOp(name + "_quant", "QuantizeLinear", [z], [y], {"scale": s_out}))
            return y
        g.initializers[name + "_M"] = Q.requant_scales(s_in, s_w, s_out)
        rq = y if act == "none" else g.add_tensor(name + "_rq", shape, "i8", s_out)
        g.ops.append(CompiledOp(name + "_requant", "Requantize", [acc, name + "_M"], [rq], {"scale": None}))
        if act == "relu":
            g.ops.append(CompiledOp(name + "_relu", "Relu", [rq], [y], {}))
        elif act == "relu6":
            g.ops.append(CompiledOp(name + "_clip", "Clip", [rq], [y], {"min": 0.0, "max": 6.0}))
        return y

    def add(self, a, b, out_scale=None, name=None):
        g = self.g
        ta, tb = g.tensors[a], g.tensors[b]
        assert ta.shape == tb.shape
        s_out = out_scale if out_scale is not None else self.act_scale()
        ra, rb = Q.add_ratios(ta.scale, tb.scale, s_out)
        name = name or self._name("add")
        y = g.add_tensor(name + "_out", ta.shape, "i8", s_out)
        g.ops.append(CompiledOp(name, "AddQuantized", [a, b], [y], {"scale_a_over_out": ra, "scale_b_over_out": rb}))
        return y

    def maxpool(self, x, k, s, pad, name=None):
        g = self.g
        n, h, w, c = g.tensors[x].shape
        name = name or self._name("maxpool")
        ho, wo = (h + 2 * pad - k) // s + 1, (w + 2 * pad - k) // s + 1
        y = g.add_tensor(name + "_out", (n, ho, wo, c), "i8", g.tensors[x].scale)
        g.ops.append(CompiledOp(name, "MaxPool", [x], [y], {"k": k, "s": s, "pad": pad}))
        return y

    def concat(self, xs, name=None):
        """Channel concat.  Inputs with a different scale are first requantised
        to the first input's scale by an AddQuantized-free 1x scale op is not
        needed: the builder gives every concat input the same scale."""
        g = self.g
        t0 = g.tensors[xs[0]]
        n, h, w, _ = t0.shape
        cs = [g.tensors[x].shape[3] for x in xs]
        name = name or self._name("concat")
        y = g.add_tensor(name + "_out", (n, h, w, sum(cs)), "i8", t0.scale)
        g.ops.append(CompiledOp(name, "Concat", list(xs), [y], {"channels": cs}))
        return y

    def split(self, x, parts, name=None):
        g = self.g
        n, h, w, c = g.tensors[x].shape
        assert sum(parts) == c
        name = name or self._name("split")
        outs, c0 = [], 0
        for i, p in enumerate(parts):
            o = g.add_tensor(f"{name}_out{i}", (n, h, w, p), "i8", g.tensors[x].scale)
            g.ops.append(CompiledOp(f"{name}_{i}", "Split", [x], [o], {"c0": c0, "c_len": p}))
            outs.append(o)
            c0 += p
        return outs

    def upsample2(self, x, name=None):
        g = self.g
        n, h, w, c = g.tensors[x].shape
        name = name or self._name("resize")
        y = g.add_tensor(name + "_out", (n, 2 * h, 2 * w, c), "i8", g.tensors[x].scale)
        g.ops.append(CompiledOp(name, "Resize", [x], [y], {"mode": "nearest"}))
        return y

    def output(self, name):
        self.g.outputs.append(name)


class F16GraphBuilder:
    """Builds an fp16 graph (the reference's F16 CPU-runtime path) with seeded
    random weights: He-normal conv weights with BN folded into them and into
    an f16 bias, as the reference's loader folds BN (crates/dragonwing-onnx/src/
    graph.rs:597-613).  Weights are generated in f32 and stored as f16 with
    round-to-nearest-even (F16::from_f32); tensors are NHWC."""

    def __init__(self, seed: int):
        self.rng = np.random.default_rng(seed)
        self.g = Graph({}, [], {}, [], [])
        self._n = 0

    def _name(self, base):
        self._n += 1
        return f"{base}_{self._n}"

    @staticmethod
    def _f16(a):
        return np.asarray(a, np.float32).astype(np.float16)

    def input_f32(self, name, shape):
        """f32 NHWC graph input and its F16 conversion (runtime.rs:842-851)."""
        g = self.g
        g.add_tensor(name, shape, "f32")
        g.inputs.append(name)
        n, h, w, c = shape
        y = g.add_tensor(name + "_f16", (n, h, w, c), "f16")
        g.ops.append(CompiledOp("cast_input", "CastF32ToF16", [name], [y], {"c_src": c, "c_dst": c}))
        return y

    def conv(self, x, c_out, k=3, s=1, pad=None, relu=True, gamma=1.0, name=None):
        g = self.g
        n, h, w, c_in = g.tensors[x].shape
        p = k // 2 if pad is None else pad
        name = name or self._name("conv")
        wf = self.rng.normal(0.0, np.sqrt(2.0 / (k * k * c_in)), (k, k, c_in, c_out)).astype(np.float32)
        wf *= np.float32(gamma)
        bias = self.rng.normal(0.0, 0.05, c_out).astype(np.float32)
        desc = ConvDesc(n, h, w, c_in, c_out, k, k, s, s, (p, p, p, p), 1, L.EPI_RELU if relu else L.EPI_NONE)
        ho, wo = desc.out_hw()
        y = g.add_tensor(name + "_out", (n, ho, wo, c_out), "f16")
        g.initializers[name + "_w"] = self._f16(wf)
        g.initializers[name + "_b"] = self._f16(bias)
        g.ops.append(CompiledOp(name, "Conv2dF16", [x, name + "_w", name + "_b"], [y], {"desc": desc}))
        return y

    def add_relu(self, a, b, name=None):
        g = self.g
        assert g.tensors[a].shape == g.tensors[b].shape
        name = name or self._name("add")
        y = g.add_tensor(name + "_out", g.tensors[a].shape, "f16")
        g.ops.append(CompiledOp(name, "AddF16", [a, b], [y], {"relu": True}))
        return y

    def maxpool(self, x, k, s, pad, name=None):
        g = self.g
        n, h, w, c = g.tensors[x].shape
        name = name or self._name("maxpool")
        ho, wo = (h + 2 * pad - k) // s + 1, (w + 2 * pad - k) // s + 1
        y = g.add_tensor(name + "_out", (n, ho, wo, c), "f16")
        g.ops.append(CompiledOp(name, "MaxPoolF16", [x], [y], {"k": k, "s": s, "pad": pad}))
        return y

    def global_avgpool(self, x, name=None):
        g = self.g
        n, h, w, c = g.tensors[x].shape
        name = name or self._name("gap")
        y = g.add_tensor(name + "_out", (n, c), "f16")
        g.ops.append(CompiledOp(name, "GlobalAveragePoolF16", [x], [y], {}))
        return y

    def fc(self, x, n_out, name=None):
        """Gemm F16 with bias (runtime.rs:1247-1275): [m, k] @ [k, n_out] + bias."""
        g = self.g
        m, k = g.tensors[x].shape
        name = name or self._name("fc")
        wf = self.rng.normal(0.0, np.sqrt(1.0 / k), (k, n_out)).astype(np.float32)
        bias = self.rng.normal(0.0, 0.05, n_out).astype(np.float32)
        y = g.add_tensor(name + "_out", (m, n_out), "f16")
        g.initializers[name + "_w"] = self._f16(wf)
        g.initializers[name + "_b"] = self._f16(bias)
        g.ops.append(CompiledOp(name, "GemmF16", [x, name + "_w", name + "_b"], [y], {"m": m, "n": n_out, "k": k}))
        return y

    def output_f32(self, x, name):
        g = self.g
        y = g.add_tensor(name, g.tensors[x].shape, "f32")
        g.ops.append(CompiledOp("cast_" + name, "CastF16ToF32", [x], [y], {}))
        g.outputs.append(y)
        return y


def fuse_residual_f16(graph: Graph) -> Graph:
    """Op-fusion pass for the fp16 path (the counterpart of the reference's
    conv fusion, crates/dragonwing-core/src/fusion.rs): Conv2dF16 (no ReLU) ->
    AddF16 (+ReLU) becomes one Conv2dAddF16 op whose epilogue adds the other
    operand of the add and applies the add's ReLU.  The conv picked is a 1x1
    stride-1 conv when the add has one (its epilogue fuses on the tensor
    cores); the other operand's producer moves before it when needed.  Returns a
    new Graph; the arithmetic is unchanged (conv, bias, add, ReLU in the same
    order and rounding)."""
    ops_ = list(graph.ops)
    producer = {o: i for i, op in enumerate(ops_) for o in op.outputs}
    consumers: dict = {}
    for op in ops_:
        for i in op.inputs:
            consumers.setdefault(i, []).append(op)
    tensors = dict(graph.tensors)
    fused_any = True
    while fused_any:
        fused_any = False
        for ai, add in enumerate(ops_):
            if add.op_type != "AddF16":
                continue
            cands = []
            for k, t in enumerate(add.inputs):
                pi = producer.get(t)
                if pi is None:
                    continue
                cv = ops_[pi]
                if (cv.op_type != "Conv2dF16" or cv.params["desc"].epilogue != L.EPI_NONE
                        or len(consumers.get(t, [])) != 1 or t in graph.outputs):
                    continue
                d = cv.params["desc"]
                flat = d.k_h == 1 and d.k_w == 1 and d.stride_h == 1 and d.stride_w == 1 and d.pads == (0, 0, 0, 0)
                cands.append((0 if flat else 1, pi, k))
            if not cands:
                continue
            _, ci, k = min(cands)
            cv = ops_[ci]
            res = add.inputs[1 - k]
            ri = producer.get(res, -1)
            new_list = [op for j, op in enumerate(ops_) if j != ai]
            conv_pos = new_list.index(cv)
            if ri > ci:  # the residual is produced later: move its producer before the conv if it can be
                rop = ops_[ri]
                ready = all(producer.get(i, -1) < ci for i in rop.inputs if i in producer)
                if not ready:
                    continue
                new_list.remove(rop)
                conv_pos = new_list.index(cv)
                new_list.insert(conv_pos, rop)
                conv_pos += 1
            d0 = cv.params["desc"]
            d = ConvDesc(d0.n, d0.h, d0.w, d0.c_in, d0.c_out, d0.k_h, d0.k_w, d0.stride_h, d0.stride_w, d0.pads,
                         d0.group, L.EPI_RELU if add.params.get("relu") else L.EPI_NONE)
            params = dict(cv.params, desc=d)
            fused = CompiledOp(cv.name + "+" + add.name, "Conv2dAddF16", list(cv.inputs) + [res], list(add.outputs),
                               params)
            new_list[conv_pos] = fused
            tensors.pop(cv.outputs[0], None)
            ops_ = new_list
            producer = {o: i for i, op in enumerate(ops_) for o in op.outputs}
            consumers = {}
            for op in ops_:
                for i in op.inputs:
                    consumers.setdefault(i, []).append(op)
            fused_any = True
            break
    return Graph(tensors, ops_, graph.initializers, list(graph.inputs), list(graph.outputs))


def lower_unfold_stem_f16(graph: Graph) -> Graph:
    """Device lowering of a network's first conv on a few-channel f16 image:
    CastF32ToF16 (c channels, c % 8 != 0) -> Conv2dF16 (k_h x k_w, stride
    (s_h, s_w)) becomes UnfoldF32ToF16 (the cast fused with a horizontal
    unfold, c_u = k_w * c rounded up to 16 channels) -> Conv2dF16 (k_h x 1,
    stride (s_h, 1)) whose kernel rows hold the k_w taps side by side.  The
    products are the same, summed in the same (kh, kw, c) order; the tensor
    cores then load rows of c_u channels instead of c (= 3).  Returns a new
    Graph; the source graph keeps the reference ops."""
    ops_ = list(graph.ops)
    consumers: dict = {}
    for op in ops_:
        for i in op.inputs:
            consumers.setdefault(i, []).append(op)
    tensors, inits = dict(graph.tensors), dict(graph.initializers)
    for ci, cast in enumerate(ops_):
        if cast.op_type != "CastF32ToF16" or cast.params["c_dst"] % 8 == 0:
            continue
        users = consumers.get(cast.outputs[0], [])
        if len(users) != 1 or users[0].op_type != "Conv2dF16" or cast.outputs[0] in graph.outputs:
            continue
        conv = users[0]
        d = conv.params["desc"]
        c = cast.params["c_src"]
        if d.group != 1 or d.k_w == 1 or d.k_w * c > 64:
            continue
        _, wo = d.out_hw()
        c_u = (d.k_w * c + 15) // 16 * 16
        pt, pl, pb, pr = d.pads
        if d.h % d.stride_h:
            continue
        u = cast.outputs[0] + "_unfold"
        tensors[u] = TensorInfo(u, (d.n, d.h, wo, c_u), "f16")
        tensors.pop(cast.outputs[0], None)
        w = graph.initializers[conv.inputs[1]].view(np.uint16).reshape(d.k_h, d.k_w * c, d.c_out)
        wu = np.zeros((d.k_h, 1, c_u, d.c_out), np.uint16)
        wu[:, 0, :d.k_w * c, :] = w
        inits[conv.inputs[1] + "_unfold"] = wu.view(np.float16)
        unfold = CompiledOp(cast.name + "_unfold", "UnfoldF32ToF16", list(cast.inputs), [u],
                            {"k_w": d.k_w, "stride_w": d.stride_w, "pad_l": pl, "w_out": wo, "c_src": c, "c_dst": c_u})
        d2 = ConvDesc(d.n, d.h, wo, c_u, d.c_out, d.k_h, 1, d.stride_h, 1, (pt, 0, pb, 0), 1, d.epilogue)
        conv2 = CompiledOp(conv.name, "Conv2dF16", [u, conv.inputs[1] + "_unfold"] + list(conv.inputs[2:]),
                           list(conv.outputs), dict(conv.params, desc=d2, c_in_real=c * d.k_w))
        ops_ = [unfold if op is cast else conv2 if op is conv else op for op in ops_]
        break  # a network has one such input conv
    return Graph(tensors, ops_, inits, list(graph.inputs), list(graph.outputs))


def stem_conv_fits(n, h, w, c, d) -> bool:
    """The shapes dw_conv2d_stem_u8_i8 takes (csrc/elementwise.cu,
    launch_stem3_conv_u8_i8): a 3x3 group-1 conv on 3 channels, c_out a
    multiple of 16 up to 64, the image width a multiple of 16, left padding
    <= 5, and a band of input rows within the kernel's shared-memory budget."""
    if c != 3 or d.k_h != 3 or d.k_w != 3 or d.group != 1 or d.c_out % 16 or d.c_out > 64 or w % 16:
        return False
    pt, pl, _, _ = d.pads
    if pl > 5 or pt < 0:
        return False
    ho, wo = d.out_hw()
    last = 16 + ((wo - 1) * d.stride_w - pl) * 3 + 12
    row_bytes = (max(16 + w * 3, last) + 15) // 16 * 16
    return (3 * d.stride_h + 3) * row_bytes <= 36 * 1024 and n * ((ho + 3) // 4) < 2 ** 31


def lower_im2col_input_i8(graph: Graph) -> Graph:
    """Device lowering of an int8 network's first conv on a few-channel image:
    QuantizeU8 (c channels, c % 16 != 0) -> Conv2dRequantReluI8Nhwc (k_h x k_w,
    k_h*k_w*c <= 64).  The 3x3 conv on a 3-channel image (YOLOv8n's stem)
    becomes one Conv2dStemU8I8 (quantisation, conv and epilogue in one kernel
    on the CUDA cores: the conv is 27 MACs per output, and the 32-byte im2col
    rows the tensor cores need would be written and read again); other shapes
    become Im2colU8ToI8 (the quantisation fused with an
    im2col into c_dst = k_h*k_w*c rounded up to 16 channels) -> a 1x1 conv
    whose kernel rows are the original taps in (kh, kw, c) order, zero rows for
    the padding channels.  The integer products are the same, so the result is
    bit-identical; the tensor cores then see 16-byte-aligned channel rows."""
    ops_ = list(graph.ops)
    consumers: dict = {}
    for op in ops_:
        for i in op.inputs:
            consumers.setdefault(i, []).append(op)
    tensors, inits = dict(graph.tensors), dict(graph.initializers)
    for q in ops_:
        if q.op_type != "QuantizeU8":
            continue
        t = tensors[q.outputs[0]]
        n, h, w, c = t.shape
        users = consumers.get(q.outputs[0], [])
        if c % 16 == 0 or len(users) != 1 or users[0].op_type != "Conv2dRequantReluI8Nhwc" or q.outputs[0] in graph.outputs:
            continue
        conv = users[0]
        d = conv.params["desc"]
        kc = d.k_h * d.k_w * c
        if d.group != 1 or kc > 64:
            continue
        ho, wo = d.out_hw()
        if stem_conv_fits(n, h, w, c, d):
            # one pass: quantisation + the 3x3 conv on the CUDA cores (dw_conv2d_stem_u8_i8)
            tensors.pop(q.outputs[0], None)
            stem = CompiledOp(conv.name, "Conv2dStemU8I8", [q.inputs[0]] + list(conv.inputs[1:]), list(conv.outputs),
                              dict(conv.params, in_scale=q.params["scale"]))
            ops_ = [stem if op is conv else op for op in ops_ if op is not q]
            break
        c_dst = (kc + 15) // 16 * 16
        u = q.outputs[0] + "_im2col"
        tensors[u] = TensorInfo(u, (n, ho, wo, c_dst), "i8", t.scale)
        tensors.pop(q.outputs[0], None)
        wt = graph.initializers[conv.inputs[1]].reshape(kc, d.c_out)
        wu = np.zeros((1, 1, c_dst, d.c_out), np.int8)
        wu[0, 0, :kc, :] = wt
        inits[conv.inputs[1] + "_im2col"] = wu
        pt, pl, _, _ = d.pads
        im2col = CompiledOp(q.name + "_im2col", "Im2colU8ToI8", list(q.inputs), [u],
                            {"k_h": d.k_h, "k_w": d.k_w, "s_h": d.stride_h, "s_w": d.stride_w, "p_t": pt, "p_l": pl,
                             "h_out": ho, "w_out": wo, "c_dst": c_dst, "scale": q.params["scale"]})
        d2 = ConvDesc(n, ho, wo, c_dst, d.c_out, 1, 1, 1, 1, (0, 0, 0, 0), 1, d.epilogue)
        d2.q6, d2.inv_s_out = d.q6, d.inv_s_out
        conv2 = CompiledOp(conv.name, conv.op_type, [u, conv.inputs[1] + "_im2col"] + list(conv.inputs[2:]),
                           list(conv.outputs), dict(conv.params, desc=d2, c_in_real=kc))
        ops_ = [im2col if op is q else conv2 if op is conv else op for op in ops_]
        break
    return Graph(tensors, ops_, inits, list(graph.inputs), list(graph.outputs))


def fuse_residual_i8(graph: Graph) -> Graph:
    """Device pass: a tensor-core conv whose output feeds only an int8 add
    (AddQuantized) becomes one Conv2dAddI8 that applies the add to the conv's
    int8 result in its epilogue (dw_conv2d_add_i8_view): the same two
    roundings, so bit-identical, and the conv's output never reaches memory.

    The add's arithmetic then runs on the conv's epilogue warps, which bound
    the conv when its reduction is short; it pays only where the epilogue has
    slack: a narrow conv (c_out <= 16) or a long reduction (k_h * k_w * c_in
    >= 1024).  Measured on YOLOv8n's bottlenecks at batch 32 (device time,
    conv alone -> fused vs the separate add): 160x160 c16 74.3 -> 79.4 vs 12.5 us,
    20x20 c128 17.7 -> 19.1 vs 3.8 us, but 80x80 c32 37.0 -> 51.5 vs 8.0 us and
    40x40 c64 23.1 -> 34.0 vs 5.0 us."""
    ops_ = list(graph.ops)
    consumers = {}
    for op in ops_:
        for i in op.inputs:
            consumers.setdefault(i, []).append(op)
    producer = {o: op for op in ops_ for o in op.outputs}
    fused, drop = {}, set()
    for add in ops_:
        if add.op_type != "AddQuantized":
            continue
        a, b = add.inputs
        ra, rb = add.params["scale_a_over_out"], add.params["scale_b_over_out"]
        if not (abs(ra) < 1e30 and abs(rb) < 1e30):
            continue
        for h, res, r_res, r_conv in ((b, a, ra, rb), (a, b, rb, ra)):
            conv = producer.get(h)
            if conv is None or conv.op_type != "Conv2dRequantReluI8Nhwc" or id(conv) in drop or h == res:
                continue
            d = conv.params["desc"]
            if (d.group != 1 or d.c_in % 16 or d.c_out % 16 or h in graph.outputs
                    or len(consumers.get(h, [])) != 1):
                continue
            if not (d.c_out <= 16 or d.k_h * d.k_w * d.c_in >= 1024):
                continue
            fused[id(add)] = CompiledOp(conv.name + "+" + add.name, "Conv2dAddI8", list(conv.inputs) + [res],
                                        list(add.outputs), dict(conv.params, ra=r_res, rb=r_conv))
            drop.add(id(conv))
            break
    if not fused:
        return graph
    out_ops = [fused.get(id(op), op) for op in ops_ if id(op) not in drop]
    gone = {op.outputs[0] for op in ops_ if id(op) in drop}
    tensors = {k: v for k, v in graph.tensors.items() if k not in gone}
    return Graph(tensors, out_ops, dict(graph.initializers), list(graph.inputs), list(graph.outputs), dict(graph.views))


def fuse_maxpool_chain_i8(graph: Graph) -> Graph:
    """Device pass: a run of 2..4 int8 MaxPools, each k x k (k odd), stride 1,
    padding k/2, each reading the previous one's output (YOLOv8's SPPF: three
    5x5 pools in a row), becomes one MaxPoolChainI8 that writes every pooled
    map (dw_maxpool_chain_i8_view: the input is read once, the pooling steps
    are the same maxima).  The intermediate maps stay outputs of the fused op,
    so their other readers (the SPPF concat) are unchanged."""
    ops_ = list(graph.ops)

    def same_pool(op):
        p = op.params
        return op.op_type == "MaxPool" and p["s"] == 1 and p["k"] % 2 == 1 and p["pad"] == p["k"] // 2

    readers = {}
    for op in ops_:
        for i in op.inputs:
            readers.setdefault(i, []).append(op)
    chained, head_of = set(), {}
    for op in ops_:
        if not same_pool(op) or id(op) in chained or graph.tensors[op.inputs[0]].shape[3] % 16:
            continue
        run = [op]
        while len(run) < 4:
            nxt = [q for q in readers.get(run[-1].outputs[0], []) if same_pool(q) and q.params["k"] == op.params["k"]]
            if len(nxt) != 1 or id(nxt[0]) in chained:
                break
            run.append(nxt[0])
        if len(run) < 2:
            continue
        chained.update(id(q) for q in run)
        head_of[id(op)] = CompiledOp("+".join(q.name for q in run), "MaxPoolChainI8", [op.inputs[0]],
                                     [q.outputs[0] for q in run], {"k": op.params["k"]})
    if not head_of:
        return graph
    out_ops = [head_of.get(id(op), op) for op in ops_ if id(op) in head_of or id(op) not in chained]
    return Graph(dict(graph.tensors), out_ops, dict(graph.initializers), list(graph.inputs), list(graph.outputs),
                 dict(graph.views))


def lower_concat_views_i8(graph: Graph) -> Graph:
    """Device lowering of int8 channel concats: when every input of a Concat is
    written by an op that can write a channel-range view (a tensor-core conv,
    an int8 add, a maxpool) and read only by ops that can read one (stride-1
    tensor-core convs, adds, maxpools, or the concat), the inputs become views
    of the concat's output buffer (producers write their channel ranges in
    place) and the Concat disappears.  An input that is a channel Split of a
    tensor makes that tensor a view too, and the Split disappears: this is the
    C2f block (split, bottlenecks, concat) and SPPF (maxpools, concat) of
    YOLOv8.  The same bytes end up in the same places, so the result is
    bit-identical; the copies are gone."""
    ops_ = list(graph.ops)
    T = graph.tensors
    producer, consumers = {}, {}
    for op in ops_:
        for o in op.outputs:
            producer[o] = op
        for i in op.inputs:
            consumers.setdefault(i, []).append(op)
    views = dict(graph.views)
    protected = set(graph.inputs) | set(graph.outputs)
    removed = set()

    def tc_conv(op):
        d = op.params["desc"]
        return d.group == 1 and d.c_in % 16 == 0 and d.c_out % 16 == 0

    def can_write(op):
        if op.op_type == "Conv2dRequantReluI8Nhwc":
            return tc_conv(op)
        return op.op_type in ("AddQuantized", "MaxPool", "Conv2dAddI8", "MaxPoolChainI8")

    def can_read(op, t):
        if op.op_type in ("Conv2dRequantReluI8Nhwc", "Conv2dAddI8"):
            if op.op_type == "Conv2dAddI8" and op.inputs[5] == t and op.inputs[0] != t:
                return True  # the residual
            return tc_conv(op) and op.inputs[0] == t and op.params["desc"].stride_w == 1
        return op.op_type in ("AddQuantized", "MaxPool", "MaxPoolChainI8")

    for cat in ops_:
        if cat.op_type != "Concat" or cat.outputs[0] in protected:
            continue
        out = cat.outputs[0]
        plan, splits, ok, off = {}, [], True, 0
        for t in cat.inputs:
            c = T[t].shape[3]
            p = producer.get(t)
            if t in protected or t in views or c % 16 or p is None:
                ok = False
                break
            if p.op_type == "Split":
                src, c0 = p.inputs[0], p.params["c0"]
                want = (out, off - c0)
                sp = producer.get(src)
                if (off - c0 < 0 or src in protected or src in views or plan.get(src, want) != want or sp is None
                        or not can_write(sp) or T[src].shape[3] % 16
                        or any(q.op_type != "Split" or q.outputs[0] not in cat.inputs for q in consumers.get(src, []))):
                    ok = False
                    break
                plan[src] = want
                plan[t] = (src, c0)
                splits.append(p)
            elif can_write(p):
                plan[t] = (out, off)
            else:
                ok = False
                break
            if any(q is not cat and q.op_type != "Split" and not can_read(q, t) for q in consumers.get(t, [])):
                ok = False
                break
            off += c
        if not ok:
            continue
        views.update(plan)
        removed.add(id(cat))
        removed.update(id(q) for q in splits)
    if not removed:
        return graph
    return Graph(dict(graph.tensors), [op for op in ops_ if id(op) not in removed], dict(graph.initializers),
                 list(graph.inputs), list(graph.outputs), views)


# ---------------------------------------------------------------------------
# the reference's op-fusion passes over the unfused int8 IR
# (crates/dragonwing-onnx/src/fusion.rs:42-334), extended to the contract
# ---------------------------------------------------------------------------

UNFUSED_OPS = ("Conv", "Requantize", "DequantizeLinear", "Sigmoid", "Mul", "SiLU", "QuantizeLinear", "Relu", "Clip")


def conv_desc_of(graph: Graph, op: CompiledOp, epilogue: int = L.EPI_NONE) -> ConvDesc:
    """ConvDesc of an unfused Conv op from its OpParams::Conv2d fields
    (builder.rs:204-361) and its tensors' NHWC shapes."""
    n, h, w, c_in = graph.tensors[op.inputs[0]].shape
    c_out = graph.tensors[op.outputs[0]].shape[3]
    kh, kw = op.params["kernel_shape"]
    sh, sw = op.params["strides"]
    return ConvDesc(n, h, w, c_in, c_out, kh, kw, sh, sw, tuple(op.params["pads"]), op.params["group"], epilogue)


@dataclass
class FusionStats:
    """Fuseable patterns of a graph (fusion.rs:404-420, FusionStats)."""
    conv_relu: int = 0            # f32 Conv -> Relu
    silu: int = 0                 # Mul(x, Sigmoid(x))
    conv_requant_relu_i8: int = 0  # int8 Conv -> Requantize / DequantizeLinear

    def total(self) -> int:
        return self.conv_relu + self.silu + self.conv_requant_relu_i8


def _producers(graph: Graph) -> dict:
    return {o: i for i, op in enumerate(graph.ops) for o in op.outputs}


def _consumers(graph: Graph) -> dict:
    cons = {}
    for i, op in enumerate(graph.ops):
        for t in op.inputs:
            cons.setdefault(t, []).append(i)
    return cons


def count_fuseable_patterns(graph: Graph) -> FusionStats:
    """count_fuseable_patterns (fusion.rs:351-402): Relu fed by a Conv with a
    float output, Mul with a Sigmoid operand, and the int8 anchor -- a
    Requantize (or, for SiLU, a DequantizeLinear) fed by a Conv's int32
    accumulators."""
    prod = _producers(graph)
    st = FusionStats()
    for op in graph.ops:
        src = [graph.ops[prod[t]] for t in op.inputs if t in prod]
        if op.op_type == "Relu" and src and src[0].op_type == "Conv" and \
                graph.tensors[src[0].outputs[0]].dtype in ("f32", "f16"):
            st.conv_relu += 1
        if op.op_type == "Mul" and len(op.inputs) == 2 and any(s.op_type == "Sigmoid" for s in src):
            st.silu += 1
        if op.op_type in ("Requantize", "DequantizeLinear") and src and src[0].op_type == "Conv":
            st.conv_requant_relu_i8 += 1
    return st


def _rebuild(graph: Graph, ops: list) -> Graph:
    used = {t for op in ops for t in op.inputs + op.outputs} | set(graph.inputs) | set(graph.outputs)
    tensors = {k: v for k, v in graph.tensors.items() if k in used}
    inits = {k: v for k, v in graph.initializers.items() if k in used}
    return Graph(tensors, ops, inits, list(graph.inputs), list(graph.outputs), dict(graph.views))


def fuse_silu(graph: Graph) -> Graph:
    """Pass 2 (fusion.rs:126-190): Mul(x, Sigmoid(x)), either operand order,
    where the Sigmoid's output feeds only that Mul, becomes one SiLU(x) op
    (y = x * sigmoid(x), the reference's order of the two ops)."""
    prod, cons = _producers(graph), _consumers(graph)
    drop, repl = set(), {}
    for i, op in enumerate(graph.ops):
        if op.op_type != "Mul" or len(op.inputs) != 2:
            continue
        a, b = op.inputs
        match = None
        for sig_in, x in ((a, b), (b, a)):
            j = prod.get(sig_in)
            if j is not None and graph.ops[j].op_type == "Sigmoid" and graph.ops[j].inputs[0] == x:
                match = (j, x)
                break
        if match is None:
            continue
        j, x = match
        sig_out = graph.ops[j].outputs[0]
        if len(cons.get(sig_out, [])) != 1 or sig_out in graph.outputs:
            continue
        drop.add(j)
        repl[i] = CompiledOp(op.name + "_silu", "SiLU", [x], list(op.outputs), {})
    ops = [repl.get(i, op) for i, op in enumerate(graph.ops) if i not in drop]
    return _rebuild(graph, ops)


def fuse_conv_requant_i8(graph: Graph) -> Graph:
    """Pass 3 (fusion.rs:192-334), extended to the contract.  The reference
    collapses Conv -> Requantize (-> Relu) into Conv2dRequantReluI8Nhwc for
    unbiased group-1 convs with a scalar scale.  Here the anchor is a
    Requantize (or a DequantizeLinear, for SiLU) that is the only reader of a
    Conv's int32 accumulators, and the op absorbs:
      * the Conv's int32 bias (BN-folded convs: reference defect 4),
      * a per-channel M initializer or the reference's scalar scale,
      * Relu, or Clip(0, 6) (ReLU6, bound q6 = quantize(6, s_out)) when it is
        the requantised tensor's only reader (the reference's live-consumer rule),
      * SiLU: DequantizeLinear(D) -> SiLU -> QuantizeLinear(s_out), each the
        previous op's only reader,
      * depthwise convs (group == c_in, c_out a multiple of c_in).
    Dilation must be 1 and other groups are refused, as the reference refuses
    every group != 1.  The fused op keeps the Conv's name and writes the
    chain's last tensor; a tensor the chain would swallow that is a graph
    output stops the chain there."""
    prod, cons = _producers(graph), _consumers(graph)
    drop, repl = set(), {}
    inits = dict(graph.initializers)

    def only_reader(t, i):
        c = cons.get(t, [])
        return len(c) == 1 and c[0] == i and t not in graph.outputs

    for i, op in enumerate(graph.ops):
        if op.op_type not in ("Requantize", "DequantizeLinear") or i in drop:
            continue
        j = prod.get(op.inputs[0])
        if j is None or j in drop or graph.ops[j].op_type != "Conv":
            continue
        conv = graph.ops[j]
        if not only_reader(conv.outputs[0], i):
            continue
        pr = conv.params
        if tuple(pr["dilations"]) != (1, 1):
            continue
        d = conv_desc_of(graph, conv)
        if d.group != 1 and not (d.group == d.c_in and d.c_out % d.c_in == 0):
            continue
        chain = [i]
        if op.op_type == "Requantize":
            if len(op.inputs) > 1:
                M = np.asarray(inits[op.inputs[1]], np.float32)
            else:
                M = np.full(d.c_out, np.float32(op.params["scale"]), np.float32)
            D = M
            out = op.outputs[0]
            s_out = graph.tensors[out].scale
            d.epilogue = L.EPI_NONE
            nxt = cons.get(out, [])
            if len(nxt) == 1 and out not in graph.outputs:
                k = nxt[0]
                a = graph.ops[k]
                if a.op_type == "Relu":
                    d.epilogue, out = L.EPI_RELU, a.outputs[0]
                    chain.append(k)
                elif a.op_type == "Clip" and float(a.params.get("min", 0.0)) == 0.0 and \
                        float(a.params.get("max", 0.0)) == 6.0 and s_out:
                    d.epilogue, out = L.EPI_RELU6, a.outputs[0]
                    chain.append(k)
            d.q6 = Q.relu6_ceiling(s_out) if s_out else 127
            d.inv_s_out = float(np.float32(1.0) / np.float32(s_out)) if s_out else 0.0
        else:
            # SiLU: DequantizeLinear -> SiLU -> QuantizeLinear, each the previous one's only reader
            D = np.asarray(inits[op.inputs[1]], np.float32)
            M = D
            t1 = op.outputs[0]
            c1 = cons.get(t1, [])
            if len(c1) != 1 or t1 in graph.outputs or graph.ops[c1[0]].op_type != "SiLU":
                continue
            k1 = c1[0]
            t2 = graph.ops[k1].outputs[0]
            c2 = cons.get(t2, [])
            if len(c2) != 1 or t2 in graph.outputs or graph.ops[c2[0]].op_type != "QuantizeLinear":
                continue
            k2 = c2[0]
            s_out = float(graph.ops[k2].params["scale"])
            out = graph.ops[k2].outputs[0]
            chain += [k1, k2]
            d.epilogue = L.EPI_SILU
            d.q6 = Q.relu6_ceiling(s_out)
            d.inv_s_out = float(np.float32(1.0) / np.float32(s_out))
        x, wn = conv.inputs[0], conv.inputs[1]
        bn = conv.inputs[2] if len(conv.inputs) > 2 and conv.inputs[2] else None
        if bn is None:
            bn = conv.name + "_b"
            inits[bn] = np.zeros(d.c_out, np.int32)
        mn, dn = conv.name + "_M", conv.name + "_D"
        inits[mn] = np.ascontiguousarray(M, np.float32)
        inits[dn] = np.ascontiguousarray(D, np.float32)
        repl[j] = CompiledOp(conv.name, "Conv2dRequantReluI8Nhwc", [x, wn, bn, mn, dn], [out], {"desc": d})
        drop.update(chain)
    ops = [repl.get(i, op) for i, op in enumerate(graph.ops) if i not in drop]
    g = Graph(dict(graph.tensors), ops, inits, list(graph.inputs), list(graph.outputs), dict(graph.views))
    return _rebuild(g, ops)


def apply_fusion_passes(graph: Graph) -> Graph:
    """apply_fusion_passes (fusion.rs:42): the SiLU pass, then the int8
    Conv -> Requantize / DequantizeLinear chain pass."""
    if any(op.op_type == "Sigmoid" for op in graph.ops):
        graph = fuse_silu(graph)
    if any(op.op_type in ("Requantize", "DequantizeLinear") for op in graph.ops):
        graph = fuse_conv_requant_i8(graph)
    return graph


def lower_for_device(graph: Graph, residual_i8: bool = False) -> Graph:
    """The device passes: the op-fusion passes over an unfused int8 graph, fp16
    residual fusion, the input-conv unfold / im2col,
    int8 residual fusion (opt-in, `residual_i8`: on YOLOv8n at batch 32 the
    two pairs it takes are faster per kernel, yet the whole step measured
    2.177 ms against 2.159 without it), chained maxpools, then concat views."""
    if any(op.op_type in UNFUSED_OPS for op in graph.ops):
        graph = apply_fusion_passes(graph)
    if any(op.op_type == "AddF16" for op in graph.ops):
        graph = fuse_residual_f16(graph)
    if any(op.op_type == "CastF32ToF16" for op in graph.ops):
        graph = lower_unfold_stem_f16(graph)
    if any(op.op_type == "QuantizeU8" for op in graph.ops):
        graph = lower_im2col_input_i8(graph)
    if residual_i8 and any(op.op_type == "AddQuantized" for op in graph.ops):
        graph = fuse_residual_i8(graph)
    if sum(op.op_type == "MaxPool" for op in graph.ops) > 1:
        graph = fuse_maxpool_chain_i8(graph)
    if any(op.op_type == "Concat" for op in graph.ops):
        graph = lower_concat_views_i8(graph)
    return graph


# ---------------------------------------------------------------------------
# network builders (synthetic weights with the published architectures' shapes)
# ---------------------------------------------------------------------------

def resnet50_fp16(batch=128, size=224, classes=1000, seed=50, stages=(3, 4, 6, 3)):
    """ResNet-50-architecture fp16 graph: 7x7/2 stem + 3x3/2 max pool, bottleneck
    stages [3, 4, 6, 3] at output widths 256/512/1024/2048 (stride 2 in the 3x3
    conv of each stage's first block, 1x1 projection shortcut there), BN folded
    into every conv, ReLU, global average pool, FC to `classes`.  Input f32 NHWC
    (3 channels); output f32 logits.  The
    last conv of each residual branch carries a folded-BN scale of 0.5 so the
    residual stream of random weights stays well inside the f16 range."""
    b = F16GraphBuilder(seed)
    x = b.input_f32("image", (batch, size, size, 3))
    x = b.conv(x, 64, k=7, s=2, name="stem")
    x = b.maxpool(x, 3, 2, 1, name="stem_pool")
    c = 64
    for si, (nb, width) in enumerate(zip(stages, (64, 128, 256, 512))):
        for bi in range(nb):
            s = 2 if (bi == 0 and si > 0) else 1
            pre = f"s{si + 1}b{bi + 1}"
            y = b.conv(x, width, k=1, name=pre + "_a")
            y = b.conv(y, width, k=3, s=s, name=pre + "_b")
            y = b.conv(y, 4 * width, k=1, relu=False, gamma=0.5, name=pre + "_c")
            sc = b.conv(x, 4 * width, k=1, s=s, relu=False, name=pre + "_proj") if bi == 0 else x
            x = b.add_relu(y, sc, name=pre + "_add")
            c = 4 * width
    x = b.global_avgpool(x, name="gap")
    x = b.fc(x, classes, name="fc")
    b.output_f32(x, "logits")
    return b.g


def mobilenetv2_block(batch=32, h=112, w=112, c=96, expand=6, seed=2, unfused=False):
    """MobileNetV2 inverted-residual block: 1x1 expand + ReLU6, depthwise 3x3 s1
    + ReLU6, 1x1 project (linear), residual add with requantisation.
    `unfused`: the convs in the reference quantizer's unfused form."""
    b = GraphBuilder(seed, unfused=unfused)
    x = b.input("x", (batch, h, w, c), "i8", b.act_scale())
    e = b.conv(x, c * expand, k=1, act="relu6", name="expand")
    d = b.conv(e, c * expand, k=3, group=c * expand, act="relu6", name="dw")
    p = b.conv(d, c, k=1, act="none", name="project")
    y = b.add(x, p, name="residual")
    b.output(y)
    return b.g


# postprocess_yolo's usual arguments (postprocess.rs:313-314): 0.25 / 0.45, for a 640x640 image
YOLO_POSTPROCESS = {"img_width": 640, "img_height": 640, "conf_threshold": 0.25, "iou_threshold": 0.45}


def yolov8n(batch=1, size=640, nc=80, reg_max=16, seed=8, width=0.25, depth=0.33, head="detections",
            unfused=False):
    """YOLOv8n-architecture INT8 graph: width 0.25, depth 0.33;
    CSPDarknet backbone of Conv(+folded BN)+SiLU layers and C2f blocks, SPPF with
    5x5 max pooling, PAN neck with nearest 2x upsampling and channel concat, and
    the decoupled detection head (box branch 4*reg_max channels, class branch nc
    channels) at strides 8/16/32.  The graph input is the uint8 image, normalised
    by 1/255 and quantised (QuantizeU8).  Tensors joined by a concat share one
    activation scale, so the concat moves bytes unchanged (the builder passes
    the scale to their producers).

    head: "raw" ends with the six head outputs dequantised to f32; "detect"
    adds the exported model's Detect tail (YoloDetect: output0 f32
    [batch, 4 + nc, 8400]); "detections" also runs postprocess_yolo on the
    device (YoloPostprocess: `detections` = dw_detection records [batch, 8400],
    image i's first `num_detections[i]` records its detections, the rest zero).
    `unfused`: every conv in the reference quantizer's unfused form (Conv ->
    Requantize, or the f32 SiLU chain), for the fusion passes."""
    ch = lambda c: int(round(c * width))  # noqa: E731
    rep = lambda n: max(round(n * depth), 1)  # noqa: E731
    b = GraphBuilder(seed, act_scale_range=(0.01, 0.1), unfused=unfused)
    img = b.input("image", (batch, size, size, 3), "u8", None)
    s_img = float(np.float32(1.0) / np.float32(127.0))
    x = b.g.add_tensor("image_q", (batch, size, size, 3), "i8", s_img)
    b.g.ops.append(CompiledOp("quantize_input", "QuantizeU8", [img], [x], {"scale": s_img}))

    def conv(t, c, k=3, s=1, act="silu", out_scale=None):
        return b.conv(t, c, k=k, s=s, act=act, out_scale=out_scale)

    def c2f(t, c_out, n, shortcut, out_scale=None):
        c = c_out // 2
        s_mid = b.act_scale()                       # cv1 output, both halves and the m outputs share it
        y = conv(t, 2 * c, k=1, out_scale=s_mid)
        parts = b.split(y, [c, c])
        outs = list(parts)
        cur = parts[1]
        for _ in range(n):
            h = conv(cur, c, k=3)
            if shortcut:
                h2 = conv(h, c, k=3)
                cur = b.add(cur, h2, out_scale=s_mid)
            else:
                cur = conv(h, c, k=3, out_scale=s_mid)
            outs.append(cur)
        cat = b.concat(outs)
        return conv(cat, c_out, k=1, out_scale=out_scale)

    def sppf(t, c_out, out_scale=None):
        c_ = b.g.tensors[t].shape[3] // 2
        s_mid = b.act_scale()
        y = conv(t, c_, k=1, out_scale=s_mid)
        ys = [y]
        for _ in range(3):
            ys.append(b.maxpool(ys[-1], 5, 1, 2))
        return conv(b.concat(ys), c_out, k=1, out_scale=out_scale)

    s_a = b.act_scale()  # shared by P4, P5 and the N4'->N5 downsample (joined by concats)
    s_b = b.act_scale()  # shared by P3, N4 and the N3->N4' downsample
    x = conv(x, ch(64), 3, 2)                        # 0  P1/2
    x = conv(x, ch(128), 3, 2)                       # 1  P2/4
    x = c2f(x, ch(128), rep(3), True)                # 2
    x = conv(x, ch(256), 3, 2)                       # 3  P3/8
    p3 = c2f(x, ch(256), rep(6), True, out_scale=s_b)  # 4
    x = conv(p3, ch(512), 3, 2)                      # 5  P4/16
    p4 = c2f(x, ch(512), rep(6), True, out_scale=s_a)  # 6
    x = conv(p4, ch(1024), 3, 2)                     # 7  P5/32
    x = c2f(x, ch(1024), rep(3), True)               # 8
    p5 = sppf(x, ch(1024), out_scale=s_a)            # 9
    x = b.concat([b.upsample2(p5), p4])              # 10, 11
    n4 = c2f(x, ch(512), rep(3), False, out_scale=s_b)  # 12
    x = b.concat([b.upsample2(n4), p3])              # 13, 14
    out3 = c2f(x, ch(256), rep(3), False)            # 15 (P3/8)
    x = b.concat([conv(out3, ch(256), 3, 2, out_scale=s_b), n4])  # 16, 17
    out4 = c2f(x, ch(512), rep(3), False)            # 18 (P4/16)
    x = b.concat([conv(out4, ch(512), 3, 2, out_scale=s_a), p5])  # 19, 20
    out5 = c2f(x, ch(1024), rep(3), False)           # 21 (P5/32)

    c_box = max(16, ch(256) // 4, reg_max * 4)
    c_cls = max(ch(256), min(nc, 100))
    heads = []
    for t in (out3, out4, out5):
        r = conv(conv(t, c_box, 3), c_box, 3)
        r = conv(r, 4 * reg_max, k=1, act="none")
        c = conv(conv(t, c_cls, 3), c_cls, 3)
        c = conv(c, nc, k=1, act="none")
        heads.append((r, c))
    if head == "raw":
        for i, (r, c) in enumerate(heads):
            for name, tq in ((f"box{i}", r), (f"cls{i}", c)):
                ti = b.g.tensors[tq]
                out = b.g.add_tensor(name, ti.shape, "f32", None)
                b.g.ops.append(CompiledOp(f"dequantize_{name}", "Dequantize", [tq], [out], {"scale": ti.scale}))
                b.output(out)
        return b.g
    # the exported model's Detect tail: DFL, dist2bbox x stride, sigmoid, concat
    anchors = sum(b.g.tensors[r].shape[1] * b.g.tensors[r].shape[2] for r, _ in heads)
    out0 = b.g.add_tensor("output0", (batch, 4 + nc, anchors), "f32", None)
    b.g.ops.append(CompiledOp("detect", "YoloDetect", [t for pair in heads for t in pair], [out0], {
        "nc": nc, "reg_max": reg_max, "strides": [8.0, 16.0, 32.0],
        "box_scales": [b.g.tensors[r].scale for r, _ in heads],
        "cls_scales": [b.g.tensors[c].scale for _, c in heads]}))
    if head == "detect":
        b.output(out0)
        return b.g
    dets = b.g.add_tensor("detections", (batch, anchors, ops.DETECTION_DTYPE.itemsize), "u8", None)
    cnt = b.g.add_tensor("num_detections", (batch,), "i32", None)
    b.g.ops.append(CompiledOp("postprocess", "YoloPostprocess", [out0], [dets, cnt],
                              dict(YOLO_POSTPROCESS, nc=nc, num_detections=anchors, flags=0)))
    b.output(dets)
    b.output(cnt)
    return b.g


# ---------------------------------------------------------------------------
# runtime
# ---------------------------------------------------------------------------

class CudaGraphRuntime:
    """Executes a Graph on one GPU (VulkanGraphRuntime::new / set_input_bytes /
    run / get_output_bytes, vulkan_runtime.rs:115, 359)."""

    def __init__(self, graph: Graph, backend: CudaBackend, fuse: bool = True, residual_i8: bool = False):
        if fuse:
            graph = lower_for_device(graph, residual_i8=residual_i8)
        self.graph = graph
        self.be = backend
        self.bufs: dict[str, CudaBuffer] = {}
        self._dispatch = []
        self._cgraph = None
        self._slot_graphs = []
        for name, t in graph.tensors.items():
            if name not in graph.views:
                self.bufs[name] = backend.alloc(t.nbytes)
        consts = {}
        for name, arr in graph.initializers.items():
            consts[name] = backend.upload_array(np.ascontiguousarray(arr))
        self._consts = consts
        for op in graph.ops:
            self._dispatch.append(self._compile(op))
        backend.synchronize(60000)

    def _loc(self, name):
        """(buffer, byte offset, pixel pitch, is_view) of a tensor (int8)."""
        root, off = name, 0
        while root in self.graph.views:
            root, o = self.graph.views[root]
            off += o
        return self.bufs[root], off, self.graph.tensors[root].shape[3], root != name

    def _cached(self, key, make):
        """A prepared constant (repacked weights, tables, workspaces), made once:
        compiling the op list again (slot graphs) reuses it."""
        if key not in self._consts:
            self._consts[key] = make()
        return self._consts[key]

    def _compile(self, op: CompiledOp):
        be, bufs, consts = self.be, self.bufs, self._consts
        t = op.op_type
        if t == "Conv2dRequantReluI8Nhwc":
            desc: ConvDesc = op.params["desc"]
            x, wn, bn, mn, dn = op.inputs
            wp = self._cached(wn + "_prep", lambda: ops.prepare_weights_i8(be, desc, consts[wn]))
            bb, bm, bd = consts[bn], consts[mn], consts[dn]
            xl, yl = self._loc(x), self._loc(op.outputs[0])
            if xl[3] or yl[3]:
                return lambda: ops.conv2d_i8_view(be, desc, xl[:3], wp, bb, bm, bd, yl[:3])
            bx, y = xl[0], yl[0]
            return lambda: ops.conv2d_i8(be, desc, bx, wp, bb, bm, bd, y)
        if t == "Conv2dAddI8":
            desc = op.params["desc"]
            x, wn, bn, mn, dn, rn = op.inputs
            wp = self._cached(wn + "_prep", lambda: ops.prepare_weights_i8(be, desc, consts[wn]))
            bb, bm, bd = consts[bn], consts[mn], consts[dn]
            xl, rl, yl = self._loc(x), self._loc(rn), self._loc(op.outputs[0])
            ra, rb = op.params["ra"], op.params["rb"]
            return lambda: ops.conv2d_add_i8_view(be, desc, xl[:3], wp, bb, bm, bd, rl[:3], ra, rb, yl[:3])
        if t == "AddQuantized":
            al, bl, ol = self._loc(op.inputs[0]), self._loc(op.inputs[1]), self._loc(op.outputs[0])
            ra, rb = op.params["scale_a_over_out"], op.params["scale_b_over_out"]
            if al[3] or bl[3] or ol[3]:
                n, h, w, c = self.graph.tensors[op.outputs[0]].shape
                return lambda: ops.add_i8_view(be, al[:3], bl[:3], ol[:3], n * h * w, c, ra, rb)
            a, b_, y = al[0], bl[0], ol[0]
            return lambda: ops.add_i8_packed(be, a, b_, y, ra, rb)
        if t == "MaxPoolChainI8":
            n, h, w, c = self.graph.tensors[op.inputs[0]].shape
            xl = self._loc(op.inputs[0])
            yls = [self._loc(o)[:3] for o in op.outputs]
            k = op.params["k"]
            return lambda: ops.maxpool_chain_i8_view(be, xl[:3], yls, n, h, w, c, k)
        if t == "MaxPool":
            n, h, w, c = self.graph.tensors[op.inputs[0]].shape
            k, s, p = op.params["k"], op.params["s"], op.params["pad"]
            xl, yl = self._loc(op.inputs[0]), self._loc(op.outputs[0])
            if xl[3] or yl[3]:
                return lambda: ops.maxpool_i8_view(be, xl[:3], yl[:3], n, h, w, c, k, k, s, s, (p, p, p, p))
            x, y = xl[0], yl[0]
            return lambda: ops.maxpool_i8(be, x, y, n, h, w, c, k, k, s, s, (p, p, p, p))
        if t == "Concat":
            xs = [bufs[i] for i in op.inputs]
            cs = op.params["channels"]
            n, h, w, _ = self.graph.tensors[op.outputs[0]].shape
            y = bufs[op.outputs[0]]
            return lambda: ops.concat_i8(be, xs, cs, n * h * w, y)
        if t == "Split":
            n, h, w, c = self.graph.tensors[op.inputs[0]].shape
            x, y = bufs[op.inputs[0]], bufs[op.outputs[0]]
            c0, cl = op.params["c0"], op.params["c_len"]
            return lambda: ops.slice_c_i8(be, x, y, n * h * w, c, c0, cl)
        if t == "Resize":
            n, h, w, c = self.graph.tensors[op.inputs[0]].shape
            _, ho, wo, _ = self.graph.tensors[op.outputs[0]].shape
            x, y = bufs[op.inputs[0]], bufs[op.outputs[0]]
            return lambda: ops.resize_nearest_i8(be, x, y, n, h, w, ho, wo, c)
        if t == "Conv2dStemU8I8":
            desc = op.params["desc"]
            x, wn, bn, mn, dn = op.inputs
            bx, y = bufs[x], bufs[op.outputs[0]]
            bw, bb, bm, bd = consts[wn], consts[bn], consts[mn], consts[dn]
            return lambda: ops.conv2d_stem_u8_i8(be, desc, bx, op.params["in_scale"], bw, bb, bm, bd, y)
        if t == "Im2colU8ToI8":
            x, y = bufs[op.inputs[0]], bufs[op.outputs[0]]
            n, h, w, c = self.graph.tensors[op.inputs[0]].shape
            pr = op.params
            return lambda: ops.im2col_u8_to_i8(be, x, y, n, h, w, c, pr["k_h"], pr["k_w"], pr["s_h"], pr["s_w"], pr["p_t"],
                                               pr["p_l"], pr["h_out"], pr["w_out"], pr["c_dst"], pr["scale"])
        if t == "QuantizeU8":
            x, y = bufs[op.inputs[0]], bufs[op.outputs[0]]
            s = op.params["scale"]
            return lambda: ops.quantize_u8_to_i8(be, x, y, s)
        if t == "Dequantize":
            x, y = bufs[op.inputs[0]], bufs[op.outputs[0]]
            s = op.params["scale"]
            return lambda: ops.dequantize_i8_packed_to_f32(be, x, y, s)
        if t == "YoloDetect":
            pr = op.params
            n = self.graph.tensors[op.inputs[0]].shape[0]
            grids = [tuple(self.graph.tensors[x].shape[1:3]) for x in op.inputs[0::2]]
            desc = ops.YoloDetectDesc(n, pr["nc"], grids, pr["strides"], pr["box_scales"], pr["cls_scales"],
                                      pr["reg_max"])
            tables = self._cached(op.name + "_tables", lambda: ops.prepare_yolo_detect(be, desc))
            boxes, clss = [bufs[x] for x in op.inputs[0::2]], [bufs[x] for x in op.inputs[1::2]]
            y = bufs[op.outputs[0]]
            return lambda: ops.yolo_detect_i8(be, desc, tables, boxes, clss, y)
        if t == "YoloPostprocess":
            pr = op.params
            n, A = self.graph.tensors[op.inputs[0]].shape[0], pr["num_detections"]
            ws = self._cached(op.name + "_workspace", lambda: be.alloc(ops.postprocess_yolo_workspace(n, A)))
            x, dets, cnt = bufs[op.inputs[0]], bufs[op.outputs[0]], bufs[op.outputs[1]]
            return lambda: ops.postprocess_yolo_device(be, x, n, pr["nc"], A, pr["img_width"], pr["img_height"],
                                                       pr["conf_threshold"], pr["iou_threshold"], pr["flags"], ws,
                                                       dets, cnt)
        # ---- fp16 path
        if t == "CastF32ToF16":
            x, y = bufs[op.inputs[0]], bufs[op.outputs[0]]
            n, h, w, _ = self.graph.tensors[op.inputs[0]].shape
            cs, cd = op.params["c_src"], op.params["c_dst"]
            return lambda: ops.cast_f32_to_f16(be, x, y, n * h * w, cs, cd)
        if t == "UnfoldF32ToF16":
            x, y = bufs[op.inputs[0]], bufs[op.outputs[0]]
            n, h, w, c = self.graph.tensors[op.inputs[0]].shape
            pr = op.params
            return lambda: ops.unfold_w_f32_to_f16(be, x, y, n, h, w, c, pr["k_w"], pr["stride_w"], pr["pad_l"],
                                                   pr["w_out"], pr["c_dst"])
        if t == "Conv2dF16":
            desc = op.params["desc"]
            x, wn, bn = op.inputs
            wp = self._cached(wn + "_prep", lambda: ops.prepare_weights_f16(be, desc, consts[wn]))
            bx, bb, y = bufs[x], consts[bn], bufs[op.outputs[0]]
            return lambda: ops.conv2d_f16(be, desc, bx, wp, bb, y)
        if t == "Conv2dAddF16":
            desc = op.params["desc"]
            x, wn, bn, rn = op.inputs
            wp = self._cached(wn + "_prep", lambda: ops.prepare_weights_f16(be, desc, consts[wn]))
            bx, bb, br, y = bufs[x], consts[bn], bufs[rn], bufs[op.outputs[0]]
            return lambda: ops.conv2d_add_f16(be, desc, bx, wp, bb, br, y)
        if t == "AddF16":
            a, b_ = bufs[op.inputs[0]], bufs[op.inputs[1]]
            y = bufs[op.outputs[0]]
            fn = ops.add_relu_fp16 if op.params.get("relu") else ops.add_fp16
            return lambda: fn(be, a, b_, y)
        if t == "MaxPoolF16":
            n, h, w, c = self.graph.tensors[op.inputs[0]].shape
            k, s, p = op.params["k"], op.params["s"], op.params["pad"]
            x, y = bufs[op.inputs[0]], bufs[op.outputs[0]]
            return lambda: ops.maxpool_f16(be, x, y, n, h, w, c, k, k, s, s, (p, p, p, p))
        if t == "GlobalAveragePoolF16":
            n, h, w, c = self.graph.tensors[op.inputs[0]].shape
            x, y = bufs[op.inputs[0]], bufs[op.outputs[0]]
            return lambda: ops.global_avgpool_f16(be, x, y, n, h, w, c)
        if t == "GemmF16":
            m, n, k = op.params["m"], op.params["n"], op.params["k"]
            x, wn, bn = op.inputs
            wp = self._cached(wn + "_prep", lambda: ops.prepare_gemm_b_f16(be, consts[wn], k, n))
            bx, bb, y = bufs[x], consts[bn], bufs[op.outputs[0]]
            return lambda: ops.gemm_f16_bias(be, bx, wp, bb, y, m, n, k)
        if t == "CastF16ToF32":
            x, y = bufs[op.inputs[0]], bufs[op.outputs[0]]
            return lambda: ops.cast_f16_to_f32(be, x, y)
        # ---- the reference's unfused int8 ops, where the fusion passes left them
        # (a conv whose accumulators have several readers): its own op set
        if t == "Conv":
            d = conv_desc_of(self.graph, op)
            pt, pl, pb, pr = d.pads
            bias = self.graph.initializers.get(op.inputs[2]) if len(op.inputs) > 2 and op.inputs[2] else None
            if d.group != 1 or pt != pb or pl != pr or (bias is not None and np.any(bias)):
                raise BackendError(L.DW_ERR_UNSUPPORTED, f"unfused Conv {op.name}: only the reference's form "
                                   "(group 1, symmetric pads, no bias) runs unfused; it did not fuse")
            x, wk, y = bufs[op.inputs[0]], consts[op.inputs[1]], bufs[op.outputs[0]]
            return lambda: ops.conv2d_i8_nhwc_packed(be, x, wk, y, d.n, d.h, d.w, d.c_in, d.c_out, d.k_h, d.k_w,
                                                     d.stride_h, d.stride_w, pt, pl)
        if t == "Requantize":
            M = (np.asarray(self.graph.initializers[op.inputs[1]], np.float32) if len(op.inputs) > 1
                 else np.array([op.params["scale"]], np.float32))
            if np.any(M != M[0]):
                raise BackendError(L.DW_ERR_UNSUPPORTED, f"unfused Requantize {op.name}: per-channel scales run "
                                   "only fused into the conv")
            x, y = bufs[op.inputs[0]], bufs[op.outputs[0]]
            scale = float(M[0])
            return lambda: ops.requantize_i32_to_i8_packed(be, x, y, scale)
        if t == "Relu":
            x, y = bufs[op.inputs[0]], bufs[op.outputs[0]]
            return lambda: ops.relu_i8_packed(be, x, y)
        raise BackendError(L.DW_ERR_UNSUPPORTED, f"unsupported op type {t} ({op.name})")

    # -- reference-style API ----------------------------------------------------
    def set_input_bytes(self, name: str, data) -> None:
        self.be.upload(self.bufs[name], data)

    def get_output_bytes(self, name: str) -> np.ndarray:
        return self.be.download_array(self.bufs[name], np.uint8)

    def get_output(self, name: str) -> np.ndarray:
        t = self.graph.tensors[name]
        return self.be.download_array(self.bufs[name], _NP[t.dtype], t.shape)

    def run(self) -> None:
        """Enqueues the whole forward pass (asynchronous; use synchronize or a
        download to wait).  Uses the captured CUDA graph when one exists."""
        if self._cgraph is not None:
            self.be._check(L.load().dw_graph_launch(self.be.handle, self._cgraph))
            return
        for fn in self._dispatch:
            fn()

    def _record(self, dispatch) -> ctypes.c_void_p:
        lib = L.load()
        self.be._check(lib.dw_capture_begin(self.be.handle))
        try:
            for fn in dispatch:
                fn()
        finally:
            g = ctypes.c_void_p()
            st = lib.dw_capture_end(self.be.handle, ctypes.byref(g))
        self.be._check(st)
        return g

    def capture(self) -> int:
        """Records the op list once as a CUDA graph; returns its kernel count."""
        before = self.be.launch_count()
        self._cgraph = self._record(self._dispatch)
        # a launch records its kernels; count them by replaying once
        self.run()
        self.be.synchronize(60000)
        return self.be.launch_count() - before

    def capture_slots(self, depth: int) -> list:
        """Records `depth` CUDA graphs of the op list for a serving loop.  Graph d
        reads the graph input from its own buffer and writes the graph outputs to
        its own buffers (slot 0: the runtime's buffers), so step i + 1's input can
        be uploaded and step i - 1's outputs read back while step i runs, with no
        device-side staging copies.  Intermediate tensors are shared: the graphs
        must run one after another on the backend stream.  Returns one
        (graph, {tensor name: buffer}) pair per slot."""
        g = self.graph
        if len(g.inputs) != 1:
            raise BackendError(L.DW_ERR_UNSUPPORTED, "capture_slots: one graph input expected")
        names = [g.inputs[0]] + list(g.outputs)
        if any(n in g.views for n in names):
            raise BackendError(L.DW_ERR_UNSUPPORTED, "capture_slots: graph input or output is a view")
        if self._slot_graphs:
            return self._slot_graphs
        base = {n: self.bufs[n] for n in names}
        try:
            for d in range(depth):
                slot = dict(base) if d == 0 else {n: self.be.alloc(g.tensors[n].nbytes) for n in names}
                self.bufs.update(slot)
                dispatch = [self._compile(op) for op in g.ops]
                self._slot_graphs.append((self._record(dispatch), slot))
        finally:
            self.bufs.update(base)
        return self._slot_graphs

    def launch_slot(self, d: int) -> None:
        self.be._check(L.load().dw_graph_launch(self.be.handle, self._slot_graphs[d][0]))

    def release(self) -> None:
        if self._cgraph is not None:
            L.load().dw_graph_destroy(self._cgraph)
            self._cgraph = None
        for graph, _ in self._slot_graphs:
            L.load().dw_graph_destroy(graph)
        self._slot_graphs = []

    def __del__(self):
        try:
            self.release()
        except Exception:
            pass


class PipelinedRunner:
    """Serving loop over a CudaGraphRuntime with the host copies overlapped.

    Two copy backends (their own streams on the same GPU) move data while the
    compute backend runs.  The runtime records `depth` CUDA graphs, each bound
    to its own input and output buffers (CudaGraphRuntime.capture_slots): step
    i uploads straight into slot i % depth's input buffer while step i - 1
    computes, runs that slot's graph, and its outputs are read back from the
    slot's output buffers while step i + 1 computes.  Events order the three
    streams; no device-to-device copy is made.  Every step copies its whole
    input to the device and its whole output to the host (what `run_steps`
    returns)."""

    def __init__(self, rt: "CudaGraphRuntime", depth: int = 2):
        self.rt, self.depth = rt, depth
        be = rt.be
        g = rt.graph
        if len(g.inputs) != 1:
            raise BackendError(L.DW_ERR_UNSUPPORTED, "PipelinedRunner: one graph input expected")
        self.up, self.down = CudaBackend(be.device), CudaBackend(be.device)
        self.in_name = g.inputs[0]
        self.in_bytes = g.tensors[self.in_name].nbytes
        self.out_names = list(g.outputs)
        self.out_sizes = [g.tensors[o].nbytes for o in self.out_names]
        self.out_bytes = sum(self.out_sizes)
        self.slots = rt.capture_slots(depth)
        ev = lambda b: [b.event() for _ in range(depth)]  # noqa: E731
        self.h2d_done, self.run_done, self.d2h_done = ev(self.up), ev(be), ev(self.down)
        self.steps = 0

    def step(self, host_in_ptr: int, host_out_ptr: int) -> None:
        """Enqueues one step: upload `in_bytes` from pinned `host_in_ptr`, run the
        graph, read all outputs back (concatenated) into pinned `host_out_ptr`."""
        i, d, be, rt = self.steps, self.steps % self.depth, self.rt.be, self.rt
        bufs = self.slots[d][1]
        if i >= self.depth:
            self.up.wait(self.run_done[d])  # the slot's previous step has read its input
        self.up.upload_async(bufs[self.in_name], host_in_ptr, self.in_bytes)
        self.up.record(self.h2d_done[d])
        be.wait(self.h2d_done[d])
        if i >= self.depth:
            be.wait(self.d2h_done[d])  # the slot's previous outputs reached the host
        rt.launch_slot(d)
        be.record(self.run_done[d])
        self.down.wait(self.run_done[d])
        off = 0
        for name, n in zip(self.out_names, self.out_sizes):
            self.down.download_async(bufs[name], host_out_ptr + off, n)
            off += n
        self.down.record(self.d2h_done[d])
        self.steps += 1

    def synchronize(self, timeout_ms: int = 600000) -> None:
        for b in (self.up, self.rt.be, self.down):
            b.synchronize(timeout_ms)

    def close(self) -> None:
        self.synchronize()
        for evs in (self.h2d_done, self.run_done, self.d2h_done):
            for e in evs:
                e.close()
        self.up.close()
        self.down.close()
