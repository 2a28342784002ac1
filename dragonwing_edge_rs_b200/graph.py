"""Graph IR and CUDA graph runtime for fused-INT8 networks.

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

_NP = {"i8": np.int8, "u8": np.uint8, "f32": np.float32, "i32": np.int32}


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
    Resize, QuantizeU8, Dequantize."""

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

    def add_tensor(self, name, shape, dtype="i8", scale=None):
        self.tensors[name] = TensorInfo(name, tuple(int(s) for s in shape), dtype, scale)
        return name

    # ---- work accounting (algorithmic ops = 2*MACs, padding taps included) ----
    def conv_ops(self):
        total = 0
        for op in self.ops:
            if op.op_type == "Conv2dRequantReluI8Nhwc":
                d: ConvDesc = op.params["desc"]
                ho, wo = d.out_hw()
                per = d.k_h * d.k_w * (d.c_in if d.group == 1 else 1)
                total += 2 * d.n * ho * wo * d.c_out * per
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

    def __init__(self, seed: int, act_scale_range=(0.01, 0.05)):
        self.rng = np.random.default_rng(seed)
        self.lo, self.hi = act_scale_range
        self.g = Graph({}, [], {}, [], [])
        self._n = 0

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
        for suffix, arr in (("_w", w_layout), ("_b", bias), ("_M", Q.requant_scales(s_in, s_w, s_out)),
                            ("_D", Q.dequant_scales(s_in, s_w))):
            g.initializers[name + suffix] = arr
        g.ops.append(CompiledOp(name, "Conv2dRequantReluI8Nhwc", [x, name + "_w", name + "_b", name + "_M", name + "_D"],
                                [y], {"desc": desc}))
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


# ---------------------------------------------------------------------------
# network builders (synthetic weights with the published architectures' shapes)
# ---------------------------------------------------------------------------

def mobilenetv2_block(batch=32, h=112, w=112, c=96, expand=6, seed=2):
    """MobileNetV2 inverted-residual block: 1x1 expand + ReLU6, depthwise 3x3 s1
    + ReLU6, 1x1 project (linear), residual add with requantisation."""
    b = GraphBuilder(seed)
    x = b.input("x", (batch, h, w, c), "i8", b.act_scale())
    e = b.conv(x, c * expand, k=1, act="relu6", name="expand")
    d = b.conv(e, c * expand, k=3, group=c * expand, act="relu6", name="dw")
    p = b.conv(d, c, k=1, act="none", name="project")
    y = b.add(x, p, name="residual")
    b.output(y)
    return b.g


# ---------------------------------------------------------------------------
# runtime
# ---------------------------------------------------------------------------

class CudaGraphRuntime:
    """Executes a Graph on one GPU (VulkanGraphRuntime::new / set_input_bytes /
    run / get_output_bytes, vulkan_runtime.rs:115, 359)."""

    def __init__(self, graph: Graph, backend: CudaBackend):
        self.graph = graph
        self.be = backend
        self.bufs: dict[str, CudaBuffer] = {}
        self._dispatch = []
        self._cgraph = None
        for name, t in graph.tensors.items():
            self.bufs[name] = backend.alloc(t.nbytes)
        consts = {}
        for name, arr in graph.initializers.items():
            consts[name] = backend.upload_array(np.ascontiguousarray(arr))
        self._consts = consts
        for op in graph.ops:
            self._dispatch.append(self._compile(op))
        backend.synchronize(60000)

    def _compile(self, op: CompiledOp):
        be, bufs, consts = self.be, self.bufs, self._consts
        t = op.op_type
        if t == "Conv2dRequantReluI8Nhwc":
            desc: ConvDesc = op.params["desc"]
            x, wn, bn, mn, dn = op.inputs
            wp = ops.prepare_weights_i8(be, desc, consts[wn])
            consts[wn + "_prep"] = wp
            y = bufs[op.outputs[0]]
            bx, bb, bm, bd = bufs[x], consts[bn], consts[mn], consts[dn]
            return lambda: ops.conv2d_i8(be, desc, bx, wp, bb, bm, bd, y)
        if t == "AddQuantized":
            a, b_ = bufs[op.inputs[0]], bufs[op.inputs[1]]
            y = bufs[op.outputs[0]]
            ra, rb = op.params["scale_a_over_out"], op.params["scale_b_over_out"]
            return lambda: ops.add_i8_packed(be, a, b_, y, ra, rb)
        if t == "MaxPool":
            n, h, w, c = self.graph.tensors[op.inputs[0]].shape
            k, s, p = op.params["k"], op.params["s"], op.params["pad"]
            x, y = bufs[op.inputs[0]], bufs[op.outputs[0]]
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
        if t == "QuantizeU8":
            x, y = bufs[op.inputs[0]], bufs[op.outputs[0]]
            s = op.params["scale"]
            return lambda: ops.quantize_u8_to_i8(be, x, y, s)
        if t == "Dequantize":
            x, y = bufs[op.inputs[0]], bufs[op.outputs[0]]
            s = op.params["scale"]
            return lambda: ops.dequantize_i8_packed_to_f32(be, x, y, s)
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

    def capture(self) -> int:
        """Records the op list once as a CUDA graph; returns its kernel count."""
        lib = L.load()
        before = self.be.launch_count()
        self.be._check(lib.dw_capture_begin(self.be.handle))
        try:
            for fn in self._dispatch:
                fn()
        finally:
            g = ctypes.c_void_p()
            st = lib.dw_capture_end(self.be.handle, ctypes.byref(g))
        self.be._check(st)
        self._cgraph = g
        # a launch records its kernels; count them by replaying once
        self.run()
        self.be.synchronize(60000)
        return self.be.launch_count() - before

    def release(self) -> None:
        if self._cgraph is not None:
            L.load().dw_graph_destroy(self._cgraph)
            self._cgraph = None

    def __del__(self):
        try:
            self.release()
        except Exception:
            pass
