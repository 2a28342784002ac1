"""The op-fusion passes over the reference's unfused int8 IR (CPU).

Mirrors the reference's fusion tests (crates/dragonwing-onnx/src/fusion.rs:
424-706): pattern counts, the Conv -> Requantize -> Relu 3 -> 1 collapse and
its has_relu flag, the Conv -> Requantize collapse, the group != 1 refusal;
plus the contract's extensions (int32 bias, per-channel M, Clip(0, 6) as
ReLU6, the SiLU chain, depthwise) and the consumer rules (a tensor with
several readers, or a graph output, stops the chain).  Then whole graphs:
YOLOv8n and the MobileNetV2 block built unfused collapse to exactly the fused
builders' op lists, and the oracle gives identical outputs for both forms."""
import numpy as np
import pytest

from dragonwing_edge_rs_b200 import _lib as L
from dragonwing_edge_rs_b200 import graph as G
from dragonwing_edge_rs_b200.graph import CompiledOp, Graph
from oracle.graph_ref import run_graph


def conv_params(k=3, s=1, p=1, group=1):
    return {"kernel_shape": (k, k), "strides": (s, s), "pads": (p, p, p, p), "dilations": (1, 1), "group": group}


def base_graph(c_in=8, c_out=8, group=1, bias=False, k=3):
    """x [1, 6, 6, c_in] -> Conv -> conv_out_i32 (the accumulator, shaped)."""
    g = Graph({}, [], {}, ["x"], [])
    g.add_tensor("x", (1, 6, 6, c_in), "i8", 0.02)
    g.add_tensor("conv_out_i32", (1, 6, 6, c_out), "i32")
    g.initializers["w"] = np.ones((k, k, c_in if group == 1 else 1, c_out if group == 1 else c_out // c_in), np.int8)
    ins = ["x", "w"]
    if bias:
        g.initializers["b"] = np.arange(c_out, dtype=np.int32)
        ins.append("b")
    g.ops.append(CompiledOp("conv1", "Conv", ins, ["conv_out_i32"], conv_params(k=k, group=group)))
    return g


def add_requant(g, scale=0.0125, out="conv_out", per_channel=None):
    g.add_tensor(out, g.tensors["conv_out_i32"].shape, "i8", 0.05)
    ins = ["conv_out_i32"]
    if per_channel is not None:
        g.initializers["M"] = np.asarray(per_channel, np.float32)
        ins.append("M")
    g.ops.append(CompiledOp("conv1_requant", "Requantize", ins, [out], {"scale": scale}))
    return out


def test_fusion_stats_empty():
    assert G.count_fuseable_patterns(Graph({}, [], {}, [], [])).total() == 0


def test_conv_relu_detection():
    g = Graph({}, [], {}, ["input"], ["relu_out"])
    g.add_tensor("input", (1, 4, 4, 4), "f32")
    g.add_tensor("conv_out", (1, 4, 4, 4), "f32")
    g.add_tensor("relu_out", (1, 4, 4, 4), "f32")
    g.ops += [CompiledOp("conv1", "Conv", ["input"], ["conv_out"], conv_params()),
              CompiledOp("relu1", "Relu", ["conv_out"], ["relu_out"], {})]
    assert G.count_fuseable_patterns(g).conv_relu == 1


def test_silu_detection_and_pass2():
    g = Graph({}, [], {}, ["x"], ["silu_out"])
    for t in ("x", "sig_out", "silu_out"):
        g.add_tensor(t, (1, 4, 4, 4), "f32")
    g.ops += [CompiledOp("sigmoid1", "Sigmoid", ["x"], ["sig_out"], {}),
              CompiledOp("mul1", "Mul", ["x", "sig_out"], ["silu_out"], {})]
    assert G.count_fuseable_patterns(g).silu == 1
    f = G.fuse_silu(g)
    assert [op.op_type for op in f.ops] == ["SiLU"]
    assert f.ops[0].inputs == ["x"] and f.ops[0].outputs == ["silu_out"]
    # operand order does not matter; a Sigmoid output with another reader does not fuse
    g.ops[1].inputs = ["sig_out", "x"]
    assert [op.op_type for op in G.fuse_silu(g).ops] == ["SiLU"]
    g.outputs.append("sig_out")
    assert [op.op_type for op in G.fuse_silu(g).ops] == ["Sigmoid", "Mul"]


def test_conv_requant_relu_i8_fusion():
    """fusion.rs:511-569: Conv -> Requantize -> Relu collapses 3 -> 1."""
    g = base_graph()
    add_requant(g)
    g.add_tensor("relu_out", (1, 6, 6, 8), "i8", 0.05)
    g.ops.append(CompiledOp("relu1", "Relu", ["conv_out"], ["relu_out"], {}))
    g.outputs.append("relu_out")
    assert G.count_fuseable_patterns(g).conv_requant_relu_i8 == 1
    f = G.apply_fusion_passes(g)
    assert len(f.ops) == 1, "should collapse 3 ops to 1"
    op = f.ops[0]
    assert op.op_type == "Conv2dRequantReluI8Nhwc"
    assert op.outputs == ["relu_out"]
    d = op.params["desc"]
    assert (d.k_h, d.k_w, d.stride_h, d.stride_w, d.pads, d.group) == (3, 3, 1, 1, (1, 1, 1, 1), 1)
    assert d.epilogue == L.EPI_RELU                                   # has_relu
    assert np.all(f.initializers[op.inputs[3]] == np.float32(0.0125))  # the scalar scale as M
    assert not np.any(f.initializers[op.inputs[2]])                    # no bias: zeros
    assert "conv_out" not in f.tensors and "conv_out_i32" not in f.tensors


def test_conv_requant_only_fusion():
    """fusion.rs:572-614: no Relu -> still fused, has_relu false."""
    g = base_graph()
    add_requant(g, scale=0.02)
    g.outputs.append("conv_out")
    f = G.apply_fusion_passes(g)
    assert len(f.ops) == 1 and f.ops[0].outputs == ["conv_out"]
    assert f.ops[0].params["desc"].epilogue == L.EPI_NONE


def test_conv_requant_skipped_when_group_ne_1():
    """fusion.rs:617-660: a grouped conv is not fused.  The contract's
    extension fuses depthwise (group == c_in) convs; other groups still refuse."""
    g = base_graph(c_in=8, c_out=8, group=2)
    g.initializers["w"] = np.ones((3, 3, 4, 8), np.int8)
    add_requant(g)
    g.outputs.append("conv_out")
    assert len(G.apply_fusion_passes(g).ops) == 2
    d = base_graph(c_in=8, c_out=16, group=8)
    add_requant(d)
    d.outputs.append("conv_out")
    f = G.apply_fusion_passes(d)
    assert len(f.ops) == 1 and f.ops[0].params["desc"].group == 8


def test_biased_conv_and_per_channel_scales_fuse():
    """The reference refuses biased convs (fusion.rs:303-309) and averages the
    channel scales (quantize.rs:307-325): the contract keeps both."""
    g = base_graph(bias=True)
    M = np.linspace(0.001, 0.002, 8).astype(np.float32)
    add_requant(g, per_channel=M)
    g.outputs.append("conv_out")
    f = G.apply_fusion_passes(g)
    op = f.ops[0]
    assert op.inputs[2] == "b" and np.array_equal(f.initializers["b"], np.arange(8, dtype=np.int32))
    assert np.array_equal(f.initializers[op.inputs[3]], M)


def test_clip_0_6_is_relu6_and_other_clips_stay():
    g = base_graph()
    add_requant(g)
    g.add_tensor("y", (1, 6, 6, 8), "i8", 0.05)
    g.ops.append(CompiledOp("clip1", "Clip", ["conv_out"], ["y"], {"min": 0.0, "max": 6.0}))
    g.outputs.append("y")
    f = G.apply_fusion_passes(g)
    d = f.ops[0].params["desc"]
    assert len(f.ops) == 1 and d.epilogue == L.EPI_RELU6 and d.q6 == 120  # round(6 / 0.05)
    g.ops[-1].params["max"] = 4.0
    f = G.apply_fusion_passes(g)
    assert [op.op_type for op in f.ops] == ["Conv2dRequantReluI8Nhwc", "Clip"]
    assert f.ops[0].params["desc"].epilogue == L.EPI_NONE


def test_silu_chain_fuses():
    g = base_graph()
    shape = (1, 6, 6, 8)
    g.initializers["D"] = np.full(8, 0.0004, np.float32)
    for t in ("deq", "sig", "silu"):
        g.add_tensor(t, shape, "f32")
    g.add_tensor("y", shape, "i8", 0.04)
    g.ops += [CompiledOp("deq", "DequantizeLinear", ["conv_out_i32", "D"], ["deq"], {}),
              CompiledOp("sigmoid", "Sigmoid", ["deq"], ["sig"], {}),
              CompiledOp("mul", "Mul", ["deq", "sig"], ["silu"], {}),
              CompiledOp("quant", "QuantizeLinear", ["silu"], ["y"], {"scale": 0.04})]
    g.outputs.append("y")
    f = G.apply_fusion_passes(g)
    assert len(f.ops) == 1 and f.ops[0].outputs == ["y"]
    d = f.ops[0].params["desc"]
    assert d.epilogue == L.EPI_SILU and d.inv_s_out == pytest.approx(25.0)
    assert np.array_equal(f.initializers[f.ops[0].inputs[4]], g.initializers["D"])


def test_consumer_rules_stop_the_chain():
    # the accumulator has a second reader: nothing fuses
    g = base_graph()
    add_requant(g)
    g.add_tensor("conv_out2", (1, 6, 6, 8), "i8", 0.05)
    g.ops.append(CompiledOp("requant2", "Requantize", ["conv_out_i32"], ["conv_out2"], {"scale": 0.01}))
    g.outputs += ["conv_out", "conv_out2"]
    assert [op.op_type for op in G.apply_fusion_passes(g).ops] == ["Conv", "Requantize", "Requantize"]
    # the requantised tensor has two readers: Conv + Requantize fuse, the Relu stays
    g = base_graph()
    add_requant(g)
    for t in ("r1", "r2"):
        g.add_tensor(t, (1, 6, 6, 8), "i8", 0.05)
    g.ops += [CompiledOp("relu1", "Relu", ["conv_out"], ["r1"], {}),
              CompiledOp("relu2", "Relu", ["conv_out"], ["r2"], {})]
    g.outputs += ["r1", "r2"]
    f = G.apply_fusion_passes(g)
    assert [op.op_type for op in f.ops] == ["Conv2dRequantReluI8Nhwc", "Relu", "Relu"]
    assert f.ops[0].params["desc"].epilogue == L.EPI_NONE and f.ops[0].outputs == ["conv_out"]
    # a graph output in the middle keeps that tensor: the Relu is not absorbed
    g = base_graph()
    add_requant(g)
    g.add_tensor("relu_out", (1, 6, 6, 8), "i8", 0.05)
    g.ops.append(CompiledOp("relu1", "Relu", ["conv_out"], ["relu_out"], {}))
    g.outputs += ["conv_out", "relu_out"]
    assert [op.op_type for op in G.apply_fusion_passes(g).ops] == ["Conv2dRequantReluI8Nhwc", "Relu"]


@pytest.mark.parametrize("builder,kw", [(G.yolov8n, {"batch": 1, "size": 128, "head": "raw"}),
                                        (G.mobilenetv2_block, {"batch": 2, "h": 16, "w": 16})],
                         ids=["yolov8n", "mbv2_block"])
def test_unfused_graphs_collapse_to_the_fused_builders(builder, kw):
    fused = builder(**kw)
    unfused = builder(unfused=True, **kw)
    assert G.count_fuseable_patterns(unfused).conv_requant_relu_i8 == sum(
        op.op_type == "Conv2dRequantReluI8Nhwc" for op in fused.ops)
    got = G.apply_fusion_passes(unfused)
    assert [op.op_type for op in got.ops] == [op.op_type for op in fused.ops]
    for a, b in zip(got.ops, fused.ops):
        assert a.name == b.name and a.outputs == b.outputs and a.inputs[:3] == b.inputs[:3]
        if a.op_type == "Conv2dRequantReluI8Nhwc":
            assert a.params["desc"] == b.params["desc"]
            used = 4 if a.params["desc"].epilogue == L.EPI_SILU else 3
            assert np.array_equal(got.initializers[a.inputs[used]], fused.initializers[b.inputs[used]])
    # the oracle: the unfused graph (the reference's op-by-op composition, the
    # SiLU chain with libm's expf) gives the fused graph's outputs
    rng = np.random.default_rng(3)
    t = unfused.tensors[unfused.inputs[0]]
    x = (rng.integers(0, 256, t.nbytes).astype(np.uint8) if t.dtype == "u8"
         else rng.integers(-128, 128, t.nbytes).astype(np.int8))
    a = run_graph(unfused, {unfused.inputs[0]: x}, threads=8)
    b = run_graph(fused, {fused.inputs[0]: x}, threads=8)
    for name in fused.outputs:
        assert np.array_equal(a[name], b[name]), name
