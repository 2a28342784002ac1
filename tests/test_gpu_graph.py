"""GPU parity of whole graphs: CudaGraphRuntime (eager dispatch and CUDA-graph
replay) against the oracle graph runner, bit-exact on every output; plus
size-independent properties on the full benchmark batch."""
import numpy as np
import pytest

import dragonwing_edge_rs_b200 as dw
from dragonwing_edge_rs_b200 import graph as G
from oracle.graph_ref import run_graph

pytestmark = pytest.mark.gpu


@pytest.fixture(scope="module")
def be():
    b = dw.CudaBackend(0)
    yield b
    b.close()


def test_mobilenetv2_block_small_batch(be):
    g = G.mobilenetv2_block(batch=2, seed=7)
    x = np.random.default_rng(3).integers(-128, 128, g.tensors["x"].nbytes).astype(np.int8)
    rt = G.CudaGraphRuntime(g, be)
    rt.set_input_bytes("x", x)
    rt.run()
    y_eager = rt.get_output(g.outputs[0])
    ref = run_graph(g, {"x": x}, threads=8)[g.outputs[0]]
    assert np.array_equal(y_eager, ref.reshape(y_eager.shape))
    kernels = rt.capture()
    assert kernels == len(rt.graph.ops) == len(g.ops)
    rt.run()
    y_graph = rt.get_output(g.outputs[0])
    assert np.array_equal(y_graph, y_eager)
    rt.release()


@pytest.mark.parametrize("head", ["raw", "detect", "detections"])
def test_yolov8n_int8_batch1_bit_exact(be, head):
    """BASELINE config 4 architecture at 640x640, batch 1, identical to the
    oracle graph run: the six head outputs (dequantised int8), the Detect
    tail's output0, or the post-processed detections and their counts."""
    g = G.yolov8n(batch=1, seed=8, head=head)
    img = np.random.default_rng(5).integers(0, 256, g.tensors["image"].nbytes).astype(np.uint8)
    rt = G.CudaGraphRuntime(g, be)
    rt.set_input_bytes("image", img)
    rt.capture()
    rt.run()
    ref = run_graph(g, {"image": img}, threads=8)
    for name in g.outputs:
        got = rt.get_output(name)
        exp = ref[name].reshape(got.shape)
        assert np.array_equal(got, exp), f"{name}: {int((got != exp).sum())} of {got.size} differ"
    rt.release()


def test_yolov8n_int8_residual_fusion_bit_exact(be):
    """The opt-in int8 residual fusion (two bottleneck convs carry their
    shortcut add, reading and writing concat views): output0 identical to
    the oracle's unfused graph."""
    g = G.yolov8n(batch=2, size=320, seed=8, head="detect")
    img = np.random.default_rng(6).integers(0, 256, g.tensors["image"].nbytes).astype(np.uint8)
    rt = G.CudaGraphRuntime(g, be, residual_i8=True)
    assert [op.op_type for op in rt.graph.ops].count("Conv2dAddI8") == 2
    rt.set_input_bytes("image", img)
    rt.run()
    ref = run_graph(g, {"image": img}, threads=8)
    for name in g.outputs:
        got = rt.get_output(name)
        assert np.array_equal(got, ref[name].reshape(got.shape)), name
    rt.release()


def test_yolov8n_batch_independence(be):
    """Batch 4: image i of the batch equals the same image run in a batch of 1
    (per-image independence, the property the multi-GPU sharding relies on)."""
    g4 = G.yolov8n(batch=4, seed=8)
    g1 = G.yolov8n(batch=1, seed=8)
    imgs = np.random.default_rng(6).integers(0, 256, g4.tensors["image"].nbytes).astype(np.uint8)
    rt4, rt1 = G.CudaGraphRuntime(g4, be), G.CudaGraphRuntime(g1, be)
    rt4.set_input_bytes("image", imgs)
    rt4.run()
    per = imgs.reshape(4, -1)
    for i in (0, 3):
        rt1.set_input_bytes("image", per[i])
        rt1.run()
        for name in g1.outputs:
            assert np.array_equal(rt4.get_output(name)[i], rt1.get_output(name)[0]), (i, name)


def test_mobilenetv2_block_full_batch_sampled(be):
    """BASELINE config 2 at its full batch (32): whole batch on the GPU, two
    sampled images checked against the oracle, and the per-image independence
    property (image i of the batch == the same image run alone)."""
    g = G.mobilenetv2_block(batch=32, seed=1234)
    x = np.random.default_rng(11).integers(-128, 128, g.tensors["x"].nbytes).astype(np.int8)
    rt = G.CudaGraphRuntime(g, be)
    rt.set_input_bytes("x", x)
    rt.capture()
    rt.run()
    y = rt.get_output(g.outputs[0])
    for i in (0, 31):
        ref = run_graph(g, {"x": x}, threads=8, batch_slice=(i, i + 1))[g.outputs[0]]
        assert np.array_equal(y[i], ref.reshape(y[i].shape)), f"image {i}"
    rt.release()


@pytest.mark.parametrize("depth", [2, 3])
def test_pipelined_runner_matches_sequential_runs(be, depth):
    """PipelinedRunner (one CUDA graph per slot bound to the slot's own input and
    output buffers; uploads and read-backs on copy streams, `depth` steps in
    flight) returns, per step, exactly what a plain run of that step's input
    returns."""
    from dragonwing_edge_rs_b200.graph import CudaGraphRuntime, PipelinedRunner, yolov8n
    g = yolov8n(batch=2, size=128, seed=21)
    rt = CudaGraphRuntime(g, be)
    name = rt.graph.inputs[0]
    n_in = rt.graph.tensors[name].nbytes
    outs = list(rt.graph.outputs)
    n_out = sum(rt.graph.tensors[o].nbytes for o in outs)
    rng = np.random.default_rng(22)
    inputs = [rng.integers(0, 256, n_in).astype(np.uint8) for _ in range(5)]
    expected = []
    for x in inputs:
        rt.set_input_bytes(name, x)
        rt.run()
        expected.append(np.concatenate([rt.get_output_bytes(o) for o in outs]))
    pr = PipelinedRunner(rt, depth=depth)
    hin = [be.host_alloc(n_in) for _ in inputs]
    hout = [be.host_alloc(n_out) for _ in inputs]
    for (p_in, a_in), x in zip(hin, inputs):
        a_in[:] = x
    for (p_in, _), (p_out, _) in zip(hin, hout):
        pr.step(p_in, p_out)
    pr.synchronize()
    for (_, a_out), e in zip(hout, expected):
        assert np.array_equal(a_out, e)
    pr.close()
    for p_, _ in hin + hout:
        be.host_free(p_)
    rt.release()


# ------------------------------------------------- graphs in the reference's unfused form

@pytest.mark.parametrize("head", ["raw", "detections"])
def test_unfused_yolov8n_fused_on_device_matches_unfused_oracle(be, head):
    """YOLOv8n built in the reference quantizer's unfused form (Conv ->
    Requantize, the f32 SiLU chain DequantizeLinear -> Sigmoid -> Mul ->
    QuantizeLinear): the runtime's fusion passes collapse it to the fused op and
    the device's outputs are identical to the oracle running the unfused graph op
    by op (its Sigmoid with the host libm's expf, as the reference's f32::exp)."""
    g = G.yolov8n(batch=1, seed=8, head=head, unfused=True)
    rt = G.CudaGraphRuntime(g, be)
    assert not any(op.op_type in G.UNFUSED_OPS for op in rt.graph.ops)
    x = np.random.default_rng(41).integers(0, 256, g.tensors[g.inputs[0]].nbytes).astype(np.uint8)
    rt.set_input_bytes(g.inputs[0], x)
    rt.run()
    ref = run_graph(g, {g.inputs[0]: x}, threads=16)
    for name in g.outputs:
        got = rt.get_output_bytes(name)
        exp = np.ascontiguousarray(ref[name]).view(np.uint8).reshape(-1)
        assert np.array_equal(got, exp), f"{name}: {int((got != exp).sum())} of {got.size} bytes differ"
    rt.release()


def test_unfused_mbv2_block_fused_on_device(be):
    g = G.mobilenetv2_block(batch=2, seed=7, unfused=True)
    rt = G.CudaGraphRuntime(g, be)
    assert [op.op_type for op in rt.graph.ops].count("Conv2dRequantReluI8Nhwc") == 3
    x = np.random.default_rng(5).integers(-128, 128, g.tensors["x"].nbytes).astype(np.int8)
    rt.set_input_bytes("x", x)
    rt.run()
    y = rt.get_output(g.outputs[0])
    ref = run_graph(g, {"x": x}, threads=16)[g.outputs[0]]
    assert np.array_equal(y, ref.reshape(y.shape))
    rt.release()


def test_unfused_reference_form_ops_run_on_device(be):
    """A conv whose accumulators have two readers stays unfused; its ops in the
    reference's own form (unbiased Conv to int32, scalar Requantize, Relu) run as
    the device's unfused entry points and match the oracle."""
    from dragonwing_edge_rs_b200.graph import CompiledOp, Graph
    rng = np.random.default_rng(17)
    g = Graph({}, [], {}, ["x"], ["r1", "q2"])
    g.add_tensor("x", (2, 12, 10, 16), "i8", 0.02)
    g.add_tensor("acc", (2, 12, 10, 32), "i32")
    g.initializers["w"] = rng.integers(-127, 128, (3, 3, 16, 32)).astype(np.int8)
    g.ops.append(CompiledOp("conv", "Conv", ["x", "w"], ["acc"],
                            {"kernel_shape": (3, 3), "strides": (1, 1), "pads": (1, 1, 1, 1), "dilations": (1, 1),
                             "group": 1}))
    for t in ("q1", "r1", "q2"):
        g.add_tensor(t, (2, 12, 10, 32), "i8", 0.05)
    g.ops += [CompiledOp("rq1", "Requantize", ["acc"], ["q1"], {"scale": 0.0021}),
              CompiledOp("relu", "Relu", ["q1"], ["r1"], {}),
              CompiledOp("rq2", "Requantize", ["acc"], ["q2"], {"scale": 0.0013})]
    rt = G.CudaGraphRuntime(g, be)
    assert [op.op_type for op in rt.graph.ops] == ["Conv", "Requantize", "Relu", "Requantize"]
    x = rng.integers(-64, 64, g.tensors["x"].nbytes).astype(np.int8)
    rt.set_input_bytes("x", x)
    rt.run()
    ref = run_graph(g, {"x": x}, threads=8)
    for name in g.outputs:
        assert np.array_equal(rt.get_output(name), ref[name].reshape(g.tensors[name].shape)), name
    rt.release()
