"""The int8 device passes' host logic on the CPU: which ops
fuse_maxpool_chain_i8 and fuse_residual_i8 take (run lengths, strided or
branching pools, channel counts, the epilogue-slack rule, a conv output read
twice or exported), and that the lowered graph, run op by op with the
oracle's ops, gives exactly the unlowered graph's outputs."""
import numpy as np

from dragonwing_edge_rs_b200 import graph as G
from oracle.graph_ref import run_graph


def _same_outputs(g0, g1, seed):
    x = np.random.default_rng(seed).integers(-128, 128, g0.tensors[g0.inputs[0]].nbytes).astype(np.int8)
    ref = run_graph(g0, {g0.inputs[0]: x}, threads=4)
    got = run_graph(g1, {g0.inputs[0]: x}, threads=4)
    for name in g0.outputs:
        assert np.array_equal(got[name], ref[name]), name


def test_maxpool_chain_runs():
    b = G.GraphBuilder(3)
    x = b.input("x", (2, 9, 11, 32), "i8", 0.05)
    p = x
    run = []
    for _ in range(5):                      # five 5x5 pools in a row: a run of four, then one alone
        p = b.maxpool(p, 5, 1, 2)
        run.append(p)
    q = b.maxpool(p, 3, 2, 1)               # strided: not chained
    r1 = b.maxpool(x, 3, 1, 1)              # read by two pools: no run
    s1, s2 = b.maxpool(r1, 3, 1, 1), b.maxpool(r1, 3, 1, 1)
    y = b.input("y", (2, 7, 7, 8), "i8", 0.05)  # 8 channels: not fused
    t = b.maxpool(b.maxpool(y, 3, 1, 1), 3, 1, 1)
    for o in (run[1], run[3], q, s1, s2, t):
        b.output(o)
    g0 = b.g
    g1 = G.fuse_maxpool_chain_i8(g0)
    kinds = [op.op_type for op in g1.ops]
    assert kinds.count("MaxPoolChainI8") == 1 and kinds.count("MaxPool") == 7
    chain = next(op for op in g1.ops if op.op_type == "MaxPoolChainI8")
    assert chain.inputs == [x] and chain.outputs == run[:4] and chain.params["k"] == 5
    # every tensor still has its producer, before its readers
    made = set(g1.inputs)
    for op in g1.ops:
        assert all(i in made or i in g1.initializers for i in op.inputs)
        made.update(op.outputs)
    xs = np.random.default_rng(4)
    feeds = {n: xs.integers(-128, 128, g0.tensors[n].nbytes).astype(np.int8) for n in g0.inputs}
    ref, got = run_graph(g0, feeds, threads=4), run_graph(g1, feeds, threads=4)
    for name in g0.outputs:
        assert np.array_equal(got[name], ref[name]), name


def test_residual_fusion_rules():
    b = G.GraphBuilder(5)
    x = b.input("x", (1, 6, 6, 16), "i8", 0.05)
    c1 = b.conv(x, 16, k=3, act="silu")
    a1 = b.add(c1, x)                        # the conv is the add's first operand: roles swapped
    c5 = b.conv(a1, 16, k=3, act="silu")
    a4 = b.add(a1, c5)                       # fused
    c6 = b.conv(a4, 16, k=3, act="silu")
    b.output(c6)                             # exported: not fused
    a6 = b.add(a4, c6)
    c7, c8 = b.conv(a6, 32, k=1, act="relu"), b.conv(a6, 32, k=1, act="relu")
    a7 = b.add(c7, c8)                       # 1x1 on 16 channels into 32: no epilogue slack, not fused
    b.output(a7)
    g0 = b.g
    g1 = G.fuse_residual_i8(g0)
    fused = [op for op in g1.ops if op.op_type == "Conv2dAddI8"]
    assert [op.name for op in fused] == [f"{c1[:-4]}+{a1[:-4]}", f"{c5[:-4]}+{a4[:-4]}"]
    r0 = next(op for op in g0.ops if op.outputs[0] == a1).params
    assert fused[0].inputs[5] == x and fused[0].params["ra"] == r0["scale_b_over_out"]
    assert fused[0].params["rb"] == r0["scale_a_over_out"]
    assert c1 not in g1.tensors and c6 in g1.tensors
    _same_outputs(g0, g1, 6)
