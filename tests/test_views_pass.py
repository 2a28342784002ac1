"""The concat-view and residual-fusion device passes
(dragonwing_edge_rs_b200.graph.lower_concat_views_i8, fuse_residual_i8) on the CPU: the lowered YOLOv8n graph, executed op by op with the oracle's
ops and the views honoured (a producer writes its channel range of the root
buffer, a consumer reads its range), gives exactly the unlowered graph's
outputs; and the views are well formed."""
import numpy as np

from dragonwing_edge_rs_b200 import graph as G
from oracle.graph_ref import run_graph


def resolve(g, t):
    root, off = t, 0
    while root in g.views:
        root, o = g.views[root]
        off += o
    return root, off


def run_with_views(g, feeds):
    vals, roots = {}, {}
    for name, arr in feeds.items():
        vals[name] = np.asarray(arr).reshape(g.tensors[name].shape)

    def read(t):
        root, off = resolve(g, t)
        if root == t and t not in roots:
            return vals[t]
        c = g.tensors[t].shape[3]
        return np.ascontiguousarray(roots[root][..., off:off + c])

    def write(t, arr):
        root, off = resolve(g, t)
        arr = np.asarray(arr).reshape(g.tensors[t].shape)
        if root == t:
            if t in roots:
                roots[t][...] = arr
            else:
                vals[t] = arr
            return
        if root not in roots:
            rt = g.tensors[root]
            roots[root] = np.full(rt.shape, 99, np.int8)  # unwritten channels would show
        c = g.tensors[t].shape[3]
        roots[root][..., off:off + c] = arr

    for op in g.ops:
        ins = [i for i in op.inputs if i in g.tensors]
        sub = G.Graph({k: g.tensors[k] for k in ins + op.outputs}, [op],
                      {k: g.initializers[k] for k in op.inputs if k in g.initializers}, ins, list(op.outputs))
        out = run_graph(sub, {i: read(i) for i in ins}, threads=8)
        for o in op.outputs:
            write(o, out[o])
    return {o: read(o) for o in g.outputs}


def test_views_pass_yolov8n_equals_unlowered():
    g0 = G.yolov8n(batch=1, size=320, seed=8, head="detect")
    g = G.lower_concat_views_i8(G.fuse_maxpool_chain_i8(G.fuse_residual_i8(G.lower_im2col_input_i8(g0))))
    kinds = [op.op_type for op in g.ops]
    assert kinds.count("MaxPoolChainI8") == 1 and kinds.count("MaxPool") == 0  # SPPF
    assert kinds.count("Split") == 0 and kinds.count("Concat") == 4  # C2f and SPPF concats are views now
    assert kinds.count("Conv2dAddI8") == 2 and kinds.count("AddQuantized") == 4  # c_out 16 and 128 bottlenecks
    for t, (parent, off) in g.views.items():
        assert off % 16 == 0 and off + g.tensors[t].shape[3] <= g.tensors[parent].shape[3]
        assert g.tensors[t].shape[:3] == g.tensors[parent].shape[:3]
    img = np.random.default_rng(5).integers(0, 256, g0.tensors["image"].nbytes).astype(np.uint8)
    ref = run_graph(g0, {"image": img}, threads=8)
    got = run_with_views(g, {"image": img})
    for name in g0.outputs:
        assert np.array_equal(got[name], ref[name].reshape(got[name].shape)), name
