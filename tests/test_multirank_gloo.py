"""Multi-rank host logic on CPU (gloo, world size 2): batch sharding, sharded
replicas reproducing the single-process result, max-over-ranks timing, and a
rank failure injected on the host (a rank reporting an error status, a rank
that never joins a collective) that the other rank observes without hanging."""
import datetime
import os
import socket

import numpy as np
import pytest
import torch.multiprocessing as mp

from dragonwing_edge_rs_b200 import _lib as L
from dragonwing_edge_rs_b200.replicas import shard


def _free_port():
    s = socket.socket()
    s.bind(("127.0.0.1", 0))
    p = s.getsockname()[1]
    s.close()
    return p


@pytest.mark.parametrize("B,W", [(256, 8), (1024, 8), (10, 4), (7, 2), (3, 4), (1, 1)])
def test_shard_covers_batch_exactly(B, W):
    seen = []
    for r in range(W):
        s, c = shard(B, W, r)
        seen.extend(range(s, s + c))
    assert seen == list(range(B))
    counts = [shard(B, W, r)[1] for r in range(W)]
    assert max(counts) - min(counts) <= 1
    assert counts == sorted(counts)  # the remainder goes to the last ranks


def _worker(rank, world, port, mode, out_q):
    import torch
    import torch.distributed as dist
    os.environ["MASTER_ADDR"] = "127.0.0.1"
    os.environ["MASTER_PORT"] = str(port)
    dist.init_process_group("gloo", rank=rank, world_size=world, timeout=datetime.timedelta(seconds=6))
    try:
        from dragonwing_edge_rs_b200 import graph as G
        from dragonwing_edge_rs_b200.replicas import exchange_status, max_over_ranks, shard
        from oracle.graph_ref import run_graph
        if mode == "replicas":
            g = G.mobilenetv2_block(batch=3, h=12, w=12, c=16, seed=5)
            x = np.random.default_rng(9).integers(-128, 128, g.tensors["x"].nbytes).astype(np.int8)
            s, c = shard(3, world, rank)
            y = run_graph(g, {"x": x}, batch_slice=(s, s + c))[g.outputs[0]]
            parts = [None] * world
            dist.all_gather_object(parts, y.tobytes())
            t = max_over_ranks(dist, float(rank + 1.5))
            if rank == 0:
                full = run_graph(g, {"x": x})[g.outputs[0]].tobytes()
                out_q.put(("replicas", b"".join(parts) == full, t))
        elif mode == "status":
            st = L.DW_ERR_DEVICE if rank == 1 else L.DW_OK  # rank 1's (fake) device call failed
            statuses = exchange_status(dist, st, "injected device failure" if rank == 1 else "")
            out_q.put(("status", rank, [(s.rank, s.status, s.message) for s in statuses]))
        elif mode == "dead":
            if rank == 1:
                return  # never joins the collective (and leaves without shutting down)
            t0 = datetime.datetime.now()
            try:
                dist.all_reduce(torch.zeros(1))
                out_q.put(("dead", "no-error", 0.0))
            except Exception as e:  # the short process-group timeout ends the wait with an error
                out_q.put(("dead", type(e).__name__, (datetime.datetime.now() - t0).total_seconds()))
    finally:
        if mode != "dead":
            dist.destroy_process_group()


def _run(mode, world=2, timeout=120):
    ctx = mp.get_context("spawn")
    q = ctx.Queue()
    port = _free_port()
    procs = [ctx.Process(target=_worker, args=(r, world, port, mode, q)) for r in range(world)]
    for p in procs:
        p.start()
    results = []
    for p in procs:
        p.join(timeout)
        if p.is_alive():
            p.kill()
    while not q.empty():
        results.append(q.get())
    return results


def test_sharded_replicas_match_single_process():
    res = _run("replicas")
    assert res and res[0][0] == "replicas"
    assert res[0][1] is True
    assert res[0][2] == 2.5  # max over ranks of (rank + 1.5)


def test_failed_rank_status_reaches_every_rank():
    res = _run("status")
    assert len(res) == 2
    for _, rank, statuses in res:
        assert statuses[0][1] == L.DW_OK
        assert statuses[1][1] == L.DW_ERR_DEVICE and "injected" in statuses[1][2]


def test_rank_that_never_joins_ends_in_error_not_hang():
    res = _run("dead", timeout=60)
    assert res and res[0][0] == "dead"
    assert res[0][1] != "no-error"
    assert res[0][2] < 45.0
