#!/usr/bin/env python3
"""Benchmark of the fused-INT8 convolution path on B200.

    python bench.py [--gpus N] [--steps K] [--warmup W] [--impl ours|reference] [--workload NAME]
    torchrun --nproc-per-node N bench.py --gpus N ...        (one process per GPU)

A step is one forward pass of the workload graph over one batch of synthetic
int8 input already resident in HBM, replayed from a CUDA graph.  Each rank
runs its own replica on its own batch slice (no collective on the data path:
weak scaling); torch.distributed (NCCL) is used only for the barrier and the
max-over-ranks of the device-timed region.  Rank 0 prints one JSON line.

Workloads (synthetic data and weights with the configs' shapes and value
distributions, seeded):
  yolov8n     (default) YOLOv8n-architecture INT8 graph, 640x640 uint8 images,
              batch 32 per GPU (256 over 8 GPUs), through the Detect tail and
              postprocess_yolo to the detections; value = images/s
              conv TOPS and % of int8 peak beside it.
  mbv2_block  MobileNetV2 inverted-residual block, batch 32 per GPU, 112x112x96,
              1x1 expand 576 + ReLU6, depthwise 3x3 + ReLU6, 1x1 project 96,
              residual add with requantisation.
  resnet50_fp16  ResNet-50-architecture fp16 graph, 224x224x3 f32 input
              normal(0,1), batch 128 per GPU (1024 over 8 GPUs); value =
              images/s, conv TFLOP/s and % of the fp16
              (= bf16) tensor peak beside it.

The default run (one GPU) also times, after the headline and outside its
timed region, every other BASELINE config on the same GPU -- config 1 at N=1
and N=256, the MobileNetV2 block, the three QGemm shapes, ResNet-50 fp16 --
each with its own roofline block, plus YOLOv8n at batch 1 (latency) and the
reference's fused-vs-unfused micro-benchmark; they go under "configs".

--impl reference times the reference's CPU implementation of the same
workload (the oracle restatement of dragonwing-cpu's scalar ops) on rank 0:
the same image sample per step as the cpu_baseline leg, the requested
warm-up, all host threads (the line's value) and one thread beside it.
"""
from __future__ import annotations

import argparse
import json
import os
import statistics
import subprocess
import sys
import threading
import time

ROOT = os.path.dirname(os.path.abspath(__file__))
if ROOT not in sys.path:
    sys.path.insert(0, ROOT)

METRIC = "fused INT8 conv TOPS (% peak); YOLO-shape images/sec at 1/2/4/8 B200 vs CPU"
FALLBACK_PEAKS = {"hbm_gbs": 6650.0, "bf16_tflops": 1590.0}


def load_peaks():
    p = os.path.join(ROOT, "MEASURED_PEAKS.json")
    try:
        with open(p) as f:
            d = json.load(f)
        return d, "measured"
    except Exception:
        return dict(FALLBACK_PEAKS), "fallback"


# ---------------------------------------------------------------------------
# clocks sampling (nvidia-smi, during the timed region)
# ---------------------------------------------------------------------------

class ClockSampler:
    FIELDS = ("index,timestamp,clocks.sm,clocks.max.sm,power.draw,clocks_event_reasons.active,"
              "clocks_event_reasons.hw_slowdown,clocks_event_reasons.hw_thermal_slowdown,"
              "clocks_event_reasons.sw_thermal_slowdown,clocks_event_reasons.sw_power_cap")

    def __init__(self, gpu_index: int):
        self.gpu = gpu_index
        self.proc = None
        self.lines = []
        self.t_start = self.t_end = None

    def start(self):
        try:
            self.proc = subprocess.Popen(
                ["nvidia-smi", f"--query-gpu={self.FIELDS}", "--format=csv,noheader,nounits", "-lms", "50",
                 "-i", str(self.gpu)], stdout=subprocess.PIPE, stderr=subprocess.DEVNULL, text=True)
            threading.Thread(target=self._read, daemon=True).start()
        except Exception:
            self.proc = None

    def _read(self):
        for line in self.proc.stdout:
            self.lines.append((time.time(), line.strip()))

    def mark_start(self):
        self.t_start = time.time()

    def mark_end(self):
        self.t_end = time.time()

    def stop(self):
        if self.proc:
            time.sleep(0.12)
            self.proc.terminate()
            try:
                self.proc.wait(timeout=5)
            except Exception:
                self.proc.kill()

    def summary(self):
        rows = []
        for t, line in self.lines:
            parts = [p.strip() for p in line.split(",")]
            if len(parts) < 10:
                continue
            rows.append((t, parts))
        inside = [r for r in rows if self.t_start and self.t_end and self.t_start - 0.06 <= r[0] <= self.t_end + 0.06]
        use = inside if inside else rows[-3:]
        if not use:
            return {"sm_mhz": None, "sm_max_mhz": None, "reasons": ["nvidia-smi unavailable"], "samples": 0}

        def num(x):
            try:
                return float(x)
            except ValueError:
                return None
        sm = [num(p[2]) for _, p in use if num(p[2]) is not None]
        smax = [num(p[3]) for _, p in use if num(p[3]) is not None]
        reasons = set()
        names = ["hw_slowdown", "hw_thermal_slowdown", "sw_thermal_slowdown", "sw_power_cap"]
        for _, p in use:
            for i, nm in enumerate(names):
                if p[6 + i].lower().startswith("active"):
                    reasons.add(nm)
        return {"sm_mhz": statistics.median(sm) if sm else None, "sm_max_mhz": max(smax) if smax else None,
                "reasons": sorted(reasons), "samples": len(use), "in_region": bool(inside)}


# ---------------------------------------------------------------------------
# workloads
# ---------------------------------------------------------------------------

WORKLOADS = {
    # name: (default per-GPU batch, value unit, description)
    "yolov8n": (32, "images/s", "yolov8n_int8 640x640 (BASELINE config 4)"),
    "mbv2_block": (32, "TOPS", "mobilenetv2_int8_block 112x112x96 (BASELINE config 2)"),
    "resnet50_fp16": (128, "images/s", "resnet50_fp16 224x224 (BASELINE config 5)"),
    "conv3x3_int8": (1, "TOPS", "fused int8 conv 3x3 s1 p1 56x56x64->64 + bias + per-channel requant + ReLU (BASELINE config 1)"),
    "qgemm_int8_4096": (1, "TOPS", "int8 QGemm M=N=K=4096, int32 bias, per-column requant (BASELINE config 3)"),
    "qgemm_int8_8192x1024x4096": (1, "TOPS", "int8 QGemm M=8192 N=1024 K=4096 (BASELINE config 3)"),
    "qgemm_int8_256x4096x11008": (1, "TOPS", "int8 QGemm M=256 N=4096 K=11008 (BASELINE config 3)"),
}
QGEMM_SHAPES = {"qgemm_int8_4096": (4096, 4096, 4096), "qgemm_int8_8192x1024x4096": (8192, 1024, 4096),
                "qgemm_int8_256x4096x11008": (256, 4096, 11008)}
FP16_WORKLOADS = {"resnet50_fp16"}
DEFAULT_WORKLOAD = "yolov8n"


def build_workload(name: str, batch: int, seed: int):
    from dragonwing_edge_rs_b200 import graph as G
    if name not in WORKLOADS:
        raise SystemExit(f"unknown workload {name}")
    desc = WORKLOADS[name][2]
    if name == "conv3x3_int8":
        b = G.GraphBuilder(seed)
        x = b.input("x", (batch, 56, 56, 64), "i8", 0.02)
        b.output(b.conv(x, 64, k=3, act="relu", out_scale=0.05, name="conv"))
        return b.g, {"workload": desc, "batch_per_gpu": batch, "layers": "one fused conv (input scale 0.02, output 0.05)"}
    if name in QGEMM_SHAPES:
        m, n, k = QGEMM_SHAPES[name]
        b = G.GraphBuilder(seed, act_scale_range=(0.001, 0.01))
        x = b.input("a", (batch, 1, m, k), "i8", 0.005)
        b.output(b.conv(x, n, k=1, act="none", name="qgemm"))
        return b.g, {"workload": desc, "batch_per_gpu": batch, "m": m, "n": n, "k": k,
                     "layers": "QGemm as a 1x1 conv over M rows (int32 bias, per-column M)"}
    if name == "resnet50_fp16":
        g = G.resnet50_fp16(batch=batch, seed=seed)
        cfg = {"workload": desc, "batch_per_gpu": batch, "stages": [3, 4, 6, 3], "classes": 1000,
               "layers": "53 fp16 convs (BN folded, bias, ReLU), 3x3/2 max pool, 16 residual add+ReLU, GAP, FC 1000",
               "input": "f32 NHWC normal(0,1) -> f16 (3 channels zero-padded to 16)", "outputs": "f32 logits"}
    elif name == "mbv2_block":
        g = G.mobilenetv2_block(batch=batch, seed=seed)
        cfg = {"workload": desc, "batch_per_gpu": batch, "expand": 576,
               "layers": "1x1 expand+ReLU6, dw3x3+ReLU6, 1x1 project, add"}
    else:
        g = G.yolov8n(batch=batch, seed=seed)
        cfg = {"workload": desc, "batch_per_gpu": batch, "width": 0.25, "depth": 0.33, "classes": 80, "reg_max": 16,
               "layers": "63 fused int8 convs (SiLU), C2f, SPPF 5x5, PAN upsample+concat, decoupled head, "
                         "Detect tail (DFL, dist2bbox, sigmoid: output0 [b, 84, 8400] f32), postprocess_yolo "
                         "(decode, conf 0.25, class-aware NMS IoU 0.45)",
               "input": "uint8 image /255 -> int8",
               "outputs": "detections (24-byte records [b, 8400], zero after each image's count) + counts"}
    return g, cfg


def workload_defaults(name):
    return WORKLOADS[name][0]


def make_input(graph, seed):
    import numpy as np
    t = graph.tensors[graph.inputs[0]]
    rng = np.random.default_rng(seed)
    if t.dtype == "u8":
        return rng.integers(0, 256, t.nbytes).astype(np.uint8)
    if t.dtype == "f32":
        return rng.standard_normal(t.nbytes // 4).astype(np.float32)
    return rng.integers(-128, 128, t.nbytes).astype(np.int8)


def op_bytes(graph, op):
    """Algorithmic (compulsory) bytes of one op: inputs + weights/scales + outputs, each once."""
    t = graph.tensors
    total = 0
    for i in op.inputs:
        if i in t:
            total += t[i].nbytes
        elif i in graph.initializers:
            total += graph.initializers[i].nbytes
    for o in op.outputs:
        total += t[o].nbytes
    return total


def op_flops(op):
    """Algorithmic ops (2 x MACs; a zero-padded input channel does not count)."""
    if op.op_type == "GemmF16":
        return 2 * op.params["m"] * op.params["n"] * op.params["k"]
    if op.op_type not in ("Conv2dRequantReluI8Nhwc", "Conv2dAddI8", "Conv2dF16", "Conv2dAddF16", "Conv2dStemU8I8"):
        return 0
    d = op.params["desc"]
    ho, wo = d.out_hw()
    c_in = op.params.get("c_in_real", d.c_in)
    return 2 * d.n * ho * wo * d.c_out * d.k_h * d.k_w * (c_in if d.group == 1 else 1)


# ---------------------------------------------------------------------------
# timing helpers (CUDA events on the backend stream)
# ---------------------------------------------------------------------------

L2_FLUSH_BYTES = 256 << 20  # larger than the B200's 126 MB L2


class Flusher:
    """Writes a buffer larger than L2 on the backend stream between timed
    launches (outside their events), so each launch starts with a cold L2."""

    def __init__(self, stream):
        import torch
        self.stream = stream
        self.buf = torch.empty(L2_FLUSH_BYTES, dtype=torch.uint8, device="cuda")

    def __call__(self):
        import torch
        with torch.cuda.stream(self.stream):
            self.buf.zero_()


def time_launches(fn, stream, steps, flush=None):
    """Per-launch device times (ms) of `fn` (enqueues work on `stream`), each
    bracketed by its own events; `flush` runs between launches, untimed."""
    import torch
    evs = [(torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)) for _ in range(steps)]
    for a, b in evs:
        if flush:
            flush()
        a.record(stream)
        fn()
        b.record(stream)
    stream.synchronize()
    return [a.elapsed_time(b) for a, b in evs]


def per_op_times(rt, stream, steps, flush=None):
    """Device time of every op of the runtime's op list (eager dispatch, events
    around each op on the backend stream), averaged over `steps` passes."""
    import torch
    n_ops = len(rt._dispatch)
    acc = [0.0] * n_ops
    for _ in range(steps):
        if flush:
            flush()
        evs = [torch.cuda.Event(enable_timing=True) for _ in range(n_ops + 1)]
        evs[0].record(stream)
        for i, fn in enumerate(rt._dispatch):
            fn()
            evs[i + 1].record(stream)
        stream.synchronize()
        for i in range(n_ops):
            acc[i] += evs[i].elapsed_time(evs[i + 1])
    return [a / steps for a in acc]


def pct(vals, q):
    v = sorted(vals)
    if not v:
        return None
    k = min(len(v) - 1, max(0, int(round(q / 100.0 * (len(v) - 1)))))
    return v[k]


# ---------------------------------------------------------------------------
# roofline
# ---------------------------------------------------------------------------

def per_op_records(graph, op_ms):
    return [{"op": op.name, "type": op.op_type, "ms": round(t, 5), "bytes": op_bytes(graph, op), "ops": op_flops(op)}
            for op, t in zip(graph.ops, op_ms)]


def roofline_units(graph, per_op):
    """Groups per-op records into roofline units.  The 3x3 stem on a 3-channel
    image is one op (Conv2dStemU8I8: uint8 image in, conv output out) where
    its shape allows; otherwise the stem pair the device lowering makes of it
    (Im2colU8ToI8, then the 1x1 conv that reads its 27 -> 32 channel rows) is
    one unit whose compulsory bytes
    are the uint8 image, the conv's weights and per-channel arrays, and its
    output: the im2col tensor is an artefact of the lowering, not algorithmic
    traffic.  Every other op is its own unit."""
    by_name = {op.name: op for op in graph.ops}
    consumer = {}
    for op in graph.ops:
        for i in op.inputs:
            consumer.setdefault(i, []).append(op.name)
    rec = {r["op"]: r for r in per_op}
    units, used = [], set()
    for r in per_op:
        if r["op"] in used:
            continue
        op = by_name[r["op"]]
        if op.op_type == "Im2colU8ToI8":
            cons = consumer.get(op.outputs[0], [])
            if len(cons) == 1 and by_name[cons[0]].op_type == "Conv2dRequantReluI8Nhwc":
                conv = by_name[cons[0]]
                c = rec[conv.name]
                img = graph.tensors[op.inputs[0]].nbytes
                col = graph.tensors[op.outputs[0]].nbytes
                units.append({"kernel": f"{op.name}+{conv.name}", "ops_in_unit": [op.name, conv.name],
                              "ms": r["ms"] + c["ms"], "bytes": img + c["bytes"] - col, "ops": c["ops"],
                              "note": "stem: uint8 image in, int8 conv output; the im2col tensor the device "
                                      "lowering writes and reads is not counted as algorithmic traffic"})
                used.update({op.name, conv.name})
                continue
        units.append({"kernel": r["op"], "ops_in_unit": [r["op"]], "ms": r["ms"], "bytes": r["bytes"],
                      "ops": r["ops"]})
        used.add(r["op"])
    return units


def load_traffic():
    """DRAM traffic per launch from the committed ncu summaries
    (profiles/traffic.json: workload -> op name -> bytes), else {}."""
    p = os.path.join(ROOT, "profiles", "traffic.json")
    try:
        with open(p) as f:
            return json.load(f)
    except Exception:
        return {}


def roofline_of(graph, per_op, workload, peaks, f16, exclude_types=("YoloPostprocess",), config_key=None):
    """Roofline block of the unit with the largest device time."""
    peak_d, peak_src = peaks
    hbm_peak = float(peak_d.get("hbm_gbs", FALLBACK_PEAKS["hbm_gbs"]))
    bf16_peak = float(peak_d.get("bf16_tflops", FALLBACK_PEAKS["bf16_tflops"]))
    tensor_peak = bf16_peak if f16 else 2.0 * bf16_peak
    units = [u for u in roofline_units(graph, per_op)
             if not any(next(r for r in per_op if r["op"] == o)["type"] in exclude_types for o in u["ops_in_unit"])]
    dom = max(units, key=lambda u: u["ms"])
    ridge = tensor_peak * 1e12 / (hbm_peak * 1e9)
    ai = dom["ops"] / dom["bytes"] if dom["bytes"] else 0.0
    if dom["ops"] and ai > ridge:
        ach = dom["ops"] / (dom["ms"] * 1e-3) / 1e12
        roof = {"bound": "tensor", "achieved": round(ach, 2), "peak": round(tensor_peak, 1),
                "unit": "TFLOP/s" if f16 else "TOP/s", "frac": round(ach / tensor_peak, 4)}
    else:
        ach = dom["bytes"] / (dom["ms"] * 1e-3) / 1e9
        roof = {"bound": "hbm", "achieved": round(ach, 1), "peak": hbm_peak, "unit": "GB/s",
                "frac": round(ach / hbm_peak, 4)}
    # per-config captures (a workload timed at several batches) are keyed by the config
    tr_all = load_traffic()
    tr = tr_all.get(config_key) if config_key in tr_all else tr_all.get(workload, {})
    parts = [tr.get(o) for o in dom["ops_in_unit"]]
    traffic = sum(parts) if parts and all(isinstance(t, (int, float)) for t in parts) else None
    roof.update({"kernel": dom["kernel"], "kernel_ms": round(dom["ms"], 5), "algorithmic_bytes": dom["bytes"],
                 "algorithmic_ops": dom["ops"], "arithmetic_intensity": round(ai, 1), "ridge": round(ridge, 1),
                 "traffic": traffic,
                 "peak_source": "measured (MEASURED_PEAKS.json)" if peak_src == "measured" else "fallback",
                 "peak_note": "fp16 dense peak = the measured bf16 cuBLAS figure" if f16 else
                 "int8 dense peak taken as 2x the measured bf16 cuBLAS figure"})
    if "note" in dom:
        roof["unit_note"] = dom["note"]
    return roof


# ---------------------------------------------------------------------------
# our arm
# ---------------------------------------------------------------------------

def run_ours(args, rank, world, local_rank):
    import numpy as np
    import torch

    import dragonwing_edge_rs_b200 as dw
    from dragonwing_edge_rs_b200.graph import CudaGraphRuntime

    torch.cuda.set_device(local_rank)
    dist = None
    if world > 1:
        import datetime

        import torch.distributed as tdist
        tdist.init_process_group("nccl", timeout=datetime.timedelta(seconds=180))
        dist = tdist

    def barrier():
        if dist:
            t = torch.zeros(1, device="cuda")
            dist.all_reduce(t)
            torch.cuda.synchronize()

    from dragonwing_edge_rs_b200 import replicas

    def max_over_ranks(v: float) -> float:
        return replicas.max_over_ranks(dist, v, device="cuda")

    batch = args.batch or workload_defaults(args.workload)
    graph, cfg = build_workload(args.workload, batch, seed=1234)
    be = dw.CudaBackend(local_rank)
    rt = CudaGraphRuntime(graph, be)
    graph0, graph = graph, rt.graph  # after the device passes (fusion, input unfold); same work, fewer ops
    x_name = graph.inputs[0]
    xt = graph.tensors[x_name]
    x_host = make_input(graph, 1000 + rank)
    rt.set_input_bytes(x_name, x_host)
    kernels_per_step = rt.capture()
    stream = torch.cuda.ExternalStream(be.stream())
    step_ops = graph.conv_ops()
    out_names = list(graph.outputs)

    # ---- warm-up
    for _ in range(args.warmup):
        rt.run()
    be.synchronize(120000)

    # ---- timed region: K graph replays, inputs resident in HBM
    sampler = ClockSampler(local_rank)
    sampler.start()
    time.sleep(0.2)
    barrier()
    be.synchronize(120000)
    torch.cuda.synchronize()
    e0, e1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
    launches0 = be.launch_count()
    sampler.mark_start()
    e0.record(stream)
    for _ in range(args.steps):
        rt.run()
    e1.record(stream)
    be.synchronize(600000)
    sampler.mark_end()
    torch.cuda.synchronize()
    barrier()
    launches = replicas.sum_over_ranks(dist, be.launch_count() - launches0, device="cuda")
    sampler.stop()
    ms_local = e0.elapsed_time(e1)
    ms = max_over_ranks(ms_local)
    ms_per_step = ms / args.steps
    clocks = sampler.summary()

    # ---- per-op device time (eager dispatch bracketed by events on the launch stream)
    be.synchronize(120000)
    per_op = per_op_records(graph, per_op_times(rt, stream, args.kernel_steps))

    # ---- end to end through the public API: pinned host input -> graph -> pinned host output.
    # PipelinedRunner runs one CUDA graph per slot, each bound to its own input and
    # output buffers: step i's upload and step i-1's read-back overlap step i's compute
    # on two copy streams, with no device-side staging copy; every step copies its whole
    # input in and its whole output out.
    from dragonwing_edge_rs_b200.graph import PipelinedRunner
    in_bytes = xt.nbytes
    out_sizes = [graph.tensors[o].nbytes for o in out_names]
    out_bytes = sum(out_sizes)
    depth = 2
    hins = [be.host_alloc(in_bytes) for _ in range(depth)]
    houts = [be.host_alloc(out_bytes) for _ in range(depth)]
    for _, arr in hins:
        arr[:] = x_host.view(np.uint8)
    pr = PipelinedRunner(rt, depth=depth)
    for i in range(2 * depth):
        pr.step(hins[i % depth][0], houts[i % depth][0])
    pr.synchronize()
    barrier()
    f0, f1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
    t_wall0 = time.perf_counter()
    f0.record(stream)
    for i in range(args.steps):
        pr.step(hins[i % depth][0], houts[i % depth][0])
    f1.record(stream)
    pr.synchronize()
    t_wall = time.perf_counter() - t_wall0
    barrier()
    e2e_ms = max_over_ranks(max(f0.elapsed_time(f1), t_wall * 1000.0))
    pr.close()
    for ptr, _ in hins + houts:
        be.host_free(ptr)

    # ---- the other BASELINE configs (one GPU only; not part of `value`)
    configs = None
    if rank == 0 and world == 1 and args.workload == DEFAULT_WORKLOAD and not args.no_configs:
        rt.release()
        configs = run_configs(be, stream, args)

    # ---- CPU baseline (rank 0, single GPU only): the oracle on a bounded sample
    cpu = None
    if rank == 0 and world == 1 and not args.no_cpu:
        cpu = cpu_reference(graph0, x_host, args, WORKLOADS[args.workload][1], steps=args.cpu_reps, warmup=1)

    if rank == 0:
        peaks = load_peaks()
        f16 = args.workload in FP16_WORKLOADS
        bf16_peak = float(peaks[0].get("bf16_tflops", FALLBACK_PEAKS["bf16_tflops"]))
        int8_peak = bf16_peak if f16 else 2.0 * bf16_peak
        # the roofline is the hot path's (fused conv, depthwise, glue): the detection
        # post-processing after the graph is latency-bound and reported on its own
        post = [r for r in per_op if r["type"] == "YoloPostprocess"]
        roof = roofline_of(graph, per_op, args.workload, peaks, f16)
        roof["selection"] = ("the unit (op, or the stem's im2col + conv pair) with the largest device time on the "
                             "fused-conv path; postprocess_yolo is reported apart (latency-bound: the serial greedy "
                             "NMS of its largest class)")
        images = batch * world
        ws = sum(t.nbytes for t in graph.tensors.values()) + sum(a.nbytes for a in graph.initializers.values())
        l2_note = (f"per-step working set {ws / 1e6:.0f} MB, larger than the 126 MB L2 (no flush needed)"
                   if ws > 126e6 else f"per-step working set {ws / 1e6:.1f} MB fits in the 126 MB L2: cache-warm figure")
        tops = step_ops * world / (ms_per_step * 1e-3) / 1e12
        ips = images / (ms_per_step * 1e-3)
        unit = WORKLOADS[args.workload][1]
        e2e_ips = images * args.steps / (e2e_ms * 1e-3)
        e2e_tops = step_ops * world * args.steps / (e2e_ms * 1e-3) / 1e12
        line = {
            "metric": METRIC,
            "value": round(ips if unit == "images/s" else tops, 3),
            "unit": unit,
            "n_gpus": world,
            "steps": args.steps,
            "warmup": args.warmup,
            "ms_per_step": round(ms_per_step, 5),
            "higher_is_better": True,
            "scaling": "weak",
            "vs_baseline": None,
            "dtype": "f16 (f32 accumulate)" if f16 else "int8 (i32 accumulate, f32 requant)",
            "data": "synthetic (seeded normal(0,1) f32 images, He-normal f16 weights, BN folded)" if f16 else
                    "synthetic (seeded int8 activations, He-normal weights quantised per channel)",
            "images_per_s": round(ips, 1),
            "conv_tops": round(tops, 3),
            "pct_of_tensor_peak": round(100.0 * tops / (int8_peak * world), 2),
            "config": dict(cfg, parallelism=f"replicas x{world} (batch-sharded, no collective)",
                           global_batch=images, l2=l2_note),
            "e2e": {"value": round(e2e_ips if unit == "images/s" else e2e_tops, 3), "unit": unit,
                    "images_per_s": round(e2e_ips, 1), "conv_tops": round(e2e_tops, 3),
                    "h2d_bytes_per_step": in_bytes, "d2h_bytes_per_step": out_bytes,
                    "path": "PipelinedRunner over CudaGraphRuntime: dw_upload_async (pinned, copy stream) into the "
                            "slot's input buffer -> the slot's CUDA graph -> dw_download_async (pinned, copy "
                            "stream) from the slot's output buffers, two steps in flight, no device-side copies"},
            "gpu_launches": int(launches),  # all ranks
            "kernels_per_step": int(kernels_per_step),
            "roofline": roof,
            "per_op": per_op,
            "postprocess": ({"ms": post[0]["ms"], "share_of_step": round(post[0]["ms"] / ms_per_step, 4),
                             "kernels": "yolo_decode, yolo_rank, yolo_nms_small, yolo_nms_segment, yolo_order"}
                            if post else None),
            "clocks": clocks,
        }
        if configs is not None:
            line["configs"] = configs
        if cpu:
            line["cpu_baseline"] = cpu
        print(json.dumps(line), flush=True)
    # every rank reports its backend status; a failed rank fails the run on all ranks
    statuses = replicas.exchange_status(dist, 0)
    rt.release()
    be.close()
    if any(not st.ok for st in statuses):
        raise SystemExit(f"rank failures: {[(st.rank, st.status, st.message) for st in statuses if not st.ok]}")
    if dist:
        dist.destroy_process_group()


# ---------------------------------------------------------------------------
# the other BASELINE configs, timed after the headline on the same GPU
# ---------------------------------------------------------------------------

CONFIG_RUNS = [
    # (key, workload, per-GPU batch)
    ("conv3x3_int8_n1", "conv3x3_int8", 1),
    ("conv3x3_int8_n256", "conv3x3_int8", 256),
    ("mbv2_block_b32", "mbv2_block", 32),
    ("qgemm_int8_4096x4096x4096", "qgemm_int8_4096", 1),
    ("qgemm_int8_8192x1024x4096", "qgemm_int8_8192x1024x4096", 1),
    ("qgemm_int8_256x4096x11008", "qgemm_int8_256x4096x11008", 1),
    ("resnet50_fp16_b128", "resnet50_fp16", 128),
]


def run_configs(be, stream, args):
    """Times every other BASELINE config on this GPU (CUDA-graph replay, each
    launch bracketed by events, L2 flushed between launches), each with the
    roofline of its largest unit; then YOLOv8n at batch 1 (latency) and the
    reference's fused-vs-unfused micro-benchmark."""
    import gc

    from dragonwing_edge_rs_b200.graph import CudaGraphRuntime
    peaks = load_peaks()
    flush = Flusher(stream)
    out = {}
    steps = max(args.steps, 20)
    for key, name, batch in CONFIG_RUNS:
        graph, cfg = build_workload(name, batch, seed=1234)
        rt = CudaGraphRuntime(graph, be)
        g = rt.graph
        rt.set_input_bytes(g.inputs[0], make_input(g, 1000))
        kernels = rt.capture()
        for _ in range(max(args.warmup, 3)):
            rt.run()
        be.synchronize(120000)
        ms = time_launches(rt.run, stream, steps, flush)
        per_op = per_op_records(g, per_op_times(rt, stream, args.kernel_steps, flush))
        f16 = name in FP16_WORKLOADS
        mean = sum(ms) / len(ms)
        ops = g.conv_ops()
        unit = WORKLOADS[name][1]
        tops = ops / (mean * 1e-3) / 1e12
        ips = batch / (mean * 1e-3)
        bf16_peak = float(peaks[0].get("bf16_tflops", FALLBACK_PEAKS["bf16_tflops"]))
        tensor_peak = bf16_peak if f16 else 2.0 * bf16_peak
        out[key] = {
            "workload": cfg["workload"], "batch": batch,
            "value": round(ips if unit == "images/s" else tops, 3), "unit": unit,
            "ms_per_step": round(mean, 5), "ms_p50": round(pct(ms, 50), 5), "steps": steps,
            "images_per_s": round(ips, 1), "tops" if not f16 else "tflops": round(tops, 2),
            "pct_of_tensor_peak": round(100.0 * tops / tensor_peak, 2),
            "kernels_per_step": kernels,
            "l2": "flushed between timed launches (256 MB write, outside the events)",
            "roofline": roofline_of(g, per_op, name, peaks, f16, config_key=key),
            "per_op": per_op if len(per_op) <= 8 else None,
        }
        rt.release()
        del rt, g, graph
        gc.collect()
    out["yolov8n_b1_latency"] = yolo_b1_latency(be, stream, flush, args)
    out["reference_microbench"] = reference_microbench(be, stream, args)
    return out


def yolo_b1_latency(be, stream, flush, args):
    """YOLOv8n (to the detections) at batch 1: per-image latency of the
    replayed graph (device events, L2 flushed before each launch) and through
    the serving API (pinned host image in, detections out, host wall clock
    from the upload call to the synchronised read-back); the reference's own
    whole-graph benchmark reports single-image latency
    (crates/dragonwing-test/src/bin/yolo_benchmark.rs:219-243)."""
    import gc

    import numpy as np

    from dragonwing_edge_rs_b200.graph import CudaGraphRuntime
    graph, _ = build_workload("yolov8n", 1, seed=1234)
    rt = CudaGraphRuntime(graph, be)
    g = rt.graph
    x = make_input(g, 1000)
    rt.set_input_bytes(g.inputs[0], x)
    rt.capture()
    for _ in range(5):
        rt.run()
    be.synchronize(60000)
    n = max(100, args.steps)
    dev = time_launches(rt.run, stream, n, flush)
    in_name = g.inputs[0]
    outs = list(g.outputs)
    in_bytes = g.tensors[in_name].nbytes
    out_sizes = [g.tensors[o].nbytes for o in outs]
    hin, ain = be.host_alloc(in_bytes)
    hout, _ = be.host_alloc(sum(out_sizes))
    ain[:] = x.view(np.uint8)
    wall = []
    for i in range(n + 5):
        t0 = time.perf_counter()
        be.upload_async(rt.bufs[in_name], hin, in_bytes)
        rt.run()
        off = 0
        for o, sz in zip(outs, out_sizes):
            be.download_async(rt.bufs[o], hout + off, sz)
            off += sz
        be.synchronize(60000)
        if i >= 5:
            wall.append((time.perf_counter() - t0) * 1000.0)
    be.host_free(hin)
    be.host_free(hout)
    rt.release()
    del rt
    gc.collect()
    return {"workload": "yolov8n_int8 640x640, batch 1, to the detections (BASELINE config 4 at batch 1)",
            "launches": n,
            "device_ms": {"p50": round(pct(dev, 50), 4), "p95": round(pct(dev, 95), 4), "min": round(min(dev), 4)},
            "serving_api_ms": {"p50": round(pct(wall, 50), 4), "p95": round(pct(wall, 95), 4),
                               "min": round(min(wall), 4)},
            "images_per_s_at_p50": round(1000.0 / pct(dev, 50), 1),
            "l2": "flushed before each device-timed launch",
            "serving_path": "dw_upload_async (pinned) -> CUDA graph -> dw_download_async (pinned) -> "
                            "dw_synchronize, one image at a time, host wall clock"}


def reference_microbench(be, stream, args):
    """The reference's only published comparison for this path
    (crates/dragonwing-test/src/bin/device_benchmark.rs:269-353): unfused
    conv2d_i8_nhwc_packed (int32 out) against fused conv2d_requant_relu_i8_packed
    (requant scale 0.001, ReLU) on three 3x3 s1 p1 shapes, 5 warm-up and 10
    timed calls, each call synchronised; the same entry points through the C
    ABI, with the reference's input bytes (i & 0x3f) and kernel bytes (i & 0x1f).
    Device time = CUDA events around the call on the backend stream (the
    weight repack the HWIO signature implies included); wall = call +
    dw_synchronize on the host."""
    import numpy as np

    from dragonwing_edge_rs_b200 import ops
    shapes = [(1, 32, 32, 16, 16, 3, 1, 1), (1, 32, 32, 32, 32, 3, 1, 1), (1, 16, 16, 64, 64, 3, 1, 1)]
    res = []
    for n, h, w, ci, co, k, s, p in shapes:
        ho, wo = (h + 2 * p - k) // s + 1, (w + 2 * p - k) // s + 1
        x = be.upload_array((np.arange(n * h * w * ci) & 0x3F).astype(np.uint8).view(np.int8))
        wt = be.upload_array((np.arange(k * k * ci * co) & 0x1F).astype(np.uint8).view(np.int8))
        y32 = be.alloc(4 * n * ho * wo * co)
        y8 = be.alloc(n * ho * wo * co)

        def unfused():
            ops.conv2d_i8_nhwc_packed(be, x, wt, y32, n, h, w, ci, co, k, k, s, s, p, p)

        def fused():
            ops.conv2d_requant_relu_i8_packed(be, x, wt, y8, n, h, w, ci, co, k, k, s, s, p, p, 0.001, True)

        row = {"shape": {"n": n, "h": h, "w": w, "c_in": ci, "c_out": co, "k": k, "stride": s, "pad": p}}
        for label, fn in (("unfused", unfused), ("fused", fused)):
            for _ in range(5):
                fn()
                be.synchronize(10000)
            dev = []
            wall = []
            for _ in range(10):
                dev += time_launches(fn, stream, 1)
                t0 = time.perf_counter()
                fn()
                be.synchronize(10000)
                wall.append((time.perf_counter() - t0) * 1e6)
            row[label] = {"device_us": round(1000.0 * sum(dev) / len(dev), 2), "wall_us": round(sum(wall) / len(wall), 2)}
        row["unfused_over_fused_device"] = round(row["unfused"]["device_us"] / row["fused"]["device_us"], 3)
        row["unfused_over_fused_wall"] = round(row["unfused"]["wall_us"] / row["fused"]["wall_us"], 3)
        res.append(row)
        for b in (x, wt, y32, y8):
            b.free()
    return {"source": "crates/dragonwing-test/src/bin/device_benchmark.rs:269-353; published ratio 1.6-1.7x "
                      "on Adreno A702 (docs/vulkan-runtime-integration.md:270)", "shapes": res}


# ---------------------------------------------------------------------------
# the reference's CPU path (the oracle restatement), timed on the host cores
# ---------------------------------------------------------------------------

def cpu_model():
    try:
        with open("/proc/cpuinfo") as f:
            for line in f:
                if line.startswith("model name"):
                    return line.split(":", 1)[1].strip()
    except Exception:
        pass
    return "unknown"


def cpu_reference(graph, x_host, args, unit, steps, warmup, single_thread_steps=None):
    """Times the oracle (C restatement of dragonwing-cpu's scalar ops) on the
    reference-shaped (unlowered) graph over a bounded sample: `args.cpu_images`
    images of the batch per step, `warmup` untimed steps, then `steps` timed
    steps (fewer if they would exceed args.cpu_budget_s; the count is
    reported).  Two figures, labelled:
      * all host threads, ops row-partitioned like dragonwing-cpu's pool.rs
        (crates/dragonwing-cpu/src/pool.rs:317-350) -- the line's value;
      * one thread: the reference's int8 conv and gemm_i8 are single-threaded
        (crates/dragonwing-cpu/src/ops.rs:2964, 3086), so for the int8
        workloads this is the reference-faithful figure."""
    from oracle import dwref
    from oracle.graph_ref import run_graph
    feeds = {graph.inputs[0]: x_host}
    batch = graph.tensors[graph.inputs[0]].shape[0]
    images = max(1, min(batch, args.cpu_images))
    ops_per_image = graph.conv_ops() / batch

    def run(threads, k, w):
        for _ in range(w):
            run_graph(graph, feeds, threads=threads, batch_slice=(0, images))
        t = []
        for _ in range(k):
            t0 = time.perf_counter()
            run_graph(graph, feeds, threads=threads, batch_slice=(0, images))
            t.append(time.perf_counter() - t0)
            if sum(t) > args.cpu_budget_s and len(t) >= 1:
                break
        return t

    def summary(t, threads, label):
        med = pct(t, 50)
        ips = images / med
        value = ips if unit == "images/s" else ops_per_image * images / med / 1e12
        return {"value": round(value, 6), "unit": unit, "cores": threads, "images_per_s": round(ips, 4),
                "steps_timed": len(t), "step_s": {"min": round(min(t), 3), "median": round(med, 3),
                                                  "max": round(max(t), 3)},
                "sample": f"{images} image(s) of the same workload per step, median of {len(t)} step(s)",
                "threading": label}

    threads = dwref.num_cpus()
    t_all = run(threads, steps, warmup)
    res = summary(t_all, threads, "all host threads, row-partitioned (pool.rs:317-350)")
    res.update({"kind": "port", "cpu": cpu_model(),
                "note": "reference = C restatement of dragonwing-cpu's scalar ops (the Rust crate cannot be "
                        "compiled here)"})
    k1 = single_thread_steps if single_thread_steps is not None else max(1, min(3, steps))
    t_one = run(1, k1, 0)
    res["single_thread"] = summary(t_one, 1, "one thread: the reference's int8 conv and gemm_i8 are "
                                              "single-threaded (ops.rs:2964, 3086)")
    return res


def run_reference(args, rank, world):
    if rank != 0:
        return
    batch = args.batch or workload_defaults(args.workload)
    graph, cfg = build_workload(args.workload, batch, seed=1234)
    x = make_input(graph, 1000)
    unit = WORKLOADS[args.workload][1]
    cpu = cpu_reference(graph, x, args, unit, steps=args.steps, warmup=args.warmup)
    value = cpu["value"]
    images = max(1, min(batch, args.cpu_images))
    ms_per_step = 1000.0 * cpu["step_s"]["median"]
    line = {"metric": METRIC, "value": value, "unit": unit, "impl": "reference", "n_gpus": world,
            "steps": cpu["steps_timed"], "steps_requested": args.steps, "warmup": args.warmup,
            "ms_per_step": round(ms_per_step, 3),
            "higher_is_better": True, "scaling": "weak", "vs_baseline": None,
            "dtype": "f16 (f32 accumulate)" if args.workload in FP16_WORKLOADS else "int8 (i32 accumulate, f32 requant)",
            "data": "synthetic",
            "images_per_s": cpu["images_per_s"],
            "config": dict(cfg, sample_images_per_step=images),
            "cpu_baseline": cpu,
            "e2e": {"value": value, "unit": unit, "h2d_bytes_per_step": 0, "d2h_bytes_per_step": 0},
            "note": cpu["note"]}
    print(json.dumps(line), flush=True)


def profile_op(args):
    """Runs one op of the workload graph (after the device passes) eagerly:
    one untimed launch, then --steps launches.  No timing, no JSON."""
    import dragonwing_edge_rs_b200 as dw
    from dragonwing_edge_rs_b200.graph import CudaGraphRuntime
    batch = args.batch or workload_defaults(args.workload)
    graph, _ = build_workload(args.workload, batch, seed=1234)
    be = dw.CudaBackend(0)
    rt = CudaGraphRuntime(graph, be)
    rt.set_input_bytes(graph.inputs[0], make_input(graph, 1000))
    rt.run()  # every tensor holds real data
    names = [op.name for op in rt.graph.ops]
    if args.profile_op not in names:
        raise SystemExit(f"unknown op {args.profile_op}; ops: {' '.join(names)}")
    fn = rt._dispatch[names.index(args.profile_op)]
    be.synchronize(120000)
    import torch
    torch.cuda.set_device(0)
    torch.cuda.profiler.start()  # for `ncu --profile-from-start off`: only this op's launches
    for _ in range(1 + args.steps):
        fn()
    be.synchronize(120000)
    torch.cuda.profiler.stop()
    print(f"profiled {args.profile_op} x{1 + args.steps} ({args.workload}, batch {batch})")
    rt.release()
    be.close()


def main():
    ap = argparse.ArgumentParser()
    ap.add_argument("--gpus", type=int, default=1)
    ap.add_argument("--steps", type=int, default=200)
    ap.add_argument("--warmup", type=int, default=5)
    ap.add_argument("--impl", choices=["ours", "reference"], default="ours")
    ap.add_argument("--workload", default=DEFAULT_WORKLOAD, choices=sorted(WORKLOADS))
    ap.add_argument("--batch", type=int, default=0, help="per-GPU batch (default: the workload's)")
    ap.add_argument("--kernel-steps", type=int, default=5)
    ap.add_argument("--cpu-images", type=int, default=2, help="images per CPU step (reference arm and cpu_baseline)")
    ap.add_argument("--cpu-reps", type=int, default=5, help="timed steps of the cpu_baseline leg")
    ap.add_argument("--no-cpu", action="store_true")
    ap.add_argument("--no-configs", action="store_true", help="skip the other BASELINE configs after the headline")
    ap.add_argument("--cpu-budget-s", type=float, default=120.0)
    ap.add_argument("--profile-op", default="",
                    help="profiling aid: run the workload graph once, then only this op (of the graph after the "
                         "device passes) 1 + --steps times inside cudaProfilerStart/Stop, and exit "
                         "(for ncu --profile-from-start off captures of one kernel)")
    args = ap.parse_args()
    if args.profile_op:
        profile_op(args)
        return
    rank = int(os.environ.get("RANK", "0"))
    world = int(os.environ.get("WORLD_SIZE", str(args.gpus if args.gpus == 1 else 1)))
    local_rank = int(os.environ.get("LOCAL_RANK", "0"))
    if args.impl == "reference":
        run_reference(args, rank, world)
        return
    run_ours(args, rank, world, local_rank)


if __name__ == "__main__":
    main()
