"""Shared helpers for the parity tests: seeded synthetic data in the value
distributions of the benchmark configs, and runners that execute one fused
conv through the C ABI and through the CPU oracle."""
from __future__ import annotations

import numpy as np

from dragonwing_edge_rs_b200 import ConvDesc, ops
from dragonwing_edge_rs_b200 import quantization as Q
from oracle import dwref


def conv_case(rng, n, h, w, c_in, c_out, k=3, s=1, pads=None, group=1, epilogue=1, bias=True,
              x_range=(-64, 63), s_in=0.02, s_out=0.05, mult=None):
    """Inputs of one fused conv (config-1 style distributions by default)."""
    if pads is None:
        p = k // 2
        pads = (p, p, p, p)
    desc = ConvDesc(n, h, w, c_in, c_out, k, k, s, s, pads, group, epilogue)
    x = rng.integers(x_range[0], x_range[1] + 1, n * h * w * c_in).astype(np.int8)
    if group == 1:
        wt = rng.integers(-127, 128, k * k * c_in * c_out).astype(np.int8)
    else:
        wt = rng.integers(-127, 128, k * k * c_out).astype(np.int8)
    s_w = rng.uniform(0.001, 0.01, c_out).astype(np.float32)
    M = Q.requant_scales(s_in, s_w, s_out)
    D = Q.dequant_scales(s_in, s_w)
    b = rng.integers(-1000, 1001, c_out).astype(np.int32) if bias else None
    desc.q6 = Q.relu6_ceiling(s_out)
    desc.inv_s_out = float(np.float32(1.0) / np.float32(s_out))
    return desc, x, wt, b, M, D


def oracle_conv(desc: ConvDesc, x, wt, b, M, D, threads=8):
    d = dwref.conv_desc(desc.n, desc.h, desc.w, desc.c_in, desc.c_out, desc.k_h, desc.k_w, desc.stride_h,
                        desc.stride_w, desc.pads, desc.group, desc.epilogue, desc.q6, desc.inv_s_out)
    return dwref.conv2d_fused_i8(x, wt, b, M, D if desc.epilogue == 3 else None, d, threads=threads)


def cuda_conv(be, desc: ConvDesc, x, wt, b, M, D):
    bx = be.upload_array(x)
    bw = be.upload_array(wt)
    wp = ops.prepare_weights_i8(be, desc, bw)
    bb = be.upload_array(b) if b is not None else None
    bm = be.upload_array(M)
    bd = be.upload_array(D)
    ho, wo = desc.out_hw()
    by = be.alloc(desc.n * ho * wo * desc.c_out)
    ops.conv2d_i8(be, desc, bx, wp, bb, bm, bd, by)
    y = be.download_array(by, np.int8)
    be.synchronize(timeout_ms=20000)
    return y


def mismatch_report(a, b, shape=None):
    bad = np.nonzero(a != b)[0]
    if bad.size == 0:
        return "ok"
    i = bad[0]
    return f"{bad.size} mismatches of {a.size}; first at {i}: got {a[i]} expected {b[i]}"
