"""Host-side quantisation formulas of the path (numpy, float32 arithmetic).

These compute the per-channel scale arrays handed to the fused op; the same
float32 arrays are given to the device kernels and to any checker, so the
requantisation is bit-exact by construction.
"""
from __future__ import annotations

import numpy as np


def roundf_away(x) -> np.ndarray:
    """C roundf / Rust f32::round (half away from zero), exact for float32 input:
    floor(|x|) + (frac(|x|) >= 0.5), both steps exact in float32."""
    x = np.asarray(x, np.float32)
    a = np.abs(x)
    fl = np.floor(a)
    r = fl + (a - fl >= np.float32(0.5)).astype(np.float32)
    return np.copysign(r, x)


def requant_scales(s_in: float, s_w, s_out: float) -> np.ndarray:
    """M[oc] = (s_in * s_w[oc]) / s_out in float32
    (crates/dragonwing-onnx/src/quantize.rs:245, per channel instead of the
    reference's averaged scalar, quantize.rs:307-325)."""
    s_w = np.asarray(s_w, np.float32)
    return (np.float32(s_in) * s_w) / np.float32(s_out)


def dequant_scales(s_in: float, s_w) -> np.ndarray:
    """D[oc] = s_in * s_w[oc] (float32): the SiLU epilogue dequantises with it."""
    return np.float32(s_in) * np.asarray(s_w, np.float32)


def relu6_ceiling(s_out: float) -> int:
    """q6 = (int8) round(clamp(6 * (1/s_out), -128, 127)): quantize_f32_to_i8
    (crates/dragonwing-cpu/src/ops.rs:3503-3525) applied to 6.0."""
    v = np.float32(6.0) * (np.float32(1.0) / np.float32(s_out))
    v = min(max(float(v), -128.0), 127.0)
    return int(np.sign(v) * np.floor(abs(v) + 0.5))


def add_ratios(s_a: float, s_b: float, s_out: float):
    """AddQuantized ratios (crates/dragonwing-onnx/src/quantize.rs:275-276)."""
    return float(np.float32(s_a) / np.float32(s_out)), float(np.float32(s_b) / np.float32(s_out))


def per_channel_symmetric(w_oc_first: np.ndarray):
    """PerChannelScale::from_weights + quantize_weights
    (crates/dragonwing-core/src/quantization.rs:154-195) on a [C_out, ...] float array."""
    w = np.asarray(w_oc_first, np.float32)
    c_out = w.shape[0]
    flat = w.reshape(c_out, -1)
    amax = np.abs(flat).max(axis=1)
    scales = np.where(amax > 0, amax / np.float32(127.0), np.float32(1.0)).astype(np.float32)
    q = flat / scales[:, None]
    q = np.clip(q, np.float32(-128.0), np.float32(127.0))
    q = roundf_away(q).astype(np.int8)
    return q.reshape(w.shape), scales
