"""GPU test of dw_conv2d_requant_relu_i8_noalloc, the fused conv for callers that
cannot allocate device memory per call (a fixed memory plan reserved at
start-up, or an inference loop where an allocator call is not allowed).  The
entry point keeps its temporaries in a fixed array inside the library instead
of the backend's growable scratch.

Called through the C ABI and compared with the allocating entry point
(dw_conv2d_requant_relu_i8) on two calls in a row with different shapes — the
second call must not see anything of the first call's contents.  int8 results
must be identical (tolerance 0, as in every int8 parity test).  The file name
makes pytest collect it last.
"""
import ctypes

import numpy as np
import pytest

import dragonwing_edge_rs_b200 as dw
from dragonwing_edge_rs_b200 import _lib as L
from dragonwing_edge_rs_b200 import ops

pytestmark = pytest.mark.gpu

CASES = [
    # n, h, w, c_in, c_out, k, stride, pad, requant_scale, relu
    (1, 28, 28, 64, 64, 3, 1, 1, 0.0011, True),     # tensor-core path, 36 KiB kernel
    (2, 17, 13, 32, 48, 3, 2, 1, 0.0023, False),    # strided, different shape and scale
]


def _noalloc(be, x, w, y, case):
    n, h, wd, ci, co, k, s, p, scale, relu = case
    return L.load().dw_conv2d_requant_relu_i8_noalloc(be.handle, x.handle, w.handle, y.handle, n, h, wd, ci, co, k,
                                                       k, s, s, p, p, ctypes.c_float(scale), 1 if relu else 0)


def test_noalloc_matches_allocating_entry_point_two_calls():
    with dw.CudaBackend(0) as be:
        rng = np.random.default_rng(2024)
        for case in CASES:
            n, h, wd, ci, co, k, s, p, scale, relu = case
            ho, wo = (h + 2 * p - k) // s + 1, (wd + 2 * p - k) // s + 1
            x = be.upload_array(rng.integers(-64, 64, n * h * wd * ci).astype(np.int8))
            w = be.upload_array(rng.integers(-127, 128, k * k * ci * co).astype(np.int8))
            y_ref = be.alloc(n * ho * wo * co)
            y_new = be.alloc(n * ho * wo * co)
            ops.conv2d_requant_relu_i8_packed(be, x, w, y_ref, n, h, wd, ci, co, k, k, s, s, p, p, scale, relu)
            st = _noalloc(be, x, w, y_new, case)
            assert st == L.DW_OK, be.last_error()
            be.synchronize(20000)
            a = be.download_array(y_new, np.int8)
            b = be.download_array(y_ref, np.int8)
            assert np.array_equal(a, b), f"{int((a != b).sum())} of {a.size} outputs differ for {case}"


def test_noalloc_rejects_kernels_beyond_the_fixed_scratch():
    with dw.CudaBackend(0) as be:
        n, h, wd, ci, co, k = 1, 8, 8, 512, 512, 3      # 2.25 MiB of weights > 1 MiB
        x = be.alloc(n * h * wd * ci)
        w = be.alloc(k * k * ci * co)
        y = be.alloc(n * h * wd * co)
        st = L.load().dw_conv2d_requant_relu_i8_noalloc(be.handle, x.handle, w.handle, y.handle, n, h, wd, ci, co,
                                                         k, k, 1, 1, 1, 1, ctypes.c_float(0.01), 1)
        assert st == L.DW_ERR_INVALID_ARG
        assert "exceeds the fixed scratch" in be.last_error()
