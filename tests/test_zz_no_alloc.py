"""GPU tests of dw_conv2d_requant_relu_i8_noalloc, the fused conv for callers that
cannot allocate device memory per call: applications that reserve all device
memory at start-up and run a fixed memory plan, and inference loops where an
allocator call (which can synchronise the device and take unbounded time) is not
allowed after start-up.  The entry point keeps its temporaries in a fixed array
inside the library instead of the backend's growable scratch.

Every case runs through the C ABI on a fresh backend with the no-allocation call
first, two calls in a row with different shapes (the second must not see
anything of the first call's contents), and checks that the backend's scratch
never grew.  Results are compared with the CPU oracle (the reference's
conv2d_i8_nhwc -> requantize_i32_to_i8 -> relu_i8 composition) and with the
allocating entry point (dw_conv2d_requant_relu_i8).  int8 results must be
identical (tolerance 0, as in every int8 parity test).  The file name makes
pytest collect it last.
"""
import ctypes

import numpy as np
import pytest

import dragonwing_edge_rs_b200 as dw
from dragonwing_edge_rs_b200 import ConvDesc, ops
from dragonwing_edge_rs_b200 import _lib as L
from tests._util import oracle_conv

pytestmark = pytest.mark.gpu

CASES = [
    # n, h, w, c_in, c_out, k, stride, pad, requant_scale, relu
    (1, 28, 28, 64, 64, 3, 1, 1, 0.0011, True),     # tensor-core branch, 36 KiB kernel
    (2, 17, 13, 32, 48, 3, 2, 1, 0.0023, False),    # strided, different shape and scale
]
# c_in % 16 != 0: the CUDA-core branch
CASES_DIRECT = [
    (1, 19, 23, 12, 20, 3, 1, 1, 0.0031, True),     # general CUDA-core kernel
    (2, 9, 11, 20, 8, 1, 1, 0, 0.0047, False),
    (2, 15, 15, 12, 16, 3, 1, 1, 0.0029, True),     # the small-reduction kernel (k*k*c_in <= 256)
]


def _noalloc(be, x, w, y, case):
    n, h, wd, ci, co, k, s, p, scale, relu = case
    return L.load().dw_conv2d_requant_relu_i8_noalloc(be.handle, x.handle, w.handle, y.handle, n, h, wd, ci, co, k,
                                                       k, s, s, p, p, ctypes.c_float(scale), 1 if relu else 0)


def _oracle(case, x, w):
    n, h, wd, ci, co, k, s, p, scale, relu = case
    desc = ConvDesc(n, h, wd, ci, co, k, k, s, s, (p, p, p, p), 1, dw.EPI_RELU if relu else dw.EPI_NONE)
    M = np.full(co, scale, np.float32)
    return oracle_conv(desc, x, w, None, M, M)


def _run_cases(be, cases, seed):
    rng = np.random.default_rng(seed)
    inputs = []
    for case in cases:
        n, h, wd, ci, co, k, s, p, scale, relu = case
        ho, wo = (h + 2 * p - k) // s + 1, (wd + 2 * p - k) // s + 1
        x = rng.integers(-64, 64, n * h * wd * ci).astype(np.int8)
        w = rng.integers(-127, 128, k * k * ci * co).astype(np.int8)
        inputs.append((case, x, w, n * ho * wo * co))
    # the no-allocation calls first, on a backend that has never grown its scratch
    assert be.scratch_bytes() == 0
    got = []
    for case, x, w, out_len in inputs:
        bx, bw, by = be.upload_array(x), be.upload_array(w), be.alloc(out_len)
        st = _noalloc(be, bx, bw, by, case)
        assert st == L.DW_OK, be.last_error()
        be.synchronize(20000)
        got.append(be.download_array(by, np.int8))
    assert be.scratch_bytes() == 0, "the no-allocation entry point grew the backend scratch"
    for (case, x, w, out_len), a in zip(inputs, got):
        ref = _oracle(case, x, w)
        assert np.array_equal(a, ref), f"{int((a != ref).sum())} of {a.size} outputs differ from the oracle for {case}"
        n, h, wd, ci, co, k, s, p, scale, relu = case
        bx, bw, by = be.upload_array(x), be.upload_array(w), be.alloc(out_len)
        ops.conv2d_requant_relu_i8_packed(be, bx, bw, by, n, h, wd, ci, co, k, k, s, s, p, p, scale, relu)
        be.synchronize(20000)
        b = be.download_array(by, np.int8)
        assert np.array_equal(a, b), f"{int((a != b).sum())} of {a.size} outputs differ from the allocating op"


def test_noalloc_tensor_core_branch_two_calls():
    with dw.CudaBackend(0) as be:
        _run_cases(be, CASES, 2024)


def test_noalloc_cuda_core_branch_two_calls():
    with dw.CudaBackend(0) as be:
        _run_cases(be, CASES_DIRECT, 2025)


def test_noalloc_direct_path_config_two_calls():
    # a backend configured for the CUDA-core path takes that branch for every shape
    with dw.CudaBackend(0, conv_path=dw.PATH_DIRECT) as be:
        _run_cases(be, CASES, 2026)


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
        assert be.scratch_bytes() == 0


def test_noalloc_rejects_what_the_allocating_op_rejects():
    with dw.CudaBackend(0) as be:
        lib = L.load()
        x, w, y = be.alloc(64), be.alloc(64), be.alloc(64)
        # a stride beyond int32 (the descriptor's field width); buffers of the sizes it implies
        w16, y16 = be.alloc(16), be.alloc(16)
        st = lib.dw_conv2d_requant_relu_i8_noalloc(be.handle, x.handle, w16.handle, y16.handle, 1, 4, 4, 4, 4, 1, 1,
                                                   1 << 33, 1, 0, 0, ctypes.c_float(0.01), 1)
        assert st == L.DW_ERR_INVALID_ARG, be.last_error()
        assert "exceeds int32" in be.last_error()
        # a shape both entry points reject the same way
        for fn in (lib.dw_conv2d_requant_relu_i8_noalloc, lib.dw_conv2d_requant_relu_i8):
            st = fn(be.handle, x.handle, w.handle, y.handle, 1, 4, 4, 6, 4, 1, 1, 1, 1, 0, 0, ctypes.c_float(0.01), 1)
            assert st == L.DW_ERR_INVALID_ARG
            assert "c_in=6 must be multiple of 4" in be.last_error()
        assert be.scratch_bytes() == 0
