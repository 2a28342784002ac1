"""GPU parity at the benchmark configurations' own shapes.

BASELINE config 3 (standalone INT8 QGemm with int32 accumulation, int32 bias and
per-column requantisation to int8) at its three shapes (4096,4096,4096),
(8192,1024,4096) and (256,4096,11008), with config 3's distributions: operands
int8 U[-127,127], scales U[0.001,0.01].  The reference's gemm_i8_scalar
(crates/dragonwing-cpu/src/ops.rs:2981-2995) followed by
requantize_i32_to_i8_scalar (ops.rs:3380-3386) per column is the oracle; every
output of every shape is compared (the threaded oracle takes a few seconds for
4096^3).  K = 11008 is also driven to accumulators of
+-177,548,032 (> 2^24, where the int -> float conversion must round to
nearest) by constant rows and columns.

BASELINE config 1 (3x3 s1 p1, 56x56, 64 -> 64, int32 bias, per-channel M,
ReLU) at its throughput batch N=256, compared on sampled images (every image
is an independent conv).  int8 results must be identical (tolerance 0).
"""
import numpy as np
import pytest

import dragonwing_edge_rs_b200 as dw
from dragonwing_edge_rs_b200 import ops
from dragonwing_edge_rs_b200 import quantization as Q
from oracle import dwref
from tests._util import conv_case, mismatch_report, oracle_conv

pytestmark = pytest.mark.gpu

QGEMM_SHAPES = [(4096, 4096, 4096), (8192, 1024, 4096), (256, 4096, 11008)]


@pytest.fixture(scope="module")
def be():
    b = dw.CudaBackend(0)
    yield b
    b.close()


def _config3_operands(rng, m, n, k, spread):
    a = rng.integers(-127, 128, (m, k), dtype=np.int8)
    b = rng.integers(-127, 128, (k, n), dtype=np.int8)
    bias = rng.integers(-1000, 1001, n).astype(np.int32)
    s_a, s_out = (np.float32(v) for v in rng.uniform(0.001, 0.01, 2))
    s_b = rng.uniform(0.001, 0.01, n).astype(np.float32)
    M = Q.requant_scales(s_a, s_b, s_out)
    if spread:
        # Scales that keep most outputs inside (-128, 127): the accumulator's
        # standard deviation is about 127^2 / 3 * sqrt(k).
        M = (M / M.mean() * np.float32(40.0 / (127.0 * 127.0 / 3.0 * np.sqrt(k)))).astype(np.float32)
    return a, b, bias, M


def _run_qgemm(be, a, b, bias, M, m, n, k, epi, q6=100):
    ba, bb = be.upload_array(a.reshape(-1)), be.upload_array(b.reshape(-1))
    bp = ops.prepare_gemm_b_i8(be, bb, k, n)
    y = be.alloc(m * n)
    ops.qgemm_i8(be, ba, bp, be.upload_array(bias), be.upload_array(M), y, m, n, k, epi, q6)
    got = be.download_array(y, np.int8).reshape(m, n)
    be.synchronize(60000)
    for buf in (ba, bb, bp, y):
        buf.free()
    return got


@pytest.mark.parametrize("m,n,k", QGEMM_SHAPES, ids=[f"{m}x{n}x{k}" for m, n, k in QGEMM_SHAPES])
@pytest.mark.parametrize("spread", [False, True], ids=["config_scales", "spread_scales"])
def test_qgemm_config3_shapes(be, m, n, k, spread):
    rng = np.random.default_rng(m + 7 * n + 13 * k + (1 if spread else 0))
    a, b, bias, M = _config3_operands(rng, m, n, k, spread)
    epi = dw.EPI_RELU if spread else dw.EPI_NONE
    got = _run_qgemm(be, a, b, bias, M, m, n, k, epi)
    ref = dwref.qgemm_i8(a, b, bias, M, m, n, k, epi, 100, threads=dwref.num_cpus()).reshape(m, n)
    assert np.array_equal(got, ref), mismatch_report(got.reshape(-1), ref.reshape(-1))
    if spread:
        # the comparison is not only of saturated values
        assert np.mean(np.abs(ref.astype(np.int32)) < 127) > 0.5


def test_qgemm_k11008_accumulators_beyond_2_24(be):
    """Rows and columns of constant +-127 drive |acc| to 127*127*11008 =
    177,548,032 (> 2^24: the conversion to float rounds); per-column scales put
    those products near a rounding boundary of the int8 result."""
    m, n, k = 256, 4096, 11008
    rng = np.random.default_rng(11008)
    a = rng.integers(-127, 128, (m, k), dtype=np.int8)
    b = rng.integers(-127, 128, (k, n), dtype=np.int8)
    a[0, :] = 127
    a[1, :] = -127
    a[2, ::2], a[2, 1::2] = 127, -127
    b[:, :64] = 127
    b[:, 64:80] = -127
    bias = rng.integers(-1000, 1001, n).astype(np.int32)
    bias[:4] = [0, 1, -1, 2 ** 31 - 1 - 127 * 127 * k]
    peak = np.float32(127 * 127 * k)
    # M so that peak * M lands on and near the half-integers of [-127, 127]
    targets = np.linspace(-126.5, 126.5, n).astype(np.float32)
    M = (targets / peak).astype(np.float32)
    for epi in (dw.EPI_NONE, dw.EPI_RELU):
        got = _run_qgemm(be, a, b, bias, M, m, n, k, epi)
        ref = dwref.qgemm_i8(a, b, bias, M, m, n, k, epi, 100, threads=dwref.num_cpus()).reshape(m, n)
        assert np.array_equal(got, ref), mismatch_report(got.reshape(-1), ref.reshape(-1))


def test_config1_n256_sampled_images(be):
    """Config 1 at its throughput batch: 256 x 56x56x64 -> 64, 3x3 s1 p1, int32
    bias, per-channel M, ReLU; 8 images (first, last, random) against the oracle."""
    rng = np.random.default_rng(256)
    desc, x, wt, b, M, D = conv_case(rng, 256, 56, 56, 64, 64, k=3, s=1, epilogue=dw.EPI_RELU)
    bx, bw = be.upload_array(x), be.upload_array(wt)
    wp = ops.prepare_weights_i8(be, desc, bw)
    bb, bm, bd = be.upload_array(b), be.upload_array(M), be.upload_array(D)
    ho, wo = desc.out_hw()
    by = be.alloc(desc.n * ho * wo * desc.c_out)
    ops.conv2d_i8(be, desc, bx, wp, bb, bm, bd, by)
    y = be.download_array(by, np.int8).reshape(256, -1)
    be.synchronize(60000)
    img_in = 56 * 56 * 64
    images = sorted({0, 255, *(int(i) for i in rng.integers(1, 255, 6))})
    for i in images:
        d1 = dw.ConvDesc(1, 56, 56, 64, 64, 3, 3, 1, 1, desc.pads, 1, desc.epilogue)
        d1.q6, d1.inv_s_out = desc.q6, desc.inv_s_out
        ref = oracle_conv(d1, x[i * img_in:(i + 1) * img_in], wt, b, M, D, threads=dwref.num_cpus())
        assert np.array_equal(y[i], ref), f"image {i}: " + mismatch_report(y[i], ref)
