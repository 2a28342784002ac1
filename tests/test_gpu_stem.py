"""The fused input stem (dw_conv2d_stem_u8_i8): the uint8 image's
quantisation and the 3x3 conv on its 3 channels in one kernel, bit-exact
against the oracle's two steps (quantize_u8_to_i8, then the fused conv of
the reference's scalar path) on the GPU."""
import numpy as np
import pytest

import dragonwing_edge_rs_b200 as dw
from dragonwing_edge_rs_b200 import ConvDesc, ops
from dragonwing_edge_rs_b200 import _lib as L
from dragonwing_edge_rs_b200 import quantization as Q
from oracle import dwref
from tests._util import mismatch_report, oracle_conv

pytestmark = pytest.mark.gpu

S_IN = 1.0 / 127.0


@pytest.fixture(scope="module")
def be():
    b = dw.CudaBackend(0)
    yield b
    b.close()


def _case(rng, n, h, w, c_out, s, pads, epilogue, s_out=0.05, w_range=127):
    desc = ConvDesc(n, h, w, 3, c_out, 3, 3, s, s, pads, 1, epilogue)
    x = rng.integers(0, 256, n * h * w * 3).astype(np.uint8)
    wt = rng.integers(-w_range, w_range + 1, 27 * c_out).astype(np.int8)
    s_w = rng.uniform(0.001, 0.01, c_out).astype(np.float32)
    M = Q.requant_scales(S_IN, s_w, s_out)
    D = Q.dequant_scales(S_IN, s_w)
    b = rng.integers(-1000, 1001, c_out).astype(np.int32)
    desc.q6 = Q.relu6_ceiling(s_out)
    desc.inv_s_out = float(np.float32(1.0) / np.float32(s_out))
    return desc, x, wt, b, M, D


def _run(be, desc, x, wt, b, M, D):
    ho, wo = desc.out_hw()
    bx, bw, bb, bm, bd = (be.upload_array(a) for a in (x, wt, b, M, D))
    by = be.alloc(desc.n * ho * wo * desc.c_out)
    ops.conv2d_stem_u8_i8(be, desc, bx, S_IN, bw, bb, bm, bd, by)
    got = be.download_array(by, np.int8)
    be.synchronize(timeout_ms=20000)
    for buf in (bx, bw, bb, bm, bd, by):
        buf.free()
    return got


def _expect(desc, x, wt, b, M, D):
    q = dwref.quantize_u8_to_i8(x, S_IN).astype(np.int8)
    return oracle_conv(desc, q, wt, b, M, D).ravel()


@pytest.mark.parametrize("geo", [
    # n, h, w, c_out, stride, pads, epilogue
    (2, 64, 64, 16, 2, (1, 1, 1, 1), dw.EPI_SILU),      # YOLOv8n's stem shape, small
    (1, 37, 48, 32, 2, (1, 1, 1, 1), dw.EPI_SILU),      # odd height: a partial last band
    (1, 24, 32, 64, 1, (1, 1, 1, 1), dw.EPI_RELU6),     # stride 1, four channel groups
    (3, 20, 16, 16, 2, (0, 0, 1, 1), dw.EPI_NONE),      # asymmetric padding, linear
    (1, 30, 48, 48, 2, (2, 5, 2, 5), dw.EPI_RELU),      # wide left padding
])
def test_stem_conv_matches_oracle(be, geo):
    n, h, w, c_out, s, pads, epi = geo
    rng = np.random.default_rng(sum(geo[:5]) + epi)
    case = _case(rng, n, h, w, c_out, s, pads, epi)
    got, exp = _run(be, *case), _expect(*case)
    assert np.array_equal(got, exp), mismatch_report(got, exp)


def test_stem_conv_full_yolov8n_batch(be):
    """The bench's stem at batch 32 (640x640, 3 -> 16, stride 2, SiLU): two
    images checked against the oracle, and a second call on the same buffers
    gives the same bytes."""
    rng = np.random.default_rng(640)
    desc, x, wt, b, M, D = _case(rng, 32, 640, 640, 16, 2, (1, 1, 1, 1), dw.EPI_SILU)
    got = _run(be, desc, x, wt, b, M, D)
    ho, wo = desc.out_hw()
    per = ho * wo * 16
    for i in (0, 31):
        d1 = ConvDesc(1, 640, 640, 3, 16, 3, 3, 2, 2, (1, 1, 1, 1), 1, dw.EPI_SILU)
        d1.q6, d1.inv_s_out = desc.q6, desc.inv_s_out
        xi = x[i * 640 * 640 * 3:(i + 1) * 640 * 640 * 3]
        exp = _expect(d1, xi, wt, b, M, D)
        assert np.array_equal(got[i * per:(i + 1) * per], exp), f"image {i}: " + mismatch_report(got[i * per:(i + 1) * per], exp)
    assert np.array_equal(_run(be, desc, x, wt, b, M, D), got)


def test_stem_conv_exact_fallbacks(be):
    """Large accumulators and uncertain SiLU results take the exact
    per-element path: full-range weights, a tiny output scale (most results
    saturate or sit near rounding ties) and one channel with a non-finite
    dequant scale (the whole block then computes every element exactly)."""
    rng = np.random.default_rng(7)
    desc, x, wt, b, M, D = _case(rng, 2, 32, 32, 32, 2, (1, 1, 1, 1), dw.EPI_SILU, s_out=0.0005)
    got, exp = _run(be, desc, x, wt, b, M, D), _expect(desc, x, wt, b, M, D)
    assert np.array_equal(got, exp), mismatch_report(got, exp)
    D2 = D.copy()
    D2[5] = np.float32(np.inf)
    got, exp = _run(be, desc, x, wt, b, M, D2), _expect(desc, x, wt, b, M, D2)
    assert np.array_equal(got, exp), mismatch_report(got, exp)


def test_stem_conv_rejects_other_shapes(be):
    rng = np.random.default_rng(3)
    desc, x, wt, b, M, D = _case(rng, 1, 16, 24, 16, 2, (1, 1, 1, 1), dw.EPI_SILU)  # width not a multiple of 16
    with pytest.raises(dw.BackendError) as e:
        _run(be, desc, x, wt, b, M, D)
    assert e.value.status == L.DW_ERR_UNSUPPORTED
