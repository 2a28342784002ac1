"""GPU parity of the tensor-core conv's halo mode: stride-1 convs with several
taps whose maps fill 8 x 16 output tiles (YOLOv8n's C2f and head 3x3 convs,
config 1, the MobileNet/ResNet-style 3x3s).  Per K block the producer loads
one zero-padded halo tile per 16-byte channel chunk and every tap reads it at
a shifted address.  The shapes cover every branch of that path: one to eight
row blocks per tile, odd chunk counts (the last K step's second half reads a
neighbouring pixel against zero weights), two taps per K step for 16-channel
inputs, several channel tiles, 5x5 and 1x3
kernels, asymmetric pads, ragged right and bottom edges, channel-range views,
every epilogue, and accumulators beyond 2^24.  int8 results must be identical
to the oracle's (tolerance 0)."""
import numpy as np
import pytest

import dragonwing_edge_rs_b200 as dw
from dragonwing_edge_rs_b200 import ConvDesc, ops
from dragonwing_edge_rs_b200 import quantization as Q
from tests._util import conv_case, cuda_conv, mismatch_report, oracle_conv

pytestmark = pytest.mark.gpu


def halo_eligible(desc: ConvDesc, esize=1, wide=False) -> bool:
    """The planner's rule for the halo mode (stride 1, several taps, 16-byte
    channel chunks, channel rows of at most 32 bytes unless DW_UMMA_HALO_WIDE
    is set, and 8 x 16 tiles covering the map at >= 70% utilisation)."""
    ho, wo = desc.out_hw()
    tiles_w, tiles_h = (wo + 7) // 8, (ho + 15) // 16
    return (desc.stride_h == 1 and desc.stride_w == 1 and desc.k_h * desc.k_w > 1 and desc.group == 1
            and (desc.c_in * esize) % 16 == 0 and (wide or desc.c_in * esize <= 32)
            and ho * wo >= 0.7 * tiles_w * 8 * tiles_h * 16)


@pytest.fixture(autouse=True)
def _wide_halo(monkeypatch):
    """Every shape here runs the halo producer: the wide-row ones too, the
    small ones that the planner would otherwise give the per-tap producer, and
    stride-2 convs of any channel count (it reads DW_UMMA_HALO_WIDE,
    DW_UMMA_HALO_ANY_SIZE and DW_UMMA_HALO_S2 at each launch)."""
    monkeypatch.setenv("DW_UMMA_HALO_WIDE", "1")
    monkeypatch.setenv("DW_UMMA_HALO_ANY_SIZE", "1")
    monkeypatch.setenv("DW_UMMA_HALO_S2", "2")


@pytest.fixture(scope="module")
def be():
    b = dw.CudaBackend(0, conv_path=dw.PATH_UMMA)
    yield b
    b.close()


HALO_SHAPES = [
    # n, h, w, c_in, c_out, k, epilogue
    (2, 40, 40, 16, 16, 3, dw.EPI_SILU),     # C2f 16 -> 16 (one chunk, up to 8 row blocks)
    (1, 80, 80, 32, 32, 3, dw.EPI_SILU),     # C2f 32 -> 32
    (2, 40, 40, 64, 64, 3, dw.EPI_RELU),
    (1, 40, 48, 64, 80, 3, dw.EPI_SILU),     # head 64 -> 80 (80-wide channel tile)
    (1, 30, 50, 48, 80, 3, dw.EPI_RELU6),    # three chunks: odd count, ragged right edge
    (1, 28, 28, 256, 256, 3, dw.EPI_RELU),   # channel tiles of 128, 16 chunks
    (2, 28, 24, 64, 48, 5, dw.EPI_NONE),     # 5x5, 25 taps
    (1, 56, 56, 64, 64, 3, dw.EPI_RELU),     # config 1 geometry
    (1, 45, 23, 128, 64, 3, dw.EPI_SILU),    # ragged bottom and right
]


@pytest.mark.parametrize("shape", HALO_SHAPES, ids=lambda s: "x".join(map(str, s)))
def test_halo_conv_bit_exact(be, shape):
    n, h, w, ci, co, k, epi = shape
    rng = np.random.default_rng(hash(shape) & 0xFFFFFFFF)
    desc, x, wt, b, M, D = conv_case(rng, n, h, w, ci, co, k=k, s=1, epilogue=epi)
    assert halo_eligible(desc, wide=True)
    y = cuda_conv(be, desc, x, wt, b, M, D)
    ref = oracle_conv(desc, x, wt, b, M, D)
    assert np.array_equal(y, ref), mismatch_report(y, ref)


@pytest.mark.parametrize("kh,kw,pads", [(1, 3, (0, 1, 0, 1)), (3, 1, (1, 0, 1, 0)), (3, 3, (1, 0, 2, 1)),
                                        (3, 3, (0, 0, 0, 0)), (5, 3, (2, 1, 2, 1))])
def test_halo_rectangular_kernels_and_asymmetric_pads(be, kh, kw, pads):
    rng = np.random.default_rng(kh * 31 + kw * 7 + sum(pads))
    n, h, w, ci, co = 2, 46, 40, 32, 48
    desc = ConvDesc(n, h, w, ci, co, kh, kw, 1, 1, pads, 1, dw.EPI_RELU)
    x = rng.integers(-64, 64, n * h * w * ci).astype(np.int8)
    wt = rng.integers(-127, 128, kh * kw * ci * co).astype(np.int8)
    s_w = rng.uniform(0.001, 0.01, co).astype(np.float32)
    M = Q.requant_scales(0.02, s_w, 0.05)
    D = Q.dequant_scales(0.02, s_w)
    b = rng.integers(-1000, 1001, co).astype(np.int32)
    desc.q6, desc.inv_s_out = 127, float(np.float32(1.0) / np.float32(0.05))
    assert halo_eligible(desc, wide=True)
    y = cuda_conv(be, desc, x, wt, b, M, D)
    ref = oracle_conv(desc, x, wt, b, M, D)
    assert np.array_equal(y, ref), mismatch_report(y, ref)


@pytest.mark.parametrize("kh,kw,pads", [(3, 3, (1, 1, 1, 1)), (5, 5, (2, 2, 2, 2)), (1, 3, (0, 1, 0, 1)),
                                        (3, 1, (1, 0, 1, 0)), (2, 2, (0, 0, 1, 1)), (3, 4, (1, 1, 1, 2))])
@pytest.mark.parametrize("epi", [dw.EPI_SILU, dw.EPI_RELU])
def test_halo_two_tap_k_steps_c16(be, kh, kw, pads, epi):
    """16 input channels: one 32-byte K step takes two horizontal taps (the
    pixel one to the right is the next tap's pixel), the row's last tap of an
    odd-width kernel pairs with an all-zero weight slice."""
    rng = np.random.default_rng(kh * 13 + kw * 7 + sum(pads) + epi)
    n, h, w, ci, co = 2, 46, 40, 16, 32
    desc = ConvDesc(n, h, w, ci, co, kh, kw, 1, 1, pads, 1, epi)
    x = rng.integers(-128, 128, n * h * w * ci).astype(np.int8)
    wt = rng.integers(-127, 128, kh * kw * ci * co).astype(np.int8)
    s_w = rng.uniform(0.001, 0.01, co).astype(np.float32)
    M = Q.requant_scales(0.02, s_w, 0.05)
    D = Q.dequant_scales(0.02, s_w)
    b = rng.integers(-1000, 1001, co).astype(np.int32)
    desc.q6, desc.inv_s_out = Q.relu6_ceiling(0.05), float(np.float32(1.0) / np.float32(0.05))
    assert halo_eligible(desc)
    y = cuda_conv(be, desc, x, wt, b, M, D)
    ref = oracle_conv(desc, x, wt, b, M, D)
    assert np.array_equal(y, ref), mismatch_report(y, ref)


def test_halo_extreme_accumulators(be):
    """All-extreme inputs and weights: |acc| up to 9 * 256 * 128 * 128 > 2^24
    (the exact epilogue path), through the halo producer."""
    rng = np.random.default_rng(99)
    desc, x, wt, b, M, D = conv_case(rng, 1, 24, 24, 256, 64, k=3, s=1, epilogue=dw.EPI_NONE)
    x = np.where(rng.random(x.size) < 0.5, -128, 127).astype(np.int8)
    wt = np.where(rng.random(wt.size) < 0.9, -128, 127).astype(np.int8)
    M = (M * np.float32(1e-3)).astype(np.float32)
    y = cuda_conv(be, desc, x, wt, b, M, D)
    ref = oracle_conv(desc, x, wt, b, M, D)
    assert np.array_equal(y, ref), mismatch_report(y, ref)


@pytest.mark.parametrize("ci", [16, 32])
@pytest.mark.parametrize("in_view,out_view", [(True, True), (True, False), (False, True)])
def test_halo_channel_range_views(be, ci, in_view, out_view):
    """Input and/or output as channel ranges of wider tensors (the C2f concat
    views): the halo boxes read only the view's channels, the stores write only
    the view's.  A dense side takes the whole-row boxes (16-channel input rows,
    outputs of exactly one channel tile), the view side the 16-byte rows."""
    rng = np.random.default_rng(7 + ci + 2 * in_view + out_view)
    n, h, w, co = 2, 41, 37, 32
    c_tot_in = 96 if in_view else ci
    c_tot_out = 64 if out_view else co
    in_off, out_off = (32 if in_view else 0), (16 if out_view else 0)
    desc, x, wt, b, M, D = conv_case(rng, n, h, w, ci, co, k=3, s=1, epilogue=dw.EPI_SILU)
    big_in = rng.integers(-128, 128, (n, h, w, c_tot_in)).astype(np.int8)
    big_in[..., in_off:in_off + ci] = x.reshape(n, h, w, ci)
    bx = be.upload_array(big_in.reshape(-1))
    wp = ops.prepare_weights_i8(be, desc, be.upload_array(wt))
    bb, bm, bd = be.upload_array(b), be.upload_array(M), be.upload_array(D)
    out0 = rng.integers(-128, 128, (n, h, w, c_tot_out)).astype(np.int8)
    by = be.upload_array(out0.reshape(-1))
    ops.conv2d_i8_view(be, desc, (bx, in_off, c_tot_in), wp, bb, bm, bd, (by, out_off, c_tot_out))
    got = be.download_array(by, np.int8).reshape(n, h, w, c_tot_out)
    be.synchronize(20000)
    ref = oracle_conv(desc, x, wt, b, M, D).reshape(n, h, w, co)
    sel = got[..., out_off:out_off + co]
    assert np.array_equal(sel, ref), mismatch_report(sel.reshape(-1), ref.reshape(-1))
    # channels outside the view are untouched
    assert np.array_equal(got[..., :out_off], out0[..., :out_off])
    assert np.array_equal(got[..., out_off + co:], out0[..., out_off + co:])


S2_SHAPES = [
    # n, h, w, c_in, c_out, k, pads (t, l, b, r), epilogue -- stride 2
    (2, 64, 64, 16, 32, 3, (1, 1, 1, 1), dw.EPI_SILU),     # YOLOv8n's conv_2 shape class
    (1, 80, 96, 32, 64, 3, (1, 1, 1, 1), dw.EPI_SILU),     # conv_10 class
    (1, 60, 44, 64, 64, 3, (1, 1, 1, 1), dw.EPI_RELU),     # ragged output (30 x 22)
    (2, 64, 48, 16, 48, 3, (0, 0, 1, 1), dw.EPI_RELU6),    # asymmetric pads: taps from (0, 0)
    (1, 48, 64, 32, 32, 5, (2, 2, 2, 2), dw.EPI_NONE),     # 5x5: 3 x 3 taps over the parity planes
    (2, 32, 48, 48, 16, 2, (0, 0, 0, 0), dw.EPI_SILU),     # 2x2: one tap, every parity in K
]


@pytest.mark.parametrize("shape", S2_SHAPES, ids=lambda s: "x".join(map(str, s[:6])) + f"_p{''.join(map(str, s[6]))}")
def test_halo_stride2_parity_planes(be, shape):
    """Stride-2 convs through the halo producer over the input's four parity
    planes: a stride-1 conv over x'[i][j][(ph, pw, c)] = x[2i + ph][2j + pw][c]
    with the kernel taps regrouped (zero weight slices where no tap lands)."""
    n, h, w, ci, co, k, pads, epi = shape
    rng = np.random.default_rng(sum(shape[:6]) + 7 * sum(pads) + epi)
    desc = ConvDesc(n, h, w, ci, co, k, k, 2, 2, pads, 1, epi)
    x = rng.integers(-128, 128, n * h * w * ci).astype(np.int8)
    wt = rng.integers(-127, 128, k * k * ci * co).astype(np.int8)
    s_w = rng.uniform(0.001, 0.01, co).astype(np.float32)
    M = Q.requant_scales(0.02, s_w, 0.05)
    D = Q.dequant_scales(0.02, s_w)
    b = rng.integers(-1000, 1001, co).astype(np.int32)
    desc.q6, desc.inv_s_out = Q.relu6_ceiling(0.05), float(np.float32(1.0) / np.float32(0.05))
    y = cuda_conv(be, desc, x, wt, b, M, D)
    ref = oracle_conv(desc, x, wt, b, M, D)
    assert np.array_equal(y, ref), mismatch_report(y, ref)


def test_halo_stride2_extreme_and_views(be):
    """Saturated inputs and weights (|acc| > 2^24) through the parity planes,
    the output written into a channel range of a wider tensor."""
    rng = np.random.default_rng(2202)
    n, h, w, ci, co, c_tot_out = 2, 64, 48, 64, 32, 96
    desc, x, wt, b, M, D = conv_case(rng, n, h, w, ci, co, k=3, s=2, epilogue=dw.EPI_NONE)
    x = np.where(rng.random(x.size) < 0.5, -128, 127).astype(np.int8)
    wt = np.where(rng.random(wt.size) < 0.9, -128, 127).astype(np.int8)
    M = (M * np.float32(1e-3)).astype(np.float32)
    bx = be.upload_array(x)
    wp = ops.prepare_weights_i8(be, desc, be.upload_array(wt))
    bb, bm, bd = be.upload_array(b), be.upload_array(M), be.upload_array(D)
    ho, wo = desc.out_hw()
    out0 = rng.integers(-128, 128, (n, ho, wo, c_tot_out)).astype(np.int8)
    by = be.upload_array(out0.reshape(-1))
    ops.conv2d_i8_view(be, desc, (bx, 0, ci), wp, bb, bm, bd, (by, 32, c_tot_out))
    got = be.download_array(by, np.int8).reshape(n, ho, wo, c_tot_out)
    be.synchronize(20000)
    ref = oracle_conv(desc, x, wt, b, M, D).reshape(n, ho, wo, co)
    assert np.array_equal(got[..., 32:64], ref), mismatch_report(got[..., 32:64].reshape(-1), ref.reshape(-1))
    assert np.array_equal(got[..., :32], out0[..., :32])
    assert np.array_equal(got[..., 64:], out0[..., 64:])
