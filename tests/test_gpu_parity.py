"""GPU parity: every op through the C ABI against the CPU oracle (bit-exact for
int8), on seeded inputs; the reference KATs through the device path; error
behaviour; the bounded-wait expiry path."""
import numpy as np
import pytest

import dragonwing_edge_rs_b200 as dw
from dragonwing_edge_rs_b200 import ops
from dragonwing_edge_rs_b200 import quantization as Q
from oracle import dwref
from tests._util import conv_case, cuda_conv, mismatch_report, oracle_conv

pytestmark = pytest.mark.gpu


@pytest.fixture(scope="module")
def be():
    b = dw.CudaBackend(0)
    yield b
    b.close()


@pytest.fixture(scope="module")
def be_direct():
    b = dw.CudaBackend(0, conv_path=dw.PATH_DIRECT)
    yield b
    b.close()


@pytest.fixture(scope="module", params=[dw.DWV_SLAB, dw.DWV_STREAM2, dw.DWV_STREAM2X2, dw.DWV_STREAM4],
                ids=["slab", "stream2", "stream2x2", "stream4"])
def be_dwv(request):
    """A backend forced onto one int8 depthwise 3x3 s1 kernel variant."""
    b = dw.CudaBackend(0, dw_variant=request.param)
    yield b
    b.close()


@pytest.fixture(scope="module")
def be_umma():
    b = dw.CudaBackend(0, conv_path=dw.PATH_UMMA)
    yield b
    b.close()


# ---------------------------------------------------------------- reference KATs

def test_kat_gemm_i8(be):
    a = be.upload_array(np.array([1, 2, 3, 4, 5, 6], np.int8))
    b = be.upload_array(np.array([7, 8, 9, 10, 11, 12], np.int8))
    c = be.alloc(16)
    ops.gemm_i8_packed(be, a, b, c, 2, 2, 3)
    assert be.download_array(c, np.int32).tolist() == [58, 64, 139, 154]  # ops.rs:1111-1125


def test_kat_conv2d_i8_basic(be):
    x = be.upload_array(np.ones(25, np.int8))
    w = be.upload_array(np.ones(9, np.int8))
    out = be.alloc(9 * 4)
    ops.conv2d_i8_nhwc_packed(be, x, w, out, 1, 5, 5, 1, 1, 3, 3, 1, 1, 0, 0)
    assert (be.download_array(out, np.int32) == 9).all()  # ops.rs:1148-1173


@pytest.mark.parametrize("acc,scale,expected", [
    ([1000, 2000, -1000, -2000, 0], 0.1, [100, 127, -100, -128, 0]),
    ([0, 1000, 5000, -2000, -5000], 0.01, [0, 10, 50, -20, -50]),
    ([0, 100, -100, 12700, -12700, 25400, -25400, 500, -500, 1234, -1234, 5, -5, 9999, -9999, 12700], 0.01,
     [0, 1, -1, 127, -127, 127, -128, 5, -5, 12, -12, 0, 0, 100, -100, 127]),
])
def test_kat_requantize(be, acc, scale, expected):
    bi = be.upload_array(np.array(acc, np.int32))
    bo = be.alloc(len(acc))
    ops.requantize_i32_to_i8_packed(be, bi, bo, scale)
    assert be.download_array(bo, np.int8).tolist() == expected


def test_kat_add_relu_quant_dequant(be):
    a = be.upload_array(np.array([10, 20, 30, 40, 50], np.int8))
    b = be.upload_array(np.array([5, 10, 15, 20, 25], np.int8))
    o = be.alloc(5)
    ops.add_i8_packed(be, a, b, o, 1.0, 1.0)
    assert be.download_array(o, np.int8).tolist() == [15, 30, 45, 60, 75]
    a = be.upload_array(np.array([100, 100, 100], np.int8))
    o3 = be.alloc(3)
    ops.add_i8_packed(be, a, a, o3, 0.5, 0.5)
    assert be.download_array(o3, np.int8).tolist() == [100, 100, 100]
    r = be.upload_array(np.array([-50, -10, 0, 10, 50], np.int8))
    ops.relu_i8_packed(be, r, o)
    assert be.download_array(o, np.int8).tolist() == [0, 0, 0, 10, 50]
    f = be.upload_array(np.array([0.0, 5.0, -5.0, 200.0, -200.0], np.float32))
    ops.quantize_f32_to_i8_packed(be, f, o, 1.0)
    assert be.download_array(o, np.int8).tolist() == [0, 5, -5, 127, -128]
    q = be.upload_array(np.array([0, 10, -10, 127, -128], np.int8))
    fo = be.alloc(20)
    ops.dequantize_i8_packed_to_f32(be, q, fo, 0.5)
    assert be.download_array(fo, np.float32).tolist() == [0.0, 5.0, -5.0, 63.5, -64.0]


# ---------------------------------------------------------------- elementwise parity

@pytest.mark.parametrize("n", [1, 15, 16, 17, 4099, 1 << 20])
def test_elementwise_parity(be, n):
    rng = np.random.default_rng(n)
    acc = rng.integers(-2**31, 2**31 - 1, n, dtype=np.int64).astype(np.int32)
    acc[: n // 2] = rng.integers(-30000, 30000, n // 2)
    bi = be.upload_array(acc)
    bo = be.alloc(n)
    for s in (0.001, 0.0123, 7.5e-6):
        ops.requantize_i32_to_i8_packed(be, bi, bo, s)
        assert np.array_equal(be.download_array(bo, np.int8), dwref.requantize_i32_to_i8(acc, s))
    a = rng.integers(-128, 128, n).astype(np.int8)
    b = rng.integers(-128, 128, n).astype(np.int8)
    ba, bb = be.upload_array(a), be.upload_array(b)
    ops.add_i8_packed(be, ba, bb, bo, 0.731, 1.27)
    assert np.array_equal(be.download_array(bo, np.int8), dwref.add_i8(a, b, 0.731, 1.27))
    ops.relu_i8_packed(be, ba, bo)
    assert np.array_equal(be.download_array(bo, np.int8), dwref.relu_i8(a))
    f = (rng.standard_normal(n) * 3).astype(np.float32)
    bf = be.upload_array(f)
    ops.quantize_f32_to_i8_packed(be, bf, bo, 0.037)
    assert np.array_equal(be.download_array(bo, np.int8), dwref.quantize_f32_to_i8(f, 0.037))
    bfo = be.alloc(4 * n)
    ops.dequantize_i8_packed_to_f32(be, ba, bfo, 0.037)
    assert np.array_equal(be.download_array(bfo, np.float32), dwref.dequantize_i8_to_f32(a, 0.037))
    u = rng.integers(0, 256, n).astype(np.uint8)
    bu = be.upload_array(u)
    ops.quantize_u8_to_i8(be, bu, bo, 0.0123)
    assert np.array_equal(be.download_array(bo, np.int8), dwref.quantize_u8_to_i8(u, 0.0123))


@pytest.mark.parametrize("n", [16, 4096, 65536, 4099])
@pytest.mark.parametrize("ra,rb", [(0.5, 0.25), (0.5, -0.5), (0.731, 1.27), (3.0e-39, 1.0), (1e30, 2.0),
                                   (-1.5, 2.5e2)])
def test_add_i8_ratios(be, n, ra, rb):
    """add_i8 over ratio pairs that make .5 ties common (0.5, 0.25, -0.5), a
    subnormal ratio, ratios at and past the packed path's limit (1e30) and
    large ones that saturate; multiples of 16 take the packed path, 4099 the
    per-element one.  Bit-exact against the reference's add_i8."""
    rng = np.random.default_rng(n + int(abs(rb) * 10))
    a = rng.integers(-128, 128, n).astype(np.int8)
    b = rng.integers(-128, 128, n).astype(np.int8)
    ba, bb, bo = be.upload_array(a), be.upload_array(b), be.alloc(n)
    ra, rb = float(np.float32(ra)), float(np.float32(rb))
    ops.add_i8_packed(be, ba, bb, bo, ra, rb)
    got, exp = be.download_array(bo, np.int8), dwref.add_i8(a, b, ra, rb)
    assert np.array_equal(got, exp), mismatch_report(got, exp)


# ---------------------------------------------------------------- fused conv parity

def _check_conv(be, case):
    desc, x, wt, b, M, D = case
    y = cuda_conv(be, desc, x, wt, b, M, D)
    ref = oracle_conv(desc, x, wt, b, M, D)
    assert np.array_equal(y, ref), mismatch_report(y, ref)


def test_config1_bit_exact_both_paths(be_direct, be_umma):
    """3x3 s1 p1, 1x56x56x64 -> 64, int32 bias, per-channel M, ReLU."""
    rng = np.random.default_rng(20250101)
    case = conv_case(rng, 1, 56, 56, 64, 64, k=3, s=1, epilogue=dw.EPI_RELU)
    _check_conv(be_direct, case)
    _check_conv(be_umma, case)


CONV_SHAPES = [
    # n, h, w, c_in, c_out, k, s, epilogue
    (1, 8, 8, 16, 16, 1, 1, dw.EPI_NONE),
    (2, 13, 11, 32, 48, 1, 1, dw.EPI_RELU),
    (1, 9, 9, 64, 64, 3, 1, dw.EPI_RELU),
    (2, 16, 16, 48, 96, 3, 2, dw.EPI_RELU6),
    (1, 20, 20, 96, 576, 1, 1, dw.EPI_RELU6),
    (1, 10, 14, 576, 96, 1, 1, dw.EPI_NONE),
    (1, 40, 40, 32, 64, 3, 2, dw.EPI_SILU),
    (1, 12, 12, 128, 80, 3, 1, dw.EPI_SILU),
    (3, 7, 7, 256, 256, 3, 1, dw.EPI_RELU),
    (1, 30, 50, 16, 32, 3, 1, dw.EPI_SILU),
    (1, 6, 6, 192, 144, 3, 1, dw.EPI_RELU6),
    (2, 5, 5, 64, 512, 1, 1, dw.EPI_RELU),
    (4, 6, 6, 64, 64, 3, 1, dw.EPI_RELU6),   # three whole images per row block (last block ragged)
    (3, 14, 14, 64, 128, 3, 2, dw.EPI_RELU),  # strided to 7x7: two images per row block
]


@pytest.mark.parametrize("shape", CONV_SHAPES, ids=lambda s: "x".join(map(str, s)))
@pytest.mark.parametrize("path", ["umma", "direct"])
def test_conv_parity_sweep(be_direct, be_umma, shape, path):
    n, h, w, ci, co, k, s, epi = shape
    rng = np.random.default_rng(hash(shape) & 0xffffffff)
    case = conv_case(rng, n, h, w, ci, co, k=k, s=s, epilogue=epi)
    _check_conv(be_umma if path == "umma" else be_direct, case)


@pytest.mark.parametrize("pads,k,s", [((0, 0, 0, 0), 3, 1), ((1, 0, 2, 1), 3, 1), ((0, 1, 1, 0), 3, 2),
                                      ((2, 2, 2, 2), 5, 1), ((1, 1, 1, 1), 3, 2)])
def test_conv_asymmetric_pads(be, pads, k, s):
    rng = np.random.default_rng(sum(pads) * 7 + k + s)
    _check_conv(be, conv_case(rng, 2, 12, 10, 32, 32, k=k, s=s, pads=pads, epilogue=dw.EPI_RELU))


def test_conv_odd_channels_direct_fallback(be):
    """C_in=3 stem (YOLO), C_out not a multiple of 16: CUDA-core path, same contract."""
    rng = np.random.default_rng(5)
    _check_conv(be, conv_case(rng, 2, 32, 32, 3, 16, k=3, s=2, epilogue=dw.EPI_SILU))
    _check_conv(be, conv_case(rng, 1, 9, 9, 8, 12, k=3, s=1, epilogue=dw.EPI_RELU))


def test_conv_extreme_values(be_umma, be_direct):
    """Saturating inputs/weights/bias: int32 accumulators far above 2^24."""
    rng = np.random.default_rng(9)
    desc, x, wt, b, M, D = conv_case(rng, 1, 8, 8, 512, 64, k=3, epilogue=dw.EPI_NONE, x_range=(-128, 127))
    x[:] = -128
    wt[: wt.size // 2] = -128
    b = rng.integers(-2**30, 2**30, 64).astype(np.int32)
    M = rng.uniform(1e-9, 1e-6, 64).astype(np.float32)
    for be in (be_umma, be_direct):
        _check_conv(be, (desc, x, wt, b, M, D))


@pytest.mark.parametrize("k,group", [(1, 1), (3, 1), (3, "dw")])
def test_conv_rounding_ties(be_umma, be_direct, k, group):
    """Requant scales of 0.5 / 0.25 / 1.5 make (float)acc * M an exact .5 tie for
    many accumulators: roundf's half-away-from-zero must be reproduced exactly."""
    rng = np.random.default_rng(31 + k)
    c = 64
    g = c if group == "dw" else 1
    desc, x, wt, b, M, D = conv_case(rng, 2, 10, 10, c, c, k=k, group=g, epilogue=dw.EPI_NONE, x_range=(-3, 3))
    wt[:] = rng.integers(-3, 4, wt.size)
    M = np.resize(np.array([0.5, 0.25, 1.5, -0.5], np.float32), c)
    b = rng.integers(-7, 8, c).astype(np.int32)
    for be in (be_umma, be_direct):
        _check_conv(be, (desc, x, wt, b, M, D))
    desc.epilogue = dw.EPI_RELU6
    desc.q6 = 5
    _check_conv(be_umma, (desc, x, wt, b, M, D))


@pytest.mark.parametrize("k", [1, 3])
@pytest.mark.parametrize("epi,q6", [(dw.EPI_RELU, 127), (dw.EPI_RELU6, 6), (dw.EPI_RELU6, 0), (dw.EPI_RELU6, 127)])
def test_conv_relu_requant_edges(be_umma, be_direct, k, epi, q6):
    """ReLU / ReLU6 requantisation of the tensor-core conv over its one-add
    path and the fall-back: scales that make .5 ties common (0.5, 0.25), zero,
    negative and tiny scales, scales at and beyond the one-add path's range
    (per 16-channel group), large biases, and ReLU6 ceilings of 0 and 127."""
    rng = np.random.default_rng(77 + k + q6)
    c_in, c_out = 32, 64
    desc, x, wt, b, M, D = conv_case(rng, 2, 12, 12, c_in, c_out, k=k, epilogue=epi, x_range=(-128, 127))
    M = M.copy()
    M[0:8] = np.float32(0.5)
    M[8:16] = np.float32(0.25)
    M[16:18] = np.float32(0.0)
    M[18:20] = np.float32(-0.3)
    M[20:24] = np.float32(1e-7)
    M[32:48] = np.float32(3.0)     # a whole 16-channel group beyond the one-add range for k = 3
    M[48:52] = np.float32(0.05)
    b = b.copy()
    b[52:56] = 1_500_000
    b[56:60] = -1_500_000
    desc.q6 = q6
    for be_ in (be_umma, be_direct):
        _check_conv(be_, (desc, x, wt, b, M, D))


@pytest.mark.parametrize("epi,q6", [(dw.EPI_RELU, 127), (dw.EPI_RELU6, 6)])
def test_conv_relu_accumulators_beyond_2_22(be_umma, epi, q6):
    """ReLU / ReLU6 where the shape's accumulator bound is above 2^22, so the
    one-add path checks each 16 accumulators (+ bias) at run time: saturated
    pixels and weights put |acc + bias| above 2^22 (up to 9.3e6) in some
    16-channel groups and rows, small values in the rest, so the two paths
    meet inside one tile; scales small enough for the one-add path, and some
    that are not (0.5)."""
    rng = np.random.default_rng(4122 + q6)
    n, h, w, c_in, c_out = 2, 20, 24, 64, 64
    desc, x, wt, b, M, D = conv_case(rng, n, h, w, c_in, c_out, k=3, epilogue=epi, x_range=(-20, 20))
    x = x.reshape(n, h, w, c_in)
    x[0, 4:12, :, :] = 127          # a band of saturated pixels in image 0
    x[1, :, 10:14, :] = -128        # and a column band in image 1
    x = x.reshape(-1)
    wt = wt.reshape(3, 3, c_in, c_out)
    wt[..., 0:16] = 127             # group 0: |acc| up to 9 * 64 * 127 * 128 on the bands
    wt[..., 16:20] = -127
    wt = wt.reshape(-1)
    M = M.copy()
    M[0:16] = np.float32(1.3e-5)
    M[16:20] = np.float32(-2.1e-5)
    M[20:24] = np.float32(0.5)
    b = b.copy()
    b[24:28] = 4_000_000            # bias alone near 2^22 for a group of the small-valued channels
    b[28:32] = -4_000_000
    desc.q6 = q6
    _check_conv(be_umma, (desc, x, wt, b, M, D))


@pytest.mark.parametrize("c_in,k,s", [(64, 1, 1), (32, 3, 1), (3, 3, 2)])
def test_silu_stress_full_range(be, be_direct, c_in, k, s):
    """SiLU over y in about [-20, 20] with t = silu(y)/s_out spanning the whole
    int8 range (many outputs near rounding boundaries): the certified fast path
    plus exact fallback must equal the oracle (shared exact exp) bit for bit,
    on the tensor-core, small-c_in and generic direct kernels."""
    rng = np.random.default_rng(77 + c_in + k)
    n, h, w, c_out = 2, 48, 48, 64
    desc, x, wt, b, M, D = conv_case(rng, n, h, w, c_in, c_out, k=k, s=s, epilogue=dw.EPI_SILU, x_range=(-128, 127))
    acc_scale = np.sqrt(k * k * c_in) * 74.0 * 73.0
    D = (rng.uniform(5.0, 20.0, c_out) / acc_scale).astype(np.float32)
    s_out = np.float32(0.0932)
    desc.inv_s_out = float(np.float32(1.0) / s_out)
    for b_ in (be, be_direct):
        _check_conv(b_, (desc, x, wt, b, M, D))


@pytest.mark.parametrize("mult,c,epi", [(1, 576, dw.EPI_RELU6), (1, 32, dw.EPI_RELU), (2, 8, dw.EPI_NONE),
                                         (1, 24, dw.EPI_SILU)])
def test_depthwise_parity(be, mult, c, epi):
    rng = np.random.default_rng(c + mult)
    case = conv_case(rng, 2, 14, 14, c, c * mult, k=3, s=1, group=c, epilogue=epi)
    _check_conv(be, case)
    case = conv_case(rng, 1, 15, 15, c, c * mult, k=3, s=2, group=c, epilogue=epi)
    _check_conv(be, case)


@pytest.mark.parametrize("shape", [(2, 57, 30, 576, (1, 1, 1, 1)), (1, 29, 9, 8, (1, 1, 1, 1)),
                                   (1, 31, 13, 12, (0, 2, 1, 0)), (3, 112, 7, 4, (1, 1, 1, 1)),
                                   (2, 30, 27, 128, (0, 2, 1, 0)), (1, 60, 120, 64, (1, 1, 1, 1))],
                         ids=lambda s: f"{s[0]}x{s[1]}x{s[2]}x{s[3]}p{''.join(map(str, s[4]))}")
@pytest.mark.parametrize("epi", [dw.EPI_RELU6, dw.EPI_SILU, dw.EPI_NONE])
def test_depthwise_s1_segments_and_edges(be, be_direct, be_dwv, shape, epi):
    """Stride-1 depthwise over row segments and column strips: heights that
    are not multiples of the segment, widths not multiples of 4, asymmetric
    pads; bit-exact against the oracle on the default path, the register-fed
    kernel (DW_PATH_DIRECT) and each TMA-fed variant (64-channel slabs; the
    persistent whole-pixel streaming kernel with 2 or 4 columns per thread)."""
    n, h, w, c, pads = shape
    rng = np.random.default_rng(h * w + c + epi)
    case = conv_case(rng, n, h, w, c, c, k=3, s=1, pads=pads, group=c, epilogue=epi)
    _check_conv(be, case)
    _check_conv(be_direct, case)
    _check_conv(be_dwv, case)


@pytest.mark.parametrize("shape", [(5, 9, 9, 64), (7, 3, 5, 16), (2, 112, 112, 32), (4, 14, 14, 960),
                                   (3, 7, 7, 160), (2, 28, 28, 144), (1, 56, 56, 96), (9, 1, 12, 48),
                                   (3, 112, 112, 576), (4, 200, 56, 160)],
                         ids=lambda s: "x".join(map(str, s)))
@pytest.mark.parametrize("epi", [dw.EPI_RELU6, dw.EPI_RELU, dw.EPI_NONE])
def test_depthwise_stream_shapes(be_dwv, shape, epi):
    """MobileNet-style channel counts (16 .. 960: one or several channel groups
    per lane), small maps where one CTA's row range crosses several images,
    a one-row image, and sizes where spare SMs take the lanes' last rows (one
    such CTA spanning several lanes); bit-exact on every variant."""
    n, h, w, c = shape
    rng = np.random.default_rng(n * h * w + c + 7 * epi)
    case = conv_case(rng, n, h, w, c, c, k=3, s=1, group=c, epilogue=epi)
    _check_conv(be_dwv, case)


@pytest.mark.parametrize("epi", [dw.EPI_RELU6, dw.EPI_RELU, dw.EPI_NONE])
def test_depthwise_requant_ties_and_slow_channels(be, be_dwv, epi):
    """Requantisation edge cases of the depthwise kernels: M = 1/8 and 1/4
    (every fourth / second odd accumulator lands exactly on a .5 tie), channels
    whose |M| or bias leave the fast range (exact per-element path), a zero
    and a negative M, large negative biases (results clamp at the bounds), and
    a ReLU6 ceiling of 0."""
    c = 64
    rng = np.random.default_rng(4242 + epi)
    desc, x, wt, b, M, D = conv_case(rng, 3, 17, 23, c, c, k=3, s=1, group=c, epilogue=epi, x_range=(-128, 127))
    M = M.copy()
    M[0:16] = np.float32(0.125)
    M[16:24] = np.float32(0.25)
    M[24] = np.float32(1.0)        # |M| * max|acc| beyond the fast range
    M[25] = np.float32(0.0)
    M[26] = np.float32(-0.01)
    M[27] = np.float32(3.0e-5)
    b = b.copy()
    b[28] = 3_000_000              # |bias| >= 2^21: exact path
    b[29] = -2_500_000
    b[30:34] = -60_000
    b[34:38] = 60_000
    for q6 in (desc.q6, 0):
        desc.q6 = q6
        _check_conv(be, (desc, x, wt, b, M, D))
        _check_conv(be_dwv, (desc, x, wt, b, M, D))


@pytest.mark.parametrize("geo", [(2, 64, 48, 3, 3, 3, 2, 2, 1, 1, 32), (1, 17, 9, 3, 3, 3, 1, 1, 1, 1, 32),
                                 (1, 20, 20, 5, 2, 3, 2, 1, 0, 1, 32), (1, 30, 30, 3, 7, 3, 2, 2, 3, 3, 64),
                                 # the row-staged stem kernel (width a multiple of 16): no padding, odd height,
                                 # stride 1, the YOLOv8n stem
                                 (1, 16, 32, 3, 3, 3, 2, 2, 0, 0, 32), (3, 33, 32, 3, 3, 3, 2, 2, 1, 1, 32),
                                 (1, 18, 16, 3, 3, 3, 1, 1, 1, 1, 32), (2, 640, 640, 3, 3, 3, 2, 2, 1, 1, 32)])
def test_im2col_u8_to_i8(be, geo):
    """Quantise + im2col of a uint8 image (the input conv's device lowering) is
    bit-exact against quantize_u8_to_i8 followed by the gather."""
    from oracle.graph_ref import im2col_u8_op
    n, h, w, c, kh, kw, sh, sw, pt, pl, cd = geo
    ho, wo = (h + 2 * pt - kh) // sh + 1, (w + 2 * pl - kw) // sw + 1
    rng = np.random.default_rng(sum(geo))
    x = rng.integers(0, 256, n * h * w * c).astype(np.uint8)
    bx, by = be.upload_array(x), be.alloc(n * ho * wo * cd)
    ops.im2col_u8_to_i8(be, bx, by, n, h, w, c, kh, kw, sh, sw, pt, pl, ho, wo, cd, 1.0 / 127.0)
    got = be.download_array(by, np.int8)

    class _Op:
        params = {"k_h": kh, "k_w": kw, "s_h": sh, "s_w": sw, "p_t": pt, "p_l": pl, "h_out": ho, "w_out": wo,
                  "c_dst": cd, "scale": 1.0 / 127.0}
    exp = im2col_u8_op(_Op, x.reshape(n, h, w, c)).ravel()
    assert np.array_equal(got, exp), mismatch_report(got, exp)


def test_reference_shim_exact_signature(be):
    """conv2d_requant_relu_i8_packed with the reference parameter list (scalar scale,
    no bias, HWIO kernel) == reference composition conv -> requantize -> relu."""
    rng = np.random.default_rng(77)
    for (n, h, w, ci, co, k, s, p, relu) in [(1, 32, 32, 16, 16, 3, 1, 1, True), (1, 16, 16, 64, 64, 3, 1, 1, True),
                                             (1, 32, 32, 32, 32, 3, 1, 1, False), (2, 9, 9, 4, 8, 3, 2, 0, True)]:
        x = rng.integers(-64, 64, n * h * w * ci).astype(np.int8)
        wt = rng.integers(-127, 128, k * k * ci * co).astype(np.int8)
        ho, wo = (h + 2 * p - k) // s + 1, (w + 2 * p - k) // s + 1
        bx, bw, by = be.upload_array(x), be.upload_array(wt), be.alloc(n * ho * wo * co)
        ops.conv2d_requant_relu_i8_packed(be, bx, bw, by, n, h, w, ci, co, k, k, s, s, p, p, 0.001, relu)
        acc = dwref.conv2d_i8_nhwc(x, wt, n, h, w, ci, co, k, k, s, s, p, p)
        ref = dwref.requantize_i32_to_i8(acc, 0.001)
        if relu:
            ref = dwref.relu_i8(ref)
        assert np.array_equal(be.download_array(by, np.int8), ref)


def test_unfused_conv_i32(be):
    rng = np.random.default_rng(8)
    n, h, w, ci, co = 2, 10, 9, 12, 20
    x = rng.integers(-128, 128, n * h * w * ci).astype(np.int8)
    wt = rng.integers(-128, 128, 9 * ci * co).astype(np.int8)
    bx, bw, bo = be.upload_array(x), be.upload_array(wt), be.alloc(4 * n * h * w * co)
    ops.conv2d_i8_nhwc_packed(be, bx, bw, bo, n, h, w, ci, co, 3, 3, 1, 1, 1, 1)
    assert np.array_equal(be.download_array(bo, np.int32), dwref.conv2d_i8_nhwc(x, wt, n, h, w, ci, co, 3, 3, 1, 1, 1, 1))


# ---------------------------------------------------------------- QGemm

@pytest.mark.parametrize("m,n,k,epi", [(128, 128, 128, dw.EPI_NONE), (200, 80, 96, dw.EPI_RELU),
                                       (256, 512, 1024, dw.EPI_RELU6), (1000, 48, 64, dw.EPI_NONE)])
def test_qgemm_parity(be, m, n, k, epi):
    rng = np.random.default_rng(m * n + k)
    a = rng.integers(-127, 128, m * k).astype(np.int8)
    b = rng.integers(-127, 128, k * n).astype(np.int8)
    bias = rng.integers(-1000, 1001, n).astype(np.int32)
    M = (rng.uniform(0.001, 0.01, n) * np.float32(0.004) / np.float32(0.05)).astype(np.float32)
    ba, bb = be.upload_array(a), be.upload_array(b)
    bp = ops.prepare_gemm_b_i8(be, bb, k, n)
    y = be.alloc(m * n)
    ops.qgemm_i8(be, ba, bp, be.upload_array(bias), be.upload_array(M), y, m, n, k, epi, 100)
    ref = dwref.qgemm_i8(a, b, bias, M, m, n, k, epi, 100, threads=8)
    got = be.download_array(y, np.int8)
    assert np.array_equal(got, ref), mismatch_report(got, ref)


def test_gemm_i8_i32_random(be):
    rng = np.random.default_rng(4)
    m, n, k = 37, 29, 45
    a = rng.integers(-128, 128, m * k).astype(np.int8)
    b = rng.integers(-128, 128, k * n).astype(np.int8)
    c = be.alloc(4 * m * n)
    ops.gemm_i8_packed(be, be.upload_array(a), be.upload_array(b), c, m, n, k)
    assert np.array_equal(be.download_array(c, np.int32), dwref.gemm_i8(a, b, m, n, k))


# ---------------------------------------------------------------- glue

def test_maxpool_concat_resize_slice(be):
    rng = np.random.default_rng(12)
    n, h, w, c = 2, 20, 20, 64
    x = rng.integers(-128, 128, n * h * w * c).astype(np.int8)
    bx = be.upload_array(x)
    by = be.alloc(x.size)
    ops.maxpool_i8(be, bx, by, n, h, w, c, 5, 5, 1, 1, (2, 2, 2, 2))  # SPPF
    assert np.array_equal(be.download_array(by, np.int8), dwref.maxpool_i8(x, n, h, w, c, 5, 5, 1, 1, (2, 2, 2, 2)))
    x3 = rng.integers(-128, 128, n * 11 * 13 * 5).astype(np.int8)
    b3 = be.upload_array(x3)
    y3 = be.alloc(n * 5 * 6 * 5)
    ops.maxpool_i8(be, b3, y3, n, 11, 13, 5, 3, 3, 2, 2, (0, 0, 0, 0))
    assert np.array_equal(be.download_array(y3, np.int8), dwref.maxpool_i8(x3, n, 11, 13, 5, 3, 3, 2, 2))
    parts = [rng.integers(-128, 128, 400 * cc).astype(np.int8) for cc in (64, 32, 16, 8)]
    bufs = [be.upload_array(p) for p in parts]
    yc = be.alloc(400 * 120)
    ops.concat_i8(be, bufs, [64, 32, 16, 8], 400, yc)
    assert np.array_equal(be.download_array(yc, np.int8), dwref.concat_c_i8(parts, [64, 32, 16, 8], 400))
    ys = be.alloc(400 * 16)
    ops.slice_c_i8(be, yc, ys, 400, 120, 96, 16)
    assert np.array_equal(be.download_array(ys, np.int8).reshape(400, 16),
                          dwref.concat_c_i8(parts, [64, 32, 16, 8], 400).reshape(400, 120)[:, 96:112])
    yr = be.alloc(n * 40 * 40 * c)
    ops.resize_nearest_i8(be, bx, yr, n, 20, 20, 40, 40, c)
    assert np.array_equal(be.download_array(yr, np.int8), dwref.resize_nearest_i8(x, n, 20, 20, 40, 40, c))
    yr2 = be.alloc(n * 7 * 9 * c)
    ops.resize_nearest_i8(be, bx, yr2, n, 20, 20, 7, 9, c)
    assert np.array_equal(be.download_array(yr2, np.int8), dwref.resize_nearest_i8(x, n, 20, 20, 7, 9, c))


# ---------------------------------------------------------------- errors

def test_error_strings_and_no_truncation(be):
    b4 = be.alloc(4)
    with pytest.raises(dw.BackendError) as ei:
        be.upload(b4, np.zeros(5, np.uint8))
    assert ei.value.status == 2 and "length mismatch" in ei.value.message
    with pytest.raises(dw.BackendError):
        be.alloc(0)
    x = be.alloc(1 * 8 * 8 * 6)
    w = be.alloc(9 * 6 * 8)
    y = be.alloc(8 * 8 * 8)
    with pytest.raises(dw.BackendError) as ei:  # vulkan/src/ops.rs:2313-2317
        ops.conv2d_requant_relu_i8_packed(be, x, w, y, 1, 8, 8, 6, 8, 3, 3, 1, 1, 1, 1, 0.01, True)
    assert "conv_fused: c_in=6 must be multiple of 4" in ei.value.message
    x = be.alloc(1 * 8 * 8 * 8)
    w = be.alloc(9 * 8 * 8)
    with pytest.raises(dw.BackendError) as ei:
        ops.conv2d_requant_relu_i8_packed(be, x, w, be.alloc(10), 1, 8, 8, 8, 8, 3, 3, 1, 1, 1, 1, 0.01, True)
    assert "conv_fused: output mismatch: expected 512, got 10" in ei.value.message
    be.synchronize(5000)


def test_bounded_wait_expiry_reports_and_recovers(be):
    """A device wait on a flag nothing sets gives up after its cap; the host
    sees DW_ERR_KERNEL_WAIT_EXPIRED and the context stays usable."""
    be.synchronize(5000)
    assert dw._lib.load().dw_debug_expire_wait(be.handle, 2000) == 0
    with pytest.raises(dw.BackendError) as ei:
        be.synchronize(10000)
    assert ei.value.status == dw._lib.DW_ERR_KERNEL_WAIT_EXPIRED
    be.synchronize(5000)  # error word cleared
    test_kat_gemm_i8(be)
