"""GPU parity of the fp16 path through the C ABI against the CPU oracle.

Bit-exact: the F16 conversions (all 65536 halves; random and special f32),
add / add+ReLU / ReLU / max pool / global average pool, the direct and
depthwise convolutions (same f32 FMA order as ops.rs:1442-1511, 2819-2937).

Tolerance (the tensor-core conv/GEMM sum in another order): per layer, fed
identical inputs, max |gpu - cpu| <= 5e-3 * max |cpu| and a relative L2 error
<= 1e-3; whole-network logits within 5e-2 of max |logit|.  The ULP histogram
is printed: both sides round an f32 sum to f16, and the CPU's sequential f32
sum carries its own error (about sqrt(K) * 2^-24 of the sum of |terms|), so
outputs that cancel to small values can sit several f16 ulps apart."""
import numpy as np
import pytest

import dragonwing_edge_rs_b200 as dw
from dragonwing_edge_rs_b200 import graph as G
from dragonwing_edge_rs_b200 import ops
from dragonwing_edge_rs_b200.backend import BackendError
from dragonwing_edge_rs_b200.ops import ConvDesc
from oracle import dwref
from oracle.graph_ref import conv_f16_op, gemm_f16_op, run_graph, unfold_f16_op

pytestmark = pytest.mark.gpu

LAYER_REL_TOL = 5e-3      # docs/parity-testing.md:120 (per layer, relative)
LOGITS_REL_TOL = 5e-2     # docs/parity-testing.md:138 (network output, relative)
LAYER_REL_L2_TOL = 1e-3


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


@pytest.fixture(scope="module")
def be_umma():
    b = dw.CudaBackend(0, conv_path=dw.PATH_UMMA)
    yield b
    b.close()


def h16(rng, size, scale=1.0):
    """Random f16 bit patterns of normal(0, scale) values."""
    return (rng.standard_normal(size) * scale).astype(np.float16).view(np.uint16)


def ordered(bits):
    b = bits.astype(np.int32)
    return np.where(b & 0x8000, -(b & 0x7FFF), b)


def ulp_diff(a, b):
    return np.abs(ordered(a) - ordered(b))


def bits_report(got, exp):
    bad = np.nonzero(got != exp)[0]
    if bad.size == 0:
        return "ok"
    i = bad[0]
    return f"{bad.size}/{got.size} differ; first at {i}: got {got[i]:#06x} expected {exp[i]:#06x}"


def tol_check(got, exp, what):
    g = got.view(np.float16).astype(np.float64)
    e = exp.view(np.float16).astype(np.float64)
    scale = np.abs(e).max()
    err = np.abs(g - e).max()
    l2 = np.linalg.norm(g - e) / max(np.linalg.norm(e), 1e-30)
    u = ulp_diff(got, exp)
    hist = [float(np.mean(u == 0)), float(np.mean(u == 1)), float(np.mean(u == 2)), float(np.mean(u > 2))]
    msg = (f"{what}: max|d|={err:.3g} max|ref|={scale:.3g} rel={err / max(scale, 1e-30):.3g} relL2={l2:.3g} "
           f"ulp 0/1/2/>2 = {hist[0]:.4f}/{hist[1]:.4f}/{hist[2]:.4f}/{hist[3]:.4f}")
    assert np.isfinite(g).all() and err <= LAYER_REL_TOL * scale, msg
    assert l2 <= LAYER_REL_L2_TOL, msg
    return msg


def run_conv_f16(be, desc, x, w_hwio, bias):
    bx, bw = be.upload_array(x), be.upload_array(w_hwio)
    wp = ops.prepare_weights_f16(be, desc, bw)
    bb = be.upload_array(bias) if bias is not None else None
    ho, wo = desc.out_hw()
    by = be.alloc(2 * desc.n * ho * wo * desc.c_out)
    ops.conv2d_f16(be, desc, bx, wp, bb, by)
    y = be.download_array(by, np.uint16)
    be.synchronize(timeout_ms=20000)
    return y


def oracle_conv_f16(desc, x, w_hwio, bias, threads=8):
    pt, pl, pb, pr = desc.pads
    relu = desc.epilogue == dw.EPI_RELU
    if desc.group == 1:
        return dwref.conv2d_f16(x, w_hwio, bias, relu, desc.n, desc.h, desc.w, desc.c_in, desc.c_out, desc.k_h,
                                desc.k_w, desc.stride_h, desc.stride_w, pt, pl, threads)
    return dwref.dwconv_f16(x, w_hwio, relu, desc.n, desc.h, desc.w, desc.c_in, desc.c_out // desc.c_in, desc.k_h,
                            desc.k_w, desc.stride_h, desc.stride_w, pt, pl, threads, bias=bias)


def conv_inputs(rng, desc):
    x = h16(rng, desc.n * desc.h * desc.w * desc.c_in)
    fan = desc.k_h * desc.k_w * (desc.c_in if desc.group == 1 else 1)
    wn = desc.k_h * desc.k_w * (desc.c_in * desc.c_out if desc.group == 1 else desc.c_out)
    w = h16(rng, wn, np.sqrt(2.0 / fan))
    b = h16(rng, desc.c_out, 0.1)
    return x, w, b


# ------------------------------------------------------------- conversions

def test_f16_to_f32_all_halves_bit_exact(be):
    allh = np.arange(65536, dtype=np.uint16)
    bx = be.upload_array(allh)
    by = be.alloc(4 * 65536)
    ops.cast_f16_to_f32(be, bx, by)
    got = be.download_array(by, np.uint32)
    exp = dwref.f16_to_f32_array(allh).view(np.uint32)
    assert np.array_equal(got, exp), f"{np.count_nonzero(got != exp)} halves convert differently"
    # the reference's subnormal defect is reproduced: 0x0001 -> 2^-25
    assert got[1] == np.float32(2.0 ** -25).view(np.uint32)


def test_f32_to_f16_random_and_special_bit_exact(be):
    rng = np.random.default_rng(3)
    bits = rng.integers(0, 2 ** 32, 1 << 20, dtype=np.uint64).astype(np.uint32)
    special = np.array([0.0, -0.0, np.inf, -np.inf, 65504.0, 65519.99, 65520.0, 2.0 ** -24, 2.0 ** -25,
                        2.0 ** -25 * 1.0000001, 2.0 ** -26, 6.1e-5, 1e-8, -1e-8], np.float32).view(np.uint32)
    nans = np.array([0x7FC00000, 0xFFC00001, 0x7F800001, 0x7FBFFFFF, 0x7FFFFFFF], np.uint32)
    x = np.concatenate([bits, special, nans]).view(np.float32)
    bx = be.upload_array(x)
    by = be.alloc(2 * x.size)
    ops.cast_f32_to_f16(be, bx, by, x.size, 1)
    got = be.download_array(by, np.uint16)
    exp = dwref.f16_from_f32_array(x)
    assert np.array_equal(got, exp), bits_report(got, exp)


def test_cast_pads_channels_with_zero(be):
    rng = np.random.default_rng(4)
    x = rng.standard_normal((5, 3)).astype(np.float32)
    bx = be.upload_array(x)
    by = be.alloc(2 * 5 * 16)
    ops.cast_f32_to_f16(be, bx, by, 5, 3, 16)
    got = be.download_array(by, np.uint16).reshape(5, 16)
    assert np.array_equal(got[:, :3], dwref.f16_from_f32_array(x).reshape(5, 3))
    assert not got[:, 3:].any()


@pytest.mark.parametrize("geo", [(2, 224, 224, 3, 7, 2, 3, 112, 32), (1, 9, 13, 3, 3, 1, 1, 13, 16),
                                 (1, 8, 10, 5, 2, 2, 0, 5, 16)])
def test_unfold_w_f32_to_f16(be, geo):
    n, h, w, c, kw, sw, pl, wo, cd = geo
    rng = np.random.default_rng(sum(geo))
    x = rng.standard_normal((n, h, w, c)).astype(np.float32)
    bx, by = be.upload_array(x), be.alloc(2 * n * h * wo * cd)
    ops.unfold_w_f32_to_f16(be, bx, by, n, h, w, c, kw, sw, pl, wo, cd)
    got = be.download_array(by, np.uint16)

    class _Op:
        params = {"k_w": kw, "stride_w": sw, "pad_l": pl, "w_out": wo, "c_dst": cd}
    exp = unfold_f16_op(_Op, x).ravel()
    assert np.array_equal(got, exp), bits_report(got, exp)


# ------------------------------------------------------------- glue (bit-exact)

def glue_data(rng, n):
    """Normal values, some subnormals and infinities (no NaN: a NaN sum's payload
    depends on the CPU's operand order)."""
    v = h16(rng, n, 4.0)
    idx = rng.choice(n, n // 50, replace=False)
    v[idx[: len(idx) // 2]] = rng.integers(1, 0x400, len(idx) // 2).astype(np.uint16) | \
        (rng.integers(0, 2, len(idx) // 2).astype(np.uint16) << 15)
    v[idx[len(idx) // 2:]] = np.where(rng.integers(0, 2, len(idx) - len(idx) // 2), 0x7C00, 0xFC00)
    return v


@pytest.mark.parametrize("n", [1, 7, 8, 4099, 1 << 20])
def test_add_and_add_relu_f16(be, n):
    rng = np.random.default_rng(n)
    a, b = glue_data(rng, n), glue_data(rng, n)
    ba, bb, by = be.upload_array(a), be.upload_array(b), be.alloc(2 * n)
    ops.add_fp16(be, ba, bb, by)
    got = be.download_array(by, np.uint16)
    exp = dwref.add_f16(a, b)
    ok = (got == exp) | ((got & 0x7C00 == 0x7C00) & (got & 0x3FF != 0) & (exp & 0x7C00 == 0x7C00) & (exp & 0x3FF != 0))
    assert ok.all(), bits_report(got, exp)  # inf - inf: both NaN
    ops.add_relu_fp16(be, ba, bb, by)
    got = be.download_array(by, np.uint16)
    exp = dwref.relu_f16(dwref.add_f16(a, b))
    assert np.array_equal(got, exp), bits_report(got, exp)


def test_relu_f16_in_place_including_nan(be):
    rng = np.random.default_rng(11)
    x = glue_data(rng, 10007)
    x[:5] = [0x7E00, 0xFE01, 0x0001, 0x8001, 0x0000]
    bx = be.upload_array(x)
    ops.relu_fp16(be, bx)
    got = be.download_array(bx, np.uint16)
    exp = dwref.relu_f16(x)
    assert np.array_equal(got, exp), bits_report(got, exp)


def test_relu_f16_unaligned_view(be):
    """A buffer view that is not 16-byte aligned takes the scalar path."""
    rng = np.random.default_rng(12)
    x = glue_data(rng, 1001)
    big = be.upload_array(np.concatenate([np.zeros(1, np.uint16), x]))
    view = be.wrap(big.device_ptr + 2, 2 * x.size)
    ops.relu_fp16(be, view)
    got = be.download_array(big, np.uint16)[1:]
    assert np.array_equal(got, dwref.relu_f16(x))


@pytest.mark.parametrize("shape,k,s,pad", [((2, 112, 112, 64), 3, 2, 1), ((1, 13, 11, 5), 3, 1, 1),
                                           ((3, 20, 20, 16), 5, 1, 2), ((1, 9, 9, 8), 2, 2, 0)])
def test_maxpool_f16(be, shape, k, s, pad):
    rng = np.random.default_rng(sum(shape))
    n, h, w, c = shape
    x = glue_data(rng, n * h * w * c)
    x[::97] = 0x7E00  # NaN taps are skipped by max
    ho, wo = (h + 2 * pad - k) // s + 1, (w + 2 * pad - k) // s + 1
    bx, by = be.upload_array(x), be.alloc(2 * n * ho * wo * c)
    ops.maxpool_f16(be, bx, by, n, h, w, c, k, k, s, s, (pad,) * 4)
    got = be.download_array(by, np.uint16)
    exp = dwref.maxpool_f16(x, n, h, w, c, k, k, s, s, (pad,) * 4)
    assert np.array_equal(got, exp), bits_report(got, exp)


@pytest.mark.parametrize("shape", [(4, 7, 7, 2048), (1, 1, 1, 8), (3, 5, 9, 33)])
def test_global_avgpool_f16(be, shape):
    rng = np.random.default_rng(sum(shape))
    n, h, w, c = shape
    x = h16(rng, n * h * w * c, 3.0)
    bx, by = be.upload_array(x), be.alloc(2 * n * c)
    ops.global_avgpool_f16(be, bx, by, n, h, w, c)
    got = be.download_array(by, np.uint16)
    exp = dwref.gap_f16(x, n, h, w, c)
    assert np.array_equal(got, exp), bits_report(got, exp)


# ------------------------------------------------------------- convolutions

DIRECT_CASES = [
    # n, h, w, c_in, c_out, k, s, pad, relu
    (1, 16, 16, 3, 64, 7, 2, 3, True),
    (2, 9, 7, 8, 24, 3, 1, 1, False),
    (1, 12, 12, 16, 16, 1, 2, 0, True),
    (1, 5, 6, 5, 7, 3, 2, 1, True),
]


@pytest.mark.parametrize("case", DIRECT_CASES)
def test_conv_f16_direct_bit_exact(be_direct, case):
    n, h, w, ci, co, k, s, p, relu = case
    rng = np.random.default_rng(sum(case))
    desc = ConvDesc(n, h, w, ci, co, k, k, s, s, (p,) * 4, 1, dw.EPI_RELU if relu else dw.EPI_NONE)
    x, wt, b = conv_inputs(rng, desc)
    got = run_conv_f16(be_direct, desc, x, wt, b)
    exp = oracle_conv_f16(desc, x, wt, b)
    assert np.array_equal(got, exp), bits_report(got, exp)


@pytest.mark.parametrize("case", [(2, 14, 14, 32, 1, 1, True), (1, 15, 17, 24, 2, 2, False),
                                  (1, 8, 8, 16, 1, 2, True)])
def test_dwconv_f16_bit_exact(be, case):
    n, h, w, c, mult, s, relu = case
    rng = np.random.default_rng(sum(case))
    desc = ConvDesc(n, h, w, c, c * mult, 3, 3, s, s, (1,) * 4, c, dw.EPI_RELU if relu else dw.EPI_NONE)
    x, wt, b = conv_inputs(rng, desc)
    got = run_conv_f16(be, desc, x, wt, b)
    exp = oracle_conv_f16(desc, x, wt, b)
    assert np.array_equal(got, exp), bits_report(got, exp)


UMMA_CASES = [
    # n, h, w, c_in, c_out, k, s, pad, relu -- ResNet-50 layer shapes (small batch) and edges
    (2, 56, 56, 64, 64, 1, 1, 0, True),
    (2, 56, 56, 64, 64, 3, 1, 1, True),
    (2, 56, 56, 64, 256, 1, 1, 0, False),
    (2, 56, 56, 256, 512, 1, 2, 0, False),
    (2, 56, 56, 128, 128, 3, 2, 1, True),
    (2, 14, 14, 1024, 256, 1, 1, 0, True),
    (2, 7, 7, 512, 2048, 1, 1, 0, False),
    (1, 64, 64, 16, 64, 7, 2, 3, True),   # the padded stem
    (1, 9, 11, 8, 24, 3, 1, 1, True),     # c_in 8, ragged tiles
    (3, 10, 10, 40, 72, 3, 1, 1, False),
    (3, 7, 7, 512, 512, 3, 1, 1, True),   # two whole 7x7 images per row block
    (3, 14, 14, 256, 512, 1, 2, 0, False),
    (5, 6, 6, 32, 64, 3, 1, 1, True),
    (2, 28, 28, 128, 128, 3, 1, 1, True),
    (2, 14, 14, 256, 256, 3, 1, 1, True),
]

# the halo producer (stride-1 multi-tap convs on maps the 8 x 16 tiles cover);
# DW_UMMA_HALO_WIDE=1 sends the wider channel rows there too
HALO_CASES = [
    (2, 28, 28, 128, 128, 3, 1, 1, True),
    (2, 14, 14, 256, 256, 3, 1, 1, True),  # channel tiles of 128
    (1, 40, 24, 32, 48, 3, 1, 1, False),
    (1, 30, 36, 16, 32, 5, 1, 2, True),
    (2, 56, 56, 64, 64, 3, 1, 1, True),
]


@pytest.mark.parametrize("case", HALO_CASES)
def test_conv_f16_halo_within_tolerance(be_umma, case, monkeypatch):
    monkeypatch.setenv("DW_UMMA_HALO_WIDE", "1")
    monkeypatch.setenv("DW_UMMA_HALO_ANY_SIZE", "1")
    n, h, w, ci, co, k, s, p, relu = case
    rng = np.random.default_rng(sum(case) + 2)
    desc = ConvDesc(n, h, w, ci, co, k, k, s, s, (p,) * 4, 1, dw.EPI_RELU if relu else dw.EPI_NONE)
    x, wt, b = conv_inputs(rng, desc)
    got = run_conv_f16(be_umma, desc, x, wt, b)
    exp = oracle_conv_f16(desc, x, wt, b)
    print(tol_check(got, exp, str(case)))


@pytest.mark.parametrize("case", UMMA_CASES)
def test_conv_f16_tensor_core_within_tolerance(be_umma, case):
    n, h, w, ci, co, k, s, p, relu = case
    rng = np.random.default_rng(sum(case) + 1)
    desc = ConvDesc(n, h, w, ci, co, k, k, s, s, (p,) * 4, 1, dw.EPI_RELU if relu else dw.EPI_NONE)
    x, wt, b = conv_inputs(rng, desc)
    got = run_conv_f16(be_umma, desc, x, wt, b)
    exp = oracle_conv_f16(desc, x, wt, b)
    print(tol_check(got, exp, str(case)))


def test_conv_f16_inf_input_stays_local(be_umma):
    """A strided conv reads no other column phase: an infinity in one pixel
    reaches only the outputs whose windows hold it (no NaN elsewhere)."""
    desc = ConvDesc(1, 16, 16, 16, 32, 3, 3, 2, 2, (1,) * 4, 1, dw.EPI_NONE)
    rng = np.random.default_rng(21)
    x, wt, b = conv_inputs(rng, desc)
    x = x.reshape(16, 16, 16)
    x[5, 5, 3] = 0x7C00
    got = run_conv_f16(be_umma, desc, x.ravel(), wt, b).reshape(8, 8, 32)
    exp = oracle_conv_f16(desc, x.ravel(), wt, b).reshape(8, 8, 32)
    nonfinite_got = (got & 0x7C00) == 0x7C00
    nonfinite_exp = (exp & 0x7C00) == 0x7C00
    assert np.array_equal(nonfinite_got.any(axis=2), nonfinite_exp.any(axis=2))


def test_conv_f16_halo_inf_input_stays_local(be_umma, monkeypatch):
    """Halo mode (stride 1, 3x3): an infinity in one pixel reaches only the
    outputs whose windows hold it; the zero-filled halo and the shifted tap
    reads touch no other pixel."""
    monkeypatch.setenv("DW_UMMA_HALO_WIDE", "1")
    monkeypatch.setenv("DW_UMMA_HALO_ANY_SIZE", "1")
    desc = ConvDesc(1, 32, 32, 32, 16, 3, 3, 1, 1, (1,) * 4, 1, dw.EPI_NONE)
    rng = np.random.default_rng(22)
    x, wt, b = conv_inputs(rng, desc)
    x = x.reshape(32, 32, 32)
    x[9, 13, 5] = 0x7C00
    got = run_conv_f16(be_umma, desc, x.ravel(), wt, b).reshape(32, 32, 16)
    exp = oracle_conv_f16(desc, x.ravel(), wt, b).reshape(32, 32, 16)
    nonfinite_got = (got & 0x7C00) == 0x7C00
    nonfinite_exp = (exp & 0x7C00) == 0x7C00
    assert np.array_equal(nonfinite_got.any(axis=2), nonfinite_exp.any(axis=2))
    assert nonfinite_got.any(axis=2).sum() <= 9


@pytest.mark.parametrize("case", [(2, 28, 28, 64, 256, 1, 1, 0, True), (2, 28, 28, 64, 256, 1, 1, 0, False),
                                  (1, 28, 28, 64, 128, 1, 2, 0, True), (1, 14, 14, 32, 32, 3, 1, 1, True)])
def test_conv_add_f16_equals_conv_then_add(be, case):
    """The fused residual epilogue gives the same bits as conv2d_f16 (no ReLU)
    followed by add_fp16 (+relu_fp16)."""
    n, h, w, ci, co, k, s, p, relu = case
    rng = np.random.default_rng(sum(case) + 7)
    desc = ConvDesc(n, h, w, ci, co, k, k, s, s, (p,) * 4, 1, dw.EPI_RELU if relu else dw.EPI_NONE)
    x, wt, b = conv_inputs(rng, desc)
    ho, wo = desc.out_hw()
    r = h16(rng, n * ho * wo * co, 2.0)
    bx, bw, bb, br = be.upload_array(x), be.upload_array(wt), be.upload_array(b), be.upload_array(r)
    wp = ops.prepare_weights_f16(be, desc, bw)
    by = be.alloc(2 * n * ho * wo * co)
    ops.conv2d_add_f16(be, desc, bx, wp, bb, br, by)
    fused = be.download_array(by, np.uint16)
    d0 = ConvDesc(n, h, w, ci, co, k, k, s, s, (p,) * 4, 1, dw.EPI_NONE)
    tmp = be.alloc(2 * n * ho * wo * co)
    ops.conv2d_f16(be, d0, bx, wp, bb, tmp)
    (ops.add_relu_fp16 if relu else ops.add_fp16)(be, tmp, br, by)
    two = be.download_array(by, np.uint16)
    assert np.array_equal(fused, two), bits_report(fused, two)
    conv = be.download_array(tmp, np.uint16)
    exp = dwref.add_f16(conv, r)
    exp = dwref.relu_f16(exp) if relu else exp
    assert np.array_equal(fused, exp), bits_report(fused, exp)


@pytest.mark.parametrize("bias_kind", ["subnormal", "normal"])
@pytest.mark.parametrize("relu", [False, True])
@pytest.mark.parametrize("residual", [False, True])
def test_f16_epilogue_subnormal_operands_bit_exact(be_umma, relu, residual, bias_kind):
    """Inputs on a 2^-12 grid make every sum exact in f32 on both sides, so the
    tensor-core result must equal the CPU's bit for bit -- including outputs,
    biases and residuals that are f16 subnormals, which F16::to_f32 halves
    (the packed path scales such operands by 0.5 inside an FMA; subnormal
    biases take the exact path)."""
    rng = np.random.default_rng(40 + relu + 2 * residual + 4 * (bias_kind == "normal"))
    n, h, w, ci, co = 1, 16, 16, 16, 64
    desc = ConvDesc(n, h, w, ci, co, 1, 1, 1, 1, (0,) * 4, 1, dw.EPI_RELU if relu else dw.EPI_NONE)
    x = (rng.integers(-8, 9, n * h * w * ci) * 2.0 ** -12).astype(np.float16).view(np.uint16)
    wt = (rng.integers(-8, 9, ci * co) * 2.0 ** -12).astype(np.float16).view(np.uint16)
    b = (rng.integers(-600, 601, co) * 2.0 ** -24).astype(np.float16).view(np.uint16)
    b[::5] = (rng.standard_normal(len(b[::5])) * 1e-3).astype(np.float16).view(np.uint16)
    if bias_kind == "normal":  # normal biases of the outputs' size: the packed path handles every element
        b = (np.sign(rng.standard_normal(co)) * rng.uniform(2.0 ** -14, 2.0 ** -12, co)).astype(np.float16)
        b = b.view(np.uint16)
    bx, bw, bb = be_umma.upload_array(x), be_umma.upload_array(wt), be_umma.upload_array(b)
    wp = ops.prepare_weights_f16(be_umma, desc, bw)
    by = be_umma.alloc(2 * n * h * w * co)
    if residual:
        r = (rng.integers(-900, 901, n * h * w * co) * 2.0 ** -24).astype(np.float16).view(np.uint16)
        ops.conv2d_add_f16(be_umma, desc, bx, wp, bb, be_umma.upload_array(r), by)
        conv = dwref.conv2d_f16(x, wt, b, False, n, h, w, ci, co, 1, 1, 1, 1, 0, 0)
        exp = dwref.add_f16(conv, r)
        exp = dwref.relu_f16(exp) if relu else exp
    else:
        ops.conv2d_f16(be_umma, desc, bx, wp, bb, by)
        exp = dwref.conv2d_f16(x, wt, b, relu, n, h, w, ci, co, 1, 1, 1, 1, 0, 0)
    got = be_umma.download_array(by, np.uint16)
    pre = dwref.conv2d_f16(x, wt, None, False, n, h, w, ci, co, 1, 1, 1, 1, 0, 0)  # the conv before its bias
    sub = np.mean(((pre & 0x7C00) == 0) & ((pre & 0x3FF) != 0))
    assert sub > 0.2, f"test data should produce many subnormal conv results ({sub:.2f})"
    assert np.array_equal(got, exp), bits_report(got, exp)


def test_shim_conv2d_fp16_nhwc_matches_conv2d_f16(be):
    rng = np.random.default_rng(31)
    desc = ConvDesc(2, 28, 28, 64, 64, 3, 3, 1, 1, (1,) * 4, 1, dw.EPI_NONE)
    x, wt, _ = conv_inputs(rng, desc)
    bx, bw = be.upload_array(x), be.upload_array(wt)
    by = be.alloc(2 * 2 * 28 * 28 * 64)
    ops.conv2d_fp16_nhwc(be, bx, bw, by, 2, 28, 28, 64, 64, 3, 3, 1, 1, 1, 1)
    got = be.download_array(by, np.uint16)
    ref = run_conv_f16(be, desc, x, wt, None)
    assert np.array_equal(got, ref)


@pytest.mark.parametrize("mnk", [(128, 1000, 2048), (7, 24, 40), (256, 512, 64)])
def test_gemm_f16_within_tolerance(be, mnk):
    m, n, k = mnk
    rng = np.random.default_rng(m + n + k)
    a = h16(rng, m * k)
    b = h16(rng, k * n, np.sqrt(1.0 / k))
    ba, bb, bc = be.upload_array(a), be.upload_array(b), be.alloc(2 * m * n)
    ops.gemm_fp16(be, ba, bb, bc, m, n, k)
    got = be.download_array(bc, np.uint16)
    exp = dwref.gemm_f16(a, b, m, n, k, threads=8)
    print(tol_check(got, exp, f"gemm {mnk}"))
    bias = h16(rng, n, 0.1)
    bp = ops.prepare_gemm_b_f16(be, bb, k, n)
    bbias = be.upload_array(bias)
    ops.gemm_f16_bias(be, ba, bp, bbias, bc, m, n, k)
    got = be.download_array(bc, np.uint16)
    exp = dwref.bias_relu_f16(exp, bias, False, m, n)
    print(tol_check(got, exp, f"gemm+bias {mnk}"))


def test_f16_error_strings(be):
    a, b, c = be.alloc(2 * 6), be.alloc(2 * 6), be.alloc(2 * 4)
    with pytest.raises(BackendError, match="gemm_fp16: C size mismatch: expected 8 got 10"):
        ops.gemm_fp16(be, a, b, be.alloc(2 * 5), 2, 2, 3)
    with pytest.raises(BackendError, match="add_fp16: buffer size mismatch"):
        ops.add_fp16(be, a, b, c)
    with pytest.raises(BackendError, match="conv2d_fp16: input size mismatch: expected"):
        ops.conv2d_fp16_nhwc(be, a, b, c, 1, 4, 4, 8, 8, 3, 3, 1, 1, 1, 1)
    odd = be.alloc(3)
    with pytest.raises(BackendError, match="relu_fp16: buffer size must be multiple of 2"):
        ops.relu_fp16(be, odd)
    desc = ConvDesc(1, 8, 8, 8, 8, 3, 3, 1, 1, (1,) * 4, 1, dw.EPI_SILU)
    with pytest.raises(BackendError, match="epilogue 3 unsupported"):
        ops.conv2d_f16(be, desc, be.alloc(2 * 512), be.alloc(2 * 576), None, be.alloc(2 * 512))


# ------------------------------------------------------------- ResNet-50 graph

def _per_layer_check(g, rt):
    """Feeds each op's GPU inputs to the oracle op and compares with the GPU
    output: convs/GEMM within the layer tolerance, everything else bit-exact."""
    worst = 0.0
    for op in g.ops:
        t = op.op_type
        out = op.outputs[0]
        if t == "UnfoldF32ToF16":
            x = rt.get_output(op.inputs[0])
            got = rt.get_output(out).view(np.uint16).ravel()
            assert np.array_equal(got, unfold_f16_op(op, x).ravel()), op.name
        elif t == "Conv2dAddF16":
            x = rt.get_output(op.inputs[0]).view(np.uint16)
            r = rt.get_output(op.inputs[3]).view(np.uint16)
            got = rt.get_output(out).view(np.uint16).ravel()
            y = dwref.add_f16(conv_f16_op(g, op, x, threads=dwref.num_cpus(), relu=False).ravel(), r.ravel())
            exp = dwref.relu_f16(y) if op.params["desc"].epilogue == dw.EPI_RELU else y
            tol_check(got, exp, op.name)
        elif t == "Conv2dF16":
            x = rt.get_output(op.inputs[0]).view(np.uint16)
            got = rt.get_output(out).view(np.uint16).ravel()
            exp = conv_f16_op(g, op, x, threads=dwref.num_cpus()).ravel()
            tol_check(got, exp, op.name)
            e = np.abs(got.view(np.float16).astype(np.float64) - exp.view(np.float16).astype(np.float64)).max()
            worst = max(worst, e / max(np.abs(exp.view(np.float16).astype(np.float64)).max(), 1e-30))
        elif t == "GemmF16":
            x = rt.get_output(op.inputs[0]).view(np.uint16)
            got = rt.get_output(out).view(np.uint16).ravel()
            tol_check(got, gemm_f16_op(g, op, x, threads=dwref.num_cpus()).ravel(), op.name)
        elif t == "AddF16":
            a = rt.get_output(op.inputs[0]).view(np.uint16)
            b = rt.get_output(op.inputs[1]).view(np.uint16)
            got = rt.get_output(out).view(np.uint16).ravel()
            assert np.array_equal(got, dwref.relu_f16(dwref.add_f16(a, b))), op.name
        elif t == "MaxPoolF16":
            x = rt.get_output(op.inputs[0]).view(np.uint16)
            n, h, w, c = x.shape
            k, s, p = op.params["k"], op.params["s"], op.params["pad"]
            got = rt.get_output(out).view(np.uint16).ravel()
            assert np.array_equal(got, dwref.maxpool_f16(x, n, h, w, c, k, k, s, s, (p,) * 4)), op.name
        elif t == "GlobalAveragePoolF16":
            x = rt.get_output(op.inputs[0]).view(np.uint16)
            n, h, w, c = x.shape
            got = rt.get_output(out).view(np.uint16).ravel()
            assert np.array_equal(got, dwref.gap_f16(x, n, h, w, c)), op.name
    return worst


def test_resnet50_fp16_small_batch_per_layer_and_logits(be):
    g = G.resnet50_fp16(batch=2, size=64, seed=5)
    x = np.random.default_rng(6).standard_normal((2, 64, 64, 3)).astype(np.float32)
    rt = G.CudaGraphRuntime(g, be)
    rt.set_input_bytes("image", x)
    rt.run()
    assert sum(op.op_type == "Conv2dAddF16" for op in rt.graph.ops) == 16  # every residual add fused
    assert rt.graph.ops[0].op_type == "UnfoldF32ToF16"  # the stem's input is unfolded for the tensor cores
    worst = _per_layer_check(rt.graph, rt)
    logits = rt.get_output("logits")
    ref = run_graph(g, {"image": x}, threads=dwref.num_cpus())["logits"]
    rel = np.abs(logits - ref).max() / np.abs(ref).max()
    print(f"worst layer rel {worst:.3g}; logits rel {rel:.3g}")
    assert rel <= LOGITS_REL_TOL
    rt.release()


def test_resnet50_fp16_full_size_logits_and_graph_replay(be):
    g = G.resnet50_fp16(batch=2, size=224, seed=7)
    x = np.random.default_rng(8).standard_normal((2, 224, 224, 3)).astype(np.float32)
    rt = G.CudaGraphRuntime(g, be)
    rt.set_input_bytes("image", x)
    rt.run()
    eager = rt.get_output("logits").copy()
    launches = rt.capture()
    assert launches >= len(rt.graph.ops)
    rt.run()
    assert np.array_equal(rt.get_output("logits"), eager)
    ref = run_graph(g, {"image": x}, threads=dwref.num_cpus(), batch_slice=(1, 2))["logits"]
    rel = np.abs(eager[1:2] - ref).max() / np.abs(ref).max()
    print(f"224x224 logits rel {rel:.3g}")
    assert rel <= LOGITS_REL_TOL
    rt.release()
