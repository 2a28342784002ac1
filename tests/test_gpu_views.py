"""GPU parity of the channel-range view entry points through the C ABI:
dw_conv2d_i8_view, dw_conv2d_add_i8_view (the conv with the int8 residual add
in its epilogue), dw_add_i8_view and dw_maxpool_i8_view, each reading and
writing (buffer, byte offset, pixel pitch) views into wider tensors.  The view's
channels are bit-identical to the oracle's conv / add_i8 / maxpool of the same
contiguous tensors, and the channels outside the output view are untouched."""
import numpy as np
import pytest

import dragonwing_edge_rs_b200 as dw
from dragonwing_edge_rs_b200 import ops
from dragonwing_edge_rs_b200.backend import BackendError
from oracle import dwref
from tests._util import conv_case, mismatch_report, oracle_conv

pytestmark = pytest.mark.gpu

SENTINEL = 77


@pytest.fixture(scope="module")
def be():
    b = dw.CudaBackend(0, conv_path=dw.PATH_UMMA)
    yield b
    b.close()


def embed(rng, x, pixels, c, pitch, off):
    """x [pixels, c] placed at channel offset `off` of a [pixels, pitch] tensor of noise."""
    full = rng.integers(-128, 128, (pixels, pitch)).astype(np.int8)
    full[:, off:off + c] = x.reshape(pixels, c)
    return full


def view_out(be, pixels, pitch):
    return be.upload_array(np.full((pixels, pitch), SENTINEL, np.int8))


def check_out(be, buf, pixels, c, pitch, off, exp):
    got = be.download_array(buf, np.int8).reshape(pixels, pitch)
    inside = np.ascontiguousarray(got[:, off:off + c]).reshape(-1)
    assert np.array_equal(inside, exp.reshape(-1)), mismatch_report(inside, exp.reshape(-1))
    outside = np.delete(got, np.s_[off:off + c], axis=1)
    assert (outside == SENTINEL).all(), "a write outside the output view"


# n, h, w, c_in, c_out, k, s, epilogue, (x pitch, x off), (residual pitch, off), (y pitch, off)
ADD_CASES = [
    (2, 20, 20, 32, 32, 1, 1, dw.EPI_RELU, (64, 32), (96, 16), (64, 0)),        # 1x1: flat tiles
    (2, 10, 12, 32, 48, 3, 1, dw.EPI_SILU, (32, 0), (48, 0), (48, 0)),          # plain pitches
    (2, 10, 12, 32, 48, 3, 1, dw.EPI_SILU, (80, 48), (64, 16), (96, 48)),
    (3, 5, 5, 16, 16, 3, 1, dw.EPI_RELU6, (48, 16), (32, 0), (32, 16)),         # boxes of fewer than 128 pixels
    (1, 40, 40, 64, 64, 3, 1, dw.EPI_SILU, (128, 64), (128, 0), (192, 128)),    # a YOLOv8n bottleneck shape
    (2, 16, 16, 32, 64, 3, 2, dw.EPI_RELU, (32, 0), (80, 16), (128, 64)),       # strided: contiguous input
    (1, 20, 20, 128, 128, 1, 1, dw.EPI_SILU, (256, 128), (128, 0), (128, 0)),
]


@pytest.mark.parametrize("case", ADD_CASES, ids=lambda c: "x".join(map(str, c[:8])) + f"_p{c[8][0]}_{c[9][0]}_{c[10][0]}")
@pytest.mark.parametrize("ratios", [(0.5, 0.25), (0.731, 1.27), (-1.5, 250.0)], ids=["ties", "mixed", "saturating"])
def test_conv_add_i8_view_matches_conv_then_add(be, case, ratios):
    n, h, w, ci, co, k, s, epi, (xp, xo), (rp, ro), (yp, yo) = case
    rng = np.random.default_rng(hash(case[:8]) & 0xffffffff)
    desc, x, wt, b, M, D = conv_case(rng, n, h, w, ci, co, k=k, s=s, epilogue=epi)
    ho, wo = desc.out_hw()
    pin, pout = n * h * w, n * ho * wo
    res = rng.integers(-128, 128, pout * co).astype(np.int8)
    ra, rb = (float(np.float32(r)) for r in ratios)
    exp = dwref.add_i8(res, oracle_conv(desc, x, wt, b, M, D), ra, rb)

    bx = be.upload_array(embed(rng, x, pin, ci, xp, xo))
    br = be.upload_array(embed(rng, res, pout, co, rp, ro))
    by = view_out(be, pout, yp)
    bw = be.upload_array(wt)
    wp = ops.prepare_weights_i8(be, desc, bw)
    bb, bm, bd = be.upload_array(b), be.upload_array(M), be.upload_array(D)
    ops.conv2d_add_i8_view(be, desc, (bx, xo, xp), wp, bb, bm, bd, (br, ro, rp), ra, rb, (by, yo, yp))
    check_out(be, by, pout, co, yp, yo, exp)
    # the same conv without the add, through the plain view entry point
    by2 = view_out(be, pout, yp)
    ops.conv2d_i8_view(be, desc, (bx, xo, xp), wp, bb, bm, bd, (by2, yo, yp))
    check_out(be, by2, pout, co, yp, yo, oracle_conv(desc, x, wt, b, M, D))
    for buf in (bx, br, by, by2, bw, wp, bb, bm, bd):
        buf.free()


def test_conv_add_i8_view_in_place_residual(be):
    """Output written over its own residual (the same view): each tile's
    residual is read before that tile's output is stored."""
    rng = np.random.default_rng(41)
    desc, x, wt, b, M, D = conv_case(rng, 2, 24, 24, 32, 32, k=3, s=1, epilogue=dw.EPI_SILU)
    pout = 2 * 24 * 24
    res = rng.integers(-128, 128, pout * 32).astype(np.int8)
    exp = dwref.add_i8(res, oracle_conv(desc, x, wt, b, M, D), 1.0, 0.8125)
    bx, br = be.upload_array(x), be.upload_array(res)
    bw = be.upload_array(wt)
    wp = ops.prepare_weights_i8(be, desc, bw)
    bb, bm, bd = be.upload_array(b), be.upload_array(M), be.upload_array(D)
    ops.conv2d_add_i8_view(be, desc, (bx, 0, 32), wp, bb, bm, bd, (br, 0, 32), 1.0, 0.8125, (br, 0, 32))
    got = be.download_array(br, np.int8)
    assert np.array_equal(got, exp), mismatch_report(got, exp)
    for buf in (bx, br, bw, wp, bb, bm, bd):
        buf.free()


def test_conv_add_i8_view_rejects(be):
    rng = np.random.default_rng(3)
    desc, x, wt, b, M, D = conv_case(rng, 1, 8, 8, 32, 32, k=1, s=1, epilogue=dw.EPI_RELU)
    bx, br, by = be.upload_array(x), be.alloc(64 * 32), be.alloc(64 * 32)
    bw = be.upload_array(wt)
    wp = ops.prepare_weights_i8(be, desc, bw)
    bm = be.upload_array(M)
    with pytest.raises(BackendError) as e:  # ratios at the packed add's limit
        ops.conv2d_add_i8_view(be, desc, (bx, 0, 32), wp, None, bm, None, (br, 0, 32), 1e30, 1.0, (by, 0, 32))
    assert e.value.status == dw._lib.DW_ERR_UNSUPPORTED
    with pytest.raises(BackendError) as e:  # residual view past its buffer
        ops.conv2d_add_i8_view(be, desc, (bx, 0, 32), wp, None, bm, None, (br, 16, 32), 1.0, 1.0, (by, 0, 32))
    assert e.value.status == dw._lib.DW_ERR_SIZE_MISMATCH
    with pytest.raises(BackendError) as e:  # pitch not a 16-byte multiple
        ops.conv2d_add_i8_view(be, desc, (bx, 0, 32), wp, None, bm, None, (br, 0, 40), 1.0, 1.0, (by, 0, 32))
    assert e.value.status == dw._lib.DW_ERR_INVALID_ARG
    for buf in (bx, br, by, bw, wp, bm):
        buf.free()


@pytest.mark.parametrize("pixels,c,pitches", [(400, 32, (64, 96, 32)), (4099, 16, (16, 48, 64)), (1, 64, (64, 64, 128))])
def test_add_i8_view(be, pixels, c, pitches):
    rng = np.random.default_rng(pixels + c)
    (pa, pb, po), (oa, ob, oo) = pitches, tuple(p - c for p in pitches)
    a = rng.integers(-128, 128, pixels * c).astype(np.int8)
    b = rng.integers(-128, 128, pixels * c).astype(np.int8)
    ba, bb = be.upload_array(embed(rng, a, pixels, c, pa, oa)), be.upload_array(embed(rng, b, pixels, c, pb, ob))
    bo = view_out(be, pixels, po)
    ops.add_i8_view(be, (ba, oa, pa), (bb, ob, pb), (bo, oo, po), pixels, c, 0.5, 0.75)
    check_out(be, bo, pixels, c, po, oo, dwref.add_i8(a, b, 0.5, 0.75))
    for buf in (ba, bb, bo):
        buf.free()


@pytest.mark.parametrize("n,h,w,c,k,s,p", [(1, 20, 20, 128, 5, 1, 2), (2, 9, 7, 32, 3, 2, 1), (1, 13, 13, 16, 2, 2, 0)])
def test_maxpool_i8_view(be, n, h, w, c, k, s, p):
    rng = np.random.default_rng(h * w + c)
    x = rng.integers(-128, 128, n * h * w * c).astype(np.int8)
    exp = dwref.maxpool_i8(x, n, h, w, c, k, k, s, s, (p, p, p, p))
    ho, wo = (h + 2 * p - k) // s + 1, (w + 2 * p - k) // s + 1
    xp, yp = 4 * c, 3 * c
    bx = be.upload_array(embed(rng, x, n * h * w, c, xp, c))
    by = view_out(be, n * ho * wo, yp)
    ops.maxpool_i8_view(be, (bx, c, xp), (by, 2 * c, yp), n, h, w, c, k, k, s, s, (p, p, p, p))
    check_out(be, by, n * ho * wo, c, yp, 2 * c, exp)
    for buf in (bx, by):
        buf.free()


@pytest.mark.parametrize("n,h,w,c,k,count", [(2, 20, 20, 128, 5, 3),   # YOLOv8n SPPF at 640x640
                                             (1, 40, 48, 32, 5, 3),    # a map too large for one block: separate pools
                                             (3, 7, 5, 16, 3, 2), (1, 4, 4, 16, 9, 1), (2, 9, 11, 48, 5, 4)])
def test_maxpool_chain_i8_view(be, n, h, w, c, k, count):
    """Chained k x k stride-1 pools (padding k/2) into views of one wider
    tensor, as SPPF's concat: identical to pooling the previous output."""
    rng = np.random.default_rng(n * h * w + c + k)
    pix, p = n * h * w, k // 2
    x = rng.integers(-128, 128, pix * c).astype(np.int8)
    pitch = (count + 1) * c
    bx = be.upload_array(embed(rng, x, pix, c, pitch, 0))
    by = view_out(be, pix, pitch)
    ops.maxpool_chain_i8_view(be, (bx, 0, pitch), [(by, (i + 1) * c, pitch) for i in range(count)], n, h, w, c, k)
    got = be.download_array(by, np.int8).reshape(pix, pitch)
    assert (got[:, :c] == SENTINEL).all()
    cur = x
    for i in range(count):
        cur = dwref.maxpool_i8(cur, n, h, w, c, k, k, 1, 1, (p, p, p, p)).reshape(-1)
        seg = np.ascontiguousarray(got[:, (i + 1) * c:(i + 2) * c]).reshape(-1)
        assert np.array_equal(seg, cur), (i, mismatch_report(seg, cur))
    for buf in (bx, by):
        buf.free()
