// conv_direct.cu -- CUDA-core int8 convolutions:
//   * k_conv_direct: any dense conv (any c_in, incl. the 3-channel stem), one
//     thread per output element, dp4a over 4 input channels when c_in % 4 == 0;
//     also produces raw int32 accumulators (conv2d_i8_nhwc, gemm_i8);
//   * k_dwconv16: depthwise conv (multiplier 1, c % 16 == 0), one thread per
//     (output pixel, 16 channels), 128-bit loads/stores;
//   * k_dwconv_generic: any depthwise conv, one thread per output element.
// Semantics: crates/dragonwing-cpu/src/ops.rs:3086-3142 (conv) and :2669-2730
// (depthwise index math), with the fused epilogue of dw_device.cuh.

#include "dw_device.cuh"

namespace dw {
namespace {

constexpr int kThreads = 256;

inline int grid_for(const dw_backend *be, size_t items) {
    size_t blocks = (items + kThreads - 1) / kThreads;
    size_t cap = (size_t)be->sm_count * 16;
    return (int)std::max<size_t>(1, std::min(blocks, cap));
}

struct ConvGeom {
    int n, h, w, c_in, c_out, kh, kw, sh, sw, pt, pl, ho, wo;
};

// Dense conv; weights OHWI [c_out][kh*kw][c_in].
template <bool kVec4>
__global__ void __launch_bounds__(kThreads) k_conv_direct(ConvGeom g, const int8_t *__restrict__ x,
                                                          const int8_t *__restrict__ w, EpiParams ep,
                                                          int8_t *__restrict__ y, int32_t *__restrict__ acc_out) {
    const size_t total = (size_t)g.n * g.ho * g.wo * g.c_out;
    const int taps = g.kh * g.kw;
    for (size_t i = blockIdx.x * (size_t)blockDim.x + threadIdx.x; i < total; i += (size_t)gridDim.x * blockDim.x) {
        const int oc = (int)(i % g.c_out);
        size_t p = i / g.c_out;
        const int ow = (int)(p % g.wo);
        size_t t = p / g.wo;
        const int oh = (int)(t % g.ho);
        const int b = (int)(t / g.ho);
        int32_t acc = 0;
        for (int a = 0; a < g.kh; a++) {
            const int ih = oh * g.sh + a - g.pt;
            if (ih < 0 || ih >= g.h) continue;
            for (int q = 0; q < g.kw; q++) {
                const int iw = ow * g.sw + q - g.pl;
                if (iw < 0 || iw >= g.w) continue;
                const int8_t *px = x + (((size_t)b * g.h + ih) * g.w + iw) * g.c_in;
                const int8_t *pw = w + ((size_t)oc * taps + (a * g.kw + q)) * g.c_in;
                if (kVec4) {
                    const int *px4 = reinterpret_cast<const int *>(px);
                    const int *pw4 = reinterpret_cast<const int *>(pw);
                    for (int c = 0; c < g.c_in / 4; c++) acc = __dp4a(__ldg(px4 + c), __ldg(pw4 + c), acc);
                } else {
                    for (int c = 0; c < g.c_in; c++) acc += (int32_t)px[c] * (int32_t)__ldg(pw + c);
                }
            }
        }
        if (acc_out) {
            acc_out[i] = acc;
        } else {
            const int32_t bias = ep.bias ? __ldg(ep.bias + oc) : 0;
            const float m = ep.M ? __ldg(ep.M + oc) : 0.0f;
            const float dsc = ep.D ? __ldg(ep.D + oc) : 0.0f;
            y[i] = (int8_t)epilogue_one_slow(acc, bias, m, dsc, ep.epilogue, ep.q6, ep.inv_s_out);
        }
    }
}

// One output element's epilogue with the certified SiLU fast path (exact result).
__device__ __forceinline__ uint32_t epilogue_byte(int32_t acc, int32_t bias, float m, float dsc, const EpiParams &ep) {
    if (ep.epilogue == DW_EPI_SILU) {
        const int32_t a = (int32_t)((uint32_t)acc + (uint32_t)bias);
        if ((uint32_t)(a + (1 << 22)) < (1u << 23) && isfinite(dsc) && isfinite(ep.inv_s_out)) {
            bool u = false;
            const uint32_t bits = silu_fast_bits(i2f_small(a), dsc, ep.inv_s_out, u);
            if (!u) return bits & 0xFFu;
        }
    }
    return (uint8_t)epilogue_one_slow(acc, bias, m, dsc, ep.epilogue, ep.q6, ep.inv_s_out);
}

// Dense conv with few input channels (the 3-channel stem, or any c_in the
// tensor-core path does not take), c_out % 16 == 0: one thread = one output
// pixel x 16 output channels.  Weights are staged once per block in shared
// memory as floats [tap][c_in][c_out]; int8 products (<= 2^14) summed over
// k_h*k_w*c_in <= 1024 taps stay below 2^24, so the FP32 accumulation is exact.
__global__ void __launch_bounds__(256) k_conv_smallc(ConvGeom g, const int8_t *__restrict__ x,
                                                     const int8_t *__restrict__ w_ohwi, EpiParams ep,
                                                     int8_t *__restrict__ y) {
    extern __shared__ float sw[];
    const int K = g.kh * g.kw * g.c_in;
    for (int i = threadIdx.x; i < K * g.c_out; i += blockDim.x) {
        const int oc = i % g.c_out, kk = i / g.c_out;
        sw[i] = (float)w_ohwi[(size_t)oc * K + kk];
    }
    __syncthreads();
    const int groups = g.c_out / 16;
    const uint32_t total = (uint32_t)g.n * g.ho * g.wo * groups;
    for (uint32_t i = blockIdx.x * blockDim.x + threadIdx.x; i < total; i += gridDim.x * blockDim.x) {
        const int cg = (int)(i % groups);
        const uint32_t p = i / groups;
        const int ow = (int)(p % g.wo);
        const uint32_t t = p / g.wo;
        const int oh = (int)(t % g.ho);
        const int b = (int)(t / g.ho);
        float acc[16];
#pragma unroll
        for (int j = 0; j < 16; j++) acc[j] = 0.0f;
        for (int a = 0; a < g.kh; a++) {
            const int ih = oh * g.sh + a - g.pt;
            if (ih < 0 || ih >= g.h) continue;
            for (int q = 0; q < g.kw; q++) {
                const int iw = ow * g.sw + q - g.pl;
                if (iw < 0 || iw >= g.w) continue;
                const int8_t *px = x + (((size_t)b * g.h + ih) * g.w + iw) * g.c_in;
                const float *ws = sw + (size_t)((a * g.kw + q) * g.c_in) * g.c_out + cg * 16;
                for (int c = 0; c < g.c_in; c++) {
                    const float xv = i2f_small(px[c]);
                    const float4 *w4 = reinterpret_cast<const float4 *>(ws + (size_t)c * g.c_out);
#pragma unroll
                    for (int j4 = 0; j4 < 4; j4++) {
                        const float4 wv = w4[j4];
                        acc[j4 * 4 + 0] = __fmaf_rn(xv, wv.x, acc[j4 * 4 + 0]);
                        acc[j4 * 4 + 1] = __fmaf_rn(xv, wv.y, acc[j4 * 4 + 1]);
                        acc[j4 * 4 + 2] = __fmaf_rn(xv, wv.z, acc[j4 * 4 + 2]);
                        acc[j4 * 4 + 3] = __fmaf_rn(xv, wv.w, acc[j4 * 4 + 3]);
                    }
                }
            }
        }
        uint32_t out[4];
#pragma unroll
        for (int j4 = 0; j4 < 4; j4++) {
            uint32_t packed = 0;
#pragma unroll
            for (int j = 0; j < 4; j++) {
                const int oc = cg * 16 + j4 * 4 + j;
                const int32_t ai = __float_as_int(__fadd_rn(acc[j4 * 4 + j], kMagic)) - kMagicBits;
                const int32_t bias = ep.bias ? __ldg(ep.bias + oc) : 0;
                const float m = ep.M ? __ldg(ep.M + oc) : 0.0f;
                const float dsc = ep.D ? __ldg(ep.D + oc) : 0.0f;
                packed |= epilogue_byte(ai, bias, m, dsc, ep) << (8 * j);
            }
            out[j4] = packed;
        }
        *reinterpret_cast<uint4 *>(y + (size_t)p * g.c_out + cg * 16) = make_uint4(out[0], out[1], out[2], out[3]);
    }
}

// Depthwise, multiplier 1, 16 channels per thread; weights [kh*kw][c].
__global__ void __launch_bounds__(kThreads) k_dwconv16(ConvGeom g, const int8_t *__restrict__ x,
                                                       const int8_t *__restrict__ w, EpiParams ep,
                                                       int8_t *__restrict__ y) {
    const int groups = g.c_in / 16;
    const size_t total = (size_t)g.n * g.ho * g.wo * groups;
    for (size_t i = blockIdx.x * (size_t)blockDim.x + threadIdx.x; i < total; i += (size_t)gridDim.x * blockDim.x) {
        const int cg = (int)(i % groups);
        size_t p = i / groups;
        const int ow = (int)(p % g.wo);
        size_t t = p / g.wo;
        const int oh = (int)(t % g.ho);
        const int b = (int)(t / g.ho);
        int32_t acc[16];
#pragma unroll
        for (int k = 0; k < 16; k++) acc[k] = 0;
        for (int a = 0; a < g.kh; a++) {
            const int ih = oh * g.sh + a - g.pt;
            if (ih < 0 || ih >= g.h) continue;
            for (int q = 0; q < g.kw; q++) {
                const int iw = ow * g.sw + q - g.pl;
                if (iw < 0 || iw >= g.w) continue;
                const int4 xv = __ldg(reinterpret_cast<const int4 *>(x + (((size_t)b * g.h + ih) * g.w + iw) * g.c_in) + cg);
                const int4 wv = __ldg(reinterpret_cast<const int4 *>(w + (size_t)(a * g.kw + q) * g.c_in) + cg);
                const uint32_t xs[4] = {(uint32_t)xv.x, (uint32_t)xv.y, (uint32_t)xv.z, (uint32_t)xv.w};
                const uint32_t ws[4] = {(uint32_t)wv.x, (uint32_t)wv.y, (uint32_t)wv.z, (uint32_t)wv.w};
#pragma unroll
                for (int v = 0; v < 4; v++)
#pragma unroll
                    for (int k = 0; k < 4; k++)
                        acc[v * 4 + k] += (int32_t)(int8_t)(xs[v] >> (8 * k)) * (int32_t)(int8_t)(ws[v] >> (8 * k));
            }
        }
        uint32_t outw[4];
#pragma unroll
        for (int v = 0; v < 4; v++) {
            uint32_t packed = 0;
#pragma unroll
            for (int k = 0; k < 4; k++) {
                const int c = cg * 16 + v * 4 + k;
                const int32_t bias = ep.bias ? __ldg(ep.bias + c) : 0;
                const float m = ep.M ? __ldg(ep.M + c) : 0.0f;
                const float dsc = ep.D ? __ldg(ep.D + c) : 0.0f;
                packed |= (uint32_t)(uint8_t)epilogue_one_slow(acc[v * 4 + k], bias, m, dsc, ep.epilogue, ep.q6,
                                                          ep.inv_s_out)
                          << (8 * k);
            }
            outw[v] = packed;
        }
        *reinterpret_cast<int4 *>(y + p * g.c_in + cg * 16) = make_int4(outw[0], outw[1], outw[2], outw[3]);
    }
}

// Depthwise 3x3 (multiplier 1, c % 4 == 0): one thread computes an RH x RW
// block of output pixels for 4 channels (one 32-bit word per pixel, so a warp
// reads and writes 128 contiguous bytes).  int8 values are converted exactly to
// float (byte placed in the mantissa of 2^23 + 128, then 2^23 + 128 subtracted)
// and accumulated with FP32 FMAs: every product (<= 2^14) and every 9-tap sum
// (< 2^18) is an integer below 2^24, so the float accumulation is exact and the
// result equals the reference's i32 sum.
__device__ __forceinline__ void unpack4(uint32_t w, float (&f)[4]) {
    const uint32_t u = w ^ 0x80808080u;  // int8 -> excess-128 unsigned bytes
#pragma unroll
    for (int k = 0; k < 4; k++)
        f[k] = __fsub_rn(__uint_as_float(__byte_perm(u, 0x4B000000u, 0x7440 + k)), 8388736.0f);
}

template <int S, int RH, int RW>
__global__ void __launch_bounds__(256, 2) k_dwconv3x3(ConvGeom g, const int8_t *__restrict__ x,
                                                   const int8_t *__restrict__ w, EpiParams ep,
                                                   int8_t *__restrict__ y) {
    // grid: x = 32-channel-group slices, y = (image, tile row); block (32, 8):
    // threadIdx.y strides over the tile columns.  32-bit index math only.
    const int cg_n = g.c_in / 4;
    const int cg = blockIdx.x * 32 + threadIdx.x;
    if (cg >= cg_n) return;
    const int tiles_w = (g.wo + RW - 1) / RW, tiles_h = (g.ho + RH - 1) / RH;
    const int th = (int)blockIdx.y % tiles_h;
    const int b = (int)blockIdx.y / tiles_h;
    constexpr int IH = (RH - 1) * S + 3, IW = (RW - 1) * S + 3;
    const uint32_t *wg = reinterpret_cast<const uint32_t *>(w) + cg;
    // epilogue: per channel bias / M (fast exact path when |bias| < 2^21 and M finite)
    const int c0 = cg * 4;
    int32_t bias[4];
    float m[4], dsc[4], biasf[4];
    bool fast = ep.epilogue != DW_EPI_SILU;
#pragma unroll
    for (int k = 0; k < 4; k++) {
        bias[k] = ep.bias ? __ldg(ep.bias + c0 + k) : 0;
        m[k] = ep.M ? __ldg(ep.M + c0 + k) : 0.0f;
        dsc[k] = ep.D ? __ldg(ep.D + c0 + k) : 0.0f;
        fast = fast && (uint32_t)(bias[k] + (1 << 21)) < (1u << 22) && isfinite(m[k]);
        biasf[k] = fast ? i2f_small(bias[k]) : 0.0f;
    }
    const uint32_t c6 = 0x01010101u * (uint32_t)ep.q6;
    for (int tw = threadIdx.y; tw < tiles_w; tw += blockDim.y) {
        const int oh0 = th * RH, ow0 = tw * RW;
        float wf[9][4];  // reloaded per tile (L1 hits) to keep register pressure down
#pragma unroll
        for (int k = 0; k < 9; k++) unpack4(__ldg(wg + (size_t)k * cg_n), wf[k]);
        float acc[RH][RW][4];
#pragma unroll
        for (int r = 0; r < RH; r++)
#pragma unroll
            for (int q = 0; q < RW; q++)
#pragma unroll
                for (int k = 0; k < 4; k++) acc[r][q][k] = 0.0f;
        const int ih0 = oh0 * S - g.pt, iw0 = ow0 * S - g.pl;
        const uint32_t *xb = reinterpret_cast<const uint32_t *>(x + (size_t)b * g.h * g.w * g.c_in) + cg;
        const uint32_t row_words = (uint32_t)g.w * cg_n;
#pragma unroll
        for (int r = 0; r < IH; r++) {
            const int ih = ih0 + r;
            const bool rok = ih >= 0 && ih < g.h;
            float xr[IW][4];
#pragma unroll
            for (int c = 0; c < IW; c++) {
                const int iw = iw0 + c;
                uint32_t v = 0;
                if (rok && iw >= 0 && iw < g.w) v = __ldg(xb + (uint32_t)ih * row_words + (uint32_t)iw * cg_n);
                unpack4(v, xr[c]);
            }
#pragma unroll
            for (int orow = 0; orow < RH; orow++) {
                const int kh = r - orow * S;
                if (kh < 0 || kh > 2) continue;
#pragma unroll
                for (int q = 0; q < RW; q++)
#pragma unroll
                    for (int kw = 0; kw < 3; kw++)
#pragma unroll
                        for (int k = 0; k < 4; k++)
                            acc[orow][q][k] = __fmaf_rn(xr[q * S + kw][k], wf[kh * 3 + kw][k], acc[orow][q][k]);
            }
        }
#pragma unroll
        for (int r = 0; r < RH; r++) {
            const int oh = oh0 + r;
            if (oh >= g.ho) break;
#pragma unroll
            for (int q = 0; q < RW; q++) {
                const int ow = ow0 + q;
                if (ow >= g.wo) break;
                uint32_t packed = 0;
                if (fast) {
#pragma unroll
                    for (int k = 0; k < 4; k++) {
                        const float a = __fadd_rn(acc[r][q][k], biasf[k]);
                        packed |= f32_to_i8_byte_nonan(__fmul_rn(a, m[k])) << (8 * k);
                    }
                    if (ep.epilogue == DW_EPI_RELU) packed = __vmaxs4(packed, 0u);
                    else if (ep.epilogue == DW_EPI_RELU6) packed = __vmins4(__vmaxs4(packed, 0u), c6);
                } else {
#pragma unroll
                    for (int k = 0; k < 4; k++) {
                        const int32_t ai = __float_as_int(__fadd_rn(acc[r][q][k], kMagic)) - kMagicBits;
                        packed |= (uint32_t)(uint8_t)epilogue_one_slow(ai, bias[k], m[k], dsc[k], ep.epilogue, ep.q6,
                                                                  ep.inv_s_out)
                                  << (8 * k);
                    }
                }
                reinterpret_cast<uint32_t *>(y + (((size_t)b * g.ho + oh) * g.wo + ow) * g.c_in)[cg] = packed;
            }
        }
    }
}

// Depthwise, any multiplier: c_out = c_in * mult, oc = ic * mult + m, weights [kh][kw][c_in][mult].
__global__ void __launch_bounds__(kThreads) k_dwconv_generic(ConvGeom g, int mult, const int8_t *__restrict__ x,
                                                             const int8_t *__restrict__ w, EpiParams ep,
                                                             int8_t *__restrict__ y, int32_t *__restrict__ acc_out) {
    const size_t total = (size_t)g.n * g.ho * g.wo * g.c_out;
    for (size_t i = blockIdx.x * (size_t)blockDim.x + threadIdx.x; i < total; i += (size_t)gridDim.x * blockDim.x) {
        const int oc = (int)(i % g.c_out);
        size_t p = i / g.c_out;
        const int ow = (int)(p % g.wo);
        size_t t = p / g.wo;
        const int oh = (int)(t % g.ho);
        const int b = (int)(t / g.ho);
        const int ic = oc / mult, m = oc % mult;
        int32_t acc = 0;
        for (int a = 0; a < g.kh; a++) {
            const int ih = oh * g.sh + a - g.pt;
            if (ih < 0 || ih >= g.h) continue;
            for (int q = 0; q < g.kw; q++) {
                const int iw = ow * g.sw + q - g.pl;
                if (iw < 0 || iw >= g.w) continue;
                acc += (int32_t)x[(((size_t)b * g.h + ih) * g.w + iw) * g.c_in + ic] *
                       (int32_t)__ldg(w + ((size_t)(a * g.kw + q) * g.c_in + ic) * mult + m);
            }
        }
        if (acc_out) {
            acc_out[i] = acc;
        } else {
            const int32_t bias = ep.bias ? __ldg(ep.bias + oc) : 0;
            const float mm = ep.M ? __ldg(ep.M + oc) : 0.0f;
            const float dsc = ep.D ? __ldg(ep.D + oc) : 0.0f;
            y[i] = (int8_t)epilogue_one_slow(acc, bias, mm, dsc, ep.epilogue, ep.q6, ep.inv_s_out);
        }
    }
}

ConvGeom geom(const dw_conv_desc &d, int ho, int wo) {
    return ConvGeom{d.n, d.h, d.w, d.c_in, d.c_out, d.k_h, d.k_w, d.stride_h, d.stride_w, d.pad_t, d.pad_l, ho, wo};
}

// ---- depthwise 3x3, stride 1: integer dot products on per-channel column packs
// One thread: 4 channels (one 32-bit word per pixel) x 4 output columns x a
// segment of SEG output rows, sliding down the input one row at a time.  The 6
// input words of a row (columns ow0-1 .. ow0+4, 4 channels each) are
// transposed with byte permutes into, per channel, the 6 columns as bytes;
// the 3-column window of output column j is then a funnel shift, and one
// __dp4a against (w[kh][0], w[kh][1], w[kh][2], 0) adds a whole kernel row.
// Each input row feeds three output rows (kh = 0, 1, 2); the accumulator of
// the row that took its kh = 2 contribution is complete and goes through the
// requantisation epilogue.  The int32 sums are exact, as in the reference
// (sum over kh, kw of x * w; ops.rs:2669-2730 index order, integer arithmetic).
__device__ __forceinline__ void dw_row_dp4a(const uint32_t (&X)[6], const int32_t (&wk)[3][4], int32_t (&a0)[4][4],
                                            int32_t (&a1)[4][4], int32_t (&a2)[4][4]) {
    const uint32_t ta = __byte_perm(X[0], X[1], 0x5140), tb = __byte_perm(X[0], X[1], 0x7362);
    const uint32_t tc = __byte_perm(X[2], X[3], 0x5140), td = __byte_perm(X[2], X[3], 0x7362);
    const uint32_t te = __byte_perm(X[4], X[5], 0x5140), tf = __byte_perm(X[4], X[5], 0x7362);
    uint32_t P0[4], P1[4];
    P0[0] = __byte_perm(ta, tc, 0x5410);
    P0[1] = __byte_perm(ta, tc, 0x7632);
    P0[2] = __byte_perm(tb, td, 0x5410);
    P0[3] = __byte_perm(tb, td, 0x7632);
    P1[0] = te;
    P1[1] = te >> 16;
    P1[2] = tf;
    P1[3] = tf >> 16;
#pragma unroll
    for (int k = 0; k < 4; k++) {
#pragma unroll
        for (int j = 0; j < 4; j++) {
            const int win = (int)(j == 0 ? P0[k] : __funnelshift_r(P0[k], P1[k], 8 * j));
            a2[j][k] = __dp4a(win, wk[2][k], a2[j][k]);
            a1[j][k] = __dp4a(win, wk[1][k], a1[j][k]);
            a0[j][k] = __dp4a(win, wk[0][k], a0[j][k]);
        }
    }
}

template <int SEG>
__global__ void __launch_bounds__(128) k_dwconv3x3_s1_dp4a(ConvGeom g, const int8_t *__restrict__ x,
                                                           const int8_t *__restrict__ w, EpiParams ep,
                                                           int8_t *__restrict__ y) {
    const int cg_n = g.c_in >> 2;
    const int strips = (g.wo + 3) >> 2;
    const int segs = (g.ho + SEG - 1) / SEG;
    int idx = blockIdx.x * blockDim.x + threadIdx.x;  // the host checks the total fits in int
    if (idx >= cg_n * strips * segs * g.n) return;
    const int cg = idx % cg_n;
    idx /= cg_n;
    const int strip = idx % strips;
    idx /= strips;
    const int seg = idx % segs;
    const int b = idx / segs;
    const int ow0 = strip * 4, o0 = seg * SEG;

    // per channel k and kernel row kh: (w[kh][0][c], w[kh][1][c], w[kh][2][c], 0)
    const uint32_t *wq = reinterpret_cast<const uint32_t *>(w) + cg;
    int32_t wk[3][4];
#pragma unroll
    for (int kh = 0; kh < 3; kh++) {
        const uint32_t k0 = __ldg(wq + (size_t)(kh * 3 + 0) * cg_n), k1 = __ldg(wq + (size_t)(kh * 3 + 1) * cg_n);
        const uint32_t k2 = __ldg(wq + (size_t)(kh * 3 + 2) * cg_n);
#pragma unroll
        for (int k = 0; k < 4; k++) {
            const uint32_t t01 = __byte_perm(k0, k1, (uint32_t)((4 + k) << 4 | k));
            wk[kh][k] = (int32_t)(__byte_perm(t01, k2, (uint32_t)((4 + k) << 8 | 0x10)) & 0x00FFFFFFu);
        }
    }
    const int c0 = cg * 4;
    int32_t bias[4];
    float m[4], dsc[4], biasf[4];
    bool fast = ep.epilogue != DW_EPI_SILU;
#pragma unroll
    for (int k = 0; k < 4; k++) {
        bias[k] = ep.bias ? __ldg(ep.bias + c0 + k) : 0;
        m[k] = ep.M ? __ldg(ep.M + c0 + k) : 0.0f;
        dsc[k] = ep.D ? __ldg(ep.D + c0 + k) : 0.0f;
        fast = fast && (uint32_t)(bias[k] + (1 << 21)) < (1u << 22) && isfinite(m[k]);
        biasf[k] = fast ? i2f_small(bias[k]) : 0.0f;
    }
    const uint32_t c6 = 0x01010101u * (uint32_t)ep.q6;
    const uint32_t *xb = reinterpret_cast<const uint32_t *>(x + (size_t)b * g.h * g.w * g.c_in) + cg;
    uint32_t *yb = reinterpret_cast<uint32_t *>(y + (size_t)b * g.ho * g.wo * g.c_in) + cg;

    // ReLU / ReLU6 clamp before rounding: roundf commutes with a clamp to
    // integer bounds, so clamp(roundf(v), lo, hi) == roundf(clamp(v, lo, hi)).
    const float lo = (ep.epilogue == DW_EPI_RELU || ep.epilogue == DW_EPI_RELU6) ? 0.0f : -128.0f;
    const float hi = ep.epilogue == DW_EPI_RELU6 ? (float)ep.q6 : 127.0f;

    auto load_row = [&](int t, uint32_t (&X)[6]) {
        const int ih = o0 - g.pt + t;
        const bool rok = ih >= 0 && ih < g.h;
#pragma unroll
        for (int c = 0; c < 6; c++) {
            const int iw = ow0 - g.pl + c;
            X[c] = (rok && iw >= 0 && iw < g.w) ? __ldg(xb + ((size_t)ih * g.w + iw) * cg_n) : 0u;
        }
    };
    // accumulators start at the bias on the fast path (|acc + bias| < 2^22 there)
    auto reset = [&](int32_t (&acc)[4][4]) {
#pragma unroll
        for (int j = 0; j < 4; j++)
#pragma unroll
            for (int k = 0; k < 4; k++) acc[j][k] = fast ? bias[k] : 0;
    };
    auto finish = [&](int t, int32_t (&acc)[4][4]) {
        const int oh = o0 + t - 2;
        if (t >= 2 && oh < o0 + SEG && oh < g.ho) {
#pragma unroll
            for (int j = 0; j < 4; j++) {
                const int ow = ow0 + j;
                if (ow < g.wo) {
                    uint32_t packed = 0;
                    if (fast) {
#pragma unroll
                        for (int k = 0; k < 4; k++) {
                            // roundf(clamp(fl(a * M))) via one RN add of 1.5 * 2^23 and the tie fix
                            const float v = fminf(fmaxf(__fmul_rn(i2f_small(acc[j][k]), m[k]), lo), hi);
                            const float r = __fadd_rn(v, kMagic);
                            const float dlt = __fsub_rn(v, __fsub_rn(r, kMagic));
                            const uint32_t q = __float_as_uint(r) + (dlt == copysignf(0.5f, v) ? (v > 0.0f ? 1u : 0xFFFFFFFFu) : 0u);
                            packed |= (q & 0xFFu) << (8 * k);
                        }
                    } else {
#pragma unroll
                        for (int k = 0; k < 4; k++)
                            packed |= (uint32_t)(uint8_t)epilogue_one_slow(acc[j][k], bias[k], m[k], dsc[k], ep.epilogue,
                                                                          ep.q6, ep.inv_s_out)
                                      << (8 * k);
                    }
                    yb[((size_t)oh * g.wo + ow) * cg_n] = packed;
                }
            }
        }
        reset(acc);
    };
    int32_t A[4][4], B[4][4], C[4][4];
    reset(A);
    reset(B);
    reset(C);
    // step t reads input row o0 - pt + t; the kh = 0 / 1 / 2 accumulators hold
    // output rows o0 + t, o0 + t - 1, o0 + t - 2 (the roles rotate every step).
    // The next three rows are loaded while the current three are computed.
    uint32_t X0[6], X1[6], X2[6];
    load_row(0, X0);
    load_row(1, X1);
    load_row(2, X2);
#pragma unroll 1
    for (int t = 0; t < SEG + 2; t += 3) {
        uint32_t N0[6], N1[6], N2[6];
        load_row(t + 3, N0);
        load_row(t + 4, N1);
        load_row(t + 5, N2);
        dw_row_dp4a(X0, wk, A, B, C);
        finish(t, C);
        dw_row_dp4a(X1, wk, C, A, B);
        finish(t + 1, B);
        dw_row_dp4a(X2, wk, B, C, A);
        finish(t + 2, A);
#pragma unroll
        for (int c = 0; c < 6; c++) {
            X0[c] = N0[c];
            X1[c] = N1[c];
            X2[c] = N2[c];
        }
    }
}

}  // namespace

dw_status launch_conv_direct_i8(dw_backend *be, const dw_conv_desc &d, int ho, int wo, const int8_t *x,
                                const int8_t *w_ohwi, const EpiParams &ep, int8_t *y, int32_t *acc_out) {
    ConvGeom g = geom(d, ho, wo);
    size_t items = (size_t)d.n * ho * wo * d.c_out;
    const int K = d.k_h * d.k_w * d.c_in;
    const size_t sw_bytes = (size_t)K * d.c_out * sizeof(float);
    if (!acc_out && d.group == 1 && d.c_out % 16 == 0 && K <= 256 && sw_bytes <= 48 * 1024 &&
        items / 16 < (1u << 31) && (uintptr_t)y % 16 == 0) {
        const size_t threads_needed = items / 16;
        const int grid = (int)std::max<size_t>(1, std::min((threads_needed + 255) / 256, (size_t)be->sm_count * 8));
        k_conv_smallc<<<grid, 256, sw_bytes, be->stream>>>(g, x, w_ohwi, ep, y);
        return dw_after_launch(be, "conv_smallc_i8");
    }
    bool vec4 = (d.c_in % 4 == 0) && ((uintptr_t)x % 4 == 0) && ((uintptr_t)w_ohwi % 4 == 0);
    if (vec4)
        k_conv_direct<true><<<grid_for(be, items), kThreads, 0, be->stream>>>(g, x, w_ohwi, ep, y, acc_out);
    else
        k_conv_direct<false><<<grid_for(be, items), kThreads, 0, be->stream>>>(g, x, w_ohwi, ep, y, acc_out);
    return dw_after_launch(be, "conv_direct_i8");
}

dw_status launch_dwconv_i8(dw_backend *be, const dw_conv_desc &d, int ho, int wo, const int8_t *x,
                           const int8_t *w_hwcm, const EpiParams &ep, int8_t *y, int32_t *acc_out) {
    ConvGeom g = geom(d, ho, wo);
    const int mult = d.c_out / d.c_in;
    const bool aligned4 = (uintptr_t)x % 4 == 0 && (uintptr_t)w_hwcm % 4 == 0 && (uintptr_t)y % 4 == 0;
    if (mult == 1 && !acc_out && be->cfg.conv_path != DW_PATH_DIRECT) {  // DIRECT: the register-fed kernels
        const int v = be->cfg.dw_variant;
        if (v != DW_DWV_SLAB) {
            // auto: the 2-column streaming kernel with 18 consumer warps (fastest measured)
            const int shape = v == DW_DWV_STREAM2X2 ? 1 : v == DW_DWV_STREAM4 ? 2 : 0;
            const dw_status st = launch_dwconv3x3_stream_i8(be, d, ho, wo, x, w_hwcm, ep, y, shape);
            if (st != DW_ERR_UNSUPPORTED) return st;
        }
        const dw_status st = launch_dwconv3x3_tma_i8(be, d, ho, wo, x, w_hwcm, ep, y);
        if (st != DW_ERR_UNSUPPORTED) return st;
    }
    if (mult == 1 && !acc_out && d.c_in % 4 == 0 && aligned4 && d.k_h == 3 && d.k_w == 3 && d.stride_h == 1 &&
        d.stride_w == 1) {
        constexpr int SEG = 28;
        const long long threads = (long long)(d.c_in / 4) * ((wo + 3) / 4) * ((ho + SEG - 1) / SEG) * d.n;
        if (threads < (1ll << 31) - 256 && (long long)d.h * d.w * d.c_in < (1ll << 31)) {
            const unsigned blocks = (unsigned)((threads + 127) / 128);
            k_dwconv3x3_s1_dp4a<SEG><<<blocks, 128, 0, be->stream>>>(g, x, w_hwcm, ep, y);
            return dw_after_launch(be, "dwconv3x3_s1_dp4a_i8");
        }
    }
    if (mult == 1 && !acc_out && d.c_in % 4 == 0 && aligned4 && d.k_h == 3 && d.k_w == 3 &&
        d.stride_h == d.stride_w && (d.stride_h == 1 || d.stride_h == 2)) {
        constexpr int RH = 2, RW = 4;
        const long long gy = (long long)d.n * ((ho + RH - 1) / RH);
        if (gy <= 65535 && (long long)d.h * d.w * d.c_in < (1ll << 31)) {
            dim3 grid((unsigned)((d.c_in / 4 + 31) / 32), (unsigned)gy);
            dim3 block(32, 8);
            if (d.stride_h == 1)
                k_dwconv3x3<1, RH, RW><<<grid, block, 0, be->stream>>>(g, x, w_hwcm, ep, y);
            else
                k_dwconv3x3<2, RH, RW><<<grid, block, 0, be->stream>>>(g, x, w_hwcm, ep, y);
            return dw_after_launch(be, "dwconv3x3_i8");
        }
    }
    if (mult == 1 && !acc_out && d.c_in % 16 == 0 && (uintptr_t)x % 16 == 0 && (uintptr_t)w_hwcm % 16 == 0 &&
        (uintptr_t)y % 16 == 0) {
        size_t items = (size_t)d.n * ho * wo * (d.c_in / 16);
        k_dwconv16<<<grid_for(be, items), kThreads, 0, be->stream>>>(g, x, w_hwcm, ep, y);
        return dw_after_launch(be, "dwconv_i8_vec16");
    }
    size_t items = (size_t)d.n * ho * wo * d.c_out;
    k_dwconv_generic<<<grid_for(be, items), kThreads, 0, be->stream>>>(g, mult, x, w_hwcm, ep, y, acc_out);
    return dw_after_launch(be, "dwconv_i8");
}

}  // namespace dw
