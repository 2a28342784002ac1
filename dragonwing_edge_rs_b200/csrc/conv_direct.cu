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
            y[i] = (int8_t)epilogue_one(acc, bias, m, dsc, ep.epilogue, ep.q6, ep.inv_s_out);
        }
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
                packed |= (uint32_t)(uint8_t)epilogue_one(acc[v * 4 + k], bias, m, dsc, ep.epilogue, ep.q6,
                                                          ep.inv_s_out)
                          << (8 * k);
            }
            outw[v] = packed;
        }
        *reinterpret_cast<int4 *>(y + p * g.c_in + cg * 16) = make_int4(outw[0], outw[1], outw[2], outw[3]);
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
            y[i] = (int8_t)epilogue_one(acc, bias, mm, dsc, ep.epilogue, ep.q6, ep.inv_s_out);
        }
    }
}

ConvGeom geom(const dw_conv_desc &d, int ho, int wo) {
    return ConvGeom{d.n, d.h, d.w, d.c_in, d.c_out, d.k_h, d.k_w, d.stride_h, d.stride_w, d.pad_t, d.pad_l, ho, wo};
}

}  // namespace

dw_status launch_conv_direct_i8(dw_backend *be, const dw_conv_desc &d, int ho, int wo, const int8_t *x,
                                const int8_t *w_ohwi, const EpiParams &ep, int8_t *y, int32_t *acc_out) {
    ConvGeom g = geom(d, ho, wo);
    size_t items = (size_t)d.n * ho * wo * d.c_out;
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
