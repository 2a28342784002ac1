// fp16.cu -- CUDA-core kernels of the fp16 path: the direct and depthwise
// convolutions (shapes the tensor-core kernel does not take), and the
// HBM-bound glue: add (+ReLU), ReLU, max pool, global average pool and the
// f32 <-> f16 casts.
//
// Each kernel follows one CPU op of the reference operation for operation and
// converts with f16_to_f32_ref / f32_to_f16_ref (the reference's F16
// conversions), so its outputs equal the CPU op's bit for bit.  Streaming
// kernels move 16 bytes (8 halves) per thread per step when the buffers allow.

#include "dw_device.cuh"

namespace dw {
namespace {

constexpr int kThreads = 256;

inline int grid_for(const dw_backend *be, size_t work_items) {
    size_t blocks = (work_items + kThreads - 1) / kThreads;
    size_t cap = (size_t)be->sm_count * 8;
    if (blocks > cap) blocks = cap;
    if (blocks < 1) blocks = 1;
    return (int)blocks;
}

// Conv output element -> f16, then the bias as the CPU runtime adds it (the
// stored f16 converted back, plus the f16 bias, rounded again:
// crates/dragonwing-onnx/src/runtime.rs:1483-1497), then ReLU as relu_fp16
// (crates/dragonwing-cpu/src/ops.rs:345-352).
__device__ __forceinline__ uint16_t conv_finish_f16(float acc, const uint16_t *bias, int oc, int relu) {
    uint16_t o = f32_to_f16_ref(acc);
    if (bias) o = f32_to_f16_ref(__fadd_rn(f16_to_f32_ref(o), f16_to_f32_ref(__ldg(bias + oc))));
    if (relu) {
        const float f = f16_to_f32_ref(o);
        o = f32_to_f16_ref(f > 0.0f ? f : 0.0f);
    }
    return o;
}

// conv2d_fp16_nhwc (crates/dragonwing-cpu/src/ops.rs:1442-1511): per output an
// f32 accumulator updated by fused multiply-adds (`mul_add`) in (kh, kw, ic)
// order over the taps that fall inside the input (taps in the padding are
// skipped, not multiplied by zero).  One thread per output element, channels
// fastest; weights OHWI [c_out][kh*kw][c_in].
__global__ void k_conv_direct_f16(const uint16_t *__restrict__ x, const uint16_t *__restrict__ w,
                                  const uint16_t *__restrict__ bias, uint16_t *__restrict__ y, int n, int h, int wd,
                                  int c_in, int c_out, int kh, int kw, int sh, int sw, int pt, int pl, int ho, int wo,
                                  int relu) {
    const size_t total = (size_t)n * ho * wo * c_out;
    for (size_t i = blockIdx.x * (size_t)blockDim.x + threadIdx.x; i < total; i += (size_t)gridDim.x * blockDim.x) {
        const int oc = (int)(i % c_out);
        size_t p = i / c_out;
        const int ow = (int)(p % wo);
        p /= wo;
        const int oh = (int)(p % ho);
        const int b = (int)(p / ho);
        const uint16_t *wr = w + (size_t)oc * kh * kw * c_in;
        float acc = 0.0f;
        for (int a = 0; a < kh; a++) {
            const int ih = oh * sh + a - pt;
            if (ih < 0 || ih >= h) continue;
            for (int q = 0; q < kw; q++) {
                const int iw = ow * sw + q - pl;
                if (iw < 0 || iw >= wd) continue;
                const uint16_t *xp = x + (((size_t)b * h + ih) * wd + iw) * c_in;
                const uint16_t *wp = wr + (size_t)(a * kw + q) * c_in;
                for (int ic = 0; ic < c_in; ic++)
                    acc = __fmaf_rn(f16_to_f32_ref(__ldg(xp + ic)), f16_to_f32_ref(__ldg(wp + ic)), acc);
            }
        }
        y[i] = conv_finish_f16(acc, bias, oc, relu);
    }
}

// depthwise_conv2d_fp16_nhwc (ops.rs:2819-2937): kernel [kh][kw][C][mult], output
// channel oc = ic * mult + m reads input channel ic; FMA in (kh, kw) order.
__global__ void k_dwconv_f16(const uint16_t *__restrict__ x, const uint16_t *__restrict__ w,
                             const uint16_t *__restrict__ bias, uint16_t *__restrict__ y, int n, int h, int wd,
                             int c_in, int mult, int kh, int kw, int sh, int sw, int pt, int pl, int ho, int wo,
                             int relu) {
    const int c_out = c_in * mult;
    const size_t total = (size_t)n * ho * wo * c_out;
    for (size_t i = blockIdx.x * (size_t)blockDim.x + threadIdx.x; i < total; i += (size_t)gridDim.x * blockDim.x) {
        const int oc = (int)(i % c_out);
        const int ic = oc / mult;
        size_t p = i / c_out;
        const int ow = (int)(p % wo);
        p /= wo;
        const int oh = (int)(p % ho);
        const int b = (int)(p / ho);
        float acc = 0.0f;
        for (int a = 0; a < kh; a++) {
            const int ih = oh * sh + a - pt;
            if (ih < 0 || ih >= h) continue;
            for (int q = 0; q < kw; q++) {
                const int iw = ow * sw + q - pl;
                if (iw < 0 || iw >= wd) continue;
                const float xv = f16_to_f32_ref(__ldg(x + (((size_t)b * h + ih) * wd + iw) * c_in + ic));
                const float wv = f16_to_f32_ref(__ldg(w + (size_t)(a * kw + q) * c_out + oc));
                acc = __fmaf_rn(xv, wv, acc);
            }
        }
        y[i] = conv_finish_f16(acc, bias, oc, relu);
    }
}

// add_fp16 (ops.rs:434-446): y = from_f32(to_f32(a) + to_f32(b)); with `relu`,
// followed by relu_fp16 on the stored result (the graph's Add -> Relu pair).
__device__ __forceinline__ uint16_t add_one_f16(uint16_t a, uint16_t b, int relu) {
    uint16_t o = f32_to_f16_ref(__fadd_rn(f16_to_f32_ref(a), f16_to_f32_ref(b)));
    if (relu) {
        const float f = f16_to_f32_ref(o);
        o = f32_to_f16_ref(f > 0.0f ? f : 0.0f);
    }
    return o;
}

__device__ __forceinline__ uint16_t relu_one_f16(uint16_t a) {
    const float f = f16_to_f32_ref(a);
    return f32_to_f16_ref(f > 0.0f ? f : 0.0f);
}

__device__ __forceinline__ uint32_t lo16(uint32_t v) { return v & 0xFFFFu; }

__device__ __forceinline__ uint32_t add_pair(uint32_t a, uint32_t b, int relu) {
    return (uint32_t)add_one_f16((uint16_t)lo16(a), (uint16_t)lo16(b), relu) |
           ((uint32_t)add_one_f16((uint16_t)(a >> 16), (uint16_t)(b >> 16), relu) << 16);
}

__device__ __forceinline__ uint32_t relu_pair(uint32_t a) {
    return (uint32_t)relu_one_f16((uint16_t)lo16(a)) | ((uint32_t)relu_one_f16((uint16_t)(a >> 16)) << 16);
}

// n halves; `vec` = 1 when all three pointers are 16-byte aligned (8 halves per
// step, scalar tail), else scalar throughout.  `b` null = ReLU only.
__global__ void k_add_relu_f16(const uint16_t *a, const uint16_t *__restrict__ b, uint16_t *y, size_t n, int relu,
                               int vec) {  // a may alias y (in-place)
    const size_t tid = blockIdx.x * (size_t)blockDim.x + threadIdx.x;
    const size_t stride = (size_t)gridDim.x * blockDim.x;
    size_t head = 0;
    if (vec) {
        const size_t nv = n / 8;
        const uint4 *av = reinterpret_cast<const uint4 *>(a);
        const uint4 *bv = reinterpret_cast<const uint4 *>(b);
        uint4 *yv = reinterpret_cast<uint4 *>(y);
        for (size_t i = tid; i < nv; i += stride) {
            const uint4 u = av[i];
            uint4 r;
            if (b) {
                const uint4 v = __ldg(bv + i);
                r = make_uint4(add_pair(u.x, v.x, relu), add_pair(u.y, v.y, relu), add_pair(u.z, v.z, relu),
                               add_pair(u.w, v.w, relu));
            } else {
                r = make_uint4(relu_pair(u.x), relu_pair(u.y), relu_pair(u.z), relu_pair(u.w));
            }
            yv[i] = r;
        }
        head = nv * 8;
    }
    for (size_t i = head + tid; i < n; i += stride) y[i] = b ? add_one_f16(a[i], b[i], relu) : relu_one_f16(a[i]);
}

// Max pool as the CPU runtime runs it for F16 (runtime.rs:1545-1563): to_f32,
// maxpool2d_f32_nhwc (ops.rs:1513-1551: start at -inf, f32::max over the
// window), from_f32.  Taps in the padding are skipped (ONNX pads).
__global__ void k_maxpool_f16(const uint16_t *__restrict__ x, uint16_t *__restrict__ y, int n, int h, int w, int c,
                              int kh, int kw, int sh, int sw, int pt, int pl, int ho, int wo) {
    const size_t total = (size_t)n * ho * wo * c;
    for (size_t i = blockIdx.x * (size_t)blockDim.x + threadIdx.x; i < total; i += (size_t)gridDim.x * blockDim.x) {
        const int ch = (int)(i % c);
        size_t p = i / c;
        const int ow = (int)(p % wo);
        p /= wo;
        const int oh = (int)(p % ho);
        const int b = (int)(p / ho);
        float m = -INFINITY;
        for (int a = 0; a < kh; a++) {
            const int ih = oh * sh + a - pt;
            if (ih < 0 || ih >= h) continue;
            for (int q = 0; q < kw; q++) {
                const int iw = ow * sw + q - pl;
                if (iw < 0 || iw >= w) continue;
                m = fmaxf(m, f16_to_f32_ref(__ldg(x + (((size_t)b * h + ih) * w + iw) * c + ch)));
            }
        }
        y[i] = f32_to_f16_ref(m);
    }
}

// Same max pool, 8 channels per thread (c % 8 == 0, 16-byte aligned buffers):
// the max of F16::to_f32 values is F16::to_f32 of the max in f16 order
// (to_f32 is monotonic: it only halves subnormals, which stay below every
// normal value), and __hmax2 ignores a NaN operand like f32::max; the result
// then goes through to_f32 / from_f32 as the CPU does, which only changes a
// nonzero subnormal.
__global__ void k_maxpool_f16_v8(const uint4 *__restrict__ x, uint4 *__restrict__ y, int n, int h, int w, int cg,
                                 int kh, int kw, int sh, int sw, int pt, int pl, int ho, int wo) {
    const size_t total = (size_t)n * ho * wo * cg;
    for (size_t i = blockIdx.x * (size_t)blockDim.x + threadIdx.x; i < total; i += (size_t)gridDim.x * blockDim.x) {
        const int g = (int)(i % cg);
        size_t p = i / cg;
        const int ow = (int)(p % wo);
        p /= wo;
        const int oh = (int)(p % ho);
        const int b = (int)(p / ho);
        __half2 m[4];
        const __half2 ninf = __halves2half2(__ushort_as_half(0xFC00), __ushort_as_half(0xFC00));
        for (int k = 0; k < 4; k++) m[k] = ninf;
        for (int a = 0; a < kh; a++) {
            const int ih = oh * sh + a - pt;
            if (ih < 0 || ih >= h) continue;
            for (int q = 0; q < kw; q++) {
                const int iw = ow * sw + q - pl;
                if (iw < 0 || iw >= w) continue;
                const uint4 v = __ldg(x + (((size_t)b * h + ih) * w + iw) * cg + g);
                const uint32_t vv[4] = {v.x, v.y, v.z, v.w};
                for (int k = 0; k < 4; k++) m[k] = __hmax2(m[k], *reinterpret_cast<const __half2 *>(&vv[k]));
            }
        }
        uint32_t o[4];
        for (int k = 0; k < 4; k++) {
            uint32_t u = *reinterpret_cast<uint32_t *>(&m[k]);
            const uint16_t lo = (uint16_t)(u & 0xFFFFu), hi = (uint16_t)(u >> 16);
            const bool slo = (lo & 0x7C00u) == 0 && (lo & 0x03FFu), shi = (hi & 0x7C00u) == 0 && (hi & 0x03FFu);
            if (slo || shi)
                u = (uint32_t)f32_to_f16_ref(f16_to_f32_ref(lo)) | ((uint32_t)f32_to_f16_ref(f16_to_f32_ref(hi)) << 16);
            o[k] = u;
        }
        y[i] = make_uint4(o[0], o[1], o[2], o[3]);
    }
}

// Horizontal unfold of an f32 NHWC image into f16 (F16::from_f32), fused
// with the input conversion: y[n][r][j][q*c + ch] = x[n][r][j*sw + q - pl][ch]
// for q < kw (0 outside the image), channels kw*c .. c_dst-1 zero.  A k_h x
// k_w conv with horizontal stride sw on x equals a k_h x 1 conv with
// horizontal stride 1 on y whose kernel rows hold the k_w taps side by side:
// the same products, with whole rows of kw*c channels per tap for the
// tensor-core loads instead of c (= 3 for an image) channels.
__global__ void k_unfold_w_f32_to_f16(const float *__restrict__ x, uint16_t *__restrict__ y, int n, int h, int w,
                                      int c, int kw, int sw, int pl, int wo, int c_dst) {
    // One thread per output pixel (n, r, j): its kw*c values are the contiguous
    // run x[n][r][j*sw - pl ..][*] of the input row (k = q*c + ch indexes it
    // directly), zero where the run leaves the row.
    const size_t total = (size_t)n * h * wo;
    const int kc = kw * c, row_len = w * c;
    for (size_t i = blockIdx.x * (size_t)blockDim.x + threadIdx.x; i < total; i += (size_t)gridDim.x * blockDim.x) {
        const int j = (int)(i % wo);
        const size_t row = i / wo;  // n * h + r
        const float *xr = x + row * (size_t)row_len;
        const int base = (j * sw - pl) * c;
        uint4 *dst = reinterpret_cast<uint4 *>(y + i * (size_t)c_dst);
        for (int g = 0; g < c_dst; g += 8) {
            uint32_t o[4];
#pragma unroll
            for (int k2 = 0; k2 < 4; k2++) {
                uint32_t pair = 0;
#pragma unroll
                for (int e = 0; e < 2; e++) {
                    const int k = g + 2 * k2 + e, idx = base + k;
                    const uint16_t hv =
                        (k < kc && idx >= 0 && idx < row_len) ? f32_to_f16_ref(__ldg(xr + idx)) : (uint16_t)0;
                    pair |= (uint32_t)hv << (16 * e);
                }
                o[k2] = pair;
            }
            dst[g / 8] = make_uint4(o[0], o[1], o[2], o[3]);
        }
    }
}

// GlobalAveragePool F16 (runtime.rs:1155-1170): per (image, channel) a sequential
// f32 sum over rows then columns, divided by h*w, stored as f16; output [n][c].
__global__ void k_gap_f16(const uint16_t *__restrict__ x, uint16_t *__restrict__ y, int n, int h, int w, int c) {
    const size_t total = (size_t)n * c;
    const float spatial = (float)(h * w);
    for (size_t i = blockIdx.x * (size_t)blockDim.x + threadIdx.x; i < total; i += (size_t)gridDim.x * blockDim.x) {
        const int ch = (int)(i % c);
        const size_t b = i / c;
        const uint16_t *xp = x + b * (size_t)h * w * c + ch;
        float sum = 0.0f;
        for (int q = 0; q < h * w; q++) sum = __fadd_rn(sum, f16_to_f32_ref(__ldg(xp + (size_t)q * c)));
        y[i] = f32_to_f16_ref(__fdiv_rn(sum, spatial));
    }
}

// f32 [pixels][c_src] -> f16 [pixels][c_dst] with F16::from_f32 (the runtime's
// input conversion, runtime.rs:842-851); channels c_src..c_dst-1 are zero (the
// channel padding that lets a 3-channel image feed the tensor-core kernel).
__global__ void k_cast_f32_to_f16(const float *__restrict__ x, uint16_t *__restrict__ y, size_t pixels, int c_src,
                                  int c_dst) {
    const size_t total = pixels * c_dst;
    for (size_t i = blockIdx.x * (size_t)blockDim.x + threadIdx.x; i < total; i += (size_t)gridDim.x * blockDim.x) {
        const int ch = (int)(i % c_dst);
        const size_t p = i / c_dst;
        y[i] = ch < c_src ? f32_to_f16_ref(__ldg(x + p * c_src + ch)) : (uint16_t)0;
    }
}

__global__ void k_cast_f16_to_f32(const uint16_t *__restrict__ x, float *__restrict__ y, size_t n) {
    for (size_t i = blockIdx.x * (size_t)blockDim.x + threadIdx.x; i < n; i += (size_t)gridDim.x * blockDim.x)
        y[i] = f16_to_f32_ref(__ldg(x + i));
}

inline bool al16(const void *p) { return ((uintptr_t)p & 15) == 0; }

}  // namespace

dw_status launch_conv_direct_f16(dw_backend *be, const dw_conv_desc &d, int ho, int wo, const uint16_t *x,
                                 const uint16_t *w_ohwi, const uint16_t *bias, int relu, uint16_t *y) {
    const size_t items = (size_t)d.n * ho * wo * d.c_out;
    k_conv_direct_f16<<<grid_for(be, items), kThreads, 0, be->stream>>>(x, w_ohwi, bias, y, d.n, d.h, d.w, d.c_in,
                                                                         d.c_out, d.k_h, d.k_w, d.stride_h, d.stride_w,
                                                                         d.pad_t, d.pad_l, ho, wo, relu);
    return dw_after_launch(be, "conv_direct_f16");
}

dw_status launch_dwconv_f16(dw_backend *be, const dw_conv_desc &d, int ho, int wo, const uint16_t *x,
                            const uint16_t *w_hwcm, const uint16_t *bias, int relu, uint16_t *y) {
    const size_t items = (size_t)d.n * ho * wo * d.c_out;
    k_dwconv_f16<<<grid_for(be, items), kThreads, 0, be->stream>>>(x, w_hwcm, bias, y, d.n, d.h, d.w, d.c_in,
                                                                    d.c_out / d.c_in, d.k_h, d.k_w, d.stride_h,
                                                                    d.stride_w, d.pad_t, d.pad_l, ho, wo, relu);
    return dw_after_launch(be, "dwconv_f16");
}

dw_status launch_add_f16(dw_backend *be, const uint16_t *a, const uint16_t *b, uint16_t *y, size_t n, int relu) {
    const int vec = al16(a) && al16(b) && al16(y) ? 1 : 0;
    k_add_relu_f16<<<grid_for(be, vec ? n / 8 + 1 : n), kThreads, 0, be->stream>>>(a, b, y, n, relu, vec);
    return dw_after_launch(be, "add_f16");
}

dw_status launch_relu_f16(dw_backend *be, const uint16_t *x, uint16_t *y, size_t n) {
    const int vec = al16(x) && al16(y) ? 1 : 0;
    k_add_relu_f16<<<grid_for(be, vec ? n / 8 + 1 : n), kThreads, 0, be->stream>>>(x, nullptr, y, n, 1, vec);
    return dw_after_launch(be, "relu_f16");
}

dw_status launch_maxpool_f16(dw_backend *be, const uint16_t *x, uint16_t *y, int n, int h, int w, int c, int kh,
                             int kw, int sh, int sw, int pt, int pl, int ho, int wo) {
    if (c % 8 == 0 && al16(x) && al16(y)) {
        const size_t items = (size_t)n * ho * wo * (c / 8);
        k_maxpool_f16_v8<<<grid_for(be, items), kThreads, 0, be->stream>>>(
            reinterpret_cast<const uint4 *>(x), reinterpret_cast<uint4 *>(y), n, h, w, c / 8, kh, kw, sh, sw, pt, pl,
            ho, wo);
        return dw_after_launch(be, "maxpool_f16");
    }
    const size_t items = (size_t)n * ho * wo * c;
    k_maxpool_f16<<<grid_for(be, items), kThreads, 0, be->stream>>>(x, y, n, h, w, c, kh, kw, sh, sw, pt, pl, ho, wo);
    return dw_after_launch(be, "maxpool_f16");
}

dw_status launch_gap_f16(dw_backend *be, const uint16_t *x, uint16_t *y, int n, int h, int w, int c) {
    k_gap_f16<<<grid_for(be, (size_t)n * c), kThreads, 0, be->stream>>>(x, y, n, h, w, c);
    return dw_after_launch(be, "global_avgpool_f16");
}

dw_status launch_cast_f32_to_f16(dw_backend *be, const float *x, uint16_t *y, size_t pixels, int c_src, int c_dst) {
    k_cast_f32_to_f16<<<grid_for(be, pixels * c_dst), kThreads, 0, be->stream>>>(x, y, pixels, c_src, c_dst);
    return dw_after_launch(be, "cast_f32_to_f16");
}

dw_status launch_unfold_w_f32_to_f16(dw_backend *be, const float *x, uint16_t *y, int n, int h, int w, int c, int kw,
                                    int sw, int pl, int wo, int c_dst) {
    const size_t items = (size_t)n * h * wo;
    k_unfold_w_f32_to_f16<<<grid_for(be, items), kThreads, 0, be->stream>>>(x, y, n, h, w, c, kw, sw, pl, wo, c_dst);
    return dw_after_launch(be, "unfold_w_f32_to_f16");
}

dw_status launch_cast_f16_to_f32(dw_backend *be, const uint16_t *x, float *y, size_t n) {
    k_cast_f16_to_f32<<<grid_for(be, n), kThreads, 0, be->stream>>>(x, y, n);
    return dw_after_launch(be, "cast_f16_to_f32");
}

}  // namespace dw
