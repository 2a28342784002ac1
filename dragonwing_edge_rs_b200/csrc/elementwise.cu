// elementwise.cu -- HBM-bound int8 kernels: requantize, relu, add, quantize,
// dequantize, and the data-movement glue (concat, channel slice, nearest
// resize, maxpool), plus the weight repack kernels.
//
// All streaming kernels move 16 bytes per thread per step (128-bit loads and
// stores) over a grid-stride loop sized to a multiple of the SM count, with a
// scalar tail for lengths that are not multiples of 16.

#include <cmath>

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

__device__ __forceinline__ bool aligned16(const void *p) { return ((uintptr_t)p & 15) == 0; }

// Division of n < 2^31 by a run-time constant d (1 <= d < 2^31), exact and
// without a divide: a shift for a power of two, else n / d = umulhi(n, m) >> l
// with l = floor(log2 d) and m = ceil(2^(32+l) / d) (m < 2^32).  The error term
// n * (m*d - 2^(32+l)) / (d * 2^(32+l)) stays below 1/d because
// m*d - 2^(32+l) < d < 2^(l+1) and n < 2^31.  The glue kernels index with it in
// 32 bits (a 64-bit divide costs about a hundred instructions per element).
struct FastDiv {
    uint32_t d, m, l, pow2;
};
inline FastDiv make_fastdiv(uint32_t d) {
    FastDiv f{d, 0u, (uint32_t)(31 - __builtin_clz(d)), (d & (d - 1)) == 0 ? 1u : 0u};
    if (!f.pow2) f.m = (uint32_t)((((uint64_t)1 << (32 + f.l)) + d - 1) / d);
    return f;
}
__device__ __forceinline__ uint32_t fdiv(uint32_t n, const FastDiv &f) {
    return f.pow2 ? (n >> f.l) : (__umulhi(n, f.m) >> f.l);
}

template <int kVec>
__device__ __forceinline__ void copy_vec(int8_t *dst, const int8_t *src) {
    if (kVec == 16) *reinterpret_cast<int4 *>(dst) = *reinterpret_cast<const int4 *>(src);
    else if (kVec == 8) *reinterpret_cast<int2 *>(dst) = *reinterpret_cast<const int2 *>(src);
    else if (kVec == 4) *reinterpret_cast<int *>(dst) = *reinterpret_cast<const int *>(src);
    else *dst = *src;
}

// --- requantize: ops.rs:3380-3386 -----------------------------------------
__global__ void k_requantize(const int32_t *__restrict__ in, int8_t *__restrict__ out, size_t n, float s) {
    size_t tid = blockIdx.x * (size_t)blockDim.x + threadIdx.x, stride = (size_t)gridDim.x * blockDim.x;
    size_t n16 = (aligned16(in) && aligned16(out)) ? n / 16 : 0;
    for (size_t i = tid; i < n16; i += stride) {
        const int4 *src = reinterpret_cast<const int4 *>(in + i * 16);
        uint32_t packed[4];
#pragma unroll
        for (int v = 0; v < 4; v++) {
            int4 q = __ldcs(src + v);
            uint32_t b0 = (uint8_t)f32_to_i8(__fmul_rn(i2f_rn(q.x), s));
            uint32_t b1 = (uint8_t)f32_to_i8(__fmul_rn(i2f_rn(q.y), s));
            uint32_t b2 = (uint8_t)f32_to_i8(__fmul_rn(i2f_rn(q.z), s));
            uint32_t b3 = (uint8_t)f32_to_i8(__fmul_rn(i2f_rn(q.w), s));
            packed[v] = b0 | (b1 << 8) | (b2 << 16) | (b3 << 24);
        }
        __stcs(reinterpret_cast<int4 *>(out + i * 16), make_int4(packed[0], packed[1], packed[2], packed[3]));
    }
    for (size_t i = n16 * 16 + tid; i < n; i += stride) out[i] = (int8_t)f32_to_i8(__fmul_rn(i2f_rn(in[i]), s));
}

// --- relu: ops.rs:3315-3319 ------------------------------------------------
__global__ void k_relu_i8(const int8_t *__restrict__ in, int8_t *__restrict__ out, size_t n) {
    size_t tid = blockIdx.x * (size_t)blockDim.x + threadIdx.x, stride = (size_t)gridDim.x * blockDim.x;
    size_t n16 = (aligned16(in) && aligned16(out)) ? n / 16 : 0;
    for (size_t i = tid; i < n16; i += stride) {
        int4 v = __ldcs(reinterpret_cast<const int4 *>(in) + i);
        v.x = __vmaxs4(v.x, 0); v.y = __vmaxs4(v.y, 0); v.z = __vmaxs4(v.z, 0); v.w = __vmaxs4(v.w, 0);
        __stcs(reinterpret_cast<int4 *>(out) + i, v);
    }
    for (size_t i = n16 * 16 + tid; i < n; i += stride) out[i] = in[i] > 0 ? in[i] : 0;
}

// --- add: ops.rs:3197-3209 (two RN multiplies, one RN add; add4 / add16_fast in dw_device.cuh) ---
__global__ void k_add_i8(const int8_t *__restrict__ a, const int8_t *__restrict__ b, int8_t *__restrict__ out,
                         size_t n, float ra, float rb) {
    size_t tid = blockIdx.x * (size_t)blockDim.x + threadIdx.x, stride = (size_t)gridDim.x * blockDim.x;
    size_t n16 = (aligned16(a) && aligned16(b) && aligned16(out)) ? n / 16 : 0;
    for (size_t i = tid; i < n16; i += stride) {
        int4 va = __ldcs(reinterpret_cast<const int4 *>(a) + i);
        int4 vb = __ldcs(reinterpret_cast<const int4 *>(b) + i);
        int4 r;
        r.x = add4(va.x, vb.x, ra, rb); r.y = add4(va.y, vb.y, ra, rb);
        r.z = add4(va.z, vb.z, ra, rb); r.w = add4(va.w, vb.w, ra, rb);
        __stcs(reinterpret_cast<int4 *>(out) + i, r);
    }
    for (size_t i = n16 * 16 + tid; i < n; i += stride) {
        float y = __fadd_rn(__fmul_rn(i2f_small(a[i]), ra), __fmul_rn(i2f_small(b[i]), rb));
        out[i] = (int8_t)f32_to_i8(y);
    }
}

__global__ void k_add_i8_fast(const int8_t *__restrict__ a, const int8_t *__restrict__ b, int8_t *__restrict__ out,
                              size_t n16, float ra, float rb) {
    const size_t tid = blockIdx.x * (size_t)blockDim.x + threadIdx.x, stride = (size_t)gridDim.x * blockDim.x;
    const float2 ra2 = make_float2(ra, ra), rb2 = make_float2(rb, rb);
    for (size_t i = tid; i < n16; i += stride) {
        const uint4 va = __ldcs(reinterpret_cast<const uint4 *>(a) + i);
        const uint4 vb = __ldcs(reinterpret_cast<const uint4 *>(b) + i);
        __stcs(reinterpret_cast<uint4 *>(out) + i, add16_fast(va, vb, ra2, rb2, ra, rb));
    }
}

// add_i8 over channel ranges of wider tensors: 16 channels of one pixel per
// step, the same exact arithmetic as k_add_i8_fast.
__global__ void k_add_i8_view(const int8_t *__restrict__ a, int a_pitch, const int8_t *__restrict__ b, int b_pitch,
                              int8_t *__restrict__ out, int out_pitch, uint32_t total, FastDiv fcg, float ra,
                              float rb) {
    const float2 ra2 = make_float2(ra, ra), rb2 = make_float2(rb, rb);
    for (uint32_t i = blockIdx.x * blockDim.x + threadIdx.x; i < total; i += gridDim.x * blockDim.x) {
        const uint32_t p = fdiv(i, fcg);
        const int c = (int)(i - p * fcg.d) * 16;
        const uint4 va = __ldcs(reinterpret_cast<const uint4 *>(a + (size_t)p * a_pitch + c));
        const uint4 vb = __ldcs(reinterpret_cast<const uint4 *>(b + (size_t)p * b_pitch + c));
        *reinterpret_cast<uint4 *>(out + (size_t)p * out_pitch + c) = add16_fast(va, vb, ra2, rb2, ra, rb);
    }
}

// --- quantize: ops.rs:3503-3525 (x * (1/scale)) -----------------------------
__global__ void k_quantize_f32(const float *__restrict__ in, int8_t *__restrict__ out, size_t n, float inv) {
    size_t tid = blockIdx.x * (size_t)blockDim.x + threadIdx.x, stride = (size_t)gridDim.x * blockDim.x;
    size_t n16 = (aligned16(in) && aligned16(out)) ? n / 16 : 0;
    for (size_t i = tid; i < n16; i += stride) {
        const float4 *src = reinterpret_cast<const float4 *>(in + i * 16);
        uint32_t packed[4];
#pragma unroll
        for (int v = 0; v < 4; v++) {
            float4 q = __ldcs(src + v);
            packed[v] = (uint32_t)(uint8_t)f32_to_i8(__fmul_rn(q.x, inv)) |
                        ((uint32_t)(uint8_t)f32_to_i8(__fmul_rn(q.y, inv)) << 8) |
                        ((uint32_t)(uint8_t)f32_to_i8(__fmul_rn(q.z, inv)) << 16) |
                        ((uint32_t)(uint8_t)f32_to_i8(__fmul_rn(q.w, inv)) << 24);
        }
        __stcs(reinterpret_cast<int4 *>(out + i * 16), make_int4(packed[0], packed[1], packed[2], packed[3]));
    }
    for (size_t i = n16 * 16 + tid; i < n; i += stride) out[i] = (int8_t)f32_to_i8(__fmul_rn(in[i], inv));
}

// u8 image -> f32 (u8 * (1/255)) -> quantize (x * (1/scale)): the YOLO input path.
__device__ __forceinline__ uint32_t quant_u8x4(uint32_t v, float inv255, float inv) {
    uint32_t r = 0;
#pragma unroll
    for (int k = 0; k < 4; k++) {
        float x = __fmul_rn(i2f_small((int32_t)((v >> (8 * k)) & 0xff)), inv255);
        r |= (uint32_t)(uint8_t)f32_to_i8(__fmul_rn(x, inv)) << (8 * k);
    }
    return r;
}

__global__ void k_quantize_u8(const uint8_t *__restrict__ in, int8_t *__restrict__ out, size_t n, float inv255,
                              float inv) {
    size_t tid = blockIdx.x * (size_t)blockDim.x + threadIdx.x, stride = (size_t)gridDim.x * blockDim.x;
    size_t n16 = (aligned16(in) && aligned16(out)) ? n / 16 : 0;
    for (size_t i = tid; i < n16; i += stride) {
        int4 v = __ldcs(reinterpret_cast<const int4 *>(in) + i);
        int4 r;
        r.x = quant_u8x4(v.x, inv255, inv); r.y = quant_u8x4(v.y, inv255, inv);
        r.z = quant_u8x4(v.z, inv255, inv); r.w = quant_u8x4(v.w, inv255, inv);
        __stcs(reinterpret_cast<int4 *>(out) + i, r);
    }
    for (size_t i = n16 * 16 + tid; i < n; i += stride)
        out[i] = (int8_t)f32_to_i8(__fmul_rn(__fmul_rn(i2f_small((int32_t)in[i]), inv255), inv));
}

// --- im2col of a uint8 image fused with its quantisation ---------------------
// y[b][i][j][(a * kw + q) * c + ch] = quant(x[b][i*sh + a - pt][j*sw + q - pl][ch])
// (0 in the padding and in channels kh*kw*c .. c_dst-1), quant(u) = the
// QuantizeU8 result for byte u (computed exactly as k_quantize_u8 does, once
// per block into a 256-entry table).  A conv of the quantised image equals a
// 1x1 conv of y with the kernel rows flattened in (kh, kw, c) order: the same
// integer products.
template <int C, int KH, int KW>  // C = 0: runtime c, kh, kw
__global__ void k_im2col_u8_i8(const uint8_t *__restrict__ x, int8_t *__restrict__ y, int n, int h, int w, int c_rt,
                               int kh_rt, int kw_rt, int sh, int sw, int pt, int pl, int ho, int wo, int c_dst,
                               float inv255, float inv) {
    __shared__ int8_t lut[256];
    for (int u = threadIdx.x; u < 256; u += blockDim.x)
        lut[u] = (int8_t)f32_to_i8(__fmul_rn(__fmul_rn(i2f_small(u), inv255), inv));
    __syncthreads();
    const int c = C ? C : c_rt, kh = C ? KH : kh_rt, kw = C ? KW : kw_rt;
    const size_t total = (size_t)n * ho * wo;
    for (size_t i = blockIdx.x * (size_t)blockDim.x + threadIdx.x; i < total; i += (size_t)gridDim.x * blockDim.x) {
        const int j = (int)(i % wo);
        const size_t t = i / wo;
        const int oi = (int)(t % ho);
        const int b = (int)(t / ho);
        const uint8_t *xb = x + (size_t)b * h * w * c;
        uint32_t wd[16] = {};  // up to 64 output bytes
        const int ih0 = oi * sh - pt, iw0 = j * sw - pl;
#pragma unroll
        for (int a = 0; a < (C ? KH : 8); a++) {
            if (!C && a >= kh) break;
            const int ih = ih0 + a;
            if (ih < 0 || ih >= h) continue;
#pragma unroll
            for (int q = 0; q < (C ? KW : 8); q++) {
                if (!C && q >= kw) break;
                const int iw = iw0 + q;
                if (iw < 0 || iw >= w) continue;
                const uint8_t *px = xb + ((size_t)ih * w + iw) * c;
#pragma unroll
                for (int ch = 0; ch < (C ? C : 8); ch++) {
                    if (!C && ch >= c) break;
                    const int k = (a * kw + q) * c + ch;
                    if (k < 64) wd[k >> 2] |= (uint32_t)(uint8_t)lut[__ldg(px + ch)] << (8 * (k & 3));
                }
            }
        }
        uint4 *dst = reinterpret_cast<uint4 *>(y + i * (size_t)c_dst);
#pragma unroll
        for (int g = 0; g < 4; g++)
            if (g * 16 < c_dst) dst[g] = make_uint4(wd[4 * g], wd[4 * g + 1], wd[4 * g + 2], wd[4 * g + 3]);
    }
}

// The 3-channel 3x3 stem (c_dst = 32, image width a multiple of 16): one block
// per output row.  The block quantises the three input rows it reads into
// shared memory once (16-byte loads, the same table), input byte e of a row at
// shared byte 16 + e with zeros around it (the padding, and rows outside the
// image); an output pixel's 27 bytes are then three runs of 9 bytes, taps
// (a, 0..2) x channels of row a being contiguous in the input row, read as
// three aligned words per row and packed into 8 words (the last 5 bytes 0).
__global__ void k_im2col_stem3_rows(const uint8_t *__restrict__ x, int8_t *__restrict__ y, int h, int w, int sh,
                                    int sw, int pt, int pl, int ho, int wo, int row_bytes, float inv255, float inv) {
    extern __shared__ __align__(16) uint8_t rows[];  // [3][row_bytes], row_bytes a multiple of 16
    __shared__ int8_t lut[256];
    for (int u = threadIdx.x; u < 256; u += blockDim.x)
        lut[u] = (int8_t)f32_to_i8(__fmul_rn(__fmul_rn(i2f_small(u), inv255), inv));
    __syncthreads();
    const int oi = blockIdx.x % ho, b = blockIdx.x / ho;
    const int units = row_bytes / 16, data_units = w * 3 / 16;
    for (int t = threadIdx.x; t < 3 * units; t += blockDim.x) {
        const int a = t / units, u = t % units;
        const int ih = oi * sh - pt + a;
        uint4 v = make_uint4(0u, 0u, 0u, 0u);
        if (u >= 1 && u <= data_units && ih >= 0 && ih < h) {
            const uint4 s = __ldg(reinterpret_cast<const uint4 *>(x + ((size_t)b * h + ih) * w * 3) + (u - 1));
            const uint32_t sw4[4] = {s.x, s.y, s.z, s.w};
            uint32_t q[4];
#pragma unroll
            for (int k = 0; k < 4; k++)
                q[k] = (uint32_t)(uint8_t)lut[sw4[k] & 0xff] | (uint32_t)(uint8_t)lut[(sw4[k] >> 8) & 0xff] << 8 |
                       (uint32_t)(uint8_t)lut[(sw4[k] >> 16) & 0xff] << 16 | (uint32_t)(uint8_t)lut[sw4[k] >> 24] << 24;
            v = make_uint4(q[0], q[1], q[2], q[3]);
        }
        *reinterpret_cast<uint4 *>(rows + a * row_bytes + u * 16) = v;
    }
    __syncthreads();
    int8_t *yrow = y + ((size_t)b * ho + oi) * wo * 32;
    for (int j = threadIdx.x; j < wo; j += blockDim.x) {
        const int s0 = 16 + (j * sw - pl) * 3;  // first of the 9 bytes, >= 16 - 3 * pl >= 1
        const int base = s0 & ~3, sh8 = (s0 & 3) * 8;
        uint32_t r[3][3];
#pragma unroll
        for (int a = 0; a < 3; a++) {
            const uint32_t *wp = reinterpret_cast<const uint32_t *>(rows + a * row_bytes + base);
            const uint32_t w0 = wp[0], w1 = wp[1], w2 = wp[2];
            r[a][0] = __funnelshift_r(w0, w1, sh8);
            r[a][1] = __funnelshift_r(w1, w2, sh8);
            r[a][2] = (w2 >> sh8) & 0xffu;
        }
        uint4 *dst = reinterpret_cast<uint4 *>(yrow + (size_t)j * 32);
        dst[0] = make_uint4(r[0][0], r[0][1], r[0][2] | r[1][0] << 8, r[1][0] >> 24 | r[1][1] << 8);
        dst[1] = make_uint4(r[1][1] >> 24 | r[1][2] << 8 | r[2][0] << 16, r[2][0] >> 16 | r[2][1] << 16,
                            r[2][1] >> 16 | r[2][2] << 16, 0u);
    }
}

// The same stem, one block per band of kStemBand output rows: the band's
// (kStemBand - 1) * sh + 3 input rows are quantised into shared memory once
// (rows shared by neighbouring output rows are not re-read), then the band's
// pixels are packed as in k_im2col_stem3_rows.  The quantisation table is
// replicated per lane (word (u / 4) * 32 + lane holds bytes u & ~3 .. | 3), so
// the 32 lanes of a lookup hit 32 different banks.
constexpr int kStemBand = 8;
__global__ void __launch_bounds__(256) k_im2col_stem3_band(const uint8_t *__restrict__ x, int8_t *__restrict__ y, int h,
                                                           int w, int sh, int sw, int pt, int pl, int ho, int wo,
                                                           int row_bytes, int nbands, float inv255, float inv) {
    extern __shared__ __align__(16) uint8_t rows[];  // [(kStemBand - 1) * sh + 3][row_bytes]
    __shared__ uint8_t q8[256];
    __shared__ uint32_t lutw[64 * 32];
    for (int u = threadIdx.x; u < 256; u += blockDim.x)
        q8[u] = (uint8_t)f32_to_i8(__fmul_rn(__fmul_rn(i2f_small(u), inv255), inv));
    __syncthreads();
    for (int i = threadIdx.x; i < 64 * 32; i += blockDim.x) {
        const int k = i >> 5;
        lutw[i] = (uint32_t)q8[4 * k] | (uint32_t)q8[4 * k + 1] << 8 | (uint32_t)q8[4 * k + 2] << 16 |
                  (uint32_t)q8[4 * k + 3] << 24;
    }
    __syncthreads();
    const uint8_t *lut = reinterpret_cast<const uint8_t *>(lutw) + (threadIdx.x & 31) * 4;
    auto quant4 = [&](uint32_t v) {
        uint32_t r = 0;
#pragma unroll
        for (int k = 0; k < 4; k++) {
            const uint32_t u = (v >> (8 * k)) & 0xFFu;
            r |= (uint32_t)lut[((u & 0xFCu) << 5) | (u & 3u)] << (8 * k);
        }
        return r;
    };
    const int band = blockIdx.x % nbands, b = blockIdx.x / nbands;
    const int i0 = band * kStemBand;
    const int nr = (kStemBand - 1) * sh + 3;
    const int units = row_bytes / 16, data_units = w * 3 / 16;
    const int ih0 = i0 * sh - pt;
    for (int t = threadIdx.x; t < nr * units; t += blockDim.x) {
        const int a = t / units, u = t - a * units;
        const int ih = ih0 + a;
        uint4 v = make_uint4(0u, 0u, 0u, 0u);
        if (u >= 1 && u <= data_units && ih >= 0 && ih < h) {
            const uint4 s = __ldg(reinterpret_cast<const uint4 *>(x + ((size_t)b * h + ih) * w * 3) + (u - 1));
            v = make_uint4(quant4(s.x), quant4(s.y), quant4(s.z), quant4(s.w));
        }
        *reinterpret_cast<uint4 *>(rows + a * row_bytes + u * 16) = v;
    }
    __syncthreads();
    for (int r = 0; r < kStemBand; r++) {
        const int oi = i0 + r;
        if (oi >= ho) break;
        int8_t *yrow = y + ((size_t)b * ho + oi) * wo * 32;
        const uint8_t *rr = rows + r * sh * row_bytes;
        for (int j = threadIdx.x; j < wo; j += blockDim.x) {
            const int s0 = 16 + (j * sw - pl) * 3;  // first of the 9 bytes, >= 16 - 3 * pl >= 1
            const int base = s0 & ~3, sh8 = (s0 & 3) * 8;
            uint32_t q[3][3];
#pragma unroll
            for (int a = 0; a < 3; a++) {
                const uint32_t *wp = reinterpret_cast<const uint32_t *>(rr + a * row_bytes + base);
                const uint32_t w0 = wp[0], w1 = wp[1], w2 = wp[2];
                q[a][0] = __funnelshift_r(w0, w1, sh8);
                q[a][1] = __funnelshift_r(w1, w2, sh8);
                q[a][2] = (w2 >> sh8) & 0xffu;
            }
            uint4 *dst = reinterpret_cast<uint4 *>(yrow + (size_t)j * 32);
            dst[0] = make_uint4(q[0][0], q[0][1], q[0][2] | q[1][0] << 8, q[1][0] >> 24 | q[1][1] << 8);
            dst[1] = make_uint4(q[1][1] >> 24 | q[1][2] << 8 | q[2][0] << 16, q[2][0] >> 16 | q[2][1] << 16,
                                q[2][1] >> 16 | q[2][2] << 16, 0u);
        }
    }
}

// Fused input stem: quantisation of a 3-channel uint8 image + 3x3 conv (any
// stride and padding the band staging covers) + bias + requantisation epilogue,
// one pass.  The band of input rows is staged and quantised in shared memory as
// in k_im2col_stem3_band; each thread then packs one output pixel's 27 taps in
// (kh, kw, c) order into 7 words (the im2col's packing) and takes every output
// channel as 7 __dp4a against that channel's staged weight words: the same
// exact int32 sums as the reference's conv over the quantised image
// (conv2d_i8_nhwc, ops.rs:2964-2995, the padding taps 0).  The epilogue is the
// fused op's (SiLU: the certified fast path with the exact fall-back per
// element, as the tensor-core epilogue; the others: epilogue_one).  The
// 27-channel im2col tensor never reaches memory: the unit reads the uint8
// image and writes the conv output once.
constexpr int kStemMaxCout = 64;
constexpr int kStemConvBand = 4;  // output rows per block
constexpr int kStemConvRowsBytes = 36 * 1024;  // dynamic shared memory: with ~11 KB static, within the 48 KB default
template <bool kSilu>
__global__ void __launch_bounds__(256, 4) k_stem3_conv(const uint8_t *__restrict__ x, const int8_t *__restrict__ w_hwio,
                                                    EpiParams ep, int8_t *__restrict__ y, int h, int w, int sh, int sw,
                                                    int pt, int pl, int ho, int wo, int c_out, int row_bytes,
                                                    int nbands, float inv255, float inv) {
    extern __shared__ __align__(16) uint8_t rows[];  // [(kStemConvBand - 1) * sh + 3][row_bytes]
    __shared__ uint8_t q8[256];
    __shared__ uint32_t lutw[64 * 32];
    __shared__ __align__(16) uint32_t wsm[kStemMaxCout * 8];  // [oc][k word]: taps 4k .. 4k + 3, zero past 26
    __shared__ __align__(16) int32_t bias_s[kStemMaxCout];
    __shared__ __align__(16) float par_s[kStemMaxCout];  // D (SiLU) or M
    __shared__ int fast_s;
    for (int u = threadIdx.x; u < 256; u += blockDim.x)
        q8[u] = (uint8_t)f32_to_i8(__fmul_rn(__fmul_rn(i2f_small(u), inv255), inv));
    for (int i = threadIdx.x; i < c_out * 8; i += blockDim.x) {
        const int oc = i >> 3, kw4 = i & 7;
        uint32_t v = 0;
#pragma unroll
        for (int b = 0; b < 4; b++) {
            const int k = kw4 * 4 + b;
            if (k < 27) v |= (uint32_t)(uint8_t)w_hwio[(size_t)k * c_out + oc] << (8 * b);
        }
        wsm[i] = v;
    }
    if (threadIdx.x == 0) fast_s = 1;
    __syncthreads();
    for (int oc = threadIdx.x; oc < c_out; oc += blockDim.x) {
        bias_s[oc] = ep.bias ? __ldg(ep.bias + oc) : 0;
        const float pv = kSilu ? (ep.D ? __ldg(ep.D + oc) : 0.0f) : (ep.M ? __ldg(ep.M + oc) : 0.0f);
        par_s[oc] = pv;
        if (kSilu && !(isfinite(pv) && isfinite(ep.inv_s_out))) fast_s = 0;
    }
    for (int i = threadIdx.x; i < 64 * 32; i += blockDim.x) {
        const int k = i >> 5;
        lutw[i] = (uint32_t)q8[4 * k] | (uint32_t)q8[4 * k + 1] << 8 | (uint32_t)q8[4 * k + 2] << 16 |
                  (uint32_t)q8[4 * k + 3] << 24;
    }
    __syncthreads();
    const uint8_t *lut = reinterpret_cast<const uint8_t *>(lutw) + (threadIdx.x & 31) * 4;
    auto quant4 = [&](uint32_t v) {
        uint32_t r = 0;
#pragma unroll
        for (int k = 0; k < 4; k++) {
            const uint32_t u = (v >> (8 * k)) & 0xFFu;
            r |= (uint32_t)lut[((u & 0xFCu) << 5) | (u & 3u)] << (8 * k);
        }
        return r;
    };
    const int band = blockIdx.x % nbands, b = blockIdx.x / nbands;
    const int i0 = band * kStemConvBand;
    const int nr = (kStemConvBand - 1) * sh + 3;
    const int units = row_bytes / 16, data_units = w * 3 / 16;
    const int ih0 = i0 * sh - pt;
    for (int t = threadIdx.x; t < nr * units; t += blockDim.x) {
        const int a = t / units, u = t - a * units;
        const int ih = ih0 + a;
        uint4 v = make_uint4(0u, 0u, 0u, 0u);
        if (u >= 1 && u <= data_units && ih >= 0 && ih < h) {
            const uint4 s = __ldg(reinterpret_cast<const uint4 *>(x + ((size_t)b * h + ih) * w * 3) + (u - 1));
            v = make_uint4(quant4(s.x), quant4(s.y), quant4(s.z), quant4(s.w));
        }
        *reinterpret_cast<uint4 *>(rows + a * row_bytes + u * 16) = v;
    }
    __syncthreads();
    const bool fast = fast_s != 0;
    const int groups = c_out >> 3;
    for (int r = 0; r < kStemConvBand; r++) {
        const int oi = i0 + r;
        if (oi >= ho) break;
        int8_t *yrow = y + ((size_t)b * ho + oi) * wo * c_out;
        const uint8_t *rr = rows + r * sh * row_bytes;
        for (int j = threadIdx.x; j < wo; j += blockDim.x) {
            const int s0 = 16 + (j * sw - pl) * 3;  // first of the 9 bytes, >= 16 - 3 * pl >= 1
            const int base = s0 & ~3, sh8 = (s0 & 3) * 8;
            uint32_t q[3][3];
#pragma unroll
            for (int a = 0; a < 3; a++) {
                const uint32_t *wp = reinterpret_cast<const uint32_t *>(rr + a * row_bytes + base);
                const uint32_t w0 = wp[0], w1 = wp[1], w2 = wp[2];
                q[a][0] = __funnelshift_r(w0, w1, sh8);
                q[a][1] = __funnelshift_r(w1, w2, sh8);
                q[a][2] = (w2 >> sh8) & 0xffu;
            }
            // the 27 taps in (kh, kw, c) order, 4 per word (the im2col's packing)
            const int X[7] = {(int)q[0][0], (int)q[0][1], (int)(q[0][2] | q[1][0] << 8),
                              (int)(q[1][0] >> 24 | q[1][1] << 8), (int)(q[1][1] >> 24 | q[1][2] << 8 | q[2][0] << 16),
                              (int)(q[2][0] >> 16 | q[2][1] << 16), (int)(q[2][1] >> 16 | q[2][2] << 16)};
            // eight output channels at a time (fewer live registers: more warps per SM)
            for (int g = 0; g < groups; g++) {
                int32_t acc[8];
#pragma unroll
                for (int o = 0; o < 8; o++) {
                    const uint4 wa = *reinterpret_cast<const uint4 *>(&wsm[(g * 8 + o) * 8]);
                    const uint4 wb = *reinterpret_cast<const uint4 *>(&wsm[(g * 8 + o) * 8 + 4]);
                    int32_t s = __dp4a(X[0], (int)wa.x, 0);
                    s = __dp4a(X[1], (int)wa.y, s);
                    s = __dp4a(X[2], (int)wa.z, s);
                    s = __dp4a(X[3], (int)wa.w, s);
                    s = __dp4a(X[4], (int)wb.x, s);
                    s = __dp4a(X[5], (int)wb.y, s);
                    acc[o] = __dp4a(X[6], (int)wb.z, s);
                }
                uint32_t wq[2] = {0u, 0u};
                const int c0 = g * 8;
                if (kSilu) {
                    int32_t av[8];
                    bool inr = true;
#pragma unroll
                    for (int k = 0; k < 8; k++) {
                        av[k] = (int32_t)((uint32_t)acc[k] + (uint32_t)bias_s[c0 + k]);
                        inr &= (uint32_t)(av[k] + (1 << 22)) < (1u << 23);
                    }
                    uint32_t unc = 0xFFu;
                    if (fast && inr) {
                        unc = 0;
#pragma unroll
                        for (int qq = 0; qq < 2; qq++) {
                            uint32_t bq[4];
#pragma unroll
                            for (int jj = 0; jj < 4; jj += 2) {
                                const int k = qq * 4 + jj;
                                bool u0 = false, u1 = false;
                                silu_fast_bits2(av[k], av[k + 1], par_s[c0 + k], par_s[c0 + k + 1], ep.inv_s_out, bq[jj],
                                                bq[jj + 1], u0, u1);
                                unc |= ((uint32_t)u0 | (uint32_t)u1 << 1) << k;
                            }
                            wq[qq] = __byte_perm(__byte_perm(bq[0], bq[1], 0x0040), __byte_perm(bq[2], bq[3], 0x0040),
                                                 0x5410);
                        }
                    }
                    if (unc) {
#pragma unroll
                        for (int k = 0; k < 8; k++) {
                            if (unc & (1u << k)) {
                                const uint32_t bb = (uint8_t)epilogue_one_slow(acc[k], bias_s[c0 + k], 0.0f, par_s[c0 + k],
                                                                               DW_EPI_SILU, ep.q6, ep.inv_s_out);
                                wq[k >> 2] = (wq[k >> 2] & ~(0xFFu << (8 * (k & 3)))) | (bb << (8 * (k & 3)));
                            }
                        }
                    }
                } else {
#pragma unroll
                    for (int k = 0; k < 8; k++)
                        wq[k >> 2] |= (uint32_t)(uint8_t)epilogue_one(acc[k], bias_s[c0 + k], par_s[c0 + k], 0.0f,
                                                                      ep.epilogue, ep.q6, ep.inv_s_out)
                                      << (8 * (k & 3));
                }
                *reinterpret_cast<uint2 *>(yrow + (size_t)j * c_out + c0) = make_uint2(wq[0], wq[1]);
            }
        }
    }
}

// --- dequantize: ops.rs:3453-3457 ---------------------------------------------
__global__ void k_dequantize(const int8_t *__restrict__ in, float *__restrict__ out, size_t n, float s) {
    size_t tid = blockIdx.x * (size_t)blockDim.x + threadIdx.x, stride = (size_t)gridDim.x * blockDim.x;
    size_t n16 = (aligned16(in) && aligned16(out)) ? n / 16 : 0;
    for (size_t i = tid; i < n16; i += stride) {
        int4 v = __ldcs(reinterpret_cast<const int4 *>(in) + i);
        uint32_t w[4] = {(uint32_t)v.x, (uint32_t)v.y, (uint32_t)v.z, (uint32_t)v.w};
        float4 *dst = reinterpret_cast<float4 *>(out + i * 16);
#pragma unroll
        for (int q = 0; q < 4; q++) {
            float4 f;
            f.x = __fmul_rn(i2f_small((int8_t)(w[q])), s);
            f.y = __fmul_rn(i2f_small((int8_t)(w[q] >> 8)), s);
            f.z = __fmul_rn(i2f_small((int8_t)(w[q] >> 16)), s);
            f.w = __fmul_rn(i2f_small((int8_t)(w[q] >> 24)), s);
            __stcs(dst + q, f);
        }
    }
    for (size_t i = n16 * 16 + tid; i < n; i += stride) out[i] = __fmul_rn(i2f_small(in[i]), s);
}

// --- maxpool (ops.rs:1513-1551, padded taps skipped) -------------------------
// One thread per (output pixel, 4-channel group) when c % 4 == 0, else per element.
__global__ void k_maxpool_i8(const int8_t *__restrict__ x, int8_t *__restrict__ y, int n, int h, int w, int c,
                             int kh, int kw, int sh, int sw, int pt, int pl, int ho, int wo, int vec) {
    const int cg = c / vec;
    const size_t total = (size_t)n * ho * wo * cg;
    for (size_t i = blockIdx.x * (size_t)blockDim.x + threadIdx.x; i < total; i += (size_t)gridDim.x * blockDim.x) {
        int g = (int)(i % cg);
        size_t p = i / cg;
        int ow = (int)(p % wo);
        size_t t = p / wo;
        int oh = (int)(t % ho);
        int b = (int)(t / ho);
        if (vec == 4) {
            uint32_t m = 0x80808080u;  // -128 x4
            for (int a = 0; a < kh; a++) {
                int ih = oh * sh + a - pt;
                if (ih < 0 || ih >= h) continue;
                for (int q = 0; q < kw; q++) {
                    int iw = ow * sw + q - pl;
                    if (iw < 0 || iw >= w) continue;
                    uint32_t v = *reinterpret_cast<const uint32_t *>(x + (((size_t)b * h + ih) * w + iw) * c + g * 4);
                    m = __vmaxs4(m, v);
                }
            }
            *reinterpret_cast<uint32_t *>(y + p * c + g * 4) = m;
        } else {
            int m = -128;
            for (int a = 0; a < kh; a++) {
                int ih = oh * sh + a - pt;
                if (ih < 0 || ih >= h) continue;
                for (int q = 0; q < kw; q++) {
                    int iw = ow * sw + q - pl;
                    if (iw < 0 || iw >= w) continue;
                    int v = x[(((size_t)b * h + ih) * w + iw) * c + g];
                    m = v > m ? v : m;
                }
            }
            y[p * c + g] = (int8_t)m;
        }
    }
}

// --- concat along C (ops.rs:2178-2194) ---------------------------------------
struct ConcatArgs {
    const int8_t *src[16];
    int32_t c[16];
    int32_t off[16];
    int32_t count;
    int32_t c_total;
};

__global__ void k_concat_i8(ConcatArgs a, size_t pixels, int8_t *__restrict__ y, int vec) {
    // thread -> (pixel, vec-byte chunk of the output channel vector)
    const int chunks = a.c_total / vec;
    const size_t total = pixels * chunks;
    for (size_t i = blockIdx.x * (size_t)blockDim.x + threadIdx.x; i < total; i += (size_t)gridDim.x * blockDim.x) {
        size_t p = i / chunks;
        int oc = (int)(i % chunks) * vec;
        int s = 0;
        while (s + 1 < a.count && oc >= a.off[s + 1]) s++;
        const int8_t *src = a.src[s] + p * a.c[s] + (oc - a.off[s]);
        int8_t *dst = y + p * a.c_total + oc;
        if (vec == 16) *reinterpret_cast<int4 *>(dst) = *reinterpret_cast<const int4 *>(src);
        else if (vec == 8) *reinterpret_cast<int2 *>(dst) = *reinterpret_cast<const int2 *>(src);
        else if (vec == 4) *reinterpret_cast<int *>(dst) = *reinterpret_cast<const int *>(src);
        else *dst = *src;
    }
}

__global__ void k_slice_c_i8(const int8_t *__restrict__ x, int8_t *__restrict__ y, size_t pixels, int c_total,
                             int c0, int c_len, int vec) {
    const int chunks = c_len / vec;
    const size_t total = pixels * chunks;
    for (size_t i = blockIdx.x * (size_t)blockDim.x + threadIdx.x; i < total; i += (size_t)gridDim.x * blockDim.x) {
        size_t p = i / chunks;
        int c = (int)(i % chunks) * vec;
        const int8_t *src = x + p * c_total + c0 + c;
        int8_t *dst = y + p * c_len + c;
        if (vec == 16) *reinterpret_cast<int4 *>(dst) = *reinterpret_cast<const int4 *>(src);
        else if (vec == 8) *reinterpret_cast<int2 *>(dst) = *reinterpret_cast<const int2 *>(src);
        else if (vec == 4) *reinterpret_cast<int *>(dst) = *reinterpret_cast<const int *>(src);
        else *dst = *src;
    }
}

// 32-bit-index twins of the copies above (element counts below 2^31).
template <int kVec>
__global__ void k_concat_i8_32(ConcatArgs a, uint32_t total, FastDiv fch, int8_t *__restrict__ y) {
    for (uint32_t i = blockIdx.x * blockDim.x + threadIdx.x; i < total; i += gridDim.x * blockDim.x) {
        const uint32_t p = fdiv(i, fch);
        const int oc = (int)(i - p * fch.d) * kVec;
        int s = 0;
        while (s + 1 < a.count && oc >= a.off[s + 1]) s++;
        copy_vec<kVec>(y + (size_t)p * a.c_total + oc, a.src[s] + (size_t)p * a.c[s] + (oc - a.off[s]));
    }
}

template <int kVec>
__global__ void k_slice_c_i8_32(const int8_t *__restrict__ x, int8_t *__restrict__ y, uint32_t total, FastDiv fch,
                                int c_total, int c0, int c_len) {
    for (uint32_t i = blockIdx.x * blockDim.x + threadIdx.x; i < total; i += gridDim.x * blockDim.x) {
        const uint32_t p = fdiv(i, fch);
        const int c = (int)(i - p * fch.d) * kVec;
        copy_vec<kVec>(y + (size_t)p * c_len + c, x + (size_t)p * c_total + c0 + c);
    }
}

// --- nearest resize (ops.rs:2320-2348, f32 index arithmetic) -----------------
__device__ __forceinline__ int nearest_src(int o, float scale, int in_len) {
    float f = roundf(__fsub_rn(__fmul_rn(__fadd_rn((float)o, 0.5f), scale), 0.5f));
    f = fminf(fmaxf(f, 0.0f), (float)(in_len - 1));
    return (int)f;
}

__global__ void k_resize_nearest_i8(const int8_t *__restrict__ x, int8_t *__restrict__ y, int n, int hi, int wi,
                                    int ho, int wo, int c, float sh, float sw, int vec) {
    const int chunks = c / vec;
    const size_t total = (size_t)n * ho * wo * chunks;
    for (size_t i = blockIdx.x * (size_t)blockDim.x + threadIdx.x; i < total; i += (size_t)gridDim.x * blockDim.x) {
        int ch = (int)(i % chunks) * vec;
        size_t p = i / chunks;
        int ow = (int)(p % wo);
        size_t t = p / wo;
        int oh = (int)(t % ho);
        int b = (int)(t / ho);
        int ih = nearest_src(oh, sh, hi), iw = nearest_src(ow, sw, wi);
        const int8_t *src = x + (((size_t)b * hi + ih) * wi + iw) * c + ch;
        int8_t *dst = y + p * c + ch;
        if (vec == 16) *reinterpret_cast<int4 *>(dst) = *reinterpret_cast<const int4 *>(src);
        else if (vec == 8) *reinterpret_cast<int2 *>(dst) = *reinterpret_cast<const int2 *>(src);
        else if (vec == 4) *reinterpret_cast<int *>(dst) = *reinterpret_cast<const int *>(src);
        else *dst = *src;
    }
}

template <int kVec>
__global__ void k_resize_nearest_i8_32(const int8_t *__restrict__ x, int8_t *__restrict__ y, int hi, int wi, int c,
                                       float sh, float sw, uint32_t total, FastDiv fch, FastDiv fwo, FastDiv fho) {
    for (uint32_t i = blockIdx.x * blockDim.x + threadIdx.x; i < total; i += gridDim.x * blockDim.x) {
        const uint32_t p = fdiv(i, fch);
        const int ch = (int)(i - p * fch.d) * kVec;
        const uint32_t t = fdiv(p, fwo);
        const int ow = (int)(p - t * fwo.d);
        const uint32_t b = fdiv(t, fho);
        const int oh = (int)(t - b * fho.d);
        const int ih = nearest_src(oh, sh, hi), iw = nearest_src(ow, sw, wi);
        copy_vec<kVec>(y + (size_t)p * c + ch, x + (((size_t)b * hi + ih) * wi + iw) * c + ch);
    }
}

// maxpool on 16 channels per thread (c % 16 == 0), the window clipped to the
// image once (padding taps are skipped, as in k_maxpool_i8; an empty window
// leaves -128).
__global__ void k_maxpool_i8_v16(const int8_t *__restrict__ x, int8_t *__restrict__ y, int h, int w, int c, int kh,
                                 int kw, int sh, int sw, int pt, int pl, uint32_t total, FastDiv fcg, FastDiv fwo,
                                 FastDiv fho, int x_pitch, int y_pitch) {
    for (uint32_t i = blockIdx.x * blockDim.x + threadIdx.x; i < total; i += gridDim.x * blockDim.x) {
        const uint32_t p = fdiv(i, fcg);
        const int g = (int)(i - p * fcg.d);
        const uint32_t t = fdiv(p, fwo);
        const int ow = (int)(p - t * fwo.d);
        const uint32_t b = fdiv(t, fho);
        const int oh = (int)(t - b * fho.d);
        const int h0 = oh * sh - pt, w0 = ow * sw - pl;
        const int a0 = max(0, -h0), a1 = min(kh, h - h0), q0 = max(0, -w0), q1 = min(kw, w - w0);
        uint4 m = make_uint4(0x80808080u, 0x80808080u, 0x80808080u, 0x80808080u);
        for (int a = a0; a < a1; a++) {
            const int8_t *row = x + (((size_t)b * h + (h0 + a)) * w + w0) * x_pitch + g * 16;
            for (int q = q0; q < q1; q++) {
                const uint4 v = __ldg(reinterpret_cast<const uint4 *>(row + (size_t)q * x_pitch));
                m.x = __vmaxs4(m.x, v.x);
                m.y = __vmaxs4(m.y, v.y);
                m.z = __vmaxs4(m.z, v.z);
                m.w = __vmaxs4(m.w, v.w);
            }
        }
        *reinterpret_cast<uint4 *>(y + (size_t)p * y_pitch + g * 16) = m;
    }
}

// `count` chained k x k stride-1 maxpools with k/2 padding (the padding taps
// skipped), the SPPF block's y1 = pool(x), y2 = pool(y1), y3 = pool(y2): one
// block per (image, 16-channel group) keeps the map in shared memory and pools
// it separably (a clipped window is a rectangle, and max is associative and
// commutative, so the row maxima's column maximum is the window maximum), writing
// each pooled map out as it goes.  x is read once instead of pooled maps being
// re-read from memory.
__global__ void k_maxpool_chain_i8(const int8_t *__restrict__ x, int x_pitch, int8_t *__restrict__ y0, int8_t *__restrict__ y1,
                                   int8_t *__restrict__ y2, int8_t *__restrict__ y3, int p0, int p1, int p2, int p3,
                                   int count, int h, int w, int groups, int r) {
    extern __shared__ __align__(16) uint4 maps[];  // [2][h * w]: the current map, the row maxima
    const int hw = h * w, b = blockIdx.x / groups, g = blockIdx.x % groups;
    uint4 *cur = maps, *rowm = maps + hw;
    for (int p = threadIdx.x; p < hw; p += blockDim.x)
        cur[p] = __ldg(reinterpret_cast<const uint4 *>(x + ((size_t)b * hw + p) * x_pitch + g * 16));
    __syncthreads();
    int8_t *const outs[4] = {y0, y1, y2, y3};
    const int pitches[4] = {p0, p1, p2, p3};
    for (int s = 0; s < count; s++) {
        for (int p = threadIdx.x; p < hw; p += blockDim.x) {  // maxima along each row
            const int oh = p / w, ow = p % w;
            const int q0 = max(0, ow - r), q1 = min(w - 1, ow + r);
            uint4 m = cur[oh * w + q0];
            for (int q = q0 + 1; q <= q1; q++) {
                const uint4 v = cur[oh * w + q];
                m.x = __vmaxs4(m.x, v.x); m.y = __vmaxs4(m.y, v.y); m.z = __vmaxs4(m.z, v.z); m.w = __vmaxs4(m.w, v.w);
            }
            rowm[p] = m;
        }
        __syncthreads();
        for (int p = threadIdx.x; p < hw; p += blockDim.x) {  // then along each column
            const int oh = p / w, ow = p % w;
            const int a0 = max(0, oh - r), a1 = min(h - 1, oh + r);
            uint4 m = rowm[a0 * w + ow];
            for (int a = a0 + 1; a <= a1; a++) {
                const uint4 v = rowm[a * w + ow];
                m.x = __vmaxs4(m.x, v.x); m.y = __vmaxs4(m.y, v.y); m.z = __vmaxs4(m.z, v.z); m.w = __vmaxs4(m.w, v.w);
            }
            cur[p] = m;
            *reinterpret_cast<uint4 *>(outs[s] + ((size_t)b * hw + p) * pitches[s] + g * 16) = m;
        }
        __syncthreads();
    }
}

// --- weight repacks (int8 and fp16 element types) ------------------------------------------------------------
// HWIO [taps][c_in][c_out] -> OHWI [c_out][taps][c_in] (K-major rows for the MMA B operand).
template <typename T>
__global__ void k_repack_hwio_to_ohwi(const T *__restrict__ w, T *__restrict__ o, int taps, int c_in, int c_out) {
    const size_t total = (size_t)taps * c_in * c_out;
    for (size_t i = blockIdx.x * (size_t)blockDim.x + threadIdx.x; i < total; i += (size_t)gridDim.x * blockDim.x) {
        // i indexes the output: i = (oc * taps + t) * c_in + ic
        int ic = (int)(i % c_in);
        size_t r = i / c_in;
        int t = (int)(r % taps);
        int oc = (int)(r / taps);
        o[i] = w[((size_t)t * c_in + ic) * c_out + oc];
    }
}

// The reference-signature fused conv's per-call preparation in one launch: the
// HWIO -> OHWI repack, and its scalar requant scale spread over c_out slots.
__global__ void k_repack_hwio_to_ohwi_fill(const int8_t *__restrict__ w, int8_t *__restrict__ o, int taps, int c_in,
                                           int c_out, float *__restrict__ m, float v) {
    const size_t total = (size_t)taps * c_in * c_out;
    const size_t stride = (size_t)gridDim.x * blockDim.x;
    const size_t first = blockIdx.x * (size_t)blockDim.x + threadIdx.x;
    for (size_t i = first; i < (size_t)c_out; i += stride) m[i] = v;
    for (size_t i = first; i < total; i += stride) {
        const int ic = (int)(i % c_in);
        const size_t r = i / c_in;
        const int t = (int)(r % taps);
        const int oc = (int)(r / taps);
        o[i] = w[((size_t)t * c_in + ic) * c_out + oc];
    }
}

// B [k][n] row-major -> [n][k] (K-major).
template <typename T>
__global__ void k_transpose_kn_to_nk(const T *__restrict__ b, T *__restrict__ o, int k, int n) {
    __shared__ T tile[32][33];
    for (int n0 = blockIdx.x * 32; n0 < n; n0 += gridDim.x * 32)
        for (int k0 = blockIdx.y * 32; k0 < k; k0 += gridDim.y * 32) {
            int tx = threadIdx.x, ty = threadIdx.y;
            for (int r = ty; r < 32; r += blockDim.y) {
                int kk = k0 + r, nn = n0 + tx;
                tile[r][tx] = (kk < k && nn < n) ? b[(size_t)kk * n + nn] : 0;
            }
            __syncthreads();
            for (int r = ty; r < 32; r += blockDim.y) {
                int nn = n0 + r, kk = k0 + tx;
                if (nn < n && kk < k) o[(size_t)nn * k + kk] = tile[tx][r];
            }
            __syncthreads();
        }
}

// Bounded wait on a flag nothing sets: exercises the expiry path without a hang.
__global__ void k_expire_wait(const volatile int32_t *flag, int32_t *err, uint64_t cap_ns) {
    const uint64_t t0 = globaltimer_ns();
    while (*flag == 0) {
        if (globaltimer_ns() - t0 > cap_ns) {
            record_error(err, DW_DEV_WAIT_EXPIRED, /*site=*/900, 0);
            return;
        }
        __nanosleep(1000);
    }
}

inline int vec_for(size_t c, const void *const *ptrs, int nptr) {
    int v = 16;
    while (v > 1) {
        bool ok = (c % v) == 0;
        for (int i = 0; i < nptr && ok; i++) ok = ((uintptr_t)ptrs[i] % v) == 0;
        if (ok) return v;
        v /= 2;
        if (v == 2) v = 1;
    }
    return 1;
}

}  // namespace

dw_status launch_requantize(dw_backend *be, const int32_t *in, int8_t *out, size_t n, float scale) {
    k_requantize<<<grid_for(be, (n + 15) / 16), kThreads, 0, be->stream>>>(in, out, n, scale);
    return dw_after_launch(be, "requantize_i32_to_i8");
}

dw_status launch_relu_i8(dw_backend *be, const int8_t *in, int8_t *out, size_t n) {
    k_relu_i8<<<grid_for(be, (n + 15) / 16), kThreads, 0, be->stream>>>(in, out, n);
    return dw_after_launch(be, "relu_i8");
}

dw_status launch_add_i8(dw_backend *be, const int8_t *a, const int8_t *b, int8_t *out, size_t n, float ra, float rb) {
    const bool aligned = ((uintptr_t)a & 15) == 0 && ((uintptr_t)b & 15) == 0 && ((uintptr_t)out & 15) == 0;
    if (aligned && n % 16 == 0 && std::fabs(ra) < 1e30f && std::fabs(rb) < 1e30f) {
        k_add_i8_fast<<<grid_for(be, n / 16), kThreads, 0, be->stream>>>(a, b, out, n / 16, ra, rb);
        return dw_after_launch(be, "add_i8");
    }
    k_add_i8<<<grid_for(be, (n + 15) / 16), kThreads, 0, be->stream>>>(a, b, out, n, ra, rb);
    return dw_after_launch(be, "add_i8");
}

dw_status launch_add_i8_view(dw_backend *be, const int8_t *a, int a_pitch, const int8_t *b, int b_pitch, int8_t *out,
                             int out_pitch, size_t pixels, int c, float ra, float rb) {
    const size_t items = pixels * (size_t)(c / 16);
    if (c % 16 || a_pitch % 16 || b_pitch % 16 || out_pitch % 16 || ((uintptr_t)a & 15) || ((uintptr_t)b & 15) ||
        ((uintptr_t)out & 15) || !(std::fabs(ra) < 1e30f) || !(std::fabs(rb) < 1e30f) || items >= (1u << 31))
        return dw_fail(be, DW_ERR_UNSUPPORTED, "add_i8_view: needs 16-channel multiples, 16-byte alignment and ratios below 1e30");
    k_add_i8_view<<<grid_for(be, items), kThreads, 0, be->stream>>>(a, a_pitch, b, b_pitch, out, out_pitch,
                                                                     (uint32_t)items, make_fastdiv((uint32_t)(c / 16)),
                                                                     ra, rb);
    return dw_after_launch(be, "add_i8_view");
}

dw_status launch_maxpool_i8_view(dw_backend *be, const int8_t *x, int x_pitch, int8_t *y, int y_pitch, int n, int h,
                                 int w, int c, int kh, int kw, int sh, int sw, int pt, int pl, int ho, int wo) {
    const size_t groups16 = (size_t)n * ho * wo * (c / 16);
    if (c % 16 || x_pitch % 16 || y_pitch % 16 || ((uintptr_t)x & 15) || ((uintptr_t)y & 15) || groups16 >= (1u << 31))
        return dw_fail(be, DW_ERR_UNSUPPORTED, "maxpool_i8_view: needs 16-channel multiples and 16-byte alignment");
    k_maxpool_i8_v16<<<grid_for(be, groups16), kThreads, 0, be->stream>>>(
        x, y, h, w, c, kh, kw, sh, sw, pt, pl, (uint32_t)groups16, make_fastdiv((uint32_t)(c / 16)),
        make_fastdiv((uint32_t)wo), make_fastdiv((uint32_t)ho), x_pitch, y_pitch);
    return dw_after_launch(be, "maxpool_i8");
}

dw_status launch_maxpool_chain_i8_view(dw_backend *be, const int8_t *x, int x_pitch, int8_t *const *ys,
                                       const int *y_pitches, int count, int n, int h, int w, int c, int k) {
    bool aligned = !((uintptr_t)x & 15) && x_pitch % 16 == 0;
    for (int i = 0; i < count; i++) aligned = aligned && !((uintptr_t)ys[i] & 15) && y_pitches[i] % 16 == 0;
    if (c % 16 || !aligned || count < 1 || count > 4 || k % 2 == 0)
        return dw_fail(be, DW_ERR_UNSUPPORTED, "maxpool_chain_i8_view: needs 16-channel multiples, 16-byte alignment, "
                                               "1..4 pools and an odd window");
    const size_t smem = (size_t)2 * h * w * 16;
    if (smem <= 48 * 1024 && (long long)n * (c / 16) < (1LL << 31)) {
        int8_t *y[4] = {ys[0], count > 1 ? ys[1] : nullptr, count > 2 ? ys[2] : nullptr, count > 3 ? ys[3] : nullptr};
        int pp[4] = {y_pitches[0], count > 1 ? y_pitches[1] : 0, count > 2 ? y_pitches[2] : 0,
                     count > 3 ? y_pitches[3] : 0};
        k_maxpool_chain_i8<<<n * (c / 16), kThreads, smem, be->stream>>>(x, x_pitch, y[0], y[1], y[2], y[3], pp[0],
                                                                           pp[1], pp[2], pp[3], count, h, w, c / 16,
                                                                           k / 2);
        return dw_after_launch(be, "maxpool_chain_i8");
    }
    // larger maps: one pooling launch per step, each reading the previous output
    const int r = k / 2;
    for (int i = 0; i < count; i++) {
        const dw_status st = launch_maxpool_i8_view(be, i ? ys[i - 1] : x, i ? y_pitches[i - 1] : x_pitch, ys[i],
                                                    y_pitches[i], n, h, w, c, k, k, 1, 1, r, r, h, w);
        if (st != DW_OK) return st;
    }
    return DW_OK;
}

dw_status launch_quantize_f32(dw_backend *be, const float *in, int8_t *out, size_t n, float scale) {
    const float inv = 1.0f / scale;  // ops.rs:3506, computed on the host in f32 like the reference
    k_quantize_f32<<<grid_for(be, (n + 15) / 16), kThreads, 0, be->stream>>>(in, out, n, inv);
    return dw_after_launch(be, "quantize_f32_to_i8");
}

dw_status launch_quantize_u8(dw_backend *be, const uint8_t *in, int8_t *out, size_t n, float scale) {
    const float inv255 = 1.0f / 255.0f, inv = 1.0f / scale;
    k_quantize_u8<<<grid_for(be, (n + 15) / 16), kThreads, 0, be->stream>>>(in, out, n, inv255, inv);
    return dw_after_launch(be, "quantize_u8_to_i8");
}

dw_status launch_im2col_u8_i8(dw_backend *be, const uint8_t *x, int8_t *y, int n, int h, int w, int c, int kh, int kw,
                              int sh, int sw, int pt, int pl, int ho, int wo, int c_dst, float scale) {
    const float inv255 = 1.0f / 255.0f, inv = 1.0f / scale;
    if (c == 3 && kh == 3 && kw == 3 && c_dst == 32 && w % 16 == 0 && ((uintptr_t)x & 15) == 0 && pl >= 0 &&
        pl <= 5 && (long long)n * ho < (1LL << 31)) {
        // row-staged kernel: each row holds the input row at byte 16 and covers the last pixel's reads
        const long long last = 16 + ((long long)(wo - 1) * sw - pl) * 3 + 12;
        const long long need = std::max<long long>(16 + (long long)w * 3, last);
        const long long row_bytes = (need + 15) / 16 * 16;
        const long long band_rows = (long long)(kStemBand - 1) * sh + 3;
        const int nbands = (ho + kStemBand - 1) / kStemBand;
        if (band_rows * row_bytes <= 38 * 1024 && (long long)n * nbands < (1LL << 31)) {
            k_im2col_stem3_band<<<n * nbands, 256, (size_t)(band_rows * row_bytes), be->stream>>>(
                x, y, h, w, sh, sw, pt, pl, ho, wo, (int)row_bytes, nbands, inv255, inv);
            return dw_after_launch(be, "im2col_u8_i8");
        }
        if (3 * row_bytes <= 40 * 1024) {
            k_im2col_stem3_rows<<<n * ho, kThreads, (size_t)(3 * row_bytes), be->stream>>>(
                x, y, h, w, sh, sw, pt, pl, ho, wo, (int)row_bytes, inv255, inv);
            return dw_after_launch(be, "im2col_u8_i8");
        }
    }
    const int grid = grid_for(be, (size_t)n * ho * wo);
    if (c == 3 && kh == 3 && kw == 3)  // the usual image stem
        k_im2col_u8_i8<3, 3, 3><<<grid, kThreads, 0, be->stream>>>(x, y, n, h, w, c, kh, kw, sh, sw, pt, pl, ho, wo,
                                                                    c_dst, inv255, inv);
    else
        k_im2col_u8_i8<0, 0, 0><<<grid, kThreads, 0, be->stream>>>(x, y, n, h, w, c, kh, kw, sh, sw, pt, pl, ho, wo,
                                                                    c_dst, inv255, inv);
    return dw_after_launch(be, "im2col_u8_i8");
}

dw_status launch_stem3_conv_u8_i8(dw_backend *be, const uint8_t *x, const int8_t *w_hwio, const EpiParams &ep,
                                 int8_t *y, int n, int h, int w, int sh, int sw, int pt, int pl, int ho, int wo, int c_out,
                                 float scale) {
    const float inv255 = 1.0f / 255.0f, inv = 1.0f / scale;
    // the band staging of k_im2col_stem3_band: whole 16-byte units per input row,
    // the row at byte 16, the last pixel's 12-byte read inside the row
    const long long last = 16 + ((long long)(wo - 1) * sw - pl) * 3 + 12;
    const long long need = std::max<long long>(16 + (long long)w * 3, last);
    const long long row_bytes = (need + 15) / 16 * 16;
    const long long band_rows = (long long)(kStemConvBand - 1) * sh + 3;
    const int nbands = (ho + kStemConvBand - 1) / kStemConvBand;
    if (w % 16 != 0 || ((uintptr_t)x & 15) != 0 || ((uintptr_t)y & 15) != 0 || pl < 0 || pl > 5 || pt < 0 ||
        c_out % 16 != 0 || c_out > kStemMaxCout || band_rows * row_bytes > kStemConvRowsBytes ||
        (long long)n * nbands >= (1LL << 31))
        return dw_fail(be, DW_ERR_UNSUPPORTED,
                       "conv2d_stem_u8_i8: shape outside the fused stem (width a multiple of 16, c_out a multiple of 16 "
                       "<= %d, left pad <= 5, 16-byte aligned buffers, staged rows <= %d bytes)",
                       kStemMaxCout, kStemConvRowsBytes);
    const size_t smem = (size_t)(band_rows * row_bytes);
    if (ep.epilogue == DW_EPI_SILU)
        k_stem3_conv<true><<<n * nbands, 256, smem, be->stream>>>(x, w_hwio, ep, y, h, w, sh, sw, pt, pl, ho, wo, c_out,
                                                                  (int)row_bytes, nbands, inv255, inv);
    else
        k_stem3_conv<false><<<n * nbands, 256, smem, be->stream>>>(x, w_hwio, ep, y, h, w, sh, sw, pt, pl, ho, wo, c_out,
                                                                   (int)row_bytes, nbands, inv255, inv);
    return dw_after_launch(be, "conv2d_stem_u8_i8");
}

dw_status launch_dequantize(dw_backend *be, const int8_t *in, float *out, size_t n, float scale) {
    k_dequantize<<<grid_for(be, (n + 15) / 16), kThreads, 0, be->stream>>>(in, out, n, scale);
    return dw_after_launch(be, "dequantize_i8_to_f32");
}

dw_status launch_maxpool_i8(dw_backend *be, const int8_t *x, int8_t *y, int n, int h, int w, int c, int kh, int kw,
                            int sh, int sw, int pt, int pl, int ho, int wo) {
    const size_t groups16 = (size_t)n * ho * wo * (c / 16);
    if (c % 16 == 0 && ((uintptr_t)x % 16) == 0 && ((uintptr_t)y % 16) == 0 && groups16 < (1u << 31)) {
        k_maxpool_i8_v16<<<grid_for(be, groups16), kThreads, 0, be->stream>>>(
            x, y, h, w, c, kh, kw, sh, sw, pt, pl, (uint32_t)groups16, make_fastdiv((uint32_t)(c / 16)),
            make_fastdiv((uint32_t)wo), make_fastdiv((uint32_t)ho), c, c);
        return dw_after_launch(be, "maxpool_i8");
    }
    int vec = (c % 4 == 0 && ((uintptr_t)x % 4) == 0 && ((uintptr_t)y % 4) == 0) ? 4 : 1;
    size_t items = (size_t)n * ho * wo * (c / vec);
    k_maxpool_i8<<<grid_for(be, items), kThreads, 0, be->stream>>>(x, y, n, h, w, c, kh, kw, sh, sw, pt, pl, ho, wo,
                                                                    vec);
    return dw_after_launch(be, "maxpool_i8");
}

dw_status launch_concat_i8(dw_backend *be, const int8_t *const *xs, const int32_t *cs, int count, size_t pixels,
                           int8_t *y) {
    ConcatArgs a{};
    a.count = count;
    int off = 0;
    const void *ptrs[17];
    for (int i = 0; i < count; i++) {
        a.src[i] = xs[i];
        a.c[i] = cs[i];
        a.off[i] = off;
        off += cs[i];
        ptrs[i] = xs[i];
    }
    a.c_total = off;
    ptrs[count] = y;
    // Vector width: every channel count, offset and pointer must allow it.
    int vec = 16;
    for (; vec > 1; vec /= 2) {
        bool ok = (off % vec) == 0;
        for (int i = 0; i < count && ok; i++) ok = (cs[i] % vec) == 0;
        for (int i = 0; i <= count && ok; i++) ok = ((uintptr_t)ptrs[i] % vec) == 0;
        if (ok) break;
        if (vec == 4) { vec = 1; break; }
    }
    if (vec == 2) vec = 1;
    size_t items = pixels * (off / vec);
    if (items < (1u << 31) && (vec == 16 || vec == 4)) {
        const FastDiv fch = make_fastdiv((uint32_t)(off / vec));
        if (vec == 16)
            k_concat_i8_32<16><<<grid_for(be, items), kThreads, 0, be->stream>>>(a, (uint32_t)items, fch, y);
        else
            k_concat_i8_32<4><<<grid_for(be, items), kThreads, 0, be->stream>>>(a, (uint32_t)items, fch, y);
        return dw_after_launch(be, "concat_i8");
    }
    k_concat_i8<<<grid_for(be, items), kThreads, 0, be->stream>>>(a, pixels, y, vec);
    return dw_after_launch(be, "concat_i8");
}

dw_status launch_slice_c_i8(dw_backend *be, const int8_t *x, int8_t *y, size_t pixels, int c_total, int c0,
                            int c_len) {
    int vec = 16;
    for (; vec > 1; vec /= 2) {
        if (c_total % vec == 0 && c0 % vec == 0 && c_len % vec == 0 && ((uintptr_t)x % vec) == 0 &&
            ((uintptr_t)y % vec) == 0)
            break;
        if (vec == 4) { vec = 1; break; }
    }
    if (vec == 2) vec = 1;
    const size_t items = pixels * (c_len / vec);
    if (items < (1u << 31) && (vec == 16 || vec == 4)) {
        const FastDiv fch = make_fastdiv((uint32_t)(c_len / vec));
        if (vec == 16)
            k_slice_c_i8_32<16><<<grid_for(be, items), kThreads, 0, be->stream>>>(x, y, (uint32_t)items, fch, c_total,
                                                                                  c0, c_len);
        else
            k_slice_c_i8_32<4><<<grid_for(be, items), kThreads, 0, be->stream>>>(x, y, (uint32_t)items, fch, c_total,
                                                                                 c0, c_len);
        return dw_after_launch(be, "slice_c_i8");
    }
    k_slice_c_i8<<<grid_for(be, items), kThreads, 0, be->stream>>>(x, y, pixels, c_total, c0, c_len, vec);
    return dw_after_launch(be, "slice_c_i8");
}

dw_status launch_resize_nearest_i8(dw_backend *be, const int8_t *x, int8_t *y, int n, int hi, int wi, int ho, int wo,
                                   int c) {
    const void *ptrs[2] = {x, y};
    int vec = vec_for((size_t)c, ptrs, 2);
    if (vec == 2) vec = 1;
    float sh = (float)hi / (float)ho, sw = (float)wi / (float)wo;  // ops.rs:2334-2335
    size_t items = (size_t)n * ho * wo * (c / vec);
    if (items < (1u << 31) && vec == 16) {
        k_resize_nearest_i8_32<16><<<grid_for(be, items), kThreads, 0, be->stream>>>(
            x, y, hi, wi, c, sh, sw, (uint32_t)items, make_fastdiv((uint32_t)(c / 16)), make_fastdiv((uint32_t)wo),
            make_fastdiv((uint32_t)ho));
        return dw_after_launch(be, "resize_nearest_i8");
    }
    k_resize_nearest_i8<<<grid_for(be, items), kThreads, 0, be->stream>>>(x, y, n, hi, wi, ho, wo, c, sh, sw, vec);
    return dw_after_launch(be, "resize_nearest_i8");
}

dw_status launch_repack_hwio_to_ohwi(dw_backend *be, const int8_t *w, int8_t *out, int taps, int c_in, int c_out) {
    size_t items = (size_t)taps * c_in * c_out;
    k_repack_hwio_to_ohwi<int8_t><<<grid_for(be, items), kThreads, 0, be->stream>>>(w, out, taps, c_in, c_out);
    return dw_after_launch(be, "repack_hwio_to_ohwi");
}

dw_status launch_repack_hwio_to_ohwi_fill(dw_backend *be, const int8_t *w, int8_t *out, int taps, int c_in, int c_out,
                                          float *m, float v) {
    const size_t items = std::max<size_t>((size_t)taps * c_in * c_out, (size_t)c_out);
    k_repack_hwio_to_ohwi_fill<<<grid_for(be, items), kThreads, 0, be->stream>>>(w, out, taps, c_in, c_out, m, v);
    return dw_after_launch(be, "repack_hwio_to_ohwi_fill");
}

dw_status launch_repack_hwio_to_ohwi_f16(dw_backend *be, const uint16_t *w, uint16_t *out, int taps, int c_in,
                                         int c_out) {
    size_t items = (size_t)taps * c_in * c_out;
    k_repack_hwio_to_ohwi<uint16_t><<<grid_for(be, items), kThreads, 0, be->stream>>>(w, out, taps, c_in, c_out);
    return dw_after_launch(be, "repack_hwio_to_ohwi_f16");
}

dw_status launch_transpose_kn_to_nk(dw_backend *be, const int8_t *b, int8_t *out, int k, int n) {
    dim3 block(32, 8);
    dim3 grid((unsigned)std::min((n + 31) / 32, 1024), (unsigned)std::min((k + 31) / 32, 1024));
    k_transpose_kn_to_nk<int8_t><<<grid, block, 0, be->stream>>>(b, out, k, n);
    return dw_after_launch(be, "transpose_kn_to_nk");
}

dw_status launch_transpose_kn_to_nk_f16(dw_backend *be, const uint16_t *b, uint16_t *out, int k, int n) {
    dim3 block(32, 8);
    dim3 grid((unsigned)std::min((n + 31) / 32, 1024), (unsigned)std::min((k + 31) / 32, 1024));
    k_transpose_kn_to_nk<uint16_t><<<grid, block, 0, be->stream>>>(b, out, k, n);
    return dw_after_launch(be, "transpose_kn_to_nk_f16");
}

dw_status launch_expire_wait(dw_backend *be, uint64_t cap_ns) {
    // The flag lives in the backend scratch and is zeroed here; nothing sets it.
    void *flag = nullptr;
    dw_status st = dw_scratch(be, 256, &flag);
    if (st != DW_OK) return st;
    st = dw_cuda_check(be, cudaMemsetAsync(flag, 0, 4, be->stream), "expire_wait flag");
    if (st != DW_OK) return st;
    k_expire_wait<<<1, 1, 0, be->stream>>>((const volatile int32_t *)flag, be->dev_err, cap_ns);
    return dw_after_launch(be, "debug_expire_wait");
}

}  // namespace dw
