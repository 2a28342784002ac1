// ops.cu -- op entry points of the C ABI: argument and size checks that mirror
// the reference's (crates/dragonwing-vulkan/src/ops.rs, crates/dragonwing-cpu/src/ops.rs),
// then dispatch to the kernels.

#include <cmath>
#include <vector>

#include "dw_internal.h"

namespace {

inline size_t al256(size_t v) { return (v + 255) & ~size_t(255); }

dw_status need(dw_backend *be, const void *p, const char *op, const char *name) {
    if (!p) return dw_fail(be, DW_ERR_INVALID_ARG, "%s: %s is null", op, name);
    return DW_OK;
}

dw_status check_len(dw_backend *be, const dw_buf *b, size_t expected, const char *op, const char *name) {
    if (b->len != expected)
        return dw_fail(be, DW_ERR_SIZE_MISMATCH, "%s: %s mismatch: expected %zu, got %zu", op, name, expected, b->len);
    return DW_OK;
}

#define DW_TRY(x)                     \
    do {                              \
        dw_status _st = (x);          \
        if (_st != DW_OK) return _st; \
    } while (0)

}  // namespace

// Validates a conv descriptor; computes the output dims.
dw_status dw_check_conv_desc(dw_backend *be, const dw_conv_desc *d, int *ho, int *wo, const char *op) {
    if (!d) return dw_fail(be, DW_ERR_INVALID_ARG, "%s: descriptor is null", op);
    if (d->n <= 0 || d->h <= 0 || d->w <= 0 || d->c_in <= 0 || d->c_out <= 0 || d->k_h <= 0 || d->k_w <= 0 ||
        d->stride_h <= 0 || d->stride_w <= 0 || d->pad_t < 0 || d->pad_l < 0 || d->pad_b < 0 || d->pad_r < 0)
        return dw_fail(be, DW_ERR_INVALID_ARG, "%s: dims must be positive and pads non-negative", op);
    long hp = (long)d->h + d->pad_t + d->pad_b - d->k_h;
    long wp = (long)d->w + d->pad_l + d->pad_r - d->k_w;
    if (hp < 0 || wp < 0)
        return dw_fail(be, DW_ERR_INVALID_ARG, "%s: kernel %dx%d larger than padded input %ldx%ld", op, d->k_h, d->k_w,
                       hp + d->k_h, wp + d->k_w);
    *ho = (int)(hp / d->stride_h + 1);
    *wo = (int)(wp / d->stride_w + 1);
    if (d->group != 1 && !(d->group == d->c_in && d->c_out % d->c_in == 0))
        return dw_fail(be, DW_ERR_UNSUPPORTED,
                       "%s: group=%d unsupported (only 1, or c_in=%d for depthwise with c_out a multiple of c_in)", op,
                       d->group, d->c_in);
    if (d->epilogue < DW_EPI_NONE || d->epilogue > DW_EPI_SILU)
        return dw_fail(be, DW_ERR_INVALID_ARG, "%s: unknown epilogue %d", op, d->epilogue);
    if (d->epilogue == DW_EPI_RELU6 && (d->q6 < 0 || d->q6 > 127))
        return dw_fail(be, DW_ERR_INVALID_ARG, "%s: q6=%d outside [0,127]", op, d->q6);
    return DW_OK;
}

namespace {

inline dw_status check_desc(dw_backend *be, const dw_conv_desc *d, int *ho, int *wo, const char *op) {
    return dw_check_conv_desc(be, d, ho, wo, op);
}

size_t weight_len(const dw_conv_desc *d) {
    size_t taps = (size_t)d->k_h * d->k_w;
    return d->group == 1 ? taps * d->c_in * d->c_out : taps * d->c_out;
}

}  // namespace

extern "C" {

DW_API dw_status dw_prepare_weights_i8(dw_backend *be, const dw_conv_desc *d, const dw_buf *w_hwio, dw_buf **out) {
    const char *op = "prepare_weights_i8";
    if (!be) return DW_ERR_INVALID_ARG;
    DW_TRY(need(be, out, op, "out"));
    *out = nullptr;
    DW_TRY(need(be, w_hwio, op, "kernel"));
    int ho, wo;
    DW_TRY(check_desc(be, d, &ho, &wo, op));
    DW_TRY(check_len(be, w_hwio, weight_len(d), op, "kernel"));
    cudaSetDevice(be->device);
    dw_buf *o = nullptr;
    DW_TRY(dw_alloc(be, w_hwio->len, &o));
    dw_status st;
    if (d->group == 1) {
        st = dw::launch_repack_hwio_to_ohwi(be, (const int8_t *)w_hwio->ptr, (int8_t *)o->ptr, d->k_h * d->k_w,
                                            d->c_in, d->c_out);
    } else {  // depthwise: [kh, kw, C, mult] is already the kernel's layout
        st = dw_cuda_check(be, cudaMemcpyAsync(o->ptr, w_hwio->ptr, w_hwio->len, cudaMemcpyDeviceToDevice, be->stream),
                           "prepare depthwise weights");
    }
    if (st != DW_OK) {
        dw_free(be, o);
        return st;
    }
    *out = o;
    return DW_OK;
}

static dw_status conv_dispatch(dw_backend *be, const dw_conv_desc *d, int ho, int wo, const dw_buf *x,
                               const dw_buf *w_prep, const dw::EpiParams &ep, dw_buf *y, const char *op) {
    const int8_t *xp = (const int8_t *)x->ptr;
    const int8_t *wp = (const int8_t *)w_prep->ptr;
    int8_t *yp = (int8_t *)y->ptr;
    if (d->group != 1) return dw::launch_dwconv_i8(be, *d, ho, wo, xp, wp, ep, yp, nullptr);
    const int path = be->cfg.conv_path;
    if (path != DW_PATH_DIRECT && dw::umma_supported(be, *d, ho, wo))
        return dw::launch_umma_conv_i8(be, *d, ho, wo, xp, wp, ep, yp);
    if (path == DW_PATH_UMMA)
        return dw_fail(be, DW_ERR_UNSUPPORTED, "%s: shape not supported by the tensor-core kernel (c_in=%d c_out=%d)",
                       op, d->c_in, d->c_out);
    return dw::launch_conv_direct_i8(be, *d, ho, wo, xp, wp, ep, yp, nullptr);
}

DW_API dw_status dw_conv2d_i8(dw_backend *be, const dw_conv_desc *d, const dw_buf *x, const dw_buf *w_prep,
                              const dw_buf *bias, const dw_buf *M, const dw_buf *D, dw_buf *y) {
    const char *op = "conv2d_i8";
    if (!be) return DW_ERR_INVALID_ARG;
    int ho, wo;
    DW_TRY(check_desc(be, d, &ho, &wo, op));
    DW_TRY(need(be, x, op, "input"));
    DW_TRY(need(be, w_prep, op, "kernel"));
    DW_TRY(need(be, y, op, "output"));
    DW_TRY(check_len(be, x, (size_t)d->n * d->h * d->w * d->c_in, op, "input"));
    DW_TRY(check_len(be, w_prep, weight_len(d), op, "kernel"));
    DW_TRY(check_len(be, y, (size_t)d->n * ho * wo * d->c_out, op, "output"));
    if (bias) DW_TRY(check_len(be, bias, 4 * (size_t)d->c_out, op, "bias"));
    if (d->epilogue == DW_EPI_SILU) {
        DW_TRY(need(be, D, op, "D (dequant scales, required by SILU)"));
        DW_TRY(check_len(be, D, 4 * (size_t)d->c_out, op, "D"));
    } else {
        DW_TRY(need(be, M, op, "M (requant scales)"));
        DW_TRY(check_len(be, M, 4 * (size_t)d->c_out, op, "M"));
    }
    cudaSetDevice(be->device);
    dw::EpiParams ep{bias ? (const int32_t *)bias->ptr : nullptr, M ? (const float *)M->ptr : nullptr,
                     D ? (const float *)D->ptr : nullptr, d->epilogue, d->q6, d->inv_s_out};
    return conv_dispatch(be, d, ho, wo, x, w_prep, ep, y, op);
}

DW_API dw_status dw_conv2d_requant_relu_i8(dw_backend *be, const dw_buf *input, const dw_buf *kernel_hwio,
                                           dw_buf *output, size_t n, size_t h_in, size_t w_in, size_t c_in,
                                           size_t c_out, size_t k_h, size_t k_w, size_t stride_h, size_t stride_w,
                                           size_t pad_h, size_t pad_w, float requant_scale, int do_relu) {
    if (!be) return DW_ERR_INVALID_ARG;
    if (!input || !kernel_hwio || !output) return dw_fail(be, DW_ERR_INVALID_ARG, "conv_fused: null buffer");
    // crates/dragonwing-vulkan/src/ops.rs:2313-2345 (same checks, same strings)
    if (c_in % 4 != 0) return dw_fail(be, DW_ERR_INVALID_ARG, "conv_fused: c_in=%zu must be multiple of 4", c_in);
    if (c_out % 4 != 0)
        return dw_fail(be, DW_ERR_INVALID_ARG, "conv_fused: c_out=%zu must be multiple of 4 (output is packed)", c_out);
    if (stride_h == 0 || stride_w == 0 || h_in + 2 * pad_h < k_h || w_in + 2 * pad_w < k_w || n == 0 || k_h == 0 ||
        k_w == 0)
        return dw_fail(be, DW_ERR_INVALID_ARG, "conv_fused: invalid geometry");
    size_t h_out = (h_in + 2 * pad_h - k_h) / stride_h + 1;
    size_t w_out = (w_in + 2 * pad_w - k_w) / stride_w + 1;
    size_t expected_input = n * h_in * w_in * c_in;
    size_t expected_kernel = k_h * k_w * c_in * c_out;
    size_t expected_output = n * h_out * w_out * c_out;
    if (input->len != expected_input)
        return dw_fail(be, DW_ERR_SIZE_MISMATCH, "conv_fused: input mismatch: expected %zu, got %zu", expected_input,
                       input->len);
    if (kernel_hwio->len != expected_kernel)
        return dw_fail(be, DW_ERR_SIZE_MISMATCH, "conv_fused: kernel mismatch: expected %zu, got %zu",
                       expected_kernel, kernel_hwio->len);
    if (output->len != expected_output)
        return dw_fail(be, DW_ERR_SIZE_MISMATCH, "conv_fused: output mismatch: expected %zu, got %zu",
                       expected_output, output->len);
    dw_conv_desc d{};
    d.n = (int32_t)n; d.h = (int32_t)h_in; d.w = (int32_t)w_in; d.c_in = (int32_t)c_in; d.c_out = (int32_t)c_out;
    d.k_h = (int32_t)k_h; d.k_w = (int32_t)k_w; d.stride_h = (int32_t)stride_h; d.stride_w = (int32_t)stride_w;
    d.pad_t = d.pad_b = (int32_t)pad_h; d.pad_l = d.pad_r = (int32_t)pad_w;
    d.group = 1;
    d.epilogue = do_relu ? DW_EPI_RELU : DW_EPI_NONE;
    d.q6 = 127;
    int ho, wo;
    DW_TRY(check_desc(be, &d, &ho, &wo, "conv_fused"));
    cudaSetDevice(be->device);
    // Scratch: [prepared weights | M filled with the scalar requant_scale]
    void *scr = nullptr;
    size_t off_m = al256(expected_kernel);
    DW_TRY(dw_scratch(be, off_m + 4 * c_out, &scr));
    dw_buf wprep{scr, expected_kernel, false};
    dw_buf mbuf{(char *)scr + off_m, 4 * c_out, false};
    // the weights repacked and the scalar scale spread per channel by one kernel on
    // the backend stream (no host copy: the call stays asynchronous)
    DW_TRY(dw::launch_repack_hwio_to_ohwi_fill(be, (const int8_t *)kernel_hwio->ptr, (int8_t *)wprep.ptr,
                                               (int)(k_h * k_w), (int)c_in, (int)c_out, (float *)mbuf.ptr,
                                               requant_scale));
    dw::EpiParams ep{nullptr, (const float *)mbuf.ptr, nullptr, d.epilogue, 127, 0.0f};
    return conv_dispatch(be, &d, ho, wo, input, &wprep, ep, output, "conv_fused");
}

DW_API dw_status dw_conv2d_i8_nhwc(dw_backend *be, const dw_buf *input, const dw_buf *kernel_hwio,
                                   dw_buf *output_i32, size_t n, size_t h_in, size_t w_in, size_t c_in, size_t c_out,
                                   size_t k_h, size_t k_w, size_t stride_h, size_t stride_w, size_t pad_h,
                                   size_t pad_w) {
    if (!be) return DW_ERR_INVALID_ARG;
    if (!input || !kernel_hwio || !output_i32) return dw_fail(be, DW_ERR_INVALID_ARG, "conv2d_i8: null buffer");
    dw_conv_desc d{};
    d.n = (int32_t)n; d.h = (int32_t)h_in; d.w = (int32_t)w_in; d.c_in = (int32_t)c_in; d.c_out = (int32_t)c_out;
    d.k_h = (int32_t)k_h; d.k_w = (int32_t)k_w; d.stride_h = (int32_t)stride_h; d.stride_w = (int32_t)stride_w;
    d.pad_t = d.pad_b = (int32_t)pad_h; d.pad_l = d.pad_r = (int32_t)pad_w;
    d.group = 1;
    int ho, wo;
    DW_TRY(check_desc(be, &d, &ho, &wo, "conv2d_i8"));
    DW_TRY(check_len(be, input, n * h_in * w_in * c_in, "conv2d_i8", "input"));
    DW_TRY(check_len(be, kernel_hwio, k_h * k_w * c_in * c_out, "conv2d_i8", "kernel"));
    DW_TRY(check_len(be, output_i32, 4 * n * (size_t)ho * wo * c_out, "conv2d_i8", "output"));
    cudaSetDevice(be->device);
    void *scr = nullptr;
    DW_TRY(dw_scratch(be, kernel_hwio->len, &scr));
    DW_TRY(dw::launch_repack_hwio_to_ohwi(be, (const int8_t *)kernel_hwio->ptr, (int8_t *)scr, (int)(k_h * k_w),
                                          (int)c_in, (int)c_out));
    dw::EpiParams ep{nullptr, nullptr, nullptr, DW_EPI_NONE, 127, 0.0f};
    return dw::launch_conv_direct_i8(be, d, ho, wo, (const int8_t *)input->ptr, (const int8_t *)scr, ep, nullptr,
                                     (int32_t *)output_i32->ptr);
}

DW_API dw_status dw_gemm_i8(dw_backend *be, const dw_buf *a, const dw_buf *b, dw_buf *c_i32, size_t m, size_t n,
                            size_t k) {
    if (!be) return DW_ERR_INVALID_ARG;
    if (!a || !b || !c_i32) return dw_fail(be, DW_ERR_INVALID_ARG, "gemm_i8: null buffer");
    if (!m || !n || !k) return dw_fail(be, DW_ERR_INVALID_ARG, "gemm_i8: zero dimension");
    // crates/dragonwing-cpu/src/ops.rs:2965-2967
    DW_TRY(check_len(be, a, m * k, "gemm_i8", "A size"));
    DW_TRY(check_len(be, b, k * n, "gemm_i8", "B size"));
    DW_TRY(check_len(be, c_i32, 4 * m * n, "gemm_i8", "C size"));
    cudaSetDevice(be->device);
    void *scr = nullptr;
    DW_TRY(dw_scratch(be, k * n, &scr));
    DW_TRY(dw::launch_transpose_kn_to_nk(be, (const int8_t *)b->ptr, (int8_t *)scr, (int)k, (int)n));
    dw_conv_desc d{};
    d.n = 1; d.h = 1; d.w = (int32_t)m; d.c_in = (int32_t)k; d.c_out = (int32_t)n;
    d.k_h = d.k_w = d.stride_h = d.stride_w = 1;
    d.group = 1;
    dw::EpiParams ep{nullptr, nullptr, nullptr, DW_EPI_NONE, 127, 0.0f};
    return dw::launch_conv_direct_i8(be, d, 1, (int)m, (const int8_t *)a->ptr, (const int8_t *)scr, ep, nullptr,
                                     (int32_t *)c_i32->ptr);
}

DW_API dw_status dw_prepare_gemm_b_i8(dw_backend *be, const dw_buf *b_kn, size_t k, size_t n, dw_buf **out) {
    if (!be) return DW_ERR_INVALID_ARG;
    if (!b_kn || !out) return dw_fail(be, DW_ERR_INVALID_ARG, "prepare_gemm_b_i8: null argument");
    *out = nullptr;
    if (!k || !n) return dw_fail(be, DW_ERR_INVALID_ARG, "prepare_gemm_b_i8: zero dimension");
    DW_TRY(check_len(be, b_kn, k * n, "prepare_gemm_b_i8", "B size"));
    cudaSetDevice(be->device);
    dw_buf *o = nullptr;
    DW_TRY(dw_alloc(be, k * n, &o));
    dw_status st = dw::launch_transpose_kn_to_nk(be, (const int8_t *)b_kn->ptr, (int8_t *)o->ptr, (int)k, (int)n);
    if (st != DW_OK) {
        dw_free(be, o);
        return st;
    }
    *out = o;
    return DW_OK;
}

DW_API dw_status dw_qgemm_i8(dw_backend *be, const dw_buf *a, const dw_buf *b_prep, const dw_buf *bias,
                             const dw_buf *M, dw_buf *y, size_t m, size_t n, size_t k, int epilogue, int q6) {
    const char *op = "qgemm_i8";
    if (!be) return DW_ERR_INVALID_ARG;
    if (!a || !b_prep || !M || !y) return dw_fail(be, DW_ERR_INVALID_ARG, "%s: null buffer", op);
    if (!m || !n || !k) return dw_fail(be, DW_ERR_INVALID_ARG, "%s: zero dimension", op);
    if (m > 0x7fffffff || n > 0x7fffffff || k > 0x7fffffff)
        return dw_fail(be, DW_ERR_INVALID_ARG, "%s: dimension exceeds int32", op);
    if (epilogue == DW_EPI_SILU) return dw_fail(be, DW_ERR_UNSUPPORTED, "%s: SILU epilogue needs D; use conv2d_i8", op);
    dw_conv_desc d{};
    d.n = 1; d.h = 1; d.w = (int32_t)m; d.c_in = (int32_t)k; d.c_out = (int32_t)n;
    d.k_h = d.k_w = d.stride_h = d.stride_w = 1;
    d.group = 1; d.epilogue = epilogue; d.q6 = q6;
    int ho, wo;
    DW_TRY(check_desc(be, &d, &ho, &wo, op));
    DW_TRY(check_len(be, a, m * k, op, "A size"));
    DW_TRY(check_len(be, b_prep, k * n, op, "B size"));
    DW_TRY(check_len(be, y, m * n, op, "Y size"));
    DW_TRY(check_len(be, M, 4 * n, op, "M size"));
    if (bias) DW_TRY(check_len(be, bias, 4 * n, op, "bias size"));
    cudaSetDevice(be->device);
    dw::EpiParams ep{bias ? (const int32_t *)bias->ptr : nullptr, (const float *)M->ptr, nullptr, epilogue, q6, 0.0f};
    return conv_dispatch(be, &d, ho, wo, a, b_prep, ep, y, op);
}

// ---------------------------------------------------------------------------
// elementwise / glue
// ---------------------------------------------------------------------------

DW_API dw_status dw_requantize_i32_to_i8(dw_backend *be, const dw_buf *in_i32, dw_buf *out_i8, float scale) {
    if (!be) return DW_ERR_INVALID_ARG;
    if (!in_i32 || !out_i8) return dw_fail(be, DW_ERR_INVALID_ARG, "requantize_i32_to_i8: null buffer");
    if (in_i32->len % 4 || in_i32->len / 4 != out_i8->len)
        return dw_fail(be, DW_ERR_SIZE_MISMATCH, "requantize_i32_to_i8: length mismatch (%zu i32 bytes vs %zu i8)",
                       in_i32->len, out_i8->len);
    cudaSetDevice(be->device);
    return dw::launch_requantize(be, (const int32_t *)in_i32->ptr, (int8_t *)out_i8->ptr, out_i8->len, scale);
}

DW_API dw_status dw_relu_i8(dw_backend *be, const dw_buf *in, dw_buf *out) {
    if (!be) return DW_ERR_INVALID_ARG;
    if (!in || !out) return dw_fail(be, DW_ERR_INVALID_ARG, "relu_i8: null buffer");
    if (in->len != out->len) return dw_fail(be, DW_ERR_SIZE_MISMATCH, "relu_i8: length mismatch");
    cudaSetDevice(be->device);
    return dw::launch_relu_i8(be, (const int8_t *)in->ptr, (int8_t *)out->ptr, in->len);
}

DW_API dw_status dw_add_i8(dw_backend *be, const dw_buf *a, const dw_buf *b, dw_buf *out, float scale_a_over_y,
                           float scale_b_over_y) {
    if (!be) return DW_ERR_INVALID_ARG;
    if (!a || !b || !out) return dw_fail(be, DW_ERR_INVALID_ARG, "add_i8: null buffer");
    // crates/dragonwing-cpu/src/ops.rs:3183-3184
    if (out->len != a->len) return dw_fail(be, DW_ERR_SIZE_MISMATCH, "add_i8: output/a length mismatch");
    if (out->len != b->len) return dw_fail(be, DW_ERR_SIZE_MISMATCH, "add_i8: output/b length mismatch");
    cudaSetDevice(be->device);
    return dw::launch_add_i8(be, (const int8_t *)a->ptr, (const int8_t *)b->ptr, (int8_t *)out->ptr, out->len,
                             scale_a_over_y, scale_b_over_y);
}

DW_API dw_status dw_quantize_f32_to_i8(dw_backend *be, const dw_buf *in_f32, dw_buf *out_i8, float scale) {
    if (!be) return DW_ERR_INVALID_ARG;
    if (!in_f32 || !out_i8) return dw_fail(be, DW_ERR_INVALID_ARG, "quantize_f32_to_i8: null buffer");
    if (in_f32->len % 4 || in_f32->len / 4 != out_i8->len)
        return dw_fail(be, DW_ERR_SIZE_MISMATCH, "quantize_f32_to_i8: length mismatch");
    cudaSetDevice(be->device);
    return dw::launch_quantize_f32(be, (const float *)in_f32->ptr, (int8_t *)out_i8->ptr, out_i8->len, scale);
}

DW_API dw_status dw_quantize_u8_to_i8(dw_backend *be, const dw_buf *in_u8, dw_buf *out_i8, float scale) {
    if (!be) return DW_ERR_INVALID_ARG;
    if (!in_u8 || !out_i8) return dw_fail(be, DW_ERR_INVALID_ARG, "quantize_u8_to_i8: null buffer");
    if (in_u8->len != out_i8->len) return dw_fail(be, DW_ERR_SIZE_MISMATCH, "quantize_u8_to_i8: length mismatch");
    cudaSetDevice(be->device);
    return dw::launch_quantize_u8(be, (const uint8_t *)in_u8->ptr, (int8_t *)out_i8->ptr, out_i8->len, scale);
}

DW_API dw_status dw_conv2d_stem_u8_i8(dw_backend *be, const dw_conv_desc *d, const dw_buf *x_u8, float in_scale,
                                      const dw_buf *kernel_hwio, const dw_buf *bias, const dw_buf *M, const dw_buf *D,
                                      dw_buf *y) {
    const char *op = "conv2d_stem_u8_i8";
    if (!be) return DW_ERR_INVALID_ARG;
    int ho, wo;
    DW_TRY(check_desc(be, d, &ho, &wo, op));
    if (d->c_in != 3 || d->k_h != 3 || d->k_w != 3 || d->group != 1)
        return dw_fail(be, DW_ERR_UNSUPPORTED, "%s: only the 3x3 conv on a 3-channel image (c_in=%d, %dx%d, group %d)",
                       op, d->c_in, d->k_h, d->k_w, d->group);
    if (!(in_scale > 0.0f) || !std::isfinite(in_scale))
        return dw_fail(be, DW_ERR_INVALID_ARG, "%s: input scale must be positive and finite", op);
    DW_TRY(need(be, x_u8, op, "input"));
    DW_TRY(need(be, kernel_hwio, op, "kernel"));
    DW_TRY(need(be, y, op, "output"));
    DW_TRY(check_len(be, x_u8, (size_t)d->n * d->h * d->w * 3, op, "input"));
    DW_TRY(check_len(be, kernel_hwio, (size_t)27 * d->c_out, op, "kernel"));
    DW_TRY(check_len(be, y, (size_t)d->n * ho * wo * d->c_out, op, "output"));
    if (bias) DW_TRY(check_len(be, bias, 4 * (size_t)d->c_out, op, "bias"));
    if (d->epilogue == DW_EPI_SILU) {
        DW_TRY(need(be, D, op, "D (dequant scales, required by SILU)"));
        DW_TRY(check_len(be, D, 4 * (size_t)d->c_out, op, "D"));
    } else {
        DW_TRY(need(be, M, op, "M (requant scales)"));
        DW_TRY(check_len(be, M, 4 * (size_t)d->c_out, op, "M"));
    }
    cudaSetDevice(be->device);
    dw::EpiParams ep{bias ? (const int32_t *)bias->ptr : nullptr, M ? (const float *)M->ptr : nullptr,
                     D ? (const float *)D->ptr : nullptr, d->epilogue, d->q6, d->inv_s_out};
    return dw::launch_stem3_conv_u8_i8(be, (const uint8_t *)x_u8->ptr, (const int8_t *)kernel_hwio->ptr, ep,
                                       (int8_t *)y->ptr, d->n, d->h, d->w, d->stride_h, d->stride_w, d->pad_t,
                                       d->pad_l, ho, wo, d->c_out, in_scale);
}

DW_API dw_status dw_im2col_u8_to_i8(dw_backend *be, const dw_buf *x_u8, dw_buf *y_i8, size_t n, size_t h, size_t w,
                                    size_t c, size_t k_h, size_t k_w, size_t s_h, size_t s_w, size_t p_t, size_t p_l,
                                    size_t h_out, size_t w_out, size_t c_dst, float scale) {
    const char *op = "im2col_u8_to_i8";
    if (!be) return DW_ERR_INVALID_ARG;
    if (!x_u8 || !y_i8) return dw_fail(be, DW_ERR_INVALID_ARG, "%s: null buffer", op);
    if (!n || !h || !w || !c || !k_h || !k_w || !s_h || !s_w || !h_out || !w_out || c_dst % 16 || c_dst > 64 ||
        k_h > 8 || k_w > 8 || c > 8 ||
        k_h * k_w * c > c_dst || n * h_out * w_out > 0x7fffffff || n * h * w * c > 0x7fffffffffffll)
        return dw_fail(be, DW_ERR_INVALID_ARG, "%s: invalid geometry (c_dst a multiple of 16 >= k_h*k_w*c)", op);
    DW_TRY(check_len(be, x_u8, n * h * w * c, op, "input"));
    DW_TRY(check_len(be, y_i8, n * h_out * w_out * c_dst, op, "output"));
    if ((uintptr_t)y_i8->ptr & 15) return dw_fail(be, DW_ERR_INVALID_ARG, "%s: output must be 16-byte aligned", op);
    cudaSetDevice(be->device);
    return dw::launch_im2col_u8_i8(be, (const uint8_t *)x_u8->ptr, (int8_t *)y_i8->ptr, (int)n, (int)h, (int)w, (int)c,
                                   (int)k_h, (int)k_w, (int)s_h, (int)s_w, (int)p_t, (int)p_l, (int)h_out, (int)w_out,
                                   (int)c_dst, scale);
}

DW_API dw_status dw_dequantize_i8_to_f32(dw_backend *be, const dw_buf *in_i8, dw_buf *out_f32, float scale) {
    if (!be) return DW_ERR_INVALID_ARG;
    if (!in_i8 || !out_f32) return dw_fail(be, DW_ERR_INVALID_ARG, "dequantize_i8_to_f32: null buffer");
    if (out_f32->len % 4 || out_f32->len / 4 != in_i8->len)
        return dw_fail(be, DW_ERR_SIZE_MISMATCH, "dequantize_i8_to_f32: length mismatch");
    cudaSetDevice(be->device);
    return dw::launch_dequantize(be, (const int8_t *)in_i8->ptr, (float *)out_f32->ptr, in_i8->len, scale);
}

DW_API dw_status dw_maxpool_i8(dw_backend *be, const dw_buf *x, dw_buf *y, size_t n, size_t h, size_t w, size_t c,
                               size_t k_h, size_t k_w, size_t s_h, size_t s_w, size_t p_t, size_t p_l, size_t p_b,
                               size_t p_r) {
    if (!be) return DW_ERR_INVALID_ARG;
    if (!x || !y) return dw_fail(be, DW_ERR_INVALID_ARG, "maxpool_i8: null buffer");
    if (!n || !h || !w || !c || !k_h || !k_w || !s_h || !s_w || p_t >= k_h || p_b >= k_h || p_l >= k_w || p_r >= k_w ||
        h + p_t + p_b < k_h || w + p_l + p_r < k_w)
        return dw_fail(be, DW_ERR_INVALID_ARG, "maxpool_i8: invalid geometry");
    size_t ho = (h + p_t + p_b - k_h) / s_h + 1, wo = (w + p_l + p_r - k_w) / s_w + 1;
    DW_TRY(check_len(be, x, n * h * w * c, "maxpool_i8", "input"));
    DW_TRY(check_len(be, y, n * ho * wo * c, "maxpool_i8", "output"));
    cudaSetDevice(be->device);
    return dw::launch_maxpool_i8(be, (const int8_t *)x->ptr, (int8_t *)y->ptr, (int)n, (int)h, (int)w, (int)c,
                                 (int)k_h, (int)k_w, (int)s_h, (int)s_w, (int)p_t, (int)p_l, (int)ho, (int)wo);
}

namespace {
// A view of `pixels` pixels of `c` bytes must end inside its buffer.
dw_status check_view(dw_backend *be, const dw_view *v, size_t pixels, size_t c, const char *op, const char *name) {
    if (!v || !v->buf) return dw_fail(be, DW_ERR_INVALID_ARG, "%s: %s view is null", op, name);
    if (v->pitch <= 0 || (size_t)v->pitch < c || (v->offset % 16) || (v->pitch % 16))
        return dw_fail(be, DW_ERR_INVALID_ARG, "%s: %s view pitch %d / offset %zu (16-byte multiples, pitch >= %zu)", op,
                       name, (int)v->pitch, v->offset, c);
    const size_t end = pixels ? v->offset + (pixels - 1) * (size_t)v->pitch + c : v->offset;
    if (end > v->buf->len)
        return dw_fail(be, DW_ERR_SIZE_MISMATCH, "%s: %s view ends at %zu, past the buffer's %zu bytes", op, name, end,
                       v->buf->len);
    return DW_OK;
}
}  // namespace

DW_API dw_status dw_conv2d_i8_view(dw_backend *be, const dw_conv_desc *d, const dw_view *x, const dw_buf *w_prep,
                                   const dw_buf *bias, const dw_buf *M, const dw_buf *D, const dw_view *y) {
    const char *op = "conv2d_i8_view";
    if (!be) return DW_ERR_INVALID_ARG;
    int ho, wo;
    DW_TRY(check_desc(be, d, &ho, &wo, op));
    DW_TRY(need(be, w_prep, op, "kernel"));
    DW_TRY(check_view(be, x, (size_t)d->n * d->h * d->w, d->c_in, op, "input"));
    DW_TRY(check_view(be, y, (size_t)d->n * ho * wo, d->c_out, op, "output"));
    DW_TRY(check_len(be, w_prep, weight_len(d), op, "kernel"));
    if (bias) DW_TRY(check_len(be, bias, 4 * (size_t)d->c_out, op, "bias"));
    if (d->epilogue == DW_EPI_SILU) {
        DW_TRY(need(be, D, op, "D (dequant scales, required by SILU)"));
        DW_TRY(check_len(be, D, 4 * (size_t)d->c_out, op, "D"));
    } else {
        DW_TRY(need(be, M, op, "M (requant scales)"));
        DW_TRY(check_len(be, M, 4 * (size_t)d->c_out, op, "M"));
    }
    if (be->cfg.conv_path == DW_PATH_DIRECT || !dw::umma_supported(be, *d, ho, wo))
        return dw_fail(be, DW_ERR_UNSUPPORTED, "%s: views need the tensor-core path (c_in=%d c_out=%d group=%d)", op,
                       d->c_in, d->c_out, d->group);
    cudaSetDevice(be->device);
    dw::EpiParams ep{bias ? (const int32_t *)bias->ptr : nullptr, M ? (const float *)M->ptr : nullptr,
                     D ? (const float *)D->ptr : nullptr, d->epilogue, d->q6, d->inv_s_out};
    return dw::launch_umma_conv_i8_view(be, *d, ho, wo, (const int8_t *)x->buf->ptr + x->offset, x->pitch,
                                        (const int8_t *)w_prep->ptr, ep, (int8_t *)y->buf->ptr + y->offset, y->pitch);
}

DW_API dw_status dw_conv2d_add_i8_view(dw_backend *be, const dw_conv_desc *d, const dw_view *x, const dw_buf *w_prep,
                                       const dw_buf *bias, const dw_buf *M, const dw_buf *D, const dw_view *residual,
                                       float ra, float rb, const dw_view *y) {
    const char *op = "conv2d_add_i8_view";
    if (!be) return DW_ERR_INVALID_ARG;
    int ho, wo;
    DW_TRY(check_desc(be, d, &ho, &wo, op));
    DW_TRY(need(be, w_prep, op, "kernel"));
    DW_TRY(check_view(be, x, (size_t)d->n * d->h * d->w, d->c_in, op, "input"));
    DW_TRY(check_view(be, residual, (size_t)d->n * ho * wo, d->c_out, op, "residual"));
    DW_TRY(check_view(be, y, (size_t)d->n * ho * wo, d->c_out, op, "output"));
    DW_TRY(check_len(be, w_prep, weight_len(d), op, "kernel"));
    if (bias) DW_TRY(check_len(be, bias, 4 * (size_t)d->c_out, op, "bias"));
    if (d->epilogue == DW_EPI_SILU) {
        DW_TRY(need(be, D, op, "D (dequant scales, required by SILU)"));
        DW_TRY(check_len(be, D, 4 * (size_t)d->c_out, op, "D"));
    } else {
        DW_TRY(need(be, M, op, "M (requant scales)"));
        DW_TRY(check_len(be, M, 4 * (size_t)d->c_out, op, "M"));
    }
    if (!(std::fabs(ra) < 1e30f) || !(std::fabs(rb) < 1e30f))
        return dw_fail(be, DW_ERR_UNSUPPORTED, "%s: add ratios must be below 1e30 in magnitude", op);
    if (be->cfg.conv_path == DW_PATH_DIRECT || !dw::umma_supported(be, *d, ho, wo) || d->c_out % 16)
        return dw_fail(be, DW_ERR_UNSUPPORTED, "%s: needs the tensor-core path (c_in=%d c_out=%d group=%d)", op,
                       d->c_in, d->c_out, d->group);
    cudaSetDevice(be->device);
    dw::EpiParams ep{bias ? (const int32_t *)bias->ptr : nullptr, M ? (const float *)M->ptr : nullptr,
                     D ? (const float *)D->ptr : nullptr, d->epilogue, d->q6, d->inv_s_out};
    return dw::launch_umma_conv_add_i8_view(be, *d, ho, wo, (const int8_t *)x->buf->ptr + x->offset, x->pitch,
                                            (const int8_t *)w_prep->ptr, ep,
                                            (const int8_t *)residual->buf->ptr + residual->offset, residual->pitch,
                                            ra, rb, (int8_t *)y->buf->ptr + y->offset, y->pitch);
}

DW_API dw_status dw_add_i8_view(dw_backend *be, const dw_view *a, const dw_view *b, const dw_view *out, size_t pixels,
                                size_t c, float scale_a_over_y, float scale_b_over_y) {
    const char *op = "add_i8_view";
    if (!be) return DW_ERR_INVALID_ARG;
    if (!pixels || !c) return dw_fail(be, DW_ERR_INVALID_ARG, "%s: empty tensor", op);
    DW_TRY(check_view(be, a, pixels, c, op, "a"));
    DW_TRY(check_view(be, b, pixels, c, op, "b"));
    DW_TRY(check_view(be, out, pixels, c, op, "output"));
    cudaSetDevice(be->device);
    return dw::launch_add_i8_view(be, (const int8_t *)a->buf->ptr + a->offset, a->pitch,
                                  (const int8_t *)b->buf->ptr + b->offset, b->pitch,
                                  (int8_t *)out->buf->ptr + out->offset, out->pitch, pixels, (int)c, scale_a_over_y,
                                  scale_b_over_y);
}

DW_API dw_status dw_maxpool_i8_view(dw_backend *be, const dw_view *x, const dw_view *y, size_t n, size_t h, size_t w,
                                    size_t c, size_t k_h, size_t k_w, size_t s_h, size_t s_w, size_t p_t, size_t p_l,
                                    size_t p_b, size_t p_r) {
    const char *op = "maxpool_i8_view";
    if (!be) return DW_ERR_INVALID_ARG;
    if (!n || !h || !w || !c || !k_h || !k_w || !s_h || !s_w || p_t >= k_h || p_b >= k_h || p_l >= k_w || p_r >= k_w ||
        h + p_t + p_b < k_h || w + p_l + p_r < k_w)
        return dw_fail(be, DW_ERR_INVALID_ARG, "%s: invalid geometry", op);
    const size_t ho = (h + p_t + p_b - k_h) / s_h + 1, wo = (w + p_l + p_r - k_w) / s_w + 1;
    DW_TRY(check_view(be, x, n * h * w, c, op, "input"));
    DW_TRY(check_view(be, y, n * ho * wo, c, op, "output"));
    cudaSetDevice(be->device);
    return dw::launch_maxpool_i8_view(be, (const int8_t *)x->buf->ptr + x->offset, x->pitch,
                                      (int8_t *)y->buf->ptr + y->offset, y->pitch, (int)n, (int)h, (int)w, (int)c,
                                      (int)k_h, (int)k_w, (int)s_h, (int)s_w, (int)p_t, (int)p_l, (int)ho, (int)wo);
}

DW_API dw_status dw_maxpool_chain_i8_view(dw_backend *be, const dw_view *x, const dw_view *ys, int32_t count, size_t n,
                                          size_t h, size_t w, size_t c, size_t k) {
    const char *op = "maxpool_chain_i8_view";
    if (!be) return DW_ERR_INVALID_ARG;
    if (!ys || count < 1 || count > 4 || !n || !h || !w || !c || k % 2 == 0 || k > 255 ||
        n * h * w >= ((size_t)1 << 31) || c > 65536)
        return dw_fail(be, DW_ERR_INVALID_ARG, "%s: invalid geometry (1..4 pools, odd k)", op);
    DW_TRY(check_view(be, x, n * h * w, c, op, "input"));
    int8_t *yp[4];
    int pitches[4];
    for (int i = 0; i < count; i++) {
        DW_TRY(check_view(be, &ys[i], n * h * w, c, op, "output"));
        yp[i] = (int8_t *)ys[i].buf->ptr + ys[i].offset;
        pitches[i] = ys[i].pitch;
    }
    cudaSetDevice(be->device);
    return dw::launch_maxpool_chain_i8_view(be, (const int8_t *)x->buf->ptr + x->offset, x->pitch, yp, pitches, count,
                                            (int)n, (int)h, (int)w, (int)c, (int)k);
}

DW_API dw_status dw_concat_i8(dw_backend *be, const dw_buf *const *xs, const int32_t *channels, int32_t count,
                              size_t pixels, dw_buf *y) {
    if (!be) return DW_ERR_INVALID_ARG;
    if (!xs || !channels || !y || count <= 0 || count > 16 || !pixels)
        return dw_fail(be, DW_ERR_INVALID_ARG, "concat_i8: need 1..16 inputs and a non-empty output");
    size_t ct = 0;
    const int8_t *ptrs[16];
    for (int i = 0; i < count; i++) {
        if (!xs[i] || channels[i] <= 0) return dw_fail(be, DW_ERR_INVALID_ARG, "concat_i8: input %d invalid", i);
        if (xs[i]->len != pixels * (size_t)channels[i])
            return dw_fail(be, DW_ERR_SIZE_MISMATCH, "concat_i8: input size mismatch (input %d)", i);
        ct += (size_t)channels[i];
        ptrs[i] = (const int8_t *)xs[i]->ptr;
    }
    DW_TRY(check_len(be, y, pixels * ct, "concat_i8", "output size"));
    cudaSetDevice(be->device);
    return dw::launch_concat_i8(be, ptrs, channels, count, pixels, (int8_t *)y->ptr);
}

DW_API dw_status dw_slice_c_i8(dw_backend *be, const dw_buf *x, dw_buf *y, size_t pixels, size_t c_total, size_t c0,
                               size_t c_len) {
    if (!be) return DW_ERR_INVALID_ARG;
    if (!x || !y || !pixels || !c_len || c0 + c_len > c_total)
        return dw_fail(be, DW_ERR_INVALID_ARG, "slice_c_i8: invalid range");
    DW_TRY(check_len(be, x, pixels * c_total, "slice_c_i8", "input"));
    DW_TRY(check_len(be, y, pixels * c_len, "slice_c_i8", "output"));
    cudaSetDevice(be->device);
    return dw::launch_slice_c_i8(be, (const int8_t *)x->ptr, (int8_t *)y->ptr, pixels, (int)c_total, (int)c0,
                                 (int)c_len);
}

DW_API dw_status dw_resize_nearest_i8(dw_backend *be, const dw_buf *x, dw_buf *y, size_t n, size_t h_in,
                                      size_t w_in, size_t h_out, size_t w_out, size_t c) {
    if (!be) return DW_ERR_INVALID_ARG;
    if (!x || !y || !n || !h_in || !w_in || !h_out || !w_out || !c)
        return dw_fail(be, DW_ERR_INVALID_ARG, "resize_nearest_i8: invalid geometry");
    DW_TRY(check_len(be, x, n * h_in * w_in * c, "resize_nearest_i8", "input"));
    DW_TRY(check_len(be, y, n * h_out * w_out * c, "resize_nearest_i8", "output"));
    cudaSetDevice(be->device);
    return dw::launch_resize_nearest_i8(be, (const int8_t *)x->ptr, (int8_t *)y->ptr, (int)n, (int)h_in, (int)w_in,
                                        (int)h_out, (int)w_out, (int)c);
}

// ---------------------------------------------------------------------------
// fp16 path
// ---------------------------------------------------------------------------

DW_API dw_status dw_prepare_weights_f16(dw_backend *be, const dw_conv_desc *d, const dw_buf *w_hwio, dw_buf **out) {
    const char *op = "prepare_weights_f16";
    if (!be) return DW_ERR_INVALID_ARG;
    DW_TRY(need(be, out, op, "out"));
    *out = nullptr;
    DW_TRY(need(be, w_hwio, op, "kernel"));
    int ho, wo;
    DW_TRY(check_desc(be, d, &ho, &wo, op));
    DW_TRY(check_len(be, w_hwio, 2 * weight_len(d), op, "kernel"));
    cudaSetDevice(be->device);
    dw_buf *o = nullptr;
    DW_TRY(dw_alloc(be, w_hwio->len, &o));
    dw_status st;
    if (d->group == 1) {
        st = dw::launch_repack_hwio_to_ohwi_f16(be, (const uint16_t *)w_hwio->ptr, (uint16_t *)o->ptr,
                                                d->k_h * d->k_w, d->c_in, d->c_out);
    } else {
        st = dw_cuda_check(be, cudaMemcpyAsync(o->ptr, w_hwio->ptr, w_hwio->len, cudaMemcpyDeviceToDevice, be->stream),
                           "prepare depthwise weights");
    }
    if (st != DW_OK) {
        dw_free(be, o);
        return st;
    }
    *out = o;
    return DW_OK;
}

// fp16 conv (+ bias) (+ residual) (+ ReLU).  The tensor-core kernel fuses the
// residual into its epilogue for 1x1 stride-1 convs; elsewhere the residual
// is added (with the ReLU) by a second pass over y, with the same arithmetic.
static dw_status conv_dispatch_f16(dw_backend *be, const dw_conv_desc *d, int ho, int wo, const dw_buf *x,
                                   const dw_buf *w_prep, const dw_buf *bias, dw_buf *y, const char *op,
                                   const dw_buf *residual = nullptr) {
    const uint16_t *xp = (const uint16_t *)x->ptr;
    const uint16_t *wp = (const uint16_t *)w_prep->ptr;
    const uint16_t *bp = bias ? (const uint16_t *)bias->ptr : nullptr;
    const uint16_t *rp = residual ? (const uint16_t *)residual->ptr : nullptr;
    uint16_t *yp = (uint16_t *)y->ptr;
    const int relu = d->epilogue == DW_EPI_RELU ? 1 : 0;
    const bool flat = d->k_h == 1 && d->k_w == 1 && d->stride_h == 1 && d->stride_w == 1 && d->pad_t == 0 &&
                      d->pad_l == 0 && d->pad_b == 0 && d->pad_r == 0;
    const int path = be->cfg.conv_path;
    const bool umma = d->group == 1 && path != DW_PATH_DIRECT && dw::umma_supported_f16(be, *d, ho, wo);
    if (d->group == 1 && !umma && path == DW_PATH_UMMA)
        return dw_fail(be, DW_ERR_UNSUPPORTED, "%s: shape not supported by the tensor-core kernel (c_in=%d c_out=%d)",
                       op, d->c_in, d->c_out);
    if (umma && (!rp || (flat && ((uintptr_t)rp & 15) == 0)))
        return dw::launch_umma_conv_f16(be, *d, ho, wo, xp, wp, bp, relu, yp, rp);
    const int relu1 = rp ? 0 : relu;
    dw_status st;
    if (d->group != 1)
        st = dw::launch_dwconv_f16(be, *d, ho, wo, xp, wp, bp, relu1, yp);
    else if (umma)
        st = dw::launch_umma_conv_f16(be, *d, ho, wo, xp, wp, bp, relu1, yp, nullptr);
    else
        st = dw::launch_conv_direct_f16(be, *d, ho, wo, xp, wp, bp, relu1, yp);
    if (st != DW_OK || !rp) return st;
    return dw::launch_add_f16(be, yp, rp, yp, y->len / 2, relu);
}

DW_API dw_status dw_conv2d_f16(dw_backend *be, const dw_conv_desc *d, const dw_buf *x, const dw_buf *w_prep,
                               const dw_buf *bias_or_null, dw_buf *y) {
    const char *op = "conv2d_f16";
    if (!be) return DW_ERR_INVALID_ARG;
    int ho, wo;
    DW_TRY(check_desc(be, d, &ho, &wo, op));
    if (d->epilogue != DW_EPI_NONE && d->epilogue != DW_EPI_RELU)
        return dw_fail(be, DW_ERR_UNSUPPORTED, "%s: epilogue %d unsupported (NONE or RELU)", op, d->epilogue);
    DW_TRY(need(be, x, op, "input"));
    DW_TRY(need(be, w_prep, op, "kernel"));
    DW_TRY(need(be, y, op, "output"));
    DW_TRY(check_len(be, x, 2 * (size_t)d->n * d->h * d->w * d->c_in, op, "input"));
    DW_TRY(check_len(be, w_prep, 2 * weight_len(d), op, "kernel"));
    DW_TRY(check_len(be, y, 2 * (size_t)d->n * ho * wo * d->c_out, op, "output"));
    if (bias_or_null) DW_TRY(check_len(be, bias_or_null, 2 * (size_t)d->c_out, op, "bias"));
    cudaSetDevice(be->device);
    return conv_dispatch_f16(be, d, ho, wo, x, w_prep, bias_or_null, y, op);
}

DW_API dw_status dw_conv2d_add_f16(dw_backend *be, const dw_conv_desc *d, const dw_buf *x, const dw_buf *w_prep,
                                   const dw_buf *bias_or_null, const dw_buf *residual, dw_buf *y) {
    const char *op = "conv2d_add_f16";
    if (!be) return DW_ERR_INVALID_ARG;
    int ho, wo;
    DW_TRY(check_desc(be, d, &ho, &wo, op));
    if (d->epilogue != DW_EPI_NONE && d->epilogue != DW_EPI_RELU)
        return dw_fail(be, DW_ERR_UNSUPPORTED, "%s: epilogue %d unsupported (NONE or RELU)", op, d->epilogue);
    DW_TRY(need(be, x, op, "input"));
    DW_TRY(need(be, w_prep, op, "kernel"));
    DW_TRY(need(be, residual, op, "residual"));
    DW_TRY(need(be, y, op, "output"));
    DW_TRY(check_len(be, x, 2 * (size_t)d->n * d->h * d->w * d->c_in, op, "input"));
    DW_TRY(check_len(be, w_prep, 2 * weight_len(d), op, "kernel"));
    DW_TRY(check_len(be, y, 2 * (size_t)d->n * ho * wo * d->c_out, op, "output"));
    DW_TRY(check_len(be, residual, y->len, op, "residual"));
    if (bias_or_null) DW_TRY(check_len(be, bias_or_null, 2 * (size_t)d->c_out, op, "bias"));
    if (residual->ptr == y->ptr) return dw_fail(be, DW_ERR_INVALID_ARG, "%s: residual must not alias the output", op);
    cudaSetDevice(be->device);
    return conv_dispatch_f16(be, d, ho, wo, x, w_prep, bias_or_null, y, op, residual);
}

DW_API dw_status dw_conv2d_fp16_nhwc(dw_backend *be, const dw_buf *input, const dw_buf *kernel_hwio, dw_buf *output,
                                     size_t n, size_t h_in, size_t w_in, size_t c_in, size_t c_out, size_t k_h,
                                     size_t k_w, size_t stride_h, size_t stride_w, size_t pad_h, size_t pad_w) {
    const char *op = "conv2d_fp16";
    if (!be) return DW_ERR_INVALID_ARG;
    if (!input || !kernel_hwio || !output) return dw_fail(be, DW_ERR_INVALID_ARG, "%s: null buffer", op);
    if (stride_h == 0 || stride_w == 0 || h_in + 2 * pad_h < k_h || w_in + 2 * pad_w < k_w || n == 0 || k_h == 0 ||
        k_w == 0 || c_in == 0 || c_out == 0)
        return dw_fail(be, DW_ERR_INVALID_ARG, "%s: invalid geometry", op);
    // crates/dragonwing-vulkan/src/ops.rs:1401-1416 (same checks, same strings)
    const size_t h_out = (h_in + 2 * pad_h - k_h) / stride_h + 1;
    const size_t w_out = (w_in + 2 * pad_w - k_w) / stride_w + 1;
    const size_t expected_input = n * h_in * w_in * c_in * 2;
    const size_t expected_kernel = k_h * k_w * c_in * c_out * 2;
    const size_t expected_output = n * h_out * w_out * c_out * 2;
    if (input->len != expected_input)
        return dw_fail(be, DW_ERR_SIZE_MISMATCH, "%s: input size mismatch: expected %zu, got %zu", op, expected_input,
                       input->len);
    if (kernel_hwio->len != expected_kernel)
        return dw_fail(be, DW_ERR_SIZE_MISMATCH, "%s: kernel size mismatch: expected %zu, got %zu", op,
                       expected_kernel, kernel_hwio->len);
    if (output->len != expected_output)
        return dw_fail(be, DW_ERR_SIZE_MISMATCH, "%s: output size mismatch: expected %zu, got %zu", op,
                       expected_output, output->len);
    dw_conv_desc d{};
    d.n = (int32_t)n; d.h = (int32_t)h_in; d.w = (int32_t)w_in; d.c_in = (int32_t)c_in; d.c_out = (int32_t)c_out;
    d.k_h = (int32_t)k_h; d.k_w = (int32_t)k_w; d.stride_h = (int32_t)stride_h; d.stride_w = (int32_t)stride_w;
    d.pad_t = d.pad_b = (int32_t)pad_h; d.pad_l = d.pad_r = (int32_t)pad_w;
    d.group = 1;
    d.epilogue = DW_EPI_NONE;
    int ho, wo;
    DW_TRY(check_desc(be, &d, &ho, &wo, op));
    cudaSetDevice(be->device);
    void *scr = nullptr;
    DW_TRY(dw_scratch(be, expected_kernel, &scr));
    dw_buf wprep{scr, expected_kernel, false};
    DW_TRY(dw::launch_repack_hwio_to_ohwi_f16(be, (const uint16_t *)kernel_hwio->ptr, (uint16_t *)scr,
                                              (int)(k_h * k_w), (int)c_in, (int)c_out));
    return conv_dispatch_f16(be, &d, ho, wo, input, &wprep, nullptr, output, op);
}

static dw_status gemm_f16_run(dw_backend *be, const dw_buf *a, const dw_buf *b_nk, const dw_buf *bias, dw_buf *y,
                              size_t m, size_t n, size_t k, int relu, const char *op) {
    dw_conv_desc d{};
    d.n = 1; d.h = 1; d.w = (int32_t)m; d.c_in = (int32_t)k; d.c_out = (int32_t)n;
    d.k_h = d.k_w = d.stride_h = d.stride_w = 1;
    d.group = 1;
    d.epilogue = relu ? DW_EPI_RELU : DW_EPI_NONE;
    int ho, wo;
    DW_TRY(check_desc(be, &d, &ho, &wo, op));
    return conv_dispatch_f16(be, &d, ho, wo, a, b_nk, bias, y, op);
}

DW_API dw_status dw_gemm_f16(dw_backend *be, const dw_buf *a, const dw_buf *b, dw_buf *c, size_t m, size_t n,
                             size_t k) {
    const char *op = "gemm_fp16";
    if (!be) return DW_ERR_INVALID_ARG;
    if (!a || !b || !c) return dw_fail(be, DW_ERR_INVALID_ARG, "%s: null buffer", op);
    if (!m || !n || !k) return dw_fail(be, DW_ERR_INVALID_ARG, "%s: zero dimension", op);
    if (m > 0x7fffffff || n > 0x7fffffff || k > 0x7fffffff)
        return dw_fail(be, DW_ERR_INVALID_ARG, "%s: dimension exceeds int32", op);
    // crates/dragonwing-vulkan/src/ops.rs:1193-1213 (same checks, same strings)
    if (a->len != m * k * 2)
        return dw_fail(be, DW_ERR_SIZE_MISMATCH, "%s: A size mismatch: expected %zu got %zu", op, m * k * 2, a->len);
    if (b->len != k * n * 2)
        return dw_fail(be, DW_ERR_SIZE_MISMATCH, "%s: B size mismatch: expected %zu got %zu", op, k * n * 2, b->len);
    if (c->len != m * n * 2)
        return dw_fail(be, DW_ERR_SIZE_MISMATCH, "%s: C size mismatch: expected %zu got %zu", op, m * n * 2, c->len);
    cudaSetDevice(be->device);
    void *scr = nullptr;
    DW_TRY(dw_scratch(be, k * n * 2, &scr));
    DW_TRY(dw::launch_transpose_kn_to_nk_f16(be, (const uint16_t *)b->ptr, (uint16_t *)scr, (int)k, (int)n));
    dw_buf bprep{scr, k * n * 2, false};
    return gemm_f16_run(be, a, &bprep, nullptr, c, m, n, k, 0, op);
}

DW_API dw_status dw_prepare_gemm_b_f16(dw_backend *be, const dw_buf *b_kn, size_t k, size_t n, dw_buf **out) {
    if (!be) return DW_ERR_INVALID_ARG;
    if (!b_kn || !out) return dw_fail(be, DW_ERR_INVALID_ARG, "prepare_gemm_b_f16: null argument");
    *out = nullptr;
    if (!k || !n) return dw_fail(be, DW_ERR_INVALID_ARG, "prepare_gemm_b_f16: zero dimension");
    if (k > 0x7fffffff || n > 0x7fffffff)
        return dw_fail(be, DW_ERR_INVALID_ARG, "prepare_gemm_b_f16: dimension exceeds int32");
    DW_TRY(check_len(be, b_kn, k * n * 2, "prepare_gemm_b_f16", "B size"));
    cudaSetDevice(be->device);
    dw_buf *o = nullptr;
    DW_TRY(dw_alloc(be, k * n * 2, &o));
    dw_status st =
        dw::launch_transpose_kn_to_nk_f16(be, (const uint16_t *)b_kn->ptr, (uint16_t *)o->ptr, (int)k, (int)n);
    if (st != DW_OK) {
        dw_free(be, o);
        return st;
    }
    *out = o;
    return DW_OK;
}

DW_API dw_status dw_gemm_f16_bias(dw_backend *be, const dw_buf *a, const dw_buf *b_prep, const dw_buf *bias,
                                  dw_buf *y, size_t m, size_t n, size_t k, int relu) {
    const char *op = "gemm_f16";
    if (!be) return DW_ERR_INVALID_ARG;
    if (!a || !b_prep || !y) return dw_fail(be, DW_ERR_INVALID_ARG, "%s: null buffer", op);
    if (!m || !n || !k) return dw_fail(be, DW_ERR_INVALID_ARG, "%s: zero dimension", op);
    if (m > 0x7fffffff || n > 0x7fffffff || k > 0x7fffffff)
        return dw_fail(be, DW_ERR_INVALID_ARG, "%s: dimension exceeds int32", op);
    DW_TRY(check_len(be, a, m * k * 2, op, "A size"));
    DW_TRY(check_len(be, b_prep, k * n * 2, op, "B size"));
    DW_TRY(check_len(be, y, m * n * 2, op, "Y size"));
    if (bias) DW_TRY(check_len(be, bias, n * 2, op, "bias size"));
    cudaSetDevice(be->device);
    return gemm_f16_run(be, a, b_prep, bias, y, m, n, k, relu, op);
}

static dw_status add_f16_common(dw_backend *be, const dw_buf *a, const dw_buf *b, dw_buf *y, int relu,
                                const char *op) {
    if (!be) return DW_ERR_INVALID_ARG;
    if (!a || !b || !y) return dw_fail(be, DW_ERR_INVALID_ARG, "%s: null buffer", op);
    // crates/dragonwing-vulkan/src/ops.rs:939-947 (same checks, same strings)
    if (a->len != b->len || a->len != y->len) return dw_fail(be, DW_ERR_SIZE_MISMATCH, "%s: buffer size mismatch", op);
    if (a->len % 2) return dw_fail(be, DW_ERR_INVALID_ARG, "%s: buffer size must be multiple of 2", op);
    cudaSetDevice(be->device);
    return dw::launch_add_f16(be, (const uint16_t *)a->ptr, (const uint16_t *)b->ptr, (uint16_t *)y->ptr, a->len / 2,
                              relu);
}

DW_API dw_status dw_add_f16(dw_backend *be, const dw_buf *a, const dw_buf *b, dw_buf *y) {
    return add_f16_common(be, a, b, y, 0, "add_fp16");
}

DW_API dw_status dw_add_relu_f16(dw_backend *be, const dw_buf *a, const dw_buf *b, dw_buf *y) {
    return add_f16_common(be, a, b, y, 1, "add_relu_fp16");
}

DW_API dw_status dw_relu_f16(dw_backend *be, dw_buf *x) {
    if (!be) return DW_ERR_INVALID_ARG;
    if (!x) return dw_fail(be, DW_ERR_INVALID_ARG, "relu_fp16: null buffer");
    // crates/dragonwing-vulkan/src/ops.rs:857-862
    if (x->len % 2) return dw_fail(be, DW_ERR_INVALID_ARG, "relu_fp16: buffer size must be multiple of 2");
    cudaSetDevice(be->device);
    return dw::launch_relu_f16(be, (const uint16_t *)x->ptr, (uint16_t *)x->ptr, x->len / 2);
}

DW_API dw_status dw_maxpool_f16(dw_backend *be, const dw_buf *x, dw_buf *y, size_t n, size_t h, size_t w, size_t c,
                                size_t k_h, size_t k_w, size_t s_h, size_t s_w, size_t p_t, size_t p_l, size_t p_b,
                                size_t p_r) {
    if (!be) return DW_ERR_INVALID_ARG;
    if (!x || !y) return dw_fail(be, DW_ERR_INVALID_ARG, "maxpool_f16: null buffer");
    if (!n || !h || !w || !c || !k_h || !k_w || !s_h || !s_w || p_t >= k_h || p_b >= k_h || p_l >= k_w || p_r >= k_w ||
        h + p_t + p_b < k_h || w + p_l + p_r < k_w)
        return dw_fail(be, DW_ERR_INVALID_ARG, "maxpool_f16: invalid geometry");
    size_t ho = (h + p_t + p_b - k_h) / s_h + 1, wo = (w + p_l + p_r - k_w) / s_w + 1;
    DW_TRY(check_len(be, x, 2 * n * h * w * c, "maxpool_f16", "input"));
    DW_TRY(check_len(be, y, 2 * n * ho * wo * c, "maxpool_f16", "output"));
    cudaSetDevice(be->device);
    return dw::launch_maxpool_f16(be, (const uint16_t *)x->ptr, (uint16_t *)y->ptr, (int)n, (int)h, (int)w, (int)c,
                                  (int)k_h, (int)k_w, (int)s_h, (int)s_w, (int)p_t, (int)p_l, (int)ho, (int)wo);
}

DW_API dw_status dw_global_avgpool_f16(dw_backend *be, const dw_buf *x, dw_buf *y, size_t n, size_t h, size_t w,
                                       size_t c) {
    if (!be) return DW_ERR_INVALID_ARG;
    if (!x || !y) return dw_fail(be, DW_ERR_INVALID_ARG, "global_avgpool_f16: null buffer");
    if (!n || !h || !w || !c || h * w > 0x7fffffff)
        return dw_fail(be, DW_ERR_INVALID_ARG, "global_avgpool_f16: invalid geometry");
    DW_TRY(check_len(be, x, 2 * n * h * w * c, "global_avgpool_f16", "input"));
    DW_TRY(check_len(be, y, 2 * n * c, "global_avgpool_f16", "output"));
    cudaSetDevice(be->device);
    return dw::launch_gap_f16(be, (const uint16_t *)x->ptr, (uint16_t *)y->ptr, (int)n, (int)h, (int)w, (int)c);
}

DW_API dw_status dw_cast_f32_to_f16(dw_backend *be, const dw_buf *x_f32, dw_buf *y_f16, size_t pixels, size_t c_src,
                                    size_t c_dst) {
    if (!be) return DW_ERR_INVALID_ARG;
    if (!x_f32 || !y_f16) return dw_fail(be, DW_ERR_INVALID_ARG, "cast_f32_to_f16: null buffer");
    if (!c_src || c_dst < c_src || c_dst > 0x7fffffff)
        return dw_fail(be, DW_ERR_INVALID_ARG, "cast_f32_to_f16: need 0 < c_src <= c_dst");
    DW_TRY(check_len(be, x_f32, 4 * pixels * c_src, "cast_f32_to_f16", "input"));
    DW_TRY(check_len(be, y_f16, 2 * pixels * c_dst, "cast_f32_to_f16", "output"));
    cudaSetDevice(be->device);
    return dw::launch_cast_f32_to_f16(be, (const float *)x_f32->ptr, (uint16_t *)y_f16->ptr, pixels, (int)c_src,
                                      (int)c_dst);
}

DW_API dw_status dw_unfold_w_f32_to_f16(dw_backend *be, const dw_buf *x_f32, dw_buf *y_f16, size_t n, size_t h,
                                        size_t w, size_t c, size_t k_w, size_t stride_w, size_t pad_l, size_t w_out,
                                        size_t c_dst) {
    const char *op = "unfold_w_f32_to_f16";
    if (!be) return DW_ERR_INVALID_ARG;
    if (!x_f32 || !y_f16) return dw_fail(be, DW_ERR_INVALID_ARG, "%s: null buffer", op);
    if (!n || !h || !w || !c || !k_w || !stride_w || !w_out || c_dst % 8 || c_dst < k_w * c || c_dst > 4096 ||
        n * h * w > 0x7fffffff || n * h * w_out > 0x7fffffff)
        return dw_fail(be, DW_ERR_INVALID_ARG, "%s: invalid geometry (c_dst must be a multiple of 8 >= k_w*c)", op);
    DW_TRY(check_len(be, x_f32, 4 * n * h * w * c, op, "input"));
    DW_TRY(check_len(be, y_f16, 2 * n * h * w_out * c_dst, op, "output"));
    if (((uintptr_t)y_f16->ptr & 15)) return dw_fail(be, DW_ERR_INVALID_ARG, "%s: output must be 16-byte aligned", op);
    cudaSetDevice(be->device);
    return dw::launch_unfold_w_f32_to_f16(be, (const float *)x_f32->ptr, (uint16_t *)y_f16->ptr, (int)n, (int)h,
                                          (int)w, (int)c, (int)k_w, (int)stride_w, (int)pad_l, (int)w_out,
                                          (int)c_dst);
}

DW_API dw_status dw_cast_f16_to_f32(dw_backend *be, const dw_buf *x_f16, dw_buf *y_f32) {
    if (!be) return DW_ERR_INVALID_ARG;
    if (!x_f16 || !y_f32) return dw_fail(be, DW_ERR_INVALID_ARG, "cast_f16_to_f32: null buffer");
    if (x_f16->len % 2 || y_f32->len != 2 * x_f16->len)
        return dw_fail(be, DW_ERR_SIZE_MISMATCH, "cast_f16_to_f32: length mismatch (%zu f16 bytes vs %zu f32 bytes)",
                       x_f16->len, y_f32->len);
    cudaSetDevice(be->device);
    return dw::launch_cast_f16_to_f32(be, (const uint16_t *)x_f16->ptr, (float *)y_f32->ptr, x_f16->len / 2);
}

}  // extern "C"
