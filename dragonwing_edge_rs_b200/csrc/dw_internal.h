// dw_internal.h -- private types shared by the translation units of
// libdragonwing_cuda.so (backend state, buffers, error plumbing, launchers).
#pragma once

#include <cuda.h>
#include <cuda_runtime.h>

#include <cstdarg>
#include <cstdint>
#include <cstdio>
#include <string>

#include "dw_cuda.h"

// Device-side error record written by kernels whose bounded waits expire
// (never by trapping).  word[0] = error code (0 = none), word[1] = site,
// word[2] = block, word[3] = detail.
enum dw_dev_err : int32_t {
    DW_DEV_OK = 0,
    DW_DEV_WAIT_EXPIRED = 1,
    DW_DEV_BAD_ARG = 2,
};
constexpr int kDevErrWords = 4;

struct dw_buf {
    void *ptr = nullptr;
    size_t len = 0;
    bool owned = false;
};

using PFN_encodeTiled = CUresult (*)(CUtensorMap *, CUtensorMapDataType, cuuint32_t, void *, const cuuint64_t *,
                                     const cuuint64_t *, const cuuint32_t *, const cuuint32_t *,
                                     CUtensorMapInterleave, CUtensorMapSwizzle, CUtensorMapL2promotion,
                                     CUtensorMapFloatOOBfill);

struct dw_backend {
    int device = 0;
    cudaStream_t stream = nullptr;
    dw_config cfg{};
    std::string last_error;
    int32_t *dev_err = nullptr;       // kDevErrWords ints in device memory
    int sm_count = 0;
    uint64_t wait_cap_ns = 0;         // device wait limit, nanoseconds (globaltimer)
    uint64_t launches = 0;
    uint64_t capture_mark = 0;        // launch count when the current capture began
    PFN_encodeTiled encode_tiled = nullptr;
    void *scratch = nullptr;          // per-backend device scratch (tile counters etc.)
    size_t scratch_len = 0;
};

// Records an error message on the backend and returns `st`.
dw_status dw_fail(dw_backend *be, dw_status st, const char *fmt, ...) __attribute__((format(printf, 3, 4)));
// Maps a CUDA error to DW_ERR_DEVICE with context; DW_OK if e == cudaSuccess.
dw_status dw_cuda_check(dw_backend *be, cudaError_t e, const char *what);
// Checks the launch that was just made, counts it, traces it when enabled.
dw_status dw_after_launch(dw_backend *be, const char *what);
// Grows (never shrinks) the backend scratch to at least `len` bytes.
dw_status dw_scratch(dw_backend *be, size_t len, void **out);
// Validates a conv descriptor (positive dims, non-negative pads, the kernel
// within the padded input, supported group and epilogue); computes the output dims.
dw_status dw_check_conv_desc(dw_backend *be, const dw_conv_desc *d, int *ho, int *wo, const char *op);

// ---- launchers implemented in the kernel translation units ----
namespace dw {

struct EpiParams {
    const int32_t *bias;  // may be null
    const float *M;       // per-channel requant scale (NONE/RELU/RELU6)
    const float *D;       // per-channel dequant scale (SILU)
    int32_t epilogue;
    int32_t q6;
    float inv_s_out;
};

// elementwise.cu
dw_status launch_requantize(dw_backend *be, const int32_t *in, int8_t *out, size_t n, float scale);
dw_status launch_relu_i8(dw_backend *be, const int8_t *in, int8_t *out, size_t n);
dw_status launch_add_i8(dw_backend *be, const int8_t *a, const int8_t *b, int8_t *out, size_t n, float ra,
                        float rb);
dw_status launch_quantize_f32(dw_backend *be, const float *in, int8_t *out, size_t n, float scale);
dw_status launch_quantize_u8(dw_backend *be, const uint8_t *in, int8_t *out, size_t n, float scale);
dw_status launch_dequantize(dw_backend *be, const int8_t *in, float *out, size_t n, float scale);
dw_status launch_maxpool_i8(dw_backend *be, const int8_t *x, int8_t *y, int n, int h, int w, int c, int kh,
                            int kw, int sh, int sw, int pt, int pl, int ho, int wo);
dw_status launch_concat_i8(dw_backend *be, const int8_t *const *xs, const int32_t *cs, int count,
                           size_t pixels, int8_t *y);
dw_status launch_slice_c_i8(dw_backend *be, const int8_t *x, int8_t *y, size_t pixels, int c_total, int c0,
                            int c_len);
dw_status launch_resize_nearest_i8(dw_backend *be, const int8_t *x, int8_t *y, int n, int hi, int wi, int ho,
                                   int wo, int c);
dw_status launch_repack_hwio_to_ohwi(dw_backend *be, const int8_t *w, int8_t *out, int taps, int c_in,
                                     int c_out);
// The repack plus m[0..c_out) = v, in one launch.
dw_status launch_repack_hwio_to_ohwi_fill(dw_backend *be, const int8_t *w, int8_t *out, int taps, int c_in, int c_out,
                                          float *m, float v);
dw_status launch_transpose_kn_to_nk(dw_backend *be, const int8_t *b, int8_t *out, int k, int n);
dw_status launch_expire_wait(dw_backend *be, uint64_t cap_ns);

// conv_direct.cu
dw_status launch_conv_direct_i8(dw_backend *be, const dw_conv_desc &d, int ho, int wo, const int8_t *x,
                                const int8_t *w_ohwi, const EpiParams &ep, int8_t *y, int32_t *acc_out);
dw_status launch_dwconv_i8(dw_backend *be, const dw_conv_desc &d, int ho, int wo, const int8_t *x,
                           const int8_t *w_hwcm, const EpiParams &ep, int8_t *y, int32_t *acc_out);

// umma_conv.cu (tcgen05 implicit GEMM)
bool umma_supported(const dw_backend *be, const dw_conv_desc &d, int ho, int wo);
bool umma_supported_f16(const dw_backend *be, const dw_conv_desc &d, int ho, int wo);
// x / y: channel ranges of wider tensors (pitch = elements from one pixel to the next).
dw_status launch_umma_conv_i8_view(dw_backend *be, const dw_conv_desc &d, int ho, int wo, const int8_t *x, int x_pitch,
                                   const int8_t *w_ohwi, const EpiParams &ep, int8_t *y, int y_pitch);
// y = add_i8(res, conv(x)) with ratios ra (res) and rb (conv), fused in the epilogue.
dw_status launch_umma_conv_add_i8_view(dw_backend *be, const dw_conv_desc &d, int ho, int wo, const int8_t *x,
                                       int x_pitch, const int8_t *w_ohwi, const EpiParams &ep, const int8_t *res,
                                       int res_pitch, float ra, float rb, int8_t *y, int y_pitch);
dw_status launch_add_i8_view(dw_backend *be, const int8_t *a, int a_pitch, const int8_t *b, int b_pitch, int8_t *out,
                             int out_pitch, size_t pixels, int c, float ra, float rb);
dw_status launch_maxpool_i8_view(dw_backend *be, const int8_t *x, int x_pitch, int8_t *y, int y_pitch, int n, int h,
                                 int w, int c, int kh, int kw, int sh, int sw, int pt, int pl, int ho, int wo);
dw_status launch_maxpool_chain_i8_view(dw_backend *be, const int8_t *x, int x_pitch, int8_t *const *ys,
                                       const int *y_pitches, int count, int n, int h, int w, int c, int k);
dw_status launch_umma_conv_i8(dw_backend *be, const dw_conv_desc &d, int ho, int wo, const int8_t *x,
                              const int8_t *w_ohwi, const EpiParams &ep, int8_t *y);
dw_status launch_umma_conv_f16(dw_backend *be, const dw_conv_desc &d, int ho, int wo, const uint16_t *x,
                               const uint16_t *w_ohwi, const uint16_t *bias, int relu, uint16_t *y,
                               const uint16_t *residual);

dw_status launch_im2col_u8_i8(dw_backend *be, const uint8_t *x, int8_t *y, int n, int h, int w, int c, int kh, int kw,
                              int sh, int sw, int pt, int pl, int ho, int wo, int c_dst, float scale);
dw_status launch_stem3_conv_u8_i8(dw_backend *be, const uint8_t *x, const int8_t *w_hwio, const EpiParams &ep,
                                 int8_t *y, int n, int h, int w, int sh, int sw, int pt, int pl, int ho, int wo, int c_out,
                                 float scale);

// dwconv_tma.cu (TMA-fed int8 depthwise 3x3 stride 1; DW_ERR_UNSUPPORTED when the shape does not fit)
dw_status launch_dwconv3x3_stream_i8(dw_backend *be, const dw_conv_desc &d, int ho, int wo, const int8_t *x,
                                     const int8_t *w_hwcm, const EpiParams &ep, int8_t *y, int shape);
dw_status launch_dwconv3x3_tma_i8(dw_backend *be, const dw_conv_desc &d, int ho, int wo, const int8_t *x,
                                  const int8_t *w_hwcm, const EpiParams &ep, int8_t *y);

// fp16.cu (CUDA-core fp16 kernels)
dw_status launch_conv_direct_f16(dw_backend *be, const dw_conv_desc &d, int ho, int wo, const uint16_t *x,
                                 const uint16_t *w_ohwi, const uint16_t *bias, int relu, uint16_t *y);
dw_status launch_dwconv_f16(dw_backend *be, const dw_conv_desc &d, int ho, int wo, const uint16_t *x,
                            const uint16_t *w_hwcm, const uint16_t *bias, int relu, uint16_t *y);
dw_status launch_add_f16(dw_backend *be, const uint16_t *a, const uint16_t *b, uint16_t *y, size_t n, int relu);
dw_status launch_relu_f16(dw_backend *be, const uint16_t *x, uint16_t *y, size_t n);
dw_status launch_maxpool_f16(dw_backend *be, const uint16_t *x, uint16_t *y, int n, int h, int w, int c, int kh,
                             int kw, int sh, int sw, int pt, int pl, int ho, int wo);
dw_status launch_gap_f16(dw_backend *be, const uint16_t *x, uint16_t *y, int n, int h, int w, int c);
dw_status launch_repack_hwio_to_ohwi_f16(dw_backend *be, const uint16_t *w, uint16_t *out, int taps, int c_in,
                                         int c_out);
dw_status launch_transpose_kn_to_nk_f16(dw_backend *be, const uint16_t *b, uint16_t *out, int k, int n);
dw_status launch_cast_f32_to_f16(dw_backend *be, const float *x, uint16_t *y, size_t pixels, int c_src, int c_dst);
dw_status launch_cast_f16_to_f32(dw_backend *be, const uint16_t *x, float *y, size_t n);
dw_status launch_unfold_w_f32_to_f16(dw_backend *be, const float *x, uint16_t *y, int n, int h, int w, int c, int kw,
                                    int sw, int pl, int wo, int c_dst);

}  // namespace dw
