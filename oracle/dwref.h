/*
 * dwref -- CPU oracle for the B200 fused-INT8-convolution backend.
 *
 * TEST INFRASTRUCTURE ONLY.  This library is a plain-C restatement of the
 * scalar (x86_64) code path of the reference's `dragonwing-cpu` crate, plus the
 * build's documented superset of the fused op (int32 bias, per-output-channel
 * requantisation, ReLU6/SiLU epilogues, int8 depthwise).  It is used by the
 * tests, by `__graft_entry__.smoke()` and by the `cpu_baseline` leg of
 * `bench.py` as the checker / timed CPU baseline.  The product path
 * (libdragonwing_cuda.so and the Python package) never links or calls it.
 *
 * Parity pin: the reference (Rust) cannot be compiled in this environment
 * (no cargo/rustc, and the `libm 0.2.16` crate it needs is not vendored), so
 * this restatement is pinned against the known-answer tests copied, as values,
 * from the reference's own unit tests (tests/golden/reference_kats.json).
 *
 * Arithmetic rules that make the restatement exact:
 *   - Rust `f32::round` and libm `roundf` round half away from zero == C roundf;
 *   - `x.clamp(-128.0, 127.0) as i8` == clamp then (int8_t) cast; Rust's
 *     saturating float->int cast maps NaN to 0, which dwref_f32_to_i8 mirrors;
 *   - Rust never contracts a*b+c into an FMA: compile with -ffp-contract=off;
 *     `f32::mul_add` (used by the fp16 paths) is an explicit fmaf.
 */
#ifndef DWREF_H
#define DWREF_H

#include <stddef.h>
#include <stdint.h>

#ifdef __cplusplus
extern "C" {
#endif

enum { DWREF_EPI_NONE = 0, DWREF_EPI_RELU = 1, DWREF_EPI_RELU6 = 2, DWREF_EPI_SILU = 3 };

/* Geometry and epilogue of one fused convolution (same field meaning as the
 * product's dw_conv_desc). pads are [top, left, bottom, right] as in
 * OpParams::Conv2dRequantReluI8Nhwc (crates/dragonwing-onnx/src/builder.rs:345-360). */
typedef struct dwref_conv_desc {
    int32_t n, h, w, c_in, c_out;
    int32_t k_h, k_w, stride_h, stride_w;
    int32_t pad_t, pad_l, pad_b, pad_r;
    int32_t group;      /* 1 = dense; == c_in = depthwise (c_out = c_in * multiplier) */
    int32_t epilogue;   /* DWREF_EPI_* */
    int32_t q6;         /* ReLU6 ceiling in the output's int8 domain */
    float inv_s_out;    /* SiLU only: 1 / s_out */
} dwref_conv_desc;

/* ---- reference scalar ops (crates/dragonwing-cpu/src/ops.rs) ---- */
void dwref_gemm_i8(int32_t *c, const int8_t *a, const int8_t *b, size_t m, size_t n, size_t k);
void dwref_conv2d_i8_nhwc(int32_t *out, const int8_t *in, const int8_t *kernel_hwio,
                          size_t n, size_t h_in, size_t w_in, size_t c_in, size_t c_out,
                          size_t k_h, size_t k_w, size_t stride_h, size_t stride_w,
                          size_t pad_h, size_t pad_w);
void dwref_requantize_i32_to_i8(int8_t *out, const int32_t *in, size_t len, float requant_scale);
void dwref_relu_i8(int8_t *out, const int8_t *in, size_t len);
void dwref_add_i8(int8_t *out, const int8_t *a, const int8_t *b, size_t len,
                  float scale_a_over_y, float scale_b_over_y);
void dwref_quantize_f32_to_i8(int8_t *out, const float *in, size_t len, float scale);
void dwref_dequantize_i8_to_f32(float *out, const int8_t *in, size_t len, float scale);
int8_t dwref_f32_to_i8(float v);
void dwref_quantize_u8_to_i8(int8_t *out, const uint8_t *in, size_t len, float scale);

/* ---- crates/dragonwing-core/src/quantization.rs ---- */
int8_t dwref_quantscale_quantize(float scale, float value);
void dwref_per_channel_scales(float *scales, const float *weights, size_t len, size_t num_channels);
void dwref_per_channel_quantize(int8_t *out, const float *weights, const float *scales,
                                size_t len, size_t num_channels);
float dwref_requant_scale(float s_in, float s_w, float s_out); /* quantize.rs:245 */

/* ---- fused op contract (superset of the reference; see dwref.c) ---- */
int dwref_conv_out_hw(const dwref_conv_desc *d, int32_t *h_out, int32_t *w_out);
int dwref_conv2d_fused_i8(int8_t *y, const int8_t *x, const int8_t *w_hwio,
                          const int32_t *bias_or_null, const float *M, const float *D_or_null,
                          const dwref_conv_desc *d, int threads);
int dwref_conv2d_acc_i32(int32_t *acc, const int8_t *x, const int8_t *w_hwio,
                         const dwref_conv_desc *d, int threads);
int8_t dwref_epilogue_one(int32_t acc, int32_t bias, float m, float dsc, const dwref_conv_desc *d);
void dwref_qgemm_i8(int8_t *y, const int8_t *a, const int8_t *b, const int32_t *bias_or_null,
                    const float *M, size_t m, size_t n, size_t k, int epilogue, int32_t q6,
                    int threads);
float dwref_expf(float x);
float dwref_silu_f32(float x);
void dwref_set_silu_exp_libm(int on);
float dwref_silu_epilogue_f32(float y);

/* ---- glue (int8 data with a shared scale moves unchanged) ---- */
void dwref_maxpool_i8_nhwc(int8_t *y, const int8_t *x, size_t n, size_t h, size_t w, size_t c,
                           size_t k_h, size_t k_w, size_t s_h, size_t s_w,
                           size_t p_t, size_t p_l, size_t p_b, size_t p_r);
void dwref_concat_c_i8(int8_t *y, const int8_t *const *xs, const int32_t *cs, int32_t count,
                       size_t pixels);
void dwref_resize_nearest_i8(int8_t *y, const int8_t *x, size_t n, size_t h_in, size_t w_in,
                             size_t h_out, size_t w_out, size_t c);

/* ---- fp16 path (crates/dragonwing-core/src/dtype.rs, ops.rs fp16 ops) ---- */
uint16_t dwref_f16_from_f32(float v);
float dwref_f16_to_f32(uint16_t h);
void dwref_conv2d_f16_nhwc(uint16_t *y, const uint16_t *x, const uint16_t *w_hwio,
                           const uint16_t *bias_or_null, int relu,
                           size_t n, size_t h_in, size_t w_in, size_t c_in, size_t c_out,
                           size_t k_h, size_t k_w, size_t stride_h, size_t stride_w,
                           size_t pad_h, size_t pad_w, int threads);
void dwref_dwconv_f16_nhwc(uint16_t *y, const uint16_t *x, const uint16_t *w,
                           const uint16_t *bias_or_null, int relu,
                           size_t n, size_t h_in, size_t w_in, size_t c_in, size_t mult,
                           size_t k_h, size_t k_w, size_t stride_h, size_t stride_w,
                           size_t pad_h, size_t pad_w, int threads);
void dwref_gemm_f16(uint16_t *c, const uint16_t *a, const uint16_t *b, size_t m, size_t n, size_t k,
                    int threads);
void dwref_bias_relu_f16(uint16_t *y, const uint16_t *bias_or_null, int relu, size_t rows, size_t c);
void dwref_f16_from_f32_array(uint16_t *y, const float *x, size_t len);
void dwref_f16_to_f32_array(float *y, const uint16_t *x, size_t len);
void dwref_add_f16(uint16_t *y, const uint16_t *a, const uint16_t *b, size_t len);
void dwref_relu_f16(uint16_t *y, const uint16_t *x, size_t len);
void dwref_gap_f16(uint16_t *y, const uint16_t *x, size_t n, size_t h, size_t w, size_t c);
void dwref_maxpool_f16_nhwc(uint16_t *y, const uint16_t *x, size_t n, size_t h, size_t w, size_t c,
                            size_t k_h, size_t k_w, size_t s_h, size_t s_w,
                            size_t p_t, size_t p_l, size_t p_b, size_t p_r);

/* ---- YOLOv8 Detect tail and post-processing (crates/dragonwing-onnx/src/postprocess.rs) ---- */
typedef struct dwref_yolo_desc { /* same fields as dw_yolo_detect_desc */
    int32_t n, num_classes, reg_max, num_levels;
    int32_t h[4], w[4];
    float stride[4], box_scale[4], cls_scale[4];
} dwref_yolo_desc;
typedef struct dwref_detection { /* postprocess.rs:12-19 */
    float bbox[4];
    uint32_t class_id;
    float confidence;
} dwref_detection;
void dwref_sigmoid_f32(float *y, const float *x, size_t len);
void dwref_softmax_f32(float *out, const float *in, size_t len, size_t n);
void dwref_yolo_detect_i8(float *out, const int8_t *const *box, const int8_t *const *cls,
                          const dwref_yolo_desc *d);
float dwref_det_area(const dwref_detection *d);
float dwref_iou(const dwref_detection *a, const dwref_detection *b);
size_t dwref_decode_detections_v8(dwref_detection *out, const float *raw, size_t raw_len, size_t num_classes,
                                  size_t num_detections, uint32_t img_width, uint32_t img_height,
                                  float conf_threshold, int alt);
size_t dwref_nms(dwref_detection *d, size_t n, float iou_threshold, int agnostic);
size_t dwref_postprocess_yolo(dwref_detection *out, const float *raw, size_t raw_len, size_t num_classes,
                              size_t num_detections, uint32_t img_width, uint32_t img_height,
                              float conf_threshold, float iou_threshold, int flags);

int dwref_num_cpus(void);

#ifdef __cplusplus
}
#endif
#endif /* DWREF_H */
