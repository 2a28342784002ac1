/*
 * dwref.c -- CPU oracle (TEST INFRASTRUCTURE ONLY; never linked by the product).
 *
 * Plain-C restatement of the scalar code path of the reference's
 * `dragonwing-cpu` crate (the path x86_64 hosts compile: ops.rs:3373-3376),
 * of the quantisation primitives in `dragonwing-core`, and of the build's
 * superset contract for the fused op.  Every function names the reference
 * file:line it follows (paths relative to the reference repository root).
 *
 * Compile with -ffp-contract=off (Rust never contracts a*b+c into an FMA).
 */
#include "dwref.h"

#include <math.h>
#include <pthread.h>
#include <stdlib.h>
#include <string.h>
#include <unistd.h>

#include "dw_expf.h" /* the contract's shared exp (include/) */

/* ------------------------------------------------------------------------ */
/* Row-partitioned host threads: restates parallel_for_scoped                 */
/* (crates/dragonwing-cpu/src/pool.rs:317-350): ceil(total/threads) chunks.   */
/* ------------------------------------------------------------------------ */
typedef void (*range_fn)(void *ctx, size_t start, size_t end);
typedef struct { range_fn f; void *ctx; size_t start, end; } range_job;

static void *range_thread(void *p) {
    range_job *j = (range_job *)p;
    j->f(j->ctx, j->start, j->end);
    return NULL;
}

static void parallel_for(int threads, size_t total, range_fn f, void *ctx) {
    if (total == 0) return;
    size_t nt = threads < 1 ? 1 : (size_t)threads;
    if (nt > total) nt = total;
    if (nt <= 1) { f(ctx, 0, total); return; }
    size_t chunk = (total + nt - 1) / nt;
    pthread_t *tid = (pthread_t *)calloc(nt, sizeof(pthread_t));
    range_job *jobs = (range_job *)calloc(nt, sizeof(range_job));
    size_t launched = 0;
    for (size_t i = 0; i < nt; i++) {
        size_t s = i * chunk, e = (i + 1) * chunk;
        if (s >= total) break;
        if (e > total) e = total;
        jobs[i].f = f; jobs[i].ctx = ctx; jobs[i].start = s; jobs[i].end = e;
        if (pthread_create(&tid[i], NULL, range_thread, &jobs[i]) != 0) {
            f(ctx, s, e); /* could not spawn: run inline */
            jobs[i].f = NULL;
        }
        launched = i + 1;
    }
    for (size_t i = 0; i < launched; i++)
        if (jobs[i].f) pthread_join(tid[i], NULL);
    free(tid);
    free(jobs);
}

/* crates/dragonwing-cpu/src/pool.rs:222 num_cpus() */
int dwref_num_cpus(void) {
    long n = sysconf(_SC_NPROCESSORS_ONLN);
    return n > 0 ? (int)n : 1;
}

/* `v.clamp(-128.0, 127.0).round() as i8` (ops.rs:3383-3385, 3207-3208, 3522-3524).
 * Rust's float->int cast saturates and maps NaN to 0. */
int8_t dwref_f32_to_i8(float v) {
    if (v != v) return 0;
    float c = v < -128.0f ? -128.0f : (v > 127.0f ? 127.0f : v);
    return (int8_t)roundf(c);
}

/* ------------------------------------------------------------------------ */
/* Reference scalar int8 ops                                                  */
/* ------------------------------------------------------------------------ */

/* ops.rs:2981-2995 gemm_i8_scalar: C[m,n] = sum_p A[m,p] * B[p,n] (i32). */
void dwref_gemm_i8(int32_t *c, const int8_t *a, const int8_t *b, size_t m, size_t n, size_t k) {
    for (size_t i = 0; i < m; i++)
        for (size_t j = 0; j < n; j++) {
            int32_t acc = 0;
            for (size_t p = 0; p < k; p++) acc += (int32_t)a[i * k + p] * (int32_t)b[p * n + j];
            c[i * n + j] = acc;
        }
}

/* ops.rs:3086-3142 conv2d_i8_nhwc: NHWC input, HWIO kernel, symmetric pads,
 * out-of-bounds taps skipped (:3115-3120), i32 MAC (:3131). */
void dwref_conv2d_i8_nhwc(int32_t *out, const int8_t *in, const int8_t *kernel,
                          size_t n, size_t h_in, size_t w_in, size_t c_in, size_t c_out,
                          size_t k_h, size_t k_w, size_t stride_h, size_t stride_w,
                          size_t pad_h, size_t pad_w) {
    size_t h_out = (h_in + 2 * pad_h - k_h) / stride_h + 1;
    size_t w_out = (w_in + 2 * pad_w - k_w) / stride_w + 1;
    for (size_t b = 0; b < n; b++)
        for (size_t oh = 0; oh < h_out; oh++)
            for (size_t ow = 0; ow < w_out; ow++)
                for (size_t oc = 0; oc < c_out; oc++) {
                    int32_t acc = 0;
                    for (size_t kh = 0; kh < k_h; kh++)
                        for (size_t kw = 0; kw < k_w; kw++) {
                            long ih = (long)(oh * stride_h + kh) - (long)pad_h;
                            long iw = (long)(ow * stride_w + kw) - (long)pad_w;
                            if (ih < 0 || ih >= (long)h_in || iw < 0 || iw >= (long)w_in) continue;
                            for (size_t ic = 0; ic < c_in; ic++) {
                                size_t ii = ((b * h_in + (size_t)ih) * w_in + (size_t)iw) * c_in + ic;
                                size_t ki = ((kh * k_w + kw) * c_in + ic) * c_out + oc;
                                acc += (int32_t)in[ii] * (int32_t)kernel[ki];
                            }
                        }
                    out[((b * h_out + oh) * w_out + ow) * c_out + oc] = acc;
                }
}

/* ops.rs:3380-3386 requantize_i32_to_i8_scalar: (i8) round(clamp((f32)acc * s)). */
void dwref_requantize_i32_to_i8(int8_t *out, const int32_t *in, size_t len, float requant_scale) {
    for (size_t i = 0; i < len; i++) {
        float scaled = (float)in[i] * requant_scale;
        out[i] = dwref_f32_to_i8(scaled);
    }
}

/* ops.rs:3315-3319 relu_i8_scalar. */
void dwref_relu_i8(int8_t *out, const int8_t *in, size_t len) {
    for (size_t i = 0; i < len; i++) out[i] = in[i] > 0 ? in[i] : 0;
}

/* ops.rs:3197-3209 add_i8_scalar: two RN multiplies and one RN add, then clamp/round. */
void dwref_add_i8(int8_t *out, const int8_t *a, const int8_t *b, size_t len,
                  float scale_a_over_y, float scale_b_over_y) {
    for (size_t i = 0; i < len; i++) {
        float pa = (float)a[i] * scale_a_over_y;
        float pb = (float)b[i] * scale_b_over_y;
        out[i] = dwref_f32_to_i8(pa + pb);
    }
}

/* ops.rs:3503-3525 quantize_f32_to_i8 (+_scalar): inv_scale = 1.0/scale, then
 * round(clamp(x * inv_scale)). */
void dwref_quantize_f32_to_i8(int8_t *out, const float *in, size_t len, float scale) {
    float inv_scale = 1.0f / scale;
    for (size_t i = 0; i < len; i++) out[i] = dwref_f32_to_i8(in[i] * inv_scale);
}

/* ops.rs:3453-3457 dequantize_i8_to_f32_scalar: (f32)x * scale. */
void dwref_dequantize_i8_to_f32(float *out, const int8_t *in, size_t len, float scale) {
    for (size_t i = 0; i < len; i++) out[i] = (float)in[i] * scale;
}

/* ------------------------------------------------------------------------ */
/* crates/dragonwing-core/src/quantization.rs                                 */
/* ------------------------------------------------------------------------ */

/* quantization.rs:94-99 QuantScale::quantize: roundf(clamp(value / scale)). */
int8_t dwref_quantscale_quantize(float scale, float value) {
    return dwref_f32_to_i8(value / scale);
}

/* quantization.rs:154-171 PerChannelScale::from_weights ([C_out, ...] layout). */
void dwref_per_channel_scales(float *scales, const float *weights, size_t len, size_t num_channels) {
    size_t per = len / num_channels;
    for (size_t c = 0; c < num_channels; c++) {
        float abs_max = 0.0f;
        for (size_t i = 0; i < per; i++) {
            float a = fabsf(weights[c * per + i]);
            abs_max = fmaxf(abs_max, a); /* f32::max ignores NaN like fmaxf */
        }
        scales[c] = abs_max > 0.0f ? abs_max / 127.0f : 1.0f;
    }
}

/* quantization.rs:178-195 PerChannelScale::quantize_weights. */
void dwref_per_channel_quantize(int8_t *out, const float *weights, const float *scales,
                                size_t len, size_t num_channels) {
    size_t per = len / num_channels;
    for (size_t c = 0; c < num_channels; c++)
        for (size_t i = 0; i < per; i++) out[c * per + i] = dwref_f32_to_i8(weights[c * per + i] / scales[c]);
}

/* crates/dragonwing-onnx/src/quantize.rs:245: (input_scale * weight_scale) / output_scale. */
float dwref_requant_scale(float s_in, float s_w, float s_out) {
    return (s_in * s_w) / s_out;
}

/* ------------------------------------------------------------------------ */
/* Fused op contract                                                          */
/*                                                                            */
/*  acc = conv (ops.rs:3086-3142, general pads; depthwise index math          */
/*        ops.rs:2669-2730 when group == c_in)                                */
/*  acc += bias[oc]                       (two's-complement wrapping add)     */
/*  NONE/RELU/RELU6: q = requantize(acc, M[oc]) (ops.rs:3380-3386)            */
/*        RELU  -> relu_i8 (ops.rs:3315-3319); RELU6 -> min(relu(q), q6)      */
/*  SILU: y = (f32)acc * D[oc]; z = y * (1/(1+exp(-y))) (ops.rs:1865-1870);   */
/*        q = quantize(z, 1/s_out) (ops.rs:3503-3525)                         */
/* With a constant M, no bias and epilogue NONE/RELU this is exactly the      */
/* reference composition conv2d_i8_nhwc -> requantize_i32_to_i8 -> relu_i8    */
/* (crates/dragonwing-test/src/int8_e2e.rs:447-466).                          */
/* ------------------------------------------------------------------------ */

float dwref_expf(float x) { return dw_expf(x); }
float dwref_silu_f32(float x) { return dw_silu_f32(x); }

/* Measurement switch: 1 computes the SiLU epilogue with the host libm's expf,
 * the function behind the reference's f32::exp in sigmoid_f32_scalar
 * (crates/dragonwing-cpu/src/ops.rs:1865-1870), instead of the contract's
 * shared exp; used to count the int8 results the choice changes. */
static volatile int g_silu_libm = 0;
void dwref_set_silu_exp_libm(int on) { g_silu_libm = on ? 1 : 0; }

static float silu_epilogue(float y) {
    if (!g_silu_libm) return dw_silu_f32(y);
    const float e = expf(-y);
    const float sig = 1.0f / (1.0f + e);
    return y * sig;
}
float dwref_silu_epilogue_f32(float y) { return silu_epilogue(y); }

int dwref_conv_out_hw(const dwref_conv_desc *d, int32_t *h_out, int32_t *w_out) {
    if (d->n < 0 || d->h <= 0 || d->w <= 0 || d->c_in <= 0 || d->c_out <= 0 || d->k_h <= 0 ||
        d->k_w <= 0 || d->stride_h <= 0 || d->stride_w <= 0 || d->pad_t < 0 || d->pad_l < 0 ||
        d->pad_b < 0 || d->pad_r < 0)
        return -1;
    int32_t hp = d->h + d->pad_t + d->pad_b - d->k_h;
    int32_t wp = d->w + d->pad_l + d->pad_r - d->k_w;
    if (hp < 0 || wp < 0) return -1;
    *h_out = hp / d->stride_h + 1;
    *w_out = wp / d->stride_w + 1;
    return 0;
}

int8_t dwref_epilogue_one(int32_t acc, int32_t bias, float m, float dsc, const dwref_conv_desc *d) {
    int32_t a = (int32_t)((uint32_t)acc + (uint32_t)bias);
    if (d->epilogue == DWREF_EPI_SILU) {
        float y = (float)a * dsc;
        float z = silu_epilogue(y);
        return dwref_f32_to_i8(z * d->inv_s_out);
    }
    int8_t q = dwref_f32_to_i8((float)a * m);
    if (d->epilogue == DWREF_EPI_RELU) return q > 0 ? q : 0;
    if (d->epilogue == DWREF_EPI_RELU6) {
        int8_t r = q > 0 ? q : 0;
        return r < d->q6 ? r : (int8_t)d->q6;
    }
    return q;
}

typedef struct {
    const dwref_conv_desc *d;
    int32_t h_out, w_out;
    const int8_t *x, *w;
    int32_t *acc;            /* when non-NULL: write raw accumulators */
    int8_t *y;               /* else: fused epilogue output */
    const int32_t *bias;
    const float *M, *D;
} conv_ctx;

static void conv_rows(void *p, size_t start, size_t end) {
    conv_ctx *c = (conv_ctx *)p;
    const dwref_conv_desc *d = c->d;
    const size_t H = (size_t)d->h, W = (size_t)d->w, CI = (size_t)d->c_in, CO = (size_t)d->c_out;
    const int dw = d->group != 1;
    const size_t mult = dw ? CO / CI : 0;
    for (size_t row = start; row < end; row++) {
        size_t b = row / (size_t)c->h_out, oh = row % (size_t)c->h_out;
        for (size_t ow = 0; ow < (size_t)c->w_out; ow++)
            for (size_t oc = 0; oc < CO; oc++) {
                int32_t acc = 0;
                for (int32_t kh = 0; kh < d->k_h; kh++)
                    for (int32_t kw = 0; kw < d->k_w; kw++) {
                        long ih = (long)(oh * (size_t)d->stride_h) + kh - d->pad_t;
                        long iw = (long)(ow * (size_t)d->stride_w) + kw - d->pad_l;
                        if (ih < 0 || ih >= (long)H || iw < 0 || iw >= (long)W) continue;
                        const int8_t *px = c->x + ((b * H + (size_t)ih) * W + (size_t)iw) * CI;
                        if (!dw) {
                            const int8_t *pk = c->w + ((size_t)(kh * d->k_w + kw) * CI) * CO + oc;
                            for (size_t ic = 0; ic < CI; ic++) acc += (int32_t)px[ic] * (int32_t)pk[ic * CO];
                        } else {
                            size_t ic = oc / mult, m = oc % mult;
                            size_t ki = ((size_t)(kh * d->k_w + kw) * CI + ic) * mult + m; /* ops.rs:2716 */
                            acc += (int32_t)px[ic] * (int32_t)c->w[ki];
                        }
                    }
                size_t oi = ((b * (size_t)c->h_out + oh) * (size_t)c->w_out + ow) * CO + oc;
                if (c->acc) {
                    c->acc[oi] = acc;
                } else {
                    int32_t bias = c->bias ? c->bias[oc] : 0;
                    float dsc = c->D ? c->D[oc] : 0.0f;
                    c->y[oi] = dwref_epilogue_one(acc, bias, c->M ? c->M[oc] : 0.0f, dsc, d);
                }
            }
    }
}

static int check_group(const dwref_conv_desc *d) {
    if (d->group == 1) return 0;
    if (d->group == d->c_in && d->c_out % d->c_in == 0) return 0;
    return -1;
}

int dwref_conv2d_acc_i32(int32_t *acc, const int8_t *x, const int8_t *w_hwio,
                         const dwref_conv_desc *d, int threads) {
    conv_ctx c;
    memset(&c, 0, sizeof c);
    if (dwref_conv_out_hw(d, &c.h_out, &c.w_out) != 0 || check_group(d) != 0) return -1;
    c.d = d; c.x = x; c.w = w_hwio; c.acc = acc;
    parallel_for(threads, (size_t)d->n * (size_t)c.h_out, conv_rows, &c);
    return 0;
}

int dwref_conv2d_fused_i8(int8_t *y, const int8_t *x, const int8_t *w_hwio,
                          const int32_t *bias_or_null, const float *M, const float *D_or_null,
                          const dwref_conv_desc *d, int threads) {
    conv_ctx c;
    memset(&c, 0, sizeof c);
    if (dwref_conv_out_hw(d, &c.h_out, &c.w_out) != 0 || check_group(d) != 0) return -1;
    if (d->epilogue == DWREF_EPI_SILU && !D_or_null) return -1;
    if (d->epilogue != DWREF_EPI_SILU && !M) return -1;
    c.d = d; c.x = x; c.w = w_hwio; c.y = y; c.bias = bias_or_null; c.M = M; c.D = D_or_null;
    parallel_for(threads, (size_t)d->n * (size_t)c.h_out, conv_rows, &c);
    return 0;
}

/* QGemm: gemm_i8_scalar (ops.rs:2981-2995) followed by the per-column
 * epilogue (bias[n], M[n]) of the contract. */
typedef struct {
    int8_t *y; const int8_t *a, *b; const int32_t *bias; const float *M;
    size_t m, n, k; dwref_conv_desc d;
} qgemm_ctx;

static void qgemm_rows(void *p, size_t start, size_t end) {
    qgemm_ctx *c = (qgemm_ctx *)p;
    int32_t *row = (int32_t *)malloc(c->n * sizeof(int32_t));
    for (size_t i = start; i < end; i++) {
        for (size_t j = 0; j < c->n; j++) row[j] = 0;
        for (size_t p2 = 0; p2 < c->k; p2++) {
            int32_t av = c->a[i * c->k + p2];
            const int8_t *br = c->b + p2 * c->n;
            for (size_t j = 0; j < c->n; j++) row[j] += av * (int32_t)br[j];
        }
        for (size_t j = 0; j < c->n; j++)
            c->y[i * c->n + j] = dwref_epilogue_one(row[j], c->bias ? c->bias[j] : 0, c->M[j], 0.0f, &c->d);
    }
    free(row);
}

void dwref_qgemm_i8(int8_t *y, const int8_t *a, const int8_t *b, const int32_t *bias_or_null,
                    const float *M, size_t m, size_t n, size_t k, int epilogue, int32_t q6,
                    int threads) {
    qgemm_ctx c;
    memset(&c, 0, sizeof c);
    c.y = y; c.a = a; c.b = b; c.bias = bias_or_null; c.M = M; c.m = m; c.n = n; c.k = k;
    c.d.epilogue = epilogue; c.d.q6 = q6;
    parallel_for(threads, m, qgemm_rows, &c);
}

/* ------------------------------------------------------------------------ */
/* Glue                                                                       */
/* ------------------------------------------------------------------------ */

/* maxpool2d_f32_nhwc (ops.rs:1513-1551) on int8 data.  The reference ignores
 * pads (runtime.rs:1505-1544) although the builder sizes the output with
 * them (builder.rs:845-850); the contract pads with -inf, i.e. the max runs
 * over in-bounds taps only. */
void dwref_maxpool_i8_nhwc(int8_t *y, const int8_t *x, size_t n, size_t h, size_t w, size_t c,
                           size_t k_h, size_t k_w, size_t s_h, size_t s_w,
                           size_t p_t, size_t p_l, size_t p_b, size_t p_r) {
    size_t h_out = (h + p_t + p_b - k_h) / s_h + 1, w_out = (w + p_l + p_r - k_w) / s_w + 1;
    for (size_t b = 0; b < n; b++)
        for (size_t oh = 0; oh < h_out; oh++)
            for (size_t ow = 0; ow < w_out; ow++)
                for (size_t ch = 0; ch < c; ch++) {
                    int m = -128;
                    for (size_t ph = 0; ph < k_h; ph++)
                        for (size_t pw = 0; pw < k_w; pw++) {
                            long ih = (long)(oh * s_h + ph) - (long)p_t;
                            long iw = (long)(ow * s_w + pw) - (long)p_l;
                            if (ih < 0 || ih >= (long)h || iw < 0 || iw >= (long)w) continue;
                            int v = x[((b * h + (size_t)ih) * w + (size_t)iw) * c + ch];
                            if (v > m) m = v;
                        }
                    y[((b * h_out + oh) * w_out + ow) * c + ch] = (int8_t)m;
                }
}

/* concat_f32 axis 3 (ops.rs:2178-2194): per pixel, input channel vectors in order. */
void dwref_concat_c_i8(int8_t *y, const int8_t *const *xs, const int32_t *cs, int32_t count,
                       size_t pixels) {
    size_t ct = 0;
    for (int32_t i = 0; i < count; i++) ct += (size_t)cs[i];
    for (size_t p = 0; p < pixels; p++) {
        size_t off = p * ct;
        for (int32_t i = 0; i < count; i++) {
            memcpy(y + off, xs[i] + p * (size_t)cs[i], (size_t)cs[i]);
            off += (size_t)cs[i];
        }
    }
}

/* resize_f32 Nearest (ops.rs:2320-2348):
 * ih = clamp(round((oh + 0.5) * (h_in/h_out) - 0.5), 0, h_in - 1), in f32. */
void dwref_resize_nearest_i8(int8_t *y, const int8_t *x, size_t n, size_t h_in, size_t w_in,
                             size_t h_out, size_t w_out, size_t c) {
    float sh = (float)h_in / (float)h_out, sw = (float)w_in / (float)w_out;
    for (size_t b = 0; b < n; b++)
        for (size_t oh = 0; oh < h_out; oh++) {
            float fh = roundf(((float)oh + 0.5f) * sh - 0.5f);
            fh = fminf(fmaxf(fh, 0.0f), (float)(h_in - 1));
            size_t ih = (size_t)fh;
            for (size_t ow = 0; ow < w_out; ow++) {
                float fw = roundf(((float)ow + 0.5f) * sw - 0.5f);
                fw = fminf(fmaxf(fw, 0.0f), (float)(w_in - 1));
                size_t iw = (size_t)fw;
                memcpy(y + ((b * h_out + oh) * w_out + ow) * c, x + ((b * h_in + ih) * w_in + iw) * c, c);
            }
        }
}

/* ------------------------------------------------------------------------ */
/* FP16                                                                       */
/* ------------------------------------------------------------------------ */

/* dtype.rs:164-222 F16::from_f32_soft (round to nearest even). */
uint16_t dwref_f16_from_f32(float v) {
    uint32_t bits;
    memcpy(&bits, &v, 4);
    uint32_t sign = (bits >> 16) & 0x8000u;
    int32_t exp = (int32_t)((bits >> 23) & 0xFFu);
    uint32_t mant = bits & 0x007FFFFFu;
    if (exp == 255) {
        if (mant == 0) return (uint16_t)(sign | 0x7C00u);
        uint32_t m = mant >> 13;
        if (m > 0x1FFu) m = 0x1FFu;
        return (uint16_t)(sign | 0x7E00u | m);
    }
    int32_t new_exp = exp - 127 + 15;
    if (new_exp >= 31) return (uint16_t)(sign | 0x7C00u);
    if (new_exp <= 0) {
        if (new_exp < -10) return (uint16_t)sign;
        uint32_t shift = (uint32_t)(1 - new_exp);
        uint32_t mh = mant | 0x00800000u;
        uint32_t shifted = mh >> (13 + shift);
        uint32_t round_bit = (mh >> (12 + shift)) & 1u;
        uint32_t sticky = (mh & ((1u << (12 + shift)) - 1u)) != 0 ? 1u : 0u;
        uint32_t rounded = shifted + (round_bit & (sticky | (shifted & 1u)));
        return (uint16_t)(sign | rounded);
    }
    uint32_t m16 = mant >> 13;
    uint32_t round_bit = (mant >> 12) & 1u;
    uint32_t sticky = (mant & 0x0FFFu) != 0 ? 1u : 0u;
    uint32_t rounded = m16 + (round_bit & (sticky | (m16 & 1u)));
    if (rounded >= 0x400u) {
        int32_t e2 = new_exp + 1;
        if (e2 >= 31) return (uint16_t)(sign | 0x7C00u);
        return (uint16_t)(sign | ((uint32_t)e2 << 10));
    }
    return (uint16_t)(sign | ((uint32_t)new_exp << 10) | rounded);
}

/* dtype.rs:225-263 F16::to_f32_soft (exact). */
float dwref_f16_to_f32(uint16_t h) {
    uint32_t bits = h;
    uint32_t sign = (bits & 0x8000u) << 16;
    uint32_t exp = (bits >> 10) & 0x1Fu;
    uint32_t mant = bits & 0x03FFu;
    uint32_t out;
    if (exp == 0) {
        if (mant == 0) {
            out = sign;
        } else {
            uint32_t m = mant;
            int32_t e = 0;
            while ((m & 0x0400u) == 0) { m <<= 1; e++; }
            out = sign | ((uint32_t)(127 - 15 - e) << 23) | ((m & 0x03FFu) << 13);
        }
    } else if (exp == 31) {
        out = mant == 0 ? (sign | 0x7F800000u) : (sign | 0x7FC00000u | (mant << 13));
    } else {
        out = sign | ((exp + 127 - 15) << 23) | (mant << 13);
    }
    float f;
    memcpy(&f, &out, 4);
    return f;
}

typedef struct {
    uint16_t *y; const uint16_t *x, *w, *bias; int relu, dw;
    size_t n, h_in, w_in, c_in, c_out, mult, k_h, k_w, s_h, s_w, p_h, p_w, h_out, w_out;
} f16conv_ctx;

static void f16conv_rows(void *p, size_t start, size_t end) {
    f16conv_ctx *c = (f16conv_ctx *)p;
    for (size_t row = start; row < end; row++) {
        size_t b = row / c->h_out, oh = row % c->h_out;
        for (size_t ow = 0; ow < c->w_out; ow++)
            for (size_t oc = 0; oc < c->c_out; oc++) {
                float acc = 0.0f;
                for (size_t kh = 0; kh < c->k_h; kh++)
                    for (size_t kw = 0; kw < c->k_w; kw++) {
                        long ih = (long)(oh * c->s_h + kh) - (long)c->p_h;
                        long iw = (long)(ow * c->s_w + kw) - (long)c->p_w;
                        if (ih < 0 || ih >= (long)c->h_in || iw < 0 || iw >= (long)c->w_in) continue;
                        const uint16_t *px = c->x + ((b * c->h_in + (size_t)ih) * c->w_in + (size_t)iw) * c->c_in;
                        if (!c->dw) {
                            for (size_t ic = 0; ic < c->c_in; ic++) {
                                size_t ki = ((kh * c->k_w + kw) * c->c_in + ic) * c->c_out + oc;
                                acc = fmaf(dwref_f16_to_f32(px[ic]), dwref_f16_to_f32(c->w[ki]), acc);
                            }
                        } else {
                            size_t ic = oc / c->mult, m = oc % c->mult;
                            size_t ki = ((kh * c->k_w + kw) * c->c_in + ic) * c->mult + m;
                            acc = fmaf(dwref_f16_to_f32(px[ic]), dwref_f16_to_f32(c->w[ki]), acc);
                        }
                    }
                uint16_t o = dwref_f16_from_f32(acc);
                if (c->bias) /* runtime.rs:1483-1497: bias added to the stored f16, rounded again */
                    o = dwref_f16_from_f32(dwref_f16_to_f32(o) + dwref_f16_to_f32(c->bias[oc]));
                if (c->relu) { /* ops.rs:345-352 relu_fp16 */
                    float v = dwref_f16_to_f32(o);
                    o = dwref_f16_from_f32(v > 0.0f ? v : 0.0f);
                }
                c->y[((b * c->h_out + oh) * c->w_out + ow) * c->c_out + oc] = o;
            }
    }
}

/* ops.rs:1442-1511 conv2d_fp16_nhwc (and its _mt twin :2572-2655): f32 FMA
 * accumulator in (kh, kw, ic) order, F16::from_f32 store; optional bias as the
 * CPU runtime applies it (runtime.rs:1483-1497) and ReLU (ops.rs:345). */
void dwref_conv2d_f16_nhwc(uint16_t *y, const uint16_t *x, const uint16_t *w_hwio,
                           const uint16_t *bias_or_null, int relu,
                           size_t n, size_t h_in, size_t w_in, size_t c_in, size_t c_out,
                           size_t k_h, size_t k_w, size_t stride_h, size_t stride_w,
                           size_t pad_h, size_t pad_w, int threads) {
    f16conv_ctx c;
    memset(&c, 0, sizeof c);
    c.y = y; c.x = x; c.w = w_hwio; c.bias = bias_or_null; c.relu = relu;
    c.n = n; c.h_in = h_in; c.w_in = w_in; c.c_in = c_in; c.c_out = c_out;
    c.k_h = k_h; c.k_w = k_w; c.s_h = stride_h; c.s_w = stride_w; c.p_h = pad_h; c.p_w = pad_w;
    c.h_out = (h_in + 2 * pad_h - k_h) / stride_h + 1;
    c.w_out = (w_in + 2 * pad_w - k_w) / stride_w + 1;
    parallel_for(threads, n * c.h_out, f16conv_rows, &c);
}

/* ops.rs:2819-2937 depthwise_conv2d_fp16_nhwc_mt: kernel [kh, kw, C, mult]. */
void dwref_dwconv_f16_nhwc(uint16_t *y, const uint16_t *x, const uint16_t *w,
                           const uint16_t *bias_or_null, int relu,
                           size_t n, size_t h_in, size_t w_in, size_t c_in, size_t mult,
                           size_t k_h, size_t k_w, size_t stride_h, size_t stride_w,
                           size_t pad_h, size_t pad_w, int threads) {
    f16conv_ctx c;
    memset(&c, 0, sizeof c);
    c.y = y; c.x = x; c.w = w; c.bias = bias_or_null; c.relu = relu; c.dw = 1; c.mult = mult;
    c.n = n; c.h_in = h_in; c.w_in = w_in; c.c_in = c_in; c.c_out = c_in * mult;
    c.k_h = k_h; c.k_w = k_w; c.s_h = stride_h; c.s_w = stride_w; c.p_h = pad_h; c.p_w = pad_w;
    c.h_out = (h_in + 2 * pad_h - k_h) / stride_h + 1;
    c.w_out = (w_in + 2 * pad_w - k_w) / stride_w + 1;
    parallel_for(threads, n * c.h_out, f16conv_rows, &c);
}

typedef struct { uint16_t *c; const uint16_t *a, *b; size_t m, n, k; } f16gemm_ctx;

static void f16gemm_rows(void *p, size_t start, size_t end) {
    f16gemm_ctx *g = (f16gemm_ctx *)p;
    for (size_t i = start; i < end; i++)
        for (size_t j = 0; j < g->n; j++) {
            float acc = 0.0f;
            for (size_t q = 0; q < g->k; q++)
                acc = fmaf(dwref_f16_to_f32(g->a[i * g->k + q]), dwref_f16_to_f32(g->b[q * g->n + j]), acc);
            g->c[i * g->n + j] = dwref_f16_from_f32(acc);
        }
}

/* ops.rs:461-481 gemm_fp16 (row-partitioned like gemm_fp16_mt :1709-1754). */
void dwref_gemm_f16(uint16_t *c, const uint16_t *a, const uint16_t *b, size_t m, size_t n, size_t k,
                    int threads) {
    f16gemm_ctx g = {c, a, b, m, n, k};
    parallel_for(threads, m, f16gemm_rows, &g);
}

/* The bias step of the CPU runtime's F16 Gemm and Conv (runtime.rs:1264-1275,
 * 1483-1497): out = from_f32(to_f32(out) + to_f32(bias[j])) over [rows, c], in
 * place; then, with `relu`, the Relu op (runtime.rs:967-971 / ops.rs:345-352). */
void dwref_bias_relu_f16(uint16_t *y, const uint16_t *bias_or_null, int relu, size_t rows, size_t c) {
    for (size_t i = 0; i < rows; i++)
        for (size_t j = 0; j < c; j++) {
            uint16_t o = y[i * c + j];
            if (bias_or_null) o = dwref_f16_from_f32(dwref_f16_to_f32(o) + dwref_f16_to_f32(bias_or_null[j]));
            if (relu) {
                float v = dwref_f16_to_f32(o);
                o = dwref_f16_from_f32(v > 0.0f ? v : 0.0f);
            }
            y[i * c + j] = o;
        }
}

/* Element-wise F16::from_f32 / F16::to_f32 (the runtime's input conversion,
 * runtime.rs:842-851, and output read-back). */
void dwref_f16_from_f32_array(uint16_t *y, const float *x, size_t len) {
    for (size_t i = 0; i < len; i++) y[i] = dwref_f16_from_f32(x[i]);
}

void dwref_f16_to_f32_array(float *y, const uint16_t *x, size_t len) {
    for (size_t i = 0; i < len; i++) y[i] = dwref_f16_to_f32(x[i]);
}

/* ops.rs:434-446 add_fp16. */
void dwref_add_f16(uint16_t *y, const uint16_t *a, const uint16_t *b, size_t len) {
    for (size_t i = 0; i < len; i++)
        y[i] = dwref_f16_from_f32(dwref_f16_to_f32(a[i]) + dwref_f16_to_f32(b[i]));
}

/* ops.rs:345-352 relu_fp16. */
void dwref_relu_f16(uint16_t *y, const uint16_t *x, size_t len) {
    for (size_t i = 0; i < len; i++) {
        float v = dwref_f16_to_f32(x[i]);
        y[i] = dwref_f16_from_f32(v > 0.0f ? v : 0.0f);
    }
}

/* runtime.rs:1155-1170 GlobalAveragePool F16: sequential f32 sum over (row, col),
 * then sum / spatial, stored as F16.  Output [N, C]. */
void dwref_gap_f16(uint16_t *y, const uint16_t *x, size_t n, size_t h, size_t w, size_t c) {
    size_t spatial = h * w;
    for (size_t b = 0; b < n; b++)
        for (size_t ch = 0; ch < c; ch++) {
            float sum = 0.0f;
            for (size_t r = 0; r < h; r++)
                for (size_t q = 0; q < w; q++) sum += dwref_f16_to_f32(x[((b * h + r) * w + q) * c + ch]);
            y[b * c + ch] = dwref_f16_from_f32(sum / (float)spatial);
        }
}

/* runtime.rs:1545-1560 F16 maxpool: f16 -> f32, maxpool2d_f32_nhwc
 * (ops.rs:1513-1551, NEG_INFINITY start, f32::max), -> f16; padded taps skipped. */
void dwref_maxpool_f16_nhwc(uint16_t *y, const uint16_t *x, size_t n, size_t h, size_t w, size_t c,
                            size_t k_h, size_t k_w, size_t s_h, size_t s_w,
                            size_t p_t, size_t p_l, size_t p_b, size_t p_r) {
    size_t h_out = (h + p_t + p_b - k_h) / s_h + 1, w_out = (w + p_l + p_r - k_w) / s_w + 1;
    for (size_t b = 0; b < n; b++)
        for (size_t oh = 0; oh < h_out; oh++)
            for (size_t ow = 0; ow < w_out; ow++)
                for (size_t ch = 0; ch < c; ch++) {
                    float m = -INFINITY;
                    for (size_t ph = 0; ph < k_h; ph++)
                        for (size_t pw = 0; pw < k_w; pw++) {
                            long ih = (long)(oh * s_h + ph) - (long)p_t;
                            long iw = (long)(ow * s_w + pw) - (long)p_l;
                            if (ih < 0 || ih >= (long)h || iw < 0 || iw >= (long)w) continue;
                            m = fmaxf(m, dwref_f16_to_f32(x[((b * h + (size_t)ih) * w + (size_t)iw) * c + ch]));
                        }
                    y[((b * h_out + oh) * w_out + ow) * c + ch] = dwref_f16_from_f32(m);
                }
}

/* Input quantisation of a uint8 image: x = (f32)u * (1/255) (the 1/255
 * normalisation of the YOLO input), then quantize_f32_to_i8 (ops.rs:3503-3525). */
void dwref_quantize_u8_to_i8(int8_t *out, const uint8_t *in, size_t len, float scale) {
    float inv255 = 1.0f / 255.0f, inv_scale = 1.0f / scale;
    for (size_t i = 0; i < len; i++) out[i] = dwref_f32_to_i8(((float)in[i] * inv255) * inv_scale);
}

/* ------------------------------------------------------------------------ */
/* YOLOv8 Detect head tail (the f32 graph ops after DequantizeLinear)         */
/* ------------------------------------------------------------------------ */

/* softmax_f32 on one row (crates/dragonwing-cpu/src/ops.rs:1609-1640):
 * max by fold(-inf, f32::max), exp(x - max) summed in order, times 1/sum. */
static void softmax_row(float *out, const float *in, size_t n) {
    float max_val = -INFINITY;
    for (size_t i = 0; i < n; i++) max_val = fmaxf(max_val, in[i]);
    float sum = 0.0f;
    for (size_t i = 0; i < n; i++) {
        float e = expf(in[i] - max_val);
        out[i] = e;
        sum += e;
    }
    float inv_sum = 1.0f / sum;
    for (size_t i = 0; i < n; i++) out[i] *= inv_sum;
}

/* sigmoid_f32_scalar (ops.rs:1865-1870). */
static float sigmoid_one(float x) { return 1.0f / (1.0f + expf(-x)); }

void dwref_sigmoid_f32(float *y, const float *x, size_t len) {
    for (size_t i = 0; i < len; i++) y[i] = sigmoid_one(x[i]);
}

/* softmax_f32 (ops.rs:1609-1640) over rows of n. */
void dwref_softmax_f32(float *out, const float *in, size_t len, size_t n) {
    for (size_t r = 0; r + n <= len; r += n) softmax_row(out + r, in + r, n);
}

/* The exported YOLOv8 Detect tail on dequantised head outputs, per image and
 * level: DFL = softmax over reg_max bins per box side, then the 1x1 conv with
 * kernel [0, 1, ..., reg_max-1] (conv2d_f32_nhwc's sum from 0.0 in channel
 * order, ops.rs:1396-1415); dist2bbox: x1y1 = anchor - lt, x2y2 = anchor + rb,
 * centre = (x1y1 + x2y2) / 2, size = x2y2 - x1y1 (Sub/Add/Div, runtime.rs:
 * 1736-1850), times the stride (Mul); class scores = sigmoid; concat along
 * anchors.  Anchors are the cell centres (x + 0.5, y + 0.5), row-major.
 * box[l]: int8 [n, h, w, 4*reg_max]; cls[l]: int8 [n, h, w, nc];
 * out: f32 [n, 4 + nc, A]. */
void dwref_yolo_detect_i8(float *out, const int8_t *const *box, const int8_t *const *cls,
                          const dwref_yolo_desc *d) {
    size_t A = 0;
    for (int l = 0; l < d->num_levels; l++) A += (size_t)d->h[l] * d->w[l];
    const size_t R = (size_t)d->reg_max, nc = (size_t)d->num_classes, rows = 4 + nc;
    float x[64], p[64];
    for (int img = 0; img < d->n; img++) {
        size_t off = 0;
        for (int l = 0; l < d->num_levels; l++) {
            const size_t hw = (size_t)d->h[l] * d->w[l];
            for (size_t local = 0; local < hw; local++) {
                const size_t pix = (size_t)img * hw + local, a = off + local;
                const int8_t *bq = box[l] + pix * 4 * R;
                float dist[4];
                for (int s = 0; s < 4; s++) {
                    for (size_t i = 0; i < R; i++) x[i] = (float)bq[s * R + i] * d->box_scale[l];
                    softmax_row(p, x, R);
                    float acc = 0.0f;
                    for (size_t i = 0; i < R; i++) acc += p[i] * (float)i;
                    dist[s] = acc;
                }
                const float ax = (float)(local % (size_t)d->w[l]) + 0.5f;
                const float ay = (float)(local / (size_t)d->w[l]) + 0.5f;
                const float x1 = ax - dist[0], y1 = ay - dist[1], x2 = ax + dist[2], y2 = ay + dist[3];
                const float st = d->stride[l];
                float *o = out + (size_t)img * rows * A + a;
                o[0] = ((x1 + x2) / 2.0f) * st;
                o[A] = ((y1 + y2) / 2.0f) * st;
                o[2 * A] = (x2 - x1) * st;
                o[3 * A] = (y2 - y1) * st;
                const int8_t *cq = cls[l] + pix * nc;
                for (size_t c = 0; c < nc; c++) o[(4 + c) * A] = sigmoid_one((float)cq[c] * d->cls_scale[l]);
            }
            off += hw;
        }
    }
}

/* ------------------------------------------------------------------------ */
/* Detection post-processing (crates/dragonwing-onnx/src/postprocess.rs)      */
/* ------------------------------------------------------------------------ */

/* Detection::area (postprocess.rs:28-32). */
float dwref_det_area(const dwref_detection *d) {
    float w = fmaxf(d->bbox[2] - d->bbox[0], 0.0f);
    float h = fmaxf(d->bbox[3] - d->bbox[1], 0.0f);
    return w * h;
}

/* iou (postprocess.rs:36-55). */
float dwref_iou(const dwref_detection *a, const dwref_detection *b) {
    float x1 = fmaxf(a->bbox[0], b->bbox[0]);
    float y1 = fmaxf(a->bbox[1], b->bbox[1]);
    float x2 = fminf(a->bbox[2], b->bbox[2]);
    float y2 = fminf(a->bbox[3], b->bbox[3]);
    float inter_w = fmaxf(x2 - x1, 0.0f);
    float inter_h = fmaxf(y2 - y1, 0.0f);
    float inter_area = inter_w * inter_h;
    float union_area = dwref_det_area(a) + dwref_det_area(b) - inter_area;
    return union_area > 0.0f ? inter_area / union_area : 0.0f;
}

/* decode_detections_v8 (postprocess.rs:78-146; raw [4 + nc, A]) or, with alt,
 * decode_detections_v8_alt (:151-208; raw [A, 4 + nc]).  Writes at most
 * num_detections detections in anchor order; returns their count (0 when
 * raw_len is short, :92-95). */
size_t dwref_decode_detections_v8(dwref_detection *out, const float *raw, size_t raw_len, size_t num_classes,
                                  size_t num_detections, uint32_t img_width, uint32_t img_height,
                                  float conf_threshold, int alt) {
    const size_t row = 4 + num_classes;
    if (raw_len < row * num_detections) return 0;
    const float model_size = 640.0f;
    const float scale_x = (float)img_width / model_size, scale_y = (float)img_height / model_size;
    const float iw = (float)img_width, ih = (float)img_height;
    size_t n = 0;
    for (size_t a = 0; a < num_detections; a++) {
        const size_t step = alt ? 1 : num_detections;
        const float *q = alt ? raw + a * row : raw + a;
        float cx = q[0], cy = q[step], w = q[2 * step], h = q[3 * step];
        size_t best_class = 0;
        float best_conf = 0.0f;
        for (size_t c = 0; c < num_classes; c++) {
            float conf = q[(4 + c) * step];
            if (conf > best_conf) {
                best_conf = conf;
                best_class = c;
            }
        }
        if (best_conf < conf_threshold) continue;
        float x1 = (cx - w / 2.0f) * scale_x, y1 = (cy - h / 2.0f) * scale_y;
        float x2 = (cx + w / 2.0f) * scale_x, y2 = (cy + h / 2.0f) * scale_y;
        dwref_detection *o = &out[n++];
        o->bbox[0] = fminf(fmaxf(x1, 0.0f), iw);
        o->bbox[1] = fminf(fmaxf(y1, 0.0f), ih);
        o->bbox[2] = fminf(fmaxf(x2, 0.0f), iw);
        o->bbox[3] = fminf(fmaxf(y2, 0.0f), ih);
        o->class_id = (uint32_t)best_class;
        o->confidence = best_conf;
    }
    return n;
}

/* Stable merge sort by confidence descending: Vec::sort_by with
 * b.confidence.partial_cmp(&a.confidence) (postprocess.rs:229-231). */
static void sort_by_conf_desc(dwref_detection *d, dwref_detection *tmp, size_t n) {
    for (size_t width = 1; width < n; width *= 2) {
        for (size_t lo = 0; lo < n; lo += 2 * width) {
            size_t mid = lo + width < n ? lo + width : n, hi = lo + 2 * width < n ? lo + 2 * width : n;
            size_t i = lo, j = mid, k = lo;
            while (i < mid && j < hi) tmp[k++] = d[j].confidence > d[i].confidence ? d[j++] : d[i++];
            while (i < mid) tmp[k++] = d[i++];
            while (j < hi) tmp[k++] = d[j++];
        }
        memcpy(d, tmp, n * sizeof(*d));
    }
}

/* nms (postprocess.rs:227-265) or, with agnostic, nms_agnostic (:270-300), in
 * place: sort, greedy suppression when iou > iou_threshold, then the
 * swap_remove deletion from the back.  Returns the new length. */
size_t dwref_nms(dwref_detection *d, size_t n, float iou_threshold, int agnostic) {
    if (n == 0) return 0;
    dwref_detection *tmp = (dwref_detection *)malloc(n * sizeof(*d));
    unsigned char *keep = (unsigned char *)malloc(n);
    sort_by_conf_desc(d, tmp, n);
    memset(keep, 1, n);
    for (size_t i = 0; i < n; i++) {
        if (!keep[i]) continue;
        for (size_t j = i + 1; j < n; j++) {
            if (!keep[j]) continue;
            if (!agnostic && d[i].class_id != d[j].class_id) continue;
            if (dwref_iou(&d[i], &d[j]) > iou_threshold) keep[j] = 0;
        }
    }
    size_t len = n;
    for (size_t i = n; i > 0;) {
        i--;
        if (!keep[i]) {
            d[i] = d[len - 1]; /* Vec::swap_remove(i) */
            len--;
        }
    }
    free(tmp);
    free(keep);
    return len;
}

/* postprocess_yolo (postprocess.rs:319-340) on one image; out has room for
 * num_detections entries.  flags as the device API: 1 alt layout, 2 agnostic
 * NMS, 4 no NMS. */
size_t dwref_postprocess_yolo(dwref_detection *out, const float *raw, size_t raw_len, size_t num_classes,
                              size_t num_detections, uint32_t img_width, uint32_t img_height,
                              float conf_threshold, float iou_threshold, int flags) {
    size_t n = dwref_decode_detections_v8(out, raw, raw_len, num_classes, num_detections, img_width, img_height,
                                          conf_threshold, flags & 1);
    if (flags & 4) return n;
    return dwref_nms(out, n, iou_threshold, (flags & 2) != 0);
}
