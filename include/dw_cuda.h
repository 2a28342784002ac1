/*
 * dw_cuda.h -- C ABI of libdragonwing_cuda.so, the B200 (sm_100a) backend for
 * the fused quantized convolution path of dragonwing-edge-rs.
 *
 * Plain C types only (pointers, sizes, scalars); no CUDA or C++ types appear
 * in any signature, so a Rust `extern "C"` block, ctypes or cgo can bind it.
 * Every entry point names the reference interface it replaces (paths relative
 * to the reference repository root).
 *
 * Execution model: one dw_backend per host thread and per GPU.  A backend owns
 * one CUDA stream; every op is enqueued asynchronously on it.  dw_upload,
 * dw_download and dw_synchronize are the blocking calls, like the reference's
 * Backend trait (crates/dragonwing-core/src/backend.rs:127-199).  Buffers are
 * opaque byte spans with no dtype (backend.rs:21-33).  Errors never truncate
 * or abort: every call returns a dw_status, and dw_last_error() gives the
 * reason string (the reference's Error::Backend(String)).
 */
#ifndef DW_CUDA_H
#define DW_CUDA_H

#include <stddef.h>
#include <stdint.h>

#ifdef __cplusplus
extern "C" {
#endif

#if defined(__GNUC__)
#define DW_API __attribute__((visibility("default")))
#else
#define DW_API
#endif

/* Status codes.  Mirrors Result<(), Error> (crates/dragonwing-core/src/error.rs:13). */
typedef enum dw_status {
    DW_OK = 0,
    DW_ERR_INVALID_ARG = 1,        /* bad shape, null pointer, unsupported parameter value */
    DW_ERR_SIZE_MISMATCH = 2,      /* buffer length != expected (backend.rs:160-185) */
    DW_ERR_UNSUPPORTED = 3,        /* valid op the backend does not implement */
    DW_ERR_OOM = 4,                /* allocation failed */
    DW_ERR_TIMEOUT = 5,            /* dw_synchronize deadline passed; work still queued */
    DW_ERR_DEVICE = 6,             /* CUDA runtime/driver error */
    DW_ERR_KERNEL_WAIT_EXPIRED = 7 /* a kernel's bounded device-side wait gave up */
} dw_status;

typedef struct dw_backend dw_backend; /* one GPU + one stream (impl Backend) */
typedef struct dw_buf dw_buf;         /* device byte buffer (impl BackendBuffer) */

typedef struct dw_config {
    uint32_t wait_cap_ms; /* limit for every device-side wait (mbarrier/TMA); 0 = 2000 ms */
    int32_t trace;        /* nonzero: synchronize and log after every op (DRAGONWING_TRACE) */
    int32_t conv_path;    /* DW_PATH_*: which convolution kernels to use */
    int32_t dw_variant;   /* int8 depthwise 3x3 s1 kernel: 0 auto, DW_DWV_* to force one (tuning, tests) */
    int32_t reserved[4];
} dw_config;

enum dw_dw_variant {
    DW_DWV_AUTO = 0,
    DW_DWV_SLAB = 1,     /* 64-channel slabs, one row per copy */
    DW_DWV_STREAM2 = 2,   /* persistent whole-pixel streaming, 4 channels x 2 columns per thread, 18 warps (the default) */
    DW_DWV_STREAM2X2 = 3, /* the same, two CTAs of 9 consumer warps per SM */
    DW_DWV_STREAM4 = 4    /* 4 channels x 4 columns per thread, 9 consumer warps */
};

enum dw_conv_path {
    DW_PATH_AUTO = 0,   /* tensor-core (tcgen05) kernels where the shape allows, else CUDA cores */
    DW_PATH_DIRECT = 1, /* always the CUDA-core direct kernels */
    DW_PATH_UMMA = 2    /* tensor-core kernels only; DW_ERR_UNSUPPORTED where they do not apply */
};

/* Epilogue of the fused op.  The reference has NONE and RELU (has_relu,
 * crates/dragonwing-onnx/src/builder.rs:345-360); RELU6 and SILU extend it. */
enum dw_epilogue { DW_EPI_NONE = 0, DW_EPI_RELU = 1, DW_EPI_RELU6 = 2, DW_EPI_SILU = 3 };

/* One fused convolution.  Mirrors OpParams::Conv2dRequantReluI8Nhwc
 * (crates/dragonwing-onnx/src/builder.rs:345-360) plus the NHWC dims the
 * runtime reads from graph.shapes (vulkan_runtime.rs:1135-1205):
 *   pads = [top, left, bottom, right]; dilation must be 1 (builder.rs:543-551);
 *   group == 1 (dense) or group == c_in (depthwise, c_out = c_in * multiplier);
 *   epilogue = dw_epilogue; q6 = ReLU6 ceiling in the output's int8 domain;
 *   inv_s_out = 1/s_out (SiLU only). */
typedef struct dw_conv_desc {
    int32_t n, h, w, c_in, c_out;
    int32_t k_h, k_w, stride_h, stride_w;
    int32_t pad_t, pad_l, pad_b, pad_r;
    int32_t group;
    int32_t epilogue;
    int32_t q6;
    float inv_s_out;
} dw_conv_desc;

/* ---------------------------------------------------------------------- */
/* Backend trait: crates/dragonwing-core/src/backend.rs:127-199           */
/* ---------------------------------------------------------------------- */

/* Backend::name (backend.rs:141): "cuda-sm100a". */
DW_API const char *dw_name(void);
/* Library version string (for logs). */
DW_API const char *dw_version(void);
/* Creates a backend on `device_ordinal` (VulkanBackend::new, vulkan/src/lib.rs:97).
 * cfg may be NULL (defaults).  The DW_WAIT_CAP_MS / DW_TRACE / DW_CONV_PATH
 * environment variables override the config. */
DW_API dw_status dw_create(int device_ordinal, const dw_config *cfg, dw_backend **out);
DW_API void dw_destroy(dw_backend *be);
/* Reason string of the last failed call on this backend (Error::Backend(String)). */
DW_API const char *dw_last_error(const dw_backend *be);
/* Backend::alloc (backend.rs:155).  Zero-length is an error (vulkan/src/lib.rs:257-261).
 * Contents are unspecified on return. */
DW_API dw_status dw_alloc(dw_backend *be, size_t len_bytes, dw_buf **out);
/* Wraps caller-owned device memory (not freed by dw_free). */
DW_API dw_status dw_buf_wrap(dw_backend *be, void *device_ptr, size_t len_bytes, dw_buf **out);
DW_API dw_status dw_free(dw_backend *be, dw_buf *buf);
/* BackendBuffer::len_bytes (backend.rs:21-33). */
DW_API size_t dw_buf_len(const dw_buf *buf);
DW_API void *dw_buf_device_ptr(const dw_buf *buf);
/* Backend::upload (backend.rs:166-173): src_len must equal the buffer length;
 * complete when the call returns. */
DW_API dw_status dw_upload(dw_backend *be, dw_buf *dst, const void *src, size_t src_len);
/* Backend::download (backend.rs:177-185): synchronizes first, then copies. */
DW_API dw_status dw_download(dw_backend *be, const dw_buf *src, void *dst, size_t dst_len);
/* Asynchronous twins on the backend stream (host memory should be pinned). */
DW_API dw_status dw_upload_async(dw_backend *be, dw_buf *dst, size_t dst_offset, const void *src, size_t len);
DW_API dw_status dw_download_async(dw_backend *be, const dw_buf *src, size_t src_offset, void *dst, size_t len);
/* Device-to-device copy on the backend stream (staging for pipelined serving). */
DW_API dw_status dw_copy_async(dw_backend *be, dw_buf *dst, size_t dst_offset, const dw_buf *src,
                               size_t src_offset, size_t len);
/* Stream ordering between backends on one GPU (each backend owns a stream): a
 * copy backend can upload step i+1's input and read back step i's output while
 * the compute backend runs.  Buffers of one GPU may be used by any backend on it. */
typedef struct dw_event dw_event;
DW_API dw_status dw_event_create(dw_backend *be, dw_event **out);
DW_API void dw_event_destroy(dw_event *ev);
/* Records `ev` at the current end of be's stream. */
DW_API dw_status dw_event_record(dw_backend *be, dw_event *ev);
/* Work enqueued on be's stream after this call waits for `ev`. */
DW_API dw_status dw_stream_wait_event(dw_backend *be, dw_event *ev);
/* Backend::synchronize (backend.rs:187-198) with a deadline: DW_ERR_TIMEOUT when
 * the queued work has not finished after timeout_ms (0 = no deadline); also
 * reports DW_ERR_KERNEL_WAIT_EXPIRED if a kernel's bounded wait gave up. */
DW_API dw_status dw_synchronize(dw_backend *be, uint32_t timeout_ms);
/* Page-locked host memory for the asynchronous copies. */
DW_API dw_status dw_host_alloc(dw_backend *be, size_t len_bytes, void **out);
DW_API dw_status dw_host_free(dw_backend *be, void *ptr);
/* The backend's cudaStream_t, as an opaque pointer (for event timing). */
DW_API void *dw_stream(dw_backend *be);
/* Number of SMs of the backend's GPU. */
DW_API int dw_sm_count(const dw_backend *be);
/* Counts kernel launches made through this backend (diagnostics / benchmarks). */
DW_API uint64_t dw_launch_count(const dw_backend *be);
/* Bytes of device scratch the backend holds.  Ops that need temporaries (the
 * reference-signature conv's repacked weights, GEMM transposes, post-processing
 * workspaces) grow it with cudaMalloc and keep it until dw_destroy.  A
 * diagnostic with no counterpart in the reference. */
DW_API size_t dw_scratch_bytes(const dw_backend *be);
/* CUDA-graph capture of an op sequence enqueued on the backend stream (the
 * reference's OpsRecorder single-command-buffer recording,
 * crates/dragonwing-vulkan/src/record.rs:49-679): between dw_capture_begin and
 * dw_capture_end, ops are recorded instead of executed; dw_graph_launch replays
 * them with one launch.  No allocation may happen while capturing. */
typedef struct dw_graph dw_graph;
DW_API dw_status dw_capture_begin(dw_backend *be);
DW_API dw_status dw_capture_end(dw_backend *be, dw_graph **out);
DW_API dw_status dw_graph_launch(dw_backend *be, dw_graph *g);
DW_API void dw_graph_destroy(dw_graph *g);
/* Test hook: runs one bounded device-side wait on a flag that nothing sets,
 * with a cap of cap_us microseconds; the kernel gives up and records the
 * failure, and the next dw_synchronize reports DW_ERR_KERNEL_WAIT_EXPIRED. */
DW_API dw_status dw_debug_expire_wait(dw_backend *be, uint32_t cap_us);

/* ---------------------------------------------------------------------- */
/* Fused INT8 convolution (the hot path)                                   */
/* ---------------------------------------------------------------------- */

/* Repacks an HWIO int8 kernel [k_h, k_w, c_in, c_out] (the layout after
 * convert_nchw_to_nhwc, crates/dragonwing-onnx/src/graph.rs:261-275, read by
 * conv2d_i8_nhwc ops.rs:3129) once, at weight-prepare time, into the layout the
 * kernels read.  Depthwise kernels are [k_h, k_w, c_in, multiplier]
 * (ops.rs:2669-2730).  *out is a new buffer owned by the caller. */
DW_API dw_status dw_prepare_weights_i8(dw_backend *be, const dw_conv_desc *d, const dw_buf *w_hwio,
                                       dw_buf **out);

/* The fused op: y = epilogue(requant(conv(x, w) + bias)).
 * Replaces conv2d_requant_relu_i8_packed (crates/dragonwing-vulkan/src/ops.rs:2294-2417)
 * with the build's superset contract:
 *   acc  = sum x[n, oh*sh+kh-pt, ow*sw+kw-pl, ic] * w[kh,kw,ic,oc]   (i32, OOB taps skipped)
 *   acc += bias[oc]                                                  (bias may be NULL)
 *   NONE/RELU/RELU6: q = (int8) roundf(clamp((float)acc * M[oc], -128, 127)),
 *                    then max(q,0) / min(max(q,0), q6)
 *   SILU: y = (float)acc * D[oc]; q = (int8) roundf(clamp(silu(y) * inv_s_out, -128, 127))
 * x: int8 NHWC [n,h,w,c_in]; w_prep from dw_prepare_weights_i8; bias: int32 [c_out];
 * M, D: float32 [c_out] (M[oc] = (s_in*s_w[oc])/s_out, quantize.rs:245; D[oc] = s_in*s_w[oc]);
 * y: int8 NHWC [n,h_out,w_out,c_out].  Bit-exact with the reference scalar path. */
DW_API dw_status dw_conv2d_i8(dw_backend *be, const dw_conv_desc *d, const dw_buf *x, const dw_buf *w_prep,
                              const dw_buf *bias, const dw_buf *M, const dw_buf *D, dw_buf *y);

/* Exact reference parameter list of conv2d_requant_relu_i8_packed
 * (crates/dragonwing-vulkan/src/ops.rs:2294-2345): scalar requant_scale, no bias,
 * HWIO kernel, symmetric pads, same error strings ("conv_fused: ...").  Prepares
 * the weights internally on every call (use dw_conv2d_i8 to prepare once). */
DW_API dw_status dw_conv2d_requant_relu_i8(dw_backend *be, const dw_buf *input, const dw_buf *kernel_hwio,
                                           dw_buf *output, size_t n, size_t h_in, size_t w_in, size_t c_in,
                                           size_t c_out, size_t k_h, size_t k_w, size_t stride_h,
                                           size_t stride_w, size_t pad_h, size_t pad_w, float requant_scale,
                                           int do_relu);

/* Same op, parameters and checks as dw_conv2d_requant_relu_i8, for callers that
 * must not allocate device memory per call (a fixed memory plan reserved at
 * start-up, or a latency-critical loop where an allocator call is not allowed).
 * No counterpart in the reference.  Its temporaries (repacked weights and the
 * scale array) live in one fixed device array inside the library, held by every
 * GPU that loads it until exit; it accepts kernels of at most 1 MiB
 * (k_h*k_w*c_in*c_out bytes) and at most 4096 output channels and rejects larger
 * ones with DW_ERR_INVALID_ARG.  The first call on a device looks the array's
 * address up (again after the device's context was reset, e.g. by
 * cudaDeviceReset); make that call before any stream capture on the device.
 * It never grows the backend's scratch (dw_scratch_bytes stays unchanged).
 * Calls share the array: calls that overlap on the GPU race and must be
 * serialised. */
DW_API dw_status dw_conv2d_requant_relu_i8_noalloc(dw_backend *be, const dw_buf *input, const dw_buf *kernel_hwio,
                                                   dw_buf *output, size_t n, size_t h_in, size_t w_in, size_t c_in,
                                                   size_t c_out, size_t k_h, size_t k_w, size_t stride_h,
                                                   size_t stride_w, size_t pad_h, size_t pad_w,
                                                   float requant_scale, int do_relu);

/* Unfused int8 conv to int32 accumulators: conv2d_i8_nhwc_packed
 * (crates/dragonwing-vulkan/src/ops.rs:1822), CPU twin conv2d_i8_nhwc (cpu ops.rs:3086). */
DW_API dw_status dw_conv2d_i8_nhwc(dw_backend *be, const dw_buf *input, const dw_buf *kernel_hwio,
                                   dw_buf *output_i32, size_t n, size_t h_in, size_t w_in, size_t c_in,
                                   size_t c_out, size_t k_h, size_t k_w, size_t stride_h, size_t stride_w,
                                   size_t pad_h, size_t pad_w);

/* ---------------------------------------------------------------------- */
/* INT8 GEMM                                                               */
/* ---------------------------------------------------------------------- */

/* gemm_i8_packed (crates/dragonwing-vulkan/src/ops.rs:1723) / gemm_i8 (cpu ops.rs:2964):
 * C_i32[m,n] = A[m,k] * B[k,n], both row-major int8. */
DW_API dw_status dw_gemm_i8(dw_backend *be, const dw_buf *a, const dw_buf *b, dw_buf *c_i32, size_t m,
                            size_t n, size_t k);
/* Repacks B [k,n] row-major (a QGemm weight) once into the kernel layout. */
DW_API dw_status dw_prepare_gemm_b_i8(dw_backend *be, const dw_buf *b_kn, size_t k, size_t n, dw_buf **out);
/* QGemm with int32 bias[n] (may be NULL), per-column M[n] and the fused
 * epilogue (NONE/RELU/RELU6; q6 for RELU6): y_i8[m,n].  The same contract as
 * dw_conv2d_i8 with a 1x1 kernel over m pixels. */
DW_API dw_status dw_qgemm_i8(dw_backend *be, const dw_buf *a, const dw_buf *b_prep, const dw_buf *bias,
                             const dw_buf *M, dw_buf *y, size_t m, size_t n, size_t k, int epilogue, int q6);

/* ---------------------------------------------------------------------- */
/* INT8 elementwise and glue                                               */
/* ---------------------------------------------------------------------- */

/* requantize_i32_to_i8_packed (vulkan ops.rs:1998) / cpu ops.rs:3366-3386. */
DW_API dw_status dw_requantize_i32_to_i8(dw_backend *be, const dw_buf *in_i32, dw_buf *out_i8, float scale);
/* relu_i8_packed (vulkan ops.rs:2179) / cpu ops.rs:3301-3319. */
DW_API dw_status dw_relu_i8(dw_backend *be, const dw_buf *in, dw_buf *out);
/* add_i8_packed (vulkan ops.rs:2105) / cpu ops.rs:3176-3209 (OpParams::AddQuantized). */
DW_API dw_status dw_add_i8(dw_backend *be, const dw_buf *a, const dw_buf *b, dw_buf *out,
                           float scale_a_over_y, float scale_b_over_y);
/* quantize_f32_to_i8_packed (vulkan ops.rs:2032) / cpu ops.rs:3503-3525. */
DW_API dw_status dw_quantize_f32_to_i8(dw_backend *be, const dw_buf *in_f32, dw_buf *out_i8, float scale);
/* Input quantisation of uint8 images: q = quantize(u8 * (1/255), s) in one pass
 * (the YOLO input path: u8 -> /255 -> f32 -> quantize). */
DW_API dw_status dw_quantize_u8_to_i8(dw_backend *be, const dw_buf *in_u8, dw_buf *out_i8, float scale);
/* im2col of a uint8 NHWC image fused with its quantisation: y [n, h_out,
 * w_out, c_dst] int8 with y[b][i][j][(a*k_w + q)*c + ch] = the
 * dw_quantize_u8_to_i8 value of x[b][i*s_h + a - p_t][j*s_w + q - p_l][ch]
 * (0 in the padding and in channels k_h*k_w*c .. c_dst-1); c, k_h, k_w <= 8,
 * c_dst <= 64 and a multiple of 16.  The first conv of
 * a network on a few-channel image then runs as a 1x1 conv over c_dst
 * channels on the tensor cores, with the same integer products. */
DW_API dw_status dw_im2col_u8_to_i8(dw_backend *be, const dw_buf *x_u8, dw_buf *y_i8, size_t n, size_t h, size_t w,
                                    size_t c, size_t k_h, size_t k_w, size_t s_h, size_t s_w, size_t p_t, size_t p_l,
                                    size_t h_out, size_t w_out, size_t c_dst, float scale);
/* The network's input stem in one pass: dw_quantize_u8_to_i8 of a 3-channel
 * uint8 NHWC image (scale in_scale) followed by the fused op of dw_conv2d_i8
 * (d: the 3x3 conv on c_in = 3, group 1, any stride and padding; the same
 * epilogue contract and bit-exact result) without the quantised image or an
 * im2col tensor in memory.  Replaces the input path of the reference's YOLO
 * graph: QuantizeLinear of the /255 image (quantize_f32_to_i8_scalar,
 * crates/dragonwing-cpu/src/ops.rs:3503-3525) then its first
 * Conv2dRequantReluI8Nhwc (conv2d_requant_relu_i8_packed,
 * crates/dragonwing-vulkan/src/ops.rs:2294-2417).  kernel_hwio: int8 HWIO
 * [3][3][3][c_out] as given to dw_prepare_weights_i8 (not prepared); c_out a
 * multiple of 16 and <= 64; the image width a multiple of 16, pad_l <= 5,
 * 16-byte aligned input and output; other shapes return DW_ERR_UNSUPPORTED
 * (run dw_im2col_u8_to_i8 and a 1x1 dw_conv2d_i8 instead). */
DW_API dw_status dw_conv2d_stem_u8_i8(dw_backend *be, const dw_conv_desc *d, const dw_buf *x_u8, float in_scale,
                                      const dw_buf *kernel_hwio, const dw_buf *bias, const dw_buf *M, const dw_buf *D,
                                      dw_buf *y);
/* dequantize_i8_packed_to_f32 (vulkan ops.rs:2069) / cpu ops.rs:3439-3457. */
DW_API dw_status dw_dequantize_i8_to_f32(dw_backend *be, const dw_buf *in_i8, dw_buf *out_f32, float scale);
/* maxpool2d (cpu ops.rs:1513-1551) on int8 NHWC, with pads [t,l,b,r] taken as -inf. */
DW_API dw_status dw_maxpool_i8(dw_backend *be, const dw_buf *x, dw_buf *y, size_t n, size_t h, size_t w,
                               size_t c, size_t k_h, size_t k_w, size_t s_h, size_t s_w, size_t p_t,
                               size_t p_l, size_t p_b, size_t p_r);
/* concat along channels (cpu concat_f32 axis 3, ops.rs:2141-2246) of `count`
 * int8 NHWC tensors with channels[i] each over `pixels` pixels. */
DW_API dw_status dw_concat_i8(dw_backend *be, const dw_buf *const *xs, const int32_t *channels, int32_t count,
                              size_t pixels, dw_buf *y);
/* Channel slice [c0, c0+c_len) of an NHWC tensor with c_total channels
 * (Split/Slice along C, cpu ops.rs:2407, 2532). */
DW_API dw_status dw_slice_c_i8(dw_backend *be, const dw_buf *x, dw_buf *y, size_t pixels, size_t c_total,
                               size_t c0, size_t c_len);
/* Nearest resize (cpu resize_f32 Nearest, ops.rs:2320-2348) on int8 NHWC. */
DW_API dw_status dw_resize_nearest_i8(dw_backend *be, const dw_buf *x, dw_buf *y, size_t n, size_t h_in,
                                      size_t w_in, size_t h_out, size_t w_out, size_t c);

/* Channel-range views.  A dw_view is a channel range of an NHWC tensor that
 * lives inside a wider one: its element (pixel p, channel c) is the byte at
 * offset + p * pitch + c of buf (pitch >= the view's channels; int8).  A graph
 * runtime uses views to let producers write, and consumers read, the channel
 * ranges of a concat's output in place (the concat and channel-split copies
 * vanish; the values are the same). */
typedef struct dw_view {
    dw_buf *buf;
    size_t offset;  /* bytes; a multiple of 16 */
    int32_t pitch;  /* bytes from one pixel to the next; a multiple of 16 */
} dw_view;

/* dw_conv2d_i8 with the input and output as views (tensor-core path only:
 * DW_ERR_UNSUPPORTED where it does not apply, or for an input view of a conv
 * with stride_w > 1 whose pitch differs from c_in). */
DW_API dw_status dw_conv2d_i8_view(dw_backend *be, const dw_conv_desc *d, const dw_view *x, const dw_buf *w_prep,
                                   const dw_buf *bias, const dw_buf *M, const dw_buf *D, const dw_view *y);
/* Conv -> Add fused: y = add_i8(residual, conv(x)), the int8 add of the
 * reference (crates/dragonwing-cpu/src/ops.rs:3197-3209: y = round(clamp(
 * residual * ra + conv * rb))) applied to the fused conv's int8 result in its
 * epilogue, with all three tensors as views (tensor-core path only; ratios
 * below 1e30 in magnitude).  Bit-identical with dw_conv2d_i8 followed by
 * dw_add_i8; the conv's own output never reaches memory.  y may be the
 * residual view itself: each tile's residual is read before its output is
 * stored, and tiles do not overlap. */
DW_API dw_status dw_conv2d_add_i8_view(dw_backend *be, const dw_conv_desc *d, const dw_view *x, const dw_buf *w_prep,
                                       const dw_buf *bias, const dw_buf *M, const dw_buf *D, const dw_view *residual,
                                       float ra, float rb, const dw_view *y);
/* dw_add_i8 over `pixels` pixels of `c` channels (c a multiple of 16) given as views. */
DW_API dw_status dw_add_i8_view(dw_backend *be, const dw_view *a, const dw_view *b, const dw_view *out, size_t pixels,
                                size_t c, float scale_a_over_y, float scale_b_over_y);
/* dw_maxpool_i8 with the input and output as views (c a multiple of 16). */
DW_API dw_status dw_maxpool_i8_view(dw_backend *be, const dw_view *x, const dw_view *y, size_t n, size_t h, size_t w,
                                    size_t c, size_t k_h, size_t k_w, size_t s_h, size_t s_w, size_t p_t, size_t p_l,
                                    size_t p_b, size_t p_r);
/* `count` (1..4) chained maxpools of x, each k x k (k odd), stride 1, padding
 * k/2 on every side with the padded taps skipped (maxpool2d_f32_nhwc,
 * crates/dragonwing-cpu/src/ops.rs:1513-1551, as YOLOv8's SPPF block runs it
 * three times in a row): ys[0] = pool(x), ys[i] = pool(ys[i-1]), all [n, h, w,
 * c] views (c a multiple of 16).  Identical to `count` dw_maxpool_i8_view
 * calls; x is read once. */
DW_API dw_status dw_maxpool_chain_i8_view(dw_backend *be, const dw_view *x, const dw_view *ys, int32_t count, size_t n,
                                          size_t h, size_t w, size_t c, size_t k);

/* ---------------------------------------------------------------------- */
/* YOLOv8 Detect head tail and detection post-processing                   */
/* ---------------------------------------------------------------------- */

#define DW_YOLO_MAX_LEVELS 4

/* The Detect head of an exported YOLOv8 model after its last box and class
 * convolutions.  Level l has a box tensor int8 NHWC [n, h[l], w[l], 4*reg_max]
 * (dequantisation scale box_scale[l]) and a class tensor int8 NHWC
 * [n, h[l], w[l], num_classes] (cls_scale[l]); stride[l] = input pixels per
 * grid cell.  reg_max must be 16. */
typedef struct dw_yolo_detect_desc {
    int32_t n, num_classes, reg_max, num_levels;
    int32_t h[DW_YOLO_MAX_LEVELS], w[DW_YOLO_MAX_LEVELS];
    float stride[DW_YOLO_MAX_LEVELS], box_scale[DW_YOLO_MAX_LEVELS], cls_scale[DW_YOLO_MAX_LEVELS];
} dw_yolo_detect_desc;

/* Builds the tables dw_yolo_detect_i8 reads (once per model: per level, the
 * 256 sigmoid values of the class levels and the 256 x 256 softmax terms
 * exp(x_i - max) of the box levels, from the host's libm expf, the function
 * the reference's f32::exp calls).  *tables is a new buffer owned by the caller. */
DW_API dw_status dw_prepare_yolo_detect(dw_backend *be, const dw_yolo_detect_desc *d, dw_buf **tables);

/* The tail the reference runs as f32 graph ops after DequantizeLinear
 * (Softmax ops.rs:1609-1640, the DFL Conv ops.rs:1356-1420, Sub/Add/Div/Mul
 * runtime.rs:1674-1850, Sigmoid ops.rs:1865-1870, Concat), fused:
 * out f32 [n, 4 + num_classes, A], A = sum h[l]*w[l] anchors, level by level,
 * row-major in each level.  Rows 0-3: box centre x, y, width, height in input
 * pixels (DFL expectation over 16 bins per side, distances around the cell
 * centre, times the stride); rows 4..: sigmoid class scores.  box[l], cls[l]
 * are arrays of num_levels buffers.  Bit-identical with the reference's ops. */
DW_API dw_status dw_yolo_detect_i8(dw_backend *be, const dw_yolo_detect_desc *d, const dw_buf *tables,
                                   const dw_buf *const *box, const dw_buf *const *cls, dw_buf *out_f32);

/* One detection, the layout of postprocess.rs:12-19 (24 bytes). */
typedef struct dw_detection {
    float bbox[4]; /* x1, y1, x2, y2 in image pixels */
    uint32_t class_id;
    float confidence;
} dw_detection;

enum dw_yolo_flags {
    DW_YOLO_ANCHOR_ROWS = 1,  /* raw is [n, A, 4 + nc] (decode_detections_v8_alt, postprocess.rs:151) */
    DW_YOLO_NMS_AGNOSTIC = 2, /* nms_agnostic (postprocess.rs:270) instead of nms */
    DW_YOLO_NO_NMS = 4        /* decode_detections_v8 alone: candidates in anchor order */
};

/* Device bytes of the workspace dw_postprocess_yolo needs for n images of
 * num_detections anchors. */
DW_API size_t dw_postprocess_yolo_workspace(size_t n, size_t num_detections);

/* postprocess_yolo (crates/dragonwing-onnx/src/postprocess.rs:319-340) for each
 * of n images: decode_detections_v8 (:78-146; model size 640, best class by
 * strict '>' from 0, skipped when best < conf_threshold, corners scaled and
 * clamped) then nms (:227-265: stable sort by confidence, greedy same-class
 * suppression when IoU > iou_threshold, then the swap_remove deletion, whose
 * output order is reproduced).  raw: f32 [n, 4 + num_classes, num_detections]
 * on the device (the model output).  dets: dw_detection [n, num_detections];
 * image i's detections are dets[i*num_detections .. + counts[i]), the records
 * after them are zero.  counts:
 * int32 [n] (raw and dets may be NULL when num_detections is 0).  workspace: at least
 * dw_postprocess_yolo_workspace bytes, or NULL to use the backend's scratch
 * (which may grow, so pass one when capturing a CUDA graph).
 * num_detections <= 16384. */
DW_API dw_status dw_postprocess_yolo(dw_backend *be, const dw_buf *raw, size_t n, size_t num_classes,
                                     size_t num_detections, uint32_t img_width, uint32_t img_height,
                                     float conf_threshold, float iou_threshold, int32_t flags, dw_buf *workspace,
                                     dw_buf *dets, dw_buf *counts);

/* ---------------------------------------------------------------------- */
/* FP16 path (binary16 buffers, f32 accumulation)                           */
/* ---------------------------------------------------------------------- */
/* Conversions follow F16::from_f32 / F16::to_f32 (crates/dragonwing-core/src/
 * dtype.rs:164-263) exactly, including to_f32's halving of subnormal halves,
 * so the elementwise, pooling, depthwise and direct-conv ops are bit-identical
 * with the CPU ops; the tensor-core conv/GEMM sums in a different order and
 * meets a stated tolerance instead. */

/* Repacks an fp16 conv kernel: HWIO [kh,kw,c_in,c_out] -> the kernel layout
 * (group == 1), or copies a depthwise kernel [kh,kw,C,mult]. */
DW_API dw_status dw_prepare_weights_f16(dw_backend *be, const dw_conv_desc *d, const dw_buf *w_hwio,
                                        dw_buf **out);
/* Conv2D in fp16, NHWC: f32 accumulation, result stored as f16, then the f16
 * bias[c_out] (may be NULL) added as the CPU runtime adds it (runtime.rs:
 * 1483-1497: stored f16 + bias, rounded again), then ReLU when
 * d->epilogue == DW_EPI_RELU (DW_EPI_NONE otherwise).  d->group: 1, or c_in
 * (depthwise).  Tensor-core path: c_in % 8 == 0 (% 16 when strided), c_out % 8
 * == 0; other shapes run the direct kernel unless the path is DW_PATH_UMMA. */
DW_API dw_status dw_conv2d_f16(dw_backend *be, const dw_conv_desc *d, const dw_buf *x, const dw_buf *w_prep,
                               const dw_buf *bias_or_null, dw_buf *y);
/* dw_conv2d_f16 followed by the residual add of a bottleneck block, fused:
 * y = relu?(from_f32(to_f32(conv_bias) + to_f32(residual))), i.e. the CPU
 * runtime's Conv -> Add (add_fp16, cpu ops.rs:434-446) -> Relu sequence with
 * the ReLU (d->epilogue == DW_EPI_RELU) applied after the add.  residual has
 * y's shape and must not alias it.  The tensor-core kernel fuses the add into
 * its epilogue for 1x1 stride-1 convs; other shapes add in a second pass. */
DW_API dw_status dw_conv2d_add_f16(dw_backend *be, const dw_conv_desc *d, const dw_buf *x, const dw_buf *w_prep,
                                   const dw_buf *bias_or_null, const dw_buf *residual, dw_buf *y);
/* conv2d_fp16_nhwc (crates/dragonwing-vulkan/src/ops.rs:1385-1420): the
 * reference's parameter list, HWIO kernel, symmetric pads, no bias. */
DW_API dw_status dw_conv2d_fp16_nhwc(dw_backend *be, const dw_buf *input, const dw_buf *kernel_hwio,
                                     dw_buf *output, size_t n, size_t h_in, size_t w_in, size_t c_in,
                                     size_t c_out, size_t k_h, size_t k_w, size_t stride_h, size_t stride_w,
                                     size_t pad_h, size_t pad_w);
/* gemm_fp16 (vulkan ops.rs:1184-1215, cpu ops.rs:461-481): C[m,n] = A[m,k] *
 * B[k,n], row-major f16, f32 accumulation. */
DW_API dw_status dw_gemm_f16(dw_backend *be, const dw_buf *a, const dw_buf *b, dw_buf *c, size_t m, size_t n,
                             size_t k);
/* Repacks B [k,n] row-major (an fp16 Gemm weight) once into the kernel layout. */
DW_API dw_status dw_prepare_gemm_b_f16(dw_backend *be, const dw_buf *b_kn, size_t k, size_t n, dw_buf **out);
/* Gemm F16 with bias as the CPU runtime runs it (runtime.rs:1247-1275): f16
 * product, then + bias[n] (may be NULL) rounded again, then ReLU if `relu`. */
DW_API dw_status dw_gemm_f16_bias(dw_backend *be, const dw_buf *a, const dw_buf *b_prep, const dw_buf *bias,
                                  dw_buf *y, size_t m, size_t n, size_t k, int relu);
/* add_fp16 (vulkan ops.rs:933-960, cpu ops.rs:434-446): y = a + b. */
DW_API dw_status dw_add_f16(dw_backend *be, const dw_buf *a, const dw_buf *b, dw_buf *y);
/* add_fp16 followed by relu_fp16 in one pass (the Add -> Relu of a residual). */
DW_API dw_status dw_add_relu_f16(dw_backend *be, const dw_buf *a, const dw_buf *b, dw_buf *y);
/* relu_fp16 (vulkan ops.rs:856, in place; cpu ops.rs:345-352). */
DW_API dw_status dw_relu_f16(dw_backend *be, dw_buf *x);
/* F16 MaxPool (runtime.rs:1545-1563) on NHWC, pads [t,l,b,r] taken as -inf. */
DW_API dw_status dw_maxpool_f16(dw_backend *be, const dw_buf *x, dw_buf *y, size_t n, size_t h, size_t w,
                                size_t c, size_t k_h, size_t k_w, size_t s_h, size_t s_w, size_t p_t,
                                size_t p_l, size_t p_b, size_t p_r);
/* F16 GlobalAveragePool (runtime.rs:1155-1170): NHWC -> [n, c]. */
DW_API dw_status dw_global_avgpool_f16(dw_backend *be, const dw_buf *x, dw_buf *y, size_t n, size_t h,
                                       size_t w, size_t c);
/* f32 [pixels, c_src] -> f16 [pixels, c_dst] with F16::from_f32 (the runtime's
 * F16 input conversion, runtime.rs:842-851); channels c_src..c_dst-1 are 0. */
DW_API dw_status dw_cast_f32_to_f16(dw_backend *be, const dw_buf *x_f32, dw_buf *y_f16, size_t pixels,
                                    size_t c_src, size_t c_dst);
/* Horizontal unfold fused with the F16 input conversion, for the first conv
 * of a network on a few-channel image: y[n][r][j][q*c + ch] =
 * from_f32(x[n][r][j*stride_w + q - pad_l][ch]) for q < k_w (0 outside the
 * image), channels k_w*c .. c_dst-1 zero; y is [n, h, w_out, c_dst] f16.  A
 * k_h x k_w conv with stride (s_h, stride_w) and pads (t, pad_l, b, r) on x
 * equals a k_h x 1 conv with stride (s_h, 1), pads (t, 0, b, 0) on y whose
 * kernel [kh][0][q*c + ch][oc] = original [kh][q][ch][oc] (zero rows for the
 * padding channels): the same products, fed to the tensor cores in rows of
 * k_w*c channels. */
DW_API dw_status dw_unfold_w_f32_to_f16(dw_backend *be, const dw_buf *x_f32, dw_buf *y_f16, size_t n, size_t h,
                                        size_t w, size_t c, size_t k_w, size_t stride_w, size_t pad_l, size_t w_out,
                                        size_t c_dst);
/* f16 -> f32 with F16::to_f32. */
DW_API dw_status dw_cast_f16_to_f32(dw_backend *be, const dw_buf *x_f16, dw_buf *y_f32);

#ifdef __cplusplus
}
#endif
#endif /* DW_CUDA_H */
