// noalloc.cu -- dw_conv2d_requant_relu_i8_noalloc: the fused int8 conv with the
// reference's parameter list, for callers that must not allocate device memory
// per call.
//
// dw_conv2d_requant_relu_i8 needs two temporaries per call: the weights
// repacked from HWIO to the kernels' OHWI layout, and the per-channel requant
// scale array filled with the scalar scale.  It takes them from the backend's
// growable scratch, which calls cudaMalloc/cudaFree when it grows.  Some
// callers cannot allow that: applications that reserve all device memory up
// front and run a fixed plan (the reference's own Vulkan runtime carves every
// buffer out of one slab allocation, crates/dragonwing-vulkan/src/slab.rs), and
// latency-critical inference loops where an allocator call, which may
// synchronize the device and take unbounded time, is not permitted after
// start-up.  This entry point keeps those temporaries in one fixed device array
// that lives in the library instead, and calls no allocator.
//
// The array (kNoAllocBytes) is a file-scope __device__ variable: every GPU that
// loads this library holds it until the process exits.  Host code cannot use the
// variable's name as a device address (on the host it names a stand-in), so the
// address is looked up with cudaGetSymbolAddress, with the device current, and
// cached per device together with the unique ID of the CUDA context it belongs
// to.  A later call in another context of that device (after cudaDeviceReset, or
// a reset of the primary context) sees a different ID and looks the address up
// again, so no stale address is ever used.  The first call on a device (and the
// first after such a reset) does that look-up: make it before any stream capture
// begins on the device.  All calls on a device share the array and every call
// fully rewrites the part it uses (no state carries over); calls whose kernels
// overlap on the GPU (different streams or backends on one device) race on it
// and must be serialised by the caller.

#include <mutex>

#include "dw_internal.h"

namespace {

constexpr size_t kNoAllocWeightBytes = 1u << 20;  // prepared int8 weights: k_h*k_w*c_in*c_out <= 1 MiB
constexpr size_t kNoAllocMaxChannels = 4096;      // requant-scale slots: c_out <= 4096
constexpr size_t kNoAllocBytes = kNoAllocWeightBytes + kNoAllocMaxChannels * sizeof(float);
constexpr int kMaxDevices = 64;

static __device__ __align__(256) unsigned char dw_noalloc_scratch[kNoAllocBytes];

using PFN_ctxGetCurrent = CUresult (*)(CUcontext *);
using PFN_ctxGetId = CUresult (*)(CUcontext, unsigned long long *);

struct CachedAddress {
    unsigned long long ctx_id = 0;  // unique ID of the context the address belongs to (0: none yet)
    void *addr = nullptr;
};

std::mutex g_addr_mu;
CachedAddress g_addr[kMaxDevices];
PFN_ctxGetCurrent g_ctx_get_current = nullptr;
PFN_ctxGetId g_ctx_get_id = nullptr;

dw_status driver_fn(dw_backend *be, const char *name, void **fn) {
    cudaDriverEntryPointQueryResult q;
    if (cudaGetDriverEntryPoint(name, fn, cudaEnableDefault, &q) != cudaSuccess || q != cudaDriverEntryPointSuccess ||
        !*fn)
        return dw_fail(be, DW_ERR_UNSUPPORTED, "conv_fused_noalloc: driver entry point %s unavailable", name);
    return DW_OK;
}

// Device address of dw_noalloc_scratch in the context now current on the
// backend's device (looked up again whenever that context changes).
dw_status scratch_address(dw_backend *be, void **out) {
    if (be->device < 0 || be->device >= kMaxDevices)
        return dw_fail(be, DW_ERR_UNSUPPORTED, "conv_fused_noalloc: device ordinal %d out of range", be->device);
    std::lock_guard<std::mutex> lock(g_addr_mu);
    dw_status st = dw_cuda_check(be, cudaSetDevice(be->device), "conv_fused_noalloc: set device");
    if (st != DW_OK) return st;
    if (!g_ctx_get_current) {
        void *f = nullptr;
        if ((st = driver_fn(be, "cuCtxGetCurrent", &f)) != DW_OK) return st;
        g_ctx_get_current = reinterpret_cast<PFN_ctxGetCurrent>(f);
    }
    if (!g_ctx_get_id) {
        void *f = nullptr;
        if ((st = driver_fn(be, "cuCtxGetId", &f)) != DW_OK) return st;
        g_ctx_get_id = reinterpret_cast<PFN_ctxGetId>(f);
    }
    CUcontext ctx = nullptr;
    unsigned long long id = 0;
    if (g_ctx_get_current(&ctx) != CUDA_SUCCESS || !ctx || g_ctx_get_id(ctx, &id) != CUDA_SUCCESS || id == 0)
        return dw_fail(be, DW_ERR_DEVICE, "conv_fused_noalloc: no current CUDA context on device %d", be->device);
    CachedAddress &c = g_addr[be->device];
    if (c.ctx_id != id || !c.addr) {
        void *p = nullptr;
        st = dw_cuda_check(be, cudaGetSymbolAddress(&p, dw_noalloc_scratch),
                           "conv_fused_noalloc: cudaGetSymbolAddress(dw_noalloc_scratch)");
        if (st != DW_OK) return st;
        c.ctx_id = id;
        c.addr = p;
    }
    *out = c.addr;
    return DW_OK;
}

__global__ void k_fill_scale(float *dst, int n, float v) {
    for (int i = blockIdx.x * blockDim.x + threadIdx.x; i < n; i += gridDim.x * blockDim.x) dst[i] = v;
}

}  // namespace

extern "C" DW_API dw_status dw_conv2d_requant_relu_i8_noalloc(dw_backend *be, const dw_buf *input,
                                                              const dw_buf *kernel_hwio, dw_buf *output, size_t n,
                                                              size_t h_in, size_t w_in, size_t c_in, size_t c_out,
                                                              size_t k_h, size_t k_w, size_t stride_h,
                                                              size_t stride_w, size_t pad_h, size_t pad_w,
                                                              float requant_scale, int do_relu) {
    if (!be) return DW_ERR_INVALID_ARG;
    if (!input || !kernel_hwio || !output) return dw_fail(be, DW_ERR_INVALID_ARG, "conv_fused: null buffer");
    // Same checks and messages as dw_conv2d_requant_relu_i8 (vulkan/src/ops.rs:2313-2345).
    if (c_in % 4 != 0) return dw_fail(be, DW_ERR_INVALID_ARG, "conv_fused: c_in=%zu must be multiple of 4", c_in);
    if (c_out % 4 != 0)
        return dw_fail(be, DW_ERR_INVALID_ARG, "conv_fused: c_out=%zu must be multiple of 4 (output is packed)", c_out);
    if (stride_h == 0 || stride_w == 0 || h_in + 2 * pad_h < k_h || w_in + 2 * pad_w < k_w || n == 0 || k_h == 0 ||
        k_w == 0)
        return dw_fail(be, DW_ERR_INVALID_ARG, "conv_fused: invalid geometry");
    const size_t h_out = (h_in + 2 * pad_h - k_h) / stride_h + 1;
    const size_t w_out = (w_in + 2 * pad_w - k_w) / stride_w + 1;
    const size_t expected_input = n * h_in * w_in * c_in;
    const size_t expected_kernel = k_h * k_w * c_in * c_out;
    const size_t expected_output = n * h_out * w_out * c_out;
    if (input->len != expected_input)
        return dw_fail(be, DW_ERR_SIZE_MISMATCH, "conv_fused: input mismatch: expected %zu, got %zu", expected_input,
                       input->len);
    if (kernel_hwio->len != expected_kernel)
        return dw_fail(be, DW_ERR_SIZE_MISMATCH, "conv_fused: kernel mismatch: expected %zu, got %zu",
                       expected_kernel, kernel_hwio->len);
    if (output->len != expected_output)
        return dw_fail(be, DW_ERR_SIZE_MISMATCH, "conv_fused: output mismatch: expected %zu, got %zu",
                       expected_output, output->len);
    // The fixed scratch bounds what this entry point accepts.
    if (expected_kernel > kNoAllocWeightBytes || c_out > kNoAllocMaxChannels)
        return dw_fail(be, DW_ERR_INVALID_ARG,
                       "conv_fused_noalloc: kernel of %zu bytes and %zu output channels exceeds the fixed scratch "
                       "(at most %zu bytes of weights and %zu output channels); use dw_conv2d_requant_relu_i8",
                       expected_kernel, c_out, kNoAllocWeightBytes, kNoAllocMaxChannels);
    // Every size the descriptor narrows to int32 (the allocating entry point's
    // descriptor holds the same fields).
    for (size_t v : {n, h_in, w_in, c_in, c_out, k_h, k_w, stride_h, stride_w, pad_h, pad_w})
        if (v > 0x7fffffff) return dw_fail(be, DW_ERR_INVALID_ARG, "conv_fused_noalloc: dimension exceeds int32");
    dw_conv_desc d{};
    d.n = (int32_t)n; d.h = (int32_t)h_in; d.w = (int32_t)w_in; d.c_in = (int32_t)c_in; d.c_out = (int32_t)c_out;
    d.k_h = (int32_t)k_h; d.k_w = (int32_t)k_w; d.stride_h = (int32_t)stride_h; d.stride_w = (int32_t)stride_w;
    d.pad_t = d.pad_b = (int32_t)pad_h; d.pad_l = d.pad_r = (int32_t)pad_w;
    d.group = 1;
    d.epilogue = do_relu ? DW_EPI_RELU : DW_EPI_NONE;
    d.q6 = 127;
    // The allocating entry point's descriptor checks (zero channels included), same messages.
    int ho_chk = 0, wo_chk = 0;
    dw_status st = dw_check_conv_desc(be, &d, &ho_chk, &wo_chk, "conv_fused");
    if (st != DW_OK) return st;
    const int ho = (int)h_out, wo = (int)w_out;

    void *base = nullptr;
    st = scratch_address(be, &base);
    if (st != DW_OK) return st;
    st = dw_cuda_check(be, cudaSetDevice(be->device), "conv_fused_noalloc: set device");
    if (st != DW_OK) return st;
    int8_t *w_prep = static_cast<int8_t *>(base);
    float *scales = reinterpret_cast<float *>(static_cast<unsigned char *>(base) + kNoAllocWeightBytes);
    // Every byte and scale slot the conv reads is rewritten here, by kernels on the
    // backend stream, ahead of the conv itself.
    st = dw::launch_repack_hwio_to_ohwi(be, (const int8_t *)kernel_hwio->ptr, w_prep, (int)(k_h * k_w), (int)c_in,
                                        (int)c_out);
    if (st != DW_OK) return st;
    k_fill_scale<<<(unsigned)((c_out + 255) / 256), 256, 0, be->stream>>>(scales, (int)c_out, requant_scale);
    st = dw_after_launch(be, "conv_fused_noalloc: fill scales");
    if (st != DW_OK) return st;
    dw::EpiParams ep{nullptr, scales, nullptr, d.epilogue, 127, 0.0f};
    const int8_t *xp = (const int8_t *)input->ptr;
    int8_t *yp = (int8_t *)output->ptr;
    if (be->cfg.conv_path != DW_PATH_DIRECT && dw::umma_supported(be, d, ho, wo))
        return dw::launch_umma_conv_i8(be, d, ho, wo, xp, w_prep, ep, yp);
    if (be->cfg.conv_path == DW_PATH_UMMA)
        return dw_fail(be, DW_ERR_UNSUPPORTED, "conv_fused_noalloc: shape not supported by the tensor-core kernel");
    return dw::launch_conv_direct_i8(be, d, ho, wo, xp, w_prep, ep, yp, nullptr);
}
