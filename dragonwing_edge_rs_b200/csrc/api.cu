// api.cu -- the C ABI (include/dw_cuda.h): backend lifecycle, buffers, copies,
// synchronization, and the op entry points with the reference's shape checks.
//
// Backend trait: crates/dragonwing-core/src/backend.rs:127-199.
// Op signatures and error strings: crates/dragonwing-vulkan/src/ops.rs.

#include <chrono>
#include <cstdlib>
#include <cstring>
#include <thread>
#include <vector>

#include "dw_internal.h"

#define DW_VERSION_STRING "dragonwing-cuda 0.1 (sm_100a)"

// ---------------------------------------------------------------------------
// error plumbing
// ---------------------------------------------------------------------------

dw_status dw_fail(dw_backend *be, dw_status st, const char *fmt, ...) {
    char buf[512];
    va_list ap;
    va_start(ap, fmt);
    vsnprintf(buf, sizeof buf, fmt, ap);
    va_end(ap);
    if (be) be->last_error = buf;
    return st;
}

dw_status dw_cuda_check(dw_backend *be, cudaError_t e, const char *what) {
    if (e == cudaSuccess) return DW_OK;
    if (e == cudaErrorMemoryAllocation) {
        cudaGetLastError();
        return dw_fail(be, DW_ERR_OOM, "%s: %s", what, cudaGetErrorString(e));
    }
    return dw_fail(be, DW_ERR_DEVICE, "%s: %s", what, cudaGetErrorString(e));
}

dw_status dw_after_launch(dw_backend *be, const char *what) {
    be->launches++;
    dw_status st = dw_cuda_check(be, cudaGetLastError(), what);
    if (st != DW_OK) return st;
    if (be->cfg.trace) {
        st = dw_synchronize(be, be->cfg.wait_cap_ms ? be->cfg.wait_cap_ms * 4 : 10000);
        fprintf(stderr, "[dw trace] %s -> %d\n", what, (int)st);
    }
    return st;
}

dw_status dw_scratch(dw_backend *be, size_t len, void **out) {
    if (be->scratch_len < len) {
        if (be->scratch) {
            cudaStreamSynchronize(be->stream);
            cudaFree(be->scratch);
            be->scratch = nullptr;
            be->scratch_len = 0;
        }
        dw_status st = dw_cuda_check(be, cudaMalloc(&be->scratch, len), "scratch alloc");
        if (st != DW_OK) return st;
        be->scratch_len = len;
    }
    *out = be->scratch;
    return DW_OK;
}

static int env_int(const char *name, int dflt) {
    const char *v = getenv(name);
    return (v && *v) ? atoi(v) : dflt;
}

// ---------------------------------------------------------------------------
// Backend trait
// ---------------------------------------------------------------------------

extern "C" {

DW_API const char *dw_name(void) { return "cuda-sm100a"; }
DW_API const char *dw_version(void) { return DW_VERSION_STRING; }

DW_API dw_status dw_create(int device_ordinal, const dw_config *cfg, dw_backend **out) {
    if (!out) return DW_ERR_INVALID_ARG;
    *out = nullptr;
    int ndev = 0;
    cudaError_t e = cudaGetDeviceCount(&ndev);
    if (e != cudaSuccess || ndev == 0) return DW_ERR_DEVICE;
    if (device_ordinal < 0 || device_ordinal >= ndev) return DW_ERR_INVALID_ARG;
    auto *be = new dw_backend();
    be->device = device_ordinal;
    if (cfg) be->cfg = *cfg;
    be->cfg.wait_cap_ms = (uint32_t)env_int("DW_WAIT_CAP_MS", be->cfg.wait_cap_ms ? (int)be->cfg.wait_cap_ms : 2000);
    be->cfg.trace = env_int("DW_TRACE", be->cfg.trace);
    be->cfg.conv_path = env_int("DW_CONV_PATH", be->cfg.conv_path);
    be->cfg.dw_variant = env_int("DW_DW_VARIANT", be->cfg.dw_variant);
    be->wait_cap_ns = (uint64_t)be->cfg.wait_cap_ms * 1000000ull;
    if (cudaSetDevice(device_ordinal) != cudaSuccess) { delete be; return DW_ERR_DEVICE; }
    cudaDeviceProp prop;
    if (cudaGetDeviceProperties(&prop, device_ordinal) != cudaSuccess) { delete be; return DW_ERR_DEVICE; }
    if (prop.major != 10) {  // the kernels are built for sm_100a only
        delete be;
        return DW_ERR_UNSUPPORTED;
    }
    be->sm_count = prop.multiProcessorCount;
    if (cudaStreamCreateWithFlags(&be->stream, cudaStreamNonBlocking) != cudaSuccess) { delete be; return DW_ERR_DEVICE; }
    if (cudaMalloc(&be->dev_err, sizeof(int32_t) * kDevErrWords) != cudaSuccess) {
        cudaStreamDestroy(be->stream);
        delete be;
        return DW_ERR_OOM;
    }
    cudaMemset(be->dev_err, 0, sizeof(int32_t) * kDevErrWords);
    // cuTensorMapEncodeTiled through the runtime's driver entry point (no -lcuda).
    void *fn = nullptr;
    cudaDriverEntryPointQueryResult qres;
    if (cudaGetDriverEntryPoint("cuTensorMapEncodeTiled", &fn, cudaEnableDefault, &qres) == cudaSuccess &&
        qres == cudaDriverEntryPointSuccess)
        be->encode_tiled = reinterpret_cast<PFN_encodeTiled>(fn);
    cudaDeviceSynchronize();
    *out = be;
    return DW_OK;
}

DW_API void dw_destroy(dw_backend *be) {
    if (!be) return;
    cudaSetDevice(be->device);
    if (be->stream) cudaStreamSynchronize(be->stream);
    if (be->scratch) cudaFree(be->scratch);
    if (be->dev_err) cudaFree(be->dev_err);
    if (be->stream) cudaStreamDestroy(be->stream);
    delete be;
}

DW_API const char *dw_last_error(const dw_backend *be) { return be ? be->last_error.c_str() : "null backend"; }

DW_API dw_status dw_alloc(dw_backend *be, size_t len_bytes, dw_buf **out) {
    if (!be || !out) return DW_ERR_INVALID_ARG;
    *out = nullptr;
    if (len_bytes == 0) return dw_fail(be, DW_ERR_INVALID_ARG, "alloc: zero-length buffer");
    cudaSetDevice(be->device);
    void *p = nullptr;
    dw_status st = dw_cuda_check(be, cudaMalloc(&p, len_bytes), "alloc");
    if (st != DW_OK) return st;
    auto *b = new dw_buf();
    b->ptr = p;
    b->len = len_bytes;
    b->owned = true;
    *out = b;
    return DW_OK;
}

DW_API dw_status dw_buf_wrap(dw_backend *be, void *device_ptr, size_t len_bytes, dw_buf **out) {
    if (!be || !out || !device_ptr) return DW_ERR_INVALID_ARG;
    if (len_bytes == 0) return dw_fail(be, DW_ERR_INVALID_ARG, "wrap: zero-length buffer");
    auto *b = new dw_buf();
    b->ptr = device_ptr;
    b->len = len_bytes;
    b->owned = false;
    *out = b;
    return DW_OK;
}

DW_API dw_status dw_free(dw_backend *be, dw_buf *buf) {
    if (!buf) return DW_OK;
    dw_status st = DW_OK;
    if (buf->owned && buf->ptr) {
        if (be) cudaSetDevice(be->device);
        cudaError_t e = cudaFree(buf->ptr);
        if (e != cudaSuccess) st = dw_cuda_check(be, e, "free");
    }
    delete buf;
    return st;
}

DW_API size_t dw_buf_len(const dw_buf *buf) { return buf ? buf->len : 0; }
DW_API void *dw_buf_device_ptr(const dw_buf *buf) { return buf ? buf->ptr : nullptr; }

DW_API dw_status dw_upload(dw_backend *be, dw_buf *dst, const void *src, size_t src_len) {
    if (!be || !dst || (!src && src_len)) return DW_ERR_INVALID_ARG;
    if (src_len != dst->len)
        return dw_fail(be, DW_ERR_SIZE_MISMATCH, "upload: length mismatch: buffer %zu bytes, source %zu bytes",
                       dst->len, src_len);
    cudaSetDevice(be->device);
    dw_status st = dw_cuda_check(be, cudaMemcpyAsync(dst->ptr, src, src_len, cudaMemcpyHostToDevice, be->stream),
                                 "upload");
    if (st != DW_OK) return st;
    return dw_cuda_check(be, cudaStreamSynchronize(be->stream), "upload sync");
}

DW_API dw_status dw_download(dw_backend *be, const dw_buf *src, void *dst, size_t dst_len) {
    if (!be || !src || (!dst && dst_len)) return DW_ERR_INVALID_ARG;
    if (dst_len != src->len)
        return dw_fail(be, DW_ERR_SIZE_MISMATCH, "download: length mismatch: buffer %zu bytes, destination %zu bytes",
                       src->len, dst_len);
    dw_status st = dw_synchronize(be, 0);
    if (st != DW_OK) return st;
    st = dw_cuda_check(be, cudaMemcpyAsync(dst, src->ptr, dst_len, cudaMemcpyDeviceToHost, be->stream), "download");
    if (st != DW_OK) return st;
    return dw_cuda_check(be, cudaStreamSynchronize(be->stream), "download sync");
}

DW_API dw_status dw_upload_async(dw_backend *be, dw_buf *dst, size_t dst_offset, const void *src, size_t len) {
    if (!be || !dst || !src) return DW_ERR_INVALID_ARG;
    if (dst_offset > dst->len || len > dst->len - dst_offset)
        return dw_fail(be, DW_ERR_SIZE_MISMATCH, "upload_async: range [%zu, +%zu) outside buffer of %zu bytes",
                       dst_offset, len, dst->len);
    return dw_cuda_check(be,
                         cudaMemcpyAsync((char *)dst->ptr + dst_offset, src, len, cudaMemcpyHostToDevice, be->stream),
                         "upload_async");
}

DW_API dw_status dw_download_async(dw_backend *be, const dw_buf *src, size_t src_offset, void *dst, size_t len) {
    if (!be || !src || !dst) return DW_ERR_INVALID_ARG;
    if (src_offset > src->len || len > src->len - src_offset)
        return dw_fail(be, DW_ERR_SIZE_MISMATCH, "download_async: range [%zu, +%zu) outside buffer of %zu bytes",
                       src_offset, len, src->len);
    return dw_cuda_check(
        be, cudaMemcpyAsync(dst, (const char *)src->ptr + src_offset, len, cudaMemcpyDeviceToHost, be->stream),
        "download_async");
}

DW_API dw_status dw_copy_async(dw_backend *be, dw_buf *dst, size_t dst_offset, const dw_buf *src, size_t src_offset,
                               size_t len) {
    if (!be || !dst || !src) return DW_ERR_INVALID_ARG;
    if (dst_offset > dst->len || len > dst->len - dst_offset || src_offset > src->len || len > src->len - src_offset)
        return dw_fail(be, DW_ERR_SIZE_MISMATCH, "copy_async: range of %zu bytes outside a buffer", len);
    return dw_cuda_check(be,
                         cudaMemcpyAsync((char *)dst->ptr + dst_offset, (const char *)src->ptr + src_offset, len,
                                         cudaMemcpyDeviceToDevice, be->stream),
                         "copy_async");
}

struct dw_event {
    cudaEvent_t ev = nullptr;
    int device = 0;
};

DW_API dw_status dw_event_create(dw_backend *be, dw_event **out) {
    if (!be || !out) return DW_ERR_INVALID_ARG;
    *out = nullptr;
    cudaSetDevice(be->device);
    cudaEvent_t ev;
    dw_status st = dw_cuda_check(be, cudaEventCreateWithFlags(&ev, cudaEventDisableTiming), "event_create");
    if (st != DW_OK) return st;
    *out = new dw_event{ev, be->device};
    return DW_OK;
}

DW_API void dw_event_destroy(dw_event *ev) {
    if (!ev) return;
    cudaSetDevice(ev->device);
    cudaEventDestroy(ev->ev);
    delete ev;
}

DW_API dw_status dw_event_record(dw_backend *be, dw_event *ev) {
    if (!be || !ev) return DW_ERR_INVALID_ARG;
    return dw_cuda_check(be, cudaEventRecord(ev->ev, be->stream), "event_record");
}

DW_API dw_status dw_stream_wait_event(dw_backend *be, dw_event *ev) {
    if (!be || !ev) return DW_ERR_INVALID_ARG;
    return dw_cuda_check(be, cudaStreamWaitEvent(be->stream, ev->ev, 0), "stream_wait_event");
}

DW_API dw_status dw_synchronize(dw_backend *be, uint32_t timeout_ms) {
    if (!be) return DW_ERR_INVALID_ARG;
    cudaSetDevice(be->device);
    cudaEvent_t ev;
    dw_status st = dw_cuda_check(be, cudaEventCreateWithFlags(&ev, cudaEventDisableTiming), "sync event");
    if (st != DW_OK) return st;
    st = dw_cuda_check(be, cudaEventRecord(ev, be->stream), "sync record");
    if (st != DW_OK) { cudaEventDestroy(ev); return st; }
    auto t0 = std::chrono::steady_clock::now();
    for (;;) {
        cudaError_t q = cudaEventQuery(ev);
        if (q == cudaSuccess) break;
        if (q != cudaErrorNotReady) {
            cudaEventDestroy(ev);
            return dw_cuda_check(be, q, "synchronize");
        }
        if (timeout_ms) {
            auto ms = std::chrono::duration_cast<std::chrono::milliseconds>(std::chrono::steady_clock::now() - t0).count();
            if (ms >= (long long)timeout_ms) {
                cudaEventDestroy(ev);
                return dw_fail(be, DW_ERR_TIMEOUT, "synchronize: queued work not finished after %u ms", timeout_ms);
            }
        }
        std::this_thread::sleep_for(std::chrono::microseconds(20));
    }
    cudaEventDestroy(ev);
    int32_t err[kDevErrWords] = {0, 0, 0, 0};
    st = dw_cuda_check(be, cudaMemcpy(err, be->dev_err, sizeof err, cudaMemcpyDeviceToHost), "read device error word");
    if (st != DW_OK) return st;
    if (err[0] != DW_DEV_OK) {
        cudaMemset(be->dev_err, 0, sizeof err);
        if (err[0] == DW_DEV_WAIT_EXPIRED)
            return dw_fail(be, DW_ERR_KERNEL_WAIT_EXPIRED,
                           "kernel wait expired (site %d, block %d, detail %d); results of the affected launch are "
                           "invalid", err[1], err[2], err[3]);
        return dw_fail(be, DW_ERR_DEVICE, "kernel reported error %d (site %d, block %d, detail %d)", err[0], err[1],
                       err[2], err[3]);
    }
    return DW_OK;
}

DW_API dw_status dw_host_alloc(dw_backend *be, size_t len_bytes, void **out) {
    if (!be || !out || !len_bytes) return DW_ERR_INVALID_ARG;
    return dw_cuda_check(be, cudaHostAlloc(out, len_bytes, cudaHostAllocPortable), "host alloc");
}

DW_API dw_status dw_host_free(dw_backend *be, void *ptr) {
    if (!ptr) return DW_OK;
    return dw_cuda_check(be, cudaFreeHost(ptr), "host free");
}

DW_API void *dw_stream(dw_backend *be) { return be ? (void *)be->stream : nullptr; }
DW_API int dw_sm_count(const dw_backend *be) { return be ? be->sm_count : 0; }
DW_API uint64_t dw_launch_count(const dw_backend *be) { return be ? be->launches : 0; }
DW_API size_t dw_scratch_bytes(const dw_backend *be) { return be ? be->scratch_len : 0; }

struct dw_graph {
    cudaGraph_t graph = nullptr;
    cudaGraphExec_t exec = nullptr;
    uint64_t kernels = 0;  // kernel launches recorded into the graph
};

DW_API dw_status dw_capture_begin(dw_backend *be) {
    if (!be) return DW_ERR_INVALID_ARG;
    cudaSetDevice(be->device);
    be->capture_mark = be->launches;
    return dw_cuda_check(be, cudaStreamBeginCapture(be->stream, cudaStreamCaptureModeThreadLocal), "capture begin");
}

DW_API dw_status dw_capture_end(dw_backend *be, dw_graph **out) {
    if (!be || !out) return DW_ERR_INVALID_ARG;
    *out = nullptr;
    auto *g = new dw_graph();
    g->kernels = be->launches - be->capture_mark;
    be->launches = be->capture_mark;  // recorded, not launched
    dw_status st = dw_cuda_check(be, cudaStreamEndCapture(be->stream, &g->graph), "capture end");
    if (st == DW_OK) st = dw_cuda_check(be, cudaGraphInstantiate(&g->exec, g->graph, 0), "graph instantiate");
    if (st != DW_OK) {
        if (g->graph) cudaGraphDestroy(g->graph);
        delete g;
        return st;
    }
    *out = g;
    return DW_OK;
}

DW_API dw_status dw_graph_launch(dw_backend *be, dw_graph *g) {
    if (!be || !g) return DW_ERR_INVALID_ARG;
    be->launches += g->kernels;
    return dw_cuda_check(be, cudaGraphLaunch(g->exec, be->stream), "graph launch");
}

DW_API void dw_graph_destroy(dw_graph *g) {
    if (!g) return;
    if (g->exec) cudaGraphExecDestroy(g->exec);
    if (g->graph) cudaGraphDestroy(g->graph);
    delete g;
}

DW_API dw_status dw_debug_expire_wait(dw_backend *be, uint32_t cap_us) {
    if (!be) return DW_ERR_INVALID_ARG;
    cudaSetDevice(be->device);
    return dw::launch_expire_wait(be, (uint64_t)cap_us * 1000ull);
}

}  // extern "C"
