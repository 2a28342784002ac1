// dw_device.cuh -- device helpers shared by all kernels: the bit-exact
// requantisation epilogue, bounded waits and the device error record.
#pragma once

#include <cstdint>

#include "dw_expf.h"
#include "dw_internal.h"

namespace dw {

// `v.clamp(-128.0, 127.0).round() as i8` (crates/dragonwing-cpu/src/ops.rs:3383-3385):
// clamp in f32, roundf (half away from zero), saturating cast (NaN -> 0).
__device__ __forceinline__ int32_t f32_to_i8(float v) {
    if (v != v) return 0;
    v = fminf(fmaxf(v, -128.0f), 127.0f);
    return (int32_t)roundf(v);
}

// The fused epilogue for one accumulator (contract in include/dw_cuda.h):
// every float operation is a separately rounded IEEE op, as in the reference
// (Rust does not contract a*b+c), so the result is bit-exact.
__device__ __forceinline__ int32_t epilogue_one(int32_t acc, int32_t bias, float m, float dsc, int epi, int q6,
                                                float inv_s_out) {
    const int32_t a = (int32_t)((uint32_t)acc + (uint32_t)bias);
    if (epi == DW_EPI_SILU) {
        const float y = __fmul_rn(__int2float_rn(a), dsc);
        const float z = dw_silu_f32(y);
        return f32_to_i8(__fmul_rn(z, inv_s_out));
    }
    int32_t q = f32_to_i8(__fmul_rn(__int2float_rn(a), m));
    if (epi == DW_EPI_RELU) q = q > 0 ? q : 0;
    else if (epi == DW_EPI_RELU6) q = min(q > 0 ? q : 0, q6);
    return q;
}

__device__ __forceinline__ uint64_t globaltimer_ns() {
    uint64_t t;
    asm volatile("mov.u64 %0, %%globaltimer;" : "=l"(t));
    return t;
}

// Records a device-side failure (first writer wins) without trapping.
__device__ __forceinline__ void record_error(int32_t *err, int32_t code, int32_t site, int32_t detail) {
    if (atomicCAS(err, 0, code) == 0) {
        err[1] = site;
        err[2] = (int32_t)(blockIdx.x + gridDim.x * (blockIdx.y + gridDim.y * blockIdx.z));
        err[3] = detail;
        __threadfence();
    }
}

}  // namespace dw
