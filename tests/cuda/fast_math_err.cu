// Test program: the largest relative errors of ex2.approx.ftz.f32 and
// rcp.approx.ftz.f32 over every input the SiLU fast path can give them (all
// floats of each range), against double-precision references.  The certified
// SiLU epilogue (dragonwing_edge_rs_b200/csrc/dw_device.cuh) budgets these
// errors; tests/test_gpu_fast_math_bounds.py compares.  Prints one line per
// range: "<name> <max relative error> <argument>".
#include <cmath>
#include <cstdint>
#include <cstdio>
#include <cstring>
#include <cuda_runtime.h>

__device__ __forceinline__ float ex2_approx(float x) {
    float r;
    asm("ex2.approx.ftz.f32 %0, %1;" : "=f"(r) : "f"(x));
    return r;
}
__device__ __forceinline__ float rcp_approx(float x) {
    float r;
    asm("rcp.approx.ftz.f32 %0, %1;" : "=f"(r) : "f"(x));
    return r;
}

// Inputs: the floats whose bit patterns run from lo_bits to lo_bits + count - 1.
__global__ void k_max_err(uint32_t lo_bits, uint32_t count, int which, unsigned long long *max_bits,
                          unsigned int *arg_bits) {
    double m = 0.0;
    uint32_t am = 0;
    for (uint32_t i = blockIdx.x * blockDim.x + threadIdx.x; i < count; i += gridDim.x * blockDim.x) {
        const uint32_t b = lo_bits + i;
        const float x = __uint_as_float(b);
        const double exact = which == 0 ? exp2((double)x) : 1.0 / (double)x;
        if (exact < 1.1754943508222875e-38 || exact > 3.4028234663852886e38) continue;  // normal results
        const double got = which == 0 ? (double)ex2_approx(x) : (double)rcp_approx(x);
        const double e = fabs(got - exact) / exact;
        if (e > m) {
            m = e;
            am = b;
        }
    }
    // non-negative doubles order like their bit patterns
    const unsigned long long v = (unsigned long long)__double_as_longlong(m);
    if (atomicMax(max_bits, v) < v) atomicExch(arg_bits, am);
}

static uint32_t bits_of(float f) {
    uint32_t b;
    memcpy(&b, &f, 4);
    return b;
}

int main() {
    struct Range {
        const char *name;
        int which;
        uint32_t lo, hi;  // inclusive bit range
    } ranges[] = {
        {"ex2_neg", 0, bits_of(-0.0f), bits_of(-126.0f)},       // x in [-126, -0]
        {"ex2_pos", 0, bits_of(0.0f), bits_of(127.99999f)},     // x in [0, 128)
        {"rcp", 1, bits_of(1.0f), bits_of(8.507059e37f)},        // d in [1, 2^126]
    };
    unsigned long long *d_max;
    unsigned int *d_arg;
    if (cudaMalloc(&d_max, sizeof(unsigned long long)) || cudaMalloc(&d_arg, sizeof(unsigned int))) return 1;
    for (const Range &r : ranges) {
        cudaMemset(d_max, 0, sizeof(unsigned long long));
        cudaMemset(d_arg, 0, sizeof(unsigned int));
        k_max_err<<<148 * 8, 256>>>(r.lo, r.hi - r.lo + 1, r.which, d_max, d_arg);
        if (cudaDeviceSynchronize() != cudaSuccess) return 2;
        unsigned long long hm;
        unsigned int ha;
        cudaMemcpy(&hm, d_max, sizeof(hm), cudaMemcpyDeviceToHost);
        cudaMemcpy(&ha, d_arg, sizeof(ha), cudaMemcpyDeviceToHost);
        double m;
        float a;
        memcpy(&m, &hm, 8);
        memcpy(&a, &ha, 4);
        printf("%s %.6e %.9g\n", r.name, m, a);
    }
    return 0;
}
