// dw_device.cuh -- device helpers shared by all kernels: the bit-exact
// requantisation epilogue, bounded waits and the device error record.
#pragma once

#include <cuda_fp16.h>

#include <cstdint>

#include "dw_expf.h"
#include "dw_internal.h"

namespace dw {

// Conversions and rounding here avoid the XU pipe (int<->float conversion,
// roundf, directed-rounding adds), which on sm_100 issues at 1/8 of the FMA
// rate; every helper is exact and uses only round-to-nearest FMA/ALU ops.
constexpr float kMagic = 12582912.0f;          // 1.5 * 2^23: ulp 1 over [2^23, 2^24)
constexpr int32_t kMagicBits = 0x4B400000;

// (float)v, exact for |v| < 2^22 (bit pattern of kMagic + v, minus kMagic).
__device__ __forceinline__ float i2f_small(int32_t v) {
    return __fsub_rn(__int_as_float(v + kMagicBits), kMagic);
}

// (float)v with round-to-nearest for any int32 (the XU conversion only when needed).
__device__ __forceinline__ float i2f_rn(int32_t v) {
    return ((uint32_t)(v + (1 << 22)) < (1u << 23)) ? i2f_small(v) : __int2float_rn(v);
}

// roundf(c) (half away from zero) for |c| <= 2^21, returned as the float
// kMagic + roundf(c) (its low byte is the int8 two's-complement result):
// r = kMagic + rint_even(c) by one RN add; d = c - rint(c) is exact; a tie
// rounded toward zero has d == copysign(0.5, c) and moves one step away.
__device__ __forceinline__ float round_away_magic(float c) {
    const float r = __fadd_rn(c, kMagic);
    const float d = __fsub_rn(c, __fsub_rn(r, kMagic));
    const float h = copysignf(0.5f, c);
    return d == h ? __fadd_rn(r, __fadd_rn(h, h)) : r;
}

// `v.clamp(-128.0, 127.0).round() as i8` (crates/dragonwing-cpu/src/ops.rs:3383-3385):
// clamp in f32, roundf (half away from zero), saturating cast (NaN -> 0).
__device__ __forceinline__ int32_t f32_to_i8(float v) {
    if (v != v) return 0;
    v = fminf(fmaxf(v, -128.0f), 127.0f);
    return __float_as_int(round_away_magic(v)) - kMagicBits;
}

// Same for a value known not to be NaN; returns the result in the low byte.
__device__ __forceinline__ uint32_t f32_to_i8_byte_nonan(float v) {
    v = fminf(fmaxf(v, -128.0f), 127.0f);
    return __float_as_uint(round_away_magic(v)) & 0xFFu;
}

// ---- SiLU fast path with a certified result -------------------------------
// t = fl(fl(y * fl(1/fl(1 + exp(-y)))) * inv_s_out) computed with the PTX
// approximations ex2.approx / rcp.approx instead of the exact exp and division.
// Relative error of t_fast against the reference's t (first order):
//   * exp(-y) = 2^(y * -log2(e)): the f32 constant (relative error 0.23 * 2^-24)
//     and the RN product put a relative error of at most 1.23 * 2^-24 on the
//     exponent y * log2(e), which moves e by at most |y| * 1.23 * 2^-24 relative
//     (log2(e) * ln(2) = 1);
//   * ex2.approx.ftz: at most 1.459e-7 relative, rcp.approx.ftz: at most
//     9.83e-8 -- the maxima over every input these paths see (ex2 of [-126, 128),
//     whose results are normal floats; rcp of [1, 2^126]), measured exhaustively
//     on B200 and re-checked by tests/test_gpu_fast_math_bounds.py; budgeted as
//     1.5e-7 and 1.0e-7.  Outside those ranges both sides agree exactly or round
//     to the same int8 (1 + e == 1; e = inf gives sig = 0; a flushed rcp result
//     makes |t| < 1e-30 on both sides);
//   * the reference's expf (the shared dw_expf, correctly rounded): 2^-24;
//   * seven RN roundings: 1 + e, y * sig and the scaling on the fast side; 1 + e,
//     the division, y * sig and the scaling on the reference's: 7 * 2^-24;
//   * a relative error r in e moves 1 + e, and so sig, by at most r relative;
//     when e overflows (y < -88) both sides give sig = 0 and t = -0.
// So |t_fast - t| <= |t| * (|y| * 7.33e-8 + 7.27e-7); the certificate takes 1.25
// times that (second-order terms and |t_fast| for |t| are far below the margin).
// The int8 result of t_fast is certified when no rounding boundary (a
// half-integer) lies within that distance; otherwise the caller recomputes the
// element exactly.  A tight certificate matters: the exact path is about 300
// cycles of dependent double arithmetic that a warp waits out, and the epilogue
// warps meet at every tile (3.6e-6 / 2.7e-7 here cost YOLOv8n b32 11% of its
// step).
constexpr float kEx2RelErr = 1.5e-7f;   // budget for ex2.approx.ftz (measured max 1.4584e-7)
constexpr float kRcpRelErr = 1.0e-7f;   // budget for rcp.approx.ftz (measured max 9.8292e-8)
constexpr float kSiluErrPerY = 9.2e-8f;  // 1.25 * 1.23 * 2^-24 (rounded up)
constexpr float kSiluErr0 = 9.1e-7f;     // 1.25 * (1.5e-7 + 1.0e-7 + 2^-24 + 7 * 2^-24) (rounded up)

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

// Returns kMagic + rint(clamp(t_fast)) as float bits (low byte = the int8 result)
// and sets `uncertain` when the result is not certified.  Preconditions: fa, dsc
// and inv finite.  When certified, rint == roundf (a tie is never certified).
__device__ __forceinline__ uint32_t silu_fast_bits(float fa, float dsc, float inv, bool &uncertain) {
    const float y = __fmul_rn(fa, dsc);
    const float e = ex2_approx(__fmul_rn(y, -1.44269502162933349609375f));
    const float sig = rcp_approx(__fadd_rn(1.0f, e));
    const float t = __fmul_rn(__fmul_rn(y, sig), inv);
    const float c = fminf(fmaxf(t, -128.0f), 127.0f);
    const float r = __fadd_rn(c, kMagic);
    const float d = fabsf(__fsub_rn(c, __fsub_rn(r, kMagic)));
    uncertain |= !(__fsub_rn(0.5f, d) > __fmul_rn(fabsf(t), __fmaf_rn(fabsf(y), kSiluErrPerY, kSiluErr0)));
    return __float_as_uint(r);
}

// silu_fast_bits for two accumulators (|a| < 2^22) at once, the arithmetic on
// f32 pairs: each lane of a packed operation is the same RN operation, so the
// error bound and the certificate are those of silu_fast_bits.
__device__ __forceinline__ void silu_fast_bits2(int32_t a0, int32_t a1, float d0, float d1, float inv, uint32_t &b0,
                                                uint32_t &b1, bool &u0, bool &u1) {
    const float2 mag = make_float2(kMagic, kMagic), nmag = make_float2(-kMagic, -kMagic);
    const float2 fa = __fadd2_rn(make_float2(__int_as_float(a0 + kMagicBits), __int_as_float(a1 + kMagicBits)), nmag);
    const float2 y = __fmul2_rn(fa, make_float2(d0, d1));
    const float2 arg = __fmul2_rn(y, make_float2(-1.44269502162933349609375f, -1.44269502162933349609375f));
    const float2 onep = __fadd2_rn(make_float2(ex2_approx(arg.x), ex2_approx(arg.y)), make_float2(1.0f, 1.0f));
    const float2 t = __fmul2_rn(__fmul2_rn(y, make_float2(rcp_approx(onep.x), rcp_approx(onep.y))), make_float2(inv, inv));
    const float2 c = make_float2(fminf(fmaxf(t.x, -128.0f), 127.0f), fminf(fmaxf(t.y, -128.0f), 127.0f));
    const float2 r = __fadd2_rn(c, mag);
    const float2 d = __ffma2_rn(__fadd2_rn(r, nmag), make_float2(-1.0f, -1.0f), c);  // c - rint(c), exact
    // the certificate on pairs as well: 0.5 + (-|d|) is the RN subtraction
    // 0.5 - |d|, and the fma and product are the scalar ones lane by lane
    // (YOLOv8n b32 step 1.797 -> 1.784 ms on B200)
    const float2 margin = __fadd2_rn(make_float2(0.5f, 0.5f), make_float2(-fabsf(d.x), -fabsf(d.y)));
    const float2 bound = __fmul2_rn(make_float2(fabsf(t.x), fabsf(t.y)),
                                    __ffma2_rn(make_float2(fabsf(y.x), fabsf(y.y)), make_float2(kSiluErrPerY, kSiluErrPerY),
                                               make_float2(kSiluErr0, kSiluErr0)));
    u0 |= !(margin.x > bound.x);
    u1 |= !(margin.y > bound.y);
    b0 = __float_as_uint(r.x);
    b1 = __float_as_uint(r.y);
}

// The fused epilogue for one accumulator (contract in include/dw_cuda.h):
// every float operation is a separately rounded IEEE op, as in the reference
// (Rust does not contract a*b+c), so the result is bit-exact.
__device__ __forceinline__ int32_t epilogue_one(int32_t acc, int32_t bias, float m, float dsc, int epi, int q6,
                                                float inv_s_out) {
    const int32_t a = (int32_t)((uint32_t)acc + (uint32_t)bias);
    if (epi == DW_EPI_SILU) {
        const float y = __fmul_rn(i2f_rn(a), dsc);
        const float z = dw_silu_f32(y);
        return f32_to_i8(__fmul_rn(z, inv_s_out));
    }
    int32_t q = f32_to_i8(__fmul_rn(i2f_rn(a), m));
    if (epi == DW_EPI_RELU) q = q > 0 ? q : 0;
    else if (epi == DW_EPI_RELU6) q = min(q > 0 ? q : 0, q6);
    return q;
}

// Out-of-line copy of epilogue_one for the rare exact fallbacks (ties, large
// accumulators, uncertain SiLU results): keeps the double-precision exp and the
// generic paths out of the hot loops' instruction stream.
static __device__ __noinline__ int32_t epilogue_one_slow(int32_t acc, int32_t bias, float m, float dsc, int epi, int q6,
                                                  float inv_s_out) {
    return epilogue_one(acc, bias, m, dsc, epi, q6, inv_s_out);
}

// ---- fp16 conversions with the reference's exact results ---------------------
// F16::to_f32 (crates/dragonwing-core/src/dtype.rs:225-263) is exact for normal
// halves, infinities and zeros; a subnormal half converts to exactly half its
// value (the renormalisation loop's exponent is one too small), and a NaN keeps
// its payload with the quiet bit set.  Every fp16 kernel that follows a CPU op
// converting with to_f32 uses this to stay bit-identical with it.
__device__ __forceinline__ float f16_to_f32_ref(uint16_t h) {
    const uint32_t e = h & 0x7C00u;
    if (e == 0x7C00u && (h & 0x03FFu))
        return __uint_as_float(((uint32_t)(h & 0x8000u) << 16) | 0x7FC00000u | ((uint32_t)(h & 0x03FFu) << 13));
    const float f = __half2float(__ushort_as_half(h));
    return e == 0 ? __fmul_rn(f, 0.5f) : f;
}

// F16::from_f32 (dtype.rs:164-222): round to nearest even with subnormals and
// overflow to infinity, which is cvt.rn.f16.f32 for every non-NaN input; a NaN
// maps to sign | 0x7E00 | min(payload >> 13, 0x1FF).
__device__ __forceinline__ uint16_t f32_to_f16_ref(float v) {
    if (v != v) {
        const uint32_t b = __float_as_uint(v);
        const uint32_t m = min((b & 0x007FFFFFu) >> 13, 0x1FFu);
        return (uint16_t)(((b >> 16) & 0x8000u) | 0x7E00u | m);
    }
    return __half_as_ushort(__float2half_rn(v));
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

// add_i8 (crates/dragonwing-cpu/src/ops.rs:3197-3209) on 4 packed int8 pairs:
// y = fl(fl(a * ra) + fl(b * rb)), then roundf and clamp, per element.
__device__ __forceinline__ uint32_t add4(uint32_t a, uint32_t b, float ra, float rb) {
    uint32_t r = 0;
#pragma unroll
    for (int k = 0; k < 4; k++) {
        int32_t av = (int8_t)(a >> (8 * k)), bv = (int8_t)(b >> (8 * k));
        float y = __fadd_rn(__fmul_rn(i2f_small(av), ra), __fmul_rn(i2f_small(bv), rb));
        r |= (uint32_t)(uint8_t)f32_to_i8(y) << (8 * k);
    }
    return r;
}

// Fast path of add_i8 for 16 elements, taken when the ratios are finite and
// below 1e30 (no overflow to infinity, so no NaN from inf - inf): the same
// f32 operations as the reference, the conversions and rounding steps two
// elements per packed instruction.  A
// byte a placed in the low mantissa bits of 1.5 * 2^23 (after a ^ 0x80, i.e.
// a + 128) reads as 1.5 * 2^23 + 128 + a, and subtracting 1.5 * 2^23 + 128
// (exact) gives a.  y = fl(fl(a * ra) + fl(b * rb)); clamp to [-128, 127] in
// f32; rint by the magic add; ties (c - rint(c) == +-0.5, rare) are redone
// per element with roundf's half-away-from-zero.
__device__ __forceinline__ uint4 add16_fast(uint4 a, uint4 b, float2 ra2, float2 rb2, float ra, float rb) {
    const float2 off = make_float2(-(kMagic + 128.0f), -(kMagic + 128.0f));
    const float2 mag = make_float2(kMagic, kMagic), nmag = make_float2(-kMagic, -kMagic);
    const float2 neg1 = make_float2(-1.0f, -1.0f);
    const uint32_t aw[4] = {a.x, a.y, a.z, a.w}, bw[4] = {b.x, b.y, b.z, b.w};
    uint32_t out[4];
    bool tie = false;
#pragma unroll
    for (int wd = 0; wd < 4; wd++) {
        const uint32_t ax = aw[wd] ^ 0x80808080u, bx = bw[wd] ^ 0x80808080u;
        uint32_t q[4];
#pragma unroll
        for (int h = 0; h < 2; h++) {
            const uint32_t s0 = 0x7650u | (uint32_t)(2 * h), s1 = 0x7650u | (uint32_t)(2 * h + 1);
            const float2 fa = __fadd2_rn(make_float2(__uint_as_float(__byte_perm(ax, 0x4B400000u, s0)),
                                                     __uint_as_float(__byte_perm(ax, 0x4B400000u, s1))), off);
            const float2 fb = __fadd2_rn(make_float2(__uint_as_float(__byte_perm(bx, 0x4B400000u, s0)),
                                                     __uint_as_float(__byte_perm(bx, 0x4B400000u, s1))), off);
            // scalar products and sum: a packed multiply feeding a packed
            // round-to-nearest add can be fused into one multiply-add by the
            // compiler, which skips the reference's rounding of the products
            float2 c = make_float2(__fadd_rn(__fmul_rn(fa.x, ra2.x), __fmul_rn(fb.x, rb2.x)),
                                   __fadd_rn(__fmul_rn(fa.y, ra2.y), __fmul_rn(fb.y, rb2.y)));
            c.x = fminf(fmaxf(c.x, -128.0f), 127.0f);
            c.y = fminf(fmaxf(c.y, -128.0f), 127.0f);
            const float2 r = __fadd2_rn(c, mag);
            const float2 d = __ffma2_rn(__fadd2_rn(r, nmag), neg1, c);  // c - rint(c), exact
            tie |= fmaxf(fabsf(d.x), fabsf(d.y)) == 0.5f;
            q[2 * h] = __float_as_uint(r.x);
            q[2 * h + 1] = __float_as_uint(r.y);
        }
        out[wd] = __byte_perm(__byte_perm(q[0], q[1], 0x0040), __byte_perm(q[2], q[3], 0x0040), 0x5410);
    }
    if (tie) {
#pragma unroll
        for (int wd = 0; wd < 4; wd++) out[wd] = add4(aw[wd], bw[wd], ra, rb);
    }
    return make_uint4(out[0], out[1], out[2], out[3]);
}

}  // namespace dw
