// dwconv_tma.cu -- int8 depthwise 3x3 stride-1 convolution fed by TMA.
//
// One CTA: one image, one 64-channel slab, a segment of output rows, a chunk
// of at most 56 output columns (two CTAs per SM).  A producer lane streams the input rows (the slab's 64 channels over
// the row's columns plus the 1-column halos, zero-filled by the TMA outside
// the image) into a ring of shared-memory slots; the consumer threads (4
// channels x 4 output columns each) slide down the rows.  Per input row a
// consumer reads its 6 words from shared memory, transposes them with byte
// permutes into per-channel column packs, and adds each kernel row to three
// output rows with one __dp4a per output -- exact int32 sums, as in the
// reference (crates/dragonwing-cpu/src/ops.rs:2669-2730 index order).  A row
// whose three kernel rows are in goes through the requantisation epilogue
// (the contract of include/dw_cuda.h) and is stored with plain 32-bit stores.
//
// Every wait is bounded (globaltimer); a wait that gives up records
// DW_DEV_WAIT_EXPIRED, the CTA stops, and the producer lets its copies in
// flight land before the CTA exits.

#include <algorithm>

#include "dw_device.cuh"
#include "dw_ptx.cuh"

namespace dw {
namespace {

constexpr int kDwMaxSlots = 16;
constexpr int kSlabCh = 64;  // channels per CTA (16 words)

struct DwTmaParams {
    int n, h, w, c, ho, wo, pt, pl;
    int strips;          // 4-column output strips per CTA
    int wchunk, wchunks; // output columns per CTA (4 * strips), column chunks per row
    int seg, segs;       // output rows per CTA, segments per image
    int slabs;           // 64-channel slabs
    int slots;           // ring depth
    int bw;              // input columns per row in the box: 4 * strips + 2
    uint32_t box_bytes;  // bw * 64: the bytes one row copy delivers
    uint32_t row_bytes;  // slot stride (box_bytes rounded up to 128)
    int cons_threads;    // 16 * strips
    uint64_t wait_cap_ns;
    int32_t *err;
    EpiParams ep;
};

__device__ __forceinline__ bool dw_wait(uint32_t bar, uint32_t parity, const DwTmaParams &p, volatile int *abort_flag,
                                        int site) {
#pragma unroll 1
    for (int i = 0; i < 128; i++)
        if (mbar_try_wait(bar, parity)) return true;
    const uint64_t t0 = globaltimer_ns();
#pragma unroll 1
    for (;;) {
        if (mbar_try_wait(bar, parity)) return true;
        if (*abort_flag) return false;
        if (globaltimer_ns() - t0 > p.wait_cap_ns) {
            *abort_flag = 1;
            record_error(p.err, DW_DEV_WAIT_EXPIRED, site, (int)parity);
            return false;
        }
    }
}

// The per-channel column packs of one input row and the three kernel-row
// dot products per output (the same arithmetic as the register-fed kernel).
// a0 (the output row that takes this input row as kernel row 0) starts here,
// from `init`; a1 and a2 accumulate.
__device__ __forceinline__ void dw_row(const uint32_t (&X)[6], const int32_t (&wk)[3][4], const int32_t (&init)[4],
                                       int32_t (&a0)[4][4], int32_t (&a1)[4][4], int32_t (&a2)[4][4]) {
    const uint32_t ta = __byte_perm(X[0], X[1], 0x5140), tb = __byte_perm(X[0], X[1], 0x7362);
    const uint32_t tc = __byte_perm(X[2], X[3], 0x5140), td = __byte_perm(X[2], X[3], 0x7362);
    const uint32_t te = __byte_perm(X[4], X[5], 0x5140), tf = __byte_perm(X[4], X[5], 0x7362);
    uint32_t P0[4], P1[4];
    P0[0] = __byte_perm(ta, tc, 0x5410);
    P0[1] = __byte_perm(ta, tc, 0x7632);
    P0[2] = __byte_perm(tb, td, 0x5410);
    P0[3] = __byte_perm(tb, td, 0x7632);
    P1[0] = te;
    P1[1] = te >> 16;
    P1[2] = tf;
    P1[3] = tf >> 16;
#pragma unroll
    for (int k = 0; k < 4; k++) {
#pragma unroll
        for (int j = 0; j < 4; j++) {
            const int win = (int)(j == 0 ? P0[k] : __funnelshift_r(P0[k], P1[k], 8 * j));
            a2[j][k] = __dp4a(win, wk[2][k], a2[j][k]);
            a1[j][k] = __dp4a(win, wk[1][k], a1[j][k]);
            a0[j][k] = __dp4a(win, wk[0][k], init[k]);
        }
    }
}

// Fast-path requantisation of 4 channels: roundf(clamp(fl(a * M), lo, hi))
// as bytes, with packed f32x2 arithmetic.  The accumulators carry the bias and
// the bit pattern of 1.5 * 2^23 (they start there), so reading them as floats
// and subtracting 1.5 * 2^23 gives acc + bias exactly (|acc + bias| < 2^22 on
// the fast path).  The product is rounded once (RN) as in the reference; the
// clamp to integer bounds before rounding commutes with roundf; rint is one
// RN add of 1.5 * 2^23; a tie (|v - rint(v)| == 0.5, rare) then moves away
// from zero.
__device__ __forceinline__ uint32_t requant4(const int32_t (&a)[4], const float2 (&m)[2], float lo, float hi) {
    const float2 mag = make_float2(kMagic, kMagic), nmag = make_float2(-kMagic, -kMagic);
    const float2 neg1 = make_float2(-1.0f, -1.0f);
    uint32_t pk[2];
#pragma unroll
    for (int h = 0; h < 2; h++) {
        const float2 f = __fadd2_rn(make_float2(__int_as_float(a[2 * h]), __int_as_float(a[2 * h + 1])), nmag);
        float2 v = __fmul2_rn(f, m[h]);
        v.x = fminf(fmaxf(v.x, lo), hi);
        v.y = fminf(fmaxf(v.y, lo), hi);
        const float2 r = __fadd2_rn(v, mag);
        const float2 d = __ffma2_rn(__fadd2_rn(r, nmag), neg1, v);  // v - rint(v), exact
        uint32_t q0 = __float_as_uint(r.x), q1 = __float_as_uint(r.y);
        if (fmaxf(fabsf(d.x), fabsf(d.y)) == 0.5f) {
            if (d.x == copysignf(0.5f, v.x)) q0 += v.x > 0.0f ? 1u : 0xFFFFFFFFu;
            if (d.y == copysignf(0.5f, v.y)) q1 += v.y > 0.0f ? 1u : 0xFFFFFFFFu;
        }
        pk[h] = __byte_perm(q0, q1, 0x0040);  // low bytes of the two results
    }
    return __byte_perm(pk[0], pk[1], 0x5410);
}

__global__ void __launch_bounds__(256, 2) k_dwconv3x3_tma(const __grid_constant__ CUtensorMap tx,
                                                           const int8_t *__restrict__ w, int8_t *__restrict__ y,
                                                           const __grid_constant__ DwTmaParams p) {
    extern __shared__ __align__(128) uint8_t smem[];
    uint64_t *full = reinterpret_cast<uint64_t *>(smem + (size_t)p.slots * p.row_bytes);
    uint64_t *empty = full + kDwMaxSlots;
    volatile int *abort_flag = reinterpret_cast<volatile int *>(empty + kDwMaxSlots);
    const int cons_warps = p.cons_threads / 32;

    // slab fastest: CTAs running side by side read and write the channel
    // chunks of the same pixels (whole DRAM bursts, shared L2 lines)
    int bid = blockIdx.x;
    const int slab = bid % p.slabs;
    bid /= p.slabs;
    const int wc = bid % p.wchunks;
    bid /= p.wchunks;
    const int seg = bid % p.segs;
    const int b = bid / p.segs;
    const int col0 = wc * p.wchunk;  // first output column of the CTA
    const int o0 = seg * p.seg;
    const int rows = p.seg + 2;  // input rows the segment reads

    if (threadIdx.x == 0) {
        for (int s = 0; s < p.slots; s++) {
            mbar_init(smem_u32(&full[s]), 1);
            mbar_init(smem_u32(&empty[s]), cons_warps);
        }
        *abort_flag = 0;
        asm volatile("fence.mbarrier_init.release.cluster;" ::: "memory");
        asm volatile("fence.proxy.async.shared::cta;" ::: "memory");
    }
    __syncthreads();

    if (threadIdx.x >= p.cons_threads) {
        // ------------------------------------------------------------ producer
        if (threadIdx.x == p.cons_threads) {
            asm volatile("prefetch.tensormap [%0];" ::"l"(&tx) : "memory");
            int issued = 0;
            for (int t = 0; t < rows; t++) {
                const int s = t % p.slots;
                if (t >= p.slots && !dw_wait(smem_u32(&empty[s]), (uint32_t)((t / p.slots - 1) & 1), p, abort_flag, 20))
                    break;
                mbar_expect_tx(smem_u32(&full[s]), p.box_bytes);
                tma_load_4d(smem_u32(smem + (size_t)s * p.row_bytes), &tx, smem_u32(&full[s]), slab * kSlabCh,
                            col0 - p.pl, o0 - p.pt + t, b);
                issued = t + 1;
            }
            // let the copies still in flight land before the CTA can exit
            for (int t = std::max(0, issued - p.slots); t < issued; t++) {
                const int s = t % p.slots;
                const uint64_t t0 = globaltimer_ns();
                while (!mbar_try_wait(smem_u32(&full[s]), (uint32_t)((t / p.slots) & 1)) &&
                       globaltimer_ns() - t0 < p.wait_cap_ns) {
                }
            }
        }
        return;
    }

    // ---------------------------------------------------------------- consumers
    const int cg = threadIdx.x & 15;            // word (4 channels) within the slab
    const int strip = threadIdx.x >> 4;         // 4 output columns
    const int lane = threadIdx.x & 31;
    const int cg_n = p.c >> 2;
    const int gw = slab * (kSlabCh / 4) + cg;   // word index of the 4 channels
    const int ow0 = col0 + strip * 4;  // the thread's first output column
    const int bc0 = strip * 4;         // its first column in the box
    const uint32_t *wq = reinterpret_cast<const uint32_t *>(w) + gw;
    int32_t wk[3][4];
#pragma unroll
    for (int kh = 0; kh < 3; kh++) {
        const uint32_t k0 = __ldg(wq + (size_t)(kh * 3 + 0) * cg_n), k1 = __ldg(wq + (size_t)(kh * 3 + 1) * cg_n);
        const uint32_t k2 = __ldg(wq + (size_t)(kh * 3 + 2) * cg_n);
#pragma unroll
        for (int k = 0; k < 4; k++) {
            const uint32_t t01 = __byte_perm(k0, k1, (uint32_t)((4 + k) << 4 | k));
            wk[kh][k] = (int32_t)(__byte_perm(t01, k2, (uint32_t)((4 + k) << 8 | 0x10)) & 0x00FFFFFFu);
        }
    }
    const EpiParams &ep = p.ep;
    const int c0 = gw * 4;
    int32_t bias[4];
    float m[4], dsc[4];
    bool fast = ep.epilogue != DW_EPI_SILU;
#pragma unroll
    for (int k = 0; k < 4; k++) {
        bias[k] = ep.bias ? __ldg(ep.bias + c0 + k) : 0;
        m[k] = ep.M ? __ldg(ep.M + c0 + k) : 0.0f;
        dsc[k] = ep.D ? __ldg(ep.D + c0 + k) : 0.0f;
        fast = fast && (uint32_t)(bias[k] + (1 << 21)) < (1u << 22) && isfinite(m[k]);
    }
    const float2 m2[2] = {make_float2(m[0], m[1]), make_float2(m[2], m[3])};

    int32_t init[4];  // fast path: bias + the magic bit pattern; exact path: 0 (the bias is added there)
#pragma unroll
    for (int k = 0; k < 4; k++) init[k] = fast ? bias[k] + kMagicBits : 0;
    const float lo = (ep.epilogue == DW_EPI_RELU || ep.epilogue == DW_EPI_RELU6) ? 0.0f : -128.0f;
    const float hi = ep.epilogue == DW_EPI_RELU6 ? (float)ep.q6 : 127.0f;
    uint32_t *yb = reinterpret_cast<uint32_t *>(y + (size_t)b * p.ho * p.wo * p.c) + gw;

    auto finish = [&](int t, const int32_t (&acc)[4][4]) {
        const int oh = o0 + t - 2;
        if (t >= 2 && t - 2 < p.seg && oh < p.ho) {
            uint32_t *yr = yb + ((size_t)oh * p.wo + ow0) * cg_n;
#pragma unroll
            for (int j = 0; j < 4; j++) {
                if (ow0 + j < p.wo) {
                    uint32_t packed = 0;
                    if (fast) {
                        packed = requant4(acc[j], m2, lo, hi);
                    } else {
#pragma unroll
                        for (int k = 0; k < 4; k++)
                            packed |= (uint32_t)(uint8_t)epilogue_one_slow(acc[j][k], bias[k], m[k], dsc[k],
                                                                          ep.epilogue, ep.q6, ep.inv_s_out)
                                      << (8 * k);
                    }
                    yr[j * cg_n] = packed;
                }
            }
        }
    };
    // one input row from its slot: the thread's 6 words (columns ow0 .. ow0 + 5
    // of the box, which starts at input column -pl)
    auto take_row = [&](int t, uint32_t (&X)[6]) -> bool {
        const int s = t % p.slots;
        if (!dw_wait(smem_u32(&full[s]), (uint32_t)((t / p.slots) & 1), p, abort_flag, 21)) return false;
        const uint32_t *row = reinterpret_cast<const uint32_t *>(smem + (size_t)s * p.row_bytes);
#pragma unroll
        for (int c = 0; c < 6; c++) X[c] = row[(bc0 + c) * (kSlabCh / 4) + cg];
        __syncwarp();
        if (lane == 0) mbar_arrive(smem_u32(&empty[s]));
        return true;
    };

    int32_t A[4][4] = {}, B[4][4] = {}, C[4][4] = {};
    // step t reads input row o0 - pt + t; the kh = 0 / 1 / 2 accumulators hold
    // output rows o0 + t, o0 + t - 1, o0 + t - 2 (the roles rotate every step).
#pragma unroll 1
    for (int t = 0; t < rows; t += 3) {
        uint32_t X[6];
        if (!take_row(t, X)) break;
        dw_row(X, wk, init, A, B, C);
        finish(t, C);
        if (t + 1 >= rows) break;
        if (!take_row(t + 1, X)) break;
        dw_row(X, wk, init, C, A, B);
        finish(t + 1, B);
        if (t + 2 >= rows) break;
        if (!take_row(t + 2, X)) break;
        dw_row(X, wk, init, B, C, A);
        finish(t + 2, A);
    }
}

}  // namespace

// Returns DW_ERR_UNSUPPORTED (without launching) when the shape does not fit
// the kernel: stride 1, 3x3, multiplier 1, c % 64 == 0.
dw_status launch_dwconv3x3_tma_i8(dw_backend *be, const dw_conv_desc &d, int ho, int wo, const int8_t *x,
                                  const int8_t *w_hwcm, const EpiParams &ep, int8_t *y) {
    if (!be->encode_tiled || d.k_h != 3 || d.k_w != 3 || d.stride_h != 1 || d.stride_w != 1 ||
        d.c_out != d.c_in || d.c_in % kSlabCh || ((uintptr_t)x & 15) || ((uintptr_t)y & 3) ||
        ((uintptr_t)w_hwcm & 3))
        return DW_ERR_UNSUPPORTED;
    DwTmaParams p{};
    p.n = d.n; p.h = d.h; p.w = d.w; p.c = d.c_in; p.ho = ho; p.wo = wo; p.pt = d.pad_t; p.pl = d.pad_l;
    // column chunks of at most 56 output columns: CTAs of <= 224 consumers + the
    // producer warp, two per SM
    p.wchunks = (wo + 55) / 56;
    p.strips = ((wo + p.wchunks - 1) / p.wchunks + 3) / 4;
    if (p.strips % 2) p.strips++;  // whole warps of consumers
    p.wchunk = 4 * p.strips;
    p.wchunks = (wo + p.wchunk - 1) / p.wchunk;
    p.bw = p.wchunk + 2;
    if (p.bw > 256 || 16 * p.strips > 224) return DW_ERR_UNSUPPORTED;
    p.cons_threads = 16 * p.strips;
    p.box_bytes = (uint32_t)(p.bw * kSlabCh);
    p.row_bytes = (p.box_bytes + 127) & ~127u;
    p.slots = std::min<int>(kDwMaxSlots, (int)((96u * 1024u) / p.row_bytes));
    if (p.slots < 4) return DW_ERR_UNSUPPORTED;
    p.slabs = d.c_in / kSlabCh;
    // row segments: enough CTAs for the SMs, each reading its 2 halo rows
    p.seg = std::min(ho, 28);
    p.segs = (ho + p.seg - 1) / p.seg;
    const long long ctas = (long long)d.n * p.slabs * p.segs * p.wchunks;
    if (ctas >= (1ll << 31)) return DW_ERR_UNSUPPORTED;
    p.wait_cap_ns = be->wait_cap_ns;
    p.err = be->dev_err;
    p.ep = ep;

    CUtensorMap tx;
    cuuint64_t dims[4] = {(cuuint64_t)d.c_in, (cuuint64_t)d.w, (cuuint64_t)d.h, (cuuint64_t)d.n};
    cuuint64_t strides[3] = {(cuuint64_t)d.c_in, (cuuint64_t)d.w * d.c_in, (cuuint64_t)d.h * d.w * d.c_in};
    cuuint32_t box[4] = {(cuuint32_t)kSlabCh, (cuuint32_t)p.bw, 1, 1};
    cuuint32_t estr[4] = {1, 1, 1, 1};
    CUresult r = be->encode_tiled(&tx, CU_TENSOR_MAP_DATA_TYPE_UINT8, 4, const_cast<int8_t *>(x), dims, strides, box,
                                  estr, CU_TENSOR_MAP_INTERLEAVE_NONE, CU_TENSOR_MAP_SWIZZLE_NONE,
                                  CU_TENSOR_MAP_L2_PROMOTION_L2_256B, CU_TENSOR_MAP_FLOAT_OOB_FILL_NONE);
    if (r != CUDA_SUCCESS) return DW_ERR_UNSUPPORTED;
    const size_t smem = (size_t)p.slots * p.row_bytes + 2 * kDwMaxSlots * sizeof(uint64_t) + 16;
    static bool attr_set[16] = {};
    if (be->device < 16 && !attr_set[be->device]) {
        cudaFuncSetAttribute(k_dwconv3x3_tma, cudaFuncAttributeMaxDynamicSharedMemorySize, 200 * 1024);
        attr_set[be->device] = true;
    }
    k_dwconv3x3_tma<<<(unsigned)ctas, p.cons_threads + 32, smem, be->stream>>>(tx, w_hwcm, y, p);
    return dw_after_launch(be, "dwconv3x3_tma_i8");
}

}  // namespace dw
