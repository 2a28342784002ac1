// dwconv_stream.cu -- int8 depthwise 3x3 stride-1 convolution, persistent and
// streaming over whole pixels.
//
// Work layout.  A lane is a column strip of `cw` output columns over a channel
// group of `cg` channels (all the channels when they fit); its rows are the
// R = n * ho output rows, image after image.  The first lanes x per_lane CTAs
// are the main ones: CTA i streams lane i % lanes, rows [k Rm / per_lane,
// (k + 1) Rm / per_lane) of it (k = i / lanes), so CTAs that run side by side
// cover the same image rows of neighbouring strips (their halo columns meet
// in L2 and whole image rows are in flight together).  When the SMs do not
// divide into lanes evenly, `extra` more CTAs take the lanes' last R - Rm rows
// (the tails, lane after lane, split evenly), so every SM streams about the
// same number of rows.  A CTA's work is a list of pieces (lane, row range);
// a run of rows inside one image is a segment, and crossing into the next
// image or piece restarts the row rotation with two halo rows.
//
// Data movement.  A producer lane loads stages of three input rows through the
// tensor map -- each row the strip's cw + 2 columns of whole cg-channel pixels,
// contiguous in NHWC when cg == c -- into a ring of shared-memory slots; zero
// fill supplies the padding rows and columns.
//
// Arithmetic.  Consumer threads own 4 channels x kCPT output columns.  Per
// input row a thread reads its kCPT + 2 words, transposes them with byte
// permutes into per-channel column packs, and adds each kernel row to three
// output rows with one __dp4a per output and kernel row: exact int32 sums, as
// in the reference (crates/dragonwing-cpu/src/ops.rs:2669-2730 index order).
// An output row whose three kernel rows are in is requantised and stored with
// coalesced 32-bit stores (consecutive threads own consecutive channel words
// of a pixel).
//
// Requantisation (the contract of include/dw_cuda.h), exact on every path:
//  * ReLU / ReLU6: v = fl(fl(acc + bias) * M) as the reference, then
//    floor(2v + 1) from one packed add rounded toward zero (it lands in the low
//    mantissa bits of 1.5 * 2^22, where the spacing is 0.5), clamped to
//    [0, 2 hi + 1] on the packed int16 pair and halved: clamp(floor(v + 0.5),
//    0, hi).  For v >= 0, floor(v + 0.5) is roundf(v); below zero both are
//    <= 0, which the ReLU bound maps to 0.  Clamping the integer after
//    rounding equals rounding after clamping because the bounds are integers.
//  * no activation: clamp to [-128, 127] in f32, rint by the magic add, ties
//    moved away from zero.
//  The fast paths need |acc + bias| < 2^22, a finite M and, for the int16
//  pairs, |2v + 1| < 2^15.  A thread whose channels miss that (pathological scales
//  or biases) recomputes its outputs after the stream, element by element with
//  the reference epilogue, over its own earlier stores; the hot loop carries
//  no exact path.  SiLU is not taken here (the slab kernel handles it).
//
// Every wait is bounded (globaltimer); a wait that gives up records
// DW_DEV_WAIT_EXPIRED, the CTA stops, and the producer lets its copies in
// flight land before the CTA exits.

#include <algorithm>

#include "dw_device.cuh"
#include "dw_ptx.cuh"

namespace dw {
namespace {

constexpr int kStreamMaxSlots = 8;

// CTA shapes: columns per thread, the most consumer threads (plus one producer
// warp) and the CTAs per SM the register budget is compiled for.  19 warps on
// an SM leave 96 registers a thread (the register file is split four ways).
struct StShape {
    int cpt, max_cons, min_blocks;
};
constexpr StShape kStShapes[3] = {
    {2, 576, 1},  // 18 consumer warps (the default)
    {2, 288, 2},  // two CTAs of 9 consumer warps
    {4, 288, 1},  // 9 consumer warps with 4 x 4 tiles
};

struct DwStreamParams {
    int n, h, w, c, ho, wo, pt, pl;
    int cg;                // channels per lane
    int words;             // cg / 4
    int groups;            // c / cg
    int cw;                // output columns per strip
    int strips;            // column strips per row
    int bw;                // input columns per stage row: cw + 2
    uint32_t stage_bytes;  // 3 * bw * cg (the box)
    uint32_t slot_bytes;   // stage_bytes rounded up to 128
    int slots;
    int cons_threads;      // words * cw / kCPT
    int per_lane;          // main CTAs per lane
    int rows_main;         // rows of each lane the main CTAs take (Rm); the rest go to the extra CTAs
    int extra;             // extra CTAs for the lanes' tails
    const int8_t *x;       // the input (the exact recomputation reads it directly)
    uint64_t wait_cap_ns;
    int32_t *err;
    EpiParams ep;
};

__device__ __forceinline__ bool st_wait(uint32_t bar, uint32_t parity, const DwStreamParams &p,
                                        volatile int *abort_flag, int site) {
#pragma unroll 1
    for (int i = 0; i < 64; i++)
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

__device__ __forceinline__ uint32_t lds_u32(uint32_t addr) {
    uint32_t v;
    asm volatile("ld.shared.u32 %0, [%1];" : "=r"(v) : "r"(addr));
    return v;
}

// Per-channel column packs of one input row and the three kernel-row dot
// products per output.  X holds kCPT + 2 words (columns), 4 channels each.
// a0 (the output row that takes this input row as kernel row 0) starts from
// `init`; a1 and a2 accumulate.
template <int kCPT>
__device__ __forceinline__ void st_row(const uint32_t (&X)[kCPT + 2], const int32_t (&wk)[3][4],
                                       const int32_t (&init)[4], int32_t (&a0)[kCPT][4], int32_t (&a1)[kCPT][4],
                                       int32_t (&a2)[kCPT][4]) {
    const uint32_t ta = __byte_perm(X[0], X[1], 0x5140), tb = __byte_perm(X[0], X[1], 0x7362);
    const uint32_t tc = __byte_perm(X[2], X[3], 0x5140), td = __byte_perm(X[2], X[3], 0x7362);
    uint32_t P[4];  // P[k]: channel k over columns 0..3
    P[0] = __byte_perm(ta, tc, 0x5410);
    P[1] = __byte_perm(ta, tc, 0x7632);
    P[2] = __byte_perm(tb, td, 0x5410);
    P[3] = __byte_perm(tb, td, 0x7632);
    if constexpr (kCPT == 2) {
#pragma unroll
        for (int k = 0; k < 4; k++) {
#pragma unroll
            for (int j = 0; j < 2; j++) {
                const int win = (int)(j == 0 ? P[k] : P[k] >> 8);  // byte 3 meets a zero weight
                a2[j][k] = __dp4a(win, wk[2][k], a2[j][k]);
                a1[j][k] = __dp4a(win, wk[1][k], a1[j][k]);
                a0[j][k] = __dp4a(win, wk[0][k], init[k]);
            }
        }
    } else {
        // columns 4, 5: te = (X4.b0, X5.b0, X4.b1, X5.b1), tf = (X4.b2, X5.b2, X4.b3, X5.b3)
        const uint32_t te = __byte_perm(X[4], X[5], 0x5140), tf = __byte_perm(X[4], X[5], 0x7362);
#pragma unroll
        for (int k = 0; k < 4; k++) {
            const uint32_t ex = (k < 2) ? te : tf;
            // window j = columns j .. j + 2 (+ one byte that meets the zero weight)
            const uint32_t s1 = (k & 1) ? 0x6321u : 0x4321u;
            const uint32_t s2 = (k & 1) ? 0x7632u : 0x5432u;
            const uint32_t s3 = (k & 1) ? 0x7763u : 0x5543u;
            int win[4];
            win[0] = (int)P[k];
            win[1] = (int)__byte_perm(P[k], ex, s1);
            win[2] = (int)__byte_perm(P[k], ex, s2);
            win[3] = (int)__byte_perm(P[k], ex, s3);
#pragma unroll
            for (int j = 0; j < 4; j++) {
                a2[j][k] = __dp4a(win[j], wk[2][k], a2[j][k]);
                a1[j][k] = __dp4a(win[j], wk[1][k], a1[j][k]);
                a0[j][k] = __dp4a(win[j], wk[0][k], init[k]);
            }
        }
    }
}

// ReLU-family fast requantisation of 4 channels (header comment); returns the
// 4 result bytes.  The accumulators start at bias + the bit pattern of
// 1.5 * 2^23, so reading them as floats and subtracting 1.5 * 2^23 gives
// acc + bias exactly; v = fl(that * M) as the reference.  One add rounded
// toward zero of 1.5 * 2^22 + 0.5 (exact: the spacing in [2^22, 2^23) is 0.5)
// gives 1.5 * 2^22 + floor_half(v + 0.5), floor_half rounding down to a multiple
// of 0.5; its low 16 bits are floor(2v + 1) as int16 (|v| < 2^14 on the fast
// path).  Clamped to [0, 2 hi + 1] and halved, that is clamp(floor(v + 0.5), 0,
// hi): floor(v + 0.5) == roundf(v) for v >= 0, both are <= 0 below zero, and
// halving commutes with the clamp because 2 hi + 1 halves to hi.  The halving
// runs on the packed bytes (every lane is at most 255 there).  The packed
// directed-rounding add issues on the FMA pipe at the full f32x2 rate; the
// compiler does not fuse it with the round-to-nearest multiply before it (the
// rounding modes differ), so v is rounded as the reference rounds it.
__device__ __forceinline__ uint32_t requant_relu4(const int32_t (&a)[4], const float2 (&m)[2], uint32_t hi2) {
    const float2 nmag = make_float2(-kMagic, -kMagic);
    const float2 mag = make_float2(6291456.5f, 6291456.5f);  // 1.5 * 2^22 + 0.5
    uint32_t c[2];
#pragma unroll
    for (int h = 0; h < 2; h++) {
        const float2 f = __fadd2_rn(make_float2(__int_as_float(a[2 * h]), __int_as_float(a[2 * h + 1])), nmag);
        const float2 v = __fmul2_rn(f, m[h]);
        const float2 r = __fadd2_rz(v, mag);
        c[h] = __vimin_s16x2_relu(__byte_perm(__float_as_uint(r.x), __float_as_uint(r.y), 0x5410), hi2);
    }
    return (__byte_perm(c[0], c[1], 0x6420) >> 1) & 0x7F7F7F7Fu;
}

// Signed (no activation) fast requantisation of 4 channels: clamp to
// [-128, 127] in f32, rint by the magic add, ties moved away from zero.
__device__ __forceinline__ uint32_t requant_signed4(const int32_t (&a)[4], const float2 (&m)[2]) {
    const float2 mag = make_float2(kMagic, kMagic), nmag = make_float2(-kMagic, -kMagic);
    const float2 neg1 = make_float2(-1.0f, -1.0f);
    uint32_t pk[2];
#pragma unroll
    for (int h = 0; h < 2; h++) {
        const float2 f = make_float2(__fsub_rn(__int_as_float(a[2 * h]), kMagic),
                                     __fsub_rn(__int_as_float(a[2 * h + 1]), kMagic));
        float2 v = __fmul2_rn(f, m[h]);
        v.x = fminf(fmaxf(v.x, -128.0f), 127.0f);
        v.y = fminf(fmaxf(v.y, -128.0f), 127.0f);
        const float2 r = __fadd2_rn(v, mag);
        const float2 d = __ffma2_rn(__fadd2_rn(r, nmag), neg1, v);
        uint32_t q0 = __float_as_uint(r.x), q1 = __float_as_uint(r.y);
        if (fmaxf(fabsf(d.x), fabsf(d.y)) == 0.5f) {
            if (d.x == copysignf(0.5f, v.x)) q0 += v.x > 0.0f ? 1u : 0xFFFFFFFFu;
            if (d.y == copysignf(0.5f, v.y)) q1 += v.y > 0.0f ? 1u : 0xFFFFFFFFu;
        }
        pk[h] = __byte_perm(q0, q1, 0x0040);
    }
    return __byte_perm(pk[0], pk[1], 0x5410);
}

// The thread's kernel rows for channel word gw: (w0, w1, w2, 0) bytes per channel.
__device__ __forceinline__ void load_kernel_rows(const int8_t *__restrict__ w, int cwords, int gw,
                                                 int32_t (&wk)[3][4]) {
    const uint32_t *w32 = reinterpret_cast<const uint32_t *>(w);
#pragma unroll
    for (int kh = 0; kh < 3; kh++) {
        const uint32_t k0 = __ldg(w32 + (size_t)(kh * 3 + 0) * cwords + gw);
        const uint32_t k1 = __ldg(w32 + (size_t)(kh * 3 + 1) * cwords + gw);
        const uint32_t k2 = __ldg(w32 + (size_t)(kh * 3 + 2) * cwords + gw);
#pragma unroll
        for (int k = 0; k < 4; k++) {
            const uint32_t t01 = __byte_perm(k0, k1, (uint32_t)((4 + k) << 4 | k));
            wk[kh][k] = (int32_t)(__byte_perm(t01, k2, (uint32_t)((4 + k) << 8 | 0x10)) & 0x00FFFFFFu);
        }
    }
}

// Thread state the segment loop reads.
struct StThread {
    int32_t wk[3][4];  // kernel rows: (w0, w1, w2, 0) bytes per channel
    int32_t init[4];   // accumulator start: bias + the magic bits
    float2 m2[2];      // M of channels 0,1 and 2,3
    uint32_t hi2;      // 2 * (ReLU ceiling) + 1 in both int16 lanes
};

// Position in the ring of input stages, advanced without divisions.
struct RingPos {
    uint32_t slot_addr;  // shared address of the current slot (+ the thread's offset)
    uint32_t bar;        // shared address of the current slot's full barrier
    int s;               // slot index
    uint32_t ph;         // barrier phase parity of the current pass over the ring
};

// One segment: `count` (>= 3) input rows from the ring position `rp` on;
// output rows are stored from the third input row on.  The first stage (one
// output row) and a last partial stage are peeled off, so whole stages run
// without per-row tests.  kFull: every column of the thread is inside the
// image (no per-store test).  Returns false when a wait gave up.
template <int kCPT, bool kRelu, bool kFull>
__device__ __forceinline__ bool st_segment(const DwStreamParams &p, const StThread &ts, int count, RingPos &rp,
                                           uint32_t slot0_addr, uint32_t full0, uint32_t empty0,
                                           const uint32_t (&coff)[kCPT + 2], uint32_t rw4, uint32_t *yb,
                                           size_t row_words, int colmask, volatile int *abort_flag, int lane) {
    const int cwords = p.c >> 2;
    uint32_t *yr = yb;  // the next output row to store
    int32_t A[kCPT][4], B[kCPT][4], C[kCPT][4];
    // one input row at shared address `addr` into the rotation (a0 starts there)
    auto row = [&](uint32_t addr, int32_t (&a0)[kCPT][4], int32_t (&a1)[kCPT][4], int32_t (&a2)[kCPT][4]) {
        uint32_t X[kCPT + 2];
#pragma unroll
        for (int c = 0; c < kCPT + 2; c++) X[c] = lds_u32(addr + coff[c]);
        st_row<kCPT>(X, ts.wk, ts.init, a0, a1, a2);
    };
    auto store = [&](const int32_t (&acc)[kCPT][4]) {
#pragma unroll
        for (int j = 0; j < kCPT; j++) {
            const uint32_t v = kRelu ? requant_relu4(acc[j], ts.m2, ts.hi2) : requant_signed4(acc[j], ts.m2);
            if (kFull || (colmask & (1 << j))) yr[(size_t)j * cwords] = v;
        }
        yr += row_words;
    };
    // releases the stage's slot and moves to the next one
    auto next_slot = [&]() {
        __syncwarp();
        if (lane == 0) mbar_arrive(empty0 + 8u * (uint32_t)rp.s);
        rp.s++;
        rp.slot_addr += p.slot_bytes;
        rp.bar += 8u;
        if (rp.s == p.slots) {
            rp.s = 0;
            rp.slot_addr = slot0_addr;
            rp.bar = full0;
            rp.ph ^= 1u;
        }
    };
    // first stage: rows 0 and 1 start output rows, row 2 completes output row 0
    if (!st_wait(rp.bar, rp.ph, p, abort_flag, 31)) return false;
    row(rp.slot_addr, A, B, C);
    row(rp.slot_addr + rw4, C, A, B);
    row(rp.slot_addr + 2 * rw4, B, C, A);
    store(A);
    next_slot();
    const int whole = count / 3;  // stages of three rows
#pragma unroll 1
    for (int k = 1; k < whole; k++) {
        if (!st_wait(rp.bar, rp.ph, p, abort_flag, 31)) return false;
        row(rp.slot_addr, A, B, C);
        store(C);
        row(rp.slot_addr + rw4, C, A, B);
        store(B);
        row(rp.slot_addr + 2 * rw4, B, C, A);
        store(A);
        next_slot();
    }
    const int tail = count - 3 * whole;  // rows of a last partial stage
    if (tail) {
        if (!st_wait(rp.bar, rp.ph, p, abort_flag, 31)) return false;
        row(rp.slot_addr, A, B, C);
        store(C);
        if (tail == 2) {
            row(rp.slot_addr + rw4, C, A, B);
            store(B);
        }
        next_slot();
    }
    return true;
}

// Exact recomputation of a thread's outputs (4 channels from c0, columns ow0 ..
// ow0 + kCPT - 1, output rows [r0, r1) of the lane) for channels outside the
// fast range: direct 3x3 sums from the input in global memory and the
// reference epilogue per element.  Cold code, kept out of line.
template <int kCPT>
static __device__ __noinline__ void st_exact_outputs(const DwStreamParams &p, const int8_t *__restrict__ w,
                                                     int8_t *__restrict__ y, int c0, int ow0, int r0, int r1) {
    const EpiParams &ep = p.ep;
#pragma unroll 1
    for (int r = r0; r < r1; r++) {
        const int b = r / p.ho, oh = r - b * p.ho;
#pragma unroll 1
        for (int j = 0; j < kCPT; j++) {
            const int ow = ow0 + j;
            if (ow >= p.wo) break;
#pragma unroll 1
            for (int k = 0; k < 4; k++) {
                const int ch = c0 + k;
                int32_t acc = 0;
                for (int kh = 0; kh < 3; kh++) {
                    const int ih = oh - p.pt + kh;
                    if (ih < 0 || ih >= p.h) continue;
                    for (int kw = 0; kw < 3; kw++) {
                        const int iw = ow - p.pl + kw;
                        if (iw < 0 || iw >= p.w) continue;
                        acc += (int32_t)p.x[(((size_t)b * p.h + ih) * p.w + iw) * p.c + ch] *
                               (int32_t)w[(size_t)(kh * 3 + kw) * p.c + ch];
                    }
                }
                const int32_t bias = ep.bias ? ep.bias[ch] : 0;
                const float m = ep.M ? ep.M[ch] : 0.0f;
                const float dsc = ep.D ? ep.D[ch] : 0.0f;
                y[(((size_t)b * p.ho + oh) * p.wo + ow) * p.c + ch] =
                    (int8_t)epilogue_one_slow(acc, bias, m, dsc, ep.epilogue, ep.q6, ep.inv_s_out);
            }
        }
    }
}

// One piece of a CTA's work for a consumer thread: rows [r0, r1) of lane
// `my_lane`, from ring position rp on.  Returns false when a wait gave up.
template <int kCPT, bool kRelu>
__device__ __forceinline__ bool st_piece(const DwStreamParams &p, const int8_t *__restrict__ w,
                                         int8_t *__restrict__ y, int my_lane, int r0, int r1, RingPos &rp,
                                         uint32_t slot0, uint32_t full0, uint32_t empty0,
                                         volatile int *abort_flag) {
    const int grp = my_lane % p.groups, strip = my_lane / p.groups;
    const int g = threadIdx.x % p.words;  // channel word within the lane's group
    const int q = threadIdx.x / p.words;  // column group within the strip
    const int lane = threadIdx.x & 31;
    const int cwords = p.c >> 2;
    const EpiParams &ep = p.ep;
    const int gw = grp * p.words + g;  // the thread's channel word
    const int c0 = gw * 4;

    StThread ts;
    bool fast = kRelu || ep.epilogue == DW_EPI_NONE;
    {
        load_kernel_rows(w, cwords, gw, ts.wk);
        int32_t bias[4];
        float m[4];
#pragma unroll
        for (int k = 0; k < 4; k++) {
            bias[k] = ep.bias ? __ldg(ep.bias + c0 + k) : 0;
            m[k] = ep.M ? __ldg(ep.M + c0 + k) : 0.0f;
            // |acc| <= 9 * 128 * 128; the fast paths need |acc + bias| < 2^22 and, for
            // the int16 pairs, |2v + 1| < 2^15 (|v| kept below 15000)
            const float amax = 147456.0f + fabsf((float)bias[k]);
            fast = fast && (uint32_t)(bias[k] + (1 << 21)) < (1u << 22) && isfinite(m[k]) &&
                   (!kRelu || fabsf(m[k]) * amax < 15000.0f);
            ts.init[k] = (int32_t)((uint32_t)bias[k] + (uint32_t)kMagicBits);
        }
        ts.m2[0] = make_float2(m[0], m[1]);
        ts.m2[1] = make_float2(m[2], m[3]);
        // a negative ReLU6 ceiling leaves the fast range (min(max(q, 0), q6) is q6 itself)
        if (kRelu && ep.epilogue == DW_EPI_RELU6 && ep.q6 < 0) fast = false;
        const int hi = ep.epilogue == DW_EPI_RELU6 ? min(max(ep.q6, 0), 127) : 127;
        ts.hi2 = (uint32_t)(2 * hi + 1) | ((uint32_t)(2 * hi + 1) << 16);
    }

    const int ow0 = strip * p.cw + q * kCPT;  // the thread's first output column
    int colmask = 0;
#pragma unroll
    for (int j = 0; j < kCPT; j++) colmask |= (ow0 + j < p.wo) ? (1 << j) : 0;
    const bool wfull = __all_sync(0xFFFFFFFFu, colmask == (1 << kCPT) - 1);
    // the thread's column offsets and the stride of a stage row (shared bytes)
    uint32_t coff[kCPT + 2];
#pragma unroll
    for (int c = 0; c < kCPT + 2; c++) coff[c] = 4u * (uint32_t)(c * p.words);
    const uint32_t rw4 = 4u * (uint32_t)(p.bw * p.words);
    const size_t row_words = (size_t)p.wo * cwords;
    uint32_t *y32 = reinterpret_cast<uint32_t *>(y);
    bool ok = true;
#pragma unroll 1
    for (int r = r0; r < r1 && ok;) {
        const int b = r / p.ho, o0 = r - b * p.ho;
        const int len = min(r1 - r, p.ho - o0);
        r += len;
        // output word of (image b, row o0, column ow0, the thread's channel word)
        uint32_t *yb = y32 + ((size_t)b * p.ho * p.wo + (size_t)o0 * p.wo + ow0) * cwords + gw;
        if (wfull)
            ok = st_segment<kCPT, kRelu, true>(p, ts, len + 2, rp, slot0, full0, empty0, coff, rw4, yb, row_words,
                                               colmask, abort_flag, lane);
        else
            ok = st_segment<kCPT, kRelu, false>(p, ts, len + 2, rp, slot0, full0, empty0, coff, rw4, yb, row_words,
                                                colmask, abort_flag, lane);
    }
    // channels outside the fast range: exact outputs over the fast ones (same
    // thread, same addresses, later in program order)
    if (ok && !fast) st_exact_outputs<kCPT>(p, w, y, c0, ow0, r0, r1);
    return ok;
}

// The CTA's pieces of work: a lane and a row range of it (header comment).
// Call with pi = 0, 1, ...; returns false after the last piece.
__device__ __forceinline__ bool cta_piece(const DwStreamParams &p, int lanes, int pi, int &lane, int &r0, int &r1) {
    const int R = p.n * p.ho;
    const int main_ctas = lanes * p.per_lane;
    if ((int)blockIdx.x < main_ctas) {
        if (pi) return false;
        const int part = blockIdx.x / lanes;
        lane = blockIdx.x % lanes;
        r0 = (int)((long long)part * p.rows_main / p.per_lane);
        r1 = (int)((long long)(part + 1) * p.rows_main / p.per_lane);
        return r0 < r1;
    }
    // the tails of all lanes concatenated, split evenly over the extra CTAs
    const long long lt = R - p.rows_main, total = (long long)lanes * lt;
    const int e = blockIdx.x - main_ctas;
    long long g = (long long)e * total / p.extra;
    const long long g1 = (long long)(e + 1) * total / p.extra;
    for (int k = 0; g < g1; k++) {
        const int ln = (int)(g / lt);
        const long long end = std::min<long long>(g1, (long long)(ln + 1) * lt);
        if (k == pi) {
            lane = ln;
            r0 = p.rows_main + (int)(g - (long long)ln * lt);
            r1 = r0 + (int)(end - g);
            return true;
        }
        g = end;
    }
    return false;
}

template <int kShape, bool kRelu>
__global__ void __launch_bounds__(kStShapes[kShape].max_cons + 32, kStShapes[kShape].min_blocks)
    k_dwconv3x3_stream(const __grid_constant__ CUtensorMap tx, const int8_t *__restrict__ w, int8_t *__restrict__ y,
                       const __grid_constant__ DwStreamParams p) {
    constexpr int kCPT = kStShapes[kShape].cpt;
    extern __shared__ __align__(128) uint8_t smem[];
    uint64_t *full = reinterpret_cast<uint64_t *>(smem + (size_t)p.slots * p.slot_bytes);
    uint64_t *empty = full + kStreamMaxSlots;
    volatile int *abort_flag = reinterpret_cast<volatile int *>(empty + kStreamMaxSlots);
    const int cons_warps = p.cons_threads >> 5;
    const int lanes = p.groups * p.strips;

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
            int it = 0, s = 0;
            uint32_t ph = 0;  // parity of the pass over the ring
            bool ok = true;
            int my_lane, r0, r1;
            for (int pi = 0; ok && cta_piece(p, lanes, pi, my_lane, r0, r1); pi++) {
            const int grp = my_lane % p.groups, strip = my_lane / p.groups;
            for (int r = r0; r < r1 && ok;) {
                const int b = r / p.ho, o0 = r - b * p.ho;
                const int len = min(r1 - r, p.ho - o0);
                const int stages = (len + 2 + 2) / 3;
                for (int k = 0; k < stages; k++, it++) {
                    if (it >= p.slots && !st_wait(smem_u32(&empty[s]), ph ^ 1u, p, abort_flag, 30)) {
                        ok = false;
                        break;
                    }
                    mbar_expect_tx(smem_u32(&full[s]), p.stage_bytes);
                    tma_load_4d(smem_u32(smem + (size_t)s * p.slot_bytes), &tx, smem_u32(&full[s]),
                                grp * (p.cg >> 3), strip * p.cw - p.pl, o0 - p.pt + 3 * k, b);
                    if (++s == p.slots) {
                        s = 0;
                        ph ^= 1u;
                    }
                }
                r += len;
            }
            }
            // let the copies still in flight land before the CTA can exit
            for (int t = max(0, it - p.slots); t < it; t++) {
                const int sl = t % p.slots;
                const uint64_t t0 = globaltimer_ns();
                while (!mbar_try_wait(smem_u32(&full[sl]), (uint32_t)((t / p.slots) & 1)) &&
                       globaltimer_ns() - t0 < p.wait_cap_ns) {
                }
            }
        }
        return;
    }

    // ---------------------------------------------------------------- consumers
    const int full0 = smem_u32(full), empty0 = smem_u32(empty);
    // the thread's first word in slot 0 (its ring position starts there)
    const uint32_t slot0 = smem_u32(smem) + 4u * (uint32_t)((threadIdx.x / p.words) * kCPT * p.words +
                                                            threadIdx.x % p.words);
    RingPos rp{slot0, (uint32_t)full0, 0, 0u};
    int my_lane, r0, r1;
#pragma unroll 1
    for (int pi = 0; cta_piece(p, lanes, pi, my_lane, r0, r1); pi++)
        if (!st_piece<kCPT, kRelu>(p, w, y, my_lane, r0, r1, rp, slot0, (uint32_t)full0, (uint32_t)empty0,
                                   abort_flag))
            break;
}

struct StreamPlan {
    int cg = 0, groups = 0, cw = 0, q_per = 0, strips = 0;
};

// Picks the channel group (fewest groups), then the strip width: consumer
// threads words * q_per a multiple of 32 and at most max_cons, the least
// padding past the last output column, then the widest strip.
StreamPlan plan_stream(int c, int wo, int cpt, int max_cons) {
    StreamPlan best;
    for (int groups = 1; groups <= c / 16; groups++) {
        if (c % groups || (c / groups) % 16 || (c / groups) / 8 > 256) continue;
        const int cg = c / groups, words = cg / 4;
        const int wo_r = ((wo + cpt - 1) / cpt) * cpt;  // columns one strip needs at most
        long long best_waste = -1;
        for (int qp = 1; words * qp <= max_cons; qp++) {
            if ((words * qp) % 32) continue;
            const int cw = qp * cpt;
            if (cw + 2 > 256) break;
            const int strips = (wo + cw - 1) / cw;
            const long long waste = (long long)strips * cw - wo;
            if (best_waste < 0 || waste < best_waste || (waste == best_waste && cw > best.cw)) {
                best_waste = waste;
                best = StreamPlan{cg, groups, cw, qp, strips};
            }
            if (cw >= wo_r) break;  // wider strips only add idle columns
        }
        if (best.cw) return best;
    }
    return best;
}

// CTAs per SM for this instance at (threads, smem), cached per device; the first
// call on a device also raises the kernel's dynamic shared-memory limit there.
template <int kShape, bool kRelu>
int stream_occupancy(int device, int threads, size_t smem) {
    static bool attr_set[16] = {};
    static int cached[16][20][64] = {};
    if (device < 0 || device >= 16) return 1;
    if (!attr_set[device]) {
        cudaFuncSetAttribute(k_dwconv3x3_stream<kShape, kRelu>, cudaFuncAttributeMaxDynamicSharedMemorySize,
                             200 * 1024);
        attr_set[device] = true;
    }
    int &c = cached[device][std::min(19, threads / 32)][std::min<size_t>(63, smem / 4096)];
    if (!c) {
        int nb = 0;
        if (cudaOccupancyMaxActiveBlocksPerMultiprocessor(&nb, k_dwconv3x3_stream<kShape, kRelu>, threads, smem) !=
                cudaSuccess ||
            nb < 1)
            nb = 1;
        c = nb;
    }
    return c;
}

template <int kShape, bool kRelu>
dw_status launch_stream(dw_backend *be, const CUtensorMap &tx, const int8_t *w, int8_t *y, DwStreamParams &p,
                        size_t smem) {
    const int threads = p.cons_threads + 32;
    const int per_sm = stream_occupancy<kShape, kRelu>(be->device, threads, smem);
    const int lanes = p.groups * p.strips;
    const int rows = p.n * p.ho;
    const int slots_total = be->sm_count * per_sm;
    // main CTAs per lane: fill the SMs once, with at least ~24 output rows per
    // CTA so the two halo rows of a range stay a small overhead
    p.per_lane = std::max(1, std::min(slots_total / lanes, rows / 24));
    p.rows_main = rows;
    p.extra = 0;
    const int spare = slots_total - lanes * p.per_lane;
    if (spare > 0 && p.per_lane == slots_total / lanes) {
        // the spare SMs take the lanes' tails: every CTA streams about
        // lanes * rows / slots_total rows
        const long long main_rows = (long long)rows * lanes * p.per_lane / slots_total;
        const long long tail_rows = (long long)lanes * (rows - main_rows);
        if (main_rows >= p.per_lane && tail_rows / spare >= 24) {
            p.rows_main = (int)main_rows;
            p.extra = spare;
        }
    }
    const long long ctas = (long long)lanes * p.per_lane + p.extra;
    if (ctas >= (1ll << 31)) return DW_ERR_UNSUPPORTED;
    k_dwconv3x3_stream<kShape, kRelu><<<(unsigned)ctas, threads, smem, be->stream>>>(tx, w, y, p);
    return dw_after_launch(be, "dwconv3x3_stream_i8");
}

}  // namespace

// Returns DW_ERR_UNSUPPORTED (without launching) when the shape does not fit
// the kernel: stride 1, 3x3, multiplier 1, c % 16 == 0 with a lane plan, no
// SiLU.  `shape` indexes kStShapes.
dw_status launch_dwconv3x3_stream_i8(dw_backend *be, const dw_conv_desc &d, int ho, int wo, const int8_t *x,
                                     const int8_t *w_hwcm, const EpiParams &ep, int8_t *y, int shape) {
    if (!be->encode_tiled || d.k_h != 3 || d.k_w != 3 || d.stride_h != 1 || d.stride_w != 1 ||
        d.c_out != d.c_in || d.c_in % 16 || ((uintptr_t)x & 15) || ((uintptr_t)y & 3) || ((uintptr_t)w_hwcm & 3) ||
        shape < 0 || shape > 2 || ep.epilogue == DW_EPI_SILU)
        return DW_ERR_UNSUPPORTED;
    const StShape &sh = kStShapes[shape];
    const StreamPlan pl = plan_stream(d.c_in, wo, sh.cpt, sh.max_cons);
    if (!pl.cw) return DW_ERR_UNSUPPORTED;
    DwStreamParams p{};
    p.n = d.n; p.h = d.h; p.w = d.w; p.c = d.c_in; p.ho = ho; p.wo = wo; p.pt = d.pad_t; p.pl = d.pad_l;
    p.cg = pl.cg;
    p.words = pl.cg / 4;
    p.groups = pl.groups;
    p.cw = pl.cw;
    p.strips = pl.strips;
    p.bw = pl.cw + 2;
    p.stage_bytes = 3u * (uint32_t)(p.bw * p.cg);
    p.slot_bytes = (p.stage_bytes + 127) & ~127u;
    p.cons_threads = p.words * pl.q_per;
    // ring: 3..8 stages in about 200 KB per SM
    const uint32_t budget = (200u * 1024u) / (uint32_t)sh.min_blocks;
    p.slots = (int)std::min<uint32_t>(kStreamMaxSlots, budget / p.slot_bytes);
    if (p.slots < 3) return DW_ERR_UNSUPPORTED;
    if ((long long)d.n * ho >= (1ll << 31)) return DW_ERR_UNSUPPORTED;
    if (d.n == 0 || ho <= 0 || wo <= 0) return DW_OK;
    p.x = x;
    p.wait_cap_ns = be->wait_cap_ns;
    p.err = be->dev_err;
    p.ep = ep;

    // the input viewed as 8-byte elements: (c / 8, w, h, n); a box is cg / 8
    // elements x bw columns x 3 rows of one image
    CUtensorMap tx;
    cuuint64_t dims[4] = {(cuuint64_t)(d.c_in / 8), (cuuint64_t)d.w, (cuuint64_t)d.h, (cuuint64_t)d.n};
    cuuint64_t strides[3] = {(cuuint64_t)d.c_in, (cuuint64_t)d.w * d.c_in, (cuuint64_t)d.h * d.w * d.c_in};
    cuuint32_t box[4] = {(cuuint32_t)(p.cg / 8), (cuuint32_t)p.bw, 3, 1};
    cuuint32_t estr[4] = {1, 1, 1, 1};
    CUresult r = be->encode_tiled(&tx, CU_TENSOR_MAP_DATA_TYPE_UINT64, 4, const_cast<int8_t *>(x), dims, strides, box,
                                  estr, CU_TENSOR_MAP_INTERLEAVE_NONE, CU_TENSOR_MAP_SWIZZLE_NONE,
                                  CU_TENSOR_MAP_L2_PROMOTION_L2_256B, CU_TENSOR_MAP_FLOAT_OOB_FILL_NONE);
    if (r != CUDA_SUCCESS) return DW_ERR_UNSUPPORTED;
    const size_t smem = (size_t)p.slots * p.slot_bytes + 2 * kStreamMaxSlots * sizeof(uint64_t) + 16;
    const bool relu = ep.epilogue == DW_EPI_RELU || ep.epilogue == DW_EPI_RELU6;
    switch (shape) {
    case 0: return relu ? launch_stream<0, true>(be, tx, w_hwcm, y, p, smem) : launch_stream<0, false>(be, tx, w_hwcm, y, p, smem);
    case 1: return relu ? launch_stream<1, true>(be, tx, w_hwcm, y, p, smem) : launch_stream<1, false>(be, tx, w_hwcm, y, p, smem);
    default: return relu ? launch_stream<2, true>(be, tx, w_hwcm, y, p, smem) : launch_stream<2, false>(be, tx, w_hwcm, y, p, smem);
    }
}

}  // namespace dw
