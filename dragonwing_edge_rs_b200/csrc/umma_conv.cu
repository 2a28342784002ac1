// umma_conv.cu -- tcgen05 (5th-gen tensor core) implicit-GEMM int8 convolution
// with the fused requantisation epilogue, for sm_100a.
//
// GEMM view: rows = output pixels (M), columns = output channels (N),
// K = (kh, kw, c_in).  One CTA per SM (persistent), warp-specialised:
//   warp 0      : TMA producer -- per k-block, one A box (activations) and one
//                 B box (weights) into a ring of shared-memory stages;
//   warp 1      : TMEM allocator + MMA issuer -- tcgen05.mma.cta_group::1.kind::i8,
//                 128 x BN x 32 per instruction, int32 accumulators in TMEM,
//                 double-buffered so the epilogue of tile i overlaps tile i+1;
//   warps 2..9  : epilogue -- tcgen05.ld accumulators, bias + per-channel
//                 requant (bit-exact with the reference scalar path) + ReLU/ReLU6/SiLU,
//                 int8 stores to NHWC.
//
// Activation tiles come from TMA boxes of the NHWC input, viewed as a 5-D tensor
// (c', w', ph, h', n) with c' = (w mod sw)*C + c, w' = w / sw, ph = h mod sh,
// h' = h / sh, so every box is unit-stride and a stride-s conv reads, for tap
// (kh, kw), the box at w' = ow0 + floor((kw-pl)/sw), parity (kw-pl) mod sw (and
// the same along h).  Out-of-range coordinates (the conv's zero padding) are
// zero-filled by TMA.  1x1 stride-1 convs and QGemm use a flat 2-D view
// [pixels, C] instead (no spatial tile waste).  The weight operand is the
// prepared OHWI tensor viewed as (c_in, tap, c_out); channels past c_in in the
// last k-block are zero-filled, so whatever the A box holds there contributes 0.
//
// Every mbarrier wait is bounded (globaltimer); on expiry the CTA records the
// failure in the backend's device error word, stops issuing, waits (bounded)
// for its own TMA copies in flight, frees its TMEM and exits.  No multicast
// TMA is used anywhere (the same code runs on 1..8 GPUs).

#include <algorithm>
#include <tuple>
#include <cstdlib>

#include "dw_device.cuh"
#include "dw_ptx.cuh"

namespace dw {
namespace {

constexpr int kBM = 128;            // MMA M (rows per tile = pixels)
// Warp roles: 0 producer, 1 MMA, then the epilogue warps (4 per part: warps
// sharing a TMEM lane quarter split its (row block, chunk) items), then the
// store warp, then a second MMA warp (tiles of several row blocks: the two
// issue alternate row blocks -- one thread issues a tcgen05.mma only every
// ~50 cycles, and the issue competes with the epilogue for its scheduler).  The int8 SiLU epilogue (issue-bound) runs 16 epilogue warps, four
// streams per scheduler at 96 registers a thread (YOLOv8n b32's stem conv 125 ->
// 111 us, the step 1.995 -> 1.971 ms); the others keep 12 at 128 registers
// (with 16 the ReLU6 / linear int8 epilogue spills and the MobileNetV2 block
// went 0.336 -> 0.351 ms; the fp16 epilogue keeps two TMEM loads in flight per
// wait instead of four).
constexpr int epi_warps(bool silu, bool f16) { return (silu && !f16) ? 16 : 12; }
constexpr int umma_threads(bool silu, bool f16) { return 64 + 32 * epi_warps(silu, f16) + 64; }
constexpr int kMaxStages = 12;

struct UmmaParams {
    // geometry
    int mode;            // 0 = flat GEMM rows, 1 = spatial tiles
    int n_img, ho, wo, c_out;
    int tw, th, nb;      // spatial tile: tw x th pixels of nb images (tw*th*nb <= 128; nb > 1 only for whole images)
    int tiles_w, tiles_h;
    int m_tiles, n_tiles, num_tiles;
    long long rows;      // flat mode: total pixels
    int taps, k_h, kw, sh, sw, pt, pl, c_in;
    int cblocks;         // k-blocks per tap
    int bk;              // bytes of K per stage (32/64/128)
    int bn;              // N per tile
    int stages;
    uint32_t a_stage_bytes, b_stage_bytes;  // smem per stage (1 KiB aligned)
    uint32_t a_tx_bytes, b_tx_bytes;        // bytes TMA delivers per stage
    uint32_t idesc;
    uint64_t desc_hi;    // constant upper 32 bits of the smem descriptors
    uint32_t tmem_cols;
    uint32_t off_out, off_chan, off_bars;   // shared-memory layout (bytes from the 1 KiB-aligned base)
    long long acc_bound;                    // |acc| <= taps * c_in * 128 * 128
    int R;                                  // 128-row blocks per tile (R * bn <= 256)
    int chan_all;                           // 1: every output channel's parameters staged once per CTA
    int esize;                              // element bytes: 1 (int8) or 2 (fp16)
    int bk_elems;                           // bk / esize: K elements per stage
    const uint16_t *bias_f16;               // fp16 path: bias [c_out] (may be null)
    const uint16_t *res_f16;                // fp16 path, flat mode: residual [rows][c_out] added (may be null)
    float add_ra, add_rb;                   // int8 residual (kFm & 2): y = add_i8(residual, conv) with these ratios
    int relu;                               // fp16 path: ReLU last (after the bias and the residual)
    int swz;                                // fp16 path: staging in 64-channel slabs, 128-byte swizzle (bn % 64 == 0)
    int nbuf;                               // staging buffers (2: a tile's store overlaps the next tile's epilogue)
    uint32_t out_bytes;                     // bytes of one staging buffer
    // mode 2 (halo tiles, stride-1 convs with several taps): the A operand of a
    // K block is one zero-padded halo tile per 16-byte channel chunk, planes of
    // [hh rows][hw columns][16 bytes]; output tiles are 8 columns x 16 rows per
    // 128-row block, so the 8 rows of a core matrix are 8 neighbouring pixels
    // and each tap is the same tile read at a shifted start address.
    int hw, hh;                             // halo columns (8 + k_w - 1) and rows (16 R + k_h - 1)
    int chunks;                             // 16-byte channel chunks of c_in
    int cps;                                // chunks per K block (bk / 16)
    int chunk_elems;                        // elements per chunk (16 / esize)
    uint32_t plane_stride;                  // bytes between chunk planes of a stage (128-byte aligned)
    uint32_t b_tap_bytes;                   // bytes of one tap's weight slice in a stage (bn * bk)
    int rw;                                 // row blocks side by side in a tile (R / rw stacked); 1 outside mode 2
    int wres;                               // mode 2: every weight of the (single) channel tile resident in
                                            // shared memory, loaded once per CTA; stages carry halo planes only
    uint32_t off_w, w_bytes;                // resident weights: offset and bytes ([tap][K block][bn][bk])
    int tpair;                              // resident weights of a 16-byte channel row: [tap + 1][bn][16 B]
                                            // slices without swizzle (the last all zero), so that one 32-byte
                                            // K step takes two horizontal taps
    int n_issuers;                          // MMA warps (2: alternate row blocks; 1 when R == 1)
    int epi_pipe;                           // int8 epilogue without SiLU: the next TMEM load in flight
                                            // during the requantisation (convs with several taps, whose
                                            // MMAs overlap the epilogue; a kernel instance of its own),
                                            // else two loads per wait
    int s2;                                 // mode 2 for a stride-2 conv: a stride-1 conv over the input's
                                            // four (row, column) parity planes, x'[i][j][(ph, pw, c)] =
                                            // x[2i + ph][2j + pw][c]: chunk j of x' is parity plane
                                            // (ph, pw) = (j / (2 chunks0), j / chunks0 % 2) of 16-byte
                                            // channel chunk j % chunks0; taps (dy, dx) of tkh x tkw from
                                            // (dy0, dx0); weights resident as 16-byte slices [tap][chunk]
    int tkh, tkw, dy0, dx0;
    int flat_in;                            // mode 2, a dense 16-byte channel row: the activation map is
                                            // [n][h][w * 16 bytes], so a halo tile is one box of hh rows of
                                            // hw * 16 contiguous bytes (not hw * hh 16-byte rows)
    int flat_out;                           // mode 2, int8 output of exactly bn dense channels: the output
                                            // map is [n][ho][wo * bn bytes]; a row block stores as 16 rows
                                            // of 8 * bn bytes (not 128 rows of bn bytes)
    uint64_t wait_cap_ns;
    int32_t *err;
    EpiParams ep;
};

// Channel parameters staged in shared memory (structure of arrays).  With
// c_out <= kChanSlots every channel is staged once when the CTA starts (slot =
// channel); otherwise each tile stages its bn channels into half `acc` of the
// slots (slot = acc * kChanSlots / 2 + local channel).
constexpr int kChanSlots = 1024;
struct ChanSmem {
    int32_t bias[kChanSlots];
    float m[kChanSlots];
    float d[kChanSlots];
    uint32_t cflags[kChanSlots / 16];  // per 16 slots: bit0 = fast-path inputs finite, bit1 = |acc+bias| < 2^22 certain, bit2 = the one-add ReLU path applies
};






// Bounded wait: true when the phase with `parity` completed; false when the
// CTA is aborting or the cap expired (then the failure is recorded).
__device__ __forceinline__ bool mbar_wait(uint32_t bar, uint32_t parity, const UmmaParams &p,
                                          volatile int *abort_flag, int site) {
    // The MMA warp's wait for a loaded stage (site 3) and the epilogue's wait for
    // its accumulators (site 4) poll first: they are usually only a little late,
    // and a thread woken from a suspended try_wait resumes late.  The other
    // waits (a free stage, a free accumulator or staging buffer, a staged tile)
    // are long and each poll is an instruction issued beside the epilogue warps
    // of the same scheduler: they suspend at once (measured on B200: MobileNetV2's
    // expand 173 -> 166 us, YOLOv8n b32 1.809 -> 1.797 ms).  Then all wait
    // suspended in hardware while the phase stays open (at most ~20 us per try).
    if (mbar_test_wait(bar, parity)) return true;
    const int polls = (site == 3 || site == 4) ? 256 : 0;
#pragma unroll 1
    for (int i = 0; i < polls; i++)
        if (mbar_try_wait(bar, parity)) return true;
    const uint64_t t0 = globaltimer_ns();
#pragma unroll 1
    for (;;) {
        if (mbar_try_wait_sleep(bar, parity, 20000u)) return true;
        if (*abort_flag) return false;
        if (globaltimer_ns() - t0 > p.wait_cap_ns) {
            *abort_flag = 1;
            record_error(p.err, DW_DEV_WAIT_EXPIRED, site, (int)parity);
            return false;
        }
    }
}




__device__ __forceinline__ void tc_fence_before() { asm volatile("tcgen05.fence::before_thread_sync;" ::: "memory"); }
__device__ __forceinline__ void tc_fence_after() { asm volatile("tcgen05.fence::after_thread_sync;" ::: "memory"); }

__device__ __forceinline__ void tc_mma_i8(uint32_t d_tmem, uint64_t adesc, uint64_t bdesc, uint32_t idesc,
                                          uint32_t accumulate) {
    asm volatile(
        "{\n\t.reg .pred p;\n\t"
        "setp.ne.b32 p, %4, 0;\n\t"
        "tcgen05.mma.cta_group::1.kind::i8 [%0], %1, %2, %3, p;\n\t}" ::"r"(d_tmem),
        "l"(adesc), "l"(bdesc), "r"(idesc), "r"(accumulate)
        : "memory");
}

// kind::f16: A = B = fp16 (instruction descriptor formats 0), D = f32 in TMEM.
__device__ __forceinline__ void tc_mma_f16(uint32_t d_tmem, uint64_t adesc, uint64_t bdesc, uint32_t idesc,
                                           uint32_t accumulate) {
    asm volatile(
        "{\n\t.reg .pred p;\n\t"
        "setp.ne.b32 p, %4, 0;\n\t"
        "tcgen05.mma.cta_group::1.kind::f16 [%0], %1, %2, %3, p;\n\t}" ::"r"(d_tmem),
        "l"(adesc), "l"(bdesc), "r"(idesc), "r"(accumulate)
        : "memory");
}

template <bool kF16>
__device__ __forceinline__ void tc_mma(uint32_t d_tmem, uint64_t adesc, uint64_t bdesc, uint32_t idesc,
                                       uint32_t accumulate) {
    if (kF16)
        tc_mma_f16(d_tmem, adesc, bdesc, idesc, accumulate);
    else
        tc_mma_i8(d_tmem, adesc, bdesc, idesc, accumulate);
}

__device__ __forceinline__ void tc_commit(uint32_t bar) {
    asm volatile("tcgen05.commit.cta_group::1.mbarrier::arrive::one.shared::cluster.b64 [%0];" ::"r"(bar) : "memory");
}

// 32 lanes x 16 columns of 32-bit accumulators -> 16 registers per thread.
__device__ __forceinline__ void tc_ld16(uint32_t taddr, int32_t (&r)[16]) {
    asm volatile(
        "tcgen05.ld.sync.aligned.32x32b.x16.b32 {%0, %1, %2, %3, %4, %5, %6, %7, %8, %9, %10, %11, %12, %13, %14, "
        "%15}, [%16];"
        : "=r"(r[0]), "=r"(r[1]), "=r"(r[2]), "=r"(r[3]), "=r"(r[4]), "=r"(r[5]), "=r"(r[6]), "=r"(r[7]),
          "=r"(r[8]), "=r"(r[9]), "=r"(r[10]), "=r"(r[11]), "=r"(r[12]), "=r"(r[13]), "=r"(r[14]), "=r"(r[15])
        : "r"(taddr)
        : "memory");
}

__device__ __forceinline__ void tc_wait_ld() { asm volatile("tcgen05.wait::ld.sync.aligned;" ::: "memory"); }






// ---------------------------------------------------------------- epilogue math
// Loads channel `oc`'s parameters into `slot` and derives the per-16-slot
// fast-path flags.  Called by every epilogue thread (the ballots need whole
// warps; 16 consecutive slots live in one half-warp); `write` selects the
// threads that own a slot.
__device__ __forceinline__ void stage_channel(const UmmaParams &p, ChanSmem *cs, int slot, int oc, bool write) {
    int32_t bias = 0;
    float m = 0.0f, dsc = 0.0f;
    if (p.esize == 2) {
        // fp16 path: `bias` holds the f16 bias bits, `m` the bias as F16::to_f32
        // gives it; flag bit0 = some bias of the 16-slot group is a nonzero
        // subnormal or a NaN (the packed fast path does not reproduce those).
        const uint16_t hb = (write && oc < p.c_out && p.bias_f16) ? p.bias_f16[oc] : (uint16_t)0;
        const bool special = ((hb & 0x7C00u) == 0 && (hb & 0x03FFu) != 0) || ((hb & 0x7C00u) == 0x7C00u && (hb & 0x03FFu));
        const uint32_t bsp = __ballot_sync(0xffffffffu, special);
        const uint32_t hb_next = __shfl_down_sync(0xffffffffu, (uint32_t)hb, 1);
        if (write) {
            cs->bias[slot] = hb;
            cs->m[slot] = f16_to_f32_ref(hb);
            // packed (even, odd) channel pairs for the epilogue's half2 loads
            if ((slot & 1) == 0) reinterpret_cast<uint32_t *>(cs->d)[slot >> 1] = (uint32_t)hb | (hb_next << 16);
        }
        const int ln = threadIdx.x & 31;
        if ((ln & 15) == 0 && write) cs->cflags[slot >> 4] = ((bsp >> ln) & 0xFFFFu) ? 1u : 0u;
        return;
    }
    if (write && oc < p.c_out) {
        bias = p.ep.bias ? __ldg(p.ep.bias + oc) : 0;
        m = p.ep.M ? __ldg(p.ep.M + oc) : 0.0f;
        dsc = p.ep.D ? __ldg(p.ep.D + oc) : 0.0f;
    }
    // bit0: the fast path's float inputs are finite (M, or D and 1/s_out for SiLU)
    const bool finite = p.ep.epilogue == DW_EPI_SILU ? (isfinite(dsc) && isfinite(p.ep.inv_s_out)) : isfinite(m);
    const long long b = bias < 0 ? -(long long)bias : (long long)bias;
    const bool safe = p.acc_bound + b < (1ll << 22);
    // bit2: the ReLU path with one directed-rounding add applies: |v| =
    // |(acc + bias) * M| < 2^21 for every accumulator (kept below 2e6), so
    // v + 1.5 * 2^22 + 0.5 stays in [2^22, 2^23)
    const bool r16 = safe && isfinite(m) && fabsf(m) * (float)(p.acc_bound + b) < 2.0e6f;
    // bit3: the same path applies to any tile whose |acc + bias| < 2^22 (checked
    // per 16 accumulators by the epilogue): |M| < 0.47 keeps |v| below 2e6 there
    const bool mfast = isfinite(m) && fabsf(m) < 0.47f;
    const uint32_t bf = __ballot_sync(0xffffffffu, finite);
    const uint32_t bs = __ballot_sync(0xffffffffu, safe);
    const uint32_t br = __ballot_sync(0xffffffffu, r16);
    const uint32_t bm = __ballot_sync(0xffffffffu, mfast);
    if (write) {
        cs->bias[slot] = bias;
        cs->m[slot] = m;
        // SiLU: the dequant scale; otherwise the bias plus the bit pattern of
        // 1.5 * 2^23, so acc + d read as a float is 1.5 * 2^23 + acc + bias
        cs->d[slot] = p.ep.epilogue == DW_EPI_SILU ? dsc : __int_as_float(bias + kMagicBits);
    }
    const int lane = threadIdx.x & 31;
    if ((lane & 15) == 0 && write) {
        const uint32_t sh = lane;  // 0 or 16
        const uint32_t f = (((bf >> sh) & 0xFFFFu) == 0xFFFFu ? 1u : 0u) | (((bs >> sh) & 0xFFFFu) == 0xFFFFu ? 2u : 0u) |
                           (((br >> sh) & 0xFFFFu) == 0xFFFFu ? 4u : 0u) | (((bm >> sh) & 0xFFFFu) == 0xFFFFu ? 8u : 0u);
        cs->cflags[slot >> 4] = f;
    }
}


// 16 accumulators (16 consecutive channels of one row) -> 16 int8, packed.
// kSilu selects the SiLU epilogue at compile time (separate kernel instances keep
// each epilogue's code out of the other's instruction stream).
template <bool kSilu>
__device__ __forceinline__ uint4 requant16(const int32_t (&v)[16], const ChanSmem *cs, int slot0,
                                           const UmmaParams &p) {
    const int epi = kSilu ? DW_EPI_SILU : p.ep.epilogue;
    const int32_t *sb = &cs->bias[slot0];
    const float *sm = &cs->m[slot0];
    uint32_t w[4] = {0u, 0u, 0u, 0u};
    const uint32_t fl = cs->cflags[slot0 >> 4];
    if (kSilu) {
        // the 16 channels' bias and dequant scale D (shared loads, the same for all lanes)
        const uint32_t ba = smem_u32(sb), dd = smem_u32(&cs->d[slot0]);
        const uint4 b4[4] = {lds_v4(ba), lds_v4(ba + 16), lds_v4(ba + 32), lds_v4(ba + 48)};
        const uint4 s4[4] = {lds_v4(dd), lds_v4(dd + 16), lds_v4(dd + 32), lds_v4(dd + 48)};
        const int32_t *bv = reinterpret_cast<const int32_t *>(b4);
        const float *sd = reinterpret_cast<const float *>(s4);
        int32_t a[16];
        bool inrange = true;
#pragma unroll
        for (int k = 0; k < 16; k++) a[k] = (int32_t)((uint32_t)v[k] + (uint32_t)bv[k]);
        if (!(fl & 2u)) {
#pragma unroll
            for (int k = 0; k < 16; k++) inrange &= (uint32_t)(a[k] + (1 << 22)) < (1u << 23);
        }
        uint32_t unc = 0xFFFFu;  // elements still to compute exactly
        if ((fl & 1u) && __all_sync(0xffffffffu, inrange)) {
            unc = 0;
#pragma unroll
            for (int q = 0; q < 4; q++) {
                uint32_t bq[4];
#pragma unroll
                for (int j = 0; j < 4; j += 2) {
                    bool u0 = false, u1 = false;
                    silu_fast_bits2(a[q * 4 + j], a[q * 4 + j + 1], sd[q * 4 + j], sd[q * 4 + j + 1], p.ep.inv_s_out,
                                    bq[j], bq[j + 1], u0, u1);
                    unc |= ((uint32_t)u0 | (uint32_t)u1 << 1) << (q * 4 + j);
                }
                w[q] = __byte_perm(__byte_perm(bq[0], bq[1], 0x0040), __byte_perm(bq[2], bq[3], 0x0040), 0x5410);
            }
        }
        if (__any_sync(0xffffffffu, unc != 0)) {
#pragma unroll
            for (int k = 0; k < 16; k++) {
                if (unc & (1u << k)) {
                    const uint32_t b = (uint8_t)epilogue_one_slow(v[k], bv[k], 0.0f, sd[k], epi, p.ep.q6, p.ep.inv_s_out);
                    const int q = k >> 2, sh = 8 * (k & 3);
                    w[q] = (w[q] & ~(0xFFu << sh)) | (b << sh);
                }
            }
        }
        return make_uint4(w[0], w[1], w[2], w[3]);
    }
    if ((epi == DW_EPI_RELU || (epi == DW_EPI_RELU6 && p.ep.q6 >= 0)) && __all_sync(0xffffffffu, (fl & 12u) != 0)) {
        // ReLU / ReLU6, exact and branch-free: v = fl((acc + bias) * M) as the
        // reference (acc + bias + magic bits read as a float, minus 1.5 * 2^23);
        // one add rounded toward zero of 1.5 * 2^22 + 0.5 (the spacing there is
        // 0.5) gives 1.5 * 2^22 + floor(2 v + 1) / 2, whose bits minus those of
        // 1.5 * 2^22 are floor(2 v + 1); clamped to [0, 2 hi + 1] in one integer
        // op and halved, that is clamp(floor(v + 0.5), 0, hi), which equals the
        // ReLU-bounded roundf(v) (floor(v + 0.5) == roundf(v) for v >= 0, both
        // <= 0 below zero; the bounds are integers).  The compiler does not
        // fuse the round-to-nearest multiply into the round-toward-zero add
        // (the rounding modes differ), so v is rounded as the reference rounds it.
        // the 16 channels' bias + magic bits and M (shared loads, the same for all lanes)
        const uint32_t da = smem_u32(&cs->d[slot0]), ma = smem_u32(&cs->m[slot0]);
        const uint4 d4[4] = {lds_v4(da), lds_v4(da + 16), lds_v4(da + 32), lds_v4(da + 48)};
        const uint4 m4[4] = {lds_v4(ma), lds_v4(ma + 16), lds_v4(ma + 32), lds_v4(ma + 48)};
        const int32_t *bm = reinterpret_cast<const int32_t *>(d4);
        const float *mm = reinterpret_cast<const float *>(m4);
        // u = acc + bias + the magic bits (wrapping, as the reference's i32 add)
        uint32_t u[16];
#pragma unroll
        for (int k = 0; k < 16; k++) u[k] = (uint32_t)v[k] + (uint32_t)bm[k];
        bool fast = true;
        if (!(fl & 4u)) {
            // the shape's bound on |acc| does not keep acc + bias within 2^22: check
            // these 16 (u - magic + 2^22 in [0, 2^23) for each; one OR covers all)
            uint32_t orr = 0;
#pragma unroll
            for (int k = 0; k < 16; k++) orr |= u[k] - (uint32_t)(kMagicBits - (1 << 22));
            fast = orr < (1u << 23);
        }
        if (__all_sync(0xffffffffu, fast)) {
        const int hi = epi == DW_EPI_RELU6 ? min(p.ep.q6, 127) : 127;
        const float2 nmag = make_float2(-kMagic, -kMagic);
        const float2 mag = make_float2(6291456.5f, 6291456.5f);  // 1.5 * 2^22 + 0.5
#pragma unroll
        for (int q = 0; q < 4; q++) {
            int32_t t[4];
#pragma unroll
            for (int h = 0; h < 2; h++) {
                const int k0 = q * 4 + 2 * h;
                const float2 f = __fadd2_rn(make_float2(__uint_as_float(u[k0]), __uint_as_float(u[k0 + 1])), nmag);
                const float2 r = __fadd2_rz(__fmul2_rn(f, make_float2(mm[k0], mm[k0 + 1])), mag);
                t[2 * h] = __viaddmin_s32_relu(__float_as_int(r.x), -0x4AC00000, 2 * hi + 1);
                t[2 * h + 1] = __viaddmin_s32_relu(__float_as_int(r.y), -0x4AC00000, 2 * hi + 1);
            }
            const uint32_t packed = __byte_perm(__byte_perm(t[0], t[1], 0x0040), __byte_perm(t[2], t[3], 0x0040), 0x5410);
            w[q] = (packed >> 1) & 0x7F7F7F7Fu;
        }
        return make_uint4(w[0], w[1], w[2], w[3]);
        }
    }
    const uint32_t ba = smem_u32(sb), ma = smem_u32(sm);
    const uint4 b4[4] = {lds_v4(ba), lds_v4(ba + 16), lds_v4(ba + 32), lds_v4(ba + 48)};
    const uint4 m4[4] = {lds_v4(ma), lds_v4(ma + 16), lds_v4(ma + 32), lds_v4(ma + 48)};
    const int32_t *bb = reinterpret_cast<const int32_t *>(b4);
    const float *mm = reinterpret_cast<const float *>(m4);
    bool inrange = true;
    if (!(fl & 2u)) {
#pragma unroll
        for (int k = 0; k < 16; k++)
            inrange &= (uint32_t)((int32_t)((uint32_t)v[k] + (uint32_t)bb[k]) + (1 << 22)) < (1u << 23);
    }
    if ((fl & 1u) && __all_sync(0xffffffffu, inrange)) {
        // Packed f32x2: acc + (bias + magic bits) read as a float is 1.5 * 2^23 +
        // acc + bias exactly; minus 1.5 * 2^23 gives the float, times M rounded
        // once; the clamp (ReLU / ReLU6 bounds included: roundf commutes with a
        // clamp to integer bounds) and rint-to-even by one RN add.  A
        // round-half-away tie can only differ from it when c - rint(c) == +-0.5
        // exactly: such chunks (rare) are redone with the per-element tie fix.
        const uint32_t da = smem_u32(&cs->d[slot0]);
        const uint4 d4[4] = {lds_v4(da), lds_v4(da + 16), lds_v4(da + 32), lds_v4(da + 48)};
        const int32_t *bm = reinterpret_cast<const int32_t *>(d4);
        const float lo = (epi == DW_EPI_RELU || epi == DW_EPI_RELU6) ? 0.0f : -128.0f;
        const float hi = epi == DW_EPI_RELU6 ? (float)p.ep.q6 : 127.0f;
        const float2 mag = make_float2(kMagic, kMagic), nmag = make_float2(-kMagic, -kMagic);
        const float2 neg1 = make_float2(-1.0f, -1.0f);
        bool tie = false;
#pragma unroll
        for (int q = 0; q < 4; q++) {
            uint32_t bq[4];
#pragma unroll
            for (int h = 0; h < 2; h++) {
                const int k0 = q * 4 + 2 * h;
                const float2 f = __fadd2_rn(make_float2(__int_as_float((int32_t)((uint32_t)v[k0] + (uint32_t)bm[k0])),
                                                        __int_as_float((int32_t)((uint32_t)v[k0 + 1] + (uint32_t)bm[k0 + 1]))),
                                            nmag);
                float2 c = __fmul2_rn(f, make_float2(mm[k0], mm[k0 + 1]));
                c.x = fminf(fmaxf(c.x, lo), hi);
                c.y = fminf(fmaxf(c.y, lo), hi);
                const float2 r = __fadd2_rn(c, mag);
                const float2 d = __ffma2_rn(__fadd2_rn(r, nmag), neg1, c);  // c - rint(c), exact
                tie |= fmaxf(fabsf(d.x), fabsf(d.y)) == 0.5f;
                bq[2 * h] = __float_as_uint(r.x);
                bq[2 * h + 1] = __float_as_uint(r.y);
            }
            w[q] = __byte_perm(__byte_perm(bq[0], bq[1], 0x0040), __byte_perm(bq[2], bq[3], 0x0040), 0x5410);
        }
        if (__any_sync(0xffffffffu, tie)) {
#pragma unroll
            for (int q = 0; q < 4; q++) {
                uint32_t packed = 0;
#pragma unroll
                for (int j = 0; j < 4; j++) {
                    const int k = q * 4 + j;
                    packed |= (uint32_t)(uint8_t)epilogue_one_slow(v[k], bb[k], mm[k], 0.0f, epi, p.ep.q6,
                                                                  p.ep.inv_s_out)
                              << (8 * j);
                }
                w[q] = packed;
            }
        }
    } else {
#pragma unroll
        for (int q = 0; q < 4; q++) {
            uint32_t packed = 0;
#pragma unroll
            for (int j = 0; j < 4; j++) {
                const int k = q * 4 + j;
                packed |= (uint32_t)(uint8_t)epilogue_one_slow(v[k], bb[k], mm[k], 0.0f, epi, p.ep.q6, p.ep.inv_s_out)
                          << (8 * j);
            }
            w[q] = packed;
        }
    }
    return make_uint4(w[0], w[1], w[2], w[3]);
}


// Two row blocks' accumulators of the same 16 channels (one channel chunk):
// the ReLU / ReLU6 one-add path with the channels' parameters, flags and votes
// taken once and the two chunks' arithmetic interleaved (the epilogue is
// latency-bound at three warps per scheduler: MobileNetV2's expand 156 -> 146 us
// on B200); anything else goes through requant16 for each.
template <bool kSilu>
__device__ __forceinline__ void requant16x2(const int32_t (&v1)[16], const int32_t (&v2)[16], const ChanSmem *cs, int slot0,
                                            const UmmaParams &p, uint4 &o1, uint4 &o2) {
    const int epi = kSilu ? DW_EPI_SILU : p.ep.epilogue;
    const uint32_t fl = cs->cflags[slot0 >> 4];
    if (!kSilu && (epi == DW_EPI_RELU || (epi == DW_EPI_RELU6 && p.ep.q6 >= 0)) && __all_sync(0xffffffffu, (fl & 12u) != 0)) {
        const uint32_t da = smem_u32(&cs->d[slot0]), ma = smem_u32(&cs->m[slot0]);
        const uint4 d4[4] = {lds_v4(da), lds_v4(da + 16), lds_v4(da + 32), lds_v4(da + 48)};
        const uint4 m4[4] = {lds_v4(ma), lds_v4(ma + 16), lds_v4(ma + 32), lds_v4(ma + 48)};
        const int32_t *bm = reinterpret_cast<const int32_t *>(d4);
        const float *mm = reinterpret_cast<const float *>(m4);
        uint32_t u1[16], u2[16];
#pragma unroll
        for (int k = 0; k < 16; k++) {
            u1[k] = (uint32_t)v1[k] + (uint32_t)bm[k];
            u2[k] = (uint32_t)v2[k] + (uint32_t)bm[k];
        }
        bool fast = true;
        if (!(fl & 4u)) {
            uint32_t orr = 0;
#pragma unroll
            for (int k = 0; k < 16; k++) orr |= (u1[k] - (uint32_t)(kMagicBits - (1 << 22))) | (u2[k] - (uint32_t)(kMagicBits - (1 << 22)));
            fast = orr < (1u << 23);
        }
        if (__all_sync(0xffffffffu, fast)) {
            const int hi = epi == DW_EPI_RELU6 ? min(p.ep.q6, 127) : 127;
            const float2 nmag = make_float2(-kMagic, -kMagic);
            const float2 mag = make_float2(6291456.5f, 6291456.5f);  // 1.5 * 2^22 + 0.5
            uint32_t w1[4], w2[4];
#pragma unroll
            for (int q = 0; q < 4; q++) {
                int32_t t1[4], t2[4];
#pragma unroll
                for (int h = 0; h < 2; h++) {
                    const int k0 = q * 4 + 2 * h;
                    const float2 mk = make_float2(mm[k0], mm[k0 + 1]);
                    const float2 f1 = __fadd2_rn(make_float2(__uint_as_float(u1[k0]), __uint_as_float(u1[k0 + 1])), nmag);
                    const float2 f2 = __fadd2_rn(make_float2(__uint_as_float(u2[k0]), __uint_as_float(u2[k0 + 1])), nmag);
                    const float2 r1 = __fadd2_rz(__fmul2_rn(f1, mk), mag);
                    const float2 r2 = __fadd2_rz(__fmul2_rn(f2, mk), mag);
                    t1[2 * h] = __viaddmin_s32_relu(__float_as_int(r1.x), -0x4AC00000, 2 * hi + 1);
                    t1[2 * h + 1] = __viaddmin_s32_relu(__float_as_int(r1.y), -0x4AC00000, 2 * hi + 1);
                    t2[2 * h] = __viaddmin_s32_relu(__float_as_int(r2.x), -0x4AC00000, 2 * hi + 1);
                    t2[2 * h + 1] = __viaddmin_s32_relu(__float_as_int(r2.y), -0x4AC00000, 2 * hi + 1);
                }
                w1[q] = (__byte_perm(__byte_perm(t1[0], t1[1], 0x0040), __byte_perm(t1[2], t1[3], 0x0040), 0x5410) >> 1) & 0x7F7F7F7Fu;
                w2[q] = (__byte_perm(__byte_perm(t2[0], t2[1], 0x0040), __byte_perm(t2[2], t2[3], 0x0040), 0x5410) >> 1) & 0x7F7F7F7Fu;
            }
            o1 = make_uint4(w1[0], w1[1], w1[2], w1[3]);
            o2 = make_uint4(w2[0], w2[1], w2[2], w2[3]);
            return;
        }
    }
    o1 = requant16<kSilu>(v1, cs, slot0, p);
    o2 = requant16<kSilu>(v2, cs, slot0, p);
}

// fp16 epilogue for 16 f32 accumulators (16 consecutive channels of one row),
// in the order the reference's CPU runtime applies the ops: the conv result
// stored as f16 (F16::from_f32, round to nearest even), the f16 bias added in
// f32 and rounded to f16 again (crates/dragonwing-onnx/src/runtime.rs:1483-1497),
// the residual added as add_fp16 does it (crates/dragonwing-cpu/src/ops.rs:434-446),
// then ReLU (x > 0 ? x : 0, ops.rs:345-352 / runtime.rs:967-971).
//
// Packed-half path, branch-free: an add of two f16 values done in f32 and
// rounded to f16 equals the f16 add rounded once (f32 has 24 >= 2*11 + 2
// significand bits, so the double rounding is innocuous; sums below 2^-14 are
// exact in both).  The reference's F16::to_f32 halves a subnormal operand, so
// a step whose operand is below 2^-14 (zero included: halving it is harmless)
// scales that operand by 0.5 inside one fused multiply-add, which rounds
// once as the f32 path does: fma(x, 0.5, b) for the bias, the residual add
// with the subnormal operand in the multiplied slot, and x * 0.5 before the
// ReLU.  What this cannot express -- both residual-add operands subnormal, a
// NaN result without a final ReLU, a subnormal or NaN bias -- goes to the
// exact per-element path.
__device__ __forceinline__ uint32_t h2_bits(__half2 h) { return *reinterpret_cast<uint32_t *>(&h); }
__device__ __forceinline__ __half2 bits_h2(uint32_t u) { return *reinterpret_cast<__half2 *>(&u); }

// Per half 0xFFFF when |x| < 2^-14 (subnormal or zero).
__device__ __forceinline__ uint32_t h2_tiny_mask(uint32_t x) {
    return __hlt2_mask(__habs2(bits_h2(x)), bits_h2(0x04000400u));
}

// Per half: 0.5 where the mask is set, else 1.0.
__device__ __forceinline__ uint32_t half_scale(uint32_t mask) { return 0x3C003C00u ^ (mask & 0x04000400u); }

// One element on the exact path (every step through F16::to_f32 / from_f32).
// Scalar arguments, out of line: the hot loop keeps its accumulators in
// registers and the rare exact path out of its instruction stream.
static __device__ __noinline__ uint32_t f16_exact_one(float acc, float bias, uint32_t res, uint32_t flags) {
    uint16_t x = f32_to_f16_ref(acc);
    if (flags & 1u) x = f32_to_f16_ref(__fadd_rn(f16_to_f32_ref(x), bias));
    if (flags & 2u) x = f32_to_f16_ref(__fadd_rn(f16_to_f32_ref(x), f16_to_f32_ref((uint16_t)res)));
    if (flags & 4u) {
        const float f = f16_to_f32_ref(x);
        x = f32_to_f16_ref(f > 0.0f ? f : 0.0f);
    }
    return x;
}

// The 16 outputs as 8 packed pairs in w.  `rw` = the 16 residual halves as 8
// packed pairs (read when p.res_f16 is set).
// kFm: bit 0 = bias, bit 1 = residual, bit 2 = ReLU (one kernel instance each).
template <int kFm>
__device__ __forceinline__ void f16_epilogue16(const int32_t (&v)[16], const ChanSmem *cs, int slot0,
                                               const UmmaParams &p, const uint32_t (&rw)[8], uint32_t (&w)[8]) {
    constexpr bool has_bias = kFm & 1, has_res = kFm & 2, relu = kFm & 4;
    uint32_t bq[8];
    if (has_bias) {
        const uint4 b0 = reinterpret_cast<const uint4 *>(cs->d)[slot0 >> 3];
        const uint4 b1 = reinterpret_cast<const uint4 *>(cs->d)[(slot0 >> 3) + 1];
        bq[0] = b0.x; bq[1] = b0.y; bq[2] = b0.z; bq[3] = b0.w;
        bq[4] = b1.x; bq[5] = b1.y; bq[6] = b1.z; bq[7] = b1.w;
    }
    uint32_t badbits = 0;
#pragma unroll
    for (int k = 0; k < 8; k++) {
        uint32_t o = h2_bits(__floats2half2_rn(__int_as_float(v[2 * k]), __int_as_float(v[2 * k + 1])));
        uint32_t bad = 0;
        if (has_bias) o = h2_bits(__hfma2(bits_h2(o), bits_h2(half_scale(h2_tiny_mask(o))), bits_h2(bq[k])));
        if (has_res) {
            const uint32_t r = rw[k];
            const uint32_t my = h2_tiny_mask(o);
            const uint32_t mr = h2_tiny_mask(r) & __hne2_mask(bits_h2(r), bits_h2(0u));  // nonzero subnormal
            bad |= my & mr;
            const uint32_t a = (mr & r) | (~mr & o), c = (mr & o) | (~mr & r);
            o = h2_bits(__hfma2(bits_h2(a), bits_h2(half_scale(my | mr)), bits_h2(c)));
        }
        if (relu) {
            const uint32_t pos = __hgt2_mask(bits_h2(o), bits_h2(0u));
            o = h2_bits(__hmul2(bits_h2(o), bits_h2(half_scale(h2_tiny_mask(o))))) & pos;
        } else {
            bad |= __hneu2_mask(bits_h2(o), bits_h2(o));  // NaN: the reference keeps its payload bits
        }
        w[k] = o;
        badbits |= (bad & 1u) << (2 * k) | ((bad >> 16) & 1u) << (2 * k + 1);
    }
    if (has_bias && (cs->cflags[slot0 >> 4] & 1u)) badbits = 0xFFFFu;  // a subnormal or NaN bias in this group
    if (badbits) {
        const uint32_t fl = (uint32_t)kFm;
#pragma unroll
        for (int j = 0; j < 16; j++) {
            if (badbits & (1u << j)) {
                const uint32_t r = (rw[j >> 1] >> (16 * (j & 1))) & 0xFFFFu;
                const uint32_t h = f16_exact_one(__int_as_float(v[j]), cs->m[slot0 + j], r, fl);
                w[j >> 1] = (j & 1) ? ((w[j >> 1] & 0x0000FFFFu) | (h << 16)) : ((w[j >> 1] & 0xFFFF0000u) | h);
            }
        }
    }
}

// Shared-memory matrix descriptor (K-major, swizzled): start address >> 4 in
// bits [0,14); leading-byte offset (unused for swizzled K-major) = 1; the
// constant high word (stride-byte offset = 8 rows * row bytes, version 1,
// swizzle mode) is precomputed on the host.
__device__ __forceinline__ uint64_t smem_desc(uint32_t addr, uint64_t hi) {
    return hi | (uint64_t)((addr >> 4) & 0x3FFFu) | ((uint64_t)1u << 16);
}

// Shared-memory matrix descriptor, K-major without swizzle: core matrices of 8
// rows x 16 bytes (rows 16 bytes apart); `lbo` = bytes between the two 16-byte
// halves of a 32-byte K step, `sbo` = bytes between 8-row groups; version 1,
// layout type 0 (no swizzle).
__device__ __forceinline__ uint64_t smem_desc_noswz(uint32_t addr, uint32_t lbo, uint32_t sbo) {
    return (uint64_t)((addr >> 4) & 0x3FFFu) | ((uint64_t)((lbo >> 4) & 0x3FFFu) << 16) |
           ((uint64_t)((sbo >> 4) & 0x3FFFu) << 32) | (1ull << 46);
}

// One MMA with both descriptors given as 32-bit halves; kAcc folds the
// enable-input-d predicate into a constant (accumulate into D, or overwrite it).
template <bool kF16, bool kAcc>
__device__ __forceinline__ void tc_mma_w(uint32_t d, uint32_t alo, uint32_t ahi, uint32_t blo, uint32_t bhi,
                                         uint32_t idesc) {
    if (kF16)
        asm volatile(
            "{\n\t.reg .pred p;\n\t.reg .b64 a, b;\n\tsetp.ne.b32 p, %6, 0;\n\t"
            "mov.b64 a, {%1, %2};\n\tmov.b64 b, {%3, %4};\n\t"
            "tcgen05.mma.cta_group::1.kind::f16 [%0], a, b, %5, p;\n\t}" ::"r"(d),
            "r"(alo), "r"(ahi), "r"(blo), "r"(bhi), "r"(idesc), "n"(kAcc ? 1 : 0)
            : "memory");
    else
        asm volatile(
            "{\n\t.reg .pred p;\n\t.reg .b64 a, b;\n\tsetp.ne.b32 p, %6, 0;\n\t"
            "mov.b64 a, {%1, %2};\n\tmov.b64 b, {%3, %4};\n\t"
            "tcgen05.mma.cta_group::1.kind::i8 [%0], a, b, %5, p;\n\t}" ::"r"(d),
            "r"(alo), "r"(ahi), "r"(blo), "r"(bhi), "r"(idesc), "n"(kAcc ? 1 : 0)
            : "memory");
}

// Halo mode: the MMAs of one K block, kR row blocks each.  Entry q of `tab` is
// one 32-byte K step: x = the A descriptor's low word relative to the stage's
// first plane (the tap's offset, and the LBO between the step's two 16-byte
// halves), y = the B descriptor's low word (added to b16: 0 for resident
// weights, else the stage's B tile).  The i-th issued row block reads A
// roff16[i] 16-byte units further and accumulates into the columns from
// d_tmem + i * dstride.  `first`: the first step overwrites the accumulators.
template <int kR, bool kF16>
__device__ __forceinline__ void halo_mmas(const int2 *tab, int n, uint32_t a16, uint32_t b16, uint32_t ahi,
                                          uint32_t bhi, uint32_t d_tmem, uint32_t dstride, const uint32_t (&roff16)[8],
                                          uint32_t idesc, bool first) {
    uint32_t dcol[kR], ar[kR];
#pragma unroll
    for (int r = 0; r < kR; r++) {
        dcol[r] = d_tmem + (uint32_t)r * dstride;
        ar[r] = a16 + roff16[r];
    }
    int q = 0;
    if (first) {
        const int2 v = tab[0];
#pragma unroll
        for (int r = 0; r < kR; r++)
            tc_mma_w<kF16, false>(dcol[r], ar[r] + (uint32_t)v.x, ahi, b16 + (uint32_t)v.y, bhi, idesc);
        q = 1;
    }
    for (; q < n; q++) {
        const int2 v = tab[q];
#pragma unroll
        for (int r = 0; r < kR; r++)
            tc_mma_w<kF16, true>(dcol[r], ar[r] + (uint32_t)v.x, ahi, b16 + (uint32_t)v.y, bhi, idesc);
    }
}

template <bool kF16>
__device__ __forceinline__ void halo_mmas_r(int R, const int2 *tab, int n, uint32_t a16, uint32_t b16, uint32_t ahi,
                                            uint32_t bhi, uint32_t d_tmem, uint32_t bn, const uint32_t (&roff16)[8],
                                            uint32_t idesc, bool first) {  // bn: the column stride
    switch (R) {
        case 1: halo_mmas<1, kF16>(tab, n, a16, b16, ahi, bhi, d_tmem, bn, roff16, idesc, first); break;
        case 2: halo_mmas<2, kF16>(tab, n, a16, b16, ahi, bhi, d_tmem, bn, roff16, idesc, first); break;
        case 3: halo_mmas<3, kF16>(tab, n, a16, b16, ahi, bhi, d_tmem, bn, roff16, idesc, first); break;
        case 4: halo_mmas<4, kF16>(tab, n, a16, b16, ahi, bhi, d_tmem, bn, roff16, idesc, first); break;
        case 5: halo_mmas<5, kF16>(tab, n, a16, b16, ahi, bhi, d_tmem, bn, roff16, idesc, first); break;
        case 6: halo_mmas<6, kF16>(tab, n, a16, b16, ahi, bhi, d_tmem, bn, roff16, idesc, first); break;
        case 7: halo_mmas<7, kF16>(tab, n, a16, b16, ahi, bhi, d_tmem, bn, roff16, idesc, first); break;
        default: halo_mmas<8, kF16>(tab, n, a16, b16, ahi, bhi, d_tmem, bn, roff16, idesc, first); break;
    }
}

// ------------------------------------------------------------------- kernel
// Tile = R blocks of 128 output pixels x bn output channels.  Row block r of a
// tile covers pixels [tile_m0 + 128 r, +128) in flat mode, or the spatial
// sub-tile (tw x th) starting at output row oh0 + r*th in spatial mode; its
// accumulators sit in TMEM columns [acc*R*bn + r*bn, +bn).
struct TileCoord {
    int mt, nt, n0, img, oh0, ow0;
};

__device__ __forceinline__ TileCoord tile_coord(const UmmaParams &p, int tile) {
    TileCoord t;
    t.mt = tile / p.n_tiles;
    t.nt = tile % p.n_tiles;
    t.n0 = t.nt * p.bn;
    t.img = t.oh0 = t.ow0 = 0;
    if (p.mode != 0) {
        const int tw_i = t.mt % p.tiles_w;
        const int t2 = t.mt / p.tiles_w;
        t.oh0 = (t2 % p.tiles_h) * p.th * (p.R / p.rw);
        t.img = (t2 / p.tiles_h) * p.nb;
        t.ow0 = tw_i * p.tw * p.rw;
    }
    return t;
}

// Output origin of row block r of a spatial tile: blocks fill the tile rw
// across, then down.
__device__ __forceinline__ int block_x(const UmmaParams &p, const TileCoord &t, int r) { return t.ow0 + (r % p.rw) * p.tw; }
__device__ __forceinline__ int block_y(const UmmaParams &p, const TileCoord &t, int r) { return t.oh0 + (r / p.rw) * p.th; }

// Row blocks of the tile that hold at least one in-range output pixel (the
// others are neither loaded nor stored).
__device__ __forceinline__ int valid_blocks(const UmmaParams &p, const TileCoord &t) {
    if (p.mode == 0) {
        const long long first = (long long)t.mt * p.R * kBM;
        const long long left = (p.rows - first + kBM - 1) / kBM;
        return (int)(left < p.R ? left : p.R);
    }
    const int left = (p.ho - t.oh0 + p.th - 1) / p.th;
    return left < p.R ? left : p.R;
}

// Row block r holds at least one in-range output pixel (its TMA store starts
// inside the output; a block past the right or bottom edge is skipped).
__device__ __forceinline__ bool block_valid(const UmmaParams &p, const TileCoord &t, int r, int nrb) {
    if (p.mode != 2) return r < nrb;
    return block_x(p, t, r) < p.wo && block_y(p, t, r) < p.ho;
}

// int8 residual (kFm & 2): the staging unit already holds the residual's 16
// bytes (fetched by the store warp before the epilogue fills the buffer); the
// tile's output is add_i8(residual, conv) with the op's ratios, exactly as the
// separate add computes it.
template <int kFm>
__device__ __forceinline__ uint4 with_residual(uint4 conv, uint32_t staged, const UmmaParams &p) {
    if (!(kFm & 2)) return conv;
    return add16_fast(lds_v4(staged), conv, make_float2(p.add_ra, p.add_ra), make_float2(p.add_rb, p.add_rb), p.add_ra,
                      p.add_rb);
}

constexpr int kTapTable = 64;  // taps whose view coordinates the producer keeps in shared memory
constexpr int kMmaTable = 256; // halo mode: K steps (per CTA, all K blocks) the MMA issuer keeps descriptors of

// Coordinates of tap (kh, kw) in the 5-D activation view: the column phase's
// channel offset, the column shift, the row phase and the row shift.
__device__ __forceinline__ int4 tap_coord(const UmmaParams &p, int tap) {
    const int kh = tap / p.kw, kw = tap % p.kw;
    const int dh = kh - p.pt, dwc = kw - p.pl;
    const int par_h = ((dh % p.sh) + p.sh) % p.sh, par_w = ((dwc % p.sw) + p.sw) % p.sw;
    return make_int4(par_w * p.c_in, (dwc - par_w) / p.sw, par_h, (dh - par_h) / p.sh);
}

// kSilu: int8 SiLU epilogue.  kF16: fp16 operands (kind::f16) with the fp16
// epilogue; kFm its bias / residual / ReLU flags.
template <bool kSilu, bool kF16, int kFm, bool kPipe = false>
__global__ void __launch_bounds__(umma_threads(kSilu, kF16), 1)
    k_umma_conv_i8(const __grid_constant__ CUtensorMap tmap_a, const __grid_constant__ CUtensorMap tmap_b,
                   const __grid_constant__ CUtensorMap tmap_y, const __grid_constant__ CUtensorMap tmap_r,
                   const __grid_constant__ UmmaParams p) {
    constexpr int kEpiWarps = epi_warps(kSilu, kF16);
    constexpr int kF16Batch = kEpiWarps > 8 ? 2 : 4;  // fp16 TMEM loads per wait (registers)
    constexpr int kEpiParts = kEpiWarps / 4;
    constexpr int kStoreWarp = 2 + kEpiWarps;
    constexpr int kMma2Warp = kStoreWarp + 1;
    extern __shared__ __align__(1024) uint8_t smem_raw[];
    // 1 KiB-aligned base (swizzle patterns repeat every 1 KiB).
    uint8_t *smem = reinterpret_cast<uint8_t *>((reinterpret_cast<uintptr_t>(smem_raw) + 1023) & ~uintptr_t(1023));
    uint8_t *a_smem = smem;
    uint8_t *b_smem = smem + (size_t)p.stages * p.a_stage_bytes;
    uint8_t *out_stage = smem + p.off_out;                          // nbuf x [R*128 rows][bn] output tiles
    ChanSmem *chan = reinterpret_cast<ChanSmem *>(smem + p.off_chan);
    uint64_t *bars = reinterpret_cast<uint64_t *>(smem + p.off_bars);
    uint64_t *full_bar = bars;                      // [stages]
    uint64_t *empty_bar = bars + kMaxStages;        // [stages]
    uint64_t *tfull_bar = bars + 2 * kMaxStages;    // [2]
    uint64_t *tempty_bar = tfull_bar + 2;           // [2]
    uint64_t *drain_bar = tempty_bar + 2;           // [1] MMA drain on abort
    uint64_t *res_bar = drain_bar + 1;              // [2] staging buffer free for the next tile (fp16: residual in)
    uint64_t *ready_bar = res_bar + 2;              // [2] staging buffer holds a finished tile
    uint64_t *w_bar = ready_bar + 2;                // [1] resident weights landed (mode 2, wres)
    uint64_t *drain2_bar = w_bar + 1;               // [1] the second MMA warp's drain on abort
    uint32_t *tmem_slot = reinterpret_cast<uint32_t *>(drain2_bar + 1);
    volatile int *abort_flag = reinterpret_cast<volatile int *>(tmem_slot + 1);

    const int warp = threadIdx.x >> 5;
    const int lane = threadIdx.x & 31;
    // Tap table: mode 1, the producer's per-tap view coordinates; mode 2, the
    // MMA issuer's per-tap halo offsets (each written and read by one warp).
    __shared__ int4 tapc[kTapTable];
    __shared__ int2 mtab[kMmaTable];  // halo mode: the MMA issuer's K-step descriptor table

    if (threadIdx.x == 0) {
        for (int s = 0; s < p.stages; s++) {
            mbar_init(smem_u32(&full_bar[s]), 1);
            mbar_init(smem_u32(&empty_bar[s]), p.n_issuers);
        }
        for (int a = 0; a < 2; a++) {
            mbar_init(smem_u32(&tfull_bar[a]), p.n_issuers);
            mbar_init(smem_u32(&tempty_bar[a]), kEpiWarps);
        }
        mbar_init(smem_u32(drain_bar), 1);
        mbar_init(smem_u32(drain2_bar), 1);
        mbar_init(smem_u32(w_bar), 1);
        for (int b = 0; b < 2; b++) {
            mbar_init(smem_u32(&res_bar[b]), 1);
            mbar_init(smem_u32(&ready_bar[b]), kEpiWarps);
        }
        *abort_flag = 0;
        asm volatile("fence.mbarrier_init.release.cluster;" ::: "memory");
        asm volatile("fence.proxy.async.shared::cta;" ::: "memory");
    }
    if (warp == 1) {
        asm volatile("tcgen05.alloc.cta_group::1.sync.aligned.shared::cta.b32 [%0], %1;" ::"r"(smem_u32(tmem_slot)),
                     "r"(p.tmem_cols)
                     : "memory");
        asm volatile("tcgen05.relinquish_alloc_permit.cta_group::1.sync.aligned;" ::: "memory");
        // halo mode: the MMA warps' K-step descriptor table (visible to both
        // after the barrier below)
        const uint32_t w_base = smem_u32(smem + p.off_w);
        const int kn2_full = (p.cps + 1) >> 1;  // halo mode: K steps of a full K block
        const int kn2_last = (min(p.cps, p.chunks - (p.cblocks - 1) * p.cps) + 1) >> 1;
        if (p.mode == 2) {
            const uint32_t hw16 = (uint32_t)p.hw * 16u;
            // the halo's taps: the conv's own, or (stride 2) the taps over the parity planes
            const int hkw = p.s2 ? p.tkw : p.kw, htaps = p.s2 ? p.tkh * p.tkw : p.taps;
            auto tap_off = [&](int t) { return ((uint32_t)(t / hkw) * hw16) + (uint32_t)(t % hkw) * 16u; };
            if (p.tpair) {
                // taps (2q, 2q + 1) in one K step: A's second half is tap 2q + 1's
                // pixel (LBO = the offset between the two taps' pixels), B's the
                // next slice (the all-zero slice past the last tap)
                for (int q = lane; q < (p.taps + 1) / 2; q += 32) {
                    const int t = 2 * q;
                    const uint32_t off = tap_off(t);
                    const uint32_t lbo = t + 1 < p.taps ? tap_off(t + 1) - off : 16u;
                    mtab[q] = make_int2((int)((off >> 4) | ((lbo >> 4) << 16)),
                                        (int)(((w_base + (uint32_t)t * p.b_tap_bytes) >> 4) | ((p.b_tap_bytes >> 4) << 16)));
                }
            } else {
                // K block `it`, tap t, K step k: chunk planes 2k and 2k + 1 (with an
                // odd chunk count the last step's second half is the neighbouring
                // pixel, LBO 16 bytes, against zero weights)
                const int per = htaps * kn2_full;
                const int total = (p.cblocks - 1) * per + htaps * kn2_last;
                for (int i = lane; i < total; i += 32) {
                    const int it = i / per, rem = i - it * per;
                    const int knb = it == p.cblocks - 1 ? kn2_last : kn2_full;
                    const int t = rem / knb, k = rem - t * knb;
                    const int real = min(p.cps, p.chunks - it * p.cps);
                    const uint32_t off = tap_off(t) + (uint32_t)(2 * k) * p.plane_stride;
                    const uint32_t lbo = 2 * k + 1 < real ? p.plane_stride : 16u;
                    if (p.s2) {
                        // 16-byte weight slices [tap][chunk]: the step's two chunks are
                        // consecutive slices (LBO one slice)
                        const uint32_t b = w_base + (uint32_t)(t * p.chunks + it * p.cps + 2 * k) * p.b_tap_bytes;
                        mtab[i] = make_int2((int)((off >> 4) | ((lbo >> 4) << 16)),
                                            (int)((b >> 4) | ((p.b_tap_bytes >> 4) << 16)));
                        continue;
                    }
                    const uint32_t b = p.wres ? w_base + (uint32_t)(t * p.cblocks + it) * p.b_tap_bytes + 32u * k
                                              : (uint32_t)t * p.b_tap_bytes + 32u * k;
                    mtab[i] = make_int2((int)((off >> 4) | ((lbo >> 4) << 16)), (int)((b >> 4) | (1u << 16)));
                }
            }
        }
    }
    tc_fence_before();
    __syncthreads();
    tc_fence_after();
    // Programmatic dependent launch: this grid may start while the previous
    // kernel on the stream finishes (its CTAs take the SMs the previous grid's
    // last CTAs free, and run the prologue above: barriers, TMEM, descriptor
    // table).  Every read of memory another kernel writes -- inputs, weights,
    // per-channel arrays, residuals -- and every write come after this wait,
    // which returns once the previous grid has completed and its writes are
    // visible (a no-op when the launch carries no programmatic dependency).
    asm volatile("griddepcontrol.wait;" ::: "memory");
    const uint32_t tmem_base = *tmem_slot;
    const int k_iters = p.mode == 2 ? p.cblocks : p.taps * p.cblocks;  // halo mode: one stage per K block, all taps
    const uint32_t acc_cols = (uint32_t)(p.R * p.bn);

    if (warp == 0) {
        // ------------------------------------------------------------ producer
        // per-tap coordinates of the 5-D activation view (mode 1), computed once:
        // x offset (column phase * c_in), column shift, row phase, row shift
        if (p.mode == 1)
            for (int tap = lane; tap < min(p.taps, kTapTable); tap += 32) tapc[tap] = tap_coord(p, tap);
        __syncwarp();
        if (lane == 0) {
            asm volatile("prefetch.tensormap [%0];" ::"l"(&tmap_a) : "memory");
            asm volatile("prefetch.tensormap [%0];" ::"l"(&tmap_b) : "memory");
            int s = 0;
            uint32_t ph = 0;
            uint32_t issued_mask = 0, last_parity = 0;  // per stage: issued at least once / parity of last issue
            bool ok = true;
            const bool w_issued = p.wres && (int)blockIdx.x < p.num_tiles;
            if (w_issued) {
                // resident weights: every (tap, K block) slice of the channel tile, once
                const uint32_t wb = smem_u32(&w_bar[0]);
                mbar_expect_tx(wb, p.w_bytes);
                const uint32_t w_dst = smem_u32(smem + p.off_w);
                if (p.tpair) {
                    // one 16-byte slice per tap, then one past the last tap: out of range,
                    // so TMA fills it with zeros
                    for (int t = 0; t <= p.taps; t++)
                        tma_load_3d(w_dst + (uint32_t)t * p.b_tap_bytes, &tmap_b, wb, 0, t, 0);
                } else if (p.s2) {
                    // parity planes: slice (tap (dy, dx), chunk (ph, pw, cc)) holds kernel tap
                    // (2 dy + ph + pt, 2 dx + pw + pl)'s chunk cc, or zeros (tap index past
                    // the last: out of range) when no kernel tap lands there
                    const int chunks0 = p.chunks / 4;
                    for (int t2 = 0; t2 < p.tkh * p.tkw; t2++)
                        for (int c2 = 0; c2 < p.chunks; c2++) {
                            const int ph = c2 / (2 * chunks0), pw = (c2 / chunks0) & 1, cc = c2 % chunks0;
                            const int kh = 2 * (t2 / p.tkw + p.dy0) + ph + p.pt;
                            const int kw = 2 * (t2 % p.tkw + p.dx0) + pw + p.pl;
                            const int tap = (kh >= 0 && kh < p.k_h && kw >= 0 && kw < p.kw) ? kh * p.kw + kw : p.taps;
                            tma_load_3d(w_dst + (uint32_t)(t2 * p.chunks + c2) * p.b_tap_bytes, &tmap_b, wb,
                                        cc * p.chunk_elems, tap, 0);
                        }
                } else {
                    for (int t = 0; t < p.taps; t++)
                        for (int cb = 0; cb < p.cblocks; cb++)
                            tma_load_3d(w_dst + (uint32_t)(t * p.cblocks + cb) * p.b_tap_bytes, &tmap_b, wb,
                                        cb * p.bk_elems, t, 0);
                }
            }
            for (int tile = blockIdx.x; tile < p.num_tiles && ok; tile += gridDim.x) {
                const TileCoord tc = tile_coord(p, tile);
                const int nrb = valid_blocks(p, tc);
                int tap = 0, cb = 0;  // it = tap * cblocks + cb, kept incrementally
                for (int it = 0; it < k_iters; it++) {
                    if (it) {
                        if (++cb == p.cblocks) {
                            cb = 0;
                            tap++;
                        }
                    }
                    if (!mbar_wait(smem_u32(&empty_bar[s]), ph ^ 1, p, abort_flag, 1)) { ok = false; break; }
                    const uint32_t fb = smem_u32(&full_bar[s]);
                    const uint32_t a_dst = smem_u32(a_smem + (size_t)s * p.a_stage_bytes);
                    const uint32_t b_dst = smem_u32(b_smem + (size_t)s * p.b_stage_bytes);
                    if (p.mode == 2) {
                        // halo mode: K block `it` = chunks [it * cps, +real) of every tap;
                        // one halo box per chunk (zero fill = the conv's padding), one
                        // weight box per tap
                        const int real = min(p.cps, p.chunks - it * p.cps);
                        mbar_expect_tx(fb, (uint32_t)real * (uint32_t)(p.hw * p.hh * 16) +
                                               (p.wres ? 0u : (uint32_t)p.taps * p.b_tx_bytes));
                        if (p.flat_in)  // one chunk: x counts 8-byte units, two per pixel
                            tma_load_3d(a_dst, &tmap_a, fb, 2 * (tc.ow0 - p.pl), tc.oh0 - p.pt, tc.img);
                        else if (p.s2) {
                            // chunk it * cps + j of the parity planes: phase (ph, pw), channel chunk cc
                            const int chunks0 = p.chunks / 4;
                            for (int j = 0; j < real; j++) {
                                const int c2 = it * p.cps + j;
                                const int ph = c2 / (2 * chunks0), pw = (c2 / chunks0) & 1, cc = c2 % chunks0;
                                tma_load_5d(a_dst + (uint32_t)j * p.plane_stride, &tmap_a, fb,
                                            pw * p.c_in + cc * p.chunk_elems, tc.ow0 + p.dx0, ph, tc.oh0 + p.dy0,
                                            tc.img);
                            }
                        } else
                            for (int j = 0; j < real; j++)
                                tma_load_4d(a_dst + (uint32_t)j * p.plane_stride, &tmap_a, fb,
                                            it * p.bk_elems + j * p.chunk_elems, tc.ow0 - p.pl, tc.oh0 - p.pt,
                                            tc.img);
                        if (!p.wres)
                            for (int t = 0; t < p.taps; t++)
                                tma_load_3d(b_dst + (uint32_t)t * p.b_tap_bytes, &tmap_b, fb, it * p.bk_elems, t,
                                            tc.n0);
                        issued_mask |= 1u << s;
                        last_parity = (last_parity & ~(1u << s)) | (ph << s);
                        if (++s == p.stages) { s = 0; ph ^= 1; }
                        continue;
                    }
                    mbar_expect_tx(fb, (uint32_t)nrb * p.a_tx_bytes + p.b_tx_bytes);
                    if (p.mode == 0) {
                        for (int r = 0; r < nrb; r++)
                            tma_load_2d(a_dst + (uint32_t)(r * kBM * p.bk), &tmap_a, fb, cb * p.bk_elems,
                                        (tc.mt * p.R + r) * kBM);
                    } else {
                        const int4 t4 = tap < kTapTable ? tapc[tap] : tap_coord(p, tap);
                        for (int r = 0; r < nrb; r++)
                            tma_load_5d(a_dst + (uint32_t)(r * kBM * p.bk), &tmap_a, fb, t4.x + cb * p.bk_elems,
                                        tc.ow0 + t4.y, t4.z, tc.oh0 + r * p.th + t4.w, tc.img);
                    }
                    tma_load_3d(b_dst, &tmap_b, fb, cb * p.bk_elems, tap, tc.n0);
                    issued_mask |= 1u << s;
                    last_parity = (last_parity & ~(1u << s)) | (ph << s);
                    if (++s == p.stages) { s = 0; ph ^= 1; }
                }
            }
            if (!ok) {
                // Abort: wait (bounded) for this CTA's own copies still in flight.
                if (w_issued) {
                    const uint64_t t0 = globaltimer_ns();
                    while (!mbar_try_wait(smem_u32(&w_bar[0]), 0) && globaltimer_ns() - t0 < p.wait_cap_ns) {
                    }
                }
                for (int st = 0; st < p.stages; st++) {
                    if (!(issued_mask & (1u << st))) continue;
                    const uint32_t par = (last_parity >> st) & 1u;
                    const uint64_t t0 = globaltimer_ns();
                    while (!mbar_try_wait(smem_u32(&full_bar[st]), par) && globaltimer_ns() - t0 < p.wait_cap_ns) {
                    }
                }
            }
        }
    } else if (warp == 1 || warp == kMma2Warp) {
        // ------------------------------------------------------------ MMA issuers
        // The issue loop is latency-bound (one thread; each tcgen05.mma takes
        // tens of cycles to issue), so in halo mode (many small MMAs per stage)
        // the descriptors are precomputed: one table entry per 32-byte K step
        // (built once per CTA) and the row blocks unrolled for the tile's R.
        const uint32_t w_base = smem_u32(smem + p.off_w);
        const int kn2_full = (p.cps + 1) >> 1;  // halo mode: K steps of a full K block
        const int kn2_last = (min(p.cps, p.chunks - (p.cblocks - 1) * p.cps) + 1) >> 1;
        const int issuer = warp == 1 ? 0 : 1;
        if (lane == 0 && issuer < p.n_issuers) {
            int s = 0;
            uint32_t ph = 0;
            int local = 0;
            bool ok = true;
            const int kn_full = p.bk >> 5;
            const int kn_last = (p.c_in * p.esize - (p.cblocks - 1) * p.bk + 31) >> 5;
            if (p.wres && (int)blockIdx.x < p.num_tiles && !mbar_wait(smem_u32(&w_bar[0]), 0, p, abort_flag, 7))
                ok = false;
            // this warp's row blocks: issuer, issuer + n_issuers, ...
            const int nis = p.n_issuers;
            const int my_r = (p.R - issuer + nis - 1) / nis;
            // halo mode: per issued row block r, its 16 B units from the tile's halo
            // origin ((r / rw) * 16 halo rows + (r % rw) * 8 pixels); descriptor
            // high words: A, SBO = one halo row; B, SBO = 8 rows of 16 bytes
            // (two-tap slices) or of bk bytes (swizzled); version 1
            const uint32_t h_sbo = (uint32_t)p.hw * 16u;
            uint32_t roff16[8];
#pragma unroll
            for (int i = 0; i < 8; i++) {
                const int r = issuer + i * nis;
                roff16[i] = p.mode == 2 ? (((uint32_t)(r / p.rw) * 16u * h_sbo) + (uint32_t)(r % p.rw) * 128u) >> 4 : 0u;
            }
            const uint32_t hi_sw = (uint32_t)(p.desc_hi >> 32);
            const uint32_t a_hi2 = (h_sbo >> 4) | (1u << 14);
            const uint32_t b_hi2 = (p.tpair || p.s2) ? ((128u >> 4) | (1u << 14)) : hi_sw;  // 16-byte slices
            for (int tile = blockIdx.x; tile < p.num_tiles && ok; tile += gridDim.x, local++) {
                const int acc = local & 1;
                const uint32_t acc_ph = (local >> 1) & 1;
                if (!mbar_wait(smem_u32(&tempty_bar[acc]), acc_ph ^ 1, p, abort_flag, 2)) { ok = false; break; }
                tc_fence_after();
                const uint32_t d_tmem = tmem_base + (uint32_t)acc * acc_cols + (uint32_t)(issuer * p.bn);
                int cb = 0;  // channel block of this iteration (it % cblocks, kept incrementally)
                for (int it = 0; it < k_iters; it++) {
                    if (!mbar_wait(smem_u32(&full_bar[s]), ph, p, abort_flag, 3)) { ok = false; break; }
                    tc_fence_after();
                    const uint32_t a_addr = smem_u32(a_smem + (size_t)s * p.a_stage_bytes);
                    const uint32_t b_addr = smem_u32(b_smem + (size_t)s * p.b_stage_bytes);
                    if (p.mode == 2) {
                        // every tap of K block `it`: the A tile is the halo plane read from
                        // the tap's offset (8-row groups one halo row apart)
                        const int htaps = p.s2 ? p.tkh * p.tkw : p.taps;
                        const int2 *tab = p.tpair ? mtab : mtab + it * htaps * kn2_full;
                        const int n = p.tpair ? (p.taps + 1) / 2 : htaps * (it == p.cblocks - 1 ? kn2_last : kn2_full);
                        halo_mmas_r<kF16>(my_r, tab, n, a_addr >> 4, p.wres ? 0u : (b_addr >> 4), a_hi2, b_hi2, d_tmem,
                                          (uint32_t)(nis * p.bn), roff16, p.idesc, it == 0);
                    } else {
                        // 32-byte K steps holding channels below c_in (the rest of the block is zero)
                        const int kn = cb == p.cblocks - 1 ? kn_last : kn_full;
                        if (++cb == p.cblocks) cb = 0;
                        // plain loops: for 128 x 256 tiles they keep the tensor pipe busier than
                        // an unrolled per-R issue (measured on B200: QGemm 4096^3 1,768 against
                        // 1,523 TOPS); with several row blocks this warp's (issuer, issuer +
                        // n_issuers, ...) for each K step
                        if (p.R == 1) {
                            for (int k = 0; k < kn; k++) {
                                const uint64_t ad = smem_desc(a_addr + 32 * k, p.desc_hi);
                                const uint64_t bd = smem_desc(b_addr + 32 * k, p.desc_hi);
                                tc_mma<kF16>(d_tmem, ad, bd, p.idesc, (it > 0 || k > 0) ? 1u : 0u);
                            }
                        } else {
                            for (int k = 0; k < kn; k++) {
                                const uint64_t bd = smem_desc(b_addr + 32 * k, p.desc_hi);
                                for (int i = 0; i < my_r; i++) {
                                    const int r = issuer + i * nis;
                                    const uint64_t ad = smem_desc(a_addr + (uint32_t)(r * kBM * p.bk) + 32 * k, p.desc_hi);
                                    tc_mma<kF16>(d_tmem + (uint32_t)(i * nis * p.bn), ad, bd, p.idesc,
                                                 (it > 0 || k > 0) ? 1u : 0u);
                                }
                            }
                        }
                    }
                    tc_commit(smem_u32(&empty_bar[s]));  // frees the stage when these MMAs finish
                    if (++s == p.stages) { s = 0; ph ^= 1; }
                }
                if (!ok) break;
                tc_commit(smem_u32(&tfull_bar[acc]));  // accumulators ready for the epilogue
            }
            if (!ok) {
                // Abort: wait (bounded) until the MMAs this warp issued have retired,
                // so TMEM is not freed under them.
                const uint32_t db = smem_u32(issuer ? drain2_bar : drain_bar);
                tc_commit(db);
                const uint64_t t0 = globaltimer_ns();
                while (!mbar_try_wait(db, 0) && globaltimer_ns() - t0 < p.wait_cap_ns) {
                }
            }
        }
    } else if (warp < kStoreWarp) {
        // ------------------------------------------------------------ epilogue
        const int e = warp - 2;               // 0 .. kEpiWarps - 1
        const int et = threadIdx.x - 64;      // epilogue thread index
        const int quarter = warp & 3;         // TMEM lanes this warp may access
        const int part = e >> 2;              // which part of the (row block, chunk) items
        const int row = quarter * 32 + lane;  // row within a 128-row block
        const int chunks = p.bn / 16;
        const int items = p.R * chunks;
        int local = 0;
        if (p.chan_all) {
            // every output channel's parameters, once, while the first tile's MMAs
            // run (all 256 epilogue threads take part in every round: the flags use
            // warp ballots; barrier A of the first tile publishes them)
            for (int base = 0; base < p.c_out; base += kEpiWarps * 32)
                stage_channel(p, chan, base + et, base + et, base + et < p.c_out);
        }
        // Per-tile channel mode: a tile's channels are staged into half `acc` of
        // the slots one tile ahead (the global loads overlap the previous tile).
        if (!p.chan_all && (int)blockIdx.x < p.num_tiles)
            stage_channel(p, chan, et, tile_coord(p, blockIdx.x).n0 + et, et < p.bn);
        // Staging: tile `local` goes to buffer local % nbuf once the store warp
        // has released it (res_bar; for an fp16 residual the buffer then holds
        // the tile's residual rows, which each thread reads from the spot its
        // 16 outputs overwrite); ready_bar hands the finished tile back.
        constexpr bool res_tma = kF16 && (kFm & 2);
        for (int tile = blockIdx.x; tile < p.num_tiles; tile += gridDim.x, local++) {
            const int acc = local & 1;
            const uint32_t acc_ph = (local >> 1) & 1;
            const int sb = p.nbuf == 2 ? (local & 1) : 0;
            const uint32_t sb_ph = p.nbuf == 2 ? ((local >> 1) & 1) : (local & 1);
            uint8_t *const stage = out_stage + (size_t)sb * p.out_bytes;
            // the tile's first channel (tile_coord's n0 without its divisions: the
            // per-tile bookkeeping sits between every tile's requantisations)
            const int n0 = p.n_tiles == 1 ? 0 : (tile % p.n_tiles) * p.bn;
            const int slot_base = p.chan_all ? n0 : acc * (kChanSlots / 2);
            bool ok = mbar_wait(smem_u32(&tfull_bar[acc]), acc_ph, p, abort_flag, 4);
            if (ok) ok = mbar_wait(smem_u32(&res_bar[sb]), sb_ph, p, abort_flag, 5);
            // Barrier A (epilogue threads only): all-or-none abort decision; this
            // tile's staged channel parameters are visible.  With every channel
            // staged once (chan_all) only the first tile needs it: later tiles let
            // each warp run on (one slow warp no longer holds the others at every
            // tile; a warp that aborts alone leaves its arrivals missing, and the
            // MMA and store warps' bounded waits end the CTA).
            if (p.chan_all && local > 0) {
                if (!ok) break;
            } else if (named_barrier_or(1, kEpiWarps * 32, !ok)) break;
            if (!p.chan_all) {  // next tile's channels into the other half (its readers finished before barrier A)
                const int next = tile + (int)gridDim.x;
                if (next < p.num_tiles)
                    stage_channel(p, chan, (acc ^ 1) * (kChanSlots / 2) + et, tile_coord(p, next).n0 + et,
                                  et < p.bn);
            }
            tc_fence_after();
            const uint32_t tacc = tmem_base + ((uint32_t)(quarter * 32) << 16) + (uint32_t)acc * acc_cols;
            // each part of the warps takes a contiguous run of (row block, chunk)
            // items, two TMEM loads in flight per wait; (r, c) advance without division.
            if constexpr (kF16) {
                // fp16: each part of the warps takes a contiguous run of (row block,
                // chunk) items, kF16Batch TMEM loads in flight per wait; (r, c)
                // advance without division.
                const int per = (items + kEpiParts - 1) / kEpiParts;
                const int i_begin = part * per, i_end = min(items, i_begin + per);
                int r0 = i_begin / chunks, c0 = i_begin - (i_begin / chunks) * chunks;
                const uint32_t r7 = (uint32_t)(row & 7);
                for (int i = i_begin; i < i_end; i += kF16Batch) {
                    int rr[kF16Batch], cc[kF16Batch];
                    rr[0] = r0; cc[0] = c0;
#pragma unroll
                    for (int q = 1; q < kF16Batch; q++) {  // the next items; past the end repeat the last (the loads are collective)
                        int r = rr[q - 1], c = cc[q - 1] + 1;
                        if (c == chunks) { c = 0; r++; }
                        const bool in = i + q < i_end;
                        rr[q] = in ? r : rr[q - 1];
                        cc[q] = in ? c : cc[q - 1];
                    }
                    {
                        int r = rr[kF16Batch - 1], c = cc[kF16Batch - 1] + 1;
                        if (c == chunks) { c = 0; r++; }
                        r0 = r; c0 = c;
                    }
                    // Staging address of the chunk's first 16-byte unit.  Swizzled
                    // layout: [row block][64-channel slab][128 rows][128 bytes], unit u
                    // of a row stored at (u ^ (row & 7)) * 16 -- the TMA 128-byte
                    // swizzle, so the 32 rows a warp writes at once fall in distinct banks.
                    int32_t v[kF16Batch][16];
                    uint8_t *u0[kF16Batch];
#pragma unroll
                    for (int q = 0; q < kF16Batch; q++) {
                        tc_ld16(tacc + (uint32_t)(rr[q] * p.bn + cc[q] * 16), v[q]);
                        u0[q] = p.swz ? stage + (size_t)rr[q] * kBM * p.bn * 2 + (size_t)(cc[q] >> 2) * (kBM * 128) +
                                            row * 128 + (((((uint32_t)cc[q] & 3u) << 1) ^ r7) << 4)
                                      : stage + ((size_t)(rr[q] * kBM + row) * p.bn + cc[q] * 16) * 2;
                    }
                    // the second 16-byte unit: the next unit (linear), or unit ^ 1 (swizzled)
                    const uintptr_t u1x = p.swz ? 16u : 0u;
                    uint32_t rw[kF16Batch][8];
                    if (res_tma) {
#pragma unroll
                        for (int q = 0; q < kF16Batch; q++) {
                            const uint4 a0 = *reinterpret_cast<const uint4 *>(u0[q]);
                            const uint4 a1 = *reinterpret_cast<const uint4 *>(
                                u1x ? (uint8_t *)((uintptr_t)u0[q] ^ u1x) : u0[q] + 16);
                            rw[q][0] = a0.x; rw[q][1] = a0.y; rw[q][2] = a0.z; rw[q][3] = a0.w;
                            rw[q][4] = a1.x; rw[q][5] = a1.y; rw[q][6] = a1.z; rw[q][7] = a1.w;
                        }
                    }
                    tc_wait_ld();
#pragma unroll
                    for (int q = 0; q < kF16Batch; q++) {
                        if (i + q < i_end) {
                            uint32_t w[8];
                            f16_epilogue16<kFm>(v[q], chan, slot_base + cc[q] * 16, p, rw[q], w);
                            *reinterpret_cast<uint4 *>(u0[q]) = make_uint4(w[0], w[1], w[2], w[3]);
                            *reinterpret_cast<uint4 *>(u1x ? (uint8_t *)((uintptr_t)u0[q] ^ u1x) : u0[q] + 16) =
                                make_uint4(w[4], w[5], w[6], w[7]);
                        }
                    }
                }
            } else if constexpr (kPipe) {
                // int8 (instances without SiLU): each part of the warps takes a
                // contiguous run of (row block, chunk) items, kB per TMEM round.  The next round's loads are in
                // flight while this round is requantised: a TMEM load waits long
                // while the MMAs write the other accumulator buffer.  (The loads'
                // registers are read only after the wait that covers them.)
                constexpr int kB = 1;
                const int per = (items + kEpiParts - 1) / kEpiParts;
                const int i_begin = part * per, i_end = min(items, i_begin + per);
                const int rounds = i_end > i_begin ? (i_end - i_begin + kB - 1) / kB : 0;
                int cur_r = 0, cur_c = i_begin;  // the next item to load
                while (cur_c >= chunks) { cur_c -= chunks; cur_r++; }
                int lr0[kB], lc0[kB], lr1[kB], lc1[kB];
                int32_t v0[kB][16], v1[kB][16];
                // loads round j (items past the run repeat the last one: the loads are collective)
                auto load_round = [&](int j, int (&lr)[kB], int (&lc)[kB], int32_t (&v)[kB][16]) {
#pragma unroll
                    for (int q = 0; q < kB; q++) {
                        if (q == 0 || i_begin + j * kB + q < i_end) {
                            lr[q] = cur_r;
                            lc[q] = cur_c;
                            if (++cur_c == chunks) { cur_c = 0; cur_r++; }
                        } else {
                            lr[q] = lr[q - 1];
                            lc[q] = lc[q - 1];
                        }
                        tc_ld16(tacc + (uint32_t)(lr[q] * p.bn + lc[q] * 16), v[q]);
                    }
                };
                auto store_round = [&](int j, const int (&lr)[kB], const int (&lc)[kB], const int32_t (&v)[kB][16]) {
#pragma unroll
                    for (int q = 0; q < kB; q++) {
                        if (q == 0 || i_begin + j * kB + q < i_end) {
                            const uint32_t dst = smem_u32(stage + ((size_t)(lr[q] * kBM + row)) * p.bn + lc[q] * 16);
                            sts_v4(dst, with_residual<kFm>(requant16<kSilu>(v[q], chan, slot_base + lc[q] * 16, p), dst, p));
                        }
                    }
                };
                if (rounds > 0) {
                    load_round(0, lr0, lc0, v0);
                    tc_wait_ld();
                }
                for (int j = 0; j < rounds; j += 2) {
                    if (j + 1 < rounds) load_round(j + 1, lr1, lc1, v1);
                    store_round(j, lr0, lc0, v0);
                    tc_wait_ld();
                    if (j + 1 < rounds) {
                        if (j + 2 < rounds) load_round(j + 2, lr0, lc0, v0);
                        store_round(j + 1, lr1, lc1, v1);
                        tc_wait_ld();
                    }
                }
            } else {
            const int per = (items + kEpiParts - 1) / kEpiParts;
            const int i_begin = part * per, i_end = min(items, i_begin + per);
            // items in chunk-major order (row block fastest): a pair of items is
            // usually one channel chunk of two row blocks, whose parameters the
            // requantisation loads once
            int r1 = i_begin % p.R, c1 = i_begin / p.R;
            for (int i = i_begin; i < i_end; i += 2) {
                const bool two = i + 1 < i_end;
                int r2 = r1 + 1, c2 = c1;
                if (r2 >= p.R) { r2 = 0; c2++; }
                if (!two) { r2 = r1; c2 = c1; }
                int32_t v1[16], v2[16];
                tc_ld16(tacc + (uint32_t)(r1 * p.bn + c1 * 16), v1);
                tc_ld16(tacc + (uint32_t)(r2 * p.bn + c2 * 16), v2);
                uint8_t *dst1 = stage + ((size_t)(r1 * kBM + row)) * p.bn + c1 * 16;
                tc_wait_ld();
                if (kFm == 0 && !kSilu && two && c2 == c1) {
                    uint4 o1, o2;
                    requant16x2<kSilu>(v1, v2, chan, slot_base + c1 * 16, p, o1, o2);
                    sts_v4(smem_u32(dst1), o1);
                    sts_v4(smem_u32(stage + ((size_t)(r2 * kBM + row)) * p.bn + c2 * 16), o2);
                } else {
                    sts_v4(smem_u32(dst1), with_residual<kFm>(requant16<kSilu>(v1, chan, slot_base + c1 * 16, p), smem_u32(dst1), p));
                    if (two) {
                        uint8_t *dst2 = stage + ((size_t)(r2 * kBM + row)) * p.bn + c2 * 16;
                        sts_v4(smem_u32(dst2),
                               with_residual<kFm>(requant16<kSilu>(v2, chan, slot_base + c2 * 16, p), smem_u32(dst2), p));
                    }
                }
                r1 = r2 + 1; c1 = c2;
                if (r1 >= p.R) { r1 = 0; c1++; }
            }
            }
            tc_fence_before();
            asm volatile("fence.proxy.async.shared::cta;" ::: "memory");  // staging writes -> async proxy
            __syncwarp();
            if (lane == 0) {
                mbar_arrive(smem_u32(&tempty_bar[acc]));  // TMEM buffer free for the MMA warp
                mbar_arrive(smem_u32(&ready_bar[sb]));    // staged tile ready for the store warp
            }
        }
    } else {
        // ------------------------------------------------------------ store warp
        // Issues each finished tile's TMA stores, then -- once they have read the
        // buffer -- releases it for the tile nbuf tiles later (fetching that
        // tile's fp16 residual into it first).
        if (lane == 0) {
            constexpr bool res_tma = (kFm & 2) != 0;
            constexpr int es = kF16 ? 2 : 1;
            const int slabs = (kF16 && p.swz) ? p.bn / 64 : 1, sw_ch = (kF16 && p.swz) ? 64 : p.bn;
            uint32_t res_ph[2] = {0u, 0u};
            bool res_out[2] = {false, false};
            auto prepare = [&](int tile, int sb) {
                const uint32_t bar = smem_u32(&res_bar[sb]);
                if (res_tma) {
                    const TileCoord tc = tile_coord(p, tile);
                    const int nrb = valid_blocks(p, tc);
                    uint8_t *stage = out_stage + (size_t)sb * p.out_bytes;
                    // bytes per row block: its box (128 rows, or tw x th x nb pixels in mode 1)
                    const int box_rows = p.mode == 0 ? kBM : p.tw * p.th * p.nb;
                    int nvalid = 0;
                    for (int r = 0; r < p.R; r++) nvalid += block_valid(p, tc, r, nrb) ? 1 : 0;
                    mbar_expect_tx(bar, (uint32_t)(nvalid * box_rows * p.bn * es));
                    for (int r = 0; r < p.R; r++) {
                        if (!block_valid(p, tc, r, nrb)) continue;
                        for (int sl = 0; sl < slabs; sl++) {
                            const uint32_t dst =
                                smem_u32(stage + (size_t)r * kBM * p.bn * es + (size_t)sl * kBM * sw_ch * es);
                            if (p.mode == 0)
                                tma_load_2d(dst, &tmap_r, bar, tc.n0 + sl * sw_ch, (tc.mt * p.R + r) * kBM);
                            else
                                tma_load_4d(dst, &tmap_r, bar, tc.n0 + sl * sw_ch, block_x(p, tc, r),
                                            block_y(p, tc, r), tc.img);
                        }
                    }
                    res_out[sb] = true;
                } else {
                    mbar_arrive(bar);
                }
                res_ph[sb] ^= 1u;
            };
            for (int k = 0; k < p.nbuf; k++) {
                const int t = (int)blockIdx.x + k * (int)gridDim.x;
                if (t < p.num_tiles) prepare(t, k);
            }
            int local = 0;
            for (int tile = blockIdx.x; tile < p.num_tiles; tile += gridDim.x, local++) {
                const int sb = p.nbuf == 2 ? (local & 1) : 0;
                const uint32_t sb_ph = p.nbuf == 2 ? ((local >> 1) & 1) : (local & 1);
                if (!mbar_wait(smem_u32(&ready_bar[sb]), sb_ph, p, abort_flag, 6)) break;
                res_out[sb] = false;  // the epilogue waited for this buffer's residual before filling it
                const TileCoord tc = tile_coord(p, tile);
                const int nrb = valid_blocks(p, tc);
                uint8_t *stage = out_stage + (size_t)sb * p.out_bytes;
                for (int r = 0; r < p.R; r++) {
                    if (!block_valid(p, tc, r, nrb)) continue;
                    for (int sl = 0; sl < slabs; sl++) {
                        const uint32_t src =
                            smem_u32(stage + (size_t)r * kBM * p.bn * es + (size_t)sl * kBM * sw_ch * es);
                        if (p.mode == 0)
                            tma_store_2d(&tmap_y, src, tc.n0 + sl * sw_ch, (tc.mt * p.R + r) * kBM);
                        else if (p.flat_out)  // x counts 8-byte units: bn / 8 per pixel
                            tma_store_3d(&tmap_y, src, block_x(p, tc, r) * (p.bn >> 3), block_y(p, tc, r), tc.img);
                        else
                            tma_store_4d(&tmap_y, src, tc.n0 + sl * sw_ch, block_x(p, tc, r), block_y(p, tc, r),
                                         tc.img);
                    }
                }
                bulk_commit();
                const int next = tile + p.nbuf * (int)gridDim.x;
                if (next < p.num_tiles) {
                    bulk_wait_read0();  // the stores have read the buffer
                    prepare(next, sb);
                }
            }
            bulk_wait_all0();
            // residual copies issued for tiles the epilogue never took (abort): let them land
            for (int b = 0; b < 2; b++) {
                if (!res_out[b]) continue;
                const uint64_t t0 = globaltimer_ns();
                while (!mbar_try_wait(smem_u32(&res_bar[b]), res_ph[b] ^ 1u) && globaltimer_ns() - t0 < p.wait_cap_ns) {
                }
            }
        }
    }

    tc_fence_before();
    __syncthreads();
    if (warp == 1) {
        tc_fence_after();
        asm volatile("tcgen05.dealloc.cta_group::1.sync.aligned.b32 %0, %1;" ::"r"(tmem_base), "r"(p.tmem_cols)
                     : "memory");
    }
}

// ------------------------------------------------------------------- host side
struct Plan {
    int mode, tw, th, bk, bn, stages;
};

int pick_bk(int c_in) {
    // minimise padded K per tap (ceil(c/bk)*bk); prefer the wider block on ties
    int best = 128;
    long best_pad = (long)((c_in + 127) / 128) * 128;
    for (int bk : {64, 32}) {
        long pad = (long)((c_in + bk - 1) / bk) * bk;
        if (pad < best_pad) { best = bk; best_pad = pad; }
    }
    return best;
}

// Convs with several taps: the fewest K stages per tap, then the least padding
// (the TMA zero-fills a block's channels past c_in without reading memory, and
// the MMA issuer skips the 32-byte K steps past them).  Measured on YOLOv8n's
// 3x3 convs with 80 input channels: 128-byte blocks (one stage per tap) take
// two thirds of the time of 32-byte ones (three stages).
int pick_bk_taps(int c_bytes) {
    const int stages = (c_bytes + 127) / 128;
    for (int bk : {32, 64})
        if ((c_bytes + bk - 1) / bk == stages) return bk;
    return 128;
}

int pick_bn(int c_out) {
    if (c_out <= 256) return c_out;  // c_out % 16 == 0 is required
    int best = 16;
    long best_cost = -1;
    for (int bn = 256; bn >= 64; bn -= 16) {
        long tiles = (c_out + bn - 1) / bn;
        long cost = tiles * bn;  // padded columns
        if (best_cost < 0 || cost < best_cost) { best_cost = cost; best = bn; }
    }
    return best;
}

// Spatial tile: tw*th <= 128 minimising the number of tiles (then prefer wider rows).
void pick_tile(int ho, int wo, int *tw, int *th) {
    long best = -1;
    for (int w = std::min(wo, 128); w >= 1; w--) {
        int h = std::min(128 / w, ho);
        if (h < 1) continue;
        long tiles = (long)((wo + w - 1) / w) * ((ho + h - 1) / h);
        if (best < 0 || tiles < best) { best = tiles; *tw = w; *th = h; }
    }
}

size_t al1k(size_t v) { return (v + 1023) & ~size_t(1023); }

uint32_t swizzle_layout(int bk) { return bk == 128 ? 2u : (bk == 64 ? 4u : 6u); }  // SW128 / SW64 / SW32

CUtensorMapSwizzle swizzle_enum(int bk) {
    return bk == 128 ? CU_TENSOR_MAP_SWIZZLE_128B : (bk == 64 ? CU_TENSOR_MAP_SWIZZLE_64B : CU_TENSOR_MAP_SWIZZLE_32B);
}

// dynamic share (the tap and K-step tables are static)
constexpr size_t kSmemLimit = 227 * 1024 - sizeof(int4) * kTapTable - sizeof(int2) * kMmaTable;

// Halo mode plan (stride-1 convs with several taps).  A row block is 8 output
// columns x 16 rows (the 8 rows of a core matrix are 8 neighbouring pixels);
// a tile is rw blocks across and R / rw down.  A stage holds, for one K block
// of bk bytes, the halo plane of each 16-byte channel chunk, and either every
// tap's bn x bk weight slice or -- resident weights, when the conv has a single
// channel tile and all its weights fit beside the stages -- nothing else (the
// weights are loaded once per CTA).
struct HaloPlan {
    bool ok = false;
    int R = 1, rw = 1, bn = 16, bk = 32, tiles_w = 1, tiles_h = 1, n_tiles = 1, wres = 0, tpair = 0;
    int s2 = 0, tkh = 0, tkw = 0, dy0 = 0, dx0 = 0;  // stride-2 plan over the parity planes
    uint32_t plane = 0, w_bytes = 0;
};

// The taps of a stride-2 conv over the parity planes: kernel row kh reads input
// row 2 oy + kh - pt = 2 (oy + dy) + ph with ph = (kh - pt) mod 2, so dy runs
// from floor(-pt / 2) to floor((k_h - 1 - pt) / 2); likewise the columns.
struct S2Taps {
    int dy0, dx0, tkh, tkw;
};
S2Taps s2_taps(const dw_conv_desc &d) {
    auto fl2 = [](int v) { return v >= 0 ? v / 2 : -((1 - v) / 2); };
    S2Taps t;
    t.dy0 = fl2(-d.pad_t);
    t.dx0 = fl2(-d.pad_l);
    t.tkh = fl2(d.k_h - 1 - d.pad_t) - t.dy0 + 1;
    t.tkw = fl2(d.k_w - 1 - d.pad_l) - t.dx0 + 1;
    return t;
}

uint32_t halo_plane_bytes(const dw_conv_desc &d, int rw, int rh) {
    return (uint32_t)(((size_t)(16 * rh + d.k_h - 1) * (size_t)(8 * rw + d.k_w - 1) * 16 + 127) & ~size_t(127));
}

// Output-channel tile for the per-stage weights: all of c_out when the taps'
// weight slices stay small, else the width <= cap with the fewest padded columns.
int halo_bn(int c_out16, int taps) {
    int cap = (int)(40 * 1024 / ((size_t)taps * 32)) / 16 * 16;
    cap = std::max(16, std::min(256, cap));
    if (c_out16 <= cap) return c_out16;
    int best = 16;
    long best_cost = -1;
    for (int bn = cap; bn >= 16; bn -= 16) {
        const long cost = (long)((c_out16 + bn - 1) / bn) * bn;
        if (best_cost < 0 || cost < best_cost) { best_cost = cost; best = bn; }
    }
    return best;
}

HaloPlan plan_halo(const dw_backend *be, const dw_conv_desc &d, int ho, int wo, int esize, bool flat) {
    HaloPlan h;
    const int taps = d.k_h * d.k_w;
    // stride 2 (int8, 16 input channels): the parity-plane form.  It pays where
    // the per-tap producer's boxes are half empty (16-byte rows): YOLOv8n b32's
    // 16 -> 32 stem conv 80 -> 67 us; with 32 or 64 input channels the 4 x c_in
    // K of the regrouped taps costs more MMAs than the per-tap producer's TMA
    // boxes cost (47 -> 49, 29 -> 49 us).  Its zero weight slices would meet
    // infinities in fp16 (0 * inf), so fp16 stays with the per-tap producer.
    // DW_UMMA_HALO_S2: 0 = never, 2 = any channel count (tests and tuning).
    const char *s2_env = getenv("DW_UMMA_HALO_S2");
    const int s2_mode = s2_env ? atoi(s2_env) : 1;
    const bool s2 = d.stride_h == 2 && d.stride_w == 2 && esize == 1 && d.h % 2 == 0 && d.w % 2 == 0 &&
                    s2_mode != 0 && (s2_mode == 2 || d.c_in == 16);
    if (flat || (!s2 && (d.stride_h != 1 || d.stride_w != 1)) || taps < 2 || taps > kTapTable) return h;
    if ((d.c_in * esize) % 16 || (esize == 2 && d.c_in % 16)) return h;  // fp16: whole 32-byte K steps
    if (8 + d.k_w - 1 > 256 || 16 + d.k_h - 1 > 256) return h;
    if (const char *e = getenv("DW_UMMA_HALO"))  // tuning switch: 0 keeps the per-tap producer
        if (atoi(e) == 0) return h;
    const S2Taps st = s2_taps(d);
    // the halo's kernel extent: the conv's own, or the taps over the parity planes
    const int ekh = s2 ? st.tkh : d.k_h, ekw = s2 ? st.tkw : d.k_w;
    // pixel utilisation of 8 x 16 blocks; small maps keep the per-tap producer
    // (whole images side by side in one row block)
    const double util = (double)ho * wo / ((double)((wo + 7) / 8) * 8 * (double)((ho + 15) / 16) * 16);
    if (util < 0.7) return h;
    // maps of at most 40x40 pixels with 64- or 128-byte channel rows: the per-tap
    // producer's tiles fit them closer than 16 x 16-pixel halo blocks (YOLOv8n
    // b32's 40x40 3x3s with 64 channels 27 -> 23 us, the step 1.747 -> 1.725 ms;
    // with 80 channels the halo stays ahead, 29 vs 37 us)
    if (d.c_in * esize > 32 && (d.c_in * esize) % 32 == 0 && (long)ho * wo <= 40 * 40) return h;
    const int c_out16 = ((d.c_out + 15) / 16) * 16;
    const int cbytes = d.c_in * esize;
    const int chunks = cbytes / 16;
    const size_t chan = al1k(sizeof(ChanSmem));
    int r_env = 8;
    if (const char *e = getenv("DW_UMMA_RMAX")) {  // tuning override, as for the per-tap producer
        const int v = atoi(e);
        if (v >= 1 && v <= 8) r_env = v;
    }
    // K blocks: the fewest padded bytes (cblocks * bk - c_in bytes), then the widest
    auto pick_bk_res = [&]() {
        int best = 32;
        long best_pad = -1;
        for (int bk : {128, 64, 32}) {
            const long pad = (long)((cbytes + bk - 1) / bk) * bk - cbytes;
            if (best_pad < 0 || pad < best_pad) { best_pad = pad; best = bk; }
        }
        return best;
    };
    // Block arrangements, cheapest first.  Cost = waves of tiles over the SMs x
    // (blocks per tile + a tile's fixed overhead in blocks), so padding (more
    // tiles), wave quantisation and per-tile overhead all count; then the least
    // halo per output pixel.  A lexicographic key: a strict weak ordering.  The
    // overhead: 2 blocks for 16-byte channel rows (paired taps, a short K per
    // block), 0.5 for wider rows, whose longer K loop per block leaves the fixed
    // hand-offs a smaller share (measured on B200 for YOLOv8n b32's 3x3 layers:
    // at 80x80 with 32 and 64 channels 16 x 16-pixel tiles beat the 32 x 32 and
    // 16 x 32 ones, conv_78 and conv_79 -8 us each, the step 1.779 -> 1.749 ms;
    // the 16-channel 160x160 layers keep their 32 x 32 tiles).
    const double tile_overhead = cbytes == 16 ? 2.0 : 0.5;
    struct Arr { int rw, rh; long tiles; };
    auto arrangements = [&](int n_tiles, int rmax, Arr *out) {
        int n = 0;
        for (int rw : {1, 2, 4, 8})
            for (int rh = 1; rw * rh <= rmax; rh++) {
                const long tw = (wo + 8 * rw - 1) / (8 * rw), th = (ho + 16 * rh - 1) / (16 * rh);
                out[n++] = Arr{rw, rh, (long)d.n * tw * th * n_tiles};
            }
        auto key = [&](const Arr &a) {
            const long waves = (a.tiles + be->sm_count - 1) / be->sm_count;
            const double cost = (double)waves * (a.rw * a.rh + tile_overhead);
            const double halo = (double)(16 * a.rh + ekh - 1) * (8 * a.rw + ekw - 1) / (double)(a.rw * a.rh * kBM);
            return std::make_tuple(cost, halo, a.rw);
        };
        std::sort(out, out + n, [&](const Arr &a, const Arr &b) { return key(a) < key(b); });
        if (const char *e = getenv("DW_UMMA_ARR")) {  // tuning override "rw,rh": that arrangement only
            int rw = 0, rh = 0;
            if (sscanf(e, "%d,%d", &rw, &rh) == 2)
                for (int i = 0; i < n; i++)
                    if (out[i].rw == rw && out[i].rh == rh) {
                        out[0] = out[i];
                        return 1;
                    }
        }
        return n;
    };
    Arr arr[64];
    if (s2) {
        // stride 2: resident weights as 16-byte slices [tap][chunk] over the 4 x
        // c_in / 16 chunks of the parity planes (zero slices for the (tap, parity)
        // pairs no kernel tap maps to); a K block = cps chunk planes, every tap
        const int chunks2 = 4 * chunks, taps2 = st.tkh * st.tkw;
        if (c_out16 > 256 || taps2 * chunks2 / 2 > kMmaTable) return h;
        const int bn = c_out16;
        const size_t w_bytes = (size_t)taps2 * chunks2 * bn * 16;
        const int n = arrangements(1, std::min(r_env, std::max(1, std::min(8, 256 / bn))), arr);
        for (int i = 0; i < n; i++) {
            const int R = arr[i].rw * arr[i].rh;
            const uint32_t plane = (uint32_t)(((size_t)(16 * arr[i].rh + st.tkh - 1) *
                                                   (size_t)(8 * arr[i].rw + st.tkw - 1) * 16 + 127) & ~size_t(127));
            for (int cps : {8, 4, 2}) {
                if (chunks2 % cps) continue;
                const size_t stage = al1k((size_t)cps * plane);
                const size_t fixed = 1024 + al1k((size_t)R * kBM * bn) + al1k(w_bytes) + chan + 512;
                if (fixed < kSmemLimit && (kSmemLimit - fixed) / stage >= 3) {
                    if (2 * arr[i].tiles < be->sm_count && !getenv("DW_UMMA_HALO_ANY_SIZE")) return h;
                    h.ok = true; h.wres = 1; h.R = R; h.rw = arr[i].rw; h.bn = bn; h.bk = 16 * cps; h.n_tiles = 1;
                    h.s2 = 1; h.tkh = st.tkh; h.tkw = st.tkw; h.dy0 = st.dy0; h.dx0 = st.dx0;
                    h.tiles_w = (wo + 8 * h.rw - 1) / (8 * h.rw);
                    h.tiles_h = (ho + 16 * arr[i].rh - 1) / (16 * arr[i].rh);
                    h.plane = plane;
                    h.w_bytes = (uint32_t)w_bytes;
                    return h;
                }
            }
        }
        return h;
    }
    // 1. resident weights: one channel tile, all weights beside >= 3 halo
    // stages.  Arrangements in cost order; for each, the K block with the least
    // padding first, then narrower ones (smaller stages).  A single row block
    // per tile loses to the per-tap producer once channel rows are wider than
    // 32 bytes (measured: YOLOv8n's 40x40 128 -> 80 3x3 42 vs 32 us, ResNet-50's
    // 56x56 fp16 64 -> 64 3x3 185 vs 122 us), so such plans are not taken.
    if (c_out16 <= 256 && !getenv("DW_UMMA_NO_WRES")) {
        const int bn = c_out16, bk0 = pick_bk_res();
        // 16-byte channel rows (int8 c_in = 16): no-swizzle weight slices, two taps per K step
        const bool tpair = cbytes == 16 && esize == 1 && !getenv("DW_UMMA_NO_TPAIR");
        const int n = arrangements(1, std::min(r_env, std::max(1, std::min(8, 256 / bn))), arr);
        for (int i = 0; i < n; i++) {
            const int R = arr[i].rw * arr[i].rh;
            if (R == 1 && cbytes > 32) continue;
            // wide rows on maps the tiles cover with > 30% padding (40x40 under
            // 16 x 16 tiles): the per-tap producer's tiles fit them closer
            // (YOLOv8n's 40x40 3x3s: 24.4 vs 24.9 us at 64 channels, 31 vs 33-35 us at 128)
            if (cbytes > 32 && (double)arr[i].tiles * R * kBM > 1.3 * (double)d.n * ho * wo) continue;
            const uint32_t plane = halo_plane_bytes(d, arr[i].rw, arr[i].rh);
            for (int bk : {bk0, 64, 32}) {
                if (bk > bk0) continue;
                const int cblocks = (cbytes + bk - 1) / bk;
                if (!tpair && cblocks * taps * (bk / 32) > kMmaTable) continue;  // the MMA issuer's K-step table
                const size_t w_bytes = tpair ? (size_t)(taps + 1) * bn * 16 : (size_t)taps * cblocks * bn * bk;
                const size_t stage = al1k((size_t)std::min(bk / 16, chunks) * plane);
                const size_t fixed = 1024 + al1k((size_t)R * kBM * bn * esize) + al1k(w_bytes) + chan + 512;
                if (fixed < kSmemLimit && (kSmemLimit - fixed) / stage >= 3) {
                    // too few tiles to give half the SMs one (batch 1): the per-tap
                    // planner spreads such problems wider (fewer row blocks, narrower
                    // tiles); DW_UMMA_HALO_ANY_SIZE keeps them here (tests of the halo path)
                    if (2 * arr[i].tiles < be->sm_count && !getenv("DW_UMMA_HALO_ANY_SIZE")) return h;
                    h.ok = true; h.wres = 1; h.R = R; h.rw = arr[i].rw; h.bn = bn; h.bk = bk; h.n_tiles = 1;
                    h.tpair = tpair ? 1 : 0;
                    h.tiles_w = (wo + 8 * h.rw - 1) / (8 * h.rw);
                    h.tiles_h = (ho + 16 * arr[i].rh - 1) / (16 * arr[i].rh);
                    h.plane = plane;
                    h.w_bytes = (uint32_t)w_bytes;
                    return h;
                }
            }
        }
    }
    // 2. per-stage weights, for channel rows of at most 32 bytes: there the
    // per-tap producer's boxes are half empty and re-read every pixel nine
    // times, and a stage with every tap's weight slice stays small.  With wider
    // rows a stage's weight boxes need 32-byte K blocks to fit, whose TMA
    // requests cost more than the halo saves (measured on B200: YOLOv8n's
    // 64-channel 3x3s 23 -> 27 us, ResNet-50's 14x14 256-channel fp16 3x3s
    // 51 -> 141 us; 16 and 32 channels 77 -> 59 and 40 -> 30 us).
    if (cbytes > 32 && !getenv("DW_UMMA_HALO_WIDE")) return h;
    h.bn = halo_bn(c_out16, taps);
    h.n_tiles = (d.c_out + h.bn - 1) / h.bn;
    const int cap_bk = ((cbytes + 31) / 32) * 32;
    const int n = arrangements(h.n_tiles, std::min(r_env, std::max(1, std::min(8, 256 / h.bn))), arr);
    for (int i = 0; i < n; i++) {
        const int R = arr[i].rw * arr[i].rh;
        const uint32_t plane = halo_plane_bytes(d, arr[i].rw, arr[i].rh);
        const size_t fixed = 1024 + al1k((size_t)R * kBM * h.bn * esize) + chan + 512;
        for (int bk : {128, 64, 32}) {
            if (bk > cap_bk && bk != 32) continue;
            if ((cbytes + bk - 1) / bk * taps * (bk / 32) > kMmaTable) continue;  // the MMA issuer's K-step table
            const size_t stage = al1k((size_t)std::min(bk / 16, chunks) * plane) + al1k((size_t)taps * h.bn * bk);
            const size_t fit = fixed < kSmemLimit ? (kSmemLimit - fixed) / stage : 0;
            if (fit >= 3 || (bk == 32 && fit >= 2)) {
                if (2 * arr[i].tiles < be->sm_count && !getenv("DW_UMMA_HALO_ANY_SIZE")) return h;  // as above
                h.ok = true; h.R = R; h.rw = arr[i].rw; h.bk = bk; h.plane = plane;
                h.tiles_w = (wo + 8 * h.rw - 1) / (8 * h.rw);
                h.tiles_h = (ho + 16 * arr[i].rh - 1) / (16 * arr[i].rh);
                return h;
            }
        }
    }
    return h;
}

}  // namespace

bool umma_supported(const dw_backend *be, const dw_conv_desc &d, int ho, int wo) {
    if (!be->encode_tiled) return false;
    if (d.group != 1 || d.c_in % 16 || d.c_out % 16) return false;
    const bool flat = d.k_h == 1 && d.k_w == 1 && d.stride_h == 1 && d.stride_w == 1 && d.pad_t == 0 &&
                      d.pad_l == 0 && d.pad_b == 0 && d.pad_r == 0;
    if (!flat && (d.h % d.stride_h || d.w % d.stride_w)) return false;
    if ((long long)d.n * ho * wo >= (1ll << 31)) return false;
    if ((long long)d.k_h * d.k_w >= (1 << 16) || d.k_h * d.k_w * (long long)d.c_in >= (1ll << 31)) return false;
    return true;
}

bool umma_supported_f16(const dw_backend *be, const dw_conv_desc &d, int ho, int wo) {
    if (!be->encode_tiled) return false;
    // 16-byte TMA strides: c_in, c_out multiples of 8 halves
    if (d.group != 1 || d.c_in % 8 || d.c_out % 8) return false;
    const bool flat = d.k_h == 1 && d.k_w == 1 && d.stride_h == 1 && d.stride_w == 1 && d.pad_t == 0 &&
                      d.pad_l == 0 && d.pad_b == 0 && d.pad_r == 0;
    if (!flat && (d.h % d.stride_h || d.w % d.stride_w)) return false;
    // With stride_w > 1 the activation view's innermost dimension holds the
    // stride_w column phases side by side; a K block wider than the channels
    // left would read the next phase's values.  Their weights are zero, but
    // 0 * inf is NaN in floating point, so K blocks must divide c_in (32-byte
    // blocks divide c_in when c_in % 16 == 0).
    if (!flat && d.stride_w > 1 && d.c_in % 16) return false;
    if ((long long)d.n * ho * wo >= (1ll << 31)) return false;
    if ((long long)d.k_h * d.k_w >= (1 << 16) || d.k_h * d.k_w * (long long)d.c_in >= (1ll << 31)) return false;
    return true;
}

namespace {

// Shared launcher: esize 1 = int8 (kind::i8, requant epilogue), 2 = fp16
// (kind::f16, f16 epilogue with bias and ReLU).
dw_status launch_umma_conv(dw_backend *be, const dw_conv_desc &d, int ho, int wo, const void *x, const void *w_ohwi,
                           const EpiParams &ep, void *y, int esize, const uint16_t *bias_f16, int relu,
                           const uint16_t *res_f16, int x_pitch, int y_pitch, const int8_t *res_i8 = nullptr,
                           int res_pitch = 0, float add_ra = 0.0f, float add_rb = 0.0f) {
    const char *op = esize == 2 ? "conv2d_f16" : "conv2d_i8";
    if (((uintptr_t)x & 15) || ((uintptr_t)w_ohwi & 15) || ((uintptr_t)y & 15))
        return dw_fail(be, DW_ERR_INVALID_ARG, "%s (tensor-core path): buffers must be 16-byte aligned", op);
    UmmaParams p{};
    const bool flat = d.k_h == 1 && d.k_w == 1 && d.stride_h == 1 && d.stride_w == 1 && d.pad_t == 0 &&
                      d.pad_l == 0 && d.pad_b == 0 && d.pad_r == 0;
    // Pixel pitches (elements between consecutive pixels; a channel range of a
    // wider tensor).  The tensor maps keep the conv's own channel extents, so a
    // K block past c_in is zero-filled, never read; a strided conv's view packs
    // the stride's column phases side by side and needs pitch == c_in.
    if (!x_pitch) x_pitch = d.c_in;
    if (!y_pitch) y_pitch = d.c_out;
    if (x_pitch < d.c_in || y_pitch < d.c_out || (x_pitch != d.c_in && d.stride_w > 1) ||
        ((size_t)x_pitch * esize) % 16 || ((size_t)y_pitch * esize) % 16)
        return dw_fail(be, DW_ERR_UNSUPPORTED, "%s (tensor-core path): pitch %d/%d unsupported for this shape", op,
                       x_pitch, y_pitch);
    p.mode = flat ? 0 : 1;
    p.esize = esize;
    p.bias_f16 = bias_f16;
    p.res_f16 = res_f16;
    p.add_ra = add_ra;
    p.add_rb = add_rb;
    if (!res_pitch) res_pitch = d.c_out;
    if (res_i8 && (esize != 1 || ((uintptr_t)res_i8 & 15) || res_pitch < d.c_out || res_pitch % 16))
        return dw_fail(be, DW_ERR_UNSUPPORTED, "%s: an int8 residual needs 16-byte alignment and pitch", op);
    p.relu = relu;
    p.swz = 0;
    if (res_f16 && (!flat || ((uintptr_t)res_f16 & 15)))
        return dw_fail(be, DW_ERR_UNSUPPORTED, "%s: a fused residual needs a 1x1 stride-1 conv and a 16-byte aligned buffer", op);
    p.n_img = d.n; p.ho = ho; p.wo = wo; p.c_out = d.c_out;
    p.taps = d.k_h * d.k_w; p.k_h = d.k_h; p.kw = d.k_w; p.sh = d.stride_h; p.sw = d.stride_w; p.pt = d.pad_t; p.pl = d.pad_l;
    p.c_in = d.c_in;
    p.rw = 1;
    const HaloPlan hp = plan_halo(be, d, ho, wo, esize, flat);
    if (hp.ok) {
        p.mode = 2;
        p.bk = hp.bk;
        p.bk_elems = p.bk / esize;
        p.cblocks = (d.c_in + p.bk_elems - 1) / p.bk_elems;
        p.bn = hp.bn;
        p.n_tiles = hp.n_tiles;
        p.R = hp.R;
        p.rw = hp.rw;
        p.tw = 8; p.th = 16; p.nb = 1;
        p.tiles_w = hp.tiles_w;
        p.tiles_h = hp.tiles_h;
        p.m_tiles = d.n * p.tiles_w * p.tiles_h;
        p.num_tiles = p.m_tiles * p.n_tiles;
        p.s2 = hp.s2;
        p.tkh = hp.tkh; p.tkw = hp.tkw; p.dy0 = hp.dy0; p.dx0 = hp.dx0;
        p.hw = 8 * p.rw + (p.s2 ? p.tkw : d.k_w) - 1;
        p.hh = 16 * (p.R / p.rw) + (p.s2 ? p.tkh : d.k_h) - 1;
        p.wres = hp.wres;
        p.w_bytes = hp.w_bytes;
        p.chunks = d.c_in * esize / 16 * (p.s2 ? 4 : 1);
        p.cps = p.bk / 16;
        if (p.s2) p.cblocks = p.chunks / p.cps;  // K blocks over the parity planes' chunks
        p.chunk_elems = 16 / esize;
        p.plane_stride = hp.plane;
        p.tpair = hp.tpair;
        p.b_tap_bytes = (uint32_t)(p.bn * ((p.tpair || p.s2) ? 16 : p.bk));
        p.a_tx_bytes = 0;  // per chunk: hw * hh * 16 bytes (the producer counts them)
        // Whole-row boxes where the data is contiguous: the TMA moves a box row by
        // row, so a halo of hw * hh 16-byte rows costs far more than hh rows of
        // hw * 16 bytes (and likewise for the stores).
        const bool no_flat = getenv("DW_UMMA_NO_FLAT") != nullptr;  // tuning switch: 16-byte rows throughout
        p.flat_in = (!no_flat && !p.s2 && p.chunks == 1 && x_pitch == d.c_in && 2 * p.hw <= 256) ? 1 : 0;
        p.flat_out = (!no_flat && esize == 1 && p.bn == d.c_out && y_pitch == d.c_out) ? 1 : 0;
    } else {
        p.bn = pick_bn(((d.c_out + 15) / 16) * 16);
        // 1x1 convs with a short K and more than 256 output channels (epilogue-
        // bound): half-width tiles of two row blocks, both MMA issuers busy
        // (MobileNetV2's 96 -> 576 expand at b32: 128 x 192 tiles 159 us,
        // 256 x 96 tiles 151 us, measured on B200)
        if (flat && d.c_out > 256 && d.c_in * esize <= 256 && p.bn > 128 && (p.bn / 2) % 16 == 0) p.bn /= 2;
        // The fewest K blocks (then the least padding): a block's padding costs no
        // memory reads (TMA zero fill) and no MMAs (the issuer skips the 32-byte K
        // steps past c_in), while every extra block is a pipeline stage more per
        // tile.  1x1 convs take it unless the wider A stage leaves fewer row blocks
        // per tile (R is capped by a 32 KiB A stage): MobileNetV2's expand (K = 96,
        // R = 2 either way) 3 x 32-byte blocks 166 us, one 128-byte block 159 us,
        // its project (K = 576) 9 x 64 bytes 86 us, 5 x 128 bytes 80 us; YOLOv8n's
        // 96 -> 32 C2f convs keep 32-byte blocks and 8 row blocks (128-byte blocks
        // allow 2: 1.5 us slower each); measured on B200.
        p.bk = pick_bk_taps(d.c_in * esize);
        if (flat) {
            const int bk_pad = pick_bk(d.c_in * esize);
            auto rows_per_tile = [&](int bk) { return std::min({8, 256 / p.bn, 32768 / (kBM * bk)}); };
            if (rows_per_tile(p.bk) < rows_per_tile(bk_pad)) p.bk = bk_pad;
        }
        if (const char *e = getenv("DW_UMMA_BK")) {  // tuning override: 32, 64 or 128 bytes of K per stage
            const int v = atoi(e);
            if (v == 32 || v == 64 || v == 128) p.bk = v;
        }
        if (esize == 2 && !flat && d.stride_w > 1 && (d.c_in * esize) % p.bk) p.bk = pick_bk(d.c_in * esize);
        // 1x1 convs (epilogue-bound: few K steps per tile): a narrower K block when
        // that lets the staging be double-buffered (the fp16 staging of a 128 x 256
        // tile is 64 KiB) -- more K steps, but a tile's stores overlap the next
        // tile's epilogue.
        if (d.k_h * d.k_w == 1) {
            const size_t chan = al1k(sizeof(ChanSmem));
            auto fits2 = [&](int bk) {
                const int r = std::max(1, std::min({8, 256 / p.bn, 32768 / (kBM * bk)}));
                const size_t ob = al1k((size_t)r * kBM * p.bn * esize);
                const size_t sp = al1k((size_t)r * kBM * bk) + al1k((size_t)p.bn * bk);
                return 1024 + 2 * ob + chan + 512 + 2 * sp <= kSmemLimit;
            };
            if (!fits2(p.bk))
                for (int bk = p.bk / 2; bk >= 32; bk /= 2)
                    if (fits2(bk)) {
                        p.bk = bk;
                        break;
                    }
        }
        p.bk_elems = p.bk / esize;
        p.cblocks = (d.c_in + p.bk_elems - 1) / p.bk_elems;
        // Tiles for a tile width bn and at most r_cap row blocks per tile: R * bn <=
        // 256 (two TMEM accumulator buffers within 512 columns), at most 8 (16 for
        // the 16-channel 1x1 case below), and an A stage (R * 128 rows * bk) of at
        // most 32 KiB (64 KiB there).
        auto plan_tiles = [&](int bn, int r_cap) {
            p.bn = bn;
            p.n_tiles = (d.c_out + p.bn - 1) / p.bn;
            // 1x1 int8 convs with 16 output channels (YOLOv8n's stem): up to 16 row
            // blocks (all 512 TMEM columns, 64 KiB A stages) -- twice the work per
            // tile hand-off (the stem conv 102 -> 86 us at b32)
            const bool r16 = flat && bn == 16 && esize == 1;
            int R = std::max(1, std::min({r_cap, r16 ? 16 : 8, 256 / p.bn, (r16 ? 65536 : 32768) / (kBM * p.bk)}));
            if (flat) {
                p.rows = (long long)d.n * d.h * d.w;
                const long long blocks = (p.rows + kBM - 1) / kBM;
                R = (int)std::min<long long>(R, blocks);
                p.R = R;
                p.m_tiles = (int)((blocks + R - 1) / R);
                p.tw = kBM; p.th = 1; p.nb = 1;
                p.a_tx_bytes = (uint32_t)(kBM * p.bk);
            } else {
                pick_tile(ho, wo, &p.tw, &p.th);
                // small maps: a row block holds whole images side by side (7x7: 2 per block)
                p.nb = (p.tw == wo && p.th == ho) ? std::max(1, std::min(kBM / (wo * ho), d.n)) : 1;
                R = std::min(R, (ho + p.th - 1) / p.th);
                p.R = R;
                p.tiles_w = (wo + p.tw - 1) / p.tw;
                p.tiles_h = (ho + p.th * R - 1) / (p.th * R);
                p.m_tiles = ((d.n + p.nb - 1) / p.nb) * p.tiles_w * p.tiles_h;
                p.a_tx_bytes = (uint32_t)(p.tw * p.th * p.nb * p.bk);
            }
            p.num_tiles = p.m_tiles * p.n_tiles;
        };
        if (const char *e = getenv("DW_UMMA_BN")) {  // tuning override: tile width (a multiple of 16, <= 256)
            const int v = atoi(e);
            if (v >= 16 && v <= 256 && v % 16 == 0) p.bn = v;
        }
        int r_cap = 16;  // (the per-shape caps above keep most convs at 8)
        if (const char *e = getenv("DW_UMMA_RMAX")) {  // tuning override: at most this many row blocks per tile
            const int v = atoi(e);
            if (v >= 1 && v <= 16) r_cap = v;
        }
        plan_tiles(p.bn, r_cap);
        // Small problems (tiles for fewer than half the SMs): fewer row blocks per
        // tile, then narrower tiles (down to 64 channels), until half the SMs have a
        // tile -- more CTAs stream the long K loops side by side; the extra reads of
        // the A tiles come from L2.
        while (2 * p.num_tiles < be->sm_count && p.R > 1) plan_tiles(p.bn, p.R - 1);
        while (2 * p.num_tiles < be->sm_count && p.bn >= 128 && (p.bn / 2) % 16 == 0) plan_tiles(p.bn / 2, 1);
    }  // per-tap producer plan
    // fp16 staging in swizzled 64-channel slabs (conflict-free epilogue stores)
    // when every tile's channels split into whole slabs.
    if (esize == 2 && p.bn % 64 == 0 && !getenv("DW_F16_NOSWZ")) p.swz = 1;
    p.chan_all = p.n_tiles * p.bn <= kChanSlots ? 1 : 0;  // every slot a tile reads lies in the arrays
    // Convs with several taps run long MMA phases beside the epilogue, and a TMEM
    // load waits long while the MMAs write the other accumulator buffer: keep the
    // next load in flight (int8 epilogues other than SiLU).  1x1 convs (short MMA
    // phases) do better with two loads per wait (measured on B200: config 1 at
    // N=256 +3%, MobileNetV2's 96 -> 576 expand 173 -> 148 us).
    p.epi_pipe = d.k_h * d.k_w > 1 ? 1 : 0;
    p.n_issuers = (p.R >= 2 && !getenv("DW_UMMA_ONE_ISSUER")) ? 2 : 1;  // DW_UMMA_ONE_ISSUER: tuning switch
    if (const char *e = getenv("DW_UMMA_EPI_PIPE")) p.epi_pipe = atoi(e) != 0;  // tuning override
    p.b_tx_bytes = (uint32_t)(p.bn * p.bk);
    p.a_stage_bytes = (uint32_t)al1k((size_t)p.R * kBM * p.bk);
    p.b_stage_bytes = (uint32_t)al1k((size_t)p.bn * p.bk);
    if (p.mode == 2) {  // the loaded chunk planes; every tap's weight slice unless they are resident
        p.a_stage_bytes = (uint32_t)al1k((size_t)std::min(p.cps, p.chunks) * p.plane_stride);
        p.b_stage_bytes = p.wres ? 0u : (uint32_t)al1k((size_t)p.taps * p.b_tap_bytes);
    }
    const size_t w_region = p.wres ? al1k(p.w_bytes) : 0;
    const size_t out_bytes = al1k((size_t)p.R * kBM * p.bn * esize);
    const size_t chan_bytes = al1k(sizeof(ChanSmem));
    // two staging buffers when they fit beside at least two pipeline stages
    const size_t stage_pair = p.a_stage_bytes + p.b_stage_bytes;
    const size_t min_stages = p.wres ? 3 : 2;
    p.nbuf = (1024 + 2 * out_bytes + chan_bytes + 512 + w_region + min_stages * stage_pair <= kSmemLimit) ? 2 : 1;
    if (const char *e = getenv("DW_UMMA_NBUF"))  // tuning override: 1 staging buffer (room for more stages)
        if (atoi(e) == 1) p.nbuf = 1;
    p.out_bytes = (uint32_t)out_bytes;
    const size_t fixed = 1024 /*align slack*/ + p.nbuf * out_bytes + chan_bytes + 512 /*barriers*/ + w_region;
    int stages = (int)((kSmemLimit - fixed) / stage_pair);
    p.stages = std::max(2, std::min(stages, kMaxStages));
    // [stages x (A, B)] [resident weights] [staging x nbuf] [channel parameters] [barriers]
    p.off_w = (uint32_t)((size_t)p.stages * stage_pair);
    p.off_out = (uint32_t)(p.off_w + w_region);
    p.off_chan = (uint32_t)(p.off_out + p.nbuf * out_bytes);
    p.off_bars = (uint32_t)(p.off_chan + chan_bytes);
    p.acc_bound = (long long)p.taps * d.c_in * 16384ll;
    // At least 116 KiB so that a second CTA never fits on the SM: one CTA per SM
    // owns the tensor memory (its tcgen05.alloc never waits on a neighbour).
    const size_t smem = std::max<size_t>(1024 + p.off_bars + 512, 116 * 1024);
    if (smem > kSmemLimit) return dw_fail(be, DW_ERR_UNSUPPORTED, "%s: tile does not fit in shared memory", op);
    // tcgen05 instruction descriptor: kind::i8: D = s32 (bits 4-5 = 2), A = B = s8
    // (bits 7-9, 10-12 = 1); kind::f16: D = f32 (bits 4-5 = 1), A = B = f16 (0).
    // Both K-major, N >> 3 at bits 17-22, M >> 4 at bits 24-28.
    const uint32_t fmt = esize == 2 ? ((1u << 4)) : ((2u << 4) | (1u << 7) | (1u << 10));
    p.idesc = fmt | ((uint32_t)(p.bn >> 3) << 17) | ((uint32_t)(kBM >> 4) << 24);
    // descriptor high word: SBO = 8 rows * bk bytes (>> 4) at bits 32-45, version 1 at bit 46,
    // swizzle layout at bits 61-63.
    p.desc_hi = ((uint64_t)((8 * p.bk) >> 4) << 32) | (1ull << 46) | ((uint64_t)swizzle_layout(p.bk) << 61);
    uint32_t cols = 32;
    while (cols < (uint32_t)(2 * p.R * p.bn)) cols <<= 1;
    p.tmem_cols = cols;
    p.wait_cap_ns = be->wait_cap_ns;
    p.err = be->dev_err;
    p.ep = ep;

    // ---- tensor maps (dims in elements, strides in bytes)
    const CUtensorMapDataType dt = esize == 2 ? CU_TENSOR_MAP_DATA_TYPE_FLOAT16 : CU_TENSOR_MAP_DATA_TYPE_UINT8;
    const cuuint64_t es = (cuuint64_t)esize;
    CUtensorMap ta, tb;
    CUresult r;
    const CUtensorMapSwizzle sw = swizzle_enum(p.bk);
    if (p.mode == 2 && p.flat_in) {
        // one 16-byte chunk per pixel, dense: [n][h][w * 2] 8-byte units; a halo
        // box is hh rows of hw pixels, zero-filled left and right of the row and
        // above and below the map (the padding)
        cuuint64_t dims[3] = {(cuuint64_t)d.w * 2, (cuuint64_t)d.h, (cuuint64_t)d.n};
        cuuint64_t strides[2] = {(cuuint64_t)d.w * 16, (cuuint64_t)d.h * d.w * 16};
        cuuint32_t box[3] = {(cuuint32_t)(2 * p.hw), (cuuint32_t)p.hh, 1};
        cuuint32_t estr[3] = {1, 1, 1};
        r = be->encode_tiled(&ta, CU_TENSOR_MAP_DATA_TYPE_UINT64, 3, const_cast<void *>(x), dims, strides, box, estr,
                             CU_TENSOR_MAP_INTERLEAVE_NONE, CU_TENSOR_MAP_SWIZZLE_NONE,
                             CU_TENSOR_MAP_L2_PROMOTION_L2_128B, CU_TENSOR_MAP_FLOAT_OOB_FILL_NONE);
    } else if (p.mode == 2 && p.s2) {
        // parity planes: the stride-2 view [n][h/2][2 row phases][w/2][2 column
        // phases x c_in]; a box is one 16-byte chunk of one (row, column) phase,
        // hh x hw positions, zero-filled outside the image (the padding)
        cuuint64_t dims[5] = {2 * (cuuint64_t)d.c_in, (cuuint64_t)(d.w / 2), 2, (cuuint64_t)(d.h / 2), (cuuint64_t)d.n};
        cuuint64_t strides[4] = {2 * (cuuint64_t)x_pitch * es, (cuuint64_t)d.w * x_pitch * es,
                                 2 * (cuuint64_t)d.w * x_pitch * es, (cuuint64_t)d.h * d.w * x_pitch * es};
        cuuint32_t box[5] = {(cuuint32_t)p.chunk_elems, (cuuint32_t)p.hw, 1, (cuuint32_t)p.hh, 1};
        cuuint32_t estr[5] = {1, 1, 1, 1, 1};
        r = be->encode_tiled(&ta, dt, 5, const_cast<void *>(x), dims, strides, box, estr, CU_TENSOR_MAP_INTERLEAVE_NONE,
                             CU_TENSOR_MAP_SWIZZLE_NONE, CU_TENSOR_MAP_L2_PROMOTION_L2_128B,
                             CU_TENSOR_MAP_FLOAT_OOB_FILL_NONE);
    } else if (p.mode == 2) {
        // halo boxes: one 16-byte channel chunk of (16 R + k_h - 1) x (8 + k_w - 1)
        // pixels, no swizzle; out-of-range pixels (the padding) are zero-filled
        cuuint64_t dims[4] = {(cuuint64_t)d.c_in, (cuuint64_t)d.w, (cuuint64_t)d.h, (cuuint64_t)d.n};
        cuuint64_t strides[3] = {(cuuint64_t)x_pitch * es, (cuuint64_t)d.w * x_pitch * es,
                                 (cuuint64_t)d.h * d.w * x_pitch * es};
        cuuint32_t box[4] = {(cuuint32_t)p.chunk_elems, (cuuint32_t)p.hw, (cuuint32_t)p.hh, 1};
        cuuint32_t estr[4] = {1, 1, 1, 1};
        r = be->encode_tiled(&ta, dt, 4, const_cast<void *>(x), dims, strides, box, estr, CU_TENSOR_MAP_INTERLEAVE_NONE,
                             CU_TENSOR_MAP_SWIZZLE_NONE, CU_TENSOR_MAP_L2_PROMOTION_L2_128B,
                             CU_TENSOR_MAP_FLOAT_OOB_FILL_NONE);
    } else if (flat) {
        cuuint64_t dims[2] = {(cuuint64_t)d.c_in, (cuuint64_t)p.rows};
        cuuint64_t strides[1] = {(cuuint64_t)x_pitch * es};
        cuuint32_t box[2] = {(cuuint32_t)p.bk_elems, (cuuint32_t)kBM};
        cuuint32_t estr[2] = {1, 1};
        r = be->encode_tiled(&ta, dt, 2, const_cast<void *>(x), dims, strides, box, estr, CU_TENSOR_MAP_INTERLEAVE_NONE,
                             sw, CU_TENSOR_MAP_L2_PROMOTION_L2_256B, CU_TENSOR_MAP_FLOAT_OOB_FILL_NONE);
    } else {
        const int sh = d.stride_h, swd = d.stride_w;
        cuuint64_t dims[5] = {(cuuint64_t)swd * d.c_in, (cuuint64_t)(d.w / swd), (cuuint64_t)sh, (cuuint64_t)(d.h / sh),
                              (cuuint64_t)d.n};
        cuuint64_t strides[4] = {(cuuint64_t)swd * x_pitch * es, (cuuint64_t)d.w * x_pitch * es,
                                 (cuuint64_t)sh * d.w * x_pitch * es, (cuuint64_t)d.h * d.w * x_pitch * es};
        cuuint32_t box[5] = {(cuuint32_t)p.bk_elems, (cuuint32_t)p.tw, 1, (cuuint32_t)p.th, (cuuint32_t)p.nb};
        cuuint32_t estr[5] = {1, 1, 1, 1, 1};
        r = be->encode_tiled(&ta, dt, 5, const_cast<void *>(x), dims, strides, box, estr, CU_TENSOR_MAP_INTERLEAVE_NONE,
                             sw, CU_TENSOR_MAP_L2_PROMOTION_L2_256B, CU_TENSOR_MAP_FLOAT_OOB_FILL_NONE);
    }
    if (r != CUDA_SUCCESS) return dw_fail(be, DW_ERR_DEVICE, "%s: activation tensor map rejected (%d)", op, (int)r);
    {
        cuuint64_t dims[3] = {(cuuint64_t)d.c_in, (cuuint64_t)p.taps, (cuuint64_t)d.c_out};
        cuuint64_t strides[2] = {(cuuint64_t)d.c_in * es, (cuuint64_t)p.taps * d.c_in * es};
        // two-tap K steps: one tap's 16 bytes per row, no swizzle (8-row core matrices)
        cuuint32_t box[3] = {(cuuint32_t)((p.tpair || p.s2) ? 16 / esize : p.bk_elems), 1, (cuuint32_t)p.bn};
        cuuint32_t estr[3] = {1, 1, 1};
        r = be->encode_tiled(&tb, dt, 3, const_cast<void *>(w_ohwi), dims, strides, box, estr,
                             CU_TENSOR_MAP_INTERLEAVE_NONE, (p.tpair || p.s2) ? CU_TENSOR_MAP_SWIZZLE_NONE : sw,
                             CU_TENSOR_MAP_L2_PROMOTION_L2_256B, CU_TENSOR_MAP_FLOAT_OOB_FILL_NONE);
    }
    if (r != CUDA_SUCCESS) return dw_fail(be, DW_ERR_DEVICE, "%s: weight tensor map rejected (%d)", op, (int)r);
    // Output: TMA stores of the staged [rows][bn] tile (swizzled fp16 staging:
    // one store per 64-channel slab); out-of-range rows/pixels/channels are clipped.
    CUtensorMap ty;
    const cuuint32_t st_ch = p.swz ? 64u : (cuuint32_t)p.bn;
    const CUtensorMapSwizzle st_sw = p.swz ? CU_TENSOR_MAP_SWIZZLE_128B : CU_TENSOR_MAP_SWIZZLE_NONE;
    if (flat) {
        cuuint64_t dims[2] = {(cuuint64_t)d.c_out, (cuuint64_t)p.rows};
        cuuint64_t strides[1] = {(cuuint64_t)y_pitch * es};
        cuuint32_t box[2] = {st_ch, (cuuint32_t)kBM};
        cuuint32_t estr[2] = {1, 1};
        r = be->encode_tiled(&ty, dt, 2, y, dims, strides, box, estr, CU_TENSOR_MAP_INTERLEAVE_NONE, st_sw,
                             CU_TENSOR_MAP_L2_PROMOTION_NONE, CU_TENSOR_MAP_FLOAT_OOB_FILL_NONE);
    } else if (p.mode == 2 && p.flat_out) {
        // [n][ho][wo * bn / 8] 8-byte units: a row block's staging [16][8][bn] is
        // 16 rows of 8 * bn contiguous bytes; pixels past the map are clipped
        cuuint64_t dims[3] = {(cuuint64_t)wo * (p.bn / 8), (cuuint64_t)ho, (cuuint64_t)d.n};
        cuuint64_t strides[2] = {(cuuint64_t)wo * d.c_out, (cuuint64_t)ho * wo * d.c_out};
        cuuint32_t box[3] = {(cuuint32_t)p.bn, (cuuint32_t)p.th, 1};
        cuuint32_t estr[3] = {1, 1, 1};
        r = be->encode_tiled(&ty, CU_TENSOR_MAP_DATA_TYPE_UINT64, 3, y, dims, strides, box, estr,
                             CU_TENSOR_MAP_INTERLEAVE_NONE, CU_TENSOR_MAP_SWIZZLE_NONE, CU_TENSOR_MAP_L2_PROMOTION_NONE,
                             CU_TENSOR_MAP_FLOAT_OOB_FILL_NONE);
    } else {
        cuuint64_t dims[4] = {(cuuint64_t)d.c_out, (cuuint64_t)wo, (cuuint64_t)ho, (cuuint64_t)d.n};
        cuuint64_t strides[3] = {(cuuint64_t)y_pitch * es, (cuuint64_t)wo * y_pitch * es,
                                 (cuuint64_t)ho * wo * y_pitch * es};
        cuuint32_t box[4] = {st_ch, (cuuint32_t)p.tw, (cuuint32_t)p.th, (cuuint32_t)p.nb};
        cuuint32_t estr[4] = {1, 1, 1, 1};
        r = be->encode_tiled(&ty, dt, 4, y, dims, strides, box, estr, CU_TENSOR_MAP_INTERLEAVE_NONE, st_sw,
                             CU_TENSOR_MAP_L2_PROMOTION_NONE, CU_TENSOR_MAP_FLOAT_OOB_FILL_NONE);
    }
    if (r != CUDA_SUCCESS) return dw_fail(be, DW_ERR_DEVICE, "%s: output tensor map rejected (%d)", op, (int)r);
    // fp16 residual: the output's 2-D view over the residual buffer (loads into the staging tile)
    CUtensorMap tr = ty;
    if (res_f16) {
        cuuint64_t dims[2] = {(cuuint64_t)d.c_out, (cuuint64_t)p.rows};
        cuuint64_t strides[1] = {(cuuint64_t)d.c_out * es};
        cuuint32_t box[2] = {st_ch, (cuuint32_t)kBM};
        cuuint32_t estr[2] = {1, 1};
        r = be->encode_tiled(&tr, dt, 2, const_cast<uint16_t *>(res_f16), dims, strides, box, estr,
                             CU_TENSOR_MAP_INTERLEAVE_NONE, st_sw, CU_TENSOR_MAP_L2_PROMOTION_L2_256B,
                             CU_TENSOR_MAP_FLOAT_OOB_FILL_NONE);
        if (r != CUDA_SUCCESS) return dw_fail(be, DW_ERR_DEVICE, "%s: residual tensor map rejected (%d)", op, (int)r);
    }
    // int8 residual: the output's map over the residual (view) buffer
    if (res_i8) {
        const cuuint64_t rp = (cuuint64_t)res_pitch;
        if (flat) {
            cuuint64_t dims[2] = {(cuuint64_t)d.c_out, (cuuint64_t)p.rows};
            cuuint64_t strides[1] = {rp};
            cuuint32_t box[2] = {st_ch, (cuuint32_t)kBM};
            cuuint32_t estr[2] = {1, 1};
            r = be->encode_tiled(&tr, dt, 2, const_cast<int8_t *>(res_i8), dims, strides, box, estr,
                                 CU_TENSOR_MAP_INTERLEAVE_NONE, st_sw, CU_TENSOR_MAP_L2_PROMOTION_L2_256B,
                                 CU_TENSOR_MAP_FLOAT_OOB_FILL_NONE);
        } else {
            cuuint64_t dims[4] = {(cuuint64_t)d.c_out, (cuuint64_t)wo, (cuuint64_t)ho, (cuuint64_t)d.n};
            cuuint64_t strides[3] = {rp, (cuuint64_t)wo * rp, (cuuint64_t)ho * wo * rp};
            cuuint32_t box[4] = {st_ch, (cuuint32_t)p.tw, (cuuint32_t)p.th, (cuuint32_t)p.nb};
            cuuint32_t estr[4] = {1, 1, 1, 1};
            r = be->encode_tiled(&tr, dt, 4, const_cast<int8_t *>(res_i8), dims, strides, box, estr,
                                 CU_TENSOR_MAP_INTERLEAVE_NONE, st_sw, CU_TENSOR_MAP_L2_PROMOTION_L2_256B,
                                 CU_TENSOR_MAP_FLOAT_OOB_FILL_NONE);
        }
        if (r != CUDA_SUCCESS) return dw_fail(be, DW_ERR_DEVICE, "%s: residual tensor map rejected (%d)", op, (int)r);
    }

    using KernelFn = void (*)(CUtensorMap, CUtensorMap, CUtensorMap, CUtensorMap, UmmaParams);
    static const KernelFn f16_kernels[8] = {
        k_umma_conv_i8<false, true, 0>, k_umma_conv_i8<false, true, 1>, k_umma_conv_i8<false, true, 2>,
        k_umma_conv_i8<false, true, 3>, k_umma_conv_i8<false, true, 4>, k_umma_conv_i8<false, true, 5>,
        k_umma_conv_i8<false, true, 6>, k_umma_conv_i8<false, true, 7>};
    static bool attr_set[16] = {};
    int dev = be->device;
    if (dev < 16 && !attr_set[dev]) {
        cudaFuncSetAttribute(k_umma_conv_i8<false, false, 0>, cudaFuncAttributeMaxDynamicSharedMemorySize,
                             (int)kSmemLimit);
        cudaFuncSetAttribute(k_umma_conv_i8<true, false, 0>, cudaFuncAttributeMaxDynamicSharedMemorySize,
                             (int)kSmemLimit);
        cudaFuncSetAttribute(k_umma_conv_i8<false, false, 2>, cudaFuncAttributeMaxDynamicSharedMemorySize,
                             (int)kSmemLimit);
        cudaFuncSetAttribute(k_umma_conv_i8<true, false, 2>, cudaFuncAttributeMaxDynamicSharedMemorySize,
                             (int)kSmemLimit);
        cudaFuncSetAttribute(k_umma_conv_i8<false, false, 0, true>, cudaFuncAttributeMaxDynamicSharedMemorySize,
                             (int)kSmemLimit);
        cudaFuncSetAttribute(k_umma_conv_i8<false, false, 2, true>, cudaFuncAttributeMaxDynamicSharedMemorySize,
                             (int)kSmemLimit);
        for (KernelFn f : f16_kernels)
            cudaFuncSetAttribute(f, cudaFuncAttributeMaxDynamicSharedMemorySize, (int)kSmemLimit);
        attr_set[dev] = true;
    }
    const int grid = std::min(p.num_tiles, be->sm_count);
    // Launched as a programmatic dependent of the previous kernel on the stream
    // (the kernel waits for it after its prologue: griddepcontrol.wait), so the
    // launch and the prologue overlap the previous grid's last wave.
    // DW_PDL=0: tuning switch, plain stream order.
    static const bool pdl = !(getenv("DW_PDL") && atoi(getenv("DW_PDL")) == 0);
    auto launch = [&](KernelFn k, int threads) {
        cudaLaunchConfig_t cfg = {};
        cfg.gridDim = dim3((unsigned)grid);
        cfg.blockDim = dim3((unsigned)threads);
        cfg.dynamicSmemBytes = smem;
        cfg.stream = be->stream;
        cudaLaunchAttribute attr[1];
        attr[0].id = cudaLaunchAttributeProgrammaticStreamSerialization;
        attr[0].val.programmaticStreamSerializationAllowed = 1;
        cfg.attrs = attr;
        cfg.numAttrs = pdl ? 1 : 0;
        return cudaLaunchKernelEx(&cfg, k, ta, tb, ty, tr, p);
    };
    cudaError_t le;
    if (esize == 2) {
        const int fm = (bias_f16 ? 1 : 0) | (res_f16 ? 2 : 0) | (relu ? 4 : 0);
        le = launch(f16_kernels[fm], umma_threads(false, true));
    } else if (res_i8) {
        if (ep.epilogue == DW_EPI_SILU)
            le = launch(k_umma_conv_i8<true, false, 2>, umma_threads(true, false));
        else if (p.epi_pipe)
            le = launch(k_umma_conv_i8<false, false, 2, true>, umma_threads(false, false));
        else
            le = launch(k_umma_conv_i8<false, false, 2>, umma_threads(false, false));
    } else if (ep.epilogue == DW_EPI_SILU) {
        le = launch(k_umma_conv_i8<true, false, 0>, umma_threads(true, false));
    } else if (p.epi_pipe) {
        le = launch(k_umma_conv_i8<false, false, 0, true>, umma_threads(false, false));
    } else {
        le = launch(k_umma_conv_i8<false, false, 0>, umma_threads(false, false));
    }
    if (le != cudaSuccess) return dw_cuda_check(be, le, esize == 2 ? "umma_conv_f16 launch" : "umma_conv_i8 launch");
    return dw_after_launch(be, esize == 2 ? "umma_conv_f16" : "umma_conv_i8");
}

}  // namespace

dw_status launch_umma_conv_i8(dw_backend *be, const dw_conv_desc &d, int ho, int wo, const int8_t *x,
                              const int8_t *w_ohwi, const EpiParams &ep, int8_t *y) {
    return launch_umma_conv(be, d, ho, wo, x, w_ohwi, ep, y, 1, nullptr, 0, nullptr, 0, 0);
}

dw_status launch_umma_conv_i8_view(dw_backend *be, const dw_conv_desc &d, int ho, int wo, const int8_t *x, int x_pitch,
                                   const int8_t *w_ohwi, const EpiParams &ep, int8_t *y, int y_pitch) {
    return launch_umma_conv(be, d, ho, wo, x, w_ohwi, ep, y, 1, nullptr, 0, nullptr, x_pitch, y_pitch);
}

dw_status launch_umma_conv_add_i8_view(dw_backend *be, const dw_conv_desc &d, int ho, int wo, const int8_t *x,
                                       int x_pitch, const int8_t *w_ohwi, const EpiParams &ep, const int8_t *res,
                                       int res_pitch, float ra, float rb, int8_t *y, int y_pitch) {
    return launch_umma_conv(be, d, ho, wo, x, w_ohwi, ep, y, 1, nullptr, 0, nullptr, x_pitch, y_pitch, res, res_pitch,
                            ra, rb);
}

dw_status launch_umma_conv_f16(dw_backend *be, const dw_conv_desc &d, int ho, int wo, const uint16_t *x,
                               const uint16_t *w_ohwi, const uint16_t *bias, int relu, uint16_t *y,
                               const uint16_t *residual) {
    EpiParams ep{nullptr, nullptr, nullptr, DW_EPI_NONE, 127, 0.0f};
    return launch_umma_conv(be, d, ho, wo, x, w_ohwi, ep, y, 2, bias, relu, residual, 0, 0);
}

}  // namespace dw
