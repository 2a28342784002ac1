// yolo_post.cu -- the tail of the YOLOv8 Detect head and the detection
// post-processing, on the device.
//
//  * dw_yolo_detect_i8: from the int8 outputs of the head's last box and class
//    convolutions to the exported model's output [n, 4 + nc, anchors] (f32):
//    DFL (softmax over reg_max bins, then the expectation), dist2bbox around
//    the grid-cell centres times the level's stride, sigmoid of the class
//    logits, levels concatenated.  The reference runs these as separate f32
//    graph ops after DequantizeLinear: Softmax (crates/dragonwing-cpu/src/
//    ops.rs:1609-1640), Conv with the bin-index kernel (conv2d_f32_nhwc,
//    ops.rs:1356-1420), Sub/Add/Div/Mul (runtime.rs:1674-1850), Sigmoid
//    (sigmoid_f32_scalar, ops.rs:1865-1870), Concat.
//  * dw_postprocess_yolo: decode_detections_v8 / _alt, nms / nms_agnostic and
//    postprocess_yolo (crates/dragonwing-onnx/src/postprocess.rs:78-340) with the
//    reference's output order.
//
// Exactness.  Every float operation is one IEEE round-to-nearest add,
// multiply or divide in the reference's order (__fadd_rn and friends are never
// contracted into FMA).  The exponentials come from tables that
// dw_prepare_yolo_detect fills with the host's libm expf, the function the
// reference's f32::exp calls: the tail's inputs are int8 levels, so a sigmoid
// input takes one of 256 values per level and a softmax term exp(x_i - max)
// one of 256 x 256.  The tail is therefore bit-identical with the reference's
// f32 ops, and the post-processing (comparisons, IoU) with its decode and NMS.

#include <algorithm>
#include <climits>
#include <cmath>
#include <cstring>
#include <vector>

#include "dw_device.cuh"

namespace {

constexpr int kRegMax = 16;
constexpr int kTableLevel = 256 + 256 * 256;  // floats per level: sigmoid[256], then softmax terms[256][256]
constexpr int kDetThreads = 128;
constexpr int kDecodeThreads = 256;
constexpr int kMaxAnchors = 16384;  // the NMS sorts an image's candidates in shared memory
constexpr float kModelSize = 640.0f;  // postprocess.rs:98 (the reference's fixed model input size)

inline size_t al256(size_t v) { return (v + 255) & ~size_t(255); }

// ---------------------------------------------------------------------------
// Detect tail
// ---------------------------------------------------------------------------

struct DetectLevel {
    const int8_t *box;  // [n, h, w, 4 * reg_max]
    const int8_t *cls;  // [n, h, w, nc]
    int h, w, off;      // grid, first anchor index of the level
    float stride;
};

struct DetectParams {
    DetectLevel lv[DW_YOLO_MAX_LEVELS];
    int levels, nc, A;
    const float *tables;
    float *out;  // [n, 4 + nc, A]
};

__device__ __forceinline__ int sbyte(uint32_t w, int i) { return (int)(int8_t)(w >> (8 * i)); }

// One anchor per thread.  The box bytes (64 per anchor) and class bytes are
// read with 16-byte loads; the output rows are written coalesced across the
// warp (consecutive anchors are consecutive floats of each row).
template <bool kVec16>
__global__ void __launch_bounds__(kDetThreads) k_yolo_detect(const DetectParams p) {
    __shared__ float sig[DW_YOLO_MAX_LEVELS][256];
    for (int i = threadIdx.x; i < p.levels * 256; i += kDetThreads)
        sig[i >> 8][i & 255] = p.tables[(size_t)(i >> 8) * kTableLevel + (i & 255)];
    __syncthreads();
    const int a = blockIdx.x * kDetThreads + threadIdx.x;
    const int img = blockIdx.y;
    if (a >= p.A) return;
    int l = 0;
    DetectLevel L = p.lv[0];
#pragma unroll
    for (int k = 1; k < DW_YOLO_MAX_LEVELS; k++)
        if (k < p.levels && a >= p.lv[k].off) {
            l = k;
            L = p.lv[k];
        }
    const int local = a - L.off;
    const int gy = local / L.w, gx = local - gy * L.w;
    const size_t pix = (size_t)img * L.h * L.w + local;

    // DFL: per side, softmax over the 16 bins (max-subtracted, sum in bin
    // order, multiply by 1/sum: ops.rs:1621-1637), then sum_i p_i * i from 0
    // in bin order (the 1x1 conv with kernel 0..15, ops.rs:1396-1415).
    const float *dfl = p.tables + (size_t)l * kTableLevel + 256;
    const uint4 *bp = reinterpret_cast<const uint4 *>(L.box + pix * (4 * kRegMax));
    float dist[4];
#pragma unroll
    for (int s = 0; s < 4; s++) {
        const uint4 v = __ldg(bp + s);
        const uint32_t wv[4] = {v.x, v.y, v.z, v.w};
        uint32_t m = __vmaxs4(__vmaxs4(v.x, v.y), __vmaxs4(v.z, v.w));
        m = __vmaxs4(m, m >> 16);
        m = __vmaxs4(m, m >> 8);
        // x_i = q_i * s is increasing in q_i (s > 0), so max_i x_i = q_max * s
        const float *row = dfl + (sbyte(m, 0) + 128) * 256 + 128;
        float e[kRegMax];
        float sum = 0.0f;
#pragma unroll
        for (int i = 0; i < kRegMax; i++) {
            e[i] = __ldg(row + sbyte(wv[i >> 2], i & 3));
            sum = __fadd_rn(sum, e[i]);
        }
        const float inv = __fdiv_rn(1.0f, sum);
        float acc = 0.0f;
#pragma unroll
        for (int i = 0; i < kRegMax; i++) acc = __fadd_rn(acc, __fmul_rn(__fmul_rn(e[i], inv), (float)i));
        dist[s] = acc;
    }
    // dist2bbox (xywh): x1y1 = anchor - lt, x2y2 = anchor + rb, centre =
    // (x1y1 + x2y2) / 2, size = x2y2 - x1y1, all times the stride; anchors at
    // the cell centres (x + 0.5, y + 0.5).
    const float ax = (float)gx + 0.5f, ay = (float)gy + 0.5f;
    const float x1 = __fsub_rn(ax, dist[0]), y1 = __fsub_rn(ay, dist[1]);
    const float x2 = __fadd_rn(ax, dist[2]), y2 = __fadd_rn(ay, dist[3]);
    const size_t A = (size_t)p.A;
    float *o = p.out + (size_t)img * (4 + p.nc) * A + a;
    o[0] = __fmul_rn(__fdiv_rn(__fadd_rn(x1, x2), 2.0f), L.stride);
    o[A] = __fmul_rn(__fdiv_rn(__fadd_rn(y1, y2), 2.0f), L.stride);
    o[2 * A] = __fmul_rn(__fsub_rn(x2, x1), L.stride);
    o[3 * A] = __fmul_rn(__fsub_rn(y2, y1), L.stride);

    // class scores: sigmoid(q * s) from the level's table
    const float *sg = sig[l] + 128;
    float *oc = o + 4 * A;
    const int8_t *cp = L.cls + pix * p.nc;
    if (kVec16) {
        for (int c0 = 0; c0 < p.nc; c0 += 16) {
            const uint4 v = __ldg(reinterpret_cast<const uint4 *>(cp + c0));
            const uint32_t wv[4] = {v.x, v.y, v.z, v.w};
#pragma unroll
            for (int i = 0; i < 16; i++) oc[(size_t)(c0 + i) * A] = sg[sbyte(wv[i >> 2], i & 3)];
        }
    } else {
        for (int c = 0; c < p.nc; c++) oc[(size_t)c * A] = sg[cp[c]];
    }
}

// ---------------------------------------------------------------------------
// Post-processing (postprocess.rs:78-340) in four kernels:
//   decode   one thread per anchor (all images): best class, threshold, corners
//   rank     one CTA per image: candidates compacted in anchor order, stable
//            radix sort by confidence descending (= the reference's stable
//            sort_by), stable radix sort of that order by class (one segment
//            per class, rank order inside it), class-ordered boxes staged
//   nms      the greedy loop per class segment: segments of up to 64
//            candidates one warp each; larger ones taken from a work queue by
//            persistent 512-thread CTAs, in batches of 128 candidates
//   order    one CTA per image: the reference's swap_remove order, records out
// ---------------------------------------------------------------------------

constexpr int kRankThreads = 1024;
constexpr int kSegThreads = 512;
constexpr int kSegWarps = kSegThreads / 32;
constexpr int kBoxCap = 4096;  // segment staged in shared memory: boxes, spans, lists, flags (100 KB)
constexpr int kSmallSeg = 64;  // segments up to this size: one warp each
constexpr int kHugeSeg = 1024; // segments over this size are taken first

// Workspace, per image of A anchors (by anchor unless noted).
struct PostWs {
    float4 *box;      // [n, A] decoded corners
    uint32_t *cls;    // [n, A] best class
    float *conf;      // [n, A] best confidence
    uint8_t *flag;    // [n, A] 1: a candidate (best >= threshold)
    uint16_t *ra;     // [n, A] rank -> anchor
    uint16_t *crank;  // [n, A] class-grouped position -> rank
    float4 *cbox;     // [n, A] class-grouped position -> box
    uint32_t *seg;    // [n, A + 1] segment starts (class-grouped positions), then the candidate count
    uint8_t *keep;    // [n, A] by rank
    uint16_t *list0;  // [n, A] NMS live lists (class-grouped positions), double-buffered
    uint16_t *list1;
    uint32_t *cnt;    // [n] candidates
    uint32_t *nseg;   // [n] class segments
    uint32_t *qhuge;  // [n * qcap] (image << 16 | segment) of segments over kHugeSeg candidates
    uint32_t *qbig;   // [n * qcap] of segments over kSmallSeg candidates (and up to kHugeSeg)
    uint32_t *qcnt;   // [4] items in qhuge, in qbig; items taken from each
};

struct DecodeParams {
    const float *raw;
    int nc, A;
    float sx, sy, iw, ih, thr;
    PostWs w;
};

// kAlt: raw is [n, A, 4 + nc] (decode_detections_v8_alt) instead of [n, 4 + nc, A].
template <bool kAlt>
__global__ void __launch_bounds__(kDecodeThreads) k_yolo_decode(const DecodeParams p) {
    const int img = blockIdx.y;
    const int a = blockIdx.x * kDecodeThreads + threadIdx.x;
    if (a >= p.A) return;
    const size_t row = 4 + (size_t)p.nc;
    const float *r = p.raw + (size_t)img * row * p.A;
    const size_t step = kAlt ? 1 : (size_t)p.A;
    const float *q = kAlt ? r + (size_t)a * row : r + a;
    const float cx = q[0], cy = q[step], w = q[2 * step], h = q[3 * step];
    // best class: strict '>' from 0.0, class 0 by default (postprocess.rs:110-119)
    float best = 0.0f;
    uint32_t bc = 0;
    for (int c = 0; c < p.nc; c++) {
        const float v = q[(4 + (size_t)c) * step];
        if (v > best) {
            best = v;
            bc = (uint32_t)c;
        }
    }
    const bool cand = !(best < p.thr);  // skipped when best_conf < conf_threshold (:122)
    const size_t gi = (size_t)img * p.A + a;
    p.w.flag[gi] = cand ? 1 : 0;
    if (cand) {
        const float hw = __fdiv_rn(w, 2.0f), hh = __fdiv_rn(h, 2.0f);
        // (cx -/+ w / 2) * scale, then .max(0.0).min(size) (:127-136)
        const float x1 = fminf(fmaxf(__fmul_rn(__fsub_rn(cx, hw), p.sx), 0.0f), p.iw);
        const float y1 = fminf(fmaxf(__fmul_rn(__fsub_rn(cy, hh), p.sy), 0.0f), p.ih);
        const float x2 = fminf(fmaxf(__fmul_rn(__fadd_rn(cx, hw), p.sx), 0.0f), p.iw);
        const float y2 = fminf(fmaxf(__fmul_rn(__fadd_rn(cy, hh), p.sy), 0.0f), p.ih);
        p.w.box[gi] = make_float4(x1, y1, x2, y2);
        p.w.cls[gi] = bc;
        p.w.conf[gi] = best;
    }
}

// Detection::area (postprocess.rs:28-32), operation for operation.
__device__ __forceinline__ float area_ref(float4 b) {
    return __fmul_rn(fmaxf(__fsub_rn(b.z, b.x), 0.0f), fmaxf(__fsub_rn(b.w, b.y), 0.0f));
}

__device__ __forceinline__ int warp_incl_scan(int v) {
    const int lane = threadIdx.x & 31;
#pragma unroll
    for (int d = 1; d < 32; d <<= 1) {
        const int u = __shfl_up_sync(0xffffffffu, v, d);
        if (lane >= d) v += u;
    }
    return v;
}

// Exclusive prefix sum of one int per thread over a 1024-thread block; the
// block total in *total.  Every thread calls it.
__device__ int block_excl_scan(int v, int *wsum, int *total) {
    const int lane = threadIdx.x & 31, warp = threadIdx.x >> 5;
    const int incl = warp_incl_scan(v);
    if (lane == 31) wsum[warp] = incl;
    __syncthreads();
    if (warp == 0) wsum[lane] = warp_incl_scan(wsum[lane]);
    __syncthreads();
    *total = wsum[31];
    const int r = incl - v + (warp ? wsum[warp - 1] : 0);
    __syncthreads();
    return r;
}

// One stable LSD radix pass over the 8-bit digit at `sh` of ka[0, c) (payload
// va) into kb / vb, by a 1024-thread block.  Warp w owns the elements
// [w*EW, (w+1)*EW) in order; ranks inside a warp come from __match_any_sync
// over 32 elements at a time, and the (digit, warp) counts are scanned in
// digit-major order, so equal digits keep their order.  Returns false, having
// moved nothing, when every key has the same digit.
__device__ bool radix_pass(const uint32_t *ka, const uint16_t *va, uint32_t *kb, uint16_t *vb, int c, int sh,
                           uint16_t *hist, int *wsum) {
    const int tid = threadIdx.x, lane = tid & 31, warp = tid >> 5;
    const uint32_t d0 = (ka[0] >> sh) & 255u;
    bool same = true;
    for (int i = tid; i < c; i += kRankThreads) same &= ((ka[i] >> sh) & 255u) == d0;
    if (__syncthreads_and(same)) return false;
    for (int i = tid; i < 256 * 32; i += kRankThreads) hist[i] = 0;
    __syncthreads();
    const int R = (c + kRankThreads - 1) / kRankThreads;  // rounds of 32 per warp (<= 16)
    const int EW = R * 32;
    uint32_t lr[8];
#pragma unroll
    for (int r = 0; r < 16; r++) {
        if (r < R) {
            const int idx = warp * EW + r * 32 + lane;
            const bool valid = idx < c;
            const uint32_t d = valid ? (ka[idx] >> sh) & 255u : 256u;
            const unsigned peers = __match_any_sync(0xffffffffu, d);
            uint32_t base = valid ? hist[d * 32 + warp] : 0u;
            __syncwarp();
            if (valid && lane == __ffs(peers) - 1) hist[d * 32 + warp] = (uint16_t)(base + __popc(peers));
            __syncwarp();
            const uint32_t rk = base + __popc(peers & ((1u << lane) - 1));
            if (r & 1)
                lr[r >> 1] |= rk << 16;
            else
                lr[r >> 1] = rk;
        }
    }
    __syncthreads();
    uint32_t h[8];
    int sum = 0;
#pragma unroll
    for (int i = 0; i < 8; i++) {
        h[i] = hist[tid * 8 + i];
        sum += (int)h[i];
    }
    int total;
    int ex = block_excl_scan(sum, wsum, &total);
#pragma unroll
    for (int i = 0; i < 8; i++) {
        hist[tid * 8 + i] = (uint16_t)ex;
        ex += (int)h[i];
    }
    __syncthreads();
#pragma unroll
    for (int r = 0; r < 16; r++) {
        if (r < R) {
            const int idx = warp * EW + r * 32 + lane;
            if (idx < c) {
                const uint32_t k = ka[idx], d = (k >> sh) & 255u;
                const int dest = (int)hist[d * 32 + warp] + (int)((lr[r >> 1] >> ((r & 1) * 16)) & 0xFFFFu);
                kb[dest] = k;
                vb[dest] = va[idx];
            }
        }
    }
    __syncthreads();
    return true;
}

struct RankParams {
    int A, cap;
    bool sort_conf;  // false: no NMS, candidates stay in anchor order
    bool nms;
    bool group;      // class-aware: one segment per class (agnostic: one segment)
    PostWs w;
};

__global__ void __launch_bounds__(kRankThreads, 1) k_yolo_rank(const RankParams p) {
    extern __shared__ __align__(16) unsigned char sm[];
    const int cap = p.cap;
    uint32_t *ka = reinterpret_cast<uint32_t *>(sm), *kb = ka + cap;
    uint16_t *va = reinterpret_cast<uint16_t *>(kb + cap), *vb = va + cap;
    uint16_t *hist = vb + cap;  // [256 * 32]
    __shared__ int wsum[32];
    const int img = blockIdx.x, tid = threadIdx.x, A = p.A;
    const size_t base = (size_t)img * A;

    // candidates in anchor order (the order decode_detections_v8 pushes them)
    // thread t owns anchors [16t, 16t + 16) (A <= 16384); all its loads are
    // issued before any is used
    const int a0 = tid * 16;
    uint32_t fl = 0;
#pragma unroll
    for (int i = 0; i < 16; i++)
        if (a0 + i < A && p.w.flag[base + a0 + i]) fl |= 1u << i;
    float cf[16];
#pragma unroll
    for (int i = 0; i < 16; i++) cf[i] = ((fl >> i) & 1u) ? p.w.conf[base + a0 + i] : 0.0f;
    int c;
    int pos = block_excl_scan(__popc(fl), wsum, &c);
#pragma unroll
    for (int i = 0; i < 16; i++)
        if ((fl >> i) & 1u) {
            ka[pos] = ~__float_as_uint(cf[i]);  // conf >= +0, never NaN: ascending = descending conf
            va[pos] = (uint16_t)(a0 + i);
            pos++;
        }
    __syncthreads();
    if (p.sort_conf && c > 1)
        for (int sh = 0; sh < 32; sh += 8)
            if (radix_pass(ka, va, kb, vb, c, sh, hist, wsum)) {
                uint32_t *tk = ka; ka = kb; kb = tk;
                uint16_t *tv = va; va = vb; vb = tv;
            }
    for (int r = tid; r < c; r += kRankThreads) p.w.ra[base + r] = va[r];
    if (tid == 0) p.w.cnt[img] = (uint32_t)c;
    if (!p.nms) {
        if (tid == 0) p.w.nseg[img] = 0;
        return;
    }
    // class grouping: keys = class (0 for agnostic), payload = rank
    {
        uint32_t cl[kMaxAnchors / kRankThreads];
#pragma unroll
        for (int t = 0; t < kMaxAnchors / kRankThreads; t++) {
            const int r = tid + t * kRankThreads;
            cl[t] = (p.group && r < c) ? p.w.cls[base + va[r]] : 0u;
        }
#pragma unroll
        for (int t = 0; t < kMaxAnchors / kRankThreads; t++) {
            const int r = tid + t * kRankThreads;
            if (r < c) {
                kb[r] = cl[t];
                vb[r] = (uint16_t)r;
            }
        }
    }
    __syncthreads();
    {
        uint32_t *tk = ka; ka = kb; kb = tk;
        uint16_t *tv = va; va = vb; vb = tv;
    }
    if (p.group && c > 1)
        for (int sh = 0; sh < 32; sh += 8)
            if (radix_pass(ka, va, kb, vb, c, sh, hist, wsum)) {
                uint32_t *tk = ka; ka = kb; kb = tk;
                uint16_t *tv = va; va = vb; vb = tv;
            }
    // class-grouped ranks and boxes (the rank -> anchor map was stored above;
    // the barrier inside the sort or below makes it visible to the block)
    __syncthreads();
    {
        uint16_t an[kMaxAnchors / kRankThreads];
#pragma unroll
        for (int t = 0; t < kMaxAnchors / kRankThreads; t++) {
            const int k = tid + t * kRankThreads;
            an[t] = k < c ? p.w.ra[base + va[k]] : 0;
        }
#pragma unroll
        for (int t = 0; t < kMaxAnchors / kRankThreads; t++) {
            const int k = tid + t * kRankThreads;
            if (k < c) {
                p.w.crank[base + k] = va[k];
                p.w.cbox[base + k] = p.w.box[base + an[t]];
            }
        }
    }
    // segment starts in order
    const int E2 = (c + kRankThreads - 1) / kRankThreads;
    const int k0 = tid * E2;
    int local = 0;
    for (int i = 0; i < E2; i++) {
        const int k = k0 + i;
        if (k < c && (k == 0 || ka[k] != ka[k - 1])) local++;
    }
    int nseg;
    pos = block_excl_scan(local, wsum, &nseg);
    uint32_t *seg = p.w.seg + (size_t)img * (A + 1);
    for (int i = 0; i < E2; i++) {
        const int k = k0 + i;
        if (k < c && (k == 0 || ka[k] != ka[k - 1])) seg[pos++] = (uint32_t)k;
    }
    if (tid == 0) {
        seg[nseg] = (uint32_t)c;
        p.w.nseg[img] = (uint32_t)nseg;
    }
    __syncthreads();
    // large segments go to the work queues of k_yolo_nms_segment
    for (int i = tid; i < nseg; i += kRankThreads) {
        const int m = (int)(seg[i + 1] - seg[i]);
        if (m > kHugeSeg)
            p.w.qhuge[atomicAdd(&p.w.qcnt[0], 1u)] = ((uint32_t)img << 16) | (uint32_t)i;
        else if (m > kSmallSeg)
            p.w.qbig[atomicAdd(&p.w.qcnt[1], 1u)] = ((uint32_t)img << 16) | (uint32_t)i;
    }
}

struct SegNmsParams {
    int A, cap;     // cap: boxes staged in shared memory per segment
    float gx, gy;   // grid cells per pixel (kGrid / image size; 0 disables the grid)
    double mid;     // halfway between the IoU threshold t and the next float above it
    bool tie_up;    // that next float has an even significand (an exact tie rounds up to it)
    bool zero_gt;   // 0.0 > t (the IoU of a pair whose union is not positive)
    PostWs w;
};

constexpr int kBatch = 32;     // candidates resolved together by one warp (small segments)
constexpr int kBigBatch = 128; // by a block (large segments)

// iou(a, b) > t (postprocess.rs:36-55, 251) without the division: the
// reference compares q' = RN(inter / union) with t.  For union > 0, q' > t
// exactly when the real quotient q = inter / union lies above the midpoint
// between t and the next float (or on it, when rounding to even goes up).
// inter > mid * union decides q > mid exactly in double: mid has at most 25
// significant bits and union 24, so the product is exact.  inter, union and
// the areas are the reference's float operations, in its order.
__device__ __forceinline__ bool iou_gt(const SegNmsParams &p, float4 a, float area_a, float4 b, float area_b) {
    const float x1 = fmaxf(a.x, b.x), y1 = fmaxf(a.y, b.y);
    const float x2 = fminf(a.z, b.z), y2 = fminf(a.w, b.w);
    // disjoint boxes: the intersection is 0, so the IoU is 0 (the union is finite)
    if (!(x2 > x1 && y2 > y1)) return p.zero_gt;
    const float inter = __fmul_rn(fmaxf(__fsub_rn(x2, x1), 0.0f), fmaxf(__fsub_rn(y2, y1), 0.0f));
    const float uni = __fsub_rn(__fadd_rn(area_a, area_b), inter);
    if (!(uni > 0.0f)) return p.zero_gt;
    const double lhs = (double)inter, rhs = __dmul_rn(p.mid, (double)uni);
    return lhs > rhs || (lhs == rhs && p.tie_up);
}

constexpr int kGrid = 16;  // cells per image side for the overlap prefilter

// The cells [xl, xh] x [yl, yh] a box's interior can touch, packed in bytes.
// Cell of x = floor(x * gx); the ends use round-down / round-up products, so
// the span always contains the cells of the box's points, and two boxes with
// a common interior point have intersecting spans (a necessary condition for
// a positive intersection, hence for IoU > t when t >= 0).
__device__ __forceinline__ uint32_t box_span(const SegNmsParams &p, float4 b) {
    const int xl = min(max((int)floorf(__fmul_rd(b.x, p.gx)), 0), kGrid - 1);
    const int xh = min(max((int)floorf(__fmul_ru(b.z, p.gx)), 0), kGrid - 1);
    const int yl = min(max((int)floorf(__fmul_rd(b.y, p.gy)), 0), kGrid - 1);
    const int yh = min(max((int)floorf(__fmul_ru(b.w, p.gy)), 0), kGrid - 1);
    return (uint32_t)xl | ((uint32_t)xh << 8) | ((uint32_t)yl << 16) | ((uint32_t)yh << 24);
}

// Exclusive prefix sum over a kSegThreads block (every thread calls it).
__device__ int seg_excl_scan(int v, int *wsum, int *total) {
    const int lane = threadIdx.x & 31, warp = threadIdx.x >> 5;
    const int incl = warp_incl_scan(v);
    if (lane == 31) wsum[warp] = incl;
    __syncthreads();
    int before = 0, all = 0;
#pragma unroll
    for (int w = 0; w < kSegThreads / 32; w++) {
        const int t = wsum[w];
        before += w < warp ? t : 0;
        all += t;
    }
    *total = all;
    __syncthreads();
    return incl - v + before;
}

// Spans (box_span) that share a cell in both directions.
__device__ __forceinline__ bool spans_meet(uint32_t a, uint32_t b) {
    return (a & 255u) <= ((b >> 8) & 255u) && (b & 255u) <= ((a >> 8) & 255u) &&
           ((a >> 16) & 255u) <= (b >> 24) && ((b >> 16) & 255u) <= (a >> 24);
}

// nms (postprocess.rs:233-255) on the class segments of more than kSmallSeg
// candidates, taken from the work queues by persistent CTAs.  A segment is
// processed in batches.  The live list holds, in rank order, the candidates no
// kept box has suppressed yet.  Its first (up to) 128 entries are resolved in
// order: each is kept unless an earlier kept entry of the batch overlaps it by
// IoU > threshold (the boxes kept in earlier batches have already removed
// everything they suppress); the 128 x 128 overlap bits are computed in
// parallel (pairs whose grid cells do not meet are skipped) and the order is
// resolved on bit masks.  Then the threads test the rest of the list
// (round-robin) against the batch's kept boxes whose grid cells meet its own
// and the survivors are compacted, in order, into the next list.  The kept set
// equals the reference's sequential greedy loop.
__global__ void __launch_bounds__(kSegThreads) k_yolo_nms_segment(const SegNmsParams p) {
    extern __shared__ __align__(16) unsigned char smraw[];
    float4 *sb = reinterpret_cast<float4 *>(smraw);           // [cap] staged boxes
    uint32_t *ss = reinterpret_cast<uint32_t *>(sb + p.cap);     // [cap] cell spans
    uint16_t *sl = reinterpret_cast<uint16_t *>(ss + p.cap);     // [2 * cap] live lists
    uint8_t *sk = reinterpret_cast<uint8_t *>(sl + 2 * p.cap);   // [cap] kept flags
    __shared__ float4 bb[kBigBatch];
    __shared__ float ba[kBigBatch];
    __shared__ uint32_t bs[kBigBatch];
    __shared__ unsigned long long sup[2][kBigBatch];  // earlier batch entries overlapping entry b (128 bits)
    __shared__ unsigned long long s_kept[2];
    __shared__ __align__(16) unsigned colw[kGrid][4], roww[kGrid][4];  // kept entries touching each column / row
    __shared__ int wsum[kSegThreads / 32];
    __shared__ uint32_t smask[32 * kSegWarps];  // survivor ballots per (round, warp)
    __shared__ int soff[32 * kSegWarps];
    __shared__ int s_item;
    const int tid = threadIdx.x, lane = tid & 31, warp = tid >> 5;
    for (;;) {
        // next segment: the huge ones first
        if (tid == 0) {
            int it = -1;
            const uint32_t h = atomicAdd(&p.w.qcnt[2], 1u);
            if (h < p.w.qcnt[0]) {
                it = (int)p.w.qhuge[h];
            } else {
                const uint32_t g = atomicAdd(&p.w.qcnt[3], 1u);
                if (g < p.w.qcnt[1]) it = (int)p.w.qbig[g];
            }
            s_item = it;
        }
        __syncthreads();
        const int item = s_item;
        if (item < 0) return;
        const int img = item >> 16, si = item & 0xFFFF;
        const size_t base = (size_t)img * p.A;
        const uint32_t *seg = p.w.seg + (size_t)img * (p.A + 1);
        const int s = (int)seg[si], m = (int)seg[si + 1] - s;
        const float4 *gb = p.w.cbox + base + s;
        const uint16_t *cr = p.w.crank + base + s;
        const bool staged = m <= p.cap;  // boxes, spans, live lists and flags on chip
        uint16_t *cur = staged ? sl : p.w.list0 + base + s, *nxt = staged ? sl + p.cap : p.w.list1 + base + s;
        for (int j = tid; j < m; j += kSegThreads) {
            if (staged) {
                const float4 b = gb[j];
                sb[j] = b;
                ss[j] = box_span(p, b);
                sk[j] = 0;
            } else {
                p.w.keep[base + cr[j]] = 0;
            }
            cur[j] = (uint16_t)j;
        }
        __syncthreads();
        int len = m;
        while (len > 0) {
            const int nb = min(kBigBatch, len);
            if (tid < nb) {
                const int q = cur[tid];
                const float4 b = staged ? sb[q] : gb[q];
                bb[tid] = b;
                ba[tid] = area_ref(b);
                bs[tid] = staged ? ss[q] : box_span(p, b);
                sup[0][tid] = 0;
                sup[1][tid] = 0;
            }
            __syncthreads();
            {   // overlap bits: 4 threads per entry b, each over every 4th earlier entry a
                const int b = tid & (kBigBatch - 1), q = tid >> 7;
                unsigned long long m0 = 0, m1 = 0;
                if (b < nb) {
                    const float4 bx = bb[b];
                    const float ax = ba[b];
                    const uint32_t sx = bs[b];
                    for (int a = q; a < b; a += kSegThreads / kBigBatch)
                        if ((p.zero_gt || spans_meet(bs[a], sx)) && iou_gt(p, bb[a], ba[a], bx, ax)) {
                            if (a < 64)
                                m0 |= 1ull << a;
                            else
                                m1 |= 1ull << (a - 64);
                        }
                    if (m0) atomicOr(&sup[0][b], m0);
                    if (m1) atomicOr(&sup[1][b], m1);
                }
            }
            __syncthreads();
            // resolve the batch's order: entry b is kept unless a kept earlier entry
            // overlaps it.  Warp 0 settles, each round, every entry whose earlier
            // overlapping entries are all settled (the lowest unsettled one always
            // is, so at most nb rounds); lane l owns entries l, l+32, l+64, l+96.
            if (warp == 0) {
                unsigned long long d0[4], d1[4];
#pragma unroll
                for (int e = 0; e < 4; e++) {
                    const int bi = lane + 32 * e;
                    d0[e] = bi < nb ? sup[0][bi] : 0ull;
                    d1[e] = bi < nb ? sup[1][bi] : 0ull;
                }
                const unsigned long long all0 = nb >= 64 ? ~0ull : ((1ull << nb) - 1);
                const unsigned long long all1 = nb <= 64 ? 0ull : (nb == 128 ? ~0ull : ((1ull << (nb - 64)) - 1));
                unsigned long long R0 = 0, R1 = 0, K0 = 0, K1 = 0;
                unsigned settled = 0, kept = 0;  // bit e: entry lane + 32e
                for (int round = 0; round < kBigBatch && ((R0 & all0) != all0 || (R1 & all1) != all1); round++) {
#pragma unroll
                    for (int e = 0; e < 4; e++) {
                        const int bi = lane + 32 * e;
                        if (bi < nb && !((settled >> e) & 1u) && !(d0[e] & ~R0) && !(d1[e] & ~R1)) {
                            settled |= 1u << e;
                            if (!((d0[e] & K0) | (d1[e] & K1))) kept |= 1u << e;
                        }
                    }
                    const unsigned s0 = __ballot_sync(0xffffffffu, settled & 1u), s1 = __ballot_sync(0xffffffffu, settled & 2u);
                    const unsigned s2 = __ballot_sync(0xffffffffu, settled & 4u), s3 = __ballot_sync(0xffffffffu, settled & 8u);
                    const unsigned k0 = __ballot_sync(0xffffffffu, kept & 1u), k1 = __ballot_sync(0xffffffffu, kept & 2u);
                    const unsigned k2 = __ballot_sync(0xffffffffu, kept & 4u), k3 = __ballot_sync(0xffffffffu, kept & 8u);
                    R0 = (unsigned long long)s0 | ((unsigned long long)s1 << 32);
                    R1 = (unsigned long long)s2 | ((unsigned long long)s3 << 32);
                    K0 = (unsigned long long)k0 | ((unsigned long long)k1 << 32);
                    K1 = (unsigned long long)k2 | ((unsigned long long)k3 << 32);
                }
                if (lane == 0) {
                    s_kept[0] = K0;
                    s_kept[1] = K1;
                }
            }
            __syncthreads();
            const unsigned long long K0 = s_kept[0], K1 = s_kept[1];
            // kept boxes stay at their batch index; per grid column / row, which
            // of them touch it (128 bits as 4 words, word w = entries 32w..32w+31)
            if (tid < kBigBatch) {
                const bool kb = tid < nb && (((tid < 64 ? K0 : K1) >> (tid & 63)) & 1ull);
                if (kb) {
                    if (staged)
                        sk[cur[tid]] = 1;
                    else
                        p.w.keep[base + cr[cur[tid]]] = 1;
                }
                const uint32_t sp = bs[tid];
#pragma unroll
                for (int c = 0; c < kGrid; c++) {
                    const unsigned cb = __ballot_sync(0xffffffffu, kb && (int)(sp & 255u) <= c && c <= (int)((sp >> 8) & 255u));
                    const unsigned rb = __ballot_sync(0xffffffffu, kb && (int)((sp >> 16) & 255u) <= c && c <= (int)(sp >> 24));
                    if (lane == 0) {
                        colw[c][warp] = cb;
                        roww[c][warp] = rb;
                    }
                }
            }
            __syncthreads();
            // the rest of the list, round-robin over the threads (round r, thread
            // t: entry nb + r*kSegThreads + t); survivors compacted in (round,
            // warp, lane) = list order
            const int rest = len - nb;
            const int R = (rest + kSegThreads - 1) / kSegThreads;  // <= 32 (len <= 16384)
            for (int r = 0; r < R; r++) {
                const int idx = nb + r * kSegThreads + tid;
                bool ok = false;
                if (idx < len && !p.zero_gt) {  // zero_gt (t < 0): every pair suppresses
                    const int j = cur[idx];
                    const float4 bj = staged ? sb[j] : gb[j];
                    const float aj = area_ref(bj);
                    const uint32_t sp = staged ? ss[j] : box_span(p, bj);
                    uint4 cm = make_uint4(0, 0, 0, 0), rm = make_uint4(0, 0, 0, 0);
                    for (int c = sp & 255u; c <= (int)((sp >> 8) & 255u); c++) {
                        const uint4 v = *reinterpret_cast<const uint4 *>(colw[c]);
                        cm.x |= v.x; cm.y |= v.y; cm.z |= v.z; cm.w |= v.w;
                    }
                    for (int rr = (sp >> 16) & 255u; rr <= (int)(sp >> 24); rr++) {
                        const uint4 v = *reinterpret_cast<const uint4 *>(roww[rr]);
                        rm.x |= v.x; rm.y |= v.y; rm.z |= v.z; rm.w |= v.w;
                    }
                    // kept batch entries that can overlap this box
                    unsigned cw[4] = {cm.x & rm.x, cm.y & rm.y, cm.z & rm.z, cm.w & rm.w};
                    ok = true;
#pragma unroll
                    for (int w = 0; w < 4; w++) {
                        unsigned cand = cw[w];
                        while (cand && ok) {
                            const int k = 32 * w + __ffs(cand) - 1;
                            cand &= cand - 1;
                            ok = !iou_gt(p, bb[k], ba[k], bj, aj);
                        }
                    }
                }
                const unsigned bal = __ballot_sync(0xffffffffu, ok);
                if (lane == 0) smask[r * kSegWarps + warp] = bal;
            }
            __syncthreads();
            int total;
            const int ent = R * kSegWarps;  // <= kSegThreads
            const int off = seg_excl_scan(tid < ent ? __popc(smask[tid]) : 0, wsum, &total);
            if (tid < ent) soff[tid] = off;
            __syncthreads();
            for (int r = 0; r < R; r++) {
                const unsigned bal = smask[r * kSegWarps + warp];
                if ((bal >> lane) & 1u)
                    nxt[soff[r * kSegWarps + warp] + __popc(bal & ((1u << lane) - 1))] =
                        cur[nb + r * kSegThreads + tid];
            }
            __syncthreads();
            uint16_t *t = cur;
            cur = nxt;
            nxt = t;
            len = total;
        }
        if (staged)
            for (int j = tid; j < m; j += kSegThreads) p.w.keep[base + cr[j]] = sk[j];
        __syncthreads();
    }
}

constexpr int kSmallWarps = 8;

// The same batched rule for a segment of at most kSmallSeg candidates, by one
// warp without block barriers: the overlap bits of a batch come from lane
// shuffles, the order is resolved on bit masks, and the survivors of the rest
// are compacted in order with ballots.
__global__ void __launch_bounds__(kSmallWarps * 32) k_yolo_nms_small(const SegNmsParams p) {
    __shared__ float4 kb[kSmallWarps][kBatch];
    __shared__ float ka[kSmallWarps][kBatch];
    const int img = blockIdx.y, warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
    const int si = blockIdx.x * kSmallWarps + warp;
    if (si >= (int)p.w.nseg[img]) return;
    const size_t base = (size_t)img * p.A;
    const uint32_t *seg = p.w.seg + (size_t)img * (p.A + 1);
    const int s = (int)seg[si], m = (int)seg[si + 1] - s;
    if (m > kSmallSeg) return;  // k_yolo_nms_segment's
    const float4 *gb = p.w.cbox + base + s;
    const uint16_t *cr = p.w.crank + base + s;
    uint16_t *cur = p.w.list0 + base + s, *nxt = p.w.list1 + base + s;
    const unsigned lt = (1u << lane) - 1;
    for (int j = lane; j < m; j += 32) {
        cur[j] = (uint16_t)j;
        p.w.keep[base + cr[j]] = 0;
    }
    __syncwarp();
    int len = m;
    while (len > 0) {
        const int nb = min(kBatch, len);
        const int q = lane < nb ? (int)cur[lane] : 0;
        const float4 b = lane < nb ? gb[q] : make_float4(0.f, 0.f, 0.f, 0.f);
        const float ab = area_ref(b);
        uint32_t sup = 0;
        for (int a = 0; a + 1 < nb; a++) {
            const float4 x = make_float4(__shfl_sync(0xffffffffu, b.x, a), __shfl_sync(0xffffffffu, b.y, a),
                                         __shfl_sync(0xffffffffu, b.z, a), __shfl_sync(0xffffffffu, b.w, a));
            const float ax = __shfl_sync(0xffffffffu, ab, a);
            if (lane > a && lane < nb && iou_gt(p, x, ax, b, ab)) sup |= 1u << a;
        }
        uint32_t K = 0;
        for (int t = 0; t < nb; t++)
            if (!(__shfl_sync(0xffffffffu, sup, t) & K)) K |= 1u << t;
        if (lane < nb && ((K >> lane) & 1u)) {
            const int slot = __popc(K & lt);
            kb[warp][slot] = b;
            ka[warp][slot] = ab;
            p.w.keep[base + cr[q]] = 1;
        }
        __syncwarp();
        const int nk = __popc(K);
        int out = 0;
        for (int i0 = nb; i0 < len; i0 += 32) {
            const int idx = i0 + lane;
            bool ok = false;
            int j = 0;
            if (idx < len) {
                j = cur[idx];
                const float4 bj = gb[j];
                const float aj = area_ref(bj);
                ok = true;
                for (int k = 0; k < nk && ok; k++) ok = !iou_gt(p, kb[warp][k], ka[warp][k], bj, aj);
            }
            const unsigned bal = __ballot_sync(0xffffffffu, ok);
            if (ok) nxt[out + __popc(bal & lt)] = (uint16_t)j;
            out += __popc(bal);
        }
        __syncwarp();
        uint16_t *t = cur;
        cur = nxt;
        nxt = t;
        len = out;
    }
}

struct OrderParams {
    int A, cap;
    bool all_kept;   // no NMS
    PostWs w;
    uint32_t *dets;  // [n, A] records of 6 words: bbox[4], class_id, confidence
    int32_t *counts;
};

// The output order.  The reference deletes the suppressed entries of its
// sorted list with swap_remove from the back (postprocess.rs:257-264).  With K
// kept of c, removing rank r moves the then-last element (position L_r - 1,
// L_r = K + number of removed ranks <= r) into r; a position is final once
// visited, so the element that ends at position p < K is found by following
// p -> L_p - 1 -> ... until a kept rank: pointer jumping, in parallel.
__global__ void __launch_bounds__(kRankThreads, 1) k_yolo_order(const OrderParams p) {
    extern __shared__ __align__(16) unsigned char sm[];
    const int cap = p.cap;
    uint16_t *rem = reinterpret_cast<uint16_t *>(sm);  // [cap] removed ranks <= r
    uint16_t *nxt = rem + cap;                         // [cap] swap_remove links
    uint8_t *keep = reinterpret_cast<uint8_t *>(nxt + cap);
    __shared__ int wsum[32];
    const int img = blockIdx.x, tid = threadIdx.x, A = p.A;
    const size_t base = (size_t)img * A;
    const int c = (int)p.w.cnt[img];
    {
        uint8_t kv[kMaxAnchors / kRankThreads];
#pragma unroll
        for (int t = 0; t < kMaxAnchors / kRankThreads; t++) {
            const int r = tid + t * kRankThreads;
            kv[t] = r < c ? (p.all_kept ? 1 : p.w.keep[base + r]) : 0;
        }
#pragma unroll
        for (int t = 0; t < kMaxAnchors / kRankThreads; t++) {
            const int r = tid + t * kRankThreads;
            if (r < c) keep[r] = kv[t];
        }
    }
    __syncthreads();
    const int E = (c + kRankThreads - 1) / kRankThreads;
    const int r0 = tid * E;
    int local = 0;
    for (int i = 0; i < E; i++) local += (r0 + i < c && !keep[r0 + i]) ? 1 : 0;
    int removed;
    int run = block_excl_scan(local, wsum, &removed);
    for (int i = 0; i < E; i++) {
        const int r = r0 + i;
        if (r < c) {
            run += keep[r] ? 0 : 1;
            rem[r] = (uint16_t)run;
        }
    }
    const int K = c - removed;
    __syncthreads();
    for (int r = tid; r < c; r += kRankThreads) nxt[r] = (uint16_t)(keep[r] ? r : K + rem[r] - 1);
    __syncthreads();
    // chains strictly increase and end at kept ranks: <= 15 doublings for c <= 16384
    for (int it = 0; it < 16; it++) {
        uint16_t tmp[kMaxAnchors / kRankThreads];
        bool changed = false;
#pragma unroll
        for (int t = 0; t < kMaxAnchors / kRankThreads; t++) {
            const int r = tid + t * kRankThreads;
            if (r < c) {
                const uint16_t x = nxt[r], y = nxt[x];
                tmp[t] = y;
                changed |= (y != x);
            }
        }
        __syncthreads();
#pragma unroll
        for (int t = 0; t < kMaxAnchors / kRankThreads; t++) {
            const int r = tid + t * kRankThreads;
            if (r < c) nxt[r] = tmp[t];
        }
        if (!__syncthreads_or(changed)) break;
    }
    for (int q = tid; q < K; q += kRankThreads) {
        const size_t gi = base + p.w.ra[base + nxt[q]];
        const float4 b = p.w.box[gi];
        uint32_t *o = p.dets + (base + q) * 6;
        o[0] = __float_as_uint(b.x);
        o[1] = __float_as_uint(b.y);
        o[2] = __float_as_uint(b.z);
        o[3] = __float_as_uint(b.w);
        o[4] = p.w.cls[gi];
        o[5] = __float_as_uint(p.w.conf[gi]);
    }
    // the records after the last detection are zero (a defined output)
    for (size_t w = (base + K) * 6 + tid; w < (base + A) * 6; w += kRankThreads) p.dets[w] = 0u;
    if (tid == 0) p.counts[img] = K;
}

// ---------------------------------------------------------------------------
// host side
// ---------------------------------------------------------------------------

#define YT(x)                         \
    do {                              \
        dw_status _st = (x);          \
        if (_st != DW_OK) return _st; \
    } while (0)

bool pos_finite(float v) { return std::isfinite(v) && v > 0.0f; }

dw_status check_detect_desc(dw_backend *be, const dw_yolo_detect_desc *d, const char *op, size_t *anchors) {
    if (!d) return dw_fail(be, DW_ERR_INVALID_ARG, "%s: descriptor is null", op);
    if (d->n <= 0 || d->n > 65535 || d->num_classes <= 0 || d->num_classes > 65535)
        return dw_fail(be, DW_ERR_INVALID_ARG, "%s: n=%d and num_classes=%d must be in [1, 65535]", op, d->n,
                       d->num_classes);
    if (d->reg_max != kRegMax)
        return dw_fail(be, DW_ERR_UNSUPPORTED, "%s: reg_max=%d unsupported (the YOLOv8 head has 16)", op, d->reg_max);
    if (d->num_levels < 1 || d->num_levels > DW_YOLO_MAX_LEVELS)
        return dw_fail(be, DW_ERR_INVALID_ARG, "%s: num_levels=%d outside [1, %d]", op, d->num_levels,
                       DW_YOLO_MAX_LEVELS);
    size_t A = 0;
    for (int l = 0; l < d->num_levels; l++) {
        if (d->h[l] <= 0 || d->w[l] <= 0)
            return dw_fail(be, DW_ERR_INVALID_ARG, "%s: level %d grid %dx%d", op, l, d->h[l], d->w[l]);
        if (!pos_finite(d->stride[l]) || !pos_finite(d->box_scale[l]) || !pos_finite(d->cls_scale[l]))
            return dw_fail(be, DW_ERR_INVALID_ARG, "%s: level %d stride and scales must be positive and finite", op,
                           l);
        A += (size_t)d->h[l] * d->w[l];
    }
    if (A > (size_t)INT32_MAX / 4)
        return dw_fail(be, DW_ERR_INVALID_ARG, "%s: %zu anchors is too many", op, A);
    *anchors = A;
    return DW_OK;
}

dw_status check_buf(dw_backend *be, const dw_buf *b, size_t expected, const char *op, const char *name) {
    if (!b) return dw_fail(be, DW_ERR_INVALID_ARG, "%s: %s is null", op, name);
    if (b->len != expected)
        return dw_fail(be, DW_ERR_SIZE_MISMATCH, "%s: %s mismatch: expected %zu, got %zu", op, name, expected, b->len);
    return DW_OK;
}

size_t ws_part(size_t bytes) { return al256(bytes); }

// segments over kSmallSeg candidates in one image: at most A / (kSmallSeg + 1)
size_t queue_cap(size_t A) { return A / (kSmallSeg + 1) + 1; }

size_t postprocess_workspace(size_t n, size_t A) {
    const size_t na = n * A;
    return ws_part(16 * na) + ws_part(4 * na) + ws_part(4 * na) + ws_part(na) + ws_part(2 * na) + ws_part(2 * na) +
           ws_part(16 * na) + ws_part(4 * n * (A + 1)) + ws_part(na) + ws_part(2 * na) + ws_part(2 * na) +
           ws_part(4 * n) + ws_part(4 * n) + 2 * ws_part(4 * n * queue_cap(A)) + ws_part(16);
}

PostWs carve_workspace(void *p, size_t n, size_t A) {
    const size_t na = n * A;
    unsigned char *w = (unsigned char *)p;
    auto take = [&](size_t bytes) {
        unsigned char *r = w;
        w += ws_part(bytes);
        return (void *)r;
    };
    PostWs ws;
    ws.box = (float4 *)take(16 * na);
    ws.cls = (uint32_t *)take(4 * na);
    ws.conf = (float *)take(4 * na);
    ws.flag = (uint8_t *)take(na);
    ws.ra = (uint16_t *)take(2 * na);
    ws.crank = (uint16_t *)take(2 * na);
    ws.cbox = (float4 *)take(16 * na);
    ws.seg = (uint32_t *)take(4 * n * (A + 1));
    ws.keep = (uint8_t *)take(na);
    ws.list0 = (uint16_t *)take(2 * na);
    ws.list1 = (uint16_t *)take(2 * na);
    ws.cnt = (uint32_t *)take(4 * n);
    ws.nseg = (uint32_t *)take(4 * n);
    ws.qhuge = (uint32_t *)take(4 * n * queue_cap(A));
    ws.qbig = (uint32_t *)take(4 * n * queue_cap(A));
    ws.qcnt = (uint32_t *)take(16);
    return ws;
}

}  // namespace

DW_API dw_status dw_prepare_yolo_detect(dw_backend *be, const dw_yolo_detect_desc *d, dw_buf **tables) {
    const char *op = "yolo_detect_prepare";
    if (!be) return DW_ERR_INVALID_ARG;
    if (!tables) return dw_fail(be, DW_ERR_INVALID_ARG, "%s: out is null", op);
    *tables = nullptr;
    size_t A;
    YT(check_detect_desc(be, d, op, &A));
    // Host libm expf: the function behind the reference's f32::exp.  One
    // multiply, subtract, add or divide per statement (no contraction).
    std::vector<float> t((size_t)d->num_levels * kTableLevel, 0.0f);
    for (int l = 0; l < d->num_levels; l++) {
        float *sg = t.data() + (size_t)l * kTableLevel;
        float *sm = sg + 256;
        const float sc = d->cls_scale[l], sb = d->box_scale[l];
        for (int q = -128; q < 128; q++) {
            const float x = (float)q * sc;  // dequantize_i8_to_f32_scalar (ops.rs:3453-3457)
            const float e = expf(-x);
            const float den = 1.0f + e;
            sg[q + 128] = 1.0f / den;  // sigmoid_f32_scalar (ops.rs:1865-1870)
        }
        for (int qm = -128; qm < 128; qm++) {
            const float xm = (float)qm * sb;
            for (int q = -128; q <= qm; q++) {
                const float x = (float)q * sb;
                const float dx = x - xm;
                sm[(qm + 128) * 256 + (q + 128)] = expf(dx);  // softmax_f32 term (ops.rs:1626-1628)
            }
        }
    }
    dw_buf *o = nullptr;
    YT(dw_alloc(be, t.size() * sizeof(float), &o));
    dw_status st = dw_upload(be, o, t.data(), t.size() * sizeof(float));
    if (st != DW_OK) {
        dw_free(be, o);
        return st;
    }
    *tables = o;
    return DW_OK;
}

DW_API dw_status dw_yolo_detect_i8(dw_backend *be, const dw_yolo_detect_desc *d, const dw_buf *tables,
                                   const dw_buf *const *box, const dw_buf *const *cls, dw_buf *out_f32) {
    const char *op = "yolo_detect_i8";
    if (!be) return DW_ERR_INVALID_ARG;
    size_t A;
    YT(check_detect_desc(be, d, op, &A));
    if (!box || !cls) return dw_fail(be, DW_ERR_INVALID_ARG, "%s: box/cls arrays are null", op);
    YT(check_buf(be, tables, (size_t)d->num_levels * kTableLevel * sizeof(float), op, "tables"));
    YT(check_buf(be, out_f32, (size_t)d->n * (4 + d->num_classes) * A * sizeof(float), op, "output"));
    DetectParams p{};
    int off = 0;
    bool vec = d->num_classes % 16 == 0;
    for (int l = 0; l < d->num_levels; l++) {
        const size_t px = (size_t)d->n * d->h[l] * d->w[l];
        YT(check_buf(be, box[l], px * 4 * kRegMax, op, "box"));
        YT(check_buf(be, cls[l], px * d->num_classes, op, "cls"));
        p.lv[l] = {(const int8_t *)box[l]->ptr, (const int8_t *)cls[l]->ptr, d->h[l], d->w[l], off, d->stride[l]};
        if (((uintptr_t)box[l]->ptr & 15) != 0)
            return dw_fail(be, DW_ERR_INVALID_ARG, "%s: box buffer %d is not 16-byte aligned", op, l);
        vec = vec && ((uintptr_t)cls[l]->ptr & 15) == 0;
        off += d->h[l] * d->w[l];
    }
    p.levels = d->num_levels;
    p.nc = d->num_classes;
    p.A = (int)A;
    p.tables = (const float *)tables->ptr;
    p.out = (float *)out_f32->ptr;
    cudaSetDevice(be->device);
    const dim3 grid((unsigned)((A + kDetThreads - 1) / kDetThreads), (unsigned)d->n);
    if (vec)
        k_yolo_detect<true><<<grid, kDetThreads, 0, be->stream>>>(p);
    else
        k_yolo_detect<false><<<grid, kDetThreads, 0, be->stream>>>(p);
    return dw_after_launch(be, "yolo_detect_i8");
}

DW_API size_t dw_postprocess_yolo_workspace(size_t n, size_t num_detections) {
    return postprocess_workspace(n, num_detections);
}

DW_API dw_status dw_postprocess_yolo(dw_backend *be, const dw_buf *raw, size_t n, size_t num_classes,
                                     size_t num_detections, uint32_t img_width, uint32_t img_height,
                                     float conf_threshold, float iou_threshold, int32_t flags, dw_buf *workspace,
                                     dw_buf *dets, dw_buf *counts) {
    const char *op = "postprocess_yolo";
    if (!be) return DW_ERR_INVALID_ARG;
    const size_t A = num_detections;
    if (n == 0 || n > 65535) return dw_fail(be, DW_ERR_INVALID_ARG, "%s: n=%zu outside [1, 65535]", op, n);
    if (num_classes > 65535) return dw_fail(be, DW_ERR_INVALID_ARG, "%s: num_classes=%zu > 65535", op, num_classes);
    if (A > (size_t)kMaxAnchors)
        return dw_fail(be, DW_ERR_UNSUPPORTED, "%s: num_detections=%zu > %d (the per-image sort is on-chip)", op, A,
                       kMaxAnchors);
    if (flags & ~(DW_YOLO_ANCHOR_ROWS | DW_YOLO_NMS_AGNOSTIC | DW_YOLO_NO_NMS))
        return dw_fail(be, DW_ERR_INVALID_ARG, "%s: unknown flags 0x%x", op, (unsigned)flags);
    YT(check_buf(be, counts, n * sizeof(int32_t), op, "counts"));
    cudaSetDevice(be->device);
    // no anchors: no detections (decode_detections_v8 returns an empty list)
    if (A == 0) return dw_cuda_check(be, cudaMemsetAsync(counts->ptr, 0, n * sizeof(int32_t), be->stream), op);
    YT(check_buf(be, raw, n * (4 + num_classes) * A * sizeof(float), op, "raw output"));
    YT(check_buf(be, dets, n * A * sizeof(dw_detection), op, "detections"));
    const size_t ws = postprocess_workspace(n, A);
    void *wp = nullptr;
    if (workspace) {
        if (workspace->len < ws)
            return dw_fail(be, DW_ERR_SIZE_MISMATCH, "%s: workspace of %zu bytes, needs %zu", op, workspace->len, ws);
        wp = workspace->ptr;
    } else {
        YT(dw_scratch(be, ws, &wp));
    }
    const PostWs w = carve_workspace(wp, n, A);
    const bool nms = (flags & DW_YOLO_NO_NMS) == 0, agnostic = (flags & DW_YOLO_NMS_AGNOSTIC) != 0;
    DecodeParams dp{};
    dp.raw = (const float *)raw->ptr;
    dp.nc = (int)num_classes;
    dp.A = (int)A;
    dp.sx = (float)img_width / kModelSize;  // postprocess.rs:99-100
    dp.sy = (float)img_height / kModelSize;
    dp.iw = (float)img_width;
    dp.ih = (float)img_height;
    dp.thr = conf_threshold;
    dp.w = w;
    const dim3 dgrid((unsigned)((A + kDecodeThreads - 1) / kDecodeThreads), (unsigned)n);
    if (flags & DW_YOLO_ANCHOR_ROWS)
        k_yolo_decode<true><<<dgrid, kDecodeThreads, 0, be->stream>>>(dp);
    else
        k_yolo_decode<false><<<dgrid, kDecodeThreads, 0, be->stream>>>(dp);
    YT(dw_after_launch(be, "yolo_decode"));

    const int cap = (int)((A + kRankThreads - 1) / kRankThreads * kRankThreads);
    RankParams rp{};
    rp.A = (int)A;
    rp.cap = cap;
    rp.sort_conf = nms;
    rp.nms = nms;
    rp.group = nms && !agnostic;
    rp.w = w;
    const size_t rank_smem = 12 * (size_t)cap + 2 * 256 * 32;
    YT(dw_cuda_check(be, cudaFuncSetAttribute(k_yolo_rank, cudaFuncAttributeMaxDynamicSharedMemorySize, (int)rank_smem),
                     "postprocess_yolo: shared memory"));
    YT(dw_cuda_check(be, cudaMemsetAsync(w.qcnt, 0, 16, be->stream), "postprocess_yolo: queue counters"));
    k_yolo_rank<<<(unsigned)n, kRankThreads, rank_smem, be->stream>>>(rp);
    YT(dw_after_launch(be, "yolo_rank"));

    if (nms) {
        SegNmsParams sp{};
        sp.A = (int)A;
        sp.cap = (int)std::min<size_t>(A, kBoxCap);
        sp.gx = img_width > 0 ? (float)kGrid / (float)img_width : 0.0f;
        sp.gy = img_height > 0 ? (float)kGrid / (float)img_height : 0.0f;
        const float tp = std::nextafter(iou_threshold, INFINITY);
        sp.mid = ((double)iou_threshold + (double)tp) * 0.5;  // exact: two adjacent floats
        uint32_t tb;
        memcpy(&tb, &tp, 4);
        sp.tie_up = (tb & 1u) == 0;
        sp.zero_gt = 0.0f > iou_threshold;
        sp.w = w;
        const size_t segs = agnostic ? 1 : std::max<size_t>(1, std::min(num_classes, A));
        const size_t seg_smem = 25 * (size_t)sp.cap;
        YT(dw_cuda_check(be, cudaFuncSetAttribute(k_yolo_nms_segment, cudaFuncAttributeMaxDynamicSharedMemorySize,
                                                  (int)seg_smem),
                         "postprocess_yolo: shared memory"));
        k_yolo_nms_small<<<dim3((unsigned)((segs + kSmallWarps - 1) / kSmallWarps), (unsigned)n), kSmallWarps * 32, 0,
                           be->stream>>>(sp);
        YT(dw_after_launch(be, "yolo_nms_small"));
        const size_t workers = std::min<size_t>(2 * (size_t)be->sm_count, n * queue_cap(A));
        k_yolo_nms_segment<<<(unsigned)workers, kSegThreads, seg_smem, be->stream>>>(sp);
        YT(dw_after_launch(be, "yolo_nms_segment"));
    }

    OrderParams op_{};
    op_.A = (int)A;
    op_.cap = cap;
    op_.all_kept = !nms;
    op_.w = w;
    op_.dets = (uint32_t *)dets->ptr;
    op_.counts = (int32_t *)counts->ptr;
    const size_t order_smem = 5 * (size_t)cap;
    YT(dw_cuda_check(be, cudaFuncSetAttribute(k_yolo_order, cudaFuncAttributeMaxDynamicSharedMemorySize,
                                              (int)order_smem),
                     "postprocess_yolo: shared memory"));
    k_yolo_order<<<(unsigned)n, kRankThreads, order_smem, be->stream>>>(op_);
    return dw_after_launch(be, "yolo_order");
}
