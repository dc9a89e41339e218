// k_decode.cu -- on-device image preparation and one-to-one YOLO decoding.
//
// pixel_table_kernel applies the image APIs' byte table (src/unoq_dsp/modern.py:10-18,
// vision.py:20-29) to uploaded uint8 pixels. yolo_topk_kernel performs the decode of
// src/unoq_dsp/modern.py:75-103 for one image per CTA: best-class score per anchor, the first
// stage `argsort(-best, stable)[:candidates]`, the second stage `argsort(-flat, stable)[:k]` over
// the candidates' (anchor, class) scores, and the pixel boxes `(grid -/+ distance) * stride`.
//
// All comparisons are on integer order codes: the host ranks the float32 scores its own decoder
// would compute (at most 4 x 256 distinct values), so equal scores tie exactly as in the stable
// argsort and no device transcendental is involved. The boxes use the same float32 operations as
// the host decoder, each correctly rounded (no contraction), so they are bit-identical.
#include "common.cuh"
#include "decode.cuh"

namespace uq {
namespace {

constexpr int kT = 256;

__global__ void __launch_bounds__(kT) pixel_table_kernel(const uint8_t *__restrict__ px, int8_t *__restrict__ x,
                                                          size_t bytes, const int8_t *__restrict__ table,
                                                          uint32_t channels) {
    __shared__ uint8_t tab[kMaxTableChannels * 256];  // [channel][pixel]
    for (uint32_t i = threadIdx.x; i < 256 * channels; i += blockDim.x) {
        const uint32_t p = i / channels, c = i - p * channels;
        tab[c * 256 + p] = (uint8_t)table[i];
    }
    __syncthreads();
    const size_t step = (size_t)gridDim.x * blockDim.x;
    const bool vec = ((reinterpret_cast<uintptr_t>(px) | reinterpret_cast<uintptr_t>(x)) & 15) == 0;
    const size_t units = vec ? bytes / 16 : 0;
    for (size_t u = blockIdx.x * (size_t)blockDim.x + threadIdx.x; u < units; u += step) {
        const uint4 v = __ldg(reinterpret_cast<const uint4 *>(px) + u);
        uint32_t c = (uint32_t)((u * 16) % channels);
        const uint32_t in[4] = {v.x, v.y, v.z, v.w};
        uint32_t out[4];
#pragma unroll
        for (int w = 0; w < 4; w++) {
            uint32_t o = 0;
#pragma unroll
            for (int b = 0; b < 4; b++) {
                o |= (uint32_t)tab[c * 256 + ((in[w] >> (8 * b)) & 255u)] << (8 * b);
                c = c + 1 == channels ? 0 : c + 1;
            }
            out[w] = o;
        }
        reinterpret_cast<uint4 *>(x)[u] = make_uint4(out[0], out[1], out[2], out[3]);
    }
    for (size_t i = units * 16 + blockIdx.x * (size_t)blockDim.x + threadIdx.x; i < bytes; i += step)
        x[i] = (int8_t)tab[(i % channels) * 256 + px[i]];
}

// ---- YOLO top-k -----------------------------------------------------------------------------

constexpr int kDT = 512;                    // threads per image = sort width
static_assert(kDT == (int)kMaxDetections, "one sort element per thread");
constexpr uint32_t kIdxBits = 21;           // key = code << 21 | (mask - index): larger key = better
constexpr uint32_t kIdxMask = (1u << kIdxBits) - 1;

struct TopkSmem {
    uint32_t hist[kRankCodes];
    uint32_t keys[kMaxDetections];
    uint32_t sel[kMaxDetections];           // first-stage anchors, best first
    uint32_t sbase[kMaxDetections];         // byte offset of each candidate's logits in the image
    uint8_t slev[kMaxDetections];
    uint16_t rank[UG_YOLO_MAX_LEVELS][256];
    uint32_t warp_sum[kDT / 32];
    uint32_t base[UG_YOLO_MAX_LEVELS + 1];  // first anchor of each level
    uint32_t score_off[UG_YOLO_MAX_LEVELS];
    uint32_t counter, thr, gt, need;
};

__device__ __forceinline__ uint32_t level_of(const TopkSmem &S, uint32_t levels, uint32_t a) {
    uint32_t l = 0;
    while (l + 1 < levels && a >= S.base[l + 1]) l++;
    return l;
}

// Exclusive prefix sum of `v` over the block's threads (thread order).
__device__ uint32_t block_exclusive_scan(uint32_t v, uint32_t *warp_sum) {
    const uint32_t lane = threadIdx.x & 31, warp = threadIdx.x >> 5;
    uint32_t inc = v;
#pragma unroll
    for (int o = 1; o < 32; o <<= 1) {
        const uint32_t t = __shfl_up_sync(0xffffffffu, inc, o);
        if (lane >= (uint32_t)o) inc += t;
    }
    if (lane == 31) warp_sum[warp] = inc;
    __syncthreads();
    if (warp == 0) {
        const uint32_t w = lane < kDT / 32 ? warp_sum[lane] : 0;
        uint32_t wi = w;
#pragma unroll
        for (int o = 1; o < 32; o <<= 1) {
            const uint32_t t = __shfl_up_sync(0xffffffffu, wi, o);
            if (lane >= (uint32_t)o) wi += t;
        }
        if (lane < kDT / 32) warp_sum[lane] = wi - w;
    }
    __syncthreads();
    const uint32_t r = warp_sum[warp] + inc - v;
    __syncthreads();
    return r;
}

// keys[0..kDT) sorted descending (bitonic network, one element per thread).
__device__ void sort_desc(uint32_t *keys) {
    const uint32_t i = threadIdx.x;
    for (uint32_t size = 2; size <= (uint32_t)kDT; size <<= 1)
        for (uint32_t stride = size >> 1; stride > 0; stride >>= 1) {
            const uint32_t p = i ^ stride;
            if (p > i) {
                const uint32_t a = keys[i], b = keys[p];
                if ((i & size) == 0 ? a < b : a > b) {
                    keys[i] = b;
                    keys[p] = a;
                }
            }
            __syncthreads();
        }
}

// The K items of [0, n) with the largest (code, -index), as sorted keys in S.keys[0..K): a code
// histogram finds the threshold code thr, then every item above thr and the lowest-index items at
// thr are collected and sorted. Items with a code below `floor` are known to lie outside the top K
// and are not counted. Requires K >= 1 and at least K items with code >= floor.
template <class CodeFn>
__device__ void select_top(TopkSmem &S, uint32_t n, uint32_t K, uint32_t floor, CodeFn code_of) {
    const uint32_t tid = threadIdx.x, lane = tid & 31;
    for (uint32_t i = tid; i < kRankCodes; i += kDT) S.hist[i] = 0;
    if (tid == 0) {
        S.counter = 0;
        S.thr = floor;
        S.gt = 0;
        S.need = 0;
    }
    __syncthreads();
    const uint32_t n_round = (n + kDT - 1) / kDT * kDT;
    for (uint32_t i = tid; i < n_round; i += kDT) {
        uint32_t r = 0;
        bool on = false;
        if (i < n) {
            r = code_of(i);
            on = r >= floor;
        }
        const unsigned act = __ballot_sync(0xffffffffu, on);
        if (on) {
            const unsigned peers = __match_any_sync(act, r);
            if (lane == (uint32_t)(__ffs(peers) - 1)) atomicAdd(&S.hist[r], (uint32_t)__popc(peers));
        }
    }
    __syncthreads();
    if (tid < 32) {
        // lane l holds codes 1023 - 32 l - t (t = 0..31): lane 0 the highest
        uint32_t s = 0;
        for (int t = 0; t < 32; t++) s += S.hist[kRankCodes - 1 - 32 * lane - t];
        uint32_t inc = s;
#pragma unroll
        for (int o = 1; o < 32; o <<= 1) {
            const uint32_t v = __shfl_up_sync(0xffffffffu, inc, o);
            if (lane >= (uint32_t)o) inc += v;
        }
        const unsigned hit = __ballot_sync(0xffffffffu, inc >= K);
        if (hit && lane == (uint32_t)(__ffs(hit) - 1)) {
            uint32_t run = inc - s;
            for (int t = 0; t < 32; t++) {
                const uint32_t code = kRankCodes - 1 - 32 * lane - t, h = S.hist[code];
                if (run + h >= K) {
                    S.thr = code;
                    S.gt = run;
                    S.need = K - run;
                    break;
                }
                run += h;
            }
        }
    }
    __syncthreads();
    const uint32_t thr = S.thr, gt = S.gt, need = S.need;
    const uint32_t chunk = (n + kDT - 1) / kDT;
    const uint32_t lo = min(n, tid * chunk), hi = min(n, lo + chunk);
    uint32_t eq = 0;
    for (uint32_t i = lo; i < hi; i++) {
        const uint32_t r = code_of(i);
        if (r > thr) {
            const uint32_t slot = atomicAdd(&S.counter, 1u);
            if (slot < K) S.keys[slot] = r << kIdxBits | (kIdxMask - i);
        } else if (r == thr) {
            eq++;
        }
    }
    uint32_t before = block_exclusive_scan(eq, S.warp_sum);
    for (uint32_t i = lo; i < hi && before < need; i++) {
        if (code_of(i) == thr) S.keys[gt + before++] = thr << kIdxBits | (kIdxMask - i);
    }
    __syncthreads();
    for (uint32_t i = K + tid; i < (uint32_t)kDT; i += kDT) S.keys[i] = 0;
    __syncthreads();
    sort_desc(S.keys);
}

__device__ __forceinline__ uint32_t best4(const uint16_t *rk, uint32_t w, uint32_t best) {
#pragma unroll
    for (int b = 0; b < 4; b++) best = max(best, (uint32_t)rk[((w >> (8 * b)) & 255u) ^ 128u]);
    return best;
}

__global__ void __launch_bounds__(kDT) yolo_topk_kernel(const int8_t *__restrict__ y, size_t image_bytes,
                                                         const UgYoloDecode *__restrict__ cfg, YoloShape shape,
                                                         uint32_t k, bool vec, UgDetectionRecord *__restrict__ rec) {
    __shared__ TopkSmem S;
    extern __shared__ uint16_t amax[];  // best-class code of every anchor
    const uint32_t tid = threadIdx.x;
    const int8_t *img = y + (size_t)blockIdx.x * image_bytes;
    const uint32_t L = shape.levels, C = shape.classes, A = shape.anchors;
    for (uint32_t i = tid; i < L * 256; i += kDT) S.rank[i >> 8][i & 255] = cfg->level[i >> 8].rank[i & 255];
    if (tid == 0) {
        uint32_t b = 0;
        for (uint32_t l = 0; l < L; l++) {
            S.base[l] = b;
            S.score_off[l] = cfg->level[l].score_offset;
            b += cfg->level[l].height * cfg->level[l].width;
        }
        S.base[L] = b;
    }
    __syncthreads();

    // best-class code per anchor (scores.max(1) in order-code form)
    for (uint32_t a = tid; a < A; a += kDT) {
        const uint32_t l = level_of(S, L, a);
        const int8_t *p = img + S.score_off[l] + (size_t)(a - S.base[l]) * C;
        const uint16_t *rk = S.rank[l];
        uint32_t best = 0;
        if (vec) {
            for (uint32_t c = 0; c < C; c += 16) {
                const uint4 v = __ldg(reinterpret_cast<const uint4 *>(p + c));
                best = best4(rk, v.w, best4(rk, v.z, best4(rk, v.y, best4(rk, v.x, best))));
            }
        } else {
            for (uint32_t c = 0; c < C; c++) best = max(best, (uint32_t)rk[(uint8_t)p[c] ^ 128u]);
        }
        amax[a] = (uint16_t)best;
    }
    __syncthreads();

    // first stage: the best `candidates` anchors, ties by lower anchor index
    const uint32_t K1 = min(shape.candidates, A);
    select_top(S, A, K1, 0, [&](uint32_t i) { return (uint32_t)amax[i]; });
    for (uint32_t i = tid; i < K1; i += kDT) {
        const uint32_t a = kIdxMask - (S.keys[i] & kIdxMask), l = level_of(S, L, a);
        S.sel[i] = a;
        S.slev[i] = (uint8_t)l;
        S.sbase[i] = S.score_off[l] + (a - S.base[l]) * C;
    }
    __syncthreads();

    // second stage: the best k pairs (candidate i, class c), flat index j = i * C + c. When k <= K1,
    // the k-th candidate's best code bounds the k-th pair's code from below.
    const uint32_t n2 = K1 * C, K2 = min(k, n2);
    const uint32_t floor = K2 <= K1 ? (uint32_t)amax[S.sel[K2 - 1]] : 0;
    select_top(S, n2, K2, floor, [&](uint32_t j) {
        const uint32_t i = j / C;
        return (uint32_t)S.rank[S.slev[i]][(uint8_t)img[S.sbase[i] + (j - i * C)] ^ 128u];
    });

    for (uint32_t r = tid; r < k; r += kDT) {
        UgDetectionRecord out;
        if (r < K2) {
            const uint32_t j = kIdxMask - (S.keys[r] & kIdxMask), i = j / C, c = j - i * C;
            const uint32_t a = S.sel[i], l = S.slev[i], cell = a - S.base[l];
            const UgYoloLevel &lv = cfg->level[l];
            const int8_t *d = img + lv.box_offset + (size_t)cell * 4;
            const uint32_t w = lv.width;
            const float gx = (float)(cell % w) + 0.5f, gy = (float)(cell / w) + 0.5f, st = lv.stride;
            out.anchor = a;
            out.class_id = c;
            out.score = lv.score[(uint8_t)img[S.sbase[i] + c] ^ 128u];
            out.box[0] = __fmul_rn(__fsub_rn(gx, lv.distance[(uint8_t)d[0] ^ 128u]), st);
            out.box[1] = __fmul_rn(__fsub_rn(gy, lv.distance[(uint8_t)d[1] ^ 128u]), st);
            out.box[2] = __fmul_rn(__fadd_rn(gx, lv.distance[(uint8_t)d[2] ^ 128u]), st);
            out.box[3] = __fmul_rn(__fadd_rn(gy, lv.distance[(uint8_t)d[3] ^ 128u]), st);
        } else {
            out.anchor = 0xffffffffu;
            out.class_id = 0;
            out.score = 0.f;
            out.box[0] = out.box[1] = out.box[2] = out.box[3] = 0.f;
        }
        out.reserved = 0;
        rec[(size_t)blockIdx.x * k + r] = out;
    }
}

}  // namespace

void launch_pixel_table(const uint8_t *pixels, int8_t *x, size_t bytes, const int8_t *table, uint32_t channels,
                        cudaStream_t s) {
    pixel_table_kernel<<<grid_for(bytes / 16 + 1, kT), kT, 0, s>>>(pixels, x, bytes, table, channels);
}

void launch_yolo_topk(const int8_t *y, size_t image_bytes, uint32_t images, const UgYoloDecode *cfg,
                      const YoloShape &shape, uint32_t k, UgDetectionRecord *records, cudaStream_t s) {
    const int dyn = (int)(shape.anchors * sizeof(uint16_t));
    cudaFuncSetAttribute(yolo_topk_kernel, cudaFuncAttributeMaxDynamicSharedMemorySize,
                         (int)(kMaxAnchors * sizeof(uint16_t)));
    const bool vec = shape.vec && (reinterpret_cast<uintptr_t>(y) & 15) == 0 && image_bytes % 16 == 0;
    yolo_topk_kernel<<<images, kDT, dyn, s>>>(y, image_bytes, cfg, shape, k, vec, records);
}

}  // namespace uq
