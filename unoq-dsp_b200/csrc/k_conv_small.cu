// k_conv_small.cu -- direct dp4a convolution for 3x3 convs with few input channels.
//
// Plan code 14 (runtime/qnn.c:1101-1227) for the layers where an implicit GEMM's reduction is tiny:
// the 3-channel RGB stems (K = 27) and 8 / 16-channel 3x3 layers (K = 72 / 144) with at most 32
// output channels. A tcgen05 tile would be more than 95 % idle there and the im2col assembly
// would dominate; on the CUDA cores every tap is one aligned word:
//  * the input rows of an output tile are staged in shared memory with each pixel's channels
//    padded to IC4 whole words (zero weight on the padding bytes, zero point outside the image);
//  * a thread owns 4 adjacent output pixels x OCT output channels; its OCT * 9 * IC4 = 72 weight
//    words sit in registers and each feeds 4 dp4a (one per pixel);
//  * the epilogue is the exact requantisation of requant.cuh, the optional post table, and an
//    OCT-byte store.
// The reference multiplies u8 columns (x ^ 0x80) by s8 weights with K padding at xzp + 128; the
// host folds 128 * sum(w) + xzp * sum(w_kpad) into each channel's constant, so the s8 sums here
// give identical results.
#include <algorithm>
#include <cstdlib>
#include <cstring>
#include <vector>

#include "conv_small.cuh"
#include "plan.hpp"
#include "requant.cuh"

namespace uq {

namespace {

constexpr int kThreads = 256;
constexpr int kPix = 4;  // adjacent output pixels per thread (each weight word feeds kPix dp4a)

struct SmallParams {
    const int8_t *x;
    int8_t *y;
    const uint32_t *w;     // [oc / OCT][OCT][9][IC4] weight words
    const EpiChan *epi;    // [oc]
    const uint8_t *post;   // 256 bytes or null
    int n, ih, iw, ic, oh, ow, oc, pt, pl;
    int lo, hi, xzp;
    int groups;            // oc / OCT
    int tw, th, tiles_x, tiles_y;
    int br, bc;            // band rows / columns (pixels)
};

template <int EPI>
__device__ __forceinline__ int32_t requant(int32_t acc, const EpiChan &e, int lo, int hi) {
    int32_t v;
    if (EPI == 2) {
        const int32_t a = (int32_t)(((uint32_t)acc << e.ls) + (uint32_t)e.bs);
        long long p = (long long)a * e.m + e.k;
        p -= (long long)(acc <= e.cut) << 31;
        v = (int32_t)(p >> e.sh) + e.zadd;
    } else {
        long long p = (long long)acc * e.m + e.k;
        if (EPI == 1) p -= (long long)(acc <= e.cut) << 31;
        v = ((int32_t)(p >> 32)) >> e.sh;
    }
    return v < lo ? lo : (v > hi ? hi : v);
}

template <int IC4, int OCT, int S, int EPI>
__global__ void __launch_bounds__(kThreads) conv_small_kernel(const SmallParams p) {
    extern __shared__ __align__(16) uint8_t smem[];
    uint8_t *sLut = smem;                                              // 256 bytes
    EpiChan *sEpi = reinterpret_cast<EpiChan *>(smem + 256);           // [oc]
    uint32_t *sBand = reinterpret_cast<uint32_t *>(smem + 256 + (size_t)p.oc * sizeof(EpiChan));  // [br][bc][IC4]

    int tile = blockIdx.x;
    const int tx = tile % p.tiles_x;
    tile /= p.tiles_x;
    const int ty = tile % p.tiles_y;
    const int n = tile / p.tiles_y;
    const int iy0 = ty * p.th * S - p.pt, ix0 = tx * p.tw * S - p.pl;

    if (p.post)
        for (int i = threadIdx.x; i < 256; i += kThreads) sLut[i] = p.post[i];
    for (int i = threadIdx.x; i < p.oc; i += kThreads) sEpi[i] = p.epi[i];
    const uint32_t fillw = 0x01010101u * (uint8_t)p.xzp;
    if (IC4 == 1 && p.ic == 3) {
        // RGB: image-aligned groups of 4 pixels are 3 aligned words; unpack to one word per pixel
        const int g0 = (ix0 >= 0 ? ix0 : ix0 - 3) / 4;  // floor(ix0 / 4)
        const int groups = (ix0 + p.bc - 1 - g0 * 4) / 4 + 1;
        // unit = (band row, 4-pixel group), row fastest: the lanes' word stores then fall 1 band row
        // apart (an odd word count when bc is odd) instead of 4 words apart
        for (int u = threadIdx.x; u < p.br * groups; u += kThreads) {
            const int gi = u / p.br, r = u - gi * p.br, gx = g0 + gi;
            const int iy = iy0 + r, x4 = gx * 4;
            uint32_t v[4] = {fillw, fillw, fillw, fillw};
            if (iy >= 0 && iy < p.ih) {
                const int8_t *row = p.x + ((size_t)n * p.ih + iy) * p.iw * 3;
                if (x4 >= 0 && x4 + 4 <= p.iw && (p.iw & 3) == 0) {  // 4-byte aligned words
                    const uint32_t *src = reinterpret_cast<const uint32_t *>(row + x4 * 3);
                    const uint32_t a = __ldg(src), b = __ldg(src + 1), c = __ldg(src + 2);
                    v[0] = a & 0x00FFFFFFu;
                    v[1] = __byte_perm(a, b, 0x0543) & 0x00FFFFFFu;
                    v[2] = __byte_perm(b, c, 0x0432) & 0x00FFFFFFu;
                    v[3] = c >> 8;
                } else {
                    for (int k = 0; k < 4; k++) {
                        const int ix = x4 + k;
                        if (ix >= 0 && ix < p.iw)
                            v[k] = (uint32_t)(uint8_t)__ldg(row + ix * 3) | (uint32_t)(uint8_t)__ldg(row + ix * 3 + 1) << 8 |
                                   (uint32_t)(uint8_t)__ldg(row + ix * 3 + 2) << 16;
                    }
                }
            }
            for (int k = 0; k < 4; k++) {
                const int c = x4 + k - ix0;
                if (c >= 0 && c < p.bc) sBand[r * p.bc + c] = v[k];
            }
        }
    } else
    for (int u = threadIdx.x; u < p.br * p.bc; u += kThreads) {
        const int r = u / p.bc, c = u - r * p.bc;
        const int iy = iy0 + r, ix = ix0 + c;
        uint32_t v[IC4];
#pragma unroll
        for (int q = 0; q < IC4; q++) v[q] = fillw;
        if (iy >= 0 && iy < p.ih && ix >= 0 && ix < p.iw) {
            const int8_t *src = p.x + (((size_t)n * p.ih + iy) * p.iw + ix) * p.ic;
            if (IC4 == 1 && p.ic == 4) {
                v[0] = __ldg(reinterpret_cast<const uint32_t *>(src));
            } else if (IC4 == 1) {  // 3 (or fewer) channels: byte loads, pad byte 0
                uint32_t w = 0;
                for (int k = 0; k < p.ic; k++) w |= (uint32_t)(uint8_t)__ldg(src + k) << (8 * k);
                v[0] = w;
            } else if (p.ic == IC4 * 4) {
#pragma unroll
                for (int q = 0; q < IC4; q++) v[q] = __ldg(reinterpret_cast<const uint32_t *>(src) + q);
            } else {
#pragma unroll
                for (int q = 0; q < IC4; q++) {
                    uint32_t w = 0;
                    for (int k = 0; k < 4 && q * 4 + k < p.ic; k++) w |= (uint32_t)(uint8_t)__ldg(src + q * 4 + k) << (8 * k);
                    v[q] = w;
                }
            }
        }
#pragma unroll
        for (int q = 0; q < IC4; q++) sBand[u * IC4 + q] = v[q];
    }
    // this thread: output pixels px0 + s * j (j < 4) of tile row py, channels og * OCT .. + OCT - 1;
    // s = tw / 4, so the lanes of a warp read neighbouring band pixels for every tap
    const int og = threadIdx.x % p.groups, quad = threadIdx.x / p.groups;
    const int quads_x = p.tw / kPix;
    const int py = quad / quads_x, px0 = quad - py * quads_x;
    uint32_t w[OCT][9][IC4];
    const uint4 *wsrc = reinterpret_cast<const uint4 *>(p.w + (size_t)og * OCT * 9 * IC4);
#pragma unroll
    for (int i = 0; i < OCT * 9 * IC4 / 4; i++) {
        const uint4 v = __ldg(wsrc + i);
        uint32_t *flat = &w[0][0][0];
        flat[4 * i] = v.x, flat[4 * i + 1] = v.y, flat[4 * i + 2] = v.z, flat[4 * i + 3] = v.w;
    }
    __syncthreads();
    const int oy = ty * p.th + py, ox0 = tx * p.tw + px0;
    if (py >= p.th || oy >= p.oh || ox0 >= p.ow) return;
    const int pstep = quads_x;  // columns between a thread's pixels
    int acc[kPix][OCT];
#pragma unroll
    for (int j = 0; j < kPix; j++)
#pragma unroll
        for (int o = 0; o < OCT; o++) acc[j][o] = 0;
#pragma unroll
    for (int ky = 0; ky < 3; ky++)
#pragma unroll
        for (int kx = 0; kx < 3; kx++)
#pragma unroll
            for (int q = 0; q < IC4; q++) {
                const uint32_t *b = sBand + ((py * S + ky) * p.bc + px0 * S + kx) * IC4 + q;
                int xv[kPix];
#pragma unroll
                for (int j = 0; j < kPix; j++) xv[j] = (int)b[j * pstep * S * IC4];
#pragma unroll
                for (int o = 0; o < OCT; o++)
#pragma unroll
                    for (int j = 0; j < kPix; j++) acc[j][o] = __dp4a(xv[j], (int)w[o][ky * 3 + kx][q], acc[j][o]);
            }
    const uint8_t *lut = p.post ? sLut : nullptr;
    uint32_t packed[kPix][(OCT + 3) / 4] = {};
#pragma unroll
    for (int o = 0; o < OCT; o++) {
        const EpiChan e = sEpi[og * OCT + o];
#pragma unroll
        for (int j = 0; j < kPix; j++) {
            int32_t v = requant<EPI>(acc[j][o], e, p.lo, p.hi);
            if (lut) v = (int8_t)lut[v + 128];
            packed[j][o / 4] |= (uint32_t)(uint8_t)v << (8 * (o % 4));
        }
    }
#pragma unroll
    for (int j = 0; j < kPix; j++) {
        if (ox0 + j * pstep >= p.ow) break;
        int8_t *dst = p.y + (((size_t)n * p.oh + oy) * p.ow + ox0 + j * pstep) * p.oc + og * OCT;
        if (OCT == 8) *reinterpret_cast<uint2 *>(dst) = make_uint2(packed[j][0], packed[j][1]);
        else if (OCT == 4) *reinterpret_cast<uint32_t *>(dst) = packed[j][0];
        else *reinterpret_cast<uint16_t *>(dst) = (uint16_t)packed[j][0];
    }
}

template <int IC4, int OCT, int S>
void launch_s(const SmallParams &p, int epi, dim3 grid, size_t smem, cudaStream_t s) {
    if (epi == 0) conv_small_kernel<IC4, OCT, S, 0><<<grid, kThreads, smem, s>>>(p);
    else if (epi == 1) conv_small_kernel<IC4, OCT, S, 1><<<grid, kThreads, smem, s>>>(p);
    else conv_small_kernel<IC4, OCT, S, 2><<<grid, kThreads, smem, s>>>(p);
}

}  // namespace

struct ConvSmall {
    SmallParams p{};
    int ic4 = 1, oct = 8, s = 1, epi = 0;
    size_t smem = 0;
};

int conv_small_prepare(const int8_t *w_packed, const int32_t *q, const uint8_t *post_dev, const ConvGeom &g,
                       const std::function<void *(size_t)> &alloc, ConvSmall **out) {
    *out = nullptr;
    const char *env = std::getenv("UNOQ_CONV_SMALL");
    if (env && env[0] == '0') return 0;
    if (g.kh != 3 || g.kw != 3 || g.dh != 1 || g.dw != 1 || g.sh != g.sw || (g.sh != 1 && g.sh != 2)) return 0;
    const int ic4 = g.ic <= 4 ? 1 : g.ic <= 8 ? 2 : g.ic <= 16 ? 4 : 0;
    if (!ic4) return 0;
    // output channels per thread: 8 / ic4 (72 weight words in registers); 4 for 1-word pixels when
    // the layer has at most 16 output channels (more threads per tile, measured faster there)
    const int oct = (ic4 == 1 && g.oc <= 16) ? 4 : 8 / ic4, oc = g.oc;
    if (oc % oct != 0) return 0;
    const int groups = oc / oct;
    if (groups > 32 || (groups & (groups - 1)) != 0) return 0;   // power of two, divides the block
    // wider 8 / 16-channel layers measured faster on the tensor cores (dp4a count grows with oc)
    if (ic4 == 4 && oc > 16) return 0;
    if (ic4 == 2 && oc > 32) return 0;
    const int K = 9 * g.ic, kp = q[18];
    const int32_t *cbias = q + kHead, *mult = cbias + oc, *shift = mult + oc;
    const int xzp = q[12], yzp = q[13];
    auto wref = [&](int j, int t) -> int { return w_packed[(j / 4) * kp * 4 + (t / 8) * 32 + (j % 4) * 8 + t % 8]; };
    // weight words [og][o][tap][q]: byte k of word q = w[oc][tap * ic + 4 q + k] (0 past ic)
    std::vector<uint32_t> wt((size_t)oc * 9 * ic4, 0);
    std::vector<EpiChan> epi(oc);
    bool fast = true;
    for (int j = 0; j < oc; j++) {
        long long sum_all = 0, sum_pad = 0;
        for (int t = 0; t < kp; t++) {
            const int v = wref(j, t);
            sum_all += v;
            if (t >= K) sum_pad += v;
        }
        for (int tap = 0; tap < 9; tap++)
            for (int c = 0; c < g.ic; c++)
                wt[((size_t)j * 9 + tap) * ic4 + c / 4] |= (uint32_t)(uint8_t)wref(j, tap * g.ic + c) << (8 * (c % 4));
        epi[j] = make_epilogue((long long)cbias[j] + 128 * sum_all + (long long)xzp * sum_pad, mult[j], shift[j], yzp);
        fast &= epi_fast(epi[j]);
    }
    const int epi_mode = !fast ? 2 : (q[14] >= yzp ? 0 : 1);
    if (epi_mode != 2)
        for (auto &e : epi) e.sh = e.sh >= 32 ? e.sh - 32 : 0;
    ConvSmall *c = new ConvSmall();
    SmallParams &p = c->p;
    const int pixels = kThreads / groups * kPix;
    p.tw = std::min(pixels, 32);
    p.th = pixels / p.tw;
    p.tiles_x = (g.ow + p.tw - 1) / p.tw;
    p.tiles_y = (g.oh + p.th - 1) / p.th;
    p.br = (p.th - 1) * g.sh + 3;
    p.bc = (p.tw - 1) * g.sw + 3;
    if ((p.bc & 1) == 0) p.bc++;  // odd row length: a column of band words spans distinct banks
    p.groups = groups;
    c->ic4 = ic4, c->oct = oct, c->s = g.sh, c->epi = epi_mode;
    c->smem = 256 + (size_t)oc * sizeof(EpiChan) + (size_t)p.br * p.bc * ic4 * 4;
    void *dw = alloc(wt.size() * 4), *de = alloc(epi.size() * sizeof(EpiChan));
    if (!dw || !de || cudaMemcpy(dw, wt.data(), wt.size() * 4, cudaMemcpyHostToDevice) != cudaSuccess ||
        cudaMemcpy(de, epi.data(), epi.size() * sizeof(EpiChan), cudaMemcpyHostToDevice) != cudaSuccess) {
        delete c;
        return 2001;
    }
    p.w = static_cast<const uint32_t *>(dw);
    p.epi = static_cast<const EpiChan *>(de);
    p.post = post_dev;
    p.ih = g.ih, p.iw = g.iw, p.ic = g.ic, p.oh = g.oh, p.ow = g.ow, p.oc = oc, p.pt = g.pt, p.pl = g.pl;
    p.lo = q[14], p.hi = q[15], p.xzp = xzp;
    *out = c;
    return 0;
}

int conv_small_launch(const ConvSmall &c, const int8_t *x, int8_t *y, const ConvGeom &g, cudaStream_t s) {
    SmallParams p = c.p;
    p.x = x;
    p.y = y;
    p.n = g.n;
    const dim3 grid((unsigned)((size_t)p.n * p.tiles_y * p.tiles_x));
    if (c.ic4 == 1 && c.oct == 4)
        c.s == 1 ? launch_s<1, 4, 1>(p, c.epi, grid, c.smem, s) : launch_s<1, 4, 2>(p, c.epi, grid, c.smem, s);
    else if (c.ic4 == 1)
        c.s == 1 ? launch_s<1, 8, 1>(p, c.epi, grid, c.smem, s) : launch_s<1, 8, 2>(p, c.epi, grid, c.smem, s);
    else if (c.ic4 == 2)
        c.s == 1 ? launch_s<2, 4, 1>(p, c.epi, grid, c.smem, s) : launch_s<2, 4, 2>(p, c.epi, grid, c.smem, s);
    else
        c.s == 1 ? launch_s<4, 2, 1>(p, c.epi, grid, c.smem, s) : launch_s<4, 2, 2>(p, c.epi, grid, c.smem, s);
    return 0;
}

void conv_small_free(ConvSmall *c) { delete c; }

}  // namespace uq
