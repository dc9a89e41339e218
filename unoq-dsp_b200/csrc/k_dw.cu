// k_dw.cu -- bandwidth-bound depthwise convolution (plan code 15) on the CUDA cores.
//
// Reference semantics (runtime/qnn.c:807-983, 1228-1245; depthwise5.h): per channel
// acc = bias + sum over taps (x + 128) * w, taps outside the image reading the zero point,
// then y = post[clamp(scale(acc, m, s) + yzp)]. Here the +128 is folded into the bias on the
// host (bias' = bias + 128 * sum w), so the device accumulates signed x * w with dp4a.
//
// Block = one output tile (TH rows x TW columns) of one image for CB channels. The input tile
// plus halo is staged in shared memory with 16-byte loads (zero-point fill at the borders),
// each input byte leaving HBM once. A thread owns 4 adjacent output pixels x 4 channels; for
// every kernel row it reads the needed input words once, transposes groups of 4 taps x 4
// channels with byte permutes so that one dp4a adds 4 taps of one channel, and uses a masked
// dp4a for a fifth tap. Requantisation is the exact constant form of requant.cuh, with the
// thread's 4 channel constants held in registers.
#include <cstring>
#include <vector>

#include "dw.cuh"
#include "plan.hpp"
#include "requant.cuh"

namespace uq {

namespace {

constexpr int kThreads = 256;

struct DwParams {
    const int8_t *x;
    int8_t *y;
    const uint32_t *wt;     // [C/4][KH][8] transposed weight words (see dw_prepare)
    const EpiChan *epi;     // [C]
    const uint8_t *post;    // 256 bytes or null
    int n, ih, iw, c, oh, ow, pt, pl;
    int lo, hi, xzp;
    int cb, tw, th;         // channels per block, tile width / height (output pixels)
    int tiles_x, tiles_y;
};

__device__ __forceinline__ void transpose4(uint32_t x0, uint32_t x1, uint32_t x2, uint32_t x3, uint32_t (&y)[4]) {
    const uint32_t a = __byte_perm(x0, x1, 0x5140), b = __byte_perm(x0, x1, 0x7362);
    const uint32_t c = __byte_perm(x2, x3, 0x5140), d = __byte_perm(x2, x3, 0x7362);
    y[0] = __byte_perm(a, c, 0x5410);
    y[1] = __byte_perm(a, c, 0x7632);
    y[2] = __byte_perm(b, d, 0x5410);
    y[3] = __byte_perm(b, d, 0x7632);
}

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

template <int KH, int KW, int SH, int EPI>
__global__ void __launch_bounds__(kThreads) dw_kernel(const DwParams p) {
    extern __shared__ __align__(16) uint8_t smem[];
    constexpr int NW = 3 * SH + KW;  // input words per kernel row for 4 output pixels
    const int cb = p.cb, tw = p.tw, th = p.th;
    const int ir = (th - 1) * SH + KH, icol = (tw - 1) * SH + KW;
    uint8_t *sLut = smem;                       // 256 bytes
    uint8_t *sIn = smem + 256;                  // [ir][icol][cb]

    int tile = blockIdx.x;
    const int tx = tile % p.tiles_x;
    tile /= p.tiles_x;
    const int ty = tile % p.tiles_y;
    const int n = tile / p.tiles_y;
    const int c0 = blockIdx.y * cb;
    const int iy0 = ty * th * SH - p.pt, ix0 = tx * tw * SH - p.pl;

    if (p.post)
        for (int i = threadIdx.x; i < 256; i += kThreads) sLut[i] = p.post[i];
    const uint32_t fillw = 0x01010101u * (uint8_t)p.xzp;
    const uint4 fill = make_uint4(fillw, fillw, fillw, fillw);
    const int c16 = cb / 16;
    for (int i = threadIdx.x; i < ir * icol * c16; i += kThreads) {
        const int cc = i % c16, pix = i / c16;
        const int col = pix % icol, row = pix / icol;
        const int iy = iy0 + row, ix = ix0 + col;
        uint4 v = fill;
        if (iy >= 0 && ix >= 0 && iy < p.ih && ix < p.iw)
            v = __ldg(reinterpret_cast<const uint4 *>(p.x + (((size_t)n * p.ih + iy) * p.iw + ix) * p.c + c0 + cc * 16));
        *reinterpret_cast<uint4 *>(sIn + (size_t)pix * cb + cc * 16) = v;
    }

    const int cgs = cb / 4;
    const int cg = threadIdx.x % cgs;
    const int slot = threadIdx.x / cgs;
    const int quads = tw / 4;
    const int r = slot / quads, q = slot % quads;
    const int c = c0 + cg * 4;
    const int oy = ty * th + r;
    const int ox = tx * tw + q * 4;

    // weights: per kernel row, 4 words of 4 taps (one per channel) + 4 mask words for a 5th tap
    uint32_t w4[KH][4], wm[KH][4];
    const uint32_t *wsrc = p.wt + (size_t)(c / 4) * KH * 8;
#pragma unroll
    for (int ky = 0; ky < KH; ky++)
#pragma unroll
        for (int ch = 0; ch < 4; ch++) {
            w4[ky][ch] = __ldg(wsrc + ky * 8 + ch);
            wm[ky][ch] = KW == 5 ? __ldg(wsrc + ky * 8 + 4 + ch) : 0u;
        }
    EpiChan e[4];
#pragma unroll
    for (int ch = 0; ch < 4; ch++) e[ch] = p.epi[c + ch];
    __syncthreads();

    int acc[4][4];
#pragma unroll
    for (int j = 0; j < 4; j++)
#pragma unroll
        for (int ch = 0; ch < 4; ch++) acc[j][ch] = 0;
    const uint8_t *base = sIn + ((size_t)(r * SH) * icol + q * 4 * SH) * cb + cg * 4;
#pragma unroll
    for (int ky = 0; ky < KH; ky++) {
        uint32_t xw[NW];
#pragma unroll
        for (int i = 0; i < NW; i++)
            xw[i] = *reinterpret_cast<const uint32_t *>(base + ((size_t)ky * icol + i) * cb);
#pragma unroll
        for (int j = 0; j < 4; j++) {
            const int b = j * SH;
            uint32_t t[4];
            transpose4(xw[b], xw[b + 1], xw[b + 2], KW > 3 ? xw[b + 3] : xw[b], t);
#pragma unroll
            for (int ch = 0; ch < 4; ch++) {
                acc[j][ch] = __dp4a((int)t[ch], (int)w4[ky][ch], acc[j][ch]);
                if (KW == 5) acc[j][ch] = __dp4a((int)xw[b + 4], (int)wm[ky][ch], acc[j][ch]);
            }
        }
    }
    if (r >= th || oy >= p.oh) return;
    const uint8_t *lut = p.post ? sLut : nullptr;
#pragma unroll
    for (int j = 0; j < 4; j++) {
        if (ox + j >= p.ow) break;
        uint32_t packed = 0;
#pragma unroll
        for (int ch = 0; ch < 4; ch++) {
            int32_t v = requant<EPI>(acc[j][ch], e[ch], p.lo, p.hi);
            if (lut) v = (int8_t)lut[v + 128];
            packed |= (uint32_t)(uint8_t)v << (8 * ch);
        }
        *reinterpret_cast<uint32_t *>(p.y + (((size_t)n * p.oh + oy) * p.ow + ox + j) * p.c + c) = packed;
    }
}

template <int KH, int KW, int SH>
void launch_shape(const DwParams &p, int epi, dim3 grid, size_t smem, cudaStream_t s) {
    if (epi == 0) dw_kernel<KH, KW, SH, 0><<<grid, kThreads, smem, s>>>(p);
    else if (epi == 1) dw_kernel<KH, KW, SH, 1><<<grid, kThreads, smem, s>>>(p);
    else dw_kernel<KH, KW, SH, 2><<<grid, kThreads, smem, s>>>(p);
}

}  // namespace

struct DwFast {
    DwParams p{};
    int kh = 3, kw = 3, sh = 1, epi = 0;
    size_t smem = 0;
};

int dw_prepare(const int8_t *w, const int32_t *q, const uint8_t *post_dev, const ConvGeom &g,
               const std::function<void *(size_t)> &alloc, DwFast **out) {
    *out = nullptr;
    // Shapes taken: 3x3 or 5x5, equal strides of 1 or 2, no dilation, 16-channel blocks.
    if (!((g.kh == 3 && g.kw == 3) || (g.kh == 5 && g.kw == 5)) || g.sh != g.sw || (g.sh != 1 && g.sh != 2) ||
        g.dh != 1 || g.dw != 1 || g.oc % 16 != 0)
        return 0;
    const int C = g.oc, K = g.kh;
    const int32_t *bias = q + kHead, *mult = bias + C, *shift = mult + C;
    const int yzp = q[13];
    // weight words: [C/4][KH][ w4 x4 | mask x4 ]
    std::vector<uint32_t> wt((size_t)C / 4 * K * 8, 0);
    std::vector<EpiChan> epi(C);
    bool fast = true;
    for (int c = 0; c < C; c++) {
        long long sum = 0;
        for (int t = 0; t < g.kh * g.kw; t++) sum += w[t * C + c];
        epi[c] = make_epilogue((long long)bias[c] + 128 * sum, mult[c], shift[c], yzp);
        fast &= shift[c] <= -1 && shift[c] >= -15;
    }
    for (int c4 = 0; c4 < C / 4; c4++)
        for (int ky = 0; ky < K; ky++)
            for (int ch = 0; ch < 4; ch++) {
                const int c = c4 * 4 + ch;
                uint32_t word = 0;
                for (int kx = 0; kx < 4 && kx < g.kw; kx++)
                    word |= (uint32_t)(uint8_t)w[(ky * g.kw + kx) * C + c] << (8 * kx);
                wt[((size_t)c4 * K + ky) * 8 + ch] = word;
                if (g.kw == 5) wt[((size_t)c4 * K + ky) * 8 + 4 + ch] = (uint32_t)(uint8_t)w[(ky * 5 + 4) * C + c] << (8 * ch);
            }
    const int epi_mode = !fast ? 2 : (q[14] >= yzp ? 0 : 1);
    if (epi_mode != 2)
        for (auto &e : epi) e.sh = e.sh >= 32 ? e.sh - 32 : 0;
    void *dwt = alloc(wt.size() * 4), *de = alloc(epi.size() * sizeof(EpiChan));
    if (!dwt || !de) return 2001;
    if (cudaMemcpy(dwt, wt.data(), wt.size() * 4, cudaMemcpyHostToDevice) != cudaSuccess ||
        cudaMemcpy(de, epi.data(), epi.size() * sizeof(EpiChan), cudaMemcpyHostToDevice) != cudaSuccess)
        return 2001;
    DwFast *d = new DwFast();
    DwParams &p = d->p;
    p.wt = static_cast<const uint32_t *>(dwt);
    p.epi = static_cast<const EpiChan *>(de);
    p.post = post_dev;
    p.ih = g.ih, p.iw = g.iw, p.c = C, p.oh = g.oh, p.ow = g.ow, p.pt = g.pt, p.pl = g.pl;
    p.lo = q[14], p.hi = q[15], p.xzp = q[12];
    p.cb = C % 64 == 0 ? 64 : C % 32 == 0 ? 32 : 16;
    p.tw = g.ow <= 8 ? 8 : 16;
    p.th = (kThreads / (p.cb / 4)) / (p.tw / 4);
    p.tiles_x = (g.ow + p.tw - 1) / p.tw;
    p.tiles_y = (g.oh + p.th - 1) / p.th;
    d->kh = g.kh, d->kw = g.kw, d->sh = g.sh, d->epi = epi_mode;
    const int ir = (p.th - 1) * g.sh + g.kh, icol = (p.tw - 1) * g.sh + g.kw;
    d->smem = 256 + (size_t)ir * icol * p.cb;
    if (d->smem > 48 * 1024) {
        static bool attr = false;
        if (!attr) {
            // every instantiation may need more than the default 48 KB
            cudaFuncSetAttribute(dw_kernel<5, 5, 2, 0>, cudaFuncAttributeMaxDynamicSharedMemorySize, 100 * 1024);
            cudaFuncSetAttribute(dw_kernel<5, 5, 2, 1>, cudaFuncAttributeMaxDynamicSharedMemorySize, 100 * 1024);
            cudaFuncSetAttribute(dw_kernel<5, 5, 2, 2>, cudaFuncAttributeMaxDynamicSharedMemorySize, 100 * 1024);
            attr = true;
        }
        if (d->smem > 100 * 1024) {
            delete d;
            return 0;
        }
    }
    *out = d;
    return 0;
}

int dw_launch(const DwFast &d, const int8_t *x, int8_t *y, const ConvGeom &g, cudaStream_t s) {
    DwParams p = d.p;
    p.x = x;
    p.y = y;
    p.n = g.n;
    dim3 grid((unsigned)(p.n * p.tiles_y * p.tiles_x), (unsigned)(p.c / p.cb));
    if (d.kh == 3 && d.sh == 1) launch_shape<3, 3, 1>(p, d.epi, grid, d.smem, s);
    else if (d.kh == 3) launch_shape<3, 3, 2>(p, d.epi, grid, d.smem, s);
    else if (d.sh == 1) launch_shape<5, 5, 1>(p, d.epi, grid, d.smem, s);
    else launch_shape<5, 5, 2>(p, d.epi, grid, d.smem, s);
    return 0;
}

void dw_free(DwFast *d) { delete d; }

}  // namespace uq
