// k_dw.cu -- bandwidth-bound depthwise convolution (plan code 15) on the CUDA cores.
//
// Reference semantics (runtime/qnn.c:807-983, 1228-1245; depthwise5.h): per channel
// acc = bias + sum over taps (x + 128) * w, taps outside the image reading the zero point,
// then y = post[clamp(scale(acc, m, s) + yzp)]. Here the +128 is folded into the bias on the
// host (bias' = bias + 128 * sum w), so the device accumulates signed x * w with dp4a.
//
// Block = one output tile (TH rows x TW = 7 or 8 columns) of one image for CB channels.
//  * Fill: the input tile plus halo is read with 16-byte loads (4 pixels x 16 channels per
//    thread, zero point outside the image), transposed in registers with byte permutes, and
//    stored as byte planes: plane[channel][row][column], 4 columns per 32-bit word. Each input
//    byte leaves HBM once per tile.
//  * Compute: a thread owns one channel x TW adjacent output pixels x 2 output rows. For every
//    input row it loads the row's words once, forms the sliding 4-column windows with funnel
//    shifts, and adds 4 taps per dp4a against the channel's weight words; the 5th tap of a
//    5-wide row is byte 3 of the next window, so it costs one dp4a and no shift. Each loaded row
//    feeds both output rows.
//  * Epilogue: exact requantisation (requant.cuh constants in registers) and the optional post
//    table; the bytes are staged NHWC in shared memory and written with 16-byte stores.
#include <cstdlib>
#include <cstring>
#include <vector>

#include "dw.cuh"
#include "plan.hpp"
#include "requant.cuh"

namespace uq {

namespace {


struct DwParams {
    const int8_t *x;
    int8_t *y;
    const uint32_t *wt;     // [C][KH][2] weight words: taps 0-3 (0 past KW), 5th tap in byte 3
    const EpiChan *epi;     // [C]
    const uint8_t *post;    // 256 bytes or null
    int n, ih, iw, c, oh, ow, pt, pl;
    int lo, hi, xzp;
    int cb, th;             // channels per block, output rows per tile
    int tiles_x, tiles_y;
    int ir, pw, plane;      // input rows per tile, words per plane row, words per plane (odd)
    int cb_shift;           // log2(cb)
    // multiply-shift division (no run-time divide in the per-unit index arithmetic)
    FastDiv f_tx, f_ty, f_pw, f_ir;
};

__device__ __forceinline__ void transpose4(uint32_t x0, uint32_t x1, uint32_t x2, uint32_t x3, uint32_t (&y)[4]) {
    const uint32_t a = __byte_perm(x0, x1, 0x5140), b = __byte_perm(x0, x1, 0x7362);
    const uint32_t c = __byte_perm(x2, x3, 0x5140), d = __byte_perm(x2, x3, 0x7362);
    y[0] = __byte_perm(a, c, 0x5410);
    y[1] = __byte_perm(a, c, 0x7632);
    y[2] = __byte_perm(b, d, 0x5410);
    y[3] = __byte_perm(b, d, 0x7632);
}

// Exact requantisation before the clamp (the forms of requant.cuh's EpiChan).
template <int EPI>
__device__ __forceinline__ int32_t requant_raw(int32_t acc, const EpiChan &e) {
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
    return v;
}
template <int EPI>
__device__ __forceinline__ int32_t requant(int32_t acc, const EpiChan &e, int lo, int hi) {
    const int32_t v = requant_raw<EPI>(acc, e);
    return v < lo ? lo : (v > hi ? hi : v);
}
// Clamp to [-128, 127] in one saturating conversion.
__device__ __forceinline__ int32_t sat_s8(int32_t v) {
    int32_t r;
    asm("cvt.sat.s8.s32 %0, %1;" : "=r"(r) : "r"(v));
    return r;
}

// Blocks per SM the compiler must fit in registers: with 2 output rows per thread, 4 for 3x3
// stride 1 (14% faster on 14x14x192 than 2), 3 elsewhere (4 spills on the 5x5 and stride-2
// shapes); with 4 rows per thread, 2 (64 registers). Each block's fill, compute and store run back
// to back, so resident blocks are what overlaps one block's loads with another's arithmetic.
// TW = output columns per tile (one thread's row of outputs): 7 or 8, whichever wastes fewer
// columns of the layer's width (7 for MobileNetV4's 28 / 14 / 7-wide layers).
// kR = output rows per thread: 4 for stride-1 layers whose whole image height is one tile (each
// loaded input row and its windows then feed up to 3-5 outputs per tap row: 15-17% faster on
// 28x28x64 5x5 and 7x7x512 3x3), else 2 (4 rows was 68% slower on 28x28x192 5x5 stride 2).
template <int K, int S, int EPI, int TW, int kR>
__global__ void __launch_bounds__(512, kR == 4 ? 2 : ((K == 3 && S == 1) ? 4 : 3)) dw_kernel(const DwParams p) {
    extern __shared__ __align__(16) uint8_t smem[];
    constexpr int TWIN = (TW - 1) * S + K;       // input columns per tile
    constexpr int NWORD = (TWIN + 3) / 4;         // words per input row
    constexpr int NWIN = (TW - 1) * S + 2;        // window starts 0 .. ((TW - 1) * S + 1)
    const int cb = p.cb, th = p.th;
    uint8_t *sLut = smem;                                                   // 256 bytes
    uint32_t *sPlane = reinterpret_cast<uint32_t *>(smem + 256);            // [cb][plane words]
    uint8_t *sOut = smem + 256 + (size_t)cb * p.plane * 4;                  // [th][8][cb]

    const int t1 = p.f_tx.div((int)blockIdx.x), tx = (int)blockIdx.x - t1 * p.tiles_x;
    const int n = p.f_ty.div(t1), ty = t1 - n * p.tiles_y;
    const int c0 = blockIdx.y * cb;
    const int iy0 = ty * th * S - p.pt, ix0 = tx * TW * S - p.pl;

    // Launched with programmatic serialization: the next kernel may be scheduled once every block
    // has started; the input is read only after the previous kernel has completed.
    grid_dep_launch();
    if (p.post)
        for (int i = threadIdx.x; i < 256; i += blockDim.x) sLut[i] = p.post[i];
    grid_dep_wait();
    // ---- fill: unit = (16-channel chunk, input row, 4-column group)
    {
        const uint32_t fillw = 0x01010101u * (uint8_t)p.xzp;
        const uint4 fill = make_uint4(fillw, fillw, fillw, fillw);
        const int units = (cb / 16) * p.ir * p.pw;
        for (int u = threadIdx.x; u < units; u += blockDim.x) {
            const int rest = p.f_pw.div(u), wc = u - rest * p.pw;
            const int chunk = p.f_ir.div(rest), row = rest - chunk * p.ir;
            const int iy = iy0 + row;
            uint4 px[4];
#pragma unroll
            for (int i = 0; i < 4; i++) {
                const int ix = ix0 + wc * 4 + i;
                px[i] = fill;
                if (iy >= 0 && iy < p.ih && ix >= 0 && ix < p.iw)
                    px[i] = __ldg(reinterpret_cast<const uint4 *>(
                        p.x + (((size_t)n * p.ih + iy) * p.iw + ix) * p.c + c0 + chunk * 16));
            }
            const uint32_t w0[4] = {px[0].x, px[0].y, px[0].z, px[0].w}, w1[4] = {px[1].x, px[1].y, px[1].z, px[1].w};
            const uint32_t w2[4] = {px[2].x, px[2].y, px[2].z, px[2].w}, w3[4] = {px[3].x, px[3].y, px[3].z, px[3].w};
            uint32_t *dst = sPlane + (size_t)(chunk * 16) * p.plane + row * p.pw + wc;
#pragma unroll
            for (int g = 0; g < 4; g++) {
                uint32_t t[4];
                transpose4(w0[g], w1[g], w2[g], w3[g], t);
#pragma unroll
                for (int k = 0; k < 4; k++) dst[(size_t)(g * 4 + k) * p.plane] = t[k];
            }
        }
    }

    // ---- this thread: channel ch, output rows kR * rg .. kR * rg + kR - 1 of the tile
    const int ch = threadIdx.x & (cb - 1), rg = threadIdx.x >> p.cb_shift;
    const int c = c0 + ch;
    uint32_t wa[K], wb[K];
#pragma unroll
    for (int ky = 0; ky < K; ky++) {
        wa[ky] = __ldg(p.wt + ((size_t)c * K + ky) * 2);
        wb[ky] = K == 5 ? __ldg(p.wt + ((size_t)c * K + ky) * 2 + 1) : 0u;
    }
    const EpiChan e = p.epi[c];
    __syncthreads();

    int acc[kR][TW];
#pragma unroll
    for (int r = 0; r < kR; r++)
#pragma unroll
        for (int j = 0; j < TW; j++) acc[r][j] = 0;
    const uint32_t *plane = sPlane + (size_t)ch * p.plane + (size_t)(rg * kR * S) * p.pw;
    // input rows used by the thread's kR output rows: (kR - 1) * S + K
#pragma unroll
    for (int ir = 0; ir < (kR - 1) * S + K; ir++) {
        uint32_t wd[NWORD + 1];
#pragma unroll
        for (int i = 0; i < NWORD; i++) wd[i] = plane[ir * p.pw + i];
        wd[NWORD] = 0;
        uint32_t win[NWIN];
#pragma unroll
        for (int s = 0; s < NWIN; s++) win[s] = (s & 3) ? __funnelshift_r(wd[s >> 2], wd[(s >> 2) + 1], 8 * (s & 3)) : wd[s >> 2];
#pragma unroll
        for (int r = 0; r < kR; r++) {
            const int ky = ir - r * S;
            if (ky < 0 || ky >= K) continue;
#pragma unroll
            for (int j = 0; j < TW; j++) {
                acc[r][j] = __dp4a((int)win[j * S], (int)wa[ky], acc[r][j]);
                if (K == 5) acc[r][j] = __dp4a((int)win[j * S + 1], (int)wb[ky], acc[r][j]);
            }
        }
    }
    const uint8_t *lut = p.post ? sLut : nullptr;
    if (!lut && p.lo == -128 && p.hi == 127) {  // the clamp is the int8 range: one saturating step
#pragma unroll
        for (int r = 0; r < kR; r++)
#pragma unroll
            for (int j = 0; j < TW; j++)
                sOut[((size_t)(rg * kR + r) * TW + j) * cb + ch] = (uint8_t)sat_s8(requant_raw<EPI>(acc[r][j], e));
    } else {
#pragma unroll
        for (int r = 0; r < kR; r++)
#pragma unroll
            for (int j = 0; j < TW; j++) {
                int32_t v = requant<EPI>(acc[r][j], e, p.lo, p.hi);
                if (lut) v = (int8_t)lut[v + 128];
                sOut[((size_t)(rg * kR + r) * TW + j) * cb + ch] = (uint8_t)v;
            }
    }
    __syncthreads();
    // ---- copy-out: 16 channels of one pixel per store
    const int units = th * TW * (cb / 16);
    for (int u = threadIdx.x; u < units; u += blockDim.x) {
        const int chunk = u & ((cb >> 4) - 1), pix = u >> (p.cb_shift - 4);
        const int j = pix % TW, row = pix / TW;
        const int oy = ty * th + row, ox = tx * TW + j;
        if (oy >= p.oh || ox >= p.ow) continue;
        *reinterpret_cast<uint4 *>(p.y + (((size_t)n * p.oh + oy) * p.ow + ox) * p.c + c0 + chunk * 16) =
            *reinterpret_cast<const uint4 *>(sOut + (size_t)pix * cb + chunk * 16);
    }
}

template <int K, int S, int TW, int R>
void launch_shape(const DwParams &p, int epi, dim3 grid, int threads, size_t smem, cudaStream_t s) {
    if (epi == 0) launch_pdl(kPdlDw, dw_kernel<K, S, 0, TW, R>, grid, threads, smem, s, p);
    else if (epi == 1) launch_pdl(kPdlDw, dw_kernel<K, S, 1, TW, R>, grid, threads, smem, s, p);
    else launch_pdl(kPdlDw, dw_kernel<K, S, 2, TW, R>, grid, threads, smem, s, p);
}

template <int K, int S, int TW, int R>
bool allow_smem_tw(size_t bytes) {
    return cudaFuncSetAttribute(dw_kernel<K, S, 0, TW, R>, cudaFuncAttributeMaxDynamicSharedMemorySize, (int)bytes) ==
               cudaSuccess &&
           cudaFuncSetAttribute(dw_kernel<K, S, 1, TW, R>, cudaFuncAttributeMaxDynamicSharedMemorySize, (int)bytes) ==
               cudaSuccess &&
           cudaFuncSetAttribute(dw_kernel<K, S, 2, TW, R>, cudaFuncAttributeMaxDynamicSharedMemorySize, (int)bytes) ==
               cudaSuccess;
}

// Stride 1 has both row counts per thread; stride 2 only 2.
template <int K, int S>
bool allow_smem(size_t bytes) {
    bool ok = allow_smem_tw<K, S, 7, 2>(bytes) && allow_smem_tw<K, S, 8, 2>(bytes);
    if constexpr (S == 1) ok = ok && allow_smem_tw<K, S, 7, 4>(bytes) && allow_smem_tw<K, S, 8, 4>(bytes);
    return ok;
}

template <int K, int S>
void launch_tw(const DwParams &p, int tw, int rows, int epi, dim3 grid, int threads, size_t smem, cudaStream_t s) {
    if constexpr (S == 1) {
        if (rows == 4) {
            if (tw == 7) launch_shape<K, S, 7, 4>(p, epi, grid, threads, smem, s);
            else launch_shape<K, S, 8, 4>(p, epi, grid, threads, smem, s);
            return;
        }
    }
    if (tw == 7) launch_shape<K, S, 7, 2>(p, epi, grid, threads, smem, s);
    else launch_shape<K, S, 8, 2>(p, epi, grid, threads, smem, s);
}

}  // namespace

struct DwFast {
    DwParams p{};
    int k = 3, s = 1, epi = 0, threads = 0, tw = 8, rows = 2;
    size_t smem = 0;
};

int dw_prepare(const int8_t *w, const int32_t *q, const uint8_t *post_dev, const ConvGeom &g,
               const std::function<void *(size_t)> &alloc, DwFast **out) {
    *out = nullptr;
    // Shapes taken: 3x3 or 5x5, equal strides of 1 or 2, no dilation, 16-channel blocks.
    if (!((g.kh == 3 && g.kw == 3) || (g.kh == 5 && g.kw == 5)) || g.sh != g.sw || (g.sh != 1 && g.sh != 2) ||
        g.dh != 1 || g.dw != 1 || g.oc % 16 != 0)
        return 0;
    const int C = g.oc, K = g.kh, S = g.sh;
    const int32_t *bias = q + kHead, *mult = bias + C, *shift = mult + C;
    const int yzp = q[13];
    // weight words per channel and kernel row: taps 0..3 (zero past KW), then tap 4 in byte 3
    std::vector<uint32_t> wt((size_t)C * K * 2, 0);
    std::vector<EpiChan> epi(C);
    bool fast = true;
    for (int c = 0; c < C; c++) {
        long long sum = 0;
        for (int t = 0; t < K * K; t++) sum += w[t * C + c];
        epi[c] = make_epilogue((long long)bias[c] + 128 * sum, mult[c], shift[c], yzp);
        fast &= epi_fast(epi[c]);
        for (int ky = 0; ky < K; ky++) {
            uint32_t a = 0;
            for (int kx = 0; kx < 4 && kx < K; kx++) a |= (uint32_t)(uint8_t)w[(ky * K + kx) * C + c] << (8 * kx);
            wt[((size_t)c * K + ky) * 2] = a;
            if (K == 5) wt[((size_t)c * K + ky) * 2 + 1] = (uint32_t)(uint8_t)w[(ky * K + 4) * C + c] << 24;
        }
    }
    const int epi_mode = !fast ? 2 : (q[14] >= yzp ? 0 : 1);
    if (epi_mode != 2)
        for (auto &e : epi) e.sh = e.sh >= 32 ? e.sh - 32 : 0;
    // Tile: 7 or 8 columns; the whole image height when it is at most 32 rows, else 16 rows
    // (UNOQ_DW_ROWS=r caps the output rows per tile; a tuning switch, results are unchanged).
    // Output rows per thread: 4 at stride 1 on whole-image tiles, else 2 (see dw_kernel;
    // UNOQ_DW_ROWS4=0 keeps 2 everywhere).
    const char *e4 = std::getenv("UNOQ_DW_ROWS4");
    const int kR = (S == 1 && g.oh <= 32 && !(e4 && e4[0] == '0')) ? 4 : 2;
    int rg = g.oh <= 32 ? (g.oh + kR - 1) / kR : 16 / kR;
    if (const char *er = std::getenv("UNOQ_DW_ROWS")) {
        const int cap = std::atoi(er) / kR;
        if (cap >= 1 && cap < rg) rg = cap;
    }
    // tile width: 7 or 8 output columns, whichever leaves fewer computed columns past the image
    const int tw = ((g.ow + 6) / 7 * 7 - g.ow) < ((g.ow + 7) / 8 * 8 - g.ow) ? 7 : 8;
    // channels per block: 32 for stride 1 on images over 16 rows (smaller blocks, more of them
    // resident: 16% faster than 64 on 28x28x64 5x5), 64 for stride 1 on smaller images (the whole
    // image is one tile, and 32-channel blocks of 64 threads pay their set-up too often: 8-9%
    // faster on 7x7x512 5x5) and for stride 2 (wider halo reuse; 32 was up to 45% slower)
    int cb = S == 1 && g.oh > 16 ? 32 : 64;
    if (const char *ec = std::getenv(S == 1 ? "UNOQ_DW_CB1" : "UNOQ_DW_CB2")) {  // tuning switch
        const int v = std::atoi(ec);
        if (v == 16 || v == 32 || v == 64) cb = v;
    }
    while (cb > 16 && (C % cb != 0 || cb * rg > 512)) cb /= 2;
    if (C % cb != 0 || cb * rg > 512) return 0;
    DwFast *d = new DwFast();
    DwParams &p = d->p;
    p.cb = cb;
    p.th = rg * kR;
    p.tiles_x = (g.ow + tw - 1) / tw;
    p.tiles_y = (g.oh + p.th - 1) / p.th;
    p.ir = (p.th - 1) * S + K;
    p.pw = ((tw - 1) * S + K + 3) / 4;
    p.cb_shift = cb == 16 ? 4 : cb == 32 ? 5 : 6;
    p.f_tx = FastDiv(p.tiles_x);
    p.f_ty = FastDiv(p.tiles_y);
    p.f_pw = FastDiv(p.pw);
    p.f_ir = FastDiv(p.ir);
    p.plane = p.ir * p.pw;
    if ((p.plane & 1) == 0) p.plane++;  // odd plane stride: lanes (channels) fall in distinct banks
    d->k = K, d->s = S, d->epi = epi_mode, d->threads = cb * rg, d->tw = tw, d->rows = kR;
    d->smem = 256 + (size_t)cb * p.plane * 4 + (size_t)p.th * tw * cb;
    if (d->smem > 200 * 1024) {
        delete d;
        return 0;
    }
    if (d->smem > 48 * 1024) {
        const bool ok = K == 3 ? (S == 1 ? allow_smem<3, 1>(d->smem) : allow_smem<3, 2>(d->smem))
                               : (S == 1 ? allow_smem<5, 1>(d->smem) : allow_smem<5, 2>(d->smem));
        if (!ok) {
            delete d;
            return 0;
        }
    }
    void *dwt = alloc(wt.size() * 4), *de = alloc(epi.size() * sizeof(EpiChan));
    if (!dwt || !de ||
        cudaMemcpy(dwt, wt.data(), wt.size() * 4, cudaMemcpyHostToDevice) != cudaSuccess ||
        cudaMemcpy(de, epi.data(), epi.size() * sizeof(EpiChan), cudaMemcpyHostToDevice) != cudaSuccess) {
        delete d;
        return 2001;
    }
    p.wt = static_cast<const uint32_t *>(dwt);
    p.epi = static_cast<const EpiChan *>(de);
    p.post = post_dev;
    p.ih = g.ih, p.iw = g.iw, p.c = C, p.oh = g.oh, p.ow = g.ow, p.pt = g.pt, p.pl = g.pl;
    p.lo = q[14], p.hi = q[15], p.xzp = q[12];
    *out = d;
    return 0;
}

int dw_launch(const DwFast &d, const int8_t *x, int8_t *y, const ConvGeom &g, cudaStream_t s) {
    DwParams p = d.p;
    p.x = x;
    p.y = y;
    p.n = g.n;
    dim3 grid((unsigned)(p.n * p.tiles_y * p.tiles_x), (unsigned)(p.c / p.cb));
    if (d.k == 3 && d.s == 1) launch_tw<3, 1>(p, d.tw, d.rows, d.epi, grid, d.threads, d.smem, s);
    else if (d.k == 3) launch_tw<3, 2>(p, d.tw, d.rows, d.epi, grid, d.threads, d.smem, s);
    else if (d.s == 1) launch_tw<5, 1>(p, d.tw, d.rows, d.epi, grid, d.threads, d.smem, s);
    else launch_tw<5, 2>(p, d.tw, d.rows, d.epi, grid, d.threads, d.smem, s);
    return 0;
}

void dw_free(DwFast *d) { delete d; }

}  // namespace uq
