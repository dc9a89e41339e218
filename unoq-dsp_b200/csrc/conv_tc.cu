// conv_tc.cu -- INT8 implicit-GEMM convolution on the 5th-generation tensor cores (sm_100a).
//
// Computes plan code 14 (runtime/qnn.c:1101-1227) as Y[m, n] = requant(sum_k A[m, k] W[n, k]):
// m = output pixel, n = output channel, k = (ky, kx, ic) reduction index (tflite.py:155 order).
//
// One persistent CTA per SM loops over 128-pixel M tiles of one N tile (grid.y = N tiles):
//   * W: the N tile's weights, prepared on the host in the UMMA K-major SWIZZLE_128B layout
//     (8-row x 128-byte atoms, 16-byte chunks XOR-swizzled by row), copied to shared memory
//     once and kept resident.
//   * A (producer warps, 4 or 8): the im2col rows of a tile, 128 reduction bytes per pipeline
//     stage, in the swizzled layout.
//       - pointwise: one 128 x 128-byte TMA box per stage, issued by one producer thread.
//       - other spatial convs whose input rows fit: the input rows a tile touches (a "band") are
//         copied to shared memory by a loader warp (one bulk copy per row, 2-3 bands in flight),
//         and the producers assemble each pixel's K bytes from the band.
//       - the rest (ic % 16 == 0): cp.async per (pixel, 16 channels); taps outside the image get
//         16 bytes of the input zero point by a plain shared store -- the value the reference
//         feeds its dot product there (qnn.c:1166-1168) -- so no border correction is needed. A
//         warp signals a stage a few stages after issuing it, once its copies have landed.
//   * the MMA warp (one thread) issues tcgen05.mma.kind::i8 (s8 x s8 -> s32, M=128, N=BN, K=32)
//     into 2-4 TMEM accumulators in rotation, so the epilogue of tile i overlaps later MMAs.
//   * the epilogue warps (8 or 16) read the accumulator with tcgen05.ld (thread = pixel row, 16
//     channels per load; each warp owns an equal column part of the tile), requantise with the
//     exact branch-free form of the reference's `scale` (make_epilogue), apply the optional post
//     table or fused residual add, stage the int8 part in shared memory and write it out with
//     their own TMA tensor stores.
//
// Reference arithmetic: the reference multiplies u8 columns (x ^ 0x80) by s8 weights and adds a
// corrected bias; with s8 columns the same sum is  sum x*w + 128*sum(w) + xzp*sum(w_kpad), which
// the host folds into the epilogue constants, so results are bit-identical.
//
// Every wait (mbarrier phases, including the ones that stand in for sub-CTA barriers) is bounded
// by about 2 s of SM clock; on expiry the kernel records a site code in g_tc_error, drains its
// MMAs, frees its TMEM and exits.
#include <cstdio>
#include <cstdlib>
#include <cstring>
#include <numeric>
#include <type_traits>
#include <vector>

#include <cuda.h>

#include "conv_tc.cuh"
#include "device_state.hpp"
#include "plan.hpp"
#include "requant.cuh"
#include "tc_common.cuh"

namespace uq {

namespace {

// Warp roles by index: producers [0, PW), epilogue [PW, PW + EW), MMA issuer PW + EW.
// PW = 4 for pointwise convs (light copies; fewer warps leave more registers), 8 for band / gather
// convs (assembly-heavy). EW = 8 or 16 epilogue warps: EW / 4 warps per TMEM lane quarter, each
// taking a contiguous column part of the tile.
template <int PW, int EW = 8>
struct Roles {
    static constexpr int kProducerWarps = PW;
    static constexpr int kEpilogueWarps = EW;
    static constexpr int kEpilogues = EW * 32;
    static constexpr int kParts = EW / 4;
    static constexpr int kMmaWarp = PW + EW;
    // band / gather configurations (8 producer warps) add one warp that fetches the bands
    static constexpr bool kLoader = PW == 8;
    static constexpr int kLoaderWarp = kMmaWarp + 1;
    static constexpr int kThreads = (kMmaWarp + 1 + (kLoader ? 1 : 0)) * 32;
    static constexpr int kProducers = PW * 32;
    // 16-byte-chunk producers: thread t builds chunk t % 8 of rows t / 8 + kRowStep * i, i < kRowIters.
    static constexpr int kRowStep = kProducers / 8;
    static constexpr int kRowIters = kBM / kRowStep;
    // word-assembly producers: thread t builds chunks t / kBM + kChunkStep * k of row t % kBM.
    static constexpr int kChunkStep = kProducers / kBM;
    static_assert(kBM % kRowStep == 0 && kProducers % kBM == 0, "producer mapping");
};
constexpr int kMaxSmem = 227 * 1024;
constexpr int kWeightBudget = 96 * 1024;

enum Mode { kPointwise = 0, kGather16 = 1, kBand = 2 };

struct Params {
    CUtensorMap ymap;          // output [M rows][oc] int8, box {min(bn,128), 128}, swizzled (TMA store)
    CUtensorMap xmap;          // pointwise input [M rows][ic] int8, box {128, 128}, SWIZZLE_128B (a_tma)
    int a_tma;                 // pointwise A tiles by TMA (one thread) instead of cp.async
    int withhold;              // failure-detection tests only: CTA (0, 0) never signals its first accumulator
    const int8_t *x;
    int8_t *y;
    const int8_t *w;           // [n_tiles][kc][BN x 128] swizzled
    const EpiChan *epi;        // [n_tiles * BN]
    const uint8_t *post;       // 256 bytes or null
    const int *tab;            // band mode: chunk taps (ic % 16 == 0) or word sources (else), see conv_tc_prepare
    long long x_bytes;         // bytes of the whole (batched) input tensor
    int M;                     // total output pixels
    FastDiv f_ow, f_img;       // division by ow and by oh*ow (pixel index -> n, oy, ox)
    int ih, iw, ic, oh, ow, oc;
    int kh, kw, sh, sw, dh, dw, pt, pl;
    int K;                     // kh*kw*ic (unpadded)
    int kc;                    // reduction stages per tile
    int bn;                    // N tile width (multiple of 16, <= 256)
    int stages;
    int lo, hi;
    int xzp;
    int tmem_cols;
    int mode;
    int band_bytes;            // per band buffer (band mode): band_rows x pitch
    int nbands;                // band buffers in rotation (band mode)
    int band_rows;             // most input rows any tile's band spans
    int pitch;                 // band row: ml margin bytes, iw*ic data bytes, right margin (multiple of 16)
    int ml;                    // left margin bytes (multiple of 16)
    int row16;                 // 16-byte chunks of one input row
    int fill_bytes;            // zero-point row read for taps above / below the image
    int K32;                   // K rounded up to 32
    int tab_bytes;             // size of the band table
    int epi_mode;              // EpiMode
    int n_acc;                 // TMEM accumulators in rotation (2 or 4)
    int fold;                  // tiles in flight per epilogue warp group: EW/4 warps per lane quarter split
                               // into column parts (bn / box) x fold tile phases (TMA-store path)
    int store_tma;             // 1: staged tile leaves by TMA tensor store; 0: cooperative stores
    int box;                   // TMA store box: columns of one epilogue warp x 32 rows
    int out_bytes;             // output staging: per-warp double buffers (TMA) or two whole tiles
    // Fused residual add (plan code 18 consuming this conv's output; 0 / null when not fused):
    // y = clamp(scale(T_conv[v + 128] + T_res[r + 128]) + zp) with the add's two 256-entry tables.
    const int8_t *res;         // residual tensor [M][oc] (the add's other operand)
    const int32_t *add_tab;    // the add's q block on the device: tables at +8 (input a), +264 (input b)
    int res_side;              // 0: this conv is the add's input a (table at +8), 1: input b
    AddEpi add;                // the add's scale as requant.cuh constants (bias 0) and clamp
    int swz;                   // staging swizzle: 0 none (16 B rows), 1 = 32 B, 2 = 64 B, 3 = 128 B span
};

// One staging buffer of the output tile for cooperative stores: 128 padded rows.
__host__ __device__ inline size_t out_stride(int bn) { return ((size_t)kBM * (bn + 16) + 1023) & ~(size_t)1023; }
// One epilogue warp's staging buffer for the TMA store: 32 rows x box bytes, swizzled like the
// box, 1024-byte aligned so swizzle atoms line up.
__host__ __device__ inline size_t warp_stage_bytes(int box) { return ((size_t)32 * box + 1023) & ~(size_t)1023; }

// Shared-memory carve-up, identical on host (sizing) and device.
struct Layout {
    size_t a, b, out, band, epi, lut, addt, tab, bars, total;
    __host__ __device__ Layout(int stages, int kc, int bn, int band_bytes, int nbands, int fill_bytes, int tab_bytes,
                               int out_bytes) {
        size_t o = 0;
        a = o;
        o += (size_t)stages * kStageBytes;
        b = o;
        o += (size_t)kc * bn * kBK;
        out = o;
        o += (size_t)out_bytes;
        band = o;
        o += (size_t)nbands * (size_t)band_bytes + (size_t)fill_bytes;
        epi = (o + 31) & ~(size_t)31;
        o = epi + (size_t)bn * sizeof(EpiChan);
        lut = o;
        o += 256;
        addt = (o + 15) & ~(size_t)15;  // fused-add tables: conv side, residual side (256 int32 each)
        o = addt + 2048;
        tab = (o + 15) & ~(size_t)15;
        o = tab + (size_t)tab_bytes;
        bars = (o + 7) & ~(size_t)7;
        o = bars + (size_t)(2 * stages + 22) * 8 + 16;
        total = o + 1024;  // base alignment slack
    }
};

}  // namespace

namespace {

// A fused residual add (qnn.c:175-183) runs inside epilogue_chunk on the requantised int32 values:
// y = clamp(scale(T_conv[v + 128] + T_res[r + 128]) + zp) with the add's scale as requant.cuh
// constants; rows past M (the last tile) read no residual and are never stored.

__device__ __forceinline__ void mbar_expect_tx(uint32_t bar, uint32_t bytes) {
    asm volatile("mbarrier.arrive.expect_tx.shared::cta.b64 _, [%0], %1;" ::"r"(bar), "r"(bytes) : "memory");
}

__device__ __forceinline__ void tma_load_2d(uint32_t dst, const CUtensorMap *map, int x, int y, uint32_t bar) {
    asm volatile(
        "cp.async.bulk.tensor.2d.shared::cluster.global.tile.mbarrier::complete_tx::bytes [%0], [%1, {%2, %3}], "
        "[%4];" ::"r"(dst),
        "l"(reinterpret_cast<uint64_t>(map)), "r"(x), "r"(y), "r"(bar)
        : "memory");
}

// One contiguous global -> shared bulk copy (no tensor map, no multicast); both addresses 16-byte
// aligned, `bytes` a multiple of 16. Completes `bytes` of transactions on `bar`.
__device__ __forceinline__ void bulk_load(uint32_t dst, const void *src, uint32_t bytes, uint32_t bar) {
    asm volatile("cp.async.bulk.shared::cluster.global.mbarrier::complete_tx::bytes [%0], [%1], %2, [%3];" ::"r"(dst),
                 "l"(src), "r"(bytes), "r"(bar)
                 : "memory");
}

// Band of M tile `mt` (band mode): global input rows [g_lo, g_lo + rows), image-major rows being
// contiguous in memory.
__device__ __forceinline__ void band_of(const Params &p, int mt, long long &g_lo, int &rows) {
    const int m0 = mt * kBM, m1 = min(p.M, m0 + kBM) - 1;
    const int n0 = p.f_img.div(m0), oy0 = p.f_ow.div(m0 - n0 * p.f_img.d);
    const int n1 = p.f_img.div(m1), oy1 = p.f_ow.div(m1 - n1 * p.f_img.d);
    g_lo = (long long)n0 * p.ih + max(0, oy0 * p.sh - p.pt);
    const long long g_hi = (long long)n1 * p.ih + max(-1, min(p.ih - 1, oy1 * p.sh - p.pt + (p.kh - 1) * p.dh));
    rows = g_hi >= g_lo ? (int)(g_hi - g_lo + 1) : 0;
}

template <int EPI, int PW, int EW>
__global__ void __launch_bounds__(Roles<PW, EW>::kThreads, 1) conv_tc_kernel(const __grid_constant__ Params p) {
    using R = Roles<PW, EW>;
    constexpr int kProducerWarps = R::kProducerWarps, kMmaWarp = R::kMmaWarp;
    constexpr int kProducers = R::kProducers, kRowStep = R::kRowStep;
    constexpr int kRowIters = R::kRowIters, kChunkStep = R::kChunkStep;
    constexpr int kEpilogueWarps = R::kEpilogueWarps, kEpilogues = R::kEpilogues, kParts = R::kParts;
    extern __shared__ uint8_t smem_raw[];
    // 1024-byte aligned base, formed by pointer arithmetic on the __shared__ array so that every
    // pointer derived from it stays in the shared address space (ld.shared, not generic loads).
    uint8_t *smem = smem_raw + ((1024u - (smem_u32(smem_raw) & 1023u)) & 1023u);
    const int S = p.stages;
    const Layout L(S, p.kc, p.bn, p.band_bytes, p.nbands, p.fill_bytes, p.tab_bytes, p.out_bytes);
    uint8_t *sA = smem + L.a;
    uint8_t *sB = smem + L.b;
    uint8_t *sOut = smem + L.out;
    uint8_t *sBand = smem + L.band;
    // per-channel constants, structure of arrays (k: int64[bn], then six int32[bn])
    long long *sK = reinterpret_cast<long long *>(smem + L.epi);
    int *sI = reinterpret_cast<int *>(sK + p.bn);
    const EpiSoA E{sK, sI, sI + p.bn, sI + 2 * p.bn, sI + 3 * p.bn, sI + 4 * p.bn, sI + 5 * p.bn};
    uint8_t *sLut = smem + L.lut;
    int32_t *sAdd = reinterpret_cast<int32_t *>(smem + L.addt);  // [0,256) conv side, [256,512) residual
    int *sTab = reinterpret_cast<int *>(smem + L.tab);
    uint64_t *bars = reinterpret_cast<uint64_t *>(smem + L.bars);
    uint64_t *full = bars, *empty = bars + S;
    uint64_t *tfull = bars + 2 * S, *tempty = bars + 2 * S + 4;
    uint64_t *bfull = bars + 2 * S + 8, *drain = bars + 2 * S + 9;
    uint64_t *psync = bars + 2 * S + 10, *esync = bars + 2 * S + 11;
    uint64_t *bandfull = bars + 2 * S + 14, *bandfree = bars + 2 * S + 18;  // band buffers (<= 4)
    uint32_t *tmem_slot = reinterpret_cast<uint32_t *>(bars + 2 * S + 22);
    volatile int *abort = reinterpret_cast<volatile int *>(tmem_slot + 1);

    const int warp = threadIdx.x / 32, lane = threadIdx.x % 32;
    const int ntile = blockIdx.y;
    const int m_tiles = (p.M + kBM - 1) / kBM;
    const size_t b_bytes = (size_t)p.kc * p.bn * kBK;

    if (threadIdx.x == 0) {
        for (int s = 0; s < S; s++) {
            mbar_init(smem_u32(full + s), p.a_tma ? 1 : kProducerWarps);
            mbar_init(smem_u32(empty + s), 1);
        }
        for (int a = 0; a < 4; a++) {
            mbar_init(smem_u32(tfull + a), 1);
            mbar_init(smem_u32(tempty + a), kEpilogueWarps / p.fold);
        }
        mbar_init(smem_u32(bfull), kProducerWarps);
        mbar_init(smem_u32(drain), 1);
        mbar_init(smem_u32(psync), kProducerWarps);
        for (int b = 0; b < 4; b++) {
            mbar_init(smem_u32(bandfull + b), 1);  // the loader's expect_tx; its bulk copies complete the bytes
            mbar_init(smem_u32(bandfree + b), kProducerWarps);
        }
        mbar_init(smem_u32(esync), kEpilogueWarps);
        *abort = 0;
        asm volatile("fence.mbarrier_init.release.cluster;" ::: "memory");
    }
    for (int i = threadIdx.x; i < p.bn; i += blockDim.x) {
        const EpiChan c = p.epi[(size_t)ntile * p.bn + i];
        sK[i] = c.k;
        sI[i] = c.m;
        sI[p.bn + i] = c.cut;
        sI[2 * p.bn + i] = c.sh;
        sI[3 * p.bn + i] = c.ls;
        sI[4 * p.bn + i] = c.bs;
        sI[5 * p.bn + i] = c.zadd;
    }
    if (p.post)
        for (int i = threadIdx.x; i < 256; i += blockDim.x) sLut[i] = p.post[i];
    if (p.res)
        for (int i = threadIdx.x; i < 512; i += blockDim.x) {
            const int side = (i >> 8) ^ p.res_side;  // conv side first
            sAdd[i] = p.add_tab[8 + 256 * side + (i & 255)];
        }
    if (p.mode == kBand)
        for (int i = threadIdx.x; i < (p.tab_bytes >> 2); i += blockDim.x) sTab[i] = p.tab[i];
    if (warp == kMmaWarp) {  // the MMA warp owns the TMEM allocation
        asm volatile("tcgen05.alloc.cta_group::1.sync.aligned.shared::cta.b32 [%0], %1;" ::"r"(smem_u32(tmem_slot)),
                     "r"(p.tmem_cols));
        asm volatile("tcgen05.relinquish_alloc_permit.cta_group::1.sync.aligned;");
    }
    tc_fence_before();
    __syncthreads();
    tc_fence_after();
    const uint32_t tmem_base = *tmem_slot;
    // Launched with programmatic serialization: every role but the MMA warp (shared memory and TMEM
    // only) waits here for the previous kernel's activations -- the producers after their weight
    // copy, which reads load-time constants.
    if (warp >= kProducerWarps && warp != kMmaWarp) grid_dep_wait();

    if (warp < kProducerWarps) {
        // ------------------------------------------------------------------ producers
        const int t = threadIdx.x;  // 0..127
        const uint8_t *wsrc = reinterpret_cast<const uint8_t *>(p.w) + (size_t)ntile * b_bytes;
        for (size_t off = (size_t)t * 16; off < b_bytes; off += kProducers * 16) cp_async16(smem_u32(sB + off), wsrc + off);
        cp_async_commit();
        cp_async_wait<0>();
        fence_proxy_async();
        __syncwarp();
        if (lane == 0) mbar_arrive(smem_u32(bfull));
        grid_dep_wait();

        long long it = 0;
        if (p.a_tma) {
            // Pointwise A tiles by TMA: producer thread 0 loads each stage as one 128 x 128-byte box
            // of the [M][ic] input, already in the SWIZZLE_128B layout. Columns past ic and rows past
            // M read as zero (the zero columns meet zero weights; those rows are never stored).
            if (t == 0) {
                bool ok = true;
                for (int mt = blockIdx.x; mt < m_tiles && ok; mt += gridDim.x)
                    for (int kc = 0; kc < p.kc; kc++, it++) {
                        const int s = (int)(it % S);
                        if (!mbar_wait(smem_u32(empty + s), (uint32_t)(((it / S) & 1) ^ 1), abort, 111)) {
                            ok = false;
                            break;
                        }
                        mbar_expect_tx(smem_u32(full + s), (uint32_t)kStageBytes);
                        tma_load_2d(smem_u32(sA + (size_t)s * kStageBytes), &p.xmap, kc * kBK, mt * kBM,
                                    smem_u32(full + s));
                    }
                // every load issued has landed before the CTA may exit (bounded)
                for (long long q = it - (it < S ? it : S); q < it; q++) {
                    const long long start = clock64();
                    while (!mbar_try_wait(smem_u32(full + (int)(q % S)), (uint32_t)((q / S) & 1), 200000) &&
                           clock64() - start < kTimeoutCycles) {
                    }
                }
            }
        } else if (p.mode != kBand) {
            const int j = t & 7;    // 16-byte chunk of the 128-byte stage row
            const int r0 = t >> 3;  // rows r0 + kRowStep i
            const uint32_t fillw = 0x01010101u * (uint32_t)(uint8_t)p.xzp;
            const uint4 fill16 = make_uint4(fillw, fillw, fillw, fillw);
            // Each stage's copies are tracked per thread with cp.async groups; a warp signals
            // stage `it - lag` once all its lanes have seen that group land (one barrier arrival
            // per warp). The lag keeps up to lag + 1 stages of copies in flight per thread.
            const int lag = S - 1 < 3 ? S - 1 : 3;
            int pending = 0;
            for (int mt = blockIdx.x; mt < m_tiles; mt += gridDim.x) {
                const int8_t *rbase[kRowIters];
                int ry[kRowIters], rx[kRowIters];
                bool rvalid[kRowIters];
#pragma unroll
                for (int i = 0; i < kRowIters; i++) {
                    const int m = mt * kBM + r0 + kRowStep * i;
                    rvalid[i] = m < p.M;
                    const int mm = rvalid[i] ? m : 0;
                    if (p.mode == kPointwise) {
                        rbase[i] = p.x + (size_t)mm * p.ic;
                        ry[i] = rx[i] = 0;
                    } else {
                        const int n = p.f_img.div(mm), rem = mm - n * p.f_img.d;
                        const int oy = p.f_ow.div(rem), ox = rem - oy * p.ow;
                        rbase[i] = p.x + (size_t)n * p.ih * p.iw * p.ic;
                        ry[i] = oy * p.sh - p.pt;
                        rx[i] = ox * p.sw - p.pl;
                    }
                }
                bool ok = true;
                for (int kc = 0; kc < p.kc; kc++, it++) {
                    const int s = (int)(it % S);
                    if (!mbar_wait(smem_u32(empty + s), (uint32_t)(((it / S) & 1) ^ 1), abort, 101)) {
                        ok = false;
                        break;
                    }
                    const uint32_t stage = smem_u32(sA + (size_t)s * kStageBytes);
                    const int k = kc * kBK + j * 16;
                    if (k < p.K) {
                        if (p.mode == kPointwise) {
#pragma unroll
                            for (int i = 0; i < kRowIters; i++) {
                                const int r = r0 + kRowStep * i;
                                const uint32_t dst = stage + (r >> 3) * 1024 + (r & 7) * 128 + ((j ^ (r & 7)) << 4);
                                if (rvalid[i]) cp_async16(dst, rbase[i] + k);
                            }
                        } else {
                            const int tap = k / p.ic, c = k - tap * p.ic;
                            const int ky = tap / p.kw, kx = tap - ky * p.kw;
                            const int dy = ky * p.dh, dx = kx * p.dw;
#pragma unroll
                            for (int i = 0; i < kRowIters; i++) {
                                const int r = r0 + kRowStep * i;
                                const uint32_t dst = stage + (r >> 3) * 1024 + (r & 7) * 128 + ((j ^ (r & 7)) << 4);
                                if (!rvalid[i]) continue;
                                const int iy = ry[i] + dy, ix = rx[i] + dx;
                                // taps outside the image hold the zero point, stored directly: a
                                // shared global source would put every CTA's border copies on one
                                // L2 slice
                                if (iy >= 0 && ix >= 0 && iy < p.ih && ix < p.iw)
                                    cp_async16(dst, rbase[i] + ((size_t)iy * p.iw + ix) * p.ic + c);
                                else
                                    st_shared16(dst, fill16);
                            }
                        }
                    }
                    cp_async_commit();
                    if (++pending > lag) {
                        cp_async_wait_dyn(lag);
                        fence_proxy_async();
                        __syncwarp();
                        if (lane == 0) mbar_arrive(smem_u32(full + (int)((it - lag) % S)));
                        pending--;
                    }
                }
                if (!ok) break;
            }
            cp_async_wait<0>();
            fence_proxy_async();
            __syncwarp();
            if (lane == 0)
                for (long long q = it - pending; q < it; q++) mbar_arrive(smem_u32(full + (int)(q % S)));
        } else {
            // Band mode: the input rows a tile touches (its "band") sit in shared memory, each row
            // framed by margins of the input zero point, with up to nb bands in flight (fetched by
            // the loader warp); A rows are assembled from the band. Rows above or below the image
            // read a shared row of zero-point bytes instead.
            const int pitch = p.pitch, ML = p.ml;
            const uint32_t buf_bytes = (uint32_t)p.band_bytes;
            const uint32_t band0 = smem_u32(sBand), fillrow = band0 + (uint32_t)p.nbands * buf_bytes + 16;
            const uint32_t fill4 = 0x01010101u * (uint32_t)(uint8_t)p.xzp;
            {
                const uint4 f = make_uint4(fill4, fill4, fill4, fill4);
                const int data16 = p.row16, margin16 = (pitch >> 4) - data16;
                const int slots = p.nbands * p.band_rows;
                for (int q = t; q < slots * margin16; q += kProducers) {
                    const int row = q / margin16, c = q - row * margin16;
                    const int col = c < (ML >> 4) ? c * 16 : ML + data16 * 16 + (c - (ML >> 4)) * 16;
                    const int b = row / p.band_rows, r = row - b * p.band_rows;
                    st_shared16(band0 + (uint32_t)b * buf_bytes + (uint32_t)(r * pitch + col), f);
                }
                for (int q = t; q < (p.fill_bytes >> 4); q += kProducers) st_shared16(fillrow - 16 + q * 16, f);
            }
            unsigned round = 0;
            // The loader warp fetches each tile's band into buffer (tile index) % nb; the producers
            // wait for it, assemble, and release the buffer.
            const int nb = p.nbands;
            // the zero-point margins written above are read by every warp
            bool ok = role_sync(smem_u32(psync), round, abort, 109);
            int i_tile = 0;
            for (int mt = blockIdx.x; mt < m_tiles && ok; mt += gridDim.x, i_tile++) {
                const int bsel = i_tile % nb;
                const uint32_t bandb = band0 + (uint32_t)bsel * buf_bytes;
                if (!mbar_wait(smem_u32(bandfull + bsel), (uint32_t)((i_tile / nb) & 1), abort, 110)) break;
                long long g_lo;
                int rows;
                band_of(p, mt, g_lo, rows);
                if (p.ic % 16 == 0) {
                    // 16-byte chunks: thread (j = t % 8, r0 = t / 8) builds chunk j of rows r0 + kRowStep i.
                    const int j = t & 7, r0 = t >> 3;
                    int y0[kRowIters], rb[kRowIters], cb[kRowIters];
#pragma unroll
                    for (int i = 0; i < kRowIters; i++) {
                        const int m = mt * kBM + r0 + kRowStep * i;
                        const int n = p.f_img.div(m), rem = m - n * p.f_img.d;
                        const int oy = p.f_ow.div(rem), ox = rem - oy * p.ow;
                        y0[i] = m < p.M ? oy * p.sh - p.pt : -(1 << 20);  // rows past M read the fill row
                        rb[i] = (int)((long long)n * p.ih - g_lo);
                        cb[i] = ML + (ox * p.sw - p.pl) * p.ic;
                    }
                    for (int kc = 0; kc < p.kc; kc++, it++) {
                        const int s = (int)(it % S);
                        if (!mbar_wait(smem_u32(empty + s), (uint32_t)(((it / S) & 1) ^ 1), abort, 101)) {
                            ok = false;
                            break;
                        }
                        const uint32_t stage = smem_u32(sA + (size_t)s * kStageBytes);
                        const int e = sTab[kc * 8 + j];
                        if (e >= 0) {
                            const int dy = e >> 20, off = e & 0xFFFFF;
                            // all loads first: each store waits only for its own load, not in turn
                            uint4 v[kRowIters];
#pragma unroll
                            for (int i = 0; i < kRowIters; i++) {
                                const int iy = y0[i] + dy;
                                v[i] = ld_shared16((iy >= 0 && iy < p.ih)
                                                       ? bandb + (uint32_t)((rb[i] + iy) * pitch + cb[i] + off)
                                                       : fillrow + (uint32_t)off);
                            }
#pragma unroll
                            for (int i = 0; i < kRowIters; i++) {
                                const int r = r0 + kRowStep * i;
                                st_shared16(stage + (r >> 3) * 1024 + (r & 7) * 128 + ((j ^ (r & 7)) << 4), v[i]);
                            }
                        }
                        fence_proxy_async();
                        __syncwarp();
                        if (lane == 0) mbar_arrive(smem_u32(full + s));
                    }
                } else {
                    // One K stage (K <= 128); thread t builds row t % 128 word by word, chunks
                    // t / 128 + kChunkStep k. Word w takes its
                    // bytes from at most two kernel rows (runs of kw*ic contiguous band bytes):
                    // table entry {dy_a, off_a, dy_b, off_b, mask_a, mask_b}, dy = -1 for none.
                    const int s = (int)(it % S);
                    if (!mbar_wait(smem_u32(empty + s), (uint32_t)(((it / S) & 1) ^ 1), abort, 101)) break;
                    const uint32_t stage = smem_u32(sA + (size_t)s * kStageBytes);
                    const int row = t % kBM;
                    const int m = mt * kBM + row;
                    if (m < p.M) {
                        const int n = p.f_img.div(m), rem = m - n * p.f_img.d;
                        const int oy = p.f_ow.div(rem), ox = rem - oy * p.ow;
                        const int y0 = oy * p.sh - p.pt, rb = (int)((long long)n * p.ih - g_lo);
                        const int cb = ML + (ox * p.sw - p.pl) * p.ic;
                        auto run = [&](int dy) -> uint32_t {
                            const int iy = y0 + dy;
                            return (iy >= 0 && iy < p.ih) ? bandb + (uint32_t)((rb + iy) * pitch + cb) : fillrow;
                        };
                        const int4 *wt = reinterpret_cast<const int4 *>(sTab);
                        const int chunks = p.K32 >> 4;
                        for (int c = t / kBM; c < chunks; c += kChunkStep) {
                            uint32_t words[4];
#pragma unroll
                            for (int w4 = 0; w4 < 4; w4++) {
                                const int4 ea = wt[2 * (c * 4 + w4)], eb = wt[2 * (c * 4 + w4) + 1];
                                uint32_t v = 0;
                                if (ea.x >= 0) v = ld_shared_u32_unaligned(run(ea.x) + ea.y) & (uint32_t)eb.x;
                                if (ea.z >= 0) v |= ld_shared_u32_unaligned(run(ea.z) + ea.w) & (uint32_t)eb.y;
                                words[w4] = v;
                            }
                            st_shared16(stage + (row >> 3) * 1024 + (row & 7) * 128 + ((c ^ (row & 7)) << 4),
                                        make_uint4(words[0], words[1], words[2], words[3]));
                        }
                    }
                    fence_proxy_async();
                    __syncwarp();
                    if (lane == 0) mbar_arrive(smem_u32(full + s));
                    it++;
                }
                __syncwarp();
                if (!ok) break;
                if (lane == 0) mbar_arrive(smem_u32(bandfree + bsel));  // this warp is done with the band
            }
        }
        cp_async_wait<0>();
    } else if (warp == kMmaWarp) {
        // ------------------------------------------------------------------ MMA issuer
        if (lane == 0) {
            const uint32_t idesc = instr_desc(p.bn);
            const uint32_t a0 = smem_u32(sA), b0 = smem_u32(sB);
            bool ok = mbar_wait(smem_u32(bfull), 0, abort, 102);
            tc_fence_after();
            long long it = 0;
            int lt = 0;
            for (int mt = blockIdx.x; mt < m_tiles && ok; mt += gridDim.x, lt++) {
                const int acc = lt % p.n_acc;
                if (!mbar_wait(smem_u32(tempty + acc), (uint32_t)(((lt / p.n_acc) & 1) ^ 1), abort, 103)) break;
                tc_fence_after();
                const uint32_t tmem_d = tmem_base + (uint32_t)(acc * p.bn);
                for (int kc = 0; kc < p.kc; kc++, it++) {
                    const int s = (int)(it % S);
                    if (!mbar_wait(smem_u32(full + s), (uint32_t)((it / S) & 1), abort, 104)) {
                        ok = false;
                        break;
                    }
                    // the stage was written through the generic proxy (cp.async / st.shared)
                    fence_proxy_async();
                    tc_fence_after();
                    const int kbytes = min(kBK, ((p.K + 31) & ~31) - kc * kBK);
                    for (int kk = 0; kk < kbytes / 32; kk++) {
                        const uint64_t ad = smem_desc(a0 + (uint32_t)(s * kStageBytes + kk * 32));
                        const uint64_t bd = smem_desc(b0 + (uint32_t)(kc * p.bn * kBK + kk * 32));
                        mma_i8(tmem_d, ad, bd, idesc, (kc | kk) ? 1u : 0u);
                    }
                    mma_commit(smem_u32(empty + s));
                }
                if (!ok) break;
                // p.withhold (tests of the bounded waits): the epilogue of this CTA's first tile is
                // never released, so its wait runs out and every role leaves by its abort path
                if (!(p.withhold && lt == 0 && blockIdx.x == 0 && blockIdx.y == 0)) mma_commit(smem_u32(tfull + acc));
            }
            // All MMAs are issued: the next kernel's CTAs may be scheduled once every CTA is here
            // (earlier, they would sit beside this CTA for its whole run, taking issue slots).
            grid_dep_launch();
            // Drain: every MMA this thread issued has completed before TMEM can be freed,
            // including on the abort path.
            mma_commit(smem_u32(drain));
            const long long start = clock64();
            while (!mbar_try_wait(smem_u32(drain), 0, 200000) && clock64() - start < kTimeoutCycles) {
            }
        }
        __syncwarp();
    } else if (R::kLoader && warp == R::kLoaderWarp) {
        // ------------------------------------------------------------------ band loader
        // One thread fetches the band of this CTA's tile f into buffer f % nb, one bulk copy per
        // input row into its slot between the zero-point margins, once the producers have released
        // that buffer's previous band (tile f - nb). The copies complete their bytes on the buffer's
        // band-full barrier. A warp of its own, so the assembling producer warps stay in step.
        if (lane == 0 && p.mode == kBand) {
            const int nb = p.nbands;
            const int my_tiles = blockIdx.x < m_tiles ? (m_tiles - 1 - blockIdx.x) / gridDim.x + 1 : 0;
            const long long row_bytes = (long long)p.iw * p.ic;
            const uint32_t band0 = smem_u32(sBand), buf_bytes = (uint32_t)p.band_bytes;
            int f = 0;
            for (; f < my_tiles; f++) {
                const int b = f % nb;
                if (f >= nb && !mbar_wait(smem_u32(bandfree + b), (uint32_t)((f / nb - 1) & 1), abort, 106)) break;
                long long g_lo;
                int rows;
                band_of(p, blockIdx.x + f * gridDim.x, g_lo, rows);
                const uint8_t *src = reinterpret_cast<const uint8_t *>(p.x) + g_lo * row_bytes;
                const uint32_t dst = band0 + (uint32_t)b * buf_bytes + (uint32_t)p.ml;
                const uint32_t bar = smem_u32(bandfull + b);
                mbar_expect_tx(bar, (uint32_t)(rows * row_bytes));
                for (int r = 0; r < rows; r++)
                    bulk_load(dst + (uint32_t)(r * p.pitch), src + r * row_bytes, (uint32_t)row_bytes, bar);
            }
            // every band issued has landed before the CTA may exit (bounded)
            for (int q = f - (f < nb ? f : nb); q < f; q++) {
                const long long start = clock64();
                while (!mbar_try_wait(smem_u32(bandfull + q % nb), (uint32_t)((q / nb) & 1), 200000) &&
                       clock64() - start < kTimeoutCycles) {
                }
            }
        }
        __syncwarp();
    } else {
        // ------------------------------------------------------------------ epilogue
        const int e = warp - kProducerWarps;
        const int et = threadIdx.x - kProducers;  // 0..kEpilogues-1
        const int quarter = warp & 3;             // TMEM lanes 32*quarter .. +31 (warp id % 4 rule)
        const int half = e >> 2;                  // which column part of the tile this warp takes
        const int row = quarter * 32 + lane;
        const uint8_t *lut = p.post ? sLut : nullptr;
        const int n0 = ntile * p.bn;
        const int cols = min(p.bn, p.oc - n0);
        const int live_chunks = (cols + 15) / 16;
        const int vw = (p.oc & 15) == 0 ? 16 : (p.oc & 7) == 0 ? 8 : (p.oc & 3) == 0 ? 4 : 1;
        unsigned round = 0;
        int lt = 0;
        if (p.store_tma) {
            // Each warp owns rows 32*quarter.. and one column part [c0, c0 + box) of every fold-th
            // tile (phase ph): it stages them in its own double buffer (swizzled like the box) and
            // stores them with its own TMA store, so no epilogue warp ever waits for another. When a
            // tile has fewer column parts than warps per lane quarter (narrow N tiles), the spare
            // warps take the following tiles of the accumulator ring instead of idling.
            const int nparts = kParts / p.fold;
            const int c0 = (half % nparts) * p.box, ph = half / nparts;
            const int my_chunks = c0 < cols ? (min(p.box, cols - c0) + 15) / 16 : 0;
            const int swz_row = p.swz == 3 ? (lane & 7) : p.swz == 2 ? ((lane >> 1) & 3) : p.swz == 1 ? ((lane >> 2) & 1) : 0;
            const size_t wsb = warp_stage_bytes(p.box);
            uint8_t *wstage0 = sOut + (size_t)e * 2 * wsb;
            int k = 0;  // tiles this warp has staged
            lt = ph;
            for (int mt = blockIdx.x + ph * gridDim.x; mt < m_tiles; mt += p.fold * gridDim.x, lt += p.fold, k++) {
                const int acc = lt % p.n_acc;
                if (!mbar_wait(smem_u32(tfull + acc), (uint32_t)((lt / p.n_acc) & 1), abort, 105)) break;
                tc_fence_after();
                uint8_t *stage = wstage0 + (size_t)(k & 1) * wsb;
                // this buffer's previous store (two tiles back) must have been read out
                if (lane == 0) asm volatile("cp.async.bulk.wait_group.read 1;" ::: "memory");
                __syncwarp();
                const uint32_t taddr = tmem_base + ((uint32_t)(quarter * 32) << 16) + (uint32_t)(acc * p.bn + c0);
                uint32_t ra[16], rb[16];
                if (my_chunks > 0) {
                    tmem_ld16_nowait(taddr, ra);
                    tmem_wait_ld(ra);
                }
                for (int ci = 0; ci < my_chunks; ci++) {
                    const bool more = ci + 1 < my_chunks;
                    if (more) tmem_ld16_nowait(taddr + (ci + 1) * 16, rb);
                    uint4 v;
                    if (p.res) {
                        const int row = mt * kBM + quarter * 32 + lane;
                        uint4 rr = make_uint4(0, 0, 0, 0);  // rows past M read no residual (never stored)
                        if (row < p.M)
                            rr = __ldg(reinterpret_cast<const uint4 *>(p.res + (size_t)row * p.oc + n0 + c0 + ci * 16));
                        v = epilogue_chunk<EPI>(ra, E, lut, c0 + ci * 16, p.lo, p.hi, &p.add, sAdd, rr);
                    } else {
                        v = epilogue_chunk<EPI>(ra, E, lut, c0 + ci * 16, p.lo, p.hi);
                    }
                    st_shared16(smem_u32(stage + (size_t)lane * p.box + ((ci ^ swz_row) << 4)), v);
                    if (more) tmem_wait_ld(rb);
#pragma unroll
                    for (int q = 0; q < 16; q++) ra[q] = rb[q];
                }
                tc_fence_before();
                fence_proxy_async();  // staged bytes visible to the TMA (async proxy)
                __syncwarp();
                if (lane == 0) {
                    mbar_arrive(smem_u32(tempty + acc));  // accumulator free for reuse
                    const int r0 = mt * kBM + quarter * 32;
                    if (my_chunks > 0 && r0 < p.M)
                        asm volatile(
                            "cp.async.bulk.tensor.2d.global.shared::cta.bulk_group [%0, {%2, %3}], [%1];" ::"l"(
                                reinterpret_cast<uint64_t>(&p.ymap)),
                            "r"(smem_u32(stage)), "r"(n0 + c0), "r"(r0)
                            : "memory");
                    asm volatile("cp.async.bulk.commit_group;" ::: "memory");
                }
            }
            if (lane == 0) asm volatile("cp.async.bulk.wait_group 0;" ::: "memory");
        } else {
            for (int mt = blockIdx.x; mt < m_tiles; mt += gridDim.x, lt++) {
                const int acc = lt % p.n_acc;
                if (!mbar_wait(smem_u32(tfull + acc), (uint32_t)((lt / p.n_acc) & 1), abort, 105)) break;
                tc_fence_after();
                uint8_t *stage = sOut + (size_t)(lt & 1) * out_stride(p.bn);
                const uint32_t taddr = tmem_base + ((uint32_t)(quarter * 32) << 16) + (uint32_t)(acc * p.bn);
                uint32_t ra[16], rb[16];
                int ci = half;  // chunks half, half + kParts, ...
                if (ci < live_chunks) {
                    tmem_ld16_nowait(taddr + ci * 16, ra);
                    tmem_wait_ld(ra);
                }
                while (ci < live_chunks) {
                    const int next = ci + kParts;
                    if (next < live_chunks) tmem_ld16_nowait(taddr + next * 16, rb);
                    const uint4 v = epilogue_chunk<EPI>(ra, E, lut, ci * 16, p.lo, p.hi);
                    st_shared16(smem_u32(stage + (size_t)row * (p.bn + 16) + ci * 16), v);
                    if (next < live_chunks) tmem_wait_ld(rb);
#pragma unroll
                    for (int q = 0; q < 16; q++) ra[q] = rb[q];
                    ci = next;
                }
                tc_fence_before();
                __syncwarp();
                if (lane == 0) mbar_arrive(smem_u32(tempty + acc));  // accumulator free for reuse
                const int m0 = mt * kBM;
                if (!role_sync(smem_u32(esync), round, abort, 108)) break;  // tile staged by all threads
                // cooperative coalesced copy-out of the staged tile: rows m0.., columns n0..n0+cols
                const int rows = min(kBM, p.M - m0);
                const int cpr = cols / vw;
                const int total = rows * cpr;
                int8_t *ybase = p.y + (size_t)m0 * p.oc + n0;
                for (int q = et; q < total; q += kEpilogues) {
                    const int rr = q / cpr, cc = (q - rr * cpr) * vw;
                    const uint8_t *src = stage + (size_t)rr * (p.bn + 16) + cc;
                    int8_t *dst = ybase + (size_t)rr * p.oc + cc;
                    if (vw == 16) *reinterpret_cast<uint4 *>(dst) = *reinterpret_cast<const uint4 *>(src);
                    else if (vw == 8) *reinterpret_cast<uint2 *>(dst) = *reinterpret_cast<const uint2 *>(src);
                    else if (vw == 4) *reinterpret_cast<uint32_t *>(dst) = *reinterpret_cast<const uint32_t *>(src);
                    else *dst = (int8_t)*src;
                }
            }
        }
    }

    tc_fence_before();
    __syncthreads();
    tc_fence_after();
    if (warp == kMmaWarp) {
        asm volatile("tcgen05.dealloc.cta_group::1.sync.aligned.b32 %0, %1;" ::"r"(tmem_base), "r"(p.tmem_cols));
    }
}

}  // namespace

struct ConvTc {
    Params p{};
    int sm_count = 148;  // of the device the op was prepared on
    int n_tiles = 1;
    size_t smem = 0;
    int producer_warps = 8;
    int epilogue_warps = 8;
    bool fused = false;  // a residual add is fused into the epilogue
};

// Band geometry of a layer. Each band row holds one input row (iw*ic bytes, a multiple of 16 so
// rows copy as whole 16-byte chunks) between margins of the input zero point wide enough for every
// tap left / right of the image plus the few bytes a word read may run over; rows = the most input
// rows any 128-pixel tile touches (the pattern repeats every lcm(128, oh*ow) pixels).
struct BandGeom {
    int rows = 0, pitch = 0, ml = 0, fill_bytes = 0;
    long long bytes() const { return (long long)rows * pitch; }
};

static long long round16(long long v) { return (v + 15) & ~15ll; }

static bool band_geometry(const ConvGeom &g, BandGeom &bg) {
    const long long row_bytes = (long long)g.iw * g.ic;
    if (row_bytes % 16 != 0) return false;
    if (g.ic % 16 != 0 && g.dw != 1) return false;  // word assembly needs contiguous kx runs
    const long long x0_max = (long long)(g.ow - 1) * g.sw - g.pl;
    const long long over = std::max<long long>(0, (x0_max + (long long)(g.kw - 1) * g.dw + 1 - g.iw) * g.ic);
    const long long ml = round16((long long)g.pl * g.ic + 8), mr = round16(over + 16);
    const long long pitch = ml + row_bytes + mr;
    const long long span = ((long long)(g.kw - 1) * g.dw + 1) * g.ic;
    const long long img = (long long)g.oh * g.ow;
    const long long period = img / std::gcd(img, (long long)kBM) * kBM;
    long long rows = 0;
    for (long long m0 = 0; m0 < period; m0 += kBM) {
        const long long m1 = m0 + kBM - 1;
        const long long n0 = m0 / img, oy0 = (m0 / g.ow) % g.oh, n1 = m1 / img, oy1 = (m1 / g.ow) % g.oh;
        const long long lo = n0 * g.ih + std::max<long long>(0, oy0 * g.sh - g.pt);
        const long long hi =
            n1 * g.ih + std::max<long long>(-1, std::min<long long>(g.ih - 1, oy1 * g.sh - g.pt + (long long)(g.kh - 1) * g.dh));
        rows = std::max(rows, hi - lo + 1);
    }
    if (rows * pitch > 64 * 1024 || pitch > (1 << 20) || (long long)(g.kh - 1) * g.dh >= 2048) return false;
    bg.rows = (int)std::max<long long>(rows, 1);
    bg.pitch = (int)pitch;
    bg.ml = (int)ml;
    bg.fill_bytes = (int)round16(16 + span + 16);
    return true;
}

int conv_tc_prepare(const int8_t *w_packed, const int32_t *q, const uint8_t *post_dev, const ConvGeom &g,
                    const std::function<void *(size_t)> &alloc, ConvTc **out, const FusedAdd *add) {
    *out = nullptr;
    if (add && (g.oc % 16 != 0)) return 0;  // fused add needs whole 16-byte column chunks (TMA store)
    const char *env = std::getenv("UNOQ_CONV_TC");
    if (env && env[0] == '0') return 0;
    const int K = g.kh * g.kw * g.ic;
    const int K32 = (K + 31) & ~31;
    const int kc = (K32 + kBK - 1) / kBK;
    int mode = kGather16;
    if (g.kh == 1 && g.kw == 1 && g.sh == 1 && g.sw == 1 && g.pt == 0 && g.pl == 0 && g.ih == g.oh && g.iw == g.ow &&
        g.ic % 16 == 0)
        mode = kPointwise;
    BandGeom bg;
    if (mode != kPointwise && (g.ic % 16 == 0 || kc == 1) && band_geometry(g, bg)) mode = kBand;
    if (mode == kGather16 && g.ic % 16 != 0) return 0;
    // epilogue warps: 16 for pointwise convs (4 producer warps leave room; more warps hide the
    // epilogue's latency), 8 for the other modes (8 producer warps)
    const int ew = mode == kPointwise ? 16 : 8;
    // N tiling: the fewest tiles of equal width (at most 256) that cover oc, each tile's weights
    // resident in shared memory. The width is a multiple of 16 columns per epilogue part (see
    // nparts below), so that no part's store box reaches into the next tile: 192 channels are one
    // 192-wide tile and 576 three, where power-of-two widths would leave a quarter idle.
    int n_tiles = (g.oc + 255) / 256, bn = 16;
    for (;; n_tiles++) {
        bn = std::max(16, ((g.oc + n_tiles - 1) / n_tiles + 15) & ~15);
        const int align = bn > 128 && ew == 16 ? 64 : bn > 64 ? 32 : 16;
        bn = (bn + align - 1) / align * align;
        if ((size_t)kc * bn * kBK <= (size_t)kWeightBudget) break;
        if (bn == 16) return 0;
    }
    // Band table: per 16-byte chunk (ic % 16 == 0) one int, else per 4-byte word eight ints.
    const int tab_bytes = mode != kBand ? 16 : g.ic % 16 == 0 ? kc * 8 * 4 : (K32 / 4) * 32;
    int stages = 8, nbands = 0;
    const bool store_tma = (g.oc % 16) == 0;
    // column parts per tile (1, 2 or ew / 4 warps of each lane quarter): the fewest that keep a part
    // within 64 columns, so narrow N tiles leave spare warps to take other tiles (see fold) and pay
    // fewer per-warp, per-tile fixed costs. Parts are equal (bn / nparts, a multiple of 16 by the
    // choice of bn); a 32 / 64 / 128-byte part is stored swizzled, others unswizzled, whose odd
    // 16-byte multiples (48, 80, 112) still put the lanes of a 16-byte store in distinct banks.
    int nparts = 1;
    while (nparts < ew / 4 && bn / nparts > 64) nparts *= 2;
    const int box = bn / nparts;
    if (box % 16 != 0) return 0;
    const int out_bytes = store_tma ? (int)(2 * ew * warp_stage_bytes(box)) : (int)(2 * out_stride(bn));
    auto layout = [&]() {
        return Layout(stages, kc, bn, mode == kBand ? (int)bg.bytes() : 0, nbands, mode == kBand ? bg.fill_bytes : 0,
                      tab_bytes, out_bytes);
    };
    if (mode == kBand) {
        nbands = 3;
        while (stages > 4 && layout().total > (size_t)kMaxSmem) stages--;
        while (nbands > 2 && layout().total > (size_t)kMaxSmem) nbands--;
        while (stages > 2 && layout().total > (size_t)kMaxSmem) stages--;
        if (layout().total > (size_t)kMaxSmem) {
            if (g.ic % 16 != 0) return 0;
            mode = kGather16;
            nbands = 0;
            stages = 8;
        }
    }
    while (stages > 2 && layout().total > (size_t)kMaxSmem) stages--;
    if (layout().total > (size_t)kMaxSmem) return 0;

    // Weights: reference packed layout (gemm.h:9) -> per N tile, per K stage, UMMA SW128 K-major.
    const int kp = q[18];
    const int oc = g.oc;
    std::vector<uint8_t> wt((size_t)n_tiles * kc * bn * kBK, 0);
    std::vector<EpiChan> epi((size_t)n_tiles * bn);
    auto wref = [&](int j, int t) -> int { return w_packed[(j / 4) * kp * 4 + (t / 8) * 32 + (j % 4) * 8 + t % 8]; };
    const int32_t *cbias = q + kHead, *mult = cbias + oc, *shift = mult + oc;
    const int xzp = q[12], yzp = q[13];
    for (int nt = 0; nt < n_tiles; nt++)
        for (int r = 0; r < bn; r++) {
            const int j = nt * bn + r;
            if (j >= oc) {
                epi[(size_t)nt * bn + r] = make_epilogue(0, 0, 0, 0);
                continue;
            }
            long long sum_all = 0, sum_pad = 0;
            for (int t = 0; t < kp; t++) {
                const int v = wref(j, t);
                sum_all += v;
                if (t >= K) sum_pad += v;
                if (t < K) {
                    const int c = t / kBK, byte = t % kBK, chunk = byte / 16;
                    const size_t off = ((size_t)(nt * kc + c) * bn + (r / 8) * 8) * kBK + (r % 8) * kBK +
                                       ((chunk ^ (r % 8)) * 16) + byte % 16;
                    wt[off] = (uint8_t)(int8_t)v;
                }
            }
            const long long bias = (long long)cbias[j] + 128ll * sum_all + (long long)xzp * sum_pad;
            epi[(size_t)nt * bn + r] = make_epilogue(bias, mult[j], shift[j], yzp);
        }
    // Epilogue mode (see EpiMode): the fast forms need every live channel in the short form.
    bool fast = true;
    for (int j = 0; j < oc; j++) fast &= epi_fast(epi[j]);  // channel j sits at nt * bn + r = j
    const int epi_mode = !fast ? kGeneral : (q[14] >= yzp ? kRelu : kTies);
    if (epi_mode != kGeneral)
        for (auto &e : epi) e.sh = e.sh >= 32 ? e.sh - 32 : 0;  // shift of the high word
    std::vector<int> tab(tab_bytes / 4, 0);
    if (mode == kBand && g.ic % 16 == 0) {
        // chunk j = reduction bytes [16 j, 16 j + 16): (ky*dh) << 20 | byte offset in the kernel-row
        // run (kx*dw*ic + c); -1 past K (its weights are zero, the A bytes are left as they are)
        for (int j = 0; j < kc * 8; j++) {
            const int t0 = j * 16;
            if (t0 >= K) {
                tab[j] = -1;
                continue;
            }
            const int tap = t0 / g.ic, c = t0 % g.ic, ky = tap / g.kw, kx = tap % g.kw;
            tab[j] = (ky * g.dh) << 20 | (kx * g.dw * g.ic + c);
        }
    } else if (mode == kBand) {
        // word w = reduction bytes [4 w, 4 w + 4); kernel row ky contributes bytes [ky*L, ky*L + L) of
        // the row, L = kw*ic, read from the run that starts at that tap row's first column.
        const int L = g.kw * g.ic;
        for (int w = 0; w < K32 / 4; w++) {
            int *e = &tab[(size_t)w * 8];
            e[0] = e[2] = -1;
            for (int b = 0; b < 4; b++) {
                const int q = 4 * w + b;
                if (q >= K) continue;
                const int ky = q / L;
                if (e[0] < 0 || ky * g.dh == e[0]) {
                    if (e[0] < 0) e[0] = ky * g.dh, e[1] = 4 * w - ky * L;
                    e[4] |= (int)(0xFFu << (8 * b));
                } else {
                    if (e[2] < 0) e[2] = ky * g.dh, e[3] = 4 * w - ky * L;
                    e[5] |= (int)(0xFFu << (8 * b));
                }
            }
        }
    }
    void *dw = alloc(wt.size());
    void *de = alloc(epi.size() * sizeof(EpiChan));
    void *dt = alloc(tab.size() * sizeof(int));
    if (!dw || !de || !dt) return 2001;
    if (cudaMemcpy(dw, wt.data(), wt.size(), cudaMemcpyHostToDevice) != cudaSuccess ||
        cudaMemcpy(de, epi.data(), epi.size() * sizeof(EpiChan), cudaMemcpyHostToDevice) != cudaSuccess ||
        cudaMemcpy(dt, tab.data(), tab.size() * sizeof(int), cudaMemcpyHostToDevice) != cudaSuccess)
        return 2001;
    const bool attrs = once_per_device(kFamilyConvTc, [] {
        auto allow = [](auto fn) {
            return cudaFuncSetAttribute(fn, cudaFuncAttributeMaxDynamicSharedMemorySize, kMaxSmem) == cudaSuccess;
        };
        return allow(conv_tc_kernel<kRelu, 4, 8>) && allow(conv_tc_kernel<kTies, 4, 8>) &&
               allow(conv_tc_kernel<kGeneral, 4, 8>) && allow(conv_tc_kernel<kRelu, 8, 8>) &&
               allow(conv_tc_kernel<kTies, 8, 8>) && allow(conv_tc_kernel<kGeneral, 8, 8>) &&
               allow(conv_tc_kernel<kRelu, 4, 16>) && allow(conv_tc_kernel<kTies, 4, 16>) &&
               allow(conv_tc_kernel<kGeneral, 4, 16>);
    });
    if (!attrs) return 2001;
    ConvTc *c = new ConvTc();
    c->sm_count = current_sm_count();
    Params &p = c->p;
    p.w = static_cast<const int8_t *>(dw);
    p.epi = static_cast<const EpiChan *>(de);
    p.post = post_dev;
    p.tab = static_cast<const int *>(dt);
    p.ih = g.ih, p.iw = g.iw, p.ic = g.ic, p.oh = g.oh, p.ow = g.ow, p.oc = g.oc;
    p.f_ow = FastDiv(g.ow);
    p.f_img = FastDiv(g.oh * g.ow);
    p.kh = g.kh, p.kw = g.kw, p.sh = g.sh, p.sw = g.sw, p.dh = g.dh, p.dw = g.dw, p.pt = g.pt, p.pl = g.pl;
    p.K = K;
    p.kc = kc;
    p.bn = bn;
    p.stages = stages;
    p.lo = q[14], p.hi = q[15];
    p.xzp = xzp;
    p.n_acc = bn <= 128 ? 4 : 2;
    p.tmem_cols = 32;  // a power of two (tcgen05.alloc)
    while (p.tmem_cols < p.n_acc * bn) p.tmem_cols *= 2;
    p.store_tma = store_tma;
    if (add) {
        p.add_tab = add->q_dev;
        p.res_side = add->conv_is_b ? 1 : 0;
        p.add.epi = make_epilogue(0, add->q_host[0], add->q_host[1], add->q_host[2]);
        p.add.lo = add->q_host[3];
        p.add.hi = add->q_host[4];
        c->fused = true;
    }
    p.box = box;
    // narrow N tiles: spare epilogue warps of each lane quarter take alternate tiles; the kernel
    // splits each quarter's ew / 4 warps into (ew / 4) / fold column parts x fold tile phases
    p.fold = store_tma ? (ew / 4) / nparts : 1;
    p.out_bytes = out_bytes;
    p.swz = p.box == 128 ? 3 : p.box == 64 ? 2 : p.box == 32 ? 1 : 0;
    p.mode = mode;
    {
        // pointwise A tiles by TMA unless switched off (UNOQ_CONV_TC_ATMA=0: per-thread cp.async)
        const char *ea = std::getenv("UNOQ_CONV_TC_ATMA");
        p.a_tma = mode == kPointwise && !(ea && ea[0] == '0');
        // test-only fault injection for the bounded device waits (UNOQ_FAULT_WITHHOLD_COMMIT=1): the
        // launch then takes about 2 s, records a timeout and the run returns 2003
        const char *fw = std::getenv("UNOQ_FAULT_WITHHOLD_COMMIT");
        p.withhold = fw && fw[0] == '1';
    }
    p.band_bytes = mode == kBand ? (int)bg.bytes() : 0;
    p.nbands = nbands;
    p.band_rows = bg.rows;
    p.pitch = bg.pitch;
    p.ml = bg.ml;
    p.row16 = (int)((long long)g.iw * g.ic / 16);
    p.fill_bytes = mode == kBand ? bg.fill_bytes : 0;
    p.K32 = K32;
    p.tab_bytes = tab_bytes;
    p.epi_mode = epi_mode;
    c->n_tiles = n_tiles;
    c->producer_warps = mode == kPointwise ? 4 : 8;
    c->epilogue_warps = ew;
    c->smem = layout().total;
    *out = c;
    return 0;
}

int conv_tc_launch(const ConvTc &c, const int8_t *x, int8_t *y, const ConvGeom &g, cudaStream_t s,
                   const int8_t *res) {
    Params p = c.p;
    p.x = x;
    p.y = y;
    p.res = c.fused ? res : nullptr;
    if (c.fused && !res) return 2001;
    if ((long long)g.n * g.oh * g.ow >= (1ll << 31)) return 2001;  // pixel indices are 31-bit
    p.M = g.n * g.oh * g.ow;
    if (p.store_tma) {
        // Output tensor [M][oc] int8; the box is one staged sub-tile, swizzled like the staging.
        EncodeTiled enc = encoder();
        if (!enc) return 2001;
        const cuuint64_t dims[2] = {(cuuint64_t)g.oc, (cuuint64_t)p.M};
        const cuuint64_t strides[1] = {(cuuint64_t)g.oc};
        const cuuint32_t box[2] = {(cuuint32_t)p.box, 32};
        const cuuint32_t estr[2] = {1, 1};
        const CUtensorMapSwizzle sw = p.swz == 3   ? CU_TENSOR_MAP_SWIZZLE_128B
                                      : p.swz == 2 ? CU_TENSOR_MAP_SWIZZLE_64B
                                      : p.swz == 1 ? CU_TENSOR_MAP_SWIZZLE_32B
                                                   : CU_TENSOR_MAP_SWIZZLE_NONE;
        if (enc(&p.ymap, CU_TENSOR_MAP_DATA_TYPE_UINT8, 2, y, dims, strides, box, estr, CU_TENSOR_MAP_INTERLEAVE_NONE, sw,
                CU_TENSOR_MAP_L2_PROMOTION_NONE, CU_TENSOR_MAP_FLOAT_OOB_FILL_NONE) != CUDA_SUCCESS)
            return 2001;
    }
    if (p.a_tma) {
        // Input [M][ic] int8. The box is one A stage: 128 reduction bytes x 128 pixels; its x
        // coordinate (a multiple of 128) meets the 16-byte rule of tiled TMA loads.
        EncodeTiled enc = encoder();
        if (!enc || (reinterpret_cast<uintptr_t>(x) & 15) != 0) return 2001;
        const cuuint64_t dims[2] = {(cuuint64_t)g.ic, (cuuint64_t)p.M};
        const cuuint64_t strides[1] = {(cuuint64_t)g.ic};
        const cuuint32_t box[2] = {(cuuint32_t)kBK, (cuuint32_t)kBM};
        const cuuint32_t estr[2] = {1, 1};
        if (enc(&p.xmap, CU_TENSOR_MAP_DATA_TYPE_UINT8, 2, const_cast<int8_t *>(x), dims, strides, box, estr,
                CU_TENSOR_MAP_INTERLEAVE_NONE, CU_TENSOR_MAP_SWIZZLE_128B, CU_TENSOR_MAP_L2_PROMOTION_L2_128B,
                CU_TENSOR_MAP_FLOAT_OOB_FILL_NONE) != CUDA_SUCCESS)
            return 2001;
    }
    p.x_bytes = (long long)g.n * g.ih * g.iw * g.ic;
    const int m_tiles = (p.M + kBM - 1) / kBM;
    // CTAs per N tile: floor, so that all n_tiles * per_tile CTAs are resident at once (one per SM).
    // Rounding up would start the extra CTAs only after a first wave had finished, and the static
    // tile schedule would make them run a full share of tiles on their own.
    int per_tile = c.sm_count / c.n_tiles;
    if (per_tile < 1) per_tile = 1;
    if (per_tile > m_tiles) per_tile = m_tiles;
    dim3 grid(per_tile, c.n_tiles);
    auto go = [&](auto pw, auto ew) {
        constexpr int PWv = decltype(pw)::value, EWv = decltype(ew)::value;
        constexpr int T = Roles<PWv, EWv>::kThreads;
        if (p.epi_mode == kRelu) launch_pdl(kPdlConvTc, conv_tc_kernel<kRelu, PWv, EWv>, grid, T, c.smem, s, p);
        else if (p.epi_mode == kTies) launch_pdl(kPdlConvTc, conv_tc_kernel<kTies, PWv, EWv>, grid, T, c.smem, s, p);
        else launch_pdl(kPdlConvTc, conv_tc_kernel<kGeneral, PWv, EWv>, grid, T, c.smem, s, p);
    };
    if (c.producer_warps == 4 && c.epilogue_warps == 16) go(std::integral_constant<int, 4>{}, std::integral_constant<int, 16>{});
    else if (c.producer_warps == 4) go(std::integral_constant<int, 4>{}, std::integral_constant<int, 8>{});
    else go(std::integral_constant<int, 8>{}, std::integral_constant<int, 8>{});
    return 0;
}

void conv_tc_free(ConvTc *c) { delete c; }

int conv_tc_error(bool reset) {
    int v = 0;
    cudaMemcpyFromSymbol(&v, g_tc_error, sizeof(int));
    if (reset && v) {
        int z = 0;
        cudaMemcpyToSymbol(g_tc_error, &z, sizeof(int));
    }
    return v;
}

}  // namespace uq
