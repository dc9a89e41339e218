// dw_tc.cu -- depthwise convolution (plan code 15) on the 5th-generation tensor cores.
//
// Reference semantics (runtime/qnn.c:807-983, 1228-1245; depthwise5.h): per channel
// acc = bias + sum over taps (x + 128) * w with taps outside the image reading the input zero
// point, then y = post[clamp(scale(acc, m, s) + yzp)]. The +128 is folded into the bias on the
// host (bias' = bias + 128 * sum w), so the device accumulates signed x * w.
//
// A depthwise conv is C independent one-channel convolutions; on a slice of cw channels it is a
// dense conv whose weights are block diagonal. For a tile of output pixels and one tap (ky, kx)
// the products x[pixel + tap][c] * w[c][tap] of 32 channels are one MMA of M = 128 pixels, N = 32
// channels, K = 32 channels against a 32 x 32 diagonal block: D[:, 32k..32k+31] += A_tap * B_tap,k.
// The tensor core does 32x the useful multiplies. Measured on B200 this does not pay: an MMA of
// M = 128, N = 32, K = 32 holds the tensor pipe for about 96 cycles, and a layer needs
// taps x C / 32 of them per 128 pixels, so 5x5 layers ran 2.5-4x and 3x3 layers 1.5-2x slower
// than the dp4a kernel (k_dw.cu), with the producer and epilogue alone already as slow as that
// kernel. The path is therefore off by default (UNOQ_DW_TC=1 selects it) and kept bit-exact
// under test as the tensor-core formulation of code 15.
//
// Window layout. The input rows a tile needs (its window: tr output rows plus the kernel's halo,
// wp = ow + halo columns) sit in shared memory as "chunk planes": plane[16-channel chunk][pixel][16 B]
// with pixel = v * wp + u. In that layout 8 consecutive pixels of one chunk are one 128-byte UMMA
// core matrix (K-major, no swizzle; K-adjacent core matrices one chunk plane apart, M-adjacent
// ones 128 bytes apart), so the A operand of tap (ky, kx) is the same buffer read from pixel offset
// ky * wp + kx: output pixel m = r * wp + c (c < ow; the columns c >= ow are computed and dropped)
// reads window pixel m + ky * wp + kx. No im2col, no per-tap copies. Stride 2 uses four phase
// planes (even / odd input rows x columns), so every tap is again a whole-row offset: tap
// (2a + py, 2b + px) reads phase plane (py, px) at a * wp + b. When a whole image fits a tile
// twice, two images share it (image slots `slot` pixels apart).
//
// Loading: four producer warps copy the window with 16-byte cp.async (lanes over the chunks of a
// pixel, so each warp reads whole runs of a pixel's channels) and store the input zero point into
// the window pixels outside the image (the reference's padding value), so the MMA sees exactly the
// reference's padded input and the epilogue needs no correction. (TMA boxes with 16-byte rows,
// the layout's natural TMA form, ran at about 6 bytes per cycle per SM: 3-5x slower overall.)
//
// Roles (one persistent CTA per SM on one channel slice): warps 0-3 load windows, warp 4 issues
// the MMAs into a ring of TMEM accumulators, warps 5..20 requantise (the exact epilogue shared
// with the dense convs) and store each valid pixel's channels with 16-byte stores. Every wait is
// bounded (about 2 s); on expiry the kernel records a site code, waits for its copies and MMAs,
// frees its TMEM and exits.
#include <algorithm>
#include <cstdlib>
#include <vector>

#include "device_state.hpp"
#include "dw_tc.cuh"
#include "plan.hpp"
#include "tc_common.cuh"

namespace uq {

namespace {

constexpr int kDwMaxSmem = 227 * 1024;
constexpr int kDwPW = 4;       // producer warps
constexpr int kDwMmaWarp = kDwPW;
constexpr int kDwEW = 16;      // epilogue warps
constexpr int kDwThreads = (kDwPW + 1 + kDwEW) * 32;
constexpr int kDwMaxAcc = 8;   // TMEM accumulators in rotation (at most)

struct DwTcParams {
    const int8_t *x;
    int8_t *y;
    const uint8_t *wd;      // [slice][tap][cw / 32][2 chunks][32 rows][16 B] diagonal blocks
    const EpiChan *epi;     // [C]
    const uint8_t *post;    // 256 bytes or null
    int n, ih, iw, c, oh, ow;
    int k, s, lo, hi, xzp;
    int cw, lchunks;        // channels per slice (32, 64 or 128); log2(cw / 16)
    int wp, wrows;          // window width (pixels) and rows per phase plane
    int tr;                 // output rows per tile
    int ipt, slot;          // images per tile, window pixels per image slot (multiple of 8)
    int row_tiles, tiles;   // tiles per image, tiles per slice
    int npix;               // pixels per chunk plane (window slots + read margin, multiple of 8)
    int planes;             // 1 (stride 1) or 4 (stride 2)
    int rowoff[4], coloff[4];  // per plane: input row = s * (r0 + v) + rowoff, column = s * u + coloff
    int stages, nparts, fold, n_acc, acc_shift, tmem_cols;
    int stage_bytes;
    FastDiv f_row, f_wrows, f_ipt;  // by wp * chunks (items per window row), wrows, ipt
};

struct DwLayout {
    size_t a, b, epi, lut, taps_off, bars, total;
    __host__ __device__ DwLayout(int stages, int stage_bytes, int taps, int cw) {
        size_t o = 0;
        a = o;
        o += (size_t)stages * stage_bytes;
        b = (o + 1023) & ~(size_t)1023;
        o = b + (size_t)taps * (cw / 32) * 1024;
        epi = (o + 31) & ~(size_t)31;
        o = epi + (size_t)cw * sizeof(EpiChan);
        lut = o;
        o += 256;
        taps_off = o;
        o += 32 * 4;  // per tap: A operand offset in 16-byte units (phase plane and pixel offset)
        bars = (o + 7) & ~(size_t)7;
        o = bars + (size_t)(2 * stages + 2 * kDwMaxAcc + 1) * 8 + 16;
        total = o + 1024;  // base alignment slack
    }
};

// UMMA shared-memory descriptor, K-major without swizzle: 8-row x 16-byte core matrices stored
// contiguously, `lbo` bytes between core matrices adjacent in K, `sbo` bytes between core matrices
// adjacent in M (or N).
__device__ __forceinline__ uint64_t desc_noswz(uint32_t addr, uint32_t lbo, uint32_t sbo) {
    return (uint64_t)((addr >> 4) & 0x3FFF) | ((uint64_t)((lbo >> 4) & 0x3FFF) << 16) |
           ((uint64_t)((sbo >> 4) & 0x3FFF) << 32) | (1ull << 46);
}

__device__ __forceinline__ void st_global16(int8_t *dst, uint4 v) {
    asm volatile("st.global.v4.b32 [%0], {%1, %2, %3, %4};" ::"l"(dst), "r"(v.x), "r"(v.y), "r"(v.z), "r"(v.w)
                 : "memory");
}

template <int EPI>
__global__ void __launch_bounds__(kDwThreads, 1) dw_tc_kernel(const __grid_constant__ DwTcParams p) {
    extern __shared__ uint8_t smem_raw[];
    uint8_t *smem = smem_raw + ((1024u - (smem_u32(smem_raw) & 1023u)) & 1023u);
    const int S = p.stages, taps = p.k * p.k, ksl = p.cw / 32, chunks = p.cw / 16;
    const DwLayout L(S, p.stage_bytes, taps, p.cw);
    uint8_t *sA = smem + L.a;
    uint8_t *sB = smem + L.b;
    long long *sK = reinterpret_cast<long long *>(smem + L.epi);
    int *sI = reinterpret_cast<int *>(sK + p.cw);
    const EpiSoA E{sK, sI, sI + p.cw, sI + 2 * p.cw, sI + 3 * p.cw, sI + 4 * p.cw, sI + 5 * p.cw};
    uint8_t *sLut = smem + L.lut;
    uint32_t *sTap = reinterpret_cast<uint32_t *>(smem + L.taps_off);
    uint64_t *bars = reinterpret_cast<uint64_t *>(smem + L.bars);
    uint64_t *full = bars, *empty = bars + S;
    uint64_t *tfull = bars + 2 * S, *tempty = tfull + kDwMaxAcc, *drain = tempty + kDwMaxAcc;
    uint32_t *tmem_slot = reinterpret_cast<uint32_t *>(drain + 1);
    volatile int *abort = reinterpret_cast<volatile int *>(tmem_slot + 1);
    const int warp = threadIdx.x / 32, lane = threadIdx.x % 32;
    const int c0 = blockIdx.y * p.cw;  // this CTA's channel slice

    if (threadIdx.x == 0) {
        for (int s = 0; s < S; s++) {
            mbar_init(smem_u32(full + s), kDwPW);  // one arrival per producer warp
            mbar_init(smem_u32(empty + s), 1);
        }
        for (int a = 0; a < p.n_acc; a++) {
            mbar_init(smem_u32(tfull + a), 1);
            mbar_init(smem_u32(tempty + a), 4 * p.nparts);  // the warps that take that tile
        }
        mbar_init(smem_u32(drain), 1);
        *abort = 0;
        asm volatile("fence.mbarrier_init.release.cluster;" ::: "memory");
    }
    for (int i = threadIdx.x; i < p.cw; i += blockDim.x) {
        const EpiChan c = p.epi[c0 + i];
        sK[i] = c.k;
        sI[i] = c.m;
        sI[p.cw + i] = c.cut;
        sI[2 * p.cw + i] = c.sh;
        sI[3 * p.cw + i] = c.ls;
        sI[4 * p.cw + i] = c.bs;
        sI[5 * p.cw + i] = c.zadd;
    }
    if (p.post)
        for (int i = threadIdx.x; i < 256; i += blockDim.x) sLut[i] = p.post[i];
    if (threadIdx.x < taps) {
        // tap (ky, kx) reads phase plane pl from window pixel off (stride 1: one plane)
        const int ky = threadIdx.x / p.k, kx = threadIdx.x - ky * p.k;
        const int pl = p.s == 1 ? 0 : (ky & 1) * 2 + (kx & 1);
        const int off = p.s == 1 ? ky * p.wp + kx : (ky >> 1) * p.wp + (kx >> 1);
        sTap[threadIdx.x] = (uint32_t)((pl * chunks) * p.npix + off);
    }
    {
        // this slice's diagonal weight blocks, resident for the whole kernel (tensor core: async proxy)
        const size_t bbytes = (size_t)taps * ksl * 1024;
        const uint4 *src = reinterpret_cast<const uint4 *>(p.wd + (size_t)blockIdx.y * bbytes);
        for (size_t i = threadIdx.x; i < bbytes / 16; i += blockDim.x)
            st_shared16(smem_u32(sB) + (uint32_t)(i * 16), __ldg(src + i));
        fence_proxy_async();
    }
    if (warp == kDwMmaWarp) {  // the MMA warp owns the TMEM allocation
        asm volatile("tcgen05.alloc.cta_group::1.sync.aligned.shared::cta.b32 [%0], %1;" ::"r"(smem_u32(tmem_slot)),
                     "r"(p.tmem_cols));
        asm volatile("tcgen05.relinquish_alloc_permit.cta_group::1.sync.aligned;");
    }
    tc_fence_before();
    __syncthreads();
    tc_fence_after();
    const uint32_t tmem_base = *tmem_slot;
    // Launched with programmatic serialization: the producer and epilogue warps wait here for the
    // previous kernel's activations (the MMA warp touches only shared memory and TMEM).
    if (warp != kDwMmaWarp) grid_dep_wait();

    if (warp < kDwPW) {
        // ------------------------------------------------------------------ window producers
        // Item q of a tile = (phase plane, image slot, window row v, pixel u, chunk j), chunk
        // fastest: a warp reads whole runs of pixels' channels. Each stage's copies are tracked per
        // thread with cp.async groups; a warp signals stage `k - lag` once all its lanes have seen
        // that group land (one arrival per warp), keeping up to lag + 1 windows of copies in flight.
        const int t = threadIdx.x;  // 0..127
        const uint32_t fw = 0x01010101u * (uint32_t)(uint8_t)p.xzp;
        const uint4 fill = make_uint4(fw, fw, fw, fw);
        const int row_items = p.wp << p.lchunks;
        const int items = p.planes * p.ipt * p.wrows * row_items;
        const int lag = S - 1 < 2 ? S - 1 : 2;
        int pending = 0;
        long long k = 0;
        for (int tile = blockIdx.x; tile < p.tiles; tile += gridDim.x, k++) {
            const int st = (int)(k % S);
            if (!mbar_wait(smem_u32(empty + st), (uint32_t)(((k / S) & 1) ^ 1), abort, 301)) break;
            const int ig = tile / p.row_tiles, r0 = (tile - ig * p.row_tiles) * p.tr;
            const uint32_t stage = smem_u32(sA) + (uint32_t)(st * p.stage_bytes);
            for (int q = t; q < items; q += kDwPW * 32) {
                const int row = p.f_row.div(q), rem = q - row * row_items;
                const int j = rem & (chunks - 1), u = rem >> p.lchunks;
                const int pi = p.f_wrows.div(row), v = row - pi * p.wrows;
                const int pl = p.f_ipt.div(pi), i = pi - pl * p.ipt;
                const int img = ig * p.ipt + i;
                const int iy = p.s * (r0 + v) + p.rowoff[pl], ix = p.s * u + p.coloff[pl];
                const uint32_t dst =
                    stage + (uint32_t)((((pl << p.lchunks) + j) * p.npix + i * p.slot + v * p.wp + u) * 16);
                if (img < p.n && (unsigned)iy < (unsigned)p.ih && (unsigned)ix < (unsigned)p.iw)
                    cp_async16(dst, p.x + (((size_t)img * p.ih + iy) * p.iw + ix) * p.c + c0 + 16 * j);
                else
                    st_shared16(dst, fill);  // the reference's padding value (and images past the batch)
            }
            cp_async_commit();
            if (++pending > lag) {
                cp_async_wait_dyn(lag);
                fence_proxy_async();  // the window visible to the tensor core (async proxy)
                __syncwarp();
                if (lane == 0) mbar_arrive(smem_u32(full + (int)((k - lag) % S)));
                pending--;
            }
        }
        cp_async_wait<0>();
        fence_proxy_async();
        __syncwarp();
        if (lane == 0)
            for (long long q = k - pending; q < k; q++) mbar_arrive(smem_u32(full + (int)(q % S)));
    } else if (warp == kDwMmaWarp) {
        // ------------------------------------------------------------------ MMA issuer
        if (lane == 0) {
            // Descriptors are built once; an operand's start address is the low field (16-byte units),
            // so each MMA adds its offset to the base descriptor (shared memory stays below 256 KB).
            const uint32_t idesc = instr_desc(32);
            const uint64_t adesc0 = desc_noswz(smem_u32(sA), (uint32_t)p.npix * 16, 128);
            const uint64_t bdesc0 = desc_noswz(smem_u32(sB), 512, 128);
            const uint32_t kk_step = 2u * (uint32_t)p.npix;  // two chunk planes per 32-channel K step
            long long k = 0;
            int lt = 0;
            for (int t = blockIdx.x; t < p.tiles; t += gridDim.x, k++, lt++) {
                const int st = (int)(k % S), acc = lt & (p.n_acc - 1);
                if (!mbar_wait(smem_u32(tempty + acc), (uint32_t)(((lt >> p.acc_shift) & 1) ^ 1), abort, 304)) break;
                if (!mbar_wait(smem_u32(full + st), (uint32_t)((k / S) & 1), abort, 305)) break;
                tc_fence_after();
                const uint64_t ad_st = adesc0 + (uint64_t)((uint32_t)(st * p.stage_bytes) >> 4);
                const uint32_t tmem_d = tmem_base + (uint32_t)(acc * p.cw);
                for (int tap = 0; tap < taps; tap++) {
                    const uint64_t ad = ad_st + sTap[tap], bd = bdesc0 + (uint64_t)(tap * ksl * 64);
                    const uint32_t accum = tap > 0 ? 1u : 0u;
                    mma_i8(tmem_d, ad, bd, idesc, accum);
                    if (ksl > 1) mma_i8(tmem_d + 32, ad + kk_step, bd + 64, idesc, accum);
                    if (ksl > 2) {
                        mma_i8(tmem_d + 64, ad + 2 * kk_step, bd + 128, idesc, accum);
                        mma_i8(tmem_d + 96, ad + 3 * kk_step, bd + 192, idesc, accum);
                    }
                }
                mma_commit(smem_u32(empty + st));  // window buffer free once these MMAs have read it
                mma_commit(smem_u32(tfull + acc));
            }
            // all MMAs are issued: the next kernel's CTAs may be scheduled once every CTA is here
            grid_dep_launch();
            // every MMA issued has completed before TMEM is freed, on the abort path too
            mma_commit(smem_u32(drain));
            const long long start = clock64();
            while (!mbar_try_wait(smem_u32(drain), 0, 200000) && clock64() - start < kTimeoutCycles) {
            }
        }
        __syncwarp();
    } else {
        // ------------------------------------------------------------------ epilogue
        const int e = warp - (kDwPW + 1);
        const int quarter = warp & 3;  // TMEM lanes 32*quarter .. +31 (warp id % 4 rule)
        // The 4 warps of a lane quarter split into fold groups of nparts: a warp takes 32 channels
        // (part) of every fold-th tile, starting with tile ph.
        const int part = (e >> 2) % p.nparts, ph = (e >> 2) / p.nparts;
        const int col = part * 32;
        const uint8_t *lut = p.post ? sLut : nullptr;
        // this lane's TMEM row: image slot, output row and column within the tile
        const int m = quarter * 32 + lane;
        const int si = p.ipt > 1 ? m / p.slot : 0;
        const int rem = m - si * p.slot, r = rem / p.wp, cc = rem - r * p.wp;
        const bool lane_ok = si < p.ipt && cc < p.ow && r < p.tr;
        int lt = ph;
        for (int t = blockIdx.x + ph * gridDim.x; t < p.tiles; t += p.fold * gridDim.x, lt += p.fold) {
            const int acc = lt & (p.n_acc - 1);
            if (!mbar_wait(smem_u32(tfull + acc), (uint32_t)((lt >> p.acc_shift) & 1), abort, 306)) break;
            tc_fence_after();
            const int ig = t / p.row_tiles;
            const int img = ig * p.ipt + si, oy = (t - ig * p.row_tiles) * p.tr + r;
            const bool valid = lane_ok && oy < p.oh && img < p.n;
            if (__any_sync(0xffffffffu, valid)) {
                const uint32_t taddr = tmem_base + ((uint32_t)(quarter * 32) << 16) + (uint32_t)(acc * p.cw + col);
                uint32_t ra[16], rb[16];
                tmem_ld16_nowait(taddr, ra);
                tmem_wait_ld(ra);
                tmem_ld16_nowait(taddr + 16, rb);
                const uint4 v0 = epilogue_chunk<EPI>(ra, E, lut, col, p.lo, p.hi);
                tmem_wait_ld(rb);
                const uint4 v1 = epilogue_chunk<EPI>(rb, E, lut, col + 16, p.lo, p.hi);
                if (valid) {
                    int8_t *dst = p.y + (((size_t)img * p.oh + oy) * p.ow + cc) * p.c + c0 + col;
                    st_global16(dst, v0);
                    st_global16(dst + 16, v1);
                }
            }
            tc_fence_before();
            __syncwarp();
            if (lane == 0) mbar_arrive(smem_u32(tempty + acc));  // accumulator free for reuse
        }
    }

    tc_fence_before();
    __syncthreads();
    tc_fence_after();
    if (warp == kDwMmaWarp) {
        asm volatile("tcgen05.dealloc.cta_group::1.sync.aligned.b32 %0, %1;" ::"r"(tmem_base), "r"(p.tmem_cols));
    }
}

}  // namespace

struct DwTc {
    int sm_count = 148;  // of the device the op was prepared on
    DwTcParams p{};
    size_t smem = 0;
    int epi_mode = kGeneral;
    int slices = 1;
};

int dw_tc_prepare(const int8_t *w, const int32_t *q, const uint8_t *post_dev, const ConvGeom &g,
                  const std::function<void *(size_t)> &alloc, DwTc **out) {
    *out = nullptr;
    // Off unless UNOQ_DW_TC=1: the dp4a kernel (k_dw.cu) is faster on every measured layer (see
    // the comment at the top of this file), so this path is an alternative kept tested, not the default.
    const char *env = std::getenv("UNOQ_DW_TC");
    if (!(env && env[0] == '1')) return 0;
    const int K = g.kh, S = g.sh, C = g.oc;
    if ((K != 3 && K != 5) || g.kw != K || g.sw != S || (S != 1 && S != 2) || g.dh != 1 || g.dw != 1) return 0;
    if (C % 32 != 0 || g.ic != C || g.pt < 0 || g.pt >= K || g.pl < 0 || g.pl >= K) return 0;
    if (g.ow < 1 || g.ow > 120 || g.oh < 1 || g.ih < 1 || g.iw < 1) return 0;
    if ((long long)g.ih * g.iw * C >= (1ll << 31) || (long long)g.oh * g.ow * C >= (1ll << 31)) return 0;
    // Window geometry: halo = the taps' reach in window pixels (one phase plane at stride 2).
    const int halo = S == 1 ? K - 1 : (K - 1) / 2;
    const int wp = g.ow + halo;
    int tr = (kBM - g.ow) / wp + 1;  // output rows whose M rows (r * wp + c) fit 128
    if (tr > g.oh) tr = g.oh;
    const int wrows = tr + halo;
    const int slot = (wrows * wp + 7) & ~7;
    int ipt = 1;
    if (tr == g.oh) {  // a whole image per tile: more images while their M rows still fit
        const int last = (g.oh - 1) * wp + g.ow;
        ipt = 1 + (kBM - last) / slot;
        if (ipt < 1) ipt = 1;
    }
    const int max_off = halo * wp + halo;  // the farthest tap offset (window pixels)
    const int npix = (std::max(ipt * slot, kBM + max_off) + 7) & ~7;
    const int planes = S == 1 ? 1 : 4, taps = K * K;
    // Channels per slice: the widest of 128 / 64 / 32 that divides C and fits shared memory with
    // at least two window stages.
    int cw = 0, stages = 0, stage_bytes = 0;
    for (int cand = 128; cand >= 32 && !cw; cand /= 2) {
        if (C % cand) continue;
        const int sb = (planes * (cand / 16) * npix * 16 + 1023) & ~1023;
        for (int st = 4; st >= 2; st--)
            if (DwLayout(st, sb, taps, cand).total <= (size_t)kDwMaxSmem) {
                cw = cand, stages = st, stage_bytes = sb;
                break;
            }
    }
    if (!cw) return 0;
    const int slices = C / cw, ksl = cw / 32;

    // Diagonal weight blocks: block (tap, kk) holds w[tap][c] at row n = c - 32 kk, column k = n of
    // the 32 x 32 B operand (K-major, no swizzle: byte (n, k) at (k / 16) * 512 + n * 16 + k % 16).
    // Plan weights are [kh * kw][C] (tflite.py:153).
    std::vector<uint8_t> wd((size_t)slices * taps * ksl * 1024, 0);
    for (int sl = 0; sl < slices; sl++)
        for (int t = 0; t < taps; t++)
            for (int kk = 0; kk < ksl; kk++)
                for (int n = 0; n < 32; n++) {
                    const int c = sl * cw + kk * 32 + n;
                    wd[(((size_t)sl * taps + t) * ksl + kk) * 1024 + (n / 16) * 512 + n * 16 + n % 16] =
                        (uint8_t)w[(size_t)t * C + c];
                }
    const int32_t *bias = q + kHead, *mult = bias + C, *shift = mult + C;
    const int yzp = q[13];
    std::vector<EpiChan> epi(C);
    bool fast = true;
    for (int c = 0; c < C; c++) {
        long long sum = 0;
        for (int t = 0; t < taps; t++) sum += w[(size_t)t * C + c];
        epi[c] = make_epilogue((long long)bias[c] + 128 * sum, mult[c], shift[c], yzp);
        fast &= epi_fast(epi[c]);
    }
    const int epi_mode = !fast ? kGeneral : (q[14] >= yzp ? kRelu : kTies);
    if (epi_mode != kGeneral)
        for (auto &e : epi) e.sh = e.sh >= 32 ? e.sh - 32 : 0;  // shift of the high word
    void *dwd = alloc(wd.size()), *de = alloc(epi.size() * sizeof(EpiChan));
    if (!dwd || !de || cudaMemcpy(dwd, wd.data(), wd.size(), cudaMemcpyHostToDevice) != cudaSuccess ||
        cudaMemcpy(de, epi.data(), epi.size() * sizeof(EpiChan), cudaMemcpyHostToDevice) != cudaSuccess)
        return 2001;
    const bool attrs = once_per_device(kFamilyDwTc, [] {
        auto allow = [](auto fn) {
            return cudaFuncSetAttribute(fn, cudaFuncAttributeMaxDynamicSharedMemorySize, kDwMaxSmem) == cudaSuccess;
        };
        return allow(dw_tc_kernel<kRelu>) && allow(dw_tc_kernel<kTies>) && allow(dw_tc_kernel<kGeneral>);
    });
    if (!attrs) return 2001;

    DwTc *d = new DwTc();
    d->sm_count = current_sm_count();
    d->slices = slices;
    d->epi_mode = epi_mode;
    d->smem = DwLayout(stages, stage_bytes, taps, cw).total;
    DwTcParams &p = d->p;
    p.wd = static_cast<const uint8_t *>(dwd);
    p.epi = static_cast<const EpiChan *>(de);
    p.post = post_dev;
    p.ih = g.ih, p.iw = g.iw, p.c = C, p.oh = g.oh, p.ow = g.ow;
    p.k = K, p.s = S, p.lo = q[14], p.hi = q[15], p.xzp = q[12];
    p.cw = cw;
    p.wp = wp, p.wrows = wrows, p.tr = tr, p.ipt = ipt, p.slot = slot;
    p.row_tiles = (g.oh + tr - 1) / tr;
    p.npix = npix;
    p.planes = planes;
    // phase plane (py, px): window pixel (u, v) is input (s (r0 + v) + py - pt, s u + px - pl)
    for (int pl = 0; pl < planes; pl++) p.rowoff[pl] = (pl >> 1) - g.pt, p.coloff[pl] = (pl & 1) - g.pl;
    p.lchunks = cw == 128 ? 3 : cw == 64 ? 2 : 1;
    p.f_row = FastDiv(wp * (cw / 16));
    p.f_wrows = FastDiv(wrows);
    p.f_ipt = FastDiv(ipt);
    p.stages = stages;
    p.stage_bytes = stage_bytes;
    p.nparts = cw / 32;
    p.fold = 4 / p.nparts;
    p.n_acc = std::min(kDwMaxAcc, 512 / cw);
    p.acc_shift = p.n_acc == 8 ? 3 : p.n_acc == 4 ? 2 : 1;
    int cols = 32;
    while (cols < p.n_acc * cw) cols *= 2;
    p.tmem_cols = cols;
    *out = d;
    return 0;
}

int dw_tc_launch(const DwTc &d, const int8_t *x, int8_t *y, const ConvGeom &g, cudaStream_t s) {
    DwTcParams p = d.p;
    p.n = g.n;
    p.y = y;
    const long long groups = (g.n + p.ipt - 1) / p.ipt;
    if (groups * p.row_tiles >= (1ll << 31)) return 2001;
    p.tiles = (int)(groups * p.row_tiles);
    p.x = x;
    int per_slice = d.sm_count / d.slices;
    if (per_slice < 1) per_slice = 1;
    if (per_slice > p.tiles) per_slice = p.tiles;
    const dim3 grid(per_slice, d.slices);
    if (d.epi_mode == kRelu) launch_pdl(kPdlDwTc, dw_tc_kernel<kRelu>, grid, kDwThreads, d.smem, s, p);
    else if (d.epi_mode == kTies) launch_pdl(kPdlDwTc, dw_tc_kernel<kTies>, grid, kDwThreads, d.smem, s, p);
    else launch_pdl(kPdlDwTc, dw_tc_kernel<kGeneral>, grid, kDwThreads, d.smem, s, p);
    return 0;
}

void dw_tc_free(DwTc *d) { delete d; }

int dw_tc_error(bool reset) {
    int v = 0;
    cudaMemcpyFromSymbol(&v, g_tc_error, sizeof(int));
    if (reset && v) {
        int z = 0;
        cudaMemcpyToSymbol(g_tc_error, &z, sizeof(int));
    }
    return v;
}

}  // namespace uq
