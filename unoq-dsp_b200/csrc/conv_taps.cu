// conv_taps.cu -- spatial convolutions over wide inputs as implicit GEMMs whose A tiles are loaded
// by TMA, one box per filter tap (tcgen05 kind::i8).
//
// Plan code 14 (runtime/qnn.c:1101-1227) for kh x kw <= 3 x 3 kernels over ic % 128 == 0 channels
// (ic % 32 == 0 on request), stride 1 or 2, any dilation. A tile is P x R output pixels (R
// output rows of P columns) of one image, MMA row m = r * P + p. For filter tap (ky, kx) the A rows of the tile are the input
// pixels (s*(oy0 + r) - pt + ky*dh, s*(ox0 + p) - pl + kx*dw): a strided 4-D box of the NHWC
// input {channels, columns, rows, images} with traversal stride s in both spatial dimensions,
// which TMA loads straight into the UMMA K-major swizzled layout (one box per tap and 128-byte
// channel chunk; taps outside the image read as zero). The reduction index order is the plan's
// (ky, kx, ic) (tflite.py:155), so B is the plan's weights re-tiled per (tap, channel chunk). No
// thread assembles im2col rows: the only SIMT work is the epilogue.
//
// Zero fill stands where the reference reads the input zero point (qnn.c:1166-1168): an output
// pixel whose taps leave the image gets xzp * (sum of those taps' weights) added to its
// accumulators, from a table indexed by which kernel rows and columns are outside; the u8 / s8
// difference of the reference's columns is folded into the per-channel constants as in
// conv_tc.cu, so results are bit-identical.
//
// Roles: warp 0 issues the TMA loads, warp 1 the MMAs (M=128, N=BN, K=32 per instruction) into a
// ring of TMEM accumulators, warps 2..17 requantise (tcgen05.ld, exact scale, clamp, post table)
// and store each pixel's 16-channel chunks with 16-byte stores. Every wait is bounded (about 2 s);
// on expiry the kernel records a site code, waits for its copies and MMAs, frees its TMEM and exits.
#include <algorithm>
#include <cstdlib>
#include <cstring>
#include <type_traits>
#include <vector>

#include "device_state.hpp"
#include "conv_taps.cuh"
#include "plan.hpp"
#include "tc_common.cuh"

namespace uq {

namespace {

constexpr int kTapsMaxSmem = 227 * 1024;
constexpr int kTapsWeightBudget = 96 * 1024;
constexpr int kTapsEW = 16;  // epilogue warps, 4 per TMEM lane quarter

struct TapsParams {
    CUtensorMap xmap;       // input {ic, iw, ih, n}, box {icc, P*s, R*s, 1}, traversal stride {1, s, s, 1}
    const int8_t *w;        // [n_tiles][taps][nchunks][bn x icc], UMMA K-major, swizzle span icc
    const EpiChan *epi;     // [n_tiles * bn]
    const uint8_t *post;    // 256 bytes or null
    const int32_t *corr;    // [(rowmask << kw) | colmask][oc]
    int8_t *y;
    int ih, iw, ic, oh, ow, oc;
    int kh, kw, s, dh, dw, pt, pl;
    int P, R;               // tile: R output rows x P output columns
    int tiles_x, tiles_y, tiles;  // column blocks, row blocks per image; M tiles in all
    int bn, icc, nchunks;   // N tile width, channel chunk bytes (32 / 64 / 128), chunks per tap
    int stage_bytes;        // bytes one tap's box writes: P * R * icc
    int stages, lo, hi, n_acc, fold, tmem_cols;
};

struct TapsLayout {
    size_t a, b, epi, lut, bars, total;
    __host__ __device__ TapsLayout(int stages, int icc, int taps, int nchunks, int bn) {
        size_t o = 0;
        a = o;
        o += (size_t)stages * kBM * icc;
        b = o;
        o += (size_t)taps * nchunks * bn * icc;
        epi = (o + 31) & ~(size_t)31;
        o = epi + (size_t)bn * sizeof(EpiChan);
        lut = o;
        o += 256;
        bars = (o + 7) & ~(size_t)7;
        o = bars + (size_t)(2 * stages + 9) * 8 + 16;
        total = o + 1024;  // base alignment slack
    }
};

// UMMA shared-memory descriptor, K-major, swizzle span `span` bytes (32 / 64 / 128): 8-row atoms
// of 8 * span bytes.
__device__ __forceinline__ uint64_t smem_desc_span(uint32_t addr, int span) {
    const uint64_t mode = span == 128 ? 2ull : span == 64 ? 4ull : 6ull;
    return (uint64_t)((addr >> 4) & 0x3FFF) | (1ull << 16) | ((uint64_t)((8 * span) >> 4) << 32) | (1ull << 46) |
           (mode << 61);
}

__device__ __forceinline__ void taps_expect_tx(uint32_t bar, uint32_t bytes) {
    asm volatile("mbarrier.arrive.expect_tx.shared::cta.b64 _, [%0], %1;" ::"r"(bar), "r"(bytes) : "memory");
}

__device__ __forceinline__ void tma_load_4d(uint32_t dst, const CUtensorMap *map, int c0, int c1, int c2, int c3,
                                            uint32_t bar) {
    asm volatile(
        "cp.async.bulk.tensor.4d.shared::cluster.global.tile.mbarrier::complete_tx::bytes [%0], [%1, {%2, %3, %4, "
        "%5}], [%6];" ::"r"(dst),
        "l"(reinterpret_cast<uint64_t>(map)), "r"(c0), "r"(c1), "r"(c2), "r"(c3), "r"(bar)
        : "memory");
}

template <int EPI>
__global__ void __launch_bounds__((2 + kTapsEW) * 32, 1) conv_taps_kernel(const __grid_constant__ TapsParams p) {
    constexpr int kParts = kTapsEW / 4;
    extern __shared__ uint8_t smem_raw[];
    uint8_t *smem = smem_raw + ((1024u - (smem_u32(smem_raw) & 1023u)) & 1023u);
    const int S = p.stages, taps = p.kh * p.kw;
    const TapsLayout L(S, p.icc, taps, p.nchunks, p.bn);
    uint8_t *sA = smem + L.a;
    uint8_t *sB = smem + L.b;
    long long *sK = reinterpret_cast<long long *>(smem + L.epi);
    int *sI = reinterpret_cast<int *>(sK + p.bn);
    const EpiSoA E{sK, sI, sI + p.bn, sI + 2 * p.bn, sI + 3 * p.bn, sI + 4 * p.bn, sI + 5 * p.bn};
    uint8_t *sLut = smem + L.lut;
    uint64_t *bars = reinterpret_cast<uint64_t *>(smem + L.bars);
    uint64_t *full = bars, *empty = bars + S;
    uint64_t *tfull = bars + 2 * S, *tempty = bars + 2 * S + 4, *drain = bars + 2 * S + 8;
    uint32_t *tmem_slot = reinterpret_cast<uint32_t *>(bars + 2 * S + 9);
    volatile int *abort = reinterpret_cast<volatile int *>(tmem_slot + 1);
    const int warp = threadIdx.x / 32, lane = threadIdx.x % 32;
    const int ntile = blockIdx.y;
    const size_t stage_alloc = (size_t)kBM * p.icc;
    const size_t b_tile = (size_t)taps * p.nchunks * p.bn * p.icc;

    if (threadIdx.x == 0) {
        for (int s = 0; s < S; s++) {
            mbar_init(smem_u32(full + s), 1);
            mbar_init(smem_u32(empty + s), 1);
        }
        for (int a = 0; a < 4; a++) {
            mbar_init(smem_u32(tfull + a), 1);
            mbar_init(smem_u32(tempty + a), kTapsEW / p.fold);
        }
        mbar_init(smem_u32(drain), 1);
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
    {
        // this N tile's weights, resident for the whole kernel (read by the tensor core: async proxy)
        const uint4 *src = reinterpret_cast<const uint4 *>(p.w + (size_t)ntile * b_tile);
        for (size_t i = threadIdx.x; i < b_tile / 16; i += blockDim.x)
            st_shared16(smem_u32(sB) + (uint32_t)(i * 16), __ldg(src + i));
        fence_proxy_async();
    }
    if (warp == 1) {  // the MMA warp owns the TMEM allocation
        asm volatile("tcgen05.alloc.cta_group::1.sync.aligned.shared::cta.b32 [%0], %1;" ::"r"(smem_u32(tmem_slot)),
                     "r"(p.tmem_cols));
        asm volatile("tcgen05.relinquish_alloc_permit.cta_group::1.sync.aligned;");
    }
    tc_fence_before();
    __syncthreads();
    tc_fence_after();
    const uint32_t tmem_base = *tmem_slot;
    // Launched with programmatic serialization: the TMA and epilogue warps wait here for the
    // previous kernel's activations (the MMA warp touches only shared memory and TMEM).
    if (warp != 1) grid_dep_wait();
    const int per_image = p.tiles_y * p.tiles_x;

    if (warp == 0) {
        // ------------------------------------------------------------------ TMA producer
        if (lane == 0) {
            long long it = 0;
            bool ok = true;
            for (int t = blockIdx.x; t < p.tiles && ok; t += gridDim.x) {
                const int img = t / per_image, rem = t - img * per_image;
                const int ty = rem / p.tiles_x, tx = rem - ty * p.tiles_x;
                const int y0 = p.s * ty * p.R - p.pt, x0 = p.s * tx * p.P - p.pl;
                for (int tap = 0; tap < taps && ok; tap++) {
                    const int ky = tap / p.kw, kx = tap - ky * p.kw;
                    for (int c = 0; c < p.nchunks; c++, it++) {
                        const int s = (int)(it % S);
                        if (!mbar_wait(smem_u32(empty + s), (uint32_t)(((it / S) & 1) ^ 1), abort, 301)) {
                            ok = false;
                            break;
                        }
                        taps_expect_tx(smem_u32(full + s), (uint32_t)p.stage_bytes);
                        tma_load_4d(smem_u32(sA + (size_t)s * stage_alloc), &p.xmap, c * p.icc, x0 + kx * p.dw,
                                    y0 + ky * p.dh, img, smem_u32(full + s));
                    }
                }
            }
            // every load issued has landed before the CTA may exit (bounded)
            for (long long q = it - (it < S ? it : S); q < it; q++) {
                const long long start = clock64();
                while (!mbar_try_wait(smem_u32(full + (int)(q % S)), (uint32_t)((q / S) & 1), 200000) &&
                       clock64() - start < kTimeoutCycles) {
                }
            }
        }
        __syncwarp();
    } else if (warp == 1) {
        // ------------------------------------------------------------------ MMA issuer
        if (lane == 0) {
            const uint32_t idesc = instr_desc(p.bn);
            const uint32_t a0 = smem_u32(sA), b0 = smem_u32(sB);
            const int ksteps = p.icc / 32;
            long long it = 0;
            bool ok = true;
            int lt = 0;
            for (int t = blockIdx.x; t < p.tiles && ok; t += gridDim.x, lt++) {
                const int acc = lt % p.n_acc;
                if (!mbar_wait(smem_u32(tempty + acc), (uint32_t)(((lt / p.n_acc) & 1) ^ 1), abort, 302)) break;
                tc_fence_after();
                const uint32_t tmem_d = tmem_base + (uint32_t)(acc * p.bn);
                for (int q = 0; q < taps * p.nchunks; q++, it++) {
                    const int s = (int)(it % S);
                    if (!mbar_wait(smem_u32(full + s), (uint32_t)((it / S) & 1), abort, 303)) {
                        ok = false;
                        break;
                    }
                    tc_fence_after();
                    for (int kk = 0; kk < ksteps; kk++) {
                        const uint64_t ad = smem_desc_span(a0 + (uint32_t)(s * stage_alloc + kk * 32), p.icc);
                        const uint64_t bd =
                            smem_desc_span(b0 + (uint32_t)((size_t)q * p.bn * p.icc + kk * 32), p.icc);
                        mma_i8(tmem_d, ad, bd, idesc, (q | kk) ? 1u : 0u);
                    }
                    mma_commit(smem_u32(empty + s));
                }
                if (!ok) break;
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
        const int e = warp - 2;
        const int quarter = warp & 3;  // TMEM lanes 32*quarter .. +31 (warp id % 4 rule)
        const int half = e >> 2;
        // column parts of a tile (16-column chunks part, part + nparts, ...) x tile phases (fold)
        const int nparts = kParts / p.fold;
        const int part = half % nparts, ph = half / nparts;
        const uint8_t *lut = p.post ? sLut : nullptr;
        const int n0 = ntile * p.bn;
        const int cols = min(p.bn, p.oc - n0);
        const int live_chunks = cols / 16;
        const int m = quarter * 32 + lane;  // MMA row of this thread: output pixel (r, pc) of the tile
        const int r = m / p.P, pc = m - r * p.P;
        const bool in_tile = m < p.P * p.R;
        int lt = ph;
        for (int t = blockIdx.x + ph * gridDim.x; t < p.tiles; t += p.fold * gridDim.x, lt += p.fold) {
            const int img = t / per_image, rem = t - img * per_image;
            const int ty = rem / p.tiles_x, tx = rem - ty * p.tiles_x;
            const int oy = ty * p.R + r, ox = tx * p.P + pc;
            const bool valid = in_tile && oy < p.oh && ox < p.ow;
            const int acc = lt % p.n_acc;
            if (!mbar_wait(smem_u32(tfull + acc), (uint32_t)((lt / p.n_acc) & 1), abort, 304)) break;
            tc_fence_after();
            // kernel rows / columns of this pixel's taps that fall outside the image
            int rmask = 0, cmask = 0;
            for (int ky = 0; ky < p.kh; ky++) {
                const int iy = p.s * oy - p.pt + ky * p.dh;
                rmask |= (iy < 0 || iy >= p.ih) ? 1 << ky : 0;
            }
            for (int kx = 0; kx < p.kw; kx++) {
                const int ix = p.s * ox - p.pl + kx * p.dw;
                cmask |= (ix < 0 || ix >= p.iw) ? 1 << kx : 0;
            }
            const int32_t *cr = (rmask | cmask) && valid ? p.corr + (size_t)((rmask << p.kw) | cmask) * p.oc + n0 : nullptr;
            int8_t *dst = p.y + (((size_t)img * p.oh + oy) * p.ow + ox) * p.oc + n0;
            const uint32_t taddr = tmem_base + ((uint32_t)(quarter * 32) << 16) + (uint32_t)(acc * p.bn);
            uint32_t ra[16], rb[16];
            int ci = part;
            if (ci < live_chunks) {
                tmem_ld16_nowait(taddr + ci * 16, ra);
                tmem_wait_ld(ra);
            }
            while (ci < live_chunks) {
                const int next = ci + nparts;
                if (next < live_chunks) tmem_ld16_nowait(taddr + next * 16, rb);
                if (valid) {
                    if (cr) {
#pragma unroll
                        for (int i = 0; i < 16; i++) ra[i] = (uint32_t)((int32_t)ra[i] + __ldg(cr + ci * 16 + i));
                    }
                    const uint4 v = epilogue_chunk<EPI>(ra, E, lut, ci * 16, p.lo, p.hi);
                    *reinterpret_cast<uint4 *>(dst + ci * 16) = v;
                }
                if (next < live_chunks) tmem_wait_ld(rb);
#pragma unroll
                for (int q = 0; q < 16; q++) ra[q] = rb[q];
                ci = next;
            }
            tc_fence_before();
            __syncwarp();
            if (lane == 0) mbar_arrive(smem_u32(tempty + acc));  // accumulator free for reuse
        }
    }

    tc_fence_before();
    __syncthreads();
    tc_fence_after();
    if (warp == 1) {
        asm volatile("tcgen05.dealloc.cta_group::1.sync.aligned.b32 %0, %1;" ::"r"(tmem_base), "r"(p.tmem_cols));
    }
}


}  // namespace

struct ConvTaps {
    int sm_count = 148;  // of the device the op was prepared on
    TapsParams p{};
    size_t smem = 0;
    int epi_mode = kGeneral;
    int n_tiles = 1;
};

int conv_taps_prepare(const int8_t *w_packed, const int32_t *q, const uint8_t *post_dev, const ConvGeom &g,
                      const std::function<void *(size_t)> &alloc, ConvTaps **out) {
    *out = nullptr;
    // Taken by default for 128-byte channel chunks (ic % 128 == 0): with 32- or 64-byte rows the TMA
    // gathers rows too slowly and the band producer of conv_tc.cu is faster. UNOQ_CONV_TAPS=all takes
    // every ic % 32 == 0 conv (for tests), UNOQ_CONV_TAPS=0 none.
    const char *env = std::getenv("UNOQ_CONV_TAPS");
    if (env && env[0] == '0') return 0;
    const bool all = env && std::strcmp(env, "all") == 0;
    const int s = g.sh;
    if (g.ic % (all ? 32 : 128) != 0 || g.kh > 3 || g.kw > 3 || g.kh * g.kw < 2 || g.sw != s || (s != 1 && s != 2))
        return 0;
    if (g.oc % 16 != 0 || g.dh < 1 || g.dw < 1) return 0;
    if ((long long)g.ih * g.iw * g.ic >= (1ll << 31) || (long long)g.oh * g.ow * g.oc >= (1ll << 31)) return 0;
    const int taps = g.kh * g.kw;
    const int icc = g.ic % 128 == 0 ? 128 : g.ic % 64 == 0 ? 64 : 32;  // channel chunk = swizzle span
    const int nchunks = g.ic / icc;
    // N tile: a power of two (16..256) no wider than the channel count needs, weights resident
    int bn = 16;
    while (bn < 256 && bn < g.oc) bn *= 2;
    while (bn > 16 && (size_t)taps * g.ic * bn > (size_t)kTapsWeightBudget) bn /= 2;
    if ((size_t)taps * g.ic * bn > (size_t)kTapsWeightBudget) return 0;
    const int n_tiles = (g.oc + bn - 1) / bn;
    // tile shape: R rows x P columns (P * R <= 128) with the fewest tiles per image
    int P = 0, R = 0;
    long long best = -1;
    for (int pc = std::min(g.ow, 128); pc >= 1; pc--) {
        const int rr = std::min(128 / pc, g.oh);
        if (pc * s > 256 || rr * s > 256 || rr < 1) continue;
        const long long n = (long long)((g.ow + pc - 1) / pc) * ((g.oh + rr - 1) / rr);
        if (best < 0 || n < best) best = n, P = pc, R = rr;
    }
    if (!P) return 0;
    int stages = 8;
    while (stages > 2 && TapsLayout(stages, icc, taps, nchunks, bn).total > (size_t)kTapsMaxSmem) stages--;
    const TapsLayout L(stages, icc, taps, nchunks, bn);
    if (L.total > (size_t)kTapsMaxSmem) return 0;

    // Weights: reference packed layout (gemm.h:9) -> per N tile, per (tap, channel chunk), a bn x icc
    // K-major block in the UMMA swizzle of span icc (16-byte chunk index XOR row bits).
    const int kp = q[18], oc = g.oc, K = taps * g.ic;
    auto wref = [&](int j, int t) -> int { return w_packed[(j / 4) * kp * 4 + (t / 8) * 32 + (j % 4) * 8 + t % 8]; };
    const size_t b_tile = (size_t)taps * nchunks * bn * icc;
    std::vector<uint8_t> wt((size_t)n_tiles * b_tile, 0);
    auto swz = [&](int row, int chunk) {
        return icc == 128 ? chunk ^ (row & 7) : icc == 64 ? chunk ^ ((row >> 1) & 3) : chunk ^ ((row >> 2) & 1);
    };
    for (int nt = 0; nt < n_tiles; nt++)
        for (int r = 0; r < bn; r++) {
            const int j = nt * bn + r;
            if (j >= oc) continue;
            for (int tap = 0; tap < taps; tap++)
                for (int c = 0; c < nchunks; c++)
                    for (int k = 0; k < icc; k++) {
                        const size_t blk = (size_t)nt * b_tile + ((size_t)(tap * nchunks + c) * bn) * icc;
                        const size_t off = blk + (size_t)(r / 8) * 8 * icc + (size_t)(r % 8) * icc + swz(r % 8, k / 16) * 16 + k % 16;
                        wt[off] = (uint8_t)(int8_t)wref(j, tap * g.ic + c * icc + k);
                    }
        }
    const int32_t *cbias = q + kHead, *mult = cbias + oc, *shift = mult + oc;
    const int xzp = q[12], yzp = q[13];
    std::vector<EpiChan> epi((size_t)n_tiles * bn);
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
            }
            epi[(size_t)nt * bn + r] =
                make_epilogue((long long)cbias[j] + 128ll * sum_all + (long long)xzp * sum_pad, mult[j], shift[j], yzp);
        }
    bool fast = true;
    for (int j = 0; j < oc; j++) fast &= epi_fast(epi[j]);  // channel j sits at nt * bn + r = j
    const int epi_mode = !fast ? kGeneral : (q[14] >= yzp ? kRelu : kTies);
    if (epi_mode != kGeneral)
        for (auto &e : epi) e.sh = e.sh >= 32 ? e.sh - 32 : 0;  // shift of the high word
    // xzp * sum of the weights of the taps outside the image, per (rows outside, columns outside)
    std::vector<int32_t> corr((size_t)(1 << g.kh) * (1 << g.kw) * oc, 0);
    for (int rm = 0; rm < (1 << g.kh); rm++)
        for (int cm = 0; cm < (1 << g.kw); cm++)
            for (int j = 0; j < oc; j++) {
                long long sum = 0;
                for (int ky = 0; ky < g.kh; ky++)
                    for (int kx = 0; kx < g.kw; kx++)
                        if ((rm >> ky & 1) || (cm >> kx & 1))
                            for (int c = 0; c < g.ic; c++) sum += wref(j, (ky * g.kw + kx) * g.ic + c);
                corr[((size_t)(rm << g.kw) | cm) * oc + j] = (int32_t)((long long)xzp * sum);
            }
    void *dw = alloc(wt.size());
    void *de = alloc(epi.size() * sizeof(EpiChan));
    void *dc = alloc(corr.size() * sizeof(int32_t));
    if (!dw || !de || !dc) return 2001;
    if (cudaMemcpy(dw, wt.data(), wt.size(), cudaMemcpyHostToDevice) != cudaSuccess ||
        cudaMemcpy(de, epi.data(), epi.size() * sizeof(EpiChan), cudaMemcpyHostToDevice) != cudaSuccess ||
        cudaMemcpy(dc, corr.data(), corr.size() * sizeof(int32_t), cudaMemcpyHostToDevice) != cudaSuccess)
        return 2001;
    const bool attrs = once_per_device(kFamilyConvTaps, [] {
        auto allow = [](auto fn) {
            return cudaFuncSetAttribute(fn, cudaFuncAttributeMaxDynamicSharedMemorySize, kTapsMaxSmem) == cudaSuccess;
        };
        return allow(conv_taps_kernel<kRelu>) && allow(conv_taps_kernel<kTies>) && allow(conv_taps_kernel<kGeneral>);
    });
    if (!attrs) return 2001;
    ConvTaps *c = new ConvTaps();
    c->sm_count = current_sm_count();
    TapsParams &p = c->p;
    p.w = static_cast<const int8_t *>(dw);
    p.epi = static_cast<const EpiChan *>(de);
    p.corr = static_cast<const int32_t *>(dc);
    p.post = post_dev;
    p.ih = g.ih, p.iw = g.iw, p.ic = g.ic, p.oh = g.oh, p.ow = g.ow, p.oc = g.oc;
    p.kh = g.kh, p.kw = g.kw, p.s = s, p.dh = g.dh, p.dw = g.dw, p.pt = g.pt, p.pl = g.pl;
    p.P = P, p.R = R;
    p.tiles_x = (g.ow + P - 1) / P;
    p.tiles_y = (g.oh + R - 1) / R;
    p.bn = bn, p.icc = icc, p.nchunks = nchunks;
    p.stage_bytes = P * R * icc;
    p.stages = stages;
    p.lo = q[14], p.hi = q[15];
    p.n_acc = bn <= 128 ? 4 : 2;
    p.tmem_cols = std::max(32, p.n_acc * bn);
    // narrow N tiles: spare epilogue warps of each lane quarter take alternate tiles (divides n_acc)
    p.fold = 4 / std::min(4, bn / 16);
    c->smem = L.total;
    c->epi_mode = epi_mode;
    c->n_tiles = n_tiles;
    *out = c;
    return 0;
}

int conv_taps_launch(const ConvTaps &c, const int8_t *x, int8_t *y, const ConvGeom &g, cudaStream_t s) {
    TapsParams p = c.p;
    p.y = y;
    const long long tiles = (long long)g.n * p.tiles_y * p.tiles_x;
    if (tiles >= (1ll << 31)) return 2001;
    p.tiles = (int)tiles;
    EncodeTiled enc = encoder();
    if (!enc) return 2001;
    const cuuint64_t dims[4] = {(cuuint64_t)g.ic, (cuuint64_t)g.iw, (cuuint64_t)g.ih, (cuuint64_t)g.n};
    const cuuint64_t strides[3] = {(cuuint64_t)g.ic, (cuuint64_t)g.iw * g.ic, (cuuint64_t)g.ih * g.iw * g.ic};
    const cuuint32_t box[4] = {(cuuint32_t)p.icc, (cuuint32_t)(p.P * p.s), (cuuint32_t)(p.R * p.s), 1};
    const cuuint32_t estr[4] = {1, (cuuint32_t)p.s, (cuuint32_t)p.s, 1};
    const CUtensorMapSwizzle sw = p.icc == 128  ? CU_TENSOR_MAP_SWIZZLE_128B
                                  : p.icc == 64 ? CU_TENSOR_MAP_SWIZZLE_64B
                                                : CU_TENSOR_MAP_SWIZZLE_32B;
    if (enc(&p.xmap, CU_TENSOR_MAP_DATA_TYPE_UINT8, 4, const_cast<int8_t *>(x), dims, strides, box, estr,
            CU_TENSOR_MAP_INTERLEAVE_NONE, sw, CU_TENSOR_MAP_L2_PROMOTION_L2_128B,
            CU_TENSOR_MAP_FLOAT_OOB_FILL_NONE) != CUDA_SUCCESS)
        return 2001;
    // CTAs per N tile: floor, so that all n_tiles * per_tile CTAs are resident at once (one per SM).
    // Rounding up would start the extra CTAs only after a first wave had finished, and the static
    // tile schedule would make them run a full share of tiles on their own.
    int per_tile = c.sm_count / c.n_tiles;
    if (per_tile < 1) per_tile = 1;
    if (per_tile > p.tiles) per_tile = p.tiles;
    const dim3 grid(per_tile, c.n_tiles);
    constexpr int T = (2 + kTapsEW) * 32;
    if (c.epi_mode == kRelu) launch_pdl(kPdlConvTaps, conv_taps_kernel<kRelu>, grid, T, c.smem, s, p);
    else if (c.epi_mode == kTies) launch_pdl(kPdlConvTaps, conv_taps_kernel<kTies>, grid, T, c.smem, s, p);
    else launch_pdl(kPdlConvTaps, conv_taps_kernel<kGeneral>, grid, T, c.smem, s, p);
    return 0;
}

void conv_taps_free(ConvTaps *c) { delete c; }

int conv_taps_error(bool reset) {
    int v = 0;
    cudaMemcpyFromSymbol(&v, g_tc_error, sizeof(int));
    if (reset && v) {
        int z = 0;
        cudaMemcpyToSymbol(g_tc_error, &z, sizeof(int));
    }
    return v;
}

}  // namespace uq
