// conv_rows.cu -- convolutions over few input channels (the RGB stems) as row GEMMs on the
// 5th-generation tensor cores (tcgen05 kind::i8).
//
// Plan code 14 (runtime/qnn.c:1101-1227) for kh x kw kernels (kh, kw <= 3) over ic <= 32 channels
// (or <= 64 with at most 32 outputs) with stride s in both directions: the RGB stems, the 8 /
// 16-channel layers of YOLO26n, 24 / 32-channel 3x3 layers and YOLO26n's 64 -> 16 head conv. For
// G adjacent output columns ox0..ox0+G-1 of output row oy, every tap of kernel row ky reads input
// row iy = s*oy - pt + ky, and all their bytes lie in one window of that row: bytes
// [X, X + s*ic*(G-1) + kw*ic) with X = (s*ox0 - pl)*ic. Hence
//
//     Y[oy][ox0 + j][oc] = sum_ky sum_b  In[iy][A + b] * W_ky[j*OC + oc][b]      (0 <= b < span)
//
// with A = X rounded down to 16 bytes and W_ky[j*OC + oc][b] = w[oc][ky][kx][c] where
// b = (X - A) + s*ic*j + kx*ic + c (zero elsewhere). That is a GEMM with M = 128 output rows (R
// rows from each of 128 / R consecutive images), N = G*OC (G output pixels x OC channels, <= 256)
// and K = one to four 128-byte blocks ("atoms") of window per kernel row: more than one when a
// 17-64-channel input leaves no tile width whose window fits one. The A operand of each (tile,
// ky, atom) is a plain box {128 bytes, R rows, 128 / R images} of the input tensor, loaded by TMA
// straight into the UMMA SWIZZLE_128B layout from a 3-D tensor map {row bytes, every s-th row,
// images} whose out-of-range rows, columns and images read as zero: no im2col assembly at all.
// The banded B matrix is built once at load time and stays resident in shared memory.
//
// Zero fill stands where the reference reads the input zero point (qnn.c:1166-1168): an output
// whose taps leave the image gets xzp * (sum of those taps' weights) added to its accumulator,
// from a table indexed by which kernel rows and columns are outside. The u8 / s8 difference of
// the reference's columns is folded into the per-channel constants as in conv_tc.cu.
//
// Roles: warp 0 issues the TMA loads, warp 1 the MMAs (M=128, N=G*OC, K=32 per instruction) into
// two TMEM accumulators, warps 2.. requantise (tcgen05.ld, exact scale, clamp, post table) into
// per-warp staging buffers and write them with 3-D TMA tensor stores, which clip the rows and
// images past the tensor. Every wait is bounded (about 2 s); on expiry the kernel records a site code, waits
// for its copies and MMAs, frees its TMEM and exits.
#include <algorithm>
#include <cstdlib>
#include <cstring>
#include <type_traits>
#include <vector>

#include "device_state.hpp"
#include "conv_rows.cuh"
#include "plan.hpp"
#include "tc_common.cuh"

namespace uq {

namespace {

constexpr int kRowsMaxSmem = 227 * 1024;

struct RowsParams {
    CUtensorMap xmap[2];   // input views: rows v, v + s, v + 2s, ... of every image (v = 0, 1)
    CUtensorMap ymap;      // output {ow*oc, oh, n}, box {box, 32, 1}, swizzled like the staging
    const int8_t *w;       // [kh][bn x 128] UMMA SWIZZLE_128B K-major
    const EpiChan *epi;    // [oc]
    const uint8_t *post;   // 256 bytes or null
    const int32_t *corr;   // [(rowmask << kw) | colmask][oc]: xzp * weights of the taps outside
    int n, ih, iw, ic, oh, ow, oc;
    int ec;                // epilogue constant entries: oc, or 16 (oc = 4 / 8: entry i is channel i % oc)
    int loc;               // log2 of the columns of one pixel within a 16-column chunk (oc < 16), else 4
    int kh, kw, s, pt, pl;
    int G, bn;             // output pixels per column group; bn = G * oc
    int groups, row_tiles, tiles;
    int R, ipt;            // M tile = R output rows of each of ipt = 128 / R consecutive images
    int span;              // bytes of a kernel row's window (from its 16-byte-aligned start)
    int atoms;             // 128-byte K blocks per kernel row (1-4): stages per tile = kh * atoms
    int x0;                // window start (bytes, 16-aligned, may be negative) of group 0; group g adds g * gstep
    int gstep;
    int view[3], dy[3];    // per kernel row: input view and row offset (view row = oy + dy)
    int stages, lo, hi, box, swz, out_bytes, tmem_cols;
    int nparts;            // epilogue warps of a lane quarter that share one tile (1, 2 or 4), box = bn / nparts
    int fold;              // tiles in flight per lane quarter: 4 / nparts (a warp takes every fold-th tile)
    int n_acc;             // TMEM accumulators in rotation (2, 4 or 8)
    int acc_shift;         // log2(n_acc)
};

constexpr int kRowsMaxAcc = 8;

struct RowsLayout {
    size_t a, b, out, epi, lut, bars, total;
    __host__ __device__ RowsLayout(int stages, int kblocks, int bn, int oc, int out_bytes) {
        size_t o = 0;
        a = o;
        o += (size_t)stages * kStageBytes;
        b = o;
        o += (size_t)kblocks * bn * kBK;
        out = o;
        o += (size_t)out_bytes;
        epi = (o + 31) & ~(size_t)31;
        o = epi + (size_t)oc * sizeof(EpiChan);
        lut = o;
        o += 256;
        bars = (o + 7) & ~(size_t)7;
        o = bars + (size_t)(2 * stages + 2 * kRowsMaxAcc + 1) * 8 + 16;
        total = o + 1024;  // base alignment slack
    }
};

__host__ __device__ inline size_t rows_warp_stage(int box) { return ((size_t)32 * box + 1023) & ~(size_t)1023; }

__device__ __forceinline__ void mbar_expect_tx(uint32_t bar, uint32_t bytes) {
    asm volatile("mbarrier.arrive.expect_tx.shared::cta.b64 _, [%0], %1;" ::"r"(bar), "r"(bytes) : "memory");
}

__device__ __forceinline__ void tma_load_3d(uint32_t dst, const CUtensorMap *map, int x, int y, int z, uint32_t bar) {
    asm volatile(
        "cp.async.bulk.tensor.3d.shared::cluster.global.tile.mbarrier::complete_tx::bytes [%0], [%1, {%2, %3, %4}], "
        "[%5];" ::"r"(dst),
        "l"(reinterpret_cast<uint64_t>(map)), "r"(x), "r"(y), "r"(z), "r"(bar)
        : "memory");
}

// 16 epilogue warps (4 per TMEM lane quarter), each owning CHUNKS 16-column chunks of a tile.
constexpr int kRowsEW = 16;

// SUB: fewer than 16 output channels, so a 16-column chunk holds several pixels, each with its
// own border correction (a variant of its own, so that the common path compiles as before).
template <int EPI, int CHUNKS, bool SUB>
__global__ void __launch_bounds__((2 + kRowsEW) * 32, 1) conv_rows_kernel(const __grid_constant__ RowsParams p) {
    extern __shared__ uint8_t smem_raw[];
    uint8_t *smem = smem_raw + ((1024u - (smem_u32(smem_raw) & 1023u)) & 1023u);
    const int S = p.stages;
    const RowsLayout L(S, p.kh * p.atoms, p.bn, p.ec, p.out_bytes);
    uint8_t *sA = smem + L.a;
    uint8_t *sB = smem + L.b;
    uint8_t *sOut = smem + L.out;
    long long *sK = reinterpret_cast<long long *>(smem + L.epi);
    int *sI = reinterpret_cast<int *>(sK + p.ec);
    const EpiSoA E{sK, sI, sI + p.ec, sI + 2 * p.ec, sI + 3 * p.ec, sI + 4 * p.ec, sI + 5 * p.ec};
    uint8_t *sLut = smem + L.lut;
    uint64_t *bars = reinterpret_cast<uint64_t *>(smem + L.bars);
    uint64_t *full = bars, *empty = bars + S;
    uint64_t *tfull = bars + 2 * S, *tempty = bars + 2 * S + kRowsMaxAcc, *drain = bars + 2 * S + 2 * kRowsMaxAcc;
    uint32_t *tmem_slot = reinterpret_cast<uint32_t *>(bars + 2 * S + 2 * kRowsMaxAcc + 1);
    volatile int *abort = reinterpret_cast<volatile int *>(tmem_slot + 1);
    const int warp = threadIdx.x / 32, lane = threadIdx.x % 32;

    if (threadIdx.x == 0) {
        for (int s = 0; s < S; s++) {
            mbar_init(smem_u32(full + s), 1);
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
    for (int i = threadIdx.x; i < p.ec; i += blockDim.x) {
        const EpiChan c = p.epi[SUB ? i % p.oc : i];
        sK[i] = c.k;
        sI[i] = c.m;
        sI[p.ec + i] = c.cut;
        sI[2 * p.ec + i] = c.sh;
        sI[3 * p.ec + i] = c.ls;
        sI[4 * p.ec + i] = c.bs;
        sI[5 * p.ec + i] = c.zadd;
    }
    if (p.post)
        for (int i = threadIdx.x; i < 256; i += blockDim.x) sLut[i] = p.post[i];
    {
        // the banded weights, resident for the whole kernel (read by the tensor core: async proxy)
        const size_t bbytes = (size_t)p.kh * p.atoms * p.bn * kBK;
        const uint4 *src = reinterpret_cast<const uint4 *>(p.w);
        for (size_t i = threadIdx.x; i < bbytes / 16; i += blockDim.x) st_shared16(smem_u32(sB) + (uint32_t)(i * 16), __ldg(src + i));
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
    const int per_group = p.row_tiles * p.groups;  // tiles per group of ipt images
    // Launched with programmatic serialization: the TMA and epilogue warps wait here for the
    // previous kernel's activations (the MMA warp touches only shared memory and TMEM).
    if (warp != 1) grid_dep_wait();

    if (warp == 0) {
        // ------------------------------------------------------------------ TMA producer
        if (lane == 0) {
            long long it = 0;
            bool ok = true;
            for (int t = blockIdx.x; t < p.tiles && ok; t += gridDim.x) {
                const int ig = t / per_group, rem = t - ig * per_group;
                const int rt = rem / p.groups, g = rem - rt * p.groups;
                const int x = p.x0 + g * p.gstep, oy0 = rt * p.R, img = ig * p.ipt;
                for (int kb = 0; kb < p.kh * p.atoms; kb++, it++) {  // K block kb: kernel row ky, atom a
                    const int ky = kb / p.atoms, a = kb - ky * p.atoms;
                    const int s = (int)(it % S);
                    if (!mbar_wait(smem_u32(empty + s), (uint32_t)(((it / S) & 1) ^ 1), abort, 201)) {
                        ok = false;
                        break;
                    }
                    mbar_expect_tx(smem_u32(full + s), (uint32_t)kStageBytes);
                    tma_load_3d(smem_u32(sA + (size_t)s * kStageBytes), &p.xmap[p.view[ky]], x + a * kBK,
                                oy0 + p.dy[ky], img, smem_u32(full + s));
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
            long long it = 0;
            bool ok = true;
            int lt = 0;
            for (int t = blockIdx.x; t < p.tiles && ok; t += gridDim.x, lt++) {
                const int acc = lt & (p.n_acc - 1);
                if (!mbar_wait(smem_u32(tempty + acc), (uint32_t)(((lt >> p.acc_shift) & 1) ^ 1), abort, 202)) break;
                tc_fence_after();
                const uint32_t tmem_d = tmem_base + (uint32_t)(acc * p.bn);
                for (int kb = 0; kb < p.kh * p.atoms; kb++, it++) {
                    const int a = kb % p.atoms;
                    const int s = (int)(it % S);
                    if (!mbar_wait(smem_u32(full + s), (uint32_t)((it / S) & 1), abort, 203)) {
                        ok = false;
                        break;
                    }
                    tc_fence_after();
                    const int ksteps = min(kBK, p.span - a * kBK + 31) / 32;  // 32-byte K steps of this atom
                    for (int kk = 0; kk < ksteps; kk++) {
                        const uint64_t ad = smem_desc(a0 + (uint32_t)(s * kStageBytes + kk * 32));
                        const uint64_t bd = smem_desc(b0 + (uint32_t)(kb * p.bn * kBK + kk * 32));
                        mma_i8(tmem_d, ad, bd, idesc, (kb | kk) ? 1u : 0u);
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
        // The 4 warps of a lane quarter split into fold groups of nparts: a warp takes column part
        // [part * box, part * box + box) of every fold-th tile, starting with tile ph. On narrow
        // tiles (nparts 1 or 2) a warp thus covers more columns per tile, and the per-tile fixed
        // costs (tile indices, masks, waits, store issue) are paid over more outputs.
        const int part = (e >> 2) % p.nparts, ph = (e >> 2) / p.nparts;
        constexpr int kBox = CHUNKS * 16;
        const int c0 = part * kBox;
        const uint8_t *lut = p.post ? sLut : nullptr;
        const int swz_row = kBox == 128 ? (lane & 7) : kBox == 64 ? ((lane >> 1) & 3) : kBox == 32 ? ((lane >> 2) & 1) : 0;
        const size_t wsb = rows_warp_stage(kBox);
        uint8_t *wstage0 = sOut + (size_t)e * 2 * wsb;
        // output pixel (within the group) and first channel of each chunk: fixed for the kernel
        int jj[CHUNKS], oo[CHUNKS];
#pragma unroll
        for (int ci = 0; ci < CHUNKS; ci++) {
            jj[ci] = (c0 + ci * 16) / p.oc;
            oo[ci] = c0 + ci * 16 - jj[ci] * p.oc;
        }
        // output columns whose taps all lie inside the image: [ox_lo, ox_hi]
        const int ox_lo = (p.pl + p.s - 1) / p.s, ox_hi = (p.iw - p.kw + p.pl) / p.s;
        int lt = ph, k = 0;
        for (int t = blockIdx.x + ph * gridDim.x; t < p.tiles; t += p.fold * gridDim.x, lt += p.fold, k++) {
            const int ig = t / per_group, rem = t - ig * per_group;
            const int rt = rem / p.groups, g = rem - rt * p.groups;
            const int oy0 = rt * p.R, ox0 = g * p.G;
            const int acc = lt & (p.n_acc - 1);
            if (!mbar_wait(smem_u32(tfull + acc), (uint32_t)((lt >> p.acc_shift) & 1), abort, 204)) break;
            tc_fence_after();
            // TMEM lane m = (image ig * ipt + m / R, row oy0 + m % R). A lane quarter covers rows
            // r0.. of one image when R >= 32, else 32 / R whole images (rows oy0 .. oy0 + R - 1).
            const int m0 = quarter * 32;
            const int r0 = oy0 + (p.R >= 32 ? m0 % p.R : 0);  // first output row of this warp
            const int img = ig * p.ipt + m0 / p.R;            // first image of this warp
            const bool live = r0 < p.oh;
            uint8_t *stage = wstage0 + (size_t)(k & 1) * wsb;
            // this buffer's previous store (two tiles back) must have been read out
            if (lane == 0) asm volatile("cp.async.bulk.wait_group.read 1;" ::: "memory");
            __syncwarp();
            if (live) {
                const int oy = p.R >= 32 ? r0 + lane : oy0 + lane % p.R;
                // kernel rows of this output row that fall outside the image
                int rmask = 0;
                for (int ky = 0; ky < p.kh; ky++) {
                    const int iy = p.s * oy - p.pt + ky;
                    rmask |= (iy < 0 || iy >= p.ih) ? 1 << ky : 0;
                }
                if (oy >= p.oh) rmask = 0;  // past the image: never stored
                const bool edge_cols = ox0 < ox_lo || ox0 + p.G - 1 > ox_hi;
                auto chunk = [&](const uint32_t(&rr)[16], int ci) {
                    uint32_t a[16];
#pragma unroll
                    for (int i = 0; i < 16; i++) a[i] = rr[i];
                    if (SUB && (rmask | (edge_cols ? 1 : 0))) {
                        // the chunk's 16 / oc pixels: each one's correction row, or -1 when all
                        // its taps lie inside the image
                        auto crow = [&](int q) {
                            if (q >= (16 >> p.loc)) return -1;
                            const int ox = ox0 + jj[ci] + q;
                            int cmask = 0;
                            for (int kx = 0; kx < p.kw; kx++) {
                                const int ix = p.s * ox - p.pl + kx;
                                cmask |= (ix < 0 || ix >= p.iw) ? 1 << kx : 0;
                            }
                            return (rmask | cmask) && ox < p.ow ? ((rmask << p.kw) | cmask) * p.oc + oo[ci] : -1;
                        };
                        const int r0c = crow(0), r1c = crow(1), r2c = crow(2), r3c = crow(3);
#pragma unroll
                        for (int i = 0; i < 16; i++) {
                            const int q = i >> p.loc;
                            const int o = q == 0 ? r0c : q == 1 ? r1c : q == 2 ? r2c : r3c;
                            if (o >= 0) a[i] = (uint32_t)((int32_t)a[i] + __ldg(p.corr + o + (i & ((1 << p.loc) - 1))));
                        }
                    } else if (!SUB && (rmask | (edge_cols ? 1 : 0))) {
                        const int ox = ox0 + jj[ci];
                        int cmask = 0;
                        for (int kx = 0; kx < p.kw; kx++) {
                            const int ix = p.s * ox - p.pl + kx;
                            cmask |= (ix < 0 || ix >= p.iw) ? 1 << kx : 0;
                        }
                        if ((rmask | cmask) && ox < p.ow) {
                            const int32_t *cr = p.corr + (size_t)((rmask << p.kw) | cmask) * p.oc + oo[ci];
#pragma unroll
                            for (int i = 0; i < 16; i++) a[i] = (uint32_t)((int32_t)a[i] + __ldg(cr + i));
                        }
                    }
                    const uint4 v = epilogue_chunk<EPI>(a, E, lut, oo[ci], p.lo, p.hi);
                    st_shared16(smem_u32(stage + (size_t)lane * kBox + ((ci ^ swz_row) << 4)), v);
                };
                const uint32_t taddr = tmem_base + ((uint32_t)(quarter * 32) << 16) + (uint32_t)(acc * p.bn + c0);
                uint32_t ra[16], rb[16];
                tmem_ld16_nowait(taddr, ra);
                tmem_wait_ld(ra);
#pragma unroll
                for (int ci = 0; ci < CHUNKS; ci += 2) {
                    if (ci + 1 < CHUNKS) tmem_ld16_nowait(taddr + (ci + 1) * 16, rb);
                    chunk(ra, ci);
                    if (ci + 1 < CHUNKS) {
                        tmem_wait_ld(rb);
                        if (ci + 2 < CHUNKS) tmem_ld16_nowait(taddr + (ci + 2) * 16, ra);
                        chunk(rb, ci + 1);
                        if (ci + 2 < CHUNKS) tmem_wait_ld(ra);
                    }
                }
            }
            tc_fence_before();
            fence_proxy_async();  // staged bytes visible to the TMA (async proxy)
            __syncwarp();
            if (lane == 0) {
                mbar_arrive(smem_u32(tempty + acc));  // accumulator free for reuse
                if (live)
                    asm volatile(
                        "cp.async.bulk.tensor.3d.global.shared::cta.bulk_group [%0, {%2, %3, %4}], [%1];" ::"l"(
                            reinterpret_cast<uint64_t>(&p.ymap)),
                        "r"(smem_u32(stage)), "r"(ox0 * p.oc + c0), "r"(r0), "r"(img)
                        : "memory");
                asm volatile("cp.async.bulk.commit_group;" ::: "memory");
            }
        }
        if (lane == 0) asm volatile("cp.async.bulk.wait_group 0;" ::: "memory");
    }

    tc_fence_before();
    __syncthreads();
    tc_fence_after();
    if (warp == 1) {
        asm volatile("tcgen05.dealloc.cta_group::1.sync.aligned.b32 %0, %1;" ::"r"(tmem_base), "r"(p.tmem_cols));
    }
}


}  // namespace

struct ConvRows {
    int sm_count = 148;  // of the device the op was prepared on
    RowsParams p{};
    size_t smem = 0;
    int epi_mode = kGeneral;
    int chunks = 4;  // 16-column chunks per epilogue warp
};

int conv_rows_prepare(const int8_t *w_packed, const int32_t *q, const uint8_t *post_dev, const ConvGeom &g,
                      const std::function<void *(size_t)> &alloc, ConvRows **out) {
    *out = nullptr;
    const char *env = std::getenv("UNOQ_CONV_ROWS");
    if (env && env[0] == '0') return 0;
    const int s = g.sh;
    const char *env_ic = std::getenv("UNOQ_CONV_ROWS_IC");  // widest input taken (default 64)
    const int max_ic = env_ic ? std::atoi(env_ic) : 64;
    if (g.ic < 1 || g.ic > max_ic || g.kh < 1 || g.kh > 3 || g.kw < 1 || g.kw > 3 || g.dh != 1 || g.dw != 1) return 0;
    if (g.sw != s || (s != 1 && s != 2)) return 0;
    if (!((g.oc % 16 == 0 && g.oc <= 256) || g.oc == 8 || g.oc == 4)) return 0;
    const int ec = g.oc < 16 ? 16 : g.oc;  // epilogue constant entries (see RowsParams::ec)
    if (g.pt < 0 || g.pt >= g.kh || g.pl < 0 || g.pl >= g.kw) return 0;
    const long long row_bytes = (long long)g.iw * g.ic;
    if (row_bytes % 16 != 0 || ((long long)g.ow * g.oc) % 16 != 0) return 0;  // tensor-map strides: 16-byte units
    if ((long long)g.ih * row_bytes >= (1ll << 31) || (long long)g.oh * g.ow * g.oc >= (1ll << 31)) return 0;
    // window offset of every group (constant because a group advances by whole 16-byte units)
    const int o = (((-g.pl * g.ic) % 16) + 16) % 16;
    // G output pixels per column group: the most (a power of two) whose window fits the fewest
    // 128-byte K blocks per kernel row (one for few channels, up to four for 64), with bn = G * oc
    // split into 16 / 32 / 48 / 64 columns per epilogue warp (48-byte staging rows are stored
    // unswizzled: their 16-byte lanes still fall in distinct banks) and the banded weights
    // resident. Inputs of 33-64 channels only with oc <= 32, where band-mode tiles are narrowest
    // (64 -> 16 channels: 2.2x faster than band mode; 64 -> 64 stride 2: 9% slower)
    const int ew = kRowsEW;
    const int max_atoms = g.ic <= 32 ? 3 : (g.oc <= 32 ? 4 : 0);
    // Among the (G, atoms) whose window fits and whose layout fits shared memory with two stages,
    // the fewest K blocks per output pixel (atoms / G: A bytes loaded and MMA work per output),
    // then the fewest atoms. 32 -> 32 channels, 3x3 stride 2 thus takes G = 4 over 3 atoms rather
    // than G = 2 over 2 (UNOQ_CONV_ROWS_ATOMS=2 restores the old two-atom limit).
    const char *env_atoms = std::getenv("UNOQ_CONV_ROWS_ATOMS");
    const int atom_cap = env_atoms ? std::atoi(env_atoms) : max_atoms;
    int G = 0, atoms = 0;
    for (int na = 1; na <= max_atoms && na <= atom_cap; na++)
        for (int c = 256 / g.oc; c >= 1; c /= 2) {
            if (G && na * G >= atoms * c) break;  // not fewer blocks per pixel than the choice so far
            const int b = c * g.oc / (ew / 4);
            if ((s * g.ic * c) % 16 != 0 || (b != 16 && b != 32 && b != 48 && b != 64)) continue;
            if (o + s * g.ic * (c - 1) + g.kw * g.ic > na * kBK) continue;
            // the narrowest staging the epilogue split allows (nparts = ew / 4)
            const int ob = (int)(2 * ew * rows_warp_stage(b));
            if (RowsLayout(2, g.kh * na, c * g.oc, ec, ob).total > (size_t)kRowsMaxSmem) continue;
            G = c, atoms = na;
            break;
        }
    if (!G) return 0;
    const int bn = G * g.oc;
    const int span = o + s * g.ic * (G - 1) + g.kw * g.ic;
    // Epilogue split: the fewest warps per tile (nparts of each lane quarter) whose column part is
    // at most 64 columns and a staging width the swizzle / bank rules take (16 / 32 / 48 / 64); the
    // other warps of the quarter take the next tiles (fold = 4 / nparts tiles in flight), over a
    // ring of as many accumulators as TMEM holds (up to 8). UNOQ_CONV_ROWS_FOLD=0 keeps one tile
    // per quarter (every warp a quarter of the tile's columns).
    const char *env_fold = std::getenv("UNOQ_CONV_ROWS_FOLD");
    const bool allow_fold = !(env_fold && env_fold[0] == '0');
    int nparts = ew / 4, box = bn / nparts, stages = 4, out_bytes = 0;
    for (int np = allow_fold ? 1 : ew / 4; np <= ew / 4; np *= 2) {
        const int b = bn / np;
        if (bn % np || (b != 16 && b != 32 && b != 48 && b != 64)) continue;
        const int ob = (int)(2 * ew * rows_warp_stage(b));
        if (RowsLayout(2, g.kh * atoms, bn, ec, ob).total > (size_t)kRowsMaxSmem) continue;
        nparts = np, box = b;
        break;
    }
    out_bytes = (int)(2 * ew * rows_warp_stage(box));
    while (stages > 2 && RowsLayout(stages, g.kh * atoms, bn, ec, out_bytes).total > (size_t)kRowsMaxSmem) stages--;
    const RowsLayout L(stages, g.kh * atoms, bn, ec, out_bytes);
    if (L.total > (size_t)kRowsMaxSmem) return 0;
    int n_acc = 2;
    while (n_acc * 2 <= kRowsMaxAcc && n_acc * 2 * bn <= 512) n_acc *= 2;

    // Weights: reference packed layout (gemm.h:9), reduction index t = (ky*kw + kx)*ic + c
    // (tflite.py:155), into the banded B matrix, one SW128 K-major block per (kernel row, atom).
    const int kp = q[18], oc = g.oc, K = g.kh * g.kw * g.ic;
    auto wref = [&](int j, int t) -> int { return w_packed[(j / 4) * kp * 4 + (t / 8) * 32 + (j % 4) * 8 + t % 8]; };
    std::vector<uint8_t> wt((size_t)g.kh * atoms * bn * kBK, 0);
    for (int ky = 0; ky < g.kh; ky++)
        for (int n = 0; n < bn; n++) {
            const int j = n / oc, ch = n % oc;
            for (int kx = 0; kx < g.kw; kx++)
                for (int c = 0; c < g.ic; c++) {
                    const int bw = o + s * g.ic * j + kx * g.ic + c;  // byte of the window
                    const int a = bw / kBK, b = bw % kBK, chunk = b / 16;
                    const size_t off = ((size_t)(ky * atoms + a) * bn + (n / 8) * 8) * kBK + (n % 8) * kBK +
                                       ((chunk ^ (n % 8)) * 16) + b % 16;
                    wt[off] = (uint8_t)(int8_t)wref(ch, (ky * g.kw + kx) * g.ic + c);
                }
        }
    const int32_t *cbias = q + kHead, *mult = cbias + oc, *shift = mult + oc;
    const int xzp = q[12], yzp = q[13];
    std::vector<EpiChan> epi(oc);
    for (int j = 0; j < oc; j++) {
        long long sum_all = 0, sum_pad = 0;
        for (int t = 0; t < kp; t++) {
            const int v = wref(j, t);
            sum_all += v;
            if (t >= K) sum_pad += v;
        }
        epi[j] = make_epilogue((long long)cbias[j] + 128ll * sum_all + (long long)xzp * sum_pad, mult[j], shift[j], yzp);
    }
    bool fast = true;
    for (int j = 0; j < oc; j++) fast &= epi_fast(epi[j]);
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
    const bool attrs = once_per_device(kFamilyConvRows, [] {
        auto allow = [](auto fn) {
            return cudaFuncSetAttribute(fn, cudaFuncAttributeMaxDynamicSharedMemorySize, kRowsMaxSmem) == cudaSuccess;
        };
        auto allow_all = [&](auto sub) {
            constexpr bool SB = decltype(sub)::value;
            return allow(conv_rows_kernel<kRelu, 1, SB>) && allow(conv_rows_kernel<kTies, 1, SB>) &&
                   allow(conv_rows_kernel<kGeneral, 1, SB>) && allow(conv_rows_kernel<kRelu, 2, SB>) &&
                   allow(conv_rows_kernel<kTies, 2, SB>) && allow(conv_rows_kernel<kGeneral, 2, SB>) &&
                   allow(conv_rows_kernel<kRelu, 3, SB>) && allow(conv_rows_kernel<kTies, 3, SB>) &&
                   allow(conv_rows_kernel<kGeneral, 3, SB>) && allow(conv_rows_kernel<kRelu, 4, SB>) &&
                   allow(conv_rows_kernel<kTies, 4, SB>) && allow(conv_rows_kernel<kGeneral, 4, SB>);
        };
        return allow_all(std::false_type{}) && allow_all(std::true_type{});
    });
    if (!attrs) return 2001;
    ConvRows *c = new ConvRows();
    c->sm_count = current_sm_count();
    RowsParams &p = c->p;
    p.w = static_cast<const int8_t *>(dw);
    p.epi = static_cast<const EpiChan *>(de);
    p.corr = static_cast<const int32_t *>(dc);
    p.post = post_dev;
    p.ih = g.ih, p.iw = g.iw, p.ic = g.ic, p.oh = g.oh, p.ow = g.ow, p.oc = g.oc;
    p.ec = ec;
    p.loc = g.oc == 4 ? 2 : g.oc == 8 ? 3 : 4;
    p.kh = g.kh, p.kw = g.kw, p.s = s, p.pt = g.pt, p.pl = g.pl;
    p.G = G;
    p.bn = bn;
    p.groups = (g.ow + G - 1) / G;
    // rows per image in an M tile: the power of two R in [8, 128] that leaves the fewest computed
    // rows past the image (ties: larger R); the tile then holds R rows of 128 / R images
    {
        int best = kBM;
        auto waste = [&](int r) { return (double)(((g.oh + r - 1) / r) * r - g.oh) / ((g.oh + r - 1) / r * r); };
        for (int r = kBM / 2; r >= 8; r /= 2)
            if (waste(r) < waste(best) - 1e-9) best = r;
        p.R = best;
        p.ipt = kBM / best;
    }
    p.row_tiles = (g.oh + p.R - 1) / p.R;
    p.span = span;
    p.atoms = atoms;
    p.x0 = -g.pl * g.ic - o;  // = (s*0 - pl)*ic rounded down to 16 bytes
    p.gstep = s * g.ic * G;
    for (int ky = 0; ky < g.kh; ky++) {
        const int r = ky - g.pt;  // input row = s*oy + r
        const int v = ((r % s) + s) % s;
        p.view[ky] = v;
        p.dy[ky] = (r - v) / s;
    }
    p.stages = stages;
    p.lo = q[14], p.hi = q[15];
    p.box = box;
    p.swz = box == 128 ? 3 : box == 64 ? 2 : box == 32 ? 1 : 0;
    p.out_bytes = out_bytes;
    p.nparts = nparts;
    p.fold = (ew / 4) / nparts;
    p.n_acc = n_acc;
    p.acc_shift = n_acc == 8 ? 3 : n_acc == 4 ? 2 : 1;
    int cols = 32;
    while (cols < n_acc * bn) cols *= 2;
    p.tmem_cols = cols;
    c->smem = L.total;
    c->epi_mode = epi_mode;
    c->chunks = box / 16;
    *out = c;
    return 0;
}

int conv_rows_launch(const ConvRows &c, const int8_t *x, int8_t *y, const ConvGeom &g, cudaStream_t s) {
    RowsParams p = c.p;
    p.n = g.n;
    const long long igroups = (g.n + p.ipt - 1) / p.ipt;
    if (igroups * p.row_tiles * p.groups >= (1ll << 31)) return 2001;
    p.tiles = (int)(igroups * p.row_tiles * p.groups);
    EncodeTiled enc = encoder();
    if (!enc) return 2001;
    const cuuint64_t row_bytes = (cuuint64_t)g.iw * g.ic, img_bytes = row_bytes * (cuuint64_t)g.ih;
    for (int v = 0; v < p.s; v++) {
        // view v: input rows v, v + s, ... of every image
        const cuuint64_t dims[3] = {row_bytes, (cuuint64_t)((g.ih - v + p.s - 1) / p.s), (cuuint64_t)g.n};
        const cuuint64_t strides[2] = {row_bytes * (cuuint64_t)p.s, img_bytes};
        const cuuint32_t box[3] = {(cuuint32_t)kBK, (cuuint32_t)p.R, (cuuint32_t)p.ipt};
        const cuuint32_t estr[3] = {1, 1, 1};
        if (enc(&p.xmap[v], CU_TENSOR_MAP_DATA_TYPE_UINT8, 3, const_cast<int8_t *>(x) + (size_t)v * row_bytes, dims, strides,
                box, estr, CU_TENSOR_MAP_INTERLEAVE_NONE, CU_TENSOR_MAP_SWIZZLE_128B, CU_TENSOR_MAP_L2_PROMOTION_L2_128B,
                CU_TENSOR_MAP_FLOAT_OOB_FILL_NONE) != CUDA_SUCCESS)
            return 2001;
    }
    {
        const cuuint64_t dims[3] = {(cuuint64_t)g.ow * g.oc, (cuuint64_t)g.oh, (cuuint64_t)g.n};
        const cuuint64_t strides[2] = {(cuuint64_t)g.ow * g.oc, (cuuint64_t)g.oh * g.ow * g.oc};
        // one lane quarter: 32 rows of one image, or R rows of 32 / R images
        const cuuint32_t box[3] = {(cuuint32_t)p.box, (cuuint32_t)std::min(p.R, 32), (cuuint32_t)std::max(1, 32 / p.R)};
        const cuuint32_t estr[3] = {1, 1, 1};
        const CUtensorMapSwizzle sw = p.swz == 3   ? CU_TENSOR_MAP_SWIZZLE_128B
                                      : p.swz == 2 ? CU_TENSOR_MAP_SWIZZLE_64B
                                      : p.swz == 1 ? CU_TENSOR_MAP_SWIZZLE_32B
                                                   : CU_TENSOR_MAP_SWIZZLE_NONE;
        if (enc(&p.ymap, CU_TENSOR_MAP_DATA_TYPE_UINT8, 3, y, dims, strides, box, estr, CU_TENSOR_MAP_INTERLEAVE_NONE, sw,
                CU_TENSOR_MAP_L2_PROMOTION_NONE, CU_TENSOR_MAP_FLOAT_OOB_FILL_NONE) != CUDA_SUCCESS)
            return 2001;
    }
    const int grid = std::min(c.sm_count, p.tiles);
    constexpr int T = (2 + kRowsEW) * 32;
    auto go = [&](auto chunks) {
        constexpr int CH = decltype(chunks)::value;
        auto run = [&](auto sub) {
            constexpr bool SB = decltype(sub)::value;
            if (c.epi_mode == kRelu) launch_pdl(kPdlConvRows, conv_rows_kernel<kRelu, CH, SB>, grid, T, c.smem, s, p);
            else if (c.epi_mode == kTies) launch_pdl(kPdlConvRows, conv_rows_kernel<kTies, CH, SB>, grid, T, c.smem, s, p);
            else launch_pdl(kPdlConvRows, conv_rows_kernel<kGeneral, CH, SB>, grid, T, c.smem, s, p);
        };
        if (p.oc < 16) run(std::true_type{});
        else run(std::false_type{});
    };
    if (c.chunks == 4) go(std::integral_constant<int, 4>{});
    else if (c.chunks == 3) go(std::integral_constant<int, 3>{});
    else if (c.chunks == 2) go(std::integral_constant<int, 2>{});
    else go(std::integral_constant<int, 1>{});
    return 0;
}

void conv_rows_free(ConvRows *c) { delete c; }

int conv_rows_error(bool reset) {
    int v = 0;
    cudaMemcpyFromSymbol(&v, g_tc_error, sizeof(int));
    if (reset && v) {
        int z = 0;
        cudaMemcpyToSymbol(g_tc_error, &z, sizeof(int));
    }
    return v;
}

}  // namespace uq
