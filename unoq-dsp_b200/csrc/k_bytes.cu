// k_bytes.cu -- byte-movement and small integer ops of the plan, vectorised.
//
// Plan codes 10 (transpose), 16 (pool), 19 (pack), 20 (concat), 21 (nearest resize),
// 26 (slice) and 27 (bmm) (runtime/graph.c:306-391, qnn.c:119-153, 1228-1245). All are exact byte
// permutations or integer arithmetic; results are bit-identical to the reference.
//
// The movement kernels work in the widest unit (16, 4 or 1 bytes) that every run length, offset
// and base address allows, and decode indices once per unit rather than once per byte:
//  * slice / concat / pack: strided copies of contiguous runs (a channel range of each pixel, a
//    block of rows, a whole segment);
//  * transpose: a permutation that reduces to a batched 2-D transpose after merging adjacent
//    axes goes through a shared-memory tile; any other permutation uses the element-wise path;
//  * resize: one output pixel's channels per run, from the prepared row / column offsets;
//  * max pool: 16 channels per thread with __vmaxs4.
// bmm keeps a whole batch matrix's operands (zero points subtracted) in shared memory and gives
// each thread a 4 x 4 register tile; large matrices use a 32 x 32 tiled path.
#include <algorithm>

#include "kernels.cuh"

namespace uq {

namespace {

constexpr int kT = 256;

inline int unit_for(uint64_t a, uint64_t b = 0, uint64_t c = 0, uint64_t d = 0) {
    const uint64_t m = a | b | c | d;
    return (m & 15) == 0 ? 16 : (m & 3) == 0 ? 4 : 1;
}

template <int V>
struct Unit;
template <>
struct Unit<16> {
    using T = uint4;
};
template <>
struct Unit<4> {
    using T = uint32_t;
};
template <>
struct Unit<1> {
    using T = uint8_t;
};

// ---------------------------------------------------------------- strided run copy -----------
// Row r (r = sum idx_d * prod(extent[d+1..])) copies `run` bytes from
// src + base + sum idx_d * stride[d] to dst + r * dst_stride + dst_base.
struct RunCopy {
    int ndim;
    uint32_t extent[4];
    uint64_t stride[4];
    uint64_t base, dst_stride, dst_base;
    uint64_t rows;
    uint32_t run;
};

template <int V>
__global__ void run_copy_kernel(const uint8_t *__restrict__ src, uint8_t *__restrict__ dst, RunCopy rc) {
    using T = typename Unit<V>::T;
    const uint32_t per_row = rc.run / V;
    const uint64_t units = rc.rows * per_row;
    for (uint64_t u = (uint64_t)blockIdx.x * blockDim.x + threadIdx.x; u < units; u += (uint64_t)gridDim.x * blockDim.x) {
        const uint64_t row = u / per_row;
        const uint32_t col = (uint32_t)(u - row * per_row);
        uint64_t rem = row, off = rc.base;
        for (int d = rc.ndim - 1; d >= 0; d--) {
            const uint64_t idx = rem % rc.extent[d];
            rem /= rc.extent[d];
            off += idx * rc.stride[d];
        }
        reinterpret_cast<T *>(dst + rc.dst_base + row * rc.dst_stride)[col] = reinterpret_cast<const T *>(src + off)[col];
    }
}

void run_copy(const uint8_t *src, uint8_t *dst, const RunCopy &rc, cudaStream_t s) {
    if (!rc.rows || !rc.run) return;
    uint64_t strides = 0;
    for (int d = 0; d < rc.ndim; d++) strides |= rc.stride[d];
    const int v = unit_for(rc.run, rc.base | strides, rc.dst_stride | rc.dst_base,
                           reinterpret_cast<uintptr_t>(src) | reinterpret_cast<uintptr_t>(dst));
    const uint64_t units = rc.rows * (rc.run / v);
    if (v == 16) run_copy_kernel<16><<<grid_for(units, kT), kT, 0, s>>>(src, dst, rc);
    else if (v == 4) run_copy_kernel<4><<<grid_for(units, kT), kT, 0, s>>>(src, dst, rc);
    else run_copy_kernel<1><<<grid_for(units, kT), kT, 0, s>>>(src, dst, rc);
}

// ---------------------------------------------------------------- concat (code 20) -----------
template <int V>
__global__ void concat_kernel(const uint8_t *__restrict__ a, const uint8_t *__restrict__ b, uint8_t *__restrict__ z,
                              uint64_t outer, uint32_t ac, uint32_t bc) {
    using T = typename Unit<V>::T;
    const uint32_t ua = ac / V, ub = bc / V, row = ua + ub;
    const uint64_t units = outer * row;
    for (uint64_t u = (uint64_t)blockIdx.x * blockDim.x + threadIdx.x; u < units; u += (uint64_t)gridDim.x * blockDim.x) {
        const uint64_t r = u / row;
        const uint32_t c = (uint32_t)(u - r * row);
        reinterpret_cast<T *>(z)[u] = c < ua ? reinterpret_cast<const T *>(a)[r * ua + c]
                                             : reinterpret_cast<const T *>(b)[r * ub + (c - ua)];
    }
}

// Concat chain: up to 8 inputs along the innermost axis; the inputs' row widths are staged in
// shared memory so the input lookup indexes no kernel parameter dynamically.
template <int V>
__global__ void concat_multi_kernel(const ConcatInputs in, uint8_t *__restrict__ z, uint64_t rows, uint32_t row_units) {
    using T = typename Unit<V>::T;
    __shared__ const T *src[8];
    __shared__ uint32_t units[8];
    if (threadIdx.x < 8) {
        src[threadIdx.x] = threadIdx.x < (unsigned)in.count ? reinterpret_cast<const T *>(in.src[threadIdx.x]) : nullptr;
        units[threadIdx.x] = threadIdx.x < (unsigned)in.count ? in.width[threadIdx.x] / V : 0u;
    }
    __syncthreads();
    const uint64_t total = rows * row_units;
    for (uint64_t u = (uint64_t)blockIdx.x * blockDim.x + threadIdx.x; u < total; u += (uint64_t)gridDim.x * blockDim.x) {
        const uint64_t r = u / row_units;
        uint32_t c = (uint32_t)(u - r * row_units);
        int i = 0;
        while (c >= units[i]) c -= units[i++];
        reinterpret_cast<T *>(z)[u] = src[i][r * units[i] + c];
    }
}

// Concat chain whose parts may read a slice of a wider row and map it through a byte table (the
// concat absorbed the table ops that only it read).
template <int V>
__global__ void concat_parts_kernel(const ConcatParts in, uint8_t *__restrict__ z, uint64_t rows, uint32_t row_units) {
    using T = typename Unit<V>::T;
    __shared__ uint8_t tab[8][256];
    __shared__ const uint8_t *src[8];
    __shared__ uint32_t units[8], in_w[8], off[8], flip[8];
    __shared__ int mapped[8];
    if (threadIdx.x < 8) {
        const int k = threadIdx.x;
        const bool live = k < in.count;
        src[k] = live ? in.src[k] : nullptr;
        units[k] = live ? in.out_w[k] / V : 0u;
        in_w[k] = live ? in.in_w[k] : 0u;
        off[k] = live ? in.off[k] : 0u;
        flip[k] = live ? in.flip[k] : 0u;
        mapped[k] = live && in.table[k] != nullptr;
    }
    for (int k = 0; k < in.count; k++)
        if (in.table[k])
            for (int i = threadIdx.x; i < 256; i += blockDim.x) tab[k][i] = in.table[k][i];
    __syncthreads();
    const uint64_t total = rows * row_units;
    for (uint64_t u = (uint64_t)blockIdx.x * blockDim.x + threadIdx.x; u < total; u += (uint64_t)gridDim.x * blockDim.x) {
        const uint64_t r = u / row_units;
        uint32_t c = (uint32_t)(u - r * row_units);
        int i = 0;
        while (c >= units[i]) c -= units[i++];
        T v = *reinterpret_cast<const T *>(src[i] + r * in_w[i] + off[i] + (size_t)c * V);
        if (mapped[i]) {
            uint8_t *b = reinterpret_cast<uint8_t *>(&v);
#pragma unroll
            for (int k = 0; k < V; k++) b[k] = tab[i][b[k] ^ flip[i]];
        }
        reinterpret_cast<T *>(z)[u] = v;
    }
}

// Slice of the innermost axis followed by a byte table, in one pass.
template <int V>
__global__ void lut_rows_kernel(const uint8_t *__restrict__ x, uint8_t *__restrict__ y, uint64_t rows, uint32_t in_w,
                                uint32_t off, uint32_t out_w, const uint8_t *__restrict__ table, unsigned flip) {
    using T = typename Unit<V>::T;
    __shared__ uint8_t t[256];
    for (int i = threadIdx.x; i < 256; i += blockDim.x) t[i] = table[i];
    __syncthreads();
    const uint32_t per_row = out_w / V;
    const uint64_t total = rows * per_row;
    for (uint64_t u = (uint64_t)blockIdx.x * blockDim.x + threadIdx.x; u < total; u += (uint64_t)gridDim.x * blockDim.x) {
        const uint64_t r = u / per_row;
        const uint32_t c = (uint32_t)(u - r * per_row) * V;
        T v = *reinterpret_cast<const T *>(x + r * in_w + off + c);
        uint8_t *b = reinterpret_cast<uint8_t *>(&v);
#pragma unroll
        for (int k = 0; k < V; k++) b[k] = t[b[k] ^ flip];
        *reinterpret_cast<T *>(y + r * out_w + c) = v;
    }
}

// ---------------------------------------------------------------- transpose (code 10) --------
// Batched 2-D transpose of elements of `E` bytes: z[b][c][r] = a[b][r][c].
template <int E>
__global__ void transpose2d_kernel(const uint8_t *__restrict__ a, uint8_t *__restrict__ z, uint32_t batches, uint32_t rows,
                                   uint32_t cols) {
    using T = typename Unit<E>::T;
    __shared__ T tile[32][33];
    const uint32_t tiles_r = (rows + 31) / 32, tiles_c = (cols + 31) / 32;
    const uint64_t tiles = (uint64_t)batches * tiles_r * tiles_c;
    for (uint64_t t = blockIdx.x; t < tiles; t += gridDim.x) {
        const uint32_t tc = (uint32_t)(t % tiles_c), tr = (uint32_t)((t / tiles_c) % tiles_r);
        const uint64_t bt = t / ((uint64_t)tiles_c * tiles_r);
        const T *src = reinterpret_cast<const T *>(a) + bt * rows * cols;
        T *dst = reinterpret_cast<T *>(z) + bt * rows * cols;
        const uint32_t c = tc * 32 + threadIdx.x % 32;
        for (uint32_t i = threadIdx.x / 32; i < 32; i += blockDim.x / 32) {
            const uint32_t r = tr * 32 + i;
            if (r < rows && c < cols) tile[i][threadIdx.x % 32] = src[(uint64_t)r * cols + c];
        }
        __syncthreads();
        const uint32_t r = tr * 32 + threadIdx.x % 32;
        for (uint32_t i = threadIdx.x / 32; i < 32; i += blockDim.x / 32) {
            const uint32_t cc = tc * 32 + i;
            if (r < rows && cc < cols) dst[(uint64_t)cc * rows + r] = tile[threadIdx.x % 32][i];
        }
        __syncthreads();
    }
}

// Byte transpose for rows % 4 == 0 and cols % 4 == 0 with 4-byte aligned buffers. A block stages
// `per` whole matrices (contiguous in memory) in shared memory with an odd word stride per row,
// then each thread transposes a 4 x 4 byte block in registers with byte permutes and writes one
// word into each of four output rows; consecutive lanes take consecutive 4-byte runs of an output
// row, so both the global loads and the global stores are contiguous across a warp.
constexpr int kTrSmem = 40 * 1024;

__global__ void transpose_b4_kernel(const uint32_t *__restrict__ a, uint32_t *__restrict__ z, uint32_t batches,
                                    uint32_t rows, uint32_t cols, uint32_t per, FastDiv div_cw, FastDiv div_blocks,
                                    FastDiv div_rb) {
    extern __shared__ uint32_t tsm[];
    const uint32_t cw = cols / 4, cs = cw | 1, rb = rows / 4;
    const uint32_t mat_words = rows * cw, blocks_per = rb * cw;
    const uint32_t chunks = (batches + per - 1) / per;
    for (uint32_t ch = blockIdx.x; ch < chunks; ch += gridDim.x) {
        const uint32_t m0 = ch * per, cnt = min(per, batches - m0);
        const uint32_t *src = a + (size_t)m0 * mat_words;
        uint32_t *dst = z + (size_t)m0 * mat_words;
        for (uint32_t g = threadIdx.x; g < cnt * mat_words; g += blockDim.x) {
            const uint32_t row = (uint32_t)div_cw.div((int)g);
            tsm[row * cs + (g - row * cw)] = __ldg(src + g);
        }
        __syncthreads();
        for (uint32_t q = threadIdx.x; q < cnt * blocks_per; q += blockDim.x) {
            const uint32_t mat = (uint32_t)div_blocks.div((int)q), rem = q - mat * blocks_per;
            const uint32_t cb = (uint32_t)div_rb.div((int)rem), r = rem - cb * rb;
            const uint32_t *t = tsm + (mat * rows + 4 * r) * cs + cb;
            const uint32_t v0 = t[0], v1 = t[cs], v2 = t[2 * cs], v3 = t[3 * cs];
            const uint32_t t0 = __byte_perm(v0, v1, 0x5140), t1 = __byte_perm(v0, v1, 0x7362);
            const uint32_t t2 = __byte_perm(v2, v3, 0x5140), t3 = __byte_perm(v2, v3, 0x7362);
            uint32_t *d = dst + (size_t)mat * mat_words + (size_t)(4 * cb) * rb + r;
            d[0] = __byte_perm(t0, t2, 0x5410);
            d[rb] = __byte_perm(t0, t2, 0x7632);
            d[2 * rb] = __byte_perm(t1, t3, 0x5410);
            d[3 * rb] = __byte_perm(t1, t3, 0x7632);
        }
        __syncthreads();
    }
}

struct Perm5 {
    int p[5];
};

__global__ void permute_kernel(const uint8_t *__restrict__ a, uint8_t *__restrict__ z, Shape5 in, Perm5 pm, int elem,
                               uint64_t count) {
    const int *perm = pm.p;
    uint64_t istride[5];
    uint64_t acc = 1;
    for (int d = in.rank - 1; d >= 0; d--) {
        istride[d] = acc;
        acc *= in.d[d];
    }
    for (uint64_t i = (uint64_t)blockIdx.x * blockDim.x + threadIdx.x; i < count; i += (uint64_t)gridDim.x * blockDim.x) {
        uint64_t rem = i, src = 0;
        for (int d = in.rank - 1; d >= 0; d--) {
            const uint32_t extent = in.d[perm[d]];
            const uint64_t idx = rem % extent;
            rem /= extent;
            src += idx * istride[perm[d]];
        }
        for (int e = 0; e < elem; e++) z[i * elem + e] = a[src * elem + e];
    }
}

// ---------------------------------------------------------------- resize (code 21) -----------
template <int V>
__global__ void resize_kernel(const uint8_t *__restrict__ a, uint8_t *__restrict__ z, uint64_t pixels, int oh, int ow,
                              uint32_t c, uint64_t img_bytes, const uint32_t *__restrict__ offsets) {
    using T = typename Unit<V>::T;
    const uint32_t per = c / V;
    const uint64_t units = pixels * per;
    for (uint64_t u = (uint64_t)blockIdx.x * blockDim.x + threadIdx.x; u < units; u += (uint64_t)gridDim.x * blockDim.x) {
        const uint64_t pix = u / per;
        const uint32_t k = (uint32_t)(u - pix * per);
        const int x = (int)(pix % ow), y = (int)((pix / ow) % oh);
        const uint64_t img = pix / ((uint64_t)ow * oh);
        const uint8_t *src = a + img * img_bytes + offsets[y] + offsets[oh + x];
        reinterpret_cast<T *>(z)[u] = reinterpret_cast<const T *>(src)[k];
    }
}

// ---------------------------------------------------------------- pool (code 16) -------------
// Max starts at -128 and takes valid taps; average sums raw int8 over valid taps and rounds
// half away from zero with truncating division (qnn.c:1228-1243; global_pool9 agrees).
__global__ void pool_kernel(const int8_t *__restrict__ x, int8_t *__restrict__ y, ConvGeom g, int is_max, int lo, int hi) {
    const uint64_t total = (uint64_t)g.n * g.oh * g.ow * g.oc;
    for (uint64_t idx = (uint64_t)blockIdx.x * blockDim.x + threadIdx.x; idx < total;
         idx += (uint64_t)gridDim.x * blockDim.x) {
        const int c = (int)(idx % g.oc);
        const uint64_t pix = idx / g.oc;
        const int ox = (int)(pix % g.ow);
        const int oy = (int)((pix / g.ow) % g.oh);
        const uint64_t n = pix / ((uint64_t)g.ow * g.oh);
        int acc = is_max ? -128 : 0, count = 0;
        for (int ky = 0; ky < g.kh; ky++) {
            const int iy = oy * g.sh - g.pt + ky;
            if (iy < 0 || iy >= g.ih) continue;
            for (int kx = 0; kx < g.kw; kx++) {
                const int ix = ox * g.sw - g.pl + kx;
                if (ix < 0 || ix >= g.iw) continue;
                const int v = x[((n * g.ih + iy) * g.iw + ix) * g.ic + c];
                count++;
                if (is_max) acc = v > acc ? v : acc;
                else acc += v;
            }
        }
        if (!is_max) {
            const int half = count / 2;
            acc = count ? (acc + (acc > 0 ? half : -half)) / count : 0;
        }
        y[idx] = (int8_t)dev_clamp(acc, lo, hi);
    }
}

// Max pool, 16 channels per thread (ic % 16 == 0): byte-wise signed max, then the clamp.
__global__ void maxpool16_kernel(const int8_t *__restrict__ x, int8_t *__restrict__ y, ConvGeom g, uint32_t lo4,
                                 uint32_t hi4) {
    const int c16 = g.oc / 16;
    const uint64_t total = (uint64_t)g.n * g.oh * g.ow * c16;
    for (uint64_t u = (uint64_t)blockIdx.x * blockDim.x + threadIdx.x; u < total; u += (uint64_t)gridDim.x * blockDim.x) {
        const int cg = (int)(u % c16);
        const uint64_t pix = u / c16;
        const int ox = (int)(pix % g.ow), oy = (int)((pix / g.ow) % g.oh);
        const uint64_t n = pix / ((uint64_t)g.ow * g.oh);
        uint4 m = make_uint4(0x80808080u, 0x80808080u, 0x80808080u, 0x80808080u);
        for (int ky = 0; ky < g.kh; ky++) {
            const int iy = oy * g.sh - g.pt + ky;
            if (iy < 0 || iy >= g.ih) continue;
            for (int kx = 0; kx < g.kw; kx++) {
                const int ix = ox * g.sw - g.pl + kx;
                if (ix < 0 || ix >= g.iw) continue;
                const uint4 v = __ldg(reinterpret_cast<const uint4 *>(x + ((n * g.ih + iy) * g.iw + ix) * g.ic) + cg);
                m.x = __vmaxs4(m.x, v.x);
                m.y = __vmaxs4(m.y, v.y);
                m.z = __vmaxs4(m.z, v.z);
                m.w = __vmaxs4(m.w, v.w);
            }
        }
        m.x = __vmins4(__vmaxs4(m.x, lo4), hi4);
        m.y = __vmins4(__vmaxs4(m.y, lo4), hi4);
        m.z = __vmins4(__vmaxs4(m.z, lo4), hi4);
        m.w = __vmins4(__vmaxs4(m.w, lo4), hi4);
        reinterpret_cast<uint4 *>(y + pix * g.oc)[cg] = m;
    }
}

// ---------------------------------------------------------------- bmm (code 27) --------------
// qnn.c:119-153 computes sum (x + 128) w - (xz + 128) sum w - wz sum (x + 128) + k (xz + 128) wz
// in wrapping int32, which is sum (x - xz)(w - wz) = sum x w - wz sum x - xz sum w + k xz wz. The
// small-matrix kernel takes that last form: block = one batch matrix, up to `rows_cap` output rows
// at a time, both operands raw int8 in shared memory packed four reduction steps to a word (zero
// padded, X rows x K, W K x N, both K-major per output index, odd word stride per row), sum x w
// through __dp4a, the row sums of X and column sums of W once per block. Each thread accumulates a
// 4 x 4 register tile whose rows and columns lie a quarter of the block's extent apart, so the lanes
// of a warp read consecutive W rows (distinct banks) and share X rows (broadcast). Matrices too
// large for the shared-memory budget use the 32 x 32 tiled path.
constexpr int kBmmSmem = 48 * 1024;

__host__ __device__ inline size_t bmm_small_smem(int n, int k, int rows_cap) {
    const size_t kp = (size_t)((k + 3) / 4) | 1;
    return ((size_t)n + rows_cap) * (kp + 1) * sizeof(int32_t);
}

__global__ void bmm_small_kernel(const int8_t *__restrict__ x, const int8_t *__restrict__ w, int8_t *__restrict__ y,
                                 uint32_t batches, int m, int n, int k, int xz, int wz, int yz, int mult, int s,
                                 int adj_x, int adj_y, int rows_cap) {
    extern __shared__ int32_t bsm[];
    const int kw = (k + 3) / 4, kp = kw | 1;
    int32_t *ws = bsm;                        // [n][kp]: word t4 of column c = w[4 t4 .. 4 t4 + 3][c]
    int32_t *xs = ws + (size_t)n * kp;        // [rows_cap][kp]
    int32_t *sw = xs + (size_t)rows_cap * kp; // [n] column sums of W
    int32_t *sx = sw + n;                     // [rows_cap] row sums of X
    const uint32_t kzz = (uint32_t)k * (uint32_t)xz * (uint32_t)wz;
    const uint32_t row_jobs = (uint32_t)((m + rows_cap - 1) / rows_cap);
    for (uint32_t job = blockIdx.x; job < batches * row_jobs; job += gridDim.x) {
        const uint32_t bt = job / row_jobs;
        const int r0 = (int)(job - bt * row_jobs) * rows_cap;
        const int rows = min(rows_cap, m - r0);
        const int8_t *xb = x + (size_t)bt * m * k, *wb = w + (size_t)bt * k * n;
        for (int i = threadIdx.x; i < n * kw; i += blockDim.x) {
            int c, t4;  // the stored layout's contiguous index runs fastest across the threads
            if (adj_y) t4 = i % kw, c = i / kw;
            else c = i % n, t4 = i / n;
            uint32_t v = 0;
#pragma unroll
            for (int b = 0; b < 4; b++) {
                const int t = 4 * t4 + b;
                if (t < k) v |= (uint32_t)(uint8_t)wb[adj_y ? (size_t)c * k + t : (size_t)t * n + c] << (8 * b);
            }
            ws[c * kp + t4] = (int32_t)v;
        }
        for (int i = threadIdx.x; i < rows * kw; i += blockDim.x) {
            int r, t4;
            if (adj_x) r = i % rows, t4 = i / rows;
            else t4 = i % kw, r = i / kw;
            uint32_t v = 0;
#pragma unroll
            for (int b = 0; b < 4; b++) {
                const int t = 4 * t4 + b;
                if (t < k) v |= (uint32_t)(uint8_t)xb[adj_x ? (size_t)t * m + r0 + r : (size_t)(r0 + r) * k + t] << (8 * b);
            }
            xs[r * kp + t4] = (int32_t)v;
        }
        __syncthreads();
        for (int i = threadIdx.x; i < n + rows; i += blockDim.x) {
            const int32_t *src = i < n ? ws + (size_t)i * kp : xs + (size_t)(i - n) * kp;
            int32_t acc = 0;
            for (int t4 = 0; t4 < kw; t4++) acc = __dp4a(src[t4], 0x01010101, acc);
            (i < n ? sw[i] : sx[i - n]) = acc;
        }
        __syncthreads();
        const int rq = (rows + 3) / 4, cq = (n + 3) / 4;
        for (int gi = threadIdx.x; gi < rq * cq; gi += blockDim.x) {
            const int rr = gi / cq, cc = gi - rr * cq;
            const int32_t *xp[4], *wp[4];
#pragma unroll
            for (int i = 0; i < 4; i++) {
                xp[i] = xs + (size_t)min(rr + i * rq, rows - 1) * kp;
                wp[i] = ws + (size_t)min(cc + i * cq, n - 1) * kp;
            }
            int32_t acc[4][4] = {};
            for (int t4 = 0; t4 < kw; t4++) {
                int32_t xv[4], wv[4];
#pragma unroll
                for (int i = 0; i < 4; i++) xv[i] = xp[i][t4], wv[i] = wp[i][t4];
#pragma unroll
                for (int i = 0; i < 4; i++)
#pragma unroll
                    for (int j = 0; j < 4; j++) acc[i][j] = __dp4a(xv[i], wv[j], acc[i][j]);
            }
#pragma unroll
            for (int i = 0; i < 4; i++) {
                const int r = rr + i * rq;
                if (r >= rows) break;
                const uint32_t rowc = kzz - (uint32_t)wz * (uint32_t)sx[r];
#pragma unroll
                for (int j = 0; j < 4; j++) {
                    const int c = cc + j * cq;
                    if (c < n) {
                        const int32_t v = (int32_t)((uint32_t)acc[i][j] + rowc - (uint32_t)xz * (uint32_t)sw[c]);
                        y[((size_t)bt * m + r0 + r) * n + c] = (int8_t)dev_clamp(dev_scale(v, mult, s) + yz, -128, 127);
                    }
                }
            }
        }
        __syncthreads();
    }
}

// 32 x 32 output tile per block, operands through shared memory 32 reduction steps at a time.
__global__ void bmm_kernel(const int8_t *__restrict__ x, const int8_t *__restrict__ w, int8_t *__restrict__ y,
                           uint32_t batches, int m, int n, int k, int xz, int wz, int yz, int mult, int s, int adj_x,
                           int adj_y) {
    __shared__ int16_t xs[32][33], ws[32][33];
    const int tx = threadIdx.x % 32, ty = threadIdx.x / 32;  // 32 x 8 threads
    const int tm = (m + 31) / 32, tn = (n + 31) / 32;
    const uint64_t tiles = (uint64_t)batches * tm * tn;
    for (uint64_t t = blockIdx.x; t < tiles; t += gridDim.x) {
        const int bn = (int)(t % tn), bm = (int)((t / tn) % tm);
        const uint64_t bt = t / ((uint64_t)tn * tm);
        const int8_t *xb = x + bt * (uint64_t)m * k, *wb = w + bt * (uint64_t)k * n;
        int32_t acc[4] = {0, 0, 0, 0};
        for (int k0 = 0; k0 < k; k0 += 32) {
            for (int i = ty; i < 32; i += 8) {
                const int r = bm * 32 + i, kk = k0 + tx;
                xs[i][tx] = (r < m && kk < k) ? (int16_t)(xb[adj_x ? (uint64_t)kk * m + r : (uint64_t)r * k + kk] - xz) : 0;
                const int kr = k0 + i, cc = bn * 32 + tx;
                ws[i][tx] = (kr < k && cc < n) ? (int16_t)(wb[adj_y ? (uint64_t)cc * k + kr : (uint64_t)kr * n + cc] - wz)
                                               : 0;
            }
            __syncthreads();
#pragma unroll 8
            for (int kk = 0; kk < 32; kk++) {
                const int wv = ws[kk][tx];
#pragma unroll
                for (int i = 0; i < 4; i++) acc[i] += (int)xs[ty + 8 * i][kk] * wv;
            }
            __syncthreads();
        }
#pragma unroll
        for (int i = 0; i < 4; i++) {
            const int r = bm * 32 + ty + 8 * i, c = bn * 32 + tx;
            if (r < m && c < n)
                y[bt * (uint64_t)m * n + (uint64_t)r * n + c] = (int8_t)dev_clamp(dev_scale(acc[i], mult, s) + yz, -128, 127);
        }
    }
}

// ---------------------------------------------------------------- pack (code 19) -------------
template <int V>
__global__ void pack_kernel(Segments segs, uint8_t *__restrict__ z, uint32_t z_bytes, int images) {
    using T = typename Unit<V>::T;
    const uint32_t per = z_bytes / V;
    const uint64_t units = (uint64_t)per * images;
    for (uint64_t u = (uint64_t)blockIdx.x * blockDim.x + threadIdx.x; u < units; u += (uint64_t)gridDim.x * blockDim.x) {
        const uint64_t img = u / per;
        const uint32_t off = (uint32_t)(u - img * per) * V;
        int s = 0;
        while (s + 1 < segs.count && off >= segs.dst_offset[s + 1]) s++;
        reinterpret_cast<T *>(z)[u] =
            *reinterpret_cast<const T *>(segs.src[s] + img * segs.bytes[s] + (off - segs.dst_offset[s]));
    }
}

}  // namespace

void launch_pool(const int8_t *x, int8_t *y, const ConvGeom &g, int is_max, int lo, int hi, cudaStream_t s) {
    if (is_max && g.ic == g.oc && g.oc % 16 == 0 && unit_for(reinterpret_cast<uintptr_t>(x) | reinterpret_cast<uintptr_t>(y)) == 16) {
        const uint64_t total = (uint64_t)g.n * g.oh * g.ow * (g.oc / 16);
        maxpool16_kernel<<<grid_for(total, kT), kT, 0, s>>>(x, y, g, 0x01010101u * (uint8_t)lo, 0x01010101u * (uint8_t)hi);
        return;
    }
    const uint64_t total = (uint64_t)g.n * g.oh * g.ow * g.oc;
    pool_kernel<<<grid_for(total, kT), kT, 0, s>>>(x, y, g, is_max, lo, hi);
}

void launch_bmm(const int8_t *x, const int8_t *w, int8_t *y, size_t batches, int m, int n, int k, const int32_t q7[7],
                cudaStream_t s) {
    for (int rows_cap = 128; rows_cap >= 32; rows_cap /= 2) {
        const size_t smem = bmm_small_smem(n, k, rows_cap);
        if (smem > (size_t)kBmmSmem || (rows_cap > 32 && rows_cap / 2 >= m)) continue;
        const uint64_t jobs = (uint64_t)batches * ((m + rows_cap - 1) / rows_cap);
        bmm_small_kernel<<<grid_for(jobs, 1), kT, smem, s>>>(x, w, y, (uint32_t)batches, m, n, k, q7[0], q7[1], q7[2],
                                                             q7[3], q7[4], q7[5], q7[6], rows_cap);
        return;
    }
    const uint64_t tiles = (uint64_t)batches * ((m + 31) / 32) * ((n + 31) / 32);
    bmm_kernel<<<grid_for(tiles, 1), kT, 0, s>>>(x, w, y, (uint32_t)batches, m, n, k, q7[0], q7[1], q7[2], q7[3], q7[4],
                                                  q7[5], q7[6]);
}

void launch_permute(const uint8_t *a, uint8_t *z, const Shape5 &in, const int perm[5], int elem_bytes, cudaStream_t s) {
    uint64_t count = 1;
    for (int d = 0; d < in.rank; d++) count *= in.d[d];
    // Merge runs of input axes that stay adjacent and in order in the output.
    int groups[5][2], ng = 0;  // [first input axis, last input axis] per output group
    for (int d = 0; d < in.rank; d++) {
        if (ng && perm[d] == groups[ng - 1][1] + 1) groups[ng - 1][1] = perm[d];
        else groups[ng][0] = groups[ng][1] = perm[d], ng++;
    }
    auto extent = [&](int g) {
        uint64_t e = 1;
        for (int d = groups[g][0]; d <= groups[g][1]; d++) e *= in.d[d];
        return e;
    };
    // batched 2-D transpose: output groups (B, C, R) with input order (B, R, C)
    bool t2 = false;
    uint64_t B = 1, R = 0, Cc = 0;
    if (ng == 2 && groups[0][0] > groups[1][0]) t2 = true, R = extent(1), Cc = extent(0);
    if (ng == 3 && groups[0][0] == 0 && groups[1][0] > groups[2][0]) t2 = true, B = extent(0), R = extent(2), Cc = extent(1);
    if (t2 && B * R * Cc == count && R < (1u << 31) && Cc < (1u << 31)) {
        const uint64_t tiles = B * ((R + 31) / 32) * ((Cc + 31) / 32);
        const unsigned grid = (unsigned)std::min<uint64_t>(tiles, 148ull * 16);
        const size_t mat_smem = R * ((Cc / 4) | 1) * sizeof(uint32_t);
        if (elem_bytes == 1 && R >= 4 && Cc >= 4 && R % 4 == 0 && Cc % 4 == 0 && mat_smem <= (size_t)kTrSmem && B < (1u << 31) &&
            unit_for(reinterpret_cast<uintptr_t>(a) | reinterpret_cast<uintptr_t>(z)) >= 4) {
            // matrices per block: fill about a quarter of the budget, keeping the word counts < 2^31
            const uint64_t per = std::max<uint64_t>(1, std::min<uint64_t>(B, (kTrSmem / 4) / mat_smem));
            const uint64_t chunks = (B + per - 1) / per;
            const int cw = (int)(Cc / 4);
            transpose_b4_kernel<<<(unsigned)std::min<uint64_t>(chunks, 148ull * 16), kT, per * mat_smem, s>>>(
                reinterpret_cast<const uint32_t *>(a), reinterpret_cast<uint32_t *>(z), (uint32_t)B, (uint32_t)R,
                (uint32_t)Cc, (uint32_t)per, FastDiv(cw), FastDiv((int)(R / 4) * cw), FastDiv((int)(R / 4)));
            return;
        }
        if (elem_bytes == 1) transpose2d_kernel<1><<<grid, kT, 0, s>>>(a, z, (uint32_t)B, (uint32_t)R, (uint32_t)Cc);
        else if (elem_bytes == 4) transpose2d_kernel<4><<<grid, kT, 0, s>>>(a, z, (uint32_t)B, (uint32_t)R, (uint32_t)Cc);
        else t2 = false;
        if (t2) return;
    }
    Perm5 p;
    for (int d = 0; d < 5; d++) p.p[d] = perm[d];
    permute_kernel<<<grid_for(count, kT), kT, 0, s>>>(a, z, in, p, elem_bytes, count);
}

void launch_slice(const uint8_t *a, uint8_t *z, const Shape5 &in, const Shape5 &out, const uint32_t begin[5],
                  cudaStream_t s) {
    uint64_t istride[5], acc = 1;
    for (int d = in.rank - 1; d >= 0; d--) istride[d] = acc, acc *= in.d[d];
    int k = -1;  // innermost sliced axis
    for (int d = 0; d < in.rank; d++)
        if (out.d[d] != in.d[d]) k = d;
    RunCopy rc{};
    if (k < 0) {
        rc.ndim = 0, rc.rows = 1, rc.run = (uint32_t)acc;
    } else {
        // run: out.d[k] * (full trailing axes) contiguous bytes; rows over the axes before k
        rc.run = (uint32_t)(out.d[k] * istride[k]);
        rc.base = begin[k] * istride[k];
        rc.rows = 1;
        // axes before k, merged into at most 4 mixed-radix digits (leading ones first)
        int nd = 0;
        for (int d = 0; d < k; d++) {
            rc.base += (uint64_t)begin[d] * istride[d];
            if (out.d[d] == 1) continue;
            rc.rows *= out.d[d];
            rc.extent[nd] = out.d[d];  // k <= 4, so at most 4 digits
            rc.stride[nd] = istride[d];
            nd++;
        }
        rc.ndim = nd;
    }
    rc.dst_stride = rc.run;
    run_copy(a, z, rc, s);
}

void launch_concat(const uint8_t *a, const uint8_t *b, uint8_t *z, size_t outer, size_t ac, size_t bc, cudaStream_t s) {
    const int v = unit_for(ac, bc, reinterpret_cast<uintptr_t>(a) | reinterpret_cast<uintptr_t>(b) |
                                       reinterpret_cast<uintptr_t>(z));
    const uint64_t units = outer * (ac + bc) / v;
    if (v == 16) concat_kernel<16><<<grid_for(units, kT), kT, 0, s>>>(a, b, z, outer, (uint32_t)ac, (uint32_t)bc);
    else if (v == 4) concat_kernel<4><<<grid_for(units, kT), kT, 0, s>>>(a, b, z, outer, (uint32_t)ac, (uint32_t)bc);
    else concat_kernel<1><<<grid_for(units, kT), kT, 0, s>>>(a, b, z, outer, (uint32_t)ac, (uint32_t)bc);
}

void launch_resize(const uint8_t *a, uint8_t *z, int n, int ih, int iw, int c, int oh, int ow, const uint32_t *offsets,
                   cudaStream_t s) {
    const uint64_t pixels = (uint64_t)n * oh * ow, img = (uint64_t)ih * iw * c;
    const int v = unit_for((uint64_t)c, img, reinterpret_cast<uintptr_t>(a) | reinterpret_cast<uintptr_t>(z));
    const uint64_t units = pixels * (c / v);
    if (v == 16) resize_kernel<16><<<grid_for(units, kT), kT, 0, s>>>(a, z, pixels, oh, ow, (uint32_t)c, img, offsets);
    else if (v == 4) resize_kernel<4><<<grid_for(units, kT), kT, 0, s>>>(a, z, pixels, oh, ow, (uint32_t)c, img, offsets);
    else resize_kernel<1><<<grid_for(units, kT), kT, 0, s>>>(a, z, pixels, oh, ow, (uint32_t)c, img, offsets);
}

void launch_concat_multi(const ConcatInputs &in, uint8_t *z, size_t rows, cudaStream_t s) {
    uint64_t m = reinterpret_cast<uintptr_t>(z), row = 0;
    for (int i = 0; i < in.count; i++) {
        m |= in.width[i] | reinterpret_cast<uintptr_t>(in.src[i]);
        row += in.width[i];
    }
    const int v = unit_for(m);
    const uint64_t units = rows * (row / v);
    if (v == 16) concat_multi_kernel<16><<<grid_for(units, kT), kT, 0, s>>>(in, z, rows, (uint32_t)(row / 16));
    else if (v == 4) concat_multi_kernel<4><<<grid_for(units, kT), kT, 0, s>>>(in, z, rows, (uint32_t)(row / 4));
    else concat_multi_kernel<1><<<grid_for(units, kT), kT, 0, s>>>(in, z, rows, (uint32_t)row);
}

void launch_concat_parts(const ConcatParts &in, uint8_t *z, size_t rows, cudaStream_t s) {
    uint64_t m = reinterpret_cast<uintptr_t>(z), row = 0;
    for (int i = 0; i < in.count; i++) {
        m |= in.out_w[i] | in.in_w[i] | in.off[i] | reinterpret_cast<uintptr_t>(in.src[i]);
        row += in.out_w[i];
    }
    const int v = unit_for(m);
    const uint64_t units = rows * (row / v);
    if (v == 16) concat_parts_kernel<16><<<grid_for(units, kT), kT, 0, s>>>(in, z, rows, (uint32_t)(row / 16));
    else if (v == 4) concat_parts_kernel<4><<<grid_for(units, kT), kT, 0, s>>>(in, z, rows, (uint32_t)(row / 4));
    else concat_parts_kernel<1><<<grid_for(units, kT), kT, 0, s>>>(in, z, rows, (uint32_t)row);
}

void launch_lut_rows(const uint8_t *x, uint8_t *y, size_t rows, uint32_t in_w, uint32_t off, uint32_t out_w,
                     const uint8_t *table, unsigned flip, cudaStream_t s) {
    const int v = unit_for((uint64_t)in_w | off | out_w | reinterpret_cast<uintptr_t>(x) | reinterpret_cast<uintptr_t>(y));
    const uint64_t units = (uint64_t)rows * (out_w / v);
    if (v == 16) lut_rows_kernel<16><<<grid_for(units, kT), kT, 0, s>>>(x, y, rows, in_w, off, out_w, table, flip);
    else if (v == 4) lut_rows_kernel<4><<<grid_for(units, kT), kT, 0, s>>>(x, y, rows, in_w, off, out_w, table, flip);
    else lut_rows_kernel<1><<<grid_for(units, kT), kT, 0, s>>>(x, y, rows, in_w, off, out_w, table, flip);
}

void launch_pack(const Segments &segs, uint8_t *z, uint32_t z_bytes, int images, cudaStream_t s) {
    uint64_t m = z_bytes | reinterpret_cast<uintptr_t>(z);
    for (int i = 0; i < segs.count; i++) m |= segs.bytes[i] | segs.dst_offset[i] | reinterpret_cast<uintptr_t>(segs.src[i]);
    const int v = unit_for(m);
    const uint64_t units = (uint64_t)z_bytes / v * images;
    if (v == 16) pack_kernel<16><<<grid_for(units, kT), kT, 0, s>>>(segs, z, z_bytes, images);
    else if (v == 4) pack_kernel<4><<<grid_for(units, kT), kT, 0, s>>>(segs, z, z_bytes, images);
    else pack_kernel<1><<<grid_for(units, kT), kT, 0, s>>>(segs, z, z_bytes, images);
}

}  // namespace uq
