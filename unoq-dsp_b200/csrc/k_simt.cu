// k_simt.cu -- CUDA-core kernels for every INT8 opcode of the plan ABI.
//
// These are the bandwidth-bound ops (depthwise, pooling, element-wise, byte movement) plus a
// general CUDA-core convolution used for shapes the tensor-core path does not take. All
// arithmetic is integer and follows the reference's scalar definitions (cited per kernel).
#include "kernels.cuh"

namespace uq {

namespace {

constexpr int kThreads = 256;

// ---------------------------------------------------------------- code 14, CUDA cores ----
// One thread = one output pixel x four output channels (one packed weight group, gemm.h:9).
// The column value is the reference's u8 form: x ^ 0x80 inside the image, xzp + 128 on
// borders and in the K padding (qnn.c:1155-1168), so acc equals the reference accumulator.
__global__ void conv_simt_kernel(const int8_t *__restrict__ x, const int8_t *__restrict__ w, int8_t *__restrict__ y,
                                 ConvGeom g, Requant r) {
    const int groups = (g.oc + 3) / 4;
    const uint64_t total = (uint64_t)g.n * g.oh * g.ow * groups;
    const int fill = g.xzp + 128;
    for (uint64_t idx = (uint64_t)blockIdx.x * blockDim.x + threadIdx.x; idx < total;
         idx += (uint64_t)gridDim.x * blockDim.x) {
        const int grp = (int)(idx % groups);
        const uint64_t pix = idx / groups;
        const int ox = (int)(pix % g.ow);
        const int oy = (int)((pix / g.ow) % g.oh);
        const uint64_t n = pix / ((uint64_t)g.ow * g.oh);
        const int8_t *wg = w + (size_t)grp * g.kp * 4;
        int acc0 = 0, acc1 = 0, acc2 = 0, acc3 = 0;
        int t = 0;
        for (int ky = 0; ky < g.kh; ky++) {
            const int iy = oy * g.sh - g.pt + ky * g.dh;
            for (int kx = 0; kx < g.kw; kx++) {
                const int ix = ox * g.sw - g.pl + kx * g.dw;
                const bool valid = iy >= 0 && ix >= 0 && iy < g.ih && ix < g.iw;
                const int8_t *src = valid ? x + ((n * g.ih + iy) * g.iw + ix) * g.ic : nullptr;
                for (int c = 0; c < g.ic; c++, t++) {
                    const int v = valid ? (int)(uint8_t)(src[c] ^ 0x80) : fill;
                    const int8_t *wt = wg + (t / 8) * 32 + t % 8;
                    acc0 += v * wt[0];
                    acc1 += v * wt[8];
                    acc2 += v * wt[16];
                    acc3 += v * wt[24];
                }
            }
        }
        for (; t < g.kp; t++) {
            const int8_t *wt = wg + (t / 8) * 32 + t % 8;
            acc0 += fill * wt[0];
            acc1 += fill * wt[8];
            acc2 += fill * wt[16];
            acc3 += fill * wt[24];
        }
        int8_t *out = y + pix * g.oc + grp * 4;
        const int j = grp * 4;
        out[0] = requant_one(acc0, j, r);
        if (j + 1 < g.oc) out[1] = requant_one(acc1, j + 1, r);
        if (j + 2 < g.oc) out[2] = requant_one(acc2, j + 2, r);
        if (j + 3 < g.oc) out[3] = requant_one(acc3, j + 3, r);
    }
}

// ---------------------------------------------------------------- code 15 -------------
// acc = sum over taps of (x + 128) * w, borders contributing (xzp + 128) * w; the bias is
// added by the requantisation (qnn.c:1228-1245, depthwise3 qnn.c:807-983 agree).
template <int VEC>
__global__ void depthwise_kernel(const int8_t *__restrict__ x, const int8_t *__restrict__ w, int8_t *__restrict__ y,
                                 ConvGeom g, Requant r) {
    const int cgroups = g.oc / VEC;
    const uint64_t total = (uint64_t)g.n * g.oh * g.ow * cgroups;
    const int fill = g.xzp + 128;
    for (uint64_t idx = (uint64_t)blockIdx.x * blockDim.x + threadIdx.x; idx < total;
         idx += (uint64_t)gridDim.x * blockDim.x) {
        const int cg = (int)(idx % cgroups);
        const uint64_t pix = idx / cgroups;
        const int ox = (int)(pix % g.ow);
        const int oy = (int)((pix / g.ow) % g.oh);
        const uint64_t n = pix / ((uint64_t)g.ow * g.oh);
        const int c0 = cg * VEC;
        int acc[VEC];
#pragma unroll
        for (int v = 0; v < VEC; v++) acc[v] = 0;
        for (int ky = 0; ky < g.kh; ky++) {
            const int iy = oy * g.sh - g.pt + ky * g.dh;
            for (int kx = 0; kx < g.kw; kx++) {
                const int ix = ox * g.sw - g.pl + kx * g.dw;
                const bool valid = iy >= 0 && ix >= 0 && iy < g.ih && ix < g.iw;
                const int8_t *wt = w + (size_t)(ky * g.kw + kx) * g.oc + c0;
                if (VEC == 4) {
                    const char4 wv = *reinterpret_cast<const char4 *>(wt);
                    int x0 = fill, x1 = fill, x2 = fill, x3 = fill;
                    if (valid) {
                        const char4 xv = *reinterpret_cast<const char4 *>(x + ((n * g.ih + iy) * g.iw + ix) * g.ic + c0);
                        x0 = xv.x + 128;
                        x1 = xv.y + 128;
                        x2 = xv.z + 128;
                        x3 = xv.w + 128;
                    }
                    acc[0] += x0 * wv.x;
                    acc[1] += x1 * wv.y;
                    acc[2] += x2 * wv.z;
                    acc[3] += x3 * wv.w;
                } else {
                    const int xv = valid ? x[((n * g.ih + iy) * g.iw + ix) * g.ic + c0] + 128 : fill;
                    acc[0] += xv * wt[0];
                }
            }
        }
        int8_t *out = y + pix * g.oc + c0;
#pragma unroll
        for (int v = 0; v < VEC; v++) out[v] = requant_one(acc[v], c0 + v, r);
    }
}

// ---------------------------------------------------------------- code 17 -------------
// qnn.c:1082-1088: table softmax, one thread per row.
__global__ void softmax_table_kernel(const int8_t *__restrict__ x, int8_t *__restrict__ y, size_t rows, int width,
                                     const int32_t *__restrict__ table, int lo, int hi) {
    for (size_t row = (size_t)blockIdx.x * blockDim.x + threadIdx.x; row < rows; row += (size_t)gridDim.x * blockDim.x) {
        const int8_t *xr = x + row * width;
        int mx = -128;
        for (int c = 0; c < width; c++) mx = xr[c] > mx ? xr[c] : mx;
        uint64_t sum = 0;
        for (int c = 0; c < width; c++) sum += (uint32_t)table[mx - xr[c]];
        for (int c = 0; c < width; c++) {
            const uint64_t v = (uint64_t)(uint32_t)table[mx - xr[c]] * 256u;
            const int32_t rr = (int32_t)((v + sum / 2) / sum) - 128;
            y[row * width + c] = (int8_t)dev_clamp(rr, lo, hi);
        }
    }
}

// ---------------------------------------------------------------- code 28 -------------
// qnn.c:87-107: gemmlowp-style exact softmax; one warp per row, lanes stride the row.
__global__ void softmax_exact_kernel(const int8_t *__restrict__ x, int8_t *__restrict__ y, size_t rows, int width,
                                     const int32_t *__restrict__ q) {
    const int lane = threadIdx.x & 31;
    const int32_t *lut = q + 1;
    for (size_t row = ((size_t)blockIdx.x * blockDim.x + threadIdx.x) / 32; row < rows;
         row += ((size_t)gridDim.x * blockDim.x) / 32) {
        const int8_t *xr = x + row * width;
        int mx = -128;
        for (int j = lane; j < width; j += 32) mx = xr[j] > mx ? xr[j] : mx;
        for (int o = 16; o; o >>= 1) {
            const int other = __shfl_xor_sync(0xffffffffu, mx, o);
            mx = other > mx ? other : mx;
        }
        uint32_t sum = 0;
        for (int j = lane; j < width; j += 32) sum += ((uint32_t)__ldg(lut + mx - xr[j]) + 2048u) >> 12;
        for (int o = 16; o; o >>= 1) sum += __shfl_xor_sync(0xffffffffu, sum, o);
        const unsigned leading = (unsigned)__clz(sum), exponent = 35u - leading;
        const uint32_t normalized = (sum << leading) - 0x80000000u;
        const int32_t half = (int32_t)(((uint64_t)normalized + 2147483648ull) >> 1);
        int32_t rcp = (int32_t)(1515870810u + (uint32_t)dev_scale(half, -1010580540, 0));
        for (int step = 0; step < 3; step++) {
            const int32_t err = (int32_t)(536870912u - (uint32_t)dev_scale(half, rcp, 0));
            rcp = (int32_t)((uint32_t)rcp + (uint32_t)dev_scale(rcp, err, 0) * 4u);
        }
        const int64_t doubled = (int64_t)rcp * 2;
        rcp = doubled > 2147483647ll ? 2147483647 : (int32_t)doubled;
        for (int j = lane; j < width; j += 32) {
            const uint32_t value = (uint32_t)dev_scale(rcp, __ldg(lut + mx - xr[j]), 0);
            const unsigned rounded = exponent >= 32 ? 0u : (value + (1u << (exponent - 1))) >> exponent;
            y[row * width + j] = (int8_t)(rounded > 255 ? 127 : (int)rounded - 128);
        }
    }
}

// Code 28 for the operator ABI (uq_softmax_exact over caller rows): one thread per row, the
// reference's three passes over the row in order (qnn.c:87-107).
__global__ void softmax_exact_rows_kernel(const int8_t *__restrict__ x, int8_t *__restrict__ y, size_t rows, int width,
                                          const int32_t *__restrict__ q) {
    const int32_t *lut = q + 1;
    for (size_t row = (size_t)blockIdx.x * blockDim.x + threadIdx.x; row < rows; row += (size_t)gridDim.x * blockDim.x) {
        const int8_t *xr = x + row * width;
        int mx = -128;
        for (int j = 0; j < width; j++) mx = xr[j] > mx ? xr[j] : mx;
        uint32_t sum = 0;
        for (int j = 0; j < width; j++) sum += ((uint32_t)lut[mx - xr[j]] + 2048u) >> 12;
        const unsigned leading = (unsigned)__clz(sum), exponent = 35u - leading;
        const uint32_t normalized = (sum << leading) - 0x80000000u;
        const int32_t half = (int32_t)(((uint64_t)normalized + 2147483648ull) >> 1);
        int32_t rcp = (int32_t)(1515870810u + (uint32_t)dev_scale(half, -1010580540, 0));
        for (int step = 0; step < 3; step++) {
            const int32_t err = (int32_t)(536870912u - (uint32_t)dev_scale(half, rcp, 0));
            rcp = (int32_t)((uint32_t)rcp + (uint32_t)dev_scale(rcp, err, 0) * 4u);
        }
        const int64_t doubled = (int64_t)rcp * 2;
        rcp = doubled > 2147483647ll ? 2147483647 : (int32_t)doubled;
        for (int j = 0; j < width; j++) {
            const uint32_t value = (uint32_t)dev_scale(rcp, lut[mx - xr[j]], 0);
            const unsigned rounded = exponent >= 32 ? 0u : (value + (1u << (exponent - 1))) >> exponent;
            y[row * width + j] = (int8_t)(rounded > 255 ? 127 : (int)rounded - 128);
        }
    }
}

// ---------------------------------------------------------------- code 18 -------------
// qnn.c:175-183: y = clamp(scale(TX[x+128] + TB[b+128], m, s) + yzp). Tables staged in
// shared memory; 16 bytes per thread per step.
__global__ void add_kernel(const int8_t *__restrict__ x, const int8_t *__restrict__ b, int8_t *__restrict__ y, size_t count,
                           const int32_t *__restrict__ q) {
    __shared__ int32_t tx[256], tb[256];
    for (int i = threadIdx.x; i < 256; i += blockDim.x) {
        tx[i] = q[8 + i];
        tb[i] = q[264 + i];
    }
    __syncthreads();
    const int32_t m = q[0], s = q[1], zp = q[2], lo = q[3], hi = q[4];
    const size_t vecs = count / 16;
    for (size_t i = (size_t)blockIdx.x * blockDim.x + threadIdx.x; i < vecs; i += (size_t)gridDim.x * blockDim.x) {
        const int4 xv = reinterpret_cast<const int4 *>(x)[i];
        const int4 bv = reinterpret_cast<const int4 *>(b)[i];
        const int8_t *xa = reinterpret_cast<const int8_t *>(&xv), *ba = reinterpret_cast<const int8_t *>(&bv);
        int4 out;
        int8_t *oa = reinterpret_cast<int8_t *>(&out);
#pragma unroll
        for (int k = 0; k < 16; k++) {
            const int32_t sum = (int32_t)((uint32_t)tx[xa[k] + 128] + (uint32_t)tb[ba[k] + 128]);
            oa[k] = (int8_t)dev_clamp(dev_scale(sum, m, s) + zp, lo, hi);
        }
        reinterpret_cast<int4 *>(y)[i] = out;
    }
    for (size_t i = vecs * 16 + (size_t)blockIdx.x * blockDim.x + threadIdx.x; i < count;
         i += (size_t)gridDim.x * blockDim.x) {
        const int32_t sum = (int32_t)((uint32_t)tx[x[i] + 128] + (uint32_t)tb[b[i] + 128]);
        y[i] = (int8_t)dev_clamp(dev_scale(sum, m, s) + zp, lo, hi);
    }
}

// ---------------------------------------------------------------- code 25 -------------
// qnn.c:112-117.
__global__ void mul_kernel(const int8_t *__restrict__ x, const int8_t *__restrict__ b, int8_t *__restrict__ y, size_t count,
                           int xz, int bz, int yz, int m, int s, int lo, int hi) {
    for (size_t i = (size_t)blockIdx.x * blockDim.x + threadIdx.x; i < count; i += (size_t)gridDim.x * blockDim.x)
        y[i] = (int8_t)dev_clamp(dev_scale((x[i] - xz) * (b[i] - bz), m, s) + yz, lo, hi);
}

// ---------------------------------------------------------------- code 22 -------------
// graph.c:331-341.
__global__ void lut_kernel(const uint8_t *__restrict__ x, uint8_t *__restrict__ y, size_t count,
                           const uint8_t *__restrict__ table, unsigned flip) {
    __shared__ uint8_t t[256];
    for (int i = threadIdx.x; i < 256; i += blockDim.x) t[i] = table[i];
    __syncthreads();
    const size_t vecs = count / 16;
    for (size_t i = (size_t)blockIdx.x * blockDim.x + threadIdx.x; i < vecs; i += (size_t)gridDim.x * blockDim.x) {
        uint4 v = reinterpret_cast<const uint4 *>(x)[i];
        uint8_t *a = reinterpret_cast<uint8_t *>(&v);
#pragma unroll
        for (int k = 0; k < 16; k++) a[k] = t[a[k] ^ flip];
        reinterpret_cast<uint4 *>(y)[i] = v;
    }
    for (size_t i = vecs * 16 + (size_t)blockIdx.x * blockDim.x + threadIdx.x; i < count;
         i += (size_t)gridDim.x * blockDim.x)
        y[i] = t[x[i] ^ flip];
}

// ---------------------------------------------------------------- code 24 -------------
// qnn.c:184-198: one thread per (batch, channel); channel-contiguous rows coalesce.
__global__ void mean_kernel(const int8_t *__restrict__ x, int8_t *__restrict__ y, size_t batches, int channels, int count,
                            int xzp, int yzp, int m, int s) {
    const size_t total = batches * channels;
    for (size_t i = (size_t)blockIdx.x * blockDim.x + threadIdx.x; i < total; i += (size_t)gridDim.x * blockDim.x) {
        const size_t n = i / channels;
        const int c = (int)(i % channels);
        const int8_t *xb = x + n * (size_t)count * channels + c;
        int32_t sum = 0;
        for (int p = 0; p < count; p++) sum += xb[(size_t)p * channels];
        y[i] = (int8_t)dev_clamp(dev_scale(sum - count * xzp, m, s) + yzp, -128, 127);
    }
}

// ---------------------------------------------------------------- byte movement -------
__global__ void pad_kernel(const uint8_t *__restrict__ a, uint8_t *__restrict__ z, int images, uint4 ad, uint4 zd, int4 lo4,
                           int8_t value) {
    const uint64_t zimg = (uint64_t)zd.x * zd.y * zd.z * zd.w, aimg = (uint64_t)ad.x * ad.y * ad.z * ad.w;
    const uint64_t total = zimg * images;
    for (uint64_t i = (uint64_t)blockIdx.x * blockDim.x + threadIdx.x; i < total; i += (uint64_t)gridDim.x * blockDim.x) {
        const uint64_t img = i / zimg;
        uint64_t rem = i % zimg;
        const int c = (int)(rem % zd.w);
        rem /= zd.w;
        const int w = (int)(rem % zd.z);
        rem /= zd.z;
        const int h = (int)(rem % zd.y);
        const int n = (int)(rem / zd.y);
        const int an = n - lo4.x, ah = h - lo4.y, aw = w - lo4.z, ac = c - lo4.w;
        uint8_t v = (uint8_t)value;
        if (an >= 0 && an < (int)ad.x && ah >= 0 && ah < (int)ad.y && aw >= 0 && aw < (int)ad.z && ac >= 0 && ac < (int)ad.w)
            v = a[img * aimg + (((uint64_t)an * ad.y + ah) * ad.z + aw) * ad.w + ac];
        z[i] = v;
    }
}

}  // namespace

void launch_conv_simt(const int8_t *x, const int8_t *w_packed, int8_t *y, const ConvGeom &g, const Requant &r,
                      cudaStream_t s) {
    const uint64_t total = (uint64_t)g.n * g.oh * g.ow * ((g.oc + 3) / 4);
    conv_simt_kernel<<<grid_for(total, kThreads), kThreads, 0, s>>>(x, w_packed, y, g, r);
}

void launch_depthwise(const int8_t *x, const int8_t *w, int8_t *y, const ConvGeom &g, const Requant &r, cudaStream_t s) {
    if (g.oc % 4 == 0) {
        const uint64_t total = (uint64_t)g.n * g.oh * g.ow * (g.oc / 4);
        depthwise_kernel<4><<<grid_for(total, kThreads), kThreads, 0, s>>>(x, w, y, g, r);
    } else {
        const uint64_t total = (uint64_t)g.n * g.oh * g.ow * g.oc;
        depthwise_kernel<1><<<grid_for(total, kThreads), kThreads, 0, s>>>(x, w, y, g, r);
    }
}

void launch_softmax_table(const int8_t *x, int8_t *y, size_t rows, int width, const int32_t *table, int lo, int hi,
                          cudaStream_t s) {
    softmax_table_kernel<<<grid_for(rows, kThreads), kThreads, 0, s>>>(x, y, rows, width, table, lo, hi);
}

void launch_softmax_exact(const int8_t *x, int8_t *y, size_t rows, int width, const int32_t *q, cudaStream_t s) {
    softmax_exact_kernel<<<grid_for(rows * 32, kThreads), kThreads, 0, s>>>(x, y, rows, width, q);
}

void launch_softmax_exact_rows(const int8_t *x, int8_t *y, size_t rows, int width, const int32_t *q, cudaStream_t s) {
    softmax_exact_rows_kernel<<<grid_for(rows, 128), 128, 0, s>>>(x, y, rows, width, q);
}

void launch_add(const int8_t *x, const int8_t *b, int8_t *y, size_t count, const int32_t *q, cudaStream_t s) {
    add_kernel<<<grid_for(count / 16 + 1, kThreads), kThreads, 0, s>>>(x, b, y, count, q);
}

void launch_mul(const int8_t *x, const int8_t *b, int8_t *y, size_t count, const int32_t q7[7], cudaStream_t s) {
    mul_kernel<<<grid_for(count, kThreads), kThreads, 0, s>>>(x, b, y, count, q7[0], q7[1], q7[2], q7[3], q7[4], q7[5],
                                                               q7[6]);
}

void launch_lut(const uint8_t *x, uint8_t *y, size_t count, const uint8_t *table, unsigned flip, cudaStream_t s) {
    lut_kernel<<<grid_for(count / 16 + 1, kThreads), kThreads, 0, s>>>(x, y, count, table, flip);
}

void launch_mean(const int8_t *x, int8_t *y, size_t batches, int channels, const int32_t q5[5], cudaStream_t s) {
    mean_kernel<<<grid_for(batches * channels, kThreads), kThreads, 0, s>>>(x, y, batches, channels, q5[0], q5[1], q5[2],
                                                                            q5[3], q5[4]);
}

void launch_pad(const uint8_t *a, uint8_t *z, int images, const uint32_t ad[4], const uint32_t zd[4], const int32_t pads[8],
                int8_t value, cudaStream_t s) {
    const uint64_t total = (uint64_t)zd[0] * zd[1] * zd[2] * zd[3] * images;
    pad_kernel<<<grid_for(total, kThreads), kThreads, 0, s>>>(a, z, images, make_uint4(ad[0], ad[1], ad[2], ad[3]),
                                                             make_uint4(zd[0], zd[1], zd[2], zd[3]),
                                                             make_int4(pads[0], pads[2], pads[4], pads[6]), value);
}

void launch_copy(const void *src, void *dst, size_t bytes, cudaStream_t s) {
    cudaMemcpyAsync(dst, src, bytes, cudaMemcpyDeviceToDevice, s);
}

}  // namespace uq
