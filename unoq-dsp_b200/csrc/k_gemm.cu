// k_gemm.cu -- the reference's raw integer GEMMs (runtime/gemm.h:5-25) on the device:
// Y[m][n] = sum_t X[m * xs + t] * W(n, t), X unsigned bytes, W signed bytes, Y int32.
//
// These are the operator ABI's ug_matmul_u8i8 / _strided / _dot4 / _selected: utilities that
// return the raw int32 accumulators (the convolutions of a plan never go through them; they use
// the tensor-core convolution kernels with the requantisation fused). One kernel covers the three
// weight layouts the reference reads:
//   row-major   W(n, t) = w[n * K + t]                                  (gemm.h:10, packed = 0)
//   packed      W(n, t) = w[(n/4) K 4 + (t/8) 32 + (n%4) 8 + t%8]        (gemm.h:9)
//   dot4        W(n, t) = w[(n/4) K 4 + (t/4) 16 + (n%4) 4 + t%4]        (gemm.c:911-948)
// In every layout the four reduction bytes t..t+3 (t % 4 == 0) of one channel are contiguous, so
// the tiles are staged as words and multiplied with dp4a (u8 x s8, int32 accumulation that wraps
// like the reference's truncated sums).
//
// Tiling: a 256-thread block computes a 64 x 64 output tile; thread (tx, ty) owns rows ty + 16 i
// and columns tx + 16 j (i, j < 4), so shared-memory reads of the B tile fall in distinct banks
// (odd word stride) and every output row is written by 16 consecutive threads.
#include <cuda_runtime.h>

#include <cstdint>

#include "gemm.cuh"

namespace uq {
namespace {

constexpr int kTile = 64, kKc = 32, kKw = kKc / 4, kStride = kKw + 1;

__device__ __forceinline__ int dp4a_us(uint32_t a, uint32_t b, int c) {
    int d;
    asm("dp4a.u32.s32 %0, %1, %2, %3;" : "=r"(d) : "r"(a), "r"(b), "r"(c));
    return d;
}

__device__ __forceinline__ size_t w_offset(int layout, uint32_t n, uint32_t t, uint32_t K) {
    if (layout == kGemmRowMajor) return (size_t)n * K + t;
    if (layout == kGemmPacked) return (size_t)(n >> 2) * K * 4 + (t >> 3) * 32 + (n & 3) * 8 + (t & 7);
    return (size_t)(n >> 2) * K * 4 + (t >> 2) * 16 + (n & 3) * 4 + (t & 3);
}

// Word of four reduction bytes t..t+3; bytes at or past K are zero. `aligned`: the word is one
// aligned 32-bit load whenever t + 3 < K.
__device__ __forceinline__ uint32_t load_word(const uint8_t *p, size_t off, uint32_t t, uint32_t K, bool aligned) {
    if (aligned && t + 3 < K) return *reinterpret_cast<const uint32_t *>(p + off);
    uint32_t v = 0;
    for (int b = 0; b < 4; b++)
        if (t + b < K) v |= (uint32_t)p[off + b] << (8 * b);
    return v;
}

__global__ void __launch_bounds__(256) gemm_u8i8_kernel(const uint8_t *__restrict__ x, const int8_t *__restrict__ w,
                                                        int32_t *__restrict__ y, GemmArgs g,
                                                        const uint16_t *__restrict__ groups) {
    __shared__ uint32_t As[kTile * kStride], Bs[kTile * kStride];
    const int tx = threadIdx.x & 15, ty = threadIdx.x >> 4;
    const uint32_t row0 = blockIdx.x * kTile;
    const uint32_t col0 = blockIdx.y * kTile;  // logical column (into the selected channels)
    const uint8_t *wb = reinterpret_cast<const uint8_t *>(w);
    // each thread stages two words of A and two of B per K chunk: tile row r, word kw
    int a_row[2], a_kw[2];
    uint32_t b_chan[2];
    bool b_ok[2];
    for (int s = 0; s < 2; s++) {
        const int idx = threadIdx.x + s * 256;
        a_row[s] = idx >> 3;
        a_kw[s] = idx & 7;
        const uint32_t c = col0 + (idx >> 3);
        if (groups) {
            b_ok[s] = c < g.cols;
            b_chan[s] = b_ok[s] ? groups[c >> 2] + (c & 3) : 0;
        } else {
            b_ok[s] = c < g.n;
            b_chan[s] = c;
        }
    }
    int acc[4][4] = {};
    for (uint32_t k0 = 0; k0 < g.k; k0 += kKc) {
        for (int s = 0; s < 2; s++) {
            const uint32_t r = row0 + a_row[s], t = k0 + 4 * a_kw[s];
            As[a_row[s] * kStride + a_kw[s]] =
                r < g.m && t < g.k ? load_word(x, (size_t)r * g.xs + t, t, g.k, g.x_aligned) : 0u;
            Bs[a_row[s] * kStride + a_kw[s]] =
                b_ok[s] && t < g.k ? load_word(wb, w_offset(g.layout, b_chan[s], t, g.k), t, g.k, g.w_aligned) : 0u;
        }
        __syncthreads();
#pragma unroll
        for (int kw = 0; kw < kKw; kw++) {
            uint32_t a[4], b[4];
#pragma unroll
            for (int i = 0; i < 4; i++) a[i] = As[(ty + 16 * i) * kStride + kw];
#pragma unroll
            for (int j = 0; j < 4; j++) b[j] = Bs[(tx + 16 * j) * kStride + kw];
#pragma unroll
            for (int i = 0; i < 4; i++)
#pragma unroll
                for (int j = 0; j < 4; j++) acc[i][j] = dp4a_us(a[i], b[j], acc[i][j]);
        }
        __syncthreads();
    }
#pragma unroll
    for (int i = 0; i < 4; i++) {
        const uint32_t r = row0 + ty + 16 * i;
        if (r >= g.m) continue;
#pragma unroll
        for (int j = 0; j < 4; j++) {
            const uint32_t c = col0 + tx + 16 * j;
            if (groups) {
                if (c < g.cols) y[(size_t)r * g.n + groups[c >> 2] + (c & 3)] = acc[i][j];
            } else if (c < g.n) {
                y[(size_t)r * g.n + c] = acc[i][j];
            }
        }
    }
}

}  // namespace

void launch_gemm_u8i8(const uint8_t *x, const int8_t *w, int32_t *y, const GemmArgs &g, const uint16_t *groups,
                      cudaStream_t s) {
    const uint32_t cols = groups ? g.cols : g.n;
    if (!g.m || !cols || !g.k) return;
    const dim3 grid((g.m + kTile - 1) / kTile, (cols + kTile - 1) / kTile);
    gemm_u8i8_kernel<<<grid, 256, 0, s>>>(x, w, y, g, groups);
}

}  // namespace uq
