// gemm.cuh -- launch interface of the raw integer GEMM (k_gemm.cu) behind the operator ABI's
// ug_matmul_u8i8 family (runtime/gemm.h:5-25).
#pragma once
#include <cuda_runtime.h>

#include <cstdint>

namespace uq {

enum GemmLayout : int { kGemmRowMajor = 0, kGemmPacked = 1, kGemmDot4 = 2 };

struct GemmArgs {
    uint32_t m, n, k;     // rows, output channels (row length of Y), reduction length
    uint32_t xs;          // bytes between rows of X
    uint32_t cols;        // with a group list: 4 x the number of groups (the columns computed)
    int layout;           // GemmLayout of W
    bool x_aligned;       // X and xs allow aligned 32-bit loads
    bool w_aligned;       // W's words are 4-byte aligned
};

// Y[m][n] = sum_t X[m][t] W(n, t) as int32. With `groups` (device array of cols / 4 channel
// offsets, each a multiple of 4), only the channels groups[g] .. groups[g] + 3 are written.
void launch_gemm_u8i8(const uint8_t *x, const int8_t *w, int32_t *y, const GemmArgs &g, const uint16_t *groups,
                      cudaStream_t s);

}  // namespace uq
