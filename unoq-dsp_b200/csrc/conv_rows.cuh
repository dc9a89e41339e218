// conv_rows.cuh -- tensor-core row-GEMM convolution for few input channels (plan code 14 stems).
#pragma once
#include <cuda_runtime.h>

#include <cstddef>
#include <cstdint>
#include <functional>

#include "kernels.cuh"

namespace uq {

struct ConvRows;  // prepared banded weights, epilogue constants and border corrections

// Take the conv if it has ic <= 32, or ic <= 64 with oc <= 32 (UNOQ_CONV_ROWS_IC lowers the input
// bound), a kh x kw <= 3 x 3 kernel
// with dilation 1, equal strides 1 or 2, oc a multiple of 16 (<= 256) or 4 or 8, 16-byte input and
// output rows;
// prepare its device data with `alloc`. *out = nullptr when another path should run. Returns 0
// or 2001.
int conv_rows_prepare(const int8_t *w_packed, const int32_t *q, const uint8_t *post_dev, const ConvGeom &g,
                      const std::function<void *(size_t)> &alloc, ConvRows **out);
// Enqueue one conv; returns 0 or 2001 when a tensor map cannot be encoded.
int conv_rows_launch(const ConvRows &c, const int8_t *x, int8_t *y, const ConvGeom &g, cudaStream_t s);
void conv_rows_free(ConvRows *c);
// Site code recorded by a timed-out device wait of this kernel (0 = none); optionally cleared.
int conv_rows_error(bool reset);

}  // namespace uq
