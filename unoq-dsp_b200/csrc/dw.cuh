// dw.cuh -- tiled depthwise convolution (plan code 15) with shared-memory halo staging.
#pragma once
#include <cuda_runtime.h>

#include <cstddef>
#include <cstdint>
#include <functional>

#include "kernels.cuh"

namespace uq {

struct DwFast;  // prepared transposed weights + requantisation constants

// Prepare the tiled kernel for 3x3 / 5x5, stride 1 or 2, undilated, channels % 16 == 0; sets
// *out to nullptr for other shapes (the generic kernel then runs). Returns 0 or 2001.
int dw_prepare(const int8_t *w, const int32_t *q, const uint8_t *post_dev, const ConvGeom &g,
               const std::function<void *(size_t)> &alloc, DwFast **out);
int dw_launch(const DwFast &d, const int8_t *x, int8_t *y, const ConvGeom &g, cudaStream_t s);
void dw_free(DwFast *d);

}  // namespace uq
