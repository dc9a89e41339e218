// conv_small.cuh -- direct dp4a convolution for 3x3 convs with few input channels (plan code 14).
#pragma once
#include <cuda_runtime.h>

#include <cstddef>
#include <cstdint>
#include <functional>

#include "kernels.cuh"

namespace uq {

struct ConvSmall;  // prepared weight words + requantisation constants

// Take 3x3, undilated, stride 1 or 2 convs with ic <= 16 and few output channels (the RGB stems,
// 8- and 16-channel layers), where a tensor-core tile would be nearly empty; sets *out to nullptr
// for any other conv. Returns 0 or 2001.
int conv_small_prepare(const int8_t *w_packed, const int32_t *q, const uint8_t *post_dev, const ConvGeom &g,
                       const std::function<void *(size_t)> &alloc, ConvSmall **out);
int conv_small_launch(const ConvSmall &c, const int8_t *x, int8_t *y, const ConvGeom &g, cudaStream_t s);
void conv_small_free(ConvSmall *c);

}  // namespace uq
