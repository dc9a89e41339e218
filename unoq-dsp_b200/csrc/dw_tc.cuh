// dw_tc.cuh -- depthwise convolution (plan code 15) on the tensor cores: block-diagonal MMAs over a
// TMA-loaded input window.
#pragma once
#include <cuda_runtime.h>

#include <cstddef>
#include <cstdint>
#include <functional>

#include "kernels.cuh"

namespace uq {

struct DwTc;  // prepared diagonal weight blocks and requantisation constants

// Take a 3x3 / 5x5 depthwise conv with equal strides 1 or 2, no dilation, channels a multiple of
// 32 and output rows of at most 120 pixels, when UNOQ_DW_TC=1 (off by default: slower than the
// dp4a kernel); prepare its device data with `alloc`. *out = nullptr when another path should
// run. Returns 0 or 2001.
int dw_tc_prepare(const int8_t *w, const int32_t *q, const uint8_t *post_dev, const ConvGeom &g,
                  const std::function<void *(size_t)> &alloc, DwTc **out);
// Enqueue one depthwise conv; returns 0, or 2001 when the batch has too many tiles.
int dw_tc_launch(const DwTc &d, const int8_t *x, int8_t *y, const ConvGeom &g, cudaStream_t s);
void dw_tc_free(DwTc *d);
// Site code recorded by a timed-out device wait of this kernel (0 = none); optionally cleared.
int dw_tc_error(bool reset);

}  // namespace uq
