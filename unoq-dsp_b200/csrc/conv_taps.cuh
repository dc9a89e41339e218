// conv_taps.cuh -- tensor-core convolution with per-tap TMA-loaded A tiles (plan code 14, ic % 32 == 0).
#pragma once
#include <cuda_runtime.h>

#include <cstddef>
#include <cstdint>
#include <functional>

#include "kernels.cuh"

namespace uq {

struct ConvTaps;  // prepared weights per (tap, channel chunk), epilogue constants, border corrections

// Take the conv if ic % 128 == 0 (ic % 32 == 0 with UNOQ_CONV_TAPS=all), its kernel is at most 3 x 3
// (and not 1 x 1), its strides are equal (1 or 2) and oc % 16 == 0; prepare its device data with
// `alloc`. *out = nullptr when another path should run. Returns 0 or 2001.
int conv_taps_prepare(const int8_t *w_packed, const int32_t *q, const uint8_t *post_dev, const ConvGeom &g,
                      const std::function<void *(size_t)> &alloc, ConvTaps **out);
// Enqueue one conv; returns 0 or 2001 when the input tensor map cannot be encoded.
int conv_taps_launch(const ConvTaps &c, const int8_t *x, int8_t *y, const ConvGeom &g, cudaStream_t s);
void conv_taps_free(ConvTaps *c);
// Site code recorded by a timed-out device wait of this kernel (0 = none); optionally cleared.
int conv_taps_error(bool reset);

}  // namespace uq
