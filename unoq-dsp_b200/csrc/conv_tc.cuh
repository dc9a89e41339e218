// conv_tc.cuh -- tensor-core (tcgen05 kind::i8) implicit-GEMM convolution for plan code 14.
#pragma once
#include <cuda_runtime.h>

#include <cstddef>
#include <cstdint>
#include <functional>

#include "kernels.cuh"

namespace uq {

struct ConvTc;  // prepared weights + epilogue tables for one conv op

// Decide whether the tensor-core path takes this conv and, if so, prepare its device data
// (repacked weights, folded bias, requantisation tables) with `alloc`. Sets *out to nullptr
// when the CUDA-core path should run instead. Returns 0 or 2001.
int conv_tc_prepare(const int8_t *w_packed, const int32_t *q, const uint8_t *post_dev, const ConvGeom &g,
                    const std::function<void *(size_t)> &alloc, ConvTc **out);
// Enqueue one conv; returns 0 or 2001 when the output tensor map cannot be encoded.
int conv_tc_launch(const ConvTc &c, const int8_t *x, int8_t *y, const ConvGeom &g, cudaStream_t s);
void conv_tc_free(ConvTc *c);
// Error code recorded by a timed-out device wait (0 = none); optionally cleared.
int conv_tc_error(bool reset);

}  // namespace uq
