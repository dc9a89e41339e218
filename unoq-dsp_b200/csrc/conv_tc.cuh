// conv_tc.cuh -- tensor-core (tcgen05 kind::i8) implicit-GEMM convolution for plan code 14.
#pragma once
#include <cuda_runtime.h>

#include <cstddef>
#include <cstdint>
#include <functional>

#include "kernels.cuh"

namespace uq {

struct ConvTc;  // prepared weights + epilogue tables for one conv op

// A residual add (plan code 18) that consumes a conv's output and is computed in that conv's
// epilogue: the add's q block (host copy for its scale constants, device copy for its two
// tables) and which add operand the conv output is.
struct FusedAdd {
    const int32_t *q_host;
    const int32_t *q_dev;
    bool conv_is_b;
};

// Decide whether the tensor-core path takes this conv and, if so, prepare its device data
// (repacked weights, folded bias, requantisation tables) with `alloc`. Sets *out to nullptr
// when the CUDA-core path should run instead. Returns 0 or 2001.
// With `add`, the epilogue also applies that add (y is then the add's output, `res` its other
// operand); convs the fused form does not take get *out = nullptr.
int conv_tc_prepare(const int8_t *w_packed, const int32_t *q, const uint8_t *post_dev, const ConvGeom &g,
                    const std::function<void *(size_t)> &alloc, ConvTc **out, const FusedAdd *add = nullptr);
// Enqueue one conv; returns 0 or 2001 when the output tensor map cannot be encoded.
int conv_tc_launch(const ConvTc &c, const int8_t *x, int8_t *y, const ConvGeom &g, cudaStream_t s,
                   const int8_t *res = nullptr);
void conv_tc_free(ConvTc *c);
// Error code recorded by a timed-out device wait (0 = none); optionally cleared.
int conv_tc_error(bool reset);

}  // namespace uq
