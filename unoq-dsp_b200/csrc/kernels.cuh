// kernels.cuh -- launch interface of every device kernel in libunoq_cuda.
//
// Batching convention: every activation tensor of a plan is stored as `images` back-to-back
// copies of its batch-1 layout, so an NHWC tensor of a batch-1 plan becomes an NHWC tensor
// with n = images * d0, and element-wise ops simply see images * bytes elements.
#pragma once
#include <cuda_runtime.h>
#include <cstddef>
#include <cstdint>

#include "common.cuh"

namespace uq {

// Spatial geometry of a conv/depthwise/pool op, from the plan's q[0:20] (qnn.c:12-16).
struct ConvGeom {
    int n;                // images * d0
    int ih, iw, ic;       // input
    int oh, ow, oc;       // output
    int kh, kw, sh, sw, dh, dw, pt, pl;
    int xzp;              // input zero point (s8)
    int kp;               // padded reduction length (multiple of 8)
};

// Code 14, CUDA-core form: the reference's u8 im2col column times the plan-packed weights
// (gemm.h:9 layout), i.e. exactly sum_t col[t] * w[j][t] with borders and K padding held at
// xzp + 128, followed by requantisation. Handles every admissible conv.
void launch_conv_simt(const int8_t *x, const int8_t *w_packed, int8_t *y, const ConvGeom &g, const Requant &r,
                      cudaStream_t s);
// Code 15: depthwise, weights [kh*kw][C] as in the plan (tflite.py:153).
void launch_depthwise(const int8_t *x, const int8_t *w, int8_t *y, const ConvGeom &g, const Requant &r, cudaStream_t s);
// Code 16: average (is_max = 0) or max pool, clamp to [lo, hi].
void launch_pool(const int8_t *x, int8_t *y, const ConvGeom &g, int is_max, int lo, int hi, cudaStream_t s);
// Code 17: table softmax over rows of `width`, table = q + 20 (Q24, 256 entries).
void launch_softmax_table(const int8_t *x, int8_t *y, size_t rows, int width, const int32_t *table, int lo, int hi,
                          cudaStream_t s);
// Code 28: exact fixed-point softmax, q = [width, 256-entry Q31 exp table].
void launch_softmax_exact(const int8_t *x, int8_t *y, size_t rows, int width, const int32_t *q, cudaStream_t s);
// The same arithmetic, one thread per row (the operator ABI's uq_softmax_exact).
void launch_softmax_exact_rows(const int8_t *x, int8_t *y, size_t rows, int width, const int32_t *q, cudaStream_t s);
// Code 18: residual add through prepared tables; q is the 520-word device parameter block.
void launch_add(const int8_t *x, const int8_t *b, int8_t *y, size_t count, const int32_t *q, cudaStream_t s);
// Code 25: equal-shape multiply; q7 = xz, bz, yz, mult, shift, lo, hi (host values).
void launch_mul(const int8_t *x, const int8_t *b, int8_t *y, size_t count, const int32_t q7[7], cudaStream_t s);
// Code 22: byte table; flip = 128 for int8 sources.
void launch_lut(const uint8_t *x, uint8_t *y, size_t count, const uint8_t *table, unsigned flip, cudaStream_t s);
// Code 24: spatial mean; q5 = count, xzp, yzp, mult, shift.
void launch_mean(const int8_t *x, int8_t *y, size_t batches, int channels, const int32_t q5[5], cudaStream_t s);
// Code 27: batched matmul; q7 = xz, wz, yz, mult, shift, adj_x, adj_y. k = reduction length.
void launch_bmm(const int8_t *x, const int8_t *w, int8_t *y, size_t batches, int m, int n, int k, const int32_t q7[7],
                cudaStream_t s);

// Byte movement. Rank <= 5 (a leading image axis plus the plan's rank <= 4).
struct Shape5 {
    int rank;
    uint32_t d[5];
};
// Code 10: z[i] = a[permuted i]; perm[d] names the source axis of output axis d.
void launch_permute(const uint8_t *a, uint8_t *z, const Shape5 &in, const int perm[5], int elem_bytes, cudaStream_t s);
// Code 26: z = a[begin : begin + zshape] per axis.
void launch_slice(const uint8_t *a, uint8_t *z, const Shape5 &in, const Shape5 &out, const uint32_t begin[5],
                  cudaStream_t s);
// Code 20: rows of a (ac bytes) and b (bc bytes) interleaved into z.
void launch_concat(const uint8_t *a, const uint8_t *b, uint8_t *z, size_t outer, size_t ac, size_t bc, cudaStream_t s);
// Code 21: nearest resize from prepared byte offsets (device table of oh + ow words).
void launch_resize(const uint8_t *a, uint8_t *z, int n, int ih, int iw, int c, int oh, int ow, const uint32_t *offsets,
                   cudaStream_t s);
// Code 23: constant pad with explicit image axis; pads = before/after per plan axis.
void launch_pad(const uint8_t *a, uint8_t *z, int images, const uint32_t ad[4], const uint32_t zd[4], const int32_t pads[8],
                int8_t value, cudaStream_t s);
// Code 19 (and plain copies): per image, concatenate `count` segments of the given sizes.
struct Segments {
    int count;
    const uint8_t *src[32];
    uint32_t bytes[32];
    uint32_t dst_offset[32];
};
void launch_pack(const Segments &segs, uint8_t *z, uint32_t z_bytes, int images, cudaStream_t s);
// Code 20 chains fused: z row r = row r of each input in turn (concatenation along the innermost
// axis of up to 8 inputs; widths in bytes per row).
struct ConcatInputs {
    int count;
    const uint8_t *src[8];
    uint32_t width[8];
};
void launch_concat_multi(const ConcatInputs &in, uint8_t *z, size_t rows, cudaStream_t s);
// Code 20 chains whose inputs may be code-22 tables (of slices) read by nothing else: z row r = for
// each part k in turn, bytes [off_k, off_k + out_w_k) of row r of src_k (rows of in_w_k bytes),
// mapped through table_k (y = table[x ^ flip]) when it is set.
struct ConcatParts {
    int count;
    const uint8_t *src[8];
    uint32_t in_w[8], off[8], out_w[8];
    const uint8_t *table[8];
    unsigned flip[8];
};
void launch_concat_parts(const ConcatParts &in, uint8_t *z, size_t rows, cudaStream_t s);
// Code 26 (innermost axis) followed by code 22, in one pass: y[r][c] = table[x[r][off + c] ^ flip]
// for c < out_w, x rows of in_w bytes.
void launch_lut_rows(const uint8_t *x, uint8_t *y, size_t rows, uint32_t in_w, uint32_t off, uint32_t out_w,
                     const uint8_t *table, unsigned flip, cudaStream_t s);
void launch_copy(const void *src, void *dst, size_t bytes, cudaStream_t s);

}  // namespace uq
