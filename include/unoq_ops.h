/*
 * unoq_ops.h -- operator-level C ABI of libunoq_cuda.so: the reference's qnn.h / gemm.h /
 * kernels.h entry points (runtime/qnn.h:12-23, runtime/gemm.h:5-25, runtime/kernels.h:7) on B200.
 *
 * In the reference these are the functions graph.c calls for one op over its host arena. Here they
 * keep the names, argument meaning and return codes, with this difference: every DATA array
 * (activations x / b / y, weights w, parameter blocks q, post tables, GEMM operands) is DEVICE
 * memory of the device selected with ug_set_device (default 0). Tensor / op descriptors,
 * uq_validate's constants and ug_matmul_u8i8_selected's group list are host memory. Null or host
 * pointers where device memory is required give 22 (or, for the void functions, uq_status() 22)
 * and launch nothing. Every call is synchronous: it waits for all earlier work on the device, and
 * its outputs are written when it returns. Calls are serialised by a lock.
 *
 * Codes: 18 invalid parameters (qnn.c:209-252), 19 unsupported op code, 20 an image of the op
 * larger than 16 MiB, 22 bad call, 2001 CUDA error, 2002 no device.
 */
#ifndef UNOQ_OPS_H
#define UNOQ_OPS_H
#include <stdint.h>

#include "unoq_cuda.h"

#ifdef __cplusplus
extern "C" {
#endif

/* runtime/graph.h:16-17: 48-byte tensor and 32-byte op records of the UGN1 plan format. */
typedef struct {uint32_t offset, bytes, type, rank, d[4], flags, reserved[3];} UGTensor;
typedef struct {uint32_t code, a, b, out, p[4];} UGOp;

#define UQ_HEAD 20      /* runtime/qnn.h:8: words before the per-channel arrays of a q block */
#define UQ_MAX_K 8192   /* runtime/qnn.h:10 */
#define UQ_MAX_C 2048   /* runtime/qnn.h:11 */

/* Replaces uq_validate (runtime/qnn.c:209-252): the parameter-block check of codes 14-17, with
 * the loader's exact result (0 or 18) and the op's work added to *work. Host-only: `data` (the q
 * block) and `weights` are host copies, as the loader holds them; no GPU is touched. */
UG_API int uq_validate(const UGOp *op, const UGTensor *a, const UGTensor *b, const UGTensor *z, const UGTensor *t,
                       const void *data, const void *weights, uint64_t *work);
/* Replaces uq_run (runtime/qnn.c:1328-1382): conv (14), depthwise (15), pool (16) or table
 * softmax (17) of NHWC int8 `x` (descriptor a, any batch a->d[0]) into `y` (descriptor z) with
 * weights `w` and q block `q`. No 16 MiB arena limit on the batch: only one image of the op must
 * fit 16 MiB. A post table registered for `q` is applied (codes 14, 15). The parameters and weights
 * are read back and validated with the loader's rules (18 when they fail) and the op runs on the
 * executor's own kernels; the preparation is cached by content. `threads` is ignored. */
UG_API int uq_run(unsigned code, const UGTensor *a, const UGTensor *z, const int8_t *x, const int8_t *w, int8_t *y,
                  const int32_t *q, int threads);
/* Replace uq_add / uq_mean / uq_mul (runtime/qnn.c:175-198, 112-117): residual add through the
 * q block's two 256-entry tables (q: 520 words), spatial mean (q: count, xzp, yzp, multiplier,
 * shift), equal-shape multiply (q: xz, bz, yz, multiplier, shift, min, max). */
UG_API void uq_add(const int8_t *x, const int8_t *b, int8_t *y, uint32_t count, const int32_t *q);
UG_API void uq_mean(const int8_t *x, int8_t *y, unsigned batches, unsigned channels, const int32_t *q);
UG_API void uq_mul(const int8_t *x, const int8_t *b, int8_t *y, unsigned count, const int32_t *q);
/* Replaces uq_bmm (runtime/qnn.c:119-153): rank-3 int8 batched matmul; q = xz, wz, yz,
 * multiplier, shift, adj_x, adj_y. Returns 0 or 18. `threads` is ignored. */
UG_API int uq_bmm(const UGTensor *a, const UGTensor *b, const UGTensor *z, const int8_t *x, const int8_t *w, int8_t *y,
                  const int32_t *q, int threads);
/* Replace uq_post_reset / uq_post_register (runtime/qnn.c:158-161): the 256-byte table applied
 * after requantisation by every uq_run whose q block is `q` (both device pointers, matched by
 * address; at most 512 registrations). uq_post_reset also drops uq_run's prepared ops. */
UG_API void uq_post_reset(void);
UG_API void uq_post_register(const int32_t *q, const uint8_t *table);
/* Replaces uq_softmax_exact (runtime/qnn.c:87-107): gemmlowp-exact softmax over rows of q[0]
 * bytes, q[1..256] the Q31 exponent table. */
UG_API void uq_softmax_exact(const int8_t *x, int8_t *y, unsigned bytes, const int32_t *q);
/* Result of the last operator-ABI call (0 or a code above): the status of the void functions. */
UG_API int uq_status(void);

/* Replace the integer GEMMs of runtime/gemm.h: Y[m][n] = sum_t X_u8[m][t] * W_s8(n, t) as int32,
 * Y dense m x n. ug_matmul_u8i8 (gemm.c:667-679): X dense (row stride k); W row-major n x k
 * (packed = 0) or in the packed layout (j/4)*k*4 + (t/8)*32 + (j%4)*8 + t%8 (packed = 1, k a
 * multiple of 8). _strided (gemm.c:708-745): packed W, X row stride xs. _dot4 (gemm.c:911-948):
 * W in the dot4 layout (j/4)*k*4 + (t/4)*16 + (j%4)*4 + t%4. _selected (gemm.c:681-706): packed W,
 * only the 4-channel groups starting at groups[0..count) (host array) are written. Return 0 or 18
 * with the reference's argument rules. */
UG_API int ug_matmul_u8i8(const uint8_t *x, const int8_t *w, int32_t *y, unsigned m, unsigned n, unsigned k,
                          int packed, int threads);
UG_API int ug_matmul_u8i8_strided(const uint8_t *x, const int8_t *w, int32_t *y, unsigned m, unsigned n, unsigned k,
                                  unsigned xs);
UG_API int ug_matmul_u8i8_dot4(const uint8_t *x, const int8_t *w, int32_t *y, unsigned m, unsigned n, unsigned k,
                               unsigned xs);
UG_API int ug_matmul_u8i8_selected(const uint8_t *x, const int8_t *w, int32_t *y, unsigned m, unsigned n, unsigned k,
                                   unsigned xs, const uint16_t *groups, unsigned count);
/* Replaces ug_gemm_available (runtime/gemm.c:617): 1 when a CUDA device is present. */
UG_API int ug_gemm_available(void);

/* runtime/kernels.h:7 declares ug_dot_u8i8 as a static inline header function (a scalar dot
 * product of unsigned and signed bytes, no exported symbol); this header keeps that contract for
 * host callers. */
static inline int32_t ug_dot_u8i8(const uint8_t *x, const int8_t *w, uint32_t n) {
    int32_t sum = 0;
    for (uint32_t i = 0; i < n; i++) sum += (int32_t)x[i] * w[i];
    return sum;
}

#ifdef __cplusplus
}
#endif
#endif
