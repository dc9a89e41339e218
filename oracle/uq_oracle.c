/*
 * uq_oracle.c -- TEST INFRASTRUCTURE ONLY (parity checker), never part of the product.
 *
 * A plain-C, scalar restatement of the reference unoq-dsp INT8 graph executor
 * (runtime/graph.c run_inner + runtime/qnn.c), written from the reference's semantics
 * rather than its Hexagon-tuned code. Every vision op is evaluated in its canonical
 * scalar form: the conv uses the explicit u8 im2col column and packed-weight dot product
 * of the reference's "scalar oracle" branch (qnn.c:1197), depthwise/pool use the generic
 * row loop (qnn.c:1228-1245), and every requantisation goes through one restated
 * `scale()` (qnn.c:61-83). The reference's affine fast paths (qnn.c:264-351, 541-647,
 * requant2.S) are proven equal to that form in the reference itself.
 *
 * Only tests/, __graft_entry__.smoke() and bench.py's cpu_baseline leg may load this
 * library, and only as the checker / CPU baseline. Parity is pinned by running it next to
 * the reference runtime compiled from its own sources (oracle/_ref) on the bundled models
 * and on synthetic single-op plans; see tests/test_oracle.py.
 *
 * Entry point: uqo_run(plan, plan_bytes, input, output, images) runs `images` independent
 * images back to back (inputs and outputs contiguous, one plan-sized tensor each).
 * Returns 0, or the reference's error code for the condition (graph.h / graph.c).
 * Legacy fp32 opcodes (1-4, 6-9, 11-13) are outside the INT8 hot path and return 19.
 */
#include <stdint.h>
#include <stdlib.h>
#include <string.h>

typedef struct { uint32_t magic, version, nt, no, arena_bytes, input, output, reserved; } OHeader;
typedef struct { uint32_t offset, bytes, type, rank, d[4], flags, reserved[3]; } OTensor;
typedef struct { uint32_t code, a, b, out, p[4]; } OOp;

#define O_MAGIC 0x55474e31u
#define O_HEAD 20 /* qnn.h:8 UQ_HEAD */

/* qnn.c:61-83 `scale`: TFLite double rounding. Optional pre-multiply left shift,
 * rounding-doubling high multiply (v*m + 2^30) >> 31 on the full int64 product, then a
 * ties-away-from-zero rounding right shift for negative exponents. */
static int32_t o_scale(int32_t v, int32_t m, int shift) {
    if (shift > 0) v = (int32_t)((uint32_t)v << shift);
    int64_t p = (int64_t)v * (int64_t)m;
    int32_t h = (int32_t)((p + ((int64_t)1 << 30)) >> 31);
    if (shift >= 0) return h;
    unsigned s = (unsigned)(-shift);
    uint32_t mask = ((uint32_t)1 << s) - 1u;
    int32_t base = h >> s;
    uint32_t rem = (uint32_t)h & mask;
    return base + (rem > ((mask >> 1) + (h < 0 ? 1u : 0u)) ? 1 : 0);
}

static int8_t o_clamp(int32_t v, int32_t lo, int32_t hi) {
    return (int8_t)(v < lo ? lo : v > hi ? hi : v);
}

static uint32_t o_width(uint32_t type) { /* graph.c:31 */
    return type == 1 || type == 4 ? 4u : type == 2 || type == 3 ? 1u : 0u;
}

/* Packed INT8 weight byte for output channel j, reduction index t (gemm.h:9). */
static int8_t o_packed(const int8_t *w, unsigned kp, unsigned j, unsigned t) {
    return w[(j / 4) * kp * 4 + (t / 8) * 32 + (j % 4) * 8 + t % 8];
}

/* qnn.c:162-173 `uq_post`: optional fused 256-entry byte table after the clamp. */
static void o_post(const uint8_t *table, int8_t *y, size_t count) {
    if (!table) return;
    for (size_t j = 0; j < count; j++) y[j] = (int8_t)table[(int)y[j] + 128];
}

/* Code 14 (qnn.c:1101-1227, scalar branch qnn.c:1197 and the column builders
 * qnn.c:1139-1169 / gather_rgb3 990-1045): u8 column = x ^ 0x80, borders and the K
 * padding hold xzp + 128; acc = sum col[t] * w[j][t]; y = clamp(scale(acc + bias) + yzp). */
static void o_conv(const OTensor *a, const OTensor *z, const int8_t *x, const int8_t *w,
                   int8_t *y, const int32_t *q, const uint8_t *post) {
    unsigned ih = a->d[1], iw = a->d[2], ic = (unsigned)q[16], oc = (unsigned)q[17];
    unsigned kp = (unsigned)q[18], oh = (unsigned)q[10], ow = (unsigned)q[11];
    unsigned rows = z->d[0] * z->d[1] * z->d[2];
    const int32_t *bias = q + O_HEAD, *mult = bias + oc, *shift = mult + oc;
    uint8_t *col = (uint8_t *)malloc(kp ? kp : 1);
    uint8_t fill = (uint8_t)(q[12] + 128);
    for (unsigned row = 0; row < rows; row++) {
        unsigned n = row / (oh * ow), yy = (row / ow) % oh, xx = row % ow, c = 0;
        for (int ky = 0; ky < q[0]; ky++)
            for (int kx = 0; kx < q[1]; kx++) {
                int sy = (int)yy * q[2] - q[6] + ky * q[4], sx = (int)xx * q[3] - q[7] + kx * q[5];
                int valid = sy >= 0 && sx >= 0 && (unsigned)sy < ih && (unsigned)sx < iw;
                const int8_t *src = valid ? x + (((size_t)n * ih + (unsigned)sy) * iw + (unsigned)sx) * ic : 0;
                for (unsigned ch = 0; ch < ic; ch++) col[c++] = valid ? (uint8_t)((uint8_t)src[ch] ^ 128u) : fill;
            }
        for (; c < kp; c++) col[c] = fill;
        for (unsigned j = 0; j < oc; j++) {
            int32_t acc = 0;
            for (unsigned t = 0; t < kp; t++) acc += (int32_t)col[t] * o_packed(w, kp, j, t);
            int32_t v = o_scale((int32_t)((uint32_t)acc + (uint32_t)bias[j]), mult[j], shift[j]) + q[13];
            y[(size_t)row * oc + j] = o_clamp(v, q[14], q[15]);
        }
    }
    free(col);
    o_post(post, y, (size_t)rows * oc);
}

/* Codes 15/16 generic row loop (qnn.c:1228-1245). Depthwise: acc starts at the corrected
 * bias and adds (x + 128) * w over every tap, borders contributing (xzp + 128) * w.
 * Pool: max (start -128) or sum of raw int8 over valid taps, average rounded half away
 * from zero with C truncating division. */
static void o_window(unsigned code, const OTensor *a, const OTensor *z, const int8_t *x,
                     const int8_t *w, int8_t *y, const int32_t *q, const uint8_t *post) {
    unsigned ih = a->d[1], iw = a->d[2], ic = (unsigned)q[16], oc = (unsigned)q[17];
    unsigned oh = (unsigned)q[10], ow = (unsigned)q[11];
    unsigned rows = z->d[0] * z->d[1] * z->d[2];
    const int32_t *bias = q + O_HEAD, *mult = bias + oc, *shift = mult + oc;
    int32_t *acc = (int32_t *)malloc(sizeof(int32_t) * (oc ? oc : 1));
    for (unsigned row = 0; row < rows; row++) {
        unsigned n = row / (oh * ow), yy = (row / ow) % oh, xx = row % ow, valid_count = 0;
        for (unsigned ch = 0; ch < oc; ch++) acc[ch] = code == 15 ? bias[ch] : q[19] ? -128 : 0;
        for (int ky = 0; ky < q[0]; ky++)
            for (int kx = 0; kx < q[1]; kx++) {
                int sy = (int)yy * q[2] - q[6] + ky * q[4], sx = (int)xx * q[3] - q[7] + kx * q[5];
                int valid = sy >= 0 && sx >= 0 && (unsigned)sy < ih && (unsigned)sx < iw;
                const int8_t *src = valid ? x + (((size_t)n * ih + (unsigned)sy) * iw + (unsigned)sx) * ic : 0;
                valid_count += (unsigned)valid;
                if (code == 15) {
                    const int8_t *wt = w + (size_t)(ky * q[1] + kx) * oc;
                    for (unsigned ch = 0; ch < oc; ch++)
                        acc[ch] += (valid ? (int32_t)src[ch] + 128 : q[12] + 128) * wt[ch];
                } else if (valid) {
                    for (unsigned ch = 0; ch < oc; ch++) {
                        if (q[19]) { if (src[ch] > acc[ch]) acc[ch] = src[ch]; }
                        else acc[ch] += src[ch];
                    }
                }
            }
        for (unsigned ch = 0; ch < oc; ch++) {
            int32_t v = acc[ch];
            if (code == 15) v = o_scale(v, mult[ch], shift[ch]) + q[13];
            else if (!q[19]) {
                int half = (int)valid_count / 2;
                v = (v + (v > 0 ? half : -half)) / (int)valid_count;
            }
            y[(size_t)row * oc + ch] = o_clamp(v, q[14], q[15]);
        }
    }
    free(acc);
    if (code == 15) o_post(post, y, (size_t)rows * oc);
}

/* Code 17 (qnn.c:1082-1088): table softmax over the last axis with a Q24 table at q[20:]. */
static void o_softmax_table(const OTensor *a, const int8_t *x, int8_t *y, const int32_t *q) {
    unsigned ic = (unsigned)q[16];
    for (unsigned base = 0; base < a->bytes; base += ic) {
        int mx = -128;
        for (unsigned c = 0; c < ic; c++) if (x[base + c] > mx) mx = x[base + c];
        uint64_t sum = 0;
        for (unsigned c = 0; c < ic; c++) sum += (uint32_t)q[O_HEAD + mx - x[base + c]];
        for (unsigned c = 0; c < ic; c++) {
            uint64_t v = (uint64_t)(uint32_t)q[O_HEAD + mx - x[base + c]] * 256u;
            int32_t r = (int32_t)((v + sum / 2) / sum) - 128;
            y[base + c] = o_clamp(r, q[14], q[15]);
        }
    }
}

/* Code 28 (qnn.c:87-107): gemmlowp-style exact softmax. Sum of Q12-rounded table terms,
 * normalised reciprocal by three Newton-Raphson steps in Q31, then a rounding shift. */
static void o_softmax_exact(const int8_t *x, int8_t *y, unsigned bytes, const int32_t *q) {
    unsigned width = (unsigned)q[0];
    const int32_t *lut = q + 1;
    for (unsigned base = 0; base < bytes; base += width) {
        int mx = -128;
        for (unsigned j = 0; j < width; j++) if (x[base + j] > mx) mx = x[base + j];
        uint32_t sum = 0;
        for (unsigned j = 0; j < width; j++) sum += ((uint32_t)lut[mx - x[base + j]] + 2048u) >> 12;
        unsigned leading = (unsigned)__builtin_clz(sum), exponent = 35 - leading;
        uint32_t normalized = (sum << leading) - 0x80000000u;
        int32_t half = (int32_t)(((uint64_t)normalized + 2147483648u) >> 1);
        int32_t r = (int32_t)(1515870810u + (uint32_t)o_scale(half, -1010580540, 0));
        for (unsigned step = 0; step < 3; step++) {
            int32_t err = (int32_t)(536870912u - (uint32_t)o_scale(half, r, 0));
            r = (int32_t)((uint32_t)r + (uint32_t)o_scale(r, err, 0) * 4u);
        }
        int64_t doubled = (int64_t)r * 2;
        r = doubled > 2147483647 ? 2147483647 : (int32_t)doubled;
        for (unsigned j = 0; j < width; j++) {
            uint32_t value = (uint32_t)o_scale(r, lut[mx - x[base + j]], 0);
            unsigned rounded = exponent >= 32 ? 0u : (value + (1u << (exponent - 1))) >> exponent;
            y[base + j] = (int8_t)(rounded > 255 ? 127 : (int)rounded - 128);
        }
    }
}

/* Code 18 (qnn.c:175-183): residual add through two prepared int32 tables. */
static void o_add(const int8_t *x, const int8_t *b, int8_t *y, uint32_t count, const int32_t *q) {
    const int32_t *tx = q + 8, *tb = q + 264;
    for (uint32_t i = 0; i < count; i++) {
        int32_t sum = (int32_t)((uint32_t)tx[(int)x[i] + 128] + (uint32_t)tb[(int)b[i] + 128]);
        y[i] = o_clamp(o_scale(sum, q[0], q[1]) + q[2], q[3], q[4]);
    }
}

/* Code 24 (qnn.c:184-198): spatial mean, q = count, xzp, yzp, multiplier, shift. */
static void o_mean(const int8_t *x, int8_t *y, unsigned batches, unsigned channels, const int32_t *q) {
    for (unsigned n = 0; n < batches; n++)
        for (unsigned c = 0; c < channels; c++) {
            int32_t sum = 0;
            for (unsigned p = 0; p < (unsigned)q[0]; p++) sum += x[((size_t)n * (unsigned)q[0] + p) * channels + c];
            y[(size_t)n * channels + c] = o_clamp(o_scale(sum - q[0] * q[1], q[3], q[4]) + q[2], -128, 127);
        }
}

/* Code 25 (qnn.c:112-117): equal-shape multiply, q = xz, bz, yz, multiplier, shift, lo, hi. */
static void o_mul(const int8_t *x, const int8_t *b, int8_t *y, unsigned count, const int32_t *q) {
    for (unsigned i = 0; i < count; i++)
        y[i] = o_clamp(o_scale(((int)x[i] - q[0]) * ((int)b[i] - q[1]), q[3], q[4]) + q[2], q[5], q[6]);
}

/* Code 27 (qnn.c:119-153): batched int8 matmul. The reference's u8 column algebra
 * acc - (xz+128)*sum(w) - wz*sum(x+128) + k*(xz+128)*wz equals sum (x - xz) * (w - wz). */
static void o_bmm(const OTensor *a, const OTensor *z, const int8_t *x, const int8_t *w,
                  int8_t *y, const int32_t *q) {
    unsigned batches = z->d[0], m = z->d[1], n = z->d[2], k = a->d[q[5] ? 1 : 2];
    for (unsigned bt = 0; bt < batches; bt++) {
        const int8_t *xb = x + (size_t)bt * m * k, *wb = w + (size_t)bt * k * n;
        for (unsigned r = 0; r < m; r++)
            for (unsigned c = 0; c < n; c++) {
                int32_t v = 0;
                for (unsigned t = 0; t < k; t++) {
                    int xv = xb[q[5] ? (size_t)t * m + r : (size_t)r * k + t];
                    int wv = wb[q[6] ? (size_t)c * k + t : (size_t)t * n + c];
                    v += (xv - q[0]) * (wv - q[1]);
                }
                v = o_scale(v, q[3], q[4]) + q[2];
                y[(size_t)bt * m * n + (size_t)r * n + c] = o_clamp(v, -128, 127);
            }
    }
}

typedef struct {
    OHeader h;
    const OTensor *ts;
    const OOp *ops;
    unsigned char *arena;
} OGraph;

/* One image through the op list (graph.c:285-423, INT8 opcodes only). */
static int o_run_image(OGraph *g, const void *in, void *out) {
    const OTensor *ts = g->ts;
    unsigned char *A = g->arena;
    memcpy(A + ts[g->h.input].offset, in, ts[g->h.input].bytes);
    for (uint32_t i = 0; i < g->h.no; i++) {
        const OOp *o = g->ops + i;
        const OTensor *a = ts + o->a, *b = ts + o->b, *z = ts + o->out;
        unsigned char *ap = A + a->offset, *bp = A + b->offset, *zp = A + z->offset;
        switch (o->code) {
        case 14: case 15: case 16: case 17: {
            const int32_t *q = (const int32_t *)(A + ts[o->p[0]].offset);
            const uint8_t *post = (o->code == 14 || o->code == 15) && o->p[1] ? A + ts[o->p[1] - 1].offset : 0;
            if (o->code == 14) o_conv(a, z, (const int8_t *)ap, (const int8_t *)bp, (int8_t *)zp, q, post);
            else if (o->code == 17) o_softmax_table(a, (const int8_t *)ap, (int8_t *)zp, q);
            else o_window(o->code, a, z, (const int8_t *)ap, (const int8_t *)bp, (int8_t *)zp, q, post);
            break;
        }
        case 28: o_softmax_exact((const int8_t *)ap, (int8_t *)zp, a->bytes, (const int32_t *)bp); break;
        case 27: o_bmm(a, z, (const int8_t *)ap, (const int8_t *)bp, (int8_t *)zp, (const int32_t *)(A + ts[o->p[0]].offset)); break;
        case 26: { /* graph.c:306-313: strided slice, p = begin index per axis */
            size_t stride[4], step = 1, offset = 0;
            unsigned idx[4] = {0, 0, 0, 0}, last = a->rank - 1, span = z->d[last];
            for (int d = (int)a->rank - 1; d >= 0; d--) { stride[d] = step; offset += o->p[d] * step; step *= a->d[d]; }
            for (size_t j = 0; j < z->bytes; j += span) {
                memcpy(zp + j, ap + offset, span);
                for (int d = (int)last - 1; d >= 0; d--) {
                    offset += stride[d];
                    if (++idx[d] < z->d[d]) break;
                    offset -= idx[d] * stride[d];
                    idx[d] = 0;
                }
            }
            break;
        }
        case 25: o_mul((const int8_t *)ap, (const int8_t *)bp, (int8_t *)zp, z->bytes, (const int32_t *)(A + ts[o->p[0]].offset)); break;
        case 24: o_mean((const int8_t *)ap, (int8_t *)zp, a->d[0], a->d[3], (const int32_t *)bp); break;
        case 23: { /* graph.c:318-330: constant pad, q = before/after per axis */
            const int32_t *q = (const int32_t *)bp;
            memset(zp, (int)(int8_t)(int32_t)o->p[0], z->bytes);
            for (unsigned n = 0; n < a->d[0]; n++)
                for (unsigned h = 0; h < a->d[1]; h++)
                    for (unsigned w = 0; w < a->d[2]; w++) {
                        size_t off = ((((size_t)n + q[0]) * z->d[1] + h + q[2]) * z->d[2] + w + q[4]) * z->d[3] + q[6];
                        memcpy(zp + off, ap + (((size_t)n * a->d[1] + h) * a->d[2] + w) * a->d[3], a->d[3]);
                    }
            break;
        }
        case 22: { /* graph.c:331-341: byte table, int8 sources index with x ^ 0x80 */
            unsigned flip = a->type == 3 ? 128u : 0u;
            for (uint32_t j = 0; j < a->bytes; j++) zp[j] = bp[ap[j] ^ flip];
            break;
        }
        case 21: { /* graph.c:342-346: nearest resize from prepared byte offsets */
            const uint32_t *q = (const uint32_t *)bp;
            size_t c = a->d[3], stride = (size_t)a->d[1] * a->d[2] * c, off = 0;
            for (unsigned n = 0; n < a->d[0]; n++)
                for (unsigned h = 0; h < z->d[1]; h++)
                    for (unsigned w = 0; w < z->d[2]; w++) {
                        memcpy(zp + off, ap + n * stride + q[h] + q[z->d[1] + w], c);
                        off += c;
                    }
            break;
        }
        case 20: { /* graph.c:347-355: concatenation of a then b along p[0] */
            size_t outer = 1, inner = 1;
            unsigned axis = o->p[0];
            for (unsigned d = 0; d < axis; d++) outer *= a->d[d];
            for (unsigned d = axis + 1; d < a->rank; d++) inner *= a->d[d];
            size_t ac = a->d[axis] * inner, bc = b->d[axis] * inner;
            for (size_t r = 0; r < outer; r++) {
                memcpy(zp + r * (ac + bc), ap + r * ac, ac);
                memcpy(zp + r * (ac + bc) + ac, bp + r * bc, bc);
            }
            break;
        }
        case 19: { /* graph.c:356-360: pack listed tensors back to back */
            const uint32_t *list = (const uint32_t *)bp;
            size_t off = 0;
            for (unsigned j = 0; j < b->bytes / 4; j++) {
                const OTensor *t = ts + list[j];
                memcpy(zp + off, A + t->offset, t->bytes);
                off += t->bytes;
            }
            break;
        }
        case 18: o_add((const int8_t *)ap, (const int8_t *)bp, (int8_t *)zp, z->bytes, (const int32_t *)(A + ts[o->p[0]].offset)); break;
        case 10: { /* graph.c:385-391: general axis permutation, any element width */
            size_t stride[4], acc = 1;
            for (int d = (int)a->rank - 1; d >= 0; d--) { stride[d] = acc; acc *= a->d[d]; }
            uint32_t w = o_width(a->type), idx[4] = {0, 0, 0, 0};
            size_t src = 0, count = z->bytes / w;
            for (size_t j = 0; j < count; j++) {
                memcpy(zp + j * w, ap + src * w, w);
                for (int d = (int)z->rank - 1; d >= 0; d--) {
                    size_t step = stride[o->p[d]];
                    src += step;
                    if (++idx[d] < z->d[d]) break;
                    src -= idx[d] * step;
                    idx[d] = 0;
                }
            }
            break;
        }
        case 5: memcpy(zp, ap, z->bytes); break; /* graph.c:408 */
        default: return 19;
        }
    }
    memcpy(out, A + ts[g->h.output].offset, ts[g->h.output].bytes);
    return 0;
}

/* Structural checks only (the reference loader's full validation is pinned separately):
 * enough to keep the checker in bounds on the plans the tests feed it. */
static int o_open(OGraph *g, const void *plan, uint32_t len) {
    if (!plan || len < sizeof(OHeader)) return 10;
    memcpy(&g->h, plan, sizeof(OHeader));
    const OHeader *h = &g->h;
    if (h->magic != O_MAGIC || h->version < 1 || h->version > 3 || !h->nt || !h->no || h->input >= h->nt ||
        h->output >= h->nt || !h->arena_bytes)
        return 11;
    uint64_t meta = sizeof(OHeader) + (uint64_t)h->nt * sizeof(OTensor) + (uint64_t)h->no * sizeof(OOp);
    if ((uint64_t)len != meta + h->arena_bytes) return 12;
    g->ts = (const OTensor *)((const unsigned char *)plan + sizeof(OHeader));
    g->ops = (const OOp *)((const unsigned char *)plan + sizeof(OHeader) + h->nt * sizeof(OTensor));
    for (uint32_t i = 0; i < h->nt; i++)
        if ((uint64_t)g->ts[i].offset + g->ts[i].bytes > h->arena_bytes) return 13;
    for (uint32_t i = 0; i < h->no; i++)
        if (g->ops[i].a >= h->nt || g->ops[i].b >= h->nt || g->ops[i].out >= h->nt) return 15;
    g->arena = (unsigned char *)malloc(h->arena_bytes);
    if (!g->arena) return 1002;
    memcpy(g->arena, (const unsigned char *)plan + meta, h->arena_bytes);
    return 0;
}

uint32_t uqo_input_bytes(const void *plan, uint32_t len) {
    OGraph g;
    if (o_open(&g, plan, len)) return 0;
    uint32_t n = g.ts[g.h.input].bytes;
    free(g.arena);
    return n;
}

uint32_t uqo_output_bytes(const void *plan, uint32_t len) {
    OGraph g;
    if (o_open(&g, plan, len)) return 0;
    uint32_t n = g.ts[g.h.output].bytes;
    free(g.arena);
    return n;
}

int uqo_run(const void *plan, uint32_t len, const void *input, void *output, uint32_t images) {
    OGraph g;
    int rc = o_open(&g, plan, len);
    if (rc) return rc;
    size_t ni = g.ts[g.h.input].bytes, no = g.ts[g.h.output].bytes;
    for (uint32_t i = 0; i < images && !rc; i++)
        rc = o_run_image(&g, (const unsigned char *)input + i * ni, (unsigned char *)output + i * no);
    free(g.arena);
    return rc;
}

/* Exposed for unit tests of the requantisation contract. */
int32_t uqo_scale(int32_t v, int32_t m, int shift) { return o_scale(v, m, shift); }
