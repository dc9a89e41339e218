// common.cuh -- device helpers shared by every kernel of libunoq_cuda.
#pragma once
#include <cuda_runtime.h>
#include <cstdint>
#include <cstdlib>

namespace uq {

// Programmatic dependent launch. A kernel started by launch_pdl may begin while the kernel before
// it in the stream is still running: its CTAs take the SMs that the earlier grid's CTAs leave and
// run their prologue (barriers, per-channel constants, weights, TMEM) under the earlier grid's
// tail. Every thread that reads or writes activations first executes grid_dep_wait(), which
// returns once the earlier grid has completed and its writes are visible; nothing before it may
// touch memory that another kernel writes or reads. grid_dep_launch() allows the next kernel's
// CTAs to be scheduled once every CTA of this grid has issued it or exited.
__device__ __forceinline__ void grid_dep_wait() { asm volatile("griddepcontrol.wait;" ::: "memory"); }
__device__ __forceinline__ void grid_dep_launch() { asm volatile("griddepcontrol.launch_dependents;" ::: "memory"); }

// Kernel families that take programmatic launches: the tensor-core convolutions, whose
// prologue (barriers, constants, weights, TMEM) then overlaps the previous kernel's tail (5% faster
// steps at 512 images per GPU, 1% at 4,096). The depthwise kernel is launched in full stream order
// (early depthwise blocks measured 1-3% slower), but it still lets the next convolution start once
// all its blocks are running. UNOQ_PDL=<bits> overrides the set (a tuning and diagnosis switch;
// results are the same either way).
enum PdlKind { kPdlConvTc = 1, kPdlConvRows = 2, kPdlConvTaps = 4, kPdlDw = 8, kPdlDwTc = 16 };
inline bool pdl_enabled(int kind) {
    static const int mask = [] {
        const char *e = std::getenv("UNOQ_PDL");
        return e ? std::atoi(e) : (kPdlConvTc | kPdlConvRows | kPdlConvTaps | kPdlDwTc);
    }();
    return (mask & kind) != 0;
}

// <<<grid, block, smem, stream>>> with the programmatic-serialization attribute: only for kernels
// that call grid_dep_wait() before their first access to activations.
template <typename... KArgs, typename... Args>
inline cudaError_t launch_pdl(int kind, void (*kernel)(KArgs...), dim3 grid, dim3 block, size_t smem,
                              cudaStream_t s, const Args &...args) {
    cudaLaunchConfig_t cfg = {};
    cfg.gridDim = grid;
    cfg.blockDim = block;
    cfg.dynamicSmemBytes = smem;
    cfg.stream = s;
    cudaLaunchAttribute attr[1];
    attr[0].id = cudaLaunchAttributeProgrammaticStreamSerialization;
    attr[0].val.programmaticStreamSerializationAllowed = pdl_enabled(kind) ? 1 : 0;
    cfg.attrs = attr;
    cfg.numAttrs = 1;
    return cudaLaunchKernelEx(&cfg, kernel, args...);
}

// TFLite double-rounding requantisation, bit-exact with the reference (runtime/qnn.c:61-83):
// optional pre-multiply left shift; rounding-doubling high multiply (v*m + 2^30) >> 31 on the
// full 64-bit product; ties-away-from-zero rounding right shift for negative exponents.
__device__ __forceinline__ int32_t dev_scale(int32_t v, int32_t m, int shift) {
    if (shift > 0) v = (int32_t)((uint32_t)v << shift);
    int64_t p = (int64_t)v * (int64_t)m;
    int32_t h = (int32_t)((p + (1ll << 30)) >> 31);
    if (shift >= 0) return h;
    unsigned s = (unsigned)(-shift);
    uint32_t mask = (1u << s) - 1u;
    int32_t base = h >> s;
    uint32_t rem = (uint32_t)h & mask;
    return base + (int32_t)(rem > ((mask >> 1) + (h < 0 ? 1u : 0u)));
}

// Exact n / d for 0 <= n < 2^31 and 1 <= d < 2^31 with one 64-bit multiply and a shift, the
// invariant-divisor method of Granlund and Montgomery ("Division by invariant integers using
// multiplication", PLDI 1994): with p = ceil(log2 d) and m = ceil(2^(31+p) / d), m*d lies in
// [2^(31+p), 2^(31+p) + 2^p], hence floor(n / d) = floor(n*m / 2^(31+p)) for every n < 2^31, and
// n*m < 2^64 because m <= 2^32 + 1. Replaces the ~20-instruction dependent sequence of a run-time
// integer division in per-pixel index arithmetic.
struct FastDiv {
    unsigned long long m = 1ull << 31;
    int s = 31;
    int d = 1;
    FastDiv() = default;
    explicit FastDiv(int divisor) : d(divisor) {
        int p = 0;
        while ((1ll << p) < divisor) p++;
        m = ((1ull << (31 + p)) + (unsigned long long)divisor - 1) / (unsigned long long)divisor;
        s = 31 + p;
    }
    __host__ __device__ __forceinline__ int div(int n) const {
        return (int)(((unsigned long long)(unsigned)n * m) >> s);
    }
};

__device__ __forceinline__ int32_t dev_clamp(int32_t v, int32_t lo, int32_t hi) {
    return v < lo ? lo : (v > hi ? hi : v);
}

// Per-output-channel requantisation block prepared at load time from a plan's q tensor
// (qnn.c:12-16): y = post[clamp(scale(acc + bias[c], mult[c], shift[c]) + yzp, lo, hi)].
struct Requant {
    const int32_t *bias;   // corrected bias (plus any load-time folded terms), wraps mod 2^32
    const int32_t *mult;   // Q31 multiplier
    const int32_t *shift;  // exponent in [-31, 15]
    const uint8_t *post;   // optional 256-entry table indexed by y + 128, or nullptr
    int32_t yzp, lo, hi;
};

__device__ __forceinline__ int8_t requant_one(int32_t acc, int c, const Requant &r) {
    int32_t v = (int32_t)((uint32_t)acc + (uint32_t)__ldg(r.bias + c));
    v = dev_scale(v, __ldg(r.mult + c), __ldg(r.shift + c)) + r.yzp;
    v = dev_clamp(v, r.lo, r.hi);
    if (r.post) v = (int8_t)__ldg(r.post + v + 128);
    return (int8_t)v;
}

inline unsigned ceil_div(uint64_t a, uint64_t b) { return (unsigned)((a + b - 1) / b); }

// Grid size for a grid-stride loop over `n` items of `per_block` each, capped to keep
// every SM of a B200 (148) busy without an excessive tail.
inline unsigned grid_for(uint64_t n, unsigned per_block, unsigned cap = 148u * 32u) {
    uint64_t g = (n + per_block - 1) / per_block;
    if (g < 1) g = 1;
    if (g > cap) g = cap;
    return (unsigned)g;
}

}  // namespace uq
