// tc_common.cuh -- building blocks of the tcgen05 convolution kernels (conv_tc.cu, conv_rows.cu):
// mbarrier waits bounded in time, UMMA shared-memory / instruction descriptors and MMA issue,
// TMEM loads, the exact requantisation epilogue of 16 accumulator columns, and the driver's
// tensor-map encoder. Everything has internal linkage, the device error flag included, so each
// kernel file keeps its own flag and reads it through its own host accessor.
#pragma once
#include <cuda.h>
#include <cuda_runtime.h>

#include <cstdint>

#include "common.cuh"
#include "requant.cuh"

namespace uq {
namespace {

// Site code of the first device wait that ran out of time in this file's kernels (0 = none).
__device__ int g_tc_error = 0;

constexpr int kBM = 128;              // pixels per tile = TMEM lanes
constexpr int kBK = 128;              // reduction bytes per stage (one 128-byte swizzle row)
constexpr int kStageBytes = kBM * kBK;

__device__ __forceinline__ uint32_t smem_u32(const void *p) {
    return static_cast<uint32_t>(__cvta_generic_to_shared(p));
}

__device__ __forceinline__ void mbar_init(uint32_t bar, uint32_t count) {
    asm volatile("mbarrier.init.shared::cta.b64 [%0], %1;" ::"r"(bar), "r"(count));
}

__device__ __forceinline__ void mbar_arrive(uint32_t bar) {
    asm volatile("{\n\t.reg .b64 st;\n\tmbarrier.arrive.shared::cta.b64 st, [%0];\n\t}" ::"r"(bar) : "memory");
}

// Test a phase; while it is incomplete the thread may be suspended for up to `hint_ns`, and it
// resumes as soon as the phase completes. Without a hint the hardware's default limit is short
// and waiting warps would spin, taking issue slots from the warps doing the work.
__device__ __forceinline__ bool mbar_try_wait(uint32_t bar, uint32_t parity, uint32_t hint_ns = 0) {
    uint32_t ok;
    asm volatile(
        "{\n\t.reg .pred p;\n\t"
        "mbarrier.try_wait.parity.shared::cta.b64 p, [%1], %2, %3;\n\t"
        "selp.u32 %0, 1, 0, p;\n\t}"
        : "=r"(ok)
        : "r"(bar), "r"(parity), "r"(hint_ns)
        : "memory");
    return ok != 0;
}

// Wait bound: 4e9 SM cycles (about 2 s at the B200's 1.9-2 GHz boost clock).
constexpr long long kTimeoutCycles = 4000000000ll;

// Bounded wait: returns false (and records `code`) if the phase does not complete in time or
// another role of this CTA already gave up.
__device__ __forceinline__ bool mbar_wait(uint32_t bar, uint32_t parity, volatile int *abort, int code) {
    constexpr uint32_t kHintNs = 200000;  // one suspension of at most 0.2 ms per poll
    if (mbar_try_wait(bar, parity, kHintNs)) return true;
    const long long start = clock64();
    while (true) {
        if (mbar_try_wait(bar, parity, kHintNs)) return true;
        if (*abort) return false;
        if (clock64() - start > kTimeoutCycles) {
            *abort = 1;
            atomicCAS(&g_tc_error, 0, code);
            return false;
        }
    }
}

// A barrier among the warps of one role, built on an mbarrier so that it is bounded: each warp
// arrives once per round (lane 0, after the warp has converged) and every lane waits for the
// round's phase. One arrival per warp keeps the shared-memory atomics on the barrier word few.
__device__ __forceinline__ bool role_sync(uint32_t bar, unsigned &round, volatile int *abort, int code) {
    __syncwarp();
    if ((threadIdx.x & 31) == 0) mbar_arrive(bar);
    const bool ok = mbar_wait(bar, round & 1u, abort, code);
    round++;
    return ok;
}

__device__ __forceinline__ void cp_async16(uint32_t dst, const void *src) {
    asm volatile("cp.async.cg.shared.global [%0], [%1], 16;" ::"r"(dst), "l"(src) : "memory");
}
__device__ __forceinline__ void cp_async_commit() { asm volatile("cp.async.commit_group;" ::: "memory"); }
template <int N>
__device__ __forceinline__ void cp_async_wait() {
    asm volatile("cp.async.wait_group %0;" ::"n"(N) : "memory");
}
// cp.async.wait_group with a run-time depth (the instruction takes an immediate).
__device__ __forceinline__ void cp_async_wait_dyn(int n) {
    switch (n) {
        case 0: cp_async_wait<0>(); break;
        case 1: cp_async_wait<1>(); break;
        case 2: cp_async_wait<2>(); break;
        default: cp_async_wait<3>(); break;
    }
}
__device__ __forceinline__ void fence_proxy_async() {
    asm volatile("fence.proxy.async.shared::cta;" ::: "memory");
}
__device__ __forceinline__ void st_shared16(uint32_t dst, uint4 v) {
    asm volatile("st.shared.v4.b32 [%0], {%1, %2, %3, %4};" ::"r"(dst), "r"(v.x), "r"(v.y), "r"(v.z), "r"(v.w)
                 : "memory");
}

__device__ __forceinline__ uint4 ld_shared16(uint32_t src) {
    uint4 v;
    asm volatile("ld.shared.v4.b32 {%0, %1, %2, %3}, [%4];" : "=r"(v.x), "=r"(v.y), "=r"(v.z), "=r"(v.w) : "r"(src));
    return v;
}
// Four bytes at any shared-memory address: two aligned words joined by a funnel shift.
__device__ __forceinline__ uint32_t ld_shared_u32_unaligned(uint32_t addr) {
    const uint32_t base = addr & ~3u;
    uint32_t lo, hi;
    asm volatile("ld.shared.b32 %0, [%1];" : "=r"(lo) : "r"(base));
    asm volatile("ld.shared.b32 %0, [%1];" : "=r"(hi) : "r"(base + 4));
    return __funnelshift_r(lo, hi, (addr & 3u) * 8);
}

// UMMA shared-memory descriptor: K-major, SWIZZLE_128B, 8-row atoms 1024 bytes apart.
__device__ __forceinline__ uint64_t smem_desc(uint32_t addr) {
    return (uint64_t)((addr >> 4) & 0x3FFF) | (1ull << 16) | (64ull << 32) | (1ull << 46) | (2ull << 61);
}

// Instruction descriptor for kind::i8: s32 accumulate, signed A and B, both K-major.
__device__ __forceinline__ uint32_t instr_desc(int bn) {
    return (2u << 4) | (1u << 7) | (1u << 10) | ((uint32_t)(bn >> 3) << 17) | ((uint32_t)(kBM >> 4) << 24);
}

__device__ __forceinline__ void mma_i8(uint32_t tmem_d, uint64_t adesc, uint64_t bdesc, uint32_t idesc, uint32_t acc) {
    asm volatile(
        "{\n\t.reg .pred p;\n\t"
        "setp.ne.b32 p, %4, 0;\n\t"
        "tcgen05.mma.cta_group::1.kind::i8 [%0], %1, %2, %3, p;\n\t}" ::"r"(tmem_d),
        "l"(adesc), "l"(bdesc), "r"(idesc), "r"(acc));
}

__device__ __forceinline__ void mma_commit(uint32_t bar) {
    asm volatile("tcgen05.commit.cta_group::1.mbarrier::arrive::one.shared::cluster.b64 [%0];" ::"r"(bar) : "memory");
}

__device__ __forceinline__ void tc_fence_before() { asm volatile("tcgen05.fence::before_thread_sync;" ::: "memory"); }
__device__ __forceinline__ void tc_fence_after() { asm volatile("tcgen05.fence::after_thread_sync;" ::: "memory"); }

__device__ __forceinline__ void tmem_ld16_nowait(uint32_t taddr, uint32_t (&r)[16]) {
    asm volatile(
        "tcgen05.ld.sync.aligned.32x32b.x16.b32 {%0,%1,%2,%3,%4,%5,%6,%7,%8,%9,%10,%11,%12,%13,%14,%15}, [%16];"
        : "=r"(r[0]), "=r"(r[1]), "=r"(r[2]), "=r"(r[3]), "=r"(r[4]), "=r"(r[5]), "=r"(r[6]), "=r"(r[7]), "=r"(r[8]),
          "=r"(r[9]), "=r"(r[10]), "=r"(r[11]), "=r"(r[12]), "=r"(r[13]), "=r"(r[14]), "=r"(r[15])
        : "r"(taddr));
}

// Wait for this thread's outstanding tcgen05.ld; the registers are tied in as read-write
// operands so no use of them can be scheduled before the wait.
__device__ __forceinline__ void tmem_wait_ld(uint32_t (&r)[16]) {
    asm volatile("tcgen05.wait::ld.sync.aligned;"
                 : "+r"(r[0]), "+r"(r[1]), "+r"(r[2]), "+r"(r[3]), "+r"(r[4]), "+r"(r[5]), "+r"(r[6]), "+r"(r[7]),
                   "+r"(r[8]), "+r"(r[9]), "+r"(r[10]), "+r"(r[11]), "+r"(r[12]), "+r"(r[13]), "+r"(r[14]), "+r"(r[15])
                 :
                 : "memory");
}


// Epilogue requantisation modes, chosen per layer on the host (all exact, see make_epilogue):
//   kRelu    every channel is in the short form (epi_fast: a negative shift with yzp folded into
//            k, or a dead channel, m == 0) and the clamp floor lo >= yzp, so the tie
//            correction for negative high products can never survive the clamp:
//            y = clamp((hi32(acc*m + k)) >> (sh - 32));
//   kTies    same shifts, lo < yzp: subtract 2^31 first when acc <= cut;
//   kGeneral any live channel with a pre-shift (shift >= 0), or whose k could not take yzp: full form.
enum EpiMode { kRelu = 0, kTies = 1, kGeneral = 2 };

// Per-channel constants in shared memory as structure-of-arrays so 16 columns load as
// 128-bit broadcast vectors.
struct EpiSoA {
    const long long *k;
    const int *m, *cut, *sh, *ls, *bs, *zadd;
};

// Saturating pack of four int32 values into int8 lanes (byte i = v_i): two cvt.pack.sat, each
// putting sat(a) in byte 1 and sat(b) in byte 0 above c's low half shifted up by 16.
__device__ __forceinline__ uint32_t pack_sat_s8x4(int32_t v0, int32_t v1, int32_t v2, int32_t v3) {
    uint32_t hi, d;
    asm("cvt.pack.sat.s8.s32.b32 %0, %1, %2, %3;" : "=r"(hi) : "r"(v3), "r"(v2), "r"(0));
    asm("cvt.pack.sat.s8.s32.b32 %0, %1, %2, %3;" : "=r"(d) : "r"(v1), "r"(v0), "r"(hi));
    return d;
}

// A residual add (qnn.c:175-183) applied in the epilogue: the add's scale as requant.cuh constants
// (bias 0) and its clamp.
struct AddEpi {
    EpiChan epi;
    int lo, hi;
};

// Requantise accumulators r[4g..4g+3] (columns c0+4g.. of one row) and pack them as int8: exact
// scale, clamp to [lo, hi], then the post table (LUT 1: always, 2: when `lut` is set) and the
// residual add (ADD). HI = false leaves the upper clamp to the saturating pack (hi == 127 without
// a lookup after it), and LO = false the lower one (lo == -128, the same condition).
template <int EPI, int LUT, bool ADD, bool HI, bool LO>
__device__ __forceinline__ uint32_t epilogue_group(const uint32_t (&r)[16], int g, const EpiSoA &E, const uint8_t *lut,
                                                   int c0, int lo, int hi, const AddEpi *fp, const int32_t *tabs,
                                                   uint32_t resw) {
    const int4 mv = reinterpret_cast<const int4 *>(E.m + c0)[g], sv = reinterpret_cast<const int4 *>(E.sh + c0)[g];
    const longlong2 ka = reinterpret_cast<const longlong2 *>(E.k + c0)[2 * g];
    const longlong2 kb = reinterpret_cast<const longlong2 *>(E.k + c0)[2 * g + 1];
    int4 cv = make_int4(0, 0, 0, 0), lv = cv, bv = cv, zv = cv;
    if (EPI >= kTies) cv = reinterpret_cast<const int4 *>(E.cut + c0)[g];
    if (EPI == kGeneral) {
        lv = reinterpret_cast<const int4 *>(E.ls + c0)[g];
        bv = reinterpret_cast<const int4 *>(E.bs + c0)[g];
        zv = reinterpret_cast<const int4 *>(E.zadd + c0)[g];
    }
    const int mm[4] = {mv.x, mv.y, mv.z, mv.w}, ss[4] = {sv.x, sv.y, sv.z, sv.w};
    const int cc[4] = {cv.x, cv.y, cv.z, cv.w}, ll[4] = {lv.x, lv.y, lv.z, lv.w};
    const int bb[4] = {bv.x, bv.y, bv.z, bv.w}, zz[4] = {zv.x, zv.y, zv.z, zv.w};
    const long long kk[4] = {ka.x, ka.y, kb.x, kb.y};
    int32_t v[4];
#pragma unroll
    for (int i = 0; i < 4; i++) {
        const int32_t acc = (int32_t)r[g * 4 + i];
        if (EPI == kGeneral) {
            const int32_t a = (int32_t)(((uint32_t)acc << ll[i]) + (uint32_t)bb[i]);
            long long p = (long long)a * mm[i] + kk[i];
            p -= (long long)(acc <= cc[i]) << 31;
            v[i] = (int32_t)(p >> ss[i]) + zz[i];
        } else {
            long long p = (long long)acc * mm[i] + kk[i];
            if (EPI == kTies) p -= (long long)(acc <= cc[i]) << 31;
            v[i] = ((int32_t)(p >> 32)) >> ss[i];
        }
        if (LO || LUT || ADD) v[i] = max(v[i], lo);
        if (HI || LUT || ADD) v[i] = min(v[i], hi);
        if (LUT == 1 || (LUT == 2 && lut)) v[i] = (int8_t)lut[v[i] + 128];
        if (ADD) {  // fused residual add: the add's two tables, then its scale and clamp
            const int rv = (int)(int8_t)(resw >> (8 * i));
            const int32_t sum = (int32_t)((uint32_t)tabs[v[i] + 128] + (uint32_t)tabs[256 + rv + 128]);
            v[i] = epilogue_one(sum, fp->epi, fp->lo, fp->hi);
        }
    }
    return pack_sat_s8x4(v[0], v[1], v[2], v[3]);
}

// Requantise 16 accumulators (columns c0..c0+15 of one row) and pack them as int8. With `fp`, the
// residual add follows: y = clamp(scale(tabs[v + 128] + tabs[256 + r + 128])) with r the residual
// bytes in `res`. The layer's variant (table, add, upper clamp) is chosen once per chunk -- the
// conditions are launch parameters, uniform over the kernel -- so each value runs only the steps
// its layer needs.
template <int EPI>
__device__ __forceinline__ uint4 epilogue_chunk(const uint32_t (&r)[16], const EpiSoA &E, const uint8_t *lut, int c0,
                                                int lo, int hi, const AddEpi *fp = nullptr, const int32_t *tabs = nullptr,
                                                uint4 res = make_uint4(0, 0, 0, 0)) {
    const uint32_t resw[4] = {res.x, res.y, res.z, res.w};
    uint32_t o[4];
#define UQ_EPI_GROUPS(L, A, H, W)                                                                    \
    _Pragma("unroll") for (int g = 0; g < 4; g++) o[g] =                                             \
        epilogue_group<EPI, L, A, H, W>(r, g, E, lut, c0, lo, hi, fp, tabs, resw[g])
    if (fp) {
        UQ_EPI_GROUPS(2, true, true, true);
    } else if (lut) {
        UQ_EPI_GROUPS(1, false, true, true);
    } else if (hi < 127) {
        if (lo > -128) UQ_EPI_GROUPS(0, false, true, true);
        else UQ_EPI_GROUPS(0, false, true, false);
    } else if (lo > -128) {
        UQ_EPI_GROUPS(0, false, false, true);
    } else {
        UQ_EPI_GROUPS(0, false, false, false);
    }
#undef UQ_EPI_GROUPS
    return make_uint4(o[0], o[1], o[2], o[3]);
}

using EncodeTiled = CUresult (*)(CUtensorMap *, CUtensorMapDataType, cuuint32_t, void *, const cuuint64_t *,
                                 const cuuint64_t *, const cuuint32_t *, const cuuint32_t *, CUtensorMapInterleave,
                                 CUtensorMapSwizzle, CUtensorMapL2promotion, CUtensorMapFloatOOBfill);

static EncodeTiled encoder() {
    static EncodeTiled fn = nullptr;
    if (!fn) {
        void *ptr = nullptr;
        cudaDriverEntryPointQueryResult q;
        if (cudaGetDriverEntryPoint("cuTensorMapEncodeTiled", &ptr, cudaEnableDefault, &q) == cudaSuccess &&
            q == cudaDriverEntryPointSuccess)
            fn = reinterpret_cast<EncodeTiled>(ptr);
    }
    return fn;
}

}  // namespace
}  // namespace uq
