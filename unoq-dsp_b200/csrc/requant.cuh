// requant.cuh -- exact per-channel requantisation constants shared by the conv and depthwise
// kernels (host preparation + device evaluation).
#pragma once
#include <climits>
#include <cstdint>

namespace uq {

// Per-output-channel epilogue constants (32 bytes): one branch-free form covers every
// channel (see make_epilogue):  a = (acc << ls) + bs;  p = a*m + k;  p -= 2^31 if acc <= cut;
// y = (int32)(p >> sh) + zadd.
struct __align__(32) EpiChan {
    long long k;
    int m, cut, ls, bs, sh, zadd;
};

__host__ __device__ __forceinline__ int32_t epilogue_one(int32_t acc, const EpiChan &e, int lo, int hi) {
    const int32_t a = (int32_t)(((uint32_t)acc << e.ls) + (uint32_t)e.bs);
    long long p = (long long)a * e.m + e.k;
    p -= (long long)(acc <= e.cut) << 31;
    const int32_t v = (int32_t)(p >> e.sh) + e.zadd;
    return v < lo ? lo : (v > hi ? hi : v);
}


// Exact requantisation constants, one branch-free form for every channel. The reference
// computes y = clamp(scale(v, m, s) + yzp) with v = acc + bias (qnn.c:61-83):
//   s >= 0:  y = floor(((v<<s) * m + 2^30) / 2^31) + yzp       -> ls = s, bs = bias<<s, k = 2^30 + yzp*2^31
//   s = -n:  y = floor((v*m + 2^30 + 2^(30+n) - [v*m < -2^30]*2^31) / 2^(31+n)) + yzp
//            (nested floor divisions with integer addends collapse into one; the bracket turns
//            the ties-up of a negative high product into the reference's ties-away). With
//            v = acc + bias this is affine in acc plus one comparison: acc <= cut, where
//            cut = floor((-2^30 - 1) / m) - bias. yzp*2^(31+n) folds into k while
//            |k| <= 2^63 - 2^59, so that acc*m + k (|acc*m| < 2^58) stays inside int64;
//            beyond that it is added after the shift (zadd).
//   m == 0:  both forms give y = yzp, whatever the shift; such a channel takes the s = -1 form,
//            so that a layer's dead channels do not force the full form on its live ones.
// The accumulator of the MMA is bounded by 8192*128*127 < 2^27, so cut = INT32_MIN means never.
inline EpiChan make_epilogue(long long bias, int m, int shift, int yzp) {
    EpiChan e{};
    e.m = m;
    e.cut = INT32_MIN;
    if (m == 0 && shift >= 0) shift = -1;
    if (shift >= 0) {
        e.ls = shift;
        e.bs = (int)((uint32_t)(uint64_t)bias << shift);
        e.k = (1ll << 30) + (long long)yzp * (1ll << 31);
        e.sh = 31;
    } else {
        // m == 0 needs no special case: p = k and floor(k / 2^(31+n)) = yzp.
        const int n = -shift;
        e.k = bias * (long long)m + (1ll << 30) + (1ll << (30 + n));
        const __int128 kz = (__int128)e.k + (__int128)yzp * ((__int128)1 << (31 + n));
        const __int128 lim = ((__int128)1 << 63) - ((__int128)1 << 59);
        if (kz >= -lim && kz <= lim) e.k = (long long)kz;
        else e.zadd = yzp;
        if (m > 0) {
            const long long num = -(1ll << 30) - 1;
            long long fl = num / m;
            if (fl * m > num) fl -= 1;
            const long long cut = fl - bias;
            e.cut = (int)(cut < INT32_MIN ? INT32_MIN : (cut > INT32_MAX ? INT32_MAX : cut));
        }
        e.sh = 31 + n;
    }
    return e;
}

// True when the channel's constants are in the short form that the fast epilogue modes evaluate:
// y = (acc*m + k) >> sh with sh >= 32, no pre-shift and nothing added after the shift.
inline bool epi_fast(const EpiChan &e) { return e.sh >= 32 && e.ls == 0 && e.bs == 0 && e.zadd == 0; }

}  // namespace uq
