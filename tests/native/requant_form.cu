// Host-side check of the product's requantisation form (unoq-dsp_b200/csrc/requant.cuh) against
// the oracle's restatement of the reference `scale` (oracle/uq_oracle.c, runtime/qnn.c:61-83).
// Built and run by tests/test_requant_form.py; prints "cases N mismatches M".
#include <cstdint>
#include <cstdio>

#include "requant.cuh"

extern "C" int32_t uqo_scale(int32_t v, int32_t m, int shift);

static uint64_t state = 0x9E3779B97F4A7C15ull;
static uint64_t next() {  // splitmix64
    uint64_t z = (state += 0x9E3779B97F4A7C15ull);
    z = (z ^ (z >> 30)) * 0xBF58476D1CE4E5B9ull;
    z = (z ^ (z >> 27)) * 0x94D049BB133111EBull;
    return z ^ (z >> 31);
}
static int64_t pick(int64_t lo, int64_t hi) { return lo + (int64_t)(next() % (uint64_t)(hi - lo + 1)); }

int main() {
    long long cases = 0, bad = 0, bad_fast = 0, fast_cases = 0;
    const int32_t special_m[] = {0, 1, 2, 3, 1 << 30, (1 << 30) + 1, 0x7FFFFFFF, 0x40000000 - 1, 12345678};
    for (int trial = 0; trial < 40000; trial++) {
        const int shift = (int)pick(-31, 15);
        const int32_t m = trial % 7 == 0 ? special_m[trial / 7 % 9] : (int32_t)pick(0, 0x7FFFFFFF);
        const int64_t bias = trial % 3 == 0 ? pick(-(1 << 12), 1 << 12) : pick(-(1ll << 30), 1ll << 30);
        const int yzp = (int)pick(-128, 127);
        int lo = (int)pick(-128, 127), hi = (int)pick(-128, 127);
        if (lo > hi) { int t = lo; lo = hi; hi = t; }
        const uq::EpiChan e = uq::make_epilogue(bias, m, shift, yzp);
        // accumulators: random, near the tie / cut boundaries, and at the MMA bound
        for (int k = 0; k < 64; k++) {
            int32_t acc;
            if (k < 24) acc = (int32_t)pick(-(1 << 27), 1 << 27);
            else if (k < 40) acc = (int32_t)pick(-4096, 4096);
            else if (k < 56 && e.cut != INT32_MIN) acc = e.cut + (int32_t)pick(-3, 3);
            else acc = (int32_t)pick(-(1 << 20), 1 << 20);
            const int32_t v = (int32_t)((int64_t)acc + bias);
            int32_t want = uqo_scale(v, m, shift) + yzp;
            want = want < lo ? lo : (want > hi ? hi : want);
            const int32_t got = uq::epilogue_one(acc, e, lo, hi);
            cases++;
            if (got != want) {
                if (bad < 5) printf("mismatch acc=%d bias=%lld m=%d s=%d yzp=%d: %d vs %d\n", acc, (long long)bias, m,
                                    shift, yzp, got, want);
                bad++;
            }
            // short forms (epi_fast): kTies keeps the tie correction; kRelu drops it when lo >= yzp
            if (uq::epi_fast(e)) {
                fast_cases++;
                const long long p = (long long)acc * e.m + e.k;
                int32_t ties = ((int32_t)((p - ((long long)(acc <= e.cut) << 31)) >> 32)) >> (e.sh - 32);
                ties = ties < lo ? lo : (ties > hi ? hi : ties);
                int32_t fast = ((int32_t)(p >> 32)) >> (e.sh - 32);
                fast = fast < lo ? lo : (fast > hi ? hi : fast);
                if (ties != want || (lo >= yzp && fast != want)) bad_fast++;
            }
        }
    }
    printf("cases %lld fast_cases %lld mismatches %lld fast_mismatches %lld\n", cases, fast_cases, bad, bad_fast);
    // every shift in [-31, -1] and every dead channel must reach the short form at these biases
    return bad || bad_fast || fast_cases < cases / 2 ? 1 : 0;
}
