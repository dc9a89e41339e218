// plan.cpp -- loader validation with the reference's error codes.
//
// Each check below restates a condition of runtime/graph.c ug_load (lines 50-216) or
// runtime/qnn.c uq_validate (lines 209-252); the comments give the line each block follows.
// Beyond validation, the pass records per-tensor birth/death op indices, which the device
// memory planner reuses for batched arenas.
#include "plan.hpp"

#include <climits>
#include <cstring>

namespace uq {

int32_t host_scale(int32_t v, int32_t m, int shift) {
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

namespace {

bool same_shape(const Tensor &a, const Tensor &b) {  // graph.c:32
    if (a.type != b.type || a.rank != b.rank) return false;
    for (uint32_t i = 0; i < a.rank; i++)
        if (a.d[i] != b.d[i]) return false;
    return true;
}

bool broadcastable(const Tensor &a, const Tensor &b) {  // graph.c:33-40
    if (a.type != b.type || b.rank > a.rank) return false;
    for (uint32_t i = 0; i < b.rank; i++)
        if (b.d[i] != 1 && b.d[i] != a.d[a.rank - b.rank + i]) return false;
    if (b.bytes == type_width(b.type)) return true;
    if (b.bytes == a.d[a.rank - 1] * type_width(b.type)) {
        for (uint32_t i = 0; i + 1 < b.rank; i++)
            if (b.d[i] != 1) return false;
        return true;
    }
    return same_shape(a, b);
}


}  // namespace

// qnn.c:209-252: vision op parameter block (codes 14-17).
int validate_vision(const Op &o, const Tensor &a, const Tensor &b, const Tensor &z, const Tensor &t,
                    const int32_t *q, const int8_t *w, uint64_t &work) {
    if (a.type != 3 || z.type != 3 || !t.flags || t.type != 4 || t.bytes < kHead * 4 ||
        ((o.code != 14 && o.code != 15) && o.p[1]) || o.p[2] || o.p[3])
        return 18;
    if (q[12] < -128 || q[12] > 127 || q[13] < -128 || q[13] > 127 || q[14] < -128 || q[15] > 127 || q[14] > q[15] ||
        q[19] < 0 || q[19] > 1)
        return 18;
    if (o.code == 17) {  // qnn.c:213-219
        if (q[13] != -128 || q[14] != -128 || q[15] != 127 || a.rank != z.rank || a.bytes != z.bytes || !a.rank ||
            q[16] != (int32_t)a.d[a.rank - 1] || q[16] < 1 || q[16] > kMaxC || t.bytes != (uint32_t)(kHead + 256) * 4)
            return 18;
        for (int i = 0; i < 256; i++)
            if (q[kHead + i] < 0 || q[kHead + i] > (1 << 24)) return 18;
        for (uint32_t d = 0; d < a.rank; d++)
            if (a.d[d] != z.d[d]) return 18;
        if (q[kHead] != (1 << 24)) return 18;
        work += a.bytes;
        return 0;
    }
    if (a.rank != 4 || z.rank != 4 || a.d[0] != z.d[0] || q[16] != (int32_t)a.d[3] || q[17] != (int32_t)z.d[3] ||
        q[16] < 1 || q[16] > kMaxC || q[17] < 1 || q[17] > kMaxC)
        return 18;
    for (int i = 0; i < 6; i++)
        if (q[i] < 1 || q[i] > 4096) return 18;
    for (int i = 6; i < 12; i++)
        if (q[i] < 0 || q[i] > 4096) return 18;
    int64_t hh = (int64_t)a.d[1] + q[6] + q[8] - (int64_t)(q[0] - 1) * q[4] - 1;
    int64_t ww = (int64_t)a.d[2] + q[7] + q[9] - (int64_t)(q[1] - 1) * q[5] - 1;
    if (hh < 0 || ww < 0 || hh / q[2] + 1 != q[10] || ww / q[3] + 1 != q[11] || q[10] != (int32_t)z.d[1] ||
        q[11] != (int32_t)z.d[2])
        return 18;
    uint64_t area = (uint64_t)q[0] * q[1], rows = (uint64_t)z.d[0] * z.d[1] * z.d[2];
    if (o.code == 16) {  // qnn.c:227-232
        if (q[16] != q[17] || q[12] != q[13] || q[4] != 1 || q[5] != 1 || area > 8192 || t.bytes != kHead * 4) return 18;
        if (q[6] >= q[0] || q[7] >= q[1] || (q[10] - 1) * (int64_t)q[2] - q[6] >= a.d[1] ||
            (q[11] - 1) * (int64_t)q[3] - q[7] >= a.d[2])
            return 18;
        work += rows * area * q[16];
        return 0;
    }
    uint64_t k = area * (o.code == 15 ? 1 : q[16]);  // qnn.c:233-251
    if (k > (uint64_t)kMaxK || q[18] != (int32_t)((k + 7) & ~7ull) || !b.flags || b.type != 3 ||
        t.bytes != (uint32_t)(kHead + 3 * q[17]) * 4)
        return 18;
    if (o.code == 15) {
        if (q[16] != q[17] || b.bytes != area * q[17]) return 18;
    } else if (b.bytes != (uint32_t)((q[17] + 3) & ~3) * q[18])
        return 18;
    for (int c = 0; c < q[17]; c++) {
        int shift = q[kHead + 2 * q[17] + c];
        if (q[kHead + q[17] + c] < 0 || shift < -31 || shift > 15) return 18;
        int64_t lo = q[kHead + c], hi = lo;
        unsigned terms = o.code == 15 ? (unsigned)k : (unsigned)q[18];
        for (unsigned j = 0; j < terms; j++) {
            int v = o.code == 15 ? w[j * q[17] + c] : w[(c / 4) * terms * 4 + (j / 8) * 32 + (c % 4) * 8 + j % 8];
            if (v < 0) lo += 255 * v;
            else hi += 255 * v;
        }
        int64_t factor = 1LL << (shift > 0 ? shift : 0);
        if (lo * factor < INT32_MIN || hi * factor > INT32_MAX) return 18;
        int m = q[kHead + q[17] + c];
        if ((int64_t)host_scale((int32_t)lo, m, shift) + q[13] < INT32_MIN ||
            (int64_t)host_scale((int32_t)hi, m, shift) + q[13] > INT32_MAX)
            return 18;
    }
    work += rows * k * q[17];
    return 0;
}

int parse_plan(const void *blob, uint32_t len, Plan &out) {
    Plan P;
    Header &h = P.h;
    if (!blob || len < sizeof(Header)) return 10;  // graph.c:51
    std::memcpy(&h, blob, sizeof(Header));
    if (h.magic != kMagic || (h.version < 1 || h.version > 3) || !h.nt || h.nt > kMaxTensors || !h.no ||
        h.no > kMaxOps || !h.arena_bytes || h.arena_bytes > kArena || h.input >= h.nt || h.output >= h.nt ||
        (h.version == 1 ? h.reserved != 0 : h.reserved > 1))
        return 11;  // graph.c:52
    uint64_t meta = sizeof(Header) + (uint64_t)h.nt * sizeof(Tensor) + (uint64_t)h.no * sizeof(Op);
    if ((uint64_t)len != meta + h.arena_bytes) return 12;  // graph.c:54
    const uint8_t *p = static_cast<const uint8_t *>(blob);
    P.ts.resize(h.nt);
    P.ops.resize(h.no);
    std::memcpy(P.ts.data(), p + sizeof(Header), h.nt * sizeof(Tensor));
    std::memcpy(P.ops.data(), p + sizeof(Header) + h.nt * sizeof(Tensor), h.no * sizeof(Op));
    P.arena.assign(p + meta, p + meta + h.arena_bytes);
    std::vector<uint8_t> defined(h.nt, 0);
    P.birth.assign(h.nt, -1);
    P.death.assign(h.nt, -1);
    uint32_t end = 0;
    for (uint32_t i = 0; i < h.nt; i++) {  // graph.c:58-65
        Tensor &t = P.ts[i];
        uint32_t w = type_width(t.type);
        uint64_t count = 1;
        if (!w || t.rank > 4 || t.offset % 128 || (h.version < 3 && t.offset < end) || t.offset > h.arena_bytes ||
            t.flags > 1 || t.reserved[0] || t.reserved[1] || t.reserved[2])
            return 13;
        for (uint32_t d = 0; d < t.rank; d++) {
            if (!t.d[d] || t.d[d] > kArena) return 13;
            count *= t.d[d];
            if (count > kArena) return 13;
        }
        if (count * w != t.bytes || t.bytes > h.arena_bytes - t.offset) return 13;
        end = t.offset + t.bytes;
        defined[i] = (uint8_t)t.flags;
        P.birth[i] = -1;
        P.death[i] = t.flags ? (int)h.no : -1;
    }
    if (P.ts[h.input].flags) return 14;  // graph.c:66
    defined[h.input] = 1;
    uint64_t work = 0;
    bool vision_only = true, parallel_vision = false;
    auto Q = [&](uint32_t tensor) { return reinterpret_cast<const int32_t *>(P.arena.data() + P.ts[tensor].offset); };
    for (uint32_t i = 0; i < h.no; i++) {  // graph.c:69-201
        const Op &o = P.ops[i];
        if (o.code != 5 && o.code != 10 && (o.code < 14 || o.code > 28)) vision_only = false;
        if (o.a >= h.nt || o.b >= h.nt || o.out >= h.nt || !defined[o.a] || defined[o.out]) return 15;
        const Tensor &a = P.ts[o.a], &b = P.ts[o.b], &z = P.ts[o.out];
        if (o.code == 1 || o.code == 6 || o.code == 8 || o.code == 9) {  // graph.c:74-83
            bool integer = o.code == 6 || o.code == 9, packed = o.code == 8 || o.code == 9;
            if (packed && h.version < 2) return 16;
            if (!defined[o.b] || !b.flags || a.rank != 2 || b.rank != 2 || z.rank != 2 || a.d[1] != b.d[1] ||
                z.d[0] != a.d[0] || (packed ? ((z.d[1] + 3) / 4 * 4 != b.d[0]) : z.d[1] != b.d[0]))
                return 16;
            if (!integer && (a.type != 1 || b.type != 1 || z.type != 1)) return 16;
            if (integer && (a.type != 2 || b.type != 3 || z.type != 4 || a.d[1] > 8192 || o.p[0] > 255 ||
                            (int32_t)o.p[1] < -128 || (int32_t)o.p[1] > 127))
                return 16;
            if (integer && (o.p[3] != 1 || o.p[2] >= h.nt || !defined[o.p[2]] || !P.ts[o.p[2]].flags ||
                            P.ts[o.p[2]].type != 4 || P.ts[o.p[2]].bytes != z.d[1] * 4))
                return 16;
            if (o.code == 8 && (o.p[0] > 1 || o.p[1] || o.p[2] || o.p[3])) return 16;
            if (o.code == 9 && a.d[1] % 8) return 16;
            work += (uint64_t)a.d[0] * a.d[1] * z.d[1];
        } else if (o.code == 2 || o.code == 3) {  // graph.c:84-86
            if (!defined[o.b] || !same_shape(a, z) || !broadcastable(a, b) || (a.type != 1 && a.type != 4)) return 17;
            work += a.bytes / type_width(a.type);
        } else if (o.code == 4) {
            if (!same_shape(a, z) || (a.type != 1 && a.type != 4)) return 18;
            work += a.bytes / 4;
        } else if (o.code == 5) {
            if (a.type != z.type || a.bytes != z.bytes) return 18;
            work += a.bytes;
        } else if (o.code == 7) {
            if (a.type != 4 || z.type != 1 || a.bytes != z.bytes) return 18;
            work += a.bytes / 4;
        } else if (o.code == 10) {  // graph.c:90-95
            if (a.rank != z.rank || a.type != z.type || a.bytes != z.bytes) return 18;
            unsigned seen = 0;
            for (unsigned d = 0; d < a.rank; d++) {
                unsigned qd = o.p[d];
                if (qd >= a.rank || (seen & (1u << qd)) || z.d[d] != a.d[qd]) return 18;
                seen |= 1u << qd;
            }
            work += z.bytes;
        } else if (o.code == 11 || o.code == 12) {  // graph.c:95-106
            if (a.rank != 4 || a.type != 1 || z.type != 1 || !defined[o.b] || !b.flags || b.type != 4 || b.bytes != 48)
                return 18;
            int32_t q[12];
            std::memcpy(q, P.arena.data() + b.offset, 48);
            for (unsigned d = 0; d < 6; d++)
                if (q[d] < 1 || q[d] > 4096) return 18;
            for (unsigned d = 6; d < 12; d++)
                if (q[d] < 0 || q[d] > 4096) return 18;
            int64_t hh = (int64_t)a.d[1] + q[6] + q[8] - (q[0] - 1) * (int64_t)q[4] - 1;
            int64_t ww = (int64_t)a.d[2] + q[7] + q[9] - (q[1] - 1) * (int64_t)q[5] - 1;
            if (hh < 0 || ww < 0 || hh / q[2] + 1 != q[10] || ww / q[3] + 1 != q[11]) return 18;
            uint64_t rows = (uint64_t)a.d[0] * q[10] * q[11], k = (uint64_t)q[0] * q[1] * a.d[3];
            if (o.code == 11) {
                if (z.rank != 2 || z.d[0] != rows || z.d[1] != k) return 18;
            } else if (z.rank != 4 || z.d[0] != a.d[0] || z.d[1] != (uint32_t)q[10] || z.d[2] != (uint32_t)q[11] ||
                       z.d[3] != a.d[3])
                return 18;
            work += rows * k;
        } else if (o.code == 13) {
            if (!same_shape(a, z) || a.type != 1 || !a.rank) return 18;
            work += a.bytes / 4;
        } else if (o.code >= 14 && o.code <= 17) {  // graph.c:108-116
            if (h.version < 2 || o.p[0] >= h.nt || !defined[o.p[0]] || !defined[o.b]) return 18;
            const Tensor &t = P.ts[o.p[0]];
            int rc = validate_vision(o, a, b, z, t, Q(o.p[0]),
                                     reinterpret_cast<const int8_t *>(P.arena.data() + b.offset), work);
            if (rc) return rc;
            if (o.p[1]) {
                unsigned id = o.p[1] - 1;
                if (id >= h.nt || !P.ts[id].flags || P.ts[id].type != 2 || P.ts[id].bytes != 256) return 18;
                P.death[id] = (int)i;
                work += z.bytes;
            }
            if ((o.code == 14 || o.code == 15) && z.bytes >= 2048 && (uint64_t)z.d[0] * z.d[1] * z.d[2] >= 8)
                parallel_vision = true;
        } else if (o.code == 18) {  // graph.c:117-124
            if (h.version < 2 || !defined[o.b] || a.type != 3 || !same_shape(a, b) || !same_shape(a, z) ||
                o.p[0] >= h.nt || o.p[1] || o.p[2] || o.p[3])
                return 18;
            const Tensor &t = P.ts[o.p[0]];
            if (!t.flags || t.type != 4 || t.bytes != 520 * 4) return 18;
            const int32_t *q = Q(o.p[0]);
            if (q[0] < 0 || q[1] < -31 || q[1] > 0 || q[2] < -128 || q[2] > 127 || q[3] < -128 || q[4] > 127 ||
                q[3] > q[4] || q[5] || q[6] || q[7])
                return 18;
            for (unsigned j = 8; j < 520; j++)
                if (q[j] < -267386880 || q[j] > 267386880) return 18;
            work += z.bytes;
        } else if (o.code == 19) {  // graph.c:125-134
            if (h.version < 2 || !b.flags || b.type != 4 || !b.bytes || b.bytes > 32 * 4 || b.bytes % 4 || z.type != 3 ||
                z.rank != 1 || o.p[0] || o.p[1] || o.p[2] || o.p[3])
                return 18;
            const uint32_t *list = reinterpret_cast<const uint32_t *>(P.arena.data() + b.offset);
            uint64_t total = 0;
            if (list[0] != o.a) return 18;
            for (unsigned j = 0; j < b.bytes / 4; j++) {
                unsigned id = list[j];
                if (id >= h.nt || !defined[id] || (P.ts[id].type != 2 && P.ts[id].type != 3)) return 18;
                total += P.ts[id].bytes;
                P.death[id] = (int)i;
            }
            if (total != z.bytes) return 18;
            work += total;
        } else if (o.code == 20) {  // graph.c:135-142
            unsigned axis = o.p[0];
            if (h.version < 2 || !defined[o.b] || a.type != 3 || b.type != 3 || z.type != 3 || a.rank != b.rank ||
                a.rank != z.rank || axis >= a.rank || o.p[1] || o.p[2] || o.p[3])
                return 18;
            for (unsigned d = 0; d < a.rank; d++) {
                if (d == axis) {
                    if ((uint64_t)a.d[d] + b.d[d] != z.d[d]) return 18;
                } else if (a.d[d] != b.d[d] || a.d[d] != z.d[d])
                    return 18;
            }
            work += z.bytes;
        } else if (o.code == 21) {  // graph.c:143-148
            if (h.version < 2 || a.type != 3 || z.type != 3 || a.rank != 4 || z.rank != 4 || a.d[0] != z.d[0] ||
                a.d[3] != z.d[3] || !b.flags || b.type != 4 || b.bytes != (z.d[1] + z.d[2]) * 4 || o.p[0] || o.p[1] ||
                o.p[2] || o.p[3])
                return 18;
            const uint32_t *q = reinterpret_cast<const uint32_t *>(P.arena.data() + b.offset);
            uint32_t row = a.d[2] * a.d[3], batch = a.d[1] * row;
            for (unsigned d = 0; d < z.d[1]; d++)
                if (q[d] >= batch || q[d] % row) return 18;
            for (unsigned d = 0; d < z.d[2]; d++)
                if (q[z.d[1] + d] >= row || q[z.d[1] + d] % a.d[3]) return 18;
            work += z.bytes;
        } else if (o.code == 22) {  // graph.c:149-152
            if (h.version < 2 || (a.type != 2 && a.type != 3) || (z.type != 2 && z.type != 3) || a.rank != z.rank ||
                a.bytes != z.bytes || !b.flags || b.type != 2 || b.bytes != 256 || o.p[0] || o.p[1] || o.p[2] || o.p[3])
                return 18;
            for (unsigned d = 0; d < a.rank; d++)
                if (a.d[d] != z.d[d]) return 18;
            work += z.bytes;
        } else if (o.code == 23) {  // graph.c:153-157
            if (h.version < 2 || a.type != 3 || z.type != 3 || a.rank != 4 || z.rank != 4 || !b.flags || b.type != 4 ||
                b.bytes != 32 || (int32_t)o.p[0] < -128 || (int32_t)o.p[0] > 127 || o.p[1] || o.p[2] || o.p[3])
                return 18;
            const int32_t *q = reinterpret_cast<const int32_t *>(P.arena.data() + b.offset);
            for (unsigned d = 0; d < 4; d++)
                if (q[d * 2] < 0 || q[d * 2] > 4096 || q[d * 2 + 1] < 0 || q[d * 2 + 1] > 4096 ||
                    (uint64_t)a.d[d] + q[d * 2] + q[d * 2 + 1] != z.d[d])
                    return 18;
            work += z.bytes;
        } else if (o.code == 24) {  // graph.c:158-165
            if (h.version < 2 || a.type != 3 || z.type != 3 || a.rank != 4 || (z.rank != 2 && z.rank != 4) || !b.flags ||
                b.type != 4 || b.bytes != 20 || o.p[0] || o.p[1] || o.p[2] || o.p[3])
                return 18;
            if (z.d[0] != a.d[0] || z.d[z.rank - 1] != a.d[3] || (z.rank == 4 && (z.d[1] != 1 || z.d[2] != 1))) return 18;
            const int32_t *q = reinterpret_cast<const int32_t *>(P.arena.data() + b.offset);
            if (q[0] < 1 || (uint64_t)a.d[1] * a.d[2] != (uint32_t)q[0] || q[1] < -128 || q[1] > 127 || q[2] < -128 ||
                q[2] > 127 || q[3] < 0 || q[4] < -31 || q[4] > 30)
                return 18;
            uint64_t bound = (uint64_t)q[0] * (q[1] >= 0 ? 128 + q[1] : 127 - q[1]);
            if ((bound << (q[4] > 0 ? q[4] : 0)) > 2147483520u) return 18;
            work += a.bytes;
        } else if (o.code == 25 || o.code == 27) {  // graph.c:166-180
            if (h.version < 2 || a.type != 3 || b.type != 3 || z.type != 3 || !defined[o.b] || o.p[0] >= h.nt || o.p[1] ||
                o.p[2] || o.p[3])
                return 18;
            const Tensor &t = P.ts[o.p[0]];
            if (!t.flags || t.type != 4 || t.bytes != 28) return 18;
            const int32_t *q = Q(o.p[0]);
            for (unsigned j = 0; j < 3; j++)
                if (q[j] < -128 || q[j] > 127) return 18;
            if (q[3] < 0 || q[4] < -31 || q[4] > 15) return 18;
            uint64_t k = 1;
            if (o.code == 25) {
                if (!same_shape(a, b) || !same_shape(a, z) || q[5] < -128 || q[6] > 127 || q[5] > q[6]) return 18;
                work += z.bytes;
            } else {
                if (a.rank != 3 || b.rank != 3 || z.rank != 3 || q[5] < 0 || q[5] > 1 || q[6] < 0 || q[6] > 1 ||
                    a.d[0] != b.d[0] || a.d[0] != z.d[0])
                    return 18;
                unsigned m = a.d[q[5] ? 2 : 1], n = b.d[q[6] ? 1 : 2];
                k = a.d[q[5] ? 1 : 2];
                if (k != b.d[q[6] ? 2 : 1] || k > 8192 || n > 2048 || z.d[1] != m || z.d[2] != n) return 18;
                work += (uint64_t)z.bytes * k;
            }
            if (k * 65025 * (1ULL << (q[4] > 0 ? q[4] : 0)) > 2147483520u) return 18;
        } else if (o.code == 26) {  // graph.c:181-187
            if (h.version < 2 || a.type != 3 || z.type != 3 || a.rank != z.rank || !a.rank) return 18;
            for (unsigned d = 0; d < 4; d++) {
                if (d >= a.rank) {
                    if (o.p[d]) return 18;
                } else if ((uint64_t)o.p[d] + z.d[d] > a.d[d])
                    return 18;
            }
            work += z.bytes;
        } else if (o.code == 28) {  // graph.c:188-193
            if (h.version < 2 || a.type != 3 || !same_shape(a, z) || !a.rank || a.d[a.rank - 1] > 2048 || !b.flags ||
                b.type != 4 || b.bytes != 257 * 4 || o.p[0] || o.p[1] || o.p[2] || o.p[3])
                return 18;
            const int32_t *q = reinterpret_cast<const int32_t *>(P.arena.data() + b.offset);
            if (q[0] != (int32_t)a.d[a.rank - 1] || q[1] != 2147483647) return 18;
            for (unsigned d = 2; d <= 256; d++)
                if (q[d] < 0 || q[d] > q[d - 1]) return 18;
            work += z.bytes;
        } else
            return 19;
        if (work > kMaxWork) return 20;  // graph.c:195
        P.death[o.a] = (int)i;           // graph.c:196-200
        P.death[o.b] = (int)i;
        P.birth[o.out] = (int)i;
        P.death[o.out] = (int)i;
        if (o.code >= 14 && o.code <= 18) P.death[o.p[0]] = (int)i;
        if (o.code == 25 || o.code == 27) P.death[o.p[0]] = (int)i;
        if (o.code == 6 || o.code == 9) P.death[o.p[2]] = (int)i;
        defined[o.out] = 1;
    }
    P.vision_only = vision_only && parallel_vision;
    if (!defined[h.output]) return 21;  // graph.c:203
    P.death[h.output] = (int)h.no;
    if (h.version == 3) {  // graph.c:204-216
        for (unsigned a = 0; a < h.nt; a++) {
            if (P.ts[a].flags) {
                P.birth[a] = -1;
                P.death[a] = (int)h.no;
            }
            if (!defined[a]) return 15;
        }
        for (unsigned a = 0; a < h.nt; a++)
            for (unsigned b = a + 1; b < h.nt; b++) {
                bool memory_overlap = P.ts[a].offset < P.ts[b].offset + P.ts[b].bytes &&
                                      P.ts[b].offset < P.ts[a].offset + P.ts[a].bytes;
                bool live_overlap = P.birth[a] <= P.death[b] && P.birth[b] <= P.death[a];
                if (memory_overlap && live_overlap) return 25;
            }
    }
    out = std::move(P);
    return 0;
}

}  // namespace uq
