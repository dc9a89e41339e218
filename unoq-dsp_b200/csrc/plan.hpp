// plan.hpp -- UGN1 plan model and loader validation (host only, no CUDA).
//
// The byte layout is the reference's plan ABI (runtime/graph.h:15-38): a 32-byte header,
// 48-byte tensor descriptors, 32-byte op records, then the arena image. Validation returns
// exactly the codes of runtime/graph.c:50-216 and runtime/qnn.c:209-252 so that a plan
// rejected by the reference is rejected here with the same number.
#pragma once
#include <cstdint>
#include <vector>

namespace uq {

struct Header { uint32_t magic, version, nt, no, arena_bytes, input, output, reserved; };
struct Tensor { uint32_t offset, bytes, type, rank, d[4], flags, reserved[3]; };
struct Op { uint32_t code, a, b, out, p[4]; };
static_assert(sizeof(Header) == 32 && sizeof(Tensor) == 48 && sizeof(Op) == 32, "plan ABI sizes");

constexpr uint32_t kMagic = 0x55474e31u;
constexpr uint32_t kMaxTensors = 1024, kMaxOps = 512;
constexpr uint32_t kArena = 16u * 1024u * 1024u, kMaxPlan = 17u * 1024u * 1024u;
constexpr uint64_t kMaxWork = 2000000000ull;
constexpr int kHead = 20;      // qnn.h:8  UQ_HEAD
constexpr int kMaxK = 8192;    // qnn.h:10 UQ_MAX_K
constexpr int kMaxC = 2048;    // qnn.h:11 UQ_MAX_C

// Element width of a tensor type (graph.c:31): 1 f32, 2 u8, 3 s8, 4 s32.
inline uint32_t type_width(uint32_t t) { return t == 1 || t == 4 ? 4u : t == 2 || t == 3 ? 1u : 0u; }

struct Plan {
    Header h{};
    std::vector<Tensor> ts;
    std::vector<Op> ops;
    std::vector<uint8_t> arena;          // arena image (constants at their offsets)
    std::vector<int> birth, death;       // op index that defines / last reads each tensor
    bool vision_only = false;

    const uint8_t *bytes(uint32_t t) const { return arena.data() + ts[t].offset; }
    const int32_t *q(uint32_t t) const { return reinterpret_cast<const int32_t *>(bytes(t)); }
    const int8_t *s8(uint32_t t) const { return reinterpret_cast<const int8_t *>(bytes(t)); }
};

// The reference's TFLite fixed-point requantisation (qnn.c:61-83), host copy used by the
// loader's overflow proofs and by weight preparation.
int32_t host_scale(int32_t v, int32_t m, int shift);

// The vision ops' parameter-block check (qnn.c:209-252, uq_validate): codes 14-17, host copies of
// the q block and weights. Returns 0 (adding the op's work to `work`) or 18.
int validate_vision(const Op &o, const Tensor &a, const Tensor &b, const Tensor &z, const Tensor &t,
                    const int32_t *q, const int8_t *w, uint64_t &work);

// Parse and validate; on success `out` holds the plan and lifetimes. Returns 0 or 10..25.
int parse_plan(const void *blob, uint32_t len, Plan &out);

}  // namespace uq
