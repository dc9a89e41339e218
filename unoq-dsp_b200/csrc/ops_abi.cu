// ops_abi.cu -- the operator-level C ABI (include/unoq_ops.h): the reference's qnn.h / gemm.h entry
// points (runtime/qnn.h:12-23, runtime/gemm.h:5-25) over DEVICE buffers.
//
// Every data array (activations, weights, parameter blocks, tables, GEMM operands) is device memory
// of the device the C ABI works on (ug_set_device); the UGTensor / UGOp descriptors, uq_validate's
// constants and ug_matmul_u8i8_selected's group list are host memory, as the reference's loader
// holds them. Every call is synchronous: it first waits for the device (so that buffers written by
// any stream are complete), runs on a stream of its own and returns when its outputs are written.
//
// uq_run (codes 14-17) reads the op's parameter block and weights back, writes them into a one-op
// UGN1 plan whose tensors are one image of the op (d[0] = 1) and runs that plan through the same
// executor as ug_load: the same validation codes, kernel choice, weight repacking and epilogues as a
// whole graph. Prepared plans are cached by their bytes (parameters, weights, post table and
// shapes), so a changed constant never reuses a stale preparation. The element-wise ops launch the
// executor's own kernels directly; the raw GEMMs use k_gemm.cu.
#include <cuda_runtime.h>

#include <array>
#include <cstring>
#include <map>
#include <memory>
#include <mutex>
#include <string>
#include <vector>

#include "engine.hpp"
#include "gemm.cuh"
#include "kernels.cuh"
#include "unoq_ops.h"

namespace {

using uq::kHead;

std::mutex g_mu;        // the operator ABI is serialised (the reference's is not thread-safe at all)
int g_status = 0;       // uq_status(): result of the last call
std::map<int, cudaStream_t> g_streams;
std::vector<std::pair<const void *, const void *>> g_post;  // uq_post_register: q block -> table
std::map<std::string, std::unique_ptr<uq::Engine>> g_plans; // uq_run's prepared one-op plans
constexpr size_t kMaxCachedPlans = 64;

struct Scratch {                       // staging for uq_run operands that are not 256-byte aligned
    void *ptr = nullptr;
    size_t bytes = 0;
};
std::map<int, std::array<Scratch, 2>> g_scratch;

int fail(int code, const std::string &msg) {
    uq::set_error(msg);
    g_status = code;
    return code;
}

#define OPS_CUDA(call)                                                                   \
    do {                                                                                 \
        cudaError_t e_ = (call);                                                         \
        if (e_ != cudaSuccess) return fail(2001, std::string(#call) + ": " + cudaGetErrorString(e_)); \
    } while (0)

// Enter a call: select the device, wait for earlier work on it, get this ABI's stream.
int begin(int *device, cudaStream_t *s) {
    int count = 0;
    if (cudaGetDeviceCount(&count) != cudaSuccess || count <= 0) return fail(2002, "no CUDA device");
    *device = uq::abi_device();
    if (*device < 0 || *device >= count) return fail(2002, "device index out of range");
    OPS_CUDA(cudaSetDevice(*device));
    OPS_CUDA(cudaDeviceSynchronize());
    auto it = g_streams.find(*device);
    if (it == g_streams.end()) {
        cudaStream_t st = nullptr;
        OPS_CUDA(cudaStreamCreateWithFlags(&st, cudaStreamNonBlocking));
        it = g_streams.emplace(*device, st).first;
    }
    *s = it->second;
    return 0;
}

int finish(cudaStream_t s) {
    cudaError_t e = cudaGetLastError();
    if (e == cudaSuccess) e = cudaStreamSynchronize(s);
    if (e != cudaSuccess) return fail(2001, std::string("operator kernel: ") + cudaGetErrorString(e));
    g_status = 0;
    return 0;
}

// Device (or managed) memory of `device`; null and host pointers are refused.
bool on_device(const void *p, int device) {
    if (!p) return false;
    cudaPointerAttributes at{};
    if (cudaPointerGetAttributes(&at, p) != cudaSuccess) {
        cudaGetLastError();
        return false;
    }
    return (at.type == cudaMemoryTypeDevice || at.type == cudaMemoryTypeManaged) && at.device == device;
}

int need_device(int device, std::initializer_list<const void *> ptrs) {
    for (const void *p : ptrs)
        if (!on_device(p, device))
            return fail(22, "operator ABI: every data pointer must be device memory of device " + std::to_string(device));
    return 0;
}

int read_back(void *dst, const void *src, size_t bytes) {
    OPS_CUDA(cudaMemcpy(dst, src, bytes, cudaMemcpyDeviceToHost));
    return 0;
}

const void *post_table(const void *q) {
    for (auto &e : g_post)
        if (e.first == q) return e.second;
    return nullptr;
}

uint64_t elements(const UGTensor &t) {
    uint64_t n = t.rank ? 1 : 0;
    for (uint32_t d = 0; d < t.rank && d < 4; d++) n *= t.d[d];
    return n;
}

// One-op UGN1 plan (runtime/graph.h:15-38): tensors [0] input (one image), [1] weights (constant),
// [2] parameter block (constant), [3] output (one image), [4] post table (constant, optional).
std::string one_op_plan(unsigned code, const UGTensor &a1, const UGTensor &z1, const std::vector<uint8_t> &w,
                        const std::vector<int32_t> &q, const std::vector<uint8_t> &post) {
    auto up = [](uint32_t v) { return (v + 255u) & ~255u; };
    const uint32_t nt = post.empty() ? 4 : 5;
    uq::Tensor ts[5] = {};
    uint32_t off = 0;
    auto place = [&](uq::Tensor &t, uint32_t bytes, uint32_t type, uint32_t flags) {
        t.offset = off;
        t.bytes = bytes;
        t.type = type;
        t.flags = flags;
        off = up(off + bytes);
    };
    place(ts[0], a1.bytes, 3, 0);
    ts[0].rank = a1.rank;
    std::memcpy(ts[0].d, a1.d, sizeof(ts[0].d));
    place(ts[1], (uint32_t)w.size(), 3, 1);
    ts[1].rank = 1;
    ts[1].d[0] = (uint32_t)w.size();
    place(ts[2], (uint32_t)(q.size() * 4), 4, 1);
    ts[2].rank = 1;
    ts[2].d[0] = (uint32_t)q.size();
    place(ts[3], z1.bytes, 3, 0);
    ts[3].rank = z1.rank;
    std::memcpy(ts[3].d, z1.d, sizeof(ts[3].d));
    if (!post.empty()) {
        place(ts[4], 256, 2, 1);
        ts[4].rank = 1;
        ts[4].d[0] = 256;
    }
    uq::Header h{uq::kMagic, 2, nt, 1, off ? off : 256, 0, 3, 0};
    uq::Op o{code, 0, 1, 3, {2, post.empty() ? 0u : 5u, 0, 0}};
    std::string plan(sizeof(h) + nt * sizeof(uq::Tensor) + sizeof(o) + h.arena_bytes, '\0');
    char *p = &plan[0];
    std::memcpy(p, &h, sizeof(h));
    std::memcpy(p + sizeof(h), ts, nt * sizeof(uq::Tensor));
    std::memcpy(p + sizeof(h) + nt * sizeof(uq::Tensor), &o, sizeof(o));
    char *arena = p + sizeof(h) + nt * sizeof(uq::Tensor) + sizeof(o);
    std::memcpy(arena + ts[1].offset, w.data(), w.size());
    std::memcpy(arena + ts[2].offset, q.data(), q.size() * 4);
    if (!post.empty()) std::memcpy(arena + ts[4].offset, post.data(), 256);
    return plan;
}

// Caller operands of uq_run that are not 256-byte aligned go through aligned staging buffers.
int staging(int device, int slot, size_t bytes, void **out) {
    Scratch &sc = g_scratch[device][slot];
    if (sc.bytes < bytes) {
        if (sc.ptr) cudaFree(sc.ptr);
        sc.ptr = nullptr;
        sc.bytes = 0;
        OPS_CUDA(cudaMalloc(&sc.ptr, bytes));
        sc.bytes = bytes;
    }
    *out = sc.ptr;
    return 0;
}

bool aligned256(const void *p) { return (reinterpret_cast<uintptr_t>(p) & 255u) == 0; }

// Raw GEMM entry: argument rules per variant are checked by the callers.
int run_gemm(const uint8_t *x, const int8_t *w, int32_t *y, unsigned m, unsigned n, unsigned k, unsigned xs,
             int layout, const uint16_t *groups, unsigned count) {
    std::lock_guard<std::mutex> lk(g_mu);
    int device = 0;
    cudaStream_t s = nullptr;
    if (int rc = begin(&device, &s)) return rc;
    if (int rc = need_device(device, {x, w, y})) return rc;
    uq::GemmArgs g{};
    g.m = m;
    g.n = n;
    g.k = k;
    g.xs = xs;
    g.layout = layout;
    g.x_aligned = (reinterpret_cast<uintptr_t>(x) & 3u) == 0 && xs % 4 == 0;
    g.w_aligned = (reinterpret_cast<uintptr_t>(w) & 3u) == 0 && (layout != uq::kGemmRowMajor || k % 4 == 0);
    uint16_t *d_groups = nullptr;
    if (groups) {
        g.cols = 4 * count;
        if (!count) return finish(s);
        void *buf = nullptr;
        if (int rc = staging(device, 1, count * sizeof(uint16_t), &buf)) return rc;
        d_groups = static_cast<uint16_t *>(buf);
        OPS_CUDA(cudaMemcpyAsync(d_groups, groups, count * sizeof(uint16_t), cudaMemcpyHostToDevice, s));
    }
    uq::launch_gemm_u8i8(x, w, y, g, d_groups, s);
    return finish(s);
}

}  // namespace

extern "C" {

int uq_validate(const UGOp *o, const UGTensor *a, const UGTensor *b, const UGTensor *z, const UGTensor *t,
                const void *data, const void *weights, uint64_t *work) {
    if (!o || !a || !b || !z || !t || !data || !work || (!weights && (o->code == 14 || o->code == 15))) return 22;
    uq::Op op;
    uq::Tensor ta, tb, tz, tt;
    std::memcpy(&op, o, sizeof(op));
    std::memcpy(&ta, a, sizeof(ta));
    std::memcpy(&tb, b, sizeof(tb));
    std::memcpy(&tz, z, sizeof(tz));
    std::memcpy(&tt, t, sizeof(tt));
    static const int8_t none = 0;
    return uq::validate_vision(op, ta, tb, tz, tt, static_cast<const int32_t *>(data),
                               weights ? static_cast<const int8_t *>(weights) : &none, *work);
}

int uq_run(unsigned code, const UGTensor *a, const UGTensor *z, const int8_t *x, const int8_t *w, int8_t *y,
           const int32_t *q, int threads) {
    (void)threads;  // the grid replaces the reference's two workers
    std::lock_guard<std::mutex> lk(g_mu);
    if (code < 14 || code > 17) return fail(19, "uq_run: codes 14-17 only");
    if (!a || !z) return fail(22, "uq_run: null tensor descriptor");
    int device = 0;
    cudaStream_t s = nullptr;
    if (int rc = begin(&device, &s)) return rc;
    if (int rc = need_device(device, {x, y, q})) return rc;
    if ((code == 14 || code == 15) && !on_device(w, device)) return fail(22, "uq_run: weights must be device memory");
    // The op's images: the runs below see one image of d[0] == 1 and are repeated a->d[0] times.
    UGTensor a1 = *a, z1 = *z;
    if (!a->rank || !z->rank || a->rank > 4 || z->rank > 4 || a->type != 3 || z->type != 3 || a->d[0] != z->d[0] ||
        !a->d[0] || elements(*a) != a->bytes || elements(*z) != z->bytes)
        return fail(18, "uq_run: tensor descriptors do not describe int8 tensors with one batch axis");
    const uint32_t images = a->d[0];
    a1.d[0] = z1.d[0] = 1;
    a1.bytes = a->bytes / images;
    z1.bytes = z->bytes / images;
    a1.offset = z1.offset = 0;
    a1.flags = z1.flags = 0;
    int32_t head[kHead];
    if (int rc = read_back(head, q, sizeof(head))) return rc;
    size_t qwords = kHead, wbytes = 0;
    if (code == 14 || code == 15) {
        const int oc = head[17];
        if (oc < 1 || oc > uq::kMaxC || head[0] < 1 || head[1] < 1 || head[0] > 4096 || head[1] > 4096 ||
            (uint64_t)head[0] * head[1] > (uint64_t)uq::kMaxK || head[18] < 0 || head[18] > uq::kMaxK)
            return fail(18, "uq_run: parameter block out of range");
        qwords = kHead + 3 * (size_t)oc;
        wbytes = code == 15 ? (size_t)head[0] * head[1] * oc : (size_t)((oc + 3) & ~3) * head[18];
    } else if (code == 17) {
        qwords = kHead + 256;
    }
    std::vector<int32_t> qh(qwords);
    if (int rc = read_back(qh.data(), q, qwords * 4)) return rc;
    std::vector<uint8_t> wh(wbytes ? wbytes : 4, 0);
    if (wbytes)
        if (int rc = read_back(wh.data(), w, wbytes)) return rc;
    std::vector<uint8_t> post;
    if (const void *table = post_table(q)) {
        if (code != 14 && code != 15) return fail(18, "uq_run: a post table applies to codes 14 and 15 only");
        if (!on_device(table, device)) return fail(22, "uq_run: post table must be device memory");
        post.resize(256);
        if (int rc = read_back(post.data(), table, 256)) return rc;
    }
    if (a1.bytes > uq::kArena || z1.bytes > uq::kArena) return fail(20, "uq_run: one image exceeds 16 MiB");
    std::string plan = one_op_plan(code, a1, z1, wh, qh, post);
    auto it = g_plans.find(plan);
    if (it == g_plans.end()) {
        if (g_plans.size() >= kMaxCachedPlans) g_plans.clear();
        auto eng = std::make_unique<uq::Engine>();
        const int rc = eng->load(plan.data(), (uint32_t)plan.size(), device);
        if (rc) return fail(rc, std::string("uq_run: ") + uq::last_error());
        it = g_plans.emplace(std::move(plan), std::move(eng)).first;
    }
    uq::Engine &eng = *it->second;
    // operands the executor's kernels may read with TMA / 16-byte vectors must be aligned
    const int8_t *xin = x;
    int8_t *yout = y;
    if (!aligned256(x)) {
        void *buf = nullptr;
        if (int rc = staging(device, 0, a->bytes, &buf)) return rc;
        OPS_CUDA(cudaMemcpy(buf, x, a->bytes, cudaMemcpyDeviceToDevice));
        xin = static_cast<const int8_t *>(buf);
    }
    void *ybuf = nullptr;
    if (!aligned256(y)) {
        if (int rc = staging(device, 1, z->bytes, &ybuf)) return rc;
        yout = static_cast<int8_t *>(ybuf);
    }
    int rc = eng.run_device(xin, yout, images);
    if (rc) {
        g_plans.erase(it);  // a failed run leaves nothing prepared behind (graph.c:298-305)
        return fail(rc, std::string("uq_run: ") + uq::last_error());
    }
    if (ybuf) OPS_CUDA(cudaMemcpy(y, ybuf, z->bytes, cudaMemcpyDeviceToDevice));
    g_status = 0;
    return 0;
}

void uq_add(const int8_t *x, const int8_t *b, int8_t *y, uint32_t count, const int32_t *q) {
    std::lock_guard<std::mutex> lk(g_mu);
    int device = 0;
    cudaStream_t s = nullptr;
    if (begin(&device, &s) || need_device(device, {x, b, y, q})) return;
    uq::launch_add(x, b, y, count, q, s);
    finish(s);
}

void uq_mean(const int8_t *x, int8_t *y, unsigned batches, unsigned channels, const int32_t *q) {
    std::lock_guard<std::mutex> lk(g_mu);
    int device = 0;
    cudaStream_t s = nullptr;
    if (begin(&device, &s) || need_device(device, {x, y, q})) return;
    int32_t q5[5];
    if (read_back(q5, q, sizeof(q5))) return;
    if (q5[0] < 1 || !channels || channels > (unsigned)uq::kMaxC) {
        fail(18, "uq_mean: count must be positive and channels 1..2048");
        return;
    }
    uq::launch_mean(x, y, batches, (int)channels, q5, s);
    finish(s);
}

void uq_mul(const int8_t *x, const int8_t *b, int8_t *y, unsigned count, const int32_t *q) {
    std::lock_guard<std::mutex> lk(g_mu);
    int device = 0;
    cudaStream_t s = nullptr;
    if (begin(&device, &s) || need_device(device, {x, b, y, q})) return;
    int32_t q7[7];
    if (read_back(q7, q, sizeof(q7))) return;
    uq::launch_mul(x, b, y, count, q7, s);
    finish(s);
}

int uq_bmm(const UGTensor *a, const UGTensor *b, const UGTensor *z, const int8_t *x, const int8_t *w, int8_t *y,
           const int32_t *q, int threads) {
    (void)threads;
    std::lock_guard<std::mutex> lk(g_mu);
    if (!a || !b || !z) return fail(22, "uq_bmm: null tensor descriptor");
    int device = 0;
    cudaStream_t s = nullptr;
    if (int rc = begin(&device, &s)) return rc;
    if (int rc = need_device(device, {x, w, y, q})) return rc;
    int32_t q7[7];
    if (int rc = read_back(q7, q, sizeof(q7))) return rc;
    // the loader's rule for code 27 (graph.c:166-180, restated in plan.cpp)
    if (a->rank != 3 || b->rank != 3 || z->rank != 3 || q7[5] < 0 || q7[5] > 1 || q7[6] < 0 || q7[6] > 1 ||
        a->d[0] != b->d[0] || a->d[0] != z->d[0])
        return fail(18, "uq_bmm: shapes");
    const unsigned m = a->d[q7[5] ? 2 : 1], n = b->d[q7[6] ? 1 : 2], k = a->d[q7[5] ? 1 : 2];
    if (k != b->d[q7[6] ? 2 : 1] || k > 8192 || n > 2048 || z->d[1] != m || z->d[2] != n)
        return fail(18, "uq_bmm: shapes");
    uq::launch_bmm(x, w, y, z->d[0], (int)m, (int)n, (int)k, q7, s);
    return finish(s);
}

void uq_post_reset(void) {
    std::lock_guard<std::mutex> lk(g_mu);
    g_post.clear();
    g_plans.clear();
}

void uq_post_register(const int32_t *q, const uint8_t *table) {
    std::lock_guard<std::mutex> lk(g_mu);
    if (g_post.size() < uq::kMaxOps) g_post.emplace_back(q, table);  // qnn.c:161: at most UG_MAX_OP
}

void uq_softmax_exact(const int8_t *x, int8_t *y, unsigned bytes, const int32_t *q) {
    std::lock_guard<std::mutex> lk(g_mu);
    int device = 0;
    cudaStream_t s = nullptr;
    if (begin(&device, &s) || need_device(device, {x, y, q})) return;
    int32_t width = 0;
    if (read_back(&width, q, 4)) return;
    if (width < 1 || width > uq::kMaxC || bytes % (unsigned)width) {
        fail(18, "uq_softmax_exact: row width must be 1..2048 and divide the bytes");
        return;
    }
    // the kernel reads the exponent table through the read-only data path: give it the library's
    // own copy of the 257 words rather than the caller's buffer
    void *qcopy = nullptr;
    if (staging(device, 1, 257 * sizeof(int32_t), &qcopy)) return;
    if (cudaMemcpyAsync(qcopy, q, 257 * sizeof(int32_t), cudaMemcpyDeviceToDevice, s) != cudaSuccess) {
        fail(2001, "uq_softmax_exact: table copy");
        return;
    }
    uq::launch_softmax_exact_rows(x, y, bytes / (unsigned)width, width, static_cast<const int32_t *>(qcopy), s);
    finish(s);
}

int ug_matmul_u8i8(const uint8_t *x, const int8_t *w, int32_t *y, unsigned m, unsigned n, unsigned k, int packed,
                   int threads) {
    (void)threads;
    if (packed && k % 8) return fail(18, "ug_matmul_u8i8: packed weights need K % 8 == 0");
    return run_gemm(x, w, y, m, n, k, k, packed ? uq::kGemmPacked : uq::kGemmRowMajor, nullptr, 0);
}

int ug_matmul_u8i8_strided(const uint8_t *x, const int8_t *w, int32_t *y, unsigned m, unsigned n, unsigned k,
                           unsigned xs) {
    if (!m || !n || !k || k > 8192 || n % 4 || k % 8 || xs < k || xs % 8) return fail(18, "ug_matmul_u8i8_strided");
    return run_gemm(x, w, y, m, n, k, xs, uq::kGemmPacked, nullptr, 0);
}

int ug_matmul_u8i8_dot4(const uint8_t *x, const int8_t *w, int32_t *y, unsigned m, unsigned n, unsigned k,
                        unsigned xs) {
    if (!m || m % 2 || !n || n % 4 || !k || k % 8 || k > 8192 || xs < k || xs % 8) return fail(18, "ug_matmul_u8i8_dot4");
    return run_gemm(x, w, y, m, n, k, xs, uq::kGemmDot4, nullptr, 0);
}

int ug_matmul_u8i8_selected(const uint8_t *x, const int8_t *w, int32_t *y, unsigned m, unsigned n, unsigned k,
                            unsigned xs, const uint16_t *groups, unsigned count) {
    if (!m || !n || k < 64 || k > 8192 || n % 4 || k % 8 || xs < k || xs % 8 || count > n / 4 || (count && !groups))
        return fail(18, "ug_matmul_u8i8_selected");
    for (unsigned g = 0; g < count; g++)
        if (groups[g] % 4 || groups[g] >= n) return fail(18, "ug_matmul_u8i8_selected: group offsets");
    static const uint16_t empty = 0;
    return run_gemm(x, w, y, m, n, k, xs, uq::kGemmPacked, count ? groups : &empty, count);
}

int ug_gemm_available(void) {
    int count = 0;
    return cudaGetDeviceCount(&count) == cudaSuccess && count > 0 ? 1 : 0;
}

int uq_status(void) {
    std::lock_guard<std::mutex> lk(g_mu);
    return g_status;
}

}  // extern "C"
