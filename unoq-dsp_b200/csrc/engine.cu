// engine.cu -- plan preparation, batched arena planning, op lowering and CUDA-graph replay.
#include "engine.hpp"

#include <algorithm>
#include <chrono>
#include <cmath>
#include <cstring>
#include <mutex>
#include <numeric>
#include <thread>

#include "conv_rows.cuh"
#include "conv_taps.cuh"
#include "conv_small.cuh"
#include "conv_tc.cuh"
#include "dw.cuh"
#include "dw_tc.cuh"
#include "kernels.cuh"

namespace uq {

namespace {
std::mutex g_err_mu;
std::string g_err;

constexpr size_t kAlign = 256;
size_t align_up(size_t v, size_t a) { return (v + a - 1) / a * a; }
}  // namespace

void set_error(const std::string &msg) {
    std::lock_guard<std::mutex> lk(g_err_mu);
    g_err = msg;
}
const char *last_error() { return g_err.c_str(); }

#define UQ_CUDA(call)                                                                      \
    do {                                                                                   \
        cudaError_t e_ = (call);                                                           \
        if (e_ != cudaSuccess) {                                                           \
            set_error(std::string(#call) + ": " + cudaGetErrorString(e_));                 \
            return 2001;                                                                   \
        }                                                                                  \
    } while (0)

Engine::~Engine() { release(); }

void Engine::drop_mailbox() {
    if (mb_exec_) cudaGraphExecDestroy(mb_exec_);
    if (mb_graph_) cudaGraphDestroy(mb_graph_);
    if (mb_in_) cudaFreeHost(mb_in_);
    if (mb_out_) cudaFreeHost(mb_out_);
    mb_exec_ = nullptr;
    mb_graph_ = nullptr;
    mb_in_ = mb_out_ = nullptr;
}

void Engine::release() {
    if (device_ >= 0 && (d_const_ || stream_)) cudaSetDevice(device_);
    if (stream_) cudaStreamSynchronize(stream_);
    drop_mailbox();
    gather_.reset();
    for (auto &kv : batches_) {
        BatchCtx &b = *kv.second;
        if (b.exec) cudaGraphExecDestroy(b.exec);
        if (b.graph) cudaGraphDestroy(b.graph);
        if (b.arena) cudaFree(b.arena);
        if (b.host_in) cudaFreeHost(b.host_in);
        if (b.host_out) cudaFreeHost(b.host_out);
        if (b.pixels) cudaFree(b.pixels);
        if (b.records) cudaFree(b.records);
    }
    batches_.clear();
    if (d_table_) cudaFree(d_table_);
    if (d_yolo_) cudaFree(d_yolo_);
    d_table_ = nullptr;
    d_yolo_ = nullptr;
    table_channels_ = 0;
    yolo_ = YoloShape();
    for (void *p : prep_) cudaFree(p);
    prep_.clear();
    if (d_const_) cudaFree(d_const_);
    d_const_ = nullptr;
    if (ev0_) cudaEventDestroy(ev0_);
    if (ev1_) cudaEventDestroy(ev1_);
    ev0_ = ev1_ = nullptr;
    for (auto &e : pipe_t_) {
        if (e) cudaEventDestroy(e);
        e = nullptr;
    }
    pipe_growth_ = kInitialPieceGrowth;
    last_ctx_ = nullptr;
    last_images_ = 0;
    for (auto &row : pipe_ev_)
        for (auto &e : row) {
            if (e) cudaEventDestroy(e);
            e = nullptr;
        }
    if (h2d_) cudaStreamDestroy(h2d_);
    if (d2h_) cudaStreamDestroy(d2h_);
    h2d_ = d2h_ = nullptr;
    if (stream_) cudaStreamDestroy(stream_);
    stream_ = nullptr;
    steps_.clear();
    static_ = BatchCtx();  // the static arena is not owned; its layout belongs to this plan
    static_replicated_.clear();
    ready_ = false;
}

void *Engine::prep_alloc(size_t bytes) {
    void *p = nullptr;
    if (cudaMalloc(&p, bytes ? bytes : 1) != cudaSuccess) return nullptr;
    prep_.push_back(p);
    return p;
}

int Engine::load(const void *plan, uint32_t bytes, int device) {
    release();
    Plan P;
    int rc = parse_plan(plan, bytes, P);
    if (rc) return rc;
    int count = 0;
    if (cudaGetDeviceCount(&count) != cudaSuccess || count <= 0) {
        set_error("no CUDA device");
        return 2002;
    }
    if (device < 0 || device >= count) {
        set_error("device index out of range");
        return 2002;
    }
    device_ = device;
    P_ = std::move(P);
    UQ_CUDA(cudaSetDevice(device_));
    UQ_CUDA(cudaStreamCreateWithFlags(&stream_, cudaStreamNonBlocking));
    UQ_CUDA(cudaStreamCreateWithFlags(&h2d_, cudaStreamNonBlocking));
    UQ_CUDA(cudaStreamCreateWithFlags(&d2h_, cudaStreamNonBlocking));
    UQ_CUDA(cudaEventCreate(&ev0_));
    UQ_CUDA(cudaEventCreate(&ev1_));
    for (auto &e : pipe_t_) UQ_CUDA(cudaEventCreate(&e));
    for (auto &row : pipe_ev_)
        for (auto &e : row) UQ_CUDA(cudaEventCreateWithFlags(&e, cudaEventDisableTiming));
    UQ_CUDA(cudaMalloc(&d_const_, P_.h.arena_bytes));
    UQ_CUDA(cudaMemcpy(d_const_, P_.arena.data(), P_.h.arena_bytes, cudaMemcpyHostToDevice));
    rc = prepare();
    if (rc) {
        release();
        return rc;
    }
    ticks_.assign(kMaxOps + 2, 0);
    profiling_ = false;
    ready_ = true;
    return 0;
}

// ----------------------------------------------------------------------------------------
// Lowering: one Step per plan op. Host-side parameter words are read from the plan arena;
// device-side tables (weights, q blocks, LUTs) are used in place in the uploaded constants.
int Engine::prepare() {
    const Plan &P = P_;
    const uint32_t nt = P.h.nt;
    alias_.resize(nt);
    std::iota(alias_.begin(), alias_.end(), 0);
    steps_.clear();
    birth_ = P.birth;
    death_ = P.death;
    fused_.assign(P.h.no, 0);
    const char *fuse_env = std::getenv("UNOQ_FUSE_ADD");
    fuse_adds_ = !(fuse_env && fuse_env[0] == '0');
    skip_.assign(P.h.no, 0);
    concat_in_.assign(P.h.no, {});
    concat_parts_.assign(P.h.no, {});
    lut_src_.assign(P.h.no, LutSrc{});
    const char *bytes_env = std::getenv("UNOQ_FUSE_BYTES");
    if (!(bytes_env && bytes_env[0] == '0')) fuse_byte_ops();
    for (uint32_t i = 0; i < P.h.no; i++) {
        const Op o = P.ops[i];
        const Tensor a = P.ts[o.a], b = P.ts[o.b], z = P.ts[o.out];
        Step st;
        st.op = i;
        switch (o.code) {
            case 5: {  // graph.c:408 -- a copy of identical bytes becomes a storage alias
                int root = o.a;
                while (alias_[root] != root) root = alias_[root];
                alias_[o.out] = root;
                st.run = nullptr;
                break;
            }
            case 14: {
                const int32_t *q = P.q(o.p[0]);
                ConvGeom g{};
                g.n = (int)a.d[0];
                g.ih = (int)a.d[1], g.iw = (int)a.d[2], g.ic = q[16];
                g.oh = q[10], g.ow = q[11], g.oc = q[17];
                g.kh = q[0], g.kw = q[1], g.sh = q[2], g.sw = q[3], g.dh = q[4], g.dw = q[5], g.pt = q[6], g.pl = q[7];
                g.xzp = q[12];
                g.kp = q[18];
                const int32_t *dq = reinterpret_cast<const int32_t *>(dconst(o.p[0]));
                Requant r{dq + kHead, dq + kHead + g.oc, dq + kHead + 2 * g.oc,
                          o.p[1] ? dconst(o.p[1] - 1) : nullptr, q[13], q[14], q[15]};
                const uint32_t ta = o.a, tz = o.out;
                // a following residual add that the conv_tc epilogue can take (see below)
                const bool add_next = i + 1 < P.h.no && P.ops[i + 1].code == 18 && o.out != P.h.output &&
                                      death_[o.out] == (int)i + 1 && fuse_adds_;
                ConvRows *cr = nullptr;
                int rc = 0;
                // the row GEMM has no fused add: 17-32-channel inputs keep theirs in conv_tc
                if (!(add_next && g.ic > 16))
                    rc = conv_rows_prepare(P.s8(o.b), q, r.post, g, [this](size_t n) { return prep_alloc(n); }, &cr);
                if (rc) return rc;
                if (cr) {
                    std::shared_ptr<ConvRows> keep(cr, conv_rows_free);
                    st.run = [keep, g, ta, tz](const BatchCtx &B, cudaStream_t s) -> int {
                        ConvGeom gb = g;
                        gb.n = g.n * (int)B.images;
                        return conv_rows_launch(*keep, reinterpret_cast<const int8_t *>(B.ptr[ta]),
                                                reinterpret_cast<int8_t *>(B.ptr[tz]), gb, s);
                    };
                    break;
                }
                ConvSmall *sm = nullptr;
                rc = conv_small_prepare(P.s8(o.b), q, r.post, g, [this](size_t n) { return prep_alloc(n); }, &sm);
                if (rc) return rc;
                if (sm) {
                    std::shared_ptr<ConvSmall> keep(sm, conv_small_free);
                    st.run = [keep, g, ta, tz](const BatchCtx &B, cudaStream_t s) -> int {
                        ConvGeom gb = g;
                        gb.n = g.n * (int)B.images;
                        return conv_small_launch(*keep, reinterpret_cast<const int8_t *>(B.ptr[ta]),
                                                 reinterpret_cast<int8_t *>(B.ptr[tz]), gb, s);
                    };
                    break;
                }
                // Residual add fused into the epilogue when the next op is an add whose one input is
                // this conv's output and nothing else reads that output.
                ConvTc *tc = nullptr;
                if (add_next) {
                    const Op &n = P.ops[i + 1];
                    const bool is_a = n.a == o.out, is_b = n.b == o.out;
                    const uint32_t res = is_a ? n.b : n.a;
                    if (is_a != is_b && P.ts[res].bytes == z.bytes && P.ts[n.out].bytes == z.bytes &&
                        P.ts[res].type == z.type && P.ts[n.out].type == z.type) {
                        const FusedAdd fa{P.q(n.p[0]), reinterpret_cast<const int32_t *>(dconst(n.p[0])), is_b};
                        rc = conv_tc_prepare(P.s8(o.b), q, r.post, g, [this](size_t n2) { return prep_alloc(n2); }, &tc,
                                             &fa);
                        if (rc) return rc;
                        if (tc) {
                            std::shared_ptr<ConvTc> keep(tc, conv_tc_free);
                            const uint32_t tout = n.out, tres = res;
                            st.run = [keep, g, ta, tout, tres](const BatchCtx &B, cudaStream_t s) -> int {
                                ConvGeom gb = g;
                                gb.n = g.n * (int)B.images;
                                return conv_tc_launch(*keep, reinterpret_cast<const int8_t *>(B.ptr[ta]),
                                                      reinterpret_cast<int8_t *>(B.ptr[tout]), gb, s,
                                                      reinterpret_cast<const int8_t *>(B.ptr[tres]));
                            };
                            fused_.at(i + 1) = 1;
                            birth_[n.out] = (int)i;  // written during this op now
                            break;
                        }
                    }
                }
                ConvTaps *ct = nullptr;
                rc = conv_taps_prepare(P.s8(o.b), q, r.post, g, [this](size_t n) { return prep_alloc(n); }, &ct);
                if (rc) return rc;
                if (ct) {
                    std::shared_ptr<ConvTaps> keep(ct, conv_taps_free);
                    st.run = [keep, g, ta, tz](const BatchCtx &B, cudaStream_t s) -> int {
                        ConvGeom gb = g;
                        gb.n = g.n * (int)B.images;
                        return conv_taps_launch(*keep, reinterpret_cast<const int8_t *>(B.ptr[ta]),
                                                reinterpret_cast<int8_t *>(B.ptr[tz]), gb, s);
                    };
                    break;
                }
                rc = conv_tc_prepare(P.s8(o.b), q, r.post, g, [this](size_t n) { return prep_alloc(n); }, &tc);
                if (rc) return rc;
                const int8_t *w = reinterpret_cast<const int8_t *>(dconst(o.b));
                if (tc) {
                    std::shared_ptr<ConvTc> keep(tc, conv_tc_free);
                    st.run = [keep, g, ta, tz](const BatchCtx &B, cudaStream_t s) -> int {
                        ConvGeom gb = g;
                        gb.n = g.n * (int)B.images;
                        return conv_tc_launch(*keep, reinterpret_cast<const int8_t *>(B.ptr[ta]),
                                              reinterpret_cast<int8_t *>(B.ptr[tz]), gb, s);
                    };
                } else {
                    st.run = [g, r, w, ta, tz](const BatchCtx &B, cudaStream_t s) -> int {
                        ConvGeom gb = g;
                        gb.n = g.n * (int)B.images;
                        launch_conv_simt(reinterpret_cast<const int8_t *>(B.ptr[ta]), w,
                                         reinterpret_cast<int8_t *>(B.ptr[tz]), gb, r, s);
                        return 0;
                    };
                }
                break;
            }
            case 15:
            case 16: {
                const int32_t *q = P.q(o.p[0]);
                ConvGeom g{};
                g.n = (int)a.d[0];
                g.ih = (int)a.d[1], g.iw = (int)a.d[2], g.ic = q[16];
                g.oh = q[10], g.ow = q[11], g.oc = q[17];
                g.kh = q[0], g.kw = q[1], g.sh = q[2], g.sw = q[3], g.dh = q[4], g.dw = q[5], g.pt = q[6], g.pl = q[7];
                g.xzp = q[12];
                g.kp = q[18];
                const uint32_t ta = o.a, tz = o.out;
                if (o.code == 15) {
                    const int32_t *dq = reinterpret_cast<const int32_t *>(dconst(o.p[0]));
                    Requant r{dq + kHead, dq + kHead + g.oc, dq + kHead + 2 * g.oc,
                              o.p[1] ? dconst(o.p[1] - 1) : nullptr, q[13], q[14], q[15]};
                    const int8_t *w = reinterpret_cast<const int8_t *>(dconst(o.b));
                    DwTc *tcd = nullptr;
                    int rc = dw_tc_prepare(P.s8(o.b), q, r.post, g, [this](size_t n) { return prep_alloc(n); }, &tcd);
                    if (rc) return rc;
                    DwFast *fast = nullptr;
                    if (!tcd) rc = dw_prepare(P.s8(o.b), q, r.post, g, [this](size_t n) { return prep_alloc(n); }, &fast);
                    if (rc) return rc;
                    if (tcd) {
                        std::shared_ptr<DwTc> keep(tcd, dw_tc_free);
                        st.run = [keep, g, ta, tz](const BatchCtx &B, cudaStream_t s) -> int {
                            ConvGeom gb = g;
                            gb.n = g.n * (int)B.images;
                            return dw_tc_launch(*keep, reinterpret_cast<const int8_t *>(B.ptr[ta]),
                                                reinterpret_cast<int8_t *>(B.ptr[tz]), gb, s);
                        };
                    } else if (fast) {
                        std::shared_ptr<DwFast> keep(fast, dw_free);
                        st.run = [keep, g, ta, tz](const BatchCtx &B, cudaStream_t s) -> int {
                            ConvGeom gb = g;
                            gb.n = g.n * (int)B.images;
                            return dw_launch(*keep, reinterpret_cast<const int8_t *>(B.ptr[ta]),
                                             reinterpret_cast<int8_t *>(B.ptr[tz]), gb, s);
                        };
                    } else {
                        st.run = [g, r, w, ta, tz](const BatchCtx &B, cudaStream_t s) -> int {
                            ConvGeom gb = g;
                            gb.n = g.n * (int)B.images;
                            launch_depthwise(reinterpret_cast<const int8_t *>(B.ptr[ta]), w,
                                             reinterpret_cast<int8_t *>(B.ptr[tz]), gb, r, s);
                            return 0;
                        };
                    }
                } else {
                    const int is_max = q[19], lo = q[14], hi = q[15];
                    st.run = [g, is_max, lo, hi, ta, tz](const BatchCtx &B, cudaStream_t s) -> int {
                        ConvGeom gb = g;
                        gb.n = g.n * (int)B.images;
                        launch_pool(reinterpret_cast<const int8_t *>(B.ptr[ta]), reinterpret_cast<int8_t *>(B.ptr[tz]), gb,
                                    is_max, lo, hi, s);
                        return 0;
                    };
                }
                break;
            }
            case 17: {
                const int32_t *q = P.q(o.p[0]);
                const int width = q[16], lo = q[14], hi = q[15];
                const int32_t *table = reinterpret_cast<const int32_t *>(dconst(o.p[0])) + kHead;
                const uint32_t ta = o.a, tz = o.out, abytes = a.bytes;
                st.run = [=](const BatchCtx &B, cudaStream_t s) -> int {
                    launch_softmax_table(reinterpret_cast<const int8_t *>(B.ptr[ta]), reinterpret_cast<int8_t *>(B.ptr[tz]),
                                         (size_t)abytes / width * B.images, width, table, lo, hi, s);
                    return 0;
                };
                break;
            }
            case 28: {
                const int width = P.q(o.b)[0];
                const int32_t *dq = reinterpret_cast<const int32_t *>(dconst(o.b));
                const uint32_t ta = o.a, tz = o.out, abytes = a.bytes;
                st.run = [=](const BatchCtx &B, cudaStream_t s) -> int {
                    launch_softmax_exact(reinterpret_cast<const int8_t *>(B.ptr[ta]), reinterpret_cast<int8_t *>(B.ptr[tz]),
                                         (size_t)abytes / width * B.images, width, dq, s);
                    return 0;
                };
                break;
            }
            case 27: {
                const int32_t *q = P.q(o.p[0]);
                int32_t q7[7];
                std::memcpy(q7, q, sizeof(q7));
                const int m = (int)z.d[1], n = (int)z.d[2], k = (int)a.d[q[5] ? 1 : 2];
                const uint32_t ta = o.a, tb = o.b, tz = o.out, d0 = z.d[0];
                st.run = [=](const BatchCtx &B, cudaStream_t s) -> int {
                    int32_t qq[7];
                    std::memcpy(qq, q7, sizeof(qq));
                    launch_bmm(reinterpret_cast<const int8_t *>(B.ptr[ta]), reinterpret_cast<const int8_t *>(B.ptr[tb]),
                               reinterpret_cast<int8_t *>(B.ptr[tz]), (size_t)d0 * B.images, m, n, k, qq, s);
                    return 0;
                };
                break;
            }
            case 26: {
                if (skip_[i]) {  // read in place by the table op that consumes it
                    st.run = nullptr;
                    break;
                }
                Shape5 in{}, out{};
                in.rank = out.rank = (int)a.rank + 1;
                in.d[0] = out.d[0] = 1;
                uint32_t begin[5] = {0, 0, 0, 0, 0};
                for (uint32_t d = 0; d < a.rank; d++) {
                    in.d[d + 1] = a.d[d];
                    out.d[d + 1] = z.d[d];
                    begin[d + 1] = o.p[d];
                }
                const uint32_t ta = o.a, tz = o.out;
                st.run = [=](const BatchCtx &B, cudaStream_t s) -> int {
                    Shape5 ib = in, ob = out;
                    ib.d[0] = ob.d[0] = B.images;
                    launch_slice(B.ptr[ta], B.ptr[tz], ib, ob, begin, s);
                    return 0;
                };
                break;
            }
            case 25: {
                int32_t q7[7];
                std::memcpy(q7, P.q(o.p[0]), sizeof(q7));
                const uint32_t ta = o.a, tb = o.b, tz = o.out, zb = z.bytes;
                st.run = [=](const BatchCtx &B, cudaStream_t s) -> int {
                    int32_t qq[7];
                    std::memcpy(qq, q7, sizeof(qq));
                    launch_mul(reinterpret_cast<const int8_t *>(B.ptr[ta]), reinterpret_cast<const int8_t *>(B.ptr[tb]),
                               reinterpret_cast<int8_t *>(B.ptr[tz]), (size_t)zb * B.images, qq, s);
                    return 0;
                };
                break;
            }
            case 24: {
                int32_t q5[5];
                std::memcpy(q5, P.q(o.b), sizeof(q5));
                const uint32_t ta = o.a, tz = o.out, d0 = a.d[0], ch = a.d[3];
                st.run = [=](const BatchCtx &B, cudaStream_t s) -> int {
                    int32_t qq[5];
                    std::memcpy(qq, q5, sizeof(qq));
                    launch_mean(reinterpret_cast<const int8_t *>(B.ptr[ta]), reinterpret_cast<int8_t *>(B.ptr[tz]),
                                (size_t)d0 * B.images, (int)ch, qq, s);
                    return 0;
                };
                break;
            }
            case 23: {
                int32_t pads[8];
                std::memcpy(pads, P.q(o.b), sizeof(pads));
                uint32_t ad[4], zd[4];
                for (int d = 0; d < 4; d++) ad[d] = a.d[d], zd[d] = z.d[d];
                const int8_t value = (int8_t)(int32_t)o.p[0];
                const uint32_t ta = o.a, tz = o.out;
                st.run = [=](const BatchCtx &B, cudaStream_t s) -> int {
                    launch_pad(B.ptr[ta], B.ptr[tz], (int)B.images, ad, zd, pads, value, s);
                    return 0;
                };
                break;
            }
            case 22: {
                if (skip_[i]) {  // applied by the concat that alone reads its output
                    st.run = nullptr;
                    break;
                }
                const uint8_t *table = dconst(o.b);
                const unsigned flip = a.type == 3 ? 128u : 0u;
                if (lut_src_[i].tensor >= 0) {  // slice of the innermost axis + table in one pass
                    const LutSrc ls = lut_src_[i];
                    const uint32_t tz = o.out;
                    st.run = [=](const BatchCtx &B, cudaStream_t s) -> int {
                        launch_lut_rows(B.ptr[ls.tensor], B.ptr[tz], (size_t)ls.rows * B.images, ls.in_w, ls.off, ls.out_w,
                                        table, flip, s);
                        return 0;
                    };
                    break;
                }
                const uint32_t ta = o.a, tz = o.out, ab = a.bytes;
                st.run = [=](const BatchCtx &B, cudaStream_t s) -> int {
                    launch_lut(B.ptr[ta], B.ptr[tz], (size_t)ab * B.images, table, flip, s);
                    return 0;
                };
                break;
            }
            case 21: {
                const uint32_t *offsets = reinterpret_cast<const uint32_t *>(dconst(o.b));
                const uint32_t ta = o.a, tz = o.out;
                const int n = (int)a.d[0], ih = (int)a.d[1], iw = (int)a.d[2], c = (int)a.d[3], oh = (int)z.d[1],
                          ow = (int)z.d[2];
                st.run = [=](const BatchCtx &B, cudaStream_t s) -> int {
                    launch_resize(B.ptr[ta], B.ptr[tz], n * (int)B.images, ih, iw, c, oh, ow, offsets, s);
                    return 0;
                };
                break;
            }
            case 20: {
                if (skip_[i]) {  // collapsed into the concat that consumes it
                    st.run = nullptr;
                    break;
                }
                if (!concat_parts_[i].empty()) {
                    const std::vector<ConcatPart> parts = concat_parts_[i];
                    const std::vector<uint32_t> ins = concat_in_[i].empty() ? std::vector<uint32_t>{o.a, o.b} : concat_in_[i];
                    size_t rows = 1;
                    for (unsigned d = 0; d + 1 < z.rank; d++) rows *= z.d[d];
                    ConcatParts cp{};
                    cp.count = (int)parts.size();
                    for (size_t k = 0; k < parts.size(); k++) {
                        cp.in_w[k] = parts[k].in_w;
                        cp.off[k] = parts[k].off;
                        cp.out_w[k] = (uint32_t)(P.ts[ins[k]].bytes / rows);
                        if (parts[k].lut_op >= 0) {
                            const Op &l = P.ops[parts[k].lut_op];
                            cp.table[k] = dconst(l.b);
                            cp.flip[k] = P.ts[l.a].type == 3 ? 128u : 0u;
                        }
                    }
                    const uint32_t tz = o.out;
                    st.run = [=](const BatchCtx &B, cudaStream_t s) -> int {
                        ConcatParts c = cp;
                        for (size_t k = 0; k < parts.size(); k++) c.src[k] = B.ptr[parts[k].tensor];
                        launch_concat_parts(c, B.ptr[tz], rows * B.images, s);
                        return 0;
                    };
                    break;
                }
                if (!concat_in_[i].empty()) {
                    const std::vector<uint32_t> ins = concat_in_[i];
                    size_t rows = 1;
                    for (unsigned d = 0; d + 1 < a.rank; d++) rows *= a.d[d];
                    std::vector<uint32_t> widths;
                    for (uint32_t t : ins) widths.push_back((uint32_t)(P.ts[t].bytes / rows));
                    const uint32_t tz = o.out;
                    st.run = [=](const BatchCtx &B, cudaStream_t s) -> int {
                        ConcatInputs ci{};
                        ci.count = (int)ins.size();
                        for (size_t k = 0; k < ins.size(); k++) {
                            ci.src[k] = B.ptr[ins[k]];
                            ci.width[k] = widths[k];
                        }
                        launch_concat_multi(ci, B.ptr[tz], rows * B.images, s);
                        return 0;
                    };
                    break;
                }
                const unsigned axis = o.p[0];
                size_t outer = 1, inner = 1;
                for (unsigned d = 0; d < axis; d++) outer *= a.d[d];
                for (unsigned d = axis + 1; d < a.rank; d++) inner *= a.d[d];
                const size_t ac = a.d[axis] * inner, bc = b.d[axis] * inner;
                const uint32_t ta = o.a, tb = o.b, tz = o.out;
                st.run = [=](const BatchCtx &B, cudaStream_t s) -> int {
                    launch_concat(B.ptr[ta], B.ptr[tb], B.ptr[tz], outer * B.images, ac, bc, s);
                    return 0;
                };
                break;
            }
            case 19: {
                const uint32_t *list = reinterpret_cast<const uint32_t *>(P.bytes(o.b));
                std::vector<uint32_t> ids(list, list + b.bytes / 4);
                const uint32_t tz = o.out, zb = z.bytes;
                std::vector<uint32_t> sizes, offs;
                uint32_t off = 0;
                for (uint32_t id : ids) {
                    sizes.push_back(P.ts[id].bytes);
                    offs.push_back(off);
                    off += P.ts[id].bytes;
                }
                st.run = [=](const BatchCtx &B, cudaStream_t s) -> int {
                    Segments sg{};
                    sg.count = (int)ids.size();
                    for (size_t j = 0; j < ids.size(); j++) {
                        sg.src[j] = B.ptr[ids[j]];
                        sg.bytes[j] = sizes[j];
                        sg.dst_offset[j] = offs[j];
                    }
                    launch_pack(sg, B.ptr[tz], zb, (int)B.images, s);
                    return 0;
                };
                break;
            }
            case 18: {
                if (fused_[i]) {  // computed in the previous conv's epilogue
                    st.run = nullptr;
                    break;
                }
                const int32_t *dq = reinterpret_cast<const int32_t *>(dconst(o.p[0]));
                const uint32_t ta = o.a, tb = o.b, tz = o.out, zb = z.bytes;
                st.run = [=](const BatchCtx &B, cudaStream_t s) -> int {
                    launch_add(reinterpret_cast<const int8_t *>(B.ptr[ta]), reinterpret_cast<const int8_t *>(B.ptr[tb]),
                               reinterpret_cast<int8_t *>(B.ptr[tz]), (size_t)zb * B.images, dq, s);
                    return 0;
                };
                break;
            }
            case 10: {
                Shape5 in{};
                in.rank = (int)a.rank + 1;
                in.d[0] = 1;
                int perm[5] = {0, 0, 0, 0, 0};
                for (uint32_t d = 0; d < a.rank; d++) {
                    in.d[d + 1] = a.d[d];
                    perm[d + 1] = (int)o.p[d] + 1;
                }
                const int elem = (int)type_width(a.type);
                const uint32_t ta = o.a, tz = o.out;
                st.run = [=](const BatchCtx &B, cudaStream_t s) -> int {
                    Shape5 ib = in;
                    ib.d[0] = B.images;
                    launch_permute(B.ptr[ta], B.ptr[tz], ib, perm, elem, s);
                    return 0;
                };
                break;
            }
            default:
                // Legacy fp32 / MatMulInteger opcodes (1-4, 6-9, 11-13) are outside the INT8
                // vision path this backend implements.
                set_error("opcode " + std::to_string(o.code) + " is not implemented by the CUDA backend");
                return 19;
        }
        steps_.push_back(std::move(st));
    }
    return 0;
}

// ----------------------------------------------------------------------------------------
// Batched arena: storage groups (copy aliases share one group) placed by lifetime. A group
// lives from its first producer to its last reader; groups whose lifetimes intersect never
// share bytes. Constants read as activations are replicated per image once, up front.
// Byte-op fusion at load time (no change to any result):
//  * a concat (code 20) along the innermost axis whose first input is another such concat, read by
//    nothing else, absorbs it: one pass writes all the inputs (YOLO's C2f concat chains);
//  * a table (code 22) whose input is a slice (code 26) of the innermost axis, read by nothing
//    else, reads the slice's source in place.
// The skipped op's inputs are then read later than the plan says, so their lifetimes (death_) are
// extended for the arena planner.
void Engine::fuse_byte_ops() {
    const Plan &P = P_;
    const uint32_t nt = P.h.nt, no = P.h.no;
    std::vector<int> prod(nt, -1), uses(nt, 0);
    for (uint32_t i = 0; i < no; i++) {
        const Op &o = P.ops[i];
        prod[o.out] = (int)i;
        uses[o.a]++;
        if (o.code == 18 || o.code == 20 || o.code == 25 || o.code == 27) uses[o.b]++;
        if (o.code == 19) {
            const uint32_t *list = reinterpret_cast<const uint32_t *>(P.bytes(o.b));
            for (uint32_t j = 0; j < P.ts[o.b].bytes / 4; j++) uses[list[j]]++;
        }
    }
    uses[P.h.output]++;
    auto rows_of = [&](const Tensor &t) {
        size_t r = 1;
        for (uint32_t d = 0; d + 1 < t.rank; d++) r *= t.d[d];
        return r;
    };
    for (uint32_t i = 0; i < no; i++) {
        const Op &o = P.ops[i];
        const Tensor &a = P.ts[o.a];
        const int j = prod[o.a];
        if (j < 0 || uses[o.a] != 1 || o.a == P.h.output || P.ts[o.a].flags) continue;
        const Op &pj = P.ops[j];
        if (o.code == 20 && a.rank >= 1 && o.p[0] + 1 == a.rank && pj.code == 20 && pj.p[0] + 1 == a.rank &&
            P.ts[pj.a].rank == a.rank) {
            std::vector<uint32_t> list = concat_in_[j].empty() ? std::vector<uint32_t>{pj.a, pj.b} : concat_in_[j];
            list.push_back(o.b);
            const size_t rows = rows_of(a);
            bool ok = list.size() <= 8 && rows > 0;
            for (uint32_t t : list) ok = ok && rows_of(P.ts[t]) == rows && P.ts[t].bytes % rows == 0;
            if (!ok) continue;
            skip_[j] = 1;
            concat_in_[j].clear();
            concat_in_[i] = list;
            for (uint32_t t : list) death_[t] = std::max(death_[t], (int)i);
        } else if (o.code == 22 && pj.code == 26) {
            const Tensor &src = P.ts[pj.a], &sl = P.ts[pj.out];
            if (src.rank != sl.rank || src.rank < 1 || src.rank > 4 || src.type != sl.type) continue;
            bool inner = true;
            for (uint32_t d = 0; d + 1 < src.rank; d++) inner = inner && pj.p[d] == 0 && sl.d[d] == src.d[d];
            const size_t rows = rows_of(src);
            if (!inner || rows == 0 || src.bytes % rows || sl.bytes % rows) continue;
            const uint32_t in_w = (uint32_t)(src.bytes / rows), out_w = (uint32_t)(sl.bytes / rows);
            const uint32_t esize = in_w / src.d[src.rank - 1];
            if (esize * src.d[src.rank - 1] != in_w) continue;
            LutSrc ls;
            ls.tensor = (int)pj.a;
            ls.rows = (uint32_t)rows;
            ls.in_w = in_w;
            ls.off = pj.p[src.rank - 1] * esize;
            ls.out_w = out_w;
            if (ls.off + out_w > in_w) continue;
            lut_src_[i] = ls;
            skip_[j] = 1;
            death_[pj.a] = std::max(death_[pj.a], (int)i);
        }
    }
    // Tables folded into the concats that alone read them (YOLO's C2f blocks: the concat of the
    // activated halves of a split): the concat reads each table's source and maps its bytes.
    for (uint32_t i = 0; i < no; i++) {
        const Op &o = P.ops[i];
        if (o.code != 20 || skip_[i]) continue;
        const Tensor &z = P.ts[o.out];
        if (z.rank < 1 || o.p[0] + 1 != z.rank) continue;
        const std::vector<uint32_t> list = concat_in_[i].empty() ? std::vector<uint32_t>{o.a, o.b} : concat_in_[i];
        const size_t rows = rows_of(z);
        if (rows == 0 || list.size() > 8) continue;
        bool ok = true;
        for (uint32_t t : list) ok = ok && rows_of(P.ts[t]) == rows && P.ts[t].bytes % rows == 0;
        if (!ok) continue;
        std::vector<ConcatPart> parts;
        bool any = false;
        for (uint32_t t : list) {
            ConcatPart part;
            part.tensor = t;
            part.in_w = (uint32_t)(P.ts[t].bytes / rows);
            const int j = prod[t];
            if (j >= 0 && P.ops[j].code == 22 && !skip_[j] && uses[t] == 1 && t != P.h.output && !P.ts[t].flags) {
                const Op &l = P.ops[j];
                if (lut_src_[j].tensor >= 0 && lut_src_[j].rows == rows) {
                    part.tensor = (uint32_t)lut_src_[j].tensor;
                    part.in_w = lut_src_[j].in_w;
                    part.off = lut_src_[j].off;
                    part.lut_op = j;
                } else if (lut_src_[j].tensor < 0 && P.ts[l.a].bytes == P.ts[t].bytes) {
                    part.tensor = l.a;
                    part.lut_op = j;
                }
                if (part.lut_op >= 0) {
                    skip_[j] = 1;
                    death_[part.tensor] = std::max(death_[part.tensor], (int)i);
                    any = true;
                }
            }
            parts.push_back(part);
        }
        if (any) concat_parts_[i] = parts;
    }
}

int Engine::plan_arena(BatchCtx &B) {
    std::vector<size_t> offset;
    std::vector<uint32_t> replicated;
    size_t total = 0;
    layout(B.images, offset, replicated, total);
    const Plan &P = P_;
    const uint32_t nt = P.h.nt;
    B.arena_bytes = std::max<size_t>(total, kAlign);
    UQ_CUDA(cudaMalloc(&B.arena, B.arena_bytes));
    B.ptr.assign(nt, nullptr);
    for (uint32_t t = 0; t < nt; t++)
        B.ptr[t] = offset[t] != kNoOffset ? B.arena + offset[t] : d_const_ + P.ts[t].offset;
    for (uint32_t r : replicated) {
        const size_t bytes = P.ts[r].bytes;
        for (uint32_t i = 0; i < B.images; i++)
            UQ_CUDA(cudaMemcpyAsync(B.ptr[r] + i * bytes, d_const_ + P.ts[r].offset, bytes, cudaMemcpyDeviceToDevice,
                                    stream_));
    }
    UQ_CUDA(cudaStreamSynchronize(stream_));
    return 0;
}

// Arena layout for `images` images (host only): offset[t] of every tensor stored in the arena
// (kNoOffset for constants read in place), the replicated constants and the total bytes.
void Engine::layout(uint32_t images, std::vector<size_t> &offset, std::vector<uint32_t> &replicated,
                    size_t &total_out) const {
    const Plan &P = P_;
    const uint32_t nt = P.h.nt;
    std::vector<int> root(nt);
    for (uint32_t t = 0; t < nt; t++) {
        int r = (int)t;
        while (alias_[r] != r) r = alias_[r];
        root[t] = r;
    }
    // Constants used as activation operands need per-image copies.
    std::vector<uint8_t> replicate(nt, 0);
    auto mark = [&](uint32_t t) {
        if (P.ts[t].flags) replicate[root[t]] = 1;
    };
    for (const Op &o : P.ops) {
        mark(o.a);
        if (o.code == 18 || o.code == 20 || o.code == 25 || o.code == 27) mark(o.b);
        if (o.code == 19) {
            const uint32_t *list = reinterpret_cast<const uint32_t *>(P.bytes(o.b));
            for (uint32_t j = 0; j < P.ts[o.b].bytes / 4; j++) mark(list[j]);
        }
    }
    mark(P.h.output);
    struct Group {
        int root;
        size_t size;
        int birth, death;
        size_t offset;
    };
    std::vector<int> gid(nt, -1);
    std::vector<Group> groups;
    for (uint32_t t = 0; t < nt; t++) {
        const int r = root[t];
        const bool is_const = P.ts[r].flags != 0;
        if (is_const && !replicate[r]) continue;
        if (gid[r] < 0) {
            gid[r] = (int)groups.size();
            groups.push_back({r, align_up((size_t)P.ts[r].bytes * images, kAlign), is_const ? -1 : birth_[r],
                              is_const ? (int)P.h.no : death_[r], 0});
        }
        Group &g = groups[gid[r]];
        if (!is_const) {
            g.birth = std::min(g.birth, birth_[t]);
            g.death = std::max(g.death, death_[t]);
        }
        gid[t] = gid[r];
    }
    // The input tensor's bytes stay untouched for the whole step: a device-resident batch is
    // uploaded once and may be launched again (ug_launch_batch, ug_time_batch), so no later
    // tensor may reuse its storage after its last reader.
    if (gid[root[P.h.input]] >= 0) groups[gid[root[P.h.input]]].death = (int)P.h.no;
    std::vector<int> order(groups.size());
    std::iota(order.begin(), order.end(), 0);
    std::sort(order.begin(), order.end(), [&](int x, int y) { return groups[x].size > groups[y].size; });
    std::vector<int> placed;
    size_t total = 0;
    for (int gi : order) {
        Group &g = groups[gi];
        std::vector<std::pair<size_t, size_t>> busy;
        for (int pj : placed) {
            const Group &h = groups[pj];
            if (g.birth <= h.death && h.birth <= g.death) busy.push_back({h.offset, h.offset + h.size});
        }
        std::sort(busy.begin(), busy.end());
        size_t off = 0;
        for (auto &iv : busy) {
            if (off + g.size <= iv.first) break;
            off = std::max(off, iv.second);
        }
        g.offset = off;
        total = std::max(total, off + g.size);
        placed.push_back(gi);
    }
    offset.assign(nt, kNoOffset);
    for (uint32_t t = 0; t < nt; t++)
        if (gid[t] >= 0) offset[t] = groups[gid[t]].offset;
    replicated.clear();
    for (const Group &g : groups)
        if (P.ts[g.root].flags) replicated.push_back((uint32_t)g.root);
    total_out = total;
}

int Engine::run_steps(const BatchCtx &B, cudaStream_t s, bool profile) {
    std::vector<cudaEvent_t> evs;
    if (profile) {
        evs.resize(steps_.size() + 1);
        for (auto &e : evs) UQ_CUDA(cudaEventCreate(&e));
        UQ_CUDA(cudaEventRecord(evs[0], s));
    }
    for (size_t i = 0; i < steps_.size(); i++) {
        if (steps_[i].run) {
            const int rc = steps_[i].run(B, s);
            if (rc) {
                set_error("launch of op " + std::to_string(steps_[i].op) + " failed");
                return rc;
            }
        }
        if (profile) UQ_CUDA(cudaEventRecord(evs[i + 1], s));
    }
    cudaError_t e = cudaGetLastError();
    if (e != cudaSuccess) {
        set_error(std::string("kernel launch: ") + cudaGetErrorString(e));
        return 2001;
    }
    if (profile) {
        UQ_CUDA(cudaEventSynchronize(evs.back()));
        for (size_t i = 0; i < steps_.size(); i++) {
            float ms = 0.f;
            UQ_CUDA(cudaEventElapsedTime(&ms, evs[i], evs[i + 1]));
            ticks_[2 + steps_[i].op] += (uint64_t)(ms * 1e6);
        }
        float total = 0.f;
        UQ_CUDA(cudaEventElapsedTime(&total, evs[0], evs.back()));
        ticks_[0] += 1;
        ticks_[1] += (uint64_t)(total * 1e6);
        for (auto &ev : evs) cudaEventDestroy(ev);
        return device_status();
    }
    return 0;
}

int Engine::capture(BatchCtx &B) {
    UQ_CUDA(cudaStreamBeginCapture(stream_, cudaStreamCaptureModeThreadLocal));
    int rc = run_steps(B, stream_, false);
    cudaGraph_t g = nullptr;
    cudaError_t e = cudaStreamEndCapture(stream_, &g);
    if (rc) {
        if (g) cudaGraphDestroy(g);
        return rc;
    }
    if (e != cudaSuccess) {
        set_error(std::string("graph capture: ") + cudaGetErrorString(e));
        return 2001;
    }
    B.graph = g;
    UQ_CUDA(cudaGraphInstantiate(&B.exec, g, 0));
    size_t n = 0;
    UQ_CUDA(cudaGraphGetNodes(g, nullptr, &n));
    std::vector<cudaGraphNode_t> nodes(n);
    UQ_CUDA(cudaGraphGetNodes(g, nodes.data(), &n));
    int kernels = 0;
    for (auto nd : nodes) {
        cudaGraphNodeType ty;
        UQ_CUDA(cudaGraphNodeGetType(nd, &ty));
        kernels += ty == cudaGraphNodeTypeKernel;
    }
    B.kernel_nodes = kernels;
    return 0;
}

int Engine::batch(uint32_t images, BatchCtx **out, uint32_t slot) {
    if (!ready_) return 22;
    if (!images) return 22;
    const uint64_t key = (uint64_t)slot << 32 | images;
    auto it = batches_.find(key);
    if (it != batches_.end()) {
        *out = it->second.get();
        return 0;
    }
    UQ_CUDA(cudaSetDevice(device_));
    auto B = std::make_unique<BatchCtx>();
    B->images = images;
    int rc = plan_arena(*B);
    if (!rc) rc = capture(*B);
    if (rc) {
        if (B->exec) cudaGraphExecDestroy(B->exec);
        if (B->graph) cudaGraphDestroy(B->graph);
        if (B->arena) cudaFree(B->arena);
        return rc;
    }
    *out = B.get();
    batches_[key] = std::move(B);
    return 0;
}

int Engine::run_host(const void *in, void *out, uint32_t images) { return run_batch_host(in, out, images, 0); }

int Engine::run_batch_host(const void *in, void *out, uint32_t images, uint32_t k) {
    if (!ready_ || !in || !out) return 22;
    if (k && !yolo_.levels) return 22;
    // Large batches overlap their copies with compute, in pieces (run_pipelined).
    if (!profiling_ && images >= 512)
        return run_pipelined(static_cast<const uint8_t *>(in), static_cast<uint8_t *>(out), images, k);
    BatchCtx *B = nullptr;
    int rc = batch(images, &B);
    if (!rc) rc = stage_buffers(*B, k != 0);
    if (rc) return rc;
    UQ_CUDA(cudaSetDevice(device_));
    const size_t ni = (size_t)input_bytes() * images, no = (size_t)output_bytes() * images;
    UQ_CUDA(cudaEventRecord(ev0_, stream_));
    UQ_CUDA(cudaMemcpyAsync(landing(*B), in, ni, cudaMemcpyHostToDevice, stream_));
    if ((rc = stage_in(*B, stream_))) return rc;
    if (profiling_) rc = run_steps(*B, stream_, true);
    else if (cudaGraphLaunch(B->exec, stream_) != cudaSuccess) {
        set_error("graph launch failed");
        rc = 2001;
    }
    if (rc) return rc;
    if (k) {
        if ((rc = stage_out(*B, k, stream_))) return rc;
        UQ_CUDA(cudaMemcpyAsync(out, B->records, sizeof(UgDetectionRecord) * k * images, cudaMemcpyDeviceToHost,
                                stream_));
    } else {
        if ((rc = gather(*B))) return rc;
        if (gather_ && gather_->active()) {
            // rank 0 returns the whole gathered batch (rank-major); the other ranks return nothing
            if (gather_->rank() == 0)
                UQ_CUDA(cudaMemcpyAsync(out, gather_->root_buffer(no), no * (size_t)gather_->world(),
                                        cudaMemcpyDeviceToHost, stream_));
        } else {
            UQ_CUDA(cudaMemcpyAsync(out, B->ptr[P_.h.output], no, cudaMemcpyDeviceToHost, stream_));
        }
    }
    UQ_CUDA(cudaEventRecord(ev1_, stream_));
    if ((rc = finish(ev1_))) return rc;
    UQ_CUDA(cudaEventElapsedTime(&last_ms_, ev0_, ev1_));
    last_images_ = images;
    last_ctx_ = B;
    return device_status();
}

int Engine::run_pipelined(const uint8_t *in, uint8_t *out, uint32_t images, uint32_t k) {
    // Piece sizes grow geometrically: the first is small (1/16 of the batch, 64 to 256 images), so
    // compute starts after a short upload, and each next piece is `growth` times the previous, so
    // that its upload still fits inside the previous piece's compute while the later, larger pieces
    // run at close to whole-batch efficiency (a 512-image MobileNetV4 graph runs about 17% slower
    // per image than a 4096-image one: tail waves and launch gaps). The growth is the ratio of
    // compute to upload time per image measured on the previous call's largest piece (1.25 at
    // first; 2.7 for YOLO26n). A call whose compute per image, beyond each piece's fixed cost, is
    // below its upload per image (MobileNetV4) takes the copy-bound schedule instead (equal pieces
    // near the break-even size: pipeline_pieces, learn_pieces). Once the session has joined a multi-GPU
    // output gather the factor stays at its initial value on every rank (see pipeline_growth). At
    // most kMaxPieces; a small remainder joins the last piece. UNOQ_PIPE_GROWTH fixes the factor
    // (below 1: the copy-bound schedule).
    static const double fixed_growth = [] {
        const char *env = std::getenv("UNOQ_PIPE_GROWTH");
        const double g = env ? std::atof(env) : 0.0;
        return g > 0.0 && g <= 4.0 ? g : 0.0;
    }();
    const bool joined = gather_ && gather_->active();
    const size_t ni = input_bytes(), no = k ? sizeof(UgDetectionRecord) * k : output_bytes();
    PieceModel model = joined || fixed_growth > 0.0 ? PieceModel() : pipe_model_;
    model.down = model.up * (double)no / (double)ni;  // this call's outputs, over the same link
    std::vector<uint32_t> sizes = pipeline_pieces(images, pipeline_growth(joined, pipe_growth_, fixed_growth), model);
    // A planned schedule replaces this batch size's previous one only when the model predicts it
    // ends 2% sooner: timing noise then does not switch schedules call after call, each switch
    // capturing graphs and planning arenas for piece sizes not seen before.
    if (model.up > 0.0) {
        const auto prev = pipe_plan_.find(images);
        if (prev != pipe_plan_.end() && pipeline_end(prev->second, model) <= 1.02 * pipeline_end(sizes, model))
            sizes = prev->second;
        pipe_plan_[images] = sizes;
    }
    // one batch context per piece (slot p + 1): no arena is refilled within a call
    std::vector<BatchCtx *> ctx(sizes.size(), nullptr);
    int rc = 0;
    for (size_t p = 0; p < sizes.size() && !rc; p++) {
        rc = batch(sizes[p], &ctx[p], (uint32_t)p + 1);
        if (!rc) rc = stage_buffers(*ctx[p], k != 0);
    }
    if (rc) return rc;
    UQ_CUDA(cudaSetDevice(device_));
    const bool gathering = !k && joined;
    uint8_t *root = gathering ? gather_->root_buffer(no * images) : nullptr;
    if (gathering && gather_->rank() == 0 && !root) return 1002;
    // every stream starts after the work already queued on the compute stream
    UQ_CUDA(cudaEventRecord(ev0_, stream_));
    UQ_CUDA(cudaStreamWaitEvent(h2d_, ev0_, 0));
    UQ_CUDA(cudaStreamWaitEvent(d2h_, ev0_, 0));
    size_t off = 0;
    // the upload and compute of the largest piece are timed (one of the equal pieces of a
    // copy-bound schedule, the last of a growing one), and the compute of the smallest: they pick
    // the next call's schedule (learn_pieces)
    const size_t timed_piece = (size_t)(std::max_element(sizes.begin(), sizes.end()) - sizes.begin());
    const size_t small_piece = (size_t)(std::min_element(sizes.begin(), sizes.end()) - sizes.begin());
    const bool two_sizes = sizes[small_piece] < sizes[timed_piece];
    for (size_t piece = 0; piece < sizes.size(); piece++) {
        const int s = (int)(piece & 1);
        BatchCtx *B = ctx[piece];
        const size_t n = sizes[piece];
        const bool timed = piece == timed_piece && sizes.size() > 1;
        if (timed) UQ_CUDA(cudaEventRecord(pipe_t_[0], h2d_));
        UQ_CUDA(cudaMemcpyAsync(landing(*B), in + off * ni, n * ni, cudaMemcpyHostToDevice, h2d_));
        UQ_CUDA(cudaEventRecord(pipe_ev_[0][s], h2d_));
        if (timed) UQ_CUDA(cudaEventRecord(pipe_t_[1], h2d_));
        UQ_CUDA(cudaStreamWaitEvent(stream_, pipe_ev_[0][s], 0));
        const bool small = two_sizes && piece == small_piece;
        if (timed) UQ_CUDA(cudaEventRecord(pipe_t_[2], stream_));
        if (small) UQ_CUDA(cudaEventRecord(pipe_t_[4], stream_));
        if ((rc = stage_in(*B, stream_))) return rc;
        if (cudaGraphLaunch(B->exec, stream_) != cudaSuccess) {
            set_error("graph launch failed");
            return 2001;
        }
        if (timed) UQ_CUDA(cudaEventRecord(pipe_t_[3], stream_));
        if (small) UQ_CUDA(cudaEventRecord(pipe_t_[5], stream_));
        if (k && (rc = stage_out(*B, k, stream_))) return rc;
        if (gathering && (rc = gather_->enqueue(B->ptr[P_.h.output], n * no, no * images, off * no, stream_)))
            return rc;
        UQ_CUDA(cudaEventRecord(pipe_ev_[1][s], stream_));
        UQ_CUDA(cudaStreamWaitEvent(d2h_, pipe_ev_[1][s], 0));
        if (!gathering) {
            const void *src = k ? static_cast<const void *>(B->records) : B->ptr[P_.h.output];
            UQ_CUDA(cudaMemcpyAsync(out + off * no, src, n * no, cudaMemcpyDeviceToHost, d2h_));
        } else if (gather_->rank() == 0) {
            // rank-major result: rank r's images occupy [r * images, (r + 1) * images)
            for (int r = 0; r < gather_->world(); r++) {
                const size_t at = ((size_t)r * images + off) * no;
                UQ_CUDA(cudaMemcpyAsync(out + at, root + at, n * no, cudaMemcpyDeviceToHost, d2h_));
            }
        }
        UQ_CUDA(cudaEventRecord(pipe_ev_[2][s], d2h_));
        off += n;
    }
    UQ_CUDA(cudaEventRecord(ev1_, d2h_));
    UQ_CUDA(cudaStreamWaitEvent(stream_, ev1_, 0));
    if ((rc = finish(ev1_))) return rc;
    UQ_CUDA(cudaEventElapsedTime(&last_ms_, ev0_, ev1_));
    last_images_ = images;
    last_ctx_ = ctx.back();
    // Learn the schedule (learn_pieces) from this process's own timing only while the session has
    // no output gather (pipeline_growth ignores it afterwards anyway): per-rank timings differ.
    if (sizes.size() > 1 && !joined) {
        float up = 0.f, comp = 0.f, comp_s = 0.f;
        if (cudaEventElapsedTime(&up, pipe_t_[0], pipe_t_[1]) == cudaSuccess &&
            cudaEventElapsedTime(&comp, pipe_t_[2], pipe_t_[3]) == cudaSuccess && up > 0.f && comp > 0.f) {
            if (!two_sizes || cudaEventElapsedTime(&comp_s, pipe_t_[4], pipe_t_[5]) != cudaSuccess) comp_s = 0.f;
            const PieceChoice next = learn_pieces(pipe_growth_, sizes[timed_piece], up, comp,
                                                  two_sizes ? sizes[small_piece] : 0, comp_s);
            pipe_growth_ = next.growth;
            pipe_model_ = next.model;
        }
    }
    return device_status();
}

int Engine::run_mailbox(const void *in, void *out) {
    if (!ready_ || !in || !out) return 22;
    // profiling runs op by op, and a gathered session returns every rank's outputs: both take
    // the ordinary path
    if (profiling_ || (gather_ && gather_->active())) return run_host(in, out, 1);
    UQ_CUDA(cudaSetDevice(device_));
    const size_t ni = input_bytes(), no = output_bytes();
    if (!mb_exec_) {
        BatchCtx *B = nullptr;
        int rc = batch(1, &B);
        if (!rc) rc = stage_buffers(*B, false);
        if (rc) return rc;
        UQ_CUDA(cudaHostAlloc(&mb_in_, ni, cudaHostAllocDefault));
        UQ_CUDA(cudaHostAlloc(&mb_out_, no, cudaHostAllocDefault));
        UQ_CUDA(cudaStreamBeginCapture(stream_, cudaStreamCaptureModeThreadLocal));
        cudaMemcpyAsync(landing(*B), mb_in_, ni, cudaMemcpyHostToDevice, stream_);
        rc = stage_in(*B, stream_);
        if (!rc) rc = run_steps(*B, stream_, false);
        cudaMemcpyAsync(mb_out_, B->ptr[P_.h.output], no, cudaMemcpyDeviceToHost, stream_);
        cudaGraph_t g = nullptr;
        const cudaError_t e = cudaStreamEndCapture(stream_, &g);
        if (rc || e != cudaSuccess) {
            if (g) cudaGraphDestroy(g);
            drop_mailbox();
            if (!rc) set_error(std::string("mailbox capture: ") + cudaGetErrorString(e));
            return rc ? rc : 2001;
        }
        mb_graph_ = g;
        if (cudaGraphInstantiate(&mb_exec_, g, 0) != cudaSuccess) {
            drop_mailbox();
            set_error("mailbox graph instantiation failed");
            return 2001;
        }
        last_ctx_ = B;
    }
    std::memcpy(mb_in_, in, ni);
    UQ_CUDA(cudaEventRecord(ev0_, stream_));
    UQ_CUDA(cudaGraphLaunch(mb_exec_, stream_));
    UQ_CUDA(cudaEventRecord(ev1_, stream_));
    // bounded like the reference's mailbox response (bridge.c:172-183): 4 s, then 1006
    const auto t0 = std::chrono::steady_clock::now();
    cudaError_t q;
    while ((q = cudaEventQuery(ev1_)) == cudaErrorNotReady) {
        if (std::chrono::steady_clock::now() - t0 > std::chrono::seconds(4)) {
            set_error("mailbox response timed out");
            return 1006;
        }
        std::this_thread::yield();
    }
    if (q != cudaSuccess) {
        set_error(std::string("mailbox run: ") + cudaGetErrorString(q));
        return 2001;
    }
    UQ_CUDA(cudaEventElapsedTime(&last_ms_, ev0_, ev1_));
    last_images_ = 1;
    const int rc = device_status();
    if (rc) return rc;
    std::memcpy(out, mb_out_, no);
    return 0;
}

// Fixed device arena of the allocation-free entry point (ug_run_static): the reference's own
// arena bound (runtime/graph.h:7). Nothing in it needs to start at zero: every activation is
// written before it is read, and replicated constants are copied in at every call.
static __device__ __align__(256) uint8_t g_static_arena[kStaticArenaBytes];

int Engine::run_static(const void *in, void *out) {
    if (!ready_ || !in || !out) return 22;
    UQ_CUDA(cudaSetDevice(device_));
    if (!static_.arena) {
        // set-up, once per engine: host-side layout and the arena's device address; no allocation
        std::vector<size_t> offset;
        size_t total = 0;
        layout(1, offset, static_replicated_, total);
        if (total > kStaticArenaBytes) {
            set_error("plan needs " + std::to_string(total) + " bytes of activation arena; the static arena holds " +
                      std::to_string(kStaticArenaBytes));
            return 20;
        }
        void *base = nullptr;
        UQ_CUDA(cudaGetSymbolAddress(&base, g_static_arena));
        static_.images = 1;
        static_.arena_bytes = kStaticArenaBytes;
        static_.ptr.assign(P_.h.nt, nullptr);
        for (uint32_t t = 0; t < P_.h.nt; t++)
            static_.ptr[t] = offset[t] != kNoOffset ? static_cast<uint8_t *>(base) + offset[t] : d_const_ + P_.ts[t].offset;
        static_.arena = static_cast<uint8_t *>(base);
    }
    for (uint32_t r : static_replicated_)
        UQ_CUDA(cudaMemcpyAsync(static_.ptr[r], d_const_ + P_.ts[r].offset, P_.ts[r].bytes, cudaMemcpyDeviceToDevice,
                                stream_));
    UQ_CUDA(cudaMemcpyAsync(static_.ptr[P_.h.input], in, input_bytes(), cudaMemcpyHostToDevice, stream_));
    int rc = run_steps(static_, stream_, false);
    if (rc) return rc;
    UQ_CUDA(cudaMemcpyAsync(out, static_.ptr[P_.h.output], output_bytes(), cudaMemcpyDeviceToHost, stream_));
    const cudaError_t e = cudaStreamSynchronize(stream_);
    if (e != cudaSuccess) {
        set_error(std::string("inference: ") + cudaGetErrorString(e));
        return 2001;
    }
    last_ctx_ = &static_;
    last_images_ = 1;
    return device_status();
}

int Engine::run_device(const void *in, void *out, uint32_t images) {
    if (!ready_ || !in || !out || !images) return 22;
    BatchCtx B;
    B.images = images;
    B.ptr.assign(P_.h.nt, nullptr);
    for (uint32_t t = 0; t < P_.h.nt; t++) {
        if (t == P_.h.input) B.ptr[t] = static_cast<uint8_t *>(const_cast<void *>(in));
        else if (t == P_.h.output) B.ptr[t] = static_cast<uint8_t *>(out);
        else if (P_.ts[t].flags) B.ptr[t] = d_const_ + P_.ts[t].offset;
        else return 22;
    }
    UQ_CUDA(cudaSetDevice(device_));
    int rc = run_steps(B, stream_, false);
    if (rc) return rc;
    const cudaError_t e = cudaStreamSynchronize(stream_);
    if (e != cudaSuccess) {
        set_error(std::string("operator run: ") + cudaGetErrorString(e));
        return 2001;
    }
    return device_status();
}

// A device-side wait that gave up (bounded mbarrier waits in the tensor-core kernels) leaves a
// code in device memory; report it as 2003 and clear it.
int Engine::device_status() {
    int code = conv_tc_error(true);
    if (!code) code = conv_rows_error(true);
    if (!code) code = conv_taps_error(true);
    if (!code) code = dw_tc_error(true);
    if (code) {
        set_error("device wait timed out in the tensor-core conv (site " + std::to_string(code) + ")");
        return 2003;
    }
    return 0;
}

int Engine::buffers(uint32_t images, void **d_in, void **d_out) {
    BatchCtx *B = nullptr;
    int rc = batch(images, &B);
    if (!rc) rc = stage_buffers(*B, false);
    if (rc) return rc;
    if (d_in) *d_in = landing(*B);
    if (d_out) *d_out = B->ptr[P_.h.output];
    return 0;
}

int Engine::launch(uint32_t images) {
    BatchCtx *B = nullptr;
    int rc = batch(images, &B);
    if (rc) return rc;
    if ((rc = stage_buffers(*B, false))) return rc;
    UQ_CUDA(cudaSetDevice(device_));
    if ((rc = stage_in(*B, stream_))) return rc;
    UQ_CUDA(cudaGraphLaunch(B->exec, stream_));
    last_images_ = images;
    last_ctx_ = B;
    return gather(*B);
}

int Engine::upload(const void *in, uint32_t images) {
    BatchCtx *B = nullptr;
    int rc = batch(images, &B);
    if (!rc) rc = stage_buffers(*B, false);
    if (rc) return rc;
    UQ_CUDA(cudaSetDevice(device_));
    UQ_CUDA(cudaMemcpyAsync(landing(*B), in, (size_t)input_bytes() * images, cudaMemcpyHostToDevice, stream_));
    UQ_CUDA(cudaStreamSynchronize(stream_));
    return 0;
}

int Engine::download(void *out, uint32_t images) {
    BatchCtx *B = nullptr;
    int rc = batch(images, &B);
    if (rc) return rc;
    UQ_CUDA(cudaSetDevice(device_));
    UQ_CUDA(cudaMemcpyAsync(out, B->ptr[P_.h.output], (size_t)output_bytes() * images, cudaMemcpyDeviceToHost,
                            stream_));
    UQ_CUDA(cudaStreamSynchronize(stream_));
    return device_status();
}

int Engine::synchronize() {
    if (!stream_) return 22;
    UQ_CUDA(cudaSetDevice(device_));
    UQ_CUDA(cudaStreamSynchronize(stream_));
    return device_status();
}

int Engine::time_launches(uint32_t images, uint32_t iterations, float *ms) {
    BatchCtx *B = nullptr;
    int rc = batch(images, &B);
    if (!rc) rc = stage_buffers(*B, false);
    if (rc) return rc;
    UQ_CUDA(cudaSetDevice(device_));
    UQ_CUDA(cudaStreamSynchronize(stream_));
    UQ_CUDA(cudaEventRecord(ev0_, stream_));
    for (uint32_t i = 0; i < iterations; i++) {
        if ((rc = stage_in(*B, stream_))) return rc;
        UQ_CUDA(cudaGraphLaunch(B->exec, stream_));
        if ((rc = gather(*B))) return rc;
    }
    UQ_CUDA(cudaEventRecord(ev1_, stream_));
    if ((rc = finish(ev1_))) return rc;
    UQ_CUDA(cudaEventElapsedTime(ms, ev0_, ev1_));
    last_images_ = images;
    last_ctx_ = B;
    return device_status();
}

int Engine::stage_buffers(BatchCtx &b, bool records) {
    if (table_channels_ && !b.pixels) UQ_CUDA(cudaMalloc(&b.pixels, (size_t)input_bytes() * b.images));
    if (records && !b.records)
        UQ_CUDA(cudaMalloc(&b.records, sizeof(UgDetectionRecord) * kMaxDetections * b.images));
    return 0;
}

int Engine::stage_in(const BatchCtx &b, cudaStream_t s) {
    if (!table_channels_) return 0;
    launch_pixel_table(b.pixels, reinterpret_cast<int8_t *>(b.ptr[P_.h.input]), (size_t)input_bytes() * b.images,
                       d_table_, table_channels_, s);
    const cudaError_t e = cudaGetLastError();
    if (e != cudaSuccess) {
        set_error(std::string("input table launch: ") + cudaGetErrorString(e));
        return 2001;
    }
    return 0;
}

int Engine::stage_out(const BatchCtx &b, uint32_t k, cudaStream_t s) {
    launch_yolo_topk(reinterpret_cast<const int8_t *>(b.ptr[P_.h.output]), output_bytes(), b.images, d_yolo_, yolo_, k,
                     b.records, s);
    const cudaError_t e = cudaGetLastError();
    if (e != cudaSuccess) {
        set_error(std::string("decoder launch: ") + cudaGetErrorString(e));
        return 2001;
    }
    return 0;
}

int Engine::set_input_table(const void *table, uint32_t channels) {
    if (!ready_) return 22;
    UQ_CUDA(cudaSetDevice(device_));
    UQ_CUDA(cudaStreamSynchronize(stream_));
    drop_mailbox();  // its graph lands the input through the old table setting
    if (!table || !channels) {
        table_channels_ = 0;
        return 0;
    }
    if (channels > kMaxTableChannels || input_bytes() % channels) {
        set_error("input table: channels must be 1.." + std::to_string(kMaxTableChannels) +
                  " and divide the input tensor's bytes");
        return 22;
    }
    if (!d_table_) UQ_CUDA(cudaMalloc(&d_table_, 256 * kMaxTableChannels));
    UQ_CUDA(cudaMemcpy(d_table_, table, 256 * (size_t)channels, cudaMemcpyHostToDevice));
    table_channels_ = channels;
    return 0;
}

int Engine::set_yolo_decode(const UgYoloDecode *d) {
    if (!ready_) return 22;
    UQ_CUDA(cudaSetDevice(device_));
    UQ_CUDA(cudaStreamSynchronize(stream_));
    if (!d) {
        yolo_ = YoloShape();
        return 0;
    }
    auto bad = [](const std::string &why) {
        set_error("YOLO decoder: " + why);
        return 22;
    };
    if (d->levels < 1 || d->levels > UG_YOLO_MAX_LEVELS) return bad("levels must be 1..4");
    if (d->classes < 1 || d->classes > 4096) return bad("classes must be 1..4096");
    if (d->candidates < 1 || d->candidates > kMaxDetections) return bad("candidates must be 1..512");
    if (d->reserved) return bad("reserved field must be 0");
    const uint64_t ob = output_bytes();
    uint64_t anchors = 0;
    bool vec = d->classes % 16 == 0;
    for (uint32_t l = 0; l < d->levels; l++) {
        const UgYoloLevel &v = d->level[l];
        const uint64_t cells = (uint64_t)v.height * v.width;
        if (!cells) return bad("empty grid");
        if ((uint64_t)v.box_offset + cells * 4 > ob || (uint64_t)v.score_offset + cells * d->classes > ob)
            return bad("level " + std::to_string(l) + " lies outside the output tensor");
        if (!std::isfinite(v.stride) || !(v.stride > 0.f)) return bad("stride must be finite and positive");
        for (int q = 0; q < 256; q++)
            if (v.rank[q] >= kRankCodes) return bad("order codes must be below 1024");
        vec = vec && v.score_offset % 16 == 0;
        anchors += cells;
    }
    if (anchors > kMaxAnchors) return bad("more than 32768 anchors");
    if (!d_yolo_) UQ_CUDA(cudaMalloc(&d_yolo_, sizeof(UgYoloDecode)));
    UQ_CUDA(cudaMemcpy(d_yolo_, d, sizeof(UgYoloDecode), cudaMemcpyHostToDevice));
    yolo_.levels = d->levels;
    yolo_.classes = d->classes;
    yolo_.anchors = (uint32_t)anchors;
    yolo_.candidates = d->candidates;
    yolo_.vec = vec;
    return 0;
}

int Engine::detect_host(const void *in, uint32_t images, uint32_t k, void *records) {
    if (!yolo_.levels || !k || k > kMaxDetections) return 22;
    return run_batch_host(in, records, images, k);
}

int Engine::launch_detect(uint32_t images, uint32_t k) {
    if (!yolo_.levels || !k || k > kMaxDetections) return 22;
    BatchCtx *B = nullptr;
    int rc = batch(images, &B);
    if (!rc) rc = stage_buffers(*B, true);
    if (rc) return rc;
    UQ_CUDA(cudaSetDevice(device_));
    if ((rc = stage_in(*B, stream_))) return rc;
    UQ_CUDA(cudaGraphLaunch(B->exec, stream_));
    last_images_ = images;
    last_ctx_ = B;
    return stage_out(*B, k, stream_);
}

int Engine::detect_buffer(uint32_t images, uint32_t k, void **records) {
    if (!yolo_.levels || !k || k > kMaxDetections || !records) return 22;
    BatchCtx *B = nullptr;
    int rc = batch(images, &B);
    if (!rc) rc = stage_buffers(*B, true);
    if (rc) return rc;
    *records = B->records;
    return 0;
}

int Engine::gather(const BatchCtx &b) {
    if (!gather_ || !gather_->active()) return 0;
    const size_t bytes = (size_t)output_bytes() * b.images;
    return gather_->enqueue(b.ptr[P_.h.output], bytes, bytes, 0, stream_);
}

int Engine::finish(cudaEvent_t ev) {
    if (gather_ && gather_->active()) {
        const int rc = gather_->wait(ev, 60.0);
        if (rc) return rc;
    } else {
        const cudaError_t e = cudaEventSynchronize(ev);
        if (e != cudaSuccess) {
            set_error(std::string("inference: ") + cudaGetErrorString(e));
            return 2001;
        }
    }
    return 0;
}

int Engine::dist_init(int rank, int world, const void *id, uint32_t bytes) {
    if (!ready_) return 22;
    if (gather_) return 1003;
    auto g = std::make_unique<OutputGather>();
    const int rc = g->init(device_, rank, world, id, bytes);
    if (rc) return rc;
    gather_ = std::move(g);
    pipe_growth_ = kInitialPieceGrowth;  // nothing learned alone carries over into gathered calls
    return 0;
}

int Engine::time_gather(uint32_t images, uint32_t iterations, float *ms) {
    if (!ms || !iterations) return 22;
    if (!gather_ || !gather_->active()) return 22;
    BatchCtx *B = nullptr;
    int rc = batch(images, &B);
    if (rc) return rc;
    UQ_CUDA(cudaSetDevice(device_));
    UQ_CUDA(cudaStreamSynchronize(stream_));
    // one untimed gather first: it completes only once every rank has joined, so the timed ones
    // start with the ranks in step rather than measuring a late rank's arrival
    if ((rc = gather(*B))) return rc;
    UQ_CUDA(cudaEventRecord(ev0_, stream_));
    for (uint32_t i = 0; i < iterations; i++)
        if ((rc = gather(*B))) return rc;
    UQ_CUDA(cudaEventRecord(ev1_, stream_));
    if ((rc = finish(ev1_))) return rc;
    UQ_CUDA(cudaEventElapsedTime(ms, ev0_, ev1_));
    return 0;
}

int Engine::gather_buffer(uint32_t images, void **root) {
    if (!root) return 1003;
    *root = nullptr;
    if (!gather_ || !gather_->active()) return 22;
    UQ_CUDA(cudaSetDevice(device_));
    *root = gather_->root_buffer((size_t)output_bytes() * images);
    return gather_->rank() != 0 || *root ? 0 : 1002;
}

int Engine::kernel_count(uint32_t images) {
    BatchCtx *B = nullptr;
    int rc = batch(images, &B);
    if (rc) return -rc;
    return B->kernel_nodes + (table_channels_ ? 1 : 0);
}

int Engine::snapshot(uint32_t tensor, void *out, uint32_t bytes) {
    if (!ready_ || tensor >= P_.h.nt || !out || bytes != P_.ts[tensor].bytes) return 22;
    // The tensor as the last run left it: the last image of the context that ran last (the static
    // arena after ug_run_static, the last piece of a pipelined batch). Per-image tensors live in
    // the context's arena, one copy per image; constants read in place have a single copy.
    const uint8_t *src = d_const_ + P_.ts[tensor].offset;
    if (last_ctx_ && !last_ctx_->ptr.empty()) {
        const BatchCtx &B = *last_ctx_;
        src = B.ptr[tensor];
        if (src >= B.arena && src < B.arena + B.arena_bytes) src += (size_t)(B.images - 1) * bytes;
    }
    UQ_CUDA(cudaSetDevice(device_));
    UQ_CUDA(cudaStreamSynchronize(stream_));
    UQ_CUDA(cudaMemcpy(out, src, bytes, cudaMemcpyDeviceToHost));
    return 0;
}

int Engine::profile_batch(uint32_t images, uint32_t iterations, uint64_t *op_ns, uint32_t n, float *total_ms) {
    BatchCtx *B = nullptr;
    int rc = batch(images, &B);
    if (rc) return rc;
    if (!op_ns || n < P_.h.no) return 22;
    UQ_CUDA(cudaSetDevice(device_));
    std::vector<uint64_t> saved = ticks_;
    std::fill(ticks_.begin(), ticks_.end(), 0);
    for (uint32_t it = 0; it < iterations && !rc; it++) rc = run_steps(*B, stream_, true);
    if (!rc) {
        for (uint32_t i = 0; i < P_.h.no; i++) op_ns[i] = ticks_[2 + i];
        if (total_ms) *total_ms = (float)(ticks_[1] / 1e6);
    }
    ticks_ = saved;
    return rc;
}

int Engine::profile(uint32_t command, void *out, uint32_t bytes) {
    if (!ready_ || command > 2 || !out ||
        (bytes != (kMaxOps + 2) * sizeof(uint64_t) && !(P_.h.no <= 128 && bytes == 130 * 8)))
        return 22;
    if (command == 1) std::fill(ticks_.begin(), ticks_.end(), 0);
    if (command < 2) profiling_ = command == 1;
    std::memcpy(out, ticks_.data(), bytes);
    return 0;
}

}  // namespace uq
