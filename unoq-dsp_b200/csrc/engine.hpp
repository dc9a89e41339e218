// engine.hpp -- device-side executor of one loaded plan.
//
// Replaces the reference's run_inner dispatch loop (runtime/graph.c:285-423) and its static
// 16 MiB arena. Constants are uploaded once; activations live in a per-batch-size device
// arena laid out by a lifetime planner (each activation tensor holds `images` back-to-back
// copies of its batch-1 layout); the op sequence for a batch size is captured once into a
// CUDA graph and replayed.
#pragma once
#include <cuda_runtime.h>

#include <functional>
#include <map>
#include <memory>
#include <string>
#include <vector>

#include "decode.cuh"
#include "gather.hpp"
#include "plan.hpp"

namespace uq {

constexpr size_t kStaticArenaBytes = (size_t)16 << 20;  // fixed arena of run_static (runtime/graph.h:7)
constexpr size_t kNoOffset = ~(size_t)0;

// Piece schedule of a pipelined host batch (Engine::run_pipelined), host-only and pure so that
// every rank of a gathered run can be shown to cut the same pieces. With a timing model of the
// session's last call (learn_pieces; never for a gathered session) the schedule is the one of
// least simulated end time (planned_pieces). Without one:
//  * growth >= 1 (compute-bound calls): the first piece is 1/16 of the batch (64 to 256 images);
//    each next one is `growth` times the previous; at most kMaxPieces; a remainder under half a
//    piece joins the last one.
//  * growth < 1 (kCopyBoundPieces: copy-bound calls, compute per image below upload per image): a
//    first piece of kCopyBoundFirst images (a quarter of a smaller batch), then equal pieces of
//    about kCopyBoundPiece (at most kMaxPieces in all).
// Why equal pieces when copy-bound: the host-to-device copies run back to back, and a piece's
// compute keeps pace with the next upload only if the upload time it frees (upload minus compute
// per image, times its images) covers the per-piece fixed cost of a graph launch. On MobileNetV4
// (0.28 ms per piece beside 1.93 against 2.73 us per image) that break-even is about 350 images:
// smaller pieces, such as a ramp down at the end of the batch, leave a backlog of compute after
// the last upload. When compute-bound (YOLO26n), pieces grow so that each upload hides under the
// previous compute, and a small closing piece shortens the last read-back of large outputs.
constexpr double kInitialPieceGrowth = 1.25;
constexpr double kCopyBoundPieces = 0.5;
constexpr uint32_t kCopyBoundFirst = 192, kCopyBoundPiece = 352;  // without a model
constexpr size_t kMaxPieces = 16;
// Per-piece timing of a pipelined call (ms): a graph takes fixed + slope * images, an upload
// up * images and the read-back of its outputs down * images. Valid when up > 0.
struct PieceModel {
    double fixed = 0.0, slope = 0.0, up = 0.0, down = 0.0;
};
// First piece `f`, then `m` equal pieces of the rest.
inline std::vector<uint32_t> first_then_equal(uint32_t images, uint32_t f, uint32_t m) {
    std::vector<uint32_t> sizes{f};
    const uint32_t rest = images - f;
    for (uint32_t i = 0; i < m; i++) sizes.push_back(rest / m + (i < rest % m ? 1 : 0));
    return sizes;
}
// Pieces from `f` images up, each `g` times the previous (a remainder under half a piece joins
// the last), then a closing piece of `tail` images (0: none); empty when that takes more than
// kMaxPieces.
inline std::vector<uint32_t> growing_pieces(uint32_t images, uint32_t f, double g, uint32_t tail) {
    std::vector<uint32_t> sizes;
    if (f < 1 || tail >= images) return sizes;
    uint32_t left = images - tail;
    double cur = f;
    while (left) {
        uint32_t n = left < (uint32_t)cur ? left : (uint32_t)cur;
        if (n < 1) n = 1;
        if (left - n < (uint32_t)(cur * 0.5)) n = left;
        sizes.push_back(n);
        left -= n;
        cur *= g;
        if (sizes.size() > kMaxPieces) return {};
    }
    if (tail) sizes.push_back(tail);
    if (sizes.size() > kMaxPieces) return {};
    return sizes;
}
// End time of a schedule under the model: uploads back to back, each graph after its upload and
// the previous graph, each read-back after its graph and the previous read-back.
inline double pipeline_end(const std::vector<uint32_t> &sizes, const PieceModel &pm) {
    double t_up = 0.0, t_c = 0.0, t_d = 0.0;
    for (uint32_t n : sizes) {
        t_up += pm.up * n;
        t_c = (t_c > t_up ? t_c : t_up) + pm.fixed + pm.slope * n;
        t_d = (t_d > t_c ? t_d : t_c) + pm.down * n;
    }
    return t_d;
}
// The schedule of least simulated end time among a first piece then equal pieces, and growing
// pieces with an optional small closing piece (which shortens the last read-back); empty when
// the model is not valid or the batch is under 128 images.
inline std::vector<uint32_t> planned_pieces(uint32_t images, const PieceModel &pm) {
    std::vector<uint32_t> best_s;
    if (!(pm.up > 0.0) || images < 128) return best_s;
    double best = 0.0;
    auto consider = [&](std::vector<uint32_t> s) {
        if (s.empty()) return;
        const double e = pipeline_end(s, pm);
        if (best_s.empty() || e < best - 1e-9) best = e, best_s = std::move(s);
    };
    for (uint32_t f : {32u, 64u, 96u, 128u, 192u, 256u}) {
        if (2 * f > images) break;
        for (uint32_t m = 1; m < kMaxPieces && m <= (images - f) / 32; m++) consider(first_then_equal(images, f, m));
        for (double g : {1.2, 1.4, 1.6, 1.8, 2.0, 2.4, 2.8, 3.2})
            for (uint32_t tail : {0u, 32u, 64u, 128u})
                if (tail * 4 <= images) consider(growing_pieces(images, f, g, tail));
    }
    return best_s;
}
inline std::vector<uint32_t> pipeline_pieces(uint32_t images, double growth, const PieceModel &pm = PieceModel()) {
    std::vector<uint32_t> sizes = planned_pieces(images, pm);
    if (!sizes.empty()) return sizes;
    if (growth < 1.0) {
        const uint32_t f = images / 4 < kCopyBoundFirst ? images / 4 : kCopyBoundFirst;
        if (f >= 64) {
            const uint32_t rest = images - f;
            uint32_t m = (rest + kCopyBoundPiece / 2) / kCopyBoundPiece;
            if (m < 1) m = 1;
            if (m > kMaxPieces - 1) m = (uint32_t)kMaxPieces - 1;
            return first_then_equal(images, f, m);
        }
        growth = kInitialPieceGrowth;  // too few images to split
    }
    uint32_t left = images;
    double cur = images / 16.0 < 64.0 ? 64.0 : images / 16.0 > 256.0 ? 256.0 : images / 16.0;
    while (left) {
        uint32_t n = left < (uint32_t)cur ? left : (uint32_t)cur;
        if (left - n < (uint32_t)(cur * 0.5) || sizes.size() + 1 == kMaxPieces) n = left;
        sizes.push_back(n);
        left -= n;
        cur *= growth;
    }
    return sizes;
}
// The growth a call uses (below 1: the copy-bound schedule). `fixed` (UNOQ_PIPE_GROWTH, 0 when unset)
// wins. A session that has joined
// an output gather always uses the initial factor: each piece enqueues one gather step, so every
// rank must cut identical pieces, whatever it measured on calls made before joining or on
// calls that gather nothing (decoder calls). Otherwise the factor learned from the last call.
inline double pipeline_growth(bool gather_joined, double learned, double fixed) {
    if (fixed > 0) return fixed;
    return gather_joined ? kInitialPieceGrowth : learned;
}

// The next call's schedule, learned from two pieces of the last one: the largest (`n_l` images,
// upload `up` ms, graph `comp` ms) and the smallest (`n_s` images, graph `comp_s` ms; n_s = 0 when
// the pieces were all alike). A graph's time is a fixed cost per piece plus a cost per image, the
// slope between the two pieces. Compute per image below upload per image (10% below to enter,
// not above to stay) takes the copy-bound schedule, planned on that model (no model without a
// slope). Otherwise pieces grow by 1.1 x the ratio of compute to upload time of the largest
// piece, within [1.15, 3]. Judging by the largest piece alone would take a small batch's small
// pieces, whose fixed cost inflates their compute, for compute-bound (MobileNetV4 at 512 and
// 1,024 images).
struct PieceChoice {
    double growth;
    PieceModel model;
};
inline PieceChoice learn_pieces(double prev_growth, uint32_t n_l, float up, float comp, uint32_t n_s, float comp_s) {
    const double up1 = (double)up / n_l;
    double slope = (double)comp / n_l, fixed = 0.0;
    if (n_s > 0 && n_s < n_l && comp_s > 0.f) {
        const double sl = ((double)comp - comp_s) / (double)(n_l - n_s);
        if (sl > 0.0) {
            slope = sl;
            fixed = (double)comp - sl * n_l;
            if (fixed < 0.0) fixed = 0.0;
        }
    }
    const double margin = prev_growth < 1.0 ? 1.0 : 0.9;
    PieceModel pm;
    if (fixed > 0.0) pm.fixed = fixed, pm.slope = slope, pm.up = up1;
    if (slope < margin * up1) return {kCopyBoundPieces, pm};
    const double g = 1.1 * comp / up;
    return {g < 1.15 ? 1.15 : g > 3.0 ? 3.0 : g, pm};
}

struct BatchCtx;

// One plan op lowered to device work. `run` enqueues its kernels on the stream and returns 0
// or an error code.
struct Step {
    uint32_t op = 0;
    std::function<int(const BatchCtx &, cudaStream_t)> run;
};

struct BatchCtx {
    uint32_t images = 0;
    uint8_t *arena = nullptr;            // device activation arena
    size_t arena_bytes = 0;
    std::vector<uint8_t *> ptr;          // device address of each tensor (image 0)
    cudaGraph_t graph = nullptr;
    cudaGraphExec_t exec = nullptr;
    int kernel_nodes = 0;
    uint8_t *host_in = nullptr, *host_out = nullptr;  // pinned staging for pageable callers
    uint8_t *pixels = nullptr;           // uint8 input landing buffer while an input table is set
    UgDetectionRecord *records = nullptr;  // images x kMaxDetections decoder records
};

class Engine {
   public:
    Engine() = default;
    ~Engine();
    Engine(const Engine &) = delete;
    Engine &operator=(const Engine &) = delete;

    // Validate + prepare. Returns 0 or a reference loader code; 2001/2002 for CUDA failures.
    int load(const void *plan, uint32_t bytes, int device);
    bool ready() const { return ready_; }
    uint32_t input_bytes() const { return ready_ ? P_.ts[P_.h.input].bytes : 0; }
    uint32_t output_bytes() const { return ready_ ? P_.ts[P_.h.output].bytes : 0; }
    const Plan &plan() const { return P_; }
    int device() const { return device_; }
    cudaStream_t stream() const { return stream_; }

    // Host buffers; `pinned` skips the staging copy. Synchronous.
    int run_host(const void *in, void *out, uint32_t images);
    // One image through the session's mailbox (pipeline mode 1, runtime/bridge.c:161-184): a
    // resident CUDA graph that copies the pinned input slot in, runs the network and copies the
    // output into the pinned output slot, launched once per call. The wait for it is bounded by
    // 4 s (1006 on expiry, as the reference's mailbox response). Synchronous.
    int run_mailbox(const void *in, void *out);
    // One image through the fixed device arena g_static_arena (kStaticArenaBytes), with no device
    // allocation: eager launches on the engine stream, host buffers, synchronous. The first call
    // lays the plan out (host) and looks up the arena's address; calls that overlap on one device
    // share the arena and must be serialised by the caller.
    int run_static(const void *in, void *out);
    // Eager run over caller-owned device buffers: `in` / `out` hold `images` back-to-back copies of
    // the plan's input / output tensor. Only plans whose activations are exactly the input and the
    // output qualify (the one-op plans of the operator ABI); others get 22. Synchronous.
    int run_device(const void *in, void *out, uint32_t images);
    // Device buffers of the batch context (input tensor, output tensor of image 0).
    int buffers(uint32_t images, void **d_in, void **d_out);
    int launch(uint32_t images);   // async on stream_
    // Host <-> device-resident batch input/output (the context ug_launch_batch replays). Synchronous.
    int upload(const void *in, uint32_t images);
    int download(void *out, uint32_t images);
    int synchronize();
    int time_launches(uint32_t images, uint32_t iterations, float *ms);
    int kernel_count(uint32_t images);
    float last_ms() const { return last_ms_; }
    int snapshot(uint32_t tensor, void *out, uint32_t bytes);
    int profile(uint32_t command, void *out, uint32_t bytes);
    // Eager (non-graph) passes with a CUDA event after every op; accumulates per-op
    // nanoseconds into op_ns[0..no) and returns the summed pass time in *total_ms.
    int profile_batch(uint32_t images, uint32_t iterations, uint64_t *op_ns, uint32_t n, float *total_ms);
    // Multi-GPU: join the output gather of a `world`-rank batch-sharded run. From then on every
    // batch launch ends with the gather of this rank's outputs into rank 0's root buffer.
    int dist_init(int rank, int world, const void *id, uint32_t bytes);
    // Time `iterations` gathers alone of the batch context's outputs (every rank calls it; CUDA
    // events on the session stream, bounded wait); 22 when no gather has been joined.
    int time_gather(uint32_t images, uint32_t iterations, float *ms);
    int gather_buffer(uint32_t images, void **root);
    // On-device preparation and decoding (include/unoq_cuda.h). The table maps uploaded pixels to
    // the input tensor before the graph; the decoder turns the output tensor into k records.
    int set_input_table(const void *table, uint32_t channels);
    int set_yolo_decode(const UgYoloDecode *decode);
    int detect_host(const void *in, uint32_t images, uint32_t k, void *records);
    int launch_detect(uint32_t images, uint32_t k);
    int detect_buffer(uint32_t images, uint32_t k, void **records);

   private:
    int prepare();
    // Batch context for `images`; slot > 0 gives further contexts of the same size (own arena and
    // graph) for the copy/compute pipeline.
    int batch(uint32_t images, BatchCtx **out, uint32_t slot = 0);
    // Host batch in pieces of growing size: H2D of piece p+1, compute of piece p and D2H of piece
    // p-1 run concurrently on three streams, each piece in its own batch context.
    // k > 0: the output is k decoder records per image instead of the output tensor.
    int run_pipelined(const uint8_t *in, uint8_t *out, uint32_t images, uint32_t k = 0);
    int run_batch_host(const void *in, void *out, uint32_t images, uint32_t k);
    int stage_buffers(BatchCtx &b, bool records);
    uint8_t *landing(const BatchCtx &b) const { return table_channels_ ? b.pixels : b.ptr[P_.h.input]; }
    int stage_in(const BatchCtx &b, cudaStream_t s);              // pixel table, when set
    int stage_out(const BatchCtx &b, uint32_t k, cudaStream_t s); // YOLO decode into b.records
    int plan_arena(BatchCtx &b);
    void layout(uint32_t images, std::vector<size_t> &offset, std::vector<uint32_t> &replicated, size_t &total) const;
    int capture(BatchCtx &b);
    int run_steps(const BatchCtx &b, cudaStream_t s, bool profile);
    void release();
    int device_status();
    uint8_t *dconst(uint32_t tensor) const { return d_const_ + P_.ts[tensor].offset; }
    void *prep_alloc(size_t bytes);   // device memory owned by the engine for prepared data

    Plan P_;
    bool ready_ = false;
    int device_ = 0;
    cudaStream_t stream_ = nullptr;
    uint8_t *d_const_ = nullptr;
    std::vector<void *> prep_;
    std::vector<Step> steps_;
    std::vector<int> alias_;             // tensor -> storage root (copy ops alias their source)
    std::vector<int> birth_;             // tensor birth op, moved earlier for fused outputs
    std::vector<int> death_;             // tensor last-read op, moved later for fused byte ops
    // Byte-op fusion (fuse_byte_ops): ops computed by a later op, concat chains collapsed into their
    // last concat, and tables that read a slice's source directly.
    struct LutSrc {
        int tensor = -1;                 // the slice's source tensor (-1: not fused)
        uint32_t rows = 0, in_w = 0, off = 0, out_w = 0;
    };
    // A concat input whose producer is a table op read by nothing else: the concat reads the
    // table's source (a slice's source in place when the table read a slice) and applies it.
    struct ConcatPart {
        uint32_t tensor = 0;             // tensor read
        uint32_t in_w = 0, off = 0;      // its row width and this part's offset in it (bytes)
        int lut_op = -1;                 // table op folded into the part (-1: plain copy)
    };
    std::vector<char> skip_;
    std::vector<std::vector<uint32_t>> concat_in_;
    std::vector<std::vector<ConcatPart>> concat_parts_;
    std::vector<LutSrc> lut_src_;
    void fuse_byte_ops();
    std::vector<char> fused_;            // op computed inside the previous op's kernel
    bool fuse_adds_ = true;              // UNOQ_FUSE_ADD=0 keeps every add separate
    std::map<uint64_t, std::unique_ptr<BatchCtx>> batches_;  // key: slot << 32 | images
    cudaStream_t h2d_ = nullptr, d2h_ = nullptr;             // copy streams of the pipeline
    cudaEvent_t pipe_ev_[3][2] = {};                         // per slot: input landed, computed, output read
    cudaEvent_t ev0_ = nullptr, ev1_ = nullptr;
    cudaEvent_t pipe_t_[6] = {};         // largest piece: upload start / end, graph start / end; smallest: graph start / end
    double pipe_growth_ = kInitialPieceGrowth;  // piece schedule from the last call: growth, or kCopyBoundPieces
    PieceModel pipe_model_;                     // timing model of the last call (planned schedules)
    std::map<uint32_t, std::vector<uint32_t>> pipe_plan_;  // last planned schedule per batch size
    float last_ms_ = 0.f;
    uint32_t last_images_ = 0;
    const BatchCtx *last_ctx_ = nullptr; // context of the last run (a batch piece or the static arena)
    bool profiling_ = false;
    std::vector<uint64_t> ticks_;        // [0] runs, [1] total ns, [2+i] op ns
    std::unique_ptr<OutputGather> gather_;
    BatchCtx static_;                    // one-image context over g_static_arena (not owned)
    // mailbox mode: pinned input / output slots and the graph that runs one image between them
    uint8_t *mb_in_ = nullptr, *mb_out_ = nullptr;
    cudaGraph_t mb_graph_ = nullptr;
    cudaGraphExec_t mb_exec_ = nullptr;
    void drop_mailbox();
    std::vector<uint32_t> static_replicated_;
    int8_t *d_table_ = nullptr;          // [256][channels] input table (device)
    uint32_t table_channels_ = 0;        // 0: inputs are the int8 input tensor itself
    UgYoloDecode *d_yolo_ = nullptr;     // installed decoder (device)
    YoloShape yolo_;                     // its host-checked shape; levels == 0 when none
    int gather(const BatchCtx &b);       // enqueue the output gather when multi-rank
    int finish(cudaEvent_t ev);          // wait for `ev`, bounded when a collective is pending
};

// The CUDA device the C ABI works on: ug_set_device's choice, else UNOQ_CUDA_DEVICE, else 0.
int abi_device();

// Dense INT8 tensor-core throughput of that device (k_peak.cu): best of three launches of
// `iterations` MMA rounds per SM, in TOPS; *ms gets that launch's time.
int measure_int8_peak(uint32_t iterations, float *tops, float *ms);

// Records the last CUDA failure for ug_last_error().
void set_error(const std::string &msg);
const char *last_error();

}  // namespace uq
