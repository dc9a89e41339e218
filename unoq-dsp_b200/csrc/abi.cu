// abi.cu -- extern "C" entry points of libunoq_cuda.so (declared in include/unoq_cuda.h).
//
// Graph ABI (ug_load/ug_run/...) keeps the reference's process-global single graph
// (runtime/graph.c:4-8). Session ABI (ug_open_mode/ug_infer/...) keeps the reference bridge's
// one-active-session rule and error codes (runtime/bridge.c:99-185), with CUDA underneath.
#include <cuda_runtime.h>

#include <cstdlib>
#include <mutex>

#include "unoq_cuda.h"
#include "engine.hpp"

namespace {

std::mutex g_graph_mu;
uq::Engine *g_graph = nullptr;  // graph ABI engine
int g_device = -1;              // ug_set_device choice; -1 = UNOQ_CUDA_DEVICE env or 0

std::mutex g_session_mu;
bool g_session_active = false;

struct Session {
    uq::Engine engine;
    int pipeline = 0;
};

int pick_device() {
    if (g_device >= 0) return g_device;
    const char *env = std::getenv("UNOQ_CUDA_DEVICE");
    return env ? std::atoi(env) : 0;
}

}  // namespace

int uq::abi_device() { return pick_device(); }

extern "C" {

int ug_load(const void *plan, uint32_t bytes) {
    std::lock_guard<std::mutex> lk(g_graph_mu);
    if (!g_graph) g_graph = new uq::Engine();
    return g_graph->load(plan, bytes, pick_device());
}

int ug_run(const void *input, uint32_t input_bytes, void *output, uint32_t output_bytes) {
    std::lock_guard<std::mutex> lk(g_graph_mu);
    if (!g_graph || !g_graph->ready() || !input || !output || input_bytes != g_graph->input_bytes() ||
        output_bytes != g_graph->output_bytes())
        return 22;
    int rc = g_graph->run_host(input, output, 1);
    if (rc) {  // graph.c:298-305: any run error requires a reload
        delete g_graph;
        g_graph = nullptr;
    }
    return rc;
}

int ug_run_static(const void *input, uint32_t input_bytes, void *output, uint32_t output_bytes) {
    std::lock_guard<std::mutex> lk(g_graph_mu);
    if (!g_graph || !g_graph->ready() || !input || !output || input_bytes != g_graph->input_bytes() ||
        output_bytes != g_graph->output_bytes())
        return 22;
    const int rc = g_graph->run_static(input, output);
    if (rc && rc != 20) {  // as ug_run: a failed run requires a reload; an oversized plan just is refused
        delete g_graph;
        g_graph = nullptr;
    }
    return rc;
}

uint32_t ug_input_bytes(void) {
    std::lock_guard<std::mutex> lk(g_graph_mu);
    return g_graph ? g_graph->input_bytes() : 0;
}

uint32_t ug_output_bytes(void) {
    std::lock_guard<std::mutex> lk(g_graph_mu);
    return g_graph ? g_graph->output_bytes() : 0;
}

int ug_snapshot(uint32_t tensor, void *out, uint32_t bytes) {
    std::lock_guard<std::mutex> lk(g_graph_mu);
    return g_graph ? g_graph->snapshot(tensor, out, bytes) : 22;
}

int ug_profile(uint32_t command, void *out, uint32_t bytes) {
    std::lock_guard<std::mutex> lk(g_graph_mu);
    return g_graph ? g_graph->profile(command, out, bytes) : 22;
}

void *ug_open_mode(const void *plan, uint32_t bytes, int pipeline, int *error) {
    if (!error) return nullptr;
    *error = 1;  // bridge.c:100
    if (!plan || bytes > uq::kMaxPlan || pipeline < 0 || pipeline > 1) return nullptr;
    {
        std::lock_guard<std::mutex> lk(g_session_mu);
        if (g_session_active) {
            *error = 1001;
            return nullptr;
        }
        g_session_active = true;
    }
    Session *s = new (std::nothrow) Session();
    if (!s) {
        std::lock_guard<std::mutex> lk(g_session_mu);
        g_session_active = false;
        *error = 1002;
        return nullptr;
    }
    s->pipeline = pipeline;
    int rc = s->engine.load(plan, bytes, pick_device());
    if (rc) {
        delete s;
        std::lock_guard<std::mutex> lk(g_session_mu);
        g_session_active = false;
        *error = rc;
        return nullptr;
    }
    *error = 0;
    return s;
}

void *ug_open(const void *plan, uint32_t bytes, int *error) { return ug_open_mode(plan, bytes, 0, error); }

int ug_infer(void *session, const void *input, uint32_t input_bytes, void *output, uint32_t output_bytes) {
    Session *s = static_cast<Session *>(session);
    if (!s || !input || !output || input_bytes != s->engine.input_bytes() || output_bytes != s->engine.output_bytes())
        return 1003;  // bridge.c:149
    if (s->pipeline) return s->engine.run_mailbox(input, output);  // bridge.c:161-184
    return s->engine.run_host(input, output, 1);
}

void ug_close(void *session) {
    Session *s = static_cast<Session *>(session);
    if (!s) return;
    delete s;
    std::lock_guard<std::mutex> lk(g_session_mu);
    g_session_active = false;
}

int ug_snapshot_tensor(void *session, uint32_t tensor, void *out, uint32_t bytes) {
    Session *s = static_cast<Session *>(session);
    if (!s || s->pipeline || !out || !bytes || bytes > 4 * 1024 * 1024) return 1003;  // bridge.c:128
    int rc = s->engine.snapshot(tensor, out, bytes);
    return rc == 22 ? 1003 : rc;
}

int ug_profile_control(void *session, uint32_t command, void *out, uint32_t bytes) {
    Session *s = static_cast<Session *>(session);
    if (!s || !out || (bytes != 130 * 8 && bytes != (uq::kMaxOps + 2) * 8) || command > 2) return 1003;  // bridge.c:135
    return s->engine.profile(command, out, bytes);
}

int ug_set_device(int device) {
    int count = 0;
    if (cudaGetDeviceCount(&count) != cudaSuccess || device < 0 || device >= count) return 2002;
    g_device = device;
    return 0;
}

int ug_infer_batch(void *session, const void *input, uint32_t images, void *output) {
    Session *s = static_cast<Session *>(session);
    if (!s || !input || !output || !images) return 1003;
    return s->engine.run_host(input, output, images);
}

int ug_batch_buffers(void *session, uint32_t images, void **device_input, void **device_output) {
    Session *s = static_cast<Session *>(session);
    if (!s || !images) return 1003;
    return s->engine.buffers(images, device_input, device_output);
}

int ug_launch_batch(void *session, uint32_t images) {
    Session *s = static_cast<Session *>(session);
    if (!s || !images) return 1003;
    return s->engine.launch(images);
}

int ug_dist_unique_id(void *id, uint32_t bytes) { return uq::collective_unique_id(id, bytes); }

int ug_dist_init(void *session, int rank, int world, const void *id, uint32_t bytes) {
    Session *s = static_cast<Session *>(session);
    if (!s) return 1003;
    return s->engine.dist_init(rank, world, id, bytes);
}

int ug_time_gather(void *session, uint32_t images, uint32_t iterations, float *milliseconds) {
    Session *s = static_cast<Session *>(session);
    if (!s || !images || !iterations || !milliseconds) return 1003;
    return s->engine.time_gather(images, iterations, milliseconds);
}

int ug_gather_buffer(void *session, uint32_t images, void **root_device_output) {
    Session *s = static_cast<Session *>(session);
    if (!s || !images) return 1003;
    return s->engine.gather_buffer(images, root_device_output);
}

int ug_upload_batch(void *session, const void *input, uint32_t images) {
    Session *s = static_cast<Session *>(session);
    if (!s || !input || !images) return 1003;
    return s->engine.upload(input, images);
}

int ug_download_batch(void *session, void *output, uint32_t images) {
    Session *s = static_cast<Session *>(session);
    if (!s || !output || !images) return 1003;
    return s->engine.download(output, images);
}

int ug_synchronize(void *session) {
    Session *s = static_cast<Session *>(session);
    if (!s) return 1003;
    return s->engine.synchronize();
}

int ug_time_batch(void *session, uint32_t images, uint32_t iterations, float *milliseconds) {
    Session *s = static_cast<Session *>(session);
    if (!s || !images || !milliseconds) return 1003;
    return s->engine.time_launches(images, iterations, milliseconds);
}

float ug_last_infer_ms(void *session) {
    Session *s = static_cast<Session *>(session);
    return s ? s->engine.last_ms() : 0.f;
}

void *ug_host_alloc(size_t bytes) {
    void *p = nullptr;
    if (cudaHostAlloc(&p, bytes ? bytes : 1, cudaHostAllocPortable) != cudaSuccess) return nullptr;
    return p;
}

void ug_host_free(void *ptr) {
    if (ptr) cudaFreeHost(ptr);
}

int ug_validate_plan(const void *plan, uint32_t bytes) {
    uq::Plan p;
    return uq::parse_plan(plan, bytes, p);
}

int ug_batch_kernel_count(void *session, uint32_t images) {
    Session *s = static_cast<Session *>(session);
    if (!s || !images) return -1003;
    return s->engine.kernel_count(images);
}

int ug_profile_batch(void *session, uint32_t images, uint32_t iterations, uint64_t *op_ns, uint32_t count,
                     float *total_ms) {
    Session *s = static_cast<Session *>(session);
    if (!s || !images || !iterations) return 1003;
    return s->engine.profile_batch(images, iterations, op_ns, count, total_ms);
}

int ug_set_input_table(void *session, const void *table, uint32_t channels) {
    Session *s = static_cast<Session *>(session);
    if (!s) return 1003;
    const int rc = s->engine.set_input_table(table, channels);
    return rc == 22 ? 1003 : rc;
}

int ug_set_yolo_decode(void *session, const UgYoloDecode *decode) {
    Session *s = static_cast<Session *>(session);
    if (!s) return 1003;
    const int rc = s->engine.set_yolo_decode(decode);
    return rc == 22 ? 1003 : rc;
}

int ug_detect_batch(void *session, const void *input, uint32_t images, uint32_t k, UgDetectionRecord *records) {
    Session *s = static_cast<Session *>(session);
    if (!s || !input || !images || !records) return 1003;
    const int rc = s->engine.detect_host(input, images, k, records);
    return rc == 22 ? 1003 : rc;
}

int ug_launch_detect(void *session, uint32_t images, uint32_t k) {
    Session *s = static_cast<Session *>(session);
    if (!s || !images) return 1003;
    const int rc = s->engine.launch_detect(images, k);
    return rc == 22 ? 1003 : rc;
}

int ug_detect_buffer(void *session, uint32_t images, uint32_t k, void **device_records) {
    Session *s = static_cast<Session *>(session);
    if (!s || !images) return 1003;
    const int rc = s->engine.detect_buffer(images, k, device_records);
    return rc == 22 ? 1003 : rc;
}

int ug_measure_int8_peak(uint32_t iterations, float *tops, float *milliseconds) {
    std::lock_guard<std::mutex> lk(g_graph_mu);
    return uq::measure_int8_peak(iterations, tops, milliseconds);
}

const char *ug_last_error(void) { return uq::last_error(); }

}  // extern "C"
