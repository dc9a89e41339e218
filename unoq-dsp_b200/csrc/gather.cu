// gather.cu -- OutputGather: NCCL point-to-point gather of per-rank outputs to rank 0.
#include "gather.hpp"

#include <dlfcn.h>
#include <nccl.h>

#include <chrono>
#include <cstring>
#include <mutex>
#include <string>
#include <thread>
#include <type_traits>

#include "engine.hpp"

namespace uq {

namespace {

// NCCL is resolved at first use with dlopen("libnccl.so.2") rather than linked: a process that
// already loaded an NCCL (PyTorch bundles its own) then shares that one, and loading this library
// never pins an NCCL version that a later import would conflict with. nccl.h supplies the types.
struct NcclApi {
    bool ok = false;
    decltype(&::ncclGetUniqueId) GetUniqueId = nullptr;
    decltype(&::ncclCommInitRankConfig) CommInitRankConfig = nullptr;
    decltype(&::ncclCommGetAsyncError) CommGetAsyncError = nullptr;
    decltype(&::ncclCommFinalize) CommFinalize = nullptr;
    decltype(&::ncclCommDestroy) CommDestroy = nullptr;
    decltype(&::ncclCommAbort) CommAbort = nullptr;
    decltype(&::ncclGroupStart) GroupStart = nullptr;
    decltype(&::ncclGroupEnd) GroupEnd = nullptr;
    decltype(&::ncclSend) Send = nullptr;
    decltype(&::ncclRecv) Recv = nullptr;
    decltype(&::ncclGetErrorString) GetErrorString = nullptr;
};

const NcclApi &nccl() {
    static NcclApi api;
    static std::once_flag once;
    std::call_once(once, [] {
        void *h = dlopen("libnccl.so.2", RTLD_NOW | RTLD_LOCAL);
        if (!h) h = dlopen("libnccl.so", RTLD_NOW | RTLD_LOCAL);
        if (!h) return;
        bool all = true;
        auto get = [&](auto &fn, const char *name) {
            fn = reinterpret_cast<std::remove_reference_t<decltype(fn)>>(dlsym(h, name));
            all &= fn != nullptr;
        };
        get(api.GetUniqueId, "ncclGetUniqueId");
        get(api.CommInitRankConfig, "ncclCommInitRankConfig");
        get(api.CommGetAsyncError, "ncclCommGetAsyncError");
        get(api.CommFinalize, "ncclCommFinalize");
        get(api.CommDestroy, "ncclCommDestroy");
        get(api.CommAbort, "ncclCommAbort");
        get(api.GroupStart, "ncclGroupStart");
        get(api.GroupEnd, "ncclGroupEnd");
        get(api.Send, "ncclSend");
        get(api.Recv, "ncclRecv");
        get(api.GetErrorString, "ncclGetErrorString");
        api.ok = all;
    });
    return api;
}

constexpr double kInitSeconds = 120.0;

// Poll a non-blocking communicator until its pending work is enqueued (or it failed).
ncclResult_t settle(ncclComm_t comm, double seconds) {
    const auto start = std::chrono::steady_clock::now();
    ncclResult_t state = ncclInProgress;
    while (true) {
        if (nccl().CommGetAsyncError(comm, &state) != ncclSuccess) return ncclSystemError;
        if (state != ncclInProgress) return state;
        if (std::chrono::duration<double>(std::chrono::steady_clock::now() - start).count() > seconds)
            return ncclInProgress;
        std::this_thread::sleep_for(std::chrono::microseconds(50));
    }
}

int fail(const std::string &what, ncclResult_t r) {
    const char *why = r == ncclInProgress ? "timed out" : nccl().ok ? nccl().GetErrorString(r) : "libnccl.so.2 not found";
    set_error("collective: " + what + ": " + why);
    return kCollectiveError;
}

}  // namespace

int collective_unique_id(void *out, uint32_t bytes) {
    if (!out || bytes < sizeof(ncclUniqueId)) return 1003;
    if (!nccl().ok) return fail("load", ncclSystemError);
    ncclUniqueId id;
    const ncclResult_t r = nccl().GetUniqueId(&id);
    if (r != ncclSuccess) return fail("unique id", r);
    std::memcpy(out, &id, sizeof(id));
    return 0;
}

OutputGather::~OutputGather() {
    if (comm_) {
        cudaSetDevice(device_);
        ncclComm_t c = static_cast<ncclComm_t>(comm_);
        if (nccl().CommFinalize(c) == ncclSuccess && settle(c, 10.0) == ncclSuccess) nccl().CommDestroy(c);
        else nccl().CommAbort(c);
    }
    if (root_) cudaFree(root_);
}

int OutputGather::init(int device, int rank, int world, const void *id, uint32_t bytes) {
    if (comm_ || world < 1 || rank < 0 || rank >= world || !id || bytes < sizeof(ncclUniqueId)) return 1003;
    device_ = device;
    rank_ = rank;
    world_ = world;
    if (world == 1) return 0;
    if (!nccl().ok) return fail("load", ncclSystemError);
    if (cudaSetDevice(device) != cudaSuccess) return 2001;
    ncclUniqueId uid;
    std::memcpy(&uid, id, sizeof(uid));
    ncclConfig_t config = NCCL_CONFIG_INITIALIZER;
    config.blocking = 0;
    ncclComm_t comm = nullptr;
    ncclResult_t r = nccl().CommInitRankConfig(&comm, world, uid, rank, &config);
    if (r != ncclSuccess && r != ncclInProgress) return fail("init", r);
    r = settle(comm, kInitSeconds);
    if (r != ncclSuccess) {
        nccl().CommAbort(comm);
        return fail("init", r);
    }
    comm_ = comm;
    return 0;
}

uint8_t *OutputGather::root_buffer(size_t rank_bytes) {
    if (rank_ != 0) return nullptr;
    const size_t need = rank_bytes * (size_t)world_;
    if (need > root_bytes_) {
        if (root_) cudaFree(root_);
        root_ = nullptr;
        root_bytes_ = 0;
        if (cudaMalloc(&root_, need) != cudaSuccess) return nullptr;
        root_bytes_ = need;
    }
    return root_;
}

int OutputGather::enqueue(const void *src, size_t bytes, size_t rank_bytes, size_t offset, cudaStream_t s) {
    if (!active()) return 0;
    if (offset + bytes > rank_bytes) return 1003;
    ncclComm_t comm = static_cast<ncclComm_t>(comm_);
    uint8_t *dst = root_buffer(rank_bytes);
    if (rank_ == 0 && !dst) {
        set_error("collective: root buffer allocation failed");
        return 1002;
    }
    auto ok = [](ncclResult_t v) { return v == ncclSuccess || v == ncclInProgress; };
    ncclResult_t r = nccl().GroupStart();
    if (ok(r) && rank_ == 0)
        for (int peer = 0; peer < world_ && ok(r); peer++)
            r = nccl().Recv(dst + (size_t)peer * rank_bytes + offset, bytes, ncclInt8, peer, comm, s);
    if (ok(r)) r = nccl().Send(src, bytes, ncclInt8, 0, comm, s);
    const ncclResult_t e = nccl().GroupEnd();
    if (!ok(r)) return fail("send/recv", r);
    if (!ok(e)) return fail("group", e);
    r = settle(comm, 30.0);
    return r == ncclSuccess ? 0 : fail("enqueue", r);
}

int OutputGather::wait(cudaEvent_t ev, double seconds) {
    const auto start = std::chrono::steady_clock::now();
    while (true) {
        const cudaError_t q = cudaEventQuery(ev);
        if (q == cudaSuccess) return 0;
        if (q != cudaErrorNotReady) {
            set_error(std::string("collective wait: ") + cudaGetErrorString(q));
            return 2001;
        }
        if (active()) {
            ncclResult_t state = ncclSuccess;
            nccl().CommGetAsyncError(static_cast<ncclComm_t>(comm_), &state);
            if (state != ncclSuccess && state != ncclInProgress) {
                nccl().CommAbort(static_cast<ncclComm_t>(comm_));
                comm_ = nullptr;
                return fail("transfer", state);
            }
        }
        if (std::chrono::duration<double>(std::chrono::steady_clock::now() - start).count() > seconds) {
            if (active()) {
                nccl().CommAbort(static_cast<ncclComm_t>(comm_));
                comm_ = nullptr;
            }
            return fail("completion", ncclInProgress);
        }
        std::this_thread::sleep_for(std::chrono::microseconds(20));
    }
}

}  // namespace uq
