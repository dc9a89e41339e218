// gather.hpp -- the one collective of a batch-sharded run: every rank's int8 outputs gathered
// into rank 0's device memory (NCCL point-to-point over NVLink/NVSwitch).
//
// Images are independent, so a multi-GPU run gives each GPU (one process each) a contiguous
// slice of the global batch and needs no exchange until the end. There, each rank sends its
// output tensor ([images][output_bytes], contiguous in its arena) to rank 0, which receives
// rank r's slice at offset r * slice_bytes, so the root buffer holds the global batch in order.
// The sends are enqueued on the session stream after the CUDA graph, inside the timed region.
//
// NCCL runs in non-blocking mode so that every wait here is bounded: initialisation and
// completion are polled with a limit, after which the communicator is aborted and the call
// returns 2004 (no rank waits forever on a peer that died).
#pragma once
#include <cuda_runtime.h>

#include <cstddef>
#include <cstdint>

namespace uq {

constexpr int kCollectiveError = 2004;

// NCCL unique id (128 bytes) for rank 0 to share with the other ranks out of band.
int collective_unique_id(void *out, uint32_t bytes);

class OutputGather {
   public:
    OutputGather() = default;
    ~OutputGather();
    OutputGather(const OutputGather &) = delete;
    OutputGather &operator=(const OutputGather &) = delete;

    // Join the communicator (all `world` ranks call this with the same id). Bounded.
    int init(int device, int rank, int world, const void *id, uint32_t bytes);
    bool active() const { return comm_ != nullptr && world_ > 1; }
    int rank() const { return rank_; }
    int world() const { return world_; }
    // Rank 0's receive buffer for `rank_bytes` per rank (grown on demand); null elsewhere.
    uint8_t *root_buffer(size_t rank_bytes);
    // Enqueue on stream `s` the gather of `bytes` at `src` from every rank; rank 0 receives rank
    // r's bytes at root + r * rank_bytes + offset (offset > 0 when a batch is sent in chunks).
    int enqueue(const void *src, size_t bytes, size_t rank_bytes, size_t offset, cudaStream_t s);
    // Wait for `ev` (recorded after the gather) with a bound; aborts the communicator on expiry.
    int wait(cudaEvent_t ev, double seconds);

   private:
    void *comm_ = nullptr;  // ncclComm_t
    int rank_ = 0, world_ = 1, device_ = 0;
    uint8_t *root_ = nullptr;
    size_t root_bytes_ = 0;
};

}  // namespace uq
