// k_peak.cu -- measured dense INT8 tensor-core peak of this GPU (ug_measure_int8_peak).
//
// The roofline of the convolution kernels needs the INT8 tensor throughput of the part as it runs
// here (clocks, power cap), which no vendor figure gives. One CTA per SM keeps a 128 x 256 s32
// accumulator in TMEM and issues tcgen05.mma.cta_group::1.kind::i8 (M = 128, N = 256, K = 32) back to
// back from one thread over operands resident in shared memory: no global traffic, no epilogue, so
// the time is the tensor pipe's alone. Operations = 2 * 128 * 256 * 32 per instruction.
#include <cuda_runtime.h>

#include <algorithm>
#include <cstdint>
#include <string>

#include "engine.hpp"
#include "tc_common.cuh"

namespace uq {
namespace {

constexpr int kPeakN = 256, kPeakKSteps = 4;  // 4 x 32 bytes = one 128-byte swizzle row of K
constexpr int kPeakA = kBM * kBK, kPeakB = kPeakN * kBK;
constexpr int kPeakSmem = kPeakA + kPeakB + 1024;
__device__ int g_peak_timeout = 0;

__global__ void __launch_bounds__(128, 1) int8_mma_peak_kernel(int iterations) {
    extern __shared__ uint8_t smem_raw[];
    __shared__ __align__(8) uint64_t done;
    __shared__ uint32_t tmem_slot;
    const uint32_t base = (smem_u32(smem_raw) + 1023u) & ~1023u;
    // operands: any bytes; a varied pattern keeps the multipliers toggling like real data
    for (int i = threadIdx.x; i < (kPeakA + kPeakB) / 16; i += blockDim.x) {
        const uint32_t v = 0x9E3779B9u * (uint32_t)(i + 1);
        st_shared16(base + 16u * i, make_uint4(v, v ^ 0x5A5A5A5Au, v * 3u, ~v));
    }
    fence_proxy_async();
    if (threadIdx.x < 32) {
        asm volatile("tcgen05.alloc.cta_group::1.sync.aligned.shared::cta.b32 [%0], %1;" ::"r"(smem_u32(&tmem_slot)),
                     "r"(kPeakN));
        asm volatile("tcgen05.relinquish_alloc_permit.cta_group::1.sync.aligned;");
    }
    if (threadIdx.x == 0) mbar_init(smem_u32(&done), 1);
    asm volatile("fence.mbarrier_init.release.cluster;" ::: "memory");
    tc_fence_before();
    __syncthreads();
    tc_fence_after();
    const uint32_t tmem = tmem_slot;
    if (threadIdx.x == 0) {
        const uint32_t idesc = instr_desc(kPeakN);
        for (int it = 0; it < iterations; it++)
#pragma unroll
            for (int kk = 0; kk < kPeakKSteps; kk++)
                mma_i8(tmem, smem_desc(base + 32u * kk), smem_desc(base + kPeakA + 32u * kk), idesc,
                       (it | kk) ? 1u : 0u);
        mma_commit(smem_u32(&done));
        // every issued MMA completes before TMEM is freed; bounded like the conv kernels' waits
        const long long start = clock64();
        while (!mbar_try_wait(smem_u32(&done), 0, 200000))
            if (clock64() - start > kTimeoutCycles) {
                atomicExch(&g_peak_timeout, 1);
                break;
            }
    }
    tc_fence_before();
    __syncthreads();
    tc_fence_after();
    if (threadIdx.x < 32) asm volatile("tcgen05.dealloc.cta_group::1.sync.aligned.b32 %0, %1;" ::"r"(tmem), "r"(kPeakN));
}

}  // namespace

int measure_int8_peak(uint32_t iterations, float *tops, float *ms_out) {
    if (!tops || !iterations || iterations > (1u << 20)) return 22;
    int device = abi_device(), sms = 0;
    auto cuda = [](cudaError_t e, const char *what) {
        if (e != cudaSuccess) set_error(std::string(what) + ": " + cudaGetErrorString(e));
        return e == cudaSuccess;
    };
    if (!cuda(cudaSetDevice(device), "cudaSetDevice") ||
        !cuda(cudaDeviceGetAttribute(&sms, cudaDevAttrMultiProcessorCount, device), "SM count") ||
        !cuda(cudaFuncSetAttribute(int8_mma_peak_kernel, cudaFuncAttributeMaxDynamicSharedMemorySize, kPeakSmem),
              "shared memory attribute"))
        return 2001;
    cudaStream_t s = nullptr;
    cudaEvent_t e0 = nullptr, e1 = nullptr;
    if (!cuda(cudaStreamCreateWithFlags(&s, cudaStreamNonBlocking), "stream") || !cuda(cudaEventCreate(&e0), "event") ||
        !cuda(cudaEventCreate(&e1), "event"))
        return 2001;
    float best = 0.f;
    int rc = 0;
    for (int rep = 0; rep < 4 && !rc; rep++) {  // one warm-up, best of three
        cudaEventRecord(e0, s);
        int8_mma_peak_kernel<<<sms, 128, kPeakSmem, s>>>((int)iterations);
        cudaEventRecord(e1, s);
        if (!cuda(cudaEventSynchronize(e1), "peak kernel")) rc = 2001;
        float ms = 0.f;
        if (!rc && rep && cuda(cudaEventElapsedTime(&ms, e0, e1), "elapsed") && ms > 0.f) {
            const double ops = 2.0 * kBM * kPeakN * 32 * kPeakKSteps * (double)iterations * sms;
            const float t = (float)(ops / (ms * 1e-3) / 1e12);
            if (t > best) {
                best = t;
                if (ms_out) *ms_out = ms;
            }
        }
    }
    int timed_out = 0;
    cudaMemcpyFromSymbol(&timed_out, g_peak_timeout, sizeof(int));
    cudaEventDestroy(e0);
    cudaEventDestroy(e1);
    cudaStreamDestroy(s);
    if (!rc && timed_out) {
        set_error("INT8 peak kernel: a device wait timed out");
        rc = 2003;
    }
    *tops = rc ? 0.f : best;
    return rc;
}

}  // namespace uq
