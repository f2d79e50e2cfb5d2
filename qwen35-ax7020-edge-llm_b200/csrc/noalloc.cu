// noalloc.cu -- a single exact BFP8 GEMV that never allocates device memory.
//
// qwen_b200_gemv_dev() keeps the paired int16 activation it builds for the
// GEMV in a per-device buffer that the library allocates on first use.  Some
// callers cannot let a library allocate: a serving process whose allocator
// has reserved (almost) all of HBM up front and must account for every
// byte, a latency-critical loop where cudaMalloc's implicit device-wide
// synchronisation is not acceptable, or a host framework that only hands
// out memory from its own pools.  For them this file provides one entry
// point whose scratch is a fixed array in the library's own device image:
// it exists on every GPU that loads the library, from load until the
// process exits, and costs kNoAllocScratchWords * 4 bytes (33 KB) each.
#include "api_error.cuh"
#include "bfp8_gemv.cuh"

#include "qwen_b200.h"

#include <mutex>

namespace {

constexpr int kNoAllocMaxK = 16384;   // largest K the fixed scratch serves
constexpr size_t kNoAllocScratchWords = (size_t)kNoAllocMaxK / 2 + (size_t)kNoAllocMaxK / 64;

// Paired activation + block scales of the GEMV in flight.  In host code this
// name is only a stand-in for the symbol: the device address comes from
// cudaGetSymbolAddress below and is what the kernels receive.
static __device__ __align__(256) uint32_t g_noalloc_scratch[kNoAllocScratchWords];

constexpr int kMaxDevices = 64;
std::mutex g_setup_mu;
uint32_t* g_scratch_addr[kMaxDevices] = {};

// Device address of g_noalloc_scratch on the current device, looked up once
// per device (with that device current).  No allocation happens here.
int scratch_address(uint32_t** out) {
    int dev = 0;
    cudaError_t e = cudaGetDevice(&dev);
    if (e != cudaSuccess) return qb::api_fail(QB_ENODEV, "qwen_b200_gemv_noalloc_dev: no current device", e);
    if (dev < 0 || dev >= kMaxDevices)
        return qb::api_fail(QB_ENODEV, "qwen_b200_gemv_noalloc_dev: device index beyond 63");
    std::lock_guard<std::mutex> lk(g_setup_mu);
    if (!g_scratch_addr[dev]) {
        void* p = nullptr;
        if ((e = cudaGetSymbolAddress(&p, g_noalloc_scratch)) != cudaSuccess || !p)
            return qb::api_fail(QB_ECUDA, "qwen_b200_gemv_noalloc_dev: scratch address lookup", e);
        g_scratch_addr[dev] = static_cast<uint32_t*>(p);
    }
    *out = g_scratch_addr[dev];
    return QB_OK;
}

}  // namespace

extern "C" int qwen_b200_gemv_noalloc_dev(float* y, const float* x, const int8_t* mant, const uint8_t* exps, int M,
                                          int K, void* stream) {
    if (!y || !x || !mant || !exps) return qb::api_fail(QB_EINVAL, "qwen_b200_gemv_noalloc_dev: null pointer");
    if (M < 0 || K <= 0 || K % 64)
        return qb::api_fail(QB_EINVAL, "qwen_b200_gemv_noalloc_dev: M must be >= 0 and K a positive multiple of 64");
    if (K > kNoAllocMaxK)   // the fixed scratch holds one activation of K <= 16384
        return qb::api_fail(QB_EINVAL, "qwen_b200_gemv_noalloc_dev: K above 16384 exceeds the fixed scratch");
    if (M == 0) return QB_OK;
    uint32_t* scratch = nullptr;
    if (int rc = scratch_address(&scratch)) return rc;
    qb::GemvDesc d{};
    d.mant = mant;
    d.exps = exps;
    d.x = x;
    d.y = y;
    d.M = M;
    d.K = K;
    // every word the kernels read is written by this call's activation pass
    // first, so the previous call's contents need no clearing
    cudaError_t e = qb::launch_gemv(d, scratch, nullptr, static_cast<cudaStream_t>(stream));
    return e == cudaSuccess ? QB_OK : qb::api_fail(QB_ECUDA, "qwen_b200_gemv_noalloc_dev", e);
}
