// tma.cuh -- TMA tensor loads and mbarrier pipeline helpers (sm_100a).
//
// Weight tiles reach shared memory through 2D cp.async.bulk.tensor loads
// with SWIZZLE_128B: a box of R rows x 128 bytes lands as R 128-byte rows
// whose 16-byte chunk c sits at position c ^ (row & 7), so per-row reads by
// consecutive lanes are bank-conflict free.  Loads never use cluster
// multicast.  Every wait on an mbarrier is bounded: after kWaitLimit polls
// it records an error code in the caller's device error word and returns,
// so a lost transfer can never hang the GPU.
#pragma once
#include <cuda.h>
#include <cuda_runtime.h>
#include <cstdint>

namespace qb {

constexpr uint32_t kWaitLimit = 1u << 22;   // polls of try_wait (each may sleep ~1 us)
constexpr uint32_t kErrMbarTimeout = 1u;

__device__ __forceinline__ void mbar_init(uint64_t* bar, uint32_t count) {
    asm volatile("mbarrier.init.shared::cta.b64 [%0], %1;" ::"r"((uint32_t)__cvta_generic_to_shared(bar)),
                 "r"(count));
}
__device__ __forceinline__ void fence_barrier_init() {
    asm volatile("fence.mbarrier_init.release.cluster;" ::: "memory");
}
__device__ __forceinline__ void mbar_arrive_expect_tx(uint64_t* bar, uint32_t bytes) {
    asm volatile("mbarrier.arrive.expect_tx.shared::cta.b64 _, [%0], %1;" ::"r"(
                     (uint32_t)__cvta_generic_to_shared(bar)),
                 "r"(bytes)
                 : "memory");
}
__device__ __forceinline__ bool mbar_try_wait(uint64_t* bar, uint32_t parity) {
    uint32_t ok;
    asm volatile(
        "{\n\t.reg .pred p;\n\t"
        "mbarrier.try_wait.parity.shared::cta.b64 p, [%1], %2;\n\t"
        "selp.u32 %0, 1, 0, p;\n\t}"
        : "=r"(ok)
        : "r"((uint32_t)__cvta_generic_to_shared(bar)), "r"(parity)
        : "memory");
    return ok != 0;
}
// Bounded wait; on timeout sets kErrMbarTimeout in *err (if given) and
// returns false.
__device__ __forceinline__ bool mbar_wait(uint64_t* bar, uint32_t parity, unsigned int* err) {
    for (uint32_t i = 0; i < kWaitLimit; i++)
        if (mbar_try_wait(bar, parity)) return true;
    if (err) atomicOr(err, kErrMbarTimeout);
    return false;
}

// try_wait with a suspend-time hint: the thread may stay suspended for up
// to `ns` nanoseconds, and resumes when the phase completes, so a blocked
// waiter issues one instruction per window instead of re-polling.
__device__ __forceinline__ bool mbar_try_wait_hint(uint64_t* bar, uint32_t parity, uint32_t ns) {
    uint32_t ok;
    asm volatile(
        "{\n\t.reg .pred p;\n\t"
        "mbarrier.try_wait.parity.shared::cta.b64 p, [%1], %2, %3;\n\t"
        "selp.u32 %0, 1, 0, p;\n\t}"
        : "=r"(ok)
        : "r"((uint32_t)__cvta_generic_to_shared(bar)), "r"(parity), "r"(ns)
        : "memory");
    return ok != 0;
}
constexpr uint32_t kSleepHintNs = 1000;
constexpr uint32_t kSleepWaitLimit = 1u << 22;   // windows of at most kSleepHintNs: a bound of ~4 s
// Bounded wait for kernels whose waiters share SM sub-partitions with busy
// warps (same error contract as mbar_wait).
__device__ __forceinline__ bool mbar_wait_sleep(uint64_t* bar, uint32_t parity, unsigned int* err) {
    for (uint32_t i = 0; i < kSleepWaitLimit; i++)
        if (mbar_try_wait_hint(bar, parity, kSleepHintNs)) return true;
    if (err) atomicOr(err, kErrMbarTimeout);
    return false;
}

__device__ __forceinline__ void tma_prefetch_desc(const void* tmap) {
    asm volatile("prefetch.tensormap [%0];" ::"l"(tmap) : "memory");
}

// 2D tile load: box at (x = inner coordinate, y = row) of `tmap` into `dst`
// (1024-byte aligned for SWIZZLE_128B), completing `bytes` on `bar`.
__device__ __forceinline__ void tma_load_2d(void* dst, const void* tmap, int x, int y, uint64_t* bar) {
    asm volatile(
        "cp.async.bulk.tensor.2d.shared::cluster.global.mbarrier::complete_tx::bytes [%0], [%1, {%2, %3}], [%4];"
        ::"r"((uint32_t)__cvta_generic_to_shared(dst)), "l"(tmap), "r"(x), "r"(y),
          "r"((uint32_t)__cvta_generic_to_shared(bar))
        : "memory");
}

// 3D tile load at (x, y, z); x in elements of the innermost dimension.
__device__ __forceinline__ void tma_load_3d(void* dst, const void* tmap, int x, int y, int z, uint64_t* bar) {
    asm volatile(
        "cp.async.bulk.tensor.3d.shared::cluster.global.mbarrier::complete_tx::bytes [%0], [%1, {%2, %3, %4}], [%5];"
        ::"r"((uint32_t)__cvta_generic_to_shared(dst)), "l"(tmap), "r"(x), "r"(y), "r"(z),
          "r"((uint32_t)__cvta_generic_to_shared(bar))
        : "memory");
}

// 1D bulk copy global -> shared (16-byte aligned addresses, size a multiple
// of 16), completing on `bar`.
__device__ __forceinline__ void bulk_load(void* dst, const void* src, uint32_t bytes, uint64_t* bar) {
    asm volatile(
        "cp.async.bulk.shared::cluster.global.mbarrier::complete_tx::bytes [%0], [%1], %2, [%3];"
        ::"r"((uint32_t)__cvta_generic_to_shared(dst)), "l"(src), "r"(bytes),
          "r"((uint32_t)__cvta_generic_to_shared(bar))
        : "memory");
}

// ------------------------------------------------------------ host side
// Encode a 2D row-major tensor map (rows x cols elements of elem_bytes) with
// a box of box_rows x (128 / elem_bytes) elements and SWIZZLE_128B.
// Returns false if the driver entry point is unavailable or rejects it.
bool encode_tmap_2d(CUtensorMap* map, const void* base, int elem_bytes, uint64_t rows, uint64_t cols,
                    uint32_t box_rows);
// General tiled tensor map: `rank` dimensions innermost first, byte strides
// of dimensions 1..rank-1, box extents, element type and swizzle.
bool encode_tmap(CUtensorMap* map, CUtensorMapDataType dtype, int rank, const void* base, const uint64_t* dims,
                 const uint64_t* strides_bytes, const uint32_t* box, CUtensorMapSwizzle swizzle);

}  // namespace qb
