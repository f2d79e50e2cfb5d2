// common.cuh -- shared device helpers for the BFP8 GEMV / lm_head kernels.
//
// Floating point: the reference's vector path runs on ARMv7 Advanced SIMD,
// which always flushes subnormal inputs and results to a same-signed zero and
// never fuses multiply-add (VMLA rounds the product).  The *_ftz helpers below
// are single PTX instructions with exactly those semantics; the *_rn helpers
// are the IEEE (subnormal-preserving) forms used where the reference runs on
// scalar VFP.  Every call is an explicit instruction, so nvcc cannot contract
// a multiply and an add into an FMA.
#pragma once
#include <cstdint>
#include <cuda_runtime.h>

#include <mutex>
#include <unordered_map>
#include <vector>

namespace qb {

constexpr int kWarp = 32;

__device__ __forceinline__ float mul_ftz(float a, float b) {
    float d;
    asm("mul.rn.ftz.f32 %0, %1, %2;" : "=f"(d) : "f"(a), "f"(b));
    return d;
}
__device__ __forceinline__ float add_ftz(float a, float b) {
    float d;
    asm("add.rn.ftz.f32 %0, %1, %2;" : "=f"(d) : "f"(a), "f"(b));
    return d;
}
__device__ __forceinline__ float sub_ftz(float a, float b) {
    float d;
    asm("sub.rn.ftz.f32 %0, %1, %2;" : "=f"(d) : "f"(a), "f"(b));
    return d;
}
__device__ __forceinline__ float mul_rn(float a, float b) {
    float d;
    asm("mul.rn.f32 %0, %1, %2;" : "=f"(d) : "f"(a), "f"(b));
    return d;
}
__device__ __forceinline__ float add_rn(float a, float b) {
    float d;
    asm("add.rn.f32 %0, %1, %2;" : "=f"(d) : "f"(a), "f"(b));
    return d;
}
__device__ __forceinline__ float i2f_rn(int v) {
    float d;
    asm("cvt.rn.f32.s32 %0, %1;" : "=f"(d) : "r"(v));
    return d;
}

// exp_neon (qwen_kernels_opt.c:332-351), one lane, with the vector unit's
// flush-to-zero on every step: x clamped to [-87, 88] (a NaN stays NaN);
// fx = x * RN(1/ln 2); n = fx rounded to an integer by adding and
// subtracting 1.5 * 2^23; f = fx - n; p = the degree-6 Taylor polynomial of
// 2^f (coefficients RN((ln 2)^k / k!)) by Horner steps that round the product
// before the add (VMLA is not fused); the result p * 2^n with 2^n built from
// exponent bits (the conversion rounds toward zero and takes a NaN to 0).
__device__ __forceinline__ float exp_neon_lane(float x) {
    constexpr float kLog2e = 0x1.715476p+0f;       // RN(1/ln 2)
    constexpr float kRoundMagic = 0x1.8p+23f;      // 1.5 * 2^23
    x = mul_ftz(x, 1.0f);                          // VMAX flushes a subnormal operand
    x = (x != x) ? x : (x > -87.0f ? x : -87.0f);
    x = (x != x) ? x : (x < 88.0f ? x : 88.0f);
    const float fx = mul_ftz(x, kLog2e);
    const float n = sub_ftz(add_ftz(fx, kRoundMagic), kRoundMagic);
    const float f = sub_ftz(fx, n);
    float p = 0x1.430912p-13f;                     // k = 6
    p = add_ftz(0x1.5d87fep-10f, mul_ftz(p, f));   // k = 5
    p = add_ftz(0x1.3b2ab6p-7f, mul_ftz(p, f));    // k = 4
    p = add_ftz(0x1.c6b08ep-5f, mul_ftz(p, f));    // k = 3
    p = add_ftz(0x1.ebfbe0p-3f, mul_ftz(p, f));    // k = 2
    p = add_ftz(0x1.62e430p-1f, mul_ftz(p, f));    // k = 1
    p = add_ftz(1.0f, mul_ftz(p, f));              // k = 0
    return mul_ftz(p, __int_as_float((__float2int_rz(n) + 127) << 23));
}

// 2^(e-134) as the vector unit sees it: exact power of two for e >= 8, a
// flushed zero for the subnormal range e < 8.
__device__ __forceinline__ float exp_scale_ftz(uint32_t e) {
    return e >= 8u ? __uint_as_float((e - 7u) << 23) : 0.0f;
}
// 2^(e-134) with IEEE subnormals (scalar VFP): 2^(e-134) = 2^(e+15) * 2^-149.
__device__ __forceinline__ float exp_scale_ieee(uint32_t e) {
    return e >= 8u ? __uint_as_float((e - 7u) << 23) : __uint_as_float(1u << (e + 15u));
}

// Monotone map of a float score to an unsigned key (-0 and +0 share a key).
__device__ __forceinline__ uint32_t ord_score(float s) {
    uint32_t u = __float_as_uint(s);
    if (u == 0x80000000u) u = 0u;
    return (u & 0x80000000u) ? ~u : (u | 0x80000000u);
}
__device__ __forceinline__ float unord_score(uint32_t k) {
    uint32_t u = (k & 0x80000000u) ? (k & 0x7FFFFFFFu) : ~k;
    return __uint_as_float(u);
}
// 64-bit candidate key: higher score first, then lower id first.
__device__ __forceinline__ unsigned long long cand_key(float s, int id) {
    return ((unsigned long long)ord_score(s) << 32) | (unsigned long long)(0xFFFFFFFFu - (uint32_t)id);
}
__device__ __forceinline__ int key_id(unsigned long long k) {
    return (int)(0xFFFFFFFFu - (uint32_t)(k & 0xFFFFFFFFull));
}
__device__ __forceinline__ float key_score(unsigned long long k) {
    return unord_score((uint32_t)(k >> 32));
}

// ------------------------------------------------------------ cp.async
__device__ __forceinline__ uint32_t smem_u32(const void* p) {
    return (uint32_t)__cvta_generic_to_shared(p);
}
__device__ __forceinline__ void cp_async16(void* dst, const void* src) {
    asm volatile("cp.async.cg.shared.global [%0], [%1], 16;\n" ::"r"(smem_u32(dst)), "l"(src));
}
__device__ __forceinline__ void cp_async4(void* dst, const void* src) {
    asm volatile("cp.async.ca.shared.global [%0], [%1], 4;\n" ::"r"(smem_u32(dst)), "l"(src));
}
__device__ __forceinline__ void cp_async8(void* dst, const void* src) {
    asm volatile("cp.async.ca.shared.global [%0], [%1], 8;\n" ::"r"(smem_u32(dst)), "l"(src));
}
__device__ __forceinline__ void cp_async_commit() { asm volatile("cp.async.commit_group;\n" ::); }
template <int N>
__device__ __forceinline__ void cp_async_wait() { asm volatile("cp.async.wait_group %0;\n" ::"n"(N)); }

// ------------------------------------------------------------ host helpers
// Raise the dynamic shared-memory limit of kernel `fn` on the current device
// to at least `bytes`.  cudaFuncSetAttribute acts per device context, so the
// largest size set so far is remembered per (kernel, device); a mutex keeps
// concurrent host threads from lowering a limit another thread just raised.
inline cudaError_t raise_smem_limit(const void* fn, size_t bytes) {
    static std::mutex mu;
    static std::unordered_map<const void*, std::vector<size_t>> limits;
    int dev = 0;
    cudaError_t e = cudaGetDevice(&dev);
    if (e != cudaSuccess) return e;
    if (dev < 0) return cudaErrorInvalidDevice;
    std::lock_guard<std::mutex> lk(mu);
    std::vector<size_t>& per_dev = limits[fn];
    if ((int)per_dev.size() <= dev) per_dev.resize(dev + 1, 0);
    if (bytes <= per_dev[dev]) return cudaSuccess;
    e = cudaFuncSetAttribute(fn, cudaFuncAttributeMaxDynamicSharedMemorySize, (int)bytes);
    if (e == cudaSuccess) per_dev[dev] = bytes;
    return e;
}

}  // namespace qb
