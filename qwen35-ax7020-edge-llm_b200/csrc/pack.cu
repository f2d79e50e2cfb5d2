// pack.cu -- on-device block-64 BFP8 packer (SoA), used to build synthetic
// weight stacks at HBM speed.
//
// Rule of the reference packer (05-主机侧源码/bfp8_packer.py:53-86):
//   peak = max |w| over a 64-element row block
//   peak < 1e-12   -> e = 127, all mantissas 0
//   otherwise      e = clip(ceil(log2(peak)) + 127, 0, 255)
//                  m = clip(round_half_even(w * 2^(7 - (e - 127))), -128, 127)
// ceil(log2(peak)) is evaluated exactly from the float's bits (exponent, plus
// one unless the significand is a power of two).  The reference evaluates it
// through numpy's float32 log2, which can round log2 of a value within a
// couple of ulps above a power of two down to the integer; only such blocks
// can pack differently.
#include "common.cuh"
#include "qwen_b200.h"

#include <algorithm>

namespace {

__global__ void pack_bfp8_kernel(const float* __restrict__ w, long long nblocks, int8_t* __restrict__ mant,
                                 uint8_t* __restrict__ exps) {
    const int lane = threadIdx.x & 31;
    for (long long blk = (long long)blockIdx.x * (blockDim.x / 32) + (threadIdx.x >> 5); blk < nblocks;
         blk += (long long)gridDim.x * (blockDim.x / 32)) {
        const float2 v = reinterpret_cast<const float2*>(w + blk * 64)[lane];
        float a = fmaxf(fabsf(v.x), fabsf(v.y));
        for (int o = 16; o > 0; o >>= 1) a = fmaxf(a, __shfl_xor_sync(0xffffffffu, a, o));
        int e;
        int m0 = 0, m1 = 0;
        if (!(a >= 1e-12f)) {
            e = 127;
        } else {
            const uint32_t u = __float_as_uint(a);
            int lg = (int)((u >> 23) & 0xFF) - 127 + ((u & 0x7FFFFF) ? 1 : 0);
            e = min(max(lg + 127, 0), 255);
            const float scale = __uint_as_float((uint32_t)(134 - e + 127) << 23);   // 2^(7-(e-127))
            m0 = (int)fminf(fmaxf(rintf(__fmul_rn(v.x, scale)), -128.0f), 127.0f);
            m1 = (int)fminf(fmaxf(rintf(__fmul_rn(v.y, scale)), -128.0f), 127.0f);
        }
        reinterpret_cast<char2*>(mant + blk * 64)[lane] = make_char2((signed char)m0, (signed char)m1);
        if (lane == 0) exps[blk] = (uint8_t)e;
    }
}

}  // namespace

extern "C" int qwen_b200_pack_bfp8_dev(const float* w, int M, int K, int8_t* mant, uint8_t* exps, void* stream) {
    if (!w || !mant || !exps || M < 0 || K <= 0 || K % 64) return QB_EINVAL;
    if (reinterpret_cast<uintptr_t>(w) % 8 || reinterpret_cast<uintptr_t>(mant) % 2) return QB_EINVAL;
    const long long nblocks = (long long)M * (K / 64);
    if (nblocks == 0) return QB_OK;
    const int grid = (int)std::min<long long>((nblocks + 7) / 8, 148LL * 16);
    pack_bfp8_kernel<<<grid, 256, 0, static_cast<cudaStream_t>(stream)>>>(w, nblocks, mant, exps);
    return cudaGetLastError() == cudaSuccess ? QB_OK : QB_ECUDA;
}
