// lm_head.cu -- bf16 tied-embedding lm_head scan with fused argmax / top-k.
//
// Semantics (reference 04-板载脚本与工具/qwen_kernels_opt.c:401-488 and
// qwen_sampling.c:160-353): score_t = sum_i h_i * bf16(E[t][i]) evaluated as
// the NEON loop does -- eight fp32 chains c = i mod 8, each
// acc_c = acc_c + E*h with a rounded (flushed) product, then
// s = ((c0+c4) + (c2+c6)) + ((c1+c5) + (c3+c7)) -- so every score is
// bit-identical to the reference build.  Greedy pick: best must exceed -1e30,
// strict '>' in ascending id (ties -> lowest id).  Top-k: scores above
// -FLT_MAX, sorted descending, ties by ascending id.  The 65536 scores never
// leave the SM: each CTA keeps its candidates in shared memory.
//
// Kernel shape: a unit is 64 table rows; thread t owns row t/4 and the two
// chains 2*(t%4), 2*(t%4)+1 for the whole unit, so every chain is summed in
// one thread in element order.  Rows stream through a P-stage ring of 16 KB
// slices (64 rows x 256 bytes) loaded by TMA (two 64 x 128-byte boxes per
// slice, SWIZZLE_128B: the 16-byte chunk index XORed by row & 7), so the
// 32-bit reads of a warp (8 rows x one chunk) are conflict free.
#include "bfp8_gemv.cuh"
#include "common.cuh"
#include "lm_head.cuh"
#include "tma.cuh"
#include "topk.cuh"

#include <cub/device/device_radix_sort.cuh>

#include <algorithm>

namespace qb {

namespace {

constexpr int kThreads = 256;
constexpr int kRows = 64;                 // rows per unit
constexpr int kSegBytes = 256;            // bytes of one row per slice
constexpr int kChunks = kSegBytes / 16;   // 16-byte chunks of one row per slice
constexpr int kStage = kRows * kSegBytes; // 16 KB
constexpr int kP = 6;

struct LmArgs {
    CUtensorMap tmap;   // E as rows x hidden uint16, 64 x 64-element boxes
    const float* h;
    const uint16_t* E;
    int vocab, hidden;
    int units, slices;  // per unit
    unsigned int* err;
    LmScratch* sc;
    int kk;
    int* out_id;
    int* out_ids;
    float* out_scores;
    int* out_n;
};

__device__ __forceinline__ void issue(const LmArgs& A, int u, int s, unsigned char* st, uint64_t* bar) {
    if (threadIdx.x == 0) {
        mbar_arrive_expect_tx(bar, kStage);
        tma_load_2d(st, &A.tmap, s * (kSegBytes / 2), u * kRows, bar);
        tma_load_2d(st + kRows * 128, &A.tmap, s * (kSegBytes / 2) + 64, u * kRows, bar);
    }
}

template <bool TOPK>
__global__ void __launch_bounds__(kThreads, 1) lm_bf16_kernel(const __grid_constant__ LmArgs A) {
    extern __shared__ __align__(1024) unsigned char smem_raw[];
    unsigned char* smem = reinterpret_cast<unsigned char*>((reinterpret_cast<uintptr_t>(smem_raw) + 1023) &
                                                           ~uintptr_t(1023));
    unsigned char* stages = smem;
    uint64_t* bars = reinterpret_cast<uint64_t*>(smem + kP * kStage);
    float* hs = reinterpret_cast<float*>(smem + kP * kStage + 64);
    unsigned long long* cand = reinterpret_cast<unsigned long long*>(hs + A.hidden);
    __shared__ int s_cand_count;
    __shared__ unsigned long long s_red[kThreads / 32];

    const int tid = threadIdx.x;
    const int r = tid >> 2, p = tid & 3;
    if (tid == 0) {
        s_cand_count = 0;
        for (int k = 0; k < kP; k++) mbar_init(&bars[k], 1);
        fence_barrier_init();
        tma_prefetch_desc(&A.tmap);
    }
    __syncthreads();

    // contiguous unit range of this CTA
    const int u_begin = (int)(((long long)A.units * blockIdx.x) / gridDim.x);
    const int u_end = (int)(((long long)A.units * (blockIdx.x + 1)) / gridDim.x);
    const int total = (u_end - u_begin) * A.slices;

    // prologue: first P-1 slices, then h (overlaps the copies)
    int iu = u_begin, is = 0, issued = 0;
#pragma unroll 1
    for (int k = 0; k < kP - 1; k++) {
        if (issued < total) {
            issue(A, iu, is, stages + k * kStage, &bars[k]);
            if (++is == A.slices) { is = 0; iu++; }
            issued++;
        }
    }
    for (int i = tid; i < A.hidden; i += kThreads) hs[i] = A.h[i];

    unsigned long long best = 0ull;
    float ca = 0.0f, cb = 0.0f;
    int cu = u_begin, cs = 0;
#pragma unroll 1
    for (int it = 0; it < total; it++) {
        mbar_wait(&bars[it % kP], (uint32_t)(it / kP) & 1u, A.err);
        __syncthreads();
        if (issued < total) {
            const int ns = (it + kP - 1) % kP;
            issue(A, iu, is, stages + ns * kStage, &bars[ns]);
            if (++is == A.slices) { is = 0; iu++; }
            issued++;
        }
        if (TOPK && s_cand_count > kCandCap - 2 * kRows) cand_compact(cand, &s_cand_count, A.kk);

        const unsigned char* st = stages + (it % kP) * kStage;
        const int chunks_total = A.hidden >> 3;
        const int vc = min(kChunks, chunks_total - cs * kChunks);
        const unsigned char* rowp = st + r * 128 + 4 * p;
        const float2* hp = reinterpret_cast<const float2*>(hs + cs * (kSegBytes / 2) + 2 * p);
        const int sw = r & 7;
        if (vc == kChunks) {
#pragma unroll
            for (int q = 0; q < kChunks; q++) {
                uint32_t w = *reinterpret_cast<const uint32_t*>(rowp + (q >> 3) * (kRows * 128) +
                                                                 (((q & 7) ^ sw) << 4));
                float2 hv = hp[4 * q];
                ca = add_ftz(ca, mul_ftz(__uint_as_float(w << 16), hv.x));
                cb = add_ftz(cb, mul_ftz(__uint_as_float(w & 0xFFFF0000u), hv.y));
            }
        } else {
            for (int q = 0; q < vc; q++) {
                uint32_t w = *reinterpret_cast<const uint32_t*>(rowp + (q >> 3) * (kRows * 128) +
                                                                 (((q & 7) ^ sw) << 4));
                float2 hv = hp[4 * q];
                ca = add_ftz(ca, mul_ftz(__uint_as_float(w << 16), hv.x));
                cb = add_ftz(cb, mul_ftz(__uint_as_float(w & 0xFFFF0000u), hv.y));
            }
        }
        if (cs == A.slices - 1) {
            // thread p holds chains (2p, 2p+1); combine in the NEON order
            float oa = __shfl_xor_sync(0xffffffffu, ca, 2);
            float ob = __shfl_xor_sync(0xffffffffu, cb, 2);
            float lo = add_ftz(ca, oa), hi = add_ftz(cb, ob);   // p=0: c0+c4, c1+c5; p=1: c2+c6, c3+c7
            float lo2 = __shfl_xor_sync(0xffffffffu, lo, 1);
            float hi2 = __shfl_xor_sync(0xffffffffu, hi, 1);
            float s = add_ftz(add_ftz(lo, lo2), add_ftz(hi, hi2));
            const int row = cu * kRows + r;
            if (p == 0 && row < A.vocab) {
                if (s > -1e30f) {
                    unsigned long long key = cand_key(s, row);
                    best = key > best ? key : best;
                }
                if (TOPK && s > -3.402823466e38f) {
                    int pos = atomicAdd(&s_cand_count, 1);
                    cand[pos] = cand_key(s, row);
                }
            }
            ca = cb = 0.0f;
            cs = 0;
            cu++;
        } else {
            cs++;
        }
    }
    __syncthreads();
    unsigned long long* work = reinterpret_cast<unsigned long long*>(stages);
    lm_finish(A.sc, cand, kCandCap, &s_cand_count, work, (kP * kStage) / 8, best, TOPK ? A.kk : 0, A.out_id,
              A.out_ids, A.out_scores, A.out_n, s_red);
}

// ---------------------------------------------------------------- warp-autonomous scan
// hidden % 128 == 0 and k <= 64.  A unit is 32 table rows and a warp owns it
// from first byte to score: lane = row, the lane keeps all eight chains of
// its row in registers, so there is no CTA barrier while streaming.  Each
// warp has a private ring of kWRing 8 KB stages (two TMA boxes of 32 rows x
// 64 elements, SWIZZLE_128B), refilled by its lane 0.  Candidates: each warp
// keeps its best 64 keys in registers; the CTA merges the eight lists at
// the end.  CTA c scores the contiguous units [U*c/G, U*(c+1)/G).
constexpr int kWRows = 32;
constexpr int kWRing = 3;
constexpr int kWStage = kWRows * 256;   // 128 elements of 32 rows
constexpr int kWWarps = kThreads / 32;

__device__ __forceinline__ void wissue(const LmArgs& A, int u, int s, unsigned char* st, uint64_t* bar) {
    mbar_arrive_expect_tx(bar, kWStage);
    tma_load_2d(st, &A.tmap, s * 128, u * kWRows, bar);
    tma_load_2d(st + kWRows * 128, &A.tmap, s * 128 + 64, u * kWRows, bar);
}

template <bool TOPK>
__global__ void __launch_bounds__(kThreads, 1) lm_bf16_warp_kernel(const __grid_constant__ LmArgs A) {
    extern __shared__ __align__(1024) unsigned char smem_raw[];
    unsigned char* smem = reinterpret_cast<unsigned char*>((reinterpret_cast<uintptr_t>(smem_raw) + 1023) &
                                                           ~uintptr_t(1023));
    unsigned char* rings = smem;                                                  // [warp][slot] 8 KB
    uint64_t* bars = reinterpret_cast<uint64_t*>(rings + kWWarps * kWRing * kWStage);   // [warp][slot]
    float* hs = reinterpret_cast<float*>(bars + kWWarps * kWRing);
    unsigned long long* cand = reinterpret_cast<unsigned long long*>(hs + A.hidden);   // 64 * warps + 64
    __shared__ int s_cand_count;
    __shared__ unsigned long long s_red[kThreads / 32];

    // the next kernel on the stream may start its prologue now
    asm volatile("griddepcontrol.launch_dependents;" ::: "memory");
    const int tid = threadIdx.x, warp = tid >> 5, lane = tid & 31;
    unsigned char* ring = rings + warp * kWRing * kWStage;
    uint64_t* bar = bars + warp * kWRing;
    if (lane == 0) {
        for (int k = 0; k < kWRing; k++) mbar_init(&bar[k], 1);
        fence_barrier_init();
        tma_prefetch_desc(&A.tmap);
    }
    if (tid == 0) s_cand_count = 0;
    __syncwarp();

    const int U = (A.vocab + kWRows - 1) / kWRows;
    const int u_begin = (int)(((long long)U * blockIdx.x) / gridDim.x);
    const int u_end = (int)(((long long)U * (blockIdx.x + 1)) / gridDim.x);
    const int nst = A.hidden / 128;
    const int my_units = u_end - u_begin > warp ? (u_end - u_begin - warp + kWWarps - 1) / kWWarps : 0;
    const int total = my_units * nst;   // stages this warp streams

    // prologue: the first kWRing-1 stages, then h (overlaps the copies)
    int iu = 0, is = 0, issued = 0;
    if (lane == 0)
        for (int k = 0; k < kWRing - 1 && issued < total; k++, issued++) {
            wissue(A, u_begin + warp + iu * kWWarps, is, ring + k * kWStage, &bar[k]);
            if (++is == nst) { is = 0; iu++; }
        }
    // a programmatic dependent of the stream's previous kernel: the table
    // stages are in flight; h (maybe that kernel's output) is read, and the
    // scratch and outputs written, only once that kernel has completed
    asm volatile("griddepcontrol.wait;" ::: "memory");
    for (int i = tid; i < A.hidden; i += kThreads) hs[i] = A.h[i];
    __syncthreads();

    unsigned long long best = 0ull, r0 = 0ull, r1 = 0ull, thr = 0ull;
    float c[8];
#pragma unroll
    for (int q = 0; q < 8; q++) c[q] = 0.0f;
    const int sw = lane & 7;
    int cu = 0, cs = 0;
#pragma unroll 1
    for (int it = 0; it < total; it++) {
        const int slot = it % kWRing;
        mbar_wait(&bar[slot], (uint32_t)(it / kWRing) & 1u, A.err);
        __syncwarp();
        if (lane == 0 && issued < total) {   // refill the slot consumed last iteration
            asm volatile("fence.proxy.async.shared::cta;" ::: "memory");
            const int ns = (it + kWRing - 1) % kWRing;
            wissue(A, u_begin + warp + iu * kWWarps, is, ring + ns * kWStage, &bar[ns]);
            if (++is == nst) { is = 0; iu++; }
            issued++;
        }
        const unsigned char* rowp = ring + slot * kWStage + lane * 128;
        const float4* hp = reinterpret_cast<const float4*>(hs + cs * 128);
#pragma unroll
        for (int b = 0; b < 2; b++) {
#pragma unroll
            for (int j = 0; j < 8; j++) {
                const uint4 w = *reinterpret_cast<const uint4*>(rowp + b * (kWRows * 128) + ((j ^ sw) << 4));
                const float4 ha = hp[(b * 64 + j * 8) / 4];
                const float4 hb = hp[(b * 64 + j * 8) / 4 + 1];
                c[0] = add_ftz(c[0], mul_ftz(__uint_as_float(w.x << 16), ha.x));
                c[1] = add_ftz(c[1], mul_ftz(__uint_as_float(w.x & 0xFFFF0000u), ha.y));
                c[2] = add_ftz(c[2], mul_ftz(__uint_as_float(w.y << 16), ha.z));
                c[3] = add_ftz(c[3], mul_ftz(__uint_as_float(w.y & 0xFFFF0000u), ha.w));
                c[4] = add_ftz(c[4], mul_ftz(__uint_as_float(w.z << 16), hb.x));
                c[5] = add_ftz(c[5], mul_ftz(__uint_as_float(w.z & 0xFFFF0000u), hb.y));
                c[6] = add_ftz(c[6], mul_ftz(__uint_as_float(w.w << 16), hb.z));
                c[7] = add_ftz(c[7], mul_ftz(__uint_as_float(w.w & 0xFFFF0000u), hb.w));
            }
        }
        if (++cs == nst) {   // the row is complete: the reference's chain combine
            const float s = add_ftz(add_ftz(add_ftz(c[0], c[4]), add_ftz(c[2], c[6])),
                                    add_ftz(add_ftz(c[1], c[5]), add_ftz(c[3], c[7])));
            const int row = (u_begin + warp + cu * kWWarps) * kWRows + lane;
            const bool ok = row < A.vocab;
            if (ok && s > -1e30f) {
                const unsigned long long key = cand_key(s, row);
                best = key > best ? key : best;
            }
            if (TOPK) {
                const unsigned long long key = (ok && s > -3.402823466e38f) ? cand_key(s, row) : 0ull;
                if (__any_sync(0xffffffffu, key > thr)) {
                    warp_fold64(r0, r1, key, 0ull);
                    thr = __shfl_sync(0xffffffffu, r1, 31);
                }
            }
#pragma unroll
            for (int q = 0; q < 8; q++) c[q] = 0.0f;
            cs = 0;
            cu++;
        }
    }
    __syncthreads();
    if (TOPK) {
        cand[warp * 64 + lane] = r0;
        cand[warp * 64 + 32 + lane] = r1;
        merge_warp_lists64(cand, &s_cand_count, A.kk);
    }
    unsigned long long* work = reinterpret_cast<unsigned long long*>(rings);
    lm_finish(A.sc, cand, 64 * kWWarps + 64, &s_cand_count, work, (kWWarps * kWRing * kWStage) / 8, best, TOPK ? A.kk : 0,
              A.out_id, A.out_ids, A.out_scores, A.out_n, s_red, TOPK);
}

// Any hidden size / alignment: one thread per row, same score order; the
// with_tail flag adds the elements past the last multiple of 8 on IEEE
// scalar arithmetic (lm_head_topk) or drops them (lm_head_argmax).
__global__ void __launch_bounds__(kThreads) lm_bf16_generic_kernel(const float* h, const uint16_t* E,
                                                                  int vocab, int hidden, int with_tail,
                                                                  float* scores) {
    const int t = blockIdx.x * kThreads + threadIdx.x;
    if (t >= vocab) return;
    const uint16_t* row = E + (size_t)t * hidden;
    float c[8] = {0, 0, 0, 0, 0, 0, 0, 0};
    int i = 0;
    for (; i + 8 <= hidden; i += 8)
#pragma unroll
        for (int j = 0; j < 8; j++)
            c[j] = add_ftz(c[j], mul_ftz(__uint_as_float((uint32_t)row[i + j] << 16), h[i + j]));
    float s = add_ftz(add_ftz(add_ftz(c[0], c[4]), add_ftz(c[2], c[6])),
                      add_ftz(add_ftz(c[1], c[5]), add_ftz(c[3], c[7])));
    if (with_tail)
        for (; i < hidden; i++) s = add_rn(s, mul_rn(h[i], __uint_as_float((uint32_t)row[i] << 16)));
    scores[t] = s;
}

// Selection over a materialised score vector (generic-shape path only).
__global__ void __launch_bounds__(kThreads, 1) select_kernel(const float* scores, int vocab,
                                                             const __grid_constant__ LmArgs A) {
    extern __shared__ __align__(128) unsigned char smem[];
    unsigned long long* cand = reinterpret_cast<unsigned long long*>(smem);
    unsigned long long* work = cand + kCandCap;
    __shared__ int s_cand_count;
    __shared__ unsigned long long s_red[kThreads / 32];
    if (threadIdx.x == 0) s_cand_count = 0;
    __syncthreads();
    const int lo = (int)(((long long)vocab * blockIdx.x) / gridDim.x);
    const int hi = (int)(((long long)vocab * (blockIdx.x + 1)) / gridDim.x);
    unsigned long long best = 0ull;
    for (int base = lo; base < hi; base += kThreads) {
        if (A.kk > 0 && s_cand_count > kCandCap - kThreads) cand_compact(cand, &s_cand_count, A.kk);
        int t = base + threadIdx.x;
        if (t < hi) {
            float s = scores[t];
            if (s > -1e30f) {
                unsigned long long key = cand_key(s, t);
                best = key > best ? key : best;
            }
            if (A.kk > 0 && s > -3.402823466e38f) {
                int pos = atomicAdd(&s_cand_count, 1);
                cand[pos] = cand_key(s, t);
            }
        }
        __syncthreads();
    }
    lm_finish(A.sc, cand, kCandCap, &s_cand_count, work, kCandCap * 4, best, A.kk, A.out_id, A.out_ids,
              A.out_scores, A.out_n, s_red);
}

}  // namespace

cudaError_t launch_lm_head_bf16(const float* h, const uint16_t* E, int vocab, int hidden, int k,
                                int with_tail, LmScratch* scratch, unsigned int* err_word, float* score_buf,
                                int* out_id, int* out_ids, float* out_scores, int* out_n, cudaStream_t stream) {
    if (vocab <= 0 || hidden <= 0 || k < 0 || std::min(k, vocab) > kTopkMax) return cudaErrorInvalidValue;
    LmArgs A{};
    A.h = h;
    A.E = E;
    A.vocab = vocab;
    A.hidden = hidden;
    A.sc = scratch;
    A.kk = std::min(k, vocab);
    A.out_id = out_id;
    A.out_ids = out_ids;
    A.out_scores = out_scores;
    A.out_n = out_n;
    A.err = err_word;
    const bool warp_path = hidden % 128 == 0 && A.kk <= 64;
    const bool fast = hidden % 8 == 0 && reinterpret_cast<uintptr_t>(E) % 16 == 0 &&
                      reinterpret_cast<uintptr_t>(h) % 8 == 0 &&
                      encode_tmap_2d(&A.tmap, E, 2, (uint64_t)vocab, (uint64_t)hidden,
                                     (uint32_t)(warp_path ? kWRows : kRows));
    if (fast && warp_path) {
        const int units = (vocab + kWRows - 1) / kWRows;
        const int grid = std::min(std::min(num_sms(), units), kMaxGrid);
        const size_t smem = 1024 + (size_t)kWWarps * kWRing * kWStage + (size_t)kWWarps * kWRing * 8 +
                            4 * (size_t)hidden + (size_t)(64 * kWWarps + 64) * 8;
        if (smem > 232448) return cudaErrorInvalidValue;
        auto kern = A.kk > 0 ? lm_bf16_warp_kernel<true> : lm_bf16_warp_kernel<false>;
        cudaError_t err = raise_smem_limit(reinterpret_cast<const void*>(kern), smem);
        if (err != cudaSuccess) return err;
        cudaLaunchConfig_t cfg = {};
        cfg.gridDim = dim3(grid);
        cfg.blockDim = dim3(kThreads);
        cfg.dynamicSmemBytes = smem;
        cfg.stream = stream;
        cudaLaunchAttribute attr[1];
        attr[0].id = cudaLaunchAttributeProgrammaticStreamSerialization;
        attr[0].val.programmaticStreamSerializationAllowed = 1;
        cfg.attrs = attr;
        cfg.numAttrs = 1;   // a programmatic dependent of the stream's previous kernel
        return cudaLaunchKernelEx(&cfg, kern, A);
    }
    if (fast) {
        A.units = (vocab + kRows - 1) / kRows;
        A.slices = ((hidden >> 3) + kChunks - 1) / kChunks;
        const int grid = std::min(std::min(num_sms(), A.units), kMaxGrid);
        const size_t smem = 1024 + (size_t)kP * kStage + 64 + 4 * (size_t)hidden + (size_t)kCandCap * 8;
        cudaError_t err;
        if (A.kk > 0) {
            err = cudaFuncSetAttribute(lm_bf16_kernel<true>, cudaFuncAttributeMaxDynamicSharedMemorySize,
                                       (int)smem);
            if (err != cudaSuccess) return err;
            lm_bf16_kernel<true><<<grid, kThreads, smem, stream>>>(A);
        } else {
            err = cudaFuncSetAttribute(lm_bf16_kernel<false>, cudaFuncAttributeMaxDynamicSharedMemorySize,
                                       (int)smem);
            if (err != cudaSuccess) return err;
            lm_bf16_kernel<false><<<grid, kThreads, smem, stream>>>(A);
        }
        return cudaGetLastError();
    }
    if (!score_buf) return cudaErrorInvalidValue;
    lm_bf16_generic_kernel<<<(vocab + kThreads - 1) / kThreads, kThreads, 0, stream>>>(h, E, vocab, hidden,
                                                                                     with_tail, score_buf);
    cudaError_t err = cudaGetLastError();
    if (err != cudaSuccess) return err;
    const size_t smem = (size_t)kCandCap * 8 * 5;
    err = cudaFuncSetAttribute(select_kernel, cudaFuncAttributeMaxDynamicSharedMemorySize, (int)smem);
    if (err != cudaSuccess) return err;
    const int grid = std::max(1, std::min(std::min(num_sms(), (vocab + 1023) / 1024), kMaxGrid));
    select_kernel<<<grid, kThreads, smem, stream>>>(score_buf, vocab, A);
    return cudaGetLastError();
}

// ------------------------------------------------------------ k > 1024
// Top-k with any k (the reference's lm_head_topk serves every k): every
// score becomes a 64-bit key (ordered score, ~id), so one descending radix
// sort of the keys is the reference order -- score descending, ties by
// ascending id -- and scores not above -FLT_MAX (which the reference never
// offers to its table) get key 0 and sort last.
__global__ void topk_keys_kernel(const float* scores, int vocab, unsigned long long* keys) {
    for (int t = blockIdx.x * blockDim.x + threadIdx.x; t < vocab; t += gridDim.x * blockDim.x) {
        const float s = scores[t];
        keys[t] = s > -3.402823466e38f ? cand_key(s, t) : 0ull;
    }
}

__global__ void topk_emit_kernel(const unsigned long long* sorted, int kk, int* out_ids, float* out_scores,
                                 int* out_n) {
    __shared__ int s_n;
    if (threadIdx.x == 0) s_n = 0;
    __syncthreads();
    int valid = 0;
    for (int i = threadIdx.x; i < kk; i += blockDim.x) {
        const unsigned long long key = sorted[i];
        if (key) {
            out_ids[i] = key_id(key);
            out_scores[i] = key_score(key);
            valid++;
        }
    }
    atomicAdd(&s_n, valid);
    __syncthreads();
    if (threadIdx.x == 0) *out_n = s_n;   // the valid keys are a prefix of the sorted list
}

size_t topk_large_temp_bytes(int vocab) {
    size_t temp = 0;
    cub::DoubleBuffer<unsigned long long> db(nullptr, nullptr);
    cub::DeviceRadixSort::SortKeysDescending(nullptr, temp, db, vocab);
    return temp;
}

cudaError_t launch_topk_large(const float* scores, int vocab, int kk, unsigned long long* keys,
                              unsigned long long* keys_alt, void* temp, size_t temp_bytes, int* out_ids,
                              float* out_scores, int* out_n, cudaStream_t stream) {
    if (vocab <= 0 || kk <= 0 || kk > vocab || !keys || !keys_alt || !temp) return cudaErrorInvalidValue;
    const int grid = std::max(1, std::min((vocab + kThreads - 1) / kThreads, num_sms() * 8));
    topk_keys_kernel<<<grid, kThreads, 0, stream>>>(scores, vocab, keys);
    cudaError_t e = cudaGetLastError();
    if (e != cudaSuccess) return e;
    cub::DoubleBuffer<unsigned long long> db(keys, keys_alt);
    e = cub::DeviceRadixSort::SortKeysDescending(temp, temp_bytes, db, vocab, 0, 64, stream);
    if (e != cudaSuccess) return e;
    topk_emit_kernel<<<1, 1024, 0, stream>>>(db.Current(), kk, out_ids, out_scores, out_n);
    return cudaGetLastError();
}

cudaError_t launch_lm_scores_bf16(const float* h, const uint16_t* E, int vocab, int hidden, int with_tail,
                                  float* scores, cudaStream_t stream) {
    if (vocab <= 0 || hidden <= 0 || !scores) return cudaErrorInvalidValue;
    lm_bf16_generic_kernel<<<(vocab + kThreads - 1) / kThreads, kThreads, 0, stream>>>(h, E, vocab, hidden,
                                                                                     with_tail, scores);
    return cudaGetLastError();
}

}  // namespace qb
