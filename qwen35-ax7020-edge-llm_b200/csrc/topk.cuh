// topk.cuh -- block-level candidate selection shared by the lm_head kernels.
//
// Scores are carried as 64-bit keys (see cand_key): the high word orders the
// score (higher first, -0 == +0), the low word holds ~id so that equal
// scores rank the lower id first.  That is exactly the order the reference
// sampler produces (score descending, ties in ascending token id,
// qwen_sampling.c:117-155), so "the k largest keys, sorted descending" is the
// reference top-k.
//
// Flow per launch:
//   1. every CTA appends the keys of the rows it scores into a shared-memory
//      buffer (compacting to the best kk when it fills),
//   2. at its end the CTA sorts the buffer and writes its best kk keys to the
//      scratch lists, then takes a ticket,
//   3. the CTA with the last ticket radix-selects the kk-th largest key of
//      the union, sorts the winners and writes ids / scores, then clears the
//      ticket and the argmax word for the next launch.
#pragma once
#include "common.cuh"

namespace qb {

constexpr int kCandCap = 2048;     // per-CTA shared-memory candidate buffer
constexpr int kTopkMax = 1024;     // largest k the device path serves
constexpr int kMaxGrid = 512;      // largest grid the scratch is laid out for

// Persistent per-device scratch for the lm_head kernels.  Zeroed once when it
// is created; every launch leaves `ticket` and `argmax_key` at zero again.
struct LmScratch {
    unsigned long long argmax_key;
    unsigned int ticket;
    unsigned int n_out;
    int counts[kMaxGrid];
    unsigned long long lists[(size_t)kMaxGrid * kTopkMax];
};

__device__ __forceinline__ int next_pow2(int n) {
    int p = 1;
    while (p < n) p <<= 1;
    return p;
}

// In-place bitonic sort, descending, of a[0..n) (n a power of two), by the
// whole block.  Ends with a barrier.
__device__ inline void block_sort_desc(unsigned long long* a, int n) {
    for (int k = 2; k <= n; k <<= 1) {
        for (int j = k >> 1; j > 0; j >>= 1) {
            for (int i = threadIdx.x; i < n; i += blockDim.x) {
                int ixj = i ^ j;
                if (ixj > i) {
                    unsigned long long ai = a[i], aj = a[ixj];
                    bool down = (i & k) == 0;
                    if (down ? (ai < aj) : (ai > aj)) {
                        a[i] = aj;
                        a[ixj] = ai;
                    }
                }
            }
            __syncthreads();
        }
    }
}

// Sort the candidate buffer and keep its best `keep` keys.  Called by the
// whole block; *count is in shared memory.
__device__ inline void cand_compact(unsigned long long* cand, int* count, int keep) {
    __syncthreads();
    int n = *count;
    int p = next_pow2(n < 1 ? 1 : n);
    for (int i = n + threadIdx.x; i < p; i += blockDim.x) cand[i] = 0ull;
    __syncthreads();
    block_sort_desc(cand, p);
    if (threadIdx.x == 0) *count = n < keep ? n : keep;
    __syncthreads();
}

// Block-wide max of a 64-bit key; result valid in every thread.
__device__ inline unsigned long long block_max_u64(unsigned long long v, unsigned long long* red) {
    for (int o = 16; o > 0; o >>= 1) {
        unsigned long long w = __shfl_xor_sync(0xffffffffu, v, o);
        v = w > v ? w : v;
    }
    int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
    __syncthreads();
    if (lane == 0) red[warp] = v;
    __syncthreads();
    unsigned long long m = 0;
    int nw = blockDim.x >> 5;
    for (int i = 0; i < nw; i++) m = red[i] > m ? red[i] : m;
    __syncthreads();
    return m;
}

// End-of-CTA work for the lm_head kernels.  `cand`/`cand_count` is the CTA's
// shared buffer, `work` a shared scratch area of at least
// max(kCandCap, union) keys that may alias the CTA's stage buffers,
// `work_cap` its size in keys.  `best` is this thread's argmax key.
// Writes out_id[0] (argmax) and, for kk > 0, out_ids/out_scores[0..n) and
// *out_n.
__device__ inline void lm_finish(LmScratch* sc, unsigned long long* cand, int* cand_count,
                                 unsigned long long* work, int work_cap, unsigned long long best,
                                 int kk, int* out_id, int* out_ids, float* out_scores, int* out_n,
                                 unsigned long long* red) {
    const int tid = threadIdx.x;
    unsigned long long bm = block_max_u64(best, red);
    if (tid == 0 && bm) atomicMax(&sc->argmax_key, bm);

    if (kk > 0) {
        cand_compact(cand, cand_count, kk);
        int n = *cand_count;
        unsigned long long* dst = sc->lists + (size_t)blockIdx.x * kk;
        for (int i = tid; i < n; i += blockDim.x) dst[i] = cand[i];
        if (tid == 0) sc->counts[blockIdx.x] = n;
    }
    __threadfence();
    __syncthreads();
    __shared__ unsigned int s_ticket;
    if (tid == 0) s_ticket = atomicAdd(&sc->ticket, 1u);
    __syncthreads();
    if (s_ticket != gridDim.x - 1) return;
    __threadfence();

    // ---- last CTA: final results
    if (tid == 0) {
        unsigned long long k = *((volatile unsigned long long*)&sc->argmax_key);
        *out_id = k ? key_id(k) : 0;
    }
    if (kk > 0) {
        // gather the union of the per-CTA lists into shared memory
        __shared__ int s_total;
        __shared__ unsigned int s_hist[256];
        __shared__ unsigned long long s_prefix;
        __shared__ int s_remaining;
        __shared__ int s_nsel;
        if (tid == 0) {
            int t = 0;
            for (int c = 0; c < (int)gridDim.x; c++) t += ((volatile int*)sc->counts)[c];
            s_total = t;
        }
        __syncthreads();
        const int total = s_total;
        const bool in_smem = total <= work_cap;
        // keys live either in `work` (shared) or are read from the lists
        if (in_smem) {
            int base = 0;
            for (int c = 0; c < (int)gridDim.x; c++) {
                int n = ((volatile int*)sc->counts)[c];
                const volatile unsigned long long* src = sc->lists + (size_t)c * kk;
                for (int i = tid; i < n; i += blockDim.x) work[base + i] = src[i];
                base += n;
            }
        }
        __syncthreads();
        auto key_at = [&](int c, int i) -> unsigned long long {
            return ((const volatile unsigned long long*)sc->lists)[(size_t)c * kk + i];
        };
        // radix select of the kk-th largest key (keys are distinct)
        const int want = total < kk ? total : kk;
        if (tid == 0) {
            s_prefix = 0ull;
            s_remaining = want;
        }
        __syncthreads();
        if (want > 0 && want < total) {
            for (int pass = 0; pass < 8; pass++) {
                const int shift = 56 - 8 * pass;
                for (int i = tid; i < 256; i += blockDim.x) s_hist[i] = 0u;
                __syncthreads();
                const unsigned long long pre = s_prefix;
                auto count_key = [&](unsigned long long key) {
                    bool match = pass == 0 ? true : ((key >> (shift + 8)) == pre);
                    if (match) atomicAdd(&s_hist[(key >> shift) & 0xFFull], 1u);
                };
                if (in_smem) {
                    for (int i = tid; i < total; i += blockDim.x) count_key(work[i]);
                } else {
                    for (int c = 0; c < (int)gridDim.x; c++) {
                        int n = ((volatile int*)sc->counts)[c];
                        for (int i = tid; i < n; i += blockDim.x) count_key(key_at(c, i));
                    }
                }
                __syncthreads();
                if (tid == 0) {
                    int rem = s_remaining;
                    unsigned int cum = 0;
                    int d = 255;
                    for (; d > 0; d--) {
                        if ((int)(cum + s_hist[d]) >= rem) break;
                        cum += s_hist[d];
                    }
                    s_remaining = rem - (int)cum;
                    s_prefix = (pre << 8) | (unsigned long long)d;
                }
                __syncthreads();
            }
        }
        const unsigned long long kstar = (want > 0 && want < total) ? s_prefix : 0ull;
        // collect the winners (exactly `want` keys >= kstar) into cand[]
        if (tid == 0) s_nsel = 0;
        __syncthreads();
        auto take = [&](unsigned long long key) {
            if (key >= kstar && key != 0ull) {
                int p = atomicAdd(&s_nsel, 1);
                if (p < kTopkMax) cand[p] = key;
            }
        };
        if (in_smem) {
            for (int i = tid; i < total; i += blockDim.x) take(work[i]);
        } else {
            for (int c = 0; c < (int)gridDim.x; c++) {
                int n = ((volatile int*)sc->counts)[c];
                for (int i = tid; i < n; i += blockDim.x) take(key_at(c, i));
            }
        }
        __syncthreads();
        int nsel = s_nsel < want ? s_nsel : want;
        int p2 = next_pow2(nsel < 1 ? 1 : nsel);
        for (int i = nsel + tid; i < p2; i += blockDim.x) cand[i] = 0ull;
        __syncthreads();
        block_sort_desc(cand, p2);
        for (int i = tid; i < nsel; i += blockDim.x) {
            out_ids[i] = key_id(cand[i]);
            out_scores[i] = key_score(cand[i]);
        }
        if (tid == 0) *out_n = nsel;
    }
    if (tid == 0) {
        sc->argmax_key = 0ull;
        sc->ticket = 0u;
    }
}

}  // namespace qb
