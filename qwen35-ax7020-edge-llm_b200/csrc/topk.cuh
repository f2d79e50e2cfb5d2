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
//   3. the CTA with the last ticket selects the kk largest keys of the
//      union (see lm_finish), writes ids / scores, then clears the ticket and
//      the argmax word for the next launch.
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

// Scatter the keys of work[0..m) (distinct) by descending rank into
// out[0..min(m, keep)), by counting, O(m^2 / threads).  Ends with a barrier.
__device__ inline void rank_place(const unsigned long long* work, int m, int keep, unsigned long long* out) {
    for (int i = threadIdx.x; i < m; i += blockDim.x) {
        const unsigned long long k = work[i];
        int r = 0;
        for (int j = 0; j < m; j++) r += work[j] > k;
        if (r < keep) out[r] = k;
    }
    __syncthreads();
}

// End-of-CTA work for the lm_head kernels.  `cand`/`cand_count` is the CTA's
// shared buffer (kCandCap keys), `work` a shared scratch area of `work_cap`
// keys that may alias the CTA's stage buffers.  `best` is this thread's
// argmax key.  Writes out_id[0] (argmax) and, for kk > 0,
// out_ids/out_scores[0..n) and *out_n.
//
// Final merge in the last CTA: with L_c the sorted list of CTA c, the
// kk-th largest key K* of the union is at least T1 = max_c L_c[kk-1] and at
// least T2 = the kk-th largest head L_c[0]; every key >= T = max(T1, T2)
// is gathered (typically ~2kk of them) and ranked.  If too many qualify
// the CTA falls back to a radix select of K* over the lists.
__device__ inline void lm_finish(LmScratch* sc, unsigned long long* cand, int* cand_count,
                                 unsigned long long* work, int work_cap, unsigned long long best,
                                 int kk, int* out_id, int* out_ids, float* out_scores, int* out_n,
                                 unsigned long long* red) {
    const int tid = threadIdx.x;
    const int lane = tid & 31, warp = tid >> 5, nwarps = blockDim.x >> 5;
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
        __shared__ int s_m;
        __shared__ int s_total;
        const int G = gridDim.x;
        const volatile int* counts = sc->counts;
        const volatile unsigned long long* lists = sc->lists;
        // thresholds: heads into cand[0..pow2(G)), kth keys reduced
        const int gp = next_pow2(G);
        unsigned long long t1 = 0ull;
        int tot = 0;
        for (int c = tid; c < gp; c += blockDim.x) {
            int n = c < G ? counts[c] : 0;
            cand[c] = n > 0 ? lists[(size_t)c * kk] : 0ull;
            if (n == kk) {
                unsigned long long v = lists[(size_t)c * kk + kk - 1];
                t1 = v > t1 ? v : t1;
            }
            tot += n;
        }
        for (int o = 16; o > 0; o >>= 1) tot += __shfl_xor_sync(0xffffffffu, tot, o);
        if (tid == 0) s_total = 0;
        __syncthreads();
        if (lane == 0) atomicAdd(&s_total, tot);
        t1 = block_max_u64(t1, red);   // contains barriers
        block_sort_desc(cand, gp);
        const unsigned long long t2 = (kk <= G) ? cand[kk - 1] : 0ull;
        const unsigned long long T = t1 > t2 ? t1 : t2;
        const int total = s_total;
        const int want = total < kk ? total : kk;
        // gather keys >= T (lists are sorted: each warp walks one list)
        if (tid == 0) s_m = 0;
        __syncthreads();
        for (int c = warp; c < G; c += nwarps) {
            const int n = counts[c];
            for (int i = lane; i < n; i += 32) {
                const unsigned long long key = lists[(size_t)c * kk + i];
                const bool take = key >= T;
                if (take) {
                    int p = atomicAdd(&s_m, 1);
                    if (p < work_cap) work[p] = key;
                }
                if (!__any_sync(__activemask(), take)) break;
            }
        }
        __syncthreads();
        const int m = s_m;
        if (m <= work_cap) {
            if (m <= 1024) {
                rank_place(work, m, want, cand);
            } else {
                const int p2 = next_pow2(m);
                for (int i = m + tid; i < p2; i += blockDim.x) work[i] = 0ull;
                __syncthreads();
                if (p2 <= work_cap) {
                    block_sort_desc(work, p2);
                    for (int i = tid; i < want; i += blockDim.x) cand[i] = work[i];
                    __syncthreads();
                } else {
                    rank_place(work, m, want, cand);
                }
            }
        } else {
            // radix select of the want-th largest key over the lists, with
            // warp-private histograms (work area reused)
            unsigned int* hist = reinterpret_cast<unsigned int*>(work);   // [nwarps][256]
            __shared__ unsigned long long s_prefix;
            __shared__ int s_rem;
            if (tid == 0) {
                s_prefix = 0ull;
                s_rem = want;
            }
            __syncthreads();
            for (int pass = 0; pass < 8; pass++) {
                const int shift = 56 - 8 * pass;
                for (int i = tid; i < nwarps * 256; i += blockDim.x) hist[i] = 0u;
                __syncthreads();
                const unsigned long long pre = s_prefix;
                for (int c = warp; c < G; c += nwarps) {
                    const int n = counts[c];
                    for (int i = lane; i < n; i += 32) {
                        const unsigned long long key = lists[(size_t)c * kk + i];
                        if (pass == 0 || (key >> (shift + 8)) == pre)
                            atomicAdd(&hist[warp * 256 + ((key >> shift) & 0xFFull)], 1u);
                    }
                }
                __syncthreads();
                if (tid == 0) {
                    int rem = s_rem;
                    unsigned int cum = 0;
                    int d = 255;
                    for (; d > 0; d--) {
                        unsigned int h = 0;
                        for (int w = 0; w < nwarps; w++) h += hist[w * 256 + d];
                        if ((int)(cum + h) >= rem) break;
                        cum += h;
                    }
                    s_rem = rem - (int)cum;
                    s_prefix = (pre << 8) | (unsigned long long)d;
                }
                __syncthreads();
            }
            const unsigned long long kstar = s_prefix;
            if (tid == 0) s_m = 0;
            __syncthreads();
            for (int c = warp; c < G; c += nwarps) {
                const int n = counts[c];
                for (int i = lane; i < n; i += 32) {
                    const unsigned long long key = lists[(size_t)c * kk + i];
                    if (key >= kstar) {
                        int p = atomicAdd(&s_m, 1);
                        if (p < kTopkMax) cand[p] = key;
                    }
                }
            }
            __syncthreads();
            const int p2 = next_pow2(want < 1 ? 1 : want);
            for (int i = want + tid; i < p2; i += blockDim.x) cand[i] = 0ull;
            __syncthreads();
            block_sort_desc(cand, p2);
        }
        for (int i = tid; i < want; i += blockDim.x) {
            out_ids[i] = key_id(cand[i]);
            out_scores[i] = key_score(cand[i]);
        }
        if (tid == 0) *out_n = want;
    }
    if (tid == 0) {
        sc->argmax_key = 0ull;
        sc->ticket = 0u;
    }
}

}  // namespace qb
