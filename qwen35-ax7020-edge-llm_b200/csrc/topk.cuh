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

// ---- warp-level top-64: a warp holds 64 keys, element i = r*32 + lane in
// register a_r.  Bitonic networks on shuffles, no block barrier.
__device__ __forceinline__ void cx_desc(unsigned long long& a, unsigned long long o, bool keep_max) {
    a = keep_max ? (a > o ? a : o) : (a < o ? a : o);
}
// Merge stages j = 32..1 of a 64-element bitonic sequence into descending order.
__device__ __forceinline__ void warp_merge64_desc(unsigned long long& a0, unsigned long long& a1) {
    const int lane = threadIdx.x & 31;
    {   // j = 32: the partner is the other register of the same lane
        const unsigned long long hi = a0 > a1 ? a0 : a1, lo = a0 > a1 ? a1 : a0;
        a0 = hi;
        a1 = lo;
    }
#pragma unroll
    for (int j = 16; j > 0; j >>= 1) {
        const unsigned long long o0 = __shfl_xor_sync(0xffffffffu, a0, j);
        const unsigned long long o1 = __shfl_xor_sync(0xffffffffu, a1, j);
        const bool low = (lane & j) == 0;   // lower index of the pair keeps the larger key
        cx_desc(a0, o0, low);
        cx_desc(a1, o1, low);
    }
}
// Sort 64 keys descending.
__device__ __forceinline__ void warp_sort64_desc(unsigned long long& a0, unsigned long long& a1) {
    const int lane = threadIdx.x & 31;
#pragma unroll
    for (int k = 2; k <= 32; k <<= 1) {
#pragma unroll
        for (int j = k >> 1; j > 0; j >>= 1) {
            const unsigned long long o0 = __shfl_xor_sync(0xffffffffu, a0, j);
            const unsigned long long o1 = __shfl_xor_sync(0xffffffffu, a1, j);
            const int i0 = lane, i1 = 32 + lane;
            cx_desc(a0, o0, ((i0 & j) == 0) == ((i0 & k) == 0));
            cx_desc(a1, o1, ((i1 & j) == 0) == ((i1 & k) == 0));
        }
    }
    // two sorted 32-halves in opposite directions form a bitonic 64-sequence
    warp_merge64_desc(a0, a1);
}
// Top 64 of two descending 64-key lists held by a warp (element i = r*32 +
// lane in register r), into (r0, r1), descending.
__device__ __forceinline__ void warp_merge_sorted64(unsigned long long& r0, unsigned long long& r1,
                                                    unsigned long long c0, unsigned long long c1) {
    const int lane = threadIdx.x & 31;
    // max(r[i], c[63 - i]) holds the top 64 as a bitonic sequence
    const unsigned long long x0 = __shfl_sync(0xffffffffu, c1, 31 - lane);
    const unsigned long long x1 = __shfl_sync(0xffffffffu, c0, 31 - lane);
    r0 = r0 > x0 ? r0 : x0;
    r1 = r1 > x1 ? r1 : x1;
    warp_merge64_desc(r0, r1);
}

// Fold 64 more keys (c0, c1: element i = r*32 + lane) into a warp's running
// top-64 (r0, r1), both descending.
__device__ __forceinline__ void warp_fold64(unsigned long long& r0, unsigned long long& r1, unsigned long long c0,
                                            unsigned long long c1) {
    warp_sort64_desc(c0, c1);
    warp_merge_sorted64(r0, r1, c0, c1);
}

// cand[w*64 .. w*64+64) hold every warp's descending top-64 (zero keys
// empty).  Writes the best `keep` (<= 64) keys of their union, descending,
// to cand[0..m) and m = min(nonzero keys, keep) to *count.  A merge tree in
// registers: at level s, warp w (a multiple of 2s) absorbs warp w + s's list
// with one bitonic merge; log2(warps) levels, one barrier each.  Needs
// kCandCap >= 64 * warps.  Called by the whole block.
__device__ inline void merge_warp_lists64(unsigned long long* cand, int* count, int keep) {
    const int nw = blockDim.x >> 5, w = threadIdx.x >> 5, lane = threadIdx.x & 31;
    __syncthreads();   // every warp's list is in place
    unsigned long long r0 = cand[w * 64 + lane], r1 = cand[w * 64 + 32 + lane];
    for (int step = 1; step < nw; step <<= 1) {
        // slot w is read at this level only by a warp that does not absorb,
        // so an absorbing warp may rewrite its own slot at once
        if ((w & (2 * step - 1)) == 0 && w + step < nw) {
            warp_merge_sorted64(r0, r1, cand[(w + step) * 64 + lane], cand[(w + step) * 64 + 32 + lane]);
            cand[w * 64 + lane] = r0;
            cand[w * 64 + 32 + lane] = r1;
        }
        __syncthreads();
    }
    if (w == 0) {
        const int nz = __popc(__ballot_sync(0xffffffffu, r0 != 0ull)) + __popc(__ballot_sync(0xffffffffu, r1 != 0ull));
        const int m = nz < keep ? nz : keep;
        if (lane < m) cand[lane] = r0;
        if (32 + lane < m) cand[32 + lane] = r1;
        if (lane == 0) *count = m;
    }
    __syncthreads();
}

// Keep the best `keep` (<= 64) of the n candidate keys in cand[0..n),
// sorted descending at cand[0..min(n, keep)): every warp folds 64-key
// chunks into its own sorted top-64, then the warps' lists are merged by
// rank.  Called by the whole block.
__device__ inline void cand_topk64(unsigned long long* cand, int* count, int keep) {
    __syncthreads();
    const int n = *count;
    const int lane = threadIdx.x & 31, w = threadIdx.x >> 5, nw = blockDim.x >> 5;
    unsigned long long r0 = 0ull, r1 = 0ull;   // running top-64, descending
    for (int base = w * 64; base < n; base += nw * 64) {
        const unsigned long long c0 = base + lane < n ? cand[base + lane] : 0ull;
        const unsigned long long c1 = base + 32 + lane < n ? cand[base + 32 + lane] : 0ull;
        warp_fold64(r0, r1, c0, c1);
    }
    __syncthreads();   // every chunk read
    cand[w * 64 + lane] = r0;
    cand[w * 64 + 32 + lane] = r1;
    merge_warp_lists64(cand, count, keep);
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
#pragma unroll 8
        for (int j = 0; j < m; j++) r += work[j] > k;
        if (r < keep) out[r] = k;
    }
    __syncthreads();
}

// End-of-CTA work for the lm_head kernels.  `cand`/`cand_count` is the CTA's
// shared buffer (cand_cap keys, >= 64 * warps + 64 and >= the next power of
// two of the grid size; with `precompacted` it already holds the
// CTA's best kk keys, descending), `work` a shared scratch area of `work_cap`
// keys that may alias the CTA's stage buffers.  `best` is this thread's
// argmax key.  Writes out_id[0] (argmax) and, for kk > 0,
// out_ids/out_scores[0..n) and *out_n.
//
// Final merge in the last CTA: with L_c the sorted list of CTA c, the
// kk-th largest key K* of the union is at least T1 = max_c L_c[kk-1] and at
// least T2 = the kk-th largest head L_c[0]; every key >= T = max(T1, T2)
// is gathered (typically ~2kk of them) and ranked.  If too many qualify
// the CTA falls back to a radix select of K* over the lists.
__device__ inline void lm_finish(LmScratch* sc, unsigned long long* cand, int cand_cap, int* cand_count,
                                 unsigned long long* work, int work_cap, unsigned long long best,
                                 int kk, int* out_id, int* out_ids, float* out_scores, int* out_n,
                                 unsigned long long* red, bool precompacted = false) {
    const int tid = threadIdx.x;
    const int lane = tid & 31, warp = tid >> 5, nwarps = blockDim.x >> 5;
    unsigned long long bm = block_max_u64(best, red);
    if (tid == 0 && bm) atomicMax(&sc->argmax_key, bm);

    if (kk > 0) {
        if (precompacted)
            __syncthreads();   // cand[0..*cand_count) already holds the CTA's best kk, descending
        else if (kk <= 64 && 64 * (int)(blockDim.x >> 5) + kk <= cand_cap)
            cand_topk64(cand, cand_count, kk);
        else
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

    // ---- last CTA: final results.  The argmax word is loaded now and stored
    // at the end, so its round trip overlaps the top-k work.
    unsigned long long amax = 0ull;
    if (tid == 0) amax = *((volatile unsigned long long*)&sc->argmax_key);
    constexpr int kPre = 8;   // keys per list read by the fast path
    if (kk > 0 && (long long)gridDim.x * (kPre + 2) <= work_cap && (((int)gridDim.x + 7) & ~7) <= cand_cap) {
        // Fast path: one round of independent L2 loads brings every list's
        // count, first kPre keys and kk-th key.  Every key >= T lies in a
        // list prefix unless some list's kPre-th key is itself >= T; only
        // then does the general path below run.
        __shared__ int s_m2;
        __shared__ int s_total2;
        __shared__ int s_spill;
        __shared__ unsigned long long s_t2;
        const int G = gridDim.x;
        constexpr int E = kPre + 1;   // entries per list: prefix, then the kk-th key
        int* s_counts = reinterpret_cast<int*>(work + (size_t)G * E);
        if (tid == 0) {
            s_m2 = 0;
            s_total2 = 0;
            s_spill = 0;
            s_t2 = 0ull;
        }
        const int total_ent = G * E;
        // the counts ride in the same round of loads as the list entries
        int cnt = 0;
        if (tid < G) cnt = __ldcg(sc->counts + tid);
        for (int base = tid; base < total_ent; base += 8 * blockDim.x) {
            unsigned long long v[8];
#pragma unroll
            for (int u = 0; u < 8; u++) {
                const int idx = base + u * blockDim.x;
                v[u] = 0ull;
                if (idx < total_ent) {
                    const int c = idx / E, e = idx - c * E;
                    const int pos = e < kPre ? e : kk - 1;
                    if (pos < kk) v[u] = __ldcg(sc->lists + (size_t)c * kk + pos);
                }
            }
#pragma unroll
            for (int u = 0; u < 8; u++) {
                const int idx = base + u * blockDim.x;
                if (idx < total_ent) work[idx] = v[u];
            }
        }
        if (tid < G) s_counts[tid] = cnt;
        for (int c = tid + blockDim.x; c < G; c += blockDim.x) s_counts[c] = __ldcg(sc->counts + c);
        __syncthreads();
        for (int idx = tid; idx < total_ent; idx += blockDim.x) {   // drop entries past each list's count
            const int c = idx / E, e = idx - c * E;
            const int pos = e < kPre ? e : kk - 1;
            if (pos >= s_counts[c]) work[idx] = 0ull;
        }
        __syncthreads();
        // T1 = best kk-th key of a full list, T2 = kk-th largest head
        unsigned long long t1 = 0ull;
        int tot = 0;
        for (int c = tid; c < G; c += blockDim.x) {
            cand[c] = work[(size_t)c * E];
            const unsigned long long last = work[(size_t)c * E + kPre];
            t1 = last > t1 ? last : t1;
            tot += s_counts[c];
        }
        for (int o = 16; o > 0; o >>= 1) tot += __shfl_xor_sync(0xffffffffu, tot, o);
        if (lane == 0) atomicAdd(&s_total2, tot);
        t1 = block_max_u64(t1, red);   // contains barriers (cand heads visible after it)
        for (int i = G + tid; i < ((G + 7) & ~7); i += blockDim.x) cand[i] = 0ull;   // pad to 8 heads
        __syncthreads();
        for (int c = tid; c < G; c += blockDim.x) {
            const unsigned long long hd = cand[c];
            if (hd == 0ull) continue;
            int r = 0;
            for (int o0 = 0; o0 < G; o0 += 8) {   // 8 heads per round, loads issued together
                unsigned long long v[8];
#pragma unroll
                for (int u = 0; u < 8; u++) v[u] = cand[o0 + u];
#pragma unroll
                for (int u = 0; u < 8; u++) r += v[u] > hd;
            }
            if (r == kk - 1) s_t2 = hd;
        }
        __syncthreads();
        const unsigned long long T = t1 > s_t2 ? t1 : s_t2;
        const int total = s_total2;
        const int want = total < kk ? total : kk;
        __syncthreads();
        // gather the prefix keys >= T; flag lists whose prefix may not hold all of theirs
        for (int idx = tid; idx < G * kPre; idx += blockDim.x) {
            const int c = idx / kPre, e = idx - c * kPre;
            const unsigned long long key = work[(size_t)c * E + e];
            if (key != 0ull && key >= T) {
                const int p = atomicAdd(&s_m2, 1);
                if (p < cand_cap) cand[p] = key;
                if (e == kPre - 1 && s_counts[c] > kPre) s_spill = 1;
            }
        }
        __syncthreads();
        const int m = s_m2;
        if (!s_spill && m <= cand_cap && m <= work_cap) {
            rank_place(cand, m, want, work);   // work is free again
            for (int i = tid; i < want; i += blockDim.x) {
                out_ids[i] = key_id(work[i]);
                out_scores[i] = key_score(work[i]);
            }
            if (tid == 0) *out_n = want;
            kk = 0;   // done: skip the general path below
        }
        __syncthreads();
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
                        if (p < cand_cap) cand[p] = key;
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
        *out_id = amax ? key_id(amax) : 0;
        sc->argmax_key = 0ull;
        sc->ticket = 0u;
    }
}

}  // namespace qb
