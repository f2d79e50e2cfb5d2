// sample.cu -- temperature / top-k / top-p sampling from a device candidate
// list (the fused lm_head top-k), so the chosen token never crosses to the
// host.  The procedure and operation order are the reference sampler's
// (04-板载脚本与工具/qwen_sampling.c:411-529):
//   sort check (and a sort by score desc, id asc if needed); greedy when
//   !(T >= 1e-6); m = min(n, top_k); maxf over the first m (strict '>');
//   e_i = expf((s_i - maxf) * (1/T)); sum_all = sum of e_i in order (double);
//   keep = first i with cum += e_i / sum_all > clamp(top_p, 0, 1), plus one;
//   sum_keep over the kept prefix; u = (xorshift32 >> 8) * 2^-24;
//   r = u * sum_keep; chosen = first i with r < cumulative e_i.
// The float and double steps are the same IEEE operations as the reference;
// expf is CUDA's (the reference links its C library's, which is not correctly
// rounded either), so a draw within a few ulps of a bucket boundary may pick
// the neighbouring candidate.  The xorshift32 state advances bit-exactly.
#include <cstdint>
#include <cuda_runtime.h>

#include "sample.cuh"

namespace qb {
namespace {

__device__ __forceinline__ unsigned int xorshift32(unsigned int* st) {
    unsigned int x = *st;
    if (x == 0u) x = 0x9E3779B9u;   // a zero state is remapped (qwen_sampling.c:360-368)
    x ^= x << 13;
    x ^= x >> 17;
    x ^= x << 5;
    *st = x;
    return x;
}

// Candidate i orders before j: score descending, then id ascending (the
// reference's qsort comparator).
__device__ __forceinline__ bool before(float si, int ii, float sj, int ij) {
    return si > sj || (!(si < sj) && ii < ij);
}

__global__ void __launch_bounds__(32) sample_topk_kernel(const __grid_constant__ SampleArgs A) {
    __shared__ int s_id[kSampleMax], t_id[kSampleMax];
    __shared__ float s_sc[kSampleMax], t_sc[kSampleMax];
    __shared__ float s_e[kSampleMax];
    const unsigned full = 0xffffffffu;
    const int lane = threadIdx.x;
    int n = A.n;
    if (A.n_dev) n = min(n, *A.n_dev);
    if (n <= 0) {
        if (lane == 0) *A.out = -1;
        return;
    }
    for (int i = lane; i < n; i += 32) {
        s_id[i] = A.ids[i];
        s_sc[i] = A.scores[i];
    }
    __syncwarp();
    if (!A.rng_state) {
        if (lane == 0) *A.out = s_id[0];
        return;
    }
    bool unsorted = false;
    for (int i = 1 + lane; i < n; i += 32) unsorted |= s_sc[i] > s_sc[i - 1];
    if (__any_sync(full, unsorted)) {
        // rank sort: an element's place is the number of elements before it
        // (distinct ids make the order total unless a score is NaN, where
        // the reference's comparator is not an order either)
        for (int i = lane; i < n; i += 32) {
            t_id[i] = 0;
            t_sc[i] = 0.0f;
        }
        __syncwarp();
        for (int i = lane; i < n; i += 32) {
            const float si = s_sc[i];
            const int ii = s_id[i];
            int r = 0;
            for (int j = 0; j < n; j++) r += before(s_sc[j], s_id[j], si, ii) ? 1 : 0;
            t_id[r] = ii;
            t_sc[r] = si;
        }
        __syncwarp();
        for (int i = lane; i < n; i += 32) {
            s_id[i] = t_id[i];
            s_sc[i] = t_sc[i];
        }
        __syncwarp();
    }
    const float temperature = A.temperature;
    if (!(temperature >= 1e-6f)) {
        if (lane == 0) *A.out = s_id[0];
        return;
    }
    int m = n;
    if (A.top_k > 0 && A.top_k < m) m = A.top_k;
    // maxf: the sequential strict-'>' scan from s[0] gives s[0] when it is
    // NaN and the largest non-NaN score otherwise (the sign of a zero maximum
    // does not change any exponent below)
    float best = -__int_as_float(0x7f800000);
    for (int i = lane; i < m; i += 32)
        if (s_sc[i] > best) best = s_sc[i];
#pragma unroll
    for (int o = 16; o > 0; o >>= 1) {
        const float b = __shfl_xor_sync(full, best, o);
        if (b > best) best = b;
    }
    const float s0 = s_sc[0];
    const float maxf = (s0 != s0) ? s0 : (best > s0 ? best : s0);
    const float inv_t = __fdiv_rn(1.0f, temperature);
    for (int i = lane; i < m; i += 32) s_e[i] = expf(__fmul_rn(__fsub_rn(s_sc[i], maxf), inv_t));
    __syncwarp();
    if (lane != 0) return;
    double sum_all = 0.0;
    for (int i = 0; i < m; i++) sum_all = __dadd_rn(sum_all, (double)s_e[i]);
    if (!(sum_all > 0.0)) {
        *A.out = s_id[0];
        return;
    }
    float p_thresh = A.top_p;
    if (!(p_thresh > 0.0f)) p_thresh = 0.0f;
    if (p_thresh > 1.0f) p_thresh = 1.0f;
    int keep = m;
    double cum = 0.0;
    for (int i = 0; i < m; i++) {
        cum = __dadd_rn(cum, __ddiv_rn((double)s_e[i], sum_all));
        if (cum > (double)p_thresh) {
            keep = i + 1;
            break;
        }
    }
    double sum_keep = 0.0;
    for (int i = 0; i < keep; i++) sum_keep = __dadd_rn(sum_keep, (double)s_e[i]);
    if (!(sum_keep > 0.0)) {
        *A.out = s_id[0];
        return;
    }
    unsigned int st = *A.rng_state;
    const float uf = __fmul_rn((float)(xorshift32(&st) >> 8), 1.0f / 16777216.0f);
    *A.rng_state = st;
    const double r = __dmul_rn((double)uf, sum_keep);
    int chosen = keep - 1;
    cum = 0.0;
    for (int i = 0; i < keep; i++) {
        cum = __dadd_rn(cum, (double)s_e[i]);
        if (r < cum) {
            chosen = i;
            break;
        }
    }
    *A.out = s_id[chosen];
}

}  // namespace

cudaError_t launch_sample_topk(const SampleArgs& a, cudaStream_t stream) {
    if (!a.ids || !a.scores || !a.out || a.n < 0 || a.n > kSampleMax) return cudaErrorInvalidValue;
    sample_topk_kernel<<<1, 32, 0, stream>>>(a);
    return cudaGetLastError();
}

}  // namespace qb
