// sample.cuh -- host-visible declaration of the device sampler launcher.
#pragma once
#include <cuda_runtime.h>

namespace qb {

constexpr int kSampleMax = 1024;   // candidates (the top-k limit of the lm_head kernels)

struct SampleArgs {
    const int* ids;            // candidate ids (device)
    const float* scores;       // their scores (device)
    const int* n_dev;          // device count (e.g. the lm_head's out_n), may be null
    int n;                     // candidates (the count used is min(n, *n_dev))
    float temperature;
    int top_k;
    float top_p;
    unsigned int* rng_state;   // xorshift32 state (device), updated in place; null -> ids[0]
    int* out;                  // chosen id (device); -1 for an empty list
};

// One warp on `stream`; n <= kSampleMax.
cudaError_t launch_sample_topk(const SampleArgs& a, cudaStream_t stream);

}  // namespace qb
