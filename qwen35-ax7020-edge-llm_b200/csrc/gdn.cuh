// gdn.cuh -- host-visible declarations of the Gated-DeltaNet layer glue and
// the token loop's small kernels (qwen_kernels_opt.c:507-858, 1008-1049).
#pragma once
#include <cstdint>
#include <cuda_runtime.h>

namespace qb {

constexpr int kGdnHeadDim = 128;    // the recurrent state of a head is kGdnHeadDim x kGdnHeadDim
constexpr int kGdnMaxHidden = 6144;

// One Gated-DeltaNet step of a linear-attention layer, everything between
// the qkv / z projections and the out projection, one CTA per head:
//   conv1d + SiLU over the head's q, k and v channels (the conv state
//   shifts), q / k l2-normalised, the head's gates alpha / beta from
//   `normed` (the layer's rmsnorm(h, in_ln_w), stored by the qkv projection
//   launch), the recurrent step (the state is updated in place),
//   rmsnorm_gated with z -> out.
// Arithmetic and order are the reference's NEON build; alpha, beta and the
// SiLU of z use CUDA's expf / log1pf where the reference calls the C
// library's.  Layouts are the reference's: qkv = q | k | v (heads * 128
// channels each), conv_w [3 * heads * 128][4], conv_s three rows of
// 3 * heads * 128 floats, state [heads][128 * 128] blocked so that S[i][j]
// sits at ((j/4 * 32 + i/4) * 4 + j%4) * 4 + i%4, wa / wb [heads][hidden].
struct GdnArgs {
    const float* qkv;
    const float* z;
    const float* normed;
    const float* conv_w;
    float* conv_s;
    const float* wa;
    const float* wb;
    const float* nea;
    const float* dt;
    float* state;
    const float* norm_w;
    float* out;
    int heads, hidden;
};
cudaError_t launch_gdn_layer(const GdnArgs& a, cudaStream_t stream);

// h[0..hidden) = the bf16 row `row` of E, widened to fp32.
cudaError_t launch_embed_row(float* h, const uint16_t* E, long long row, int hidden, cudaStream_t stream);

// y = rmsnorm(x, w, eps), the reference's NEON build (four flushed lane sums
// of x*x, r = 1/sqrtf(sum/n + eps), x * (r * (1 + w))); n % 4 == 0, n <= 6144.
cudaError_t launch_rmsnorm(float* y, const float* x, const float* w, int n, float eps, cudaStream_t stream);

}  // namespace qb
