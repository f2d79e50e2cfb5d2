// lm_head.cuh -- host-visible declarations of the bf16 lm_head launchers.
#pragma once
#include <cstdint>
#include <cuda_runtime.h>

namespace qb {

struct LmScratch;

// bf16 lm_head scan over E [vocab][hidden] with fused greedy argmax and, for
// k > 0, top-k (k <= 1024).  with_tail selects the reference routine's
// treatment of hidden % 8 != 0 (1: lm_head_topk adds the tail, 0:
// lm_head_argmax drops it); it only matters on the generic-shape path, which
// also needs `score_buf` (vocab floats).  Results land in device memory.
cudaError_t launch_lm_head_bf16(const float* h, const uint16_t* E, int vocab, int hidden, int k,
                                int with_tail, LmScratch* scratch, unsigned int* err, float* score_buf,
                                int* out_id, int* out_ids, float* out_scores, int* out_n, cudaStream_t stream);

// Scores alone: scores[t] = the lm_head_topk order's score of row t.
cudaError_t launch_lm_scores_bf16(const float* h, const uint16_t* E, int vocab, int hidden, int with_tail,
                                  float* scores, cudaStream_t stream);

// Top-k of a materialised score vector for any 1 <= kk <= vocab (score
// descending, ties by ascending id, only scores above -FLT_MAX): out_ids /
// out_scores get the first *out_n <= kk entries.  keys / keys_alt hold vocab
// 64-bit keys each, temp topk_large_temp_bytes(vocab) bytes.
size_t topk_large_temp_bytes(int vocab);
cudaError_t launch_topk_large(const float* scores, int vocab, int kk, unsigned long long* keys,
                              unsigned long long* keys_alt, void* temp, size_t temp_bytes, int* out_ids,
                              float* out_scores, int* out_n, cudaStream_t stream);

}  // namespace qb
