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

}  // namespace qb
