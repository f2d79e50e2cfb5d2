// api_error.cuh -- the calling thread's last-error text behind
// qwen_b200_last_error(), shared by every translation unit of the C ABI.
#pragma once
#include <cuda_runtime.h>

namespace qb {

// Record `what` (followed by the CUDA error's text when e != cudaSuccess) as
// the calling thread's last error and return `code`.
int api_fail(int code, const char* what, cudaError_t e = cudaSuccess);

}  // namespace qb
