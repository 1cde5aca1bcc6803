// Allocation-free dense projection (split-K tcgen05 GEMM with static scratch).
#pragma once
#include <cuda_runtime.h>

#include "kernels.h"

namespace qwen {

// Bytes of the per-device static scratch array (status word + split partials).
size_t noalloc_scratch_bytes();

// y[T][W.rows] (fp32, device) = x[T][W.k] (fp16, device) . deq(W)^T, enqueued on
// `s` and waited for. Returns 0, or -1 with a message in `error`. Performs no
// device or host allocation on success.
int project_noalloc(const QMat& W, int max_splits, const gemm_in_t* x, int T, float* y, int sm_count,
                    cudaStream_t s, char* error, size_t capacity);

}  // namespace qwen
