// Host launchers for the stride-2 transition kernels (ops.cu).
#pragma once

#include <cstdint>
#include <cuda_runtime.h>

namespace msc {

// pooled: [np][c] fp32
cudaError_t launch_pool_mean(const void* x, int x_dtype, int64_t nfine, int c, const int32_t* pool_rows,
                             const float* inv_count, int64_t np, float* pooled, uint32_t* status, cudaStream_t st);
// y[i] = t[rows[i]] (+ skip[i]); t: [nsrc][c] fp32
cudaError_t launch_gather_rows(const float* t, int64_t nsrc, int c, const int32_t* rows, int64_t n, const void* skip,
                               int skip_dtype, void* y, int y_dtype, uint32_t* status, cudaStream_t st);

}  // namespace msc
