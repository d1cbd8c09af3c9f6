// GroupNorm statistics (gn.cu) for the GroupNorm residual-block variant:
// 32 groups, sample-wide, as ggml's group_norm_f32.
#pragma once

#include <cstdint>
#include <cuda_runtime.h>

namespace msc {

// Doubles in the statistics buffer for nsamples samples:
// [nsamples*32] sums | [nsamples] counts | [nsamples*32] sums of squares.
int64_t gn_stats_doubles(int nsamples);
// Adds the group sums, sums of squares and voxel counts of rows [0, n_stat)
// and checks the sample index of all n rows (MSC_DEV_BAD_COORD).  x: fp32
// [n][c], c in {64, 128}; coords: int32 [n][4], sample in field 3.
cudaError_t launch_gn_stats(const float* x, int c, const int32_t* coords, int64_t n, int64_t n_stat,
                            int nsamples, double* stats, uint32_t* status, cudaStream_t st);
// gn[b*32 + g] = {mean, 1 / sqrtf(var + eps)}.
cudaError_t launch_gn_finalize(const double* stats, int c, int nsamples, float eps, float2* gn, cudaStream_t st);

}  // namespace msc
