// Host launchers for the level-0 image topology and the refiner's per-pixel
// glue kernels (image_topo.cu).
#pragma once

#include <cstddef>
#include <cstdint>
#include <cuda_runtime.h>

namespace msc {

// Device scratch of launch_quantize_topology_z (the running min / max).
size_t quantize_z_workspace_bytes();
// factor_coord: [n][3] floats (x/z, y/z, log z); zbin: [n] int32.
cudaError_t launch_quantize_topology_z(const float* factor_coord, int64_t n, float depth_resolution, int32_t* zbin,
                                       void* ws, uint32_t* status, cudaStream_t st);
// zbin: [height * width]; coords: [n][4] (row, column, zbin, 0); nbr: [n][27].
cudaError_t launch_dense_image_level(const int32_t* zbin, int width, int height, int32_t* coords, int32_t* nbr,
                                     cudaStream_t st);
// The refiner's input rows [n][3] from factor_coord (see image_topo.cu).
cudaError_t launch_refiner_input(const float* factor_coord, int64_t n, float* feat, cudaStream_t st);
// y [rows][cout] = W [cout][c1 + c2] * [x1 | x2] + bias, wtype 0 = F32, 1 = F16.
cudaError_t launch_small_linear(const float* x1, int c1, const float* x2, int c2, int64_t rows, const void* w,
                                int wtype, int cout, const float* bias, float* y, cudaStream_t st);
cudaError_t launch_silu_inplace(float* x, int64_t n, cudaStream_t st);
// out [n][cenc] = enc [row * ew + col] for each deep voxel (row, col).
cudaError_t launch_encoder_rows(const int32_t* deep_coords, int64_t n, const float* enc, int ew, int eh, int cenc,
                                float* out, uint32_t* status, cudaStream_t st);
// factor_coord[3 i + 2] += res[i]
cudaError_t launch_logz_update(float* factor_coord, const float* res, int64_t n, cudaStream_t st);
// *differ = any(a[i] != b[i])
cudaError_t launch_keys_differ(const int32_t* a, const int32_t* b, int64_t n, int* differ, cudaStream_t st);

}  // namespace msc
