// Host launchers for the topology kernels (topology.cu).
#pragma once

#include <cstddef>
#include <cstdint>
#include <cuda_runtime.h>

namespace msc {

// Device scratch needed by launch_make_level / launch_downsample for n voxels.
size_t topology_workspace_bytes(int64_t n);

// coords: [n][4] int32 (x, y, z, b), 16-byte aligned.  nbr: [n][27] int32.
cudaError_t launch_make_level(const int32_t* coords, int64_t n, int32_t* nbr, void* ws, uint32_t* status,
                              cudaStream_t st);

// Bytes of the hash table make_level uses for n voxels, and make_level with
// that table supplied directly (table_bytes >= topology_table_bytes(n)).
size_t topology_table_bytes(int64_t n);
cudaError_t launch_make_level_in_table(const int32_t* coords, int64_t n, int32_t* nbr, void* table,
                                       size_t table_bytes, uint32_t* status, cudaStream_t st);

// parent: [n][4] capacity; np_dev: one device int32; pool_rows: [8][n]
// capacity (written slot-major with stride np); inv_count, up_rows: [n].
cudaError_t launch_downsample(const int32_t* coords, int64_t n, int32_t* parent, int32_t* np_dev, int32_t* pool_rows,
                              float* inv_count, int32_t* up_rows, void* ws, uint32_t* status, cudaStream_t st);

// Both of the above for one set of voxels, the brick table built once
// (the neighbour map and the stride-2 maps of a pyramid level).
cudaError_t launch_make_level_downsample(const int32_t* coords, int64_t n, int32_t* nbr, int32_t* parent,
                                         int32_t* np_dev, int32_t* pool_rows, float* inv_count, int32_t* up_rows,
                                         void* ws, uint32_t* status, cudaStream_t st);

// Octant maps of a stride-2 transition (pool_rows [8][np], up_rows
// [nfine]): down [np][27] (column o = the child at octant o, else nfine) and
// up [nfine][27] (column oct(c) = c's parent, else np).
cudaError_t launch_octant_maps(const int32_t* coords, int64_t nfine, const int32_t* pool_rows,
                               const int32_t* up_rows, int64_t np, int32_t* down, int32_t* up, cudaStream_t st);

}  // namespace msc
