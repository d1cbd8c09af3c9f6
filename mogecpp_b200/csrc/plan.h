// Conv plan (plan.cu): the voxels of one level sorted by their 27-tap
// neighbourhood masks, so that the 128-row tiles of the neighbour-map conv
// (conv_tc.cu) see few distinct taps, plus each tile's rows, neighbour
// lists and tap mask, laid out so that the conv stages a tile with two bulk
// copies.
#pragma once

#include <cstddef>
#include <cstdint>
#include <cuda_runtime.h>

namespace msc {

constexpr uint32_t kPlanMagic = 0x4e4c5053u;

struct PlanHeader {
    uint32_t magic;
    int32_t reserved;
    int64_t n;
};

enum PlanKind : int { PLAN_TAP_ORDER = 0 };

__host__ __device__ inline size_t plan_align(size_t v) { return (v + 255) / 256 * 256; }

constexpr int kPlanTileRows = 128;
struct PlanTiles {
    int* order;       // [n] voxel index per plan row, sorted by tap mask
    int* rows;        // [n_pad] voxel per tile row, -1 past n
    int* nbr;         // [n_pad][27] neighbour lists, -1 = missing
    uint32_t* mask;   // [n_pad / 128] tap mask of each tile
    int* sched;       // [n_pad / 128] tiles by descending cost (the conv deals them out in a snake)
};
PlanTiles plan_tiles(uint8_t* plan, int64_t n);

size_t plan_bytes(int64_t n);
size_t plan_workspace_bytes(int64_t n);
// Plans rows [0, n) of the neighbour map; indices >= n_in (n_in >= n) are
// missing taps (the sentinel).  n_in > n plans a subset of a level's rows,
// e.g. the owned rows of a z-slab whose neighbours include halo rows.
cudaError_t launch_plan_build(const int32_t* nbr, int64_t n, int64_t n_in, void* plan, void* ws, cudaStream_t st);

}  // namespace msc
