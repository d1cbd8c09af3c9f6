// Conv plan (plan.cu).  Two kinds share one buffer layout:
//  * tap order (kind 0): the voxels sorted by their tap masks, so that the
//    128-row tiles of the neighbour-map conv (conv_tc.cu) see few distinct
//    taps;
//  * row cache (kind 1): Morton-ordered subtiles with per-subtile unique
//    input row lists and 16-bit neighbour slots (conv_cached.cu).
#pragma once

#include <cstddef>
#include <cstdint>
#include <cuda_runtime.h>

namespace msc {

constexpr int kPlanCap = 384;           // max distinct input rows per subtile
constexpr uint16_t kNoSlot = 0xffffu;   // missing neighbour
constexpr uint32_t kPlanMagic = 0x4e4c5053u;

struct PlanHeader {
    uint32_t magic;
    int overflow;                    // set when the pool or descriptor space ran out
    int64_t n;
    int64_t max_desc;
    int64_t pool_cap;
    unsigned long long ndesc;        // subtiles written
    unsigned long long pool_used;    // U-list entries written (each list padded to 4)
};

enum PlanKind : int { PLAN_TAP_ORDER = 0, PLAN_ROW_CACHE = 1 };

struct PlanView {
    int* perm;        // [n] voxel index per plan row (Morton order)
    int* order;       // [n] voxel index per row, sorted by tap mask (kind 0)
    int4* desc;       // [max_desc] {row_begin, u_off, rows | u_cnt << 8, tap mask}
    uint16_t* slots;  // [n][27] slot of each (plan row, tap) in its subtile's U list
    int* pool;        // U lists
};

__host__ __device__ inline size_t plan_align(size_t v) { return (v + 255) / 256 * 256; }

// Section pointers of a plan buffer for n rows and max_desc descriptors.
__host__ __device__ inline PlanView plan_view(uint8_t* plan, int64_t n, int64_t max_desc) {
    PlanView v;
    uint8_t* p = plan + plan_align(sizeof(PlanHeader));
    v.perm = reinterpret_cast<int*>(p);
    p += plan_align(static_cast<size_t>(n) * 4);
    v.desc = reinterpret_cast<int4*>(p);
    p += plan_align(static_cast<size_t>(max_desc) * 16);
    v.slots = reinterpret_cast<uint16_t*>(p);
    p += plan_align(static_cast<size_t>(n) * 27 * 2);
    v.order = reinterpret_cast<int*>(p);
    p += plan_align(static_cast<size_t>(n) * 4);
    v.pool = reinterpret_cast<int*>(p);
    return v;
}

// Tap-order plans also hold, after the sections above, the tile rows of the
// neighbour-map conv in 128-row tiles: each tile row's voxel (-1 past n),
// its neighbour list in tap order (-1 = missing) and each tile's tap mask,
// laid out so that the conv stages a tile with two bulk copies.
constexpr int kPlanTileRows = 128;
struct PlanTiles {
    int* rows;        // [n_pad] voxel per tile row, -1 past n
    int* nbr;         // [n_pad][27] neighbour lists, -1 = missing
    uint32_t* mask;   // [n_pad / 128] tap mask of each tile
};
PlanTiles plan_tiles(uint8_t* plan, int64_t n);

int64_t plan_max_desc(int64_t n);
int64_t plan_pool_cap(int64_t n);
size_t plan_bytes(int64_t n);
size_t plan_workspace_bytes(int64_t n);
cudaError_t launch_plan_build(const int32_t* coords, const int32_t* nbr, int64_t n, int kind, void* plan, void* ws,
                              uint32_t* status, cudaStream_t st);

}  // namespace msc
