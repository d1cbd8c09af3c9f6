// Conv plans, built once per topology level (the refiner rebuilds topology
// every refine pass, src/sparse.cpp:443-472) and shared by every conv on it.
//
// Tap order.  The neighbour-map conv runs a 128-row tile over the
// union of its rows' taps, so a tile of rows with different neighbourhoods
// costs 27 taps of work for ~15 (surfaces) or ~6 (thin shells) taps of
// data.  Sorting the voxels by their 27-bit tap mask puts rows with equal
// or similar neighbourhoods together; the mask bits are ordered so that the
// rarest taps (corners, then edges, then faces, then the centre) decide the
// order first, and the masks are sorted in reflected Gray-code order (the
// key is the mask's position in that sequence), so neighbouring masks
// differ in one tap.  Useful fraction of a 128-row tile / a 32-row drain
// warp on the seeded sets: 0.21 / 0.21 in (b, z, y, x) order, 0.79 / 0.87
// sorted by mask, 0.83 / 0.90 in Gray order (shell_4m); 0.54 -> 0.70 ->
// 0.71 (res4_c128, 128 rows).  The stable sort keeps the (b, z, y, x) order
// among equal masks.
//
#include "common.cuh"
#include "plan.h"

#include <cub/device/device_radix_sort.cuh>

namespace msc {
namespace {

// Bit of each tap in the sort key: corners (|dx|+|dy|+|dz| = 3) take the
// high bits, then edges, faces and the centre.
struct TapBits {
    unsigned char bit[27];
};

TapBits make_tap_bits() {
    TapBits tb{};
    int next = 26;
    for (int cls = 3; cls >= 0; --cls)
        for (int t = 0; t < 27; ++t) {
            const int dx = t / 9 - 1, dy = (t / 3) % 3 - 1, dz = t % 3 - 1;
            if ((dx < 0 ? -dx : dx) + (dy < 0 ? -dy : dy) + (dz < 0 ? -dz : dz) == cls)
                tb.bit[t] = static_cast<unsigned char>(next--);
        }
    return tb;
}

__global__ void mask_keys_kernel(const int* __restrict__ nbr, int n, int n_in, TapBits tb, uint32_t* __restrict__ keys,
                                 int* __restrict__ vals) {
    const int i = blockIdx.x * blockDim.x + threadIdx.x;
    if (i >= n) return;
    uint32_t k = 0;
    const int* r = nbr + static_cast<int64_t>(i) * 27;
#pragma unroll
    for (int t = 0; t < 27; ++t)
        if (static_cast<unsigned>(__ldg(r + t)) < static_cast<unsigned>(n_in)) k |= 1u << tb.bit[t];
    // position of the mask in the reflected Gray-code sequence (prefix xor
    // from the high bit): sorted in that order, neighbouring masks differ in
    // one tap, so a tile's (and a warp's) tap union stays small
    k ^= k >> 1;
    k ^= k >> 2;
    k ^= k >> 4;
    k ^= k >> 8;
    k ^= k >> 16;
    keys[i] = k;
    vals[i] = i;
}

// One block per 128-row tile, 16 warps of 8 rows, lane t = tap t: each
// row's voxel, its neighbour list with -1 for missing taps (8 rows of loads
// in flight per warp), the tile's tap mask (ballots OR-ed in shared memory,
// one plain store per tile) and its cost, the key of the schedule:
// 4 x the tile's taps (each tap holds an accumulator slot of the whole CTA)
// + the taps of each 32-row quarter summed (a drain warp reads the slot
// only for the taps its quarter uses).  Balancing on this sum keeps the
// busiest CTA within a few per cent of the mean whether the slot or the
// quarters dominate.
constexpr int kTileListWarps = 16;
__global__ void __launch_bounds__(32 * kTileListWarps)
    tile_lists_kernel(const int* __restrict__ order, const int* __restrict__ nbr, int n, int n_in, PlanTiles T,
                      uint32_t* __restrict__ cost, int* __restrict__ tile_id) {
    constexpr int RPW = kPlanTileRows / kTileListWarps;
    constexpr int kQuarterWarps = 32 / RPW;  // warps per 32-row quarter
    __shared__ uint32_t smask, qmask[kPlanTileRows / 32];
    const int lane = threadIdx.x & 31;
    const int warp = threadIdx.x >> 5;
    if (threadIdx.x == 0) smask = 0u;
    if (threadIdx.x < kPlanTileRows / 32) qmask[threadIdx.x] = 0u;
    __syncthreads();
    const int64_t r0 = static_cast<int64_t>(blockIdx.x) * kPlanTileRows + warp * RPW;
    int v[RPW], j[RPW];
#pragma unroll
    for (int u = 0; u < RPW; ++u) v[u] = r0 + u < n ? __ldg(order + r0 + u) : -1;
#pragma unroll
    for (int u = 0; u < RPW; ++u) j[u] = (v[u] >= 0 && lane < 27) ? __ldg(nbr + static_cast<int64_t>(v[u]) * 27 + lane) : -1;
    uint32_t m = 0;
#pragma unroll
    for (int u = 0; u < RPW; ++u) {
        const bool ok = lane < 27 && static_cast<unsigned>(j[u]) < static_cast<unsigned>(n_in);
        if (lane < 27) T.nbr[(r0 + u) * 27 + lane] = ok ? j[u] : -1;
        m |= __ballot_sync(0xffffffffu, ok);
    }
    if (lane == 0) {
#pragma unroll
        for (int u = 0; u < RPW; ++u) T.rows[r0 + u] = v[u];
        if (m) {
            atomicOr(&smask, m);
            atomicOr(&qmask[warp / kQuarterWarps], m);
        }
    }
    __syncthreads();
    if (threadIdx.x == 0) {
        T.mask[blockIdx.x] = smask;
        uint32_t c = 4u * __popc(smask);
#pragma unroll
        for (int q = 0; q < kPlanTileRows / 32; ++q) c += __popc(qmask[q]);
        cost[blockIdx.x] = c;  // <= 216: 8 bits
        tile_id[blockIdx.x] = blockIdx.x;
    }
}

__global__ void plan_header_kernel(PlanHeader* h, int64_t n) {
    h->magic = kPlanMagic;
    h->reserved = 0;
    h->n = n;
}

size_t align256(size_t v) { return plan_align(v); }

int64_t tiles_of(int64_t n) { return (n + kPlanTileRows - 1) / kPlanTileRows; }

// Scratch of the two sorts: the voxels by tap key (27 bits) and the tiles by
// descending cost (8 bits).
size_t sort_temp_bytes(int64_t n) {
    size_t b_vox = 0, b_tile = 0;
    cub::DeviceRadixSort::SortPairs(nullptr, b_vox, static_cast<const uint32_t*>(nullptr),
                                    static_cast<uint32_t*>(nullptr), static_cast<const int*>(nullptr),
                                    static_cast<int*>(nullptr), static_cast<int>(n), 0, 27);
    cub::DeviceRadixSort::SortPairsDescending(nullptr, b_tile, static_cast<const uint32_t*>(nullptr),
                                              static_cast<uint32_t*>(nullptr), static_cast<const int*>(nullptr),
                                              static_cast<int*>(nullptr), static_cast<int>(tiles_of(n)), 0, 8);
    return b_vox > b_tile ? b_vox : b_tile;
}

}  // namespace

// Plan layout: PlanHeader | order [n] | tile rows [n_pad] | tile neighbour
// lists [n_pad][27] | tile masks [n_pad / 128] | tile schedule [n_pad / 128],
// each section 256-byte aligned.
PlanTiles plan_tiles(uint8_t* plan, int64_t n) {
    const int64_t np = tiles_of(n) * kPlanTileRows;
    uint8_t* p = plan + align256(sizeof(PlanHeader));
    PlanTiles t;
    t.order = reinterpret_cast<int*>(p);
    p += align256(static_cast<size_t>(n) * 4);
    t.rows = reinterpret_cast<int*>(p);
    p += align256(static_cast<size_t>(np) * 4);
    t.nbr = reinterpret_cast<int*>(p);
    p += align256(static_cast<size_t>(np) * 27 * 4);
    t.mask = reinterpret_cast<uint32_t*>(p);
    p += align256(static_cast<size_t>(tiles_of(n)) * 4);
    t.sched = reinterpret_cast<int*>(p);
    return t;
}

size_t plan_bytes(int64_t n) {
    const int64_t np = tiles_of(n) * kPlanTileRows;
    return align256(sizeof(PlanHeader)) + align256(static_cast<size_t>(n) * 4) + align256(static_cast<size_t>(np) * 4) +
           align256(static_cast<size_t>(np) * 27 * 4) + 2 * align256(static_cast<size_t>(tiles_of(n)) * 4);
}

size_t plan_workspace_bytes(int64_t n) {
    return 2 * align256(static_cast<size_t>(n) * 4) + align256(static_cast<size_t>(n) * 4) +
           align256(sort_temp_bytes(n)) + 256;
}

cudaError_t launch_plan_build(const int32_t* nbr, int64_t n, int64_t n_in, void* plan, void* ws, cudaStream_t st) {
    plan_header_kernel<<<1, 1, 0, st>>>(static_cast<PlanHeader*>(plan), n);
    if (n == 0) return cudaGetLastError();
    uint8_t* w = static_cast<uint8_t*>(ws);
    uint32_t* k_in = reinterpret_cast<uint32_t*>(w);
    w += align256(static_cast<size_t>(n) * 4);
    uint32_t* k_out = reinterpret_cast<uint32_t*>(w);
    w += align256(static_cast<size_t>(n) * 4);
    int* vals_in = reinterpret_cast<int*>(w);
    w += align256(static_cast<size_t>(n) * 4);
    size_t temp_bytes = sort_temp_bytes(n);
    const PlanTiles T = plan_tiles(static_cast<uint8_t*>(plan), n);
    const int ni = static_cast<int>(n);
    static const TapBits tb = make_tap_bits();
    const int nin = static_cast<int>(n_in);
    mask_keys_kernel<<<static_cast<unsigned>((n + 255) / 256), 256, 0, st>>>(nbr, ni, nin, tb, k_in, vals_in);
    cudaError_t e = cub::DeviceRadixSort::SortPairs(w, temp_bytes, k_in, k_out, vals_in, T.order, ni, 0, 27, st);
    if (e != cudaSuccess) return e;
    // the key and value buffers of the voxel sort are free again: tile costs
    // and ids, then the tiles sorted by descending cost (stable: equal costs
    // keep the tap order)
    const int nt = static_cast<int>(tiles_of(n));
    tile_lists_kernel<<<static_cast<unsigned>(nt), 32 * kTileListWarps, 0, st>>>(T.order, nbr, ni, nin, T, k_in,
                                                                                  vals_in);
    size_t tile_temp = temp_bytes;
    e = cub::DeviceRadixSort::SortPairsDescending(w, tile_temp, k_in, k_out, vals_in, T.sched, nt, 0, 8, st);
    if (e != cudaSuccess) return e;
    return cudaGetLastError();
}

}  // namespace msc
