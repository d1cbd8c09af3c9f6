// Conv plans, built once per topology level (the refiner rebuilds topology
// every refine pass, src/sparse.cpp:443-472) and shared by every conv on it.
//
// Tap order (kind 0).  The neighbour-map conv runs a 128-row tile over the
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
// Row cache (kind 1): a tiling that lets the conv load each input row once
// per tile instead of once per (tile row, tap).
//
//  1. Voxels are ordered along a Morton curve of (x, y, z) within each sample
//     (key = b << 48 | interleaved low 16 bits of x, y, z), so consecutive
//     voxels are spatial neighbours.
//  2. The order is cut into blocks of 128 rows.  A block becomes one subtile
//     of 128 rows, or 2, 4, 8 or 16 subtiles of 64..8 rows, the largest size
//     whose every subtile references at most kPlanCap distinct input rows
//     (its neighbours over all 27 taps).
//  3. Each subtile records its distinct input rows ("U list") and, per row and
//     tap, the 16-bit position of the neighbour in that list (0xFFFF = none).
//
// Plan layout (one device buffer, see plan.h):
//   PlanHeader | perm [n] int32 | desc [max_desc] int4 {row_begin, u_off,
//   rows | u_cnt << 8, tap mask} | slots [n][27] uint16 (plan order) |
//   pool [pool_cap] int32
// Subtiles start at multiples of 8 rows and U lists at multiples of 4
// entries, so a subtile's slots, rows and U list are 16-byte aligned for
// the conv's asynchronous copies.
// Descriptors and U lists are placed by atomic counters, so their order is
// not deterministic; the conv's arithmetic depends only on a subtile's rows
// and row_begin, so results are.
#include "common.cuh"
#include "plan.h"

#include <cub/device/device_radix_sort.cuh>

namespace msc {
namespace {

constexpr int kBlockRows = 128;
constexpr int kHashSize = 8192;  // open addressing over <= 128*27 entries
constexpr int kPlanThreads = 256;

__device__ __forceinline__ uint64_t spread3(uint32_t v) {
    // interleave the low 16 bits of v with two zero bits between them
    uint64_t x = v & 0xffffu;
    x = (x | (x << 32)) & 0x1f00000000ffffull;
    x = (x | (x << 16)) & 0x1f0000ff0000ffull;
    x = (x | (x << 8)) & 0x100f00f00f00f00full;
    x = (x | (x << 4)) & 0x10c30c30c30c30c3ull;
    x = (x | (x << 2)) & 0x1249249249249249ull;
    return x;
}

__global__ void morton_keys_kernel(const int4* __restrict__ coords, int n, uint64_t* __restrict__ keys,
                                   int* __restrict__ vals) {
    const int i = blockIdx.x * blockDim.x + threadIdx.x;
    if (i >= n) return;
    const int4 c = __ldg(coords + i);
    keys[i] = (static_cast<uint64_t>(c.w & 0x7f) << 48) | spread3(static_cast<uint32_t>(c.x)) |
              (spread3(static_cast<uint32_t>(c.y)) << 1) | (spread3(static_cast<uint32_t>(c.z)) << 2);
    vals[i] = i;
}

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

__global__ void mask_keys_kernel(const int* __restrict__ nbr, int n, TapBits tb, uint32_t* __restrict__ keys,
                                 int* __restrict__ vals) {
    const int i = blockIdx.x * blockDim.x + threadIdx.x;
    if (i >= n) return;
    uint32_t k = 0;
    const int* r = nbr + static_cast<int64_t>(i) * 27;
#pragma unroll
    for (int t = 0; t < 27; ++t)
        if (static_cast<unsigned>(__ldg(r + t)) < static_cast<unsigned>(n)) k |= 1u << tb.bit[t];
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
// in flight per warp), and the tile's tap mask (ballots OR-ed in shared
// memory, one plain store per tile).
constexpr int kTileListWarps = 16;
__global__ void __launch_bounds__(32 * kTileListWarps)
    tile_lists_kernel(const int* __restrict__ order, const int* __restrict__ nbr, int n, PlanTiles T) {
    constexpr int RPW = kPlanTileRows / kTileListWarps;
    __shared__ uint32_t smask;
    const int lane = threadIdx.x & 31;
    const int warp = threadIdx.x >> 5;
    if (threadIdx.x == 0) smask = 0u;
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
        const bool ok = lane < 27 && static_cast<unsigned>(j[u]) < static_cast<unsigned>(n);
        if (lane < 27) T.nbr[(r0 + u) * 27 + lane] = ok ? j[u] : -1;
        m |= __ballot_sync(0xffffffffu, ok);
    }
    if (lane == 0) {
#pragma unroll
        for (int u = 0; u < RPW; ++u) T.rows[r0 + u] = v[u];
        if (m) atomicOr(&smask, m);
    }
    __syncthreads();
    if (threadIdx.x == 0) T.mask[blockIdx.x] = smask;
}

__global__ void plan_header_kernel(PlanHeader* h, int64_t n, int64_t max_desc, int64_t pool_cap) {
    h->magic = kPlanMagic;
    h->n = n;
    h->max_desc = max_desc;
    h->pool_cap = pool_cap;
    h->ndesc = 0;
    h->pool_used = 0;
    h->overflow = 0;
}

// Inserts key (>= 0) into the shared hash; returns its slot in the subtile's
// U list, assigning the next free slot on first insert.
__device__ __forceinline__ int hash_insert(int* hkeys, int* hslot, int* counter, int* ulist, int key) {
    uint32_t h = (static_cast<uint32_t>(key) * 2654435761u) >> (32 - 13);
    for (int probe = 0; probe < kHashSize; ++probe) {
        const int prev = atomicCAS(&hkeys[h], -1, key);
        if (prev == -1) {
            const int s = atomicAdd(counter, 1);
            if (s < kPlanCap) ulist[s] = key;
            // publish the slot; readers spin until it is set (bounded)
            atomicExch(&hslot[h], s);
            return s;
        }
        if (prev == key) {
            int s = -1;
            for (int it = 0; it < (1 << 20) && s < 0; ++it) s = atomicAdd(&hslot[h], 0);
            return s;
        }
        h = (h + 1) & (kHashSize - 1);
    }
    return -1;
}

constexpr int kSubtileSmem = (kBlockRows * 27 + 2 * kHashSize + kPlanCap) * 4;

__global__ void __launch_bounds__(kPlanThreads) subtile_kernel(const int* __restrict__ perm,
                                                              const int* __restrict__ nbr, int n,
                                                              uint8_t* __restrict__ plan, uint32_t* status) {
    extern __shared__ int smem_i[];
    int* s_nbr = smem_i;                      // [kBlockRows*27]
    int* hkeys = s_nbr + kBlockRows * 27;     // [kHashSize]
    int* hslot = hkeys + kHashSize;           // [kHashSize]
    int* ulist = hslot + kHashSize;           // [kPlanCap]
    __shared__ int counter, ok, size, base_off;
    __shared__ unsigned tap_mask;
    PlanHeader* hdr = reinterpret_cast<PlanHeader*>(plan);
    PlanView P = plan_view(plan, hdr->n, hdr->max_desc);
    const int r0 = blockIdx.x * kBlockRows;
    const int nr = min(kBlockRows, n - r0);
    for (int e = threadIdx.x; e < nr * 27; e += kPlanThreads) {
        const int r = e / 27, t = e % 27;
        const int j = __ldg(nbr + static_cast<int64_t>(__ldg(perm + r0 + r)) * 27 + t);
        s_nbr[e] = (static_cast<unsigned>(j) < static_cast<unsigned>(n)) ? j : -1;
    }
    if (threadIdx.x == 0) size = kBlockRows;
    __syncthreads();
    // choose the largest subtile size whose subtiles all fit the cap
    for (;;) {
        const int s = size;
        if (threadIdx.x == 0) ok = 1;
        __syncthreads();
        for (int sub = 0; sub * s < nr; ++sub) {
            for (int e = threadIdx.x; e < kHashSize; e += kPlanThreads) {
                hkeys[e] = -1;
                hslot[e] = -1;
            }
            if (threadIdx.x == 0) counter = 0;
            __syncthreads();
            const int rb = sub * s, re = min(nr, rb + s);
            for (int e = rb * 27 + threadIdx.x; e < re * 27; e += kPlanThreads)
                if (s_nbr[e] >= 0) hash_insert(hkeys, hslot, &counter, ulist, s_nbr[e]);
            __syncthreads();
            if (threadIdx.x == 0 && counter > kPlanCap) ok = 0;
            __syncthreads();
            if (!ok) break;
        }
        if (ok || s <= 8) break;
        __syncthreads();
        if (threadIdx.x == 0) size = s / 2;
        __syncthreads();
    }
    if (!ok) {  // cannot happen: 8 rows x 27 taps <= kPlanCap
        if (threadIdx.x == 0) set_status(status, MSC_DEV_PLAN_OVERFLOW);
        return;
    }
    // emit the subtiles
    const int s = size;
    for (int sub = 0; sub * s < nr; ++sub) {
        for (int e = threadIdx.x; e < kHashSize; e += kPlanThreads) {
            hkeys[e] = -1;
            hslot[e] = -1;
        }
        if (threadIdx.x == 0) {
            counter = 0;
            tap_mask = 0;
        }
        __syncthreads();
        const int rb = sub * s, re = min(nr, rb + s);
        unsigned m = 0;
        for (int e = rb * 27 + threadIdx.x; e < re * 27; e += kPlanThreads) {
            const int j = s_nbr[e];
            const int slot = j >= 0 ? hash_insert(hkeys, hslot, &counter, ulist, j) : -1;
            if (j >= 0 && slot < 0) set_status(status, MSC_DEV_TIMEOUT);
            if (slot >= 0) m |= 1u << (e % 27);
            P.slots[static_cast<int64_t>(r0) * 27 + e] = slot >= 0 ? static_cast<uint16_t>(slot) : kNoSlot;
        }
        if (m) atomicOr(&tap_mask, m);
        __syncthreads();
        if (threadIdx.x == 0) {
            const int u = counter;
            const unsigned long long off = atomicAdd(reinterpret_cast<unsigned long long*>(&hdr->pool_used),
                                                     static_cast<unsigned long long>((u + 3) & ~3));
            const unsigned long long d =
                atomicAdd(reinterpret_cast<unsigned long long*>(&hdr->ndesc), 1ull);
            if (off + ((u + 3) & ~3) > static_cast<unsigned long long>(hdr->pool_cap) ||
                d >= static_cast<unsigned long long>(hdr->max_desc)) {
                atomicExch(&hdr->overflow, 1);
                set_status(status, MSC_DEV_PLAN_OVERFLOW);
                base_off = -1;
            } else {
                base_off = static_cast<int>(off);
                P.desc[d] = make_int4(r0 + rb, static_cast<int>(off), (re - rb) | (u << 8),
                                      static_cast<int>(tap_mask));
            }
        }
        __syncthreads();
        if (base_off >= 0)
            for (int e = threadIdx.x; e < counter; e += kPlanThreads) P.pool[base_off + e] = ulist[e];
        __syncthreads();
    }
}

size_t align256(size_t v) { return plan_align(v); }

size_t sort_temp_bytes(int64_t n) {
    size_t b64 = 0, b32 = 0;
    cub::DeviceRadixSort::SortPairs(nullptr, b64, static_cast<const uint64_t*>(nullptr),
                                    static_cast<uint64_t*>(nullptr), static_cast<const int*>(nullptr),
                                    static_cast<int*>(nullptr), static_cast<int>(n), 0, 55);
    cub::DeviceRadixSort::SortPairs(nullptr, b32, static_cast<const uint32_t*>(nullptr),
                                    static_cast<uint32_t*>(nullptr), static_cast<const int*>(nullptr),
                                    static_cast<int*>(nullptr), static_cast<int>(n), 0, 27);
    return b64 > b32 ? b64 : b32;
}

}  // namespace

int64_t plan_max_desc(int64_t n) { return 16 * ((n + kBlockRows - 1) / kBlockRows) + 16; }
// Sum of U-list lengths: 2.2-2.8 per voxel on surfaces and solids (at most 27,
// since a row is listed by at most the subtiles of its 27 neighbours).
// (+ up to 3 entries of padding per subtile).
int64_t plan_pool_cap(int64_t n) { return 8 * n + 4 * plan_max_desc(n) + 65536; }

namespace {
size_t plan_base_bytes(int64_t n) {
    return align256(sizeof(PlanHeader)) + align256(static_cast<size_t>(n) * 4) +
           align256(static_cast<size_t>(plan_max_desc(n)) * 16) + align256(static_cast<size_t>(n) * 27 * 2) +
           align256(static_cast<size_t>(n) * 4) + align256(static_cast<size_t>(plan_pool_cap(n)) * 4);
}
int64_t tiles_of(int64_t n) { return (n + kPlanTileRows - 1) / kPlanTileRows; }
}  // namespace

PlanTiles plan_tiles(uint8_t* plan, int64_t n) {
    const int64_t np = tiles_of(n) * kPlanTileRows;
    uint8_t* p = plan + plan_base_bytes(n);
    PlanTiles t;
    t.rows = reinterpret_cast<int*>(p);
    p += align256(static_cast<size_t>(np) * 4);
    t.nbr = reinterpret_cast<int*>(p);
    p += align256(static_cast<size_t>(np) * 27 * 4);
    t.mask = reinterpret_cast<uint32_t*>(p);
    return t;
}

size_t plan_bytes(int64_t n) {
    const int64_t np = tiles_of(n) * kPlanTileRows;
    return plan_base_bytes(n) + align256(static_cast<size_t>(np) * 4) + align256(static_cast<size_t>(np) * 27 * 4) +
           align256(static_cast<size_t>(tiles_of(n)) * 4);
}

size_t plan_workspace_bytes(int64_t n) {
    return 2 * align256(static_cast<size_t>(n) * 8) + align256(static_cast<size_t>(n) * 4) +
           align256(sort_temp_bytes(n)) + 256;
}

cudaError_t launch_plan_build(const int32_t* coords, const int32_t* nbr, int64_t n, int kind, void* plan, void* ws,
                              uint32_t* status, cudaStream_t st) {
    auto* hdr = static_cast<PlanHeader*>(plan);
    const int64_t max_desc = plan_max_desc(n);
    plan_header_kernel<<<1, 1, 0, st>>>(hdr, n, max_desc, plan_pool_cap(n));
    if (n == 0) return cudaGetLastError();
    uint8_t* w = static_cast<uint8_t*>(ws);
    uint64_t* keys_in = reinterpret_cast<uint64_t*>(w);
    w += align256(static_cast<size_t>(n) * 8);
    uint64_t* keys_out = reinterpret_cast<uint64_t*>(w);
    w += align256(static_cast<size_t>(n) * 8);
    int* vals_in = reinterpret_cast<int*>(w);
    w += align256(static_cast<size_t>(n) * 4);
    void* temp = w;
    size_t temp_bytes = sort_temp_bytes(n);
    PlanView P = plan_view(static_cast<uint8_t*>(plan), n, max_desc);
    const int ni = static_cast<int>(n);
    if (kind == PLAN_TAP_ORDER) {
        static const TapBits tb = make_tap_bits();
        uint32_t* k_in = reinterpret_cast<uint32_t*>(keys_in);
        uint32_t* k_out = reinterpret_cast<uint32_t*>(keys_out);
        mask_keys_kernel<<<static_cast<unsigned>((n + 255) / 256), 256, 0, st>>>(nbr, ni, tb, k_in, vals_in);
        cudaError_t e = cub::DeviceRadixSort::SortPairs(temp, temp_bytes, k_in, k_out, vals_in, P.order, ni, 0, 27, st);
        if (e != cudaSuccess) return e;
        const PlanTiles T = plan_tiles(static_cast<uint8_t*>(plan), n);
        tile_lists_kernel<<<static_cast<unsigned>(tiles_of(n)), 32 * kTileListWarps, 0, st>>>(P.order, nbr, ni, T);
        return cudaGetLastError();
    }
    morton_keys_kernel<<<static_cast<unsigned>((n + 255) / 256), 256, 0, st>>>(
        reinterpret_cast<const int4*>(coords), ni, keys_in, vals_in);
    cudaError_t e = cub::DeviceRadixSort::SortPairs(temp, temp_bytes, keys_in, keys_out, vals_in, P.perm, ni, 0, 55,
                                                    st);
    if (e != cudaSuccess) return e;
    static bool configured[64] = {false};
    int dev = 0;
    e = cudaGetDevice(&dev);
    if (e != cudaSuccess) return e;
    if (dev >= 0 && dev < 64 && !configured[dev]) {
        e = cudaFuncSetAttribute(subtile_kernel, cudaFuncAttributeMaxDynamicSharedMemorySize, kSubtileSmem);
        if (e != cudaSuccess) return e;
        configured[dev] = true;
    }
    subtile_kernel<<<static_cast<unsigned>((n + kBlockRows - 1) / kBlockRows), kPlanThreads, kSubtileSmem, st>>>(
        P.perm, nbr, ni, static_cast<uint8_t*>(plan), status);
    return cudaGetLastError();
}

}  // namespace msc
