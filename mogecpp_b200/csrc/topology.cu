// Sparse topology on the GPU: the 27-tap submanifold neighbour map and the
// stride-2 pool / upsample maps, bit-identical to the reference's host code
// (mogecpp src/sparse.cpp:238-272 make_level, :312-357 downsample).
//
// Brick records (the default).  Voxels are grouped into 4 x 4 x 4 bricks: a
// small hash table maps a brick key (b, z >> 2, y >> 2, x >> 2) to a brick id
// (numbered in arrival order) and a brick record holds the 64 voxel indices
// of its cells (empty cells INT_MAX; a duplicated coordinate keeps its
// smallest index, FlatCoordMap's first-insert rule, src/sparse.cpp:102-114).
// Surfaces put ~15-40 voxels in a brick, so the table and the records are a
// few tens of MB and stay in L2.
//   make_level: each voxel looks up the (at most 8) bricks its 27 taps reach
//     once, then every tap is one record read;
//   downsample: a voxel's 2 x 2 x 2 stride-2 cell lies inside its brick, so
//     its siblings are the cell's 8 record entries: the parent's first child
//     is their smallest index, the slot (arrival rank) the number of siblings
//     with a smaller index and the count their number.
// Parent ids follow the reference's serial loop exactly: the rank of the
// parent's first child among all first children (first-occurrence order), by
// a flag + exclusive scan; pool_rows is slot-major [8][np] with sentinel
// nfine, inv_count = 1 / count, up_rows = fine -> parent id.
//
// Per-voxel hash (inputs too sparse for the record budget, more than
// n / 4 + 1024 bricks; the choice is made on the device from the brick
// count, so both paths are launched and one returns at once).  Keys are the
// 64-bit packed (b, z, y, x) (7 + 3 x 19 bits), open addressing with linear
// probing in 16-byte slots {key, value}, capacity a power of two >= 2n.  The
// allocation-free neighbour map (noalloc.cu) uses this path only.
#include "common.cuh"
#include "topology.h"

#include <cuda_runtime.h>

namespace msc {

namespace {

constexpr unsigned long long kEmpty = ~0ull;
constexpr int kAxisMax = (1 << 19) - 1;
constexpr int kNoVoxel = 0x7fffffff;
constexpr int kBrickVox = 64;
constexpr int kMapVox = 32;       // voxels per neighbour-map block (27 x 32 threads)
constexpr int kScanBlock = 1024;  // threads of the single-block scan of the block sums
// Voxels per block of the first-child flag scan (excl[] holds exclusive
// prefixes within such a block, bsum[] the blocks' totals).  Equal to the
// neighbour-map block, so make_level_downsample's neighbour kernel scans the
// flags of the voxels it maps.
constexpr int kFirstBlock = 256;
constexpr unsigned kStrideGrid = 148 * 8;

struct __align__(16) Slot {
    unsigned long long key;
    int val;
    int pad;
};

__device__ __forceinline__ unsigned long long mix64(unsigned long long k) {
    k ^= k >> 31;
    k *= 0x7fb5d329728ea185ull;
    k ^= k >> 27;
    k *= 0x81dadef4bc2dd44dull;
    k ^= k >> 33;
    return k;
}

__device__ __forceinline__ unsigned long long pack_key(int x, int y, int z, int b) {
    return (static_cast<unsigned long long>(b) << 57) | (static_cast<unsigned long long>(z) << 38) |
           (static_cast<unsigned long long>(y) << 19) | static_cast<unsigned long long>(x);
}

__device__ __forceinline__ bool coord_ok(int4 c) {
    return c.x >= 0 && c.x <= kAxisMax && c.y >= 0 && c.y <= kAxisMax && c.z >= 0 && c.z <= kAxisMax && c.w >= 0 &&
           c.w < 127;
}

// The per-voxel path's kernels run only while *gate > budget (the brick count
// overflowed its budget), or always when gate is null.
__device__ __forceinline__ bool gated_off(const int* gate, int budget) { return gate && *gate <= budget; }

__device__ __forceinline__ uint64_t grid_index() { return blockIdx.x * static_cast<uint64_t>(blockDim.x) + threadIdx.x; }
__device__ __forceinline__ uint64_t grid_stride() { return static_cast<uint64_t>(gridDim.x) * blockDim.x; }

__global__ void table_clear_kernel(Slot* __restrict__ t, uint64_t cap, const int* gate, int budget) {
    if (gated_off(gate, budget)) return;
    Slot s;
    s.key = kEmpty;
    s.val = kNoVoxel;
    s.pad = 0;
    for (uint64_t i = grid_index(); i < cap; i += grid_stride()) t[i] = s;
}

// Inserts key -> min(index).  Returns false when the table is full.
__device__ __forceinline__ bool table_insert(Slot* t, uint64_t mask, unsigned long long key, int idx,
                                             uint32_t* status) {
    uint64_t h = mix64(key) & mask;
    for (uint64_t probe = 0; probe <= mask; ++probe) {
        const unsigned long long prev = atomicCAS(&t[h].key, kEmpty, key);
        if (prev == kEmpty || prev == key) {
            const int old = atomicMin(&t[h].val, idx);
            if (prev == key || old != kNoVoxel) set_status(status, MSC_DEV_DUP_COORD);
            return true;
        }
        h = (h + 1) & mask;
    }
    return false;
}

__device__ __forceinline__ int table_find(const Slot* __restrict__ t, uint64_t mask, unsigned long long key) {
    uint64_t h = mix64(key) & mask;
    for (uint64_t probe = 0; probe <= mask; ++probe) {
        const int4 raw = __ldg(reinterpret_cast<const int4*>(t + h));
        const unsigned long long k =
            (static_cast<unsigned long long>(static_cast<unsigned>(raw.y)) << 32) | static_cast<unsigned>(raw.x);
        if (k == key) return raw.z;
        if (k == kEmpty) return -1;
        h = (h + 1) & mask;
    }
    return -1;
}

// Validate and insert (x, y, z, b) -> index.  Out-of-range coordinates are
// reported here only when the kernel runs ungated (the brick insert reports
// them otherwise).
__global__ void insert_kernel(const int4* __restrict__ coords, int n, Slot* __restrict__ t, uint64_t mask,
                              uint32_t* status, const int* gate, int budget) {
    if (gated_off(gate, budget)) return;
    for (uint64_t i = grid_index(); i < static_cast<uint64_t>(n); i += grid_stride()) {
        const int4 c = __ldg(coords + i);
        if (!coord_ok(c)) {
            if (!gate) set_status(status, MSC_DEV_BAD_COORD);
            continue;
        }
        if (!table_insert(t, mask, pack_key(c.x, c.y, c.z, c.w), static_cast<int>(i), status))
            set_status(status, MSC_DEV_HASH_FULL);
    }
}

// Neighbour map over the per-voxel table.  A block of 27 x 32 threads covers
// groups of 32 consecutive voxels: thread (tap, v) probes one neighbour; a
// group's results are staged in shared memory and written back as one
// contiguous [32][27] run.
__global__ void __launch_bounds__(27 * kMapVox) neighbor_kernel(const int4* __restrict__ coords, int n,
                                                                const Slot* __restrict__ t, uint64_t mask,
                                                                int* __restrict__ nbr, const int* gate, int budget) {
    if (gated_off(gate, budget)) return;
    __shared__ int4 sc[kMapVox];
    __shared__ int sn[kMapVox * 27];
    const int tid = threadIdx.x;
    const int v = tid % kMapVox;
    const int tap = tid / kMapVox;
    const int dx = tap / 9 - 1, dy = (tap / 3) % 3 - 1, dz = tap % 3 - 1;
    for (int64_t base = static_cast<int64_t>(blockIdx.x) * kMapVox; base < n;
         base += static_cast<int64_t>(gridDim.x) * kMapVox) {
        if (tid < kMapVox && base + tid < n) sc[tid] = __ldg(coords + base + tid);
        __syncthreads();
        if (base + v < n) {
            const int4 c = sc[v];
            const int qx = c.x + dx, qy = c.y + dy, qz = c.z + dz;
            int found = n;
            if (coord_ok(c) && qx >= 0 && qy >= 0 && qz >= 0 && qx <= kAxisMax && qy <= kAxisMax && qz <= kAxisMax) {
                const int idx = table_find(t, mask, pack_key(qx, qy, qz, c.w));
                if (idx >= 0) found = idx;
            }
            sn[v * 27 + tap] = found;
        }
        __syncthreads();
        const int64_t count = (n - base < kMapVox ? n - base : kMapVox) * 27;
        int* out = nbr + base * 27;
        for (int k = tid; k < count; k += blockDim.x) out[k] = sn[k];
        __syncthreads();
    }
}

// ---- downsample over the per-voxel tables ---------------------------------

__global__ void parent_insert_kernel(const int4* __restrict__ coords, int n, Slot* __restrict__ tp, uint64_t pmask,
                                     uint32_t* status, const int* gate, int budget) {
    if (gated_off(gate, budget)) return;
    for (uint64_t i = grid_index(); i < static_cast<uint64_t>(n); i += grid_stride()) {
        const int4 c = __ldg(coords + i);
        if (!coord_ok(c)) continue;
        // the parent table only needs min-index semantics; duplicates of a
        // parent key are the normal case, so no duplicate flag here
        const unsigned long long key = pack_key(c.x >> 1, c.y >> 1, c.z >> 1, c.w);
        uint64_t h = mix64(key) & pmask;
        bool done = false;
        for (uint64_t probe = 0; probe <= pmask && !done; ++probe) {
            const unsigned long long prev = atomicCAS(&tp[h].key, kEmpty, key);
            if (prev == kEmpty || prev == key) {
                atomicMin(&tp[h].val, static_cast<int>(i));
                done = true;
            }
            h = (h + 1) & pmask;
        }
        if (!done) set_status(status, MSC_DEV_HASH_FULL);
    }
}

// Block-level exclusive scan of flags f (one per thread): returns the
// exclusive prefix within the block; the block total goes to *total.
// Exclusive scan of f over the block (blockDim.x a multiple of 32, at most
// 1024; warp_tot holds blockDim.x / 32 ints); the block total goes to *total.
__device__ __forceinline__ int block_exclusive_scan(int f, int* warp_tot, int* total) {
    const int lane = threadIdx.x & 31, warp = threadIdx.x >> 5;
    const int nwarps = static_cast<int>(blockDim.x >> 5);
    int inc = f;
#pragma unroll
    for (int o = 1; o < 32; o <<= 1) {
        const int v = __shfl_up_sync(0xffffffffu, inc, o);
        if (lane >= o) inc += v;
    }
    if (lane == 31) warp_tot[warp] = inc;
    __syncthreads();
    if (warp == 0) {
        const int w = lane < nwarps ? warp_tot[lane] : 0;
        int wi = w;
#pragma unroll
        for (int o = 1; o < 32; o <<= 1) {
            const int v = __shfl_up_sync(0xffffffffu, wi, o);
            if (lane >= o) wi += v;
        }
        if (lane < nwarps) warp_tot[lane] = wi - w;
        if (lane == 31) *total = wi;
    }
    __syncthreads();
    return warp_tot[warp] + inc - f;
}

// first[i] = (i is the first child of its parent); per-block exclusive scan
// into excl[], block totals into bsum[].
__global__ void __launch_bounds__(kFirstBlock) first_scan_kernel(const int4* __restrict__ coords, int n,
                                                                 const Slot* __restrict__ tp, uint64_t pmask,
                                                                 int* __restrict__ excl, int* __restrict__ bsum,
                                                                 const int* gate, int budget) {
    if (gated_off(gate, budget)) return;
    __shared__ int warp_tot[kFirstBlock / 32];
    const int i = blockIdx.x * kFirstBlock + threadIdx.x;
    int f = 0;
    if (i < n) {
        const int4 c = __ldg(coords + i);
        if (coord_ok(c)) f = table_find(tp, pmask, pack_key(c.x >> 1, c.y >> 1, c.z >> 1, c.w)) == i;
    }
    const int e = block_exclusive_scan(f, warp_tot, bsum + blockIdx.x);
    if (i < n) excl[i] = e;
}

// Single block: exclusive scan of the block totals in place; np -> *np_out.
// Thread t takes the run of `per` consecutive totals starting at t * per,
// then one block scan of the run sums.  Up to kRunRegs totals per thread
// (nblocks <= 32768, n <= 8.4M voxels) the run is held in registers: all
// its loads are issued together (one memory round trip for the array).
constexpr int kRunRegs = 32;
__global__ void __launch_bounds__(kScanBlock) block_scan_kernel(int* __restrict__ bsum, int nblocks,
                                                                int* __restrict__ np_out) {
    __shared__ int warp_tot[kScanBlock / 32];
    __shared__ int total;
    const int per = (nblocks + kScanBlock - 1) / kScanBlock;
    const int64_t b0 = static_cast<int64_t>(threadIdx.x) * per;
    if (per <= kRunRegs) {
        int v[kRunRegs];
        int s = 0;
#pragma unroll
        for (int k = 0; k < kRunRegs; ++k) {
            v[k] = (k < per && b0 + k < nblocks) ? bsum[b0 + k] : 0;
            s += v[k];
        }
        int run = block_exclusive_scan(s, warp_tot, &total);
#pragma unroll
        for (int k = 0; k < kRunRegs; ++k) {
            if (k < per && b0 + k < nblocks) bsum[b0 + k] = run;
            run += v[k];
        }
    } else {
        int s = 0;
        for (int k = 0; k < per; ++k)
            if (b0 + k < nblocks) s += bsum[b0 + k];
        int run = block_exclusive_scan(s, warp_tot, &total);
        for (int k = 0; k < per; ++k) {
            if (b0 + k < nblocks) {
                const int v = bsum[b0 + k];
                bsum[b0 + k] = run;
                run += v;
            }
        }
    }
    if (threadIdx.x == 0) *np_out = total;
}

// Parent ids, up_rows, parent coordinates.
__global__ void assign_kernel(const int4* __restrict__ coords, int n, const Slot* __restrict__ tp, uint64_t pmask,
                              const int* __restrict__ excl, const int* __restrict__ bsum, int4* __restrict__ parent,
                              int* __restrict__ up_rows, const int* gate, int budget) {
    if (gated_off(gate, budget)) return;
    for (uint64_t u = grid_index(); u < static_cast<uint64_t>(n); u += grid_stride()) {
        const int i = static_cast<int>(u);
        const int4 c = __ldg(coords + i);
        if (!coord_ok(c)) continue;
        const int first = table_find(tp, pmask, pack_key(c.x >> 1, c.y >> 1, c.z >> 1, c.w));
        if (first < 0 || first >= n) continue;
        const int pid = excl[first] + bsum[first / kFirstBlock];
        up_rows[i] = pid;
        if (first == i) parent[pid] = make_int4(c.x >> 1, c.y >> 1, c.z >> 1, c.w);
    }
}

__global__ void pool_fill_kernel(int* __restrict__ pool_rows, const int* __restrict__ np_dev, int nfine) {
    const int64_t total = 8ll * (*np_dev);
    for (int64_t k = grid_index(); k < total; k += grid_stride()) pool_rows[k] = nfine;
}

// slot = number of siblings with a smaller fine index.
__global__ void slot_kernel(const int4* __restrict__ coords, int n, const Slot* __restrict__ tf, uint64_t fmask,
                            const int* __restrict__ up_rows, const int* __restrict__ np_dev, int* __restrict__ pool_rows,
                            float* __restrict__ inv_count, uint32_t* status, const int* gate, int budget) {
    if (gated_off(gate, budget)) return;
    const int np = *np_dev;
    for (uint64_t u = grid_index(); u < static_cast<uint64_t>(n); u += grid_stride()) {
        const int i = static_cast<int>(u);
        const int4 c = __ldg(coords + i);
        if (!coord_ok(c)) continue;
        const int px = c.x >> 1, py = c.y >> 1, pz = c.z >> 1;
        int count = 0, rank = 0;
#pragma unroll
        for (int o = 0; o < 8; ++o) {
            const int j =
                table_find(tf, fmask, pack_key(2 * px + (o >> 2), 2 * py + ((o >> 1) & 1), 2 * pz + (o & 1), c.w));
            if (j >= 0) {
                ++count;
                rank += j < i;
            }
        }
        const int pid = up_rows[i];
        if (pid < 0 || pid >= np || rank >= 8) {
            set_status(status, MSC_DEV_POOL_OVERFLOW);
            continue;
        }
        pool_rows[static_cast<int64_t>(rank) * np + pid] = i;
        if (rank == 0) inv_count[pid] = 1.0f / static_cast<float>(count);
    }
}

// ---- brick records ---------------------------------------------------------

int64_t brick_budget(int64_t n) { return n / 4 + 1024; }
uint64_t brick_capacity(int64_t n) {
    uint64_t cap = 64;
    while (cap < static_cast<uint64_t>(2 * brick_budget(n))) cap <<= 1;
    return cap;
}

__device__ __forceinline__ unsigned long long brick_key(int bx, int by, int bz, int b) { return pack_key(bx, by, bz, b); }
__device__ __forceinline__ int brick_cell(int x, int y, int z) { return (x & 3) | ((y & 3) << 2) | ((z & 3) << 4); }

// Brick-table lookup shared by the lanes of a warp that hold the same key
// (neighbouring voxels of the (b, z, y, x) order share bricks): the first of
// them probes, the others take its answer.  Lanes with valid = false get -1.
__device__ __forceinline__ int warp_brick_find(const Slot* __restrict__ t, uint64_t mask, unsigned long long key,
                                               bool valid) {
    const unsigned peers = __match_any_sync(__activemask(), valid ? key : kEmpty);
    const int leader = __ffs(peers) - 1;
    int id = -1;
    if (valid && static_cast<int>(threadIdx.x & 31) == leader) id = table_find(t, mask, key);
    return __shfl_sync(peers, id, leader);
}

// ctr[0] = bricks numbered so far (forced above the budget when the table
// runs out, which selects the per-voxel hash).  Neighbouring voxels of the
// (b, z, y, x) order share bricks, so the lanes of a warp that hold the same
// brick key elect one lane to insert it: fewer atomics on the same slot.
__global__ void brick_insert_kernel(const int4* __restrict__ coords, int n, Slot* __restrict__ t, uint64_t mask,
                                    int* __restrict__ ctr, int budget, uint32_t* status) {
    for (uint64_t u = grid_index(); u < static_cast<uint64_t>(n); u += grid_stride()) {
        const int4 c = __ldg(coords + u);
        const bool ok = coord_ok(c);
        if (!ok) set_status(status, MSC_DEV_BAD_COORD);
        const unsigned long long key = ok ? brick_key(c.x >> 2, c.y >> 2, c.z >> 2, c.w) : kEmpty;
        const unsigned peers = __match_any_sync(__activemask(), key);
        if (!ok || static_cast<int>(threadIdx.x & 31) != __ffs(peers) - 1) continue;
        uint64_t h = mix64(key) & mask;
        bool done = false, fresh = false;
        for (uint64_t probe = 0; probe <= mask && !done; ++probe) {
            // most bricks are already in the table: a plain L2 read finds
            // them without an atomic (a stale empty read just takes the CAS)
            const unsigned long long cur = __ldcg(&t[h].key);
            if (cur == key) {
                done = true;
            } else if (cur == kEmpty) {
                const unsigned long long prev = atomicCAS(&t[h].key, kEmpty, key);
                fresh = prev == kEmpty;
                done = fresh || prev == key;
            }
            if (!done) h = (h + 1) & mask;
        }
        // ids for the bricks this warp inserted: one counter add per warp
        const unsigned active = __activemask();
        const unsigned won = __ballot_sync(active, fresh);
        if (won) {
            const int lead = __ffs(won) - 1;
            const int lane = static_cast<int>(threadIdx.x & 31);
            int base = 0;
            if (lane == lead) base = atomicAdd(ctr, __popc(won));
            base = __shfl_sync(active, base, lead);
            if (fresh) t[h].val = base + __popc(won & ((1u << lane) - 1u));
        }
        if (!done) atomicMax(ctr, budget + 1);
    }
}

__global__ void brick_clear_kernel(int* __restrict__ rec, const int* __restrict__ ctr, int budget) {
    const int nb = *ctr;
    if (nb > budget) return;
    const int64_t total = static_cast<int64_t>(nb) * kBrickVox;
    for (int64_t e = grid_index(); e < total; e += grid_stride()) rec[e] = kNoVoxel;
}

__global__ void brick_fill_kernel(const int4* __restrict__ coords, int n, const Slot* __restrict__ t, uint64_t mask,
                                  int* __restrict__ rec, const int* __restrict__ ctr, int budget, uint32_t* status) {
    if (*ctr > budget) return;
    for (uint64_t u = grid_index(); u < static_cast<uint64_t>(n); u += grid_stride()) {
        const int4 c = __ldg(coords + u);
        const bool ok = coord_ok(c);
        const int id = warp_brick_find(t, mask, brick_key(c.x >> 2, c.y >> 2, c.z >> 2, c.w), ok);
        if (!ok || id < 0) continue;  // id < 0 cannot happen: every voxel's brick was inserted
        const int old = atomicMin(&rec[static_cast<int64_t>(id) * kBrickVox + brick_cell(c.x, c.y, c.z)],
                                  static_cast<int>(u));
        if (old != kNoVoxel) set_status(status, MSC_DEV_DUP_COORD);
    }
}

// Neighbour map over the brick records, one thread per voxel and one block
// per 256 voxels (no grid-stride loop: shared memory holds 6 blocks per SM,
// and a fixed grid-stride grid left a second, partial wave of blocks): the
// thread looks up the bricks its taps can reach (offset bits (ox, oy, oz):
// on an axis with the bit set the neighbour brick is the one below when the
// voxel sits on its brick's low face (cell coordinate 0), above on the high
// face (3), none otherwise) into shared memory, then issues its 27 record
// reads before using any of them (27 independent loads in flight per
// thread); the block's [256][27] rows are staged in shared memory (row
// stride 27 words: conflict-free) and leave as one contiguous run.
//
// kFirst (make_level_downsample): the voxel's stride-2 cell (the 2 x 2 x 2
// cells with the same parent) lies inside its brick and its 8 cells are
// taps of the row just built, so the kernel also does the first-child pass
// of the stride-2 maps: first child (smallest index), the voxel's rank among
// its siblings and their count, and the block scan of the first-child flags
// (one block = kFirstBlock voxels), as brick_first_scan_kernel does from the
// records.
constexpr int kNbrThreads = 256;
static_assert(kNbrThreads == kFirstBlock, "the neighbour block is the first-child scan block");

template <bool kFirst>
__global__ void __launch_bounds__(kNbrThreads) brick_neighbor_kernel(const int4* __restrict__ coords, int n,
                                                                     const Slot* __restrict__ t, uint64_t mask,
                                                                     const int* __restrict__ rec,
                                                                     const int* __restrict__ ctr, int budget,
                                                                     int* __restrict__ nbr,
                                                                     int* __restrict__ first_idx,
                                                                     int* __restrict__ cell_rc,
                                                                     int* __restrict__ excl, int* __restrict__ bsum) {
    if (*ctr > budget) return;
    __shared__ __align__(16) int sn[kNbrThreads * 27];
    __shared__ int sb[8 * kNbrThreads];
    __shared__ int warp_tot[kNbrThreads / 32];
    const int tid = threadIdx.x;
    const int64_t base = static_cast<int64_t>(blockIdx.x) * kNbrThreads;
    const int64_t i = base + tid;
    int* row = sn + tid * 27;
    int first = -1, rc = 8;  // brick_first_scan_kernel's values for a voxel without a cell
    if (i < n) {
        const int4 c = __ldg(coords + i);
        if (!coord_ok(c)) {
#pragma unroll
            for (int tap = 0; tap < 27; ++tap) row[tap] = n;
        } else {
            const int lx = c.x & 3, ly = c.y & 3, lz = c.z & 3;
            const int bx = c.x >> 2, by = c.y >> 2, bz = c.z >> 2;
            constexpr int kBrickMax = kAxisMax >> 2;
#pragma unroll
            for (int o = 0; o < 8; ++o) {
                const int ox = (o & 1) ? (lx == 0 ? -1 : (lx == 3 ? 1 : 2)) : 0;
                const int oy = (o & 2) ? (ly == 0 ? -1 : (ly == 3 ? 1 : 2)) : 0;
                const int oz = (o & 4) ? (lz == 0 ? -1 : (lz == 3 ? 1 : 2)) : 0;
                const int qx = bx + ox, qy = by + oy, qz = bz + oz;
                int id = -1;
                if (ox != 2 && oy != 2 && oz != 2 && qx >= 0 && qy >= 0 && qz >= 0 && qx <= kBrickMax &&
                    qy <= kBrickMax && qz <= kBrickMax)
                    id = table_find(t, mask, brick_key(qx, qy, qz, c.w));
                sb[o * kNbrThreads + tid] = id;
            }
            // per axis and offset d in {-1, 0, 1} (index d + 1): the brick-offset
            // bit (set when the tap crosses into the neighbouring brick) and the
            // cell coordinate inside the brick reached.  A tap outside the
            // coordinate range lands in a brick that was not looked up (id -1).
            const int ox[3] = {lx == 0 ? 1 : 0, 0, lx == 3 ? 1 : 0};
            const int oy[3] = {ly == 0 ? 2 : 0, 0, ly == 3 ? 2 : 0};
            const int oz[3] = {lz == 0 ? 4 : 0, 0, lz == 3 ? 4 : 0};
            const int cx[3] = {(lx + 3) & 3, lx, (lx + 1) & 3};
            const int cy[3] = {((ly + 3) & 3) << 2, ly << 2, ((ly + 1) & 3) << 2};
            const int cz[3] = {((lz + 3) & 3) << 4, lz << 4, ((lz + 1) & 3) << 4};
            const int* sbt = sb + tid;
            int v[27];
#pragma unroll
            for (int tap = 0; tap < 27; ++tap) {
                const int ix = tap / 9, iy = (tap / 3) % 3, iz = tap % 3;
                const int id = sbt[(ox[ix] | oy[iy] | oz[iz]) * kNbrThreads];
                v[tap] = id >= 0 ? __ldg(rec + static_cast<int64_t>(id) * kBrickVox + (cx[ix] | cy[iy] | cz[iz]))
                                 : kNoVoxel;
            }
#pragma unroll
            for (int tap = 0; tap < 27; ++tap) row[tap] = v[tap] != kNoVoxel ? v[tap] : n;
            if (kFirst && sbt[0] >= 0) {
                // the cell's cells: offset 0 and s per axis, s = +1 on an even
                // coordinate and -1 on an odd one (tap digit s + 1), all in the
                // own brick; a missing cell reads n
                const int sx = (lx & 1) ? 0 : 2, sy = (ly & 1) ? 0 : 2, sz = (lz & 1) ? 0 : 2;
                int fst = kNoVoxel, cnt = 0, rnk = 0;
#pragma unroll
                for (int o = 0; o < 8; ++o) {
                    const int j = row[((o & 4) ? sx : 1) * 9 + ((o & 2) ? sy : 1) * 3 + ((o & 1) ? sz : 1)];
                    if (j < n) {
                        ++cnt;
                        rnk += j < i;
                        fst = min(fst, j);
                    }
                }
                first = fst;
                rc = rnk | (cnt << 8);
            }
        }
    }
    if constexpr (kFirst) {
        if (i < n) {
            first_idx[i] = first;
            cell_rc[i] = rc;
        }
        const int e = block_exclusive_scan(i < n && first == i ? 1 : 0, warp_tot, bsum + blockIdx.x);
        if (i < n) excl[i] = e;
    }
    __syncthreads();
    const int64_t count = (n - base < kNbrThreads ? n - base : kNbrThreads) * 27;
    int* out = nbr + base * 27;
    int64_t k0 = 0;
    if ((reinterpret_cast<uintptr_t>(nbr) & 15) == 0) {
        // a block's run starts 256 x 108 bytes after the previous one: 16-byte
        // stores when the map itself is 16-byte aligned
        const int64_t c4 = count / 4;
        for (int64_t k = tid; k < c4; k += kNbrThreads)
            reinterpret_cast<int4*>(out)[k] = reinterpret_cast<const int4*>(sn)[k];
        k0 = c4 * 4;
    }
    for (int64_t k = k0 + tid; k < count; k += kNbrThreads) out[k] = sn[k];
}

// The 8 record entries of voxel c's stride-2 cell (the 2 x 2 x 2 block of
// cells with the same parent, inside c's brick): first child (smallest
// index), the count, and the number with a smaller index than i.
struct CellInfo {
    int first, count, rank;
};
__device__ __forceinline__ CellInfo cell_info(const int* __restrict__ rec, int id, int4 c, int i) {
    const int* r = rec + static_cast<int64_t>(id) * kBrickVox;
    const int x0 = c.x & 2, y0 = c.y & 2, z0 = c.z & 2;
    CellInfo ci{kNoVoxel, 0, 0};
#pragma unroll
    for (int o = 0; o < 8; ++o) {
        const int j = __ldg(r + brick_cell(x0 + (o >> 2), y0 + ((o >> 1) & 1), z0 + (o & 1)));
        if (j != kNoVoxel) {
            ++ci.count;
            ci.rank += j < i;
            ci.first = min(ci.first, j);
        }
    }
    return ci;
}

// first_idx[i] = the first child of i's parent; per-block exclusive scan of
// the flags (i == first) into excl[], block totals into bsum[].
__global__ void __launch_bounds__(kFirstBlock) brick_first_scan_kernel(const int4* __restrict__ coords, int n,
                                                                       const Slot* __restrict__ t, uint64_t mask,
                                                                       const int* __restrict__ rec,
                                                                       const int* __restrict__ ctr, int budget,
                                                                       int* __restrict__ first_idx,
                                                                       int* __restrict__ cell_rc,
                                                                       int* __restrict__ excl, int* __restrict__ bsum) {
    if (*ctr > budget) return;
    __shared__ int warp_tot[kFirstBlock / 32];
    const int i = blockIdx.x * kFirstBlock + threadIdx.x;
    int f = 0;
    if (i < n) {
        const int4 c = __ldg(coords + i);
        int first = -1, rc = 8;
        if (coord_ok(c)) {
            const int id = table_find(t, mask, brick_key(c.x >> 2, c.y >> 2, c.z >> 2, c.w));
            if (id >= 0) {
                const CellInfo ci = cell_info(rec, id, c, i);
                first = ci.first;
                rc = ci.rank | (ci.count << 8);
            }
        }
        first_idx[i] = first;
        cell_rc[i] = rc;
        f = first == i;
    }
    const int e = block_exclusive_scan(f, warp_tot, bsum + blockIdx.x);
    if (i < n) excl[i] = e;
}

// Parent ids, up_rows, parent coordinates, pool_rows slots and inv_count.
__global__ void brick_assign_kernel(const int4* __restrict__ coords, int n, const int* __restrict__ ctr, int budget,
                                    const int* __restrict__ first_idx, const int* __restrict__ cell_rc,
                                    const int* __restrict__ excl,
                                    const int* __restrict__ bsum, const int* __restrict__ np_dev,
                                    int4* __restrict__ parent, int* __restrict__ up_rows, int* __restrict__ pool_rows,
                                    float* __restrict__ inv_count, uint32_t* status) {
    if (*ctr > budget) return;
    const int np = *np_dev;
    for (uint64_t u = grid_index(); u < static_cast<uint64_t>(n); u += grid_stride()) {
        const int i = static_cast<int>(u);
        const int first = first_idx[i];
        if (first < 0 || first >= n) continue;
        const int4 c = __ldg(coords + i);
        const int pid = excl[first] + bsum[first / kFirstBlock];
        up_rows[i] = pid;
        if (first == i) parent[pid] = make_int4(c.x >> 1, c.y >> 1, c.z >> 1, c.w);
        const int rc = cell_rc[i];  // the cell's rank and count from the first-child pass
        const CellInfo ci{first, rc >> 8, rc & 0xff};
        if (pid < 0 || pid >= np || ci.rank >= 8) {
            set_status(status, MSC_DEV_POOL_OVERFLOW);
            continue;
        }
        pool_rows[static_cast<int64_t>(ci.rank) * np + pid] = i;
        if (ci.rank == 0) inv_count[pid] = 1.0f / static_cast<float>(ci.count);
    }
}

// Octant maps of a stride-2 transition, for the octant-weighted stride-2
// conv and its transpose (an extension: the reference's stride-2 operators
// are pool + linear and linear + nearest up).  The octant of fine voxel
// (x, y, z) in its parent's 2 x 2 x 2 cell is (x & 1) * 4 + (y & 1) * 2 +
// (z & 1).  One thread per output row; a block's [256][27] rows are staged
// in shared memory and leave as one contiguous run.
//   down [np][27]: column o = the child at octant o (from pool_rows), or nfine
//   up [nfine][27]: column oct(c) = up_rows[c], every other column np
__device__ __forceinline__ int octant(int4 c) { return (c.x & 1) * 4 + (c.y & 1) * 2 + (c.z & 1); }

__device__ __forceinline__ void store_rows27(int* __restrict__ out, const int* __restrict__ sn, int64_t rows) {
    const int64_t count = rows * 27;
    int64_t k0 = 0;
    if ((reinterpret_cast<uintptr_t>(out) & 15) == 0) {
        const int64_t c4 = count / 4;
        for (int64_t k = threadIdx.x; k < c4; k += blockDim.x)
            reinterpret_cast<int4*>(out)[k] = reinterpret_cast<const int4*>(sn)[k];
        k0 = c4 * 4;
    }
    for (int64_t k = k0 + threadIdx.x; k < count; k += blockDim.x) out[k] = sn[k];
}

__global__ void __launch_bounds__(256) octant_down_kernel(const int4* __restrict__ coords, int nfine,
                                                          const int* __restrict__ pool_rows, int np,
                                                          int* __restrict__ down) {
    __shared__ __align__(16) int sn[256 * 27];
    const int64_t base = static_cast<int64_t>(blockIdx.x) * 256;
    const int64_t p = base + threadIdx.x;
    int* row = sn + threadIdx.x * 27;
#pragma unroll
    for (int t = 0; t < 27; ++t) row[t] = nfine;
    if (p < np) {
#pragma unroll
        for (int s = 0; s < 8; ++s) {
            const int c = __ldg(pool_rows + static_cast<int64_t>(s) * np + p);
            if (c >= 0 && c < nfine) row[octant(__ldg(coords + c))] = c;
        }
    }
    __syncthreads();
    store_rows27(down + base * 27, sn, np - base < 256 ? np - base : 256);
}

__global__ void __launch_bounds__(256) octant_up_kernel(const int4* __restrict__ coords, int nfine,
                                                        const int* __restrict__ up_rows, int np,
                                                        int* __restrict__ up) {
    __shared__ __align__(16) int sn[256 * 27];
    const int64_t base = static_cast<int64_t>(blockIdx.x) * 256;
    const int64_t c = base + threadIdx.x;
    int* row = sn + threadIdx.x * 27;
#pragma unroll
    for (int t = 0; t < 27; ++t) row[t] = np;
    if (c < nfine) row[octant(__ldg(coords + c))] = __ldg(up_rows + c);
    __syncthreads();
    store_rows27(up + base * 27, sn, nfine - base < 256 ? nfine - base : 256);
}

uint64_t table_capacity(int64_t n) {
    uint64_t cap = 64;
    while (cap < static_cast<uint64_t>(2 * n)) cap <<= 1;
    return cap;
}

size_t align_up(size_t v, size_t a) { return (v + a - 1) / a * a; }

unsigned stride_grid(int64_t n, int per) {
    const int64_t g = (n + per - 1) / per;
    return static_cast<unsigned>(g < kStrideGrid ? (g > 0 ? g : 1) : kStrideGrid);
}

}  // namespace

// Workspace layout (shared by make_level and downsample):
//   per-voxel tables: 2 x cap slots (make_level uses the first; downsample
//   the fine and parent tables) | excl [n + 1] | bsum | brick table (bcap
//   slots) | brick records [budget][64] | counter | first child [n] |
//   stride-2 cell rank and count [n]
namespace {
struct TopoWs {
    Slot* t;
    int* excl;
    int* bsum;
    Slot* bt;
    int* rec;
    int* ctr;
    int* first;
    int* cell;  // per voxel: the stride-2 cell's rank of it | count << 8
    uint64_t cap, bcap;
    int budget;
};

TopoWs carve(void* ws, int64_t n) {
    TopoWs w;
    w.cap = table_capacity(n);
    w.bcap = brick_capacity(n);
    w.budget = static_cast<int>(brick_budget(n));
    const int64_t nblk = (n + kFirstBlock - 1) / kFirstBlock + 1;
    char* p = static_cast<char*>(ws);
    w.t = reinterpret_cast<Slot*>(p);
    p += align_up(2 * w.cap * sizeof(Slot), 256);
    w.excl = reinterpret_cast<int*>(p);
    p += align_up(static_cast<size_t>(n + 1) * 4, 256);
    w.bsum = reinterpret_cast<int*>(p);
    p += align_up(static_cast<size_t>(nblk) * 4, 256);
    w.bt = reinterpret_cast<Slot*>(p);
    p += align_up(w.bcap * sizeof(Slot), 256);
    w.rec = reinterpret_cast<int*>(p);
    p += align_up(static_cast<size_t>(w.budget) * kBrickVox * 4, 256);
    w.ctr = reinterpret_cast<int*>(p);
    p += 256;
    w.first = reinterpret_cast<int*>(p);
    p += align_up(static_cast<size_t>(n) * 4, 256);
    w.cell = reinterpret_cast<int*>(p);
    return w;
}

// Brick table + records of the n voxels (counter, clear, insert, fill).
cudaError_t launch_brick_build(const int4* c4, int n, const TopoWs& w, uint32_t* status, cudaStream_t st) {
    cudaError_t e = cudaMemsetAsync(w.ctr, 0, sizeof(int), st);
    if (e != cudaSuccess) return e;
    table_clear_kernel<<<stride_grid(static_cast<int64_t>(w.bcap), 256), 256, 0, st>>>(w.bt, w.bcap, nullptr, 0);
    brick_insert_kernel<<<stride_grid(n, 256), 256, 0, st>>>(c4, n, w.bt, w.bcap - 1, w.ctr, w.budget, status);
    brick_clear_kernel<<<kStrideGrid, 256, 0, st>>>(w.rec, w.ctr, w.budget);
    brick_fill_kernel<<<stride_grid(n, 256), 256, 0, st>>>(c4, n, w.bt, w.bcap - 1, w.rec, w.ctr, w.budget, status);
    return cudaGetLastError();
}
}  // namespace

size_t topology_workspace_bytes(int64_t n) {
    const int64_t nblk = (n + kFirstBlock - 1) / kFirstBlock + 1;
    return align_up(2 * table_capacity(n) * sizeof(Slot), 256) + align_up(static_cast<size_t>(n + 1) * 4, 256) +
           align_up(static_cast<size_t>(nblk) * 4, 256) + align_up(brick_capacity(n) * sizeof(Slot), 256) +
           align_up(static_cast<size_t>(brick_budget(n)) * kBrickVox * 4, 256) + 256 +
           2 * align_up(static_cast<size_t>(n) * 4, 256);
}

namespace {

// The neighbour map from a built brick table (or the per-voxel hash when
// the bricks overflowed).  with_first: the brick path also runs the
// first-child pass of the stride-2 maps (launch_stride2 then skips it).
cudaError_t launch_map(const int4* c4, int64_t n, int32_t* nbr, const TopoWs& w, uint32_t* status,
                       cudaStream_t st, bool with_first) {
    const int ni = static_cast<int>(n);
    const unsigned grid = static_cast<unsigned>((n + kNbrThreads - 1) / kNbrThreads);
    if (with_first)
        brick_neighbor_kernel<true><<<grid, kNbrThreads, 0, st>>>(c4, ni, w.bt, w.bcap - 1, w.rec, w.ctr, w.budget,
                                                                  nbr, w.first, w.cell, w.excl, w.bsum);
    else
        brick_neighbor_kernel<false><<<grid, kNbrThreads, 0, st>>>(c4, ni, w.bt, w.bcap - 1, w.rec, w.ctr, w.budget,
                                                                   nbr, nullptr, nullptr, nullptr, nullptr);
    // too many bricks: the per-voxel hash (these return at once otherwise)
    table_clear_kernel<<<kStrideGrid, 256, 0, st>>>(w.t, w.cap, w.ctr, w.budget);
    insert_kernel<<<kStrideGrid, 256, 0, st>>>(c4, ni, w.t, w.cap - 1, status, w.ctr, w.budget);
    neighbor_kernel<<<stride_grid(n, kMapVox), 27 * kMapVox, 0, st>>>(c4, ni, w.t, w.cap - 1, nbr, w.ctr, w.budget);
    return cudaGetLastError();
}

}  // namespace

cudaError_t launch_make_level(const int32_t* coords, int64_t n, int32_t* nbr, void* ws, uint32_t* status,
                              cudaStream_t st) {
    if (n == 0) return cudaSuccess;
    const TopoWs w = carve(ws, n);
    const auto* c4 = reinterpret_cast<const int4*>(coords);
    cudaError_t e = launch_brick_build(c4, static_cast<int>(n), w, status, st);
    if (e != cudaSuccess) return e;
    return launch_map(c4, n, nbr, w, status, st, false);
}

size_t topology_table_bytes(int64_t n) { return table_capacity(n) * sizeof(Slot); }

cudaError_t launch_make_level_in_table(const int32_t* coords, int64_t n, int32_t* nbr, void* table,
                                       size_t table_bytes, uint32_t* status, cudaStream_t st) {
    if (n == 0) return cudaSuccess;
    const uint64_t cap = table_capacity(n);
    if (cap * sizeof(Slot) > table_bytes) return cudaErrorInvalidValue;
    Slot* t = static_cast<Slot*>(table);
    const auto* c4 = reinterpret_cast<const int4*>(coords);
    const int ni = static_cast<int>(n);
    table_clear_kernel<<<stride_grid(static_cast<int64_t>(cap), 256), 256, 0, st>>>(t, cap, nullptr, 0);
    insert_kernel<<<stride_grid(n, 256), 256, 0, st>>>(c4, ni, t, cap - 1, status, nullptr, 0);
    neighbor_kernel<<<stride_grid(n, kMapVox), 27 * kMapVox, 0, st>>>(c4, ni, t, cap - 1, nbr, nullptr, 0);
    return cudaGetLastError();
}

namespace {

// The stride-2 maps from a built brick table (or the per-voxel hashes).
// first_done: the neighbour kernel already ran the brick path's first-child
// pass (first_idx, cell ranks, flag scan).
cudaError_t launch_stride2(const int4* c4, int64_t n, int32_t* parent, int32_t* np_dev, int32_t* pool_rows,
                           float* inv_count, int32_t* up_rows, const TopoWs& w, uint32_t* status, cudaStream_t st,
                           bool first_done) {
    Slot* tf = w.t;
    Slot* tp = w.t + w.cap;
    const int nblk = static_cast<int>((n + kFirstBlock - 1) / kFirstBlock);
    const int ni = static_cast<int>(n);
    auto* par = reinterpret_cast<int4*>(parent);
    // per-voxel tables only when the bricks overflowed (gated kernels)
    table_clear_kernel<<<kStrideGrid, 256, 0, st>>>(w.t, 2 * w.cap, w.ctr, w.budget);
    insert_kernel<<<kStrideGrid, 256, 0, st>>>(c4, ni, tf, w.cap - 1, status, w.ctr, w.budget);
    parent_insert_kernel<<<kStrideGrid, 256, 0, st>>>(c4, ni, tp, w.cap - 1, status, w.ctr, w.budget);
    // first children: flags + per-block scan (one of the two runs)
    if (!first_done)
        brick_first_scan_kernel<<<nblk, kFirstBlock, 0, st>>>(c4, ni, w.bt, w.bcap - 1, w.rec, w.ctr, w.budget,
                                                              w.first, w.cell, w.excl, w.bsum);
    first_scan_kernel<<<nblk, kFirstBlock, 0, st>>>(c4, ni, tp, w.cap - 1, w.excl, w.bsum, w.ctr, w.budget);
    block_scan_kernel<<<1, kScanBlock, 0, st>>>(w.bsum, nblk, np_dev);
    pool_fill_kernel<<<kStrideGrid, 256, 0, st>>>(pool_rows, np_dev, ni);
    brick_assign_kernel<<<stride_grid(n, 256), 256, 0, st>>>(c4, ni, w.ctr, w.budget, w.first, w.cell, w.excl, w.bsum,
                                                             np_dev, par, up_rows, pool_rows, inv_count, status);
    assign_kernel<<<kStrideGrid, 256, 0, st>>>(c4, ni, tp, w.cap - 1, w.excl, w.bsum, par, up_rows, w.ctr, w.budget);
    slot_kernel<<<kStrideGrid, 256, 0, st>>>(c4, ni, tf, w.cap - 1, up_rows, np_dev, pool_rows, inv_count, status,
                                             w.ctr, w.budget);
    return cudaGetLastError();
}

}  // namespace

cudaError_t launch_downsample(const int32_t* coords, int64_t n, int32_t* parent, int32_t* np_dev, int32_t* pool_rows,
                              float* inv_count, int32_t* up_rows, void* ws, uint32_t* status, cudaStream_t st) {
    if (n == 0) return cudaMemsetAsync(np_dev, 0, sizeof(int32_t), st);
    const TopoWs w = carve(ws, n);
    const auto* c4 = reinterpret_cast<const int4*>(coords);
    cudaError_t e = launch_brick_build(c4, static_cast<int>(n), w, status, st);
    if (e != cudaSuccess) return e;
    return launch_stride2(c4, n, parent, np_dev, pool_rows, inv_count, up_rows, w, status, st, false);
}

cudaError_t launch_octant_maps(const int32_t* coords, int64_t nfine, const int32_t* pool_rows,
                               const int32_t* up_rows, int64_t np, int32_t* down, int32_t* up, cudaStream_t st) {
    const auto* c4 = reinterpret_cast<const int4*>(coords);
    if (np > 0)
        octant_down_kernel<<<static_cast<unsigned>((np + 255) / 256), 256, 0, st>>>(
            c4, static_cast<int>(nfine), pool_rows, static_cast<int>(np), down);
    if (nfine > 0)
        octant_up_kernel<<<static_cast<unsigned>((nfine + 255) / 256), 256, 0, st>>>(
            c4, static_cast<int>(nfine), up_rows, static_cast<int>(np), up);
    return cudaGetLastError();
}

cudaError_t launch_make_level_downsample(const int32_t* coords, int64_t n, int32_t* nbr, int32_t* parent,
                                         int32_t* np_dev, int32_t* pool_rows, float* inv_count, int32_t* up_rows,
                                         void* ws, uint32_t* status, cudaStream_t st) {
    if (n == 0) return cudaMemsetAsync(np_dev, 0, sizeof(int32_t), st);
    const TopoWs w = carve(ws, n);
    const auto* c4 = reinterpret_cast<const int4*>(coords);
    cudaError_t e = launch_brick_build(c4, static_cast<int>(n), w, status, st);
    if (e != cudaSuccess) return e;
    e = launch_map(c4, n, nbr, w, status, st, true);
    if (e != cudaSuccess) return e;
    return launch_stride2(c4, n, parent, np_dev, pool_rows, inv_count, up_rows, w, status, st, true);
}

}  // namespace msc
