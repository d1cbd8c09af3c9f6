// Sparse topology on the GPU: voxel hash, 27-tap submanifold neighbour map
// and the stride-2 pool / upsample maps, bit-identical to the reference's
// host code (mogecpp src/sparse.cpp:238-272 make_level, :312-357 downsample).
//
// Keys: 64-bit packed (b, z, y, x), 7 + 3 x 19 bits (x in the low bits).
// Table: open addressing, linear probing, 16-byte slots {key, value} so a
// probe is one 16-byte load; capacity = power of two >= 2n (load <= 0.5).
// The value of a key is the smallest voxel index holding it (atomicMin), the
// "first insert wins" rule of FlatCoordMap::emplace (src/sparse.cpp:102-114).
//
// Downsample numbering follows the reference's serial loop exactly:
//   parent id   = rank of the parent's first child among first children
//                 (first-occurrence order): flag + exclusive scan;
//   slot        = number of siblings with a smaller fine index (the serial
//                 arrival order), found by probing the parent's 8 child
//                 coordinates in the fine table;
//   pool_rows   = slot-major [8][np], sentinel nfine; inv_count = 1/count;
//   up_rows     = fine -> parent id.
#include "common.cuh"
#include "topology.h"

#include <cuda_runtime.h>

namespace msc {

namespace {

constexpr unsigned long long kEmpty = ~0ull;
constexpr int kAxisMax = (1 << 19) - 1;

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

__global__ void table_clear_kernel(Slot* __restrict__ t, uint64_t cap) {
    const uint64_t i = blockIdx.x * static_cast<uint64_t>(blockDim.x) + threadIdx.x;
    if (i < cap) {
        Slot s;
        s.key = kEmpty;
        s.val = 0x7fffffff;
        s.pad = 0;
        t[i] = s;
    }
}

// Inserts key -> min(index).  Returns false when the table is full.
__device__ __forceinline__ bool table_insert(Slot* t, uint64_t mask, unsigned long long key, int idx,
                                             uint32_t* status) {
    uint64_t h = mix64(key) & mask;
    for (uint64_t probe = 0; probe <= mask; ++probe) {
        const unsigned long long prev = atomicCAS(&t[h].key, kEmpty, key);
        if (prev == kEmpty || prev == key) {
            const int old = atomicMin(&t[h].val, idx);
            if (prev == key || old != 0x7fffffff) set_status(status, MSC_DEV_DUP_COORD);
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

// One thread per voxel: validate and insert (x, y, z, b) -> index.
__global__ void insert_kernel(const int4* __restrict__ coords, int n, Slot* __restrict__ t, uint64_t mask,
                              uint32_t* status) {
    const int i = blockIdx.x * blockDim.x + threadIdx.x;
    if (i >= n) return;
    const int4 c = __ldg(coords + i);
    if (!coord_ok(c)) {
        set_status(status, MSC_DEV_BAD_COORD);
        return;
    }
    if (!table_insert(t, mask, pack_key(c.x, c.y, c.z, c.w), i, status)) set_status(status, MSC_DEV_HASH_FULL);
}

// Neighbour map.  A block of 27 x 32 threads covers 32 consecutive voxels:
// thread (tap, v) probes one neighbour, results are staged in shared memory
// and written back as one contiguous [32][27] run.
constexpr int kMapVox = 32;

__global__ void __launch_bounds__(27 * kMapVox) neighbor_kernel(const int4* __restrict__ coords, int n,
                                                                const Slot* __restrict__ t, uint64_t mask,
                                                                int* __restrict__ nbr) {
    __shared__ int4 sc[kMapVox];
    __shared__ int sn[kMapVox * 27];
    const int base = blockIdx.x * kMapVox;
    const int tid = threadIdx.x;
    if (tid < kMapVox && base + tid < n) sc[tid] = __ldg(coords + base + tid);
    __syncthreads();
    const int v = tid % kMapVox;
    const int tap = tid / kMapVox;
    if (base + v < n) {
        const int4 c = sc[v];
        const int dx = tap / 9 - 1, dy = (tap / 3) % 3 - 1, dz = tap % 3 - 1;
        const int qx = c.x + dx, qy = c.y + dy, qz = c.z + dz;
        int found = n;
        if (coord_ok(c) && qx >= 0 && qy >= 0 && qz >= 0 && qx <= kAxisMax && qy <= kAxisMax && qz <= kAxisMax) {
            const int idx = table_find(t, mask, pack_key(qx, qy, qz, c.w));
            if (idx >= 0) found = idx;
        }
        sn[v * 27 + tap] = found;
    }
    __syncthreads();
    const int count = min(kMapVox, n - base) * 27;
    int* out = nbr + static_cast<int64_t>(base) * 27;
    for (int k = tid; k < count; k += blockDim.x) out[k] = sn[k];
}

// ---- downsample ----------------------------------------------------------

__global__ void parent_insert_kernel(const int4* __restrict__ coords, int n, Slot* __restrict__ tp, uint64_t pmask,
                                     uint32_t* status) {
    const int i = blockIdx.x * blockDim.x + threadIdx.x;
    if (i >= n) return;
    const int4 c = __ldg(coords + i);
    if (!coord_ok(c)) {
        set_status(status, MSC_DEV_BAD_COORD);
        return;
    }
    // the parent table only needs min-index semantics; duplicates of a
    // parent key are the normal case, so no duplicate flag here
    const unsigned long long key = pack_key(c.x >> 1, c.y >> 1, c.z >> 1, c.w);
    uint64_t h = mix64(key) & pmask;
    for (uint64_t probe = 0; probe <= pmask; ++probe) {
        const unsigned long long prev = atomicCAS(&tp[h].key, kEmpty, key);
        if (prev == kEmpty || prev == key) {
            atomicMin(&tp[h].val, i);
            return;
        }
        h = (h + 1) & pmask;
    }
    set_status(status, MSC_DEV_HASH_FULL);
}

constexpr int kScanBlock = 1024;

// Pass 1: first[i] = (i is the first child of its parent); per-block
// exclusive scan into excl[], block totals into bsum[].
__global__ void __launch_bounds__(kScanBlock) first_scan_kernel(const int4* __restrict__ coords, int n,
                                                                const Slot* __restrict__ tp, uint64_t pmask,
                                                                int* __restrict__ excl, int* __restrict__ bsum) {
    __shared__ int warp_tot[kScanBlock / 32];
    const int i = blockIdx.x * kScanBlock + threadIdx.x;
    int f = 0;
    if (i < n) {
        const int4 c = __ldg(coords + i);
        if (coord_ok(c)) f = table_find(tp, pmask, pack_key(c.x >> 1, c.y >> 1, c.z >> 1, c.w)) == i;
    }
    const int lane = threadIdx.x & 31, warp = threadIdx.x >> 5;
    int inc = f;
#pragma unroll
    for (int o = 1; o < 32; o <<= 1) {
        const int v = __shfl_up_sync(0xffffffffu, inc, o);
        if (lane >= o) inc += v;
    }
    if (lane == 31) warp_tot[warp] = inc;
    __syncthreads();
    if (warp == 0) {
        int w = warp_tot[lane];
        int wi = w;
#pragma unroll
        for (int o = 1; o < 32; o <<= 1) {
            const int v = __shfl_up_sync(0xffffffffu, wi, o);
            if (lane >= o) wi += v;
        }
        warp_tot[lane] = wi - w;
        if (lane == 31) bsum[blockIdx.x] = wi;
    }
    __syncthreads();
    if (i < n) excl[i] = warp_tot[warp] + inc - f;
}

// Pass 2: single block, exclusive scan of block totals; np -> *np_out.
__global__ void __launch_bounds__(kScanBlock) block_scan_kernel(int* __restrict__ bsum, int nblocks,
                                                                int* __restrict__ np_out) {
    __shared__ int warp_tot[kScanBlock / 32];
    __shared__ int carry;
    if (threadIdx.x == 0) carry = 0;
    __syncthreads();
    const int lane = threadIdx.x & 31, warp = threadIdx.x >> 5;
    for (int base = 0; base < nblocks; base += kScanBlock) {
        const int i = base + threadIdx.x;
        const int f = i < nblocks ? bsum[i] : 0;
        int inc = f;
#pragma unroll
        for (int o = 1; o < 32; o <<= 1) {
            const int v = __shfl_up_sync(0xffffffffu, inc, o);
            if (lane >= o) inc += v;
        }
        if (lane == 31) warp_tot[warp] = inc;
        __syncthreads();
        if (warp == 0) {
            int w = warp_tot[lane];
            int wi = w;
#pragma unroll
            for (int o = 1; o < 32; o <<= 1) {
                const int v = __shfl_up_sync(0xffffffffu, wi, o);
                if (lane >= o) wi += v;
            }
            warp_tot[lane] = wi - w;
        }
        __syncthreads();
        const int c0 = carry;
        if (i < nblocks) bsum[i] = c0 + warp_tot[warp] + inc - f;
        __syncthreads();
        if (threadIdx.x == kScanBlock - 1) carry = c0 + warp_tot[warp] + inc;
        __syncthreads();
    }
    if (threadIdx.x == 0) *np_out = carry;
}

// Pass 3: parent ids, up_rows, parent coordinates.
__global__ void assign_kernel(const int4* __restrict__ coords, int n, const Slot* __restrict__ tp, uint64_t pmask,
                              const int* __restrict__ excl, const int* __restrict__ bsum, int4* __restrict__ parent,
                              int* __restrict__ up_rows) {
    const int i = blockIdx.x * blockDim.x + threadIdx.x;
    if (i >= n) return;
    const int4 c = __ldg(coords + i);
    if (!coord_ok(c)) return;
    const int first = table_find(tp, pmask, pack_key(c.x >> 1, c.y >> 1, c.z >> 1, c.w));
    if (first < 0 || first >= n) return;
    const int pid = excl[first] + bsum[first / kScanBlock];
    up_rows[i] = pid;
    if (first == i) parent[pid] = make_int4(c.x >> 1, c.y >> 1, c.z >> 1, c.w);
}

__global__ void pool_fill_kernel(int* __restrict__ pool_rows, const int* __restrict__ np_dev, int nfine) {
    const int64_t total = 8ll * (*np_dev);
    for (int64_t k = blockIdx.x * static_cast<int64_t>(blockDim.x) + threadIdx.x; k < total;
         k += static_cast<int64_t>(gridDim.x) * blockDim.x)
        pool_rows[k] = nfine;
}

// Pass 4: slot = number of siblings with a smaller fine index.
__global__ void slot_kernel(const int4* __restrict__ coords, int n, const Slot* __restrict__ tf, uint64_t fmask,
                            const int* __restrict__ up_rows, const int* __restrict__ np_dev, int* __restrict__ pool_rows,
                            float* __restrict__ inv_count, uint32_t* status) {
    const int i = blockIdx.x * blockDim.x + threadIdx.x;
    if (i >= n) return;
    const int4 c = __ldg(coords + i);
    if (!coord_ok(c)) return;
    const int px = c.x >> 1, py = c.y >> 1, pz = c.z >> 1;
    int count = 0, rank = 0;
#pragma unroll
    for (int o = 0; o < 8; ++o) {
        const int j = table_find(tf, fmask, pack_key(2 * px + (o >> 2), 2 * py + ((o >> 1) & 1), 2 * pz + (o & 1), c.w));
        if (j >= 0) {
            ++count;
            rank += j < i;
        }
    }
    const int pid = up_rows[i];
    const int np = *np_dev;
    if (pid < 0 || pid >= np || rank >= 8) {
        set_status(status, MSC_DEV_POOL_OVERFLOW);
        return;
    }
    pool_rows[static_cast<int64_t>(rank) * np + pid] = i;
    if (rank == 0) inv_count[pid] = 1.0f / static_cast<float>(count);
}

uint64_t table_capacity(int64_t n) {
    uint64_t cap = 64;
    while (cap < static_cast<uint64_t>(2 * n)) cap <<= 1;
    return cap;
}

// ---- brick map (make_level) ----------------------------------------------
// Voxels are grouped into 4 x 4 x 4 bricks: a small hash table maps a brick
// key (b, z >> 2, y >> 2, x >> 2) to a brick id (numbered in arrival order),
// and a brick record holds the 64 voxel indices of its cells (INT_MAX =
// empty; the smallest index of a duplicated coordinate, FlatCoordMap's
// first-insert rule).  A neighbour query is one brick-table probe plus one
// record read.  Surfaces fill a brick with ~15-40 voxels, so the table and
// the records are a few tens of MB and stay in L2, and the 32 voxels of a
// query warp (consecutive rows, mostly one or two bricks) probe the same
// slots.  Inputs too sparse for the record budget (more than n / 4 + 1024
// bricks) take the per-voxel hash instead; the choice is made on the device.
constexpr int kBrickVox = 64;
constexpr int kNoVoxel = 0x7fffffff;

int64_t brick_budget(int64_t n) { return n / 4 + 1024; }
uint64_t brick_capacity(int64_t n) {
    uint64_t cap = 64;
    while (cap < static_cast<uint64_t>(2 * brick_budget(n))) cap <<= 1;
    return cap;
}

__device__ __forceinline__ unsigned long long brick_key(int x, int y, int z, int b) {
    return pack_key(x >> 2, y >> 2, z >> 2, b);
}
__device__ __forceinline__ int brick_cell(int x, int y, int z) { return (x & 3) | ((y & 3) << 2) | ((z & 3) << 4); }

// ctr[0] = bricks numbered so far (forced above the budget when the table
// runs out, which selects the per-voxel hash)
__global__ void brick_insert_kernel(const int4* __restrict__ coords, int n, Slot* __restrict__ t, uint64_t mask,
                                    int* __restrict__ ctr, int budget, uint32_t* status) {
    const int i = blockIdx.x * blockDim.x + threadIdx.x;
    if (i >= n) return;
    const int4 c = __ldg(coords + i);
    if (!coord_ok(c)) {
        set_status(status, MSC_DEV_BAD_COORD);
        return;
    }
    const unsigned long long key = brick_key(c.x, c.y, c.z, c.w);
    uint64_t h = mix64(key) & mask;
    for (uint64_t probe = 0; probe <= mask; ++probe) {
        const unsigned long long prev = atomicCAS(&t[h].key, kEmpty, key);
        if (prev == kEmpty) {
            t[h].val = atomicAdd(ctr, 1);
            return;
        }
        if (prev == key) return;
        h = (h + 1) & mask;
    }
    atomicMax(ctr, budget + 1);
}

__global__ void brick_clear_kernel(int* __restrict__ rec, const int* __restrict__ ctr, int budget) {
    const int nb = *ctr;
    if (nb > budget) return;
    const int64_t total = static_cast<int64_t>(nb) * kBrickVox;
    for (int64_t e = blockIdx.x * static_cast<int64_t>(blockDim.x) + threadIdx.x; e < total;
         e += static_cast<int64_t>(gridDim.x) * blockDim.x)
        rec[e] = kNoVoxel;
}

__device__ __forceinline__ int brick_find(const Slot* __restrict__ t, uint64_t mask, unsigned long long key) {
    return table_find(t, mask, key);
}

__global__ void brick_fill_kernel(const int4* __restrict__ coords, int n, const Slot* __restrict__ t, uint64_t mask,
                                  int* __restrict__ rec, const int* __restrict__ ctr, int budget, uint32_t* status) {
    if (*ctr > budget) return;
    const int i = blockIdx.x * blockDim.x + threadIdx.x;
    if (i >= n) return;
    const int4 c = __ldg(coords + i);
    if (!coord_ok(c)) return;
    const int id = brick_find(t, mask, brick_key(c.x, c.y, c.z, c.w));
    if (id < 0) return;  // cannot happen: every voxel's brick was inserted
    const int old = atomicMin(&rec[static_cast<int64_t>(id) * kBrickVox + brick_cell(c.x, c.y, c.z)], i);
    if (old != kNoVoxel) set_status(status, MSC_DEV_DUP_COORD);
}

__global__ void __launch_bounds__(27 * kMapVox) brick_neighbor_kernel(const int4* __restrict__ coords, int n,
                                                                      const Slot* __restrict__ t, uint64_t mask,
                                                                      const int* __restrict__ rec,
                                                                      const int* __restrict__ ctr, int budget,
                                                                      int* __restrict__ nbr) {
    if (*ctr > budget) return;
    __shared__ int4 sc[kMapVox];
    __shared__ int sn[kMapVox * 27];
    const int base = blockIdx.x * kMapVox;
    const int tid = threadIdx.x;
    if (tid < kMapVox && base + tid < n) sc[tid] = __ldg(coords + base + tid);
    __syncthreads();
    const int v = tid % kMapVox;
    const int tap = tid / kMapVox;
    if (base + v < n) {
        const int4 c = sc[v];
        const int dx = tap / 9 - 1, dy = (tap / 3) % 3 - 1, dz = tap % 3 - 1;
        const int qx = c.x + dx, qy = c.y + dy, qz = c.z + dz;
        int found = n;
        if (coord_ok(c) && qx >= 0 && qy >= 0 && qz >= 0 && qx <= kAxisMax && qy <= kAxisMax && qz <= kAxisMax) {
            const int id = brick_find(t, mask, brick_key(qx, qy, qz, c.w));
            if (id >= 0) {
                const int j = __ldg(rec + static_cast<int64_t>(id) * kBrickVox + brick_cell(qx, qy, qz));
                if (j != kNoVoxel) found = j;
            }
        }
        sn[v * 27 + tap] = found;
    }
    __syncthreads();
    const int count = min(kMapVox, n - base) * 27;
    int* out = nbr + static_cast<int64_t>(base) * 27;
    for (int k = tid; k < count; k += blockDim.x) out[k] = sn[k];
}

// The per-voxel hash path, run only when the brick count exceeded the budget.
__global__ void gated_clear_kernel(Slot* __restrict__ t, uint64_t cap, const int* __restrict__ ctr, int budget) {
    if (*ctr <= budget) return;
    for (uint64_t i = blockIdx.x * static_cast<uint64_t>(blockDim.x) + threadIdx.x; i < cap;
         i += static_cast<uint64_t>(gridDim.x) * blockDim.x) {
        Slot s;
        s.key = kEmpty;
        s.val = 0x7fffffff;
        s.pad = 0;
        t[i] = s;
    }
}

__global__ void gated_insert_kernel(const int4* __restrict__ coords, int n, Slot* __restrict__ t, uint64_t mask,
                                    const int* __restrict__ ctr, int budget, uint32_t* status) {
    if (*ctr <= budget) return;
    const int i = blockIdx.x * blockDim.x + threadIdx.x;
    if (i >= n) return;
    const int4 c = __ldg(coords + i);
    if (!coord_ok(c)) return;  // reported by the brick insert
    if (!table_insert(t, mask, pack_key(c.x, c.y, c.z, c.w), i, status)) set_status(status, MSC_DEV_HASH_FULL);
}

__global__ void __launch_bounds__(27 * kMapVox) gated_neighbor_kernel(const int4* __restrict__ coords, int n,
                                                                      const Slot* __restrict__ t, uint64_t mask,
                                                                      const int* __restrict__ ctr, int budget,
                                                                      int* __restrict__ nbr) {
    if (*ctr <= budget) return;
    __shared__ int4 sc[kMapVox];
    __shared__ int sn[kMapVox * 27];
    const int base = blockIdx.x * kMapVox;
    const int tid = threadIdx.x;
    if (tid < kMapVox && base + tid < n) sc[tid] = __ldg(coords + base + tid);
    __syncthreads();
    const int v = tid % kMapVox;
    const int tap = tid / kMapVox;
    if (base + v < n) {
        const int4 c = sc[v];
        const int dx = tap / 9 - 1, dy = (tap / 3) % 3 - 1, dz = tap % 3 - 1;
        const int qx = c.x + dx, qy = c.y + dy, qz = c.z + dz;
        int found = n;
        if (coord_ok(c) && qx >= 0 && qy >= 0 && qz >= 0 && qx <= kAxisMax && qy <= kAxisMax && qz <= kAxisMax) {
            const int idx = table_find(t, mask, pack_key(qx, qy, qz, c.w));
            if (idx >= 0) found = idx;
        }
        sn[v * 27 + tap] = found;
    }
    __syncthreads();
    const int count = min(kMapVox, n - base) * 27;
    int* out = nbr + static_cast<int64_t>(base) * 27;
    for (int k = tid; k < count; k += blockDim.x) out[k] = sn[k];
}

size_t align_up(size_t v, size_t a) { return (v + a - 1) / a * a; }

}  // namespace

size_t topology_workspace_bytes(int64_t n) {
    const uint64_t cap = table_capacity(n);
    const int64_t nblk = (n + kScanBlock - 1) / kScanBlock + 1;
    // downsample: fine and parent tables + scan arrays; make_level: the
    // per-voxel table (first half of the pair), then the brick table, the
    // brick records and the counter
    const size_t down = align_up(2 * cap * sizeof(Slot), 256) + align_up(static_cast<size_t>(n + 1) * 4, 256) +
                        align_up(static_cast<size_t>(nblk) * 4, 256) + 256;
    const size_t level = align_up(cap * sizeof(Slot), 256) + align_up(brick_capacity(n) * sizeof(Slot), 256) +
                         align_up(static_cast<size_t>(brick_budget(n)) * kBrickVox * 4, 256) + 256;
    return down > level ? down : level;
}

cudaError_t launch_make_level(const int32_t* coords, int64_t n, int32_t* nbr, void* ws, uint32_t* status,
                              cudaStream_t st) {
    if (n == 0) return cudaSuccess;
    const uint64_t cap = table_capacity(n);
    const uint64_t bcap = brick_capacity(n);
    const int budget = static_cast<int>(brick_budget(n));
    char* p = static_cast<char*>(ws);
    Slot* t = reinterpret_cast<Slot*>(p);
    p += align_up(cap * sizeof(Slot), 256);
    Slot* bt = reinterpret_cast<Slot*>(p);
    p += align_up(bcap * sizeof(Slot), 256);
    int* rec = reinterpret_cast<int*>(p);
    p += align_up(static_cast<size_t>(budget) * kBrickVox * 4, 256);
    int* ctr = reinterpret_cast<int*>(p);
    const auto* c4 = reinterpret_cast<const int4*>(coords);
    const int ni = static_cast<int>(n);
    const unsigned g = static_cast<unsigned>((n + 255) / 256);
    const unsigned gm = static_cast<unsigned>((n + kMapVox - 1) / kMapVox);
    cudaError_t e = cudaMemsetAsync(ctr, 0, sizeof(int), st);
    if (e != cudaSuccess) return e;
    table_clear_kernel<<<static_cast<unsigned>((bcap + 255) / 256), 256, 0, st>>>(bt, bcap);
    brick_insert_kernel<<<g, 256, 0, st>>>(c4, ni, bt, bcap - 1, ctr, budget, status);
    brick_clear_kernel<<<592, 256, 0, st>>>(rec, ctr, budget);
    brick_fill_kernel<<<g, 256, 0, st>>>(c4, ni, bt, bcap - 1, rec, ctr, budget, status);
    brick_neighbor_kernel<<<gm, 27 * kMapVox, 0, st>>>(c4, ni, bt, bcap - 1, rec, ctr, budget, nbr);
    // too many bricks: the per-voxel hash (these kernels return at once otherwise)
    gated_clear_kernel<<<592, 256, 0, st>>>(t, cap, ctr, budget);
    gated_insert_kernel<<<g, 256, 0, st>>>(c4, ni, t, cap - 1, ctr, budget, status);
    gated_neighbor_kernel<<<gm, 27 * kMapVox, 0, st>>>(c4, ni, t, cap - 1, ctr, budget, nbr);
    return cudaGetLastError();
}

size_t topology_table_bytes(int64_t n) { return table_capacity(n) * sizeof(Slot); }

cudaError_t launch_make_level_in_table(const int32_t* coords, int64_t n, int32_t* nbr, void* table,
                                       size_t table_bytes, uint32_t* status, cudaStream_t st) {
    if (n == 0) return cudaSuccess;
    const uint64_t cap = table_capacity(n);
    if (cap * sizeof(Slot) > table_bytes) return cudaErrorInvalidValue;
    Slot* t = static_cast<Slot*>(table);
    table_clear_kernel<<<static_cast<unsigned>((cap + 255) / 256), 256, 0, st>>>(t, cap);
    const auto* c4 = reinterpret_cast<const int4*>(coords);
    insert_kernel<<<static_cast<unsigned>((n + 255) / 256), 256, 0, st>>>(c4, static_cast<int>(n), t, cap - 1,
                                                                          status);
    neighbor_kernel<<<static_cast<unsigned>((n + kMapVox - 1) / kMapVox), 27 * kMapVox, 0, st>>>(
        c4, static_cast<int>(n), t, cap - 1, nbr);
    return cudaGetLastError();
}

cudaError_t launch_downsample(const int32_t* coords, int64_t n, int32_t* parent, int32_t* np_dev, int32_t* pool_rows,
                              float* inv_count, int32_t* up_rows, void* ws, uint32_t* status, cudaStream_t st) {
    if (n == 0) {
        return cudaMemsetAsync(np_dev, 0, sizeof(int32_t), st);
    }
    const uint64_t cap = table_capacity(n);
    char* p = static_cast<char*>(ws);
    Slot* tf = reinterpret_cast<Slot*>(p);
    Slot* tp = tf + cap;
    p += align_up(2 * cap * sizeof(Slot), 256);
    int* excl = reinterpret_cast<int*>(p);
    p += align_up(static_cast<size_t>(n + 1) * 4, 256);
    int* bsum = reinterpret_cast<int*>(p);
    const int nblk = static_cast<int>((n + kScanBlock - 1) / kScanBlock);
    const auto* c4 = reinterpret_cast<const int4*>(coords);
    const int ni = static_cast<int>(n);
    const unsigned g = static_cast<unsigned>((n + 255) / 256);
    table_clear_kernel<<<static_cast<unsigned>((2 * cap + 255) / 256), 256, 0, st>>>(tf, 2 * cap);
    insert_kernel<<<g, 256, 0, st>>>(c4, ni, tf, cap - 1, status);
    parent_insert_kernel<<<g, 256, 0, st>>>(c4, ni, tp, cap - 1, status);
    first_scan_kernel<<<nblk, kScanBlock, 0, st>>>(c4, ni, tp, cap - 1, excl, bsum);
    block_scan_kernel<<<1, kScanBlock, 0, st>>>(bsum, nblk, np_dev);
    assign_kernel<<<g, 256, 0, st>>>(c4, ni, tp, cap - 1, excl, bsum, reinterpret_cast<int4*>(parent), up_rows);
    pool_fill_kernel<<<592, 256, 0, st>>>(pool_rows, np_dev, ni);
    slot_kernel<<<g, 256, 0, st>>>(c4, ni, tf, cap - 1, up_rows, np_dev, pool_rows, inv_count, status);
    return cudaGetLastError();
}

}  // namespace msc
