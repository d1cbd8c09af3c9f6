// Neighbour-map entry point that allocates nothing.
//
// Some callers cannot allocate device memory: a host runtime whose device
// memory belongs to another allocator (a ggml backend buffer pool that hands
// out no scratch space), or latency-critical code that must not call
// cudaMalloc because it can synchronise the device.  For them the hash table
// of msc_make_level lives in a fixed array compiled into this library instead
// of a caller-provided workspace.  The caller still passes the coordinates
// and the output map.
//
// The array is kNoAllocTableBytes (16 MiB) per GPU that loads the library and
// is held until the process exits; it fits the table of up to
// kNoAllocMaxVoxels voxels.  All calls share it and it keeps the previous
// call's contents; every call clears the part it uses before inserting.
// Calls whose kernels overlap on the GPU (other streams, other host threads)
// race on the shared table and must be serialised by the caller.
#include "topology.h"

#include "../../include/moge_sparse_cuda.h"

#include <cuda_runtime.h>

#include <mutex>
#include <string>

namespace msc {
void set_last_error(const std::string& msg);
}

namespace {

constexpr size_t kNoAllocTableBytes = size_t(16) << 20;
constexpr int64_t kNoAllocMaxVoxels = 524288;  // hash capacity 2^20 slots of 16 bytes
constexpr int kMaxDevices = 64;

static __device__ __align__(256) unsigned char g_noalloc_table[kNoAllocTableBytes];

// Device address of g_noalloc_table per device.  In host code the array's
// name is a host-side stand-in, not a device address, so it is looked up
// once per device (with that device current) and cached.
void* g_table_ptr[kMaxDevices] = {nullptr};
std::mutex g_table_mu;

int fail(int code, const std::string& msg) {
    msc::set_last_error(msg);
    return code;
}

}  // namespace

extern "C" int msc_make_level_noalloc(const int32_t* coords, int64_t n, int32_t* nbr, uint32_t* status,
                                      void* stream) {
    if (n < 0 || n > kNoAllocMaxVoxels)
        return fail(MSC_E_INVALID, "msc_make_level_noalloc: voxel count " + std::to_string(n) +
                                       " outside [0, " + std::to_string(kNoAllocMaxVoxels) +
                                       "] (fixed 16 MiB table; use msc_make_level with a workspace)");
    if (n == 0) return MSC_OK;
    if (!coords || !nbr) return fail(MSC_E_INVALID, "msc_make_level_noalloc: null pointer");
    if (reinterpret_cast<uintptr_t>(coords) % 16)
        return fail(MSC_E_INVALID, "msc_make_level_noalloc: coords is not 16-byte aligned");
    int dev = -1;
    cudaError_t e = cudaGetDevice(&dev);
    if (e != cudaSuccess) return fail(MSC_E_CUDA, std::string("cudaGetDevice: ") + cudaGetErrorString(e));
    if (dev < 0 || dev >= kMaxDevices) return fail(MSC_E_INVALID, "msc_make_level_noalloc: device index out of range");
    void* table = nullptr;
    {
        std::lock_guard<std::mutex> lk(g_table_mu);
        if (!g_table_ptr[dev]) {
            e = cudaGetSymbolAddress(&g_table_ptr[dev], g_noalloc_table);
            if (e != cudaSuccess) {
                g_table_ptr[dev] = nullptr;
                return fail(MSC_E_CUDA, std::string("cudaGetSymbolAddress: ") + cudaGetErrorString(e));
            }
        }
        table = g_table_ptr[dev];
    }
    e = msc::launch_make_level_in_table(coords, n, nbr, table, kNoAllocTableBytes, status,
                                        static_cast<cudaStream_t>(stream));
    if (e != cudaSuccess) return fail(MSC_E_CUDA, std::string("msc_make_level_noalloc: ") + cudaGetErrorString(e));
    return MSC_OK;
}
