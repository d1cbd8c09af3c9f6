// Stride-2 transition kernels around the per-voxel linear layer:
//
//  * pool_mean: mean over up to 8 children (slot-major pool_rows, sentinel
//    nfine, times inv_count) in fp32, the input of the following linear
//    (mogecpp src/sparse.cpp:646-668 pool_down: the slot gathers are summed
//    in slot order, then scaled).
//  * gather_rows: y[i] = t[rows[i]] (+ skip[i]), the row gather after the
//    linear of nearest_up (src/sparse.cpp:670-674) with the U-Net's additive
//    skip fused in.
#include "common.cuh"
#include "conv.h"
#include "ops.h"

namespace msc {
namespace {

__device__ __forceinline__ float ld(const void* p, int dtype, int64_t i) {
    if (dtype == DT_F32) return static_cast<const float*>(p)[i];
    if (dtype == DT_F16) return __half2float(static_cast<const __half*>(p)[i]);
    return __bfloat162float(static_cast<const __nv_bfloat16*>(p)[i]);
}

__device__ __forceinline__ void st(void* p, int dtype, int64_t i, float v) {
    if (dtype == DT_F32)
        static_cast<float*>(p)[i] = v;
    else if (dtype == DT_F16)
        static_cast<__half*>(p)[i] = __float2half_rn(v);
    else
        static_cast<__nv_bfloat16*>(p)[i] = __float2bfloat16_rn(v);
}

// one thread per (parent, channel): pooled[p][ch] = (sum over slots) * inv_count[p]
__global__ void pool_mean_kernel(const void* x, int x_dtype, int64_t nfine, int c, const int32_t* pool_rows,
                                 const float* inv_count, int64_t np, float* pooled, uint32_t* status) {
    const int64_t total = np * c;
    for (int64_t i = blockIdx.x * static_cast<int64_t>(blockDim.x) + threadIdx.x; i < total;
         i += static_cast<int64_t>(gridDim.x) * blockDim.x) {
        const int64_t p = i / c;
        const int ch = static_cast<int>(i % c);
        float s = 0.0f;
        for (int sl = 0; sl < 8; ++sl) {
            const int32_t r = pool_rows[sl * np + p];
            if (r >= 0 && r < nfine) s += ld(x, x_dtype, static_cast<int64_t>(r) * c + ch);
            else if (r != nfine) set_status(status, MSC_DEV_BAD_INDEX);
        }
        pooled[i] = s * inv_count[p];
    }
}

__global__ void gather_rows_kernel(const float* t, int64_t nsrc, int c, const int32_t* rows, int64_t n,
                                   const void* skip, int skip_dtype, void* y, int y_dtype, uint32_t* status) {
    const int64_t total = n * c;
    for (int64_t i = blockIdx.x * static_cast<int64_t>(blockDim.x) + threadIdx.x; i < total;
         i += static_cast<int64_t>(gridDim.x) * blockDim.x) {
        const int64_t row = i / c;
        const int ch = static_cast<int>(i % c);
        const int32_t r = rows[row];
        float v = 0.0f;
        if (r >= 0 && r < nsrc) v = t[static_cast<int64_t>(r) * c + ch];
        else set_status(status, MSC_DEV_BAD_INDEX);
        if (skip) v += ld(skip, skip_dtype, i);
        st(y, y_dtype, i, v);
    }
}

unsigned grid_for(int64_t total) {
    const int64_t g = (total + 255) / 256;
    return static_cast<unsigned>(g < 148 * 32 ? (g > 0 ? g : 1) : 148 * 32);
}

}  // namespace

cudaError_t launch_pool_mean(const void* x, int x_dtype, int64_t nfine, int c, const int32_t* pool_rows,
                             const float* inv_count, int64_t np, float* pooled, uint32_t* status, cudaStream_t st) {
    if (np == 0) return cudaSuccess;
    pool_mean_kernel<<<grid_for(np * c), 256, 0, st>>>(x, x_dtype, nfine, c, pool_rows, inv_count, np, pooled,
                                                        status);
    return cudaGetLastError();
}

cudaError_t launch_gather_rows(const float* t, int64_t nsrc, int c, const int32_t* rows, int64_t n, const void* skip,
                               int skip_dtype, void* y, int y_dtype, uint32_t* status, cudaStream_t st) {
    if (n == 0) return cudaSuccess;
    gather_rows_kernel<<<grid_for(n * c), 256, 0, st>>>(t, nsrc, c, rows, n, skip, skip_dtype, y, y_dtype, status);
    return cudaGetLastError();
}

}  // namespace msc
