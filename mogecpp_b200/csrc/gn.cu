// Sample-wide GroupNorm statistics for the GroupNorm residual-block variant.
//
// Restates ggml's group_norm_f32 (ggml-cpu/ops.cpp:4208-4283) on the
// [C, N] features viewed as [N, 1, C] per sample: for each (sample, group
// of C/32 channels) the mean of the group's values over the sample's
// voxels (double sum), then the variance of the float differences x - mean
// (double sum of float squares), scale = 1 / sqrtf(var + eps).  The apply
// step (normalise, per-channel affine, SiLU, operand preparation) is fused
// into act_prepare (prep.cu).
//
// Statistics buffer (doubles, caller-owned so that sharded runs can
// all-reduce it between the passes):
//   [nsamples * 32] group sums | [nsamples] voxel counts | [nsamples * 32] squared deviations
//
// One warp per chunk of rows; lane l holds the C/32 channels of group l, so
// a lane accumulates one group (each value added in double, as ggml) and
// flushes it with one double atomic add whenever the row's sample changes
// (rows are normally sorted by sample).
#include "common.cuh"
#include "gn.h"

namespace msc {
namespace {

constexpr int kRowsPerWarp = 128;
constexpr int kUnroll = 8;

template <int C>
__device__ __forceinline__ void load_group(const float* x, int64_t row, int lane, float (&v)[C / 32]) {
    constexpr int EPL = C / 32;
    const float* p = x + row * C + lane * EPL;
    if constexpr (EPL == 4) {
        const float4 t = *reinterpret_cast<const float4*>(p);
        v[0] = t.x, v[1] = t.y, v[2] = t.z, v[3] = t.w;
    } else if constexpr (EPL == 2) {
        const float2 t = *reinterpret_cast<const float2*>(p);
        v[0] = t.x, v[1] = t.y;
    } else {
#pragma unroll
        for (int k = 0; k < EPL; ++k) v[k] = p[k];
    }
}

__device__ __forceinline__ int sample_of(const int4* coords, int64_t row, int nsamples, uint32_t* status) {
    const int b = __ldg(coords + row).w;
    if (static_cast<unsigned>(b) >= static_cast<unsigned>(nsamples)) {
        set_status(status, MSC_DEV_BAD_COORD);
        return -1;
    }
    return b;
}

// PASS 1: group sums and voxel counts of rows [0, n_stat), and the sample
// index of rows [n_stat, n) (halo rows, normalised but not counted) checked.
// PASS 2: squared deviations from the complete group means.
// A warp takes kRowsPerWarp consecutive rows: their sample indices are read
// 32 at a time (one per lane) and their features kUnroll rows at a time, all
// loads in flight before the first row is accumulated.
template <int C, int PASS>
__global__ void gn_pass_kernel(const float* __restrict__ x, const int4* __restrict__ coords, int64_t n,
                               int64_t n_stat, int nsamples, double* stats, uint32_t* status) {
    constexpr int EPL = C / 32;
    const int lane = threadIdx.x & 31;
    const int64_t warp = (blockIdx.x * static_cast<int64_t>(blockDim.x) + threadIdx.x) >> 5;
    const int64_t r0 = warp * kRowsPerWarp;
    if (r0 >= n) return;
    if (PASS == 1) {
        const int64_t r2 = r0 + kRowsPerWarp < n ? r0 + kRowsPerWarp : n;
        for (int64_t r = (r0 > n_stat ? r0 : n_stat) + lane; r < r2; r += 32) sample_of(coords, r, nsamples, status);
    }
    if (r0 >= n_stat) return;
    const int64_t r1 = r0 + kRowsPerWarp < n_stat ? r0 + kRowsPerWarp : n_stat;
    double* sums = stats;
    double* counts = stats + static_cast<int64_t>(nsamples) * 32;
    double* sq = stats + static_cast<int64_t>(nsamples) * 33;
    int cur = -1;
    float mean = 0.0f;
    double acc = 0.0, cnt = 0.0;
    for (int64_t base = r0; base < r1; base += 32) {
        const int m = r1 - base < 32 ? static_cast<int>(r1 - base) : 32;
        const int bl = lane < m ? sample_of(coords, base + lane, nsamples, PASS == 1 ? status : nullptr) : -1;
        for (int j = 0; j < m; j += kUnroll) {
            float v[kUnroll][EPL];
#pragma unroll
            for (int u = 0; u < kUnroll; ++u)
                if (j + u < m) load_group<C>(x, base + j + u, lane, v[u]);
#pragma unroll
            for (int u = 0; u < kUnroll; ++u) {
                const int b = __shfl_sync(0xffffffffu, bl, (j + u) & 31);
                if (j + u >= m || b < 0) continue;
                if (b != cur) {
                    if (cur >= 0) {
                        if (PASS == 1) {
                            atomicAdd(sums + cur * 32 + lane, acc);
                            if (lane == 0) atomicAdd(counts + cur, cnt);
                        } else {
                            atomicAdd(sq + cur * 32 + lane, acc);
                        }
                    }
                    cur = b, acc = 0.0, cnt = 0.0;
                    if (PASS == 2) {
                        const double c = counts[b] * EPL;
                        mean = c > 0.0 ? static_cast<float>(sums[b * 32 + lane] / c) : 0.0f;
                    }
                }
#pragma unroll
                for (int k = 0; k < EPL; ++k) {
                    if (PASS == 1) {
                        acc += static_cast<double>(v[u][k]);
                    } else {
                        const float d = v[u][k] - mean;
                        acc += static_cast<double>(d * d);
                    }
                }
                cnt += 1.0;
            }
        }
    }
    if (cur >= 0) {
        if (PASS == 1) {
            atomicAdd(sums + cur * 32 + lane, acc);
            if (lane == 0) atomicAdd(counts + cur, cnt);
        } else {
            atomicAdd(sq + cur * 32 + lane, acc);
        }
    }
}

// mean and 1 / sqrtf(var + eps) per (sample, group)
template <int C>
__global__ void gn_finalize_kernel(const double* stats, int nsamples, float eps, float2* gn) {
    const int i = blockIdx.x * blockDim.x + threadIdx.x;
    if (i >= nsamples * 32) return;
    const int b = i / 32;
    const double cnt = stats[static_cast<int64_t>(nsamples) * 32 + b] * (C / 32);
    const float mean = cnt > 0.0 ? static_cast<float>(stats[i] / cnt) : 0.0f;
    const float var = cnt > 0.0 ? static_cast<float>(stats[static_cast<int64_t>(nsamples) * 33 + i] / cnt) : 0.0f;
    gn[i] = make_float2(mean, 1.0f / sqrtf(var + eps));
}

template <int C>
cudaError_t launch_pass(int pass, const float* x, const int32_t* coords, int64_t n, int64_t n_stat, int nsamples,
                        double* stats, uint32_t* status, cudaStream_t st) {
    const int64_t warps = ((pass == 1 ? n : n_stat) + kRowsPerWarp - 1) / kRowsPerWarp;
    const unsigned grid = static_cast<unsigned>((warps * 32 + 255) / 256);
    const int4* c4 = reinterpret_cast<const int4*>(coords);
    if (grid == 0) return cudaSuccess;
    if (pass == 1)
        gn_pass_kernel<C, 1><<<grid, 256, 0, st>>>(x, c4, n, n_stat, nsamples, stats, status);
    else
        gn_pass_kernel<C, 2><<<grid, 256, 0, st>>>(x, c4, n, n_stat, nsamples, stats, status);
    return cudaGetLastError();
}

}  // namespace

int64_t gn_stats_doubles(int nsamples) { return static_cast<int64_t>(nsamples) * (2 * 32 + 1); }

cudaError_t launch_gn_pass(int pass, const float* x, int c, const int32_t* coords, int64_t n, int64_t n_stat,
                           int nsamples, double* stats, uint32_t* status, cudaStream_t st) {
    if (n_stat > n) return cudaErrorInvalidValue;
    if (c == 64) return launch_pass<64>(pass, x, coords, n, n_stat, nsamples, stats, status, st);
    if (c == 128) return launch_pass<128>(pass, x, coords, n, n_stat, nsamples, stats, status, st);
    return cudaErrorInvalidValue;
}

cudaError_t launch_gn_finalize(const double* stats, int c, int nsamples, float eps, float2* gn, cudaStream_t st) {
    const unsigned grid = static_cast<unsigned>((nsamples * 32 + 255) / 256);
    if (c == 64)
        gn_finalize_kernel<64><<<grid, 256, 0, st>>>(stats, nsamples, eps, gn);
    else if (c == 128)
        gn_finalize_kernel<128><<<grid, 256, 0, st>>>(stats, nsamples, eps, gn);
    else
        return cudaErrorInvalidValue;
    return cudaGetLastError();
}

}  // namespace msc
