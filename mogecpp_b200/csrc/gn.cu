// Sample-wide GroupNorm statistics for the GroupNorm residual-block variant.
//
// Follows ggml's group_norm_f32 (ggml-cpu/ops.cpp:4208-4283) on the
// [C, N] features viewed as [N, 1, C] per sample: for each (sample, group
// of C/32 channels) the mean of the group's values over the sample's
// voxels and their variance, scale = 1 / sqrtf(var + eps).  ggml makes two
// passes (a double sum for the mean, then a double sum of the float squares
// of x - mean); this makes one, with double sums of x and x * x and
// var = E[x^2] - mean^2 in double, which equals the two-pass value to
// double rounding unless |mean| / std approaches 1e6 (the float variance
// is then the same to within an ulp).  One read of the features instead of
// two, and one all-reduce of the statistics for sharded runs.  The apply
// step (normalise, per-channel affine, SiLU, operand preparation) is fused
// into act_prepare (prep.cu).
//
// Statistics buffer (doubles, caller-owned so that sharded runs can
// all-reduce it before the finalize):
//   [nsamples * 32] group sums | [nsamples] voxel counts | [nsamples * 32] group sums of squares
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

// Group sums, sums of squares and voxel counts of rows [0, n_stat); the
// sample index of rows [n_stat, n) (halo rows, normalised but not counted)
// is checked.  A warp takes kRowsPerWarp consecutive rows: their sample
// indices are read 32 at a time (one per lane) and their features kUnroll
// rows at a time, all loads in flight before the first row is accumulated.
template <int C>
__global__ void gn_stats_kernel(const float* __restrict__ x, const int4* __restrict__ coords, int64_t n,
                                int64_t n_stat, int nsamples, double* stats, uint32_t* status) {
    constexpr int EPL = C / 32;
    const int lane = threadIdx.x & 31;
    const int64_t warp = (blockIdx.x * static_cast<int64_t>(blockDim.x) + threadIdx.x) >> 5;
    const int64_t r0 = warp * kRowsPerWarp;
    if (r0 >= n) return;
    {
        const int64_t r2 = r0 + kRowsPerWarp < n ? r0 + kRowsPerWarp : n;
        for (int64_t r = (r0 > n_stat ? r0 : n_stat) + lane; r < r2; r += 32) sample_of(coords, r, nsamples, status);
    }
    if (r0 >= n_stat) return;
    const int64_t r1 = r0 + kRowsPerWarp < n_stat ? r0 + kRowsPerWarp : n_stat;
    double* sums = stats;
    double* counts = stats + static_cast<int64_t>(nsamples) * 32;
    double* sq = stats + static_cast<int64_t>(nsamples) * 33;
    int cur = -1;
    double acc = 0.0, acc2 = 0.0, cnt = 0.0;
    auto flush = [&]() {
        atomicAdd(sums + cur * 32 + lane, acc);
        atomicAdd(sq + cur * 32 + lane, acc2);
        if (lane == 0) atomicAdd(counts + cur, cnt);
    };
    for (int64_t base = r0; base < r1; base += 32) {
        const int m = r1 - base < 32 ? static_cast<int>(r1 - base) : 32;
        const int bl = lane < m ? sample_of(coords, base + lane, nsamples, status) : -1;
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
                    if (cur >= 0) flush();
                    cur = b, acc = 0.0, acc2 = 0.0, cnt = 0.0;
                }
#pragma unroll
                for (int k = 0; k < EPL; ++k) {
                    const double d = static_cast<double>(v[u][k]);
                    acc += d;
                    acc2 = fma(d, d, acc2);
                }
                cnt += 1.0;
            }
        }
    }
    if (cur >= 0) flush();
}

// mean and 1 / sqrtf(var + eps) per (sample, group)
template <int C>
__global__ void gn_finalize_kernel(const double* stats, int nsamples, float eps, float2* gn) {
    const int i = blockIdx.x * blockDim.x + threadIdx.x;
    if (i >= nsamples * 32) return;
    const int b = i / 32;
    const double cnt = stats[static_cast<int64_t>(nsamples) * 32 + b] * (C / 32);
    double mean = 0.0, var = 0.0;
    if (cnt > 0.0) {
        mean = stats[i] / cnt;
        var = stats[static_cast<int64_t>(nsamples) * 33 + i] / cnt - mean * mean;
        var = var > 0.0 ? var : 0.0;
    }
    gn[i] = make_float2(static_cast<float>(mean), 1.0f / sqrtf(static_cast<float>(var) + eps));
}

template <int C>
cudaError_t launch_stats(const float* x, const int32_t* coords, int64_t n, int64_t n_stat, int nsamples,
                         double* stats, uint32_t* status, cudaStream_t st) {
    const int64_t warps = (n + kRowsPerWarp - 1) / kRowsPerWarp;
    const unsigned grid = static_cast<unsigned>((warps * 32 + 255) / 256);
    if (grid == 0) return cudaSuccess;
    gn_stats_kernel<C><<<grid, 256, 0, st>>>(x, reinterpret_cast<const int4*>(coords), n, n_stat, nsamples, stats,
                                             status);
    return cudaGetLastError();
}

}  // namespace

int64_t gn_stats_doubles(int nsamples) { return static_cast<int64_t>(nsamples) * (2 * 32 + 1); }

cudaError_t launch_gn_stats(const float* x, int c, const int32_t* coords, int64_t n, int64_t n_stat,
                            int nsamples, double* stats, uint32_t* status, cudaStream_t st) {
    if (n_stat > n) return cudaErrorInvalidValue;
    if (c == 64) return launch_stats<64>(x, coords, n, n_stat, nsamples, stats, status, st);
    if (c == 128) return launch_stats<128>(x, coords, n, n_stat, nsamples, stats, status, st);
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
