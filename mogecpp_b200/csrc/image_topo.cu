// Level-0 topology of the refiner (one voxel per image pixel) and the
// refiner's per-pixel glue, on the GPU.
//
// quantize_topology_z (mogecpp src/sparse.cpp:363-406): for every pixel,
//     q = nearbyint(double(z * depth_resolution))     (z = log depth, float product)
// then zbin = q - min(q).  fl(z * r) converted to double is exact, so
// rounding the float product to the nearest integer, ties to even (the
// default rounding mode nearbyint uses), gives the same q.
//
// make_dense_image_level (src/sparse.cpp:274-310): pixel i = y * width + x
// holds voxel (row y, column x, zbin[i]); its neighbour at (dy, dx) is pixel
// j = (y + dy) * width + (x + dx), present at tap (dy+1)*9 + (dx+1)*3 +
// (dz+1) when dz = zbin[j] - zbin[i] is in [-1, 1]; every other tap is the
// sentinel n.  No hash: the pixel grid indexes the neighbours directly.
//
// Glue of SparseRefiner::refine_once (src/sparse.cpp:1014-1296):
//   * refiner input: upload_feature (:935-943) writes the three coordinate
//     planes one after another into the buffer that the graph reads as
//     [n][3] rows, so row k, channel c holds plane value p[3k + c] with
//     p[m] = factor_coord[3 (m mod n) + m div n];
//   * small linear layers that do not suit the tensor-core tiles
//     (input_proj 3 -> C, out_proj C -> 1, the fused projection of the
//     deepest level over [x | encoder] rows), computed as ggml's mul_mat
//     does for F32 / F16 weights (F16 weights: activations rounded to fp16);
//   * encoder rows: row of deep voxel (r, c) in the encoder matrix is
//     r * encoder_width + c (upload_encoder_rows, :958-972);
//   * the log-depth update factor_coord[3i + 2] += residual[i] (:1293-1295).
#include "common.cuh"
#include "image_topo.h"

namespace msc {
namespace {

constexpr int kAxisMax = (1 << 19) - 1;

__global__ void zq_minmax_kernel(const float* __restrict__ fc, int64_t n, float dres, long long* __restrict__ mm,
                                 uint32_t* status) {
    long long lo = LLONG_MAX, hi = LLONG_MIN;
    for (int64_t i = blockIdx.x * static_cast<int64_t>(blockDim.x) + threadIdx.x; i < n;
         i += static_cast<int64_t>(gridDim.x) * blockDim.x) {
        const float v = __fmul_rn(fc[3 * i + 2], dres);
        if (!(fabsf(v) < 4.0e18f)) {  // NaN, inf or beyond int64 range
            set_status(status, MSC_DEV_BAD_COORD);
            continue;
        }
        const long long q = __float2ll_rn(v);
        lo = min(lo, q);
        hi = max(hi, q);
    }
#pragma unroll
    for (int o = 16; o > 0; o >>= 1) {
        lo = min(lo, __shfl_xor_sync(0xffffffffu, lo, o));
        hi = max(hi, __shfl_xor_sync(0xffffffffu, hi, o));
    }
    if ((threadIdx.x & 31) == 0) {
        atomicMin(&mm[0], lo);
        atomicMax(&mm[1], hi);
    }
}

__global__ void zq_init_kernel(long long* mm) {
    mm[0] = LLONG_MAX;
    mm[1] = LLONG_MIN;
}

__global__ void zq_write_kernel(const float* __restrict__ fc, int64_t n, float dres, const long long* __restrict__ mm,
                                int32_t* __restrict__ zbin, uint32_t* status) {
    const long long zmin = mm[0];
    if (mm[1] - zmin > kAxisMax) {
        // the reference allows extents up to INT32_MAX; the 64-bit voxel keys
        // here hold 19 bits per axis
        if (blockIdx.x == 0 && threadIdx.x == 0) set_status(status, MSC_DEV_BAD_COORD);
        return;
    }
    for (int64_t i = blockIdx.x * static_cast<int64_t>(blockDim.x) + threadIdx.x; i < n;
         i += static_cast<int64_t>(gridDim.x) * blockDim.x) {
        const float v = __fmul_rn(fc[3 * i + 2], dres);
        zbin[i] = (fabsf(v) < 4.0e18f) ? static_cast<int32_t>(__float2ll_rn(v) - zmin) : 0;
    }
}

// 256 consecutive pixels per block; the [256][27] map rows are staged in
// shared memory and written back as one contiguous run.
constexpr int kImgPix = 256;

__global__ void __launch_bounds__(kImgPix) dense_level_kernel(const int32_t* __restrict__ zbin, int width,
                                                             int height, int32_t* __restrict__ nbr,
                                                             int4* __restrict__ coords) {
    __shared__ int32_t sn[kImgPix * 27];
    const int64_t n = static_cast<int64_t>(width) * height;
    const int64_t base = static_cast<int64_t>(blockIdx.x) * kImgPix;
    const int64_t i = base + threadIdx.x;
    const int32_t sentinel = static_cast<int32_t>(n);
    int32_t* row = sn + threadIdx.x * 27;
#pragma unroll
    for (int t = 0; t < 27; ++t) row[t] = sentinel;
    if (i < n) {
        const int y = static_cast<int>(i / width);
        const int x = static_cast<int>(i - static_cast<int64_t>(y) * width);
        const int z = __ldg(zbin + i);
        coords[i] = make_int4(y, x, z, 0);
#pragma unroll
        for (int dy = -1; dy <= 1; ++dy) {
            const int yy = y + dy;
            if (yy < 0 || yy >= height) continue;
#pragma unroll
            for (int dx = -1; dx <= 1; ++dx) {
                const int xx = x + dx;
                if (xx < 0 || xx >= width) continue;
                const int64_t j = static_cast<int64_t>(yy) * width + xx;
                const int dz = __ldg(zbin + j) - z;
                if (dz < -1 || dz > 1) continue;
                row[(dy + 1) * 9 + (dx + 1) * 3 + (dz + 1)] = static_cast<int32_t>(j);
            }
        }
    }
    __syncthreads();
    const int64_t count = (n - base < kImgPix ? n - base : kImgPix) * 27;
    int32_t* out = nbr + base * 27;
    for (int64_t k = threadIdx.x; k < count; k += kImgPix) out[k] = sn[k];
}

__global__ void refiner_input_kernel(const float* __restrict__ fc, int64_t n, float* __restrict__ feat) {
    for (int64_t k = blockIdx.x * static_cast<int64_t>(blockDim.x) + threadIdx.x; k < 3 * n;
         k += static_cast<int64_t>(gridDim.x) * blockDim.x) {
        const int64_t plane = k / n;
        feat[k] = fc[3 * (k - plane * n) + plane];
    }
}

__device__ __forceinline__ float weight_at(const void* w, int wtype, int64_t idx) {
    return wtype == 0 ? static_cast<const float*>(w)[idx] : __half2float(static_cast<const __half*>(w)[idx]);
}

// y[r][o] = sum_k W[o][k] * in[r][k] + b[o], in = [x1 (c1) | x2 (c2)] rows.
// F16 weights: each activation is rounded to fp16 first (ggml converts the
// activations to the weight's vec_dot type).  One thread per output.
__global__ void small_linear_kernel(const float* __restrict__ x1, int c1, const float* __restrict__ x2, int c2,
                                    int64_t rows, const void* __restrict__ w, int wtype, int cout,
                                    const float* __restrict__ bias, float* __restrict__ y) {
    const int cin = c1 + c2;
    for (int64_t e = blockIdx.x * static_cast<int64_t>(blockDim.x) + threadIdx.x; e < rows * cout;
         e += static_cast<int64_t>(gridDim.x) * blockDim.x) {
        const int64_t r = e / cout;
        const int o = static_cast<int>(e - r * cout);
        float s = 0.0f;
        for (int k = 0; k < cin; ++k) {
            float a = k < c1 ? x1[r * c1 + k] : x2[r * c2 + (k - c1)];
            if (wtype == 1) a = __half2float(__float2half_rn(a));
            s = fmaf(weight_at(w, wtype, static_cast<int64_t>(o) * cin + k), a, s);
        }
        y[e] = s + (bias ? bias[o] : 0.0f);
    }
}

__global__ void silu_inplace_kernel(float* __restrict__ x, int64_t n) {
    for (int64_t i = blockIdx.x * static_cast<int64_t>(blockDim.x) + threadIdx.x; i < n;
         i += static_cast<int64_t>(gridDim.x) * blockDim.x)
        x[i] = silu_f(x[i]);
}

__global__ void encoder_rows_kernel(const int4* __restrict__ deep, int64_t n, const float* __restrict__ enc, int ew,
                                    int eh, int cenc, float* __restrict__ out, uint32_t* status) {
    for (int64_t e = blockIdx.x * static_cast<int64_t>(blockDim.x) + threadIdx.x; e < n * cenc;
         e += static_cast<int64_t>(gridDim.x) * blockDim.x) {
        const int64_t i = e / cenc;
        const int c = static_cast<int>(e - i * cenc);
        const int4 q = deep[i];
        if (q.y < 0 || q.x < 0 || q.y >= ew || q.x >= eh) {
            set_status(status, MSC_DEV_BAD_INDEX);
            out[e] = 0.0f;
            continue;
        }
        out[e] = enc[(static_cast<int64_t>(q.x) * ew + q.y) * cenc + c];
    }
}

__global__ void logz_update_kernel(float* __restrict__ fc, const float* __restrict__ res, int64_t n) {
    for (int64_t i = blockIdx.x * static_cast<int64_t>(blockDim.x) + threadIdx.x; i < n;
         i += static_cast<int64_t>(gridDim.x) * blockDim.x)
        fc[3 * i + 2] += res[i];
}

__global__ void keys_differ_kernel(const int32_t* __restrict__ a, const int32_t* __restrict__ b, int64_t n,
                                   int* __restrict__ differ) {
    bool d = false;
    for (int64_t i = blockIdx.x * static_cast<int64_t>(blockDim.x) + threadIdx.x; i < n;
         i += static_cast<int64_t>(gridDim.x) * blockDim.x)
        d |= a[i] != b[i];
    if (__any_sync(0xffffffffu, d) && (threadIdx.x & 31) == 0) atomicOr(differ, 1);
}

unsigned grid_for(int64_t total, int per = 256) {
    const int64_t g = (total + per - 1) / per;
    return static_cast<unsigned>(g < 148 * 32 ? (g > 0 ? g : 1) : 148 * 32);
}

}  // namespace

size_t quantize_z_workspace_bytes() { return 256; }

cudaError_t launch_quantize_topology_z(const float* fc, int64_t n, float dres, int32_t* zbin, void* ws,
                                       uint32_t* status, cudaStream_t st) {
    if (n == 0) return cudaSuccess;
    auto* mm = static_cast<long long*>(ws);
    zq_init_kernel<<<1, 1, 0, st>>>(mm);
    zq_minmax_kernel<<<grid_for(n), 256, 0, st>>>(fc, n, dres, mm, status);
    zq_write_kernel<<<grid_for(n), 256, 0, st>>>(fc, n, dres, mm, zbin, status);
    return cudaGetLastError();
}

cudaError_t launch_dense_image_level(const int32_t* zbin, int width, int height, int32_t* coords, int32_t* nbr,
                                     cudaStream_t st) {
    const int64_t n = static_cast<int64_t>(width) * height;
    if (n == 0) return cudaSuccess;
    dense_level_kernel<<<static_cast<unsigned>((n + kImgPix - 1) / kImgPix), kImgPix, 0, st>>>(
        zbin, width, height, nbr, reinterpret_cast<int4*>(coords));
    return cudaGetLastError();
}

cudaError_t launch_refiner_input(const float* fc, int64_t n, float* feat, cudaStream_t st) {
    if (n == 0) return cudaSuccess;
    refiner_input_kernel<<<grid_for(3 * n), 256, 0, st>>>(fc, n, feat);
    return cudaGetLastError();
}

cudaError_t launch_small_linear(const float* x1, int c1, const float* x2, int c2, int64_t rows, const void* w,
                                int wtype, int cout, const float* bias, float* y, cudaStream_t st) {
    if (rows == 0) return cudaSuccess;
    if (wtype != 0 && wtype != 1) return cudaErrorInvalidValue;
    small_linear_kernel<<<grid_for(rows * cout), 256, 0, st>>>(x1, c1, x2, c2, rows, w, wtype, cout, bias, y);
    return cudaGetLastError();
}

cudaError_t launch_silu_inplace(float* x, int64_t n, cudaStream_t st) {
    if (n == 0) return cudaSuccess;
    silu_inplace_kernel<<<grid_for(n), 256, 0, st>>>(x, n);
    return cudaGetLastError();
}

cudaError_t launch_encoder_rows(const int32_t* deep_coords, int64_t n, const float* enc, int ew, int eh, int cenc,
                                float* out, uint32_t* status, cudaStream_t st) {
    if (n == 0) return cudaSuccess;
    encoder_rows_kernel<<<grid_for(n * cenc), 256, 0, st>>>(reinterpret_cast<const int4*>(deep_coords), n, enc, ew,
                                                            eh, cenc, out, status);
    return cudaGetLastError();
}

cudaError_t launch_logz_update(float* fc, const float* res, int64_t n, cudaStream_t st) {
    if (n == 0) return cudaSuccess;
    logz_update_kernel<<<grid_for(n), 256, 0, st>>>(fc, res, n);
    return cudaGetLastError();
}

cudaError_t launch_keys_differ(const int32_t* a, const int32_t* b, int64_t n, int* differ, cudaStream_t st) {
    cudaError_t e = cudaMemsetAsync(differ, 0, sizeof(int), st);
    if (e != cudaSuccess || n == 0) return e;
    keys_differ_kernel<<<grid_for(n), 256, 0, st>>>(a, b, n, differ);
    return cudaGetLastError();
}

}  // namespace msc
