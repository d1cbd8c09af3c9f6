// Host launchers for the sparse-conv / linear tensor-core kernels (conv_tc.cu)
// and the activation / weight preparation kernels (prep.cu).
#pragma once

#include <cstddef>
#include <cstdint>
#include <cuda_runtime.h>

namespace msc {

// dtype codes (shared with the C ABI)
enum DType : int { DT_F32 = 0, DT_F16 = 1, DT_BF16 = 2 };
// weight type codes (ggml order)
enum WType : int { WT_F32 = 0, WT_F16 = 1, WT_Q8_0 = 8 };
// activation preparation modes: fp16 rounding (1 plane), exact hi/lo split
// of the fp32 value (2 planes), Q8_0 quantise then exact split (2 planes).
enum ActMode : int { ACT_FP16 = 0, ACT_SPLIT = 1, ACT_Q8 = 2 };

// Prepared-weight blob header (first 256 bytes of the blob).
struct WeightHeader {
    uint32_t magic;
    int32_t wtype;
    int32_t cin;
    int32_t cout;
    int32_t ntaps;
    int32_t planes;
    float oscale;     // multiply accumulators by this (power of two)
    float amax;       // max |dequantised weight|
    uint32_t reserved[56];
};
static_assert(sizeof(WeightHeader) == 256, "header is 256 bytes");
constexpr uint32_t kWeightMagic = 0x4d534357u;  // "WCSM"

int weight_planes(int wtype);
size_t weight_blob_bytes(int wtype, int cin, int cout, int ntaps);
cudaError_t launch_weight_prepare(int wtype, const void* w, int cin, int cout, int ntaps, void* blob, cudaStream_t st);

int act_planes(int mode);
// x: [n][c] (dtype); planes: [act_planes][n][c] fp16.  Optional LayerNorm
// (gamma/beta may be null only if ln == 0) and SiLU before preparation.
cudaError_t launch_act_prepare(const void* x, int x_dtype, int64_t n, int c, int ln, const float* gamma,
                               const float* beta, float eps, int silu, int mode, void* planes, cudaStream_t st);

struct ConvArgs {
    const void* planes;      // [na][n][cin] fp16
    int na;                  // 1 or 2
    int64_t n;               // rows (voxels) of input and output
    int cin;
    const int32_t* nbr;      // [n][27]; null => linear (row i reads row i)
    const void* blob;        // prepared weights
    int wplanes;             // planes in blob (1 or 2)
    int cout;
    int ntaps;               // 27 or 1
    const float* bias;       // [cout] or null
    int silu_out;
    const void* residual;    // [n][cout] or null
    int res_dtype;
    void* y;                 // [n][cout]
    int y_dtype;
    uint32_t* status;
};
cudaError_t launch_conv(const ConvArgs& a, cudaStream_t st);
bool conv_supported(int cin, int cout);

}  // namespace msc
