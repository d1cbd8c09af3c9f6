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
// of the fp32 value (2 planes), Q8_0 quantisation (1 plane of the int8 codes
// as fp16, or ACT_Q8I as int8, + one fp32 scale per 32 channels).
enum ActMode : int { ACT_FP16 = 0, ACT_SPLIT = 1, ACT_Q8 = 2, ACT_Q8I = 3 };

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

// Prepared weight layouts: f16 -> one exact fp16 plane; f32 and Q8_0 with
// cin != 128 -> exact hi/lo fp16 pair of the prescaled dequantised value;
// Q8_0 with cin == 128 -> int8 code tiles followed by the fp32 block scales
// [ntaps][cin/32][cout] (the kind::i8 path).
bool weight_is_i8(int wtype, int cin);
int weight_planes(int wtype, int cin);
size_t weight_blob_bytes(int wtype, int cin, int cout, int ntaps);
cudaError_t launch_weight_prepare(int wtype, const void* w, int cin, int cout, int ntaps, void* blob, cudaStream_t st);

int act_planes(int mode);
// Bytes of the prepared activation operand for n rows of c channels.
size_t act_bytes(int mode, int64_t n, int c);
// Q8 modes: the per-block scales follow the code plane at this byte offset.
size_t act_scale_offset(int mode, int64_t n, int c);
// x: [n][c] (dtype) -> prepared operand (planes [act_planes][n][c] fp16, plus
// scales in Q8 mode).  Optional normalisation before preparation: LayerNorm
// (ln), or, when gn is given, 32-group GroupNorm with gn[sample*32 + group] =
// {mean, 1/sqrt(var + eps)} and the sample of row i in coords[i][3]
// (clamped to [0, nsamples)); both
// with the affine gamma/beta (either may be null).  Then optional SiLU.
cudaError_t launch_act_prepare(const void* x, int x_dtype, int64_t n, int c, int ln, const float* gamma,
                               const float* beta, float eps, int silu, int mode, void* planes, cudaStream_t st,
                               const float2* gn = nullptr, const int32_t* coords = nullptr, int nsamples = 0);

struct ConvArgs {
    const void* planes;      // [na][n_in][cin] fp16 operand planes (Q8: the int8 codes as fp16)
    const float* a_scale;    // Q8: [n_in][cin/32] per-block activation scales, else null
    int na;                  // 1 or 2
    int q8;                  // ggml Q8_0 x Q8_0 block arithmetic
    int i8;                  // Q8 with int8 code planes (kind::i8 MMA; cin 128)
    int64_t n_in;            // rows of the input planes (neighbour indices >= n_in are missing)
    int64_t n;               // output rows processed
    int64_t row_begin;       // output row k is row_begin + k (when perm is null)
    const int32_t* perm;     // [n] output rows to process, or null
    // With a tap-order plan: the tile rows (-1 past n), their neighbour
    // lists (-1 = missing) and each tile's tap mask (plan.h PlanTiles); the
    // conv then stages each tile with bulk copies.  Null otherwise.
    const int32_t* tile_rows;
    const int32_t* tile_nbr;
    const uint32_t* tile_mask;
    const int32_t* tile_sched;  // plan: tiles by descending cost, dealt to the CTAs in a snake (NULL: round-robin)
    int cin;
    const int32_t* nbr;      // [rows][27] indexed by output row; null => linear (row i reads row i)
    const void* blob;        // prepared weights
    int wplanes;             // planes in blob (1 or 2)
    int cout;
    int ntaps;               // 27 or 1
    const float* bias;       // [cout] or null
    int silu_out;
    const void* residual;    // [rows][cout] or null
    int res_dtype;
    void* y;                 // [rows][cout]
    int y_dtype;
    // When set (cout = 128), the output is re-quantised for the next Q8_0
    // conv instead of stored in y: int8 codes [rows][cout] and fp32(fp16(d))
    // block scales [rows][cout/32] of ggml's x86 quantiser (the ACT_Q8I
    // operand).
    int8_t* q_codes;
    float* q_scales;
    uint32_t* status;
    // z-slab halo forwarding (multi-GPU), fp16 output with fp16 residual
    // only: with store_limit > 0, output rows r < store_limit are stored
    // locally; rows r < send_lo are also stored into the lower neighbour's
    // feature buffer peer_lo at row peer_lo_off + r, rows send_hi_begin <= r
    // < store_limit into the upper neighbour's peer_hi at row peer_hi_off +
    // (r - send_hi_begin).  The peer buffers are the neighbours' device memory
    // (CUDA IPC), written over NVLink.
    int64_t store_limit;
    void* peer_lo;
    int64_t peer_lo_off;
    int64_t send_lo;
    void* peer_hi;
    int64_t peer_hi_off;
    int64_t send_hi_begin;
};
cudaError_t launch_conv(const ConvArgs& a, cudaStream_t st);

bool conv_supported(int cin, int cout);

}  // namespace msc
