/* CPU oracle for the sparse-voxel hot path: a plain-C restatement of the
 * reference algorithms (mogecpp src/sparse.cpp + the ggml 0.25.3 CPU
 * arithmetic those graphs execute).
 *
 * TEST INFRASTRUCTURE ONLY.  Tests, the smoke check and the CPU-baseline leg
 * of the benchmark use this as the checker; no product code links it.
 *
 * Coordinates are int32 rows (x, y, z, b); voxel index = row position.
 * Features are row-major [n][c] (ggml's [C, N] with ne0 = C fastest).
 * Packed conv weights are row-major [cout][27*cin] (ggml ne0 = 27*cin), cin
 * fastest within a tap, taps in neighbour-map order.
 */
#ifndef MOGE_ORACLE_H
#define MOGE_ORACLE_H

#include <stdint.h>

#ifdef __cplusplus
extern "C" {
#endif

/* weight type codes (match the C ABI) */
#define ORC_W_F32 0
#define ORC_W_F16 1
#define ORC_W_Q8_0 8

typedef struct {
    uint16_t d;      /* fp16 scale */
    int8_t qs[32];
} orc_block_q8_0;

uint16_t orc_fp32_to_fp16(float f);
float orc_fp16_to_fp32(uint16_t h);
uint16_t orc_fp32_to_bf16(float f);
float orc_bf16_to_fp32(uint16_t h);

/* ggml quantize_row_q8_0_ref (weights; round half away from zero). */
void orc_quantize_q8_0_ref(const float *x, orc_block_q8_0 *y, int64_t k);
/* ggml x86 quantize_row_q8_0 (activations; id = 127/amax, round half even). */
void orc_quantize_q8_0_act(const float *x, orc_block_q8_0 *y, int64_t k);

/* Returns 0, or -1 on invalid input (negative / out-of-range coordinate). */
int orc_make_level(const int32_t *coords, int32_t n, int32_t *nbr);
/* Stride-2 transition.  parent: [n][4] capacity; pool_rows: [8][n] capacity
 * (slot-major, stride *np_out); inv_count: [n]; up_rows: [n].
 * Returns 0, -1 on invalid input, -2 on pool occupancy > 8. */
int orc_downsample(const int32_t *coords, int32_t n, int32_t *parent, int32_t *np_out, int32_t *pool_rows,
                   float *inv_count, int32_t *up_rows);

/* y[n][cout] = sum_t W_t x[nbr[n][t]] + bias, ggml mul_mat semantics for wtype:
 *   F32: fp32 products, F16: activations rounded to fp16, Q8_0: activations
 *   quantised per 32-block, w = orc_block_q8_0 rows. */
void orc_sparse_conv(const float *x, int64_t n, int cin, const int32_t *nbr, int wtype, const void *w, int cout,
                     const float *bias, float *y);
/* Conv from n_in input rows to n_out output rows over nbr [n_out][27] (first
 * ntaps columns), W [cout][ntaps*cin]: the octant-weighted stride-2 conv and
 * its transpose (no counterpart in the reference). */
void orc_conv_rect(const float *x, int64_t n_in, int cin, const int32_t *nbr, int64_t n_out, int ntaps, int wtype,
                   const void *w, int cout, const float *bias, float *y);
/* Octant maps of a stride-2 transition: down [np][27], up [nfine][27]. */
void orc_octant_maps(const int32_t *coords, int64_t nfine, const int32_t *pool_rows, const int32_t *up_rows,
                     int64_t np, int32_t *down, int32_t *up);
/* y[n][cout] = W x + bias with W [cout][cin] (ggml linear). */
void orc_linear(const float *x, int64_t n, int cin, int wtype, const void *w, int cout, const float *bias, float *y);
void orc_layer_norm(const float *x, int64_t n, int c, const float *gamma, const float *beta, float eps, float *y);
void orc_silu(float *x, int64_t n);
/* LN -> SiLU -> conv1 -> SiLU -> conv2 -> +x; weights as in orc_sparse_conv. */
void orc_res_block(const float *x, int64_t n, int c, const int32_t *nbr, int wtype, const float *norm_w,
                   const float *norm_b, const void *w1, const float *b1, const void *w2, const float *b2, float *y);
/* Sample-wide GroupNorm, restating ggml group_norm_f32
 * (ggml-cpu/ops.cpp:4208-4283) on the [C, N] features viewed as [N, 1, C]
 * per sample: per (sample, group of c/groups channels) the mean of all the
 * sample's voxels' group values (double sum), then the variance of the
 * float differences (double sum of float squares), y = (x - mean) *
 * (1 / sqrtf(var + eps)), then the per-channel affine y * gamma + beta
 * (ggml_mul, ggml_add; either may be NULL).  sample: [n] sample index of
 * each voxel, 0 <= sample < nsamples.  No counterpart in mogecpp's
 * refiner (its blocks use LayerNorm). */
void orc_group_norm(const float *x, int64_t n, int c, const int32_t *sample, int nsamples, int groups, float eps,
                    const float *gamma, const float *beta, float *y);
/* conv1 -> GroupNorm -> SiLU -> conv2 -> +x (the GroupNorm block variant). */
void orc_res_block_gn(const float *x, int64_t n, int c, const int32_t *nbr, const int32_t *sample, int nsamples,
                      int groups, float eps, int wtype, const float *gn_w, const float *gn_b, const void *w1,
                      const float *b1, const void *w2, const float *b2, float *y);
/* mean over children (slot-major pool_rows, sentinel nfine) then linear. */
void orc_pool_down(const float *x, int64_t nfine, int c, const int32_t *pool_rows, const float *inv_count, int64_t np,
                   int slots, int wtype, const void *w, int cout, const float *bias, float *y);
/* linear then gather up_rows. */
void orc_nearest_up(const float *x, int64_t np, int c, const int32_t *up_rows, int64_t nfine, int wtype, const void *w,
                    int cout, const float *bias, float *y);

/* Log-depth bins of an image (factor_coord [n][3]); 0, or -1 when the bin
 * extent exceeds INT32_MAX. */
int orc_quantize_topology_z(const float *coord, int64_t n, float depth_resolution, int32_t *zbin);
/* Level-0 neighbour map [width*height][27] from the pixel grid. */
void orc_dense_image_level(const int32_t *zbin, int32_t width, int32_t height, int32_t *nbr);

#ifdef __cplusplus
}
#endif
#endif
