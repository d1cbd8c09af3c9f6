/* moge_sparse_cuda.h - C ABI of the B200 (sm_100a) sparse-voxel path.
 *
 * Drop-in device executor for the sparse refiner of mogecpp (moge-ggml
 * 0.4.2).  Every entry point returns 0 on success or a negative MSC_E_* code
 * and leaves a message in the calling thread's msc_last_error(), the same
 * contract as the reference's C API guard (src/moge_c.cpp:20, :65-75) and
 * moge_last_error() (include/moge_ggml/moge_c.h:80).  No C++ exception
 * crosses this boundary.
 *
 * Memory: all tensors are caller-owned device pointers (the reference keeps
 * them in ggml backend buffers, src/sparse.cpp:541-558); scratch is passed in
 * as a caller-owned workspace whose size the *_workspace_bytes queries give.
 * Streams are cudaStream_t passed as void* (NULL = legacy default stream).
 * Calls are asynchronous on the stream except where noted ("syncs").
 *
 * Layouts (identical to the reference's):
 *   coords     int32 [n][4] rows (x, y, z, b), 16-byte aligned; x = image
 *              row, y = image column, z = depth bin (Coord3,
 *              src/sparse.cpp:69-74) plus the sample index b (the reference
 *              has no batch field; b keeps samples apart).  0 <= x,y,z < 2^19,
 *              0 <= b < 127.  Voxel index = row position.
 *   features   [n][c] row-major (ggml [C, N], ne0 = C), dtype MSC_F32/F16/BF16.
 *   nbr        int32 [n][27], tap v = (dx+1)*9 + (dy+1)*3 + (dz+1), missing = n
 *              (SparseLevel::neighbors, src/sparse.cpp:132-137).
 *   pool_rows  int32 [8][np] slot-major, missing = nfine; inv_count f32 [np];
 *              up_rows int32 [nfine] (Transition, src/sparse.cpp:139-147).
 *   weights    packed [cout][27*cin] (cin fastest; "*.weight.mogg_sparse27",
 *              tools/convert_moge.py:339-349) or linear [cout][cin], as
 *              MSC_W_F32 floats, MSC_W_F16 halves or MSC_W_Q8_0 ggml
 *              block_q8_0 rows {fp16 d; int8 qs[32]}.
 */
#ifndef MOGE_SPARSE_CUDA_H
#define MOGE_SPARSE_CUDA_H

#include <stddef.h>
#include <stdint.h>

#ifdef __cplusplus
extern "C" {
#endif

#define MSC_ABI_VERSION 1

/* error codes */
#define MSC_OK 0
#define MSC_E_INVALID (-1)     /* bad argument, shape or alignment */
#define MSC_E_UNSUPPORTED (-2) /* shape/dtype combination not built */
#define MSC_E_CUDA (-3)        /* CUDA runtime error */
#define MSC_E_DEVICE (-4)      /* device-side failure (bad coordinate, hash full, timeout, ...) */
#define MSC_E_WORKSPACE (-5)   /* workspace too small */

/* feature dtypes */
#define MSC_F32 0
#define MSC_F16 1
#define MSC_BF16 2

/* weight types (ggml_type values) */
#define MSC_W_F32 0
#define MSC_W_F16 1
#define MSC_W_Q8_0 8

/* device status bits (msc_check) */
#define MSC_DEV_TIMEOUT 0x1u
#define MSC_DEV_HASH_FULL 0x2u
#define MSC_DEV_BAD_COORD 0x4u
#define MSC_DEV_DUP_COORD 0x8u
#define MSC_DEV_POOL_OVERFLOW 0x10u
#define MSC_DEV_BAD_INDEX 0x20u
#define MSC_DEV_PLAN_OVERFLOW 0x40u

typedef struct msc_context* msc_ctx_t;

/* Library ABI version (MSC_ABI_VERSION). */
int msc_abi_version(void);

/* Thread-local message of the last failed call on this thread.
 * Replaces: moge_last_error (include/moge_ggml/moge_c.h:80). */
const char* msc_last_error(void);

/* Creates an executor bound to a CUDA device (allocates its 4-byte device
 * status word).  Mirrors SparseMetalExecutor::create (src/sparse_metal.hpp:21-30):
 * fails with MSC_E_UNSUPPORTED when the device is not sm_100. */
int msc_create(int device, msc_ctx_t* out);
int msc_destroy(msc_ctx_t ctx);

/* Syncs the stream, reads and clears the device status word; returns
 * MSC_E_DEVICE if any failure bit was set (bits in *bits when non-NULL).
 * MSC_DEV_DUP_COORD alone is informational (duplicates resolve to the first
 * index, as FlatCoordMap::emplace does) and does not fail.  Syncs. */
int msc_check(msc_ctx_t ctx, void* stream, uint32_t* bits);

/* ---------------------------------------------------------------- topology */

/* Workspace bytes for msc_make_level / msc_downsample over n voxels. */
size_t msc_topology_workspace_bytes(int64_t n);

/* Submanifold neighbour map.
 * Replaces: make_level (src/sparse.cpp:238-272). */
int msc_make_level(msc_ctx_t ctx, const int32_t* coords, int64_t n, int32_t* nbr, void* ws, size_t ws_bytes,
                   void* stream);

/* Neighbour map that allocates nothing, for callers that cannot allocate
 * device memory (a host runtime whose device memory belongs to another
 * allocator and offers no scratch, or latency-critical code that must not
 * call cudaMalloc because it can synchronise the device).  Same result as
 * msc_make_level; the hash table lives in a 16 MiB array compiled into the
 * library (held by every GPU that loads it until the process exits), so
 * n <= 524288 voxels; larger n fails with MSC_E_INVALID.  No context:
 * device-side failure bits go to *status (a caller-owned device word, may be
 * NULL).  The first call on a device looks up the array's device address
 * with that device current; make it before any stream capture.  The address
 * is cached per device for the life of the process: after a device reset
 * (cudaDeviceReset, which destroys the primary context and the array with
 * it) the cached address is stale and this entry point must not be called
 * again in that process.  All calls share the array: calls that overlap on
 * the GPU race and must be serialised.
 * No counterpart in the reference. */
int msc_make_level_noalloc(const int32_t* coords, int64_t n, int32_t* nbr, uint32_t* status, void* stream);

/* Stride-2 transition: parent coords [np][4] (capacity n rows), np (device
 * int32), pool_rows (capacity 8*n, written [8][np]), inv_count, up_rows.
 * If np_host is non-NULL the call syncs and stores np there; device failures
 * (duplicate coordinates, which the reference's serial slot numbering does
 * not define on the GPU) are then reported by the return code.
 * Replaces: downsample (src/sparse.cpp:312-357) with factor 2. */
int msc_downsample(msc_ctx_t ctx, const int32_t* coords, int64_t n, int32_t* parent, int32_t* np_dev,
                   int32_t* pool_rows, float* inv_count, int32_t* up_rows, int64_t* np_host, void* ws,
                   size_t ws_bytes, void* stream);

/* msc_make_level and msc_downsample of the same voxels in one call (the
 * neighbour map and the stride-2 maps of one pyramid level): the voxel
 * table is built once instead of twice.  Same arguments and results as the
 * two calls; the workspace is msc_topology_workspace_bytes(n).
 * Replaces: make_level + downsample of one level (src/sparse.cpp:238-272,
 * 312-357) as build_topology_from_key (src/sparse.cpp:408-431) calls them. */
int msc_make_level_downsample(msc_ctx_t ctx, const int32_t* coords, int64_t n, int32_t* nbr, int32_t* parent,
                              int32_t* np_dev, int32_t* pool_rows, float* inv_count, int32_t* up_rows,
                              int64_t* np_host, void* ws, size_t ws_bytes, void* stream);

/* Log-depth voxel bins of an image: for every pixel i (factor_coord [n][3]
 * floats: x/z, y/z, log z), q = nearbyint(double(log z * depth_resolution))
 * (float product, round half to even), zbin[i] = q - min(q).  Syncs; fails
 * with MSC_E_DEVICE on a non-finite z or a bin extent beyond 2^19 - 1 (the
 * voxel keys hold 19 bits per axis).
 * Replaces: quantize_topology_z (src/sparse.cpp:363-406). */
int msc_quantize_topology_z(msc_ctx_t ctx, const float* factor_coord, int64_t n, float depth_resolution,
                            int32_t* zbin, void* stream);

/* Level-0 topology of an image (one voxel per pixel): coords [n][4] =
 * (row, column, zbin, 0) for pixel i = row * width + column, and the
 * neighbour map nbr [n][27] from the pixel grid (a neighbour pixel is at tap
 * (drow+1)*9 + (dcol+1)*3 + (dz+1) when its bin differs by at most 1).
 * Replaces: make_dense_image_level (src/sparse.cpp:274-310) with the level-0
 * coordinates of build_topology_from_key (src/sparse.cpp:408-431). */
int msc_make_dense_image_level(msc_ctx_t ctx, const int32_t* zbin, int width, int height, int32_t* coords,
                               int32_t* nbr, void* stream);

/* ----------------------------------------------------------------- refiner
 * The whole sparse refiner pass on the device.  Mirrors SparseRefiner
 * (src/sparse.hpp:21-66): the configuration is SparseConfig (read from the
 * MOGG image's refiner.* metadata, read_sparse_config src/sparse.cpp:985-1007)
 * and refine_once (src/sparse.cpp:1014-1296) updates log z in place.
 * Topology is cached across calls as get_topology_cached
 * (src/sparse.cpp:443-472) does: a pass whose quantised bins equal the
 * previous pass's reuses its levels, neighbour maps and stride-2 maps.
 * Supported: model channels 64 or 128, downsample factors 2, F32 / F16 /
 * Q8_0 weights, identity residual skips (others fail with
 * MSC_E_UNSUPPORTED).  The feature state is fp32 on every level. */
#define MSC_REFINER_MAX_LEVELS 8
typedef struct {
    int in_channels;
    int out_channels;
    int encoder_channels;
    int num_levels;
    int model_channels[MSC_REFINER_MAX_LEVELS];
    int encoder_blocks[MSC_REFINER_MAX_LEVELS];
    int decoder_blocks[MSC_REFINER_MAX_LEVELS];     /* num_levels - 1 used */
    int downsample_factors[MSC_REFINER_MAX_LEVELS]; /* num_levels - 1 used */
    int bottleneck_blocks;
    int encoder_downsample;
    float depth_resolution;
} msc_sparse_config;

typedef struct msc_refiner* msc_refiner_t;

/* Loads the refiner.* tensors of a MOGG v1 image held in host memory
 * (src/mogg.cpp:247-312; sparse conv weights "*.weight.mogg_sparse27") to the
 * context's device and prepares them for the tensor cores.  Syncs.
 * Replaces: SparseRefiner::SparseRefiner + WeightStore (src/sparse.cpp:1010,
 * src/dense.cpp:198-270). */
int msc_refiner_create(msc_ctx_t ctx, const void* mogg, size_t mogg_bytes, void* stream, msc_refiner_t* out);
int msc_refiner_destroy(msc_refiner_t r);
int msc_refiner_config(msc_refiner_t r, msc_sparse_config* out);
/* Topology cache hits and misses so far (the reference's
 * moge_sparse_topology_cache trace counters). */
int msc_refiner_cache_stats(msc_refiner_t r, uint64_t* hits, uint64_t* misses);
/* Voxels per level of the cached topology (count = 0 before the first pass). */
int msc_refiner_level_sizes(msc_refiner_t r, int64_t* sizes, int capacity, int* count);

/* One refine pass.  factor_coord: device [height * width][3] floats, log z
 * updated in place; encoder_feature: device [encoder_height *
 * encoder_width][encoder_channels] floats (the reference's [C, ew * eh]).
 * width = encoder_width * encoder_downsample, likewise height.  Syncs.
 * Replaces: SparseRefiner::refine_once (src/sparse.cpp:1014-1296). */
int msc_refiner_refine_once(msc_refiner_t r, float* factor_coord, int width, int height, const float* encoder_feature,
                            int encoder_width, int encoder_height, void* stream);
/* The same with host buffers (copied in and out inside the call), as the
 * reference's refine_once takes factor_coord as a host vector. */
int msc_refiner_refine_once_host(msc_refiner_t r, float* factor_coord, int width, int height,
                                 const float* encoder_feature, int encoder_width, int encoder_height, void* stream);

/* ----------------------------------------------------------------- weights */

/* Bytes of a prepared-weight blob (tensor-core layout). */
size_t msc_weight_blob_bytes(int wtype, int cin, int cout, int ntaps);

/* Converts packed weights (ntaps = 27 for sparse27 conv weights, 1 for a
 * linear [cout][cin]) into the blob consumed by the conv / linear calls.
 * Replaces: the WeightStore upload of "*.weight.mogg_sparse27" tensors
 * (src/dense.cpp:198-270). */
int msc_weight_prepare(msc_ctx_t ctx, int wtype, const void* w, int cin, int cout, int ntaps, void* blob,
                       size_t blob_bytes, void* stream);

/* ----------------------------------------------------------------- operators
 * Arithmetic follows ggml's mul_mat for the weight type: F32 weights use fp32
 * products, F16 weights round activations to fp16, Q8_0 weights quantise
 * activations to Q8_0 per 32 channels (ggml's x86 quantiser) and sum
 * fp16(d_a)*fp16(d_w)*int_dot per block.  Accumulation is fp32. */

/* Workspace bytes for msc_sparse_conv / msc_linear / msc_res_block /
 * msc_pool_down / msc_nearest_up on n rows of c channels. */
size_t msc_op_workspace_bytes(int64_t n, int c);

/* y = sparse_conv(x) + bias.  cin, cout in {64, 128}.
 * Replaces: sparse_conv (src/sparse.cpp:579-627). */
int msc_sparse_conv(msc_ctx_t ctx, const void* x, int x_dtype, int64_t n, int cin, const int32_t* nbr,
                    const void* blob, const float* bias, void* y, int y_dtype, void* ws, size_t ws_bytes,
                    void* stream);

/* ---------------------------------------------------------------- conv plan
 * A conv plan is a per-level reordering of the voxels for the sparse convs
 * on that level.  Build it once per level, after msc_make_level, and pass it
 * to every conv on the level.  No counterpart in the reference (its CPU
 * gather walks the neighbour map directly, src/sparse.cpp:579-627); results
 * match the unplanned calls within the features tolerance (the tap
 * summation order differs).  One kind:
 *   MSC_PLAN_TAP_ORDER  the voxels sorted by their 27-bit tap mask (rarest
 *                       taps first), so that each 128-row tile of the conv
 *                       runs over fewer taps, with each tile's rows,
 *                       neighbour lists and tap mask; any weight type. */
#define MSC_PLAN_TAP_ORDER 0

/* Bytes of the plan buffer (256-byte aligned) and of the build workspace. */
size_t msc_conv_plan_bytes(int64_t n);
size_t msc_conv_plan_workspace_bytes(int64_t n);

/* Builds a plan from a level's neighbour map (coords is not read and may be
 * NULL). */
int msc_conv_plan_build(msc_ctx_t ctx, const int32_t* coords, int64_t n, const int32_t* nbr, int kind, void* plan,
                        size_t plan_bytes, void* ws, size_t ws_bytes, void* stream);

/* msc_sparse_conv with an optional plan (NULL = msc_sparse_conv); nbr is
 * required either way. */
int msc_sparse_conv_planned(msc_ctx_t ctx, const void* x, int x_dtype, int64_t n, int cin, const int32_t* nbr,
                            const void* plan, const void* blob, const float* bias, void* y, int y_dtype, void* ws,
                            size_t ws_bytes, void* stream);

/* Prologue and epilogue of a fused sparse conv:
 *   y = [SiLU](W * gather([SiLU]([LayerNorm](x))) + bias) [+ residual]
 * The prologue runs in the operand preparation of x, the epilogue in the
 * conv's tile epilogue (no extra passes over memory). */
typedef struct {
    int layer_norm;           /* 1: LayerNorm over each input row (ggml norm, eps), then the affine */
    const float* norm_w;      /* [cin] gamma (may be NULL) */
    const float* norm_b;      /* [cin] beta (may be NULL) */
    float eps;
    int silu_in;              /* 1: SiLU on the (normalised) input */
    int silu_out;             /* 1: SiLU on conv + bias */
    const void* residual;     /* [n][cout], added last (may be NULL) */
    int residual_dtype;
} msc_conv_fusion;

/* msc_sparse_conv_planned with a fused prologue / epilogue (fusion may be
 * NULL: none).  Workspace: msc_op_workspace_bytes(n, max(cin, cout)).
 * Replaces: the layer_norm -> silu -> sparse_conv -> silu / + skip chains of
 * res_block (src/sparse.cpp:629-642), one conv at a time. */
int msc_sparse_conv_fused(msc_ctx_t ctx, const void* x, int x_dtype, int64_t n, int cin, const int32_t* nbr,
                          const void* plan, const msc_conv_fusion* fusion, const void* blob, const float* bias,
                          void* y, int y_dtype, void* ws, size_t ws_bytes, void* stream);

/* msc_res_block with an optional plan, same rules as msc_sparse_conv_planned. */
int msc_res_block_planned(msc_ctx_t ctx, void* x, int x_dtype, int64_t n, int c, const int32_t* nbr,
                          const void* plan, const float* norm_w, const float* norm_b, const void* blob1,
                          const float* b1, const void* blob2, const float* b2, void* ws, size_t ws_bytes,
                          void* stream);

/* nblocks residual blocks in a row, in place on x: msc_res_block_planned
 * per block (one call for a level's block loop).  Per-block parameters are
 * arrays of nblocks pointers (norm_w, norm_b, b1, b2 may be NULL arrays).
 * Workspace: msc_op_workspace_bytes(n, c).
 * Replaces: the level's res_block loop (src/sparse.cpp:1118-1121,
 * :1140-1143, :1173-1176). */
int msc_res_stack(msc_ctx_t ctx, void* x, int x_dtype, int64_t n, int c, const int32_t* nbr, const void* plan,
                  int nblocks, const float* const* norm_w, const float* const* norm_b, const void* const* blob1,
                  const float* const* b1, const void* const* blob2, const float* const* b2, void* ws, size_t ws_bytes,
                  void* stream);

/* A level's LayerNorm residual stack from host tensors to host tensors:
 * copies coords [n][4] and x [n][c] (x_dtype) in, builds the neighbour map
 * and the tap-order plan, runs the nblocks blocks of msc_res_stack and
 * copies the result to y_host [n][c] (may be x_host).  Everything is
 * ordered on `stream` and the call returns without waiting; with
 * copy_in_stream / copy_out_stream (may be NULL) the copies run there,
 * ordered against the compute by events, so that consecutive calls on two
 * workspaces overlap one call's copies with another's compute.  The next
 * call on the same workspace waits for this call's result copy.  Host
 * buffers must stay valid until the result copy has completed
 * (page-locked buffers let the copies run asynchronously).
 * Workspace: msc_level_stack_host_workspace_bytes(n, c) device bytes.
 * Replaces: a level's upload, make_level, res_block loop and readback
 * (src/sparse.cpp:935-952, 238-272, 1118-1121, 1293-1295). */
size_t msc_level_stack_host_workspace_bytes(int64_t n, int c);
int msc_level_stack_host(msc_ctx_t ctx, const int32_t* coords_host, const void* x_host, int x_dtype, int64_t n,
                         int c, int nblocks, const float* const* norm_w, const float* const* norm_b,
                         const void* const* blob1, const float* const* b1, const void* const* blob2,
                         const float* const* b2, void* y_host, void* ws, size_t ws_bytes, void* stream,
                         void* copy_in_stream, void* copy_out_stream);

/* --------------------------------------------------- GroupNorm res block
 * The GroupNorm variant of the residual block, in place:
 *   x = x + conv2(SiLU(GroupNorm_32(conv1(x) + b1))) + b2
 * GroupNorm is sample-wide: for each sample (coords[i][3]) and each of 32
 * groups of c/32 channels, the mean and variance of the group's values over
 * the sample's voxels (double sums of x and x*x, var = E[x^2] - mean^2 in
 * double), y = (h - mean) * (1 / sqrtf(var + eps)), then * gn_w, then + gn_b
 * (either may be NULL).  Follows ggml's group_norm_f32
 * (ggml-cpu/ops.cpp:4208-4283, two passes) on the [C, N] features viewed as
 * [N, 1, C]; the reference's res_block (src/sparse.cpp:629-642) uses
 * LayerNorm instead and has no counterpart.
 *
 * Sharded runs: rows [0, n_stat) are this rank's own voxels and enter the
 * statistics; rows [n_stat, n) are halo rows, normalised with the same
 * statistics.  stats is a caller-owned device buffer of
 * msc_gn_stats_doubles(nsamples) doubles.  When allreduce is given it is
 * called once per block on the calling thread, in stream order, with the
 * whole statistics buffer (msc_gn_stats_doubles(nsamples) doubles at
 * stats: sums, counts, sums of squares) to sum over all ranks in place,
 * enqueued on `stream` (e.g. an NCCL all-reduce).  A non-zero return fails
 * the call.  With n = 0 the callback is still called (collectives stay
 * matched across ranks). */
typedef int (*msc_allreduce_fn)(double* buf, int64_t count, void* stream, void* user);

int64_t msc_gn_stats_doubles(int nsamples);
size_t msc_res_block_gn_workspace_bytes(int64_t n, int c, int nsamples);
int msc_res_block_gn(msc_ctx_t ctx, void* x, int x_dtype, int64_t n, int64_t n_stat, int c, const int32_t* coords,
                     int nsamples, const int32_t* nbr, const void* plan, const float* gn_w, const float* gn_b,
                     float eps, const void* blob1, const float* b1, const void* blob2, const float* b2,
                     double* stats, msc_allreduce_fn allreduce, void* allreduce_user, void* ws, size_t ws_bytes,
                     void* stream);

/* y = W x + bias per row.  Replaces: linear (src/sparse.cpp:515-518). */
int msc_linear(msc_ctx_t ctx, const void* x, int x_dtype, int64_t n, int cin, const void* blob, const float* bias,
               void* y, int y_dtype, void* ws, size_t ws_bytes, void* stream);

/* In place: x = x + conv2(SiLU(conv1(SiLU(LayerNorm(x))))), LayerNorm eps 1e-6
 * with affine norm_w / norm_b (either may be NULL).
 * Replaces: res_block (src/sparse.cpp:629-642) with an identity skip. */
int msc_res_block(msc_ctx_t ctx, void* x, int x_dtype, int64_t n, int c, const int32_t* nbr, const float* norm_w,
                  const float* norm_b, const void* blob1, const float* b1, const void* blob2, const float* b2,
                  void* ws, size_t ws_bytes, void* stream);

/* y [np][cout] = Linear(mean of children).  Replaces: pool_down
 * (src/sparse.cpp:646-668) with factor 2 (8 slots). */
int msc_pool_down(msc_ctx_t ctx, const void* x, int x_dtype, int64_t nfine, int c, const int32_t* pool_rows,
                  const float* inv_count, int64_t np, const void* blob, const float* bias, void* y, int y_dtype,
                  void* ws, size_t ws_bytes, void* stream);

/* y [nfine][cout] = Linear(x)[up_rows] (+ skip [nfine][cout] when non-NULL).
 * Replaces: nearest_up (src/sparse.cpp:670-674) and the decoder's skip add
 * (src/sparse.cpp:1160-1191). */
int msc_nearest_up(msc_ctx_t ctx, const void* x, int x_dtype, int64_t np, int c, const int32_t* up_rows,
                   int64_t nfine, const void* blob, const float* bias, const void* skip, int skip_dtype, void* y,
                   int y_dtype, void* ws, size_t ws_bytes, void* stream);

/* ------------------------------------------------- octant stride-2 conv
 * An extension with no counterpart in the reference, whose stride-2
 * operators are pool_down (mean over the children + linear,
 * src/sparse.cpp:646-668) and nearest_up (linear + parent gather, :670-674):
 * the octant-weighted stride-2 conv (each parent sums W_o x[child at octant
 * o] over its 2 x 2 x 2 cell) and its transpose (each child takes W_o
 * x[parent], o its own octant).  The octant of fine voxel (x, y, z) is
 * (x & 1) * 4 + (y & 1) * 2 + (z & 1); weights are packed [cout][8 * cin]
 * (cin fastest), prepared with ntaps = 8.
 *
 * Octant maps of a transition from msc_downsample (pool_rows [8][np],
 * up_rows [nfine]; np on the host): down_nbr [np][27] (column o = the child
 * at octant o, else nfine; columns 8-26 nfine) and up_nbr [nfine][27]
 * (column oct(c) = c's parent, every other column np). */
int msc_octant_maps(msc_ctx_t ctx, const int32_t* coords, int64_t nfine, const int32_t* pool_rows,
                    const int32_t* up_rows, int64_t np, int32_t* down_nbr, int32_t* up_nbr, void* stream);

/* Tap-order conv plan for a map whose neighbour lists index another level's
 * rows: n_out output rows, entries in [0, n_in) present.  Sizes as
 * msc_conv_plan_bytes(n_out) / msc_conv_plan_workspace_bytes(n_out). */
int msc_conv_plan_build_rect(msc_ctx_t ctx, int64_t n_out, int64_t n_in, const int32_t* nbr, void* plan,
                             size_t plan_bytes, void* ws, size_t ws_bytes, void* stream);

/* y [n_out][cout] = sum_{o < 8} W_o x[nbr[i][o]] + bias (+ skip [n_out][cout],
 * may be NULL) over x [n_in][cin]: the strided conv with nbr = down_nbr
 * (n_in = nfine, n_out = np), the transposed conv with nbr = up_nbr (n_in =
 * np, n_out = nfine; the skip is the decoder's additive skip).  plan: from
 * msc_conv_plan_build_rect over the same map, or NULL (strongly advised for
 * the transpose, whose rows each have one tap).  Workspace:
 * msc_op_workspace_bytes(n_in, cin). */
int msc_octant_conv(msc_ctx_t ctx, const void* x, int x_dtype, int64_t n_in, int cin, const int32_t* nbr,
                    int64_t n_out, const void* plan, const void* blob, const float* bias, const void* skip,
                    int skip_dtype, void* y, int y_dtype, void* ws, size_t ws_bytes, void* stream);

/* ------------------------------------------------------------ multi-GPU
 * A z-slab shard of a level for one GPU of a node (one process per GPU).
 * No counterpart in the reference (its refiner is single-device,
 * src/sparse.cpp:1100-1191); this is the sharded form of its per-level
 * res_block loop.  Rows are laid out [owned | halo below | halo above]: the
 * halos are the two z-planes on either side held by the neighbouring ranks;
 * the first send_lo owned rows are the lower neighbour's halo above and the
 * last send_hi owned rows the upper neighbour's halo below, in order.
 *
 * The exchange is fused into the conv: each block's second conv computes the
 * owned rows only and its epilogue also stores the boundary rows straight
 * into the neighbours' feature buffers (CUDA IPC memory over NVLink); a
 * one-thread kernel per block waits, for at most 2 s, until both neighbours
 * have finished the previous block (flags they set in this GPU's memory; a
 * neighbour that never arrives raises MSC_DEV_TIMEOUT, read by msc_check).
 * Two feature buffers alternate between blocks.
 *
 * Setup: msc_slab_create on every rank, msc_slab_get_handle, exchange the
 * handles with the host's communicator (e.g. an all-gather), then
 * msc_slab_connect with the lower and upper neighbours' handles (NULL at the
 * ends).  Every rank must run the same number of blocks; call
 * msc_slab_destroy only after all ranks are done (a barrier). */
typedef struct {
    int rank;
    int world;
    int channels;      /* 128 */
    int64_t n_local;   /* n_owned + n_halo_lo + n_halo_hi */
    int64_t n_owned;
    int64_t n_halo_lo;
    int64_t n_halo_hi;
    int64_t send_lo;
    int64_t send_hi;
} msc_slab_desc;

typedef struct {
    unsigned char bytes[512];
} msc_slab_handle;

typedef struct msc_slab* msc_slab_t;

int msc_slab_create(msc_ctx_t ctx, const msc_slab_desc* desc, msc_slab_t* out);
int msc_slab_destroy(msc_slab_t s);
int msc_slab_get_handle(msc_slab_t s, msc_slab_handle* out);
int msc_slab_connect(msc_slab_t s, const msc_slab_handle* lower, const msc_slab_handle* upper);
/* Topology of the local rows (coords [n_local][4], device): neighbour map
 * and the conv plans of all rows and of the owned rows. */
int msc_slab_set_level(msc_slab_t s, const int32_t* coords, void* stream);
/* Loads [n_local][channels] fp16 features (device) into the current buffer;
 * reads the owned rows [n_owned][channels] back (device or pinned host). */
int msc_slab_put_features(msc_slab_t s, const void* x, void* stream);
int msc_slab_get_features(msc_slab_t s, void* owned_out, void* stream);
int msc_slab_features_ptr(msc_slab_t s, void** x);
/* One LayerNorm residual block (as msc_res_block, Q8_0 weights, C = 128)
 * over the shard, halo rows refreshed through the neighbours' conv2. */
int msc_slab_res_block(msc_slab_t s, const float* norm_w, const float* norm_b, const void* blob1, const float* b1,
                       const void* blob2, const float* b2, void* stream);

/* Failure-detection probe: runs the bounded cross-GPU wait of the slab path
 * on a flag that nothing sets, for budget_us microseconds (at most 2 s);
 * the wait gives up, sets MSC_DEV_TIMEOUT in the context's status word (read
 * and cleared by msc_check) and the context stays usable.  Lets a host test
 * its handling of a neighbour that never arrives without a second GPU. */
int msc_wait_probe(msc_ctx_t ctx, int64_t budget_us, void* stream);

/* ------------------------------------------------------------------ tracing */

typedef struct {
    char name[32];      /* kernel family: conv_tc, linear_tc, act_prepare, make_level, ... */
    int64_t launches;
    double total_ms;    /* summed CUDA-event durations on the launching stream */
} msc_profile_entry;

/* Enables / disables per-launch CUDA-event timing of this context's kernels.
 * Replaces: MOGE_OP_PROFILE's per-node eval callback (src/profiling.hpp:50-71). */
int msc_profile_enable(msc_ctx_t ctx, int enable);

/* Aggregates the recorded launches per kernel family into out[0..capacity)
 * and clears them; *count = number of families.  Syncs on the events. */
int msc_profile_read(msc_ctx_t ctx, msc_profile_entry* out, int capacity, int* count);

#ifdef __cplusplus
}
#endif

#endif /* MOGE_SPARSE_CUDA_H */
