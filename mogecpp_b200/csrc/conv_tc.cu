// Submanifold sparse 3-D convolution (and its 1-tap special case, the
// per-voxel linear layer) as a persistent implicit gather-GEMM on the sm_100a
// tensor cores.
//
// Reference semantics (mogecpp src/sparse.cpp:579-627 sparse_conv):
//   y[i, :] = sum_t W_t x[nbr[i][t], :] + bias,  nbr sentinel = zero row,
// with W packed [cout][27*cin] (cin fastest, taps in neighbour-map order).
//
// Tiles of 128 output voxels (M) x cout (N).  K runs over the taps present
// in the tile (taps with no valid neighbour in any of its rows are skipped)
// and 128-byte operand rows.  Operands sit in shared memory 128-byte
// swizzled, K-major.  Three arithmetic kinds:
//   * KIND_Q8I (ggml Q8_0 weights, cin = 128): A = the activation's int8
//     Q8_0 codes, B = the weight's int8 codes; one kind::i8 MMA per
//     32-channel block gives the exact int32 block dot product isum (two
//     blocks side by side in one accumulator slot, so that a slot's wait,
//     commit and release serve two blocks); the drain warps apply ggml's
//     per-block scale
//         acc += (d_a * d_w) * isum       (ggml-cpu x86 quants.c:1308)
//   * KIND_Q8F (ggml Q8_0 weights, cin = 64): A = the int8 codes as fp16,
//     B = the exact hi/lo fp16 pair of the prescaled weight d_w * q_w; one
//     MMA group per 32-channel block gives d_w * isum exactly (4-MMA chain),
//     the drain applies d_a.
//   * KIND_F (f32 / f16 weights): A and B are one fp16 plane or an exact
//     hi/lo pair (hi*hi + hi*lo + lo*hi); one MMA group per 64-channel chunk,
//     drained with an fp32 add.
// Draining every group keeps each tensor-core accumulation chain to a few
// MMAs: the tcgen05 fp32 accumulator does not round to nearest, and long
// chains drift by ~1e-6 relative, which ggml's activation re-quantisation
// would amplify.
//
// Persistent CTA, one per SM, 20 warps:
//   warps 0-1   producers: per tile, stage the rows' neighbour lists and the
//               tap mask; per stage, gather the 128 A rows with coalesced
//               16-byte cp.async (8 lanes per 128-byte row, swizzled straight
//               into the UMMA layout; sentinel rows zero-filled), completion
//               tracked by the stage's `gathered` barrier; thread 0
//               bulk-copies the stage's pre-swizzled B tile.  Q8I: the
//               gathered rows' activation block scales (16 bytes a row) are
//               copied into the stage too, so each scale is fetched from
//               global memory once per tile rather than by every drain warp.
//   warp 2      TMEM allocation and the single-thread MMA issue loop.
//   warps 3-18  drain + epilogue: TMEM lane quarter (warp % 4) x column quarter;
//               fp32 accumulators in registers, bias / SiLU / residual / store.
//               Q8I: a stage is released by the MMA's commit and by every drain
//               warp once it has read the stage's scales for the tap.
//   warp 19     publisher: once a stage's copies have landed, the proxy fence
//               and the stage's `full` arrival (a thread with no copies of its
//               own in flight, so the fence does not wait on them).
// Pipelines (mbarriers): smem stages gathered/full/empty, TMEM accumulator slots
// acc_full/acc_empty (NACC rotating slots), per-tile tile_ready/tile_free
// (double-buffered neighbour lists).  Taps are visited in ascending order in
// every tile (tiling-independent results); with a plan, each CTA takes its
// tiles from the plan's cost-sorted schedule in a snake order.  Every wait
// is bounded; a wait that runs out sets MSC_DEV_TIMEOUT and the CTA unwinds.
#include "common.cuh"
#include "conv.h"
#include "conv_common.cuh"

#include <mutex>

namespace msc {
namespace {

constexpr int BM = 128;
constexpr int kProducerWarps = 2;
constexpr int kDrainWarps = 16;
constexpr int kFenceWarp = kProducerWarps + 1 + kDrainWarps;  // last warp
constexpr int kThreads = 32 * (kProducerWarps + 2 + kDrainWarps);
constexpr int kProducers = 32 * kProducerWarps;
constexpr int kRowsPerProducer = BM / kProducers;
constexpr int kSmemLimit = 227 * 1024;  // max dynamic shared memory per block on sm_100
constexpr uint32_t kLazyWaitNs = 128;    // poll interval of the producers' and the publisher's waits

enum Kind : int { KIND_F = 0, KIND_Q8F = 1, KIND_Q8I = 2 };

template <int CIN, int COUT, int NA, int NB, int KIND>
struct Cfg {
    static constexpr int ELEM = KIND == KIND_Q8I ? 1 : 2;   // bytes per A/B element
    static constexpr int ROW_BYTES = CIN * ELEM;             // one activation row
    static constexpr int KCH = ROW_BYTES / 128;              // 128-byte chunks per tap
    static constexpr int NBLK = CIN / 32;                    // Q8_0 blocks per tap
    static constexpr int A_PLANE = BM * 128;
    static constexpr int B_PLANE = COUT * 128;
    static constexpr int STAGE = NA * A_PLANE + NB * B_PLANE;
    // accumulator groups per stage and MMA k-steps (32 bytes of K) per group
    // Q8I: BPG = 2 block sums side by side in one accumulator slot, so that a
    // slot's wait, commit and release are paid once per two blocks
    static constexpr int BPG = KIND == KIND_Q8I ? 2 : 1;
    static constexpr int GPS = KIND == KIND_Q8I ? 4 / BPG : (KIND == KIND_Q8F ? 2 : 1);
    static constexpr int KSPG = KIND == KIND_Q8I ? 1 : 4 / GPS;  // MMA k-steps per block (Q8I) or group
    static constexpr int SLOT = BPG * COUT;                        // TMEM columns per slot
    static constexpr int NACC = (512 / SLOT) < 4 ? (512 / SLOT) : 4;
    static constexpr int TMEM_COLS = NACC * SLOT;
    static constexpr int COLS = COUT / (kDrainWarps / 4);  // columns per drain thread
    static constexpr int NBR_BYTES = 2 * BM * 27 * 4;
    static constexpr int ROWS_BYTES = 2 * BM * 4;
    static constexpr int SB_BYTES = KIND == KIND_Q8I ? 27 * NBLK * COUT * 4 : 0;  // weight block scales
    // Q8I: the gathered rows' activation block scales ride with each stage
    // ([BM][NBLK] floats) and the drainers release the stage after reading them
    static constexpr bool STAGED_SCALES = KIND == KIND_Q8I;
    static constexpr int SC_STAGE = STAGED_SCALES ? BM * NBLK * 4 : 0;
    static constexpr int BAR_BYTES = 512;
    static constexpr int BIAS_BYTES = COUT * 4;
    static constexpr int FIXED = NBR_BYTES + ROWS_BYTES + SB_BYTES + BIAS_BYTES + BAR_BYTES;
    static constexpr int STAGES_FIT = (kSmemLimit - 1024 - FIXED) / (STAGE + SC_STAGE);
    static constexpr int STAGES = STAGES_FIT > 6 ? 6 : STAGES_FIT;
    static constexpr int SMEM = 1024 + STAGES * (STAGE + SC_STAGE) + FIXED;
    static_assert(STAGES >= 2, "at least two pipeline stages");
    static_assert(ROW_BYTES % 128 == 0, "activation rows must be whole 128-byte chunks");
    static_assert(COUT % 64 == 0 && COUT <= 256, "cout must be 64..256 in steps of 64");
    static_assert(TMEM_COLS <= 512 && (TMEM_COLS & (TMEM_COLS - 1)) == 0, "TMEM allocation");
    static_assert(KIND != KIND_Q8F || (NA == 1 && NB == 2), "Q8F: code plane x exact weight pair");
    static_assert(KIND != KIND_Q8I || (NA == 1 && NB == 1 && CIN == 128), "Q8I: int8 planes, cin 128");
    static_assert(SMEM <= kSmemLimit, "shared memory budget");
    static_assert(!STAGED_SCALES || (NBLK * 4 == 16 && KCH == 1), "staged scales: one 16-byte copy per row and tap");
};

struct Smem {
    uint8_t* stages;
    int* nbr;        // [2][BM*27], missing neighbour = -1
    int* rows;       // [2][BM]
    float* sB;       // [27][NBLK][COUT] weight block scales (Q8I)
    float* sA;       // [STAGES][BM][NBLK] gathered activation block scales (Q8I)
    float* bias;     // [COUT] output bias (zeros without one)
    uint64_t* full;
    uint64_t* empty;
    uint64_t* gathered;
    uint64_t* acc_full;
    uint64_t* acc_empty;
    uint64_t* tile_ready;  // [2]
    uint64_t* tile_free;   // [2]
    uint64_t* drained;     // MMA completion on the abort path (before TMEM release)
    uint32_t* wmask;       // [2][kProducerWarps]
    uint32_t* tmem;
    int* abort;
};

__device__ __forceinline__ uint32_t tile_mask(const Smem& S, int buf) {
    uint32_t m = 0;
#pragma unroll
    for (int w = 0; w < kProducerWarps; ++w) m |= S.wmask[buf * kProducerWarps + w];
    return m;
}

__device__ __forceinline__ int64_t tile_row(const ConvArgs& a, int64_t idx) {
    if (idx >= a.n) return -1;
    return a.perm ? static_cast<int64_t>(__ldg(a.perm + idx)) : a.row_begin + idx;
}

// The k-th tile of this CTA, or -1 past the end.  With a plan's schedule
// (tiles by descending cost) the tiles are dealt out in a snake,
// CTAs 0..G-1 then G-1..0 and so on, which evens out the CTAs' loads
// (round-robin over tiles in tap order left the busiest CTA 5 % above the
// mean at 3.1M voxels and 18 % at 400k); without one, round-robin.
__device__ __forceinline__ int64_t cta_tile(const ConvArgs& a, int64_t k, int64_t ntiles) {
    const int64_t g = gridDim.x;
    const int64_t idx = k * g + ((a.tile_sched && (k & 1)) ? g - 1 - blockIdx.x : blockIdx.x);
    if (idx >= ntiles) return -1;
    return a.tile_sched ? static_cast<int64_t>(__ldg(a.tile_sched + idx)) : idx;
}

// D[tmem] (+)= A * B^T, kind::i8 (signed int8 operands, int32 accumulator).
// ------------------------------------------------------------------ roles

template <int CIN, int COUT, int NA, int NB, int KIND>
__device__ void producer(const ConvArgs& a, const Smem& S, int64_t ntiles) {
    using C = Cfg<CIN, COUT, NA, NB, KIND>;
    const int t0 = threadIdx.x;  // 0..kProducers-1
    const int warp = t0 >> 5;
    const int lane = t0 & 31;
    const int chunk = lane & 7;            // 16-byte chunk of a 128-byte row
    const int rsub = lane >> 3;            // row within a group of 4
    constexpr int kRowsPerWarp = BM / kProducerWarps;
    constexpr int kCopies = kRowsPerWarp / 4;  // cp.async per lane per plane per stage
    const uint8_t* planes = static_cast<const uint8_t*>(a.planes);
    const uint8_t* wdata = static_cast<const uint8_t*>(a.blob) + sizeof(WeightHeader);
    const int64_t plane_bytes = a.n_in * C::ROW_BYTES;
    int64_t i = 0;  // stages issued
    bool ok = true;
    int k = 0;
    for (int64_t tile = cta_tile(a, 0, ntiles); tile >= 0 && ok; tile = cta_tile(a, ++k, ntiles)) {
        const int buf = k & 1;
        if (k >= 2 && !wait_or_abort(&S.tile_free[buf], ((k >> 1) - 1) & 1, S.abort, a.status, kLazyWaitNs)) {
            ok = false;
            break;
        }
        if (a.tile_nbr) {
            // a tap-order plan holds this tile's rows, neighbour lists and tap
            // mask: two bulk copies completing on tile_ready (no thread loads)
            if (t0 == 0) {
                S.wmask[buf * kProducerWarps] = __ldg(a.tile_mask + tile);
#pragma unroll
                for (int w = 1; w < kProducerWarps; ++w) S.wmask[buf * kProducerWarps + w] = 0u;
                mbar_arrive_expect_tx(&S.tile_ready[buf], BM * 27 * 4 + BM * 4);
                bulk_g2s(smem_u32(S.nbr + buf * BM * 27), a.tile_nbr + tile * BM * 27, BM * 27 * 4, &S.tile_ready[buf]);
                bulk_g2s(smem_u32(S.rows + buf * BM), a.tile_rows + tile * BM, BM * 4, &S.tile_ready[buf]);
            } else if ((t0 & 31) == 0) {
                mbar_arrive(&S.tile_ready[buf]);
            }
            if (!wait_or_abort(&S.tile_ready[buf], (k >> 1) & 1, S.abort, a.status)) {
                ok = false;
                break;
            }
        } else {
            // neighbour lists and tap mask of this thread's rows (t0, t0+64)
            uint32_t m = 0;
#pragma unroll
            for (int u = 0; u < kRowsPerProducer; ++u) {
                const int r = t0 + u * kProducers;
                const int64_t row = tile_row(a, tile * BM + r);
                int* nb = S.nbr + buf * BM * 27 + r * 27;
                if (row >= 0) {
                    if (a.nbr) {
                        const int* src = a.nbr + row * 27;
#pragma unroll 9
                        for (int t = 0; t < 27; ++t) {
                            const int j = __ldg(src + t);
                            const bool v = static_cast<uint64_t>(j) < static_cast<uint64_t>(a.n_in);
                            nb[t] = v ? j : -1;
                            if (v) m |= 1u << t;
                        }
                    } else {
                        nb[0] = static_cast<int>(row);
                        m = 1u;
                    }
                } else {
#pragma unroll 9
                    for (int t = 0; t < 27; ++t) nb[t] = -1;
                }
                S.rows[buf * BM + r] = static_cast<int>(row);
            }
            m = __reduce_or_sync(0xffffffffu, m);
            if (lane == 0) S.wmask[buf * kProducerWarps + warp] = m;
            asm volatile("bar.sync 1, %0;" ::"n"(kProducers) : "memory");
            warp_arrive(&S.tile_ready[buf]);
        }
        const int rot = tap_rotation(tile, a.ntaps);
        uint32_t rem = rot_mask(tile_mask(S, buf), rot);
        const int nst = __popc(rem) * C::KCH;
        int tap = -1, kc = C::KCH;
        const int* nbw = S.nbr + buf * BM * 27 + (warp * kRowsPerWarp + rsub) * 27;
        for (int st = 0; st < nst; ++st, ++i) {
            if (kc == C::KCH) {
                tap = rot_tap(__ffs(rem) - 1, rot);
                rem &= rem - 1;
                kc = 0;
            }
            const int s = static_cast<int>(i % C::STAGES);
            if (i >= C::STAGES &&
                !wait_or_abort(&S.empty[s], static_cast<uint32_t>((i / C::STAGES) - 1) & 1, S.abort, a.status,
                               kLazyWaitNs)) {
                ok = false;
                break;
            }
            uint8_t* sA = S.stages + s * C::STAGE;
            uint8_t* sB = sA + NA * C::A_PLANE;
            if (t0 == 0) {
                mbar_arrive_expect_tx(&S.full[s], NB * C::B_PLANE);
                bulk_g2s(smem_u32(sB), wdata + static_cast<int64_t>(tap * C::KCH + kc) * NB * C::B_PLANE,
                         NB * C::B_PLANE, &S.full[s]);
            }
            // coalesced gather: 8 lanes per 128-byte row, 4 rows per instruction
#pragma unroll
            for (int q = 0; q < kCopies; ++q) {
                const int r = warp * kRowsPerWarp + rsub + 4 * q;
                const int j = nbw[(4 * q) * 27 + tap];
                const uint32_t nbytes = j >= 0 ? 16u : 0u;
                const uint32_t dst = smem_u32(sA) + sw128_offset(r, chunk);
#pragma unroll
                for (int p = 0; p < NA; ++p) {
                    const uint8_t* src =
                        j >= 0 ? planes + p * plane_bytes + static_cast<int64_t>(j) * C::ROW_BYTES + kc * 128 + chunk * 16
                               : planes;
                    cp_async16(dst + p * C::A_PLANE, src, nbytes);
                }
            }
            if constexpr (C::STAGED_SCALES) {
                // the block scales of the rows gathered for this tap (zero
                // where the neighbour is missing or the row is padding)
#pragma unroll
                for (int r = t0; r < BM; r += kProducers) {
                    const int j = S.nbr[buf * BM * 27 + r * 27 + tap];
                    cp_async16(smem_u32(S.sA + (s * BM + r) * C::NBLK),
                               j >= 0 ? a.a_scale + static_cast<int64_t>(j) * C::NBLK : a.a_scale, j >= 0 ? 16u : 0u);
                }
            }
            cp_async_mbar_arrive_noinc(&S.gathered[s]);
            ++kc;
        }
    }
    cp_async_wait_all();
    if (!ok && t0 == 0) {
        // aborted: the weight-tile bulk copies this thread issued complete on
        // `full` barriers that may never finish their phase now; a bulk copy
        // of at most 32 KB lands within microseconds, so wait 100 us before
        // the CTA (and its shared memory) can go away
        const uint64_t t_end = global_timer_ns() + 100000ull;
        while (global_timer_ns() < t_end) __nanosleep(1000);
    }
}

// Publishes each stage to the MMA issuer once the producers' copies have
// landed: a proxy fence (generic-proxy cp.async writes -> async-proxy MMA
// reads) by a thread with no copies of its own in flight, so it never waits
// on them.
template <int CIN, int COUT, int NA, int NB, int KIND>
__device__ void publisher(const ConvArgs& a, const Smem& S, int64_t ntiles) {
    using C = Cfg<CIN, COUT, NA, NB, KIND>;
    int64_t i = 0;
    int k = 0;
    for (int64_t tile = cta_tile(a, 0, ntiles); tile >= 0; tile = cta_tile(a, ++k, ntiles)) {
        const int buf = k & 1;
        if (!wait_or_abort(&S.tile_ready[buf], (k >> 1) & 1, S.abort, a.status)) return;
        const int nst = __popc(tile_mask(S, buf)) * C::KCH;
        for (int st = 0; st < nst; ++st, ++i) {
            const int s = static_cast<int>(i % C::STAGES);
            if (!wait_or_abort(&S.gathered[s], static_cast<uint32_t>(i / C::STAGES) & 1, S.abort, a.status, kLazyWaitNs))
                return;
            fence_proxy_async();
            mbar_arrive(&S.full[s]);
        }
    }
}

template <int CIN, int COUT, int NA, int NB, int KIND>
__device__ void mma_issuer(const ConvArgs& a, const Smem& S, int64_t ntiles, uint32_t tmem) {
    using C = Cfg<CIN, COUT, NA, NB, KIND>;
    constexpr uint32_t idesc = KIND == KIND_Q8I ? idesc_i8(BM, COUT) : idesc_f16(BM, COUT, 0);
    int64_t i = 0, g = 0;
    int k = 0;
    for (int64_t tile = cta_tile(a, 0, ntiles); tile >= 0; tile = cta_tile(a, ++k, ntiles)) {
        const int buf = k & 1;
        if (!wait_or_abort(&S.tile_ready[buf], (k >> 1) & 1, S.abort, a.status)) return;
        const int nst = __popc(tile_mask(S, buf)) * C::KCH;
        for (int st = 0; st < nst; ++st, ++i) {
            const int s = static_cast<int>(i % C::STAGES);
            if (!wait_or_abort(&S.full[s], static_cast<uint32_t>(i / C::STAGES) & 1, S.abort, a.status)) return;
            tc_fence_after();
            const uint32_t aaddr = smem_u32(S.stages + s * C::STAGE);
            const uint32_t baddr = aaddr + NA * C::A_PLANE;
#pragma unroll
            for (int gg = 0; gg < C::GPS; ++gg, ++g) {
                const int slot = static_cast<int>(g % C::NACC);
                if (g >= C::NACC &&
                    !wait_or_abort(&S.acc_empty[slot], static_cast<uint32_t>((g / C::NACC) - 1) & 1, S.abort,
                                   a.status))
                    return;
                tc_fence_after();
                const uint32_t d = tmem + static_cast<uint32_t>(slot * C::SLOT);
                if (KIND == KIND_Q8I) {
                    // one k-step per block, each block into its own columns
#pragma unroll
                    for (int b = 0; b < C::BPG; ++b) {
                        const uint32_t off = static_cast<uint32_t>((gg * C::BPG + b) * 32);
                        umma_i8(d + static_cast<uint32_t>(b * COUT), sdesc_k_sw128(aaddr + off),
                                sdesc_k_sw128(baddr + off), idesc, 0u);
                    }
                }
#pragma unroll
                for (int ks = 0; ks < (KIND == KIND_Q8I ? 0 : C::KSPG); ++ks) {
                    const uint32_t off = static_cast<uint32_t>((gg * C::KSPG + ks) * 32);
                    const uint64_t ah = sdesc_k_sw128(aaddr + off);
                    const uint64_t bh = sdesc_k_sw128(baddr + off);
                    {
                        umma_f16(d, ah, bh, idesc, ks > 0 ? 1u : 0u);
                        if (NB == 2) umma_f16(d, ah, sdesc_k_sw128(baddr + C::B_PLANE + off), idesc, 1u);
                        if (NA == 2) umma_f16(d, sdesc_k_sw128(aaddr + C::A_PLANE + off), bh, idesc, 1u);
                    }
                }
                umma_commit(&S.acc_full[slot]);
            }
            umma_commit(&S.empty[s]);
        }
    }
}

// Magic-number conversion of an int32 in (-2^22, 2^22) to fp32: the integer
// added to the bits of 1.5*2^23 lands in the mantissa, so subtracting
// 1.5*2^23 afterwards is exact.
constexpr int kMagicBits = 0x4B400000;
constexpr float kMagic = 12582912.0f;

template <int CIN, int COUT, int NA, int NB, int KIND>
__device__ void drainer(const ConvArgs& a, const Smem& S, int64_t ntiles, uint32_t tmem) {
    using C = Cfg<CIN, COUT, NA, NB, KIND>;
    constexpr bool Q8 = KIND != KIND_F;
    constexpr int COLS = C::COLS;
    // TMEM columns per load: 16 for the int8 path keeps its drain in registers
    constexpr int CH = (COLS < 32 || KIND == KIND_Q8I) ? 16 : 32;
    const int warp = threadIdx.x >> 5;
    const int lane = threadIdx.x & 31;
    const int q = warp & 3;                              // TMEM lane quarter
    const int part = (warp - kProducerWarps - 1) >> 2;  // column slice
    const int m = q * 32 + lane;                         // tile row
    const int c_base = part * COLS;
    const uint32_t lane_addr = static_cast<uint32_t>(q * 32) << 16;
    const float oscale = static_cast<const WeightHeader*>(a.blob)->oscale;
    int64_t g = 0, i = 0;  // accumulator groups and pipeline stages seen
    int k = 0;
    for (int64_t tile = cta_tile(a, 0, ntiles); tile >= 0; tile = cta_tile(a, ++k, ntiles)) {
        const int buf = k & 1;
        if (!wait_or_abort(&S.tile_ready[buf], (k >> 1) & 1, S.abort, a.status)) return;
        const int rot = tap_rotation(tile, a.ntaps);
        uint32_t rem = rot_mask(tile_mask(S, buf), rot);
        const int row = S.rows[buf * BM + m];
        const int* nb = S.nbr + buf * BM * 27 + m * 27;
        if (a.residual && row >= 0) {
            const int es = a.res_dtype == DT_F32 ? 4 : 2;
            prefetch_l2(static_cast<const char*>(a.residual) + (static_cast<int64_t>(row) * COUT + c_base) * es);
        }
        uint64_t acc[COLS / 2];
#pragma unroll
        for (int e = 0; e < COLS / 2; ++e) acc[e] = 0ull;
        // activation block scales of this row, fetched one tap ahead
        float sa[C::NBLK], sa_next[C::NBLK];
        auto fetch_scales = [&](int tap, float (&dst)[C::NBLK]) {
            const int j = (row >= 0 && tap >= 0) ? nb[tap] : -1;
#pragma unroll
            for (int b = 0; b < C::NBLK; ++b)
                dst[b] = j >= 0 ? __ldg(a.a_scale + static_cast<int64_t>(j) * C::NBLK + b) : 0.f;
        };
        if (Q8 && !C::STAGED_SCALES) fetch_scales(rem ? rot_tap(__ffs(rem) - 1, rot) : -1, sa_next);
        while (rem) {
            const int tap = rot_tap(__ffs(rem) - 1, rot);
            rem &= rem - 1;
            // Q8 kinds: when none of this warp's 32 rows has a neighbour at
            // this tap, every block sum it would read is scaled by d_a = 0:
            // keep the slot protocol, skip the loads and the arithmetic
            const bool idle = Q8 && !__any_sync(0xffffffffu, row >= 0 && nb[tap] >= 0);
            // staged scales: this tap's stage holds the row's activation block
            // scales until every drain warp has released it after the tap
            const int ss = static_cast<int>(i % C::STAGES);
            if (C::STAGED_SCALES &&
                !wait_or_abort(&S.full[ss], static_cast<uint32_t>(i / C::STAGES) & 1, S.abort, a.status))
                return;
            if (!C::STAGED_SCALES && Q8) {
#pragma unroll
                for (int b = 0; b < C::NBLK; ++b) sa[b] = sa_next[b];
                fetch_scales(rem ? rot_tap(__ffs(rem) - 1, rot) : -1, sa_next);
            }
#pragma unroll 1
            for (int grp = 0; grp < C::KCH * C::GPS; ++grp, ++g) {
                const int slot = static_cast<int>(g % C::NACC);
                if (!wait_or_abort(&S.acc_full[slot], static_cast<uint32_t>(g / C::NACC) & 1, S.abort, a.status))
                    return;
                tc_fence_after();
                if (idle) {
                    tc_fence_before();
                    warp_arrive(&S.acc_empty[slot]);
                    continue;
                }
                float2 sg2 = make_float2(0.f, 0.f);
                if constexpr (C::STAGED_SCALES)
                    sg2 = *reinterpret_cast<const float2*>(S.sA + (ss * BM + m) * C::NBLK + grp * C::BPG);
#pragma unroll
                for (int b = 0; b < C::BPG; ++b) {
                    const int kb = grp * C::BPG + b;  // 32-channel block (Q8 kinds)
                    // this block's activation scale (select chain keeps sa in registers)
                    float sg = 0.f;
                    if constexpr (C::STAGED_SCALES) {
                        sg = b == 0 ? sg2.x : sg2.y;
                    } else if (Q8) {
                        sg = sa[0];
#pragma unroll
                        for (int bb = 1; bb < C::NBLK; ++bb) sg = kb == bb ? sa[bb] : sg;
                    }
                    // CH columns at a time: load, wait, accumulate; release the slot
                    // after the last load has landed
#pragma unroll
                    for (int c = 0; c < COLS; c += CH) {
                        uint32_t d[CH];
                        tmem_ld<CH>(tmem + lane_addr + static_cast<uint32_t>(slot * C::SLOT + b * COUT + c_base + c), d);
                        tmem_wait_ld_regs(d);
                        if (b + 1 == C::BPG && c + CH == COLS) {
                            tc_fence_before();
                            warp_arrive(&S.acc_empty[slot]);
                        }
                        if (KIND == KIND_Q8I) {
                            // acc += (d_a * d_w[n]) * isum[n]: (isum * d_a) is rounded once
                            // by an FMA that also removes the conversion offset, then
                            // fused into the accumulator with d_w[n]
                            const uint64_t s2 = pack2(sg, sg);
                            const uint64_t off2 = pack2(-kMagic * sg, -kMagic * sg);
                            const uint32_t sb = smem_u32(S.sB + (tap * C::NBLK + kb) * COUT + c_base + c);
#pragma unroll
                            for (int e = 0; e < CH / 4; ++e) {
                                uint64_t w01, w23;
                                lds_2x64(sb + 16 * e, w01, w23);
                                const uint64_t f0 = pack2(__int_as_float(static_cast<int>(d[4 * e]) + kMagicBits),
                                                          __int_as_float(static_cast<int>(d[4 * e + 1]) + kMagicBits));
                                const uint64_t f1 = pack2(__int_as_float(static_cast<int>(d[4 * e + 2]) + kMagicBits),
                                                          __int_as_float(static_cast<int>(d[4 * e + 3]) + kMagicBits));
                                acc[c / 2 + 2 * e] = fma2(fma2(f0, s2, off2), w01, acc[c / 2 + 2 * e]);
                                acc[c / 2 + 2 * e + 1] = fma2(fma2(f1, s2, off2), w23, acc[c / 2 + 2 * e + 1]);
                            }
                        } else if (KIND == KIND_Q8F) {
                            const uint64_t s2 = pack2(sg, sg);
#pragma unroll
                            for (int e = 0; e < CH / 2; ++e)
                                acc[c / 2 + e] =
                                    fma2(pack2(__uint_as_float(d[2 * e]), __uint_as_float(d[2 * e + 1])), s2, acc[c / 2 + e]);
                        } else {
#pragma unroll
                            for (int e = 0; e < CH / 2; ++e)
                                acc[c / 2 + e] = add2(acc[c / 2 + e], pack2(__uint_as_float(d[2 * e]), __uint_as_float(d[2 * e + 1])));
                        }
                    }
                }
            }
            if constexpr (C::STAGED_SCALES) {
                warp_arrive(&S.empty[ss]);
                ++i;
            }
        }
        // epilogue for this tile row / column slice
        // rows leave through lane transposes where the format allows:
        // 1 = fp16 (residual fp16 or none), 2 = fp32 without residual,
        // 3 = fused Q8_0 codes without residual; 0 = one row per lane
        int io = 0;
        if constexpr (COLS == 32) {
            if (a.q_codes)
                io = a.residual ? 0 : 3;
            else if (a.y_dtype == DT_F16 && (!a.residual || a.res_dtype == DT_F16))
                io = 1;
            else if (a.y_dtype == DT_F32 && !a.residual)
                io = 2;
        }
        if constexpr (COLS == 32) {
            if (io >= 2) {
                float v[32];
#pragma unroll
                for (int e = 0; e < 16; ++e) {
                    unpack2(acc[e], v[2 * e], v[2 * e + 1]);
#pragma unroll
                    for (int u = 0; u < 2; ++u) {
                        float t = v[2 * e + u] * oscale;
                        if (a.bias) t += S.bias[c_base + 2 * e + u];
                        if (a.silu_out) t = silu_fast(t);
                        v[2 * e + u] = t;
                    }
                }
                if (io == 3) {
                    // this thread holds one whole 32-channel block of the row:
                    // codes through a lane-pair transpose (each store covers 16
                    // rows x 32 bytes), the scale per row
                    uint32_t w[8];
                    const float d = quantize_block32(v, w);
                    const int64_t bcol = c_base / 32;
                    if (row >= 0) a.q_scales[static_cast<int64_t>(row) * (COUT / 32) + bcol] = d;
                    uint4 e[2] = {make_uint4(w[0], w[1], w[2], w[3]), make_uint4(w[4], w[5], w[6], w[7])};
                    pair_transpose(e);
                    const int pb = lane & ~1, pk = lane & 1;
#pragma unroll
                    for (int j = 0; j < 2; ++j) {
                        const int r = __shfl_sync(0xffffffffu, row, pb + j);
                        if (r >= 0)
                            reinterpret_cast<uint4*>(a.q_codes + (static_cast<int64_t>(r) * (COUT / 32) + bcol) * 32)[pk] =
                                e[j];
                    }
                } else {
                    // fp32 rows: two quad transposes (columns 0-15, 16-31); each
                    // store covers 8 rows x 64 contiguous bytes
                    const int qb = lane & ~3, qk = lane & 3;
#pragma unroll
                    for (int half = 0; half < 2; ++half) {
                        uint4 h[4];
#pragma unroll
                        for (int c4 = 0; c4 < 4; ++c4) {
                            const float* q = v + 16 * half + 4 * c4;
                            h[c4] = make_uint4(__float_as_uint(q[0]), __float_as_uint(q[1]), __float_as_uint(q[2]),
                                               __float_as_uint(q[3]));
                        }
                        quad_transpose(h);
#pragma unroll
                        for (int j = 0; j < 4; ++j) {
                            const int r = __shfl_sync(0xffffffffu, row, qb + j);
                            if (r >= 0)
                                reinterpret_cast<uint4*>(static_cast<float*>(a.y) + static_cast<int64_t>(r) * COUT +
                                                         c_base + 16 * half)[qk] = h[j];
                        }
                    }
                }
            }
            if (io == 1) {
                // fp16 rows through quad transposes: each load / store
                // instruction covers 8 rows x 64 contiguous bytes (this column
                // slice of the row) instead of 32 rows x 16 bytes
                const int qb = lane & ~3, qk = lane & 3;
                int rj[4];
#pragma unroll
                for (int j = 0; j < 4; ++j) rj[j] = __shfl_sync(0xffffffffu, row, qb + j);
                uint4 h[4];
#pragma unroll
                for (int j = 0; j < 4; ++j) h[j] = make_uint4(0u, 0u, 0u, 0u);
                if (a.residual) {
#pragma unroll
                    for (int j = 0; j < 4; ++j)
                        if (rj[j] >= 0)
                            h[j] = reinterpret_cast<const uint4*>(static_cast<const __half*>(a.residual) +
                                                                  static_cast<int64_t>(rj[j]) * COUT + c_base)[qk];
                    quad_transpose(h);  // h[c] = 16-byte chunk c of this lane's row
                }
#pragma unroll
                for (int c8 = 0; c8 < 4; ++c8) {
                    const float* bv = S.bias + c_base + 8 * c8;
                    uint32_t w[4] = {h[c8].x, h[c8].y, h[c8].z, h[c8].w};
#pragma unroll
                    for (int e2 = 0; e2 < 4; ++e2) {
                        float t[2];
                        unpack2(acc[4 * c8 + e2], t[0], t[1]);
                        const float2 r2 = __half22float2(*reinterpret_cast<const __half2*>(&w[e2]));
                        const float r[2] = {r2.x, r2.y};
#pragma unroll
                        for (int u = 0; u < 2; ++u) {
                            t[u] *= oscale;
                            if (a.bias) t[u] += bv[2 * e2 + u];
                            if (a.silu_out) t[u] = silu_fast(t[u]);
                            if (a.residual) t[u] += r[u];
                        }
                        const __half2 o = __floats2half2_rn(t[0], t[1]);
                        w[e2] = *reinterpret_cast<const uint32_t*>(&o);
                    }
                    h[c8] = make_uint4(w[0], w[1], w[2], w[3]);
                }
                quad_transpose(h);  // h[j] = chunk qk of row rj[j]
#pragma unroll
                for (int j = 0; j < 4; ++j) {
                    const int r = rj[j];
                    if (r < 0) continue;
                    if (a.store_limit <= 0 || r < a.store_limit)
                        reinterpret_cast<uint4*>(static_cast<__half*>(a.y) + static_cast<int64_t>(r) * COUT + c_base)[qk] =
                            h[j];
                    if (a.store_limit > 0) {
                        // boundary rows of a z-slab also go to the neighbour
                        // that holds them as halo rows (peer memory over NVLink)
                        if (a.peer_lo && r < a.send_lo)
                            reinterpret_cast<uint4*>(static_cast<__half*>(a.peer_lo) +
                                                     (a.peer_lo_off + r) * COUT + c_base)[qk] = h[j];
                        if (a.peer_hi && r >= a.send_hi_begin && r < a.store_limit)
                            reinterpret_cast<uint4*>(static_cast<__half*>(a.peer_hi) +
                                                     (a.peer_hi_off + (r - a.send_hi_begin)) * COUT + c_base)[qk] = h[j];
                    }
                }
            }
        }
        if (row >= 0 && io == 0) {
            constexpr int EC = COLS < 32 ? COLS : 32;
#pragma unroll
            for (int c0 = 0; c0 < COLS; c0 += EC) {
                float v[EC];
#pragma unroll
                for (int e = 0; e < EC / 2; ++e) unpack2(acc[c0 / 2 + e], v[2 * e], v[2 * e + 1]);
                // bias and residual in 8-column vector loads (the residual row
                // was prefetched to L2 at the start of the tile)
#pragma unroll
                for (int e8 = 0; e8 < EC; e8 += 8) {
                    const float* bv = S.bias + c_base + c0 + e8;
                    float rv[8];
                    if (a.residual)
                        load_row_vec<8>(a.residual, a.res_dtype, static_cast<int64_t>(row) * COUT + c_base + c0 + e8, rv);
#pragma unroll
                    for (int e = 0; e < 8; ++e) {
                        float t = v[e8 + e] * oscale;
                        if (a.bias) t += bv[e];
                        if (a.silu_out) t = silu_fast(t);
                        if (a.residual) t += rv[e];
                        v[e8 + e] = t;
                    }
                }
                if constexpr (EC == 32) {
                    // this thread holds one whole 32-channel block of the row
                    if (a.q_codes) {
                        const int64_t blk = static_cast<int64_t>(row) * (COUT / 32) + (c_base + c0) / 32;
                        quantize_store_block32(v, a.q_codes + blk * 32, a.q_scales + blk);
                        continue;
                    }
                }
                store_row<EC>(a.y, a.y_dtype, static_cast<int64_t>(row) * COUT + c_base + c0, v);
            }
        }
        warp_arrive(&S.tile_free[buf]);
    }
}

// Register budget: 20 warps x 32 threads x 96 registers = 61440.
template <int CIN, int COUT, int NA, int NB, int KIND>
__global__ void __maxnreg__(96) conv_tc_kernel(const ConvArgs a) {
    using C = Cfg<CIN, COUT, NA, NB, KIND>;
    extern __shared__ uint8_t smem_raw[];
    uint8_t* base = reinterpret_cast<uint8_t*>((reinterpret_cast<uintptr_t>(smem_raw) + 1023) & ~uintptr_t(1023));
    Smem S;
    S.stages = base;
    uint8_t* p = base + C::STAGES * C::STAGE;
    S.nbr = reinterpret_cast<int*>(p);
    p += C::NBR_BYTES;
    S.rows = reinterpret_cast<int*>(p);
    p += C::ROWS_BYTES;
    S.sB = reinterpret_cast<float*>(p);
    p += C::SB_BYTES;
    S.sA = reinterpret_cast<float*>(p);
    p += C::STAGES * C::SC_STAGE;
    S.bias = reinterpret_cast<float*>(p);
    p += C::BIAS_BYTES;
    uint64_t* bars = reinterpret_cast<uint64_t*>(p);
    S.full = bars;
    S.empty = S.full + C::STAGES;
    S.gathered = S.empty + C::STAGES;
    S.acc_full = S.gathered + C::STAGES;
    S.acc_empty = S.acc_full + C::NACC;
    S.tile_ready = S.acc_empty + C::NACC;
    S.tile_free = S.tile_ready + 2;
    S.drained = S.tile_free + 2;
    S.wmask = reinterpret_cast<uint32_t*>(S.drained + 1);
    S.tmem = S.wmask + 2 * kProducerWarps;
    S.abort = reinterpret_cast<int*>(S.tmem + 1);

    const int warp = threadIdx.x >> 5;
    if (threadIdx.x == 0) {
        for (int s = 0; s < C::STAGES; ++s) {
            mbar_init(&S.full[s], 2);  // publisher + weight tile
            mbar_init(&S.gathered[s], 32 * kProducerWarps);
            // the MMA's commit, plus every drain warp when the stage holds scales
            mbar_init(&S.empty[s], C::STAGED_SCALES ? 1 + kDrainWarps : 1);
        }
        for (int s = 0; s < C::NACC; ++s) {
            mbar_init(&S.acc_full[s], 1);
            mbar_init(&S.acc_empty[s], kDrainWarps);
        }
        for (int b = 0; b < 2; ++b) {
            mbar_init(&S.tile_ready[b], kProducerWarps);
            mbar_init(&S.tile_free[b], kDrainWarps);
        }
        mbar_init(S.drained, 1);
        *S.abort = 0;
        fence_mbar_init();
    }
    if (warp == kProducerWarps) {
        tmem_alloc(S.tmem, C::TMEM_COLS);
        tmem_relinquish();
    }
    if (KIND == KIND_Q8I) {
        // weight block scales [ntaps][NBLK][COUT] follow the code tiles
        const float4* src = reinterpret_cast<const float4*>(static_cast<const uint8_t*>(a.blob) + sizeof(WeightHeader) +
                                                            static_cast<size_t>(a.ntaps) * C::KCH * C::B_PLANE);
        float4* dst = reinterpret_cast<float4*>(S.sB);
        const int n4 = a.ntaps * C::NBLK * COUT / 4;
        for (int e = threadIdx.x; e < n4; e += kThreads) dst[e] = __ldg(src + e);
    }
    for (int e = threadIdx.x; e < COUT; e += kThreads) S.bias[e] = a.bias ? __ldg(a.bias + e) : 0.f;
    tc_fence_before();
    __syncthreads();
    tc_fence_after();
    const uint32_t tmem = *S.tmem;
    const int64_t ntiles = (a.n + BM - 1) / BM;

    if (warp < kProducerWarps) {
        producer<CIN, COUT, NA, NB, KIND>(a, S, ntiles);
    } else if (warp == kProducerWarps) {
        if ((threadIdx.x & 31) == 0) mma_issuer<CIN, COUT, NA, NB, KIND>(a, S, ntiles, tmem);
        __syncwarp();
    } else if (warp == kFenceWarp) {
        if ((threadIdx.x & 31) == 0) publisher<CIN, COUT, NA, NB, KIND>(a, S, ntiles);
        __syncwarp();
    } else {
        drainer<CIN, COUT, NA, NB, KIND>(a, S, ntiles, tmem);
    }

    tc_fence_before();
    __syncthreads();
    if (warp == kProducerWarps) {
        tc_fence_after();
        if (*reinterpret_cast<volatile int*>(S.abort)) {
            // a role gave up after a wait ran out: MMAs the issuer sent before
            // it stopped may still be writing TMEM; a commit tracks all of
            // them, so wait (bounded) for it before releasing the columns
            if ((threadIdx.x & 31) == 0) {
                umma_commit(S.drained);
                (void)mbar_wait(S.drained, 0);
            }
            __syncwarp();
        }
        tmem_dealloc(tmem, C::TMEM_COLS);
    }
}

template <int CIN, int COUT, int NA, int NB, int KIND>
cudaError_t launch_t(const ConvArgs& a, cudaStream_t st) {
    using C = Cfg<CIN, COUT, NA, NB, KIND>;
    auto kern = conv_tc_kernel<CIN, COUT, NA, NB, KIND>;
    // per device and instantiation: the shared-memory opt-in and the SM
    // count, set up once under a lock (host threads may launch concurrently)
    static std::mutex mu;
    static int num_sms[64] = {0};
    int dev = 0;
    cudaError_t e = cudaGetDevice(&dev);
    if (e != cudaSuccess) return e;
    if (dev < 0 || dev >= 64) return cudaErrorInvalidDevice;
    int sms = 0;
    {
        std::lock_guard<std::mutex> lk(mu);
        if (!num_sms[dev]) {
            e = cudaFuncSetAttribute(kern, cudaFuncAttributeMaxDynamicSharedMemorySize, C::SMEM);
            if (e != cudaSuccess) return e;
            int count = 0;
            e = cudaDeviceGetAttribute(&count, cudaDevAttrMultiProcessorCount, dev);
            if (e != cudaSuccess) return e;
            num_sms[dev] = count;
        }
        sms = num_sms[dev];
    }
    const int64_t ntiles = (a.n + BM - 1) / BM;
    const unsigned grid = static_cast<unsigned>(ntiles < sms ? ntiles : sms);
    kern<<<grid, kThreads, C::SMEM, st>>>(a);
    return cudaGetLastError();
}

template <int CIN, int COUT>
cudaError_t launch_planes(const ConvArgs& a, cudaStream_t st) {
    if (a.q8) {
        if constexpr (CIN == 128) {
            if (a.i8) return launch_t<CIN, COUT, 1, 1, KIND_Q8I>(a, st);
        }
        return a.i8 ? cudaErrorInvalidValue : launch_t<CIN, COUT, 1, 2, KIND_Q8F>(a, st);
    }
    if (a.na == 1 && a.wplanes == 1) return launch_t<CIN, COUT, 1, 1, KIND_F>(a, st);
    if (a.na == 1 && a.wplanes == 2) return launch_t<CIN, COUT, 1, 2, KIND_F>(a, st);
    if (a.na == 2 && a.wplanes == 1) return launch_t<CIN, COUT, 2, 1, KIND_F>(a, st);
    if (a.na == 2 && a.wplanes == 2) return launch_t<CIN, COUT, 2, 2, KIND_F>(a, st);
    return cudaErrorInvalidValue;
}

}  // namespace

bool conv_supported(int cin, int cout) { return (cin == 64 || cin == 128) && (cout == 64 || cout == 128); }

cudaError_t launch_conv(const ConvArgs& a, cudaStream_t st) {
    if (a.n == 0) return cudaSuccess;
    if (a.cin == 64 && a.cout == 64) return launch_planes<64, 64>(a, st);
    if (a.cin == 64 && a.cout == 128) return launch_planes<64, 128>(a, st);
    if (a.cin == 128 && a.cout == 64) return launch_planes<128, 64>(a, st);
    if (a.cin == 128 && a.cout == 128) return launch_planes<128, 128>(a, st);
    return cudaErrorInvalidValue;
}

}  // namespace msc
