// Sparse conv with ggml Q8_0 weights over a conv plan (plan.cu): each subtile
// loads its distinct input rows once into a shared-memory row cache and
// builds every tap's operand tile on chip.
//
// Arithmetic (ggml Q8_0 x Q8_0, mogecpp src/sparse.cpp:579-627 with ggml-cpu
// x86 quants.c:1308): per tap and 32-channel block, kind::i8 tensor-core MMAs
// give the exact integer block sum isum; the drain folds it in as
//     acc += (isum * d_a) * d_w[n]
// with d_a, d_w the fp16 block scales as fp32.  Each block accumulator
// starts from the int32 bit pattern of 1.5 * 2^23 (written by the drain when
// it releases the accumulator), so that after the MMA its bits read as the
// float 1.5 * 2^23 + isum (exact for |isum| < 2^22; |isum| <= 32 * 127^2) and
// one FMA with -1.5 * 2^23 * d_a yields isum * d_a rounded once.
//
// Why a row cache: on B200, random 128-byte row gathers from L2 sustain only
// ~7-15 B/clk per SM.  A Morton-ordered subtile of 128 voxels references
// ~200-300 distinct input rows rather than 27 x 128, so each is loaded once.
// Bulk copies cost ~370 cycles of copy-engine time each whatever their size
// (16 KB: 45 B/clk/SM, 32 KB: 88), so a tap's weight codes and block scales
// travel as one copy.
//
// Persistent CTA, one per SM, 20 warps (cin = 128, cout 64 or 128):
//   warps 0-2   producers.  Together, per subtile: its rows' int8 codes into
//               the row cache and their block scales (cp.async), from the U
//               list.  Per tap, warps 0-1 copy the 128 x 128 int8 operand
//               tile out of the cache (16-byte chunks, SW128 K-major) and
//               warp 2 issues one bulk copy of the tap's weight codes +
//               scales; warp 2 also prefetches the next subtile's slot map,
//               U list and output rows.  The builders never have copies in
//               flight when they execute their proxy fence: a thread's
//               fence.proxy.async waits for its own outstanding bulk and
//               cp.async copies (thousands of cycles).
//   warp 3      TMEM allocation and the single-thread MMA issue loop.
//   warps 4-19  drain + epilogue (TMEM lane quarter x column quarter).
#include "common.cuh"
#include "conv.h"
#include "conv_common.cuh"
#include "plan.h"

namespace msc {
namespace {

constexpr int BM = 128;
constexpr int CIN = 128;
constexpr int NBLK = CIN / 32;
constexpr int ROW = CIN;          // int8 codes per cache row
constexpr int NQ = ROW / 16;      // 16-byte chunks per row
constexpr int kPW = 3;            // producer warps: 2 builders + the loader
constexpr int kBW = 2;            // builder warps
constexpr int kBuilders = 32 * kBW;
constexpr int kLoader = kBuilders;  // thread index of the loader warp's lane 0
constexpr int kDW = 16;           // drain warps
constexpr int kThreads = 32 * (kPW + 1 + kDW);
constexpr int kProducers = 32 * kPW;
constexpr int kSmemLimit = 227 * 1024;
constexpr int kPrefetchTap = 3;   // taps built before the next subtile's metadata is fetched
constexpr uint32_t kMagicBits = 0x4B400000u;  // 1.5 * 2^23
constexpr float kMagic = 12582912.0f;

template <int COUT>
struct CCfg {
    static constexpr int A_BYTES = BM * ROW;                  // 16 KB
    static constexpr int B_BYTES = COUT * ROW;                // weight codes of one tap
    static constexpr int S_BYTES = NBLK * COUT * 4;           // block scales of one tap
    static constexpr int TAP_BYTES = B_BYTES + S_BYTES;       // one bulk copy
    static constexpr int STAGE = A_BYTES + TAP_BYTES;
    static constexpr int NACC = (512 / COUT) < 8 ? (512 / COUT) : 8;
    static constexpr int TMEM_COLS = NACC * COUT;
    static constexpr int COLS = COUT / 4;                     // drain columns per thread
    static constexpr int CACHE_BYTES = kPlanCap * ROW;
    static constexpr int SLOT_BYTES = 2 * BM * 27 * 2;
    static constexpr int U_BYTES = 2 * kPlanCap * 4;
    static constexpr int ROWS_BYTES = 2 * BM * 4;
    static constexpr int ASC_BYTES = 2 * kPlanCap * NBLK * 4;
    static constexpr int BAR_BYTES = 1024;
    static constexpr int FIXED = CACHE_BYTES + SLOT_BYTES + U_BYTES + ROWS_BYTES + ASC_BYTES + BAR_BYTES;
    static constexpr int STAGES_FIT = (kSmemLimit - 1024 - FIXED) / STAGE;
    static constexpr int STAGES = STAGES_FIT > 6 ? 6 : STAGES_FIT;
    static constexpr int SMEM = 1024 + STAGES * STAGE + FIXED;
    static_assert(STAGE % 1024 == 0, "SW128 tiles need 1024-byte aligned stages");
    static_assert(STAGES >= 3, "pipeline depth");
    static_assert(SMEM <= kSmemLimit, "shared memory budget");
    static_assert(TMEM_COLS == 512, "TMEM");
    static_assert(COLS % 16 == 0, "drain chunks and accumulator arming");
};

// tinfo fields (per buffer)
enum { TI_BEGIN = 0, TI_ROWS = 1, TI_UCNT = 2, TI_ROT = 3, TI_MASK = 4, TI_N = 8 };

struct CSmem {
    uint8_t* stages;     // [STAGES] {A tile | weight codes | weight block scales}
    uint8_t* cache;      // [kPlanCap][ROW] int8 codes, 16-byte chunks XOR-swizzled by slot
    uint16_t* slots;     // [2][BM*27] (row, tap) -> U-list position
    int* ulist;          // [2][kPlanCap]
    int* rows;           // [2][BM] output voxel of each tile row
    float* ascale;       // [2][kPlanCap][NBLK] activation block scales of the cached rows
    uint64_t* full;      // [STAGES] producers' tiles + the weight copy landed
    uint64_t* empty;     // [STAGES] MMAs done and every drain warp past the tap's scales
    uint64_t* acc_full;  // [NACC]
    uint64_t* acc_empty; // [NACC]
    uint64_t* tile_ready;  // [2] cache and metadata of a subtile ready
    uint64_t* tile_free;   // [2] drain done with a subtile's metadata
    uint64_t* pgrp;        // producer-group barrier (bounded wait)
    int* tinfo;            // [2][TI_N]
    uint32_t* tmem;
    int* abort;
};

// Barrier of the producer warps: an mbarrier with a bounded wait, so that a
// producer that gave up on a wait cannot leave the others blocked.
__device__ __forceinline__ bool group_sync(const CSmem& S, uint32_t n, uint32_t* status) {
    warp_arrive(S.pgrp);
    return wait_or_abort(S.pgrp, n & 1, S.abort, status);
}

struct Desc {
    int begin, uoff, rows, ucnt;
    uint32_t mask;
};

// Reads descriptor d; one outside the plan's bounds becomes an empty subtile.
__device__ __forceinline__ Desc load_desc(const ConvArgs& a, const PlanView& P, int64_t d, int64_t pool_cap,
                                          bool report) {
    const int4 v = __ldg(P.desc + d);
    Desc r{v.x, v.y, v.z & 0xff, v.z >> 8, static_cast<uint32_t>(v.w) & 0x7ffffffu};
    const bool ok = r.rows >= 1 && r.rows <= BM && r.begin >= 0 && (r.begin & 7) == 0 &&
                    static_cast<int64_t>(r.begin) + r.rows <= a.n && r.ucnt >= 0 && r.ucnt <= kPlanCap &&
                    r.uoff >= 0 && (r.uoff & 3) == 0 && static_cast<int64_t>(r.uoff) + r.ucnt <= pool_cap;
    if (!ok) {
        if (report) set_status(a.status, MSC_DEV_BAD_INDEX);
        r = Desc{0, 0, 0, 0, 0u};
    }
    return r;
}

// Issues the asynchronous copies of a subtile's slot map, U list and output
// rows into buffer `buf`, all 16-byte aligned by the plan's construction
// (subtiles start at multiples of 8 rows, U lists at multiples of 4).  A
// ragged last subtile's copies end at most 15 bytes past its sections, inside
// the plan's 256-byte section padding.
__device__ __forceinline__ void fetch_meta(const ConvArgs& a, const CSmem& S, const PlanView& P, const Desc& ds,
                                           int buf) {
    const int t0 = threadIdx.x & 31;  // the loader warp
    const int nrow = ds.rows;
    const int nslot = (nrow * 27 * 2 + 15) / 16;
    const uint8_t* src_s = reinterpret_cast<const uint8_t*>(P.slots + static_cast<int64_t>(ds.begin) * 27);
    const uint32_t dst_s = smem_u32(S.slots + buf * BM * 27);
    for (int e = t0; e < nslot; e += 32) cp_async16(dst_s + e * 16, src_s + e * 16, 16);
    const int nu = (ds.ucnt + 3) / 4;
    const uint32_t dst_u = smem_u32(S.ulist + buf * kPlanCap);
    for (int e = t0; e < nu; e += 32) cp_async16(dst_u + e * 16, P.pool + ds.uoff + 4 * e, 16);
    const uint32_t dst_r = smem_u32(S.rows + buf * BM);
    for (int e = t0; e < (nrow + 3) / 4; e += 32) cp_async16(dst_r + e * 16, P.perm + ds.begin + 4 * e, 16);
    cp_async_commit();
    if (t0 == 0) {
        int* ti = S.tinfo + buf * TI_N;
        ti[TI_BEGIN] = ds.begin;
        ti[TI_ROWS] = nrow;
        ti[TI_UCNT] = ds.ucnt;
        ti[TI_ROT] = a.ntaps == 27 ? (ds.begin / BM) % 27 : 0;
        ti[TI_MASK] = static_cast<int>(ds.mask);
    }
}

template <int COUT>
__device__ void c_producer(const ConvArgs& a, const CSmem& S, const PlanView& P, int64_t ndesc, int64_t pool_cap) {
    using C = CCfg<COUT>;
    const int t0 = threadIdx.x;
    const int8_t* codes = static_cast<const int8_t*>(a.planes);
    const uint8_t* wdata = static_cast<const uint8_t*>(a.blob);  // the blob's row-cached section
    int64_t i = 0;     // stages (taps) issued
    uint32_t pg = 0;   // producer-group syncs
    int k = 0;
    const bool loader = t0 >= kBuilders;
    int64_t d = blockIdx.x;
    if (loader && d < ndesc) fetch_meta(a, S, P, load_desc(a, P, d, pool_cap, t0 == kLoader), 0);
    for (; d < ndesc; d += gridDim.x, ++k) {
        const int buf = k & 1;
        const int64_t dn = d + gridDim.x;
        Desc next{0, 0, 0, 0, 0u};
        if (loader && dn < ndesc) next = load_desc(a, P, dn, pool_cap, t0 == kLoader);
        // this subtile's metadata has landed (its copies were the last committed)
        cp_async_wait_all();
        if (!group_sync(S, pg++, a.status)) return;
        const int* ti = S.tinfo + buf * TI_N;
        const int ucnt = ti[TI_UCNT];
        const int rows = ti[TI_ROWS];
        const int rot = ti[TI_ROT];
        const int* ul = S.ulist + buf * kPlanCap;
        float* asc = S.ascale + buf * kPlanCap * NBLK;
        // row cache (single buffer: every producer is past the previous
        // subtile's builds) and the rows' activation scales
        for (int e = t0; e < ucnt * NQ; e += kProducers) {
            const int slot = e / NQ, q = e % NQ;
            int64_t j = ul[slot];
            const bool jok = static_cast<uint64_t>(j) < static_cast<uint64_t>(a.n_in);
            if (!jok) {
                if (q == 0) set_status(a.status, MSC_DEV_BAD_INDEX);
                j = 0;
            }
            cp_async16(smem_u32(S.cache + slot * ROW + ((q ^ (slot & (NQ - 1))) << 4)), codes + j * ROW + q * 16,
                       jok ? 16u : 0u);
        }
        for (int e = t0; e < ucnt; e += kProducers) {
            const int64_t j = ul[e];
            const bool jok = static_cast<uint64_t>(j) < static_cast<uint64_t>(a.n_in);
            cp_async16(smem_u32(asc + e * NBLK), a.a_scale + (jok ? j : 0) * NBLK, jok ? 16u : 0u);
        }
        cp_async_commit();
        cp_async_wait_all();
        if (!group_sync(S, pg++, a.status)) return;
        if (t0 == 0) mbar_arrive(&S.tile_ready[buf]);  // the group is synchronised
        const uint16_t* sl = S.slots + buf * BM * 27;
        uint32_t rem = rot_mask(static_cast<uint32_t>(ti[TI_MASK]), rot);
        bool prefetched = dn >= ndesc;
        for (int tcount = 0; rem; ++tcount, ++i) {
            const int tap = rot_tap(__ffs(rem) - 1, rot);
            rem &= rem - 1;
            const int s = static_cast<int>(i % C::STAGES);
            uint8_t* sA = S.stages + s * C::STAGE;
            if (loader) {
                if (!prefetched && tcount == kPrefetchTap) {
                    // the drain has left the other buffer's metadata (subtile k-1)
                    if (k >= 1 && !wait_or_abort(&S.tile_free[buf ^ 1], ((k - 1) >> 1) & 1, S.abort, a.status))
                        return;
                    fetch_meta(a, S, P, next, buf ^ 1);
                    prefetched = true;
                }
                // every lane waits (no warp-synchronous step that a lane
                // leaving on an abort could block); lane 0 issues the copy
                if (i >= C::STAGES &&
                    !wait_or_abort(&S.empty[s], static_cast<uint32_t>((i / C::STAGES) - 1) & 1, S.abort, a.status))
                    return;
                if (t0 == kLoader) {
                    mbar_arrive_expect_tx(&S.full[s], C::TAP_BYTES);
                    bulk_g2s(smem_u32(sA + C::A_BYTES), wdata + static_cast<int64_t>(tap) * C::TAP_BYTES,
                             C::TAP_BYTES, &S.full[s]);
                }
                continue;
            }
            if (i >= C::STAGES &&
                !wait_or_abort(&S.empty[s], static_cast<uint32_t>((i / C::STAGES) - 1) & 1, S.abort, a.status))
                return;
            // operand tile: unit u = (row u/8, 16-byte chunk u%8)
#pragma unroll 4
            for (int q = 0; q < (BM * NQ) / kBuilders; ++q) {
                const int u = t0 + q * kBuilders;
                const int r = u >> 3, c = u & 7;
                const int slot = r < rows ? sl[r * 27 + tap] : kNoSlot;
                uint4 v = make_uint4(0u, 0u, 0u, 0u);
                if (slot < ucnt) v = *reinterpret_cast<const uint4*>(S.cache + slot * ROW + ((c ^ (slot & 7)) << 4));
                *reinterpret_cast<uint4*>(sA + sw128_offset(r, c)) = v;
            }
            fence_proxy_async();
            warp_arrive(&S.full[s]);
        }
        if (loader && !prefetched) {
            if (k >= 1 && !wait_or_abort(&S.tile_free[buf ^ 1], ((k - 1) >> 1) & 1, S.abort, a.status)) return;
            fetch_meta(a, S, P, next, buf ^ 1);
        }
    }
}

template <int COUT>
__device__ void c_mma(const ConvArgs& a, const CSmem& S, int64_t ndesc, uint32_t tmem) {
    using C = CCfg<COUT>;
    constexpr uint32_t idesc = idesc_i8(BM, COUT);
    int64_t i = 0, g = 0;
    int k = 0;
    for (int64_t d = blockIdx.x; d < ndesc; d += gridDim.x, ++k) {
        const int buf = k & 1;
        if (!wait_or_abort(&S.tile_ready[buf], (k >> 1) & 1, S.abort, a.status)) return;
        const int ntap = __popc(static_cast<uint32_t>(S.tinfo[buf * TI_N + TI_MASK]));
        for (int t = 0; t < ntap; ++t, ++i) {
            const int s = static_cast<int>(i % C::STAGES);
            if (!wait_or_abort(&S.full[s], static_cast<uint32_t>(i / C::STAGES) & 1, S.abort, a.status)) return;
            tc_fence_after();
            const uint32_t aaddr = smem_u32(S.stages + s * C::STAGE);
            const uint32_t baddr = aaddr + C::A_BYTES;
#pragma unroll
            for (int grp = 0; grp < NBLK; ++grp, ++g) {
                const int slot = static_cast<int>(g % C::NACC);
                if (g >= C::NACC &&
                    !wait_or_abort(&S.acc_empty[slot], static_cast<uint32_t>((g / C::NACC) - 1) & 1, S.abort,
                                   a.status))
                    return;
                tc_fence_after();
                // K = 32 int8 = one Q8_0 block; accumulate onto the magic bias
                umma_i8(tmem + static_cast<uint32_t>(slot * COUT), sdesc_k_sw128(aaddr + grp * 32),
                        sdesc_k_sw128(baddr + grp * 32), idesc, 1u);
                umma_commit(&S.acc_full[slot]);
            }
            umma_commit(&S.empty[s]);
        }
    }
}

template <int COUT>
__device__ void c_drain(const ConvArgs& a, const CSmem& S, int64_t ndesc, uint32_t tmem) {
    using C = CCfg<COUT>;
    constexpr int COLS = C::COLS;
    const int warp = threadIdx.x >> 5;
    const int q = warp & 3;
    const int part = (warp - kPW - 1) >> 2;
    const int m = q * 32 + (threadIdx.x & 31);
    const int c_base = part * COLS;
    const uint32_t lane_addr = static_cast<uint32_t>(q * 32) << 16;
    int64_t g = 0, i = 0;
    int k = 0;
    for (int64_t d = blockIdx.x; d < ndesc; d += gridDim.x, ++k) {
        const int buf = k & 1;
        if (!wait_or_abort(&S.tile_ready[buf], (k >> 1) & 1, S.abort, a.status)) return;
        const int* ti = S.tinfo + buf * TI_N;
        const int rot = ti[TI_ROT];
        const int rows = ti[TI_ROWS];
        const int ucnt = ti[TI_UCNT];
        uint32_t rem = rot_mask(static_cast<uint32_t>(ti[TI_MASK]), rot);
        const bool live_row = m < rows;
        const uint16_t* sl = S.slots + buf * BM * 27 + m * 27;
        const float* asc = S.ascale + buf * kPlanCap * NBLK;
        uint64_t acc[COLS / 2];
#pragma unroll
        for (int e = 0; e < COLS / 2; ++e) acc[e] = 0ull;
        for (; rem; ++i) {
            const int tap = rot_tap(__ffs(rem) - 1, rot);
            rem &= rem - 1;
            const int s = static_cast<int>(i % C::STAGES);
            const int us = live_row ? sl[tap] : kNoSlot;
            const bool live = us < ucnt;
            // a missing neighbour has a zero operand row and a zero scale
            const float* sap = asc + (live ? us : 0) * NBLK;
            const float* wsc = reinterpret_cast<const float*>(S.stages + s * C::STAGE + C::A_BYTES + C::B_BYTES);
#pragma unroll 1
            for (int grp = 0; grp < NBLK; ++grp, ++g) {
                const float sa = live ? sap[grp] : 0.0f;
                const int slot = static_cast<int>(g % C::NACC);
                if (!wait_or_abort(&S.acc_full[slot], static_cast<uint32_t>(g / C::NACC) & 1, S.abort, a.status))
                    return;
                tc_fence_after();
                const uint64_t s2 = pack2(sa, sa);
                const uint64_t nm2 = pack2(-kMagic * sa, -kMagic * sa);
                const float* sbrow = wsc + grp * COUT + c_base;
                const uint32_t col = tmem + lane_addr + static_cast<uint32_t>(slot * COUT + c_base);
                // 16 columns per load; after the arithmetic, re-arm the
                // accumulator and release it
#pragma unroll
                for (int c = 0; c < COLS; c += 16) {
                    uint32_t dv[16];
                    tmem_ld<16>(col + c, dv);
                    tmem_wait_ld_regs(dv);
                    const float4* sb = reinterpret_cast<const float4*>(sbrow + c);
#pragma unroll
                    for (int e = 0; e < 4; ++e) {
                        const float4 w = sb[e];
                        // (1.5*2^23 + isum) * d_a - 1.5*2^23 * d_a = isum * d_a, one rounding
                        const uint64_t t0 =
                            fma2(pack2(__uint_as_float(dv[4 * e]), __uint_as_float(dv[4 * e + 1])), s2, nm2);
                        const uint64_t t1 =
                            fma2(pack2(__uint_as_float(dv[4 * e + 2]), __uint_as_float(dv[4 * e + 3])), s2, nm2);
                        acc[c / 2 + 2 * e] = fma2(t0, pack2(w.x, w.y), acc[c / 2 + 2 * e]);
                        acc[c / 2 + 2 * e + 1] = fma2(t1, pack2(w.z, w.w), acc[c / 2 + 2 * e + 1]);
                    }
                }
#pragma unroll
                for (int c = 0; c < COLS; c += 8) tmem_st8_fill(col + c, kMagicBits);
                tmem_wait_st();
                tc_fence_before();
                warp_arrive(&S.acc_empty[slot]);
            }
            // done with this tap's weight scales in the stage
            warp_arrive(&S.empty[s]);
        }
        const int row = live_row ? S.rows[buf * BM + m] : -1;
        if (row >= 0 && static_cast<int64_t>(row) < a.n) {
            constexpr int EC = 8;  // small chunks: the accumulators already hold COLS registers
#pragma unroll
            for (int c0 = 0; c0 < COLS; c0 += EC) {
                float v[EC];
#pragma unroll
                for (int e = 0; e < EC / 2; ++e) unpack2(acc[c0 / 2 + e], v[2 * e], v[2 * e + 1]);
#pragma unroll
                for (int e = 0; e < EC; ++e) {
                    const int n = c_base + c0 + e;
                    float t = v[e];
                    if (a.bias) t += __ldg(a.bias + n);
                    if (a.silu_out) t = silu_f(t);
                    if (a.residual) t += load_elem(a.residual, a.res_dtype, static_cast<int64_t>(row) * COUT + n);
                    v[e] = t;
                }
                store_row<EC>(a.y, a.y_dtype, static_cast<int64_t>(row) * COUT + c_base + c0, v);
            }
        } else if (live_row) {
            set_status(a.status, MSC_DEV_BAD_INDEX);
        }
        warp_arrive(&S.tile_free[buf]);
    }
}

// 20 warps x 32 threads x 96 registers = 61440 of the SM's 65536.
template <int COUT>
__global__ void __maxnreg__(96) conv_cached_kernel(const ConvArgs a, const uint8_t* plan) {
    using C = CCfg<COUT>;
    // a plan that overflowed or belongs to another level is refused before
    // any barrier or TMEM is set up (every thread reads the same header)
    const PlanHeader* hdr = reinterpret_cast<const PlanHeader*>(plan);
    if (hdr->magic != kPlanMagic || hdr->overflow != 0 || hdr->n != a.n) {
        if (blockIdx.x == 0 && threadIdx.x == 0) set_status(a.status, MSC_DEV_PLAN_OVERFLOW);
        return;
    }
    extern __shared__ uint8_t smem_raw[];
    uint8_t* base = reinterpret_cast<uint8_t*>((reinterpret_cast<uintptr_t>(smem_raw) + 1023) & ~uintptr_t(1023));
    CSmem S;
    S.stages = base;
    uint8_t* p = base + C::STAGES * C::STAGE;
    S.cache = p;
    p += C::CACHE_BYTES;
    S.slots = reinterpret_cast<uint16_t*>(p);
    p += C::SLOT_BYTES;
    S.ulist = reinterpret_cast<int*>(p);
    p += C::U_BYTES;
    S.rows = reinterpret_cast<int*>(p);
    p += C::ROWS_BYTES;
    S.ascale = reinterpret_cast<float*>(p);
    p += C::ASC_BYTES;
    uint64_t* bars = reinterpret_cast<uint64_t*>(p);
    S.full = bars;
    S.empty = S.full + C::STAGES;
    S.acc_full = S.empty + C::STAGES;
    S.acc_empty = S.acc_full + C::NACC;
    S.tile_ready = S.acc_empty + C::NACC;
    S.tile_free = S.tile_ready + 2;
    S.pgrp = S.tile_free + 2;
    S.tinfo = reinterpret_cast<int*>(S.pgrp + 1);
    S.tmem = reinterpret_cast<uint32_t*>(S.tinfo + 2 * TI_N);
    S.abort = reinterpret_cast<int*>(S.tmem + 1);

    const PlanView P = plan_view(const_cast<uint8_t*>(plan), hdr->n, hdr->max_desc);
    const int64_t ndesc = static_cast<int64_t>(
        hdr->ndesc < static_cast<unsigned long long>(hdr->max_desc) ? hdr->ndesc : hdr->max_desc);
    const int64_t pool_cap = hdr->pool_cap;
    const int warp = threadIdx.x >> 5;
    if (threadIdx.x == 0) {
        for (int s = 0; s < C::STAGES; ++s) {
            mbar_init(&S.full[s], kBW + 1);
            mbar_init(&S.empty[s], 1 + kDW);
        }
        for (int s = 0; s < C::NACC; ++s) {
            mbar_init(&S.acc_full[s], 1);
            mbar_init(&S.acc_empty[s], kDW);
        }
        for (int b = 0; b < 2; ++b) {
            mbar_init(&S.tile_ready[b], 1);
            mbar_init(&S.tile_free[b], kDW);
        }
        mbar_init(S.pgrp, kPW);
        *S.abort = 0;
        fence_mbar_init();
    }
    if (warp == kPW) {
        tmem_alloc(S.tmem, C::TMEM_COLS);
        tmem_relinquish();
    }
    tc_fence_before();
    __syncthreads();
    tc_fence_after();
    const uint32_t tmem = *S.tmem;
    // arm every accumulator with the magic bias
    if (warp > kPW) {
        const int q = warp & 3;
        const int part = (warp - kPW - 1) >> 2;
        const uint32_t lane_addr = static_cast<uint32_t>(q * 32) << 16;
#pragma unroll 1
        for (int slot = 0; slot < C::NACC; ++slot)
#pragma unroll
            for (int c = 0; c < C::COLS; c += 16)
                tmem_st16_fill(tmem + lane_addr + static_cast<uint32_t>(slot * COUT + part * C::COLS + c), kMagicBits);
        tmem_wait_st();
    }
    tc_fence_before();
    __syncthreads();
    tc_fence_after();

    if (warp < kPW) {
        c_producer<COUT>(a, S, P, ndesc, pool_cap);
        cp_async_wait_all();
    } else if (warp == kPW) {
        if ((threadIdx.x & 31) == 0) c_mma<COUT>(a, S, ndesc, tmem);
        __syncwarp();
    } else {
        c_drain<COUT>(a, S, ndesc, tmem);
    }

    tc_fence_before();
    __syncthreads();
    if (warp == kPW) {
        tc_fence_after();
        tmem_dealloc(tmem, C::TMEM_COLS);
    }
}

template <int COUT>
cudaError_t launch_c(const ConvArgs& a, const void* plan, int64_t max_tiles, cudaStream_t st) {
    using C = CCfg<COUT>;
    auto kern = conv_cached_kernel<COUT>;
    static int num_sms[64] = {0};
    int dev = 0;
    cudaError_t e = cudaGetDevice(&dev);
    if (e != cudaSuccess) return e;
    if (dev < 0 || dev >= 64) return cudaErrorInvalidDevice;
    if (!num_sms[dev]) {
        e = cudaFuncSetAttribute(kern, cudaFuncAttributeMaxDynamicSharedMemorySize, C::SMEM);
        if (e != cudaSuccess) return e;
        int sms = 0;
        e = cudaDeviceGetAttribute(&sms, cudaDevAttrMultiProcessorCount, dev);
        if (e != cudaSuccess) return e;
        num_sms[dev] = sms;
    }
    const unsigned grid = static_cast<unsigned>(max_tiles < num_sms[dev] ? (max_tiles > 0 ? max_tiles : 1) : num_sms[dev]);
    kern<<<grid, kThreads, C::SMEM, st>>>(a, static_cast<const uint8_t*>(plan));
    return cudaGetLastError();
}

}  // namespace

bool conv_cached_supported(int cin, int cout) { return cin == CIN && (cout == 64 || cout == 128); }

cudaError_t launch_conv_cached(const ConvArgs& a, const void* plan, cudaStream_t st) {
    if (a.n == 0) return cudaSuccess;
    if (!conv_cached_supported(a.cin, a.cout) || a.ntaps != 27) return cudaErrorInvalidValue;
    const int64_t max_tiles = (a.n + BM - 1) / BM;
    if (a.cout == 64) return launch_c<64>(a, plan, max_tiles, st);
    return launch_c<128>(a, plan, max_tiles, st);
}

}  // namespace msc
