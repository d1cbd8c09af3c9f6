// Submanifold sparse 3-D convolution (and its 1-tap special case, the
// per-voxel linear layer) as an implicit gather-GEMM on the sm_100a tensor
// cores.
//
// Reference semantics (mogecpp src/sparse.cpp:579-627 sparse_conv):
//   y[i, :] = sum_t W_t x[nbr[i][t], :] + bias,  nbr sentinel = zero row,
// with W packed [cout][27*cin] (cin fastest, taps in neighbour-map order).
//
// Tile: 128 output voxels (M) x cout (N) accumulated in TMEM (fp32), K loops
// over (tap, 64-channel chunk) stages; taps with no valid neighbour in the
// tile are skipped.  Operands are fp16 "planes": A = gathered activation
// rows (1 plane, or an exact hi/lo pair), B = prepared weights (1 plane or
// hi/lo pair).  For two-plane operands the MMA sums hi*hi + hi*lo + lo*hi,
// which reproduces fp32 products of <=22-bit operands to ~2^-22 (used for
// fp32 weights and for ggml's Q8_0 x Q8_0 block dot products).
//
// Warp roles (160 threads):
//   warps 0-3  producers: each thread gathers one A row per stage with
//              16-byte cp.async (sentinel rows zero-filled), thread 0 also
//              issues the bulk copy of the stage's pre-swizzled B tile;
//              after the main loop the same warps run the epilogue (TMEM
//              lane 32w+l = voxel row).
//   warp 4     TMEM allocation and the single-thread MMA issue loop.
// smem stages: [A planes][B planes], 128B-swizzled K-major; mbarriers full
// (128 producer arrivals + 1 tx arrival) and empty (tcgen05.commit).
#include "common.cuh"
#include "conv.h"

#include <algorithm>

namespace msc {
namespace {

constexpr int BM = 128;
constexpr int BK = 64;                  // fp16 elements per stage row (128 B)
constexpr int kProducerThreads = 128;
constexpr int kThreads = kProducerThreads + 32;
constexpr int kSmemBudget = 200 * 1024;

template <int CIN, int COUT, int NA, int NB>
struct Cfg {
    static constexpr int KCH = CIN / BK;
    static constexpr int A_PLANE = BM * BK * 2;
    static constexpr int B_PLANE = COUT * BK * 2;
    static constexpr int STAGE = NA * A_PLANE + NB * B_PLANE;
    static constexpr int STAGES_FIT = kSmemBudget / STAGE;
    static constexpr int STAGES = STAGES_FIT > 4 ? 4 : STAGES_FIT;
    static constexpr int NBR_BYTES = BM * 27 * 4;
    static constexpr int SMEM = 1024 /*align slack*/ + STAGES * STAGE + NBR_BYTES + 256;
    static constexpr int TMEM_COLS = COUT < 32 ? 32 : COUT;
    static_assert(STAGES >= 2, "at least two pipeline stages");
    static_assert(CIN % BK == 0, "cin must be a multiple of 64");
    static_assert(COUT % 16 == 0 && COUT >= 16 && COUT <= 256, "UMMA N range for M=128");
    static_assert((COUT & (COUT - 1)) == 0, "TMEM allocation is a power of two");
};

__device__ __forceinline__ float load_elem(const void* p, int dtype, int64_t idx) {
    if (dtype == DT_F32) return static_cast<const float*>(p)[idx];
    if (dtype == DT_F16) return __half2float(static_cast<const __half*>(p)[idx]);
    return __bfloat162float(static_cast<const __nv_bfloat16*>(p)[idx]);
}

template <int CIN, int COUT, int NA, int NB>
__global__ void __launch_bounds__(kThreads, 1) conv_tc_kernel(ConvArgs a) {
    using C = Cfg<CIN, COUT, NA, NB>;
    extern __shared__ uint8_t smem_raw[];
    uint8_t* smem = reinterpret_cast<uint8_t*>((reinterpret_cast<uintptr_t>(smem_raw) + 1023) & ~uintptr_t(1023));
    uint8_t* stage_base = smem;
    int* s_nbr = reinterpret_cast<int*>(smem + C::STAGES * C::STAGE);
    uint64_t* full = reinterpret_cast<uint64_t*>(smem + C::STAGES * C::STAGE + C::NBR_BYTES);
    uint64_t* empty = full + C::STAGES;
    uint64_t* done = empty + C::STAGES;
    uint32_t* s_tmem = reinterpret_cast<uint32_t*>(done + 1);
    uint32_t* s_mask = s_tmem + 1;
    int* s_abort = reinterpret_cast<int*>(s_mask + 1);

    const int tid = threadIdx.x;
    const int warp = tid >> 5;
    const int64_t row0 = static_cast<int64_t>(blockIdx.x) * BM;
    const int64_t n = a.n;
    const int ntaps = a.ntaps;

    if (tid == 0) {
        for (int s = 0; s < C::STAGES; ++s) {
            mbar_init(&full[s], kProducerThreads + 1);
            mbar_init(&empty[s], 1);
        }
        mbar_init(done, 1);
        *s_mask = 0;
        *s_abort = 0;
        fence_mbar_init();
    }
    if (warp == 4) {
        tmem_alloc(s_tmem, C::TMEM_COLS);
        tmem_relinquish();
    }
    // stage the tile's neighbour rows and build the tap-occupancy mask
    if (a.nbr) {
        const int rows = static_cast<int>(n - row0 < BM ? n - row0 : BM);
        const int* src = a.nbr + row0 * 27;
        for (int k = tid; k < rows * 27; k += kThreads) s_nbr[k] = __ldg(src + k);
    }
    __syncthreads();
    if (tid < kProducerThreads) {
        uint32_t m = 0;
        if (row0 + tid < n) {
            if (a.nbr) {
                for (int t = 0; t < 27; ++t) {
                    const int j = s_nbr[tid * 27 + t];
                    if (static_cast<uint64_t>(j) < static_cast<uint64_t>(n)) m |= 1u << t;
                }
            } else {
                m = 1u;
            }
        }
        m |= __shfl_xor_sync(0xffffffffu, m, 1);
        m |= __shfl_xor_sync(0xffffffffu, m, 2);
        m |= __shfl_xor_sync(0xffffffffu, m, 4);
        m |= __shfl_xor_sync(0xffffffffu, m, 8);
        m |= __shfl_xor_sync(0xffffffffu, m, 16);
        if ((tid & 31) == 0 && m) atomicOr(s_mask, m);
    }
    tc_fence_before();
    __syncthreads();
    tc_fence_after();
    const uint32_t tmem = *s_tmem;
    const uint32_t mask = *s_mask;
    const int nst = __popc(mask) * C::KCH;

    const __half* planes = static_cast<const __half*>(a.planes);
    const uint8_t* wdata = static_cast<const uint8_t*>(a.blob) + sizeof(WeightHeader);
    const int64_t plane_stride = n * CIN;
    constexpr int LAG = C::STAGES - 1;

    if (tid < kProducerThreads) {
        // ---------------------------------------------------------- producer
        const int r = tid;
        const bool row_ok = row0 + r < n;
        uint32_t rem = mask;
        int tap = -1, kc = C::KCH;
        bool ok = true;
        for (int i = 0; i < nst; ++i) {
            if (kc == C::KCH) {
                tap = __ffs(rem) - 1;
                rem &= rem - 1;
                kc = 0;
            }
            const int s = i % C::STAGES;
            if (i >= C::STAGES) {
                if (!mbar_wait(&empty[s], ((i / C::STAGES) - 1) & 1)) {
                    ok = false;
                    break;
                }
            }
            uint8_t* sA = stage_base + s * C::STAGE;
            uint8_t* sB = sA + NA * C::A_PLANE;
            if (r == 0) {
                mbar_arrive_expect_tx(&full[s], NB * C::B_PLANE);
                bulk_g2s(smem_u32(sB), wdata + static_cast<int64_t>(tap * C::KCH + kc) * NB * C::B_PLANE,
                         NB * C::B_PLANE, &full[s]);
            }
            int64_t j = -1;
            if (row_ok) {
                if (a.nbr) {
                    const int jj = s_nbr[r * 27 + tap];
                    if (static_cast<uint64_t>(jj) < static_cast<uint64_t>(n)) j = jj;
                } else {
                    j = row0 + r;
                }
            }
            const uint32_t nbytes = j >= 0 ? 16u : 0u;
#pragma unroll
            for (int p = 0; p < NA; ++p) {
                const __half* src = j >= 0 ? planes + p * plane_stride + j * CIN + kc * BK : planes;
                const uint32_t dst = smem_u32(sA + p * C::A_PLANE);
#pragma unroll
                for (int c = 0; c < 8; ++c) cp_async16(dst + sw128_offset(r, c), src + (j >= 0 ? c * 8 : 0), nbytes);
            }
            cp_async_commit();
            if (i >= LAG) {
                cp_async_wait<LAG>();
                fence_proxy_async();
                mbar_arrive(&full[(i - LAG) % C::STAGES]);
            }
            ++kc;
        }
        cp_async_wait_all();
        if (ok) {
            fence_proxy_async();
            for (int i = max(0, nst - LAG); i < nst; ++i) mbar_arrive(&full[i % C::STAGES]);
        } else {
            atomicExch(s_abort, 1);
            set_status(a.status, MSC_DEV_TIMEOUT);
        }
    } else if (warp == 4) {
        // ---------------------------------------------------------- MMA
        if ((tid & 31) == 0) {
            constexpr uint32_t idesc = idesc_f16(BM, COUT, 0);
            bool ok = true;
            for (int i = 0; i < nst; ++i) {
                const int s = i % C::STAGES;
                if (!mbar_wait(&full[s], (i / C::STAGES) & 1)) {
                    ok = false;
                    break;
                }
                tc_fence_after();
                const uint32_t aaddr = smem_u32(stage_base + s * C::STAGE);
                const uint32_t baddr = aaddr + NA * C::A_PLANE;
#pragma unroll
                for (int k = 0; k < BK / 16; ++k) {
                    const uint64_t ah = sdesc_k_sw128(aaddr + k * 32);
                    const uint64_t bh = sdesc_k_sw128(baddr + k * 32);
                    umma_f16(tmem, ah, bh, idesc, (i > 0 || k > 0) ? 1u : 0u);
                    if (NB == 2) umma_f16(tmem, ah, sdesc_k_sw128(baddr + C::B_PLANE + k * 32), idesc, 1u);
                    if (NA == 2) umma_f16(tmem, sdesc_k_sw128(aaddr + C::A_PLANE + k * 32), bh, idesc, 1u);
                }
                umma_commit(&empty[s]);
            }
            if (ok) {
                umma_commit(done);
            } else {
                atomicExch(s_abort, 1);
                set_status(a.status, MSC_DEV_TIMEOUT);
                mbar_arrive(done);  // release the epilogue
            }
        }
    }

    // -------------------------------------------------------------- epilogue
    if (tid < kProducerThreads) {
        const bool ok = mbar_wait(done, 0);
        if (!ok) set_status(a.status, MSC_DEV_TIMEOUT);
        tc_fence_after();
        __syncwarp();
        const bool valid = __all_sync(0xffffffffu, ok && *reinterpret_cast<volatile int*>(s_abort) == 0);
        const int64_t row = row0 + tid;
        const auto* hdr = static_cast<const WeightHeader*>(a.blob);
        const float oscale = hdr->oscale;
#pragma unroll 1
        for (int c0 = 0; c0 < COUT; c0 += 32) {
            uint32_t acc[32];
            if (nst > 0 && valid) {
                tmem_ld32(tmem + (static_cast<uint32_t>(warp * 32) << 16) + c0, acc);
                tmem_wait_ld();
            } else {
#pragma unroll
                for (int k = 0; k < 32; ++k) acc[k] = 0u;
            }
            if (row < n && valid) {
                float v[32];
#pragma unroll
                for (int k = 0; k < 32; ++k) {
                    float t = __uint_as_float(acc[k]) * oscale;
                    if (a.bias) t += __ldg(a.bias + c0 + k);
                    if (a.silu_out) t = silu_f(t);
                    if (a.residual) t += load_elem(a.residual, a.res_dtype, row * COUT + c0 + k);
                    v[k] = t;
                }
                if (a.y_dtype == DT_F32) {
                    float4* dst = reinterpret_cast<float4*>(static_cast<float*>(a.y) + row * COUT + c0);
#pragma unroll
                    for (int k = 0; k < 8; ++k) dst[k] = make_float4(v[4 * k], v[4 * k + 1], v[4 * k + 2], v[4 * k + 3]);
                } else if (a.y_dtype == DT_F16) {
                    uint4* dst = reinterpret_cast<uint4*>(static_cast<__half*>(a.y) + row * COUT + c0);
#pragma unroll
                    for (int k = 0; k < 4; ++k) {
                        uint4 u;
                        __half2 h0 = __floats2half2_rn(v[8 * k], v[8 * k + 1]);
                        __half2 h1 = __floats2half2_rn(v[8 * k + 2], v[8 * k + 3]);
                        __half2 h2 = __floats2half2_rn(v[8 * k + 4], v[8 * k + 5]);
                        __half2 h3 = __floats2half2_rn(v[8 * k + 6], v[8 * k + 7]);
                        u.x = *reinterpret_cast<uint32_t*>(&h0);
                        u.y = *reinterpret_cast<uint32_t*>(&h1);
                        u.z = *reinterpret_cast<uint32_t*>(&h2);
                        u.w = *reinterpret_cast<uint32_t*>(&h3);
                        dst[k] = u;
                    }
                } else {
                    uint4* dst = reinterpret_cast<uint4*>(static_cast<__nv_bfloat16*>(a.y) + row * COUT + c0);
#pragma unroll
                    for (int k = 0; k < 4; ++k) {
                        uint4 u;
                        __nv_bfloat162 h0 = __floats2bfloat162_rn(v[8 * k], v[8 * k + 1]);
                        __nv_bfloat162 h1 = __floats2bfloat162_rn(v[8 * k + 2], v[8 * k + 3]);
                        __nv_bfloat162 h2 = __floats2bfloat162_rn(v[8 * k + 4], v[8 * k + 5]);
                        __nv_bfloat162 h3 = __floats2bfloat162_rn(v[8 * k + 6], v[8 * k + 7]);
                        u.x = *reinterpret_cast<uint32_t*>(&h0);
                        u.y = *reinterpret_cast<uint32_t*>(&h1);
                        u.z = *reinterpret_cast<uint32_t*>(&h2);
                        u.w = *reinterpret_cast<uint32_t*>(&h3);
                        dst[k] = u;
                    }
                }
            }
        }
    }
    tc_fence_before();
    __syncthreads();
    if (warp == 4) {
        tc_fence_after();
        tmem_dealloc(tmem, C::TMEM_COLS);
    }
}

template <int CIN, int COUT, int NA, int NB>
cudaError_t launch_t(const ConvArgs& a, cudaStream_t st) {
    using C = Cfg<CIN, COUT, NA, NB>;
    auto kern = conv_tc_kernel<CIN, COUT, NA, NB>;
    static bool configured = false;
    if (!configured) {
        cudaError_t e = cudaFuncSetAttribute(kern, cudaFuncAttributeMaxDynamicSharedMemorySize, C::SMEM);
        if (e != cudaSuccess) return e;
        configured = true;
    }
    const unsigned grid = static_cast<unsigned>((a.n + BM - 1) / BM);
    kern<<<grid, kThreads, C::SMEM, st>>>(a);
    return cudaGetLastError();
}

template <int CIN, int COUT>
cudaError_t launch_planes(const ConvArgs& a, cudaStream_t st) {
    if (a.na == 1 && a.wplanes == 1) return launch_t<CIN, COUT, 1, 1>(a, st);
    if (a.na == 1 && a.wplanes == 2) return launch_t<CIN, COUT, 1, 2>(a, st);
    if (a.na == 2 && a.wplanes == 1) return launch_t<CIN, COUT, 2, 1>(a, st);
    if (a.na == 2 && a.wplanes == 2) return launch_t<CIN, COUT, 2, 2>(a, st);
    return cudaErrorInvalidValue;
}

}  // namespace

bool conv_supported(int cin, int cout) {
    return (cin == 64 || cin == 128) && (cout == 64 || cout == 128);
}

cudaError_t launch_conv(const ConvArgs& a, cudaStream_t st) {
    if (a.n == 0) return cudaSuccess;
    if (a.cin == 64 && a.cout == 64) return launch_planes<64, 64>(a, st);
    if (a.cin == 64 && a.cout == 128) return launch_planes<64, 128>(a, st);
    if (a.cin == 128 && a.cout == 64) return launch_planes<128, 64>(a, st);
    if (a.cin == 128 && a.cout == 128) return launch_planes<128, 128>(a, st);
    return cudaErrorInvalidValue;
}

}  // namespace msc
