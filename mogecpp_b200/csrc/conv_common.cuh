// Device helpers of the tensor-core conv kernel (conv_tc.cu): bounded waits,
// tap-order rotation and row loads / stores.
#pragma once

#include "common.cuh"
#include "conv.h"

namespace msc {

// Bounded wait that also gives up once another role has aborted.  Roles
// that run ahead of the pipeline's pace (the gather producers, the
// publisher) pass sleep_ns: between polls they yield their issue slots to
// the drain warps.
__device__ __forceinline__ bool wait_or_abort(uint64_t* bar, uint32_t parity, int* abort_flag, uint32_t* status,
                                              uint32_t sleep_ns = 0) {
    if (mbar_try_wait(bar, parity)) return true;
    const uint64_t t0 = global_timer_ns();
    for (uint32_t it = 0;; ++it) {
        if (sleep_ns) __nanosleep(sleep_ns);
        if (mbar_try_wait(bar, parity)) return true;
        if ((it & 31u) == 31u) {
            if (*reinterpret_cast<volatile int*>(abort_flag)) return false;
            if (global_timer_ns() - t0 > kWaitBudgetNs) {
                atomicExch(abort_flag, 1);
                set_status(status, MSC_DEV_TIMEOUT);
                return false;
            }
        }
    }
}

// One arrival per warp on a barrier that counts warps.  Arrivals from every
// lane of a CTA on one mbarrier serialise in shared memory (hundreds of
// cycles per phase at 512 threads); the warp sync orders the lanes' prior
// writes before the elected lane's arrive.
__device__ __forceinline__ void warp_arrive(uint64_t* bar) {
    const unsigned m = __activemask();
    __syncwarp(m);
    if (static_cast<int>(threadIdx.x & 31) == __ffs(m) - 1) mbar_arrive(bar);
}

// Taps are visited in ascending order in every tile.  A row's output is
// then the fp32 sum of its taps' block products in one fixed order, whatever
// tile the row lands in, so a tap-order plan, a different tiling or a z-slab
// split over GPUs gives bit-identical rows.  (Rotating the order per tile
// spreads the CTAs' requests for the same weight tile over time, but makes
// the rounding depend on the tile.)  rot_mask() / rot_tap() map the tile's
// mask to the visiting order and a visited bit back to its tap.
constexpr bool kRotateTaps = false;
__device__ __forceinline__ int tap_rotation(int64_t tile, int ntaps) {
    return (kRotateTaps && ntaps == 27) ? static_cast<int>(tile % 27) : 0;
}
__device__ __forceinline__ uint32_t rot_mask(uint32_t m, int r) {
    return r ? ((m >> r) | (m << (27 - r))) & 0x7ffffffu : m;
}
__device__ __forceinline__ int rot_tap(int bit, int r) {
    const int t = bit + r;
    return t >= 27 ? t - 27 : t;
}

__device__ __forceinline__ float load_elem(const void* p, int dtype, int64_t idx) {
    if (dtype == DT_F32) return static_cast<const float*>(p)[idx];
    if (dtype == DT_F16) return __half2float(static_cast<const __half*>(p)[idx]);
    return __bfloat162float(static_cast<const __nv_bfloat16*>(p)[idx]);
}

// N consecutive elements (N a multiple of 8, off a multiple of 8) as floats,
// in 16-byte loads.
template <int N>
__device__ __forceinline__ void load_row_vec(const void* p, int dtype, int64_t off, float (&v)[N]) {
    if (dtype == DT_F32) {
        const float4* src = reinterpret_cast<const float4*>(static_cast<const float*>(p) + off);
#pragma unroll
        for (int k = 0; k < N / 4; ++k) {
            const float4 t = src[k];
            v[4 * k] = t.x, v[4 * k + 1] = t.y, v[4 * k + 2] = t.z, v[4 * k + 3] = t.w;
        }
    } else {
        const uint4* src = reinterpret_cast<const uint4*>(static_cast<const __half*>(p) + off);
#pragma unroll
        for (int k = 0; k < N / 8; ++k) {
            const uint4 t = src[k];
            const uint32_t w[4] = {t.x, t.y, t.z, t.w};
#pragma unroll
            for (int e = 0; e < 8; ++e) {
                const unsigned short b = static_cast<unsigned short>(w[e / 2] >> (16 * (e & 1)));
                v[8 * k + e] = dtype == DT_F16 ? __half2float(__ushort_as_half(b))
                                               : __bfloat162float(__ushort_as_bfloat16(b));
            }
        }
    }
}

// 4 x 4 transpose of 16-byte chunks within each quad of lanes (4r..4r+3):
// afterwards lane 4r+k holds in e[j] what lane 4r+j held in e[k].  Two
// butterfly exchanges (lane bit 1, then lane bit 0), each moving the two
// chunks whose index bit differs from the lane's.  All 32 lanes take part.
__device__ __forceinline__ void quad_transpose(uint4 (&e)[4]) {
    const int l = static_cast<int>(threadIdx.x & 3);
#pragma unroll
    for (int mask = 2; mask >= 1; mask >>= 1) {
        const bool up = (l & mask) != 0;
#pragma unroll
        for (int t = 0; t < 2; ++t) {
            const int lo = mask == 2 ? t : 2 * t;
            const int hi = lo + mask;
            uint4 v = up ? e[lo] : e[hi];
            v.x = __shfl_xor_sync(0xffffffffu, v.x, mask);
            v.y = __shfl_xor_sync(0xffffffffu, v.y, mask);
            v.z = __shfl_xor_sync(0xffffffffu, v.z, mask);
            v.w = __shfl_xor_sync(0xffffffffu, v.w, mask);
            if (up)
                e[lo] = v;
            else
                e[hi] = v;
        }
    }
}

// 2 x 2 transpose of 16-byte chunks within each pair of lanes (2r, 2r+1):
// afterwards lane 2r+k holds in e[j] what lane 2r+j held in e[k].
__device__ __forceinline__ void pair_transpose(uint4 (&e)[2]) {
    const bool up = (threadIdx.x & 1) != 0;
    uint4 v = up ? e[0] : e[1];
    v.x = __shfl_xor_sync(0xffffffffu, v.x, 1);
    v.y = __shfl_xor_sync(0xffffffffu, v.y, 1);
    v.z = __shfl_xor_sync(0xffffffffu, v.z, 1);
    v.w = __shfl_xor_sync(0xffffffffu, v.w, 1);
    if (up)
        e[0] = v;
    else
        e[1] = v;
}

__device__ __forceinline__ void prefetch_l2(const void* p) {
    asm volatile("prefetch.global.L2 [%0];" ::"l"(p));
}

template <int N>
__device__ __forceinline__ void store_row(void* y, int dtype, int64_t off, const float (&v)[N]) {
    if (dtype == DT_F32) {
        float4* dst = reinterpret_cast<float4*>(static_cast<float*>(y) + off);
#pragma unroll
        for (int k = 0; k < N / 4; ++k) dst[k] = make_float4(v[4 * k], v[4 * k + 1], v[4 * k + 2], v[4 * k + 3]);
    } else if (dtype == DT_F16) {
        uint4* dst = reinterpret_cast<uint4*>(static_cast<__half*>(y) + off);
#pragma unroll
        for (int k = 0; k < N / 8; ++k) {
            __half2 h[4];
#pragma unroll
            for (int e = 0; e < 4; ++e) h[e] = __floats2half2_rn(v[8 * k + 2 * e], v[8 * k + 2 * e + 1]);
            dst[k] = *reinterpret_cast<uint4*>(h);
        }
    } else {
        uint4* dst = reinterpret_cast<uint4*>(static_cast<__nv_bfloat16*>(y) + off);
#pragma unroll
        for (int k = 0; k < N / 8; ++k) {
            __nv_bfloat162 h[4];
#pragma unroll
            for (int e = 0; e < 4; ++e) h[e] = __floats2bfloat162_rn(v[8 * k + 2 * e], v[8 * k + 2 * e + 1]);
            dst[k] = *reinterpret_cast<uint4*>(h);
        }
    }
}

// Quantises one 32-channel block with ggml's x86 Q8_0 rules (d = amax/127,
// id = 127/amax, codes rounded half to even; quants.c:302), exactly as the
// ACT_Q8I activation preparation does: the 32 int8 codes packed into w, the
// scale fp32(fp16(d)) returned.
__device__ __forceinline__ float quantize_block32(const float (&v)[32], uint32_t (&w)[8]) {
    float amax = 0.0f;
#pragma unroll
    for (int e = 0; e < 32; ++e) amax = fmaxf(amax, fabsf(v[e]));
    const float d = __fdiv_rn(amax, 127.0f);
    const float id = amax != 0.0f ? __fdiv_rn(127.0f, amax) : 0.0f;
#pragma unroll
    for (int k = 0; k < 8; ++k)
        w[k] = pack_code_bytes(code_bits(v[4 * k], id), code_bits(v[4 * k + 1], id), code_bits(v[4 * k + 2], id),
                               code_bits(v[4 * k + 3], id));
    return __half2float(__float2half_rn(d));
}

// The same, storing the codes (16-byte aligned) and the scale.
__device__ __forceinline__ void quantize_store_block32(const float (&v)[32], int8_t* codes, float* scale) {
    uint32_t w[8];
    const float d = quantize_block32(v, w);
    reinterpret_cast<uint4*>(codes)[0] = make_uint4(w[0], w[1], w[2], w[3]);
    reinterpret_cast<uint4*>(codes)[1] = make_uint4(w[4], w[5], w[6], w[7]);
    *scale = d;
}

}  // namespace msc
