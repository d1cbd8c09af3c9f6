// Operand preparation for the tensor-core sparse conv:
//
//  * weights: packed [cout][ntaps*cin] (f32, f16 or ggml block_q8_0 rows) ->
//    blob of 128B-swizzled K-major fp16 tiles [tap][64-ch chunk][plane][cout][64].
//    f16 weights are one exact plane; f32 weights and Q8_0 weights with
//    cin = 64 (their exact dequantised value q * fp16(d)) become an exact
//    hi/lo pair after a power-of-two prescale that puts max|w| near 2^14
//    (undone in the conv epilogue); Q8_0 weights with cin = 128 keep their
//    int8 codes ([tap][cout][128] swizzled) plus fp32(fp16(d)) block scales.
//  * activations: [n][c] rows (f32/f16/bf16), optional LayerNorm + SiLU
//    (mogecpp src/sparse.cpp:520-526, ggml norm_f32 / silu), then
//      ACT_FP16  round to fp16                      (ggml F16 vec_dot_type)
//      ACT_SPLIT exact hi/lo fp16 pair of the fp32  (ggml F32 x F32)
//      ACT_Q8    ggml's x86 Q8_0 quantiser per 32 channels (d = amax/127,
//                id = 127/amax, round-half-even; ggml-cpu/arch/x86/quants.c:302):
//                the int8 codes as one fp16 plane (ACT_Q8I: as int8),
//                fp32(fp16(d)) per block after it (Q8_0 vec_dot_type)
#include "common.cuh"
#include "conv.h"

namespace msc {
namespace {

__host__ __device__ inline size_t scale_offset(int64_t n, int c) {
    return (static_cast<size_t>(n) * c * 2 + 255) / 256 * 256;
}

struct BlockQ8 {
    __half d;
    int8_t qs[32];
};
static_assert(sizeof(BlockQ8) == 34, "block_q8_0 is 34 bytes");

__device__ __forceinline__ float weight_value(int wtype, const void* w, int64_t row_len, int o, int64_t k) {
    if (wtype == WT_F32) return static_cast<const float*>(w)[o * row_len + k];
    if (wtype == WT_F16) return __half2float(static_cast<const __half*>(w)[o * row_len + k]);
    const BlockQ8* b = static_cast<const BlockQ8*>(w) + (o * row_len + k) / 32;
    return static_cast<float>(b->qs[k % 32]) * __half2float(b->d);
}

__global__ void weight_header_kernel(WeightHeader* h, int wtype, int cin, int cout, int ntaps, int planes) {
    h->magic = kWeightMagic;
    h->wtype = wtype;
    h->cin = cin;
    h->cout = cout;
    h->ntaps = ntaps;
    h->planes = planes;
    h->oscale = 1.0f;
    h->amax = 0.0f;
}

__global__ void weight_amax_kernel(WeightHeader* h, int wtype, const void* w, int64_t row_len, int cout) {
    float m = 0.0f;
    const int64_t total = row_len * cout;
    for (int64_t i = blockIdx.x * static_cast<int64_t>(blockDim.x) + threadIdx.x; i < total;
         i += static_cast<int64_t>(gridDim.x) * blockDim.x)
        m = fmaxf(m, fabsf(weight_value(wtype, w, row_len, static_cast<int>(i / row_len), i % row_len)));
    for (int o = 16; o > 0; o >>= 1) m = fmaxf(m, __shfl_xor_sync(0xffffffffu, m, o));
    if ((threadIdx.x & 31) == 0) atomicMax(reinterpret_cast<unsigned*>(&h->amax), __float_as_uint(m));
}

__device__ __forceinline__ int prescale_exp(float amax) {
    if (!(amax > 0.0f)) return 0;
    int e;
    frexpf(amax, &e);  // amax = f * 2^e, f in [0.5, 1)
    return 14 - e;     // amax * 2^s in [2^13, 2^14)
}

__global__ void weight_split_kernel(WeightHeader* h, int wtype, const void* w, int cin, int cout, int ntaps,
                                    int planes, uint8_t* out) {
    const int64_t row_len = static_cast<int64_t>(ntaps) * cin;
    const int64_t total = row_len * cout;
    const int s = planes == 2 ? prescale_exp(h->amax) : 0;
    const int kch = cin / 64;
    for (int64_t i = blockIdx.x * static_cast<int64_t>(blockDim.x) + threadIdx.x; i < total;
         i += static_cast<int64_t>(gridDim.x) * blockDim.x) {
        const int o = static_cast<int>(i / row_len);
        const int64_t k = i % row_len;
        const int t = static_cast<int>(k / cin);
        const int ci = static_cast<int>(k % cin);
        const int kc = ci / 64, e = ci % 64;
        __half hi, lo;
        const float v = ldexpf(weight_value(wtype, w, row_len, o, k), s);
        if (planes == 2) {
            split_f16(v, hi, lo);
        } else {
            hi = __float2half_rn(v);
            lo = __float2half_rn(0.0f);
        }
        const int64_t tile = static_cast<int64_t>(t * kch + kc) * planes;
        const uint32_t off = sw128_offset(o, e >> 3) + (e & 7) * 2;
        *reinterpret_cast<__half*>(out + (tile + 0) * cout * 128 + off) = hi;
        if (planes == 2) *reinterpret_cast<__half*>(out + (tile + 1) * cout * 128 + off) = lo;
    }
    if (blockIdx.x == 0 && threadIdx.x == 0) h->oscale = ldexpf(1.0f, -s);
}

// Q8_0 weights for the kind::i8 path: int8 codes into 128-byte swizzled rows
// (one tile of cout rows per tap), block scales as fp32 [tap][block][cout].
__global__ void weight_q8i_kernel(const BlockQ8* w, int cin, int cout, int ntaps, uint8_t* out) {
    const int64_t nblocks = static_cast<int64_t>(cout) * ntaps * (cin / 32);
    int8_t* codes = reinterpret_cast<int8_t*>(out);
    float* scales = reinterpret_cast<float*>(out + static_cast<int64_t>(ntaps) * cout * cin);
    for (int64_t bi = blockIdx.x * static_cast<int64_t>(blockDim.x) + threadIdx.x; bi < nblocks;
         bi += static_cast<int64_t>(gridDim.x) * blockDim.x) {
        const int64_t per_row = static_cast<int64_t>(ntaps) * (cin / 32);
        const int o = static_cast<int>(bi / per_row);
        const int64_t rb = bi % per_row;               // block within the packed row
        const int t = static_cast<int>(rb / (cin / 32));
        const int b = static_cast<int>(rb % (cin / 32));
        const BlockQ8 blk = w[bi];
        int8_t* tile = codes + static_cast<int64_t>(t) * cout * cin;
#pragma unroll
        for (int e = 0; e < 32; ++e) {
            const int ci = b * 32 + e;
            tile[sw128_offset(o, ci >> 4) + (ci & 15)] = blk.qs[e];
        }
        scales[(static_cast<int64_t>(t) * (cin / 32) + b) * cout + o] = __half2float(blk.d);
    }
}

// EPL consecutive 32-bit words <-> memory at p, in the widest aligned
// accesses (the row part of a lane is EPL elements at an EPL-aligned offset).
template <int NW>
__device__ __forceinline__ void load_words(const void* p, uint32_t (&w)[NW]) {
    if constexpr (NW % 4 == 0) {
#pragma unroll
        for (int k = 0; k < NW / 4; ++k) {
            const uint4 t = reinterpret_cast<const uint4*>(p)[k];
            w[4 * k] = t.x, w[4 * k + 1] = t.y, w[4 * k + 2] = t.z, w[4 * k + 3] = t.w;
        }
    } else if constexpr (NW == 2) {
        const uint2 t = *reinterpret_cast<const uint2*>(p);
        w[0] = t.x, w[1] = t.y;
    } else {
        w[0] = *reinterpret_cast<const uint32_t*>(p);
    }
}
template <int NW>
__device__ __forceinline__ void store_words(void* p, const uint32_t (&w)[NW]) {
    if constexpr (NW % 4 == 0) {
#pragma unroll
        for (int k = 0; k < NW / 4; ++k)
            reinterpret_cast<uint4*>(p)[k] = make_uint4(w[4 * k], w[4 * k + 1], w[4 * k + 2], w[4 * k + 3]);
    } else if constexpr (NW == 2) {
        *reinterpret_cast<uint2*>(p) = make_uint2(w[0], w[1]);
    } else {
        *reinterpret_cast<uint32_t*>(p) = w[0];
    }
}

// EPL fp16 values as half-words: vector stores when EPL >= 2.
template <int EPL>
__device__ __forceinline__ void store_halves(__half* dst, const __half (&h)[EPL]) {
    if constexpr (EPL >= 2) {
        uint32_t w[EPL / 2];
#pragma unroll
        for (int k = 0; k < EPL / 2; ++k)
            w[k] = static_cast<uint32_t>(__half_as_ushort(h[2 * k])) |
                   (static_cast<uint32_t>(__half_as_ushort(h[2 * k + 1])) << 16);
        store_words<EPL / 2>(dst, w);
    } else {
        dst[0] = h[0];
    }
}

// Rows are prepared by 8-lane groups (4 rows per warp instruction): lane j
// of a row's group holds channels [j*EPL, (j+1)*EPL), EPL = C/8, read and
// written with vector accesses; row reductions take 3 shuffle steps and a
// row's scalar work is shared by 4 rows per instruction.
constexpr int kLanesPerRow = 8;
constexpr int kPrepIters = 2;  // row groups per warp, all loads issued first

template <int C>
__device__ __forceinline__ void load_row8(const void* x, int x_dtype, int64_t row, int j, float (&v)[C / 8]) {
    constexpr int EPL = C / 8;
    const int64_t base = row * C + j * EPL;
    if (x_dtype == DT_F32) {
        uint32_t w[EPL];
        load_words<EPL>(static_cast<const float*>(x) + base, w);
#pragma unroll
        for (int k = 0; k < EPL; ++k) v[k] = __uint_as_float(w[k]);
    } else {
        uint32_t w[EPL / 2];
        load_words<EPL / 2>(static_cast<const __half*>(x) + base, w);
#pragma unroll
        for (int k = 0; k < EPL; ++k) {
            const unsigned short b = static_cast<unsigned short>(w[k / 2] >> (16 * (k & 1)));
            v[k] = x_dtype == DT_F16 ? __half2float(__ushort_as_half(b)) : __bfloat162float(__ushort_as_bfloat16(b));
        }
    }
}

// sum over the 8 lanes of a row group
__device__ __forceinline__ float row_sum8(float s) {
#pragma unroll
    for (int o = 4; o > 0; o >>= 1) s += __shfl_xor_sync(0xffffffffu, s, o);
    return s;
}

// Normalisation, SiLU and the operand output of one row; all 32 lanes call
// it (the shuffles need them), `valid` gates the stores.
// The affine weights of the normalisation, per row-group lane j: its EPL
// channels at j * (EPL + 4) floats in shared memory (the 4-float pad puts
// the 8 lanes' 16-byte reads in distinct banks).
template <int C>
struct Affine {
    static constexpr int EPL = C / 8;
    static constexpr int STRIDE = EPL + 4;
    const float* g;  // this lane's gamma (nullptr: none)
    const float* b;  // this lane's beta (nullptr: none)
    // channels (2k, 2k + 1) as an f32x2 pair
    __device__ __forceinline__ uint64_t gamma2(int k) const { return reinterpret_cast<const uint64_t*>(g)[k]; }
    __device__ __forceinline__ uint64_t beta2(int k) const { return reinterpret_cast<const uint64_t*>(b)[k]; }
};

template <int C>
__device__ __forceinline__ void prepare_row8(float (&v)[C / 8], int64_t row, bool valid, int j, int64_t n, int ln,
                                             const Affine<C>& aff, float eps, int silu, int mode,
                                             __half* planes, const float2* gn, const int4* coords, int nsamples) {
    constexpr int EPL = C / 8;
    constexpr int CPG = C / 32;  // channels per GroupNorm group
    const int64_t base = row * C + j * EPL;
    // the row part as f32x2 pairs (channels 2k, 2k + 1)
    uint64_t p[EPL / 2];
#pragma unroll
    for (int k = 0; k < EPL / 2; ++k) p[k] = pack2(v[2 * k], v[2 * k + 1]);
    if (gn) {
        // GroupNorm, 32 groups: ggml order ((x - mean) * scale, then * gamma,
        // then + beta); a lane holds EPL / CPG groups of CPG channels
        int b = valid ? __ldg(coords + row).w : 0;  // out-of-range samples are reported by the statistics pass
        b = b < 0 ? 0 : (b >= nsamples ? nsamples - 1 : b);
        constexpr int PPG = CPG >= 2 ? CPG / 2 : 1;  // pairs per group load
#pragma unroll
        for (int k0 = 0; k0 < EPL / 2; k0 += PPG) {
            // the pair's (or pairs') group statistics; with one channel per
            // group the two lanes of a pair have their own
            const float2 m0 = gn[b * 32 + (j * EPL + 2 * k0) / CPG];
            const float2 m1 = CPG >= 2 ? m0 : gn[b * 32 + (j * EPL + 2 * k0 + 1) / CPG];
            const uint64_t nm2 = pack2(-m0.x, -m1.x), sc2 = pack2(m0.y, m1.y);
#pragma unroll
            for (int k = k0; k < k0 + PPG; ++k) {
                uint64_t t = mul2(add2(p[k], nm2), sc2);
                if (aff.g) t = mul2(t, aff.gamma2(k));
                if (aff.b) t = add2(t, aff.beta2(k));
                p[k] = t;
            }
        }
    } else if (ln) {
        uint64_t s2 = p[0];
#pragma unroll
        for (int k = 1; k < EPL / 2; ++k) s2 = add2(s2, p[k]);
        float s0, s1;
        unpack2(s2, s0, s1);
        const float mean = row_sum8(s0 + s1) / C;
        const uint64_t nm2 = pack2(-mean, -mean);
        uint64_t q2 = 0ull;  // (+0, +0)
#pragma unroll
        for (int k = 0; k < EPL / 2; ++k) {
            p[k] = add2(p[k], nm2);  // x - mean
            q2 = fma2(p[k], p[k], q2);
        }
        float q0, q1;
        unpack2(q2, q0, q1);
        const float scale = 1.0f / sqrtf(row_sum8(q0 + q1) / C + eps);
        const uint64_t sc2 = pack2(scale, scale);
#pragma unroll
        for (int k = 0; k < EPL / 2; ++k) {
            uint64_t t = mul2(p[k], sc2);
            if (aff.g) t = mul2(t, aff.gamma2(k));
            if (aff.b) t = add2(t, aff.beta2(k));
            p[k] = t;
        }
    }
    if (silu) {
#pragma unroll
        for (int k = 0; k < EPL / 2; ++k) p[k] = silu2(p[k]);
    }
#pragma unroll
    for (int k = 0; k < EPL / 2; ++k) unpack2(p[k], v[2 * k], v[2 * k + 1]);
    const int64_t plane = n * C;
    if (mode == ACT_FP16) {
        __half h[EPL];
#pragma unroll
        for (int k = 0; k < EPL; ++k) h[k] = __float2half_rn(v[k]);
        if (valid) store_halves<EPL>(planes + base, h);
        return;
    }
    if (mode == ACT_Q8 || mode == ACT_Q8I) {
        // a 32-channel block spans LPB lanes of the row group
        constexpr int LPB = 32 / EPL > 0 ? 32 / EPL : 1;
        float amax = 0.0f;
#pragma unroll
        for (int k = 0; k < EPL; ++k) amax = fmaxf(amax, fabsf(v[k]));
#pragma unroll
        for (int o = 1; o < LPB; o <<= 1) amax = fmaxf(amax, __shfl_xor_sync(0xffffffffu, amax, o));
        const float d = __fdiv_rn(amax, 127.0f);
        const float id = amax != 0.0f ? __fdiv_rn(127.0f, amax) : 0.0f;
        if (!valid) return;
        if (mode == ACT_Q8I) {
            uint32_t w[EPL / 4];
#pragma unroll
            for (int k = 0; k < EPL / 4; ++k)
                w[k] = pack_code_bytes(code_bits(v[4 * k], id), code_bits(v[4 * k + 1], id),
                                       code_bits(v[4 * k + 2], id), code_bits(v[4 * k + 3], id));
            store_words<EPL / 4>(reinterpret_cast<int8_t*>(planes) + base, w);
        } else {
            __half h[EPL];
#pragma unroll
            for (int k = 0; k < EPL; ++k) h[k] = __int2half_rn(__float2int_rn(__fmul_rn(v[k], id)));
            store_halves<EPL>(planes + base, h);
        }
        if ((j * EPL) % 32 == 0) {
            float* scales = reinterpret_cast<float*>(reinterpret_cast<char*>(planes) +
                                                     scale_offset(n, mode == ACT_Q8I ? C / 2 : C));
            const float dh = __half2float(__float2half_rn(d));
#pragma unroll
            for (int bk = 0; bk < (EPL + 31) / 32; ++bk) scales[row * (C / 32) + (j * EPL) / 32 + bk] = dh;
        }
        return;
    }
    __half hi[EPL], lo[EPL];
#pragma unroll
    for (int k = 0; k < EPL; ++k) split_f16(v[k], hi[k], lo[k]);
    if (!valid) return;
    store_halves<EPL>(planes + base, hi);
    store_halves<EPL>(planes + plane + base, lo);
}

// 4 blocks of 256 per SM for C <= 128 (64 registers, half the warp slots
// resident: the loads of more rows in flight); C = 256 needs its registers
template <int C>
__global__ void __launch_bounds__(256, C <= 128 ? 4 : 1) act_prepare_kernel(const void* x, int x_dtype, int64_t n, int ln, const float* gamma,
                                   const float* beta, float eps, int silu, int mode, __half* planes,
                                   const float2* gn, const int4* coords, int nsamples) {
    // gamma / beta once per block into shared memory (a per-element global
    // load per row cost 32 L1 requests per lane and row)
    using A = Affine<C>;
    __shared__ __align__(16) float s_aff[2][8 * A::STRIDE];
    if (gamma || beta) {  // uniform over the block
        for (int e = threadIdx.x; e < C; e += blockDim.x) {
            const int jj = e / A::EPL, k = e % A::EPL;
            s_aff[0][jj * A::STRIDE + k] = gamma ? __ldg(gamma + e) : 1.0f;
            s_aff[1][jj * A::STRIDE + k] = beta ? __ldg(beta + e) : 0.0f;
        }
        __syncthreads();
    }
    const int64_t warp = (blockIdx.x * static_cast<int64_t>(blockDim.x) + threadIdx.x) >> 5;
    const int lane = threadIdx.x & 31;
    const int j = lane & (kLanesPerRow - 1);
    const int64_t r0 = warp * (4 * kPrepIters) + (lane >> 3);
    if (warp * (4 * kPrepIters) >= n) return;
    const A aff{gamma ? s_aff[0] + j * A::STRIDE : nullptr, beta ? s_aff[1] + j * A::STRIDE : nullptr};
    float v[kPrepIters][C / 8];
#pragma unroll
    for (int it = 0; it < kPrepIters; ++it) {
        const int64_t row = r0 + 4 * it;
        if (row < n) {
            load_row8<C>(x, x_dtype, row, j, v[it]);
        } else {
#pragma unroll
            for (int k = 0; k < C / 8; ++k) v[it][k] = 0.0f;
        }
    }
#pragma unroll
    for (int it = 0; it < kPrepIters; ++it) {
        const int64_t row = r0 + 4 * it;
        prepare_row8<C>(v[it], row, row < n, j, n, ln, aff, eps, silu, mode, planes, gn, coords, nsamples);
    }
}

}  // namespace

bool weight_is_i8(int wtype, int cin) { return wtype == WT_Q8_0 && cin == 128; }

int weight_planes(int wtype, int cin) { return (wtype == WT_F16 || weight_is_i8(wtype, cin)) ? 1 : 2; }

size_t weight_blob_bytes(int wtype, int cin, int cout, int ntaps) {
    if (weight_is_i8(wtype, cin))
        return sizeof(WeightHeader) + static_cast<size_t>(ntaps) * cin * cout +
               static_cast<size_t>(ntaps) * (cin / 32) * cout * 4;
    return sizeof(WeightHeader) + static_cast<size_t>(weight_planes(wtype, cin)) * ntaps * cin * cout * 2;
}

cudaError_t launch_weight_prepare(int wtype, const void* w, int cin, int cout, int ntaps, void* blob,
                                  cudaStream_t st) {
    auto* h = static_cast<WeightHeader*>(blob);
    const int planes = weight_planes(wtype, cin);
    const int64_t row_len = static_cast<int64_t>(ntaps) * cin;
    weight_header_kernel<<<1, 1, 0, st>>>(h, wtype, cin, cout, ntaps, planes);
    if (weight_is_i8(wtype, cin)) {
        const int64_t nblocks = row_len / 32 * cout;
        const unsigned grid = static_cast<unsigned>(std::min<int64_t>((nblocks + 255) / 256, 148 * 16));
        weight_q8i_kernel<<<grid, 256, 0, st>>>(static_cast<const BlockQ8*>(w), cin, cout, ntaps,
                                                static_cast<uint8_t*>(blob) + sizeof(WeightHeader));
        return cudaGetLastError();
    }
    if (planes == 2) weight_amax_kernel<<<148, 256, 0, st>>>(h, wtype, w, row_len, cout);
    const int64_t total = row_len * cout;
    const unsigned grid = static_cast<unsigned>(std::min<int64_t>((total + 255) / 256, 148 * 16));
    weight_split_kernel<<<grid, 256, 0, st>>>(h, wtype, w, cin, cout, ntaps, planes,
                                              static_cast<uint8_t*>(blob) + sizeof(WeightHeader));
    return cudaGetLastError();
}

int act_planes(int mode) { return mode == ACT_SPLIT ? 2 : 1; }

size_t act_scale_offset(int mode, int64_t n, int c) { return scale_offset(n, mode == ACT_Q8I ? c / 2 : c); }

size_t act_bytes(int mode, int64_t n, int c) {
    if (mode == ACT_Q8 || mode == ACT_Q8I)
        return act_scale_offset(mode, n, c) + static_cast<size_t>(n) * (c / 32) * 4;
    return static_cast<size_t>(act_planes(mode)) * n * c * 2;
}

cudaError_t launch_act_prepare(const void* x, int x_dtype, int64_t n, int c, int ln, const float* gamma,
                               const float* beta, float eps, int silu, int mode, void* planes, cudaStream_t st,
                               const float2* gn, const int32_t* coords, int nsamples) {
    if (n == 0) return cudaSuccess;
    const int64_t warps = (n + 4 * kPrepIters - 1) / (4 * kPrepIters);
    const unsigned grid = static_cast<unsigned>((warps * 32 + 255) / 256);
    auto* out = static_cast<__half*>(planes);
    const int4* c4 = reinterpret_cast<const int4*>(coords);
    if (gn && (c % 32 != 0 || !coords || nsamples < 1)) return cudaErrorInvalidValue;
    switch (c) {
        case 32: act_prepare_kernel<32><<<grid, 256, 0, st>>>(x, x_dtype, n, ln, gamma, beta, eps, silu, mode, out, gn, c4, nsamples); break;
        case 64: act_prepare_kernel<64><<<grid, 256, 0, st>>>(x, x_dtype, n, ln, gamma, beta, eps, silu, mode, out, gn, c4, nsamples); break;
        case 128: act_prepare_kernel<128><<<grid, 256, 0, st>>>(x, x_dtype, n, ln, gamma, beta, eps, silu, mode, out, gn, c4, nsamples); break;
        case 256: act_prepare_kernel<256><<<grid, 256, 0, st>>>(x, x_dtype, n, ln, gamma, beta, eps, silu, mode, out, gn, c4, nsamples); break;
        default: return cudaErrorInvalidValue;
    }
    return cudaGetLastError();
}

}  // namespace msc
