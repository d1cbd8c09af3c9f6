/* CPU oracle for the sparse-voxel hot path (test infrastructure only; see
 * oracle.h).  Each function cites the reference code it restates; paths are
 * relative to the mogecpp tree and its vendored ggml-0.25.3.
 */
#include "oracle.h"

#include <math.h>
#include <stdlib.h>
#include <string.h>

/* ------------------------------------------------------------ half floats */

/* IEEE binary16, round to nearest even (matches F16C vcvtps2ph and
 * ggml's software GGML_FP32_TO_FP16, ggml-impl.h). */
uint16_t orc_fp32_to_fp16(float f) {
    uint32_t x;
    memcpy(&x, &f, 4);
    const uint32_t sign = (x >> 16) & 0x8000u;
    uint32_t mag = x & 0x7fffffffu;
    if (mag >= 0x7f800000u) return (uint16_t)(sign | (mag > 0x7f800000u ? 0x7e00u : 0x7c00u));
    if (mag >= 0x477ff000u) return (uint16_t)(sign | 0x7c00u); /* rounds to >= 65520 -> inf */
    if (mag < 0x38800000u) {                                    /* result subnormal or zero */
        if (mag < 0x33000000u) return (uint16_t)sign;           /* < 2^-25: rounds to 0 */
        const uint32_t e = mag >> 23;
        const uint32_t m = (mag & 0x7fffffu) | 0x800000u;
        const uint32_t shift = 126u - e; /* value = m * 2^(e-150); target unit 2^-24 */
        uint32_t q = m >> shift;
        const uint32_t rem = m & ((1u << shift) - 1u);
        const uint32_t half = 1u << (shift - 1u);
        if (rem > half || (rem == half && (q & 1u))) ++q;
        return (uint16_t)(sign | q);
    }
    uint32_t h = ((mag >> 13) - (112u << 10));
    const uint32_t rem = mag & 0x1fffu;
    if (rem > 0x1000u || (rem == 0x1000u && (h & 1u))) ++h;
    return (uint16_t)(sign | h);
}

float orc_fp16_to_fp32(uint16_t h) {
    const uint32_t sign = (uint32_t)(h & 0x8000u) << 16;
    const uint32_t e = (h >> 10) & 0x1fu;
    const uint32_t m = h & 0x3ffu;
    uint32_t x;
    if (e == 0) {
        if (m == 0) {
            x = sign;
        } else {
            float v = ldexpf((float)m, -24);
            memcpy(&x, &v, 4);
            x |= sign;
        }
    } else if (e == 31) {
        x = sign | 0x7f800000u | (m << 13);
    } else {
        x = sign | ((e + 112u) << 23) | (m << 13);
    }
    float f;
    memcpy(&f, &x, 4);
    return f;
}

uint16_t orc_fp32_to_bf16(float f) {
    uint32_t x;
    memcpy(&x, &f, 4);
    if ((x & 0x7fffffffu) > 0x7f800000u) return (uint16_t)((x >> 16) | 0x40u);
    x += 0x7fffu + ((x >> 16) & 1u);
    return (uint16_t)(x >> 16);
}

float orc_bf16_to_fp32(uint16_t h) {
    uint32_t x = (uint32_t)h << 16;
    float f;
    memcpy(&f, &x, 4);
    return f;
}

/* --------------------------------------------------------------- Q8_0 */

/* ggml-quants.c:274-296 quantize_row_q8_0_ref: d = amax/127, id = 1/d,
 * q = roundf(x*id) (half away from zero); d stored as fp16. */
void orc_quantize_q8_0_ref(const float *x, orc_block_q8_0 *y, int64_t k) {
    const int64_t nb = k / 32;
    for (int64_t i = 0; i < nb; ++i) {
        float amax = 0.0f;
        for (int j = 0; j < 32; ++j) {
            const float v = fabsf(x[i * 32 + j]);
            amax = v > amax ? v : amax;
        }
        const float d = amax / 127.0f;
        const float id = d != 0.0f ? 1.0f / d : 0.0f;
        y[i].d = orc_fp32_to_fp16(d);
        for (int j = 0; j < 32; ++j) y[i].qs[j] = (int8_t)roundf(x[i * 32 + j] * id);
    }
}

/* ggml-cpu/arch/x86/quants.c:302-350 quantize_row_q8_0 (AVX2 path, the one
 * ggml's mul_mat uses for Q8_0 vec_dot_type): d = amax/127,
 * id = 127/amax, q = nearbyint(x*id) (round half to even). */
void orc_quantize_q8_0_act(const float *x, orc_block_q8_0 *y, int64_t k) {
    const int64_t nb = k / 32;
    for (int64_t i = 0; i < nb; ++i) {
        float amax = 0.0f;
        for (int j = 0; j < 32; ++j) {
            const float v = fabsf(x[i * 32 + j]);
            amax = v > amax ? v : amax;
        }
        const float d = amax / 127.0f;
        const float id = amax != 0.0f ? 127.0f / amax : 0.0f;
        y[i].d = orc_fp32_to_fp16(d);
        for (int j = 0; j < 32; ++j) y[i].qs[j] = (int8_t)nearbyintf(x[i * 32 + j] * id);
    }
}

/* ------------------------------------------------------------- topology */

/* Open-addressing map from packed voxel key to the first index inserted,
 * the semantics of FlatCoordMap::emplace/find (src/sparse.cpp:91-130).  The
 * probe sequence differs from the reference's; the mapping does not. */
typedef struct {
    uint64_t *keys;
    int32_t *vals;
    uint64_t mask;
} orc_map;

static const uint64_t ORC_EMPTY = ~(uint64_t)0;

static uint64_t orc_mix(uint64_t k) {
    k ^= k >> 31;
    k *= 0x7fb5d329728ea185ull;
    k ^= k >> 27;
    k *= 0x81dadef4bc2dd44dull;
    k ^= k >> 33;
    return k;
}

static int orc_map_init(orc_map *m, int64_t expected) {
    uint64_t cap = 16;
    while (cap < (uint64_t)(expected * 2)) cap <<= 1;
    m->keys = (uint64_t *)malloc(cap * sizeof(uint64_t));
    m->vals = (int32_t *)malloc(cap * sizeof(int32_t));
    if (!m->keys || !m->vals) return -1;
    for (uint64_t i = 0; i < cap; ++i) m->keys[i] = ORC_EMPTY;
    m->mask = cap - 1;
    return 0;
}

static void orc_map_free(orc_map *m) {
    free(m->keys);
    free(m->vals);
}

/* returns the stored value (existing or new) */
static int32_t orc_map_emplace(orc_map *m, uint64_t key, int32_t val) {
    uint64_t s = orc_mix(key) & m->mask;
    for (;;) {
        if (m->keys[s] == ORC_EMPTY) {
            m->keys[s] = key;
            m->vals[s] = val;
            return val;
        }
        if (m->keys[s] == key) return m->vals[s];
        s = (s + 1) & m->mask;
    }
}

static int32_t orc_map_find(const orc_map *m, uint64_t key) {
    uint64_t s = orc_mix(key) & m->mask;
    for (;;) {
        if (m->keys[s] == ORC_EMPTY) return -1;
        if (m->keys[s] == key) return m->vals[s];
        s = (s + 1) & m->mask;
    }
}

#define ORC_AXIS_MAX ((1 << 19) - 1)

static int orc_valid(const int32_t *c) {
    return c[0] >= 0 && c[0] <= ORC_AXIS_MAX && c[1] >= 0 && c[1] <= ORC_AXIS_MAX && c[2] >= 0 &&
           c[2] <= ORC_AXIS_MAX && c[3] >= 0 && c[3] < 127;
}

static uint64_t orc_key(int32_t x, int32_t y, int32_t z, int32_t b) {
    return ((uint64_t)b << 57) | ((uint64_t)z << 38) | ((uint64_t)y << 19) | (uint64_t)x;
}

/* src/sparse.cpp:238-272 make_level: taps v = (dx+1)*9 + (dy+1)*3 + (dz+1),
 * dx on x (row), dz fastest; missing neighbour = n. */
int orc_make_level(const int32_t *coords, int32_t n, int32_t *nbr) {
    for (int32_t i = 0; i < n; ++i)
        if (!orc_valid(coords + 4 * i)) return -1;
    orc_map m;
    if (orc_map_init(&m, n) != 0) return -3;
    for (int32_t i = 0; i < n; ++i) {
        const int32_t *c = coords + 4 * i;
        orc_map_emplace(&m, orc_key(c[0], c[1], c[2], c[3]), i);
    }
    for (int32_t i = 0; i < n; ++i) {
        const int32_t *c = coords + 4 * i;
        int v = 0;
        for (int dx = -1; dx <= 1; ++dx)
            for (int dy = -1; dy <= 1; ++dy)
                for (int dz = -1; dz <= 1; ++dz, ++v) {
                    const int32_t qx = c[0] + dx, qy = c[1] + dy, qz = c[2] + dz;
                    int32_t found = n;
                    if (qx >= 0 && qy >= 0 && qz >= 0 && qx <= ORC_AXIS_MAX && qy <= ORC_AXIS_MAX &&
                        qz <= ORC_AXIS_MAX) {
                        const int32_t idx = orc_map_find(&m, orc_key(qx, qy, qz, c[3]));
                        if (idx >= 0) found = idx;
                    }
                    nbr[(int64_t)i * 27 + v] = found;
                }
    }
    orc_map_free(&m);
    return 0;
}

/* src/sparse.cpp:312-357 downsample (factor 2): parent = c/2, parents
 * numbered by first occurrence, slot = arrival rank of the child among its
 * siblings, pool_rows slot-major [8][np] with sentinel n, inv_count =
 * 1/count, up_rows = fine -> parent. */
int orc_downsample(const int32_t *coords, int32_t n, int32_t *parent, int32_t *np_out, int32_t *pool_rows,
                   float *inv_count, int32_t *up_rows) {
    for (int32_t i = 0; i < n; ++i)
        if (!orc_valid(coords + 4 * i)) return -1;
    orc_map m;
    if (orc_map_init(&m, n) != 0) return -3;
    int32_t *counts = (int32_t *)calloc((size_t)(n > 0 ? n : 1), sizeof(int32_t));
    int32_t np = 0;
    for (int32_t i = 0; i < n; ++i) {
        const int32_t *c = coords + 4 * i;
        const int32_t px = c[0] / 2, py = c[1] / 2, pz = c[2] / 2;
        const int32_t pi = orc_map_emplace(&m, orc_key(px, py, pz, c[3]), np);
        if (pi == np) {
            parent[4 * np] = px;
            parent[4 * np + 1] = py;
            parent[4 * np + 2] = pz;
            parent[4 * np + 3] = c[3];
            ++np;
        }
        up_rows[i] = pi;
        ++counts[pi];
    }
    int rc = 0;
    for (int32_t p = 0; p < np; ++p) {
        if (counts[p] <= 0 || counts[p] > 8) rc = -2;
        inv_count[p] = 1.0f / (float)counts[p];
    }
    for (int64_t s = 0; s < (int64_t)8 * np; ++s) pool_rows[s] = n;
    memset(counts, 0, sizeof(int32_t) * (size_t)(n > 0 ? n : 1));
    for (int32_t i = 0; i < n && rc == 0; ++i) {
        const int32_t pi = up_rows[i];
        const int32_t slot = counts[pi]++;
        pool_rows[(int64_t)slot * np + pi] = i;
    }
    *np_out = np;
    free(counts);
    orc_map_free(&m);
    return rc;
}

/* ---------------------------------------------------------- dot products */

/* Dot of one output row of packed weight `w` (row o, length k) with the
 * activation vector a (length k, contiguous per the gather), by ggml
 * mul_mat semantics for the weight type (ggml-cpu.c:215-280 vec_dot_type):
 *   F32  : fp32 * fp32
 *   F16  : fp16(a) * fp16 w (products exact, fp32/double accumulation)
 *   Q8_0 : sum_b fp16(da)*fp16(dw) * isum_b (x86 quants.c:1308) */
typedef struct {
    int wtype;
    int k;
    const float *wf;
    const uint16_t *wh;
    const orc_block_q8_0 *wq;
} orc_wview;

static orc_wview orc_view(int wtype, const void *w, int k) {
    orc_wview v;
    v.wtype = wtype;
    v.k = k;
    v.wf = (const float *)w;
    v.wh = (const uint16_t *)w;
    v.wq = (const orc_block_q8_0 *)w;
    return v;
}

/* a is prepared per wtype: F32/F16 -> float array (already fp16-rounded for
 * F16); Q8_0 -> block array */
static double orc_dot_row(const orc_wview *v, int o, const float *af, const orc_block_q8_0 *aq) {
    double acc = 0.0;
    const int k = v->k;
    if (v->wtype == ORC_W_F32) {
        const float *wr = v->wf + (int64_t)o * k;
        for (int j = 0; j < k; ++j) acc += (double)wr[j] * (double)af[j];
    } else if (v->wtype == ORC_W_F16) {
        const uint16_t *wr = v->wh + (int64_t)o * k;
        for (int j = 0; j < k; ++j) acc += (double)orc_fp16_to_fp32(wr[j]) * (double)af[j];
    } else {
        const orc_block_q8_0 *wr = v->wq + (int64_t)o * (k / 32);
        for (int b = 0; b < k / 32; ++b) {
            int32_t isum = 0;
            for (int j = 0; j < 32; ++j) isum += (int32_t)wr[b].qs[j] * (int32_t)aq[b].qs[j];
            const float d = orc_fp16_to_fp32(wr[b].d) * orc_fp16_to_fp32(aq[b].d);
            acc += (double)d * (double)isum;
        }
    }
    return acc;
}

/* Prepares activation vector (length k) for the weight type. */
static void orc_prep(int wtype, const float *src, int k, float *af, orc_block_q8_0 *aq) {
    if (wtype == ORC_W_F32) {
        memcpy(af, src, sizeof(float) * (size_t)k);
    } else if (wtype == ORC_W_F16) {
        for (int j = 0; j < k; ++j) af[j] = orc_fp16_to_fp32(orc_fp32_to_fp16(src[j]));
    } else {
        orc_quantize_q8_0_act(src, aq, k);
    }
}

/* src/sparse.cpp:579-627 sparse_conv: GET_ROWS of the 27 neighbour rows
 * (sentinel = appended zero row), MUL_MAT with the packed weight, + bias. */
void orc_sparse_conv(const float *x, int64_t n, int cin, const int32_t *nbr, int wtype, const void *w, int cout,
                     const float *bias, float *y) {
    const int k = 27 * cin;
    float *g = (float *)malloc(sizeof(float) * (size_t)k);
    float *af = (float *)malloc(sizeof(float) * (size_t)k);
    orc_block_q8_0 *aq = (orc_block_q8_0 *)malloc(sizeof(orc_block_q8_0) * (size_t)(k / 32 + 1));
    const orc_wview v = orc_view(wtype, w, k);
    for (int64_t i = 0; i < n; ++i) {
        for (int t = 0; t < 27; ++t) {
            const int32_t j = nbr[i * 27 + t];
            if (j >= 0 && j < n)
                memcpy(g + t * cin, x + (int64_t)j * cin, sizeof(float) * (size_t)cin);
            else
                memset(g + t * cin, 0, sizeof(float) * (size_t)cin);
        }
        orc_prep(wtype, g, k, af, aq);
        for (int o = 0; o < cout; ++o) {
            float r = (float)orc_dot_row(&v, o, af, aq);
            if (bias) r += bias[o];
            y[i * cout + o] = r;
        }
    }
    free(g);
    free(af);
    free(aq);
}

/* Octant-weighted stride-2 conv and its transpose: an extension with no
 * counterpart in the reference, whose stride-2 operators are pool_down
 * (src/sparse.cpp:646-668) and nearest_up (:670-674).  A conv over a map
 * whose inputs are another level's rows: n_in input rows, n_out output rows,
 * nbr [n_out][27] of which the first ntaps columns are used (sentinel: any
 * value outside [0, n_in)); W packed [cout][ntaps * cin] as the 27-tap
 * conv's.  The gathered row is multiplied as orc_sparse_conv's (ggml
 * mul_mat semantics for wtype). */
void orc_conv_rect(const float *x, int64_t n_in, int cin, const int32_t *nbr, int64_t n_out, int ntaps, int wtype,
                   const void *w, int cout, const float *bias, float *y) {
    const int k = ntaps * cin;
    float *g = (float *)malloc(sizeof(float) * (size_t)k);
    float *af = (float *)malloc(sizeof(float) * (size_t)k);
    orc_block_q8_0 *aq = (orc_block_q8_0 *)malloc(sizeof(orc_block_q8_0) * (size_t)(k / 32 + 1));
    const orc_wview v = orc_view(wtype, w, k);
    for (int64_t i = 0; i < n_out; ++i) {
        for (int t = 0; t < ntaps; ++t) {
            const int32_t j = nbr[i * 27 + t];
            if (j >= 0 && j < n_in)
                memcpy(g + t * cin, x + (int64_t)j * cin, sizeof(float) * (size_t)cin);
            else
                memset(g + t * cin, 0, sizeof(float) * (size_t)cin);
        }
        orc_prep(wtype, g, k, af, aq);
        for (int o = 0; o < cout; ++o) {
            float r = (float)orc_dot_row(&v, o, af, aq);
            if (bias) r += bias[o];
            y[i * cout + o] = r;
        }
    }
    free(g);
    free(af);
    free(aq);
}

/* Octant maps of a stride-2 transition (orc_downsample's pool_rows [8][np]
 * and up_rows [nfine]).  The octant of fine voxel (x, y, z) inside its
 * parent's 2 x 2 x 2 cell is (x & 1) * 4 + (y & 1) * 2 + (z & 1).
 *   down [np][27]: column o = the child at octant o, or nfine; columns 8-26 nfine
 *   up [nfine][27]: column oct(c) = c's parent, every other column np */
void orc_octant_maps(const int32_t *coords, int64_t nfine, const int32_t *pool_rows, const int32_t *up_rows,
                     int64_t np, int32_t *down, int32_t *up) {
    for (int64_t i = 0; i < np * 27; ++i) down[i] = (int32_t)nfine;
    for (int64_t i = 0; i < nfine * 27; ++i) up[i] = (int32_t)np;
    for (int64_t p = 0; p < np; ++p)
        for (int s = 0; s < 8; ++s) {
            const int32_t c = pool_rows[(int64_t)s * np + p];
            if (c < 0 || c >= nfine) continue;
            const int32_t *q = coords + (int64_t)c * 4;
            down[p * 27 + (q[0] & 1) * 4 + (q[1] & 1) * 2 + (q[2] & 1)] = c;
        }
    for (int64_t c = 0; c < nfine; ++c) {
        const int32_t *q = coords + c * 4;
        up[c * 27 + (q[0] & 1) * 4 + (q[1] & 1) * 2 + (q[2] & 1)] = up_rows[c];
    }
}

/* src/sparse.cpp:515-518 linear: mul_mat(W [cout][cin], x) + bias. */
void orc_linear(const float *x, int64_t n, int cin, int wtype, const void *w, int cout, const float *bias, float *y) {
    float *af = (float *)malloc(sizeof(float) * (size_t)cin);
    orc_block_q8_0 *aq = (orc_block_q8_0 *)malloc(sizeof(orc_block_q8_0) * (size_t)(cin / 32 + 1));
    const orc_wview v = orc_view(wtype, w, cin);
    for (int64_t i = 0; i < n; ++i) {
        orc_prep(wtype, x + i * cin, cin, af, aq);
        for (int o = 0; o < cout; ++o) {
            float r = (float)orc_dot_row(&v, o, af, aq);
            if (bias) r += bias[o];
            y[i * cout + o] = r;
        }
    }
    free(af);
    free(aq);
}

/* src/sparse.cpp:520-526 layer_norm over ggml_norm (ggml-cpu/ops.cpp:3827-3893):
 * y = (x - mean) / sqrt(var + eps) * gamma + beta, per voxel over C. */
void orc_layer_norm(const float *x, int64_t n, int c, const float *gamma, const float *beta, float eps, float *y) {
    for (int64_t i = 0; i < n; ++i) {
        const float *xr = x + i * c;
        double s = 0.0;
        for (int j = 0; j < c; ++j) s += xr[j];
        const float mean = (float)(s / c);
        double v = 0.0;
        for (int j = 0; j < c; ++j) {
            const float d = xr[j] - mean;
            v += (double)d * d;
        }
        const float var = (float)(v / c);
        const float scale = 1.0f / sqrtf(var + eps);
        for (int j = 0; j < c; ++j) {
            float r = (xr[j] - mean) * scale;
            if (gamma) r *= gamma[j];
            if (beta) r += beta[j];
            y[i * c + j] = r;
        }
    }
}

/* ggml-cpu/vec.h:1046 ggml_silu_f32: x / (1 + exp(-x)). */
void orc_silu(float *x, int64_t n) {
    for (int64_t i = 0; i < n; ++i) x[i] = x[i] / (1.0f + expf(-x[i]));
}

/* src/sparse.cpp:629-642 res_block (identity skip). */
void orc_res_block(const float *x, int64_t n, int c, const int32_t *nbr, int wtype, const float *norm_w,
                   const float *norm_b, const void *w1, const float *b1, const void *w2, const float *b2, float *y) {
    float *h = (float *)malloc(sizeof(float) * (size_t)(n * c));
    float *h2 = (float *)malloc(sizeof(float) * (size_t)(n * c));
    orc_layer_norm(x, n, c, norm_w, norm_b, 1e-6f, h);
    orc_silu(h, n * c);
    orc_sparse_conv(h, n, c, nbr, wtype, w1, c, b1, h2);
    orc_silu(h2, n * c);
    orc_sparse_conv(h2, n, c, nbr, wtype, w2, c, b2, h);
    for (int64_t i = 0; i < n * c; ++i) y[i] = h[i] + x[i];
    free(h);
    free(h2);
}

/* ggml-cpu/ops.cpp:4208-4283 group_norm_f32 applied per sample, then the
 * affine ggml_mul / ggml_add. */
void orc_group_norm(const float *x, int64_t n, int c, const int32_t *sample, int nsamples, int groups, float eps,
                    const float *gamma, const float *beta, float *y) {
    const int cpg = (c + groups - 1) / groups;
    int64_t *count = (int64_t *)calloc((size_t)nsamples, sizeof(int64_t));
    double *sum = (double *)calloc((size_t)nsamples * (size_t)groups, sizeof(double));
    double *sum2 = (double *)calloc((size_t)nsamples * (size_t)groups, sizeof(double));
    float *mean = (float *)malloc(sizeof(float) * (size_t)nsamples * (size_t)groups);
    float *scale = (float *)malloc(sizeof(float) * (size_t)nsamples * (size_t)groups);
    for (int64_t i = 0; i < n; ++i) count[sample[i]]++;
    for (int64_t i = 0; i < n; ++i)
        for (int j = 0; j < c; ++j) sum[(int64_t)sample[i] * groups + j / cpg] += (double)x[i * c + j];
    for (int b = 0; b < nsamples; ++b)
        for (int g = 0; g < groups; ++g) {
            const int start = g * cpg, end = start + cpg > c ? c : start + cpg;
            const double cnt = (double)count[b] * (double)(end - start);
            mean[b * groups + g] = cnt > 0 ? (float)(sum[b * groups + g] / cnt) : 0.0f;
        }
    for (int64_t i = 0; i < n; ++i)
        for (int j = 0; j < c; ++j) {
            const int64_t k = (int64_t)sample[i] * groups + j / cpg;
            const float v = x[i * c + j] - mean[k];
            y[i * c + j] = v;
            sum2[k] += (double)(v * v);
        }
    for (int b = 0; b < nsamples; ++b)
        for (int g = 0; g < groups; ++g) {
            const int start = g * cpg, end = start + cpg > c ? c : start + cpg;
            const double cnt = (double)count[b] * (double)(end - start);
            const float variance = cnt > 0 ? (float)(sum2[b * groups + g] / cnt) : 0.0f;
            scale[b * groups + g] = 1.0f / sqrtf(variance + eps);
        }
    for (int64_t i = 0; i < n; ++i)
        for (int j = 0; j < c; ++j) {
            float t = y[i * c + j] * scale[(int64_t)sample[i] * groups + j / cpg];
            if (gamma) t = t * gamma[j];
            if (beta) t = t + beta[j];
            y[i * c + j] = t;
        }
    free(count);
    free(sum);
    free(sum2);
    free(mean);
    free(scale);
}

void orc_res_block_gn(const float *x, int64_t n, int c, const int32_t *nbr, const int32_t *sample, int nsamples,
                      int groups, float eps, int wtype, const float *gn_w, const float *gn_b, const void *w1,
                      const float *b1, const void *w2, const float *b2, float *y) {
    float *h = (float *)malloc(sizeof(float) * (size_t)(n * c));
    float *h2 = (float *)malloc(sizeof(float) * (size_t)(n * c));
    orc_sparse_conv(x, n, c, nbr, wtype, w1, c, b1, h);
    orc_group_norm(h, n, c, sample, nsamples, groups, eps, gn_w, gn_b, h2);
    orc_silu(h2, n * c);
    orc_sparse_conv(h2, n, c, nbr, wtype, w2, c, b2, h);
    for (int64_t i = 0; i < n * c; ++i) y[i] = h[i] + x[i];
    free(h);
    free(h2);
}

/* src/sparse.cpp:646-668 pool_down: sum of the slot gathers in slot order,
 * times inv_count, then linear. */
void orc_pool_down(const float *x, int64_t nfine, int c, const int32_t *pool_rows, const float *inv_count, int64_t np,
                   int slots, int wtype, const void *w, int cout, const float *bias, float *y) {
    float *s = (float *)malloc(sizeof(float) * (size_t)(np * c));
    for (int64_t p = 0; p < np; ++p) {
        float *sr = s + p * c;
        for (int j = 0; j < c; ++j) sr[j] = 0.0f;
        for (int sl = 0; sl < slots; ++sl) {
            const int32_t r = pool_rows[(int64_t)sl * np + p];
            if (r >= 0 && r < nfine)
                for (int j = 0; j < c; ++j) sr[j] += x[(int64_t)r * c + j];
        }
        for (int j = 0; j < c; ++j) sr[j] *= inv_count[p];
    }
    orc_linear(s, np, c, wtype, w, cout, bias, y);
    free(s);
}

/* src/sparse.cpp:670-674 nearest_up: linear, then gather the parent row. */
void orc_nearest_up(const float *x, int64_t np, int c, const int32_t *up_rows, int64_t nfine, int wtype, const void *w,
                    int cout, const float *bias, float *y) {
    float *t = (float *)malloc(sizeof(float) * (size_t)(np * cout));
    orc_linear(x, np, c, wtype, w, cout, bias, t);
    for (int64_t i = 0; i < nfine; ++i)
        memcpy(y + i * cout, t + (int64_t)up_rows[i] * cout, sizeof(float) * (size_t)cout);
    free(t);
}

/* ------------------------------------------------------ level-0 topology */

/* quantize_topology_z (src/sparse.cpp:363-406): q = nearbyint((double)(z *
 * depth_resolution)) with the product in float and the default rounding
 * mode (half to even); zbin = q - min(q).  Returns 0, or -1 when the extent
 * exceeds INT32_MAX (the reference throws). */
int orc_quantize_topology_z(const float *coord, int64_t n, float depth_resolution, int32_t *zbin) {
    if (n <= 0) return 0;
    int64_t *q = (int64_t *)malloc((size_t)n * sizeof(int64_t));
    if (!q) return -2;
    int64_t zmin = INT64_MAX, zmax = INT64_MIN;
    for (int64_t i = 0; i < n; ++i) {
        const float z = coord[3 * i + 2] * depth_resolution;
        q[i] = (int64_t)nearbyint((double)z);
        if (q[i] < zmin) zmin = q[i];
        if (q[i] > zmax) zmax = q[i];
    }
    if (zmax - zmin > INT32_MAX) {
        free(q);
        return -1;
    }
    for (int64_t i = 0; i < n; ++i) zbin[i] = (int32_t)(q[i] - zmin);
    free(q);
    return 0;
}

/* make_dense_image_level (src/sparse.cpp:274-310) on the level-0 coords of
 * build_topology_from_key (:408-431): pixel i = y*width + x is voxel
 * (y, x, zbin[i]); neighbour pixel j at (dy, dx) sits at tap
 * (dy+1)*9 + (dx+1)*3 + (dz+1) when dz = zbin[j] - zbin[i] is in [-1, 1];
 * other taps hold n. */
void orc_dense_image_level(const int32_t *zbin, int32_t width, int32_t height, int32_t *nbr) {
    const int64_t n = (int64_t)width * height;
    for (int64_t i = 0; i < n * 27; ++i) nbr[i] = (int32_t)n;
    for (int32_t y = 0; y < height; ++y)
        for (int32_t x = 0; x < width; ++x) {
            const int64_t i = (int64_t)y * width + x;
            for (int dy = -1; dy <= 1; ++dy) {
                const int32_t yy = y + dy;
                if (yy < 0 || yy >= height) continue;
                for (int dx = -1; dx <= 1; ++dx) {
                    const int32_t xx = x + dx;
                    if (xx < 0 || xx >= width) continue;
                    const int64_t j = (int64_t)yy * width + xx;
                    const int32_t dz = zbin[j] - zbin[i];
                    if (dz < -1 || dz > 1) continue;
                    nbr[i * 27 + (dy + 1) * 9 + (dx + 1) * 3 + (dz + 1)] = (int32_t)j;
                }
            }
        }
}
