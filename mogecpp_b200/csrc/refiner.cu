// Device executor of the MoGe-3 sparse refiner: SparseRefiner::refine_once
// (mogecpp src/sparse.cpp:1014-1296) with every step on the GPU.
//
// What the reference does per refine pass, and where it happens here:
//   get_topology_cached (:443-472)     quantise log z (image_topo.cu), compare
//                                      the bins with the cached ones on the
//                                      device, rebuild the pyramid on a miss:
//                                      level 0 from the pixel grid
//                                      (make_dense_image_level), coarser
//                                      levels by msc_make_level_downsample
//                                      (build_topology_from_key, :408-431),
//                                      plus one tap-order conv plan per level
//   upload_feature + input_proj        refiner input rows and a SIMT linear
//   down path (:1100-1157)             res blocks (msc_res_block_planned), pool
//                                      (msc_pool_down) into the next level;
//                                      deepest level: encoder rows, encoder_fuse,
//                                      fuse_proj.0 over [x | enc], SiLU,
//                                      fuse_proj.2, bottleneck blocks
//   up path (:1160-1191)               msc_nearest_up with the skip add, decoder
//                                      blocks, out_proj at level 0
//   residual readback (:1293-1295)     factor_coord[3i + 2] += residual[i] on the
//                                      device (no host round trip)
//
// The feature state is fp32 on every level, as the reference's CPU path
// keeps it (sparse_state_type, :560-563).  Weights come from a MOGG image
// (src/mogg.cpp:247-312): its refiner.* metadata is the SparseConfig
// (read_sparse_config, :985-1007) and its refiner.* tensors the weights
// (F32, F16 or Q8_0; sparse conv weights packed [cout][27 cin] as
// "*.weight.mogg_sparse27").
#include "../../include/moge_sparse_cuda.h"
#include "image_topo.h"

#include <cuda_fp16.h>
#include <cuda_runtime.h>

#include <cstring>
#include <map>
#include <stdexcept>
#include <string>
#include <variant>
#include <vector>

namespace msc {
void set_last_error(const std::string& msg);
}

namespace {

using namespace msc;

struct Fail : std::runtime_error {
    int code;
    Fail(int c, const std::string& m) : std::runtime_error(m), code(c) {}
};

[[noreturn]] void fail(int code, const std::string& m) { throw Fail(code, m); }

void ok(int rc, const char* what) {
    if (rc != MSC_OK) fail(rc, std::string(what) + ": " + msc_last_error());
}
void cuda(cudaError_t e, const char* what) {
    if (e != cudaSuccess) fail(MSC_E_CUDA, std::string(what) + ": " + cudaGetErrorString(e));
}

template <class F>
int guard(F&& f) {
    try {
        f();
        return MSC_OK;
    } catch (const Fail& e) {
        msc::set_last_error(e.what());
        return e.code;
    } catch (const std::exception& e) {
        msc::set_last_error(e.what());
        return MSC_E_INVALID;
    } catch (...) {
        msc::set_last_error("unknown error");
        return MSC_E_INVALID;
    }
}

// ------------------------------------------------------------------ MOGG
// MOGG v1 image (src/mogg.cpp:247-312): 8-byte magic, version, counts,
// alignment, metadata offset, data start; metadata records {u16 key length,
// key, u8 tag, u32 payload bytes, payload}; tensor records {u16 name length,
// name, u16 type, u8 ndim, u8 flags, i64 ne[4], u64 offset, u64 size}.
enum MoggTag : uint8_t { TAG_I64 = 1, TAG_F64 = 2, TAG_STR = 3, TAG_I64_LIST = 4, TAG_STR_LIST = 5, TAG_BOOL = 6 };
enum MoggType : uint16_t { MT_F32 = 1, MT_F16 = 2, MT_BF16 = 3, MT_I32 = 4, MT_Q8_0 = 12 };

using Meta = std::variant<int64_t, double, std::string, std::vector<int64_t>, bool>;

struct MoggTensor {
    uint16_t type = 0;
    int ndim = 0;
    int64_t ne[4] = {1, 1, 1, 1};
    const uint8_t* data = nullptr;
    uint64_t size = 0;
};

struct Mogg {
    std::map<std::string, Meta> meta;
    std::map<std::string, MoggTensor> tensors;
};

struct Reader {
    const uint8_t* p;
    const uint8_t* end;
    void need(size_t n) const {
        if (static_cast<size_t>(end - p) < n) fail(MSC_E_INVALID, "truncated MOGG image");
    }
    template <class T>
    T pod() {
        need(sizeof(T));
        T v;
        std::memcpy(&v, p, sizeof(T));
        p += sizeof(T);
        return v;
    }
    std::string str16() {
        const uint16_t n = pod<uint16_t>();
        need(n);
        std::string s(reinterpret_cast<const char*>(p), n);
        p += n;
        return s;
    }
};

uint64_t tensor_bytes(const MoggTensor& t) {
    uint64_t rows = 1;
    for (int d = 1; d < t.ndim; ++d) rows *= static_cast<uint64_t>(t.ne[d]);
    const uint64_t ne0 = static_cast<uint64_t>(t.ne[0]);
    switch (t.type) {
        case MT_F32:
        case MT_I32: return ne0 * 4 * rows;
        case MT_F16:
        case MT_BF16: return ne0 * 2 * rows;
        case MT_Q8_0: return (ne0 % 32) ? ~0ull : ne0 / 32 * 34 * rows;
        default: return ~0ull;  // types the refiner never holds (k-quants): size not checked
    }
}

Mogg parse_mogg(const uint8_t* data, size_t size) {
    static const uint8_t kMagic[8] = {'M', 'O', 'G', 'G', 0, 0, 0, 1};
    Reader h{data, data + size};
    h.need(40);
    if (std::memcmp(h.p, kMagic, 8) != 0) fail(MSC_E_INVALID, "not a MOGG v1 image");
    h.p += 8;
    const uint32_t version = h.pod<uint32_t>();
    const uint32_t n_meta = h.pod<uint32_t>();
    const uint32_t n_tensors = h.pod<uint32_t>();
    const uint32_t align = h.pod<uint32_t>();
    const uint64_t meta_off = h.pod<uint64_t>();
    const uint64_t data_start = h.pod<uint64_t>();
    if (version != 1) fail(MSC_E_INVALID, "unsupported MOGG version");
    if (align < 64 || (align & (align - 1))) fail(MSC_E_INVALID, "bad MOGG alignment");
    if (meta_off < 40 || meta_off >= data_start || data_start > size) fail(MSC_E_INVALID, "bad MOGG offsets");
    Mogg m;
    Reader r{data + meta_off, data + data_start};
    for (uint32_t i = 0; i < n_meta; ++i) {
        std::string key = r.str16();
        const uint8_t tag = r.pod<uint8_t>();
        const uint32_t bytes = r.pod<uint32_t>();
        r.need(bytes);
        const uint8_t* start = r.p;
        switch (tag) {
            case TAG_I64: m.meta[key] = r.pod<int64_t>(); break;
            case TAG_F64: m.meta[key] = r.pod<double>(); break;
            case TAG_BOOL: m.meta[key] = r.pod<uint8_t>() != 0; break;
            case TAG_STR: {
                const uint32_t n = r.pod<uint32_t>();
                r.need(n);
                m.meta[key] = std::string(reinterpret_cast<const char*>(r.p), n);
                r.p += n;
                break;
            }
            case TAG_I64_LIST: {
                const uint32_t n = r.pod<uint32_t>();
                std::vector<int64_t> v(n);
                for (uint32_t k = 0; k < n; ++k) v[k] = r.pod<int64_t>();
                m.meta[key] = std::move(v);
                break;
            }
            default: r.p += bytes; break;  // string lists: not read by the refiner
        }
        if (static_cast<uint64_t>(r.p - start) != bytes) fail(MSC_E_INVALID, "bad MOGG metadata record " + key);
    }
    for (uint32_t i = 0; i < n_tensors; ++i) {
        std::string name = r.str16();
        MoggTensor t;
        t.type = r.pod<uint16_t>();
        t.ndim = r.pod<uint8_t>();
        (void)r.pod<uint8_t>();  // flags
        for (int d = 0; d < 4; ++d) t.ne[d] = r.pod<int64_t>();
        const uint64_t off = r.pod<uint64_t>();
        t.size = r.pod<uint64_t>();
        if (t.ndim < 1 || t.ndim > 4) fail(MSC_E_INVALID, "bad ndim for " + name);
        if (off < data_start || off > size || t.size > size - off) fail(MSC_E_INVALID, "bad tensor extent for " + name);
        const uint64_t want = tensor_bytes(t);
        if (want != ~0ull && want != t.size) fail(MSC_E_INVALID, "tensor payload size does not match shape for " + name);
        t.data = data + off;
        m.tensors[name] = t;
    }
    return m;
}

template <class T>
T meta_get(const Mogg& m, const std::string& key) {
    auto it = m.meta.find(key);
    if (it == m.meta.end()) fail(MSC_E_INVALID, "missing metadata key: " + key);
    const T* v = std::get_if<T>(&it->second);
    if (!v) fail(MSC_E_INVALID, "metadata key has another type: " + key);
    return *v;
}

// ------------------------------------------------------------ device memory
struct DevBuf {
    void* p = nullptr;
    size_t cap = 0;
    DevBuf() = default;
    DevBuf(const DevBuf&) = delete;
    DevBuf& operator=(const DevBuf&) = delete;
    DevBuf(DevBuf&& o) noexcept : p(o.p), cap(o.cap) { o.p = nullptr, o.cap = 0; }
    DevBuf& operator=(DevBuf&& o) noexcept {
        std::swap(p, o.p);
        std::swap(cap, o.cap);
        return *this;
    }
    ~DevBuf() {
        if (p) cudaFree(p);
    }
    void* ensure(size_t bytes) {
        bytes = (bytes + 255) / 256 * 256;
        if (bytes <= cap && p) return p;
        if (p) cudaFree(p);
        p = nullptr;
        cap = 0;
        cuda(cudaMalloc(&p, bytes ? bytes : 256), "refiner device allocation");
        cap = bytes ? bytes : 256;
        return p;
    }
    template <class T>
    T* as() const {
        return static_cast<T*>(p);
    }
};

int msc_wtype(uint16_t t, const std::string& name) {
    if (t == MT_F32) return MSC_W_F32;
    if (t == MT_F16) return MSC_W_F16;
    if (t == MT_Q8_0) return MSC_W_Q8_0;
    fail(MSC_E_UNSUPPORTED, "refiner tensor " + name + " has a storage type this executor does not run (F32, F16 "
                                                       "and Q8_0 are supported)");
}

}  // namespace

struct msc_refiner {
    msc_ctx_t ctx = nullptr;
    msc_sparse_config cfg{};
    uint32_t* status = nullptr;

    // a learned vector (bias, norm affine) in fp32
    struct Vec {
        DevBuf buf;
        int n = 0;
        const float* ptr() const { return n ? buf.as<float>() : nullptr; }
    };
    // a weight prepared for the tensor-core conv / linear (msc_weight_prepare)
    struct Blob {
        DevBuf buf;
        int cin = 0, cout = 0, ntaps = 0;
    };
    // a linear weight kept raw for the SIMT linear (F32 or F16)
    struct Raw {
        DevBuf buf;
        int wtype = 0, cin = 0, cout = 0;
    };
    struct Lin {
        bool tc = false;  // tensor-core path (cin, cout in {64, 128})
        Blob blob;
        Raw raw;
        Vec bias;
    };
    struct Block {
        Vec norm_w, norm_b, b1, b2;
        Blob w1, w2;
    };

    Raw input_proj;
    Vec input_proj_b;
    std::vector<std::vector<Block>> down;  // [level][block]
    std::vector<Block> bottleneck;
    std::vector<std::vector<Block>> up;    // [u][block]
    std::vector<Lin> pool_lin, up_lin;
    Lin encoder_fuse, fuse0, fuse2;
    Raw out_proj;
    Vec out_proj_b;
    int fuse_channels = 0, fuse_hidden = 0;

    // topology cache (get_topology_cached, src/sparse.cpp:443-472)
    struct Level {
        int64_t n = 0;
        DevBuf coords, nbr, plan, state, tmp;
        // transition to the next level
        DevBuf pool_rows, inv, up_rows, np_dev;
    };
    std::vector<Level> levels;
    DevBuf zbin_cached, zbin_new, differ;
    int cache_w = 0, cache_h = 0;
    bool have_topology = false;
    uint64_t hits = 0, misses = 0;

    DevBuf ws, feat, enc_rows, enc_fused, fuse_tmp, residual, zq_ws;
    std::vector<uint8_t> host_stage;
};

namespace {

msc_refiner::Vec upload_vec(const Mogg& m, const std::string& name, int want_n, bool required, cudaStream_t st) {
    msc_refiner::Vec v;
    auto it = m.tensors.find(name);
    if (it == m.tensors.end()) {
        if (required) fail(MSC_E_INVALID, "missing refiner tensor " + name);
        return v;
    }
    const MoggTensor& t = it->second;
    const int64_t n = t.ne[0] * t.ne[1] * t.ne[2] * t.ne[3];
    if (want_n >= 0 && n != want_n)
        fail(MSC_E_INVALID, name + " has " + std::to_string(n) + " values, expected " + std::to_string(want_n));
    std::vector<float> h(static_cast<size_t>(n));
    for (int64_t i = 0; i < n; ++i) {
        if (t.type == MT_F32) {
            std::memcpy(&h[i], t.data + 4 * i, 4);
        } else if (t.type == MT_F16) {
            uint16_t b;
            std::memcpy(&b, t.data + 2 * i, 2);
            __half_raw r;
            r.x = b;
            h[i] = __half2float(__half(r));
        } else if (t.type == MT_BF16) {
            uint16_t b;
            std::memcpy(&b, t.data + 2 * i, 2);
            const uint32_t u = static_cast<uint32_t>(b) << 16;
            std::memcpy(&h[i], &u, 4);
        } else {
            fail(MSC_E_UNSUPPORTED, name + ": vectors must be F32, F16 or BF16");
        }
    }
    v.n = static_cast<int>(n);
    v.buf.ensure(4 * static_cast<size_t>(n));
    cuda(cudaMemcpyAsync(v.buf.p, h.data(), 4 * static_cast<size_t>(n), cudaMemcpyHostToDevice, st), "vector upload");
    cuda(cudaStreamSynchronize(st), "vector upload");
    return v;
}

const MoggTensor& need_tensor(const Mogg& m, const std::string& name) {
    auto it = m.tensors.find(name);
    if (it == m.tensors.end()) fail(MSC_E_INVALID, "missing refiner tensor " + name);
    return it->second;
}

void upload_raw_bytes(DevBuf& dst, const MoggTensor& t, cudaStream_t st) {
    dst.ensure(t.size);
    cuda(cudaMemcpyAsync(dst.p, t.data, t.size, cudaMemcpyHostToDevice, st), "weight upload");
    cuda(cudaStreamSynchronize(st), "weight upload");
}

// Weight [cout][ntaps * cin] (ggml ne0 = ntaps * cin, ne1 = cout) prepared
// for the tensor cores.
msc_refiner::Blob prepare_blob(msc_ctx_t ctx, const Mogg& m, const std::string& name, int cin, int cout, int ntaps,
                               cudaStream_t st) {
    const MoggTensor& t = need_tensor(m, name);
    if (t.ne[0] != static_cast<int64_t>(ntaps) * cin || t.ne[1] != cout)
        fail(MSC_E_INVALID, name + " has shape [" + std::to_string(t.ne[0]) + ", " + std::to_string(t.ne[1]) +
                                "], expected [" + std::to_string(ntaps * cin) + ", " + std::to_string(cout) + "]");
    const int wt = msc_wtype(t.type, name);
    DevBuf raw;
    upload_raw_bytes(raw, t, st);
    msc_refiner::Blob b;
    const size_t bytes = msc_weight_blob_bytes(wt, cin, cout, ntaps);
    b.buf.ensure(bytes);
    ok(msc_weight_prepare(ctx, wt, raw.p, cin, cout, ntaps, b.buf.p, bytes, st), name.c_str());
    cuda(cudaStreamSynchronize(st), "weight prepare");
    b.cin = cin, b.cout = cout, b.ntaps = ntaps;
    return b;
}

bool tc_width(int c) { return c == 64 || c == 128; }

msc_refiner::Raw upload_raw(const Mogg& m, const std::string& name, int cin, int cout, cudaStream_t st) {
    const MoggTensor& t = need_tensor(m, name);
    if (t.ne[0] != cin || t.ne[1] != cout)
        fail(MSC_E_INVALID, name + " has shape [" + std::to_string(t.ne[0]) + ", " + std::to_string(t.ne[1]) +
                                "], expected [" + std::to_string(cin) + ", " + std::to_string(cout) + "]");
    if (t.type != MT_F32 && t.type != MT_F16)
        fail(MSC_E_UNSUPPORTED, name + ": linear layers outside the tensor-core widths need F32 or F16 weights");
    msc_refiner::Raw r;
    upload_raw_bytes(r.buf, t, st);
    r.wtype = t.type == MT_F32 ? 0 : 1;
    r.cin = cin, r.cout = cout;
    return r;
}

msc_refiner::Lin load_linear(msc_ctx_t ctx, const Mogg& m, const std::string& pfx, int cin, int cout, cudaStream_t st) {
    msc_refiner::Lin l;
    const MoggTensor& t = need_tensor(m, pfx + ".weight");
    l.tc = tc_width(cin) && tc_width(cout) && (t.type == MT_F32 || t.type == MT_F16 || t.type == MT_Q8_0);
    if (l.tc)
        l.blob = prepare_blob(ctx, m, pfx + ".weight", cin, cout, 1, st);
    else
        l.raw = upload_raw(m, pfx + ".weight", cin, cout, st);
    l.bias = upload_vec(m, pfx + ".bias", cout, false, st);
    return l;
}

msc_refiner::Block load_block(msc_ctx_t ctx, const Mogg& m, const std::string& pfx, int c, cudaStream_t st) {
    if (m.tensors.count(pfx + ".skip_connection.weight"))
        fail(MSC_E_UNSUPPORTED, pfx + ": projected residual skips are not supported (identity skips only)");
    if (!tc_width(c)) fail(MSC_E_UNSUPPORTED, pfx + ": residual blocks run at 64 or 128 channels");
    msc_refiner::Block b;
    b.norm_w = upload_vec(m, pfx + ".norm1.weight", c, false, st);
    b.norm_b = upload_vec(m, pfx + ".norm1.bias", c, false, st);
    b.w1 = prepare_blob(ctx, m, pfx + ".conv1.weight.mogg_sparse27", c, c, 27, st);
    b.b1 = upload_vec(m, pfx + ".conv1.bias", c, false, st);
    b.w2 = prepare_blob(ctx, m, pfx + ".conv2.weight.mogg_sparse27", c, c, 27, st);
    b.b2 = upload_vec(m, pfx + ".conv2.bias", c, false, st);
    return b;
}

void read_config(const Mogg& m, msc_sparse_config& c) {
    auto it = m.meta.find("refiner.present");
    if (it == m.meta.end() || !std::get_if<bool>(&it->second) || !std::get<bool>(it->second))
        fail(MSC_E_INVALID, "the MOGG image has no sparse refiner (refiner.present)");
    c.in_channels = static_cast<int>(meta_get<int64_t>(m, "refiner.in_channels"));
    c.out_channels = static_cast<int>(meta_get<int64_t>(m, "refiner.out_channels"));
    c.encoder_channels = static_cast<int>(meta_get<int64_t>(m, "refiner.encoder_channels"));
    const auto mc = meta_get<std::vector<int64_t>>(m, "refiner.model_channels");
    const auto eb = meta_get<std::vector<int64_t>>(m, "refiner.encoder_blocks_per_level");
    const auto db = meta_get<std::vector<int64_t>>(m, "refiner.decoder_blocks_per_level");
    const auto df = meta_get<std::vector<int64_t>>(m, "refiner.downsample_factors");
    c.bottleneck_blocks = static_cast<int>(meta_get<int64_t>(m, "refiner.bottleneck_blocks"));
    c.encoder_downsample = static_cast<int>(meta_get<int64_t>(m, "refiner.encoder_downsample"));
    c.depth_resolution = static_cast<float>(meta_get<double>(m, "refiner.depth_resolution"));
    if (mc.size() < 2 || mc.size() > MSC_REFINER_MAX_LEVELS || eb.size() != mc.size() || db.size() + 1 != mc.size() ||
        df.size() + 1 != mc.size())
        fail(MSC_E_INVALID, "invalid sparse refiner metadata");
    c.num_levels = static_cast<int>(mc.size());
    int prod = 1;
    for (size_t i = 0; i < mc.size(); ++i) {
        c.model_channels[i] = static_cast<int>(mc[i]);
        c.encoder_blocks[i] = static_cast<int>(eb[i]);
        if (i + 1 < mc.size()) {
            c.decoder_blocks[i] = static_cast<int>(db[i]);
            c.downsample_factors[i] = static_cast<int>(df[i]);
            prod *= c.downsample_factors[i];
        }
    }
    if (prod != c.encoder_downsample) fail(MSC_E_INVALID, "refiner encoder_downsample mismatch");
    for (int i = 0; i + 1 < c.num_levels; ++i)
        if (c.downsample_factors[i] != 2)
            fail(MSC_E_UNSUPPORTED, "downsample factors other than 2 are not supported");
    if (c.out_channels != 1) fail(MSC_E_UNSUPPORTED, "MoGe-3 refiner out_channels != 1 unsupported");
    if (c.in_channels != 3) fail(MSC_E_UNSUPPORTED, "the refiner input has 3 channels (x/z, y/z, log z)");
}

// ---------------------------------------------------------------- driver

void build_topology(msc_refiner* R, const int32_t* zbin, int w, int h, cudaStream_t st) {
    msc_ctx_t ctx = R->ctx;
    const int L = R->cfg.num_levels;
    R->levels.resize(L);
    const int64_t n0 = static_cast<int64_t>(w) * h;
    auto& l0 = R->levels[0];
    l0.n = n0;
    l0.coords.ensure(16 * n0);
    l0.nbr.ensure(4 * 27 * n0);
    cuda(launch_dense_image_level(zbin, w, h, l0.coords.as<int32_t>(), l0.nbr.as<int32_t>(), st), "dense image level");
    for (int l = 0; l < L; ++l) {
        auto& lv = R->levels[l];
        const int64_t n = lv.n;
        const bool map = l > 0;          // level 0's map comes from the pixel grid
        const bool down = l + 1 < L;     // stride-2 maps into the next level
        if (map) lv.nbr.ensure(4 * 27 * (n ? n : 1));
        if (down) {
            R->levels[l + 1].coords.ensure(16 * (n ? n : 1));
            lv.pool_rows.ensure(4 * 8 * (n ? n : 1));
            lv.inv.ensure(4 * (n ? n : 1));
            lv.up_rows.ensure(4 * (n ? n : 1));
            lv.np_dev.ensure(4);
        }
        R->ws.ensure(msc_topology_workspace_bytes(n));
        int64_t np = 0;
        if (map && down) {
            // one voxel table for both maps of the level
            ok(msc_make_level_downsample(ctx, lv.coords.as<int32_t>(), n, lv.nbr.as<int32_t>(),
                                         R->levels[l + 1].coords.as<int32_t>(), lv.np_dev.as<int32_t>(),
                                         lv.pool_rows.as<int32_t>(), lv.inv.as<float>(), lv.up_rows.as<int32_t>(), &np,
                                         R->ws.p, R->ws.cap, st),
               "make_level_downsample");
        } else if (map) {
            ok(msc_make_level(ctx, lv.coords.as<int32_t>(), n, lv.nbr.as<int32_t>(), R->ws.p, R->ws.cap, st),
               "make_level");
        } else if (down) {
            ok(msc_downsample(ctx, lv.coords.as<int32_t>(), n, R->levels[l + 1].coords.as<int32_t>(),
                              lv.np_dev.as<int32_t>(), lv.pool_rows.as<int32_t>(), lv.inv.as<float>(),
                              lv.up_rows.as<int32_t>(), &np, R->ws.p, R->ws.cap, st),
               "downsample");
        }
        if (down) R->levels[l + 1].n = np;
        const size_t pb = msc_conv_plan_bytes(n);
        lv.plan.ensure(pb);
        R->ws.ensure(msc_conv_plan_workspace_bytes(n));
        ok(msc_conv_plan_build(ctx, nullptr, n, lv.nbr.as<int32_t>(), MSC_PLAN_TAP_ORDER, lv.plan.p, pb, R->ws.p,
                               R->ws.cap, st),
           "conv plan");
    }
}

void res_block(msc_refiner* R, msc_refiner::Level& lv, int c, const msc_refiner::Block& b, cudaStream_t st) {
    const size_t wsb = msc_op_workspace_bytes(lv.n, c);
    R->ws.ensure(wsb);
    ok(msc_res_block_planned(R->ctx, lv.state.p, MSC_F32, lv.n, c, lv.nbr.as<int32_t>(), lv.plan.p, b.norm_w.ptr(),
                             b.norm_b.ptr(), b.w1.buf.p, b.b1.ptr(), b.w2.buf.p, b.b2.ptr(), R->ws.p, R->ws.cap, st),
       "res_block");
}

void linear(msc_refiner* R, const msc_refiner::Lin& l, const float* x, int64_t n, int cin, float* y, cudaStream_t st) {
    if (l.tc) {
        R->ws.ensure(msc_op_workspace_bytes(n, cin > l.blob.cout ? cin : l.blob.cout));
        ok(msc_linear(R->ctx, x, MSC_F32, n, cin, l.blob.buf.p, l.bias.ptr(), y, MSC_F32, R->ws.p, R->ws.cap, st),
           "linear");
    } else {
        cuda(launch_small_linear(x, cin, nullptr, 0, n, l.raw.buf.p, l.raw.wtype, l.raw.cout, l.bias.ptr(), y, st),
             "linear");
    }
}

void refine(msc_refiner* R, float* fc, int w, int h, const float* enc, int ew, int eh, cudaStream_t st) {
    const msc_sparse_config& c = R->cfg;
    if (w != ew * c.encoder_downsample || h != eh * c.encoder_downsample)
        fail(MSC_E_INVALID, "refiner grid " + std::to_string(w) + "x" + std::to_string(h) + " does not match encoder " +
                                std::to_string(ew) + "x" + std::to_string(eh) + " * " +
                                std::to_string(c.encoder_downsample));
    if (w <= 0 || h <= 0) fail(MSC_E_INVALID, "empty image");
    if (static_cast<int64_t>(w) * h >= (int64_t(1) << 31) / 27) fail(MSC_E_INVALID, "image too large");
    if (!fc || !enc) fail(MSC_E_INVALID, "null pointer");
    const int64_t n0 = static_cast<int64_t>(w) * h;
    const int L = c.num_levels;
    const int deep = L - 1;

    // topology: quantised log z, cache check, rebuild on a miss
    R->zbin_new.ensure(4 * n0);
    R->zq_ws.ensure(quantize_z_workspace_bytes());
    cuda(launch_quantize_topology_z(fc, n0, c.depth_resolution, R->zbin_new.as<int32_t>(), R->zq_ws.p, R->status, st),
         "quantize_topology_z");
    bool hit = false;
    if (R->have_topology && R->cache_w == w && R->cache_h == h) {
        R->differ.ensure(4);
        cuda(launch_keys_differ(R->zbin_new.as<int32_t>(), R->zbin_cached.as<int32_t>(), n0, R->differ.as<int>(), st),
             "topology key compare");
        int differ = 1;
        cuda(cudaMemcpyAsync(&differ, R->differ.p, 4, cudaMemcpyDeviceToHost, st), "topology key compare");
        cuda(cudaStreamSynchronize(st), "topology key compare");
        hit = differ == 0;
    }
    uint32_t bits = 0;
    if (hit) {
        ++R->hits;
    } else {
        R->have_topology = false;
        build_topology(R, R->zbin_new.as<int32_t>(), w, h, st);
        std::swap(R->zbin_cached, R->zbin_new);
        R->cache_w = w, R->cache_h = h;
        R->have_topology = true;
        ++R->misses;
    }
    ok(msc_check(R->ctx, st, &bits), "refiner topology");

    // input rows and input_proj (3 -> C0)
    auto& l0 = R->levels[0];
    R->feat.ensure(4 * 3 * n0);
    cuda(launch_refiner_input(fc, n0, R->feat.as<float>(), st), "refiner input");
    for (int l = 0; l < L; ++l) {
        auto& lv = R->levels[l];
        const int64_t rows = lv.n ? lv.n : 1;
        lv.state.ensure(4 * rows * c.model_channels[l]);
        lv.tmp.ensure(4 * rows * c.model_channels[l]);
    }
    cuda(launch_small_linear(R->feat.as<float>(), 3, nullptr, 0, n0, R->input_proj.buf.p, R->input_proj.wtype,
                             c.model_channels[0], R->input_proj_b.ptr(), l0.state.as<float>(), st),
         "input_proj");

    // down path
    for (int l = 0; l <= deep; ++l) {
        auto& lv = R->levels[l];
        const int cl = c.model_channels[l];
        for (const auto& b : R->down[l]) res_block(R, lv, cl, b, st);
        if (l < deep) {
            auto& nx = R->levels[l + 1];
            const auto& pl = R->pool_lin[l];
            R->ws.ensure(msc_op_workspace_bytes(nx.n ? nx.n : 1, cl > c.model_channels[l + 1] ? cl : c.model_channels[l + 1]));
            ok(msc_pool_down(R->ctx, lv.state.p, MSC_F32, lv.n, cl, lv.pool_rows.as<int32_t>(), lv.inv.as<float>(), nx.n,
                             pl.blob.buf.p, pl.bias.ptr(), nx.state.p, MSC_F32, R->ws.p, R->ws.cap, st),
               "pool_down");
        } else {
            // encoder rows of the deep voxels, encoder_fuse, [x | enc] -> fuse_proj
            const int64_t n = lv.n;
            R->enc_rows.ensure(4 * (n ? n : 1) * c.encoder_channels);
            R->enc_fused.ensure(4 * (n ? n : 1) * R->fuse_channels);
            R->fuse_tmp.ensure(4 * (n ? n : 1) * R->fuse_hidden);
            cuda(launch_encoder_rows(lv.coords.as<int32_t>(), n, enc, ew, eh, c.encoder_channels,
                                     R->enc_rows.as<float>(), R->status, st),
                 "encoder rows");
            linear(R, R->encoder_fuse, R->enc_rows.as<float>(), n, c.encoder_channels, R->enc_fused.as<float>(), st);
            const auto& f0 = R->fuse0;
            cuda(launch_small_linear(lv.state.as<float>(), cl, R->enc_fused.as<float>(), R->fuse_channels, n,
                                     f0.raw.buf.p, f0.raw.wtype, R->fuse_hidden, f0.bias.ptr(), R->fuse_tmp.as<float>(),
                                     st),
                 "fuse_proj.0");
            cuda(launch_silu_inplace(R->fuse_tmp.as<float>(), n * R->fuse_hidden, st), "fuse SiLU");
            linear(R, R->fuse2, R->fuse_tmp.as<float>(), n, R->fuse_hidden, lv.state.as<float>(), st);
            for (const auto& b : R->bottleneck) res_block(R, lv, cl, b, st);
        }
    }
    // up path: the decoded feature replaces the skip on each level
    for (int u = 0; u + 1 < L; ++u) {
        const int t = L - 2 - u;
        auto& lv = R->levels[t];
        auto& src = R->levels[t + 1];
        const auto& ul = R->up_lin[u];
        const int ct = c.model_channels[t], cs = c.model_channels[t + 1];
        R->ws.ensure(msc_op_workspace_bytes(src.n ? src.n : 1, cs > ct ? cs : ct) + 4 * (src.n + 1) * ct);
        ok(msc_nearest_up(R->ctx, src.state.p, MSC_F32, src.n, cs, lv.up_rows.as<int32_t>(), lv.n, ul.blob.buf.p,
                          ul.bias.ptr(), lv.state.p, MSC_F32, lv.tmp.p, MSC_F32, R->ws.p, R->ws.cap, st),
           "nearest_up");
        std::swap(lv.state, lv.tmp);
        for (const auto& b : R->up[u]) res_block(R, lv, ct, b, st);
    }
    R->residual.ensure(4 * n0);
    cuda(launch_small_linear(l0.state.as<float>(), c.model_channels[0], nullptr, 0, n0, R->out_proj.buf.p,
                             R->out_proj.wtype, 1, R->out_proj_b.ptr(), R->residual.as<float>(), st),
         "out_proj");
    cuda(launch_logz_update(fc, R->residual.as<float>(), n0, st), "log z update");
}

}  // namespace

extern "C" {

int msc_refiner_create(msc_ctx_t ctx, const void* mogg, size_t mogg_bytes, void* stream, msc_refiner_t* out) {
    return guard([&] {
        if (!ctx || !mogg || !out) fail(MSC_E_INVALID, "null pointer");
        *out = nullptr;
        cudaStream_t st = static_cast<cudaStream_t>(stream);
        const Mogg m = parse_mogg(static_cast<const uint8_t*>(mogg), mogg_bytes);
        auto* R = new msc_refiner();
        try {
            R->ctx = ctx;
            read_config(m, R->cfg);
            const msc_sparse_config& c = R->cfg;
            cuda(cudaMalloc(&R->status, sizeof(uint32_t)), "status allocation");
            cuda(cudaMemset(R->status, 0, sizeof(uint32_t)), "status clear");
            R->input_proj = upload_raw(m, "refiner.input_proj.weight", c.in_channels, c.model_channels[0], st);
            R->input_proj_b = upload_vec(m, "refiner.input_proj.bias", c.model_channels[0], false, st);
            const int L = c.num_levels;
            R->down.resize(L);
            for (int l = 0; l < L; ++l)
                for (int b = 0; b < c.encoder_blocks[l]; ++b)
                    R->down[l].push_back(load_block(
                        ctx, m, "refiner.down_stages." + std::to_string(l) + "." + std::to_string(b), c.model_channels[l],
                        st));
            for (int l = 0; l + 1 < L; ++l) {
                R->pool_lin.push_back(load_linear(ctx, m, "refiner.downsample_blocks." + std::to_string(l) + ".linear",
                                                  c.model_channels[l], c.model_channels[l + 1], st));
                if (!R->pool_lin.back().tc) fail(MSC_E_UNSUPPORTED, "pool linear widths must be 64 or 128");
            }
            const int cd = c.model_channels[L - 1];
            const MoggTensor& ef = need_tensor(m, "refiner.encoder_fuse.weight");
            R->fuse_channels = static_cast<int>(ef.ne[1]);
            R->encoder_fuse = load_linear(ctx, m, "refiner.encoder_fuse", c.encoder_channels, R->fuse_channels, st);
            const MoggTensor& f0 = need_tensor(m, "refiner.fuse_proj.0.weight");
            R->fuse_hidden = static_cast<int>(f0.ne[1]);
            R->fuse0.raw = upload_raw(m, "refiner.fuse_proj.0.weight", cd + R->fuse_channels, R->fuse_hidden, st);
            R->fuse0.bias = upload_vec(m, "refiner.fuse_proj.0.bias", R->fuse_hidden, false, st);
            R->fuse2 = load_linear(ctx, m, "refiner.fuse_proj.2", R->fuse_hidden, cd, st);
            for (int b = 0; b < c.bottleneck_blocks; ++b)
                R->bottleneck.push_back(load_block(ctx, m, "refiner.bottleneck_stage." + std::to_string(b), cd, st));
            R->up.resize(L - 1);
            for (int u = 0; u + 1 < L; ++u) {
                const int t = L - 2 - u;
                R->up_lin.push_back(load_linear(ctx, m, "refiner.upsample_blocks." + std::to_string(u) + ".linear",
                                                c.model_channels[t + 1], c.model_channels[t], st));
                if (!R->up_lin.back().tc) fail(MSC_E_UNSUPPORTED, "upsample linear widths must be 64 or 128");
                for (int b = 0; b < c.decoder_blocks[u]; ++b)
                    R->up[u].push_back(load_block(
                        ctx, m, "refiner.up_stages." + std::to_string(u) + "." + std::to_string(b), c.model_channels[t],
                        st));
            }
            R->out_proj = upload_raw(m, "refiner.out_proj.weight", c.model_channels[0], c.out_channels, st);
            R->out_proj_b = upload_vec(m, "refiner.out_proj.bias", c.out_channels, false, st);
        } catch (...) {
            if (R->status) cudaFree(R->status);
            delete R;
            throw;
        }
        *out = R;
    });
}

int msc_refiner_destroy(msc_refiner_t r) {
    return guard([&] {
        if (!r) return;
        if (r->status) cudaFree(r->status);
        delete r;
    });
}

int msc_refiner_config(msc_refiner_t r, msc_sparse_config* out) {
    return guard([&] {
        if (!r || !out) fail(MSC_E_INVALID, "null pointer");
        *out = r->cfg;
    });
}

int msc_refiner_cache_stats(msc_refiner_t r, uint64_t* hits, uint64_t* misses) {
    return guard([&] {
        if (!r) fail(MSC_E_INVALID, "null refiner");
        if (hits) *hits = r->hits;
        if (misses) *misses = r->misses;
    });
}

int msc_refiner_level_sizes(msc_refiner_t r, int64_t* sizes, int capacity, int* count) {
    return guard([&] {
        if (!r || !count) fail(MSC_E_INVALID, "null pointer");
        *count = r->have_topology ? static_cast<int>(r->levels.size()) : 0;
        for (int i = 0; i < *count && i < capacity && sizes; ++i) sizes[i] = r->levels[i].n;
    });
}

int msc_refiner_refine_once(msc_refiner_t r, float* factor_coord, int width, int height, const float* encoder_feature,
                            int encoder_width, int encoder_height, void* stream) {
    return guard([&] {
        if (!r) fail(MSC_E_INVALID, "null refiner");
        cudaStream_t st = static_cast<cudaStream_t>(stream);
        refine(r, factor_coord, width, height, encoder_feature, encoder_width, encoder_height, st);
        uint32_t h = 0;
        cuda(cudaMemcpyAsync(&h, r->status, sizeof(h), cudaMemcpyDeviceToHost, st), "status read");
        cuda(cudaMemsetAsync(r->status, 0, sizeof(uint32_t), st), "status clear");
        cuda(cudaStreamSynchronize(st), "refine sync");
        if (h & MSC_DEV_BAD_COORD)
            fail(MSC_E_DEVICE, "log-depth bins out of range (non-finite z, or a bin extent beyond 2^19 - 1)");
        if (h & MSC_DEV_BAD_INDEX) fail(MSC_E_DEVICE, "deep sparse coord outside encoder feature map");
        ok(msc_check(r->ctx, st, nullptr), "refine");
    });
}

int msc_refiner_refine_once_host(msc_refiner_t r, float* factor_coord, int width, int height,
                                 const float* encoder_feature, int encoder_width, int encoder_height, void* stream) {
    return guard([&] {
        if (!r || !factor_coord || !encoder_feature) fail(MSC_E_INVALID, "null pointer");
        cudaStream_t st = static_cast<cudaStream_t>(stream);
        const int64_t n0 = static_cast<int64_t>(width) * height;
        const int64_t ne = static_cast<int64_t>(encoder_width) * encoder_height * r->cfg.encoder_channels;
        if (n0 <= 0 || ne <= 0) fail(MSC_E_INVALID, "empty image");
        DevBuf dfc, denc;
        dfc.ensure(4 * 3 * n0);
        denc.ensure(4 * ne);
        cuda(cudaMemcpyAsync(dfc.p, factor_coord, 4 * 3 * n0, cudaMemcpyHostToDevice, st), "factor_coord upload");
        cuda(cudaMemcpyAsync(denc.p, encoder_feature, 4 * ne, cudaMemcpyHostToDevice, st), "encoder upload");
        ok(msc_refiner_refine_once(r, dfc.as<float>(), width, height, denc.as<float>(), encoder_width, encoder_height,
                                   stream),
           "refine");
        cuda(cudaMemcpyAsync(factor_coord, dfc.p, 4 * 3 * n0, cudaMemcpyDeviceToHost, st), "factor_coord readback");
        cuda(cudaStreamSynchronize(st), "refine sync");
    });
}

int msc_quantize_topology_z(msc_ctx_t ctx, const float* factor_coord, int64_t n, float depth_resolution,
                            int32_t* zbin, void* stream) {
    return guard([&] {
        if (!ctx) fail(MSC_E_INVALID, "null context");
        if (n < 0) fail(MSC_E_INVALID, "negative pixel count");
        if (n == 0) return;
        if (!factor_coord || !zbin) fail(MSC_E_INVALID, "null pointer");
        cudaStream_t st = static_cast<cudaStream_t>(stream);
        DevBuf ws, status;
        ws.ensure(quantize_z_workspace_bytes());
        status.ensure(4);
        cuda(cudaMemsetAsync(status.p, 0, 4, st), "status clear");
        cuda(launch_quantize_topology_z(factor_coord, n, depth_resolution, zbin, ws.p, status.as<uint32_t>(), st),
             "quantize_topology_z");
        uint32_t h = 0;
        cuda(cudaMemcpyAsync(&h, status.p, 4, cudaMemcpyDeviceToHost, st), "status read");
        cuda(cudaStreamSynchronize(st), "quantize sync");
        if (h) fail(MSC_E_DEVICE, "log-depth bins out of range (non-finite z, or a bin extent beyond 2^19 - 1)");
    });
}

int msc_make_dense_image_level(msc_ctx_t ctx, const int32_t* zbin, int width, int height, int32_t* coords,
                               int32_t* nbr, void* stream) {
    return guard([&] {
        if (!ctx) fail(MSC_E_INVALID, "null context");
        if (width < 0 || height < 0) fail(MSC_E_INVALID, "negative image size");
        const int64_t n = static_cast<int64_t>(width) * height;
        if (n >= (int64_t(1) << 31) / 27) fail(MSC_E_INVALID, "image too large");
        if (n == 0) return;
        if (!zbin || !coords || !nbr) fail(MSC_E_INVALID, "null pointer");
        if (reinterpret_cast<uintptr_t>(coords) % 16) fail(MSC_E_INVALID, "coords is not 16-byte aligned");
        cuda(launch_dense_image_level(zbin, width, height, coords, nbr, static_cast<cudaStream_t>(stream)),
             "dense image level");
    });
}

}  // extern "C"
