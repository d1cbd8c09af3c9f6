// Reference harness: exposes the reference's own sparse-path functions
// (mogecpp src/sparse.cpp) behind a flat C API so that tests and the CPU
// baseline can call them on synthetic inputs.
//
// Test infrastructure only.  The harness includes the reference translation
// unit verbatim (its functions live in an anonymous namespace), builds a MOGG
// image in memory so that the reference WeightStore serves the synthetic
// weights, and runs the reference graph builders (sparse_conv, res_block,
// pool_down, nearest_up, linear) through ggml's CPU backend with the
// reference's own run_phase().  Topology comes from the reference's
// make_level() and downsample().
//
// Reference entry points used (paths inside the mogecpp tree):
//   make_level          src/sparse.cpp:238-272
//   downsample          src/sparse.cpp:312-357
//   sparse_conv         src/sparse.cpp:579-627
//   res_block           src/sparse.cpp:629-642
//   pool_down           src/sparse.cpp:646-668
//   nearest_up          src/sparse.cpp:670-674
//   linear, layer_norm  src/sparse.cpp:515-526
//   run_phase           src/sparse.cpp:850-894
//   quantize_topology_z src/sparse.cpp:363-406
//   make_dense_image_level src/sparse.cpp:274-310
//   SparseRefiner       src/sparse.cpp:985-1296 (read_sparse_config, refine_once)
//   MOGG v1 layout      src/mogg.cpp:247-312 (header 40 B, metadata, tensor records)

#include "sparse.cpp"

#include <ggml-cpu.h>

#include <chrono>
#include <cstdint>
#include <cstring>
#include <string>
#include <vector>

namespace {

thread_local std::string g_err;

// ---------------------------------------------------------------- MOGG image
struct MoggTensorSpec {
    std::string name;
    moge::MoggType type;
    int ndim;
    int64_t ne[4];
    std::vector<uint8_t> payload;
};

void put_u16(std::vector<uint8_t> & b, uint16_t v) { b.push_back(v & 0xff); b.push_back(v >> 8); }
void put_u32(std::vector<uint8_t> & b, uint32_t v) { for (int i = 0; i < 4; ++i) b.push_back((v >> (8 * i)) & 0xff); }
void put_u64(std::vector<uint8_t> & b, uint64_t v) { for (int i = 0; i < 8; ++i) b.push_back((v >> (8 * i)) & 0xff); }

// Serialise tensors into a MOGG v1 image with no metadata entries.
std::vector<uint8_t> build_mogg(const std::vector<MoggTensorSpec> & ts) {
    const uint64_t align = 64;
    std::vector<uint8_t> dir;
    // first pass: directory size (records have fixed size except names)
    size_t dir_bytes = 0;
    for (const auto & t : ts) dir_bytes += 2 + t.name.size() + 2 + 1 + 1 + 8 * 4 + 8 + 8;
    const uint64_t meta_offset = 40;
    uint64_t data_start = meta_offset + dir_bytes;
    data_start = (data_start + align - 1) / align * align;
    uint64_t off = data_start;
    std::vector<uint64_t> offsets;
    for (const auto & t : ts) {
        offsets.push_back(off);
        off += t.payload.size();
        off = (off + align - 1) / align * align;
    }
    std::vector<uint8_t> img;
    const uint8_t magic[8] = {'M', 'O', 'G', 'G', 0, 0, 0, 1};
    img.insert(img.end(), magic, magic + 8);
    put_u32(img, 1);                         // version
    put_u32(img, 0);                         // n_meta
    put_u32(img, static_cast<uint32_t>(ts.size()));
    put_u32(img, static_cast<uint32_t>(align));
    put_u64(img, meta_offset);
    put_u64(img, data_start);
    for (size_t i = 0; i < ts.size(); ++i) {
        const auto & t = ts[i];
        put_u16(img, static_cast<uint16_t>(t.name.size()));
        img.insert(img.end(), t.name.begin(), t.name.end());
        put_u16(img, static_cast<uint16_t>(t.type));
        img.push_back(static_cast<uint8_t>(t.ndim));
        img.push_back(static_cast<uint8_t>((t.name.find("mogg_sparse27") != std::string::npos)
                                               ? (moge::TF_SPARSE | moge::TF_SPARSE_PACKED) : 0));
        for (int d = 0; d < 4; ++d) put_u64(img, static_cast<uint64_t>(t.ne[d]));
        put_u64(img, offsets[i]);
        put_u64(img, t.payload.size());
    }
    img.resize(off, 0);
    for (size_t i = 0; i < ts.size(); ++i)
        std::memcpy(img.data() + offsets[i], ts[i].payload.data(), ts[i].payload.size());
    return img;
}

// wtype codes shared with the Python side: 0 = F32, 1 = F16, 8 = Q8_0.
MoggTensorSpec make_weight(const std::string & name, const float * w, int64_t ne0, int64_t ne1, int wtype) {
    MoggTensorSpec t;
    t.name = name;
    t.ndim = 2;
    t.ne[0] = ne0; t.ne[1] = ne1; t.ne[2] = 1; t.ne[3] = 1;
    const int64_t n = ne0 * ne1;
    if (wtype == 0) {
        t.type = moge::MoggType::F32;
        t.payload.resize(n * 4);
        std::memcpy(t.payload.data(), w, n * 4);
    } else if (wtype == 1) {
        t.type = moge::MoggType::F16;
        t.payload.resize(n * 2);
        ggml_fp32_to_fp16_row(w, reinterpret_cast<ggml_fp16_t *>(t.payload.data()), n);
    } else if (wtype == 8) {
        if (ne0 % 32) throw std::runtime_error("Q8_0 weight rows must be a multiple of 32");
        t.type = moge::MoggType::Q8_0;
        t.payload.resize(ggml_row_size(GGML_TYPE_Q8_0, ne0) * ne1);
        ggml_quantize_chunk(GGML_TYPE_Q8_0, w, t.payload.data(), 0, ne1, ne0, nullptr);
    } else {
        throw std::runtime_error("unsupported weight type code");
    }
    return t;
}

MoggTensorSpec make_vec(const std::string & name, const float * v, int64_t n) {
    MoggTensorSpec t;
    t.name = name;
    t.type = moge::MoggType::F32;
    t.ndim = 1;
    t.ne[0] = n; t.ne[1] = 1; t.ne[2] = 1; t.ne[3] = 1;
    t.payload.resize(n * 4);
    std::memcpy(t.payload.data(), v, n * 4);
    return t;
}

// -------------------------------------------------------- CPU backend runner
struct Runner {
    ggml_backend_t cpu = nullptr;
    ggml_backend_sched_t sched = nullptr;
    explicit Runner(int n_threads) {
        cpu = ggml_backend_cpu_init();
        if (!cpu) throw std::runtime_error("ggml_backend_cpu_init failed");
        ggml_backend_cpu_set_n_threads(cpu, n_threads > 0 ? n_threads : 1);
        sched = ggml_backend_sched_new(&cpu, nullptr, 1, 4096, false, true);
        if (!sched) throw std::runtime_error("ggml_backend_sched_new failed");
    }
    ~Runner() {
        if (sched) ggml_backend_sched_free(sched);
        if (cpu) ggml_backend_free(cpu);
    }
};

// Persistent device-side (here: CPU backend buffer) tensors.
struct State {
    ggml_context * ctx = nullptr;
    ggml_backend_buffer_t buf = nullptr;
    explicit State(size_t n_tensors) {
        ggml_init_params p{};
        p.mem_size = (n_tensors + 8) * ggml_tensor_overhead();
        p.no_alloc = true;
        ctx = ggml_init(p);
    }
    ggml_tensor * f32_2d(int64_t ne0, int64_t ne1) { return ggml_new_tensor_2d(ctx, GGML_TYPE_F32, ne0, ne1); }
    ggml_tensor * i32_1d(int64_t n) { return ggml_new_tensor_1d(ctx, GGML_TYPE_I32, n); }
    void alloc(ggml_backend_t b) {
        buf = ggml_backend_alloc_ctx_tensors(ctx, b);
        if (!buf) throw std::runtime_error("state buffer allocation failed");
    }
    ~State() {
        if (buf) ggml_backend_buffer_free(buf);
        if (ctx) ggml_free(ctx);
    }
};

template <class Fn>
int guard(Fn && fn) {
    try {
        fn();
        return 0;
    } catch (const std::exception & e) {
        g_err = e.what();
    } catch (...) {
        g_err = "unknown error";
    }
    return 1;
}

std::vector<moge::Coord3> to_coords(const int32_t * c, int32_t n) {
    std::vector<moge::Coord3> v(static_cast<size_t>(n));
    for (int32_t i = 0; i < n; ++i) v[i] = moge::Coord3{c[3 * i], c[3 * i + 1], c[3 * i + 2]};
    return v;
}

// Builds a phase graph with fn(ctx, weights) -> output tensor, copies the
// output into `out` (a state tensor) and runs it through run_phase().
template <class Fn>
void run_graph(Runner & r, const moge::WeightStore & ws, ggml_tensor * out, Fn && fn) {
    ggml_context * c = moge::make_phase_context();
    try {
        ggml_tensor * y = fn(c, ws);
        auto * cp = ggml_cpy(c, y, out);
        moge::run_phase(r.sched, c, "harness", {cp});
    } catch (...) {
        ggml_free(c);
        throw;
    }
    ggml_free(c);
}

} // namespace

extern "C" {

const char * ref_last_error(void) { return g_err.c_str(); }

// make_level: coords [n][3] (x=row, y=col, z=bin) -> nbr [n][27], sentinel n.
int ref_make_level(const int32_t * coords, int32_t n, int32_t * nbr) {
    return guard([&] {
        auto l = moge::make_level(to_coords(coords, n));
        std::memcpy(nbr, l.neighbors.data(), l.neighbors.size() * sizeof(int32_t));
    });
}

// downsample: coords [n][3] -> parents [np][3], pool_rows [slots][np] (sentinel n),
// inv_count [np], up_rows [n].  Output buffers must hold n parents.
int ref_downsample(const int32_t * coords, int32_t n, int32_t factor, int32_t * parent_coords,
                   int32_t * np_out, int32_t * pool_rows, float * inv_count, int32_t * up_rows) {
    return guard([&] {
        moge::SparseLevel fine;
        fine.coords = to_coords(coords, n);
        auto [parent, tr] = moge::downsample(fine, factor);
        const size_t np = parent.size();
        *np_out = static_cast<int32_t>(np);
        for (size_t p = 0; p < np; ++p) {
            parent_coords[3 * p] = parent[p].x;
            parent_coords[3 * p + 1] = parent[p].y;
            parent_coords[3 * p + 2] = parent[p].z;
        }
        std::memcpy(pool_rows, tr.pool_rows.data(), tr.pool_rows.size() * sizeof(int32_t));
        std::memcpy(inv_count, tr.inv_count.data(), tr.inv_count.size() * sizeof(float));
        std::memcpy(up_rows, tr.up_rows.data(), tr.up_rows.size() * sizeof(int32_t));
    });
}

// sparse_conv: x [n][cin] f32 -> y [n][cout] f32 with weight [cout][27*cin]
// (ggml ne0 = 27*cin) stored as wtype, optional bias [cout].
int ref_sparse_conv(int n_threads, const float * x, int64_t n, int64_t cin, const int32_t * nbr,
                    int wtype, const float * w, int64_t cout, const float * bias, float * y) {
    return guard([&] {
        std::vector<MoggTensorSpec> specs;
        specs.push_back(make_weight("t.weight.mogg_sparse27", w, 27 * cin, cout, wtype));
        if (bias) specs.push_back(make_vec("t.bias", bias, cout));
        auto img = build_mogg(specs);
        moge::MoggFile mf(img.data(), img.size(), true);
        Runner r(n_threads);
        moge::WeightStore ws(mf, r.cpu);
        State s(4);
        auto * tx = s.f32_2d(cin, n);
        auto * tn = s.i32_1d(27 * n);
        auto * ty = s.f32_2d(cout, n);
        s.alloc(r.cpu);
        ggml_backend_tensor_set(tx, x, 0, ggml_nbytes(tx));
        ggml_backend_tensor_set(tn, nbr, 0, ggml_nbytes(tn));
        run_graph(r, ws, ty, [&](ggml_context * c, const moge::WeightStore & w_) {
            return moge::sparse_conv(c, w_, tx, tn, "t", 0);
        });
        ggml_backend_tensor_get(ty, y, 0, ggml_nbytes(ty));
    });
}

// res_block (LayerNorm -> SiLU -> conv1 -> SiLU -> conv2 -> +x), identity skip.
// Also times `iters` repeated graph executions when iters > 0 (median seconds
// written to *seconds); the output is from the last run.
int ref_res_stack(int n_threads, const float * x, int64_t n, int64_t c, const int32_t * nbr, int wtype,
                  int n_blocks, const float * norm_w, const float * norm_b, const float * w1, const float * b1,
                  const float * w2, const float * b2, float * y, int iters, double * seconds) {
    return guard([&] {
        std::vector<MoggTensorSpec> specs;
        const int64_t wsz = c * 27 * c;
        for (int b = 0; b < n_blocks; ++b) {
            const std::string p = "blk." + std::to_string(b);
            specs.push_back(make_vec(p + ".norm1.weight", norm_w + b * c, c));
            specs.push_back(make_vec(p + ".norm1.bias", norm_b + b * c, c));
            specs.push_back(make_weight(p + ".conv1.weight.mogg_sparse27", w1 + b * wsz, 27 * c, c, wtype));
            specs.push_back(make_vec(p + ".conv1.bias", b1 + b * c, c));
            specs.push_back(make_weight(p + ".conv2.weight.mogg_sparse27", w2 + b * wsz, 27 * c, c, wtype));
            specs.push_back(make_vec(p + ".conv2.bias", b2 + b * c, c));
        }
        auto img = build_mogg(specs);
        moge::MoggFile mf(img.data(), img.size(), true);
        Runner r(n_threads);
        moge::WeightStore ws(mf, r.cpu);
        State s(4);
        auto * tx = s.f32_2d(c, n);
        auto * tn = s.i32_1d(27 * n);
        auto * ty = s.f32_2d(c, n);
        s.alloc(r.cpu);
        ggml_backend_tensor_set(tn, nbr, 0, ggml_nbytes(tn));
        std::vector<double> times;
        const int runs = iters > 0 ? iters : 1;
        for (int it = 0; it < runs; ++it) {
            ggml_backend_tensor_set(tx, x, 0, ggml_nbytes(tx));
            const auto t0 = std::chrono::steady_clock::now();
            run_graph(r, ws, ty, [&](ggml_context * cx, const moge::WeightStore & w_) {
                ggml_tensor * h = tx;
                for (int b = 0; b < n_blocks; ++b)
                    h = moge::res_block(cx, w_, h, tn, "blk." + std::to_string(b), 0);
                return h;
            });
            times.push_back(std::chrono::duration<double>(std::chrono::steady_clock::now() - t0).count());
        }
        std::sort(times.begin(), times.end());
        if (seconds) *seconds = times[times.size() / 2];
        ggml_backend_tensor_get(ty, y, 0, ggml_nbytes(ty));
    });
}

// pool_down: x [nfine][c] -> y [np][cout] = Linear(mean over children).
int ref_pool_down(int n_threads, const float * x, int64_t nfine, int64_t c, const int32_t * pool_rows,
                  const float * inv_count, int64_t np, int slots, int wtype, const float * w, int64_t cout,
                  const float * bias, float * y) {
    return guard([&] {
        std::vector<MoggTensorSpec> specs;
        specs.push_back(make_weight("p.linear.weight", w, c, cout, wtype));
        if (bias) specs.push_back(make_vec("p.linear.bias", bias, cout));
        auto img = build_mogg(specs);
        moge::MoggFile mf(img.data(), img.size(), true);
        Runner r(n_threads);
        moge::WeightStore ws(mf, r.cpu);
        State s(4);
        auto * tx = s.f32_2d(c, nfine);
        auto * tr = s.i32_1d(slots * np);
        auto * ti = s.f32_2d(1, np);
        auto * ty = s.f32_2d(cout, np);
        s.alloc(r.cpu);
        ggml_backend_tensor_set(tx, x, 0, ggml_nbytes(tx));
        ggml_backend_tensor_set(tr, pool_rows, 0, ggml_nbytes(tr));
        ggml_backend_tensor_set(ti, inv_count, 0, ggml_nbytes(ti));
        run_graph(r, ws, ty, [&](ggml_context * cx, const moge::WeightStore & w_) {
            return moge::pool_down(cx, w_, tx, tr, ti, slots, "p");
        });
        ggml_backend_tensor_get(ty, y, 0, ggml_nbytes(ty));
    });
}

// nearest_up: x [np][c] -> y [nfine][cout] = Linear(x)[up_rows].
int ref_nearest_up(int n_threads, const float * x, int64_t np, int64_t c, const int32_t * up_rows,
                   int64_t nfine, int wtype, const float * w, int64_t cout, const float * bias, float * y) {
    return guard([&] {
        std::vector<MoggTensorSpec> specs;
        specs.push_back(make_weight("u.linear.weight", w, c, cout, wtype));
        if (bias) specs.push_back(make_vec("u.linear.bias", bias, cout));
        auto img = build_mogg(specs);
        moge::MoggFile mf(img.data(), img.size(), true);
        Runner r(n_threads);
        moge::WeightStore ws(mf, r.cpu);
        State s(4);
        auto * tx = s.f32_2d(c, np);
        auto * tr = s.i32_1d(nfine);
        auto * ty = s.f32_2d(cout, nfine);
        s.alloc(r.cpu);
        ggml_backend_tensor_set(tx, x, 0, ggml_nbytes(tx));
        ggml_backend_tensor_set(tr, up_rows, 0, ggml_nbytes(tr));
        run_graph(r, ws, ty, [&](ggml_context * cx, const moge::WeightStore & w_) {
            return moge::nearest_up(cx, w_, tx, tr, "u");
        });
        ggml_backend_tensor_get(ty, y, 0, ggml_nbytes(ty));
    });
}

// Times make_level + downsample on the reference's topology threads
// (MOGE_SPARSE_TOPOLOGY_THREADS governs the thread count, as in the reference).
// ggml_group_norm (ggml.c:3233, CPU ops.cpp:4208-4283) of one sample's
// features [C, N] viewed as [N, 1, C] (groups along channels), no affine.
int ref_group_norm(int n_threads, const float * x, int64_t n, int64_t c, int groups, float eps, float * y) {
    return guard([&] {
        std::vector<float> one(1, 0.0f);
        std::vector<MoggTensorSpec> specs;
        specs.push_back(make_vec("unused.bias", one.data(), 1));
        auto img = build_mogg(specs);
        moge::MoggFile mf(img.data(), img.size(), true);
        Runner r(n_threads);
        moge::WeightStore ws(mf, r.cpu);
        State s(4);
        auto * tx = s.f32_2d(c, n);
        auto * ty = s.f32_2d(c, n);
        s.alloc(r.cpu);
        ggml_backend_tensor_set(tx, x, 0, ggml_nbytes(tx));
        run_graph(r, ws, ty, [&](ggml_context * g, const moge::WeightStore &) {
            ggml_tensor * t = ggml_cont(g, ggml_transpose(g, tx));            // [N, C]
            t = ggml_reshape_3d(g, t, n, 1, c);                               // [N, 1, C]
            t = ggml_group_norm(g, t, groups, eps);
            t = ggml_reshape_2d(g, t, n, c);                                  // [N, C]
            return ggml_cont(g, ggml_transpose(g, t));                        // [C, N]
        });
        ggml_backend_tensor_get(ty, y, 0, ggml_nbytes(ty));
    });
}

int ref_topology_timed(const int32_t * coords, int32_t n, int iters, double * make_level_s, double * downsample_s) {
    return guard([&] {
        auto cs = to_coords(coords, n);
        std::vector<double> t1, t2;
        for (int it = 0; it < (iters > 0 ? iters : 1); ++it) {
            auto a = std::chrono::steady_clock::now();
            auto l = moge::make_level(cs);
            auto b = std::chrono::steady_clock::now();
            auto d = moge::downsample(l, 2);
            auto e = std::chrono::steady_clock::now();
            t1.push_back(std::chrono::duration<double>(b - a).count());
            t2.push_back(std::chrono::duration<double>(e - b).count());
            (void) d;
        }
        std::sort(t1.begin(), t1.end());
        std::sort(t2.begin(), t2.end());
        *make_level_s = t1[t1.size() / 2];
        *downsample_s = t2[t2.size() / 2];
    });
}

// quantize_topology_z over factor_coord [w*h][3] with the given depth
// resolution -> zbin [w*h].
int ref_quantize_topology_z(const float * coord, int32_t width, int32_t height, float depth_resolution,
                            int32_t * zbin) {
    return guard([&] {
        const size_t n = static_cast<size_t>(width) * height;
        std::vector<float> fc(coord, coord + 3 * n);
        moge::SparseConfig cfg;
        cfg.depth_resolution = depth_resolution;
        auto key = moge::quantize_topology_z(fc, width, height, cfg);
        std::memcpy(zbin, key.z.data(), n * sizeof(int32_t));
    });
}

// Level 0 of build_topology_from_key: coords (row, column, zbin) and
// make_dense_image_level's neighbour map [w*h][27].
int ref_make_dense_image_level(const int32_t * zbin, int32_t width, int32_t height, int32_t * nbr) {
    return guard([&] {
        const size_t n = static_cast<size_t>(width) * height;
        std::vector<moge::Coord3> l0(n);
        for (size_t i = 0; i < n; ++i) {
            const int y = static_cast<int>(i / static_cast<size_t>(width));
            const int x = static_cast<int>(i - static_cast<size_t>(y) * width);
            l0[i] = moge::Coord3{y, x, zbin[i]};
        }
        auto l = moge::make_dense_image_level(std::move(l0), width, height);
        std::memcpy(nbr, l.neighbors.data(), l.neighbors.size() * sizeof(int32_t));
    });
}

// SparseRefiner::refine_once run `passes` times in a row on one refiner (so
// the second pass exercises the topology cache) from a MOGG image in memory:
// factor_coord [h*w][3] updated in place, encoder_feature [ew*eh][Cenc].
int ref_refine_once(int n_threads, const uint8_t * mogg, size_t mogg_bytes, float * factor_coord, int32_t width,
                    int32_t height, const float * encoder_feature, int32_t ew, int32_t eh, int passes,
                    double * seconds) {
    return guard([&] {
        moge::MoggFile mf(mogg, mogg_bytes, true);
        moge::SparseConfig cfg = moge::read_sparse_config(mf);
        Runner r(n_threads);
        moge::WeightStore ws(mf, r.cpu);
        moge::SparseRefiner refiner(ws, cfg);
        State s(2);
        auto * enc = s.f32_2d(cfg.encoder_channels, static_cast<int64_t>(ew) * eh);
        s.alloc(r.cpu);
        ggml_backend_tensor_set(enc, encoder_feature, 0, ggml_nbytes(enc));
        const size_t n = static_cast<size_t>(width) * height;
        std::vector<float> fc(factor_coord, factor_coord + 3 * n);
        std::vector<double> times;
        for (int p = 0; p < (passes > 0 ? passes : 1); ++p) {
            const auto t0 = std::chrono::steady_clock::now();
            refiner.refine_once(r.sched, fc, width, height, enc, ew, eh);
            times.push_back(std::chrono::duration<double>(std::chrono::steady_clock::now() - t0).count());
        }
        std::memcpy(factor_coord, fc.data(), 3 * n * sizeof(float));
        std::sort(times.begin(), times.end());
        if (seconds) *seconds = times[times.size() / 2];
    });
}

} // extern "C"
