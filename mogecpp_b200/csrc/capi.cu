// extern "C" boundary of the sparse-voxel path (include/moge_sparse_cuda.h).
//
// Error contract mirrors the reference C API (src/moge_c.cpp:20, :65-75):
// every call runs inside guard(), which converts exceptions into a negative
// status and a thread-local message; nothing throws across the boundary.
#include "conv.h"
#include "gn.h"
#include "ops.h"
#include "plan.h"
#include "topology.h"

#include "../../include/moge_sparse_cuda.h"

#include <cuda_runtime.h>

#include <cstdio>
#include <algorithm>
#include <mutex>
#include <stdexcept>
#include <string>
#include <unordered_map>
#include <vector>
#include <cstring>

struct msc_context {
    int device = 0;
    uint32_t* status = nullptr;  // device status word
    struct Blob {
        int wtype, cin, cout, ntaps, planes;
        size_t bytes;
    };
    std::mutex mu;
    std::unordered_map<const void*, Blob> blobs;
    struct Plan {
        int64_t n;     // output rows
        int kind;
        int64_t n_in;  // input rows its neighbour lists index
    };
    std::unordered_map<const void*, Plan> plans;  // conv plans built by this context
    // kernel profiling (msc_profile_*): one event pair per launch
    struct Rec {
        const char* name;
        cudaEvent_t a, b;
    };
    bool prof = false;
    std::vector<Rec> recs;
    std::vector<cudaEvent_t> pool;
    // msc_level_stack_host, per workspace: events after the input copies,
    // after the blocks and after the result copy of the last call on it
    // (the next call on that workspace waits for the last before
    // overwriting the device copies)
    struct WsEvents {
        cudaEvent_t in_done, blocks_done, out_done;
    };
    std::unordered_map<const void*, WsEvents> ws_events;
};

namespace {

thread_local std::string g_err;

struct Failure : std::runtime_error {
    int code;
    Failure(int c, const std::string& m) : std::runtime_error(m), code(c) {}
};

[[noreturn]] void fail(int code, const std::string& msg) { throw Failure(code, msg); }

void cuda_ok(cudaError_t e, const char* what) {
    if (e != cudaSuccess) fail(MSC_E_CUDA, std::string(what) + ": " + cudaGetErrorString(e));
}

template <class F>
int guard(F&& f) {
    try {
        f();
        return MSC_OK;
    } catch (const Failure& e) {
        g_err = e.what();
        return e.code;
    } catch (const std::exception& e) {
        g_err = e.what();
        return MSC_E_INVALID;
    } catch (...) {
        g_err = "unknown error";
        return MSC_E_INVALID;
    }
}

cudaStream_t S(void* s) { return static_cast<cudaStream_t>(s); }

cudaEvent_t take_event(msc_ctx_t ctx) {
    if (!ctx->pool.empty()) {
        cudaEvent_t e = ctx->pool.back();
        ctx->pool.pop_back();
        return e;
    }
    cudaEvent_t e = nullptr;
    if (cudaEventCreate(&e) != cudaSuccess) fail(MSC_E_CUDA, "cudaEventCreate failed");
    return e;
}

// Brackets one kernel launch with CUDA events when profiling is enabled
// (the counterpart of the reference's MOGE_OP_PROFILE per-node callback,
// src/profiling.hpp:50-71).
struct ProfScope {
    msc_ctx_t ctx;
    cudaStream_t st;
    cudaEvent_t b = nullptr;
    const char* name;
    cudaEvent_t a = nullptr;
    ProfScope(msc_ctx_t c, const char* n, cudaStream_t s) : ctx(c), st(s), name(n) {
        if (ctx->prof) {
            a = take_event(ctx);
            cudaEventRecord(a, st);
        }
    }
    ~ProfScope() {
        if (a) {
            b = take_event(ctx);
            cudaEventRecord(b, st);
            ctx->recs.push_back({name, a, b});
        }
    }
};

void need(bool cond, const char* msg) {
    if (!cond) fail(MSC_E_INVALID, msg);
}

void need_dtype(int dt, const char* what) {
    if (dt != MSC_F32 && dt != MSC_F16 && dt != MSC_BF16) fail(MSC_E_INVALID, std::string("bad dtype for ") + what);
}

void need_aligned(const void* p, size_t a, const char* what) {
    if (reinterpret_cast<uintptr_t>(p) % a) fail(MSC_E_INVALID, std::string(what) + " is not " + std::to_string(a) + "-byte aligned");
}

void need_ctx(msc_ctx_t ctx) {
    if (!ctx) fail(MSC_E_INVALID, "null context");
    int dev = -1;
    cuda_ok(cudaGetDevice(&dev), "cudaGetDevice");
    if (dev != ctx->device) fail(MSC_E_INVALID, "context belongs to device " + std::to_string(ctx->device) +
                                                  " but the current device is " + std::to_string(dev));
}

msc_context::Blob blob_info(msc_ctx_t ctx, const void* blob) {
    std::lock_guard<std::mutex> lk(ctx->mu);
    auto it = ctx->blobs.find(blob);
    if (it == ctx->blobs.end()) fail(MSC_E_INVALID, "weight blob was not prepared by this context");
    return it->second;
}

// Operand preparation mode for a weight type.
int act_mode(int wtype, int x_dtype, int cin) {
    if (wtype == MSC_W_Q8_0) return msc::weight_is_i8(wtype, cin) ? msc::ACT_Q8I : msc::ACT_Q8;
    if (wtype == MSC_W_F16) return msc::ACT_FP16;
    return x_dtype == MSC_F16 ? msc::ACT_FP16 : msc::ACT_SPLIT;
}

size_t align256(size_t v) { return (v + 255) / 256 * 256; }

cudaError_t act_prepare(msc_ctx_t ctx, const void* x, int x_dtype, int64_t n, int c, int ln, const float* gamma,
                        const float* beta, float eps, int silu, int mode, void* planes, cudaStream_t st) {
    ProfScope ps(ctx, "act_prepare", st);
    return msc::launch_act_prepare(x, x_dtype, n, c, ln, gamma, beta, eps, silu, mode, planes, st);
}

void need_ws(size_t have, size_t want) {
    if (have < want)
        fail(MSC_E_WORKSPACE, "workspace too small: " + std::to_string(have) + " < " + std::to_string(want));
}

// What a conv plan contributes to one conv: the tap order and the per-tile
// lists for the neighbour-map kernel, or nothing.
struct PlanUse {
    const int32_t* order = nullptr;
    msc::PlanTiles tiles{};
};

void run_conv(msc_ctx_t ctx, const void* planes, int mode, int64_t n, int cin, const int32_t* nbr,
              const msc_context::Blob& b, const void* blob, const float* bias, int silu_out, const void* residual,
              int res_dtype, void* y, int y_dtype, cudaStream_t st, PlanUse pu = {}, void* q_out = nullptr,
              int64_t n_in = -1, const char* family = nullptr) {
    if (n_in < 0) n_in = n;  // input rows (the prepared planes) = output rows unless given
    msc::ConvArgs a{};
    a.planes = planes;
    a.q8 = mode == msc::ACT_Q8 || mode == msc::ACT_Q8I;
    a.i8 = mode == msc::ACT_Q8I;
    a.a_scale = a.q8 ? reinterpret_cast<const float*>(static_cast<const char*>(planes) +
                                                      msc::act_scale_offset(mode, n_in, cin))
                     : nullptr;
    a.na = msc::act_planes(mode);
    a.n_in = n_in;
    a.n = n;
    a.row_begin = 0;
    a.perm = nullptr;
    a.cin = cin;
    a.nbr = nbr;
    a.blob = blob;
    a.wplanes = b.planes;
    a.cout = b.cout;
    a.ntaps = b.ntaps;
    a.bias = bias;
    a.silu_out = silu_out;
    a.residual = residual;
    a.res_dtype = res_dtype;
    a.y = y;
    a.y_dtype = y_dtype;
    if (q_out) {
        // fused re-quantisation: the ACT_Q8I operand of the next conv (no
        // caller combines it with a residual; the epilogue is only built and
        // tested without one)
        if (residual) fail(MSC_E_UNSUPPORTED, "fused Q8_0 output with a residual is not supported");
        a.q_codes = static_cast<int8_t*>(q_out);
        a.q_scales = reinterpret_cast<float*>(static_cast<char*>(q_out) +
                                              msc::act_scale_offset(msc::ACT_Q8I, n, b.cout));
    }
    a.status = ctx->status;
    a.perm = pu.order;
    a.tile_rows = pu.tiles.rows;
    a.tile_nbr = nbr ? pu.tiles.nbr : nullptr;
    a.tile_mask = pu.tiles.mask;
    a.tile_sched = nbr ? pu.tiles.sched : nullptr;
    ProfScope ps(ctx, family ? family : (nbr ? "conv_tc" : "linear_tc"), st);
    cuda_ok(msc::launch_conv(a, st), "conv launch");
}

// The plan, when given, must come from msc_conv_plan_build on this context
// for n voxels; it reorders the neighbour-map conv's tiles for every weight
// type.
PlanUse use_plan(msc_ctx_t ctx, const void* plan, int64_t n, int64_t n_in = -1) {
    if (n_in < 0) n_in = n;
    PlanUse pu;
    if (!plan) return pu;
    msc_context::Plan pl{};
    {
        std::lock_guard<std::mutex> lk(ctx->mu);
        auto it = ctx->plans.find(plan);
        if (it == ctx->plans.end()) fail(MSC_E_INVALID, "conv plan was not built by this context");
        pl = it->second;
    }
    if (pl.n != n)
        fail(MSC_E_INVALID, "conv plan covers " + std::to_string(pl.n) + " voxels, not " + std::to_string(n));
    if (pl.n_in != n_in)
        fail(MSC_E_INVALID, "conv plan indexes " + std::to_string(pl.n_in) + " input rows, not " + std::to_string(n_in));
    pu.tiles = msc::plan_tiles(static_cast<uint8_t*>(const_cast<void*>(plan)), n);
    pu.order = pu.tiles.order;
    return pu;
}

void check_conv_shape(const msc_context::Blob& b, int cin, int ntaps) {
    if (b.cin != cin) fail(MSC_E_INVALID, "weight cin " + std::to_string(b.cin) + " != input channels " + std::to_string(cin));
    if (b.ntaps != ntaps) fail(MSC_E_INVALID, "weight has " + std::to_string(b.ntaps) + " taps, expected " + std::to_string(ntaps));
    if (!msc::conv_supported(b.cin, b.cout))
        fail(MSC_E_UNSUPPORTED, "conv/linear shape " + std::to_string(b.cin) + "->" + std::to_string(b.cout) +
                                    " not built (channels must be 64 or 128)");
}

}  // namespace

namespace msc {
// Records the calling thread's error message (for entry points in other files).
void set_last_error(const std::string& msg) { g_err = msg; }

// Context services for the executors in other files (slab.cu): the device
// status word, the profiling event pair of one launch, a prepared blob's shape.
uint32_t* ctx_status(msc_ctx_t ctx) { return ctx->status; }
int ctx_device(msc_ctx_t ctx) { return ctx->device; }

void* prof_begin(msc_ctx_t ctx, const char* name, cudaStream_t st) {
    if (!ctx->prof) return nullptr;
    auto* rec = new msc_context::Rec{name, take_event(ctx), nullptr};
    cudaEventRecord(rec->a, st);
    return rec;
}

void prof_end(msc_ctx_t ctx, void* token, cudaStream_t st) {
    if (!token) return;
    auto* rec = static_cast<msc_context::Rec*>(token);
    rec->b = take_event(ctx);
    cudaEventRecord(rec->b, st);
    ctx->recs.push_back(*rec);
    delete rec;
}

bool blob_shape(msc_ctx_t ctx, const void* blob, int* wtype, int* cin, int* cout, int* ntaps, int* planes) {
    std::lock_guard<std::mutex> lk(ctx->mu);
    auto it = ctx->blobs.find(blob);
    if (it == ctx->blobs.end()) return false;
    *wtype = it->second.wtype, *cin = it->second.cin, *cout = it->second.cout, *ntaps = it->second.ntaps,
    *planes = it->second.planes;
    return true;
}
}  // namespace msc

extern "C" {

int msc_abi_version(void) { return MSC_ABI_VERSION; }

const char* msc_last_error(void) { return g_err.c_str(); }

int msc_create(int device, msc_ctx_t* out) {
    return guard([&] {
        need(out != nullptr, "null output pointer");
        cudaDeviceProp prop{};
        cuda_ok(cudaGetDeviceProperties(&prop, device), "cudaGetDeviceProperties");
        if (prop.major != 10 || prop.minor != 0)
            fail(MSC_E_UNSUPPORTED, "device " + std::to_string(device) + " is sm_" + std::to_string(prop.major) +
                                        std::to_string(prop.minor) + "; this library is built for sm_100a");
        cuda_ok(cudaSetDevice(device), "cudaSetDevice");
        auto* c = new msc_context();
        c->device = device;
        cudaError_t e = cudaMalloc(&c->status, sizeof(uint32_t));
        if (e == cudaSuccess) e = cudaMemset(c->status, 0, sizeof(uint32_t));
        if (e != cudaSuccess) {
            if (c->status) cudaFree(c->status);
            delete c;
            cuda_ok(e, "status word allocation");
        }
        *out = c;
    });
}

int msc_destroy(msc_ctx_t ctx) {
    return guard([&] {
        if (!ctx) return;
        if (ctx->status) cudaFree(ctx->status);
        for (auto& r : ctx->recs) {
            cudaEventDestroy(r.a);
            cudaEventDestroy(r.b);
        }
        for (auto e : ctx->pool) cudaEventDestroy(e);
        for (auto& kv : ctx->ws_events) {
            cudaEventDestroy(kv.second.in_done);
            cudaEventDestroy(kv.second.blocks_done);
            cudaEventDestroy(kv.second.out_done);
        }
        delete ctx;
    });
}

int msc_check(msc_ctx_t ctx, void* stream, uint32_t* bits) {
    return guard([&] {
        need_ctx(ctx);
        uint32_t h = 0;
        cuda_ok(cudaMemcpyAsync(&h, ctx->status, sizeof(h), cudaMemcpyDeviceToHost, S(stream)), "status read");
        cuda_ok(cudaMemsetAsync(ctx->status, 0, sizeof(uint32_t), S(stream)), "status clear");
        cuda_ok(cudaStreamSynchronize(S(stream)), "stream sync");
        if (bits) *bits = h;
        const uint32_t failing = h & ~MSC_DEV_DUP_COORD;
        if (failing) {
            std::string m = "device failure:";
            if (h & MSC_DEV_TIMEOUT) m += " wait-timeout";
            if (h & MSC_DEV_HASH_FULL) m += " hash-full";
            if (h & MSC_DEV_BAD_COORD) m += " coordinate-out-of-range";
            if (h & MSC_DEV_POOL_OVERFLOW) m += " pool-slot-overflow";
            if (h & MSC_DEV_BAD_INDEX) m += " index-out-of-range";
            if (h & MSC_DEV_PLAN_OVERFLOW) m += " plan-overflow";
            fail(MSC_E_DEVICE, m);
        }
    });
}

size_t msc_topology_workspace_bytes(int64_t n) { return n < 0 ? 0 : msc::topology_workspace_bytes(n); }

int msc_make_level(msc_ctx_t ctx, const int32_t* coords, int64_t n, int32_t* nbr, void* ws, size_t ws_bytes,
                   void* stream) {
    return guard([&] {
        need_ctx(ctx);
        need(n >= 0 && n < (int64_t(1) << 31) / 27, "voxel count out of range");
        if (n == 0) return;
        need(coords && nbr && ws, "null pointer");
        need_aligned(coords, 16, "coords");
        need_aligned(ws, 16, "workspace");
        need_ws(ws_bytes, msc::topology_workspace_bytes(n));
        ProfScope ps(ctx, "make_level", S(stream));
        cuda_ok(msc::launch_make_level(coords, n, nbr, ws, ctx->status, S(stream)), "make_level launch");
    });
}

namespace {
// With np_host: sync, store the parent count and report device failures of
// the stride-2 numbering (duplicate coordinates) by the return code.
void read_parent_count(msc_ctx_t ctx, const int32_t* np_dev, int64_t* np_host, cudaStream_t st) {
    if (!np_host) return;
    int32_t h = 0;
    cuda_ok(cudaMemcpyAsync(&h, np_dev, sizeof(h), cudaMemcpyDeviceToHost, st), "np read");
    uint32_t bits = 0;
    cuda_ok(cudaMemcpyAsync(&bits, ctx->status, sizeof(bits), cudaMemcpyDeviceToHost, st), "status read");
    cuda_ok(cudaStreamSynchronize(st), "stream sync");
    *np_host = h;
    if (bits & MSC_DEV_DUP_COORD) {
        cuda_ok(cudaMemsetAsync(ctx->status, 0, sizeof(uint32_t), st), "status clear");
        fail(MSC_E_DEVICE, "duplicate voxel coordinates: stride-2 slot numbering needs unique voxels");
    }
    if (bits & ~MSC_DEV_DUP_COORD) {
        cuda_ok(cudaMemsetAsync(ctx->status, 0, sizeof(uint32_t), st), "status clear");
        fail(MSC_E_DEVICE, "device failure in downsample (status bits " + std::to_string(bits) + ")");
    }
}
}  // namespace

int msc_downsample(msc_ctx_t ctx, const int32_t* coords, int64_t n, int32_t* parent, int32_t* np_dev,
                   int32_t* pool_rows, float* inv_count, int32_t* up_rows, int64_t* np_host, void* ws,
                   size_t ws_bytes, void* stream) {
    return guard([&] {
        need_ctx(ctx);
        need(n >= 0 && n < (int64_t(1) << 31) / 8, "voxel count out of range");
        need(np_dev != nullptr, "null np pointer");
        if (n > 0) {
            need(coords && parent && pool_rows && inv_count && up_rows && ws, "null pointer");
            need_aligned(coords, 16, "coords");
            need_aligned(parent, 16, "parent");
            need_aligned(ws, 16, "workspace");
            need_ws(ws_bytes, msc::topology_workspace_bytes(n));
        }
        {
            ProfScope ps(ctx, "downsample", S(stream));
            cuda_ok(msc::launch_downsample(coords, n, parent, np_dev, pool_rows, inv_count, up_rows, ws, ctx->status,
                                           S(stream)),
                    "downsample launch");
        }
        read_parent_count(ctx, np_dev, np_host, S(stream));
    });
}

int msc_make_level_downsample(msc_ctx_t ctx, const int32_t* coords, int64_t n, int32_t* nbr, int32_t* parent,
                              int32_t* np_dev, int32_t* pool_rows, float* inv_count, int32_t* up_rows,
                              int64_t* np_host, void* ws, size_t ws_bytes, void* stream) {
    return guard([&] {
        need_ctx(ctx);
        need(n >= 0 && n < (int64_t(1) << 31) / 27, "voxel count out of range");
        need(np_dev != nullptr, "null np pointer");
        if (n > 0) {
            need(coords && nbr && parent && pool_rows && inv_count && up_rows && ws, "null pointer");
            need_aligned(coords, 16, "coords");
            need_aligned(parent, 16, "parent");
            need_aligned(ws, 16, "workspace");
            need_ws(ws_bytes, msc::topology_workspace_bytes(n));
        }
        {
            ProfScope ps(ctx, "make_level_downsample", S(stream));
            cuda_ok(msc::launch_make_level_downsample(coords, n, nbr, parent, np_dev, pool_rows, inv_count, up_rows,
                                                      ws, ctx->status, S(stream)),
                    "make_level_downsample launch");
        }
        read_parent_count(ctx, np_dev, np_host, S(stream));
    });
}

size_t msc_weight_blob_bytes(int wtype, int cin, int cout, int ntaps) {
    if ((wtype != MSC_W_F32 && wtype != MSC_W_F16 && wtype != MSC_W_Q8_0) || cin <= 0 || cout <= 0 || ntaps <= 0)
        return 0;
    return msc::weight_blob_bytes(wtype, cin, cout, ntaps);
}

int msc_weight_prepare(msc_ctx_t ctx, int wtype, const void* w, int cin, int cout, int ntaps, void* blob,
                       size_t blob_bytes, void* stream) {
    return guard([&] {
        need_ctx(ctx);
        need(wtype == MSC_W_F32 || wtype == MSC_W_F16 || wtype == MSC_W_Q8_0, "unknown weight type");
        need(ntaps == 27 || ntaps == 8 || ntaps == 1,
             "ntaps must be 27 (sparse conv), 8 (octant-weighted stride-2 conv) or 1 (linear)");
        need(w && blob, "null pointer");
        need(cin > 0 && cout > 0, "bad channel counts");
        if (cin % 64 != 0) fail(MSC_E_UNSUPPORTED, "cin must be a multiple of 64");
        if (wtype == MSC_W_Q8_0) need(cin % 32 == 0, "Q8_0 rows need cin % 32 == 0");
        need_aligned(blob, 256, "weight blob");
        const size_t want = msc::weight_blob_bytes(wtype, cin, cout, ntaps);
        need_ws(blob_bytes, want);
        cuda_ok(msc::launch_weight_prepare(wtype, w, cin, cout, ntaps, blob, S(stream)), "weight prepare launch");
        std::lock_guard<std::mutex> lk(ctx->mu);
        ctx->blobs[blob] = msc_context::Blob{wtype, cin, cout, ntaps, msc::weight_planes(wtype, cin), want};
    });
}

size_t msc_op_workspace_bytes(int64_t n, int c) {
    if (n < 0 || c <= 0) return 0;
    return align256(static_cast<size_t>(n) * c * 4) + align256(static_cast<size_t>(n) * c * 4) + 256;
}

int64_t msc_gn_stats_doubles(int nsamples) { return nsamples < 1 ? 0 : msc::gn_stats_doubles(nsamples); }

size_t msc_res_block_gn_workspace_bytes(int64_t n, int c, int nsamples) {
    if (n < 0 || c <= 0 || nsamples < 1) return 0;
    return msc_op_workspace_bytes(n, c) + align256(static_cast<size_t>(nsamples) * 32 * sizeof(float2));
}

size_t msc_conv_plan_bytes(int64_t n) { return n < 0 ? 0 : msc::plan_bytes(n); }

size_t msc_conv_plan_workspace_bytes(int64_t n) { return n < 0 ? 0 : msc::plan_workspace_bytes(n); }

int msc_conv_plan_build(msc_ctx_t ctx, const int32_t* coords, int64_t n, const int32_t* nbr, int kind, void* plan,
                        size_t plan_bytes, void* ws, size_t ws_bytes, void* stream) {
    return guard([&] {
        need_ctx(ctx);
        (void)coords;
        need(kind == MSC_PLAN_TAP_ORDER, "unknown plan kind");
        need(n >= 0 && n < (int64_t(1) << 31) / 27, "voxel count out of range");
        need(plan != nullptr, "null plan pointer");
        need_aligned(plan, 256, "plan");
        need_ws(plan_bytes, msc::plan_bytes(n));
        if (n > 0) {
            need(nbr && ws, "null pointer");
            need_aligned(ws, 256, "workspace");
            need_ws(ws_bytes, msc::plan_workspace_bytes(n));
        }
        {
            ProfScope ps(ctx, "plan_build", S(stream));
            cuda_ok(msc::launch_plan_build(nbr, n, n, plan, ws, S(stream)), "plan build launch");
        }
        std::lock_guard<std::mutex> lk(ctx->mu);
        ctx->plans[plan] = msc_context::Plan{n, kind, n};
    });
}

int msc_conv_plan_build_rect(msc_ctx_t ctx, int64_t n_out, int64_t n_in, const int32_t* nbr, void* plan,
                             size_t plan_bytes, void* ws, size_t ws_bytes, void* stream) {
    return guard([&] {
        need_ctx(ctx);
        need(n_out >= 0 && n_out < (int64_t(1) << 31) / 27, "voxel count out of range");
        need(n_in >= 0 && n_in < (int64_t(1) << 31), "input row count out of range");
        need(plan != nullptr, "null plan pointer");
        need_aligned(plan, 256, "plan");
        need_ws(plan_bytes, msc::plan_bytes(n_out));
        if (n_out > 0) {
            need(nbr && ws, "null pointer");
            need_aligned(ws, 256, "workspace");
            need_ws(ws_bytes, msc::plan_workspace_bytes(n_out));
        }
        {
            ProfScope ps(ctx, "plan_build", S(stream));
            cuda_ok(msc::launch_plan_build(nbr, n_out, n_in, plan, ws, S(stream)), "plan build launch");
        }
        std::lock_guard<std::mutex> lk(ctx->mu);
        ctx->plans[plan] = msc_context::Plan{n_out, MSC_PLAN_TAP_ORDER, n_in};
    });
}

int msc_sparse_conv_planned(msc_ctx_t ctx, const void* x, int x_dtype, int64_t n, int cin, const int32_t* nbr,
                            const void* plan, const void* blob, const float* bias, void* y, int y_dtype, void* ws,
                            size_t ws_bytes, void* stream) {
    return guard([&] {
        need_ctx(ctx);
        need_dtype(x_dtype, "x");
        need_dtype(y_dtype, "y");
        const auto b = blob_info(ctx, blob);
        check_conv_shape(b, cin, 27);
        need(n >= 0 && n < (int64_t(1) << 31) / 27, "voxel count out of range");
        if (n == 0) return;
        const PlanUse pl = use_plan(ctx, plan, n);
        need(x && nbr && y && ws, "null pointer");
        need_aligned(x, 16, "x");
        need_aligned(y, 16, "y");
        need_aligned(ws, 256, "workspace");
        const int mode = act_mode(b.wtype, x_dtype, b.cin);
        need_ws(ws_bytes, msc::act_bytes(mode, n, cin));
        cuda_ok(act_prepare(ctx, x, x_dtype, n, cin, 0, nullptr, nullptr, 0.f, 0, mode, ws, S(stream)),
                "activation prepare");
        run_conv(ctx, ws, mode, n, cin, nbr, b, blob, bias, 0, nullptr, 0, y, y_dtype, S(stream), pl);
    });
}

int msc_octant_maps(msc_ctx_t ctx, const int32_t* coords, int64_t nfine, const int32_t* pool_rows,
                    const int32_t* up_rows, int64_t np, int32_t* down_nbr, int32_t* up_nbr, void* stream) {
    return guard([&] {
        need_ctx(ctx);
        need(nfine >= 0 && nfine < (int64_t(1) << 31) / 27, "voxel count out of range");
        need(np >= 0 && np <= nfine, "parent count out of range");
        if (nfine == 0) return;
        need(coords && pool_rows && up_rows && down_nbr && up_nbr, "null pointer");
        need_aligned(coords, 16, "coords");
        ProfScope ps(ctx, "octant_maps", S(stream));
        cuda_ok(msc::launch_octant_maps(coords, nfine, pool_rows, up_rows, np, down_nbr, up_nbr, S(stream)),
                "octant maps launch");
    });
}

int msc_octant_conv(msc_ctx_t ctx, const void* x, int x_dtype, int64_t n_in, int cin, const int32_t* nbr,
                    int64_t n_out, const void* plan, const void* blob, const float* bias, const void* skip,
                    int skip_dtype, void* y, int y_dtype, void* ws, size_t ws_bytes, void* stream) {
    return guard([&] {
        need_ctx(ctx);
        need_dtype(x_dtype, "x");
        need_dtype(y_dtype, "y");
        const auto b = blob_info(ctx, blob);
        check_conv_shape(b, cin, 8);
        need(n_in >= 0 && n_in < (int64_t(1) << 31), "input row count out of range");
        need(n_out >= 0 && n_out < (int64_t(1) << 31) / 27, "output row count out of range");
        if (n_out == 0) return;
        const PlanUse pl = use_plan(ctx, plan, n_out, n_in);
        need(nbr && y && ws && (x || n_in == 0), "null pointer");
        need_aligned(x, 16, "x");
        need_aligned(y, 16, "y");
        need_aligned(ws, 256, "workspace");
        if (skip) {
            need_dtype(skip_dtype, "skip");
            need_aligned(skip, 16, "skip");
        }
        const int mode = act_mode(b.wtype, x_dtype, b.cin);
        need_ws(ws_bytes, msc::act_bytes(mode, n_in, cin));
        if (n_in > 0)
            cuda_ok(act_prepare(ctx, x, x_dtype, n_in, cin, 0, nullptr, nullptr, 0.f, 0, mode, ws, S(stream)),
                    "activation prepare");
        run_conv(ctx, ws, mode, n_out, cin, nbr, b, blob, bias, 0, skip, skip ? skip_dtype : 0, y, y_dtype,
                 S(stream), pl, nullptr, n_in, "octant_conv");
    });
}

int msc_sparse_conv_fused(msc_ctx_t ctx, const void* x, int x_dtype, int64_t n, int cin, const int32_t* nbr,
                          const void* plan, const msc_conv_fusion* fusion, const void* blob, const float* bias,
                          void* y, int y_dtype, void* ws, size_t ws_bytes, void* stream) {
    return guard([&] {
        need_ctx(ctx);
        need_dtype(x_dtype, "x");
        need_dtype(y_dtype, "y");
        const auto b = blob_info(ctx, blob);
        check_conv_shape(b, cin, 27);
        need(n >= 0 && n < (int64_t(1) << 31) / 27, "voxel count out of range");
        if (n == 0) return;
        const msc_conv_fusion f = fusion ? *fusion : msc_conv_fusion{};
        need(!f.layer_norm || f.eps > 0.0f, "LayerNorm eps must be positive");
        if (f.residual) {
            need_dtype(f.residual_dtype, "residual");
            need_aligned(f.residual, 16, "residual");
        }
        const PlanUse pl = use_plan(ctx, plan, n);
        need(x && nbr && y && ws, "null pointer");
        need_aligned(x, 16, "x");
        need_aligned(y, 16, "y");
        need_aligned(ws, 256, "workspace");
        const int mode = act_mode(b.wtype, x_dtype, b.cin);
        need_ws(ws_bytes, msc::act_bytes(mode, n, cin));
        cuda_ok(act_prepare(ctx, x, x_dtype, n, cin, f.layer_norm ? 1 : 0, f.layer_norm ? f.norm_w : nullptr,
                            f.layer_norm ? f.norm_b : nullptr, f.eps, f.silu_in ? 1 : 0, mode, ws, S(stream)),
                "activation prepare");
        run_conv(ctx, ws, mode, n, cin, nbr, b, blob, bias, f.silu_out ? 1 : 0, f.residual,
                 f.residual ? f.residual_dtype : 0, y, y_dtype, S(stream), pl);
    });
}

int msc_sparse_conv(msc_ctx_t ctx, const void* x, int x_dtype, int64_t n, int cin, const int32_t* nbr,
                    const void* blob, const float* bias, void* y, int y_dtype, void* ws, size_t ws_bytes,
                    void* stream) {
    return msc_sparse_conv_planned(ctx, x, x_dtype, n, cin, nbr, nullptr, blob, bias, y, y_dtype, ws, ws_bytes,
                                   stream);
}

int msc_linear(msc_ctx_t ctx, const void* x, int x_dtype, int64_t n, int cin, const void* blob, const float* bias,
               void* y, int y_dtype, void* ws, size_t ws_bytes, void* stream) {
    return guard([&] {
        need_ctx(ctx);
        need_dtype(x_dtype, "x");
        need_dtype(y_dtype, "y");
        const auto b = blob_info(ctx, blob);
        check_conv_shape(b, cin, 1);
        need(n >= 0, "negative row count");
        if (n == 0) return;
        need(x && y && ws, "null pointer");
        need_aligned(x, 16, "x");
        need_aligned(y, 16, "y");
        need_aligned(ws, 256, "workspace");
        const int mode = act_mode(b.wtype, x_dtype, b.cin);
        need_ws(ws_bytes, msc::act_bytes(mode, n, cin));
        cuda_ok(act_prepare(ctx, x, x_dtype, n, cin, 0, nullptr, nullptr, 0.f, 0, mode, ws, S(stream)),
                "activation prepare");
        run_conv(ctx, ws, mode, n, cin, nullptr, b, blob, bias, 0, nullptr, 0, y, y_dtype, S(stream));
    });
}

int msc_res_block(msc_ctx_t ctx, void* x, int x_dtype, int64_t n, int c, const int32_t* nbr, const float* norm_w,
                  const float* norm_b, const void* blob1, const float* b1, const void* blob2, const float* b2,
                  void* ws, size_t ws_bytes, void* stream) {
    return msc_res_block_planned(ctx, x, x_dtype, n, c, nbr, nullptr, norm_w, norm_b, blob1, b1, blob2, b2, ws,
                                 ws_bytes, stream);
}

int msc_res_block_planned(msc_ctx_t ctx, void* x, int x_dtype, int64_t n, int c, const int32_t* nbr,
                          const void* plan, const float* norm_w, const float* norm_b, const void* blob1,
                          const float* b1, const void* blob2, const float* b2, void* ws, size_t ws_bytes,
                          void* stream) {
    return guard([&] {
        need_ctx(ctx);
        need_dtype(x_dtype, "x");
        const auto w1 = blob_info(ctx, blob1);
        const auto w2 = blob_info(ctx, blob2);
        check_conv_shape(w1, c, 27);
        check_conv_shape(w2, c, 27);
        need(w1.cout == c && w2.cout == c, "res_block convs must map c -> c");
        need(n >= 0 && n < (int64_t(1) << 31) / 27, "voxel count out of range");
        if (n == 0) return;
        const PlanUse pl = use_plan(ctx, plan, n);
        need(x && nbr && ws, "null pointer");
        need_aligned(x, 16, "x");
        need_aligned(ws, 256, "workspace");
        const size_t planes_bytes = align256(static_cast<size_t>(n) * c * 4);
        need_ws(ws_bytes, planes_bytes + static_cast<size_t>(n) * c * 4);
        void* planes = ws;
        float* h = reinterpret_cast<float*>(static_cast<char*>(ws) + planes_bytes);
        const int m1 = act_mode(w1.wtype, x_dtype, w1.cin);
        cuda_ok(act_prepare(ctx, x, x_dtype, n, c, 1, norm_w, norm_b, 1e-6f, 1, m1, planes, S(stream)),
                "norm1 prepare");
        const int m2 = act_mode(w2.wtype, MSC_F32, w2.cin);
        if (m2 == msc::ACT_Q8I && c == 128) {
            // conv1's epilogue quantises SiLU(conv1 + b1) for conv2 in place of
            // an fp32 intermediate and a separate preparation pass (same ggml
            // quantiser, same values: identical operand)
            run_conv(ctx, planes, m1, n, c, nbr, w1, blob1, b1, 1, nullptr, 0, h, MSC_F32, S(stream), pl, h);
            run_conv(ctx, h, m2, n, c, nbr, w2, blob2, b2, 0, x, x_dtype, x, x_dtype, S(stream), pl);
            return;
        }
        run_conv(ctx, planes, m1, n, c, nbr, w1, blob1, b1, 1, nullptr, 0, h, MSC_F32, S(stream), pl);
        cuda_ok(act_prepare(ctx, h, MSC_F32, n, c, 0, nullptr, nullptr, 0.f, 0, m2, planes, S(stream)),
                "conv2 prepare");
        run_conv(ctx, planes, m2, n, c, nbr, w2, blob2, b2, 0, x, x_dtype, x, x_dtype, S(stream), pl);
    });
}

int msc_res_stack(msc_ctx_t ctx, void* x, int x_dtype, int64_t n, int c, const int32_t* nbr, const void* plan,
                  int nblocks, const float* const* norm_w, const float* const* norm_b, const void* const* blob1,
                  const float* const* b1, const void* const* blob2, const float* const* b2, void* ws, size_t ws_bytes,
                  void* stream) {
    return guard([&] {
        need_ctx(ctx);
        need(nblocks >= 0, "negative block count");
        if (n == 0 || nblocks == 0) return;
        need(blob1 && blob2, "null weight arrays");
        auto opt = [](const float* const* a, int i) { return a ? a[i] : nullptr; };
        for (int i = 0; i < nblocks; ++i) {
            const int rc = msc_res_block_planned(ctx, x, x_dtype, n, c, nbr, plan, opt(norm_w, i), opt(norm_b, i),
                                                 blob1[i], opt(b1, i), blob2[i], opt(b2, i), ws, ws_bytes, stream);
            if (rc != MSC_OK) fail(rc, "block " + std::to_string(i) + ": " + g_err);
        }
    });
}

namespace {
// Section offsets of the msc_level_stack_host workspace: device coords,
// features, neighbour map, plan, then scratch shared by the topology, the
// plan build and the blocks.
struct StackHostWs {
    size_t coords, x, nbr, plan, scratch, scratch_bytes, total;
};
StackHostWs stack_host_ws(int64_t n, int c, int es) {
    StackHostWs w{};
    w.coords = 0;
    w.x = w.coords + align256(static_cast<size_t>(n) * 16);
    w.nbr = w.x + align256(static_cast<size_t>(n) * c * es);
    w.plan = w.nbr + align256(static_cast<size_t>(n) * 27 * 4);
    w.scratch = w.plan + align256(msc::plan_bytes(n));
    w.scratch_bytes = std::max({msc::topology_workspace_bytes(n), msc::plan_workspace_bytes(n),
                                msc_op_workspace_bytes(n, c)});
    w.total = w.scratch + align256(w.scratch_bytes);
    return w;
}
}  // namespace

size_t msc_level_stack_host_workspace_bytes(int64_t n, int c) {
    if (n < 0 || c <= 0) return 0;
    return stack_host_ws(n, c, 4).total;  // sized for fp32 features (fp16 / bf16 fit)
}

int msc_level_stack_host(msc_ctx_t ctx, const int32_t* coords_host, const void* x_host, int x_dtype, int64_t n,
                         int c, int nblocks, const float* const* norm_w, const float* const* norm_b,
                         const void* const* blob1, const float* const* b1, const void* const* blob2,
                         const float* const* b2, void* y_host, void* ws, size_t ws_bytes, void* stream,
                         void* copy_in_stream, void* copy_out_stream) {
    return guard([&] {
        need_ctx(ctx);
        need_dtype(x_dtype, "x");
        need(n >= 0 && n < (int64_t(1) << 31) / 27, "voxel count out of range");
        need(c > 0 && c % 32 == 0, "channels must be a positive multiple of 32");
        need(nblocks >= 0, "negative block count");
        if (n == 0) return;
        need(coords_host && x_host && y_host && ws, "null pointer");
        need_aligned(ws, 256, "workspace");
        const int es = x_dtype == MSC_F32 ? 4 : 2;
        const StackHostWs L = stack_host_ws(n, c, es);
        need_ws(ws_bytes, msc_level_stack_host_workspace_bytes(n, c));
        char* base = static_cast<char*>(ws);
        auto* coords = reinterpret_cast<int32_t*>(base + L.coords);
        void* x = base + L.x;
        auto* nbr = reinterpret_cast<int32_t*>(base + L.nbr);
        void* plan = base + L.plan;
        void* scratch = base + L.scratch;
        const size_t xbytes = static_cast<size_t>(n) * c * es;
        cudaStream_t st = S(stream);
        cudaStream_t in = copy_in_stream ? S(copy_in_stream) : st;
        cudaStream_t out = copy_out_stream ? S(copy_out_stream) : st;
        msc_context::WsEvents ev{};
        bool fresh = false;
        {
            std::lock_guard<std::mutex> lk(ctx->mu);
            auto it = ctx->ws_events.find(ws);
            if (it == ctx->ws_events.end()) {
                msc_context::WsEvents e{};
                cuda_ok(cudaEventCreateWithFlags(&e.in_done, cudaEventDisableTiming), "event create");
                cuda_ok(cudaEventCreateWithFlags(&e.blocks_done, cudaEventDisableTiming), "event create");
                cuda_ok(cudaEventCreateWithFlags(&e.out_done, cudaEventDisableTiming), "event create");
                it = ctx->ws_events.emplace(ws, e).first;
                fresh = true;
            }
            ev = it->second;
        }
        // inputs: after the previous call on this workspace has copied its result out
        if (!fresh) cuda_ok(cudaStreamWaitEvent(in, ev.out_done, 0), "wait previous result copy");
        cuda_ok(cudaMemcpyAsync(coords, coords_host, static_cast<size_t>(n) * 16, cudaMemcpyHostToDevice, in),
                "coords copy");
        cuda_ok(cudaMemcpyAsync(x, x_host, xbytes, cudaMemcpyHostToDevice, in), "features copy");
        if (in != st) {
            cuda_ok(cudaEventRecord(ev.in_done, in), "event record");
            cuda_ok(cudaStreamWaitEvent(st, ev.in_done, 0), "wait inputs");
        }
        int rc = msc_make_level(ctx, coords, n, nbr, scratch, L.scratch_bytes, st);
        if (rc != MSC_OK) fail(rc, "make_level: " + g_err);
        rc = msc_conv_plan_build(ctx, coords, n, nbr, MSC_PLAN_TAP_ORDER, plan, msc::plan_bytes(n), scratch,
                                 L.scratch_bytes, st);
        if (rc != MSC_OK) fail(rc, "plan: " + g_err);
        rc = msc_res_stack(ctx, x, x_dtype, n, c, nbr, plan, nblocks, norm_w, norm_b, blob1, b1, blob2, b2, scratch,
                           L.scratch_bytes, st);
        if (rc != MSC_OK) fail(rc, g_err);
        if (out != st) {
            cuda_ok(cudaEventRecord(ev.blocks_done, st), "event record");
            cuda_ok(cudaStreamWaitEvent(out, ev.blocks_done, 0), "wait blocks");
        }
        cuda_ok(cudaMemcpyAsync(y_host, x, xbytes, cudaMemcpyDeviceToHost, out), "result copy");
        cuda_ok(cudaEventRecord(ev.out_done, out), "event record");
    });
}

int msc_res_block_gn(msc_ctx_t ctx, void* x, int x_dtype, int64_t n, int64_t n_stat, int c, const int32_t* coords,
                     int nsamples, const int32_t* nbr, const void* plan, const float* gn_w, const float* gn_b,
                     float eps, const void* blob1, const float* b1, const void* blob2, const float* b2,
                     double* stats, msc_allreduce_fn allreduce, void* allreduce_user, void* ws, size_t ws_bytes,
                     void* stream) {
    return guard([&] {
        need_ctx(ctx);
        need_dtype(x_dtype, "x");
        const auto w1 = blob_info(ctx, blob1);
        const auto w2 = blob_info(ctx, blob2);
        check_conv_shape(w1, c, 27);
        check_conv_shape(w2, c, 27);
        need(w1.cout == c && w2.cout == c, "res_block convs must map c -> c");
        need(n >= 0 && n < (int64_t(1) << 31) / 27, "voxel count out of range");
        need(n_stat >= 0 && n_stat <= n, "n_stat must be in [0, n]");
        need(nsamples >= 1 && nsamples <= (1 << 20), "nsamples out of range");
        need(eps > 0.0f, "eps must be positive");
        if (n == 0 && !allreduce) return;
        const PlanUse pl = use_plan(ctx, plan, n);
        need(stats && ws && (n == 0 || (x && coords && nbr)), "null pointer");
        need_aligned(x, 16, "x");
        need_aligned(coords, 16, "coords");
        need_aligned(stats, 8, "stats");
        need_aligned(ws, 256, "workspace");
        need_ws(ws_bytes, msc_res_block_gn_workspace_bytes(n, c, nsamples));
        const size_t planes_bytes = align256(static_cast<size_t>(n) * c * 4);
        void* planes = ws;
        float* h = reinterpret_cast<float*>(static_cast<char*>(ws) + planes_bytes);
        float2* gn = reinterpret_cast<float2*>(static_cast<char*>(ws) + 2 * planes_bytes + 256);
        cudaStream_t st = S(stream);
        auto reduce = [&](double* buf, int64_t count, const char* what) {
            if (allreduce && allreduce(buf, count, stream, allreduce_user) != 0)
                fail(MSC_E_INVALID, std::string("GroupNorm statistics all-reduce failed (") + what + ")");
        };
        // conv1 + b1 on the raw features
        if (n > 0) {
            const int m1 = act_mode(w1.wtype, x_dtype, w1.cin);
            cuda_ok(act_prepare(ctx, x, x_dtype, n, c, 0, nullptr, nullptr, 0.f, 0, m1, planes, st), "conv1 prepare");
            run_conv(ctx, planes, m1, n, c, nbr, w1, blob1, b1, 0, nullptr, 0, h, MSC_F32, st, pl);
        }
        // sample-wide statistics of the owned rows (sums, counts, sums of
        // squares), summed over the ranks by the hook
        cuda_ok(cudaMemsetAsync(stats, 0, sizeof(double) * msc::gn_stats_doubles(nsamples), st), "stats clear");
        if (n > 0) {
            ProfScope ps(ctx, "gn_stats", st);
            cuda_ok(msc::launch_gn_stats(h, c, coords, n, n_stat, nsamples, stats, ctx->status, st),
                    "GroupNorm statistics");
        }
        reduce(stats, msc::gn_stats_doubles(nsamples), "statistics");
        if (n == 0) return;
        {
            ProfScope ps(ctx, "gn_finalize", st);
            cuda_ok(msc::launch_gn_finalize(stats, c, nsamples, eps, gn, st), "GroupNorm finalize");
        }
        // GroupNorm + SiLU fused into conv2's operand preparation, then
        // conv2 + b2 + x into x
        const int m2 = act_mode(w2.wtype, MSC_F32, w2.cin);
        {
            ProfScope ps(ctx, "act_prepare", st);
            cuda_ok(msc::launch_act_prepare(h, MSC_F32, n, c, 0, gn_w, gn_b, eps, 1, m2, planes, st, gn, coords,
                                            nsamples),
                    "GroupNorm apply");
        }
        run_conv(ctx, planes, m2, n, c, nbr, w2, blob2, b2, 0, x, x_dtype, x, x_dtype, st, pl);
    });
}

int msc_pool_down(msc_ctx_t ctx, const void* x, int x_dtype, int64_t nfine, int c, const int32_t* pool_rows,
                  const float* inv_count, int64_t np, const void* blob, const float* bias, void* y, int y_dtype,
                  void* ws, size_t ws_bytes, void* stream) {
    return guard([&] {
        need_ctx(ctx);
        need_dtype(x_dtype, "x");
        need_dtype(y_dtype, "y");
        const auto b = blob_info(ctx, blob);
        check_conv_shape(b, c, 1);
        need(np >= 0 && np <= nfine, "parent count out of range");
        if (np == 0) return;
        need(x && pool_rows && inv_count && y && ws, "null pointer");
        need_aligned(y, 16, "y");
        need_aligned(ws, 256, "workspace");
        const size_t pooled_bytes = align256(static_cast<size_t>(np) * c * 4);
        const int mode = act_mode(b.wtype, MSC_F32, b.cin);
        need_ws(ws_bytes, pooled_bytes + msc::act_bytes(mode, np, c));
        float* pooled = static_cast<float*>(ws);
        void* planes = static_cast<char*>(ws) + pooled_bytes;
        ProfScope pm(ctx, "pool_mean", S(stream));
        cuda_ok(msc::launch_pool_mean(x, x_dtype, nfine, c, pool_rows, inv_count, np, pooled, ctx->status, S(stream)),
                "pool mean");
        cuda_ok(act_prepare(ctx, pooled, MSC_F32, np, c, 0, nullptr, nullptr, 0.f, 0, mode, planes, S(stream)),
                "pool prepare");
        run_conv(ctx, planes, mode, np, c, nullptr, b, blob, bias, 0, nullptr, 0, y, y_dtype,
                 S(stream));
    });
}

int msc_nearest_up(msc_ctx_t ctx, const void* x, int x_dtype, int64_t np, int c, const int32_t* up_rows,
                   int64_t nfine, const void* blob, const float* bias, const void* skip, int skip_dtype, void* y,
                   int y_dtype, void* ws, size_t ws_bytes, void* stream) {
    return guard([&] {
        need_ctx(ctx);
        need_dtype(x_dtype, "x");
        need_dtype(y_dtype, "y");
        if (skip) need_dtype(skip_dtype, "skip");
        const auto b = blob_info(ctx, blob);
        check_conv_shape(b, c, 1);
        need(np >= 0 && nfine >= 0, "negative sizes");
        if (nfine == 0) return;
        need(np > 0, "upsampling from an empty level");
        need(x && up_rows && y && ws, "null pointer");
        need_aligned(x, 16, "x");
        need_aligned(ws, 256, "workspace");
        const int mode = act_mode(b.wtype, x_dtype, b.cin);
        const size_t planes_bytes = align256(msc::act_bytes(mode, np, c));
        need_ws(ws_bytes, planes_bytes + static_cast<size_t>(np) * b.cout * 4);
        void* planes = ws;
        float* t = reinterpret_cast<float*>(static_cast<char*>(ws) + planes_bytes);
        cuda_ok(act_prepare(ctx, x, x_dtype, np, c, 0, nullptr, nullptr, 0.f, 0, mode, planes, S(stream)),
                "up prepare");
        run_conv(ctx, planes, mode, np, c, nullptr, b, blob, bias, 0, nullptr, 0, t, MSC_F32,
                 S(stream));
        ProfScope pg(ctx, "gather_rows", S(stream));
        cuda_ok(msc::launch_gather_rows(t, np, b.cout, up_rows, nfine, skip, skip_dtype, y, y_dtype, ctx->status,
                                        S(stream)),
                "up gather");
    });
}

int msc_profile_enable(msc_ctx_t ctx, int enable) {
    return guard([&] {
        need_ctx(ctx);
        ctx->prof = enable != 0;
    });
}

int msc_profile_read(msc_ctx_t ctx, msc_profile_entry* out, int capacity, int* count) {
    return guard([&] {
        need_ctx(ctx);
        need(count != nullptr, "null count pointer");
        std::vector<msc_profile_entry> agg;
        for (auto& r : ctx->recs) {
            cuda_ok(cudaEventSynchronize(r.b), "profile event sync");
            float ms = 0.f;
            cuda_ok(cudaEventElapsedTime(&ms, r.a, r.b), "profile elapsed time");
            msc_profile_entry* e = nullptr;
            for (auto& x : agg)
                if (std::strncmp(x.name, r.name, sizeof(x.name)) == 0) e = &x;
            if (!e) {
                agg.push_back(msc_profile_entry{});
                e = &agg.back();
                std::strncpy(e->name, r.name, sizeof(e->name) - 1);
            }
            e->launches += 1;
            e->total_ms += ms;
            ctx->pool.push_back(r.a);
            ctx->pool.push_back(r.b);
        }
        ctx->recs.clear();
        *count = static_cast<int>(agg.size());
        for (int i = 0; i < static_cast<int>(agg.size()) && i < capacity && out; ++i) out[i] = agg[i];
    });
}

}  // extern "C"
