// Z-slab shard of the residual stack on one GPU of a multi-GPU node, with
// the halo exchange fused into the second conv of every block.
//
// Layout of a rank's rows (the z-slab partition, voxel-count quantiles cut on
// z-plane boundaries): [owned | halo below | halo above], the halos being the
// two z-planes on either side owned by the neighbouring ranks; the first
// send_lo owned rows are the lower neighbour's "halo above", the last send_hi
// owned rows the upper neighbour's "halo below", in the same order.
//
// Per residual block k (LayerNorm -> SiLU -> conv1 -> SiLU -> conv2 -> +x,
// mogecpp src/sparse.cpp:629-642):
//   1. wait until both neighbours have finished block k-1 (their flags in this
//      GPU's memory reach k; a bounded one-thread poll: a neighbour that never
//      arrives sets MSC_DEV_TIMEOUT after 2 s and the block runs on);
//   2. operand preparation of all local rows of buffer x[k % 2];
//   3. conv1 over all local rows (its output on the inner halo plane is what
//      conv2 needs at the slab edge), Q8_0 operand of conv2 fused in;
//   4. conv2 over the owned rows only, into x[(k + 1) % 2]; its epilogue also
//      stores the boundary rows straight into the neighbours' x[(k + 1) % 2]
//      halo rows (CUDA IPC pointers, NVLink);
//   5. signal: a system-scope release store of k + 1 into each neighbour's
//      flag for this rank.
// The two feature buffers alternate, so a neighbour writing block k's halo
// rows never touches the buffer this rank still reads for block k (and step
// 1 orders the reuse two blocks later).  No NCCL call on this path: the
// exchange is the conv epilogue's peer stores.
#include "../../include/moge_sparse_cuda.h"
#include "conv.h"
#include "plan.h"
#include "topology.h"

#include <cuda_runtime.h>

#include <cstring>
#include <stdexcept>
#include <string>

namespace msc {
void set_last_error(const std::string& msg);
uint32_t* ctx_status(msc_ctx_t ctx);
int ctx_device(msc_ctx_t ctx);
void* prof_begin(msc_ctx_t ctx, const char* name, cudaStream_t st);
void prof_end(msc_ctx_t ctx, void* token, cudaStream_t st);
bool blob_shape(msc_ctx_t ctx, const void* blob, int* wtype, int* cin, int* cout, int* ntaps, int* planes);
}  // namespace msc

namespace {

using namespace msc;

struct Fail : std::runtime_error {
    int code;
    Fail(int c, const std::string& m) : std::runtime_error(m), code(c) {}
};
[[noreturn]] void fail(int code, const std::string& m) { throw Fail(code, m); }
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
    }
}

constexpr uint32_t kHandleMagic = 0x534c4142u;  // "SLAB"
constexpr unsigned long long kWaitNs = 2000000000ull;

struct Handle {
    uint32_t magic;
    int32_t rank, world, channels;
    int64_t n_local, n_owned, n_halo_lo, n_halo_hi, send_lo, send_hi;
    cudaIpcMemHandle_t x[2];
    cudaIpcMemHandle_t flags;
};
static_assert(sizeof(Handle) <= sizeof(msc_slab_handle), "handle size");

__device__ __forceinline__ unsigned long long timer_ns() {
    unsigned long long t;
    asm volatile("mov.u64 %0, %%globaltimer;" : "=l"(t));
    return t;
}

__device__ __forceinline__ int ld_acquire_sys(const int* p) {
    int v;
    asm volatile("ld.acquire.sys.global.b32 %0, [%1];" : "=r"(v) : "l"(p) : "memory");
    return v;
}

__device__ __forceinline__ void st_release_sys(int* p, int v) {
    asm volatile("st.release.sys.global.b32 [%0], %1;" ::"l"(p), "r"(v) : "memory");
}

// One thread polls this GPU's flags (written by the neighbours over
// NVLink) until both reach `target`, for at most 2 s.
__global__ void slab_wait_kernel(const int* flags, int need_lo, int need_hi, int target, uint32_t* status,
                                 unsigned long long budget_ns) {
    if (threadIdx.x != 0) return;
    const unsigned long long t0 = timer_ns();
    for (;;) {
        const bool lo = !need_lo || ld_acquire_sys(flags) >= target;
        const bool hi = !need_hi || ld_acquire_sys(flags + 1) >= target;
        if (lo && hi) return;
        if (timer_ns() - t0 > budget_ns) {
            atomicOr(status, MSC_DEV_TIMEOUT);
            return;
        }
        __nanosleep(256);
    }
}

// Publishes "this rank finished block value - 1" to each neighbour: every
// store of the preceding kernels (the conv's peer stores included) is
// ordered before the flag by the system-scope fence and release.
__global__ void slab_signal_kernel(int* lo_flag, int* hi_flag, int value) {
    if (threadIdx.x != 0) return;
    asm volatile("fence.acq_rel.sys;" ::: "memory");
    if (lo_flag) st_release_sys(lo_flag, value);
    if (hi_flag) st_release_sys(hi_flag, value);
}

size_t align256(size_t v) { return (v + 255) / 256 * 256; }

}  // namespace

struct msc_slab {
    msc_ctx_t ctx = nullptr;
    msc_slab_desc d{};
    void* x[2] = {nullptr, nullptr};
    int* flags = nullptr;  // [0]: blocks the lower neighbour finished, [1]: the upper one
    struct Peer {
        void* x[2] = {nullptr, nullptr};
        int* flags = nullptr;
        int64_t off = 0;
    } lo, hi;
    int cur = 0;
    int32_t done = 0;
    int32_t* nbr = nullptr;
    void* plan_all = nullptr;
    void* plan_own = nullptr;
    void* ws = nullptr;
    size_t ws_bytes = 0;
    bool level = false;

    ~msc_slab() {
        for (Peer* p : {&lo, &hi}) {
            for (void* v : p->x)
                if (v) cudaIpcCloseMemHandle(v);
            if (p->flags) cudaIpcCloseMemHandle(p->flags);
        }
        for (void* v : {x[0], x[1], static_cast<void*>(flags), static_cast<void*>(nbr), plan_all, plan_own, ws})
            if (v) cudaFree(v);
    }
};

extern "C" {

int msc_slab_create(msc_ctx_t ctx, const msc_slab_desc* desc, msc_slab_t* out) {
    return guard([&] {
        if (!ctx || !desc || !out) fail(MSC_E_INVALID, "null pointer");
        *out = nullptr;
        const msc_slab_desc& d = *desc;
        if (d.world < 1 || d.rank < 0 || d.rank >= d.world) fail(MSC_E_INVALID, "bad rank / world");
        if (d.channels != 128) fail(MSC_E_UNSUPPORTED, "slab residual stacks run at 128 channels");
        if (d.n_owned < 0 || d.n_halo_lo < 0 || d.n_halo_hi < 0 || d.n_local != d.n_owned + d.n_halo_lo + d.n_halo_hi)
            fail(MSC_E_INVALID, "n_local must be n_owned + n_halo_lo + n_halo_hi");
        if (d.send_lo < 0 || d.send_hi < 0 || d.send_lo > d.n_owned || d.send_hi > d.n_owned)
            fail(MSC_E_INVALID, "send ranges out of the owned rows");
        if ((d.rank == 0 && (d.n_halo_lo || d.send_lo)) || (d.rank == d.world - 1 && (d.n_halo_hi || d.send_hi)))
            fail(MSC_E_INVALID, "the outermost ranks have no neighbour on that side");
        if (d.n_local >= (int64_t(1) << 31) / 27) fail(MSC_E_INVALID, "too many local rows");
        int dev = -1;
        cuda(cudaGetDevice(&dev), "cudaGetDevice");
        if (dev != ctx_device(ctx)) fail(MSC_E_INVALID, "the context belongs to another device");
        auto* s = new msc_slab();
        try {
            s->ctx = ctx;
            s->d = d;
            const size_t xb = align256(static_cast<size_t>(d.n_local ? d.n_local : 1) * d.channels * 2);
            for (int i = 0; i < 2; ++i) {
                cuda(cudaMalloc(&s->x[i], xb), "feature buffer");
                cuda(cudaMemset(s->x[i], 0, xb), "feature buffer clear");
            }
            cuda(cudaMalloc(&s->flags, 256), "flag allocation");
            cuda(cudaMemset(s->flags, 0, 256), "flag clear");
        } catch (...) {
            delete s;
            throw;
        }
        *out = s;
    });
}

int msc_slab_destroy(msc_slab_t s) {
    return guard([&] { delete s; });
}

int msc_slab_get_handle(msc_slab_t s, msc_slab_handle* out) {
    return guard([&] {
        if (!s || !out) fail(MSC_E_INVALID, "null pointer");
        Handle h{};
        h.magic = kHandleMagic;
        h.rank = s->d.rank, h.world = s->d.world, h.channels = s->d.channels;
        h.n_local = s->d.n_local, h.n_owned = s->d.n_owned, h.n_halo_lo = s->d.n_halo_lo;
        h.n_halo_hi = s->d.n_halo_hi, h.send_lo = s->d.send_lo, h.send_hi = s->d.send_hi;
        for (int i = 0; i < 2; ++i) cuda(cudaIpcGetMemHandle(&h.x[i], s->x[i]), "feature buffer IPC handle");
        cuda(cudaIpcGetMemHandle(&h.flags, s->flags), "flag IPC handle");
        std::memset(out, 0, sizeof(*out));
        std::memcpy(out, &h, sizeof(h));
    });
}

int msc_slab_connect(msc_slab_t s, const msc_slab_handle* lower, const msc_slab_handle* upper) {
    return guard([&] {
        if (!s) fail(MSC_E_INVALID, "null slab");
        const msc_slab_desc& d = s->d;
        if ((d.rank > 0) != (lower != nullptr) || (d.rank < d.world - 1) != (upper != nullptr))
            fail(MSC_E_INVALID, "a rank connects to exactly the neighbours it has");
        auto open = [&](const msc_slab_handle* raw, msc_slab::Peer& p, int want_rank, bool is_lower) {
            Handle h;
            std::memcpy(&h, raw, sizeof(h));
            if (h.magic != kHandleMagic || h.rank != want_rank || h.world != d.world || h.channels != d.channels)
                fail(MSC_E_INVALID, "neighbour handle does not belong to rank " + std::to_string(want_rank));
            // my first send_lo owned rows are the lower neighbour's halo above;
            // my last send_hi owned rows the upper neighbour's halo below
            if (is_lower && h.n_halo_hi != d.send_lo)
                fail(MSC_E_INVALID, "lower neighbour's halo above does not match send_lo");
            if (!is_lower && h.n_halo_lo != d.send_hi)
                fail(MSC_E_INVALID, "upper neighbour's halo below does not match send_hi");
            p.off = is_lower ? h.n_owned + h.n_halo_lo : h.n_owned;
            for (int i = 0; i < 2; ++i)
                cuda(cudaIpcOpenMemHandle(&p.x[i], h.x[i], cudaIpcMemLazyEnablePeerAccess), "open neighbour buffer");
            void* f = nullptr;
            cuda(cudaIpcOpenMemHandle(&f, h.flags, cudaIpcMemLazyEnablePeerAccess), "open neighbour flags");
            p.flags = static_cast<int*>(f);
        };
        if (lower) open(lower, s->lo, d.rank - 1, true);
        if (upper) open(upper, s->hi, d.rank + 1, false);
    });
}

int msc_slab_set_level(msc_slab_t s, const int32_t* coords, void* stream) {
    return guard([&] {
        if (!s || !coords) fail(MSC_E_INVALID, "null pointer");
        if (reinterpret_cast<uintptr_t>(coords) % 16) fail(MSC_E_INVALID, "coords is not 16-byte aligned");
        cudaStream_t st = static_cast<cudaStream_t>(stream);
        const int64_t n = s->d.n_local, no = s->d.n_owned;
        const int c = s->d.channels;
        if (!s->nbr) {
            cuda(cudaMalloc(&s->nbr, static_cast<size_t>(n ? n : 1) * 27 * 4), "neighbour map");
            cuda(cudaMalloc(&s->plan_all, plan_bytes(n)), "plan");
            cuda(cudaMalloc(&s->plan_own, plan_bytes(no)), "plan");
            size_t w = topology_workspace_bytes(n);
            w = w > plan_workspace_bytes(n) ? w : plan_workspace_bytes(n);
            // operand planes (int8 codes + scales) and conv1's fused Q8_0 output
            const size_t op = 2 * (align256(act_bytes(ACT_Q8I, n, c)) + 256);
            s->ws_bytes = w > op ? w : op;
            cuda(cudaMalloc(&s->ws, s->ws_bytes), "slab workspace");
        }
        if (n == 0) {
            s->level = true;
            return;
        }
        void* t = prof_begin(s->ctx, "make_level", st);
        cuda(launch_make_level(coords, n, s->nbr, s->ws, ctx_status(s->ctx), st), "make_level");
        prof_end(s->ctx, t, st);
        t = prof_begin(s->ctx, "plan_build", st);
        cuda(launch_plan_build(s->nbr, n, n, s->plan_all, s->ws, st), "plan (all rows)");
        cuda(launch_plan_build(s->nbr, no, n, s->plan_own, s->ws, st), "plan (owned rows)");
        prof_end(s->ctx, t, st);
        s->level = true;
    });
}

int msc_slab_put_features(msc_slab_t s, const void* x, void* stream) {
    return guard([&] {
        if (!s || !x) fail(MSC_E_INVALID, "null pointer");
        const size_t b = static_cast<size_t>(s->d.n_local) * s->d.channels * 2;
        if (b)
            cuda(cudaMemcpyAsync(s->x[s->cur], x, b, cudaMemcpyDeviceToDevice, static_cast<cudaStream_t>(stream)),
                 "feature copy");
    });
}

int msc_slab_get_features(msc_slab_t s, void* owned_out, void* stream) {
    return guard([&] {
        if (!s || !owned_out) fail(MSC_E_INVALID, "null pointer");
        const size_t b = static_cast<size_t>(s->d.n_owned) * s->d.channels * 2;
        if (b)
            cuda(cudaMemcpyAsync(owned_out, s->x[s->cur], b, cudaMemcpyDefault, static_cast<cudaStream_t>(stream)),
                 "feature copy");
    });
}

int msc_slab_features_ptr(msc_slab_t s, void** x) {
    return guard([&] {
        if (!s || !x) fail(MSC_E_INVALID, "null pointer");
        *x = s->x[s->cur];
    });
}

int msc_slab_res_block(msc_slab_t s, const float* norm_w, const float* norm_b, const void* blob1, const float* b1,
                       const void* blob2, const float* b2, void* stream) {
    return guard([&] {
        if (!s) fail(MSC_E_INVALID, "null slab");
        if (!s->level) fail(MSC_E_INVALID, "msc_slab_set_level has not been called");
        const msc_slab_desc& d = s->d;
        const int c = d.channels;
        for (const void* blob : {blob1, blob2}) {
            int wt, ci, co, nt, pl;
            if (!blob || !blob_shape(s->ctx, blob, &wt, &ci, &co, &nt, &pl))
                fail(MSC_E_INVALID, "weight blob was not prepared by this context");
            if (wt != MSC_W_Q8_0 || ci != c || co != c || nt != 27)
                fail(MSC_E_UNSUPPORTED, "slab residual blocks take Q8_0 sparse27 weights c -> c");
        }
        if ((d.rank > 0 && !s->lo.flags) || (d.rank < d.world - 1 && !s->hi.flags))
            fail(MSC_E_INVALID, "msc_slab_connect has not been called");
        cudaStream_t st = static_cast<cudaStream_t>(stream);
        uint32_t* status = ctx_status(s->ctx);
        const int64_t n = d.n_local;
        const int k = s->done;
        if (k > 0 && d.world > 1) {
            void* t = prof_begin(s->ctx, "halo_wait", st);
            slab_wait_kernel<<<1, 32, 0, st>>>(s->flags, d.rank > 0, d.rank < d.world - 1, k, status, kWaitNs);
            cuda(cudaGetLastError(), "halo wait");
            prof_end(s->ctx, t, st);
        }
        void* xin = s->x[s->cur];
        void* xout = s->x[1 - s->cur];
        if (n > 0) {
            uint8_t* planes = static_cast<uint8_t*>(s->ws);
            uint8_t* h = planes + align256(act_bytes(ACT_Q8I, n, c)) + 256;
            void* t = prof_begin(s->ctx, "act_prepare", st);
            cuda(launch_act_prepare(xin, DT_F16, n, c, 1, norm_w, norm_b, 1e-6f, 1, ACT_Q8I, planes, st),
                 "norm1 prepare");
            prof_end(s->ctx, t, st);
            auto conv = [&](const void* src, const void* blob, const float* bias, const void* plan, int64_t rows) {
                ConvArgs a{};
                a.planes = src;
                a.a_scale = reinterpret_cast<const float*>(static_cast<const uint8_t*>(src) +
                                                           act_scale_offset(ACT_Q8I, n, c));
                a.na = 1, a.q8 = 1, a.i8 = 1;
                a.n_in = n;
                a.n = rows;
                const PlanTiles T = plan_tiles(static_cast<uint8_t*>(const_cast<void*>(plan)), rows);
                a.perm = T.order, a.tile_rows = T.rows, a.tile_nbr = T.nbr, a.tile_mask = T.mask, a.tile_sched = T.sched;
                a.cin = c, a.nbr = s->nbr, a.blob = blob, a.wplanes = 1, a.cout = c, a.ntaps = 27;
                a.bias = bias;
                a.status = status;
                return a;
            };
            // conv1 over all local rows, SiLU, conv2's Q8_0 operand fused in
            ConvArgs a1 = conv(planes, blob1, b1, s->plan_all, n);
            a1.silu_out = 1;
            a1.y = h, a1.y_dtype = DT_F32;
            a1.q_codes = reinterpret_cast<int8_t*>(h);
            a1.q_scales = reinterpret_cast<float*>(h + act_scale_offset(ACT_Q8I, n, c));
            t = prof_begin(s->ctx, "conv_tc", st);
            cuda(launch_conv(a1, st), "conv1");
            prof_end(s->ctx, t, st);
            // conv2 over the owned rows into the other buffer, boundary rows
            // also into the neighbours' halo rows
            if (d.n_owned > 0) {
                ConvArgs a2 = conv(h, blob2, b2, s->plan_own, d.n_owned);
                a2.residual = xin, a2.res_dtype = DT_F16;
                a2.y = xout, a2.y_dtype = DT_F16;
                a2.store_limit = d.n_owned;
                a2.peer_lo = s->lo.x[1 - s->cur], a2.peer_lo_off = s->lo.off, a2.send_lo = d.send_lo;
                a2.peer_hi = s->hi.x[1 - s->cur], a2.peer_hi_off = s->hi.off, a2.send_hi_begin = d.n_owned - d.send_hi;
                t = prof_begin(s->ctx, "conv_tc", st);
                cuda(launch_conv(a2, st), "conv2");
                prof_end(s->ctx, t, st);
            }
        }
        if (d.world > 1) {
            slab_signal_kernel<<<1, 32, 0, st>>>(s->lo.flags ? s->lo.flags + 1 : nullptr,
                                                 s->hi.flags ? s->hi.flags : nullptr, k + 1);
            cuda(cudaGetLastError(), "halo signal");
        }
        s->cur ^= 1;
        ++s->done;
    });
}

int msc_wait_probe(msc_ctx_t ctx, int64_t budget_us, void* stream) {
    return guard([&] {
        if (!ctx) fail(MSC_E_INVALID, "null context");
        if (budget_us < 0 || budget_us > 2000000) fail(MSC_E_INVALID, "budget must be in [0, 2 s]");
        cudaStream_t st = static_cast<cudaStream_t>(stream);
        int* flag = nullptr;
        cuda(cudaMallocAsync(reinterpret_cast<void**>(&flag), 256, st), "probe flag");
        cuda(cudaMemsetAsync(flag, 0, 256, st), "probe flag clear");
        // a flag nothing sets: the wait runs out and reports MSC_DEV_TIMEOUT
        slab_wait_kernel<<<1, 32, 0, st>>>(flag, 1, 1, 1, ctx_status(ctx),
                                           static_cast<unsigned long long>(budget_us) * 1000ull);
        cuda(cudaGetLastError(), "probe wait");
        cuda(cudaFreeAsync(flag, st), "probe flag free");
    });
}

}  // extern "C"
