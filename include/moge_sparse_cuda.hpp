// moge_sparse_cuda.hpp - C++17 seam over the C ABI (header only).
//
// The operator surface mogecpp's host code uses for the sparse refiner
// (src/sparse.hpp:21-66: SparseConfig, SparseRefiner::refine_once) on the
// B200 library, so that the refiner loop of moge::Model::Impl::infer
// (src/moge.cpp:2118-2131) can hand its passes to the device the way it
// hands residual blocks to SparseMetalExecutor (src/sparse_metal.hpp:21-52):
//   * Device::create(device) returns nullptr where the device is not an
//     sm_100 GPU, the SparseMetalExecutor::create convention (its stub
//     reports "unavailable", src/sparse_metal_stub.cpp:18-20); the caller
//     keeps its CPU path;
//   * failures throw moge_cuda::Error (a std::runtime_error, as the
//     reference's operators throw) carrying the C ABI status code and the
//     msc_last_error() text; nothing else of the C ABI leaks.
// Only the C ABI is called: no CUDA header is needed to include this file,
// and the library links the CUDA runtime statically.
#ifndef MOGE_SPARSE_CUDA_HPP
#define MOGE_SPARSE_CUDA_HPP

#include "moge_sparse_cuda.h"

#include <cstddef>
#include <cstdint>
#include <memory>
#include <stdexcept>
#include <string>
#include <utility>
#include <vector>

namespace moge_cuda {

class Error : public std::runtime_error {
public:
    Error(int code, const std::string& what) : std::runtime_error(what), code_(code) {}
    int code() const noexcept { return code_; }

private:
    int code_;
};

// Throws Error for a non-zero C ABI status.
inline void check(int rc, const char* what) {
    if (rc != MSC_OK) throw Error(rc, std::string(what) + ": " + msc_last_error());
}

// One GPU's context (msc_ctx_t): device status word, events, profiling.
class Device {
public:
    static std::unique_ptr<Device> create(int device = 0) {
        msc_ctx_t ctx = nullptr;
        if (msc_create(device, &ctx) != MSC_OK) return nullptr;
        return std::unique_ptr<Device>(new Device(ctx));
    }
    ~Device() { msc_destroy(ctx_); }
    Device(const Device&) = delete;
    Device& operator=(const Device&) = delete;

    msc_ctx_t handle() const noexcept { return ctx_; }

    // Device-side status bits (MSC_DEV_*) raised since the last call, which
    // it clears; throws Error (MSC_E_DEVICE) when any failure bit is set
    // (MSC_DEV_DUP_COORD alone is informational and returned).  Syncs the
    // stream.
    uint32_t status(void* stream = nullptr) const {
        uint32_t bits = 0;
        check(msc_check(ctx_, stream, &bits), "msc_check");
        return bits;
    }

private:
    explicit Device(msc_ctx_t ctx) : ctx_(ctx) {}
    msc_ctx_t ctx_;
};

// moge::SparseConfig (src/sparse.hpp:21-33) as the MOGG image's refiner.*
// metadata gives it (read_sparse_config, src/sparse.cpp:985-1007).
struct SparseConfig {
    bool present = false;
    int in_channels = 3;
    int out_channels = 1;
    int encoder_channels = 0;
    std::vector<int> model_channels;
    std::vector<int> encoder_blocks;
    std::vector<int> decoder_blocks;
    int bottleneck_blocks = 1;
    std::vector<int> downsample_factors;
    int encoder_downsample = 16;
    float depth_resolution = 256.0f;
};

// moge::SparseRefiner (src/sparse.hpp:41-66) on the device: built from the
// MOGG v1 image in host memory (the bytes mogecpp memory-maps), weights
// prepared once; refine_once keeps the reference's arguments without the
// ggml scheduler, and the topology of the previous pass is reused when the
// quantised log-depth bins are unchanged (get_topology_cached,
// src/sparse.cpp:443-472).
class SparseRefiner {
public:
    SparseRefiner(const Device& device, const void* mogg, size_t mogg_bytes, void* stream = nullptr) {
        check(msc_refiner_create(device.handle(), mogg, mogg_bytes, stream, &r_), "msc_refiner_create");
        try {
            read_config();
        } catch (...) {
            msc_refiner_destroy(r_);
            throw;
        }
    }
    ~SparseRefiner() { msc_refiner_destroy(r_); }
    SparseRefiner(const SparseRefiner&) = delete;
    SparseRefiner& operator=(const SparseRefiner&) = delete;

    const SparseConfig& config() const noexcept { return cfg_; }

    // factor_coord: width * height * 3 interleaved (x/z, y/z, log z); only
    // log z is updated.  encoder_feature: host floats, the reference's
    // [C, encoder_width * encoder_height] (C fastest).  Syncs.
    void refine_once(std::vector<float>& factor_coord, int width, int height, const float* encoder_feature,
                     int encoder_width, int encoder_height, void* stream = nullptr) const {
        if (width <= 0 || height <= 0 ||
            factor_coord.size() != static_cast<size_t>(width) * static_cast<size_t>(height) * 3)
            throw Error(MSC_E_INVALID, "refine_once: factor_coord must hold width * height * 3 floats");
        check(msc_refiner_refine_once_host(r_, factor_coord.data(), width, height, encoder_feature, encoder_width,
                                           encoder_height, stream),
              "msc_refiner_refine_once_host");
    }

    // (hits, misses) of the topology cache so far.
    std::pair<uint64_t, uint64_t> cache_stats() const {
        uint64_t hits = 0, misses = 0;
        check(msc_refiner_cache_stats(r_, &hits, &misses), "msc_refiner_cache_stats");
        return {hits, misses};
    }

    // Voxels per level of the cached topology (empty before the first pass).
    std::vector<int64_t> level_sizes() const {
        int64_t sizes[MSC_REFINER_MAX_LEVELS] = {0};
        int count = 0;
        check(msc_refiner_level_sizes(r_, sizes, MSC_REFINER_MAX_LEVELS, &count), "msc_refiner_level_sizes");
        return std::vector<int64_t>(sizes, sizes + count);
    }

private:
    void read_config() {
        msc_sparse_config c{};
        check(msc_refiner_config(r_, &c), "msc_refiner_config");
        cfg_.present = true;
        cfg_.in_channels = c.in_channels;
        cfg_.out_channels = c.out_channels;
        cfg_.encoder_channels = c.encoder_channels;
        const int levels = c.num_levels < 0 ? 0 : (c.num_levels > MSC_REFINER_MAX_LEVELS ? MSC_REFINER_MAX_LEVELS
                                                                                        : c.num_levels);
        cfg_.model_channels.assign(c.model_channels, c.model_channels + levels);
        cfg_.encoder_blocks.assign(c.encoder_blocks, c.encoder_blocks + levels);
        const int inner = levels > 0 ? levels - 1 : 0;
        cfg_.decoder_blocks.assign(c.decoder_blocks, c.decoder_blocks + inner);
        cfg_.downsample_factors.assign(c.downsample_factors, c.downsample_factors + inner);
        cfg_.bottleneck_blocks = c.bottleneck_blocks;
        cfg_.encoder_downsample = c.encoder_downsample;
        cfg_.depth_resolution = c.depth_resolution;
    }

    msc_refiner_t r_ = nullptr;
    SparseConfig cfg_;
};

}  // namespace moge_cuda

#endif  // MOGE_SPARSE_CUDA_HPP
