// Host-side probe of the C++ seam (include/moge_sparse_cuda.hpp), built and
// run by tests/test_capi_host.py on a machine without an sm_100 GPU:
// Device::create reports the device as unavailable (nullptr, the caller
// keeps its CPU path), C ABI failures surface as moge_cuda::Error with the
// status code and message, and SparseConfig has the reference's defaults.
#include "moge_sparse_cuda.hpp"

#include <cstdio>
#include <cstring>
#include <vector>

int main() {
    std::unique_ptr<moge_cuda::Device> dev = moge_cuda::Device::create(0);
    std::printf("device %s\n", dev ? "sm100" : "none");

    int code = 0;
    bool names_context = false;
    try {
        moge_cuda::check(msc_make_level(nullptr, nullptr, 0, nullptr, nullptr, 0, nullptr), "make_level");
    } catch (const moge_cuda::Error& e) {
        code = e.code();
        names_context = std::strstr(e.what(), "make_level: ") == e.what() && std::strstr(e.what(), "context");
    }
    std::printf("null_ctx_code %d\n", code);
    std::printf("null_ctx_message %d\n", names_context ? 1 : 0);

    moge_cuda::SparseConfig cfg;
    std::printf("default_config %d %d %d %.1f\n", cfg.present ? 1 : 0, cfg.in_channels, cfg.encoder_downsample,
                static_cast<double>(cfg.depth_resolution));

    if (dev) {
        // an sm_100 device: a refiner needs a MOGG image, which this probe
        // does not carry (the msc_refiner_* entry points the seam forwards
        // to run in the GPU tests through the Python binding)
        std::printf("status %u\n", dev->status());
    }
    return 0;
}
