// C entry point over the reference's calibrator cache I/O (calibrator.cpp of
// pplmx/nova, compiled from the reference tree by oracle/Makefile into
// _ref/libnova_ref_calib.so).  Pinning only: a cache file is loaded and saved
// again by the reference's own MinMax / Histogram / MSE / PerChannel
// calibrators.
#include <cuda/quantize/calibrator.hpp>

#include <cstdlib>

namespace nova {
namespace quantize {
namespace cuda {
// calibrator.cpp refers to the device reductions (int8_kernels.cu); the cache
// round trips never calibrate, so these are never called.
void build_histogram(const float*, uint32_t*, size_t, float, float, int, cudaStream_t) { std::abort(); }
void compute_minmax(const float*, size_t, float*, float*, cudaStream_t) { std::abort(); }
}  // namespace cuda
}  // namespace quantize
}  // namespace nova

extern "C" int ref_calib_cache_roundtrip(int kind, const char* in, const char* out) {
    using namespace nova::quantize;
    switch (kind) {
        case 0: { MinMaxCalibrator c(true); c.load_cache(in); c.save_cache(out); return 0; }
        case 1: { HistogramCalibrator c; c.load_cache(in); c.save_cache(out); return 0; }
        case 2: { MSECalibrator c; c.load_cache(in); c.save_cache(out); return 0; }
        case 3: { PerChannelCalibrator c(0); c.load_cache(in); c.save_cache(out); return 0; }
        default: return -1;
    }
}
