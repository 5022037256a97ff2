// Calibrator cache files through the drop-in header (calibrator.hpp): load a
// cache and save it again, for the cross-check against the reference's own
// calibrator.cpp (tests/test_cpp_calib.py).  No GPU needed.
//   test_calib <kind> <in> <out>   kind 0 MinMax, 1 Histogram, 2 MSE, 3 PerChannel
#include <cuda/quantize/calibrator.hpp>

#include <cstdio>
#include <cstdlib>

using namespace nova::quantize;

int main(int argc, char** argv) {
    if (argc != 4) {
        std::fprintf(stderr, "usage: test_calib <kind> <in> <out>\n");
        return 2;
    }
    switch (std::atoi(argv[1])) {
        case 0: { MinMaxCalibrator c(true); c.load_cache(argv[2]); c.save_cache(argv[3]); break; }
        case 1: { HistogramCalibrator c; c.load_cache(argv[2]); c.save_cache(argv[3]); break; }
        case 2: { MSECalibrator c; c.load_cache(argv[2]); c.save_cache(argv[3]); break; }
        case 3: { PerChannelCalibrator c(0); c.load_cache(argv[2]); c.save_cache(argv[3]); break; }
        default: return 2;
    }
    return 0;
}
