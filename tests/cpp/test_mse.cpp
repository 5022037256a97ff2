// Drop-in MSECalibrator::calibrate (include/cuda/quantize/calibrator.hpp) on a
// file of fp32 values, from host memory or from a device copy; prints the
// CalibrationResult fields as float bit patterns for tests/test_ref_gpu_pin.py.
//   test_mse <data.bin> <symmetric 0|1> <host|device>
#include <cuda/quantize/calibrator.hpp>

#include <cstdio>
#include <cstring>
#include <vector>

int main(int argc, char** argv) {
    if (argc != 4) {
        std::fprintf(stderr, "usage: test_mse <data.bin> <symmetric> <host|device>\n");
        return 2;
    }
    std::FILE* f = std::fopen(argv[1], "rb");
    if (!f) return 2;
    std::vector<float> h;
    float v;
    while (std::fread(&v, sizeof(float), 1, f) == 1) h.push_back(v);
    std::fclose(f);
    const bool device = std::strcmp(argv[3], "device") == 0;
    const float* data = h.data();
    float* d = nullptr;
    if (device) {
        if (cudaMalloc(&d, h.size() * sizeof(float) + 16) != cudaSuccess) return 3;
        cudaMemcpy(d, h.data(), h.size() * sizeof(float), cudaMemcpyHostToDevice);
        data = d;
    }
    nova::quantize::MSECalibrator c(argv[2][0] == '1');
    nova::quantize::CalibrationResult r = c.calibrate(data, h.size(), 0);
    const float out[5] = {r.scale, r.zero_point, r.symmetric ? 1.0f : 0.0f, r.min_val, r.max_val};
    for (float x : out) {
        unsigned u;
        std::memcpy(&u, &x, 4);
        std::printf("%08x ", u);
    }
    std::printf("\n");
    if (d) cudaFree(d);
    return 0;
}
