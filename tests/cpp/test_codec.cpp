// Host side of the drop-in FP8 classes (include/cuda/quantize/fp8_types.hpp):
// reads little-endian float32 values from stdin and writes, per value, the
// FP8E4M3 and FP8E5M2 codes (two bytes) to stdout; then the decoded float of
// each of the 256 codes of both formats (2 x 256 float32).  No GPU needed.
#include <cuda/quantize/fp8_types.hpp>

#include <cstdio>
#include <vector>

using namespace nova::quantize;

int main() {
    std::vector<float> x;
    float v;
    while (std::fread(&v, sizeof(float), 1, stdin) == 1) x.push_back(v);
    for (float f : x) {
        const uint8_t c[2] = {FP8E4M3(f).to_bits(), FP8E5M2(f).to_bits()};
        std::fwrite(c, 1, 2, stdout);
    }
    for (int c = 0; c < 256; ++c) {
        const float d = static_cast<float>(FP8E4M3::from_bits(static_cast<uint8_t>(c)));
        std::fwrite(&d, sizeof(float), 1, stdout);
    }
    for (int c = 0; c < 256; ++c) {
        const float d = static_cast<float>(FP8E5M2::from_bits(static_cast<uint8_t>(c)));
        std::fwrite(&d, sizeof(float), 1, stdout);
    }
    return 0;
}
