// Host side of the FP8 activation drop-in header (fp8_activation.hpp): prints,
// for every one of the 256 codes, the output code of relu / gelu / sigmoid /
// leaky_relu(0.01) through the activation:: functions and the *_scalar
// helpers, E4M3 then E5M2, one line per format and activation.  No GPU needed.
#include <cuda/quantize/fp8_activation.hpp>

#include <cstdio>

using namespace nova::quantize;
namespace act = nova::quantize::cuda::activation;

template <typename T>
static void dump() {
    for (int op = 0; op < 4; ++op) {
        for (int c = 0; c < 256; ++c) {
            const T x = T::from_bits(static_cast<uint8_t>(c));
            T y;
            if (op == 0) y = nova::quantize::cuda::relu_fp8_scalar(x);
            else if (op == 1) y = nova::quantize::cuda::gelu_fp8_scalar(x);
            else if (op == 2) y = act::sigmoid_fp8(x);
            else y = act::leaky_relu_fp8(x, 0.01f);
            std::printf("%d%c", static_cast<int>(y.to_bits()), c == 255 ? '\n' : ' ');
        }
    }
}

int main() {
    dump<FP8E4M3>();
    dump<FP8E5M2>();
    return 0;
}
