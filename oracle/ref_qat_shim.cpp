// C entry points over the reference's QAT host code (qat.hpp, qat.cpp of
// pplmx/nova), compiled from the reference tree by oracle/Makefile.  A
// separate translation unit: qat.hpp's Precision enum clashes with the one of
// quantize_ops.hpp (qat.hpp:31-37 vs quantize_ops.hpp:28).  Pinning only.
#include <cuda/quantize/qat.hpp>

#include <cstddef>
#include <string>

using namespace nova::quantize;

extern "C" {

// FakeQuantize::forward (qat.hpp:64-72) element by element
void ref_fake_quantize(const float* src, float* dst, size_t n, float scale, float zero_point) {
    FakeQuantize::Config c;
    c.scale = scale;
    c.zero_point = zero_point;
    FakeQuantize fq(c);
    for (size_t i = 0; i < n; ++i) dst[i] = fq.forward(src[i]);
}

// AMPManager::load_config (qat.cpp:31-62): number of layers read, and the
// precision / scale / zero point / trainable flag of layer `name` (-1 when absent)
int ref_amp_load(const char* path, const char* name, int* precision, float* scale, float* zero_point,
                 int* trainable) {
    AMPManager amp;
    amp.load_config(path);
    const LayerConfig& c = amp.get_config(name);
    if (c.name != name) return -1;
    *precision = static_cast<int>(c.precision);
    *scale = c.scale;
    *zero_point = c.zero_point;
    *trainable = c.trainable ? 1 : 0;
    return static_cast<int>(amp.num_layers());
}

// AMPManager::save_config (qat.cpp:7-29) of two layers, for the reverse check
void ref_amp_save_two(const char* path) {
    AMPManager amp;
    amp.add_layer("attn.qkv", Precision::FP8_E4M3);
    amp.set_scale("attn.qkv", 0.125f);
    amp.add_layer("mlp.down", Precision::INT8);
    amp.set_scale("mlp.down", 0.03125f);
    amp.save_config(path);
}

}  // extern "C"
