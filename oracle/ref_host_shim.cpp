// C entry points over the reference's own host code (pplmx/nova headers,
// compiled from the reference tree by oracle/Makefile).  Used only to pin the
// oracle restatement and as the timed CPU reference arm.
#include <cuda/quantize/fp8_types.hpp>
#include <cuda/quantize/quantize_tensor.hpp>
#include <cuda/quantize/quantize_ops.hpp>

#include <cstdint>
#include <cstring>

using namespace nova::quantize;

extern "C" {

uint8_t ref_e4m3_encode(float f) { return FP8E4M3(f).to_bits(); }
float ref_e4m3_decode(uint8_t b) { return static_cast<float>(FP8E4M3::from_bits(b)); }
uint8_t ref_e5m2_encode(float f) { return FP8E5M2(f).to_bits(); }
float ref_e5m2_decode(uint8_t b) { return static_cast<float>(FP8E5M2::from_bits(b)); }

void ref_e4m3_encode_array(const float* src, uint8_t* dst, size_t n) {
    for (size_t i = 0; i < n; ++i) dst[i] = FP8E4M3(src[i]).to_bits();
}

// QuantizedTensor<int8_t>::FromFloat (quantize_tensor.hpp:160-191)
int ref_from_float_int8(const float* data, size_t n, float scale, int8_t* q, float* scale_out) {
    auto t = QuantizedTensor<int8_t>::FromFloat(data, n, scale);
    if (!t) return 0;
    std::memcpy(q, t->data(), n);
    *scale_out = t->metadata().scale;
    return 1;
}

// QuantizedMatmul::forward (quantize_ops.hpp:54-81)
void ref_quantized_matmul(const int8_t* a, const int8_t* b, int8_t* out, int m, int k, int n,
                          float sa, float sb) {
    QuantizationMetadata ma{QuantizationMode::PerTensor, sa, 0.0f, 8};
    QuantizationMetadata mb{QuantizationMode::PerTensor, sb, 0.0f, 8};
    QuantizedInt8 qa(std::vector<int8_t>(a, a + (size_t)m * k), ma, {m, k});
    QuantizedInt8 qb(std::vector<int8_t>(b, b + (size_t)k * n), mb, {k, n});
    QuantizedInt8 qc;
    QuantizedMatmul::forward(qa, qb, qc, m, k, n);
    std::memcpy(out, qc.data(), (size_t)m * n);
}

}  // extern "C"
