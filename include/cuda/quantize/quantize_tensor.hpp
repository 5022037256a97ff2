// quantize_tensor.hpp -- drop-in for pplmx/nova include/cuda/quantize/quantize_tensor.hpp
// (QuantizationMode :45, QuantizationMetadata :52-64, float16 :71-126,
// QuantizedTensor :128-231).
//
// QuantizedTensor keeps host vectors, as in the reference.  FromFloat for int8
// runs on the GPU: the input is staged to device memory, the amax comes from
// the library's reduction, and the codes from nq_quantize_f32_to_int8_round_away
// (std::round semantics, quantize_tensor.hpp:176-182), so the codes and scale
// equal the reference's host loop.  The float16 type keeps the reference's
// truncating conversion (no rounding, no subnormals) because it is part of the
// stored format.
#ifndef NOVA_B200_QUANTIZE_TENSOR_HPP
#define NOVA_B200_QUANTIZE_TENSOR_HPP

#include <cuda_runtime.h>

#include <cmath>
#include <cstdint>
#include <optional>
#include <type_traits>
#include <vector>

#include "nq_check.hpp"

namespace nova {
namespace quantize {

enum class QuantizationMode { PerTensor, PerChannel };

struct QuantizationMetadata {
    QuantizationMode mode;
    float scale;
    float zero_point;
    int num_bits;
};

// The reference's 16-bit float: exponent = frexp exponent + 15, mantissa
// truncated to 10 bits, zero for exponents <= 0, Inf for >= 31.
struct alignas(2) float16 {
    uint16_t value;

    float16() = default;
    explicit float16(float f) {
        if (f == 0.0f) {
            value = 0;
            return;
        }
        const bool negative = f < 0;
        f = std::abs(f);
        int e;
        float m = std::frexp(f, &e);
        e += 15;
        if (e <= 0) {
            value = negative ? 0x8000 : 0;
            return;
        }
        if (e >= 31) {
            value = negative ? 0xFC00 : 0x7C00;
            return;
        }
        m = (m * 2.0f - 1.0f) * 1024.0f;
        value = static_cast<uint16_t>((negative ? 0x8000 : 0) | (static_cast<uint16_t>(e) << 10) |
                                      static_cast<uint16_t>(m));
    }
    operator float() const {
        if (value == 0) return 0.0f;
        const int e = static_cast<int>((value & 0x7C00) >> 10) - 15;
        const float m = 1.0f + static_cast<float>(value & 0x03FF) / 1024.0f;
        const float r = m * std::ldexp(1.0f, e);
        return (value & 0x8000) ? -r : r;
    }
};

template <typename T>
class QuantizedTensor {
public:
    QuantizedTensor() = default;
    QuantizedTensor(std::vector<T> data, QuantizationMetadata meta, std::vector<int> shape)
        : data_(std::move(data)), metadata_(meta), shape_(std::move(shape)) {}

    static std::optional<QuantizedTensor<int8_t>> FromFloat(const float* data, size_t size, float scale = 0.0f);
    static std::optional<QuantizedTensor<float16>> FromFloat(const float* data, size_t size);

    std::vector<float> ToFloat() const {
        std::vector<float> r(size());
        if constexpr (std::is_same_v<T, int8_t>) {
            for (size_t i = 0; i < size(); ++i) r[i] = static_cast<float>(data_[i]) * metadata_.scale;
        } else if constexpr (std::is_same_v<T, float16>) {
            for (size_t i = 0; i < size(); ++i) r[i] = static_cast<float>(data_[i]);
        }
        return r;
    }

    const T* data() const { return data_.data(); }
    T* data() { return data_.data(); }
    const QuantizationMetadata& metadata() const { return metadata_; }
    const std::vector<int>& shape() const { return shape_; }
    size_t size() const { return data_.size(); }

private:
    std::vector<T> data_;
    QuantizationMetadata metadata_{};
    std::vector<int> shape_;
};

using QuantizedInt8 = QuantizedTensor<int8_t>;
using QuantizedFP16 = QuantizedTensor<float16>;

namespace detail {
// FromFloat<int8_t> on the GPU (quantize_tensor.hpp:160-191 semantics).
inline std::optional<QuantizedTensor<int8_t>> from_float_int8(const float* data, size_t size, float scale) {
    if (size == 0) return std::nullopt;
    cudaStream_t s = 0;
    float* d_x = nullptr;
    int8_t* d_q = nullptr;
    float* d_as = nullptr;
    auto ok = [](cudaError_t e) { return e == cudaSuccess ? NQ_SUCCESS : NQ_ERROR_CUDA; };
    nq_status_t st = ok(cudaMallocAsync(reinterpret_cast<void**>(&d_x), size * sizeof(float), s));
    if (st == NQ_SUCCESS) st = ok(cudaMallocAsync(reinterpret_cast<void**>(&d_q), size, s));
    if (st == NQ_SUCCESS) st = ok(cudaMallocAsync(reinterpret_cast<void**>(&d_as), 2 * sizeof(float), s));
    if (st == NQ_SUCCESS) st = ok(cudaMemcpyAsync(d_x, data, size * sizeof(float), cudaMemcpyHostToDevice, s));
    if (st == NQ_SUCCESS && scale <= 0.0f) {
        float h[2] = {0.0f, 0.0f};
        st = nq_amax_scale_async(d_x, NQ_F32, size, NQ_INT8, d_as, s);
        if (st == NQ_SUCCESS) st = ok(cudaMemcpyAsync(h, d_as, sizeof(h), cudaMemcpyDeviceToHost, s));
        if (st == NQ_SUCCESS) st = ok(cudaStreamSynchronize(s));
        scale = h[0] / 127.0f;  // max |x| / 127, quantize_tensor.hpp:166-172
    }
    if (scale == 0.0f) scale = 1.0f;
    std::vector<int8_t> q(size);
    if (st == NQ_SUCCESS) st = nq_quantize_f32_to_int8_round_away(d_x, d_q, size, scale, s);
    if (st == NQ_SUCCESS) st = ok(cudaMemcpyAsync(q.data(), d_q, size, cudaMemcpyDeviceToHost, s));
    if (d_x) cudaFreeAsync(d_x, s);
    if (d_q) cudaFreeAsync(d_q, s);
    if (d_as) cudaFreeAsync(d_as, s);
    if (st == NQ_SUCCESS) st = ok(cudaStreamSynchronize(s));
    nq_throw_if(st, "QuantizedTensor<int8_t>::FromFloat");
    QuantizationMetadata meta{QuantizationMode::PerTensor, scale, 0.0f, 8};
    return QuantizedTensor<int8_t>(std::move(q), meta, {static_cast<int>(size)});
}
inline std::optional<QuantizedTensor<float16>> from_float_fp16(const float* data, size_t size) {
    if (size == 0) return std::nullopt;
    std::vector<float16> q(size);
    for (size_t i = 0; i < size; ++i) q[i] = float16(data[i]);
    QuantizationMetadata meta{QuantizationMode::PerTensor, 1.0f, 0.0f, 16};
    return QuantizedTensor<float16>(std::move(q), meta, {static_cast<int>(size)});
}
}  // namespace detail

template <typename T>
inline std::optional<QuantizedTensor<int8_t>> QuantizedTensor<T>::FromFloat(const float* data, size_t size,
                                                                            float scale) {
    return detail::from_float_int8(data, size, scale);
}
template <typename T>
inline std::optional<QuantizedTensor<float16>> QuantizedTensor<T>::FromFloat(const float* data, size_t size) {
    return detail::from_float_fp16(data, size);
}

}  // namespace quantize
}  // namespace nova

#endif
