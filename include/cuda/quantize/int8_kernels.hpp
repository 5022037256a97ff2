// int8_kernels.hpp -- drop-in for pplmx/nova include/cuda/quantize/int8_kernels.hpp
// (QuantizationParams :28-49 and the functions :51-92), over libnova_q.
#ifndef NOVA_B200_INT8_KERNELS_HPP
#define NOVA_B200_INT8_KERNELS_HPP

#include <cuda_runtime.h>

#include <cstddef>
#include <cstdint>

#include "nq_check.hpp"

namespace nova {
namespace quantize {
namespace cuda {

struct QuantizationParams {
    float scale{1.0f};
    float zero_point{0.0f};
    bool symmetric{true};

    QuantizationParams() = default;
    QuantizationParams(float s, float zp = 0.0f, bool sym = true) : scale(s), zero_point(zp), symmetric(sym) {}
};

inline void quantize_f32_to_int8(const float* src, int8_t* dst, size_t n, QuantizationParams params,
                                 cudaStream_t stream = 0) {
    detail::nq_report(nq_quantize_f32_to_int8(src, dst, n, params.scale, params.zero_point, params.symmetric, stream),
                      "quantize_f32_to_int8");
}
inline void dequantize_int8_to_f32(const int8_t* src, float* dst, size_t n, QuantizationParams params,
                                   cudaStream_t stream = 0) {
    detail::nq_report(nq_dequantize_int8_to_f32(src, dst, n, params.scale, params.zero_point, params.symmetric, stream),
                      "dequantize_int8_to_f32");
}
inline void quantize_f32_to_int8_async(const float* src, int8_t* dst, size_t n, QuantizationParams params,
                                       cudaStream_t stream = 0) {
    quantize_f32_to_int8(src, dst, n, params, stream);
}
inline void dequantize_int8_to_f32_async(const int8_t* src, float* dst, size_t n, QuantizationParams params,
                                         cudaStream_t stream = 0) {
    dequantize_int8_to_f32(src, dst, n, params, stream);
}
inline void quantize_f32_to_int8_with_calibration(const float* src, int8_t* dst, size_t n, float min_val,
                                                  float max_val, cudaStream_t stream = 0) {
    detail::nq_report(nq_quantize_f32_to_int8_with_calibration(src, dst, n, min_val, max_val, stream),
                      "quantize_f32_to_int8_with_calibration");
}
// Host or device `data`; synchronises `stream`.  Any num_bins in [1, 65536].
inline void build_histogram(const float* data, uint32_t* histogram, size_t n, float min_val, float max_val,
                            int num_bins = 256, cudaStream_t stream = 0) {
    detail::nq_throw_if(nq_build_histogram(data, histogram, n, min_val, max_val, num_bins, stream), "build_histogram");
}
// Host or device `data` and outputs; synchronises `stream`.
inline void compute_minmax(const float* data, size_t n, float* min_val, float* max_val, cudaStream_t stream = 0) {
    detail::nq_throw_if(nq_compute_minmax(data, n, min_val, max_val, stream), "compute_minmax");
}

}  // namespace cuda
}  // namespace quantize
}  // namespace nova

#endif
