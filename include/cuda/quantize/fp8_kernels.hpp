// fp8_kernels.hpp -- drop-in for pplmx/nova include/cuda/quantize/fp8_kernels.hpp
// (signatures of :30-59), implemented by libnova_q (nova_q.h).
#ifndef NOVA_B200_FP8_KERNELS_HPP
#define NOVA_B200_FP8_KERNELS_HPP

#include <cuda_runtime.h>

#include <cstddef>

#include "fp8_types.hpp"
#include "nq_check.hpp"

namespace nova {
namespace quantize {
namespace cuda {

inline void quantize_f32_to_fp8e4m3(const float* src, FP8E4M3* dst, size_t n, cudaStream_t stream = 0) {
    detail::nq_report(nq_quantize_f32_to_fp8e4m3(src, reinterpret_cast<uint8_t*>(dst), n, stream),
                      "quantize_f32_to_fp8e4m3");
}
inline void quantize_f32_to_fp8e5m2(const float* src, FP8E5M2* dst, size_t n, cudaStream_t stream = 0) {
    detail::nq_report(nq_quantize_f32_to_fp8e5m2(src, reinterpret_cast<uint8_t*>(dst), n, stream),
                      "quantize_f32_to_fp8e5m2");
}
inline void dequantize_fp8e4m3_to_f32(const FP8E4M3* src, float* dst, size_t n, float scale, cudaStream_t stream = 0) {
    detail::nq_report(nq_dequantize_fp8e4m3_to_f32(reinterpret_cast<const uint8_t*>(src), dst, n, scale, stream),
                      "dequantize_fp8e4m3_to_f32");
}
inline void dequantize_fp8e5m2_to_f32(const FP8E5M2* src, float* dst, size_t n, float scale, cudaStream_t stream = 0) {
    detail::nq_report(nq_dequantize_fp8e5m2_to_f32(reinterpret_cast<const uint8_t*>(src), dst, n, scale, stream),
                      "dequantize_fp8e5m2_to_f32");
}
inline void quantize_batched_f32_to_fp8e4m3(const float** src, FP8E4M3** dst, int batch_size, const size_t* sizes,
                                            const float* scales, cudaStream_t stream = 0) {
    detail::nq_report(nq_quantize_batched_f32_to_fp8e4m3(src, reinterpret_cast<uint8_t* const*>(dst), batch_size,
                                                         sizes, scales, stream),
                      "quantize_batched_f32_to_fp8e4m3");
}
inline void dequantize_batched_fp8e4m3_to_f32(const FP8E4M3** src, float** dst, int batch_size, const size_t* sizes,
                                              const float* scales, cudaStream_t stream = 0) {
    detail::nq_report(nq_dequantize_batched_fp8e4m3_to_f32(reinterpret_cast<const uint8_t* const*>(src), dst,
                                                           batch_size, sizes, scales, stream),
                      "dequantize_batched_fp8e4m3_to_f32");
}

}  // namespace cuda
}  // namespace quantize
}  // namespace nova

#endif
