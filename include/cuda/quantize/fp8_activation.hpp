// fp8_activation.hpp -- drop-in for pplmx/nova include/cuda/quantize/fp8_activation.hpp
// (activation:: device functions :26-59, kernels :62-98, host launchers and
// scalar helpers :100-170), element-wise activations on FP8 codes of the
// reference codec: decode, activate in fp32, re-encode.
//
// The host launchers run libnova_q's kernel (nq_fp8_activation: 16 codes per
// thread step instead of one thread per element, same arithmetic); the
// activation:: functions are __host__ __device__ here (device-only in the
// reference), so the *_scalar helpers also work on the host.
#ifndef NOVA_B200_FP8_ACTIVATION_HPP
#define NOVA_B200_FP8_ACTIVATION_HPP

#include <cuda_runtime.h>

#include <cmath>
#include <cstddef>

#include "fp8_types.hpp"
#include "nq_check.hpp"

namespace nova {
namespace quantize {
namespace cuda {

namespace activation {

NOVA_HD inline float sigmoidf(float x) { return 1.0f / (1.0f + expf(-x)); }

NOVA_HD inline float geluf(float x) {
    const float cdf = 0.5f * (1.0f + erff(x * 0.7071067811865476f));
    return x * cdf;
}

template <typename T>
NOVA_HD inline T relu_fp8(T x) {
    return static_cast<float>(x) < 0.0f ? T(0.0f) : x;
}
template <typename T>
NOVA_HD inline T gelu_fp8(T x) {
    return T(geluf(static_cast<float>(x)));
}
template <typename T>
NOVA_HD inline T sigmoid_fp8(T x) {
    return T(sigmoidf(static_cast<float>(x)));
}
template <typename T>
NOVA_HD inline T leaky_relu_fp8(T x, float alpha = 0.01f) {
    const float f = static_cast<float>(x);
    return T(f >= 0.0f ? f : alpha * f);
}

}  // namespace activation

#ifdef __CUDACC__
// one element per thread, as the reference's kernels (for callers that launch them)
template <typename T>
__global__ void relu_kernel(const T* input, T* output, size_t n) {
    const size_t i = static_cast<size_t>(blockIdx.x) * blockDim.x + threadIdx.x;
    if (i < n) output[i] = activation::relu_fp8(input[i]);
}
template <typename T>
__global__ void gelu_kernel(const T* input, T* output, size_t n) {
    const size_t i = static_cast<size_t>(blockIdx.x) * blockDim.x + threadIdx.x;
    if (i < n) output[i] = activation::gelu_fp8(input[i]);
}
template <typename T>
__global__ void sigmoid_kernel(const T* input, T* output, size_t n) {
    const size_t i = static_cast<size_t>(blockIdx.x) * blockDim.x + threadIdx.x;
    if (i < n) output[i] = activation::sigmoid_fp8(input[i]);
}
template <typename T>
__global__ void leaky_relu_kernel(const T* input, T* output, size_t n, float alpha) {
    const size_t i = static_cast<size_t>(blockIdx.x) * blockDim.x + threadIdx.x;
    if (i < n) output[i] = activation::leaky_relu_fp8(input[i], alpha);
}
#endif

namespace act_detail {
template <typename T>
struct Fp8Format;
template <>
struct Fp8Format<FP8E4M3> {
    static constexpr nq_format_t value = NQ_E4M3;
};
template <>
struct Fp8Format<FP8E5M2> {
    static constexpr nq_format_t value = NQ_E5M2;
};
template <typename T>
inline void run_activation(const T* input, T* output, size_t n, nq_activation_t op, float alpha, cudaStream_t s,
                           const char* what) {
    nova::quantize::detail::nq_report(nq_fp8_activation(reinterpret_cast<const uint8_t*>(input),
                                                        reinterpret_cast<uint8_t*>(output), n, Fp8Format<T>::value,
                                                        op, alpha, s),
                                      what);
}
}  // namespace act_detail

// Device arrays, asynchronous on `stream`; errors are printed, as in the reference.
template <typename T>
void relu(const T* input, T* output, size_t n, cudaStream_t stream = 0) {
    act_detail::run_activation(input, output, n, NQ_ACT_RELU, 0.0f, stream, "relu");
}
template <typename T>
void gelu(const T* input, T* output, size_t n, cudaStream_t stream = 0) {
    act_detail::run_activation(input, output, n, NQ_ACT_GELU, 0.0f, stream, "gelu");
}
template <typename T>
void sigmoid(const T* input, T* output, size_t n, cudaStream_t stream = 0) {
    act_detail::run_activation(input, output, n, NQ_ACT_SIGMOID, 0.0f, stream, "sigmoid");
}
template <typename T>
void leaky_relu(const T* input, T* output, size_t n, float alpha = 0.01f, cudaStream_t stream = 0) {
    act_detail::run_activation(input, output, n, NQ_ACT_LEAKY_RELU, alpha, stream, "leaky_relu");
}

template <typename T>
T relu_fp8_scalar(T x) {
    return activation::relu_fp8(x);
}
template <typename T>
T gelu_fp8_scalar(T x) {
    return activation::gelu_fp8(x);
}

}  // namespace cuda
}  // namespace quantize
}  // namespace nova

#endif  // NOVA_B200_FP8_ACTIVATION_HPP
