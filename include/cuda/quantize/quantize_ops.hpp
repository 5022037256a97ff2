// quantize_ops.hpp -- drop-in for pplmx/nova include/cuda/quantize/quantize_ops.hpp
// (Precision :28, QuantizedMatmul :35-117).
//
// QuantizedMatmul::forward runs the INT8 tcgen05 GEMM (exact int32
// accumulation) with the int8 requantizing epilogue: (float)sum * (sa*sb),
// clamp to +-127, std::round -- the reference host loop's arithmetic
// (:66-77), so outputs are identical.  As in the reference, the output
// carries A's metadata (:80).  mixed_precision runs a GPU kernel with the
// reference's order of operations (:83-102).  Inputs and outputs are host
// memory, as in the reference.
#ifndef NOVA_B200_QUANTIZE_OPS_HPP
#define NOVA_B200_QUANTIZE_OPS_HPP

#include <cuda_runtime.h>

#include <cstring>
#include <vector>

#include "nq_check.hpp"
#include "quantize_tensor.hpp"

namespace nova {
namespace quantize {

enum class Precision { FP32, FP16, INT8 };

class QuantizedMatmul {
public:
    static void forward(const QuantizedInt8& a, const QuantizedInt8& b, QuantizedInt8& output, int m, int k, int n) {
        const size_t na = static_cast<size_t>(m) * k, nb = static_cast<size_t>(k) * n, nc = static_cast<size_t>(m) * n;
        std::vector<int8_t> out(nc);
        if (nc) {
            cudaStream_t s = 0;
            void *d_a = nullptr, *d_b = nullptr, *d_c = nullptr;
            auto ok = [](cudaError_t e) { return e == cudaSuccess ? NQ_SUCCESS : NQ_ERROR_CUDA; };
            nq_status_t st = ok(cudaMallocAsync(&d_a, na ? na : 1, s));
            if (st == NQ_SUCCESS) st = ok(cudaMallocAsync(&d_b, nb ? nb : 1, s));
            if (st == NQ_SUCCESS) st = ok(cudaMallocAsync(&d_c, nc, s));
            if (st == NQ_SUCCESS && na) st = ok(cudaMemcpyAsync(d_a, a.data(), na, cudaMemcpyHostToDevice, s));
            if (st == NQ_SUCCESS && nb) st = ok(cudaMemcpyAsync(d_b, b.data(), nb, cudaMemcpyHostToDevice, s));
            if (st == NQ_SUCCESS) {
                nq_gemm_desc_t d;
                std::memset(&d, 0, sizeof(d));
                d.m = m; d.n = n; d.k = k;
                d.a_format = NQ_INT8; d.b_format = NQ_INT8;
                d.b_layout = NQ_B_KN;
                d.out_dtype = NQ_S8;
                d.alpha = a.metadata().scale * b.metadata().scale;
                st = nq_gemm(&d, d_a, d_b, d_c, s);
            }
            if (st == NQ_SUCCESS) st = ok(cudaMemcpyAsync(out.data(), d_c, nc, cudaMemcpyDeviceToHost, s));
            if (d_a) cudaFreeAsync(d_a, s);
            if (d_b) cudaFreeAsync(d_b, s);
            if (d_c) cudaFreeAsync(d_c, s);
            if (st == NQ_SUCCESS) st = ok(cudaStreamSynchronize(s));
            detail::nq_throw_if(st, "QuantizedMatmul::forward");
        }
        output = QuantizedInt8(std::move(out), a.metadata(), {m, n});
    }

    static std::vector<float> mixed_precision(const float* a, const int8_t* b, const float* scale_b, int m, int k,
                                              int n, Precision /*output_precision*/) {
        const size_t na = static_cast<size_t>(m) * k, nb = static_cast<size_t>(k) * n, nc = static_cast<size_t>(m) * n;
        std::vector<float> out(nc, 0.0f);
        if (!nc) return out;
        cudaStream_t s = 0;
        void *d_a = nullptr, *d_b = nullptr, *d_s = nullptr, *d_c = nullptr;
        auto ok = [](cudaError_t e) { return e == cudaSuccess ? NQ_SUCCESS : NQ_ERROR_CUDA; };
        nq_status_t st = ok(cudaMallocAsync(&d_a, (na ? na : 1) * sizeof(float), s));
        if (st == NQ_SUCCESS) st = ok(cudaMallocAsync(&d_b, nb ? nb : 1, s));
        if (st == NQ_SUCCESS) st = ok(cudaMallocAsync(&d_s, (k ? k : 1) * sizeof(float), s));
        if (st == NQ_SUCCESS) st = ok(cudaMallocAsync(&d_c, nc * sizeof(float), s));
        if (st == NQ_SUCCESS && na) st = ok(cudaMemcpyAsync(d_a, a, na * sizeof(float), cudaMemcpyHostToDevice, s));
        if (st == NQ_SUCCESS && nb) st = ok(cudaMemcpyAsync(d_b, b, nb, cudaMemcpyHostToDevice, s));
        if (st == NQ_SUCCESS && k) st = ok(cudaMemcpyAsync(d_s, scale_b, k * sizeof(float), cudaMemcpyHostToDevice, s));
        if (st == NQ_SUCCESS)
            st = nq_mixed_precision_matmul(static_cast<const float*>(d_a), static_cast<const int8_t*>(d_b),
                                           static_cast<const float*>(d_s), static_cast<float*>(d_c), m, k, n, s);
        if (st == NQ_SUCCESS) st = ok(cudaMemcpyAsync(out.data(), d_c, nc * sizeof(float), cudaMemcpyDeviceToHost, s));
        for (void* p : {d_a, d_b, d_s, d_c})
            if (p) cudaFreeAsync(p, s);
        if (st == NQ_SUCCESS) st = ok(cudaStreamSynchronize(s));
        detail::nq_throw_if(st, "QuantizedMatmul::mixed_precision");
        return out;
    }
};

inline void quantized_matmul(const QuantizedInt8& a, const QuantizedInt8& b, QuantizedInt8& output, int m, int k,
                             int n) {
    QuantizedMatmul::forward(a, b, output, m, k, n);
}

inline std::vector<float> mixed_precision_matmul(const float* a, const int8_t* b, const float* scale_b, int m, int k,
                                                 int n, Precision precision = Precision::FP32) {
    return QuantizedMatmul::mixed_precision(a, b, scale_b, m, k, n, precision);
}

}  // namespace quantize
}  // namespace nova

#endif
