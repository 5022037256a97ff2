// fp8_gemm.hpp -- drop-in for pplmx/nova include/cuda/quantize/fp8_gemm.hpp
// (FP8GEMM :28-82, FP8E5M2GEMM :84-108), over the tcgen05 GEMM of libnova_q.
//
// forward: C[m x n] (fp32) = scale_out * sum_k (A*scale_a)(B*scale_b), A m x k
// and B k x n row-major codes.  The tensor cores read E4M3 codes as OCP
// E4M3FN; the 19 codes whose reading differs from the reference decoder
// (exponent field 0, 0x7C/0x7D/0x7F and their negatives) are therefore values
// of the OCP format here.  FP8E5M2GEMM decodes E5M2 (the reference passed the
// bytes to its E4M3 kernel, fp8_gemm.cu:247-249).
#ifndef NOVA_B200_FP8_GEMM_HPP
#define NOVA_B200_FP8_GEMM_HPP

#include <cuda_runtime.h>

#include <cstddef>

#include "fp8_types.hpp"
#include "nq_check.hpp"

namespace nova {
namespace quantize {

class FP8GEMM {
public:
    struct Config {
        float scale_a;
        float scale_b;
        float scale_out;
        bool use_tensor_core;
        int num_streams;

        Config() : scale_a(1.0f), scale_b(1.0f), scale_out(1.0f), use_tensor_core(false), num_streams(1) {}
        Config(float sa, float sb, float so, bool utc = false, int ns = 1)
            : scale_a(sa), scale_b(sb), scale_out(so), use_tensor_core(utc), num_streams(ns) {}
    };

    static void forward(const FP8E4M3* a, const FP8E4M3* b, float* output, int m, int k, int n,
                        Config config = Config{}, cudaStream_t stream = 0) {
        detail::nq_report(nq_fp8_gemm_forward(reinterpret_cast<const uint8_t*>(a), reinterpret_cast<const uint8_t*>(b),
                                              output, m, k, n, config.scale_a, config.scale_b, config.scale_out, stream),
                          "FP8GEMM::forward");
    }

    static void forward_async(const FP8E4M3* a, const FP8E4M3* b, float* output, int m, int k, int n,
                              Config config = Config{}, cudaStream_t stream = 0) {
        forward(a, b, output, m, k, n, config, stream);
    }

    // Same two calls as the reference (fp8_gemm.cu:200-230).
    static void backward(const FP8E4M3* grad_output, const FP8E4M3* a, const FP8E4M3* b, float* grad_a, float* grad_b,
                         int m, int k, int n, Config config = Config{}, cudaStream_t stream = 0) {
        Config g;
        g.scale_a = config.scale_a;
        g.scale_b = config.scale_out;
        forward(grad_output, b, grad_a, m, n, k, g, stream);
        g.scale_a = config.scale_out;
        g.scale_b = config.scale_b;
        forward(grad_output, a, grad_b, n, m, k, g, stream);
    }

    // Additive: the true gradients of output = (a.b) * scale_a * scale_b for a
    // gradient grad_output (M x N) quantized with scale_grad, E4M3 or E5M2
    // (nq_fp8_gemm_backward): grad_a = grad_output . b^T, grad_b = a^T . grad_output.
    static void backward_exact(const FP8E4M3* grad_output, float scale_grad, const FP8E4M3* a, const FP8E4M3* b,
                               float* grad_a, float* grad_b, int m, int k, int n, Config config = Config{},
                               cudaStream_t stream = 0) {
        detail::nq_report(nq_fp8_gemm_backward(reinterpret_cast<const uint8_t*>(grad_output), NQ_E4M3,
                                               reinterpret_cast<const uint8_t*>(a), reinterpret_cast<const uint8_t*>(b),
                                               grad_a, grad_b, m, k, n, scale_grad, config.scale_a, config.scale_b,
                                               stream),
                          "FP8GEMM::backward_exact");
    }
    static void backward_exact(const FP8E5M2* grad_output, float scale_grad, const FP8E4M3* a, const FP8E4M3* b,
                               float* grad_a, float* grad_b, int m, int k, int n, Config config = Config{},
                               cudaStream_t stream = 0) {
        detail::nq_report(nq_fp8_gemm_backward(reinterpret_cast<const uint8_t*>(grad_output), NQ_E5M2,
                                               reinterpret_cast<const uint8_t*>(a), reinterpret_cast<const uint8_t*>(b),
                                               grad_a, grad_b, m, k, n, scale_grad, config.scale_a, config.scale_b,
                                               stream),
                          "FP8GEMM::backward_exact");
    }

    static size_t get_workspace_size(int m, int k, int n, const Config&) { return nq_fp8_gemm_workspace_size(m, k, n); }
};

class FP8E5M2GEMM {
public:
    struct Config {
        float scale_a;
        float scale_b;
        float scale_out;
        int num_streams;

        Config() : scale_a(1.0f), scale_b(1.0f), scale_out(1.0f), num_streams(1) {}
        Config(float sa, float sb, float so, int ns = 1) : scale_a(sa), scale_b(sb), scale_out(so), num_streams(ns) {}
    };

    static void forward(const FP8E5M2* a, const FP8E5M2* b, float* output, int m, int k, int n,
                        Config config = Config{}, cudaStream_t stream = 0) {
        detail::nq_report(nq_fp8e5m2_gemm_forward(reinterpret_cast<const uint8_t*>(a),
                                                  reinterpret_cast<const uint8_t*>(b), output, m, k, n, config.scale_a,
                                                  config.scale_b, config.scale_out, stream),
                          "FP8E5M2GEMM::forward");
    }
};

}  // namespace quantize
}  // namespace nova

#endif
