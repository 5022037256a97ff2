// C entry points over the reference's own GPU kernels (pplmx/nova
// src/cuda/quantize/*.cu compiled for sm_100a by oracle/Makefile).  Used only
// by tests/test_ref_gpu_pin.py to pin the oracle against the reference run on
// the same GPU.  Histograms are only requested with <= 256 bins: the
// reference kernel writes shared memory out of bounds above that.
#include <cuda/quantize/int8_kernels.hpp>
#include <cuda/quantize/fp8_kernels.hpp>
#include <cuda/quantize/fp8_gemm.hpp>
#include <cuda/quantize/calibrator.hpp>

using namespace nova::quantize;
namespace qc = nova::quantize::cuda;

extern "C" {

int ref_gpu_quantize_f32_to_int8(const float* src, int8_t* dst, size_t n, float scale,
                                 float zp, int sym) {
    qc::quantize_f32_to_int8(src, dst, n, qc::QuantizationParams(scale, zp, sym != 0), 0);
    return (int)cudaDeviceSynchronize();
}

int ref_gpu_dequantize_int8_to_f32(const int8_t* src, float* dst, size_t n, float scale,
                                   float zp, int sym) {
    qc::dequantize_int8_to_f32(src, dst, n, qc::QuantizationParams(scale, zp, sym != 0), 0);
    return (int)cudaDeviceSynchronize();
}

int ref_gpu_quantize_with_calibration(const float* src, int8_t* dst, size_t n, float mn, float mx) {
    qc::quantize_f32_to_int8_with_calibration(src, dst, n, mn, mx, 0);
    return (int)cudaDeviceSynchronize();
}

int ref_gpu_quantize_fp8(const float* src, uint8_t* dst, size_t n, int e5m2) {
    if (e5m2) qc::quantize_f32_to_fp8e5m2(src, reinterpret_cast<FP8E5M2*>(dst), n, 0);
    else qc::quantize_f32_to_fp8e4m3(src, reinterpret_cast<FP8E4M3*>(dst), n, 0);
    return (int)cudaDeviceSynchronize();
}

int ref_gpu_dequantize_fp8(const uint8_t* src, float* dst, size_t n, float scale, int e5m2) {
    if (e5m2) qc::dequantize_fp8e5m2_to_f32(reinterpret_cast<const FP8E5M2*>(src), dst, n, scale, 0);
    else qc::dequantize_fp8e4m3_to_f32(reinterpret_cast<const FP8E4M3*>(src), dst, n, scale, 0);
    return (int)cudaDeviceSynchronize();
}

int ref_gpu_compute_minmax(const float* data, size_t n, float* mn, float* mx) {
    qc::compute_minmax(data, n, mn, mx, 0);
    return (int)cudaDeviceSynchronize();
}

int ref_gpu_build_histogram(const float* data, uint32_t* hist, size_t n, float mn, float mx,
                            int bins) {
    if (bins > 256) return -1;
    qc::build_histogram(data, hist, n, mn, mx, bins, 0);
    return (int)cudaDeviceSynchronize();
}

int ref_gpu_fp8_gemm(const uint8_t* a, const uint8_t* b, float* c, int m, int k, int n,
                     float sa, float sb, float so) {
    FP8GEMM::forward(reinterpret_cast<const FP8E4M3*>(a), reinterpret_cast<const FP8E4M3*>(b),
                     c, m, k, n, FP8GEMM::Config(sa, sb, so), 0);
    return (int)cudaDeviceSynchronize();
}

// MSECalibrator::calibrate of the reference (calibrator.cpp:158-190) on a
// HOST pointer: its scale search reads data[i] on the host, so only host
// memory is valid there.
int ref_gpu_mse_calibrate(const float* host_data, size_t n, int sym, float* out5) {
    MSECalibrator c(sym != 0);
    CalibrationResult r = c.calibrate(host_data, n, 0);
    out5[0] = r.scale; out5[1] = r.zero_point; out5[2] = r.symmetric ? 1.0f : 0.0f;
    out5[3] = r.min_val; out5[4] = r.max_val;
    return (int)cudaDeviceSynchronize();
}

int ref_gpu_minmax_calibrate(const float* data, size_t n, int sym, float* out5) {
    MinMaxCalibrator c(sym != 0);
    CalibrationResult r = c.calibrate(data, n, 0);
    out5[0] = r.scale; out5[1] = r.zero_point; out5[2] = r.symmetric ? 1.0f : 0.0f;
    out5[3] = r.min_val; out5[4] = r.max_val;
    return (int)cudaDeviceSynchronize();
}

}  // extern "C"
