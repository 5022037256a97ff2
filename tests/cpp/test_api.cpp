// C++ drop-in API test: the assertions of the reference's own gtests
// (tests/quantize/*.cpp of pplmx/nova), re-expressed against the headers in
// include/cuda/quantize/ over libnova_q.  Runs on a GPU (tests/test_cpp_api.py).
#include <cuda/quantize/calibrator.hpp>
#include <cuda/quantize/fp8_gemm.hpp>
#include <cuda/quantize/fp8_kernels.hpp>
#include <cuda/quantize/fp8_types.hpp>
#include <cuda/quantize/int8_kernels.hpp>
#include <cuda/quantize/quantize_ops.hpp>
#include <cuda/quantize/quantize_tensor.hpp>

#include <cmath>
#include <cstdio>
#include <cstdlib>
#include <limits>
#include <random>
#include <vector>

using namespace nova::quantize;

static int g_fail = 0, g_checks = 0;
#define CHECK(cond)                                                              \
    do {                                                                         \
        ++g_checks;                                                              \
        if (!(cond)) {                                                           \
            ++g_fail;                                                            \
            std::fprintf(stderr, "FAIL %s:%d: %s\n", __FILE__, __LINE__, #cond); \
        }                                                                        \
    } while (0)

template <class T>
static T* dalloc(size_t n) {
    T* p = nullptr;
    cudaMalloc(&p, n * sizeof(T) + 16);
    return p;
}

// fp8_types_test.cpp
static void test_types() {
    CHECK(FP8E4M3(0.0f).to_bits() == 0);
    CHECK(FP8E4M3(std::numeric_limits<float>::infinity()).to_bits() == FP8E4M3::POS_INF);
    CHECK(FP8E4M3(-std::numeric_limits<float>::infinity()).to_bits() == FP8E4M3::NEG_INF);
    CHECK(FP8E4M3(std::numeric_limits<float>::quiet_NaN()).to_bits() == FP8E4M3::NAN_VAL);
    CHECK(FP8E4M3(-0.0f).to_bits() == FP8E4M3::NEG_ZERO);
    CHECK(std::isnan(static_cast<float>(FP8E4M3::from_bits(FP8E4M3::NAN_VAL))));
    CHECK(FP8E4M3::from_bits(0x3C).to_bits() == 0x3C);
    for (float v : {0.1f, 0.5f, 1.0f, 2.0f, 10.0f, 50.0f, 100.0f, 200.0f}) {
        float r = static_cast<float>(FP8E4M3(v));
        CHECK(std::abs(v - r) / v <= 0.15f);
    }
    CHECK(std::abs(static_cast<float>(FP8E4M3(1.5f)) - 1.5f) <= 0.1f);
    CHECK(static_cast<float>(FP8E5M2(100.0f)) > 0 && static_cast<float>(FP8E5M2(100.0f)) <= 256.0f);
    CHECK(FP8E5M2(std::numeric_limits<float>::infinity()).to_bits() == FP8E5M2::POS_INF);
    CHECK(is_fp8_type_v<FP8E4M3> && is_fp8_type_v<FP8E5M2> && !is_fp8_type_v<float>);
}

// int8_kernels_test.cpp:47-268
static void test_int8_kernels() {
    const size_t n = 1024;
    std::mt19937 rng(7);
    std::uniform_real_distribution<float> u(-10.0f, 10.0f);
    std::vector<float> src(n);
    for (auto& v : src) v = u(rng);
    float* d_src = dalloc<float>(n);
    int8_t* d_q = dalloc<int8_t>(n);
    float* d_y = dalloc<float>(n);
    cudaMemcpy(d_src, src.data(), n * 4, cudaMemcpyHostToDevice);
    cuda::QuantizationParams params(0.1f, 0.0f, true);
    cuda::quantize_f32_to_int8(d_src, d_q, n, params);
    std::vector<int8_t> q(n);
    cudaMemcpy(q.data(), d_q, n, cudaMemcpyDeviceToHost);
    int exact = 0;
    for (size_t i = 0; i < n; ++i) {
        int r = static_cast<int>(std::nearbyint(src[i] / 0.1f));
        r = std::max(-127, std::min(127, r));
        exact += (q[i] == r);
    }
    CHECK(exact == static_cast<int>(n));
    cuda::dequantize_int8_to_f32(d_q, d_y, n, params);
    std::vector<float> y(n);
    cudaMemcpy(y.data(), d_y, n * 4, cudaMemcpyDeviceToHost);
    int close = 0;
    for (size_t i = 0; i < n; ++i) close += std::abs(y[i] - q[i] * 0.1f) <= 0.01f;
    CHECK(close == static_cast<int>(n));
    // ramp min/max with device outputs (:207-236)
    std::vector<float> ramp(n);
    for (size_t i = 0; i < n; ++i) ramp[i] = static_cast<float>(i) / n * 100.0f - 50.0f;
    cudaMemcpy(d_src, ramp.data(), n * 4, cudaMemcpyHostToDevice);
    float* d_mm = dalloc<float>(2);
    cuda::compute_minmax(d_src, n, d_mm, d_mm + 1);
    float mm[2];
    cudaMemcpy(mm, d_mm, 8, cudaMemcpyDeviceToHost);
    CHECK(std::abs(mm[0] + 50.0f) <= 0.5f && std::abs(mm[1] - 49.9f) <= 0.5f);
    // histogram total (:238-268), 2048 bins as HistogramCalibrator's default
    uint32_t* d_h = dalloc<uint32_t>(2048);
    cuda::build_histogram(d_src, d_h, n, -50.0f, 50.0f, 2048);
    std::vector<uint32_t> h(2048);
    cudaMemcpy(h.data(), d_h, 2048 * 4, cudaMemcpyDeviceToHost);
    uint64_t tot = 0;
    for (auto c : h) tot += c;
    CHECK(tot == n);
    cudaFree(d_src); cudaFree(d_q); cudaFree(d_y); cudaFree(d_mm); cudaFree(d_h);
}

static std::vector<float> ramp(float lo, float hi, size_t n) {
    std::vector<float> d(n);
    for (size_t i = 0; i < n; ++i) d[i] = lo + static_cast<float>(i) / n * (hi - lo);
    return d;
}

// calibrator_test.cpp:32-188
static void test_calibrators() {
    auto d = ramp(-10, 10, 1024);
    MinMaxCalibrator c(true);
    auto r = c.calibrate(d.data(), d.size());
    CHECK(std::abs(r.scale - 10.0f / 127.0f) <= 0.01f && r.zero_point == 0.0f && r.symmetric);
    auto d2 = ramp(-5, 15, 1024);
    MinMaxCalibrator ca(false);
    auto r2 = ca.calibrate(d2.data(), d2.size());
    CHECK(std::abs(r2.scale - 20.0f / 254.0f) <= 0.01f && !r2.symmetric);
    MinMaxCalibrator c3(true);
    auto d3 = ramp(-8, 12, 1024);
    c3.calibrate(d3.data(), d3.size());
    c3.save_cache("/tmp/nova_b200_minmax_cache.bin");
    MinMaxCalibrator c4(true);
    c4.load_cache("/tmp/nova_b200_minmax_cache.bin");
    CHECK(c4.get_min() == c3.get_min() && c4.get_max() == c3.get_max());
    HistogramCalibrator hc(256, 99.99f, true);
    auto hr = hc.calibrate(d.data(), d.size());
    CHECK(hr.scale > 0 && hr.symmetric && hc.get_num_bins() == 256);
    std::mt19937 rng(3);
    std::vector<float> mix(10000);
    for (auto& v : mix) v = (rng() % 100 < 95) ? (rng() % 10000) / 1000.0f : (rng() % 100000) / 1000.0f;
    HistogramCalibrator h1(256, 99.0f, true), h2(256, 99.9f, true);
    CHECK(h2.calibrate(mix.data(), mix.size()).scale >= h1.calibrate(mix.data(), mix.size()).scale);
    HistogramCalibrator hdef;  // 2048 bins: correct here (the reference kernel kept 256)
    hdef.calibrate(mix.data(), mix.size());
    uint64_t tot = 0;
    for (auto v : hdef.histogram()) tot += v;
    CHECK(hdef.get_num_bins() == 2048 && tot == mix.size());
    MSECalibrator mc(true);
    auto d5 = ramp(-5, 5, 1024);
    CHECK(mc.calibrate(d5.data(), d5.size()).scale > 0);
    PerChannelCalibrator pc(0, true);
    auto d6 = ramp(-10, 10, 512);
    auto pr = pc.calibrate_per_channel(d6.data(), {4, 128});
    CHECK(pr.size() == 4);
    for (int ch = 0; ch < 4; ++ch) {
        MinMaxCalibrator one(true);
        auto o = one.calibrate(d6.data() + ch * 128, 128);
        CHECK(pr[ch].scale == o.scale && pr[ch].min_val == o.min_val && pr[ch].max_val == o.max_val);
    }
    std::vector<float> small(100, 0.001f), flat(100, 5.0f);
    CHECK(MinMaxCalibrator(true).calibrate(small.data(), 100).scale >= 1e-6f);
    CHECK(MinMaxCalibrator(true).calibrate(flat.data(), 100).scale >= 1e-6f);
}

// fp8_gemm_test.cpp:58-287
static void test_fp8_gemm() {
    const int m = 4, k = 4, n = 4;
    std::vector<FP8E4M3> a(16), b(16);
    for (int i = 0; i < 16; ++i) a[i] = FP8E4M3(static_cast<float>(i + 1));
    for (int i = 0; i < 16; ++i) b[i] = FP8E4M3((i / 4 == i % 4) ? 1.0f : 0.0f);
    FP8E4M3 *d_a = dalloc<FP8E4M3>(16), *d_b = dalloc<FP8E4M3>(16);
    float* d_c = dalloc<float>(16);
    cudaMemcpy(d_a, a.data(), 16, cudaMemcpyHostToDevice);
    cudaMemcpy(d_b, b.data(), 16, cudaMemcpyHostToDevice);
    FP8GEMM::forward(d_a, d_b, d_c, m, k, n, FP8GEMM::Config{}, 0);
    std::vector<float> c(16);
    cudaMemcpy(c.data(), d_c, 64, cudaMemcpyDeviceToHost);
    int ok = 0;
    for (int i = 0; i < 16; ++i) ok += std::abs(c[i] - static_cast<float>(i + 1)) <= 0.05f * (i + 1);
    CHECK(ok == 16);
    FP8GEMM::forward(d_a, d_b, d_c, m, k, n, FP8GEMM::Config(2.0f, 0.5f, 1.0f), 0);
    cudaMemcpy(c.data(), d_c, 64, cudaMemcpyDeviceToHost);
    CHECK(std::abs(c[5] - 6.0f) <= 1.0f);
    CHECK(FP8GEMM::get_workspace_size(128, 256, 128, FP8GEMM::Config{}) >= 128 * 128 * sizeof(float));
    cudaFree(d_a); cudaFree(d_b); cudaFree(d_c);
}

// quantize_ops_test.cpp:55-77 / quantize_tensor_test.cpp
static void test_quantized_tensor_and_matmul() {
    std::vector<float> x = {0.5f, -1.0f, 2.0f, -2.5f, 3.0f, 0.0f};
    auto q = QuantizedTensor<int8_t>::FromFloat(x.data(), x.size(), 0.0f);
    CHECK(q.has_value() && q->size() == 6 && std::abs(q->metadata().scale - 3.0f / 127.0f) < 1e-7f);
    auto back = q->ToFloat();
    for (size_t i = 0; i < x.size(); ++i) CHECK(std::abs(back[i] - x[i]) <= q->metadata().scale);
    CHECK(!QuantizedTensor<int8_t>::FromFloat(x.data(), 0, 0.0f).has_value());
    std::vector<float> af = {1, 2, 3, 4, 5, 6}, bf = {1, 0, 0, 1, 1, 1};
    auto qa = QuantizedTensor<int8_t>::FromFloat(af.data(), 6, 0.0f);
    auto qb = QuantizedTensor<int8_t>::FromFloat(bf.data(), 6, 0.0f);
    QuantizedInt8 out;
    QuantizedMatmul::forward(*qa, *qb, out, 2, 3, 2);
    CHECK(out.size() == 4 && out.shape().size() == 2 && out.shape()[0] == 2);
    // the reference's host loop on the same codes
    for (int i = 0; i < 2; ++i)
        for (int j = 0; j < 2; ++j) {
            int32_t s = 0;
            for (int p = 0; p < 3; ++p) s += qa->data()[i * 3 + p] * qb->data()[p * 2 + j];
            float v = s * (qa->metadata().scale * qb->metadata().scale);
            v = std::max(-127.0f, std::min(127.0f, v));
            CHECK(out.data()[i * 2 + j] == static_cast<int8_t>(std::round(v)));
        }
    std::vector<int8_t> bw = {1, -2, 3, -4, 5, -6};
    std::vector<float> sb = {0.5f, 0.25f, 2.0f};
    auto mp = mixed_precision_matmul(af.data(), bw.data(), sb.data(), 2, 3, 2);
    for (int i = 0; i < 2; ++i)
        for (int j = 0; j < 2; ++j) {
            float s = 0.0f;
            for (int p = 0; p < 3; ++p) s += af[i * 3 + p] * (static_cast<float>(bw[p * 2 + j]) * sb[p]);
            CHECK(mp[i * 2 + j] == s);
        }
}

int main() {
    if (cudaSetDevice(0) != cudaSuccess) {
        std::printf("SKIP: no CUDA device\n");
        return 0;
    }
    test_types();
    test_int8_kernels();
    test_calibrators();
    test_fp8_gemm();
    test_quantized_tensor_and_matmul();
    std::printf("%d checks, %d failures\n", g_checks, g_fail);
    return g_fail ? 1 : 0;
}
