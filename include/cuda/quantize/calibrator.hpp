// calibrator.hpp -- drop-in for pplmx/nova include/cuda/quantize/calibrator.hpp
// (CalibrationResult :39-68, Calibrator :70-82, MinMax :84-104, Histogram
// :106-135, MSE :137-156, PerChannel :158-183), over libnova_q.
//
// The scalar formulas after the reductions are the reference's host code
// (src/cuda/quantize/calibrator.cpp) in the same operation order, so results
// are bit-identical given bit-identical reductions.  Differences: no per-call
// cudaMalloc of reduction scratch (the library pools it), histograms are
// correct for any bin count, per-channel calibration is one kernel for all
// channels, and MSECalibrator also accepts device pointers.
#ifndef NOVA_B200_CALIBRATOR_HPP
#define NOVA_B200_CALIBRATOR_HPP

#include <cuda_runtime.h>

#include <algorithm>
#include <cmath>
#include <cstdint>
#include <fstream>
#include <limits>
#include <string>
#include <vector>

#include "int8_kernels.hpp"
#include "nq_check.hpp"

namespace nova {
namespace quantize {

struct CalibrationResult {
    float scale;
    float zero_point;
    bool symmetric;
    float min_val;
    float max_val;

    CalibrationResult() : scale(1.0f), zero_point(0.0f), symmetric(true), min_val(0.0f), max_val(0.0f) {}
    CalibrationResult(float s, float zp, bool sym, float min_v, float max_v)
        : scale(s), zero_point(zp), symmetric(sym), min_val(min_v), max_val(max_v) {}
};

class Calibrator {
public:
    virtual ~Calibrator() = default;
    virtual CalibrationResult calibrate(const float* data, size_t n, cudaStream_t stream = 0) = 0;
    virtual void save_cache(const std::string& path) const = 0;
    virtual void load_cache(const std::string& path) = 0;
    virtual std::string name() const = 0;
};

namespace detail {
// calibrator.cpp:27-37 (and :218-228): symmetric max(|min|,|max|)/127,
// asymmetric (max-min)/254 with zp = -min/scale - 127; scale floored at 1e-6
// after the zero point is computed.
inline CalibrationResult minmax_result(float lo, float hi, bool symmetric) {
    float scale, zero_point;
    if (symmetric) {
        float abs_max = std::max(std::abs(lo), std::abs(hi));
        scale = abs_max / 127.0f;
        zero_point = 0.0f;
    } else {
        scale = (hi - lo) / 254.0f;
        zero_point = -lo / scale - 127.0f;
    }
    if (scale < 1e-6f) scale = 1e-6f;
    return CalibrationResult(scale, zero_point, symmetric, lo, hi);
}
inline bool is_device_ptr(const void* p) {
    cudaPointerAttributes a;
    if (cudaPointerGetAttributes(&a, p) != cudaSuccess) {
        cudaGetLastError();
        return false;
    }
    return a.type == cudaMemoryTypeDevice || a.type == cudaMemoryTypeManaged;
}
}  // namespace detail

class MinMaxCalibrator : public Calibrator {
public:
    explicit MinMaxCalibrator(bool symmetric = true) : symmetric_(symmetric), min_val_(0.0f), max_val_(0.0f) {}

    CalibrationResult calibrate(const float* data, size_t n, cudaStream_t stream = 0) override {
        float lo = 0.0f, hi = 0.0f;
        cuda::compute_minmax(data, n, &lo, &hi, stream);
        min_val_ = lo;
        max_val_ = hi;
        return detail::minmax_result(min_val_, max_val_, symmetric_);
    }
    void save_cache(const std::string& path) const override {
        std::ofstream f(path, std::ios::binary);
        if (f.is_open()) {
            f.write(reinterpret_cast<const char*>(&min_val_), sizeof(float));
            f.write(reinterpret_cast<const char*>(&max_val_), sizeof(float));
        }
    }
    void load_cache(const std::string& path) override {
        std::ifstream f(path, std::ios::binary);
        if (f.is_open()) {
            f.read(reinterpret_cast<char*>(&min_val_), sizeof(float));
            f.read(reinterpret_cast<char*>(&max_val_), sizeof(float));
        }
    }
    std::string name() const override { return "MinMax"; }
    float get_min() const { return min_val_; }
    float get_max() const { return max_val_; }

private:
    bool symmetric_;
    float min_val_;
    float max_val_;
};

class HistogramCalibrator : public Calibrator {
public:
    explicit HistogramCalibrator(int num_bins = 2048, float percentile = 99.99f, bool symmetric = true)
        : num_bins_(num_bins), percentile_(percentile), symmetric_(symmetric), min_val_(0.0f), max_val_(0.0f) {
        histogram_.resize(num_bins_, 0);
    }

    // calibrator.cpp:65-107
    CalibrationResult calibrate(const float* data, size_t n, cudaStream_t stream = 0) override {
        float lo = 0.0f, hi = 0.0f;
        cuda::compute_minmax(data, n, &lo, &hi, stream);
        min_val_ = lo;
        max_val_ = hi;
        histogram_.assign(num_bins_, 0);
        uint32_t* d_hist = nullptr;
        detail::nq_throw_if(cudaMallocAsync(reinterpret_cast<void**>(&d_hist), sizeof(uint32_t) * num_bins_, stream) ==
                                    cudaSuccess ? NQ_SUCCESS : NQ_ERROR_OUT_OF_MEMORY,
                            "HistogramCalibrator::calibrate");
        nq_status_t st = nq_build_histogram(data, d_hist, n, min_val_, max_val_, num_bins_, stream);
        if (st == NQ_SUCCESS &&
            cudaMemcpyAsync(histogram_.data(), d_hist, sizeof(uint32_t) * num_bins_, cudaMemcpyDeviceToHost, stream) !=
                cudaSuccess)
            st = NQ_ERROR_CUDA;
        cudaFreeAsync(d_hist, stream);
        if (st == NQ_SUCCESS && cudaStreamSynchronize(stream) != cudaSuccess) st = NQ_ERROR_CUDA;
        detail::nq_throw_if(st, "HistogramCalibrator::calibrate");
        const float threshold = find_threshold_percentile(percentile_);
        const float abs_max = std::max(std::abs(threshold), std::abs(-threshold));
        float scale = abs_max / 127.0f;
        if (scale < 1e-6f) scale = 1e-6f;
        return CalibrationResult(scale, 0.0f, symmetric_, min_val_, max_val_);
    }
    void save_cache(const std::string& path) const override {
        std::ofstream f(path, std::ios::binary);
        if (f.is_open()) {
            f.write(reinterpret_cast<const char*>(&num_bins_), sizeof(int));
            f.write(reinterpret_cast<const char*>(&min_val_), sizeof(float));
            f.write(reinterpret_cast<const char*>(&max_val_), sizeof(float));
            f.write(reinterpret_cast<const char*>(histogram_.data()), num_bins_ * sizeof(uint32_t));
        }
    }
    void load_cache(const std::string& path) override {
        std::ifstream f(path, std::ios::binary);
        if (f.is_open()) {
            f.read(reinterpret_cast<char*>(&num_bins_), sizeof(int));
            f.read(reinterpret_cast<char*>(&min_val_), sizeof(float));
            f.read(reinterpret_cast<char*>(&max_val_), sizeof(float));
            histogram_.resize(num_bins_);
            f.read(reinterpret_cast<char*>(histogram_.data()), num_bins_ * sizeof(uint32_t));
        }
    }
    std::string name() const override { return "Histogram"; }
    int get_num_bins() const { return num_bins_; }
    float get_percentile() const { return percentile_; }
    const std::vector<uint32_t>& histogram() const { return histogram_; }

private:
    int num_bins_;
    float percentile_;
    bool symmetric_;
    float min_val_;
    float max_val_;
    std::vector<uint32_t> histogram_;

    // calibrator.cpp:109-129
    float find_threshold_percentile(float percentile) {
        uint64_t total = 0;
        for (uint32_t c : histogram_) total += c;
        const uint64_t target = static_cast<uint64_t>(static_cast<float>(total) * percentile / 100.0f);
        const float range = max_val_ - min_val_;
        const float bin_width = range / static_cast<float>(num_bins_);
        uint64_t cumulative = 0;
        for (int i = 0; i < num_bins_; ++i) {
            cumulative += histogram_[i];
            if (cumulative >= target) return min_val_ + (static_cast<float>(i) + 0.5f) * bin_width;
        }
        return max_val_;
    }
};

class MSECalibrator : public Calibrator {
public:
    explicit MSECalibrator(bool symmetric = true)
        : symmetric_(symmetric), min_val_(0.0f), max_val_(0.0f), best_scale_(1.0f), best_zero_point_(0.0f) {}

    // calibrator.cpp:158-190: power-of-two scale search on the first 10000
    // elements (copied to the host when `data` is device memory).
    CalibrationResult calibrate(const float* data, size_t n, cudaStream_t stream = 0) override {
        float lo = 0.0f, hi = 0.0f;
        cuda::compute_minmax(data, n, &lo, &hi, stream);
        min_val_ = lo;
        max_val_ = hi;
        const size_t cnt = std::min(n, static_cast<size_t>(10000));
        std::vector<float> h;
        const float* x = data;
        if (cnt && detail::is_device_ptr(data)) {
            h.resize(cnt);
            detail::nq_throw_if(cudaMemcpy(h.data(), data, cnt * sizeof(float), cudaMemcpyDeviceToHost) == cudaSuccess
                                    ? NQ_SUCCESS : NQ_ERROR_CUDA,
                                "MSECalibrator::calibrate");
            x = h.data();
        }
        float best_mse = std::numeric_limits<float>::max();
        float best = 1.0f;
        for (float cs = 0.001f; cs <= (max_val_ - min_val_); cs *= 2.0f) {
            float mse = 0.0f;
            for (size_t i = 0; i < cnt; ++i) {
                const float q = std::round(x[i] / cs) * cs;
                const float e = (x[i] - q) * (x[i] - q);
                mse += e;
            }
            mse /= static_cast<float>(cnt);
            if (mse < best_mse) {
                best_mse = mse;
                best = cs;
            }
        }
        best_scale_ = best;
        best_zero_point_ = 0.0f;
        return CalibrationResult(best_scale_, best_zero_point_, symmetric_, min_val_, max_val_);
    }
    void save_cache(const std::string& path) const override {
        std::ofstream f(path, std::ios::binary);
        if (f.is_open()) {
            f.write(reinterpret_cast<const char*>(&best_scale_), sizeof(float));
            f.write(reinterpret_cast<const char*>(&best_zero_point_), sizeof(float));
        }
    }
    void load_cache(const std::string& path) override {
        std::ifstream f(path, std::ios::binary);
        if (f.is_open()) {
            f.read(reinterpret_cast<char*>(&best_scale_), sizeof(float));
            f.read(reinterpret_cast<char*>(&best_zero_point_), sizeof(float));
        }
    }
    std::string name() const override { return "MSE"; }

private:
    bool symmetric_;
    float min_val_;
    float max_val_;
    float best_scale_;
    float best_zero_point_;
};

class PerChannelCalibrator : public Calibrator {
public:
    explicit PerChannelCalibrator(int channel_dim = 0, bool symmetric = true)
        : channel_dim_(channel_dim), symmetric_(symmetric) {}

    // calibrator.cpp:233-253 walks channel c as the contiguous slice
    // [c*inner, (c+1)*inner); here every slice's min/max comes from one
    // launch (nq_minmax_rows) and the per-channel formula is calibrate()'s.
    std::vector<CalibrationResult> calibrate_per_channel(const float* data, const std::vector<int>& shape,
                                                         cudaStream_t stream = 0) {
        channel_results_.clear();
        const int channels = shape.at(static_cast<size_t>(channel_dim_));
        int inner = 1;
        for (size_t i = 0; i < shape.size(); ++i)
            if (static_cast<int>(i) != channel_dim_) inner *= shape[i];
        if (channels <= 0) return channel_results_;
        const size_t n = static_cast<size_t>(channels) * inner;
        const bool dev = detail::is_device_ptr(data);
        float* staged = nullptr;
        float* mm = nullptr;
        auto ok = [](cudaError_t e) { return e == cudaSuccess ? NQ_SUCCESS : NQ_ERROR_CUDA; };
        nq_status_t st = NQ_SUCCESS;
        if (!dev) {
            st = ok(cudaMallocAsync(reinterpret_cast<void**>(&staged), n * sizeof(float), stream));
            if (st == NQ_SUCCESS) st = ok(cudaMemcpyAsync(staged, data, n * sizeof(float), cudaMemcpyHostToDevice, stream));
        }
        if (st == NQ_SUCCESS) st = ok(cudaMallocAsync(reinterpret_cast<void**>(&mm), 2 * sizeof(float) * channels, stream));
        std::vector<float> lo(channels), hi(channels);
        if (st == NQ_SUCCESS) st = nq_minmax_rows(dev ? data : staged, channels, inner, mm, mm + channels, stream);
        if (st == NQ_SUCCESS)
            st = ok(cudaMemcpyAsync(lo.data(), mm, sizeof(float) * channels, cudaMemcpyDeviceToHost, stream));
        if (st == NQ_SUCCESS)
            st = ok(cudaMemcpyAsync(hi.data(), mm + channels, sizeof(float) * channels, cudaMemcpyDeviceToHost, stream));
        if (staged) cudaFreeAsync(staged, stream);
        if (mm) cudaFreeAsync(mm, stream);
        if (st == NQ_SUCCESS) st = ok(cudaStreamSynchronize(stream));
        detail::nq_throw_if(st, "PerChannelCalibrator::calibrate_per_channel");
        for (int c = 0; c < channels; ++c) channel_results_.push_back(detail::minmax_result(lo[c], hi[c], symmetric_));
        return channel_results_;
    }

    CalibrationResult calibrate(const float* data, size_t n, cudaStream_t stream = 0) override {
        float lo = 0.0f, hi = 0.0f;
        cuda::compute_minmax(data, n, &lo, &hi, stream);
        return detail::minmax_result(lo, hi, symmetric_);
    }
    void save_cache(const std::string& path) const override {
        std::ofstream f(path, std::ios::binary);
        if (f.is_open()) {
            int c = static_cast<int>(channel_results_.size());
            f.write(reinterpret_cast<const char*>(&c), sizeof(int));
            for (const auto& r : channel_results_) {
                f.write(reinterpret_cast<const char*>(&r.scale), sizeof(float));
                f.write(reinterpret_cast<const char*>(&r.zero_point), sizeof(float));
            }
        }
    }
    void load_cache(const std::string& path) override {
        std::ifstream f(path, std::ios::binary);
        if (f.is_open()) {
            int c = 0;
            f.read(reinterpret_cast<char*>(&c), sizeof(int));
            channel_results_.resize(c);
            for (int i = 0; i < c; ++i) {
                f.read(reinterpret_cast<char*>(&channel_results_[i].scale), sizeof(float));
                f.read(reinterpret_cast<char*>(&channel_results_[i].zero_point), sizeof(float));
            }
        }
    }
    std::string name() const override { return "PerChannel"; }
    int get_channel_dim() const { return channel_dim_; }

private:
    int channel_dim_;
    bool symmetric_;
    std::vector<CalibrationResult> channel_results_;
};

}  // namespace quantize
}  // namespace nova

#endif
