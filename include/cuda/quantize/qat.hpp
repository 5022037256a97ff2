// qat.hpp -- drop-in for pplmx/nova include/cuda/quantize/qat.hpp
// (quantization-aware training helpers: Precision :31-37, LayerConfig :39-50,
// FakeQuantize :51-85, AMPManager :87-132 with the file format of
// src/cuda/quantize/qat.cpp:7-62, SensitivityAnalyzer :134-200).
//
// Same names, members and behaviour as the reference, host side.  Like the
// reference, this header's Precision enum clashes with the one of
// quantize_ops.hpp: include one of the two per translation unit.  Additive:
// FakeQuantize::forward over a device array (nq_fake_quantize_int8), the same
// arithmetic as the scalar forward element by element.
#ifndef NOVA_B200_QAT_HPP
#define NOVA_B200_QAT_HPP

#include <cuda_runtime.h>

#include <algorithm>
#include <cmath>
#include <cstdint>
#include <fstream>
#include <map>
#include <string>
#include <vector>

#include "calibrator.hpp"
#include "fp8_types.hpp"
#include "nq_check.hpp"

namespace nova {
namespace quantize {

enum class Precision { FP32, FP16, INT8, FP8_E4M3, FP8_E5M2 };

struct LayerConfig {
    std::string name;
    Precision precision{Precision::FP32};
    float scale{1.0f};
    float zero_point{0.0f};
    bool trainable{true};

    LayerConfig() = default;
    LayerConfig(const std::string& n, Precision p) : name(n), precision(p) {}
};

class FakeQuantize {
public:
    struct Config {
        Precision precision{Precision::INT8};
        float scale{1.0f};
        float zero_point{0.0f};
        int quant_bits{8};
        bool per_channel{false};
    };

    FakeQuantize(const Config& config) : config_(config) {}

    Config get_config() const { return config_; }

    // q = clamp(round_half_away((x - zp) / scale), +-127) * scale + zp, the
    // scale floored at 1e-6
    float forward(float x) const {
        const float s = config_.scale < 1e-6f ? 1e-6f : config_.scale;
        const float q = std::round((x - config_.zero_point) / s);
        const float c = std::max(-127.0f, std::min(127.0f, q));
        return c * s + config_.zero_point;
    }

    // Device arrays (n elements), asynchronous on `stream`.
    void forward(const float* d_input, float* d_output, size_t n, cudaStream_t stream = 0) const {
        detail::nq_report(nq_fake_quantize_int8(d_input, d_output, n, config_.scale, config_.zero_point, stream),
                          "FakeQuantize::forward");
    }

    // straight-through estimator
    float backward(float grad_output, float /*x*/) const { return grad_output; }

    void update_scale(float new_scale) { config_.scale = new_scale; }
    void update_zero_point(float new_zp) { config_.zero_point = new_zp; }

private:
    Config config_;
};

class AMPManager {
public:
    AMPManager() = default;

    void add_layer(const std::string& name, Precision precision = Precision::FP16) {
        configs_[name] = LayerConfig(name, precision);
    }
    void set_precision(const std::string& name, Precision precision) {
        auto it = configs_.find(name);
        if (it != configs_.end()) it->second.precision = precision;
    }
    void set_scale(const std::string& name, float scale) {
        auto it = configs_.find(name);
        if (it != configs_.end()) it->second.scale = scale;
    }
    Precision get_precision(const std::string& name) const {
        auto it = configs_.find(name);
        return it != configs_.end() ? it->second.precision : Precision::FP32;
    }
    const LayerConfig& get_config(const std::string& name) const {
        static const LayerConfig fallback;
        auto it = configs_.find(name);
        return it != configs_.end() ? it->second : fallback;
    }
    std::vector<LayerConfig> get_all_configs() const {
        std::vector<LayerConfig> out;
        out.reserve(configs_.size());
        for (const auto& kv : configs_) out.push_back(kv.second);
        return out;
    }

    // Binary layout kept from the reference (qat.cpp:7-29) so existing files
    // load: size_t count, then per layer in name order: size_t name length,
    // the name bytes, int precision, float scale, float zero point, int
    // trainable.  A file that cannot be opened is ignored, as there.
    void save_config(const std::string& path) const {
        std::ofstream f(path, std::ios::binary);
        if (!f) return;
        put(f, static_cast<size_t>(configs_.size()));
        for (const auto& kv : configs_) {
            put(f, static_cast<size_t>(kv.first.size()));
            f.write(kv.first.data(), static_cast<std::streamsize>(kv.first.size()));
            put(f, static_cast<int>(kv.second.precision));
            put(f, kv.second.scale);
            put(f, kv.second.zero_point);
            put(f, static_cast<int>(kv.second.trainable ? 1 : 0));
        }
    }
    void load_config(const std::string& path) {
        std::ifstream f(path, std::ios::binary);
        if (!f) return;
        configs_.clear();
        size_t count = 0;
        get(f, count);
        for (size_t i = 0; i < count && f; ++i) {
            size_t len = 0;
            get(f, len);
            std::string name(len, '\0');
            f.read(&name[0], static_cast<std::streamsize>(len));
            int prec = 0, trainable = 0;
            float scale = 1.0f, zp = 0.0f;
            get(f, prec);
            get(f, scale);
            get(f, zp);
            get(f, trainable);
            LayerConfig c(name, static_cast<Precision>(prec));
            c.scale = scale;
            c.zero_point = zp;
            c.trainable = trainable != 0;
            configs_[name] = c;
        }
    }

    size_t num_layers() const { return configs_.size(); }

private:
    template <class T>
    static void put(std::ofstream& f, const T& v) {
        f.write(reinterpret_cast<const char*>(&v), sizeof(T));
    }
    template <class T>
    static void get(std::ifstream& f, T& v) {
        f.read(reinterpret_cast<char*>(&v), sizeof(T));
    }

    std::map<std::string, LayerConfig> configs_;
};

class SensitivityAnalyzer {
public:
    struct LayerSensitivity {
        std::string name;
        float gradient_magnitude{0.0f};
        Precision recommended_precision{Precision::FP16};
        float confidence{0.0f};
    };

    // magnitude = max|activation| * max|gradient| over the common prefix;
    // above 10 the layer stays FP16, else INT8 (confidence 0.7).  Host arrays.
    void analyze_layer(const std::string& name, const float* activations, size_t n, const float* gradients,
                       size_t grad_n) {
        float amax = 0.0f, gmax = 0.0f;
        const size_t m = std::min(n, grad_n);
        for (size_t i = 0; i < m; ++i) {
            amax = std::max(amax, std::abs(activations[i]));
            gmax = std::max(gmax, std::abs(gradients[i]));
        }
        LayerSensitivity r;
        r.name = name;
        r.gradient_magnitude = amax * gmax;
        r.recommended_precision = r.gradient_magnitude > 10.0f ? Precision::FP16 : Precision::INT8;
        r.confidence = 0.7f;
        sensitivities_[name] = r;
    }

    Precision get_recommended_precision(const std::string& name) const {
        auto it = sensitivities_.find(name);
        return it != sensitivities_.end() ? it->second.recommended_precision : Precision::FP16;
    }
    const LayerSensitivity& get_sensitivity(const std::string& name) const {
        static const LayerSensitivity fallback;
        auto it = sensitivities_.find(name);
        return it != sensitivities_.end() ? it->second : fallback;
    }
    std::vector<LayerSensitivity> get_all_sensitivities() const {
        std::vector<LayerSensitivity> out;
        out.reserve(sensitivities_.size());
        for (const auto& kv : sensitivities_) out.push_back(kv.second);
        return out;
    }
    void auto_assign_precision(AMPManager& amp) const {
        for (const auto& kv : sensitivities_) amp.set_precision(kv.first, kv.second.recommended_precision);
    }

private:
    std::map<std::string, LayerSensitivity> sensitivities_;
};

}  // namespace quantize
}  // namespace nova

#endif  // NOVA_B200_QAT_HPP
