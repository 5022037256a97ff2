// Host-side checks of the QAT drop-in header (include/cuda/quantize/qat.hpp),
// restating the reference tests' expectations (tests/quantize/qat_test.cpp of
// pplmx/nova) in our own words.  No GPU needed.
//   test_qat                 run the checks
//   test_qat write <path>    save an AMPManager config (three layers)
//   test_qat read <path>     load a config and print "layers name prec scale zp trainable" per layer
#include <cuda/quantize/qat.hpp>

#include <cmath>
#include <cstdio>
#include <cstring>
#include <string>

using namespace nova::quantize;

static int failures = 0;
#define CHECK(cond)                                                      \
    do {                                                                 \
        if (!(cond)) {                                                   \
            std::printf("FAIL %s:%d: %s\n", __FILE__, __LINE__, #cond); \
            ++failures;                                                  \
        }                                                                \
    } while (0)

static void checks() {
    FakeQuantize::Config c;
    c.scale = 0.5f;
    FakeQuantize fq(c);
    CHECK(fq.forward(1.0f) == 1.0f);
    CHECK(fq.forward(0.26f) == 0.5f);      // 0.52 -> 1 step
    CHECK(fq.forward(0.25f) == 0.5f);      // 0.5 rounds away from zero
    CHECK(fq.forward(-0.25f) == -0.5f);
    CHECK(fq.forward(1000.0f) == 63.5f);   // clamped to 127 steps
    CHECK(fq.forward(-1000.0f) == -63.5f);
    CHECK(fq.backward(3.0f, 123.0f) == 3.0f);
    fq.update_scale(0.0f);                 // floored at 1e-6
    CHECK(fq.forward(1.0f) == 127.0f * 1e-6f);
    fq.update_scale(1.0f);
    fq.update_zero_point(2.0f);
    CHECK(fq.forward(2.4f) == 2.0f);
    CHECK(fq.get_config().zero_point == 2.0f);

    AMPManager amp;
    amp.add_layer("fc1");
    CHECK(amp.get_precision("fc1") == Precision::FP16);
    amp.set_precision("fc1", Precision::FP8_E4M3);
    amp.set_scale("fc1", 0.25f);
    CHECK(amp.get_precision("fc1") == Precision::FP8_E4M3);
    CHECK(amp.get_config("fc1").scale == 0.25f);
    CHECK(amp.get_precision("missing") == Precision::FP32);
    CHECK(amp.get_config("missing").name.empty());
    amp.set_scale("missing", 3.0f);        // ignored
    CHECK(amp.num_layers() == 1);
    amp.add_layer("fc2", Precision::INT8);
    CHECK(amp.get_all_configs().size() == 2);
    const std::string path = "/tmp/nova_b200_qat_roundtrip.bin";
    amp.save_config(path);
    AMPManager back;
    back.load_config(path);
    CHECK(back.num_layers() == 2);
    CHECK(back.get_precision("fc1") == Precision::FP8_E4M3 && back.get_config("fc1").scale == 0.25f);
    CHECK(back.get_precision("fc2") == Precision::INT8 && back.get_config("fc2").trainable);
    std::remove(path.c_str());

    SensitivityAnalyzer sa;
    const float act[4] = {1.0f, -4.0f, 2.0f, 0.5f};
    const float grad_small[4] = {0.1f, 0.2f, -0.5f, 1.0f};
    const float grad_big[4] = {3.0f, -2.0f, 1.0f, 0.0f};
    sa.analyze_layer("small", act, 4, grad_small, 4);  // 4 * 1 = 4 -> INT8
    sa.analyze_layer("big", act, 4, grad_big, 4);      // 4 * 3 = 12 -> FP16
    sa.analyze_layer("edge", act, 2, grad_small, 4);   // common prefix of 2: 4 * 0.2
    CHECK(sa.get_recommended_precision("small") == Precision::INT8);
    CHECK(sa.get_recommended_precision("big") == Precision::FP16);
    CHECK(std::fabs(sa.get_sensitivity("edge").gradient_magnitude - 0.8f) < 1e-6f);
    CHECK(sa.get_sensitivity("big").confidence == 0.7f);
    CHECK(sa.get_recommended_precision("none") == Precision::FP16);
    CHECK(sa.get_all_sensitivities().size() == 3);
    AMPManager amp2;
    amp2.add_layer("small");
    amp2.add_layer("big");
    sa.auto_assign_precision(amp2);
    CHECK(amp2.get_precision("small") == Precision::INT8 && amp2.get_precision("big") == Precision::FP16);
    CHECK(static_cast<int>(Precision::FP8_E5M2) == 4);
}

int main(int argc, char** argv) {
    if (argc == 3 && std::strcmp(argv[1], "write") == 0) {
        AMPManager amp;
        amp.add_layer("q_proj", Precision::INT8);
        amp.set_scale("q_proj", 0.0625f);
        amp.add_layer("k_proj", Precision::FP8_E5M2);
        amp.add_layer("gate", Precision::FP8_E4M3);
        amp.set_scale("gate", 1.5f);
        amp.save_config(argv[2]);
        return 0;
    }
    if (argc == 3 && std::strcmp(argv[1], "read") == 0) {
        AMPManager amp;
        amp.load_config(argv[2]);
        std::printf("%zu\n", amp.num_layers());
        for (const auto& c : amp.get_all_configs())
            std::printf("%s %d %.9g %.9g %d\n", c.name.c_str(), static_cast<int>(c.precision), c.scale, c.zero_point,
                        c.trainable ? 1 : 0);
        return 0;
    }
    checks();
    std::printf("%d failures\n", failures);
    return failures ? 1 : 0;
}
