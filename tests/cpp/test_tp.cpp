// The drop-in C++ tensor-parallel layers (include/cuda/neural/
// tensor_parallel_layers.h, include/cuda/nccl/nccl_context.h) driven the way
// the reference's own tests drive theirs (tests/neural/
// tensor_parallel_multigpu_test.cpp:578-621): one host thread per GPU, each
// building its rank's layer on a shared NcclContext, set_weight with the full
// host weights, forward on device fp32 buffers.
//
//   test_tp checks           argument and shape errors, no GPU needed
//   test_tp run <tp> <dir>   tp GPUs (tp == 1: an uninitialized context, the
//                            reference's single-GPU fallback); writes every
//                            case's inputs and each rank's output to <dir>
//                            for tests/test_cpp_tp.py to check against the
//                            oracle.
#include <cuda/nccl/nccl_context.h>
#include <cuda/neural/tensor_parallel_layers.h>

#include <cmath>
#include <cstdio>
#include <cstdlib>
#include <cstring>
#include <functional>
#include <string>
#include <thread>
#include <vector>

using cuda::neural::ColumnParallelLayer;
using cuda::neural::RowParallelLayer;
using cuda::neural::TensorParallelMLP;
using cuda::neural::TpAllReduce;
using cuda::nccl::NcclContext;

static int g_fail = 0;
#define CHECK(cond)                                                              \
    do {                                                                         \
        if (!(cond)) {                                                           \
            ++g_fail;                                                            \
            std::fprintf(stderr, "FAIL %s:%d: %s\n", __FILE__, __LINE__, #cond); \
        }                                                                        \
    } while (0)

template <class E, class F>
static bool throws(F f) {
    try {
        f();
    } catch (const E&) {
        return true;
    } catch (...) {
        return false;
    }
    return false;
}

// Seeded normal values (xorshift + Box-Muller), written out for the checker.
static std::vector<float> normal(size_t n, uint64_t seed, float scale) {
    std::vector<float> v(n);
    uint64_t s = seed * 0x9E3779B97F4A7C15ull + 1;
    auto u01 = [&]() {
        s ^= s << 13;
        s ^= s >> 7;
        s ^= s << 17;
        return (static_cast<double>(s >> 11) + 0.5) / 9007199254740992.0;
    };
    for (size_t i = 0; i < n; ++i) {
        const double a = u01(), b = u01();
        v[i] = static_cast<float>(std::sqrt(-2.0 * std::log(a)) * std::cos(6.283185307179586 * b) * scale);
    }
    return v;
}

static void save(const std::string& path, const std::vector<float>& v) {
    FILE* f = std::fopen(path.c_str(), "wb");
    if (!f) {
        std::perror(path.c_str());
        std::exit(2);
    }
    std::fwrite(v.data(), sizeof(float), v.size(), f);
    std::fclose(f);
}

static int checks() {
    NcclContext ctx;  // uninitialized: tp degree 1
    CHECK(ctx.device_count() == 0 && !ctx.initialized() && !ctx.has_nccl());
    CHECK(throws<cuda::nccl::NcclException>([&] { (void)ctx.get_comm(0); }));
    CHECK(throws<cuda::nccl::NcclException>([&] { (void)ctx.rank_of_device(0); }));
    CHECK(throws<std::invalid_argument>([&] { ColumnParallelLayer l(ctx, 0, 16); }));
    CHECK(throws<std::invalid_argument>([&] { ColumnParallelLayer l(ctx, 16, -1); }));
    CHECK(throws<std::invalid_argument>([&] { RowParallelLayer l(ctx, -4, 16); }));
    CHECK(throws<std::invalid_argument>([&] { TensorParallelMLP l(ctx, 16, 0); }));
    CHECK(throws<std::invalid_argument>([&] { TensorParallelMLP l(ctx, 20, 64); }));  // hidden % 16
    {
        ColumnParallelLayer l(ctx, 16, 32);
        CHECK(l.tp_degree() == 1 && l.in_features() == 16 && l.out_features() == 32);
        CHECK(throws<std::invalid_argument>([&] { l.forward(nullptr, nullptr, 0, 4); }));
        CHECK(throws<std::runtime_error>([&] { l.forward(nullptr, nullptr, 2, 4); }));  // before set_weight
    }
    {
        RowParallelLayer l(ctx, 16, 32);
        CHECK(throws<std::invalid_argument>([&] { l.forward(nullptr, nullptr, 3, -1); }));
        CHECK(throws<std::runtime_error>([&] { l.forward(nullptr, nullptr, 1, 1); }));
    }
    {
        TensorParallelMLP l(ctx, 16, 48);
        CHECK(l.hidden_dim() == 16 && l.intermediate_size() == 48 && l.tp_degree() == 1);
        CHECK(!l.fused_all_reduce());
        CHECK(throws<std::invalid_argument>([&] { l.forward(nullptr, nullptr, 0, 0); }));
        CHECK(throws<std::runtime_error>([&] { l.forward(nullptr, nullptr, 8, 1); }));
    }
    cuda::nccl::NcclResult r;
    CHECK(r.ok() && static_cast<bool>(r));
    r.timed_out = true;
    CHECK(!r.ok());
    std::printf("%d failures\n", g_fail);
    return g_fail ? 1 : 0;
}

struct MlpCase {
    const char* name;
    int m, h, inter;
    TpAllReduce mode;
};
struct LinCase {
    const char* name;
    int m, k, n;
    bool row;
    TpAllReduce mode;
};

// Runs fn(rank) on one thread per rank with that rank's device current.
static void per_rank(NcclContext& ctx, int tp, const std::function<void(int)>& fn) {
    std::vector<std::thread> ts;
    std::vector<std::string> errors(tp);
    for (int r = 0; r < tp; ++r)
        ts.emplace_back([&, r] {
            try {
                cudaSetDevice(tp > 1 ? ctx.device_ids()[r] : 0);
                fn(r);
            } catch (const std::exception& e) {
                errors[r] = e.what();
            }
        });
    for (auto& t : ts) t.join();
    for (int r = 0; r < tp; ++r)
        if (!errors[r].empty()) {
            std::fprintf(stderr, "rank %d: %s\n", r, errors[r].c_str());
            ++g_fail;
        }
}

static std::vector<float> device_run(const std::vector<float>& in, size_t out_n,
                                     const std::function<void(const float*, float*)>& fwd) {
    float *din = nullptr, *dout = nullptr;
    cudaMalloc(&din, in.size() * sizeof(float));
    cudaMalloc(&dout, out_n * sizeof(float));
    cudaMemcpy(din, in.data(), in.size() * sizeof(float), cudaMemcpyHostToDevice);
    cudaMemset(dout, 0, out_n * sizeof(float));
    fwd(din, dout);
    std::vector<float> out(out_n);
    cudaMemcpy(out.data(), dout, out_n * sizeof(float), cudaMemcpyDeviceToHost);
    cudaFree(din);
    cudaFree(dout);
    return out;
}

static int run(int tp, const std::string& dir) {
    NcclContext ctx;
    if (tp > 1) {
        cuda::nccl::NcclContextConfig cfg;
        for (int d = 0; d < tp; ++d) cfg.device_ids.push_back(d);
        cfg.timeout_ms = 20000;
        ctx.initialize(cfg);
        std::printf("peer_access=%d\n", ctx.peer_access() ? 1 : 0);
    }
    const std::vector<MlpCase> mlps = {
        {"mlp_ref", 8, 16, tp > 1 ? 8 * tp : 48, TpAllReduce::Auto},   // the reference test's shapes
        {"mlp_mid", 200, 512, 768 * tp, TpAllReduce::Auto},             // fused all-reduce when tp > 1
        {"mlp_mid_nccl", 200, 512, 768 * tp, TpAllReduce::Nccl},        // the reference's fp32 ncclAllReduce
        {"mlp_odd", 37, 48, 96 * tp, TpAllReduce::Auto},                // padded shard, ncclAllReduce
    };
    for (const auto& c : mlps) {
        const auto x = normal(static_cast<size_t>(c.m) * c.h, 1, 1.0f);
        const auto wg = normal(static_cast<size_t>(c.h) * c.inter, 2, 0.05f);
        const auto wu = normal(static_cast<size_t>(c.h) * c.inter, 3, 0.05f);
        const auto wd = normal(static_cast<size_t>(c.inter) * c.h, 4, 0.05f);
        const std::string p = dir + "/" + c.name;
        save(p + "_x.bin", x);
        save(p + "_wg.bin", wg);
        save(p + "_wu.bin", wu);
        save(p + "_wd.bin", wd);
        std::vector<int> fused(tp, 0);
        per_rank(ctx, tp, [&](int r) {
            TensorParallelMLP mlp(ctx, c.h, c.inter, c.mode);
            mlp.set_weight(wg.data(), wu.data(), wd.data());
            fused[r] = mlp.fused_all_reduce() ? 1 : 0;
            std::vector<float> out;
            for (int rep = 0; rep < 2; ++rep)  // the fused path's counters move on every call
                out = device_run(x, static_cast<size_t>(c.m) * c.h,
                                 [&](const float* in, float* o) { mlp.forward(in, o, c.m, 1); });
            save(p + "_out" + std::to_string(r) + ".bin", out);
        });
        std::printf("case %s m=%d h=%d inter=%d tp=%d fused=%d\n", c.name, c.m, c.h, c.inter, tp, fused[0]);
    }
    const std::vector<LinCase> lins = {
        {"col_ref", 8, 16, 32, false, TpAllReduce::Auto},
        {"row_ref", 8, 16 * tp, 32, true, TpAllReduce::Auto},
        {"row_big", 200, 256 * tp, 512, true, TpAllReduce::Auto},
        {"row_big_nccl", 200, 256 * tp, 512, true, TpAllReduce::Nccl},
    };
    for (const auto& c : lins) {
        const auto x = normal(static_cast<size_t>(c.m) * c.k, 5, 1.0f);
        const auto w = normal(static_cast<size_t>(c.k) * c.n, 6, 0.05f);
        const std::string p = dir + "/" + c.name;
        save(p + "_x.bin", x);
        save(p + "_w.bin", w);
        per_rank(ctx, tp, [&](int r) {
            std::vector<float> out;
            if (c.row) {
                RowParallelLayer l(ctx, c.k, c.n, c.mode);
                l.set_weight(w.data());
                const int kl = c.k / l.tp_degree();
                std::vector<float> xs(static_cast<size_t>(c.m) * kl);  // this rank's input shard (columns)
                for (int i = 0; i < c.m; ++i)
                    std::memcpy(&xs[static_cast<size_t>(i) * kl], &x[static_cast<size_t>(i) * c.k + r * kl],
                                kl * sizeof(float));
                for (int rep = 0; rep < 2; ++rep)
                    out = device_run(xs, static_cast<size_t>(c.m) * c.n,
                                     [&](const float* in, float* o) { l.forward(in, o, 1, c.m); });
            } else {
                ColumnParallelLayer l(ctx, c.k, c.n);
                l.set_weight(w.data());
                out = device_run(x, static_cast<size_t>(c.m) * (c.n / l.tp_degree()),
                                 [&](const float* in, float* o) { l.forward(in, o, c.m, 1); });
            }
            save(p + "_out" + std::to_string(r) + ".bin", out);
        });
        std::printf("case %s m=%d k=%d n=%d tp=%d\n", c.name, c.m, c.k, c.n, tp);
    }
    std::printf("%d failures\n", g_fail);
    return g_fail ? 1 : 0;
}

int main(int argc, char** argv) {
    if (argc >= 2 && std::strcmp(argv[1], "checks") == 0) return checks();
    if (argc >= 4 && std::strcmp(argv[1], "run") == 0) return run(std::atoi(argv[2]), argv[3]);
    std::fprintf(stderr, "usage: test_tp checks | run <tp> <dir>\n");
    return 2;
}
