// tensor_parallel_layers.h -- drop-in for pplmx/nova's cuda::neural
// ColumnParallelLayer, RowParallelLayer and TensorParallelMLP
// (include/cuda/neural/tensor_parallel_layers.h:51, :194, :328;
// src/cuda/neural/tensor_parallel_layers.cpp), header-only, over libnova_q.
//
// Same constructors (NcclContext&, sizes), set_weight(host fp32, full weight;
// this rank keeps its shard as the reference slices it, :111-136 / :344-368),
// synchronous forward(device fp32 input, device fp32 output, batch, seq),
// tp_degree() = max(1, ctx.device_count()), the rank from
// ctx.rank_of_device(cudaGetDevice()), std::invalid_argument for shape errors
// and NcclException when the all-reduce fails.  The arithmetic is W8A8 FP8
// instead of fp32: weight shards are quantized per output channel to E4M3 at
// set_weight (scale = column amax / 448), activations per token at forward,
// and the GEMMs run on the tcgen05 tensor cores with the scales in the
// epilogue.  TensorParallelMLP packs its gate and up shards into one weight
// (alternating 128-column blocks, zero-padded to a multiple of 128) so one
// GEMM writes silu(gate) * up directly.
//
// The row-parallel all-reduce (the reference's fp32 ncclAllReduce, :406)
// runs, when every GPU of the group can address the others' memory and the
// output width is a multiple of 256, inside the down GEMM (nq_gemm_allreduce:
// bf16 partials summed in fp32 over peer memory, bf16 result, converted to
// the fp32 output); otherwise as the reference does it, an fp32
// ncclAllReduce.  The choice is the same on every rank.  Either way a timed
// out or failed collective throws NcclException.
//
// Not provided: the training surface (backward, step, AdamW) of the
// reference layers; this path is inference.
#pragma once

#include <cuda_runtime.h>

#include <algorithm>
#include <cstdint>
#include <cstring>
#include <limits>
#include <map>
#include <memory>
#include <stdexcept>
#include <string>
#include <vector>

#include "../../nova_q.h"
#include "../nccl/nccl_all_reduce.h"
#include "../nccl/nccl_context.h"

namespace cuda {
namespace neural {

// How RowParallelLayer (and the MLP's down projection) reduces across ranks;
// an addition to the reference API (default Auto).
enum class TpAllReduce { Auto, Fused, Nccl };

namespace tp_detail {

inline void check(nq_status_t st, const char* where) {
    if (st != NQ_SUCCESS)
        throw std::runtime_error(std::string(where) + ": " + nq_status_string(st) + ": " + nq_last_error());
}
inline void cuda_check(cudaError_t e, const char* where) {
    if (e != cudaSuccess) throw std::runtime_error(std::string(where) + ": " + cudaGetErrorString(e));
}
inline int current_device() {
    int d = 0;
    cuda_check(cudaGetDevice(&d), "cudaGetDevice");
    return d;
}

// Device memory owned by the GPU that was current when it was allocated.
class DeviceBuffer {
public:
    DeviceBuffer() = default;
    DeviceBuffer(const DeviceBuffer&) = delete;
    DeviceBuffer& operator=(const DeviceBuffer&) = delete;
    ~DeviceBuffer() { reset(); }
    void ensure(size_t bytes) {
        if (bytes <= size_ && p_) return;
        reset();
        cuda_check(cudaMalloc(&p_, std::max<size_t>(bytes, 16)), "cudaMalloc");
        size_ = bytes;
        dev_ = current_device();
    }
    void reset() {
        if (!p_) return;
        int prev = 0;
        cudaGetDevice(&prev);
        cudaSetDevice(dev_);
        cudaFree(p_);
        cudaSetDevice(prev);
        p_ = nullptr;
        size_ = 0;
    }
    template <class T>
    T* as() const {
        return static_cast<T*>(p_);
    }
    bool empty() const { return p_ == nullptr; }

private:
    void* p_ = nullptr;
    size_t size_ = 0;
    int dev_ = 0;
};

// OCP E4M3FN code -> float (exact; copy_weight_shard).
inline float e4m3_value(uint8_t c) {
    const int s = c >> 7, e = (c >> 3) & 15, m = c & 7;
    float v;
    if (e == 15 && m == 7) v = std::numeric_limits<float>::quiet_NaN();
    else if (e == 0) v = static_cast<float>(m) * (1.0f / 512.0f);
    else v = (1.0f + static_cast<float>(m) / 8.0f) * static_cast<float>(1 << e) * (1.0f / 128.0f);
    return s ? -v : v;
}

// A K x N row-major weight quantized per output column to E4M3.
struct Fp8Weight {
    DeviceBuffer codes, scales;
    int k = 0, n = 0;
    void load(const float* host, int k_, int n_, cudaStream_t s) {
        k = k_;
        n = n_;
        DeviceBuffer tmp;
        const size_t elems = static_cast<size_t>(k) * n;
        tmp.ensure(elems * sizeof(float));
        codes.ensure(elems);
        scales.ensure(static_cast<size_t>(n) * sizeof(float));
        cuda_check(cudaMemcpyAsync(tmp.as<float>(), host, elems * sizeof(float), cudaMemcpyHostToDevice, s),
                   "set_weight: upload");
        check(nq_quantize_cols(tmp.as<float>(), codes.as<uint8_t>(), scales.as<float>(), k, n, NQ_E4M3, s),
              "set_weight: nq_quantize_cols");
        cuda_check(cudaStreamSynchronize(s), "set_weight: synchronize");
    }
    // The dequantized weight (codes x column scales), K x N.
    std::vector<float> dequantized() const {
        const size_t elems = static_cast<size_t>(k) * n;
        std::vector<uint8_t> c(elems);
        std::vector<float> sc(n), out(elems);
        cuda_check(cudaMemcpy(c.data(), codes.as<uint8_t>(), elems, cudaMemcpyDeviceToHost), "copy weight");
        cuda_check(cudaMemcpy(sc.data(), scales.as<float>(), n * sizeof(float), cudaMemcpyDeviceToHost), "copy scales");
        for (size_t i = 0; i < elems; ++i) out[i] = e4m3_value(c[i]) * sc[i % n];
        return out;
    }
};

// Per-token E4M3 codes and scales of m activation rows (nq_quantize_rows).
struct TokenCodes {
    DeviceBuffer codes, scales;
    void quantize(const void* x, nq_dtype_t dt, int m, int k, cudaStream_t s) {
        codes.ensure(static_cast<size_t>(m) * k);
        scales.ensure(static_cast<size_t>(m) * sizeof(float));
        check(nq_quantize_rows(x, dt, codes.as<uint8_t>(), scales.as<float>(), m, k, NQ_E4M3, s),
              "forward: nq_quantize_rows");
    }
};

inline nq_gemm_desc_t gemm_desc(int m, int n, int k, nq_dtype_t out, const float* row_scale, const float* col_scale,
                                nq_epilogue_t epi = NQ_EPI_NONE) {
    nq_gemm_desc_t d;
    std::memset(&d, 0, sizeof(d));
    d.m = m;
    d.n = n;
    d.k = k;
    d.a_format = NQ_E4M3;
    d.b_format = NQ_E4M3;
    d.b_layout = NQ_B_KN;
    d.out_dtype = out;
    d.alpha = 1.0f;
    d.row_scale = row_scale;
    d.col_scale = col_scale;
    d.epilogue = epi;
    return d;
}

// The row-parallel reduction of one layer: rank, stream, and for the fused
// all-reduce the per-token-count buffers (bf16 partial and output, tile and
// completion counters) with every rank's addresses.
class RowReducer {
public:
    RowReducer(::cuda::nccl::NcclContext& ctx, int out_features, TpAllReduce mode)
        : ctx_(ctx), n_(out_features), mode_(mode), reducer_(ctx) {
        tp_ = std::max(1, ctx.device_count());
        if (tp_ > 1 && ctx.initialized()) layer_id_ = ctx.next_layer_id(current_device());
    }
    int tp() const { return tp_; }
    // The reduction the group uses for a k-deep GEMM (identical on every rank).
    bool fused(int k) const {
        if (tp_ <= 1 || mode_ == TpAllReduce::Nccl) return false;
        const bool ok = ctx_.peer_access() && tp_ <= NQ_MAX_TP && n_ % 256 == 0 && k % 16 == 0;
        if (mode_ == TpAllReduce::Fused && !ok)
            throw std::invalid_argument("TpAllReduce::Fused needs peer access between the group's GPUs, "
                                        "tp <= 8, out_features % 256 == 0 and k % 16 == 0");
        return ok;
    }
    // out (m x n fp32, device) = sum over ranks of codes x weight; synchronous.
    void run(const TokenCodes& a, const Fp8Weight& w, float* output, int m, cudaStream_t s) {
        const int k = w.k;
        if (tp_ <= 1) {
            const nq_gemm_desc_t d = gemm_desc(m, n_, k, NQ_F32, a.scales.as<float>(), w.scales.as<float>());
            check(nq_gemm(&d, a.codes.as<uint8_t>(), w.codes.as<uint8_t>(), output, s), "forward: nq_gemm");
            cuda_check(cudaStreamSynchronize(s), "forward: synchronize");
            return;
        }
        if (!ctx_.has_nccl())
            throw std::invalid_argument("RowParallelLayer::forward on multi-GPU requires an initialized NCCL context");
        const int rank = ctx_.rank_of_device(current_device());
        if (!fused(k)) {
            // the reference's path: fp32 partial, fp32 ncclAllReduce in place
            const nq_gemm_desc_t d = gemm_desc(m, n_, k, NQ_F32, a.scales.as<float>(), w.scales.as<float>());
            check(nq_gemm(&d, a.codes.as<uint8_t>(), w.codes.as<uint8_t>(), output, s), "forward: nq_gemm");
            const ::cuda::nccl::NcclResult r =
                reducer_.all_reduce_async(output, output, static_cast<size_t>(m) * n_, ncclFloat32, ncclSum, s);
            if (!r.ok())
                throw ::cuda::nccl::NcclException(r.error_message.c_str(), r.code, "RowParallelLayer::forward AllReduce",
                                                  __FILE__, __LINE__);
            return;
        }
        Shape& sh = shape(m, rank);
        ++sh.epoch;
        nq_allreduce_desc_t ar;
        std::memset(&ar, 0, sizeof(ar));
        ar.tp = tp_;
        ar.rank = rank;
        ar.epoch = sh.epoch;
        ar.signal = 1;
        ar.m = m;
        ar.n = n_;
        ar.flags = sh.flags_of[rank];
        for (int r = 0; r < tp_; ++r) {
            ar.signal_flags[r] = sh.flags_of[r];
            ar.peer_partial[r] = reinterpret_cast<void*>(sh.partial_of[r]);
            ar.peer_out[r] = reinterpret_cast<void*>(sh.out_of[r]);
            ar.peer_done[r] = sh.done_of[r];
        }
        ar.done = sh.done_of[rank];
        ar.done_target = sh.epoch * sh.per_forward;  // both modulo 2^32
        const nq_gemm_desc_t d = gemm_desc(m, n_, k, NQ_BF16, a.scales.as<float>(), w.scales.as<float>());
        check(nq_gemm_allreduce(&d, &ar, a.codes.as<uint8_t>(), w.codes.as<uint8_t>(),
                                reinterpret_cast<void*>(sh.partial_of[rank]), s),
              "forward: nq_gemm_allreduce");
        check(nq_convert_bf16_to_f32(reinterpret_cast<void*>(sh.out_of[rank]), output, static_cast<size_t>(m) * n_, s),
              "forward: nq_convert_bf16_to_f32");
        cuda_check(cudaStreamSynchronize(s), "forward: synchronize");
        uint32_t flags = 0;
        check(nq_device_error_flags(&flags, 1), "forward: nq_device_error_flags");
        if (flags)
            throw ::cuda::nccl::NcclException("GEMM-fused all-reduce: a wait on another GPU timed out", ncclSystemError,
                                              "RowParallelLayer::forward", __FILE__, __LINE__);
    }

private:
    struct Shape {
        DeviceBuffer partial, out, counters;
        uint32_t epoch = 0, per_forward = 0;
        std::vector<uintptr_t> partial_of, out_of;
        std::vector<uint32_t*> flags_of, done_of;
    };
    // Buffers for m tokens, allocated and zeroed by every rank, then swapped
    // with the other ranks through the context (collective on first use).
    Shape& shape(int m, int rank) {
        auto it = shapes_.find(m);
        if (it != shapes_.end()) return *it->second;
        auto sh = std::make_unique<Shape>();
        const size_t bytes = static_cast<size_t>(m) * n_ * 2;
        const int tiles = nq_gemm_allreduce_counters(m, n_);
        sh->partial.ensure(bytes);
        sh->out.ensure(bytes);
        sh->counters.ensure(static_cast<size_t>(tiles + 1) * sizeof(uint32_t));
        cuda_check(cudaMemset(sh->counters.as<uint32_t>(), 0, static_cast<size_t>(tiles + 1) * sizeof(uint32_t)),
                   "zero all-reduce counters");
        cuda_check(cudaDeviceSynchronize(), "zero all-reduce counters");
        sh->per_forward = static_cast<uint32_t>(nq_allreduce_done_per_job(m, n_, 1));
        const uint64_t key = (static_cast<uint64_t>(layer_id_) << 40) | (static_cast<uint64_t>(m) << 4);
        const auto p = ctx_.exchange(key | 0, rank, reinterpret_cast<uintptr_t>(sh->partial.as<void>()));
        const auto o = ctx_.exchange(key | 1, rank, reinterpret_cast<uintptr_t>(sh->out.as<void>()));
        const auto c = ctx_.exchange(key | 2, rank, reinterpret_cast<uintptr_t>(sh->counters.as<uint32_t>()));
        sh->partial_of = p;
        sh->out_of = o;
        for (int r = 0; r < tp_; ++r) {
            uint32_t* base = reinterpret_cast<uint32_t*>(c[r]);
            sh->flags_of.push_back(base);
            sh->done_of.push_back(base + tiles);
        }
        return *(shapes_[m] = std::move(sh));
    }

    ::cuda::nccl::NcclContext& ctx_;
    int n_;
    TpAllReduce mode_;
    int tp_ = 1;
    int layer_id_ = 0;
    ::cuda::nccl::NcclAllReduce reducer_;
    std::map<int, std::unique_ptr<Shape>> shapes_;
};

// A layer's stream on its device (the reference creates one per call).
class LayerStream {
public:
    ~LayerStream() {
        if (s_) {
            int prev = 0;
            cudaGetDevice(&prev);
            cudaSetDevice(dev_);
            cudaStreamDestroy(s_);
            cudaSetDevice(prev);
        }
    }
    cudaStream_t get() {
        if (!s_) {
            cuda_check(cudaStreamCreateWithFlags(&s_, cudaStreamNonBlocking), "cudaStreamCreate");
            dev_ = current_device();
        }
        return s_;
    }

private:
    cudaStream_t s_ = nullptr;
    int dev_ = 0;
};

}  // namespace tp_detail

// Column-parallel linear layer (tensor_parallel_layers.h:51): rank r keeps
// columns [r*out/tp, (r+1)*out/tp) of the weight; input replicated, output
// sharded, no communication.
class ColumnParallelLayer {
public:
    ColumnParallelLayer(::cuda::nccl::NcclContext& ctx, int in_features, int out_features)
        : ctx_(ctx), in_features_(in_features), out_features_(out_features) {
        if (in_features_ <= 0) throw std::invalid_argument("ColumnParallelLayer requires a positive in_features");
        if (out_features_ <= 0) throw std::invalid_argument("ColumnParallelLayer requires a positive out_features");
        if (tp_degree() > 1 && out_features_ % tp_degree() != 0)
            throw std::invalid_argument("ColumnParallelLayer requires out_features divisible by the tp degree");
    }
    ColumnParallelLayer(const ColumnParallelLayer&) = delete;
    ColumnParallelLayer& operator=(const ColumnParallelLayer&) = delete;

    // Full weight [in_features x out_features], row-major, host memory.
    void set_weight(const float* weight) {
        const int tp = tp_degree(), nl = out_features_ / tp;
        const int rank = tp > 1 ? ctx_.rank_of_device(tp_detail::current_device()) : 0;
        std::vector<float> shard(static_cast<size_t>(in_features_) * nl);
        for (int i = 0; i < in_features_; ++i)
            std::memcpy(&shard[static_cast<size_t>(i) * nl], weight + static_cast<size_t>(i) * out_features_ + rank * nl,
                        nl * sizeof(float));
        weight_.load(shard.data(), in_features_, nl, stream_.get());
    }
    // input [batch*seq x in_features] -> output [batch*seq x out_features/tp],
    // device fp32, synchronous.
    void forward(const float* input, float* output, int batch, int seq) {
        const int m = batch * seq;
        if (m <= 0) throw std::invalid_argument("ColumnParallelLayer::forward requires batch*seq > 0");
        if (weight_.codes.empty())
            throw std::runtime_error("ColumnParallelLayer::forward called before set_weight");
        cudaStream_t s = stream_.get();
        act_.quantize(input, NQ_F32, m, in_features_, s);
        const nq_gemm_desc_t d = tp_detail::gemm_desc(m, weight_.n, in_features_, NQ_F32, act_.scales.as<float>(),
                                                      weight_.scales.as<float>());
        tp_detail::check(nq_gemm(&d, act_.codes.as<uint8_t>(), weight_.codes.as<uint8_t>(), output, s),
                         "ColumnParallelLayer::forward");
        tp_detail::cuda_check(cudaStreamSynchronize(s), "ColumnParallelLayer::forward");
    }
    // This rank's shard, dequantized, [in_features x out_features/tp].
    void copy_weight_shard(float* host_out) const {
        const auto w = weight_.dequantized();
        std::memcpy(host_out, w.data(), w.size() * sizeof(float));
    }
    [[nodiscard]] int in_features() const { return in_features_; }
    [[nodiscard]] int out_features() const { return out_features_; }
    [[nodiscard]] int tp_degree() const { return std::max(1, ctx_.device_count()); }

private:
    ::cuda::nccl::NcclContext& ctx_;
    int in_features_, out_features_;
    tp_detail::Fp8Weight weight_;
    tp_detail::TokenCodes act_;
    tp_detail::LayerStream stream_;
};

// Row-parallel linear layer (tensor_parallel_layers.h:194): rank r keeps rows
// [r*in/tp, (r+1)*in/tp); input sharded, output replicated by the all-reduce.
class RowParallelLayer {
public:
    RowParallelLayer(::cuda::nccl::NcclContext& ctx, int in_features, int out_features,
                     TpAllReduce mode = TpAllReduce::Auto)
        : ctx_(ctx), in_features_(in_features), out_features_(out_features),
          reducer_(ctx, out_features > 0 ? out_features : 1, mode) {
        if (in_features_ <= 0) throw std::invalid_argument("RowParallelLayer requires a positive in_features");
        if (out_features_ <= 0) throw std::invalid_argument("RowParallelLayer requires a positive out_features");
        if (tp_degree() > 1 && in_features_ % tp_degree() != 0)
            throw std::invalid_argument("RowParallelLayer requires in_features divisible by the tp degree");
    }
    RowParallelLayer(const RowParallelLayer&) = delete;
    RowParallelLayer& operator=(const RowParallelLayer&) = delete;

    // Full weight [in_features x out_features], row-major, host memory.
    void set_weight(const float* weight) {
        const int tp = tp_degree(), kl = in_features_ / tp;
        const int rank = tp > 1 ? ctx_.rank_of_device(tp_detail::current_device()) : 0;
        weight_.load(weight + static_cast<size_t>(rank) * kl * out_features_, kl, out_features_, stream_.get());
    }
    // input [batch*seq x in_features/tp] -> output [batch*seq x out_features]
    // (replicated), device fp32, synchronous.
    void forward(const float* input, float* output, int batch, int seq) {
        const int m = batch * seq;
        if (m <= 0) throw std::invalid_argument("RowParallelLayer::forward requires batch*seq > 0");
        if (weight_.codes.empty()) throw std::runtime_error("RowParallelLayer::forward called before set_weight");
        cudaStream_t s = stream_.get();
        act_.quantize(input, NQ_F32, m, weight_.k, s);
        reducer_.run(act_, weight_, output, m, s);
    }
    // The same from per-token codes already made (TensorParallelMLP's h).
    void forward_codes(const tp_detail::TokenCodes& codes, float* output, int m) {
        reducer_.run(codes, weight_, output, m, stream_.get());
    }
    void copy_weight_shard(float* host_out) const {
        const auto w = weight_.dequantized();
        std::memcpy(host_out, w.data(), w.size() * sizeof(float));
    }
    // Loads an already-sliced (and, for the MLP, zero-padded) shard.
    void set_weight_shard(const float* shard, int k_local) { weight_.load(shard, k_local, out_features_, stream_.get()); }
    cudaStream_t stream() { return stream_.get(); }
    bool fused_all_reduce(int k) const { return reducer_.fused(k); }
    [[nodiscard]] int in_features() const { return in_features_; }
    [[nodiscard]] int out_features() const { return out_features_; }
    [[nodiscard]] int tp_degree() const { return std::max(1, ctx_.device_count()); }

private:
    ::cuda::nccl::NcclContext& ctx_;
    int in_features_, out_features_;
    tp_detail::RowReducer reducer_;
    tp_detail::Fp8Weight weight_;
    tp_detail::TokenCodes act_;
    tp_detail::LayerStream stream_;
};

// out = down( silu(x W_gate) .* (x W_up) ) (tensor_parallel_layers.h:328,
// forward :561-579): gate/up column-parallel, down row-parallel.
class TensorParallelMLP {
public:
    TensorParallelMLP(::cuda::nccl::NcclContext& ctx, int hidden_dim, int intermediate_size,
                      TpAllReduce mode = TpAllReduce::Auto)
        : ctx_(ctx), hidden_dim_(hidden_dim), intermediate_size_(intermediate_size),
          down_(ctx, intermediate_size > 0 ? intermediate_size : 1, hidden_dim > 0 ? hidden_dim : 1, mode) {
        if (hidden_dim_ <= 0 || intermediate_size_ <= 0)
            throw std::invalid_argument("TensorParallelMLP requires positive hidden_dim and intermediate_size");
        if (tp_degree() > 1 && intermediate_size_ % tp_degree() != 0)
            throw std::invalid_argument("TensorParallelMLP requires intermediate_size divisible by the tp degree");
        if (hidden_dim_ % 16 != 0)
            throw std::invalid_argument("TensorParallelMLP requires hidden_dim % 16 == 0 (tensor-core GEMM rows)");
        local_ = intermediate_size_ / tp_degree();
        pad_ = (local_ + 127) / 128 * 128;
    }
    TensorParallelMLP(const TensorParallelMLP&) = delete;
    TensorParallelMLP& operator=(const TensorParallelMLP&) = delete;

    // Full weights, host fp32: gate / up [hidden x intermediate], down
    // [intermediate x hidden], row-major.
    void set_weight(const float* gate_weight, const float* up_weight, const float* down_weight) {
        const int tp = tp_degree();
        const int rank = tp > 1 ? ctx_.rank_of_device(tp_detail::current_device()) : 0;
        const int H = hidden_dim_, I = intermediate_size_;
        // [g_0 | u_0 | g_1 | u_1 | ...], 128-column blocks of this rank's shard, zero past local_
        std::vector<float> packed(static_cast<size_t>(H) * 2 * pad_, 0.0f);
        for (int i = 0; i < H; ++i)
            for (int c = 0; c < local_; ++c) {
                const int blk = c / 128, col = c % 128;
                const size_t src = static_cast<size_t>(i) * I + static_cast<size_t>(rank) * local_ + c;
                float* row = &packed[static_cast<size_t>(i) * 2 * pad_ + static_cast<size_t>(blk) * 256];
                row[col] = gate_weight[src];
                row[128 + col] = up_weight[src];
            }
        gate_up_.load(packed.data(), H, 2 * pad_, down_.stream());
        std::vector<float> down(static_cast<size_t>(pad_) * H, 0.0f);
        std::memcpy(down.data(), down_weight + static_cast<size_t>(rank) * local_ * H,
                    static_cast<size_t>(local_) * H * sizeof(float));
        down_.set_weight_shard(down.data(), pad_);
    }
    // input [batch*seq x hidden] -> output [batch*seq x hidden] (replicated),
    // device fp32, synchronous.
    void forward(const float* input, float* output, int batch, int seq) {
        const int m = batch * seq;
        if (m <= 0) throw std::invalid_argument("TensorParallelMLP::forward requires batch*seq > 0");
        if (gate_up_.codes.empty()) throw std::runtime_error("TensorParallelMLP::forward called before set_weight");
        cudaStream_t s = down_.stream();
        x_.quantize(input, NQ_F32, m, hidden_dim_, s);
        h_.ensure(static_cast<size_t>(m) * pad_ * 2);
        const nq_gemm_desc_t d = tp_detail::gemm_desc(m, 2 * pad_, hidden_dim_, NQ_BF16, x_.scales.as<float>(),
                                                      gate_up_.scales.as<float>(), NQ_EPI_SWIGLU);
        tp_detail::check(nq_gemm(&d, x_.codes.as<uint8_t>(), gate_up_.codes.as<uint8_t>(), h_.as<void>(), s),
                         "TensorParallelMLP::forward: gate/up");
        hq_.quantize(h_.as<void>(), NQ_BF16, m, pad_, s);
        down_.forward_codes(hq_, output, m);
    }
    // This rank's shards, dequantized: gate / up [hidden x intermediate/tp],
    // down [intermediate/tp x hidden].
    void copy_weights(float* host_gate, float* host_up, float* host_down) const {
        const auto gu = gate_up_.dequantized();
        for (int i = 0; i < hidden_dim_; ++i)
            for (int c = 0; c < local_; ++c) {
                const size_t p = static_cast<size_t>(i) * 2 * pad_ + static_cast<size_t>(c / 128) * 256 + c % 128;
                host_gate[static_cast<size_t>(i) * local_ + c] = gu[p];
                host_up[static_cast<size_t>(i) * local_ + c] = gu[p + 128];
            }
        std::vector<float> dw(static_cast<size_t>(pad_) * hidden_dim_);
        down_.copy_weight_shard(dw.data());
        std::memcpy(host_down, dw.data(), static_cast<size_t>(local_) * hidden_dim_ * sizeof(float));
    }
    [[nodiscard]] int hidden_dim() const { return hidden_dim_; }
    [[nodiscard]] int intermediate_size() const { return intermediate_size_; }
    [[nodiscard]] int tp_degree() const { return std::max(1, ctx_.device_count()); }
    // True when the down projection reduces inside its GEMM (else ncclAllReduce).
    bool fused_all_reduce() const { return down_.fused_all_reduce(pad_); }

private:
    ::cuda::nccl::NcclContext& ctx_;
    int hidden_dim_, intermediate_size_;
    int local_ = 0, pad_ = 0;
    RowParallelLayer down_;
    tp_detail::Fp8Weight gate_up_;
    tp_detail::TokenCodes x_, hq_;
    tp_detail::DeviceBuffer h_;
};

}  // namespace neural
}  // namespace cuda
