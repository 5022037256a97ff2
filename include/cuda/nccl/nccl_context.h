// nccl_context.h -- drop-in for pplmx/nova's cuda::nccl::NcclContext
// (include/cuda/nccl/nccl_context.h), NcclException, NcclResult
// (include/cuda/nccl/nccl_error.h:61) and safe_stream_wait
// (src/cuda/nccl/nccl_error.cpp:13-83), header-only.
//
// One process drives every GPU of the group, one host thread per GPU (the
// reference's model): initialize() creates one communicator and one stream per
// device with ncclCommInitAll and, beyond the reference, enables peer access
// between every pair of the group's GPUs, so that the GEMM-fused all-reduce of
// the TP layers (libnova_q, nq_gemm_allreduce) can read and write the other
// GPUs' buffers through their plain device pointers.  Two more additions serve
// those layers: next_layer_id() numbers the layers each device builds (the
// n-th layer built on every device is the same logical layer) and exchange()
// is a host rendezvous through which the per-device instances of a layer
// swap buffer addresses.
#pragma once

#include <cuda_runtime.h>
#include <nccl.h>

#include <algorithm>
#include <atomic>
#include <chrono>
#include <condition_variable>
#include <cstdint>
#include <map>
#include <mutex>
#include <stdexcept>
#include <string>
#include <thread>
#include <vector>

namespace cuda {
namespace nccl {

#define NCCL_CHECK(call)                                                                     \
    do {                                                                                     \
        ncclResult_t nccl_err__ = (call);                                                    \
        if (nccl_err__ != ncclSuccess) {                                                     \
            throw ::cuda::nccl::NcclException(ncclGetErrorString(nccl_err__), nccl_err__, #call, \
                                              __FILE__, __LINE__);                           \
        }                                                                                    \
    } while (0)

// An NCCL (or collective) failure with its code, the failed expression and
// where it happened (nccl_context.h of the reference).
class NcclException : public std::runtime_error {
public:
    NcclException(const char* msg, ncclResult_t code, const char* expr, const char* file, int line)
        : std::runtime_error(format_message(msg, expr, file, line)),
          error_code_(code), expression_(expr), file_(file), line_(line) {}
    [[nodiscard]] ncclResult_t error_code() const noexcept { return error_code_; }
    [[nodiscard]] const char* expression() const noexcept { return expression_; }
    [[nodiscard]] const char* file() const noexcept { return file_; }
    [[nodiscard]] int line() const noexcept { return line_; }

private:
    ncclResult_t error_code_;
    const char* expression_;
    const char* file_;
    int line_;
    static std::string format_message(const char* msg, const char* expr, const char* file, int line) {
        return std::string("NCCL error: ") + (msg ? msg : "") + " in " + (expr ? expr : "?") + " at " +
               (file ? file : "?") + ":" + std::to_string(line);
    }
};

// Outcome of a collective: the NCCL code, whether a deadline ran out, whether
// the communicator reported an asynchronous error (nccl_error.h:61).
struct NcclResult {
    ncclResult_t code = ncclSuccess;
    bool timed_out = false;
    bool async_error = false;
    std::string error_message;
    [[nodiscard]] bool ok() const { return code == ncclSuccess && !timed_out && !async_error; }
    explicit operator bool() const { return ok(); }
};

struct NcclContextConfig {
    std::vector<int> device_ids;  // empty: every visible device
    bool debug = false;
    int timeout_ms = 30000;       // bound of collectives and of the layers' rendezvous
};

class NcclContext {
public:
    static NcclContext& instance() {
        static NcclContext ctx;
        return ctx;
    }
    NcclContext() = default;
    explicit NcclContext(const NcclContextConfig& config) { initialize(config); }
    NcclContext(const NcclContext&) = delete;
    NcclContext& operator=(const NcclContext&) = delete;
    NcclContext(NcclContext&& other) noexcept { take(other); }
    NcclContext& operator=(NcclContext&& other) noexcept {
        if (this != &other) {
            destroy();
            take(other);
        }
        return *this;
    }
    ~NcclContext() { destroy(); }

    void initialize() { initialize(NcclContextConfig{}); }

    // One communicator and stream per device of the group (ncclCommInitAll),
    // peer access between every pair; the calling thread's device is restored.
    void initialize(const NcclContextConfig& config) {
        std::lock_guard<std::mutex> lk(init_mutex_);
        if (initialized_) return;
        int prev = 0;
        cudaGetDevice(&prev);
        std::vector<int> ids = config.device_ids;
        if (ids.empty()) {
            int n = 0;
            if (cudaGetDeviceCount(&n) != cudaSuccess || n <= 0)
                throw NcclException("no CUDA device", ncclInvalidUsage, "cudaGetDeviceCount", __FILE__, __LINE__);
            for (int d = 0; d < n; ++d) ids.push_back(d);
        }
        std::vector<ncclComm_t> comms(ids.size(), nullptr);
        NCCL_CHECK(ncclCommInitAll(comms.data(), static_cast<int>(ids.size()), ids.data()));
        std::vector<cudaStream_t> streams(ids.size(), nullptr);
        bool peers = true;
        for (size_t i = 0; i < ids.size(); ++i) {
            cudaSetDevice(ids[i]);
            if (cudaStreamCreateWithFlags(&streams[i], cudaStreamNonBlocking) != cudaSuccess) {
                for (auto c : comms) ncclCommDestroy(c);
                cudaSetDevice(prev);
                throw NcclException("cudaStreamCreate failed", ncclUnhandledCudaError, "initialize", __FILE__, __LINE__);
            }
            for (size_t j = 0; j < ids.size(); ++j) {
                if (i == j) continue;
                int can = 0;
                cudaDeviceCanAccessPeer(&can, ids[i], ids[j]);
                if (!can) {
                    peers = false;
                    continue;
                }
                const cudaError_t e = cudaDeviceEnablePeerAccess(ids[j], 0);
                if (e == cudaErrorPeerAccessAlreadyEnabled) cudaGetLastError();
                else if (e != cudaSuccess) peers = false;
            }
        }
        cudaSetDevice(prev);
        device_ids_ = ids;
        communicators_ = comms;
        streams_ = streams;
        device_count_ = static_cast<int>(ids.size());
        timeout_ms_ = config.timeout_ms > 0 ? config.timeout_ms : 30000;
        peer_access_ = peers;
        broken_.store(false, std::memory_order_release);
        initialized_ = true;
    }

    ncclComm_t get_comm(int device) const { return communicators_.at(index_of(device)); }
    [[nodiscard]] ncclComm_t current_comm() const {
        int d = 0;
        cudaGetDevice(&d);
        return get_comm(d);
    }
    cudaStream_t get_stream(int device) const { return streams_.at(index_of(device)); }
    // The device's NCCL rank: its position in the configured device list.
    [[nodiscard]] int rank_of_device(int device) const { return index_of(device); }
    [[nodiscard]] bool initialized() const { return initialized_; }
    [[nodiscard]] int device_count() const { return device_count_; }
    [[nodiscard]] bool has_nccl() const {
        return initialized_ && !broken_.load(std::memory_order_acquire) && !communicators_.empty();
    }
    // Forgets a communicator aborted after a timeout or an asynchronous error
    // and marks the context broken (has_nccl() false) until destroy() and a
    // new initialize().
    bool mark_comm_aborted(ncclComm_t comm) noexcept {
        std::lock_guard<std::mutex> lk(init_mutex_);
        for (auto& c : communicators_) {
            if (c == comm) {
                c = nullptr;
                broken_.store(true, std::memory_order_release);
                return true;
            }
        }
        return false;
    }
    [[nodiscard]] bool broken() const { return broken_.load(std::memory_order_acquire); }
    void destroy() {
        std::lock_guard<std::mutex> lk(init_mutex_);
        if (!initialized_) return;
        int prev = 0;
        cudaGetDevice(&prev);
        for (size_t i = 0; i < communicators_.size(); ++i) {
            if (communicators_[i]) ncclCommDestroy(communicators_[i]);
            if (streams_[i]) {
                cudaSetDevice(device_ids_[i]);
                cudaStreamDestroy(streams_[i]);
            }
        }
        cudaSetDevice(prev);
        communicators_.clear();
        streams_.clear();
        device_ids_.clear();
        device_count_ = 0;
        initialized_ = false;
        broken_.store(false, std::memory_order_release);
    }
    [[nodiscard]] const std::vector<int>& device_ids() const { return device_ids_; }
    [[nodiscard]] int timeout_ms() const { return timeout_ms_; }

    // ---- additions for the GEMM-fused all-reduce (no reference counterpart) ----
    // True when every pair of the group's GPUs can address each other's memory.
    [[nodiscard]] bool peer_access() const { return initialized_ && peer_access_; }
    // 0, 1, 2, ... for the TP layers built on `device`, in construction order.
    int next_layer_id(int device) {
        std::lock_guard<std::mutex> lk(rv_mutex_);
        return layer_ids_[device]++;
    }
    // Rendezvous of the group's ranks on `key`: rank r posts `value`, and every
    // rank gets all device_count() values in rank order once all have posted.
    // Throws NcclException (ncclSystemError) when a rank does not post within
    // timeout_ms().  Each key is used once by each rank.
    std::vector<uintptr_t> exchange(uint64_t key, int rank, uintptr_t value) {
        std::unique_lock<std::mutex> lk(rv_mutex_);
        Rendezvous& rv = rendezvous_[key];
        if (rv.values.empty()) rv.values.assign(device_count_, 0);
        rv.values.at(rank) = value;
        ++rv.posted;
        rv_cv_.notify_all();
        const bool all = rv_cv_.wait_for(lk, std::chrono::milliseconds(timeout_ms_),
                                         [&] { return rv.posted >= device_count_; });
        if (!all)
            throw NcclException("a rank did not reach the TP layer rendezvous in time", ncclSystemError,
                                "NcclContext::exchange", __FILE__, __LINE__);
        std::vector<uintptr_t> out = rv.values;
        if (++rv.taken == device_count_) rendezvous_.erase(key);
        return out;
    }

private:
    struct Rendezvous {
        std::vector<uintptr_t> values;
        int posted = 0;
        int taken = 0;
    };
    int index_of(int device) const {
        if (!initialized_) throw NcclException("NCCL context not initialized", ncclInvalidUsage, "NcclContext", __FILE__, __LINE__);
        const auto it = std::find(device_ids_.begin(), device_ids_.end(), device);
        if (it == device_ids_.end())
            throw NcclException(("device " + std::to_string(device) + " is not in the NCCL group").c_str(),
                                ncclInvalidArgument, "NcclContext::rank_of_device", __FILE__, __LINE__);
        return static_cast<int>(it - device_ids_.begin());
    }
    void take(NcclContext& o) {
        std::lock_guard<std::mutex> lk(o.init_mutex_);
        device_count_ = o.device_count_;
        communicators_ = std::move(o.communicators_);
        streams_ = std::move(o.streams_);
        device_ids_ = std::move(o.device_ids_);
        initialized_ = o.initialized_;
        timeout_ms_ = o.timeout_ms_;
        peer_access_ = o.peer_access_;
        broken_.store(o.broken_.load());
        o.device_count_ = 0;
        o.initialized_ = false;
    }

    int device_count_ = 0;
    std::vector<ncclComm_t> communicators_;
    std::vector<cudaStream_t> streams_;
    std::vector<int> device_ids_;
    bool initialized_ = false;
    bool peer_access_ = false;
    int timeout_ms_ = 30000;
    std::atomic<bool> broken_{false};
    mutable std::mutex init_mutex_;
    std::mutex rv_mutex_;
    std::condition_variable rv_cv_;
    std::map<uint64_t, Rendezvous> rendezvous_;
    std::map<int, int> layer_ids_;
};

// Waits for `stream` with a deadline, watching the communicator for
// asynchronous errors (nccl_error.cpp:13-83): on a CUDA error, an async NCCL
// error or the deadline, the communicator is aborted, the context (if given)
// marks it, and the result says which.
inline NcclResult safe_stream_wait(ncclComm_t comm, cudaStream_t stream, int timeout_ms, NcclContext* ctx = nullptr) {
    NcclResult result;
    const auto deadline = std::chrono::steady_clock::now() + std::chrono::milliseconds(timeout_ms);
    while (std::chrono::steady_clock::now() < deadline) {
        const cudaError_t e = cudaStreamQuery(stream);
        if (e == cudaSuccess) return result;
        if (e != cudaErrorNotReady) {
            result.code = ncclUnhandledCudaError;
            result.error_message = cudaGetErrorString(e);
            return result;
        }
        ncclResult_t async_err = ncclSuccess;
        if (comm && ncclCommGetAsyncError(comm, &async_err) != ncclSuccess) {
            result.code = ncclInternalError;
            result.error_message = "ncclCommGetAsyncError failed";
            return result;
        }
        if (async_err != ncclSuccess && async_err != ncclInProgress) {
            result.async_error = true;
            result.code = async_err;
            result.error_message = ncclGetErrorString(async_err);
            if (comm) ncclCommAbort(comm);
            if (ctx) ctx->mark_comm_aborted(comm);
            return result;
        }
        std::this_thread::sleep_for(std::chrono::milliseconds(1));
    }
    result.timed_out = true;
    result.code = ncclSystemError;
    result.error_message = "Stream wait timed out after " + std::to_string(timeout_ms) + "ms";
    if (comm) ncclCommAbort(comm);
    if (ctx) ctx->mark_comm_aborted(comm);
    return result;
}

}  // namespace nccl
}  // namespace cuda
