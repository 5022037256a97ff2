// Runtime support of libnova_q: status strings, thread-local error text,
// device properties, the scratch pool and the device-side error word.
#include <atomic>
#include <cstdio>
#include <mutex>
#include <vector>

#include "nq_internal.h"
#include "ptx.cuh"

// Device error word: kernels OR bits in here instead of trapping (bit 0: a
// bounded wait gave up).  One per device, read by nq_device_error_flags.
__device__ uint32_t nq_device_error_word = 0;

namespace nq {

// Per-device caches are filled once under g_mu and then read without a lock
// (an acquire load of the slot), so no launch path takes a lock after a
// device's first call.
namespace {
thread_local std::string g_last_error;
std::mutex g_mu;
DeviceInfo g_info[64];
std::atomic<bool> g_info_ready[64];
std::atomic<cudaMemPool_t> g_pool[64];
std::atomic<uint32_t*> g_err_word[64];
constexpr uint64_t kDefaultPeerWaitNs = 5000000000ull;  // 5 s: a peer's kernel may start a little later
std::atomic<uint64_t> g_peer_wait_ns{kDefaultPeerWaitNs};
}  // namespace

uint64_t peer_wait_limit_ns() { return g_peer_wait_ns.load(std::memory_order_relaxed); }

nq_status_t fail(nq_status_t st, const std::string& msg) {
    g_last_error = msg;
    return st;
}

nq_status_t cuda_status(cudaError_t e, const char* what) {
    if (e == cudaSuccess) return NQ_SUCCESS;
    std::string m = std::string(what) + ": " + cudaGetErrorName(e) + " (" + cudaGetErrorString(e) + ")";
    if (e == cudaErrorMemoryAllocation) return fail(NQ_ERROR_OUT_OF_MEMORY, m);
    if (e == cudaErrorNoDevice || e == cudaErrorInsufficientDriver) return fail(NQ_ERROR_NO_DEVICE, m);
    return fail(NQ_ERROR_CUDA, m);
}

nq_status_t current_device(DeviceInfo* out) {
    int dev = -1;
    cudaError_t e = cudaGetDevice(&dev);
    if (e != cudaSuccess) return cuda_status(e, "cudaGetDevice");
    if (dev < 0 || dev >= 64) return fail(NQ_ERROR_NO_DEVICE, "device ordinal out of range");
    if (!g_info_ready[dev].load(std::memory_order_acquire)) {
        std::lock_guard<std::mutex> lk(g_mu);
        if (!g_info_ready[dev].load(std::memory_order_relaxed)) {
            cudaDeviceProp p;
            e = cudaGetDeviceProperties(&p, dev);
            if (e != cudaSuccess) return cuda_status(e, "cudaGetDeviceProperties");
            DeviceInfo& w = g_info[dev];
            w.device = dev;
            w.sm_count = p.multiProcessorCount;
            w.major = p.major;
            w.minor = p.minor;
            w.max_smem_optin = p.sharedMemPerBlockOptin;
            g_info_ready[dev].store(true, std::memory_order_release);
        }
    }
    const DeviceInfo& d = g_info[dev];
    if (d.major != 10)
        return fail(NQ_ERROR_NO_DEVICE, "libnova_q is built for sm_100a (B200); the current device is sm_" +
                                            std::to_string(d.major) + std::to_string(d.minor));
    *out = d;
    return NQ_SUCCESS;
}

nq_status_t scratch_alloc(void** p, size_t bytes, cudaStream_t s) {
    int dev = -1;
    NQ_CHECK_CUDA(cudaGetDevice(&dev), "cudaGetDevice");
    if (dev < 0 || dev >= 64) return fail(NQ_ERROR_NO_DEVICE, "device ordinal out of range");
    cudaMemPool_t pool = g_pool[dev].load(std::memory_order_acquire);
    if (!pool) {
        std::lock_guard<std::mutex> lk(g_mu);
        pool = g_pool[dev].load(std::memory_order_relaxed);
        if (!pool) {
            cudaMemPoolProps props = {};
            props.allocType = cudaMemAllocationTypePinned;
            props.location.type = cudaMemLocationTypeDevice;
            props.location.id = dev;
            NQ_CHECK_CUDA(cudaMemPoolCreate(&pool, &props), "cudaMemPoolCreate");
            uint64_t keep = UINT64_MAX;  // keep freed blocks cached in the pool
            NQ_CHECK_CUDA(cudaMemPoolSetAttribute(pool, cudaMemPoolAttrReleaseThreshold, &keep),
                          "cudaMemPoolSetAttribute");
            g_pool[dev].store(pool, std::memory_order_release);
        }
    }
    NQ_CHECK_CUDA(cudaMallocFromPoolAsync(p, bytes, pool, s), "cudaMallocFromPoolAsync");
    return NQ_SUCCESS;
}

void scratch_free(void* p, cudaStream_t s) {
    if (p) cudaFreeAsync(p, s);
}

namespace {
constexpr int kStreamFlagWords = 4096;
struct StreamFlags {
    int device;
    cudaStream_t stream;
    uint32_t* words;
};
std::mutex g_flags_mu;
std::vector<StreamFlags> g_flags;  // kept for the life of the process (16 KB per stream used)
}  // namespace

nq_status_t stream_flags(uint32_t** p, int count, cudaStream_t s) {
    *p = nullptr;
    if (count > kStreamFlagWords) return fail(NQ_ERROR_INVALID_VALUE, "stream flags: too many words requested");
    cudaStreamCaptureStatus cs = cudaStreamCaptureStatusNone;
    NQ_CHECK_CUDA(cudaStreamIsCapturing(s, &cs), "cudaStreamIsCapturing");
    if (cs != cudaStreamCaptureStatusNone) return NQ_SUCCESS;
    int dev = -1;
    NQ_CHECK_CUDA(cudaGetDevice(&dev), "cudaGetDevice");
    std::lock_guard<std::mutex> lk(g_flags_mu);
    for (const auto& f : g_flags)
        if (f.device == dev && f.stream == s) {
            *p = f.words;
            return NQ_SUCCESS;
        }
    uint32_t* w = nullptr;
    if (cudaMalloc(&w, kStreamFlagWords * sizeof(uint32_t)) != cudaSuccess) {
        // e.g. another thread is capturing a graph in global mode: the caller
        // takes per-launch flags this time
        (void)cudaGetLastError();
        return NQ_SUCCESS;
    }
    cudaError_t e = cudaMemsetAsync(w, 0, kStreamFlagWords * sizeof(uint32_t), s);
    if (e != cudaSuccess) {
        cudaFree(w);
        return cuda_status(e, "cudaMemsetAsync(stream flags)");
    }
    g_flags.push_back({dev, s, w});
    *p = w;
    return NQ_SUCCESS;
}

nq_status_t clear_stream_flags() {
    int dev = -1;
    NQ_CHECK_CUDA(cudaGetDevice(&dev), "cudaGetDevice");
    std::lock_guard<std::mutex> lk(g_flags_mu);
    for (const auto& f : g_flags)
        if (f.device == dev)
            NQ_CHECK_CUDA(cudaMemset(f.words, 0, kStreamFlagWords * sizeof(uint32_t)), "cudaMemset(stream flags)");
    return NQ_SUCCESS;
}

uint32_t* device_error_word() {
    // Host code cannot name a __device__ variable's address directly: the
    // symbol's address is looked up once per device with that device current.
    int dev = 0;
    if (cudaGetDevice(&dev) != cudaSuccess || dev < 0 || dev >= 64) return nullptr;
    uint32_t* a = g_err_word[dev].load(std::memory_order_acquire);
    if (a) return a;
    std::lock_guard<std::mutex> lk(g_mu);
    a = g_err_word[dev].load(std::memory_order_relaxed);
    if (!a) {
        void* p = nullptr;
        if (cudaGetSymbolAddress(&p, nq_device_error_word) != cudaSuccess) return nullptr;
        a = static_cast<uint32_t*>(p);
        g_err_word[dev].store(a, std::memory_order_release);
    }
    return a;
}

}  // namespace nq

extern "C" {

const char* nq_status_string(nq_status_t s) {
    switch (s) {
        case NQ_SUCCESS: return "NQ_SUCCESS";
        case NQ_ERROR_INVALID_VALUE: return "NQ_ERROR_INVALID_VALUE";
        case NQ_ERROR_UNSUPPORTED: return "NQ_ERROR_UNSUPPORTED";
        case NQ_ERROR_CUDA: return "NQ_ERROR_CUDA";
        case NQ_ERROR_OUT_OF_MEMORY: return "NQ_ERROR_OUT_OF_MEMORY";
        case NQ_ERROR_NO_DEVICE: return "NQ_ERROR_NO_DEVICE";
        case NQ_ERROR_DEVICE_TIMEOUT: return "NQ_ERROR_DEVICE_TIMEOUT";
    }
    return "NQ_UNKNOWN_STATUS";
}

const char* nq_last_error(void) { return nq::g_last_error.c_str(); }

int nq_version(void) { return 100; }

nq_status_t nq_set_peer_wait_limit(uint64_t ns) {
    nq::g_peer_wait_ns.store(ns ? ns : nq::kDefaultPeerWaitNs, std::memory_order_relaxed);
    return NQ_SUCCESS;
}

uint64_t nq_peer_wait_limit(void) { return nq::peer_wait_limit_ns(); }

nq_status_t nq_device_error_flags(uint32_t* flags, int clear) {
    if (!flags) return nq::fail(NQ_ERROR_INVALID_VALUE, "nq_device_error_flags: flags is null");
    nq::DeviceInfo di;
    nq_status_t st = nq::current_device(&di);
    if (st != NQ_SUCCESS) return st;
    NQ_CHECK_CUDA(cudaDeviceSynchronize(), "nq_device_error_flags: synchronize");
    NQ_CHECK_CUDA(cudaMemcpyFromSymbol(flags, nq_device_error_word, sizeof(uint32_t)),
                  "nq_device_error_flags: read");
    if (clear) {
        uint32_t z = 0;
        NQ_CHECK_CUDA(cudaMemcpyToSymbol(nq_device_error_word, &z, sizeof(uint32_t)),
                      "nq_device_error_flags: clear");
        st = nq::clear_stream_flags();
        if (st != NQ_SUCCESS) return st;
        NQ_CHECK_CUDA(cudaDeviceSynchronize(), "nq_device_error_flags: clear flags");
    }
    return NQ_SUCCESS;
}

}  // extern "C"
