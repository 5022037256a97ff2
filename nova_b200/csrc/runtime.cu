// Runtime support of libnova_q: status strings, thread-local error text,
// device properties, the scratch pool and the device-side error word.
#include <cstdio>
#include <mutex>

#include "nq_internal.h"
#include "ptx.cuh"

// Device error word: kernels OR bits in here instead of trapping (bit 0: a
// bounded wait gave up).  One per device, read by nq_device_error_flags.
__device__ uint32_t nq_device_error_word = 0;

namespace nq {

namespace {
thread_local std::string g_last_error;
std::mutex g_mu;
DeviceInfo g_info[64];
cudaMemPool_t g_pool[64] = {};
}  // namespace

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
    std::lock_guard<std::mutex> lk(g_mu);
    DeviceInfo& d = g_info[dev];
    if (d.device != dev) {
        cudaDeviceProp p;
        e = cudaGetDeviceProperties(&p, dev);
        if (e != cudaSuccess) return cuda_status(e, "cudaGetDeviceProperties");
        d.device = dev;
        d.sm_count = p.multiProcessorCount;
        d.major = p.major;
        d.minor = p.minor;
        d.max_smem_optin = p.sharedMemPerBlockOptin;
    }
    if (d.major != 10)
        return fail(NQ_ERROR_NO_DEVICE, "libnova_q is built for sm_100a (B200); the current device is sm_" +
                                            std::to_string(d.major) + std::to_string(d.minor));
    *out = d;
    return NQ_SUCCESS;
}

nq_status_t scratch_alloc(void** p, size_t bytes, cudaStream_t s) {
    int dev = -1;
    NQ_CHECK_CUDA(cudaGetDevice(&dev), "cudaGetDevice");
    cudaMemPool_t pool;
    {
        std::lock_guard<std::mutex> lk(g_mu);
        if (!g_pool[dev]) {
            cudaMemPoolProps props = {};
            props.allocType = cudaMemAllocationTypePinned;
            props.location.type = cudaMemLocationTypeDevice;
            props.location.id = dev;
            NQ_CHECK_CUDA(cudaMemPoolCreate(&g_pool[dev], &props), "cudaMemPoolCreate");
            uint64_t keep = UINT64_MAX;  // keep freed blocks cached in the pool
            NQ_CHECK_CUDA(cudaMemPoolSetAttribute(g_pool[dev], cudaMemPoolAttrReleaseThreshold, &keep),
                          "cudaMemPoolSetAttribute");
        }
        pool = g_pool[dev];
    }
    NQ_CHECK_CUDA(cudaMallocFromPoolAsync(p, bytes, pool, s), "cudaMallocFromPoolAsync");
    return NQ_SUCCESS;
}

void scratch_free(void* p, cudaStream_t s) {
    if (p) cudaFreeAsync(p, s);
}

uint32_t* device_error_word() {
    // Host code cannot name a __device__ variable's address directly: the
    // symbol's address is looked up once per device with that device current.
    static uint32_t* addr[64] = {};
    int dev = 0;
    if (cudaGetDevice(&dev) != cudaSuccess || dev < 0 || dev >= 64) return nullptr;
    std::lock_guard<std::mutex> lk(g_mu);
    if (!addr[dev]) {
        void* p = nullptr;
        if (cudaGetSymbolAddress(&p, nq_device_error_word) != cudaSuccess) return nullptr;
        addr[dev] = static_cast<uint32_t*>(p);
    }
    return addr[dev];
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
    }
    return NQ_SUCCESS;
}

}  // extern "C"
