// Internal host-side helpers shared by the libnova_q translation units.
#pragma once

#include <cuda_runtime.h>

#include <atomic>
#include <cstddef>
#include <cstdint>
#include <mutex>
#include <string>
#include <utility>

#include "../../include/nova_q.h"

namespace nq {

// Records `msg` as this thread's last error and returns `st`.
nq_status_t fail(nq_status_t st, const std::string& msg);
// Maps a CUDA error to a status (with context) or NQ_SUCCESS.
nq_status_t cuda_status(cudaError_t e, const char* what);

struct DeviceInfo {
    int device = -1;
    int sm_count = 0;
    int major = 0, minor = 0;
    size_t max_smem_optin = 0;
};
// Properties of the current device (cached per device).
nq_status_t current_device(DeviceInfo* out);

// Launch with programmatic stream serialization: the kernel triggers its
// dependents early (griddepcontrol.launch_dependents) and waits for its
// predecessors (griddepcontrol.wait) before it touches memory they may write,
// so its prologue overlaps the previous kernel's tail.
template <class... P, class... A>
cudaError_t launch_pdl(void (*kern)(P...), dim3 grid, dim3 block, size_t smem, cudaStream_t s, A&&... args) {
    cudaLaunchConfig_t cfg = {};
    cfg.gridDim = grid;
    cfg.blockDim = block;
    cfg.dynamicSmemBytes = smem;
    cfg.stream = s;
    cudaLaunchAttribute at[1];
    at[0].id = cudaLaunchAttributeProgrammaticStreamSerialization;
    at[0].val.programmaticStreamSerializationAllowed = 1;
    cfg.attrs = at;
    cfg.numAttrs = 1;
    return cudaLaunchKernelEx(&cfg, kern, std::forward<A>(args)...);
}

// Stream-ordered scratch from a library-owned memory pool of the current
// device: cudaMallocAsync after the first call on a device reuses the pool's
// cached blocks instead of reaching the driver.
nq_status_t scratch_alloc(void** p, size_t bytes, cudaStream_t s);
void scratch_free(void* p, cudaStream_t s);

// Zero-initialised flag words owned by (current device, stream), at least
// `count` of them, for kernels that clear every flag they raise before they
// finish (so the next launch on the stream finds them zero without a memset).
// While the stream is capturing a graph *p is nullptr: the caller then takes
// flags from its scratch and clears them inside the graph.
nq_status_t stream_flags(uint32_t** p, int count, cudaStream_t s);
// Clears every stream's flags of the current device (after a bounded wait has
// given up, a flag may have been left raised).  The device must be idle.
nq_status_t clear_stream_flags();

// Device address of the error word of the current device (kernels OR their
// error bits into it), or nullptr if it cannot be resolved.
uint32_t* device_error_word();

// Bound (ns) of a kernel's wait on counts that other GPUs send (the fused
// all-reduce); nq_set_peer_wait_limit changes it for kernels launched later.
uint64_t peer_wait_limit_ns();

inline bool aligned16(const void* p) { return (reinterpret_cast<uintptr_t>(p) & 15u) == 0; }

// Runs init() once per device for one call site (e.g. a kernel's shared-memory
// opt-in, a per-device function attribute).  Bit `device` of `done` is read
// without a lock; only a device's first call takes `mu`.
template <class F>
nq_status_t once_per_device(std::atomic<uint64_t>& done, std::mutex& mu, int device, F init) {
    const uint64_t bit = 1ull << (device & 63);
    if (done.load(std::memory_order_acquire) & bit) return NQ_SUCCESS;
    std::lock_guard<std::mutex> lk(mu);
    if (done.load(std::memory_order_relaxed) & bit) return NQ_SUCCESS;
    nq_status_t st = init();
    if (st == NQ_SUCCESS) done.fetch_or(bit, std::memory_order_release);
    return st;
}

}  // namespace nq

#define NQ_CHECK_CUDA(call, what)                                   \
    do {                                                            \
        cudaError_t e__ = (call);                                   \
        if (e__ != cudaSuccess) return ::nq::cuda_status(e__, what); \
    } while (0)

#define NQ_LAUNCH_CHECK(what) NQ_CHECK_CUDA(cudaGetLastError(), what)
