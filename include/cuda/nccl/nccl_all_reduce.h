// nccl_all_reduce.h -- drop-in for pplmx/nova's cuda::nccl::NcclAllReduce
// (include/cuda/nccl/nccl_all_reduce.h, src/cuda/nccl/nccl_all_reduce.cpp:
// 21-61), header-only: ncclAllReduce on the calling thread's device
// communicator, then a bounded wait for the stream (safe_stream_wait) that
// reports timeouts and asynchronous errors as an NcclResult.
#pragma once

#include "nccl_context.h"

namespace cuda {
namespace nccl {

class NcclAllReduce {
public:
    explicit NcclAllReduce(NcclContext& ctx) : ctx_(&ctx) {}
    NcclAllReduce(const NcclAllReduce&) = delete;
    NcclAllReduce& operator=(const NcclAllReduce&) = delete;
    NcclAllReduce(NcclAllReduce&&) = default;
    NcclAllReduce& operator=(NcclAllReduce&&) = default;

    // Enqueues the all-reduce on `stream` and waits for it (bounded by the
    // context's timeout); the result carries the NCCL code, timed_out or
    // async_error.
    NcclResult all_reduce_async(const void* send_data, void* recv_data, size_t count, ncclDataType_t dtype,
                                ncclRedOp_t op, cudaStream_t stream) {
        NcclResult r;
        if (!ctx_->has_nccl()) {
            r.code = ncclInternalError;
            r.error_message = "NCCL context not initialized";
            return r;
        }
        ncclComm_t comm = nullptr;
        try {
            comm = ctx_->current_comm();
        } catch (const std::exception& e) {
            r.code = ncclInvalidArgument;
            r.error_message = e.what();
            return r;
        }
        const ncclResult_t e = ncclAllReduce(send_data, recv_data, count, dtype, op, comm, stream);
        if (e != ncclSuccess) {
            r.code = e;
            r.error_message = ncclGetErrorString(e);
            return r;
        }
        return safe_stream_wait(comm, stream, ctx_->timeout_ms(), ctx_);
    }
    NcclResult all_reduce(const void* send_data, void* recv_data, size_t count, ncclDataType_t dtype, ncclRedOp_t op,
                          cudaStream_t stream) {
        return all_reduce_async(send_data, recv_data, count, dtype, op, stream);
    }

private:
    NcclContext* ctx_;
};

}  // namespace nccl
}  // namespace cuda
