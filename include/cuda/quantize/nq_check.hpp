// nq_check.hpp -- error plumbing shared by the drop-in C++ headers.
//
// The reference reports kernel-launch errors on stderr and continues
// (e.g. src/cuda/quantize/int8_kernels.cu:214-217) and throws
// ::cuda::device::CudaException for allocation / synchronisation errors
// (include/cuda/device/error.h:13, calibrator.cpp:22).  The shims keep the two
// behaviours: nq_report() prints, nq_throw_if() throws nova::quantize::NqError.
#ifndef NOVA_B200_NQ_CHECK_HPP
#define NOVA_B200_NQ_CHECK_HPP

#include <cstdio>
#include <stdexcept>
#include <string>

#include "../../nova_q.h"

namespace nova {
namespace quantize {

class NqError : public std::runtime_error {
public:
    NqError(nq_status_t st, const std::string& where)
        : std::runtime_error(where + ": " + nq_status_string(st) + ": " + nq_last_error()), status_(st) {}
    nq_status_t status() const noexcept { return status_; }

private:
    nq_status_t status_;
};

namespace detail {
inline void nq_report(nq_status_t st, const char* where) {
    if (st != NQ_SUCCESS) std::fprintf(stderr, "CUDA error in %s: %s: %s\n", where, nq_status_string(st), nq_last_error());
}
inline void nq_throw_if(nq_status_t st, const char* where) {
    if (st != NQ_SUCCESS) throw NqError(st, where);
}
}  // namespace detail

}  // namespace quantize
}  // namespace nova

#endif
