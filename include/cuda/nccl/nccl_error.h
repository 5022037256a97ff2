// nccl_error.h -- drop-in include path of pplmx/nova's NcclResult and
// safe_stream_wait (include/cuda/nccl/nccl_error.h, src/cuda/nccl/
// nccl_error.cpp:13-83); both are defined in nccl_context.h.
#pragma once

#include "nccl_context.h"
