// fcai_common.h -- error reporting and small device helpers shared by the
// library's translation units.
#pragma once

#include <cuda_runtime.h>
#include <stdint.h>

#include <cstdarg>
#include <cstdio>

namespace fcai {

// Records a message for fcai_last_error() on the calling thread and returns
// `code`, so call sites can write `return fail(code, ...)`.
int fail(int code, const char *fmt, ...);
void clear_error();

// Multiprocessor count of the current device (cached per device).
int sm_count();

}  // namespace fcai

#define FCAI_CUDA_TRY(expr)                                                                  \
    do {                                                                                     \
        cudaError_t fcai_e_ = (expr);                                                        \
        if (fcai_e_ != cudaSuccess)                                                          \
            return ::fcai::fail(FCAI_ERR_CUDA, "%s failed: %s", #expr, cudaGetErrorString(fcai_e_)); \
    } while (0)
