// Shared helpers for the unum_ops_b200 kernels: error reporting across the
// C ABI and small device utilities.
#pragma once

#include <cuda_runtime.h>
#include <stdint.h>
#include <cstdarg>
#include <cstdio>

#include "../../include/unum_ops_b200.h"

namespace unum {

// Thread-local message of the last failing entry point (read by unum_last_error).
void set_error(const char *fmt, ...);
void clear_error();

#define UNUM_CHECK_ARG(cond, ...)              \
    do {                                       \
        if (!(cond)) {                         \
            ::unum::set_error(__VA_ARGS__);    \
            return UNUM_ERR_INVALID;           \
        }                                      \
    } while (0)

#define UNUM_CHECK_CUDA(expr)                                                          \
    do {                                                                               \
        cudaError_t e_ = (expr);                                                       \
        if (e_ != cudaSuccess) {                                                       \
            ::unum::set_error("%s failed: %s", #expr, cudaGetErrorString(e_));         \
            return UNUM_ERR_CUDA;                                                      \
        }                                                                              \
    } while (0)

// Check the launch that was just enqueued.
inline int check_launch(const char *what) {
    cudaError_t e = cudaGetLastError();
    if (e != cudaSuccess) {
        set_error("%s launch failed: %s", what, cudaGetErrorString(e));
        return UNUM_ERR_CUDA;
    }
    return UNUM_OK;
}

inline int sm_count() {
    int dev = 0, n = 0;
    cudaGetDevice(&dev);
    cudaDeviceGetAttribute(&n, cudaDevAttrMultiProcessorCount, dev);
    return n > 0 ? n : 148;
}

inline bool aligned16(const void *p) { return (reinterpret_cast<uintptr_t>(p) & 15u) == 0; }

}  // namespace unum
