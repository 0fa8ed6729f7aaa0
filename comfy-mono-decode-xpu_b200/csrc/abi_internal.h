// Internal helpers shared by the C-ABI translation units: status codes, the thread-local error message.
#pragma once
#include <cstdarg>
#include <cstdint>
#include <cstdio>
#include <cuda_runtime.h>

#include "../../include/mono_b200.h"

namespace mono {

// Record an error message for mono_last_error() and return `code`.
int fail(int code, const char* fmt, ...);

#define CUDA_TRY(expr)                                                                                  \
    do {                                                                                                \
        cudaError_t err_ = (expr);                                                                      \
        if (err_ != cudaSuccess)                                                                        \
            return ::mono::fail(MONO_ECUDA, "%s failed: %s (%s:%d)", #expr, cudaGetErrorString(err_), __FILE__, \
                                __LINE__);                                                              \
    } while (0)

#define MONO_CHECK(cond, ...)                                    \
    do {                                                         \
        if (!(cond)) return ::mono::fail(MONO_EINVAL, __VA_ARGS__); \
    } while (0)

inline bool aligned(const void* p, uintptr_t a) { return (reinterpret_cast<uintptr_t>(p) & (a - 1)) == 0; }

// Per-device SM count, cached.
int sm_count();

}  // namespace mono
