// common.cuh - status codes, error reporting and small device helpers shared by every kernel file.
//
// Every C-ABI entry point returns an int status (SPLAT_OK == 0) and never throws. A failing call
// stores a one-line message in a thread-local buffer that splat_last_error() returns, so the Python
// layer can raise the same RuntimeError text the reference's TORCH_CHECKs raise.
#pragma once

#include <cuda_runtime.h>
#include <stdint.h>
#include <stdio.h>
#include <stdarg.h>

#include "../../include/splat_b200.h"

namespace splat {

void set_error(const char* fmt, ...);

// Records the pending launch error (if any) and converts it to a status.
int check_launch(const char* what);

#define SPLAT_REQUIRE(cond, ...)                 \
    do {                                         \
        if (!(cond)) {                           \
            ::splat::set_error(__VA_ARGS__);     \
            return SPLAT_ERR_ARG;                \
        }                                        \
    } while (0)

#define SPLAT_CUDA(call)                                                           \
    do {                                                                           \
        cudaError_t e_ = (call);                                                   \
        if (e_ != cudaSuccess) {                                                   \
            ::splat::set_error("%s failed: %s", #call, cudaGetErrorString(e_));    \
            return SPLAT_ERR_CUDA;                                                 \
        }                                                                          \
    } while (0)

#define SPLAT_TRY(expr)             \
    do {                            \
        int s_ = (expr);            \
        if (s_ != SPLAT_OK) return s_; \
    } while (0)

inline unsigned int div_up(long long a, long long b) { return static_cast<unsigned int>((a + b - 1) / b); }

inline cudaStream_t as_stream(void* s) { return reinterpret_cast<cudaStream_t>(s); }

// Number of SMs of the current device (cached per device id).
int sm_count();

// Counts one kernel launch of this library (every launch site calls it; read by splat_launch_count).
void note_launch();

constexpr unsigned int kFullMask = 0xffffffffu;

// ---- workspace carving: one caller-owned byte buffer split into 256-byte aligned pieces ----
struct Carver {
    char* base;
    size_t size;
    size_t used;
    __host__ Carver(void* b, size_t s) : base(static_cast<char*>(b)), size(s), used(0) {}
    template <typename T>
    __host__ T* take(size_t count) {
        used = (used + 255) & ~size_t(255);
        T* p = reinterpret_cast<T*>(base ? base + used : nullptr);
        used += count * sizeof(T);
        return p;
    }
    __host__ bool fits() const { return used <= size; }
};

}  // namespace splat
