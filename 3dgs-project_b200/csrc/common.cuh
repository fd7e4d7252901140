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

// A size bound of the caller's inputs is exceeded (e.g. more instances than 32-bit lists index, a capacity
// below its bound): SPLAT_ERR_OVERFLOW before any device work.
#define SPLAT_BOUND(cond, ...)                   \
    do {                                         \
        if (!(cond)) {                           \
            ::splat::set_error(__VA_ARGS__);     \
            return SPLAT_ERR_OVERFLOW;           \
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

// Records the caller's CUDA events (splat_time_kernel) on `st` just before (begin) and after (end) a launch of the
// named kernel; a no-op unless a timer is set. `kernel` must be the literal name the timer table lists.
void timer_mark(const char* kernel, bool begin, cudaStream_t st);

// Launches `launch` (a kernel launch statement) on stream `st` between the timer marks of `name`.
#define SPLAT_TIMED_LAUNCH(name, st, launch)    \
    do {                                        \
        ::splat::timer_mark(name, true, st);    \
        launch;                                 \
        ::splat::timer_mark(name, false, st);   \
    } while (0)

constexpr unsigned int kFullMask = 0xffffffffu;

// One halving step of a warp sum of N values per lane: lanes with the `off` bit clear keep the first ceil(N/2)
// partial sums, the others the rest, each adding its partner's copy of the half it keeps. Four steps (16, 8, 4,
// 2) and a last exchange (1) leave value k's total in the lanes whose bits 4..1 spell k's position.
template <int N>
__device__ __forceinline__ void fold_half(const float (&v)[N], float (&out)[(N + 1) / 2], int off, bool upper) {
    constexpr int H = (N + 1) / 2;
#pragma unroll
    for (int i = 0; i < H; ++i) {
        const float hi = i + H < N ? v[i + H] : 0.f;
        const float recv = __shfl_xor_sync(kFullMask, upper ? v[i] : hi, off);
        out[i] = (upper ? hi : v[i]) + recv;
    }
}

// Warp sums of nine values: after the call, every lane's t holds one total; the totals of values 0..8 are in
// lanes 0, 2, 4, 8, 10, 16, 18, 20, 24 (kFold9Lane).
__device__ __forceinline__ float warp_fold9(const float (&v9)[9], int lane) {
    float f5[5], f3[3], f2[2], f1[1];
    fold_half<9>(v9, f5, 16, lane & 16);
    fold_half<5>(f5, f3, 8, lane & 8);
    fold_half<3>(f3, f2, 4, lane & 4);
    fold_half<2>(f2, f1, 2, lane & 2);
    return f1[0] + __shfl_xor_sync(kFullMask, f1[0], 1);
}
constexpr int kFold9Lane[9] = {0, 2, 4, 8, 10, 16, 18, 20, 24};

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
