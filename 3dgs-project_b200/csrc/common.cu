// common.cu - error reporting and the launch counter shared by all entry points.
#include <atomic>

#include "common.cuh"

namespace splat {

namespace {
thread_local char g_error[1024] = "";
std::atomic<long long> g_launches{0};
}  // namespace

void note_launch() { g_launches.fetch_add(1, std::memory_order_relaxed); }

void set_error(const char* fmt, ...) {
    va_list ap;
    va_start(ap, fmt);
    vsnprintf(g_error, sizeof(g_error), fmt, ap);
    va_end(ap);
}

int check_launch(const char* what) {
    const cudaError_t e = cudaGetLastError();
    if (e != cudaSuccess) {
        set_error("%s: kernel launch failed: %s", what, cudaGetErrorString(e));
        return SPLAT_ERR_CUDA;
    }
    return SPLAT_OK;
}

int sm_count() {
    static int cached[64] = {0};
    int dev = 0;
    if (cudaGetDevice(&dev) != cudaSuccess || dev < 0 || dev >= 64) return 148;
    if (cached[dev] == 0) {
        int n = 0;
        if (cudaDeviceGetAttribute(&n, cudaDevAttrMultiProcessorCount, dev) != cudaSuccess || n <= 0) n = 148;
        cached[dev] = n;
    }
    return cached[dev];
}

}  // namespace splat

extern "C" {

const char* splat_last_error(void) { return splat::g_error; }

int splat_abi_version(void) { return SPLAT_ABI_VERSION; }

long long splat_launch_count(void) { return splat::g_launches.load(std::memory_order_relaxed); }

}  // extern "C"
