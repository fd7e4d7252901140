// common.cu - error reporting, the launch counter and the kernel timers shared by all entry points.
#include <atomic>
#include <cstring>
#include <mutex>

#include "common.cuh"

namespace splat {

namespace {
thread_local char g_error[1024] = "";
std::atomic<long long> g_launches{0};
}  // namespace

void note_launch() { g_launches.fetch_add(1, std::memory_order_relaxed); }

// ---- kernel timers: caller-owned CUDA events recorded around the launches of named kernels ----
namespace {
constexpr int kTimerSlots = 4;
struct Timer {
    const char* name;  // one of kTimedKernels (static storage), nullptr = free slot
    cudaEvent_t begin, end;
};
Timer g_timers[kTimerSlots] = {};
std::atomic<int> g_timers_active{0};
std::mutex g_timer_mutex;
constexpr const char* kTimedKernels[] = {"k_preprocess", "k_duplicate", "k_blend", "k_blend_backward",
                                         "k_preprocess_backward", "k_adam", "gs2d_k_render", "gs2d_k_backward_splat"};
}  // namespace

void timer_mark(const char* kernel, bool begin, cudaStream_t st) {
    if (g_timers_active.load(std::memory_order_relaxed) == 0) return;
    std::lock_guard<std::mutex> lock(g_timer_mutex);
    for (auto& t : g_timers)
        if (t.name != nullptr && strcmp(t.name, kernel) == 0) cudaEventRecord(begin ? t.begin : t.end, st);
}

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

int splat_time_kernel(const char* kernel, void* begin_event, void* end_event) {
    using namespace splat;
    SPLAT_REQUIRE(kernel != nullptr, "splat_time_kernel: kernel name missing");
    const char* name = nullptr;
    for (const char* k : kTimedKernels)
        if (strcmp(k, kernel) == 0) name = k;
    SPLAT_REQUIRE(name != nullptr, "splat_time_kernel: no timer for kernel '%s'", kernel);
    std::lock_guard<std::mutex> lock(g_timer_mutex);
    int slot = -1;
    for (int i = 0; i < kTimerSlots; ++i)
        if (g_timers[i].name == name) slot = i;
    if (begin_event == nullptr || end_event == nullptr) {  // stop timing this kernel
        if (slot >= 0) {
            g_timers[slot] = Timer{};
            g_timers_active.fetch_sub(1, std::memory_order_relaxed);
        }
        return SPLAT_OK;
    }
    if (slot < 0) {
        for (int i = 0; i < kTimerSlots && slot < 0; ++i)
            if (g_timers[i].name == nullptr) slot = i;
        SPLAT_REQUIRE(slot >= 0, "splat_time_kernel: at most %d kernels are timed at once", kTimerSlots);
        g_timers_active.fetch_add(1, std::memory_order_relaxed);
    }
    g_timers[slot] = Timer{name, static_cast<cudaEvent_t>(begin_event), static_cast<cudaEvent_t>(end_event)};
    return SPLAT_OK;
}

}  // extern "C"
