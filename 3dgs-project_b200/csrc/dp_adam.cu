// dp_adam.cu - data-parallel Adam as one kernel over peer memory (the exchange step of multi-view training).
//
// With G ranks (one per GPU, NVLink / NVSwitch between them), rank r owns the slice [lo, hi) of the flat
// parameter vector. Its kernel reads the gradients of that slice from every rank's memory (peer loads), sums
// them in rank order, applies Adam with the moments kept for the slice only, and stores the updated parameters
// of the slice into every rank's parameter vector (peer stores). This replaces an all-reduce of the whole
// gradient followed by G identical Adam steps: the same bytes cross NVLink once in each direction (the slice's
// gradients in, its parameters out) and each rank does 1/G of the optimizer work. The kernel waits on nothing;
// the caller orders it between two device-side barriers (see the header).
#include <algorithm>
#include <cstring>

#include "adam_math.cuh"
#include "common.cuh"

namespace splat {
namespace dp {

constexpr int kThreads = 256;

struct Segment {
    long long begin, end;
    float step_size;
};

struct Args {
    const float* grads[SPLAT_DP_MAX_RANKS];
    float* params[SPLAT_DP_MAX_RANKS];
    float* exp_avg;
    float* exp_avg_sq;
    long long lo, hi;
    Segment seg[SPLAT_DP_MAX_SEGMENTS];
    int nseg;
    int world, rank;
    float beta1, beta2, eps, bc2_sqrt_rcp;
};

__device__ __forceinline__ float step_size_of(const Args& a, long long i) {
    float s = 0.f;
#pragma unroll
    for (int k = 0; k < SPLAT_DP_MAX_SEGMENTS; ++k)
        if (k < a.nseg && i >= a.seg[k].begin && i < a.seg[k].end) s = a.seg[k].step_size;
    return s;
}

__device__ __forceinline__ float adam(float p, float g, float& m, float& v, float step_size, const Args& a) {
    adam_element(p, g, m, v, step_size, a.bc2_sqrt_rcp, a.beta1, a.beta2, a.eps);
    return p;
}

// kWorld: the number of ranks, a template argument so that the per-rank loads live in exactly that many registers.
// Each thread takes kUnroll float4 groups per round (8 / kWorld of them, at least one), so that every peer load of
// the round is in flight before the first sum.
template <int kWorld>
__global__ void __launch_bounds__(kThreads) k_dp_adam(Args a) {
    constexpr int kUnroll = kWorld >= 8 ? 1 : 8 / kWorld;
    const long long n = a.hi - a.lo;
    const long long n4 = n / 4;  // lo is a multiple of 4 and the buffers 16-byte aligned
    const long long stride = static_cast<long long>(gridDim.x) * kThreads;
    for (long long q0 = static_cast<long long>(blockIdx.x) * kThreads + threadIdx.x; q0 < n4; q0 += stride * kUnroll) {
        float4 gv[kUnroll][kWorld], p[kUnroll], m[kUnroll], v[kUnroll];
#pragma unroll
        for (int u = 0; u < kUnroll; ++u) {
            const long long q = q0 + u * stride;
            if (q < n4) {
                const long long e = a.lo + 4 * q;
#pragma unroll
                for (int k = 0; k < kWorld; ++k) gv[u][k] = *reinterpret_cast<const float4*>(a.grads[k] + e);
                p[u] = *reinterpret_cast<const float4*>(a.params[a.rank] + e);  // this rank's own copy
                m[u] = *reinterpret_cast<const float4*>(a.exp_avg + 4 * q);
                v[u] = *reinterpret_cast<const float4*>(a.exp_avg_sq + 4 * q);
            }
        }
#pragma unroll
        for (int u = 0; u < kUnroll; ++u) {
            const long long q = q0 + u * stride;
            if (q < n4) {
                const long long e = a.lo + 4 * q;
                float4 g = gv[u][0];
#pragma unroll
                for (int k = 1; k < kWorld; ++k) {  // in rank order
                    g.x += gv[u][k].x;
                    g.y += gv[u][k].y;
                    g.z += gv[u][k].z;
                    g.w += gv[u][k].w;
                }
                p[u].x = adam(p[u].x, g.x, m[u].x, v[u].x, step_size_of(a, e), a);
                p[u].y = adam(p[u].y, g.y, m[u].y, v[u].y, step_size_of(a, e + 1), a);
                p[u].z = adam(p[u].z, g.z, m[u].z, v[u].z, step_size_of(a, e + 2), a);
                p[u].w = adam(p[u].w, g.w, m[u].w, v[u].w, step_size_of(a, e + 3), a);
                *reinterpret_cast<float4*>(a.exp_avg + 4 * q) = m[u];
                *reinterpret_cast<float4*>(a.exp_avg_sq + 4 * q) = v[u];
#pragma unroll
                for (int k = 0; k < kWorld; ++k) *reinterpret_cast<float4*>(a.params[k] + e) = p[u];
            }
        }
    }
    // the last n % 4 elements, one thread
    if (blockIdx.x == 0 && threadIdx.x == 0) {
        for (long long i = a.lo + 4 * n4; i < a.hi; ++i) {
            float g = 0.f;
            for (int k = 0; k < a.world; ++k) g += a.grads[k][i];
            const long long j = i - a.lo;
            float mm = a.exp_avg[j], vv = a.exp_avg_sq[j];
            const float p = adam(a.params[a.rank][i], g, mm, vv, step_size_of(a, i), a);
            a.exp_avg[j] = mm;
            a.exp_avg_sq[j] = vv;
            for (int k = 0; k < a.world; ++k) a.params[k][i] = p;
        }
    }
    __threadfence_system();  // the peer stores are visible to every GPU before the caller's barrier completes
}

// The same step through NVLink SHARP (multicast memory): each 16-byte group of the slice's gradients is summed
// over the ranks by the switch (multimem.ld_reduce) and the updated parameters are written to every rank with one
// multicast store (multimem.st), so each rank's links carry the slice once in and once out per direction instead
// of G - 1 times. grads_mc / params_mc are multicast addresses of the flat vectors; params_local this rank's copy.
struct NvlsArgs {
    const float* grads_mc;
    float* params_mc;
    const float* params_local;
    float* exp_avg;
    float* exp_avg_sq;
    long long lo, hi;
    Segment seg[SPLAT_DP_MAX_SEGMENTS];
    int nseg;
    float beta1, beta2, eps, bc2_sqrt_rcp;
};

__device__ __forceinline__ float step_size_nvls(const NvlsArgs& a, long long i) {
    float s = 0.f;
#pragma unroll
    for (int k = 0; k < SPLAT_DP_MAX_SEGMENTS; ++k)
        if (k < a.nseg && i >= a.seg[k].begin && i < a.seg[k].end) s = a.seg[k].step_size;
    return s;
}

__device__ __forceinline__ float adam_nvls(float p, float g, float& m, float& v, float step_size, const NvlsArgs& a) {
    adam_element(p, g, m, v, step_size, a.bc2_sqrt_rcp, a.beta1, a.beta2, a.eps);
    return p;
}

// Four float4 groups per thread per round: their four multimem loads are in flight together.
constexpr int kNvlsUnroll = 4;

__global__ void __launch_bounds__(kThreads) k_dp_adam_nvls(NvlsArgs a) {
    const long long n4 = (a.hi - a.lo) / 4;  // lo and hi are multiples of 4
    const long long stride = static_cast<long long>(gridDim.x) * kThreads;
    for (long long q0 = static_cast<long long>(blockIdx.x) * kThreads + threadIdx.x; q0 < n4;
         q0 += stride * kNvlsUnroll) {
        float4 g[kNvlsUnroll], p[kNvlsUnroll], m[kNvlsUnroll], v[kNvlsUnroll];
#pragma unroll
        for (int u = 0; u < kNvlsUnroll; ++u) {
            const long long q = q0 + u * stride;
            if (q < n4) {
                const long long e = a.lo + 4 * q;
                asm volatile("multimem.ld_reduce.relaxed.sys.global.add.v4.f32 {%0, %1, %2, %3}, [%4];"
                             : "=f"(g[u].x), "=f"(g[u].y), "=f"(g[u].z), "=f"(g[u].w)
                             : "l"(a.grads_mc + e)
                             : "memory");
                p[u] = *reinterpret_cast<const float4*>(a.params_local + e);
                m[u] = *reinterpret_cast<const float4*>(a.exp_avg + 4 * q);
                v[u] = *reinterpret_cast<const float4*>(a.exp_avg_sq + 4 * q);
            }
        }
#pragma unroll
        for (int u = 0; u < kNvlsUnroll; ++u) {
            const long long q = q0 + u * stride;
            if (q < n4) {
                const long long e = a.lo + 4 * q;
                p[u].x = adam_nvls(p[u].x, g[u].x, m[u].x, v[u].x, step_size_nvls(a, e), a);
                p[u].y = adam_nvls(p[u].y, g[u].y, m[u].y, v[u].y, step_size_nvls(a, e + 1), a);
                p[u].z = adam_nvls(p[u].z, g[u].z, m[u].z, v[u].z, step_size_nvls(a, e + 2), a);
                p[u].w = adam_nvls(p[u].w, g[u].w, m[u].w, v[u].w, step_size_nvls(a, e + 3), a);
                *reinterpret_cast<float4*>(a.exp_avg + 4 * q) = m[u];
                *reinterpret_cast<float4*>(a.exp_avg_sq + 4 * q) = v[u];
                asm volatile("multimem.st.relaxed.sys.global.v4.f32 [%0], {%1, %2, %3, %4};"
                             :
                             : "l"(a.params_mc + e), "f"(p[u].x), "f"(p[u].y), "f"(p[u].z), "f"(p[u].w)
                             : "memory");
            }
        }
    }
    __threadfence_system();
}

}  // namespace dp
}  // namespace splat

using namespace splat;

namespace {
// Resident 256-thread blocks per SM of the exchange kernels' grids. A sweep at two ranks on the C3-sized vector
// (1, 2, 4, 8 and 16 blocks per SM) measured the same time within 5%.
constexpr long long kDpBlocksPerSm = 8;
long long dp_blocks_per_sm() { return kDpBlocksPerSm; }
}  // namespace

extern "C" {

int splat_peer_alloc(size_t bytes, void** ptr, unsigned char* ipc_handle) {
    SPLAT_REQUIRE(ptr && ipc_handle && bytes > 0, "splat_peer_alloc: bad arguments");
    void* p = nullptr;
    SPLAT_CUDA(cudaMalloc(&p, bytes));
    cudaIpcMemHandle_t h;
    const cudaError_t e = cudaIpcGetMemHandle(&h, p);
    if (e != cudaSuccess) {
        cudaFree(p);
        set_error("cudaIpcGetMemHandle failed: %s", cudaGetErrorString(e));
        return SPLAT_ERR_CUDA;
    }
    SPLAT_CUDA(cudaMemset(p, 0, bytes));
    memcpy(ipc_handle, &h, sizeof(h));
    *ptr = p;
    return SPLAT_OK;
}

int splat_peer_open(const unsigned char* ipc_handle, void** ptr) {
    SPLAT_REQUIRE(ptr && ipc_handle, "splat_peer_open: bad arguments");
    cudaIpcMemHandle_t h;
    memcpy(&h, ipc_handle, sizeof(h));
    SPLAT_CUDA(cudaIpcOpenMemHandle(ptr, h, cudaIpcMemLazyEnablePeerAccess));
    return SPLAT_OK;
}

int splat_peer_close(void* ptr) {
    SPLAT_CUDA(cudaIpcCloseMemHandle(ptr));
    return SPLAT_OK;
}

int splat_peer_free(void* ptr) {
    SPLAT_CUDA(cudaFree(ptr));
    return SPLAT_OK;
}

int adam_step_dp_fused(int world, int rank, const float* const* grads, float* const* params, long long lo,
                       long long hi, float* exp_avg, float* exp_avg_sq, int segment_count,
                       const dp_adam_segment* segments, int step, double beta1, double beta2, double eps,
                       void* stream) {
    SPLAT_REQUIRE(world >= 1 && world <= SPLAT_DP_MAX_RANKS && rank >= 0 && rank < world,
                  "adam_step_dp_fused: rank %d of %d (at most %d ranks)", rank, world, SPLAT_DP_MAX_RANKS);
    SPLAT_REQUIRE(step >= 1, "adam_step_dp_fused: step must be >= 1");
    SPLAT_REQUIRE(segment_count >= 1 && segment_count <= SPLAT_DP_MAX_SEGMENTS,
                  "adam_step_dp_fused: %d segments (1 to %d)", segment_count, SPLAT_DP_MAX_SEGMENTS);
    SPLAT_REQUIRE(0 <= lo && lo <= hi, "adam_step_dp_fused: slice [%lld, %lld)", lo, hi);
    if (hi == lo) return SPLAT_OK;
    SPLAT_REQUIRE(lo % 4 == 0, "adam_step_dp_fused: slice [%lld, %lld) must start at a multiple of 4", lo, hi);
    SPLAT_REQUIRE(exp_avg && exp_avg_sq, "adam_step_dp_fused: null moments");
    dp::Args a{};
    uintptr_t align = reinterpret_cast<uintptr_t>(exp_avg) | reinterpret_cast<uintptr_t>(exp_avg_sq);
    for (int k = 0; k < world; ++k) {
        SPLAT_REQUIRE(grads[k] && params[k], "adam_step_dp_fused: null buffer of rank %d", k);
        a.grads[k] = grads[k];
        a.params[k] = params[k];
        align |= reinterpret_cast<uintptr_t>(grads[k]) | reinterpret_cast<uintptr_t>(params[k]);
    }
    SPLAT_REQUIRE((align & 15u) == 0, "adam_step_dp_fused: buffers must be 16-byte aligned");
    a.exp_avg = exp_avg;
    a.exp_avg_sq = exp_avg_sq;
    a.lo = lo;
    a.hi = hi;
    a.world = world;
    a.rank = rank;
    a.nseg = segment_count;
    // the reference wrapper's host arithmetic (fastergs_lean_adam.patch:162-164), per segment
    const double bc1_rcp = 1.0 / (1.0 - pow(beta1, step));
    for (int k = 0; k < segment_count; ++k) {
        SPLAT_REQUIRE(segments[k].begin <= segments[k].end, "adam_step_dp_fused: segment %d is reversed", k);
        a.seg[k].begin = segments[k].begin;
        a.seg[k].end = segments[k].end;
        a.seg[k].step_size = static_cast<float>(segments[k].lr * bc1_rcp);
    }
    a.beta1 = static_cast<float>(beta1);
    a.beta2 = static_cast<float>(beta2);
    a.eps = static_cast<float>(eps);
    a.bc2_sqrt_rcp = static_cast<float>(1.0 / sqrt(1.0 - pow(beta2, step)));
    const long long n4 = (hi - lo) / 4;
    const long long blocks = std::max<long long>(1, std::min<long long>(div_up(n4, dp::kThreads), dp_blocks_per_sm() * sm_count()));
    cudaStream_t st = as_stream(stream);
    const unsigned nb = static_cast<unsigned>(blocks);
    switch (world) {
        case 1: dp::k_dp_adam<1><<<nb, dp::kThreads, 0, st>>>(a); break;
        case 2: dp::k_dp_adam<2><<<nb, dp::kThreads, 0, st>>>(a); break;
        case 3: dp::k_dp_adam<3><<<nb, dp::kThreads, 0, st>>>(a); break;
        case 4: dp::k_dp_adam<4><<<nb, dp::kThreads, 0, st>>>(a); break;
        case 5: dp::k_dp_adam<5><<<nb, dp::kThreads, 0, st>>>(a); break;
        case 6: dp::k_dp_adam<6><<<nb, dp::kThreads, 0, st>>>(a); break;
        case 7: dp::k_dp_adam<7><<<nb, dp::kThreads, 0, st>>>(a); break;
        default: dp::k_dp_adam<8><<<nb, dp::kThreads, 0, st>>>(a); break;
    }
    note_launch();
    return check_launch("adam_step_dp_fused");
}

int adam_step_dp_nvls(long long lo, long long hi, const float* grads_mc, float* params_mc, const float* params_local,
                      float* exp_avg, float* exp_avg_sq, int segment_count, const dp_adam_segment* segments, int step,
                      double beta1, double beta2, double eps, void* stream) {
    SPLAT_REQUIRE(step >= 1, "adam_step_dp_nvls: step must be >= 1");
    SPLAT_REQUIRE(segment_count >= 1 && segment_count <= SPLAT_DP_MAX_SEGMENTS,
                  "adam_step_dp_nvls: %d segments (1 to %d)", segment_count, SPLAT_DP_MAX_SEGMENTS);
    SPLAT_REQUIRE(0 <= lo && lo <= hi && lo % 4 == 0 && hi % 4 == 0,
                  "adam_step_dp_nvls: slice [%lld, %lld) must start and end at multiples of 4", lo, hi);
    if (hi == lo) return SPLAT_OK;
    SPLAT_REQUIRE(grads_mc && params_mc && params_local && exp_avg && exp_avg_sq, "adam_step_dp_nvls: null buffer");
    SPLAT_REQUIRE(((reinterpret_cast<uintptr_t>(grads_mc) | reinterpret_cast<uintptr_t>(params_mc) |
                    reinterpret_cast<uintptr_t>(params_local) | reinterpret_cast<uintptr_t>(exp_avg) |
                    reinterpret_cast<uintptr_t>(exp_avg_sq)) & 15u) == 0,
                  "adam_step_dp_nvls: buffers must be 16-byte aligned");
    dp::NvlsArgs a{};
    a.grads_mc = grads_mc;
    a.params_mc = params_mc;
    a.params_local = params_local;
    a.exp_avg = exp_avg;
    a.exp_avg_sq = exp_avg_sq;
    a.lo = lo;
    a.hi = hi;
    a.nseg = segment_count;
    const double bc1_rcp = 1.0 / (1.0 - pow(beta1, step));
    for (int k = 0; k < segment_count; ++k) {
        SPLAT_REQUIRE(segments[k].begin <= segments[k].end, "adam_step_dp_nvls: segment %d is reversed", k);
        a.seg[k].begin = segments[k].begin;
        a.seg[k].end = segments[k].end;
        a.seg[k].step_size = static_cast<float>(segments[k].lr * bc1_rcp);
    }
    a.beta1 = static_cast<float>(beta1);
    a.beta2 = static_cast<float>(beta2);
    a.eps = static_cast<float>(eps);
    a.bc2_sqrt_rcp = static_cast<float>(1.0 / sqrt(1.0 - pow(beta2, step)));
    const long long n4 = (hi - lo) / 4;
    const long long blocks = std::max<long long>(1, std::min<long long>(div_up(n4, dp::kThreads), dp_blocks_per_sm() * sm_count()));
    dp::k_dp_adam_nvls<<<static_cast<unsigned>(blocks), dp::kThreads, 0, as_stream(stream)>>>(a);
    note_launch();
    return check_launch("adam_step_dp_nvls");
}

}  // extern "C"
