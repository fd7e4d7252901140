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
#include "gs3d_common.cuh"

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

// ---- the compact form: SH gradients sent as (colour gradient, view direction) records ----
//
// A view's SH gradients are products: for SH coefficient k of colour channel c, basis_k(d) * g_c, with d the unit
// view direction of the Gaussian and g the colour gradient masked by the colour clamp. So each rank sends, per view
// and Gaussian, the six floats (g, d) (gs3d_backward_preprocess_records) instead of 3 * (rest_bases + 1) gradients,
// and the owner forms every rank's products itself, with the same rounding as the preprocess backward
// (sh_basis_rn, __fmul_rn), sums them over the rank's views in view order and then over the ranks in rank order.
// The other four groups (means, scales, rotations, opacities) are summed over the ranks as in k_dp_adam.
//
// Rank r owns the Gaussians [lo, hi) and updates all of their parameters. Layouts (elements; n Gaussians, R
// rest bases, V views):
//   parameters (every rank): means 3n | scales 3n | rotations 4n | opacities n | sh0 3n | sh_rest 3Rn
//   gradients (every rank):  means 3n | scales 3n | rotations 4n | opacities n | records 6n per view
//   moments (owner):         the parameter layout over the owned Gaussians, with c = hi - lo rounded up to 4
constexpr int kCompactThreads = 256;
constexpr int kChunk = 80;       // Gaussians per block iteration (3 x 80 sum threads of the 256)
constexpr int kRecBatch = 8;     // (rank, view) record blocks staged in shared memory at a time
constexpr int kMaxBases = 16;

struct CompactArgs {
    const float* grads[SPLAT_DP_MAX_RANKS];
    float* params[SPLAT_DP_MAX_RANKS];
    float* exp_avg;
    float* exp_avg_sq;
    long long n, lo, hi, cpad;
    int world, rank, views, active_bases, rest_bases;
    int small_blocks;  // blocks [0, small_blocks) take the non-SH groups, the others the SH chunks
    float step_size[6];
    float beta1, beta2, eps, bc2_sqrt_rcp;
};

__device__ __forceinline__ long long group_base(int gi, long long n) {
    return gi == 0 ? 0 : gi == 1 ? 3 * n : gi == 2 ? 6 * n : gi == 3 ? 10 * n : gi == 4 ? 11 * n : 14 * n;
}

__device__ __forceinline__ float4 add4(float4 a, float4 b) {
    return make_float4(__fadd_rn(a.x, b.x), __fadd_rn(a.y, b.y), __fadd_rn(a.z, b.z), __fadd_rn(a.w, b.w));
}

// Adam over the elements of group gi of the Gaussians [i0, i0 + cnt): the gradient is the rank-ordered sum of the
// ranks' gradients (g_smem null) or SH sums in shared memory; the parameter is written to every rank. The calling
// threads take the elements first, first + step, ... (16-byte groups of four where kVec: every group start is a
// multiple of 4 elements and the buffers 16-byte aligned). kWorld: the number of ranks, so that the per-rank loads
// live in exactly that many registers.
template <bool kVec, int kWorld>
__device__ __forceinline__ void adam_span(const CompactArgs& a, int gi, int w, long long i0, long long cnt,
                                          const float* g_smem, long long first, long long step) {
    const long long e0 = group_base(gi, a.n) + w * i0;
    const long long m0 = group_base(gi, a.cpad) + w * (i0 - a.lo);
    const long long ne = w * cnt;
    const float ss = a.step_size[gi];
    long long done = 0;
    if (kVec) {
        const long long n4 = ne / 4;
        for (long long q = first; q < n4; q += step) {
            float4 g;
            if (g_smem) {
                g = *reinterpret_cast<const float4*>(g_smem + 4 * q);
            } else {
                float4 gv[kWorld];
#pragma unroll
                for (int r = 0; r < kWorld; ++r)  // every rank's load in flight before the sum
                    gv[r] = *reinterpret_cast<const float4*>(a.grads[r] + e0 + 4 * q);
                g = gv[0];
#pragma unroll
                for (int r = 1; r < kWorld; ++r) g = add4(g, gv[r]);
            }
            float4 p = *reinterpret_cast<const float4*>(a.params[a.rank] + e0 + 4 * q);
            float4 m = *reinterpret_cast<const float4*>(a.exp_avg + m0 + 4 * q);
            float4 v = *reinterpret_cast<const float4*>(a.exp_avg_sq + m0 + 4 * q);
            adam_element(p.x, g.x, m.x, v.x, ss, a.bc2_sqrt_rcp, a.beta1, a.beta2, a.eps);
            adam_element(p.y, g.y, m.y, v.y, ss, a.bc2_sqrt_rcp, a.beta1, a.beta2, a.eps);
            adam_element(p.z, g.z, m.z, v.z, ss, a.bc2_sqrt_rcp, a.beta1, a.beta2, a.eps);
            adam_element(p.w, g.w, m.w, v.w, ss, a.bc2_sqrt_rcp, a.beta1, a.beta2, a.eps);
            *reinterpret_cast<float4*>(a.exp_avg + m0 + 4 * q) = m;
            *reinterpret_cast<float4*>(a.exp_avg_sq + m0 + 4 * q) = v;
#pragma unroll
            for (int r = 0; r < kWorld; ++r) *reinterpret_cast<float4*>(a.params[r] + e0 + 4 * q) = p;
        }
        done = 4 * n4;
    }
    for (long long k = done + first; k < ne; k += step) {
        float g;
        if (g_smem) {
            g = g_smem[k];
        } else {
            g = a.grads[0][e0 + k];
#pragma unroll
            for (int r = 1; r < kWorld; ++r) g = __fadd_rn(g, a.grads[r][e0 + k]);
        }
        float p = a.params[a.rank][e0 + k], m = a.exp_avg[m0 + k], v = a.exp_avg_sq[m0 + k];
        adam_element(p, g, m, v, ss, a.bc2_sqrt_rcp, a.beta1, a.beta2, a.eps);
        a.exp_avg[m0 + k] = m;
        a.exp_avg_sq[m0 + k] = v;
#pragma unroll
        for (int r = 0; r < kWorld; ++r) a.params[r][e0 + k] = p;
    }
}

// Two kinds of blocks run side by side: the first a.small_blocks stream the four non-SH groups of the owned
// Gaussians (grid-stride, every rank's load in flight), the others take chunks of kChunk Gaussians for the SH
// groups (records staged in shared memory, sums, then Adam through shared memory). The grid is resident at once.
template <bool kVec, int kWorld>
__global__ void __launch_bounds__(kCompactThreads, 2) k_dp_adam_compact(CompactArgs a) {
    __shared__ __align__(16) float s_rec[kRecBatch * kChunk * 6];
    __shared__ __align__(16) float s_g[kChunk * 3 * kMaxBases];  // sh0 sums [Gaussian][channel], then sh_rest
    const int tid = threadIdx.x;
    if (static_cast<int>(blockIdx.x) < a.small_blocks) {
        const long long first = static_cast<long long>(blockIdx.x) * kCompactThreads + tid;
        const long long step = static_cast<long long>(a.small_blocks) * kCompactThreads;
        adam_span<kVec, kWorld>(a, 0, 3, a.lo, a.hi - a.lo, nullptr, first, step);
        adam_span<kVec, kWorld>(a, 1, 3, a.lo, a.hi - a.lo, nullptr, first, step);
        adam_span<kVec, kWorld>(a, 2, 4, a.lo, a.hi - a.lo, nullptr, first, step);
        adam_span<kVec, kWorld>(a, 3, 1, a.lo, a.hi - a.lo, nullptr, first, step);
        __threadfence_system();
        return;
    }
    const int R = a.rest_bases;
    const int nb = min(a.active_bases, R + 1);  // bases with a gradient; the others get zeros
    const int rv = a.world * a.views;
    const long long owned = a.hi - a.lo;
    const long long chunks = (owned + kChunk - 1) / kChunk;
    for (long long ch = blockIdx.x - a.small_blocks; ch < chunks; ch += gridDim.x - a.small_blocks) {
        const long long i0 = a.lo + ch * kChunk;
        const int cnt = static_cast<int>(min(static_cast<long long>(kChunk), a.hi - i0));
        // thread (il, c) forms the sums of Gaussian i0 + il, colour channel c
        const int il = tid / 3, c = tid - 3 * il;
        const bool mine = tid < 3 * cnt;
        float tot[kMaxBases], acc[kMaxBases];
#pragma unroll
        for (int k = 0; k < kMaxBases; ++k) tot[k] = acc[k] = 0.f;
        for (int q0 = 0; q0 < rv; q0 += kRecBatch) {
            const int nq = min(kRecBatch, rv - q0);
            __syncthreads();  // s_rec of the previous batch (or chunk) is consumed
            const int span = 6 * cnt;  // floats of one (rank, view) block of the chunk
            if (kVec && (span & 3) == 0) {
                const int s4 = span / 4;
                for (int t = tid; t < nq * s4; t += kCompactThreads) {
                    const int qq = t / s4, k4 = t - qq * s4;
                    const int q = q0 + qq, r = q / a.views, v = q - r * a.views;
                    const float* src = a.grads[r] + 11 * a.n + (6 * a.n) * v + 6 * i0;
                    reinterpret_cast<float4*>(s_rec + qq * kChunk * 6)[k4] = reinterpret_cast<const float4*>(src)[k4];
                }
            } else {
                for (int t = tid; t < nq * span; t += kCompactThreads) {
                    const int qq = t / span, k = t - qq * span;
                    const int q = q0 + qq, r = q / a.views, v = q - r * a.views;
                    s_rec[qq * kChunk * 6 + k] = a.grads[r][11 * a.n + (6 * a.n) * v + 6 * i0 + k];
                }
            }
            __syncthreads();
            if (mine) {
                for (int qq = 0; qq < nq; ++qq) {
                    const int q = q0 + qq, r = q / a.views, v = q - r * a.views;
                    const float* rec = s_rec + (qq * kChunk + il) * 6;
                    const float g = rec[c];
                    float bas[kMaxBases];
                    gs3d::sh_basis_rn(rec[3], rec[4], rec[5], a.active_bases, bas);
#pragma unroll
                    for (int k = 0; k < kMaxBases; ++k) {
                        if (k > R) continue;
                        const float t = k == 0 ? __fmul_rn(gs3d::kSH0, g) : (k < nb ? __fmul_rn(bas[k], g) : 0.f);
                        acc[k] = v == 0 ? t : __fadd_rn(acc[k], t);  // the rank's views in view order
                        if (v == a.views - 1) tot[k] = r == 0 ? acc[k] : __fadd_rn(tot[k], acc[k]);  // rank order
                    }
                }
            }
        }
        if (mine) {
            s_g[3 * il + c] = tot[0];
#pragma unroll
            for (int k = 1; k < kMaxBases; ++k)
                if (k <= R) s_g[3 * kChunk + 3 * R * il + 3 * (k - 1) + c] = tot[k];
        }
        __syncthreads();
        adam_span<kVec, kWorld>(a, 4, 3, i0, cnt, s_g, tid, kCompactThreads);
        if (R > 0) adam_span<kVec, kWorld>(a, 5, 3 * R, i0, cnt, s_g + 3 * kChunk, tid, kCompactThreads);
        __syncthreads();  // s_g is rewritten by the next chunk
    }
    __threadfence_system();  // the peer stores are visible to every GPU before the caller's barrier completes
}

}  // namespace dp
}  // namespace splat

using namespace splat;

namespace {
// Resident 256-thread blocks per SM of the exchange kernels' grids. A sweep at two ranks on the C3-sized vector
// (1, 2, 4, 8 and 16 blocks per SM) measured the same time within 5%.
constexpr long long kDpBlocksPerSm = 8;
long long dp_blocks_per_sm() { return kDpBlocksPerSm; }

template <int kWorld>
void launch_compact_for(bool vec, unsigned blocks, cudaStream_t st, const dp::CompactArgs& a) {
    if (vec)
        dp::k_dp_adam_compact<true, kWorld><<<blocks, dp::kCompactThreads, 0, st>>>(a);
    else
        dp::k_dp_adam_compact<false, kWorld><<<blocks, dp::kCompactThreads, 0, st>>>(a);
}

int launch_compact(bool vec, int world, unsigned blocks, cudaStream_t st, const dp::CompactArgs& a) {
    switch (world) {
        case 1: launch_compact_for<1>(vec, blocks, st, a); break;
        case 2: launch_compact_for<2>(vec, blocks, st, a); break;
        case 3: launch_compact_for<3>(vec, blocks, st, a); break;
        case 4: launch_compact_for<4>(vec, blocks, st, a); break;
        case 5: launch_compact_for<5>(vec, blocks, st, a); break;
        case 6: launch_compact_for<6>(vec, blocks, st, a); break;
        case 7: launch_compact_for<7>(vec, blocks, st, a); break;
        case 8: launch_compact_for<8>(vec, blocks, st, a); break;
        default: return SPLAT_ERR_ARG;
    }
    return SPLAT_OK;
}
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

int adam_step_dp_compact(int world, int rank, const float* const* grads, float* const* params, long long n,
                         long long lo, long long hi, int views, int active_sh_bases, int rest_bases, float* exp_avg,
                         float* exp_avg_sq, const double* lr, int step, double beta1, double beta2, double eps,
                         void* stream) {
    SPLAT_REQUIRE(world >= 1 && world <= SPLAT_DP_MAX_RANKS && rank >= 0 && rank < world,
                  "adam_step_dp_compact: rank %d of %d (at most %d ranks)", rank, world, SPLAT_DP_MAX_RANKS);
    SPLAT_REQUIRE(step >= 1, "adam_step_dp_compact: step must be >= 1");
    SPLAT_REQUIRE(views >= 1, "adam_step_dp_compact: views must be >= 1 (got %d)", views);
    SPLAT_REQUIRE(rest_bases >= 0 && rest_bases <= 15 && active_sh_bases >= 1 && active_sh_bases <= 16,
                  "adam_step_dp_compact: rest_bases %d / active_sh_bases %d out of range", rest_bases,
                  active_sh_bases);
    SPLAT_REQUIRE(n >= 0 && 0 <= lo && lo <= hi && hi <= n, "adam_step_dp_compact: Gaussians [%lld, %lld) of %lld",
                  lo, hi, n);
    if (hi == lo) return SPLAT_OK;
    SPLAT_REQUIRE(lo % 4 == 0, "adam_step_dp_compact: the owned Gaussians must start at a multiple of 4 (%lld)", lo);
    SPLAT_REQUIRE(exp_avg && exp_avg_sq && lr, "adam_step_dp_compact: null moments or learning rates");
    dp::CompactArgs a{};
    uintptr_t align = reinterpret_cast<uintptr_t>(exp_avg) | reinterpret_cast<uintptr_t>(exp_avg_sq);
    for (int k = 0; k < world; ++k) {
        SPLAT_REQUIRE(grads[k] && params[k], "adam_step_dp_compact: null buffer of rank %d", k);
        a.grads[k] = grads[k];
        a.params[k] = params[k];
        align |= reinterpret_cast<uintptr_t>(grads[k]) | reinterpret_cast<uintptr_t>(params[k]);
    }
    a.exp_avg = exp_avg;
    a.exp_avg_sq = exp_avg_sq;
    a.n = n;
    a.lo = lo;
    a.hi = hi;
    a.cpad = (hi - lo + 3) / 4 * 4;
    a.world = world;
    a.rank = rank;
    a.views = views;
    a.active_bases = active_sh_bases;
    a.rest_bases = rest_bases;
    for (int gi = 0; gi < 6; ++gi) {
        float bc2 = 0.f;
        adam_bias_corrections(lr[gi], beta1, beta2, step, a.step_size[gi], bc2);
        a.bc2_sqrt_rcp = bc2;
    }
    a.beta1 = static_cast<float>(beta1);
    a.beta2 = static_cast<float>(beta2);
    a.eps = static_cast<float>(eps);
    const bool vec = (align & 15u) == 0 && n % 4 == 0;
    // a resident grid (two blocks per SM), about 3 / 10 of it on the non-SH groups: their share of the bytes that
    // cross NVLink per Gaussian (11 of 11 + 48 + 6 views floats each way at one view)
    const long long chunks = div_up(hi - lo, static_cast<long long>(dp::kChunk));
    const long long resident = 2ll * sm_count();
    a.small_blocks = static_cast<int>(std::max<long long>(1, resident * 3 / 10));
    const unsigned blocks = static_cast<unsigned>(a.small_blocks + std::max<long long>(1, std::min<long long>(chunks, resident - a.small_blocks)));
    cudaStream_t st = as_stream(stream);
    SPLAT_TRY(launch_compact(vec, world, blocks, st, a));
    note_launch();
    return check_launch("adam_step_dp_compact");
}

}  // extern "C"
