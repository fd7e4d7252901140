// adam.cu - fused Adam over all parameter groups in one launch.
//
// Per element, the update of Faster-GS's adam_step_cu / adam_step_sparse_cu<false>
// (cluster/patches/fastergs_lean_adam.patch:88-130):
//   m = beta1 (m - g) + g;  v = beta2 (v - g^2) + g^2
//   p -= lr / (1 - beta1^t) * m / (sqrt(v) / sqrt(1 - beta2^t) + eps)
// Groups (means, scales, rotations, opacities, sh0, sh_rest) are described by a table passed by value;
// each 256-thread block owns a contiguous run of one group and streams it with 16-byte accesses when
// the group's buffers allow, so a step reads 4 and writes 3 floats per element and nothing else.
#include "common.cuh"

namespace splat {
namespace adam {

constexpr int kThreads = 256;
constexpr int kVec = 4;
constexpr int kPerBlock = kThreads * kVec * 4;  // 4096 elements per block

struct Group {
    float* param;
    const float* grad;
    float* exp_avg;
    float* exp_avg_sq;
    long long n;
    float step_size;       // lr / (1 - beta1^t)
    float bc2_sqrt_rcp;    // 1 / sqrt(1 - beta2^t)
    long long first_block;  // prefix of blocks over the groups
    int vec;               // all four buffers 16-byte aligned
};

struct Table {
    Group g[SPLAT_ADAM_MAX_GROUPS];
    int count;
    float beta1, beta2, eps;
};

__device__ __forceinline__ float upd(float& p, float g, float& m, float& v, const Group& G, const Table& t) {
    const float g2 = g * g;
    m = fmaf(t.beta1, m - g, g);
    v = fmaf(t.beta2, v - g2, g2);
    const float denom = sqrtf(v) * G.bc2_sqrt_rcp + t.eps;
    p -= G.step_size * m / denom;
    return p;
}

__global__ void __launch_bounds__(kThreads) k_adam(Table t) {
    int gi = 0;
#pragma unroll 1
    while (gi + 1 < t.count && static_cast<long long>(blockIdx.x) >= t.g[gi + 1].first_block) ++gi;
    const Group& G = t.g[gi];
    const long long base = (static_cast<long long>(blockIdx.x) - G.first_block) * kPerBlock;
    if (G.vec) {
#pragma unroll
        for (int k = 0; k < kPerBlock / (kThreads * kVec); ++k) {
            const long long e = base + (static_cast<long long>(k) * kThreads + threadIdx.x) * kVec;
            if (e + kVec <= G.n) {
                float4 p = *reinterpret_cast<const float4*>(G.param + e);
                const float4 g = __ldg(reinterpret_cast<const float4*>(G.grad + e));
                float4 m = *reinterpret_cast<const float4*>(G.exp_avg + e);
                float4 v = *reinterpret_cast<const float4*>(G.exp_avg_sq + e);
                upd(p.x, g.x, m.x, v.x, G, t);
                upd(p.y, g.y, m.y, v.y, G, t);
                upd(p.z, g.z, m.z, v.z, G, t);
                upd(p.w, g.w, m.w, v.w, G, t);
                *reinterpret_cast<float4*>(G.param + e) = p;
                *reinterpret_cast<float4*>(G.exp_avg + e) = m;
                *reinterpret_cast<float4*>(G.exp_avg_sq + e) = v;
            } else {
                for (long long j = e; j < G.n; ++j) upd(G.param[j], G.grad[j], G.exp_avg[j], G.exp_avg_sq[j], G, t);
            }
        }
    } else {
        for (long long e = base + threadIdx.x; e < base + kPerBlock && e < G.n; e += kThreads)
            upd(G.param[e], G.grad[e], G.exp_avg[e], G.exp_avg_sq[e], G, t);
    }
}

}  // namespace adam
}  // namespace splat

using namespace splat;

extern "C" {

int adam_step_multi(int count, const adam_group* groups, int step, float beta1, float beta2, float eps,
                    void* stream) {
    SPLAT_REQUIRE(count >= 0 && count <= SPLAT_ADAM_MAX_GROUPS, "adam_step_multi: %d groups (at most %d)", count,
                  SPLAT_ADAM_MAX_GROUPS);
    SPLAT_REQUIRE(step >= 1, "adam_step_multi: step must be >= 1");
    adam::Table t{};
    t.beta1 = beta1;
    t.beta2 = beta2;
    t.eps = eps;
    long long blocks = 0;
    int k = 0;
    for (int i = 0; i < count; ++i) {
        const adam_group& g = groups[i];
        SPLAT_REQUIRE(g.n >= 0, "adam_step_multi: group %d has negative size", i);
        if (g.n == 0) continue;
        SPLAT_REQUIRE(g.param && g.grad && g.exp_avg && g.exp_avg_sq, "adam_step_multi: group %d has a null buffer", i);
        adam::Group& G = t.g[k++];
        G.param = g.param;
        G.grad = g.grad;
        G.exp_avg = g.exp_avg;
        G.exp_avg_sq = g.exp_avg_sq;
        G.n = g.n;
        const double bc1 = 1.0 - pow(static_cast<double>(beta1), step);
        const double bc2 = 1.0 - pow(static_cast<double>(beta2), step);
        G.step_size = static_cast<float>(static_cast<double>(g.lr) / bc1);
        G.bc2_sqrt_rcp = static_cast<float>(1.0 / sqrt(bc2));
        G.first_block = blocks;
        G.vec = ((reinterpret_cast<uintptr_t>(g.param) | reinterpret_cast<uintptr_t>(g.grad) |
                  reinterpret_cast<uintptr_t>(g.exp_avg) | reinterpret_cast<uintptr_t>(g.exp_avg_sq)) & 15u) == 0;
        blocks += (g.n + adam::kPerBlock - 1) / adam::kPerBlock;
    }
    t.count = k;
    if (blocks == 0) return SPLAT_OK;
    SPLAT_REQUIRE(blocks < (1ll << 31), "adam_step_multi: too many elements");
    adam::k_adam<<<static_cast<unsigned int>(blocks), adam::kThreads, 0, as_stream(stream)>>>(t);
    note_launch();
    return check_launch("adam_step_multi");
}

}  // extern "C"
