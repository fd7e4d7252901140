// adam.cu - fused Adam over all parameter groups in one launch.
//
// Per element, the update of Faster-GS's adam_step_cu / adam_step_sparse_cu<false>
// (cluster/patches/fastergs_lean_adam.patch:88-130):
//   m = beta1 (m - g) + g;  v = beta2 (v - g^2) + g^2
//   p -= lr / (1 - beta1^t) * m / (sqrt(v) / sqrt(1 - beta2^t) + eps)
// Groups (means, scales, rotations, opacities, sh0, sh_rest) are described by a table passed by value;
// each 256-thread block owns a contiguous run of one group and streams it with 16-byte accesses when
// the group's buffers allow, so a step reads 4 and writes 3 floats per element and nothing else.
// k_adam_lean adds the two options of the reference's lean Adam (adam_step_sparse_cu<LOWP>, same patch):
// a per-primitive visibility mask and bfloat16 moments written with stochastic rounding.
#include "adam_math.cuh"
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
    adam_element(p, g, m, v, G.step_size, G.bc2_sqrt_rcp, t.beta1, t.beta2, t.eps);
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

// ---- lean Adam: visibility mask and bfloat16 moments with stochastic rounding ----

struct LeanGroup {
    float* param;
    const float* grad;
    void* exp_avg;
    void* exp_avg_sq;
    long long n;
    float step_size;
    float bc2_sqrt_rcp;
    long long first_block;
    int features;
    int lowp;
    int vec;  // 16-byte (fp32 moments) / 8-byte (bf16 moments) accesses possible
};

struct LeanTable {
    LeanGroup g[SPLAT_ADAM_MAX_GROUPS];
    int count;
    float beta1, beta2, eps;
    uint32_t seed;
    const int32_t* visibility;  // may be null
};

// lowbias32 (C. Wellons, "hash prospector", 2018): a 32-bit integer hash with two multiply-xorshift rounds.
__device__ __forceinline__ uint32_t lowbias32(uint32_t x) {
    x ^= x >> 16;
    x *= 0x7feb352du;
    x ^= x >> 15;
    x *= 0x846ca68bu;
    x ^= x >> 16;
    return x;
}

__device__ __forceinline__ float bf16_to_float(uint16_t b) { return __uint_as_float(static_cast<uint32_t>(b) << 16); }

// Stochastic rounding to bfloat16: uniform noise in the 16 bits that are dropped, then truncation.
__device__ __forceinline__ uint16_t float_to_bf16_sr(float f, uint32_t rnd) {
    return static_cast<uint16_t>((__float_as_uint(f) + (rnd & 0xFFFFu)) >> 16);
}

// The primitive that element i of the group belongs to: a 32-bit division where the group's element count allows
// (every group of a scene below 2^32 elements), a 64-bit one otherwise.
__device__ __forceinline__ long long primitive_of(const LeanGroup& G, long long i) {
    if (G.n <= 0xFFFFFFFFll) return static_cast<uint32_t>(i) / static_cast<uint32_t>(G.features);
    return i / G.features;
}

template <bool kLowp>
__device__ __forceinline__ void lean_one(const LeanGroup& G, const LeanTable& t, long long i) {
    if (t.visibility && t.visibility[primitive_of(G, i)] == 0) return;
    const float g = G.grad[i];
    float m, v;
    if (kLowp) {
        m = bf16_to_float(static_cast<const uint16_t*>(G.exp_avg)[i]);
        v = bf16_to_float(static_cast<const uint16_t*>(G.exp_avg_sq)[i]);
    } else {
        m = static_cast<const float*>(G.exp_avg)[i];
        v = static_cast<const float*>(G.exp_avg_sq)[i];
    }
    adam_element(G.param[i], g, m, v, G.step_size, G.bc2_sqrt_rcp, t.beta1, t.beta2, t.eps);
    if (kLowp) {
        const uint32_t r1 = lowbias32(static_cast<uint32_t>(i) ^ t.seed);
        const uint32_t r2 = lowbias32(r1);
        static_cast<uint16_t*>(G.exp_avg)[i] = float_to_bf16_sr(m, r1);
        static_cast<uint16_t*>(G.exp_avg_sq)[i] = float_to_bf16_sr(v, r2);
    } else {
        static_cast<float*>(G.exp_avg)[i] = m;
        static_cast<float*>(G.exp_avg_sq)[i] = v;
    }
}

// Which of the four consecutive elements from e belong to visible primitives (bit k for element e + k): one
// division per four elements, walking from the first element's primitive across the (at most four) primitives
// they belong to and loading each one's visibility once.
__device__ __forceinline__ unsigned lean_mask(const LeanGroup& G, const LeanTable& t, long long e) {
    if (!t.visibility) return (1u << kVec) - 1u;
    long long prim = primitive_of(G, e);
    int r = static_cast<int>(e - prim * G.features);
    bool vis = t.visibility[prim] != 0;
    unsigned mask = 0u;
#pragma unroll
    for (int k = 0; k < kVec; ++k) {
        mask |= static_cast<unsigned>(vis) << k;
        if (++r == G.features && k + 1 < kVec) {
            r = 0;
            ++prim;
            vis = t.visibility[prim] != 0;
        }
    }
    return mask;
}

// Four consecutive elements with vector accesses, `mask` from lean_mask (non-zero): elements of primitives that
// are not visible keep their parameter and moments.
template <bool kLowp>
__device__ __forceinline__ void lean_four(const LeanGroup& G, const LeanTable& t, long long e, unsigned mask) {
    bool on[kVec];
#pragma unroll
    for (int k = 0; k < kVec; ++k) on[k] = (mask >> k) & 1u;
    float4 p = *reinterpret_cast<const float4*>(G.param + e);
    const float4 g4 = __ldg(reinterpret_cast<const float4*>(G.grad + e));
    float pv[kVec] = {p.x, p.y, p.z, p.w}, gv[kVec] = {g4.x, g4.y, g4.z, g4.w}, mv[kVec], vv[kVec];
    uint2 mb{}, vb{};
    if (kLowp) {
        mb = *reinterpret_cast<const uint2*>(static_cast<const uint16_t*>(G.exp_avg) + e);
        vb = *reinterpret_cast<const uint2*>(static_cast<const uint16_t*>(G.exp_avg_sq) + e);
        const uint32_t mw[2] = {mb.x, mb.y}, vw[2] = {vb.x, vb.y};
#pragma unroll
        for (int k = 0; k < kVec; ++k) {
            mv[k] = bf16_to_float(static_cast<uint16_t>(mw[k >> 1] >> (16 * (k & 1))));
            vv[k] = bf16_to_float(static_cast<uint16_t>(vw[k >> 1] >> (16 * (k & 1))));
        }
    } else {
        const float4 m4 = *reinterpret_cast<const float4*>(static_cast<const float*>(G.exp_avg) + e);
        const float4 v4 = *reinterpret_cast<const float4*>(static_cast<const float*>(G.exp_avg_sq) + e);
        mv[0] = m4.x, mv[1] = m4.y, mv[2] = m4.z, mv[3] = m4.w;
        vv[0] = v4.x, vv[1] = v4.y, vv[2] = v4.z, vv[3] = v4.w;
    }
    uint32_t mo[2] = {mb.x, mb.y}, vo[2] = {vb.x, vb.y};
#pragma unroll
    for (int k = 0; k < kVec; ++k) {
        if (!on[k]) continue;
        adam_element(pv[k], gv[k], mv[k], vv[k], G.step_size, G.bc2_sqrt_rcp, t.beta1, t.beta2, t.eps);
        const float m = mv[k], v = vv[k];
        if (kLowp) {
            const uint32_t r1 = lowbias32(static_cast<uint32_t>(e + k) ^ t.seed);
            const uint32_t r2 = lowbias32(r1);
            const int sh = 16 * (k & 1);
            mo[k >> 1] = (mo[k >> 1] & ~(0xFFFFu << sh)) | (static_cast<uint32_t>(float_to_bf16_sr(m, r1)) << sh);
            vo[k >> 1] = (vo[k >> 1] & ~(0xFFFFu << sh)) | (static_cast<uint32_t>(float_to_bf16_sr(v, r2)) << sh);
        }
    }
    *reinterpret_cast<float4*>(G.param + e) = make_float4(pv[0], pv[1], pv[2], pv[3]);
    if (kLowp) {
        *reinterpret_cast<uint2*>(static_cast<uint16_t*>(G.exp_avg) + e) = make_uint2(mo[0], mo[1]);
        *reinterpret_cast<uint2*>(static_cast<uint16_t*>(G.exp_avg_sq) + e) = make_uint2(vo[0], vo[1]);
    } else {
        *reinterpret_cast<float4*>(static_cast<float*>(G.exp_avg) + e) = make_float4(mv[0], mv[1], mv[2], mv[3]);
        *reinterpret_cast<float4*>(static_cast<float*>(G.exp_avg_sq) + e) = make_float4(vv[0], vv[1], vv[2], vv[3]);
    }
}

template <bool kLowp>
__device__ __forceinline__ void lean_block(const LeanGroup& G, const LeanTable& t, long long base) {
    if (G.vec) {
        // the visibility of all of this thread's groups of four first, so that their loads overlap one another
        // instead of each one delaying its group's data loads
        constexpr int kIters = kPerBlock / (kThreads * kVec);
        unsigned mask[kIters];
#pragma unroll
        for (int k = 0; k < kIters; ++k) {
            const long long e = base + (static_cast<long long>(k) * kThreads + threadIdx.x) * kVec;
            mask[k] = e + kVec <= G.n ? lean_mask(G, t, e) : 0u;
        }
#pragma unroll
        for (int k = 0; k < kIters; ++k) {
            const long long e = base + (static_cast<long long>(k) * kThreads + threadIdx.x) * kVec;
            if (e + kVec <= G.n) {
                if (mask[k]) lean_four<kLowp>(G, t, e, mask[k]);
            } else {
                for (long long j = e; j < G.n; ++j) lean_one<kLowp>(G, t, j);
            }
        }
    } else {
        for (long long e = base + threadIdx.x; e < base + kPerBlock && e < G.n; e += kThreads)
            lean_one<kLowp>(G, t, e);
    }
}

__global__ void __launch_bounds__(kThreads) k_adam_lean(LeanTable t) {
    int gi = 0;
#pragma unroll 1
    while (gi + 1 < t.count && static_cast<long long>(blockIdx.x) >= t.g[gi + 1].first_block) ++gi;
    const LeanGroup& G = t.g[gi];
    const long long base = (static_cast<long long>(blockIdx.x) - G.first_block) * kPerBlock;
    if (G.lowp)
        lean_block<true>(G, t, base);
    else
        lean_block<false>(G, t, base);
}

}  // namespace adam
}  // namespace splat

using namespace splat;

namespace {

// The reference wrapper's host arithmetic (fastergs_lean_adam.patch:162-164): in double, rounded once to float.
void bias_corrections(double lr, double beta1, double beta2, int step, float& step_size, float& bc2_sqrt_rcp) {
    adam_bias_corrections(lr, beta1, beta2, step, step_size, bc2_sqrt_rcp);
}

}  // namespace

extern "C" {

int adam_step_multi(int count, const adam_group* groups, int step, double beta1, double beta2, double eps,
                    void* stream) {
    SPLAT_REQUIRE(count >= 0 && count <= SPLAT_ADAM_MAX_GROUPS, "adam_step_multi: %d groups (at most %d)", count,
                  SPLAT_ADAM_MAX_GROUPS);
    SPLAT_REQUIRE(step >= 1, "adam_step_multi: step must be >= 1");
    adam::Table t{};
    t.beta1 = static_cast<float>(beta1);
    t.beta2 = static_cast<float>(beta2);
    t.eps = static_cast<float>(eps);
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
        bias_corrections(g.lr, beta1, beta2, step, G.step_size, G.bc2_sqrt_rcp);
        G.first_block = blocks;
        G.vec = ((reinterpret_cast<uintptr_t>(g.param) | reinterpret_cast<uintptr_t>(g.grad) |
                  reinterpret_cast<uintptr_t>(g.exp_avg) | reinterpret_cast<uintptr_t>(g.exp_avg_sq)) & 15u) == 0;
        blocks += (g.n + adam::kPerBlock - 1) / adam::kPerBlock;
    }
    t.count = k;
    if (blocks == 0) return SPLAT_OK;
    SPLAT_REQUIRE(blocks < (1ll << 31), "adam_step_multi: too many elements");
    SPLAT_TIMED_LAUNCH("k_adam", as_stream(stream),
                       (adam::k_adam<<<static_cast<unsigned int>(blocks), adam::kThreads, 0, as_stream(stream)>>>(t)));
    note_launch();
    return check_launch("adam_step_multi");
}

int adam_step_multi_lean(int count, const adam_lean_group* groups, int step, double beta1, double beta2,
                         double eps, const int32_t* visibility, long long n_primitives, void* stream) {
    SPLAT_REQUIRE(count >= 0 && count <= SPLAT_ADAM_MAX_GROUPS, "adam_step_multi_lean: %d groups (at most %d)",
                  count, SPLAT_ADAM_MAX_GROUPS);
    SPLAT_REQUIRE(step >= 1, "adam_step_multi_lean: step must be >= 1");
    adam::LeanTable t{};
    t.beta1 = static_cast<float>(beta1);
    t.beta2 = static_cast<float>(beta2);
    t.eps = static_cast<float>(eps);
    t.seed = 0x9E3779B9u * static_cast<uint32_t>(step) + 0x85EBCA6Bu;
    t.visibility = visibility;
    long long blocks = 0;
    int k = 0;
    for (int i = 0; i < count; ++i) {
        const adam_lean_group& g = groups[i];
        SPLAT_REQUIRE(g.n >= 0 && g.features >= 1, "adam_step_multi_lean: group %d has a bad size", i);
        if (g.n == 0) continue;
        SPLAT_REQUIRE(g.param && g.grad && g.exp_avg && g.exp_avg_sq, "adam_step_multi_lean: group %d has a null buffer",
                      i);
        SPLAT_REQUIRE(!visibility || g.n == static_cast<long long>(g.features) * n_primitives,
                      "adam_step_multi_lean: group %d has %lld elements, not %d x %lld primitives", i, g.n, g.features,
                      n_primitives);
        adam::LeanGroup& G = t.g[k++];
        G.param = g.param;
        G.grad = g.grad;
        G.exp_avg = g.exp_avg;
        G.exp_avg_sq = g.exp_avg_sq;
        G.n = g.n;
        bias_corrections(g.lr, beta1, beta2, step, G.step_size, G.bc2_sqrt_rcp);
        G.first_block = blocks;
        G.features = g.features;
        G.lowp = g.lowp_moments != 0;
        const uintptr_t moment_align = G.lowp ? 7u : 15u;
        G.vec = ((reinterpret_cast<uintptr_t>(g.param) | reinterpret_cast<uintptr_t>(g.grad)) & 15u) == 0 &&
                ((reinterpret_cast<uintptr_t>(g.exp_avg) | reinterpret_cast<uintptr_t>(g.exp_avg_sq)) & moment_align) == 0;
        blocks += (g.n + adam::kPerBlock - 1) / adam::kPerBlock;
    }
    t.count = k;
    if (blocks == 0) return SPLAT_OK;
    SPLAT_REQUIRE(blocks < (1ll << 31), "adam_step_multi_lean: too many elements");
    adam::k_adam_lean<<<static_cast<unsigned int>(blocks), adam::kThreads, 0, as_stream(stream)>>>(t);
    note_launch();
    return check_launch("adam_step_multi_lean");
}

}  // extern "C"
