// gs3d_backward.cu - 3DGS backward: per-Gaussian warp-bucketed blend backward, then the preprocess
// backward to the six parameter gradients.
//
// k_blend_backward: persistent warps (a grid sized to the SMs) take, from an atomic work counter, the
// buckets the forward listed as reached (those before their tile's last contributor); one warp per
// (tile, 32-splat bucket) at a time. Lane l owns the 8 pixels r*32 + l of the
// 16x16 tile (column l % 16, rows 2r + l / 16). From the bucket's (C, T) checkpoint each pixel keeps
// T and rho = G . (image - C) (image with background), so that
//     dL/dalpha_j = T_j (G . c_j) - rho_after_j / max(1 - alpha_j, 1e-6),  rho_after_j = rho_j - T_j alpha_j (G . c_j)
// (the formulation of phase1/fastergs_macro.patch:22-31,186-198), and replays the bucket's splats in
// front-to-back order up to the pixel's last contributor. Row bands whose culling rectangle misses
// the splat are skipped by the whole warp. Per splat the lanes' nine sums (mean2d 2, conic 3,
// opacity, colour 3) are reduced with shuffles and lane 0 issues three vector atomics (float2,
// float4, float4) instead of nine scalar ones; the reduction halves the nine sums across the lanes (9 -> 5 ->
// 3 -> 2 -> 1 per lane, 12 shuffles) and lane 0 collects the totals (8 shuffles) instead of 45 butterfly
// shuffles. With three densification rows it also sums the per-pixel absolute mean2d gradients (two more
// values and one more float2 atomic per splat).
//
// k_preprocess_backward: one thread per Gaussian recomputes the projection and chains
// (dL/dmean2d, dL/dconic, dL/dopacity, dL/dcolour) to means, scales, rotations, opacity logits,
// sh0 and sh_rest. SH rows are read and their gradients written per warp through shared memory with
// 16-byte accesses (the coalesced layout of upstream/sh_coalesced_loads.patch:12-52). Gaussians
// that were not visible get zero gradients.
#include <algorithm>

#include "adam_math.cuh"
#include "gs3d_common.cuh"

namespace splat {
namespace gs3d {

constexpr int kBwdWarps = 4;
#ifndef SPLAT_BWD_MIN_BLOCKS
#define SPLAT_BWD_MIN_BLOCKS 7  // 72 registers, no spills: 28 warps per SM instead of 20
#endif
constexpr int kPxPerLane = kTilePixels / 32;  // 8
constexpr int kPbThreads = 128;
constexpr int kPbWarps = kPbThreads / 32;
constexpr float kLn2 = 0.6931471805599453f;

struct GradAcc {
    uint32_t* work;  // next entry of the replayed-bucket list for the blend backward's persistent warps
    float2* mean2d;  // [N] dL/dmean2d
    float4* conic_o;  // [N] (dL/dA, dL/dB, dL/dC, dL/dopacity)
    float4* color;   // [N] dL/d max(colour, 0), w unused
    float2* mean2d_abs;  // [N] sums of |per-pixel dL/dmean2d| (cleared and written only for 3 densification rows)
};

inline GradAcc carve_grad(Carver& c, int n) {
    const size_t nn = static_cast<size_t>(n < 1 ? 1 : n);
    GradAcc g;
    g.work = c.take<uint32_t>(1);
    g.mean2d = c.take<float2>(nn);
    g.conic_o = c.take<float4>(nn);
    g.color = c.take<float4>(nn);
    g.mean2d_abs = c.take<float2>(nn);
    return g;
}

// kAbs: also accumulate the per-pixel absolute values of the mean2d gradient (the third densification row).
template <bool kAbs>
__global__ void __launch_bounds__(32 * kBwdWarps, SPLAT_BWD_MIN_BLOCKS) k_blend_backward(
    Cam cam, const uint32_t* __restrict__ counters, const uint32_t* __restrict__ reached, uint32_t* __restrict__ work,
    const uint32_t* __restrict__ bucket_tile, const uint2* __restrict__ ranges, const uint32_t* __restrict__ bstart,
    const uint32_t* __restrict__ max_contrib, const uint32_t* __restrict__ point_list,
    const float2* __restrict__ mean2d, const float4* __restrict__ conic_o, const float4* __restrict__ color_z,
    const ushort4* __restrict__ rect, const float* __restrict__ grad_image, const float* __restrict__ image,
    const uint32_t* __restrict__ n_contrib, const float4* __restrict__ ckpt, int n, int m, long long bcap,
    GradAcc acc) {
    __shared__ float2 s_mean[kBwdWarps][kBucket];
    __shared__ float4 s_con[kBwdWarps][kBucket];
    __shared__ float4 s_col[kBwdWarps][kBucket];
    __shared__ ushort4 s_rect[kBwdWarps][kBucket];
    __shared__ uint32_t s_id[kBwdWarps][kBucket];
    __shared__ float4 s_grad[kBwdWarps][kTilePixels];

    const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
    const long long nbuckets = min(static_cast<long long>(counters[1]), bcap);
    const long long nwork = min(static_cast<long long>(counters[2]), bcap);
    const int T_tiles = cam.tiles_x * cam.tiles_y;
    // Persistent warps: each takes the next replayed bucket from the work counter until the list is done, so
    // no warp is launched for a bucket past its tile's last contributor and heavy buckets do not leave a tail.
    for (;;) {
        uint32_t k = 0u;
        if (lane == 0) k = atomicAdd(work, 1u);
        k = __shfl_sync(kFullMask, k, 0);
        if (k >= nwork) break;
        const long long b = reached[k];
        if (b >= nbuckets) continue;
        const uint32_t tile = bucket_tile[b];
        if (tile >= static_cast<uint32_t>(T_tiles)) continue;
        uint2 rg = ranges[tile];
        rg.y = min(rg.y, static_cast<uint32_t>(m));
        rg.x = min(rg.x, rg.y);
        const long long bucket_start = (b - static_cast<long long>(bstart[tile])) * kBucket;
        const long long tile_last = min(static_cast<long long>(max_contrib[tile]), static_cast<long long>(rg.y - rg.x));
        if (bucket_start < 0 || bucket_start >= tile_last) continue;
        const int bsize = static_cast<int>(min(static_cast<long long>(kBucket), tile_last - bucket_start));
        __syncwarp();  // this warp's staging below is rewritten only after every lane finished the previous bucket

        const int tx0 = (tile % cam.tiles_x) * kTile, ty0 = (tile / cam.tiles_x) * kTile;
        if (lane < bsize) {
            const int g = min(static_cast<int>(point_list[rg.x + bucket_start + lane]), n - 1);
            s_id[warp][lane] = g;
            s_mean[warp][lane] = mean2d[g];
            const float4 co = conic_o[g];
            s_con[warp][lane] = make_float4(-0.5f * kLog2e * co.x, -kLog2e * co.y, -0.5f * kLog2e * co.z, co.w);
            const float4 cz = color_z[g];
            s_col[warp][lane] = make_float4(fmaxf(cz.x, 0.f), fmaxf(cz.y, 0.f), fmaxf(cz.z, 0.f), 0.f);
            s_rect[warp][lane] = rect[g];
        }

        const int x = tx0 + (lane & 15);
        const int y0 = ty0 + (lane >> 4);
        const float pxf = static_cast<float>(x) + 0.5f;
        const size_t HW = static_cast<size_t>(cam.width) * cam.height;
        const float4* ck = ckpt + b * kTilePixels;
        float T[kPxPerLane], rho[kPxPerLane];
        // per pixel, how many of this bucket's splats it used in the forward, clamped to [0, 32], 8 bits each
        uint32_t lim_lo = 0u, lim_hi = 0u;
        // Every load of the prologue is issued without waiting on another: addresses are clamped into the image
        // (and the checkpoint block of this bucket), and pixels outside the image or already finished before
        // this bucket get their values replaced by zeros afterwards.
#pragma unroll
        for (int r = 0; r < kPxPerLane; ++r) {
            const int y = y0 + 2 * r;
            const bool inside = x < cam.width && y < cam.height;
            const int pix = inside ? y * cam.width + x : 0;
            const long long used_here = static_cast<long long>(__ldg(n_contrib + pix)) - bucket_start;
            const float4 st = ck[r * 32 + lane];
            const float gx = __ldg(grad_image + pix), gy = __ldg(grad_image + HW + pix), gz = __ldg(grad_image + 2 * HW + pix);
            const float ix = __ldg(image + pix), iy = __ldg(image + HW + pix), iz = __ldg(image + 2 * HW + pix);
            const bool live = inside && used_here > 0;
            const uint32_t l = live ? static_cast<uint32_t>(min(used_here, 32ll)) : 0u;
            if (r < 4)
                lim_lo |= l << (8 * r);
            else
                lim_hi |= l << (8 * (r - 4));
            const float4 G = live ? make_float4(gx, gy, gz, 0.f) : make_float4(0.f, 0.f, 0.f, 0.f);
            T[r] = live ? st.w : 0.f;
            rho[r] = live ? G.x * (ix - st.x) + G.y * (iy - st.y) + G.z * (iz - st.z) : 0.f;
            s_grad[warp][r * 32 + lane] = G;
        }
        __syncwarp();

        for (int j = 0; j < bsize; ++j) {
            const float2 mm = s_mean[warp][j];
            const float4 co = s_con[warp][j];
            const float4 c = s_col[warp][j];
            const ushort4 rc = s_rect[warp][j];
            // per-lane sums over its pixels of t = G dL/dalpha: its moments (for mean2d and conic; dL/dq2 is
            // t opacity ln 2, a per-splat factor applied once to the warp's totals), t itself (opacity), colour
            float s_x = 0.f, s_y = 0.f, s_xx = 0.f, s_xy = 0.f, s_yy = 0.f, g_o = 0.f, g_r = 0.f, g_g = 0.f, g_bl = 0.f;
            float a_x = 0.f, a_y = 0.f;  // kAbs: sums of |per-pixel dL/dmean2d|
            bool used = false;
            const bool col_hit = x >= rc.x && x <= rc.z;
#pragma unroll
            for (int r = 0; r < kPxPerLane; ++r) {
                const int yb = ty0 + 2 * r;  // rows yb, yb + 1 of this band
                if (rc.y > yb + 1 || rc.w < yb) continue;  // warp-uniform
                const uint32_t l = ((r < 4 ? lim_lo : lim_hi) >> (8 * (r & 3))) & 0xffu;
                if (!col_hit || static_cast<uint32_t>(j) >= l) continue;
                const float dx = mm.x - pxf, dy = mm.y - (static_cast<float>(y0 + 2 * r) + 0.5f);
                const float G = hw_exp2(fminf(blend_q2(co.x, co.y, co.z, dx, dy), 0.f));
                const float alpha = co.w * G;
                if (alpha < kAlphaMin) continue;
                used = true;
                const float4 gp = s_grad[warp][r * 32 + lane];
                const float w = alpha * T[r];
                const float dot_c = gp.x * c.x + gp.y * c.y + gp.z * c.z;
                g_r += w * gp.x;
                g_g += w * gp.y;
                g_bl += w * gp.z;
                rho[r] -= w * dot_c;
                const float one_minus = 1.f - alpha;
                const float dL_dalpha = T[r] * dot_c - __fdividef(rho[r], fmaxf(one_minus, kOneMinusAlphaEps));
                const float t = G * dL_dalpha;
                g_o += t;
                const float tx = t * dx, ty = t * dy;
                s_x += tx;
                s_y += ty;
                s_xx += tx * dx;
                s_xy += tx * dy;
                s_yy += ty * dy;
                if (kAbs) {
                    a_x += fabsf(2.f * co.x * tx + co.y * ty);
                    a_y += fabsf(co.y * tx + 2.f * co.z * ty);
                }
                T[r] *= one_minus;
            }
            const unsigned used_mask = __ballot_sync(kFullMask, used);
            if (used_mask == 0u) continue;
            const int g = s_id[warp][j];
            {
                // halving exchanges: 9 -> 5 -> 3 -> 2 -> 1 partial sums per lane (11 shuffles), a last exchange,
                // then lane 0 collects the nine totals from the lanes that hold them (8 shuffles)
                const float v9[9] = {s_x, s_y, s_xx, s_xy, s_yy, g_o, g_r, g_g, g_bl};
                const float t = warp_fold9(v9, lane);
                s_x = t;
                s_y = __shfl_sync(kFullMask, t, 2);
                s_xx = __shfl_sync(kFullMask, t, 4);
                s_xy = __shfl_sync(kFullMask, t, 8);
                s_yy = __shfl_sync(kFullMask, t, 10);
                g_o = __shfl_sync(kFullMask, t, 16);
                g_r = __shfl_sync(kFullMask, t, 18);
                g_g = __shfl_sync(kFullMask, t, 20);
                g_bl = __shfl_sync(kFullMask, t, 24);
                if (kAbs) {
#pragma unroll
                    for (int o = 16; o > 0; o >>= 1) {
                        a_x += __shfl_down_sync(kFullMask, a_x, o);
                        a_y += __shfl_down_sync(kFullMask, a_y, o);
                    }
                }
            }
            if (lane == 0) {
                // dL/dq2 = t opacity ln 2 (alpha = opacity 2^q2). q2 = a2 dx^2 + b2 dx dy + c2 dy^2: dq2/dmx =
                // 2 a2 dx + b2 dy, dq2/dmy = b2 dx + 2 c2 dy; back from the exp2-scaled conic (a2, b2, c2) =
                // log2(e) (-0.5 A, -B, -0.5 C) to (A, B, C), log2(e) ln 2 = 1
                const float k = co.w * kLn2;
                atomicAdd(acc.mean2d + g,
                          make_float2(k * (2.f * co.x * s_x + co.y * s_y), k * (co.y * s_x + 2.f * co.z * s_y)));
                atomicAdd(acc.conic_o + g,
                          make_float4(-0.5f * co.w * s_xx, -co.w * s_xy, -0.5f * co.w * s_yy, g_o));
                atomicAdd(acc.color + g, make_float4(g_r, g_g, g_bl, 0.f));
                if (kAbs) atomicAdd(acc.mean2d_abs + g, make_float2(k * a_x, k * a_y));
            }
        }
    }
}

struct PParams {
    const float* means;
    const float* scales;
    const float* rotations;
    const float* opacities;
    const float* sh_rest;
    const float* w2c;
    const float* cam_pos;
    int n;
};

// The six gradient outputs (means, scales, rotations, opacities, sh0, sh_rest) of the unfused preprocess backward.
struct Grads {
    float* ptr[6];
    int vec;         // the SH-rest output 16-byte aligned
    int accumulate;  // add into the outputs instead of storing (the gradients of several views of one batch)
    // When set, the SH gradients are not formed: per Gaussian, six floats (dL/dcolour masked by the colour clamp,
    // then the unit view direction) are stored here instead, zeros for a Gaussian the view does not see; ptr[4]
    // and ptr[5] are unused. Always stored, also with accumulate (each view has its own records).
    float* records;
};

__device__ __forceinline__ void sh_backward(float x, float y, float z, int bases, const float* v, float& gx, float& gy,
                                            float& gz) {
    // v[k] = sum over channels of dL/dcolour * coefficient k; returns dL/d(direction)
    gx = gy = gz = 0.f;
    if (bases > 1) {
        gy += -kSH1 * v[1];
        gz += kSH1 * v[2];
        gx += -kSH1 * v[3];
    }
    if (bases > 4) {
        const float xx = x * x, yy = y * y, zz = z * z;
        gx += kSH2_0 * y * v[4];
        gy += kSH2_0 * x * v[4];
        gy += kSH2_1 * z * v[5];
        gz += kSH2_1 * y * v[5];
        gx += -2.f * kSH2_2 * x * v[6];
        gy += -2.f * kSH2_2 * y * v[6];
        gz += 4.f * kSH2_2 * z * v[6];
        gx += kSH2_3 * z * v[7];
        gz += kSH2_3 * x * v[7];
        gx += 2.f * kSH2_4 * x * v[8];
        gy += -2.f * kSH2_4 * y * v[8];
        if (bases > 9) {
            gx += 6.f * kSH3_0 * x * y * v[9];
            gy += kSH3_0 * (3.f * xx - 3.f * yy) * v[9];
            gx += kSH3_1 * y * z * v[10];
            gy += kSH3_1 * x * z * v[10];
            gz += kSH3_1 * x * y * v[10];
            gx += -2.f * kSH3_2 * x * y * v[11];
            gy += kSH3_2 * (4.f * zz - xx - 3.f * yy) * v[11];
            gz += 8.f * kSH3_2 * y * z * v[11];
            gx += -6.f * kSH3_3 * x * z * v[12];
            gy += -6.f * kSH3_3 * y * z * v[12];
            gz += kSH3_3 * (6.f * zz - 3.f * xx - 3.f * yy) * v[12];
            gx += kSH3_4 * (4.f * zz - 3.f * xx - yy) * v[13];
            gy += -2.f * kSH3_4 * x * y * v[13];
            gz += 8.f * kSH3_4 * x * z * v[13];
            gx += 2.f * kSH3_5 * x * z * v[14];
            gy += -2.f * kSH3_5 * y * z * v[14];
            gz += kSH3_5 * (xx - yy) * v[14];
            gx += kSH3_6 * (3.f * xx - 3.f * yy) * v[15];
            gy += -6.f * kSH3_6 * x * y * v[15];
        }
    }
}

struct Densification {
    float* info;  // [rows, N], accumulated in place
    int rows;     // 0, 2 or 3
};

// Densification statistics of visible Gaussian i: visible count, |dL/dmean2d| in normalised device units (pixels
// scaled by half the image size), and with three rows the same norm of the summed per-pixel |dL/dmean2d|.
__device__ __forceinline__ void accumulate_densification(const Densification& dens, const GradAcc& acc, const Cam& cam,
                                                         int n, int i, float2 gm) {
    // each operation rounded on its own: the rows do not depend on how the calling kernel was compiled
    const float hw = 0.5f * static_cast<float>(cam.width), hh = 0.5f * static_cast<float>(cam.height);
    auto norm = [&](float2 g) {
        const float a = __fmul_rn(g.x, hw), b = __fmul_rn(g.y, hh);
        return __fsqrt_rn(__fadd_rn(__fmul_rn(a, a), __fmul_rn(b, b)));
    };
    dens.info[i] = __fadd_rn(dens.info[i], 1.f);
    float* row1 = dens.info + static_cast<size_t>(n) + i;
    *row1 = __fadd_rn(*row1, norm(gm));
    if (dens.rows == 3) {
        float* row2 = dens.info + 2 * static_cast<size_t>(n) + i;
        *row2 = __fadd_rn(*row2, norm(acc.mean2d_abs[i]));
    }
}

// The densification rows alone (when the preprocess backward is deferred to a fused Adam step).
__global__ void k_densification(int n, Cam cam, PrimBuffers pb, GradAcc acc, Densification dens) {
    const int i = blockIdx.x * blockDim.x + threadIdx.x;
    if (i >= n || pb.n_touched[i] == 0) return;
    accumulate_densification(dens, acc, cam, n, i, acc.mean2d[i]);
}

// The Adam step fused into the preprocess backward (when `fused`): groups in the order means, scales, rotations,
// opacities, sh0, sh_rest. Each gradient element is added to grad_in (the gradient other terms of the loss left,
// when given: autograd's accumulation, existing + new) and applied to its parameter and moments in place; the
// gradient itself is never stored.
struct AdamArgs {
    float* param[6];
    float* exp_avg[6];
    float* exp_avg_sq[6];
    const float* grad_in[6];
    float step_size[6];
    float bc2_sqrt_rcp[6];
    float beta1, beta2, eps;
    int vec;    // every buffer of every group 16-byte aligned
    int fused;  // 0: the gradients are stored (Grads) instead
};

__device__ __forceinline__ void fused_adam(const AdamArgs& A, int gi, size_t e, float g) {
    if (A.grad_in[gi]) g = __fadd_rn(A.grad_in[gi][e], g);  // rounded on its own: no contraction with g's product
    float p = A.param[gi][e], m = A.exp_avg[gi][e], v = A.exp_avg_sq[gi][e];
    adam_element(p, g, m, v, A.step_size[gi], A.bc2_sqrt_rcp[gi], A.beta1, A.beta2, A.eps);
    A.param[gi][e] = p;
    A.exp_avg[gi][e] = m;
    A.exp_avg_sq[gi][e] = v;
}

// Shared-memory staging of one warp's gradients for the fused step: the five small groups of its 32 Gaussians in
// Gaussian-major order (means 96, scales 96, rotations 128, opacities 32, sh0 96 floats), after its SH-rest block.
constexpr int kSmallFloats = 448;
__host__ __device__ constexpr int small_offset(int gi) {
    return gi == 0 ? 0 : gi == 1 ? 96 : gi == 2 ? 192 : gi == 3 ? 320 : 352;
}
__host__ __device__ constexpr int group_width(int gi, int rest3) {
    return gi == 0 || gi == 1 || gi == 4 ? 3 : gi == 2 ? 4 : gi == 3 ? 1 : rest3;
}
template <int GI>
__device__ __forceinline__ void adam4_load(const AdamArgs& A, size_t e, float4& p, float4& m, float4& v, float4& h) {
    p = *reinterpret_cast<const float4*>(A.param[GI] + e);
    m = *reinterpret_cast<const float4*>(A.exp_avg[GI] + e);
    v = *reinterpret_cast<const float4*>(A.exp_avg_sq[GI] + e);
    h = A.grad_in[GI] ? *reinterpret_cast<const float4*>(A.grad_in[GI] + e) : make_float4(0.f, 0.f, 0.f, 0.f);
}

template <int GI>
__device__ __forceinline__ void adam4_apply(const AdamArgs& A, size_t e, float4 p, float4 m, float4 v, float4 h,
                                            float4 g) {
    if (A.grad_in[GI])
        g = make_float4(__fadd_rn(h.x, g.x), __fadd_rn(h.y, g.y), __fadd_rn(h.z, g.z), __fadd_rn(h.w, g.w));
    const float ss = A.step_size[GI], bc = A.bc2_sqrt_rcp[GI];
    adam_element(p.x, g.x, m.x, v.x, ss, bc, A.beta1, A.beta2, A.eps);
    adam_element(p.y, g.y, m.y, v.y, ss, bc, A.beta1, A.beta2, A.eps);
    adam_element(p.z, g.z, m.z, v.z, ss, bc, A.beta1, A.beta2, A.eps);
    adam_element(p.w, g.w, m.w, v.w, ss, bc, A.beta1, A.beta2, A.eps);
    *reinterpret_cast<float4*>(A.param[GI] + e) = p;
    *reinterpret_cast<float4*>(A.exp_avg[GI] + e) = m;
    *reinterpret_cast<float4*>(A.exp_avg_sq[GI] + e) = v;
}

// The Adam phase of one warp whose 32 Gaussians' gradients are staged (sh: SH rest, zeros when !sh_staged; sg: the
// small groups): the warp's contiguous block of every group is streamed with 16-byte accesses, the small groups in
// two passes, then the SH-rest block two float4 per lane at a time; each pass loads all its parameters, moments and
// grad_in before it stores any. A partial warp, or buffers that are not 16-byte aligned, take element-wise accesses.
__device__ __forceinline__ void warp_adam(const AdamArgs& A, int first, int cnt, int rest3, const float* sh,
                                          bool sh_staged, const float* sg, int lane) {
    if (cnt == 32 && A.vec) {
        const float4 z = make_float4(0.f, 0.f, 0.f, 0.f);
        {
            float4 p0 = z, m0 = z, v0 = z, h0 = z, p1 = z, m1 = z, v1 = z, h1 = z, p3 = z, m3 = z, v3 = z, h3 = z;
            const size_t e3w = 3 * static_cast<size_t>(first) + 4 * lane, e1w = static_cast<size_t>(first) + 4 * lane;
            if (lane < 24) {
                adam4_load<0>(A, e3w, p0, m0, v0, h0);
                adam4_load<1>(A, e3w, p1, m1, v1, h1);
            }
            if (lane < 8) adam4_load<3>(A, e1w, p3, m3, v3, h3);
            if (lane < 24) {
                adam4_apply<0>(A, e3w, p0, m0, v0, h0, *reinterpret_cast<const float4*>(sg + small_offset(0) + 4 * lane));
                adam4_apply<1>(A, e3w, p1, m1, v1, h1, *reinterpret_cast<const float4*>(sg + small_offset(1) + 4 * lane));
            }
            if (lane < 8)
                adam4_apply<3>(A, e1w, p3, m3, v3, h3, *reinterpret_cast<const float4*>(sg + small_offset(3) + 4 * lane));
        }
        {
            float4 p2 = z, m2 = z, v2 = z, h2 = z, p4 = z, m4 = z, v4 = z, h4 = z;
            const size_t e4w = 4 * static_cast<size_t>(first) + 4 * lane, e3w = 3 * static_cast<size_t>(first) + 4 * lane;
            adam4_load<2>(A, e4w, p2, m2, v2, h2);
            if (lane < 24) adam4_load<4>(A, e3w, p4, m4, v4, h4);
            adam4_apply<2>(A, e4w, p2, m2, v2, h2, *reinterpret_cast<const float4*>(sg + small_offset(2) + 4 * lane));
            if (lane < 24)
                adam4_apply<4>(A, e3w, p4, m4, v4, h4, *reinterpret_cast<const float4*>(sg + small_offset(4) + 4 * lane));
        }
        const int n4 = 8 * rest3;
        const size_t e0 = static_cast<size_t>(rest3) * first;
        for (int k0 = lane; k0 < n4; k0 += 64) {
            const int k1 = k0 + 32;
            float4 pa, ma, va, ha, pb = z, mb = z, vb = z, hb = z;
            adam4_load<5>(A, e0 + 4 * k0, pa, ma, va, ha);
            if (k1 < n4) adam4_load<5>(A, e0 + 4 * k1, pb, mb, vb, hb);
            adam4_apply<5>(A, e0 + 4 * k0, pa, ma, va, ha, sh_staged ? *reinterpret_cast<const float4*>(sh + 4 * k0) : z);
            if (k1 < n4)
                adam4_apply<5>(A, e0 + 4 * k1, pb, mb, vb, hb,
                               sh_staged ? *reinterpret_cast<const float4*>(sh + 4 * k1) : z);
        }
        return;
    }
#pragma unroll 1
    for (int gi = 0; gi < 6; ++gi) {
        const int w = group_width(gi, rest3);
        const size_t e0 = static_cast<size_t>(w) * first;
        for (int k = lane; k < cnt * w; k += 32) {
            const float g = gi < 5 ? sg[small_offset(gi) + k] : (sh_staged ? sh[k] : 0.f);
            fused_adam(A, gi, e0 + k, g);
        }
    }
}

#ifndef SPLAT_PB_MIN_BLOCKS
#define SPLAT_PB_MIN_BLOCKS 8  // 64 registers, no spills: 32 warps per SM
#endif
// One kernel for both modes, so that the gradient arithmetic is the same machine code. Unfused, each gradient is
// stored as it is found (SH rest through shared memory, per warp). Fused (A.fused), every gradient of the warp is
// staged in shared memory and the warp then streams its blocks through the Adam step.
__global__ void __launch_bounds__(kPbThreads, SPLAT_PB_MIN_BLOCKS) k_preprocess_backward(
    PParams P, Cam cam, PrimBuffers pb, GradAcc acc, const __grid_constant__ Grads out, Densification dens,
    const __grid_constant__ AdamArgs A) {
    // [kPbWarps][32 * rest_bases * 3 (+ kSmallFloats when fused)]
    extern __shared__ __align__(16) float s_sh[];
    const int i = blockIdx.x * kPbThreads + threadIdx.x;
    const int lane = threadIdx.x & 31, warp = threadIdx.x >> 5;
    if (i - lane >= P.n) return;  // whole warp past the end
    const bool valid = i < P.n;
    const bool vis = valid && pb.n_touched[i] > 0;
    const int rest3 = cam.rest_bases * 3;
    float* sh = s_sh + warp * (32 * rest3 + (A.fused ? kSmallFloats : 0));
    float* sg = sh + 32 * rest3;  // fused: the small groups' gradients
    const int first = i - lane;
    const int cnt = min(32, P.n - first);
    const int nfl = cnt * rest3;
    // one gradient element of group gi: stored, or staged for the warp's Adam phase
    auto emit = [&](int gi, size_t e, float g) {
        if (gi == 4 && out.records) return;  // the records carry the SH gradients
        if (A.fused)
            sg[small_offset(gi) + static_cast<int>(e - static_cast<size_t>(group_width(gi, rest3)) * first)] = g;
        else if (out.accumulate)
            out.ptr[gi][e] += g;
        else
            out.ptr[gi][e] = g;
    };
    const unsigned any_vis = __ballot_sync(kFullMask, vis);
    // The warp's SH rows stream into shared memory while every per-Gaussian input is loaded into registers.
    const bool stage = any_vis && cam.active_sh_bases > 1 && rest3 > 0;
    const float* sh_src = P.sh_rest + static_cast<size_t>(first) * rest3;
    const int staged = stage ? stage_sh_begin(sh, sh_src, nfl, lane) : 0;
    float px = 0.f, py = 0.f, pz = 0.f, ls0 = 0.f, ls1 = 0.f, ls2 = 0.f, op_logit = 0.f;
    float2 gm = make_float2(0.f, 0.f);
    float4 gco = make_float4(0.f, 0.f, 0.f, 0.f), gcl = gco, cz = gco, q = make_float4(1.f, 0.f, 0.f, 0.f);
    if (vis) {
        px = P.means[3 * i];
        py = P.means[3 * i + 1];
        pz = P.means[3 * i + 2];
        gm = acc.mean2d[i];
        gco = acc.conic_o[i];
        gcl = acc.color[i];
        cz = pb.color_z[i];
        q = make_float4(P.rotations[4 * i], P.rotations[4 * i + 1], P.rotations[4 * i + 2], P.rotations[4 * i + 3]);
        ls0 = P.scales[3 * i];
        ls1 = P.scales[3 * i + 1];
        ls2 = P.scales[3 * i + 2];
        op_logit = P.opacities[i];
    }
    if (stage) stage_sh_end(sh, sh_src, nfl, staged, lane);
    __syncwarp();

    float* my_sh = sh + lane * rest3;  // this Gaussian's coefficients, overwritten by their gradients
    if (vis) {
        float w2c[12];
#pragma unroll
        for (int k = 0; k < 12; ++k) w2c[k] = __ldg(P.w2c + k);
        const float xc = w2c[0] * px + w2c[1] * py + w2c[2] * pz + w2c[3];
        const float yc = w2c[4] * px + w2c[5] * py + w2c[6] * pz + w2c[7];
        const float zc = w2c[8] * px + w2c[9] * py + w2c[10] * pz + w2c[11];

        const float gr = cz.x >= 0.f ? gcl.x : 0.f, gg = cz.y >= 0.f ? gcl.y : 0.f, gb = cz.z >= 0.f ? gcl.z : 0.f;

        // ---- SH: colour = sum_k basis_k(d) sh_k + 0.5, d = (p - cam) / |p - cam|
        float ux = px - __ldg(P.cam_pos), uy = py - __ldg(P.cam_pos + 1), uz = pz - __ldg(P.cam_pos + 2);
        const float inv_len = rsqrtf(ux * ux + uy * uy + uz * uz);
        const float dx = ux * inv_len, dy = uy * inv_len, dz = uz * inv_len;
        float bas[16];
        sh_basis_rn(dx, dy, dz, cam.active_sh_bases, bas);
        // each product rounded on its own, as the compact exchange forms it from the records
        emit(4, 3 * i, __fmul_rn(bas[0], gr));
        emit(4, 3 * i + 1, __fmul_rn(bas[0], gg));
        emit(4, 3 * i + 2, __fmul_rn(bas[0], gb));
        if (out.records) {
            float* rec = out.records + 6 * static_cast<size_t>(i);
            rec[0] = gr;
            rec[1] = gg;
            rec[2] = gb;
            rec[3] = dx;
            rec[4] = dy;
            rec[5] = dz;
        }
        float v[16];
        v[0] = 0.f;
        const int nb = min(cam.active_sh_bases, cam.rest_bases + 1);
#pragma unroll
        for (int k = 1; k < 16; ++k) {  // unrolled, so bas and v stay in registers
            v[k] = 0.f;
            if (k < nb) {
                const float cr = my_sh[3 * (k - 1)], cg = my_sh[3 * (k - 1) + 1], cb = my_sh[3 * (k - 1) + 2];
                v[k] = gr * cr + gg * cg + gb * cb;
                my_sh[3 * (k - 1)] = __fmul_rn(bas[k], gr);
                my_sh[3 * (k - 1) + 1] = __fmul_rn(bas[k], gg);
                my_sh[3 * (k - 1) + 2] = __fmul_rn(bas[k], gb);
            }
        }
        for (int k = max(nb, 1); k <= cam.rest_bases; ++k) {
            my_sh[3 * (k - 1)] = 0.f;
            my_sh[3 * (k - 1) + 1] = 0.f;
            my_sh[3 * (k - 1) + 2] = 0.f;
        }
        float gdx, gdy, gdz;
        sh_backward(dx, dy, dz, nb, v, gdx, gdy, gdz);
        const float dd = gdx * dx + gdy * dy + gdz * dz;
        float gpx = (gdx - dx * dd) * inv_len, gpy = (gdy - dy * dd) * inv_len, gpz = (gdz - dz * dd) * inv_len;

        // ---- recompute the projection
        float nsq;
        const Mat3 R = quat_to_rot(q, nsq);
        const float s[3] = {expf(ls0), expf(ls1), expf(ls2)};
        float M[3][3];
#pragma unroll
        for (int r = 0; r < 3; ++r)
#pragma unroll
            for (int c = 0; c < 3; ++c) M[r][c] = R.m[r][c] * s[c];
        float S3[3][3];
#pragma unroll
        for (int r = 0; r < 3; ++r)
#pragma unroll
            for (int c = 0; c < 3; ++c) S3[r][c] = M[r][0] * M[c][0] + M[r][1] * M[c][1] + M[r][2] * M[c][2];
        float T1[3][3], Sc[3][3];
#pragma unroll
        for (int r = 0; r < 3; ++r)
#pragma unroll
            for (int c = 0; c < 3; ++c)
                T1[r][c] = w2c[4 * r] * S3[0][c] + w2c[4 * r + 1] * S3[1][c] + w2c[4 * r + 2] * S3[2][c];
#pragma unroll
        for (int r = 0; r < 3; ++r)
#pragma unroll
            for (int c = 0; c < 3; ++c)
                Sc[r][c] = T1[r][0] * w2c[4 * c] + T1[r][1] * w2c[4 * c + 1] + T1[r][2] * w2c[4 * c + 2];
        const float inv_z = 1.f / zc;
        const float lox = -1.3f * cam.cx / cam.fx, hix = 1.3f * (cam.width - cam.cx) / cam.fx;
        const float loy = -1.3f * cam.cy / cam.fy, hiy = 1.3f * (cam.height - cam.cy) / cam.fy;
        const float rx = xc * inv_z, ry = yc * inv_z;
        const float tx = fminf(fmaxf(rx, lox), hix), ty = fminf(fmaxf(ry, loy), hiy);
        const bool free_x = rx >= lox && rx <= hix, free_y = ry >= loy && ry <= hiy;
        const float j00 = cam.fx * inv_z, j02 = -cam.fx * tx * inv_z;
        const float j11 = cam.fy * inv_z, j12 = -cam.fy * ty * inv_z;
        const float a = j00 * (j00 * Sc[0][0] + j02 * Sc[0][2]) + j02 * (j00 * Sc[2][0] + j02 * Sc[2][2]);
        const float b = j00 * (j11 * Sc[0][1] + j12 * Sc[0][2]) + j02 * (j11 * Sc[2][1] + j12 * Sc[2][2]);
        const float c = j11 * (j11 * Sc[1][1] + j12 * Sc[1][2]) + j12 * (j11 * Sc[2][1] + j12 * Sc[2][2]);
        const float ad = a + kDilation, cd = c + kDilation;
        const float det = ad * cd - b * b;
        const float inv_det = 1.f / det;
        const float A = cd * inv_det, B = -b * inv_det, C = ad * inv_det;
        const float sig = 1.f / (1.f + expf(-op_logit));

        // ---- opacity (and the antialiasing factor f = sqrt(det(Sigma2) / det(Sigma2 + 0.3 I)))
        float ga = 0.f, gb2 = 0.f, gc = 0.f;  // dL/d(a, b, c) of Sigma2 (b = the off-diagonal value)
        float f = 1.f;
        if (cam.proper_aa) {
            const float det0 = a * c - b * b;
            const float ratio = det0 * inv_det;
            if (ratio > 0.f) {
                f = sqrtf(ratio);
                const float dL_dratio = gco.w * sig * 0.5f / f;
                const float id2 = inv_det * inv_det;
                ga += dL_dratio * (c * det - det0 * cd) * id2;
                gc += dL_dratio * (a * det - det0 * ad) * id2;
                gb2 += dL_dratio * (-2.f * b * (det - det0)) * id2;
            } else {
                f = 0.f;
            }
        }
        emit(3, i, gco.w * f * sig * (1.f - sig));

        // ---- conic = inverse of [[ad, b], [b, cd]]: dL/dS = -K G K with G = [[gA, gB/2], [gB/2, gC]]
        {
            const float g0 = gco.x, g1 = 0.5f * gco.y, g2 = gco.z;
            const float k00 = A * g0 + B * g1, k01 = A * g1 + B * g2, k10 = B * g0 + C * g1, k11 = B * g1 + C * g2;
            const float p00 = k00 * A + k01 * B, p01 = k00 * B + k01 * C, p11 = k10 * B + k11 * C;
            ga += -p00;
            gc += -p11;
            gb2 += -2.f * p01;
        }

        // ---- Sigma2 = J Sc J^T: dL/dSc = J^T G2 J, dL/dJ = 2 G2 J Sc, G2 = [[ga, gb2/2], [gb2/2, gc]]
        const float G2[2][2] = {{ga, 0.5f * gb2}, {0.5f * gb2, gc}};
        const float J[2][3] = {{j00, 0.f, j02}, {0.f, j11, j12}};
        float GJ[2][3];
#pragma unroll
        for (int r = 0; r < 2; ++r)
#pragma unroll
            for (int k = 0; k < 3; ++k) GJ[r][k] = G2[r][0] * J[0][k] + G2[r][1] * J[1][k];
        float gSc[3][3];
#pragma unroll
        for (int r = 0; r < 3; ++r)
#pragma unroll
            for (int k = 0; k < 3; ++k) gSc[r][k] = J[0][r] * GJ[0][k] + J[1][r] * GJ[1][k];
        float gJ[2][3];
#pragma unroll
        for (int r = 0; r < 2; ++r)
#pragma unroll
            for (int k = 0; k < 3; ++k)
                gJ[r][k] = 2.f * (GJ[r][0] * Sc[0][k] + GJ[r][1] * Sc[1][k] + GJ[r][2] * Sc[2][k]);

        // ---- J and mean2d to camera coordinates
        const float iz2 = inv_z * inv_z;
        float gxc = cam.fx * inv_z * gm.x;
        float gyc = cam.fy * inv_z * gm.y;
        float gzc = -cam.fx * xc * iz2 * gm.x - cam.fy * yc * iz2 * gm.y;
        gzc += -cam.fx * iz2 * gJ[0][0] - cam.fy * iz2 * gJ[1][1];
        // j02 = -fx tx / z with tx = x / z inside the clamp window (dtx/dz = -x / z^2), constant outside:
        // dj02/dz = fx tx / z^2 - (fx / z) dtx/dz, dj02/dx = -(fx / z) dtx/dx
        gzc += gJ[0][2] * (cam.fx * tx * iz2 + (free_x ? cam.fx * inv_z * xc * iz2 : 0.f));
        gxc += free_x ? gJ[0][2] * (-cam.fx * iz2) : 0.f;
        gzc += gJ[1][2] * (cam.fy * ty * iz2 + (free_y ? cam.fy * inv_z * yc * iz2 : 0.f));
        gyc += free_y ? gJ[1][2] * (-cam.fy * iz2) : 0.f;
        gpx += w2c[0] * gxc + w2c[4] * gyc + w2c[8] * gzc;
        gpy += w2c[1] * gxc + w2c[5] * gyc + w2c[9] * gzc;
        gpz += w2c[2] * gxc + w2c[6] * gyc + w2c[10] * gzc;
        emit(0, 3 * i, gpx);
        emit(0, 3 * i + 1, gpy);
        emit(0, 3 * i + 2, gpz);

        // ---- densification statistics: visible count, |dL/dmean2d| in normalised device units (pixels scaled
        // by half the image size), and with three rows the same norm of the summed per-pixel |dL/dmean2d|
        if (dens.rows >= 2) accumulate_densification(dens, acc, cam, P.n, i, gm);

        // ---- Sc = Wr S3 Wr^T: dL/dS3 = Wr^T gSc Wr; S3 = M M^T: dL/dM = 2 dL/dS3 M
        float t1[3][3], gS3[3][3];
#pragma unroll
        for (int r = 0; r < 3; ++r)
#pragma unroll
            for (int k = 0; k < 3; ++k) t1[r][k] = w2c[r] * gSc[0][k] + w2c[4 + r] * gSc[1][k] + w2c[8 + r] * gSc[2][k];
#pragma unroll
        for (int r = 0; r < 3; ++r)
#pragma unroll
            for (int k = 0; k < 3; ++k) gS3[r][k] = t1[r][0] * w2c[k] + t1[r][1] * w2c[4 + k] + t1[r][2] * w2c[8 + k];
        float gM[3][3];
#pragma unroll
        for (int r = 0; r < 3; ++r)
#pragma unroll
            for (int k = 0; k < 3; ++k)
                gM[r][k] = 2.f * (gS3[r][0] * M[0][k] + gS3[r][1] * M[1][k] + gS3[r][2] * M[2][k]);
        float gR[3][3];
#pragma unroll
        for (int k = 0; k < 3; ++k) {
            const float gs = gM[0][k] * R.m[0][k] + gM[1][k] * R.m[1][k] + gM[2][k] * R.m[2][k];
            emit(1, 3 * i + k, gs * s[k]);
#pragma unroll
            for (int r = 0; r < 3; ++r) gR[r][k] = gM[r][k] * s[k];
        }
        // ---- rotation of the normalised quaternion (w, x, y, z), then the normalisation
        const float inv_n = rsqrtf(fmaxf(nsq, 1e-30f));
        const float w = q.x * inv_n, qx = q.y * inv_n, qy = q.z * inv_n, qz = q.w * inv_n;
        const float gw = 2.f * (-qz * gR[0][1] + qy * gR[0][2] + qz * gR[1][0] - qx * gR[1][2] - qy * gR[2][0] +
                                qx * gR[2][1]);
        const float gx = 2.f * (qy * gR[0][1] + qz * gR[0][2] + qy * gR[1][0] - 2.f * qx * gR[1][1] - w * gR[1][2] +
                                qz * gR[2][0] + w * gR[2][1] - 2.f * qx * gR[2][2]);
        const float gy = 2.f * (-2.f * qy * gR[0][0] + qx * gR[0][1] + w * gR[0][2] + qx * gR[1][0] + qz * gR[1][2] -
                                w * gR[2][0] + qz * gR[2][1] - 2.f * qy * gR[2][2]);
        const float gz = 2.f * (-2.f * qz * gR[0][0] - w * gR[0][1] + qx * gR[0][2] + w * gR[1][0] -
                                2.f * qz * gR[1][1] + qy * gR[1][2] + qx * gR[2][0] + qy * gR[2][1]);
        const float qd = gw * w + gx * qx + gy * qy + gz * qz;
        emit(2, 4 * i, (gw - w * qd) * inv_n);
        emit(2, 4 * i + 1, (gx - qx * qd) * inv_n);
        emit(2, 4 * i + 2, (gy - qy * qd) * inv_n);
        emit(2, 4 * i + 3, (gz - qz * qd) * inv_n);
    } else if (valid) {
        if (!out.accumulate) {  // zero gradients (nothing to add when accumulating)
#pragma unroll
            for (int k = 0; k < 3; ++k) {
                emit(0, 3 * i + k, 0.f);
                emit(1, 3 * i + k, 0.f);
                emit(4, 3 * i + k, 0.f);
            }
#pragma unroll
            for (int k = 0; k < 4; ++k) emit(2, 4 * i + k, 0.f);
            emit(3, i, 0.f);
        }
        if (out.records) {  // not seen by this view: its records are zeros
            float* rec = out.records + 6 * static_cast<size_t>(i);
#pragma unroll
            for (int k = 0; k < 6; ++k) rec[k] = 0.f;
        }
        // this Gaussian's row of the warp's staged block still holds its SH coefficients: its gradients are zeros
        if (rest3 > 0 && any_vis && cam.active_sh_bases > 1)
            for (int k = 0; k < rest3; ++k) my_sh[k] = 0.f;
    }
    __syncwarp();
    const bool sh_staged = any_vis && cam.active_sh_bases > 1;
    if (A.fused) {  // every gradient of the warp is staged: one streaming Adam phase over its blocks
        warp_adam(A, first, cnt, rest3, sh, sh_staged, sg, lane);
        return;
    }
    if (out.records) return;  // no SH-rest gradients are formed
    // the warp's SH-rest gradients as one contiguous block
    if (rest3 > 0 && out.accumulate) {
        if (!sh_staged) return;  // all zeros
        float* dst = out.ptr[5] + static_cast<size_t>(first) * rest3;
        int done = 0;
        if (out.vec) {
            const int n4 = nfl / 4;
            for (int k = lane; k < n4; k += 32) {
                float4 d = reinterpret_cast<float4*>(dst)[k];
                const float4 a = reinterpret_cast<const float4*>(sh)[k];
                d.x += a.x;
                d.y += a.y;
                d.z += a.z;
                d.w += a.w;
                reinterpret_cast<float4*>(dst)[k] = d;
            }
            done = n4 * 4;
        }
        for (int k = done + lane; k < nfl; k += 32) dst[k] += sh[k];
    } else if (rest3 > 0) {
        float* dst = out.ptr[5] + static_cast<size_t>(first) * rest3;
        int done = 0;
        if (out.vec) {
            const int n4 = nfl / 4;
            for (int k = lane; k < n4; k += 32)
                reinterpret_cast<float4*>(dst)[k] = sh_staged ? reinterpret_cast<const float4*>(sh)[k]
                                                              : make_float4(0.f, 0.f, 0.f, 0.f);
            done = n4 * 4;
        }
        for (int k = done + lane; k < nfl; k += 32) dst[k] = sh_staged ? sh[k] : 0.f;
    }
}

}  // namespace gs3d
}  // namespace splat

using namespace splat;
using namespace splat::gs3d;

extern "C" {

size_t gs3d_backward_workspace_size(int n) {
    Carver c(nullptr, 0);
    carve_grad(c, n);
    return c.used + 256;
}

int gs3d_backward_blend(const float* grad_image, const float* image, int n, long long num_instances,
                        const gs3d_settings* settings, void* prim_buf, size_t prim_bytes_, void* tile_buf,
                        size_t tile_bytes_, void* inst_buf, size_t inst_bytes_, void* bucket_buf,
                        size_t bucket_bytes_, long long bucket_capacity, void* workspace, size_t workspace_bytes,
                        int densification_rows, void* stream) {
    Cam cam;
    SPLAT_TRY(fill_cam(settings, cam));
    const long long m = num_instances;
    const int T = cam.tiles_x * cam.tiles_y;
    SPLAT_REQUIRE(n >= 0 && m >= 0 && m < (1ll << 31), "gs3d_backward: bad sizes n=%d M=%lld", n, m);
    SPLAT_REQUIRE(prim_bytes_ >= prim_bytes(n) && tile_bytes_ >= tile_bytes(cam.width, cam.height) &&
                      inst_bytes_ >= inst_bytes(m) && bucket_capacity >= bucket_bound(m, T) &&
                      bucket_bytes_ >= bucket_bytes(bucket_capacity) &&
                      workspace_bytes >= gs3d_backward_workspace_size(n),
                  "gs3d_backward: a buffer is smaller than its size query");
    if (n == 0) return SPLAT_OK;
    cudaStream_t st = as_stream(stream);
    Carver cp(prim_buf, prim_bytes_), ct(tile_buf, tile_bytes_), ci(inst_buf, inst_bytes_),
        cb(bucket_buf, bucket_bytes_), cw(workspace, workspace_bytes);
    PrimBuffers pb = carve_prim(cp, n);
    TileBuffers tb = carve_tile(ct, cam.width, cam.height);
    InstBuffers ib = carve_inst(ci, m);
    BucketBuffers bb = carve_bucket(cb, bucket_capacity);
    SPLAT_REQUIRE(densification_rows == 0 || densification_rows == 2 || densification_rows == 3,
                  "gs3d_backward: densification_info must have 0, 2 or 3 rows (got %d)", densification_rows);
    GradAcc acc = carve_grad(cw, n);
    const bool abs_grad = densification_rows == 3;
    // the |dL/dmean2d| sums come last in the workspace and are cleared only when they are accumulated
    const size_t clear = abs_grad ? cw.used : static_cast<size_t>(reinterpret_cast<char*>(acc.mean2d_abs) -
                                                                  static_cast<char*>(workspace));
    SPLAT_CUDA(cudaMemsetAsync(workspace, 0, clear, st));
    if (m > 0) {
        const long long blocks = std::min<long long>(static_cast<long long>(sm_count()) * SPLAT_BWD_MIN_BLOCKS,
                                                     div_up(bucket_capacity, kBwdWarps));
        auto kernel = abs_grad ? k_blend_backward<true> : k_blend_backward<false>;
        SPLAT_TIMED_LAUNCH("k_blend_backward", st,
                           (kernel<<<static_cast<unsigned>(blocks), 32 * kBwdWarps, 0, st>>>(
                               cam, pb.counters, bb.reached, acc.work, bb.tile, tb.ranges, tb.bstart, tb.max_contrib,
                               ib.point_list, pb.mean2d, pb.conic_o, pb.color_z, pb.rect, grad_image, image,
                               tb.n_contrib, bb.ckpt, n, static_cast<int>(m), bucket_capacity, acc)));
        note_launch();
        SPLAT_TRY(check_launch("gs3d_blend_backward"));
    }
    return SPLAT_OK;
}

namespace {
int preprocess_backward(const float* means, const float* scales, const float* rotations, const float* opacities,
                        const float* sh_rest, int n, const gs3d_settings* settings, void* prim_buf, size_t prim_bytes_,
                        void* workspace, size_t workspace_bytes, float* grad_means, float* grad_scales,
                        float* grad_rotations, float* grad_opacities, float* grad_sh0, float* grad_sh_rest,
                        float* densification_info, int densification_rows, int accumulate, void* stream,
                        float* records = nullptr) {
    Cam cam;
    SPLAT_TRY(fill_cam(settings, cam));
    SPLAT_REQUIRE(n >= 0, "gs3d_backward: bad size n=%d", n);
    SPLAT_REQUIRE(densification_rows == 0 || ((densification_rows == 2 || densification_rows == 3) &&
                                              densification_info != nullptr),
                  "gs3d_backward: densification_info must have 0, 2 or 3 rows (got %d)", densification_rows);
    SPLAT_REQUIRE(prim_bytes_ >= prim_bytes(n) && workspace_bytes >= gs3d_backward_workspace_size(n),
                  "gs3d_backward: a buffer is smaller than its size query");
    if (n == 0) return SPLAT_OK;
    Carver cp(prim_buf, prim_bytes_), cw(workspace, workspace_bytes);
    PrimBuffers pb = carve_prim(cp, n);
    GradAcc acc = carve_grad(cw, n);
    PParams P{means, scales, rotations, opacities, sh_rest, settings->w2c, settings->cam_position, n};
    Grads g{{grad_means, grad_scales, grad_rotations, grad_opacities, grad_sh0, grad_sh_rest}, 0, accumulate,
            records};
    for (int gi = 0; gi < 6; ++gi)
        SPLAT_REQUIRE(g.ptr[gi] || (gi >= 4 && records) || (gi == 5 && cam.rest_bases == 0),
                      "gs3d_backward: gradient output %d is null", gi);
    g.vec = (reinterpret_cast<uintptr_t>(grad_sh_rest) & 15u) == 0;
    const size_t smem = static_cast<size_t>(kPbWarps) * 32 * cam.rest_bases * 3 * sizeof(float);
    const Densification dens{densification_info, densification_rows};
    SPLAT_TIMED_LAUNCH("k_preprocess_backward", as_stream(stream),
                       (k_preprocess_backward<<<div_up(n, kPbThreads), kPbThreads, smem, as_stream(stream)>>>(
                           P, cam, pb, acc, g, dens, AdamArgs{})));
    note_launch();
    return check_launch("gs3d_preprocess_backward");
}
}  // namespace

int gs3d_backward_preprocess(const float* means, const float* scales, const float* rotations,
                             const float* opacities, const float* sh_rest, int n, const gs3d_settings* settings,
                             void* prim_buf, size_t prim_bytes_, void* workspace, size_t workspace_bytes,
                             float* grad_means, float* grad_scales, float* grad_rotations, float* grad_opacities,
                             float* grad_sh0, float* grad_sh_rest, float* densification_info,
                             int densification_rows, void* stream) {
    return preprocess_backward(means, scales, rotations, opacities, sh_rest, n, settings, prim_buf, prim_bytes_,
                               workspace, workspace_bytes, grad_means, grad_scales, grad_rotations, grad_opacities,
                               grad_sh0, grad_sh_rest, densification_info, densification_rows, 0, stream);
}

int gs3d_backward_preprocess_accumulate(const float* means, const float* scales, const float* rotations,
                                        const float* opacities, const float* sh_rest, int n,
                                        const gs3d_settings* settings, void* prim_buf, size_t prim_bytes_,
                                        void* workspace, size_t workspace_bytes, float* grad_means,
                                        float* grad_scales, float* grad_rotations, float* grad_opacities,
                                        float* grad_sh0, float* grad_sh_rest, float* densification_info,
                                        int densification_rows, void* stream) {
    return preprocess_backward(means, scales, rotations, opacities, sh_rest, n, settings, prim_buf, prim_bytes_,
                               workspace, workspace_bytes, grad_means, grad_scales, grad_rotations, grad_opacities,
                               grad_sh0, grad_sh_rest, densification_info, densification_rows, 1, stream);
}

int gs3d_backward_preprocess_records(const float* means, const float* scales, const float* rotations,
                                     const float* opacities, const float* sh_rest, int n,
                                     const gs3d_settings* settings, void* prim_buf, size_t prim_bytes_,
                                     void* workspace, size_t workspace_bytes, float* grad_means, float* grad_scales,
                                     float* grad_rotations, float* grad_opacities, float* sh_records,
                                     int accumulate, float* densification_info, int densification_rows,
                                     void* stream) {
    SPLAT_REQUIRE(sh_records != nullptr, "gs3d_backward_preprocess_records: sh_records is null");
    return preprocess_backward(means, scales, rotations, opacities, sh_rest, n, settings, prim_buf, prim_bytes_,
                               workspace, workspace_bytes, grad_means, grad_scales, grad_rotations, grad_opacities,
                               nullptr, nullptr, densification_info, densification_rows, accumulate ? 1 : 0, stream,
                               sh_records);
}

int gs3d_backward_densification(int n, const gs3d_settings* settings, void* prim_buf, size_t prim_bytes_,
                                void* workspace, size_t workspace_bytes, float* densification_info,
                                int densification_rows, void* stream) {
    Cam cam;
    SPLAT_TRY(fill_cam(settings, cam));
    SPLAT_REQUIRE(n >= 0, "gs3d_backward_densification: bad size n=%d", n);
    SPLAT_REQUIRE(densification_rows == 0 || ((densification_rows == 2 || densification_rows == 3) &&
                                              densification_info != nullptr),
                  "gs3d_backward_densification: densification_info must have 0, 2 or 3 rows (got %d)",
                  densification_rows);
    SPLAT_REQUIRE(prim_bytes_ >= prim_bytes(n) && workspace_bytes >= gs3d_backward_workspace_size(n),
                  "gs3d_backward_densification: a buffer is smaller than its size query");
    if (n == 0 || densification_rows == 0) return SPLAT_OK;
    Carver cp(prim_buf, prim_bytes_), cw(workspace, workspace_bytes);
    PrimBuffers pb = carve_prim(cp, n);
    GradAcc acc = carve_grad(cw, n);
    k_densification<<<div_up(n, 256), 256, 0, as_stream(stream)>>>(n, cam, pb, acc,
                                                                   Densification{densification_info,
                                                                                 densification_rows});
    note_launch();
    return check_launch("gs3d_backward_densification");
}

int gs3d_backward_preprocess_adam(float* means, float* scales, float* rotations, float* opacities, float* sh0,
                                  float* sh_rest, int n, const gs3d_settings* settings, void* prim_buf,
                                  size_t prim_bytes_, void* workspace, size_t workspace_bytes,
                                  const gs3d_adam_state* adam, void* stream) {
    Cam cam;
    SPLAT_TRY(fill_cam(settings, cam));
    SPLAT_REQUIRE(n >= 0, "gs3d_backward_preprocess_adam: bad size n=%d", n);
    SPLAT_REQUIRE(adam != nullptr, "gs3d_backward_preprocess_adam: no Adam state");
    SPLAT_REQUIRE(prim_bytes_ >= prim_bytes(n) && workspace_bytes >= gs3d_backward_workspace_size(n),
                  "gs3d_backward_preprocess_adam: a buffer is smaller than its size query");
    if (n == 0) return SPLAT_OK;
    float* params[6] = {means, scales, rotations, opacities, sh0, sh_rest};
    AdamArgs A{};
    for (int gi = 0; gi < 6; ++gi) {
        const bool empty = gi == 5 && cam.rest_bases == 0;  // no SH-rest coefficients: nothing to update
        SPLAT_REQUIRE(empty || (params[gi] && adam->exp_avg[gi] && adam->exp_avg_sq[gi]),
                      "gs3d_backward_preprocess_adam: group %d has a null buffer", gi);
        SPLAT_REQUIRE(adam->step[gi] >= 1, "gs3d_backward_preprocess_adam: group %d step must be >= 1", gi);
        A.param[gi] = params[gi];
        A.exp_avg[gi] = adam->exp_avg[gi];
        A.exp_avg_sq[gi] = adam->exp_avg_sq[gi];
        A.grad_in[gi] = adam->grad_in[gi];
        adam_bias_corrections(adam->lr[gi], adam->beta1, adam->beta2, adam->step[gi], A.step_size[gi],
                              A.bc2_sqrt_rcp[gi]);
    }
    A.beta1 = static_cast<float>(adam->beta1);
    A.beta2 = static_cast<float>(adam->beta2);
    A.eps = static_cast<float>(adam->eps);
    uintptr_t align = 0;
    for (int gi = 0; gi < 6; ++gi)
        align |= reinterpret_cast<uintptr_t>(A.param[gi]) | reinterpret_cast<uintptr_t>(A.exp_avg[gi]) |
                 reinterpret_cast<uintptr_t>(A.exp_avg_sq[gi]) | reinterpret_cast<uintptr_t>(A.grad_in[gi]);
    A.vec = (align & 15u) == 0;
    A.fused = 1;
    Carver cp(prim_buf, prim_bytes_), cw(workspace, workspace_bytes);
    PrimBuffers pb = carve_prim(cp, n);
    GradAcc acc = carve_grad(cw, n);
    PParams P{means, scales, rotations, opacities, sh_rest, settings->w2c, settings->cam_position, n};
    const size_t smem = static_cast<size_t>(kPbWarps) * (32 * cam.rest_bases * 3 + kSmallFloats) * sizeof(float);
    k_preprocess_backward<<<div_up(n, kPbThreads), kPbThreads, smem, as_stream(stream)>>>(
        P, cam, pb, acc, Grads{}, Densification{nullptr, 0}, A);
    note_launch();
    return check_launch("gs3d_backward_preprocess_adam");
}

int gs3d_backward(const float* grad_image, const float* image, const float* means, const float* scales,
                  const float* rotations, const float* opacities, const float* sh_rest, int n, long long num_instances,
                  const gs3d_settings* settings, void* prim_buf, size_t prim_bytes_, void* tile_buf,
                  size_t tile_bytes_, void* inst_buf, size_t inst_bytes_, void* bucket_buf, size_t bucket_bytes_,
                  long long bucket_capacity, void* workspace, size_t workspace_bytes, float* grad_means,
                  float* grad_scales, float* grad_rotations, float* grad_opacities, float* grad_sh0,
                  float* grad_sh_rest, float* densification_info, int densification_rows, void* stream) {
    SPLAT_TRY(gs3d_backward_blend(grad_image, image, n, num_instances, settings, prim_buf, prim_bytes_, tile_buf,
                                  tile_bytes_, inst_buf, inst_bytes_, bucket_buf, bucket_bytes_, bucket_capacity,
                                  workspace, workspace_bytes, densification_rows, stream));
    return gs3d_backward_preprocess(means, scales, rotations, opacities, sh_rest, n, settings, prim_buf,
                                    prim_bytes_, workspace, workspace_bytes, grad_means, grad_scales, grad_rotations,
                                    grad_opacities, grad_sh0, grad_sh_rest, densification_info, densification_rows,
                                    stream);
}

}  // extern "C"
