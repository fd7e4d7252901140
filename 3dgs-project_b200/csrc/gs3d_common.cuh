// gs3d_common.cuh - the 3DGS rasterization rules and buffer layouts shared by the forward and
// backward kernels.
//
// The rules are this library's restatement of Faster-GS's (nerficg-project/faster-gaussian-splatting
// @ c60ea26, not vendored in the reference; its blend rules are visible in
// phase1/fastergs_macro.patch:174-211 and upstream/upstream_main_kernels.patch:9-13,100-103):
//   * camera: x_c = w2c[:3,:3] p + w2c[:3,3]; visible if near <= z <= far
//   * Sigma3 = R S S^T R^T (R from the normalised quaternion (w, x, y, z), S = diag(exp(scales)))
//   * EWA: Sigma2 = J W Sigma3 W^T J^T with J the projection Jacobian at the clamped
//     x/z in [-1.3 cx/fx, 1.3 (W-cx)/fx] (and likewise y), low-pass dilation +0.3 on the diagonal;
//     proper antialiasing scales opacity by sqrt(det(Sigma2) / det(Sigma2 + 0.3 I))
//   * mean2d = (fx x/z + cx, fy y/z + cy) in pixel units, pixel (i, j) has its centre at (i+0.5, j+0.5)
//   * colour = real SH of degree <= 3 in the view direction (p - cam_position) / |.|, + 0.5; the
//     blend uses max(colour, 0) and the gradient passes where colour >= 0
//   * opacity = sigmoid(logit); a Gaussian with opacity < 1/255 can never reach the alpha cut-off
//   * blend: G = exp2(min(q2, 0)) with q2 = log2(e) * (-0.5 d^T conic d), d = mean2d - centre;
//     alpha = opacity G; skipped if alpha < 1/255; C += T alpha c; T *= 1 - alpha; the pixel
//     stops after the splat that drops T below 1e-4; image = C + T bg
//   * a Gaussian is listed in a 16x16 tile iff the ellipse alpha >= 1/255 (q <= 2 ln(255 opacity))
//     meets the tile's pixel-centre rectangle (closed-form x-extent per tile row, below)
//   * tile lists are ordered by the 64-bit key (tile << 32 | float bits of z), ties by Gaussian index
#pragma once

#include "common.cuh"
#include "sort.cuh"

namespace splat {
namespace gs3d {

constexpr int kTile = 16;
constexpr int kTilePixels = kTile * kTile;
constexpr int kBucket = 32;
constexpr float kAlphaMin = 1.0f / 255.0f;
constexpr float kTMin = 1e-4f;
constexpr float kOneMinusAlphaEps = 1e-6f;
constexpr float kDilation = 0.3f;
constexpr float kLog2e = 1.4426950408889634f;
constexpr float kCullMargin = 0.01f;  // log-domain margin of the per-warp culling rectangle

// Real spherical-harmonics constants (degrees 0-3), the published values used by 3DGS.
constexpr float kSH0 = 0.28209479177387814f;
constexpr float kSH1 = 0.4886025119029199f;
constexpr float kSH2_0 = 1.0925484305920792f;
constexpr float kSH2_1 = -1.0925484305920792f;
constexpr float kSH2_2 = 0.31539156525252005f;
constexpr float kSH2_3 = -1.0925484305920792f;
constexpr float kSH2_4 = 0.5462742152960396f;
constexpr float kSH3_0 = -0.5900435899266435f;
constexpr float kSH3_1 = 2.890611442640554f;
constexpr float kSH3_2 = -0.4570457994644658f;
constexpr float kSH3_3 = 0.3731763325901154f;
constexpr float kSH3_4 = -0.4570457994644658f;
constexpr float kSH3_5 = 1.445305721320277f;
constexpr float kSH3_6 = -0.5900435899266435f;

// Camera and image, passed by value to every kernel.
struct Cam {
    float fx, fy, cx, cy, near_plane, far_plane;
    int width, height, tiles_x, tiles_y;
    int active_sh_bases;  // 1, 4, 9 or 16
    int rest_bases;       // coefficients per Gaussian in sh_rest (15 for degree 3)
    int proper_aa;
};

// ---------------------------------------------------------------------------------------------
// Per-Gaussian ("primitive") buffer, sized by N
// ---------------------------------------------------------------------------------------------
constexpr int kCounters = 8;  // the primitive buffer's device counters

struct PrimBuffers {
    float2* mean2d;        // pixel units
    float4* conic_o;       // (A, B, C, opacity); power = -0.5 (A dx^2 + 2B dx dy + C dy^2)
    float4* color_z;       // (r, g, b) unclamped SH colour, w = camera depth z
    ushort4* rect;         // culling rectangle in pixels (x0, y0, x1, y1), inclusive, with margin
    float* thr;            // ln(255 opacity): the ellipse q <= 2 thr holds every alpha >= 1/255
    uint32_t* n_touched;   // listed tiles (0 = not visible)
    uint32_t* depth_key;   // float bits of z (visible), 0xffffffff (not visible)
    uint32_t* ids;         // 0..N-1
    uint32_t* depth_key_sorted;
    uint32_t* order;       // Gaussian ids in (depth, id) order: the depth passes of the 64-bit key sort
    uint32_t* offsets;     // exclusive prefix of n_touched, in that order
    uint32_t* counters;    // [0] = instance count M (offsets scan), [1] = bucket count B, [2] = buckets the
                           // backward replays, [3] = M (k_count_instances, read by the host)
    void* scan_ws;
    size_t scan_bytes;
    void* sort_ws;
    size_t sort_bytes;
};

// Per-tile and per-pixel buffer, sized by the image
struct TileBuffers {
    uint2* ranges;          // [T] (start, end) into the instance list
    uint32_t* nb;           // [T + 1] buckets per tile
    uint32_t* bstart;       // [T + 1] first bucket of each tile (exclusive prefix of nb)
    uint32_t* max_contrib;  // [T] max over the tile's pixels of n_contrib
    float* final_T;         // [H * W]
    uint32_t* n_contrib;    // [H * W] list position of the last contributor + 1
    uint32_t* lb;           // [T + 1] first sorted-list position whose tile key is >= t (scratch)
};

// Per-instance buffer, sized by M. Instances are written in depth order, so a stable sort on the tile
// alone finishes the LSD sort of the 64-bit (tile << 32 | depth) keys.
struct InstBuffers {
    uint32_t* keys;         // tile index, generation (depth) order
    uint32_t* vals;         // Gaussian id
    uint32_t* keys_sorted;  // tile index, final order
    uint32_t* point_list;   // sorted Gaussian ids
    void* sort_ws;
    size_t sort_bytes;
};

// Per-bucket buffer, sized by the bucket bound floor((M + 31 T) / 32) + 1
struct BucketBuffers {
    uint32_t* tile;     // [B] tile of each bucket
    uint32_t* reached;  // [B] the buckets before their tile's last contributor, in no set order (count: counters[2])
    float4* ckpt;       // [B * 256] (C.r, C.g, C.b, T) at the bucket start, per tile pixel
};

inline long long bucket_bound(long long m, int T) { return (m + 31ll * T) / 32 + 1; }

// Validates the settings and fills the kernel-side camera (gs3d_forward.cu).
int fill_cam(const gs3d_settings* s, Cam& cam);

inline PrimBuffers carve_prim(Carver& c, int n) {
    PrimBuffers b;
    const size_t nn = static_cast<size_t>(n < 1 ? 1 : n);
    b.mean2d = c.take<float2>(nn);
    b.conic_o = c.take<float4>(nn);
    b.color_z = c.take<float4>(nn);
    b.rect = c.take<ushort4>(nn);
    b.thr = c.take<float>(nn);
    b.n_touched = c.take<uint32_t>(nn);
    b.depth_key = c.take<uint32_t>(nn);
    b.ids = c.take<uint32_t>(nn);
    b.depth_key_sorted = c.take<uint32_t>(nn);
    b.order = c.take<uint32_t>(nn);
    b.offsets = c.take<uint32_t>(nn);
    b.counters = c.take<uint32_t>(kCounters);
    b.scan_bytes = scan_workspace_bytes(static_cast<long long>(nn));
    b.scan_ws = c.take<unsigned char>(b.scan_bytes);
    b.sort_bytes = sort_workspace_bytes<uint32_t>(static_cast<long long>(nn));
    b.sort_ws = c.take<unsigned char>(b.sort_bytes);
    return b;
}

inline TileBuffers carve_tile(Carver& c, int W, int H) {
    const int T = ((W + kTile - 1) / kTile) * ((H + kTile - 1) / kTile);
    TileBuffers b;
    b.ranges = c.take<uint2>(T);
    b.nb = c.take<uint32_t>(T + 1);
    b.bstart = c.take<uint32_t>(T + 1);
    b.max_contrib = c.take<uint32_t>(T);
    b.final_T = c.take<float>(static_cast<size_t>(W) * H);
    b.n_contrib = c.take<uint32_t>(static_cast<size_t>(W) * H);
    b.lb = c.take<uint32_t>(T + 1);
    return b;
}

inline InstBuffers carve_inst(Carver& c, long long m) {
    const size_t mm = static_cast<size_t>(m < 1 ? 1 : m);
    InstBuffers b;
    b.keys = c.take<uint32_t>(mm);
    b.vals = c.take<uint32_t>(mm);
    b.keys_sorted = c.take<uint32_t>(mm);
    b.point_list = c.take<uint32_t>(mm);
    b.sort_bytes = sort_workspace_bytes<uint32_t>(static_cast<long long>(mm));
    b.sort_ws = c.take<unsigned char>(b.sort_bytes);
    return b;
}

inline BucketBuffers carve_bucket(Carver& c, long long bcap) {
    BucketBuffers b;
    b.tile = c.take<uint32_t>(static_cast<size_t>(bcap < 1 ? 1 : bcap));
    b.reached = c.take<uint32_t>(static_cast<size_t>(bcap < 1 ? 1 : bcap));
    b.ckpt = c.take<float4>(static_cast<size_t>(bcap < 1 ? 1 : bcap) * kTilePixels);
    return b;
}

inline size_t prim_bytes(int n) {
    Carver c(nullptr, 0);
    carve_prim(c, n);
    return c.used + 256;
}
inline size_t tile_bytes(int W, int H) {
    Carver c(nullptr, 0);
    carve_tile(c, W, H);
    return c.used + 256;
}
inline size_t inst_bytes(long long m) {
    Carver c(nullptr, 0);
    carve_inst(c, m);
    return c.used + 256;
}
inline size_t bucket_bytes(long long bcap) {
    Carver c(nullptr, 0);
    carve_bucket(c, bcap);
    return c.used + 256;
}

// ---------------------------------------------------------------------------------------------
// Device math
// ---------------------------------------------------------------------------------------------
struct Mat3 {
    float m[3][3];
};

// Rotation of the normalised quaternion q = (w, x, y, z); returns |q|^2 for the backward.
__device__ __forceinline__ Mat3 quat_to_rot(float4 q, float& norm_sq) {
    norm_sq = q.x * q.x + q.y * q.y + q.z * q.z + q.w * q.w;
    const float inv = rsqrtf(fmaxf(norm_sq, 1e-30f));
    const float w = q.x * inv, x = q.y * inv, y = q.z * inv, z = q.w * inv;
    Mat3 R;
    R.m[0][0] = 1.f - 2.f * (y * y + z * z);
    R.m[0][1] = 2.f * (x * y - w * z);
    R.m[0][2] = 2.f * (x * z + w * y);
    R.m[1][0] = 2.f * (x * y + w * z);
    R.m[1][1] = 1.f - 2.f * (x * x + z * z);
    R.m[1][2] = 2.f * (y * z - w * x);
    R.m[2][0] = 2.f * (x * z - w * y);
    R.m[2][1] = 2.f * (y * z + w * x);
    R.m[2][2] = 1.f - 2.f * (x * x + y * y);
    return R;
}

// SH basis values b[0..15] (b[0] = SH0) for the unit direction (x, y, z).
__device__ __forceinline__ void sh_basis(float x, float y, float z, int bases, float* b) {
    b[0] = kSH0;
    if (bases > 1) {
        b[1] = -kSH1 * y;
        b[2] = kSH1 * z;
        b[3] = -kSH1 * x;
    }
    if (bases > 4) {
        const float xx = x * x, yy = y * y, zz = z * z;
        b[4] = kSH2_0 * x * y;
        b[5] = kSH2_1 * y * z;
        b[6] = kSH2_2 * (2.f * zz - xx - yy);
        b[7] = kSH2_3 * x * z;
        b[8] = kSH2_4 * (xx - yy);
        if (bases > 9) {
            b[9] = kSH3_0 * y * (3.f * xx - yy);
            b[10] = kSH3_1 * x * y * z;
            b[11] = kSH3_2 * y * (4.f * zz - xx - yy);
            b[12] = kSH3_3 * z * (2.f * zz - 3.f * xx - 3.f * yy);
            b[13] = kSH3_4 * x * (4.f * zz - xx - yy);
            b[14] = kSH3_5 * z * (xx - yy);
            b[15] = kSH3_6 * x * (xx - 3.f * yy);
        }
    }
}

// sh_basis with every operation rounded on its own (no contraction into fused multiply-adds), so that the basis of
// a direction has the same bits in every kernel that evaluates it: the preprocess backward forms the SH gradients
// basis_k(d) * dL/dcolour from it, and the compact exchange (dp_adam.cu) forms the same products again from the
// direction and the colour gradient that a rank sends in their place.
__device__ __forceinline__ void sh_basis_rn(float x, float y, float z, int bases, float* b) {
    b[0] = kSH0;
    if (bases > 1) {
        b[1] = __fmul_rn(-kSH1, y);
        b[2] = __fmul_rn(kSH1, z);
        b[3] = __fmul_rn(-kSH1, x);
    }
    if (bases > 4) {
        const float xx = __fmul_rn(x, x), yy = __fmul_rn(y, y), zz = __fmul_rn(z, z);
        b[4] = __fmul_rn(__fmul_rn(kSH2_0, x), y);
        b[5] = __fmul_rn(__fmul_rn(kSH2_1, y), z);
        b[6] = __fmul_rn(kSH2_2, __fsub_rn(__fsub_rn(__fmul_rn(2.f, zz), xx), yy));
        b[7] = __fmul_rn(__fmul_rn(kSH2_3, x), z);
        b[8] = __fmul_rn(kSH2_4, __fsub_rn(xx, yy));
        if (bases > 9) {
            const float t4 = __fsub_rn(__fsub_rn(__fmul_rn(4.f, zz), xx), yy);
            b[9] = __fmul_rn(__fmul_rn(kSH3_0, y), __fsub_rn(__fmul_rn(3.f, xx), yy));
            b[10] = __fmul_rn(__fmul_rn(__fmul_rn(kSH3_1, x), y), z);
            b[11] = __fmul_rn(__fmul_rn(kSH3_2, y), t4);
            b[12] = __fmul_rn(__fmul_rn(kSH3_3, z),
                              __fsub_rn(__fsub_rn(__fmul_rn(2.f, zz), __fmul_rn(3.f, xx)), __fmul_rn(3.f, yy)));
            b[13] = __fmul_rn(__fmul_rn(kSH3_4, x), t4);
            b[14] = __fmul_rn(__fmul_rn(kSH3_5, z), __fsub_rn(xx, yy));
            b[15] = __fmul_rn(__fmul_rn(kSH3_6, x), __fsub_rn(xx, __fmul_rn(3.f, yy)));
        }
    }
}

// ---------------------------------------------------------------------------------------------
// Blend evaluation shared by the forward and the backward, with explicit fused multiply-adds so both
// kernels take the same alpha >= 1/255 decisions bit for bit. (a2, b2, c2) is the conic scaled by
// log2(e) (-0.5 A, -B, -0.5 C), so q2 = log2(e) * power and G = 2^min(q2, 0). The hardware ex2 is used:
// below 2^-126 it flushes to 0, where alpha is far under the 1/255 cut-off anyway.
// ---------------------------------------------------------------------------------------------
__device__ __forceinline__ float hw_exp2(float x) {
    float y;
    asm("ex2.approx.ftz.f32 %0, %1;" : "=f"(y) : "f"(x));
    return y;
}

// ---- warp staging of a contiguous block of SH-rest rows in shared memory ----
// The warp's rows [first, first + 32) are one contiguous block of nfl floats. stage_sh_begin starts 16-byte
// asynchronous copies (cp.async, L1 bypassed) of its aligned part, so other loads and arithmetic overlap them;
// stage_sh_end loads the unaligned remainder, waits for the copies and synchronises the warp. Both must be
// called by all 32 lanes.
__device__ __forceinline__ int stage_sh_begin(float* sh, const float* src, int nfl, int lane) {
    int done = 0;
    if ((reinterpret_cast<uintptr_t>(src) & 15u) == 0) {
        const int n4 = nfl / 4;
        for (int k = lane; k < n4; k += 32) {
            const unsigned dst = static_cast<unsigned>(__cvta_generic_to_shared(sh + 4 * k));
            asm volatile("cp.async.cg.shared.global [%0], [%1], 16;\n" ::"r"(dst), "l"(src + 4 * k) : "memory");
        }
        done = n4 * 4;
    }
    asm volatile("cp.async.commit_group;\n" ::: "memory");
    return done;
}

__device__ __forceinline__ void stage_sh_end(float* sh, const float* src, int nfl, int done, int lane) {
    for (int k = done + lane; k < nfl; k += 32) sh[k] = __ldg(src + k);
    asm volatile("cp.async.wait_group 0;\n" ::: "memory");
    __syncwarp();
}

__device__ __forceinline__ float blend_q2(float a2, float b2, float c2, float dx, float dy) {
    return __fmaf_rn(dx, __fmaf_rn(a2, dx, __fmul_rn(b2, dy)), __fmul_rn(c2, __fmul_rn(dy, dy)));
}

// ---------------------------------------------------------------------------------------------
// Listing test: which tiles the ellipse q = A dx^2 + 2B dx dy + C dy^2 <= R = 2 thr (every pixel
// with alpha >= 1/255) reaches, each tile taken as the continuous rectangle of its pixel centres.
// Per tile row, the ellipse's x-extent over the row band is found in closed form (the rightmost /
// leftmost point on the band: x(dy) = (-B dy +- sqrt(A R - D dy^2)) / A is concave / convex, so its
// extreme on the band is at the clamped stationary dy = -+B sqrt(R / (D C)), D = AC - B^2), and the
// tiles whose centre range meets that interval are listed. Every operation is rounded on its own
// (no fused multiply-add), so the count pass, the write pass and the numpy oracle agree bit for bit.
// ---------------------------------------------------------------------------------------------
struct Ellipse {
    float mx, my, A, B, R, D, ey, s, inv_a;
};

// Reciprocals are taken once per Gaussian (correctly rounded), the per-row work is products, sums and two
// square roots; divisions by 16 are products by 1/16 (exact).
__device__ __forceinline__ Ellipse make_ellipse(float mx, float my, float A, float B, float C, float thr) {
    Ellipse e;
    e.mx = mx;
    e.my = my;
    e.A = A;
    e.B = B;
    e.R = __fmul_rn(2.f, thr);
    e.D = __fsub_rn(__fmul_rn(A, C), __fmul_rn(B, B));
    const float inv_d = __frcp_rn(e.D);
    e.ey = __fsqrt_rn(__fmul_rn(__fmul_rn(A, e.R), inv_d));
    e.s = __fsqrt_rn(__fmul_rn(__fmul_rn(e.R, inv_d), __frcp_rn(C)));
    e.inv_a = __frcp_rn(A);
    return e;
}

// First and last tile row the ellipse can reach (empty when lo > hi).
__device__ __forceinline__ int2 ellipse_rows(const Ellipse& e, int H, int tiles_y) {
    const float top = __fsub_rn(e.my, e.ey), bot = __fadd_rn(e.my, e.ey);
    if (!(bot >= 0.5f && top <= static_cast<float>(H) - 0.5f)) return make_int2(1, 0);
    const int lo = max(static_cast<int>(ceilf(__fmul_rn(__fsub_rn(top, 15.5f), 0.0625f))), 0);
    const int hi = min(static_cast<int>(floorf(__fmul_rn(__fsub_rn(bot, 0.5f), 0.0625f))), tiles_y - 1);
    return make_int2(lo, hi);
}

__device__ __forceinline__ float ellipse_x(const Ellipse& e, float dy, float sign) {
    const float disc = fmaxf(__fsub_rn(__fmul_rn(e.A, e.R), __fmul_rn(__fmul_rn(e.D, dy), dy)), 0.f);
    return __fmul_rn(__fadd_rn(__fmul_rn(-e.B, dy), __fmul_rn(sign, __fsqrt_rn(disc))), e.inv_a);
}

// Listed tiles [x, y] of tile row ty (empty when x > y).
__device__ __forceinline__ int2 ellipse_row_tiles(const Ellipse& e, int ty, int W, int H, int tiles_x) {
    const float y0 = static_cast<float>(ty * kTile) + 0.5f;
    const float y1 = static_cast<float>(min(ty * kTile + kTile, H)) - 0.5f;
    const float lo = fmaxf(__fsub_rn(y0, e.my), -e.ey), hi = fminf(__fsub_rn(y1, e.my), e.ey);
    if (!(lo <= hi)) return make_int2(1, 0);
    const float dyr = fminf(fmaxf(__fmul_rn(-e.B, e.s), lo), hi);
    const float dyl = fminf(fmaxf(__fmul_rn(e.B, e.s), lo), hi);
    const float xr = __fadd_rn(e.mx, ellipse_x(e, dyr, 1.f));
    const float xl = __fadd_rn(e.mx, ellipse_x(e, dyl, -1.f));
    if (!(xr >= 0.5f && xl <= static_cast<float>(W) - 0.5f)) return make_int2(1, 0);
    const int tlo = max(static_cast<int>(ceilf(__fmul_rn(__fsub_rn(xl, 15.5f), 0.0625f))), 0);
    const int thi = min(static_cast<int>(floorf(__fmul_rn(__fsub_rn(xr, 0.5f), 0.0625f))), tiles_x - 1);
    return make_int2(tlo, thi);
}

}  // namespace gs3d
}  // namespace splat
