// gs3d_oracle.cpp - CPU restatement of the 3DGS training step (TEST INFRASTRUCTURE: the tests, smoke()
// and bench.py's CPU baseline use it; the product never links it).
//
// The rules are those listed in 3dgs-project_b200/csrc/gs3d_common.cuh (this library's restatement of
// Faster-GS @ c60ea26, whose blend rules phase1/fastergs_macro.patch:174-211 shows; Faster-GS is not vendored
// in the reference, so this path's parity is UNPINNED - no reference output exists to check it against):
//   preprocess      float32 EWA projection, +0.3 dilation, optional antialiasing factor, sigmoid opacity,
//                   degree <= 3 real SH + 0.5, culling rectangle, ln(255 opacity)
//   listing         per tile row, closed-form x-extent of the ellipse q <= 2 ln(255 opacity), every product
//                   and sum rounded separately (compile with -ffp-contract=off), so the tiles match the device
//   sort            std::stable_sort on (tile << 32 | order-preserving depth bits), ties by Gaussian id
//   blend           per pixel, front to back over its tile's list; alpha = o exp2(min(q2, 0)), skip < 1/255,
//                   stop after T < 1e-4; image = C + T bg. A pixel is flagged "near" when one of its decisions
//                   (alpha >= 1/255, T < 1e-4) lies within the error bound of two exp2 implementations (the
//                   device's hardware ex2 and the C library's exp2f); counts are compared on the others
//   blend backward  per pixel: the forward's splat set (its float alpha >= 1/255 decisions before the pixel's
//                   contributor count), then exact float64 values of the float inputs (exponent, G, alpha, T as
//                   the product of (1 - alpha)); back to front with T recovered by division (the 3DGS per-pixel
//                   scheme); gradients into mean2d / conic / opacity / colour accumulated in double
//   preprocess bwd  the analytic chain to means, scales, rotations, opacity logits, sh0, sh_rest
//   adam            the update of cluster/patches/fastergs_lean_adam.patch:112-117
// OpenMP parallelises over Gaussians and over tile rows; a row range [row0, row1) bounds the blend work so
// the timed CPU baseline can run a sample of the image.
#include <math.h>
#include <omp.h>
#include <stdint.h>
#include <string.h>

#include <xmmintrin.h>

#include <algorithm>
#include <cstdio>
#include <parallel/algorithm>
#include <numeric>
#include <vector>

namespace {

constexpr int kTile = 16;
constexpr float kAlphaMin = 1.0f / 255.0f;
constexpr float kTMin = 1e-4f;
constexpr float kDilation = 0.3f;
constexpr float kLog2e = 1.4426950408889634f;
constexpr float kCullMargin = 0.01f;
constexpr double kOneMinusAlphaEps = 1e-6;
// Relative difference allowed between two float exp2 evaluations of the same argument (a few ulp: the
// device's ex2.approx is within 2 ulp, the C library's exp2f within 1), times a safety factor of 4.
constexpr float kExp2Tol = 0x1p-19f;

const float SH0 = 0.28209479177387814f, SH1 = 0.4886025119029199f;
const float SH2[5] = {1.0925484305920792f, -1.0925484305920792f, 0.31539156525252005f, -1.0925484305920792f,
                      0.5462742152960396f};
const float SH3[7] = {-0.5900435899266435f, 2.890611442640554f, -0.4570457994644658f, 0.3731763325901154f,
                      -0.4570457994644658f, 1.445305721320277f, -0.5900435899266435f};

}  // namespace

extern "C" {

struct gs3o_settings {
    float w2c[16];
    float cam_position[3];
    float bg[3];
    int active_sh_bases, rest_bases, width, height;
    float fx, fy, cx, cy, near_plane, far_plane;
    int proper_antialiasing;
};

struct gs3o_ctx {
    int n = 0;
    gs3o_settings s;
    int tiles_x = 0, tiles_y = 0;
    // preprocess outputs
    std::vector<float> mean2d, conic_o, color_z, thr;
    std::vector<int> rect, n_touched;
    // listing
    std::vector<int64_t> point_list;
    std::vector<uint64_t> keys_sorted;
    std::vector<int64_t> ranges;
    // forward per pixel
    std::vector<float> image, final_T;
    std::vector<int> n_contrib;
    std::vector<unsigned char> near;  // 1 = a decision of this pixel is within exp2 rounding of its threshold
    // backward accumulators (double)
    std::vector<double> g_mean2d, g_conic_o, g_color;
};

}  // extern "C"

namespace {

void sh_basis(float x, float y, float z, int bases, float* b) {
    b[0] = SH0;
    if (bases > 1) {
        b[1] = -SH1 * y;
        b[2] = SH1 * z;
        b[3] = -SH1 * x;
    }
    if (bases > 4) {
        const float xx = x * x, yy = y * y, zz = z * z;
        b[4] = SH2[0] * x * y;
        b[5] = SH2[1] * y * z;
        b[6] = SH2[2] * (2.f * zz - xx - yy);
        b[7] = SH2[3] * x * z;
        b[8] = SH2[4] * (xx - yy);
        if (bases > 9) {
            b[9] = SH3[0] * y * (3.f * xx - yy);
            b[10] = SH3[1] * x * y * z;
            b[11] = SH3[2] * y * (4.f * zz - xx - yy);
            b[12] = SH3[3] * z * (2.f * zz - 3.f * xx - 3.f * yy);
            b[13] = SH3[4] * x * (4.f * zz - xx - yy);
            b[14] = SH3[5] * z * (xx - yy);
            b[15] = SH3[6] * x * (xx - 3.f * yy);
        }
    }
}

void quat_rot(const float* q, float R[3][3], float& nsq) {
    nsq = q[0] * q[0] + q[1] * q[1] + q[2] * q[2] + q[3] * q[3];
    const float inv = 1.f / sqrtf(std::max(nsq, 1e-30f));
    const float w = q[0] * inv, x = q[1] * inv, y = q[2] * inv, z = q[3] * inv;
    R[0][0] = 1.f - 2.f * (y * y + z * z);
    R[0][1] = 2.f * (x * y - w * z);
    R[0][2] = 2.f * (x * z + w * y);
    R[1][0] = 2.f * (x * y + w * z);
    R[1][1] = 1.f - 2.f * (x * x + z * z);
    R[1][2] = 2.f * (y * z - w * x);
    R[2][0] = 2.f * (x * z - w * y);
    R[2][1] = 2.f * (y * z + w * x);
    R[2][2] = 1.f - 2.f * (x * x + y * y);
}

// Listing test (every operation rounded on its own; the file is built with -ffp-contract=off).
struct Ell {
    float mx, my, A, B, R, D, ey, s, inv_a;
};

Ell make_ell(float mx, float my, float A, float B, float C, float thr) {
    Ell e;
    e.mx = mx;
    e.my = my;
    e.A = A;
    e.B = B;
    e.R = 2.f * thr;
    e.D = A * C - B * B;
    const float inv_d = 1.f / e.D;
    e.ey = sqrtf((A * e.R) * inv_d);
    e.s = sqrtf((e.R * inv_d) * (1.f / C));
    e.inv_a = 1.f / A;
    return e;
}

void ell_rows(const Ell& e, int H, int tiles_y, int& lo, int& hi) {
    const float top = e.my - e.ey, bot = e.my + e.ey;
    if (!(bot >= 0.5f && top <= static_cast<float>(H) - 0.5f)) {
        lo = 1;
        hi = 0;
        return;
    }
    lo = std::max(static_cast<int>(std::max(ceilf((top - 15.5f) * 0.0625f), -1.f)), 0);
    hi = std::min(static_cast<int>(std::min(floorf((bot - 0.5f) * 0.0625f), static_cast<float>(tiles_y))),
                  tiles_y - 1);
}

float ell_x(const Ell& e, float dy, float sign) {
    const float disc = std::max(e.A * e.R - (e.D * dy) * dy, 0.f);
    return ((-e.B) * dy + sign * sqrtf(disc)) * e.inv_a;
}

void ell_row_tiles(const Ell& e, int ty, int W, int H, int tiles_x, int& tlo, int& thi) {
    const float y0 = static_cast<float>(ty * kTile) + 0.5f;
    const float y1 = static_cast<float>(std::min(ty * kTile + kTile, H)) - 0.5f;
    const float lo = std::max(y0 - e.my, -e.ey), hi = std::min(y1 - e.my, e.ey);
    tlo = 1;
    thi = 0;
    if (!(lo <= hi)) return;
    const float dyr = std::min(std::max((-e.B) * e.s, lo), hi);
    const float dyl = std::min(std::max(e.B * e.s, lo), hi);
    const float xr = e.mx + ell_x(e, dyr, 1.f);
    const float xl = e.mx + ell_x(e, dyl, -1.f);
    if (!(xr >= 0.5f && xl <= static_cast<float>(W) - 0.5f)) return;
    tlo = std::max(static_cast<int>(std::max(ceilf((xl - 15.5f) * 0.0625f), -1.f)), 0);
    thi = std::min(static_cast<int>(std::min(floorf((xr - 0.5f) * 0.0625f), static_cast<float>(tiles_x))),
                   tiles_x - 1);
}

uint32_t depth_order_key(float z) {
    uint32_t b;
    memcpy(&b, &z, 4);
    return (b & 0x80000000u) ? ~b : (b | 0x80000000u);
}

}  // namespace

extern "C" {

gs3o_ctx* gs3o_create(void) { return new gs3o_ctx(); }
void gs3o_destroy(gs3o_ctx* c) { delete c; }
int gs3o_threads(void) { return omp_get_max_threads(); }
void gs3o_set_threads(int t) { omp_set_num_threads(t > 0 ? t : 1); }

void gs3o_preprocess(gs3o_ctx* c, const float* means, const float* scales, const float* rotations,
                     const float* opacities, const float* sh0, const float* sh_rest, int n, const gs3o_settings* s) {
    c->n = n;
    c->s = *s;
    c->tiles_x = (s->width + kTile - 1) / kTile;
    c->tiles_y = (s->height + kTile - 1) / kTile;
    c->mean2d.assign(2 * (size_t)n, 0.f);
    c->conic_o.assign(4 * (size_t)n, 0.f);
    c->color_z.assign(4 * (size_t)n, 0.f);
    c->thr.assign(n, 0.f);
    c->rect.assign(4 * (size_t)n, 0);
    c->n_touched.assign(n, 0);
    const float* w = s->w2c;
    const int rest3 = 3 * s->rest_bases;
#pragma omp parallel for schedule(static)
    for (int i = 0; i < n; ++i) {
        const float px = means[3 * i], py = means[3 * i + 1], pz = means[3 * i + 2];
        const float xc = w[0] * px + w[1] * py + w[2] * pz + w[3];
        const float yc = w[4] * px + w[5] * py + w[6] * pz + w[7];
        const float zc = w[8] * px + w[9] * py + w[10] * pz + w[11];
        if (!(zc >= s->near_plane && zc <= s->far_plane)) continue;
        float R[3][3], nsq;
        quat_rot(rotations + 4 * i, R, nsq);
        const float sc[3] = {expf(scales[3 * i]), expf(scales[3 * i + 1]), expf(scales[3 * i + 2])};
        float M[3][3], S3[3][3], T1[3][3], Sc[3][3];
        for (int r = 0; r < 3; ++r)
            for (int k = 0; k < 3; ++k) M[r][k] = R[r][k] * sc[k];
        for (int r = 0; r < 3; ++r)
            for (int k = 0; k < 3; ++k) S3[r][k] = M[r][0] * M[k][0] + M[r][1] * M[k][1] + M[r][2] * M[k][2];
        for (int r = 0; r < 3; ++r)
            for (int k = 0; k < 3; ++k) T1[r][k] = w[4 * r] * S3[0][k] + w[4 * r + 1] * S3[1][k] + w[4 * r + 2] * S3[2][k];
        for (int r = 0; r < 3; ++r)
            for (int k = 0; k < 3; ++k) Sc[r][k] = T1[r][0] * w[4 * k] + T1[r][1] * w[4 * k + 1] + T1[r][2] * w[4 * k + 2];
        const float inv_z = 1.f / zc;
        const float tx = std::min(std::max(xc * inv_z, -1.3f * s->cx / s->fx), 1.3f * (s->width - s->cx) / s->fx);
        const float ty = std::min(std::max(yc * inv_z, -1.3f * s->cy / s->fy), 1.3f * (s->height - s->cy) / s->fy);
        const float j00 = s->fx * inv_z, j02 = -s->fx * tx * inv_z, j11 = s->fy * inv_z, j12 = -s->fy * ty * inv_z;
        const float a = j00 * (j00 * Sc[0][0] + j02 * Sc[0][2]) + j02 * (j00 * Sc[2][0] + j02 * Sc[2][2]);
        const float b = j00 * (j11 * Sc[0][1] + j12 * Sc[0][2]) + j02 * (j11 * Sc[2][1] + j12 * Sc[2][2]);
        const float cc = j11 * (j11 * Sc[1][1] + j12 * Sc[1][2]) + j12 * (j11 * Sc[2][1] + j12 * Sc[2][2]);
        const float ad = a + kDilation, cd = cc + kDilation;
        const float det = ad * cd - b * b;
        float o = 1.f / (1.f + expf(-opacities[i]));
        if (s->proper_antialiasing) o *= sqrtf(std::max((a * cc - b * b) / det, 0.f));
        const float mx = s->fx * xc * inv_z + s->cx, my = s->fy * yc * inv_z + s->cy;
        if (!(det > 0.f && o * 255.f >= 1.f && std::isfinite(mx) && std::isfinite(my))) continue;
        const float inv_det = 1.f / det;
        const float A = cd * inv_det, B = -b * inv_det, C = ad * inv_det;
        const float th = logf(255.f * o);
        const float r2 = 2.f * (th + kCullMargin);
        const float ex = sqrtf(r2 * ad), ey = sqrtf(r2 * cd);
        const float fx0 = ceilf(mx - ex - 0.5f) - 1.f, fx1 = floorf(mx + ex - 0.5f) + 1.f;
        const float fy0 = ceilf(my - ey - 0.5f) - 1.f, fy1 = floorf(my + ey - 0.5f) + 1.f;
        if (!(fx1 >= 0.f && fy1 >= 0.f && fx0 <= s->width - 1 && fy0 <= s->height - 1)) continue;
        const Ell e = make_ell(mx, my, A, B, C, th);
        int lo, hi, touched = 0;
        ell_rows(e, s->height, c->tiles_y, lo, hi);
        for (int r = lo; r <= hi; ++r) {
            int tlo, thi;
            ell_row_tiles(e, r, s->width, s->height, c->tiles_x, tlo, thi);
            touched += std::max(thi - tlo + 1, 0);
        }
        if (touched == 0) continue;
        float dx = px - s->cam_position[0], dy = py - s->cam_position[1], dz = pz - s->cam_position[2];
        const float inv_len = 1.f / sqrtf(dx * dx + dy * dy + dz * dz);
        dx *= inv_len;
        dy *= inv_len;
        dz *= inv_len;
        float bas[16];
        sh_basis(dx, dy, dz, s->active_sh_bases, bas);
        float col[3];
        for (int ch = 0; ch < 3; ++ch) {
            float v = bas[0] * sh0[3 * i + ch] + 0.5f;
            for (int k = 1; k < s->active_sh_bases && k <= s->rest_bases; ++k) v += bas[k] * sh_rest[(size_t)i * rest3 + 3 * (k - 1) + ch];
            col[ch] = v;
        }
        c->mean2d[2 * i] = mx;
        c->mean2d[2 * i + 1] = my;
        c->conic_o[4 * i] = A;
        c->conic_o[4 * i + 1] = B;
        c->conic_o[4 * i + 2] = C;
        c->conic_o[4 * i + 3] = o;
        c->color_z[4 * i] = col[0];
        c->color_z[4 * i + 1] = col[1];
        c->color_z[4 * i + 2] = col[2];
        c->color_z[4 * i + 3] = zc;
        c->thr[i] = th;
        c->rect[4 * i] = (int)std::max(fx0, 0.f);
        c->rect[4 * i + 1] = (int)std::max(fy0, 0.f);
        c->rect[4 * i + 2] = (int)std::min(fx1, (float)(s->width - 1));
        c->rect[4 * i + 3] = (int)std::min(fy1, (float)(s->height - 1));
        c->n_touched[i] = touched;
    }
}

// Replace the preprocess outputs (e.g. with a device's own) before binning.
void gs3o_set_primitives(gs3o_ctx* c, const float* mean2d, const float* conic_o, const float* color_z,
                         const float* thr, const int* n_touched) {
    const size_t n = c->n;
    memcpy(c->mean2d.data(), mean2d, 8 * n);
    memcpy(c->conic_o.data(), conic_o, 16 * n);
    memcpy(c->color_z.data(), color_z, 16 * n);
    memcpy(c->thr.data(), thr, 4 * n);
    memcpy(c->n_touched.data(), n_touched, 4 * n);
}

long long gs3o_bin(gs3o_ctx* c) {
    const int n = c->n, W = c->s.width, H = c->s.height, T = c->tiles_x * c->tiles_y;
    std::vector<long long> off(n + 1, 0);
    for (int i = 0; i < n; ++i) off[i + 1] = off[i] + c->n_touched[i];
    const long long m = off[n];
    std::vector<uint64_t> keys(m);
    std::vector<int64_t> ids(m);
#pragma omp parallel for schedule(dynamic, 1024)
    for (int i = 0; i < n; ++i) {
        if (c->n_touched[i] == 0) continue;
        const Ell e = make_ell(c->mean2d[2 * i], c->mean2d[2 * i + 1], c->conic_o[4 * i], c->conic_o[4 * i + 1],
                               c->conic_o[4 * i + 2], c->thr[i]);
        const uint64_t zk = depth_order_key(c->color_z[4 * i + 3]);
        int lo, hi;
        ell_rows(e, H, c->tiles_y, lo, hi);
        long long k = off[i];
        for (int r = lo; r <= hi; ++r) {
            int tlo, thi;
            ell_row_tiles(e, r, W, H, c->tiles_x, tlo, thi);
            for (int t = tlo; t <= thi && k < off[i + 1]; ++t, ++k) {
                keys[k] = ((uint64_t)(r * c->tiles_x + t) << 32) | zk;
                ids[k] = i;
            }
        }
        for (; k < off[i + 1]; ++k) {
            keys[k] = (uint64_t)T << 32;
            ids[k] = i;
        }
    }
    std::vector<int64_t> perm(m);
    std::iota(perm.begin(), perm.end(), 0);
    __gnu_parallel::stable_sort(perm.begin(), perm.end(), [&](int64_t a, int64_t b) { return keys[a] < keys[b]; });
    c->point_list.resize(m);
    c->keys_sorted.resize(m);
    for (long long k = 0; k < m; ++k) {
        c->point_list[k] = ids[perm[k]];
        c->keys_sorted[k] = keys[perm[k]];
    }
    c->ranges.assign(2 * (size_t)T, 0);
    for (long long k = 0; k < m; ++k) {
        const uint64_t t = c->keys_sorted[k] >> 32;
        if (t >= (uint64_t)T) continue;
        if (k == 0 || (c->keys_sorted[k - 1] >> 32) != t) c->ranges[2 * t] = k;
        if (k == m - 1 || (c->keys_sorted[k + 1] >> 32) != t) c->ranges[2 * t + 1] = k + 1;
    }
    const size_t P = (size_t)W * H;
    c->image.assign(3 * P, 0.f);
    c->final_T.assign(P, 1.f);
    c->n_contrib.assign(P, 0);
    c->near.assign(P, 0);
    return m;
}

void gs3o_blend(gs3o_ctx* c, int row0, int row1) {
    const int W = c->s.width, H = c->s.height;
    const size_t P = (size_t)W * H;
    row0 = std::max(row0, 0);
    row1 = std::min(row1, c->tiles_y);
#pragma omp parallel for schedule(dynamic, 1)
    for (int t = row0 * c->tiles_x; t < row1 * c->tiles_x; ++t) {
        const int tx0 = (t % c->tiles_x) * kTile, ty0 = (t / c->tiles_x) * kTile;
        const int64_t s0 = c->ranges[2 * t], s1 = c->ranges[2 * t + 1];
        for (int y = ty0; y < std::min(ty0 + kTile, H); ++y)
            for (int x = tx0; x < std::min(tx0 + kTile, W); ++x) {
                const float pxf = x + 0.5f, pyf = y + 0.5f;
                float T = 1.f, C[3] = {0.f, 0.f, 0.f};
                int last = 0;
                unsigned char near = 0;
                double eT = 0.0;  // bound on the relative difference of T between two exp2 implementations
                for (int64_t k = s0; k < s1; ++k) {
                    const int64_t g = c->point_list[k];
                    const float* co = &c->conic_o[4 * g];
                    const float dx = c->mean2d[2 * g] - pxf, dy = c->mean2d[2 * g + 1] - pyf;
                    const float a2 = -0.5f * kLog2e * co[0], b2 = -kLog2e * co[1], c2 = -0.5f * kLog2e * co[2];
                    const float q2 = fmaf(dx, fmaf(a2, dx, b2 * dy), c2 * (dy * dy));  // the device's blend_q2
                    const float alpha = co[3] * exp2f(std::min(q2, 0.f));
                    if (fabsf(alpha - kAlphaMin) <= kExp2Tol * kAlphaMin) near = 1;
                    if (alpha < kAlphaMin) continue;
                    const float w = alpha * T;
                    for (int ch = 0; ch < 3; ++ch) C[ch] += w * std::max(c->color_z[4 * g + ch], 0.f);
                    T *= 1.f - alpha;
                    eT += (double)kExp2Tol * alpha / std::max(1.0 - alpha, 1e-30) + 0x1p-22;
                    last = (int)(k - s0 + 1);
                    if (fabs((double)T - kTMin) <= eT * kTMin) near = 1;
                    if (T < kTMin) break;
                }
                const size_t pix = (size_t)y * W + x;
                c->near[pix] = near;
                for (int ch = 0; ch < 3; ++ch) c->image[ch * P + pix] = C[ch] + T * c->s.bg[ch];
                c->final_T[pix] = T;
                c->n_contrib[pix] = last;
            }
    }
}

// Per-pixel backward over tile rows [row0, row1); accumulates into the double buffers (zeroed by
// gs3o_backward_reset).
void gs3o_backward_reset(gs3o_ctx* c) {
    c->g_mean2d.assign(2 * (size_t)c->n, 0.0);
    c->g_conic_o.assign(4 * (size_t)c->n, 0.0);
    c->g_color.assign(3 * (size_t)c->n, 0.0);
}

void gs3o_blend_backward(gs3o_ctx* c, const float* grad_image, int row0, int row1) {
    const int W = c->s.width, H = c->s.height;
    const size_t P = (size_t)W * H;
    row0 = std::max(row0, 0);
    row1 = std::min(row1, c->tiles_y);
#pragma omp parallel
    {
        std::vector<double> alpha_d, G_d;  // this thread's per-contributor values of one pixel
        std::vector<int64_t> ids;
#pragma omp for schedule(dynamic, 1)
        for (int t = row0 * c->tiles_x; t < row1 * c->tiles_x; ++t) {
            const int tx0 = (t % c->tiles_x) * kTile, ty0 = (t / c->tiles_x) * kTile;
            const int64_t s0 = c->ranges[2 * t];
            for (int y = ty0; y < std::min(ty0 + kTile, H); ++y)
                for (int x = tx0; x < std::min(tx0 + kTile, W); ++x) {
                    const size_t pix = (size_t)y * W + x;
                    const double Gr[3] = {grad_image[pix], grad_image[P + pix], grad_image[2 * P + pix]};
                    const float pxf = x + 0.5f, pyf = y + 0.5f;
                    // The forward's splat set: its float decisions (the same evaluation as the blend) over the
                    // positions before its contributor count. The values are then exact float64 functions of the
                    // float inputs: the exponent -0.5 d^T K d from the float conic and offsets, G = e^min(., 0),
                    // alpha = opacity G, and T as the product of (1 - alpha) in front.
                    alpha_d.clear();
                    G_d.clear();
                    ids.clear();
                    double T = 1.0;
                    for (int64_t k = s0; k < s0 + c->n_contrib[pix]; ++k) {
                        const int64_t g = c->point_list[k];
                        const float* co = &c->conic_o[4 * g];
                        const float dxf = c->mean2d[2 * g] - pxf, dyf = c->mean2d[2 * g + 1] - pyf;
                        const float a2 = -0.5f * kLog2e * co[0], b2 = -kLog2e * co[1], c2 = -0.5f * kLog2e * co[2];
                        const float q2 = fmaf(dxf, fmaf(a2, dxf, b2 * dyf), c2 * (dyf * dyf));
                        if (co[3] * exp2f(std::min(q2, 0.f)) < kAlphaMin) continue;
                        const double dx = (double)c->mean2d[2 * g] - (x + 0.5), dy = (double)c->mean2d[2 * g + 1] - (y + 0.5);
                        const double pw = -0.5 * ((double)co[0] * dx * dx + 2.0 * (double)co[1] * dx * dy +
                                                  (double)co[2] * dy * dy);
                        const double Gs = exp(std::min(pw, 0.0));
                        ids.push_back(g);
                        G_d.push_back(Gs);
                        alpha_d.push_back((double)co[3] * Gs);
                        T *= 1.0 - alpha_d.back();
                    }
                    double acc[3];  // colour behind the current splat, background included, / T
                    for (int ch = 0; ch < 3; ++ch) acc[ch] = c->s.bg[ch];
                    for (int64_t i = (int64_t)ids.size() - 1; i >= 0; --i) {
                        const int64_t g = ids[i];
                        const float* co = &c->conic_o[4 * g];
                        const double alpha = alpha_d[i], Gs = G_d[i];
                        const double om = std::max(1.0 - alpha, kOneMinusAlphaEps);
                        T = T / om;  // T before this splat
                        double col[3], dot = 0.0;
                        for (int ch = 0; ch < 3; ++ch) {
                            col[ch] = std::max(c->color_z[4 * g + ch], 0.f);
                            dot += Gr[ch] * (col[ch] - acc[ch]);
                        }
                        const double dL_dalpha = T * dot;
                        for (int ch = 0; ch < 3; ++ch) {
#pragma omp atomic
                            c->g_color[3 * g + ch] += Gr[ch] * alpha * T;
                            acc[ch] = alpha * col[ch] + (1.0 - alpha) * acc[ch];
                        }
                        const double dx = (double)c->mean2d[2 * g] - (x + 0.5), dy = (double)c->mean2d[2 * g + 1] - (y + 0.5);
                        const double h = alpha * dL_dalpha;  // dL/dpower (power = -0.5 d^T K d)
                        const double A = co[0], B = co[1], C = co[2];
#pragma omp atomic
                        c->g_mean2d[2 * g] += -h * (A * dx + B * dy);
#pragma omp atomic
                        c->g_mean2d[2 * g + 1] += -h * (B * dx + C * dy);
#pragma omp atomic
                        c->g_conic_o[4 * g] += -0.5 * h * dx * dx;
#pragma omp atomic
                        c->g_conic_o[4 * g + 1] += -h * dx * dy;
#pragma omp atomic
                        c->g_conic_o[4 * g + 2] += -0.5 * h * dy * dy;
#pragma omp atomic
                        c->g_conic_o[4 * g + 3] += Gs * dL_dalpha;
                    }
                }
        }
    }
}

// The same sums by the 3DGS per-pixel scheme in its float form, for the timed CPU baseline: alpha and G in float
// (the forward's evaluation), T recovered by division from the forward's final T, accumulation in double.
void gs3o_blend_backward_fast(gs3o_ctx* c, const float* grad_image, int row0, int row1) {
    const int W = c->s.width, H = c->s.height;
    const size_t P = (size_t)W * H;
    row0 = std::max(row0, 0);
    row1 = std::min(row1, c->tiles_y);
#pragma omp parallel for schedule(dynamic, 1)
    for (int t = row0 * c->tiles_x; t < row1 * c->tiles_x; ++t) {
        const int tx0 = (t % c->tiles_x) * kTile, ty0 = (t / c->tiles_x) * kTile;
        const int64_t s0 = c->ranges[2 * t];
        for (int y = ty0; y < std::min(ty0 + kTile, H); ++y)
            for (int x = tx0; x < std::min(tx0 + kTile, W); ++x) {
                const size_t pix = (size_t)y * W + x;
                const double G[3] = {grad_image[pix], grad_image[P + pix], grad_image[2 * P + pix]};
                double T = c->final_T[pix];
                double acc[3] = {0.0, 0.0, 0.0};  // colour behind the current splat, background included, / T
                for (int ch = 0; ch < 3; ++ch) acc[ch] = c->s.bg[ch];
                const double pxf = x + 0.5, pyf = y + 0.5;
                for (int64_t k = s0 + c->n_contrib[pix] - 1; k >= s0; --k) {
                    const int64_t g = c->point_list[k];
                    const float* co = &c->conic_o[4 * g];
                    // same float evaluation as the forward, so the same splats pass
                    const float dxf = c->mean2d[2 * g] - (float)pxf, dyf = c->mean2d[2 * g + 1] - (float)pyf;
                    const float a2 = -0.5f * kLog2e * co[0], b2 = -kLog2e * co[1], c2 = -0.5f * kLog2e * co[2];
                    const float q2 = fmaf(dxf, fmaf(a2, dxf, b2 * dyf), c2 * (dyf * dyf));
                    const float Gs = exp2f(std::min(q2, 0.f));
                    const float alpha_f = co[3] * Gs;
                    if (alpha_f < kAlphaMin) continue;
                    const double alpha = alpha_f;
                    const double om = std::max(1.0 - alpha, kOneMinusAlphaEps);
                    T = T / om;  // T before this splat
                    double col[3], dot = 0.0;
                    for (int ch = 0; ch < 3; ++ch) {
                        col[ch] = std::max(c->color_z[4 * g + ch], 0.f);
                        dot += G[ch] * (col[ch] - acc[ch]);
                    }
                    const double dL_dalpha = T * dot;
                    for (int ch = 0; ch < 3; ++ch) {
#pragma omp atomic
                        c->g_color[3 * g + ch] += G[ch] * alpha * T;
                        acc[ch] = alpha * col[ch] + (1.0 - alpha) * acc[ch];
                    }
                    const double dx = dxf, dy = dyf;
                    const double h = alpha * dL_dalpha;  // dL/dpower (power = -0.5 d^T K d)
                    const double A = co[0], B = co[1], C = co[2];
#pragma omp atomic
                    c->g_mean2d[2 * g] += -h * (A * dx + B * dy);
#pragma omp atomic
                    c->g_mean2d[2 * g + 1] += -h * (B * dx + C * dy);
#pragma omp atomic
                    c->g_conic_o[4 * g] += -0.5 * h * dx * dx;
#pragma omp atomic
                    c->g_conic_o[4 * g + 1] += -h * dx * dy;
#pragma omp atomic
                    c->g_conic_o[4 * g + 2] += -0.5 * h * dy * dy;
#pragma omp atomic
                    c->g_conic_o[4 * g + 3] += (double)Gs * dL_dalpha;
                }
            }
    }
}

// Chain rule from the accumulated (mean2d, conic, opacity, colour) gradients to the parameters.
void gs3o_preprocess_backward(gs3o_ctx* c, const float* means, const float* scales, const float* rotations,
                              const float* opacities, const float* sh_rest, float* g_means, float* g_scales,
                              float* g_rot, float* g_op, float* g_sh0, float* g_rest) {
    const gs3o_settings* s = &c->s;
    const int n = c->n;
    const int rest3 = 3 * s->rest_bases;
    const double* w0 = nullptr;
    (void)w0;
    double w[12];
    for (int k = 0; k < 12; ++k) w[k] = s->w2c[k];
#pragma omp parallel for schedule(static)
    for (int i = 0; i < n; ++i) {
        for (int k = 0; k < 3; ++k) g_means[3 * i + k] = g_scales[3 * i + k] = g_sh0[3 * i + k] = 0.f;
        for (int k = 0; k < 4; ++k) g_rot[4 * i + k] = 0.f;
        g_op[i] = 0.f;
        for (int k = 0; k < rest3; ++k) g_rest[(size_t)i * rest3 + k] = 0.f;
        if (c->n_touched[i] == 0) continue;
        const double px = means[3 * i], py = means[3 * i + 1], pz = means[3 * i + 2];
        const double xc = w[0] * px + w[1] * py + w[2] * pz + w[3];
        const double yc = w[4] * px + w[5] * py + w[6] * pz + w[7];
        const double zc = w[8] * px + w[9] * py + w[10] * pz + w[11];
        double gc[3];
        for (int ch = 0; ch < 3; ++ch) gc[ch] = c->color_z[4 * i + ch] >= 0.f ? c->g_color[3 * i + ch] : 0.0;
        // SH
        double ux = px - s->cam_position[0], uy = py - s->cam_position[1], uz = pz - s->cam_position[2];
        const double len = sqrt(ux * ux + uy * uy + uz * uz);
        const double x = ux / len, y = uy / len, z = uz / len;
        float bas[16];
        sh_basis((float)x, (float)y, (float)z, s->active_sh_bases, bas);
        for (int ch = 0; ch < 3; ++ch) g_sh0[3 * i + ch] = (float)(SH0 * gc[ch]);
        const int nb = std::min(s->active_sh_bases, s->rest_bases + 1);
        double v[16] = {0};
        for (int k = 1; k < nb; ++k) {
            for (int ch = 0; ch < 3; ++ch) {
                v[k] += gc[ch] * sh_rest[(size_t)i * rest3 + 3 * (k - 1) + ch];
                g_rest[(size_t)i * rest3 + 3 * (k - 1) + ch] = (float)(bas[k] * gc[ch]);
            }
        }
        double gdx = 0, gdy = 0, gdz = 0;
        if (nb > 1) {
            gdy += -SH1 * v[1];
            gdz += SH1 * v[2];
            gdx += -SH1 * v[3];
        }
        if (nb > 4) {
            const double xx = x * x, yy = y * y, zz = z * z;
            gdx += SH2[0] * y * v[4]; gdy += SH2[0] * x * v[4];
            gdy += SH2[1] * z * v[5]; gdz += SH2[1] * y * v[5];
            gdx += -2 * SH2[2] * x * v[6]; gdy += -2 * SH2[2] * y * v[6]; gdz += 4 * SH2[2] * z * v[6];
            gdx += SH2[3] * z * v[7]; gdz += SH2[3] * x * v[7];
            gdx += 2 * SH2[4] * x * v[8]; gdy += -2 * SH2[4] * y * v[8];
            if (nb > 9) {
                gdx += 6 * SH3[0] * x * y * v[9]; gdy += SH3[0] * (3 * xx - 3 * yy) * v[9];
                gdx += SH3[1] * y * z * v[10]; gdy += SH3[1] * x * z * v[10]; gdz += SH3[1] * x * y * v[10];
                gdx += -2 * SH3[2] * x * y * v[11]; gdy += SH3[2] * (4 * zz - xx - 3 * yy) * v[11];
                gdz += 8 * SH3[2] * y * z * v[11];
                gdx += -6 * SH3[3] * x * z * v[12]; gdy += -6 * SH3[3] * y * z * v[12];
                gdz += SH3[3] * (6 * zz - 3 * xx - 3 * yy) * v[12];
                gdx += SH3[4] * (4 * zz - 3 * xx - yy) * v[13]; gdy += -2 * SH3[4] * x * y * v[13];
                gdz += 8 * SH3[4] * x * z * v[13];
                gdx += 2 * SH3[5] * x * z * v[14]; gdy += -2 * SH3[5] * y * z * v[14]; gdz += SH3[5] * (xx - yy) * v[14];
                gdx += SH3[6] * (3 * xx - 3 * yy) * v[15]; gdy += -6 * SH3[6] * x * y * v[15];
            }
        }
        const double dd = gdx * x + gdy * y + gdz * z;
        double gp[3] = {(gdx - x * dd) / len, (gdy - y * dd) / len, (gdz - z * dd) / len};
        // projection, recomputed in double
        float Rf[3][3], nsq;
        quat_rot(rotations + 4 * i, Rf, nsq);
        double R[3][3], M[3][3], S3[3][3], T1[3][3], Sc[3][3];
        const double sc[3] = {exp((double)scales[3 * i]), exp((double)scales[3 * i + 1]), exp((double)scales[3 * i + 2])};
        for (int r = 0; r < 3; ++r)
            for (int k = 0; k < 3; ++k) {
                R[r][k] = Rf[r][k];
                M[r][k] = R[r][k] * sc[k];
            }
        for (int r = 0; r < 3; ++r)
            for (int k = 0; k < 3; ++k) S3[r][k] = M[r][0] * M[k][0] + M[r][1] * M[k][1] + M[r][2] * M[k][2];
        for (int r = 0; r < 3; ++r)
            for (int k = 0; k < 3; ++k) T1[r][k] = w[4 * r] * S3[0][k] + w[4 * r + 1] * S3[1][k] + w[4 * r + 2] * S3[2][k];
        for (int r = 0; r < 3; ++r)
            for (int k = 0; k < 3; ++k) Sc[r][k] = T1[r][0] * w[4 * k] + T1[r][1] * w[4 * k + 1] + T1[r][2] * w[4 * k + 2];
        const double iz = 1.0 / zc;
        const double lox = -1.3 * s->cx / s->fx, hix = 1.3 * (s->width - s->cx) / s->fx;
        const double loy = -1.3 * s->cy / s->fy, hiy = 1.3 * (s->height - s->cy) / s->fy;
        const double rx = xc * iz, ry = yc * iz;
        const double tx = std::min(std::max(rx, lox), hix), ty = std::min(std::max(ry, loy), hiy);
        const bool fxr = rx >= lox && rx <= hix, fyr = ry >= loy && ry <= hiy;
        const double J[2][3] = {{s->fx * iz, 0.0, -s->fx * tx * iz}, {0.0, s->fy * iz, -s->fy * ty * iz}};
        double S2[2][2];
        for (int r = 0; r < 2; ++r)
            for (int k = 0; k < 2; ++k) {
                double acc = 0;
                for (int p = 0; p < 3; ++p)
                    for (int q = 0; q < 3; ++q) acc += J[r][p] * Sc[p][q] * J[k][q];
                S2[r][k] = acc;
            }
        const double a = S2[0][0], b = S2[0][1], cc = S2[1][1];
        const double ad = a + kDilation, cd = cc + kDilation, det = ad * cd - b * b;
        const double A = cd / det, B = -b / det, C = ad / det;
        const double sig = 1.0 / (1.0 + exp(-(double)opacities[i]));
        double ga = 0, gb = 0, gcv = 0, f = 1.0;
        const double gA = c->g_conic_o[4 * i], gB = c->g_conic_o[4 * i + 1], gC = c->g_conic_o[4 * i + 2];
        const double go = c->g_conic_o[4 * i + 3];
        if (s->proper_antialiasing) {
            const double det0 = a * cc - b * b, ratio = det0 / det;
            if (ratio > 0) {
                f = sqrt(ratio);
                const double dr = go * sig * 0.5 / f;
                ga += dr * (cc * det - det0 * cd) / (det * det);
                gcv += dr * (a * det - det0 * ad) / (det * det);
                gb += dr * (-2 * b * (det - det0)) / (det * det);
            } else {
                f = 0;
            }
        }
        g_op[i] = (float)(go * f * sig * (1 - sig));
        {
            const double g0 = gA, g1 = 0.5 * gB, g2 = gC;
            const double k00 = A * g0 + B * g1, k01 = A * g1 + B * g2, k10 = B * g0 + C * g1, k11 = B * g1 + C * g2;
            ga += -(k00 * A + k01 * B);
            gcv += -(k10 * B + k11 * C);
            gb += -2 * (k00 * B + k01 * C);
        }
        const double G2[2][2] = {{ga, 0.5 * gb}, {0.5 * gb, gcv}};
        double GJ[2][3], gSc[3][3], gJ[2][3];
        for (int r = 0; r < 2; ++r)
            for (int k = 0; k < 3; ++k) GJ[r][k] = G2[r][0] * J[0][k] + G2[r][1] * J[1][k];
        for (int r = 0; r < 3; ++r)
            for (int k = 0; k < 3; ++k) gSc[r][k] = J[0][r] * GJ[0][k] + J[1][r] * GJ[1][k];
        for (int r = 0; r < 2; ++r)
            for (int k = 0; k < 3; ++k) gJ[r][k] = 2 * (GJ[r][0] * Sc[0][k] + GJ[r][1] * Sc[1][k] + GJ[r][2] * Sc[2][k]);
        const double gmx = c->g_mean2d[2 * i], gmy = c->g_mean2d[2 * i + 1];
        const double iz2 = iz * iz;
        double gxc = s->fx * iz * gmx, gyc = s->fy * iz * gmy;
        double gzc = -s->fx * xc * iz2 * gmx - s->fy * yc * iz2 * gmy;
        gzc += -s->fx * iz2 * gJ[0][0] - s->fy * iz2 * gJ[1][1];
        gzc += gJ[0][2] * (s->fx * tx * iz2 + (fxr ? s->fx * iz * xc * iz2 : 0.0));
        gxc += fxr ? gJ[0][2] * (-s->fx * iz2) : 0.0;
        gzc += gJ[1][2] * (s->fy * ty * iz2 + (fyr ? s->fy * iz * yc * iz2 : 0.0));
        gyc += fyr ? gJ[1][2] * (-s->fy * iz2) : 0.0;
        for (int k = 0; k < 3; ++k) gp[k] += w[k] * gxc + w[4 + k] * gyc + w[8 + k] * gzc;
        for (int k = 0; k < 3; ++k) g_means[3 * i + k] = (float)gp[k];
        double t1[3][3], gS3[3][3], gM[3][3], gR[3][3];
        for (int r = 0; r < 3; ++r)
            for (int k = 0; k < 3; ++k) t1[r][k] = w[r] * gSc[0][k] + w[4 + r] * gSc[1][k] + w[8 + r] * gSc[2][k];
        for (int r = 0; r < 3; ++r)
            for (int k = 0; k < 3; ++k) gS3[r][k] = t1[r][0] * w[k] + t1[r][1] * w[4 + k] + t1[r][2] * w[8 + k];
        for (int r = 0; r < 3; ++r)
            for (int k = 0; k < 3; ++k) gM[r][k] = 2 * (gS3[r][0] * M[0][k] + gS3[r][1] * M[1][k] + gS3[r][2] * M[2][k]);
        for (int k = 0; k < 3; ++k) {
            const double gs = gM[0][k] * R[0][k] + gM[1][k] * R[1][k] + gM[2][k] * R[2][k];
            g_scales[3 * i + k] = (float)(gs * sc[k]);
            for (int r = 0; r < 3; ++r) gR[r][k] = gM[r][k] * sc[k];
        }
        const double inv = 1.0 / sqrt(std::max((double)nsq, 1e-30));
        const float* q = rotations + 4 * i;
        const double qw = q[0] * inv, qx = q[1] * inv, qy = q[2] * inv, qz = q[3] * inv;
        const double gw = 2 * (-qz * gR[0][1] + qy * gR[0][2] + qz * gR[1][0] - qx * gR[1][2] - qy * gR[2][0] + qx * gR[2][1]);
        const double gx = 2 * (qy * gR[0][1] + qz * gR[0][2] + qy * gR[1][0] - 2 * qx * gR[1][1] - qw * gR[1][2] +
                               qz * gR[2][0] + qw * gR[2][1] - 2 * qx * gR[2][2]);
        const double gy = 2 * (-2 * qy * gR[0][0] + qx * gR[0][1] + qw * gR[0][2] + qx * gR[1][0] + qz * gR[1][2] -
                               qw * gR[2][0] + qz * gR[2][1] - 2 * qy * gR[2][2]);
        const double gz = 2 * (-2 * qz * gR[0][0] - qw * gR[0][1] + qx * gR[0][2] + qw * gR[1][0] - 2 * qz * gR[1][1] +
                               qy * gR[1][2] + qx * gR[2][0] + qy * gR[2][1]);
        const double qd = gw * qw + gx * qx + gy * qy + gz * qz;
        g_rot[4 * i] = (float)((gw - qw * qd) * inv);
        g_rot[4 * i + 1] = (float)((gx - qx * qd) * inv);
        g_rot[4 * i + 2] = (float)((gy - qy * qd) * inv);
        g_rot[4 * i + 3] = (float)((gz - qz * qd) * inv);
    }
}

void gs3o_adam(float* param, const float* grad, float* m, float* v, long long n, int step, double lr_d, double b1_d,
               double b2_d, double eps_d) {
    // host arithmetic of the reference wrapper (fastergs_lean_adam.patch:162-164), kernel values in float
    const float step_size = (float)(lr_d * (1.0 / (1.0 - pow(b1_d, step))));
    const float bc2r = (float)(1.0 / sqrt(1.0 - pow(b2_d, step)));
    const float b1 = (float)b1_d, b2 = (float)b2_d, eps = (float)eps_d;
    // squared tiny gradients are subnormal; x86 handles those in microcode, so flush them (each thread)
#pragma omp parallel for schedule(static)
    for (long long e = 0; e < n; ++e) {
        if ((_mm_getcsr() & 0x8040) != 0x8040) _mm_setcsr(_mm_getcsr() | 0x8040);
        const float g = grad[e], g2 = g * g;
        m[e] = fmaf(b1, m[e] - g, g);
        v[e] = fmaf(b2, v[e] - g2, g2);
        param[e] -= step_size * m[e] / fmaf(sqrtf(v[e]), bc2r, eps);  // the device's denominator
    }
}

// Accessors for the Python wrapper (pointers into the context's buffers; valid until the next call).
const float* gs3o_mean2d(gs3o_ctx* c) { return c->mean2d.data(); }
const float* gs3o_conic_o(gs3o_ctx* c) { return c->conic_o.data(); }
const float* gs3o_color_z(gs3o_ctx* c) { return c->color_z.data(); }
const float* gs3o_thr(gs3o_ctx* c) { return c->thr.data(); }
const int* gs3o_n_touched(gs3o_ctx* c) { return c->n_touched.data(); }
const int64_t* gs3o_point_list(gs3o_ctx* c) { return c->point_list.data(); }
const uint64_t* gs3o_keys_sorted(gs3o_ctx* c) { return c->keys_sorted.data(); }
const int64_t* gs3o_ranges(gs3o_ctx* c) { return c->ranges.data(); }
const float* gs3o_image(gs3o_ctx* c) { return c->image.data(); }
const float* gs3o_final_T(gs3o_ctx* c) { return c->final_T.data(); }
const int* gs3o_n_contrib(gs3o_ctx* c) { return c->n_contrib.data(); }
const unsigned char* gs3o_near(gs3o_ctx* c) { return c->near.data(); }
// The blend backward's float64 per-Gaussian sums: dL/dmean2d [N, 2], (dL/dA, dL/dB, dL/dC, dL/dopacity) [N, 4],
// dL/dcolour [N, 3] (before the colour >= 0 mask).
const double* gs3o_g_mean2d(gs3o_ctx* c) { return c->g_mean2d.data(); }
const double* gs3o_g_conic_o(gs3o_ctx* c) { return c->g_conic_o.data(); }
const double* gs3o_g_color(gs3o_ctx* c) { return c->g_color.data(); }

}  // extern "C"
