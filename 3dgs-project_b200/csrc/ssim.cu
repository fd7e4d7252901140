// ssim.cu - fused L1 + SSIM training loss and its gradient (the fused-ssim step that sits beside the
// rasterizer in the reference's training loop; the fused-ssim package itself is not vendored).
//
// loss = (1 - lambda) mean|x - y| + lambda (1 - mean SSIM(x, y)), SSIM per pixel and channel with the 11x11
// Gaussian window (sigma 1.5, normalised), C1 = 0.01^2, C2 = 0.03^2, zero padding; "same" averages the SSIM map
// over every pixel, "valid" over the pixels whose window lies inside the image.
//
// k_ssim_forward: one 256-thread block per 32x16 output tile of one (image, channel) plane. The 42x26 input
// region (5-pixel halo) of x and y is loaded once into shared memory; a horizontal pass forms the five
// window sums (x, y, x^2, y^2, xy) for the 26 rows, a vertical pass finishes them per output pixel. Per pixel
// it writes the three partial derivatives of SSIM the backward needs (w.r.t. mu_x, E[x^2], E[xy]) and adds
// its SSIM and |x - y| to the block's sums; one deterministic reduction turns the block sums into the loss.
// k_ssim_backward: the same tiling over the derivative maps, d(sum SSIM)/dx(p) = (G*A)(p) + 2 x(p) (G*B)(p) +
// y(p) (G*C)(p) with G the (symmetric) window, plus the L1 term.
#include "common.cuh"

namespace splat {
namespace ssim {

constexpr int kTW = 32, kTH = 16, kR = 5, kWin = 2 * kR + 1;
constexpr int kInW = kTW + 2 * kR, kInH = kTH + 2 * kR;  // 42 x 26
constexpr int kThreads = 256;
constexpr float kC1 = 0.01f * 0.01f, kC2 = 0.03f * 0.03f;

// normalised 1-D Gaussian, sigma 1.5 (host-computed once, passed by value)
struct Window {
    float w[kWin];
};

Window make_window() {
    Window g{};
    double sum = 0.0, v[kWin];
    for (int k = 0; k < kWin; ++k) {
        const double d = k - kR;
        v[k] = exp(-d * d / (2.0 * 1.5 * 1.5));
        sum += v[k];
    }
    for (int k = 0; k < kWin; ++k) g.w[k] = static_cast<float>(v[k] / sum);
    return g;
}

struct Plane {
    int B, C, H, W;
    int tiles_x, tiles_y;
};

__device__ __forceinline__ float ld(const float* p, int H, int W, int y, int x) {
    return (y >= 0 && y < H && x >= 0 && x < W) ? __ldg(p + static_cast<size_t>(y) * W + x) : 0.f;
}

// sums[blockIdx] = (sum of SSIM over the counted pixels, sum of |x - y|)
__global__ void __launch_bounds__(kThreads) k_ssim_forward(const float* __restrict__ x, const float* __restrict__ y,
                                                          Plane pl, Window g, int valid_only,
                                                          float* __restrict__ dA, float* __restrict__ dB,
                                                          float* __restrict__ dC, float2* __restrict__ sums) {
    __shared__ float sx[kInH][kInW], sy[kInH][kInW];
    __shared__ float hs[5][kInH][kTW];  // horizontal window sums of x, y, x^2, y^2, xy
    __shared__ float red[2][kThreads / 32];
    const int tiles = pl.tiles_x * pl.tiles_y;
    const int plane = blockIdx.x / tiles, t = blockIdx.x % tiles;
    const int ox = (t % pl.tiles_x) * kTW, oy = (t / pl.tiles_x) * kTH;
    const size_t off = static_cast<size_t>(plane) * pl.H * pl.W;
    const float* xp = x + off;
    const float* yp = y + off;
    for (int k = threadIdx.x; k < kInH * kInW; k += kThreads) {
        const int r = k / kInW, c = k % kInW;
        sx[r][c] = ld(xp, pl.H, pl.W, oy - kR + r, ox - kR + c);
        sy[r][c] = ld(yp, pl.H, pl.W, oy - kR + r, ox - kR + c);
    }
    __syncthreads();
    for (int k = threadIdx.x; k < kInH * kTW; k += kThreads) {
        const int r = k / kTW, c = k % kTW;
        float a = 0.f, b = 0.f, aa = 0.f, bb = 0.f, ab = 0.f;
#pragma unroll
        for (int j = 0; j < kWin; ++j) {
            const float u = sx[r][c + j], v = sy[r][c + j], w = g.w[j];
            a += w * u;
            b += w * v;
            aa += w * u * u;
            bb += w * v * v;
            ab += w * u * v;
        }
        hs[0][r][c] = a;
        hs[1][r][c] = b;
        hs[2][r][c] = aa;
        hs[3][r][c] = bb;
        hs[4][r][c] = ab;
    }
    __syncthreads();
    float s_sum = 0.f, l_sum = 0.f;
    for (int k = threadIdx.x; k < kTH * kTW; k += kThreads) {
        const int r = k / kTW, c = k % kTW;
        const int py = oy + r, px = ox + c;
        if (py >= pl.H || px >= pl.W) continue;
        float m1 = 0.f, m2 = 0.f, e11 = 0.f, e22 = 0.f, e12 = 0.f;
#pragma unroll
        for (int j = 0; j < kWin; ++j) {
            const float w = g.w[j];
            m1 += w * hs[0][r + j][c];
            m2 += w * hs[1][r + j][c];
            e11 += w * hs[2][r + j][c];
            e22 += w * hs[3][r + j][c];
            e12 += w * hs[4][r + j][c];
        }
        const float s1 = e11 - m1 * m1, s2 = e22 - m2 * m2, s12 = e12 - m1 * m2;
        const float n1 = 2.f * m1 * m2 + kC1, n2 = 2.f * s12 + kC2;
        const float d1 = m1 * m1 + m2 * m2 + kC1, d2 = s1 + s2 + kC2;
        const float inv = 1.f / (d1 * d2);
        const float S = n1 * n2 * inv;
        const bool counted = !valid_only || (py >= kR && py < pl.H - kR && px >= kR && px < pl.W - kR);
        // dS/dmu_x, dS/dE[x^2], dS/dE[xy] (mu_x also enters sigma_x^2 and sigma_xy)
        const float a = 2.f * m2 * (n2 - n1) * inv - 2.f * m1 * S * (1.f / d1 - 1.f / d2);
        const float b = -S / d2;
        const float cc = 2.f * n1 * inv;
        const size_t o = off + static_cast<size_t>(py) * pl.W + px;
        dA[o] = counted ? a : 0.f;
        dB[o] = counted ? b : 0.f;
        dC[o] = counted ? cc : 0.f;
        if (counted) s_sum += S;
        l_sum += fabsf(sx[r + kR][c + kR] - sy[r + kR][c + kR]);
    }
    // block sums in a fixed order
#pragma unroll
    for (int o = 16; o > 0; o >>= 1) {
        s_sum += __shfl_down_sync(kFullMask, s_sum, o);
        l_sum += __shfl_down_sync(kFullMask, l_sum, o);
    }
    const int lane = threadIdx.x & 31, warp = threadIdx.x >> 5;
    if (lane == 0) {
        red[0][warp] = s_sum;
        red[1][warp] = l_sum;
    }
    __syncthreads();
    if (threadIdx.x == 0) {
        float a = 0.f, b = 0.f;
        for (int w = 0; w < kThreads / 32; ++w) {
            a += red[0][w];
            b += red[1][w];
        }
        sums[blockIdx.x] = make_float2(a, b);
    }
}

// One block: the block sums in a fixed order (in double), then the loss and the mean SSIM.
__global__ void __launch_bounds__(kThreads) k_ssim_reduce(const float2* __restrict__ sums, int nblocks,
                                                         double n_ssim, double n_l1, float lambda,
                                                         float* __restrict__ loss, float* __restrict__ ssim_mean) {
    __shared__ double red[2][kThreads];
    double a = 0.0, b = 0.0;
    for (int k = threadIdx.x; k < nblocks; k += kThreads) {
        a += sums[k].x;
        b += sums[k].y;
    }
    red[0][threadIdx.x] = a;
    red[1][threadIdx.x] = b;
    __syncthreads();
    for (int s = kThreads / 2; s > 0; s >>= 1) {
        if (threadIdx.x < s) {
            red[0][threadIdx.x] += red[0][threadIdx.x + s];
            red[1][threadIdx.x] += red[1][threadIdx.x + s];
        }
        __syncthreads();
    }
    if (threadIdx.x == 0) {
        const double ms = red[0][0] / n_ssim, ml = red[1][0] / n_l1;
        if (loss) *loss = static_cast<float>((1.0 - lambda) * ml + lambda * (1.0 - ms));
        if (ssim_mean) *ssim_mean = static_cast<float>(ms);
    }
}

__global__ void __launch_bounds__(kThreads) k_ssim_backward(const float* __restrict__ x, const float* __restrict__ y,
                                                           Plane pl, Window g, const float* __restrict__ dA,
                                                           const float* __restrict__ dB, const float* __restrict__ dC,
                                                           float w_ssim, float w_l1,
                                                           const float* __restrict__ grad_loss,
                                                           float* __restrict__ grad_x) {
    __shared__ float sa[kInH][kInW], sb[kInH][kInW], sc[kInH][kInW];
    __shared__ float hs[3][kInH][kTW];
    const int tiles = pl.tiles_x * pl.tiles_y;
    const int plane = blockIdx.x / tiles, t = blockIdx.x % tiles;
    const int ox = (t % pl.tiles_x) * kTW, oy = (t / pl.tiles_x) * kTH;
    const size_t off = static_cast<size_t>(plane) * pl.H * pl.W;
    for (int k = threadIdx.x; k < kInH * kInW; k += kThreads) {
        const int r = k / kInW, c = k % kInW;
        sa[r][c] = ld(dA + off, pl.H, pl.W, oy - kR + r, ox - kR + c);
        sb[r][c] = ld(dB + off, pl.H, pl.W, oy - kR + r, ox - kR + c);
        sc[r][c] = ld(dC + off, pl.H, pl.W, oy - kR + r, ox - kR + c);
    }
    __syncthreads();
    for (int k = threadIdx.x; k < kInH * kTW; k += kThreads) {
        const int r = k / kTW, c = k % kTW;
        float a = 0.f, b = 0.f, cc = 0.f;
#pragma unroll
        for (int j = 0; j < kWin; ++j) {
            const float w = g.w[j];
            a += w * sa[r][c + j];
            b += w * sb[r][c + j];
            cc += w * sc[r][c + j];
        }
        hs[0][r][c] = a;
        hs[1][r][c] = b;
        hs[2][r][c] = cc;
    }
    __syncthreads();
    const float scale = grad_loss ? __ldg(grad_loss) : 1.f;
    for (int k = threadIdx.x; k < kTH * kTW; k += kThreads) {
        const int r = k / kTW, c = k % kTW;
        const int py = oy + r, px = ox + c;
        if (py >= pl.H || px >= pl.W) continue;
        float a = 0.f, b = 0.f, cc = 0.f;
#pragma unroll
        for (int j = 0; j < kWin; ++j) {
            const float w = g.w[j];
            a += w * hs[0][r + j][c];
            b += w * hs[1][r + j][c];
            cc += w * hs[2][r + j][c];
        }
        const size_t o = off + static_cast<size_t>(py) * pl.W + px;
        const float xv = __ldg(x + o), yv = __ldg(y + o);
        const float d_ssim = a + 2.f * xv * b + yv * cc;
        const float diff = xv - yv;
        const float sgn = diff > 0.f ? 1.f : (diff < 0.f ? -1.f : 0.f);
        grad_x[o] = scale * (w_l1 * sgn - w_ssim * d_ssim);
    }
}

Plane make_plane(int B, int C, int H, int W) {
    Plane p;
    p.B = B;
    p.C = C;
    p.H = H;
    p.W = W;
    p.tiles_x = static_cast<int>(div_up(W, kTW));
    p.tiles_y = static_cast<int>(div_up(H, kTH));
    return p;
}

size_t workspace_bytes(int B, int C, int H, int W) {
    const size_t n = static_cast<size_t>(B) * C * H * W;
    const Plane p = make_plane(B, C, H, W);
    Carver c(nullptr, 0);
    c.take<float>(n);
    c.take<float>(n);
    c.take<float>(n);
    c.take<float2>(static_cast<size_t>(B) * C * p.tiles_x * p.tiles_y);
    return c.used + 256;
}

struct Work {
    float *dA, *dB, *dC;
    float2* sums;
};

Work carve(void* ws, size_t bytes, int B, int C, int H, int W) {
    const size_t n = static_cast<size_t>(B) * C * H * W;
    const Plane p = make_plane(B, C, H, W);
    Carver c(ws, bytes);
    Work w;
    w.dA = c.take<float>(n);
    w.dB = c.take<float>(n);
    w.dC = c.take<float>(n);
    w.sums = c.take<float2>(static_cast<size_t>(B) * C * p.tiles_x * p.tiles_y);
    return w;
}

int check_sizes(int B, int C, int H, int W, int padding_valid) {
    SPLAT_REQUIRE(B >= 1 && C >= 1 && H >= 1 && W >= 1, "l1_ssim: bad shape [%d, %d, %d, %d]", B, C, H, W);
    SPLAT_REQUIRE(!padding_valid || (H > 2 * kR && W > 2 * kR), "l1_ssim: 'valid' needs images larger than 10x10");
    SPLAT_REQUIRE(static_cast<long long>(B) * C * div_up(W, kTW) * div_up(H, kTH) < (1ll << 31),
                  "l1_ssim: image too large");
    return SPLAT_OK;
}

}  // namespace ssim
}  // namespace splat

using namespace splat;

extern "C" {

size_t splat_l1_ssim_workspace_size(int B, int C, int H, int W) {
    if (B < 1 || C < 1 || H < 1 || W < 1) return 0;
    return ssim::workspace_bytes(B, C, H, W);
}

int splat_l1_ssim_forward(const float* img, const float* gt, int B, int C, int H, int W, float lambda,
                          int padding_valid, float* loss, float* ssim_mean, void* workspace, size_t workspace_bytes,
                          void* stream) {
    SPLAT_TRY(ssim::check_sizes(B, C, H, W, padding_valid));
    SPLAT_REQUIRE(img && gt && workspace, "l1_ssim_forward: null pointer");
    SPLAT_REQUIRE(workspace_bytes >= ssim::workspace_bytes(B, C, H, W), "l1_ssim_forward: workspace too small");
    const ssim::Plane pl = ssim::make_plane(B, C, H, W);
    const ssim::Work w = ssim::carve(workspace, workspace_bytes, B, C, H, W);
    static const ssim::Window g = ssim::make_window();
    const unsigned blocks = static_cast<unsigned>(static_cast<long long>(B) * C * pl.tiles_x * pl.tiles_y);
    cudaStream_t st = as_stream(stream);
    ssim::k_ssim_forward<<<blocks, ssim::kThreads, 0, st>>>(img, gt, pl, g, padding_valid, w.dA, w.dB, w.dC,
                                                           w.sums);
    note_launch();
    const double n_all = static_cast<double>(B) * C * H * W;
    const double n_ssim = padding_valid ? static_cast<double>(B) * C * (H - 2 * ssim::kR) * (W - 2 * ssim::kR) : n_all;
    ssim::k_ssim_reduce<<<1, ssim::kThreads, 0, st>>>(w.sums, static_cast<int>(blocks), n_ssim, n_all, lambda, loss,
                                                      ssim_mean);
    note_launch();
    return check_launch("l1_ssim_forward");
}

int splat_l1_ssim_backward(const float* img, const float* gt, int B, int C, int H, int W, float lambda,
                           int padding_valid, const float* grad_loss, float* grad_img, const void* workspace,
                           size_t workspace_bytes, void* stream) {
    SPLAT_TRY(ssim::check_sizes(B, C, H, W, padding_valid));
    SPLAT_REQUIRE(img && gt && grad_img && workspace, "l1_ssim_backward: null pointer");
    SPLAT_REQUIRE(workspace_bytes >= ssim::workspace_bytes(B, C, H, W), "l1_ssim_backward: workspace too small");
    const ssim::Plane pl = ssim::make_plane(B, C, H, W);
    const ssim::Work w = ssim::carve(const_cast<void*>(workspace), workspace_bytes, B, C, H, W);
    static const ssim::Window g = ssim::make_window();
    const double n_all = static_cast<double>(B) * C * H * W;
    const double n_ssim = padding_valid ? static_cast<double>(B) * C * (H - 2 * ssim::kR) * (W - 2 * ssim::kR) : n_all;
    const unsigned blocks = static_cast<unsigned>(static_cast<long long>(B) * C * pl.tiles_x * pl.tiles_y);
    ssim::k_ssim_backward<<<blocks, ssim::kThreads, 0, as_stream(stream)>>>(
        img, gt, pl, g, w.dA, w.dB, w.dC, static_cast<float>(lambda / n_ssim),
        static_cast<float>((1.0 - lambda) / n_all), grad_loss, grad_img);
    note_launch();
    return check_launch("l1_ssim_backward");
}

}  // extern "C"
