// splat2d.cu - the phase0 "splat2d" 2D op: tile binning, forward, per-pixel and per-splat backward,
// in float and double.
//
// The MODEL is phase0/csrc/macrotile/splat2d_common.h:7-11:
//   q = (l0 dx + l1 dy)^2 + (l2 dy)^2 with (dx, dy) = pixel centre (x + 0.5, y + 0.5) - mean,
//   o = sigmoid(z), alpha = min(0.99, o exp(-q / 2)), skipped below 1/255; front to back,
//   C += c alpha T, T *= (1 - alpha); a pixel stops once T < 1e-4 (checked before each splat).
// Outputs as phase0/csrc/macrotile/bindings.cpp:156-178: image [H,W,3], t_final, n_contrib (count),
// last_contrib (list position + 1), ckpt [B,256,4] = (C, T) at every bucket start, every slot written.
//
// Kernels (own design, same arithmetic per (pixel, splat) as splat2d_common.h:132-246):
//   forward          one 128-thread block per 16x16 tile, two pixels per thread (warp per 8x8 subtile);
//                    batches of 256 splats staged in shared memory with the sigmoid applied once per splat
//                    and the box of pixels each can reach (alpha >= 1/255); a warp evaluates only the splats
//                    whose box meets its subtile; once every pixel of the tile has stopped, the block only
//                    fills the remaining checkpoints
//   backward_pixel   one thread per pixel walking back from last_contrib (T by division), 9 atomics
//                    per (pixel, splat): the baseline mode
//   backward_splat   one warp per (tile, 32-splat bucket), lane owns the 8 pixels r*32 + lane, keeps
//                    (T, rho = G . (C_final - C)) replayed from the checkpoint, warp-reduces the 9
//                    parameter sums per splat and issues one atomic per parameter from lane 0
// Op counters (get_counters / reset_counters, bindings.cpp:222-230) count on the device when enabled.
#include "common.cuh"
#include "sort.cuh"

namespace splat {
namespace s2 {

constexpr int kTile = 16;
constexpr int kBlock = kTile * kTile;
constexpr int kBucket = 32;
constexpr int kPxPerLane = kBlock / kBucket;  // 8
constexpr int kBwdWarps = 4;
constexpr int kParams = 9;

enum Counter { kAtomics = 0, kEvals = 1, kNumCounters = 2 };
__device__ unsigned long long g_counters[kNumCounters];

template <typename S>
struct P {
    S mx, my, l0, l1, l2, o, cr, cg, cb;
};

template <typename S>
__device__ __forceinline__ S sp_exp(S x);
template <>
__device__ __forceinline__ float sp_exp<float>(float x) { return expf(x); }
template <>
__device__ __forceinline__ double sp_exp<double>(double x) { return exp(x); }

template <typename S>
__device__ __forceinline__ P<S> load_params(int id, const S* __restrict__ means, const S* __restrict__ chol,
                                            const S* __restrict__ zlogit, const S* __restrict__ colors) {
    P<S> p;
    p.mx = means[2 * id];
    p.my = means[2 * id + 1];
    p.l0 = chol[3 * id];
    p.l1 = chol[3 * id + 1];
    p.l2 = chol[3 * id + 2];
    p.o = S(1) / (S(1) + sp_exp<S>(-zlogit[id]));
    p.cr = colors[3 * id];
    p.cg = colors[3 * id + 1];
    p.cb = colors[3 * id + 2];
    return p;
}

template <typename S>
struct Eval {
    S dx, dy, a, b, g, alpha;
    bool clamped;
};

// splat2d_common.h:132-146, expression for expression.
template <typename S>
__device__ __forceinline__ Eval<S> eval(const P<S>& p, S px, S py) {
    Eval<S> e;
    e.dx = px - p.mx;
    e.dy = py - p.my;
    e.a = p.l0 * e.dx + p.l1 * e.dy;
    e.b = p.l2 * e.dy;
    const S q = e.a * e.a + e.b * e.b;
    e.g = sp_exp<S>(S(-0.5) * q);
    const S raw = p.o * e.g;
    e.clamped = raw > S(0.99);
    e.alpha = e.clamped ? S(0.99) : raw;
    return e;
}

// Chain rule to (mu_x, mu_y, l0, l1, l2, z, c_r, c_g, c_b): splat2d_common.h:227-246.
template <typename S>
__device__ __forceinline__ void chain(const P<S>& p, const Eval<S>& e, S dL_dalpha, S dcr, S dcg, S dcb, S* g) {
    const S d_alpha = e.clamped ? S(0) : dL_dalpha;
    const S d_z = d_alpha * e.g * p.o * (S(1) - p.o);
    const S d_q = S(-0.5) * e.g * p.o * d_alpha;
    const S two_a = S(2) * e.a;
    const S two_b = S(2) * e.b;
    g[0] = -d_q * two_a * p.l0;
    g[1] = -d_q * (two_a * p.l1 + two_b * p.l2);
    g[2] = d_q * two_a * e.dx;
    g[3] = d_q * two_a * e.dy;
    g[4] = d_q * two_b * e.dy;
    g[5] = d_z;
    g[6] = dcr;
    g[7] = dcg;
    g[8] = dcb;
}

template <typename S>
__device__ __forceinline__ void add_grads(const S* g, int id, S* gm, S* gc, S* gz, S* gcol) {
    atomicAdd(&gm[2 * id], g[0]);
    atomicAdd(&gm[2 * id + 1], g[1]);
    atomicAdd(&gc[3 * id], g[2]);
    atomicAdd(&gc[3 * id + 1], g[3]);
    atomicAdd(&gc[3 * id + 2], g[4]);
    atomicAdd(&gz[id], g[5]);
    atomicAdd(&gcol[3 * id], g[6]);
    atomicAdd(&gcol[3 * id + 1], g[7]);
    atomicAdd(&gcol[3 * id + 2], g[8]);
}

// One warp-aggregated add per counter and warp.
__device__ __forceinline__ void count(Counter c, unsigned long long v) {
    unsigned long long s = v;
#pragma unroll
    for (int o = 16; o > 0; o >>= 1) s += __shfl_xor_sync(kFullMask, s, o);
    if ((threadIdx.x & 31) == 0 && s) atomicAdd(&g_counters[c], s);
}

struct Tables {
    const int32_t* tile_off;     // [T + 1]
    const int32_t* tile_ids;     // [M]
    const int32_t* bucket_off;   // [T + 1]
    const int32_t* bucket_tile;  // [B]
    int N, M, T, B, H, W, tiles_x;
};

__device__ __forceinline__ int2 tile_range(const Tables& t, int tile) {
    int b = min(max(t.tile_off[tile], 0), t.M);
    int e = min(max(t.tile_off[tile + 1], b), t.M);
    return make_int2(b, e);
}

__device__ __forceinline__ int safe_id(const Tables& t, int k) { return min(max(t.tile_ids[k], 0), t.N - 1); }

// ---------------------------------------------------------------------------------------------
// Forward
// ---------------------------------------------------------------------------------------------
constexpr int kFwdThreads = kBlock / 2;  // two pixels per thread

// Box (x0, x1, y0, y1) of the pixel centres where alpha = min(0.99, o e^(-q/2)) can reach 1/255: those satisfy
// q = (l0 dx + l1 dy)^2 + (l2 dy)^2 <= R = 2 ln(255 o), an ellipse with half-extents sqrt(R (l1^2 + l2^2)) / |l0 l2|
// in x and sqrt(R) / |l2| in y. R is widened by 0.1% and the box by one pixel, so the rounding of the per-pixel
// evaluation never reaches outside it. An opacity below 1/255 reaches nothing; a degenerate factor or values that
// are not finite (which the per-pixel rules may turn into alpha = 0.99) give the unbounded box.
template <typename S>
__device__ __forceinline__ void reach_box(const P<S>& p, S (&box)[4]) {
    const S inf = S(INFINITY);
    box[0] = -inf;
    box[1] = inf;
    box[2] = -inf;
    box[3] = inf;
    if (!isfinite(p.mx) || !isfinite(p.my) || p.o != p.o) return;
    if (!(p.o * S(255) >= S(1))) {
        box[0] = inf;
        box[1] = -inf;
        return;
    }
    const S d = fabs(p.l0 * p.l2);
    if (!(d > S(0)) || !isfinite(d)) return;
    const S R = S(2.002) * log(S(255) * p.o) + S(1e-3);
    const S ex = sqrt(R * (p.l1 * p.l1 + p.l2 * p.l2)) / d + S(1), ey = sqrt(R) / fabs(p.l2) + S(1);
    if (!(ex == ex && ey == ey)) return;
    box[0] = p.mx - ex;
    box[1] = p.mx + ex;
    box[2] = p.my - ey;
    box[3] = p.my + ey;
}

// 128 threads per 16x16 tile, two pixels per thread: warp w owns the 8x8 subtile (w & 1, w >> 1), lane (column
// lane & 7, rows lane >> 3 and (lane >> 3) + 4). A round stages 256 splats of the tile's list (two per thread) with
// their reach boxes; each warp walks them 32 at a time, evaluating in list order only those whose box meets its
// subtile. The (C, T) checkpoint of both pixels is written at every bucket start; once every pixel of the tile
// has stopped, the remaining checkpoints are filled with the final (C, T), so every slot is written.
template <typename S, bool kCount>
__global__ void __launch_bounds__(kFwdThreads) k_forward(Tables t, const S* __restrict__ means,
                                                         const S* __restrict__ chol, const S* __restrict__ zlogit,
                                                         const S* __restrict__ colors, S* __restrict__ image,
                                                         S* __restrict__ t_final, int32_t* __restrict__ n_contrib,
                                                         int32_t* __restrict__ last_contrib, S* __restrict__ ckpt) {
    __shared__ P<S> s_p[kBlock];
    __shared__ S s_box[kBlock][4];
    const int tile = blockIdx.x;
    const int tid = threadIdx.x, lane = tid & 31, warp = tid >> 5;
    const int tx0 = (tile % t.tiles_x) * kTile, ty0 = (tile / t.tiles_x) * kTile;
    const int sx0 = tx0 + (warp & 1) * 8, sy0 = ty0 + (warp >> 1) * 8;
    const int x = sx0 + (lane & 7), ya = sy0 + (lane >> 3), yb = ya + 4;
    const int la = (ya - ty0) * kTile + (x - tx0), lb = la + 4 * kTile;
    const bool in_a = x < t.W && ya < t.H, in_b = x < t.W && yb < t.H;
    const S px = S(x) + S(0.5), pya = S(ya) + S(0.5), pyb = S(yb) + S(0.5);
    const S bx0 = S(sx0) + S(0.5), bx1 = S(sx0) + S(7.5), by0 = S(sy0) + S(0.5), by1 = S(sy0) + S(7.5);
    const int2 rg = tile_range(t, tile);
    const int bucket0 = t.bucket_off[tile];
    S Ra = S(0), Ga = S(0), Ba = S(0), Ta = S(1), Rb = S(0), Gb = S(0), Bb = S(0), Tb = S(1);
    int cnt_a = 0, cnt_b = 0, last_a = 0, last_b = 0;
    unsigned long long evals = 0;
    auto store_ckpt = [&](int local) {
        const int bk = bucket0 + local / kBucket;
        if (bk >= 0 && bk < t.B) {
            S* d = ckpt + (static_cast<size_t>(bk) * kBlock + la) * 4;
            d[0] = Ra;
            d[1] = Ga;
            d[2] = Ba;
            d[3] = Ta;
            d = ckpt + (static_cast<size_t>(bk) * kBlock + lb) * 4;
            d[0] = Rb;
            d[1] = Gb;
            d[2] = Bb;
            d[3] = Tb;
        }
    };
    for (int batch = rg.x; batch < rg.y; batch += kBlock) {
        const bool live = (in_a && !(Ta < S(1e-4))) || (in_b && !(Tb < S(1e-4)));
        if (__syncthreads_count(live) == 0) {
            // every pixel has stopped: the remaining checkpoints all hold the final (C, T)
            for (int local = (batch - rg.x + kBucket - 1) / kBucket * kBucket; local < rg.y - rg.x; local += kBucket)
                store_ckpt(local);
            break;
        }
#pragma unroll
        for (int h = 0; h < kBlock / kFwdThreads; ++h) {
            const int slot = tid + h * kFwdThreads;
            if (batch + slot < rg.y) {
                const P<S> p = load_params<S>(safe_id(t, batch + slot), means, chol, zlogit, colors);
                s_p[slot] = p;
                reach_box<S>(p, s_box[slot]);
            }
        }
        __syncthreads();
        const int nb = min(kBlock, rg.y - batch);
        for (int j0 = 0; j0 < nb; j0 += kBucket) {
            store_ckpt(batch - rg.x + j0);
            const bool run_a = in_a && !(Ta < S(1e-4)), run_b = in_b && !(Tb < S(1e-4));
            if (!__any_sync(kFullMask, run_a || run_b)) continue;
            bool hit = false;
            if (lane < nb - j0) {
                const S* bx = s_box[j0 + lane];
                hit = bx[0] <= bx1 && bx[1] >= bx0 && bx[2] <= by1 && bx[3] >= by0;
            }
            unsigned pending = __ballot_sync(kFullMask, hit);
            while (pending != 0u) {
                const int j = j0 + __ffs(pending) - 1;
                pending &= pending - 1u;
                const P<S>& p = s_p[j];
                const int local = batch - rg.x + j;
                if (in_a && !(Ta < S(1e-4))) {
                    const Eval<S> e = eval<S>(p, px, pya);
                    if (kCount) ++evals;
                    if (!(e.alpha < S(1.0 / 255.0))) {
                        Ra = Ra + p.cr * e.alpha * Ta;
                        Ga = Ga + p.cg * e.alpha * Ta;
                        Ba = Ba + p.cb * e.alpha * Ta;
                        Ta = Ta * (S(1) - e.alpha);
                        ++cnt_a;
                        last_a = local + 1;
                    }
                }
                if (in_b && !(Tb < S(1e-4))) {
                    const Eval<S> e = eval<S>(p, px, pyb);
                    if (kCount) ++evals;
                    if (!(e.alpha < S(1.0 / 255.0))) {
                        Rb = Rb + p.cr * e.alpha * Tb;
                        Gb = Gb + p.cg * e.alpha * Tb;
                        Bb = Bb + p.cb * e.alpha * Tb;
                        Tb = Tb * (S(1) - e.alpha);
                        ++cnt_b;
                        last_b = local + 1;
                    }
                }
            }
        }
        __syncthreads();
    }
    if (kCount) count(kEvals, evals);
    if (in_a) {
        const int pix = ya * t.W + x;
        image[3 * pix] = Ra;
        image[3 * pix + 1] = Ga;
        image[3 * pix + 2] = Ba;
        t_final[pix] = Ta;
        n_contrib[pix] = cnt_a;
        last_contrib[pix] = last_a;
    }
    if (in_b) {
        const int pix = yb * t.W + x;
        image[3 * pix] = Rb;
        image[3 * pix + 1] = Gb;
        image[3 * pix + 2] = Bb;
        t_final[pix] = Tb;
        n_contrib[pix] = cnt_b;
        last_contrib[pix] = last_b;
    }
}

// ---------------------------------------------------------------------------------------------
// Backward (A): per pixel, back to front
// ---------------------------------------------------------------------------------------------
template <typename S, bool kCount>
__global__ void __launch_bounds__(kBlock) k_backward_pixel(Tables t, const S* __restrict__ grad_image,
                                                           const S* __restrict__ means, const S* __restrict__ chol,
                                                           const S* __restrict__ zlogit, const S* __restrict__ colors,
                                                           const S* __restrict__ t_final,
                                                           const int32_t* __restrict__ last_contrib, S* gm, S* gc,
                                                           S* gz, S* gcol) {
    __shared__ P<S> s_p[kBlock];
    __shared__ int s_id[kBlock];
    const int tile = blockIdx.x;
    const int lane = threadIdx.x;
    const int x = (tile % t.tiles_x) * kTile + lane % kTile;
    const int y = (tile / t.tiles_x) * kTile + lane / kTile;
    const bool inside = x < t.W && y < t.H;
    const int pix = inside ? y * t.W + x : 0;
    const S px = S(x) + S(0.5), py = S(y) + S(0.5);
    S Gr = S(0), Gg = S(0), Gb = S(0), T_after = S(1);
    int last = 0;
    if (inside) {
        Gr = grad_image[3 * pix];
        Gg = grad_image[3 * pix + 1];
        Gb = grad_image[3 * pix + 2];
        T_after = t_final[pix];
        last = last_contrib[pix];
    }
    S Ar = S(0), Ag = S(0), Ab = S(0);
    const int2 rg = tile_range(t, tile);
    unsigned long long evals = 0, atomics = 0;
    for (int hi = rg.y; hi > rg.x; hi -= kBlock) {
        const int lo = max(hi - kBlock, rg.x);
        __syncthreads();
        if (lo + lane < hi) {
            const int id = safe_id(t, lo + lane);
            s_id[lane] = id;
            s_p[lane] = load_params<S>(id, means, chol, zlogit, colors);
        }
        __syncthreads();
        for (int j = hi - lo - 1; j >= 0; --j) {
            const int local = lo - rg.x + j;
            if (local >= last) continue;
            const P<S>& p = s_p[j];
            const Eval<S> e = eval<S>(p, px, py);
            if (kCount) ++evals;
            if (e.alpha < S(1.0 / 255.0)) continue;
            // splat2d_common.h:179-193
            const S one_minus = S(1) - e.alpha;
            const S T = T_after / one_minus;
            const S dcr = Gr * e.alpha * T, dcg = Gg * e.alpha * T, dcb = Gb * e.alpha * T;
            const S dot = Gr * (p.cr - Ar) + Gg * (p.cg - Ag) + Gb * (p.cb - Ab);
            Ar = e.alpha * p.cr + one_minus * Ar;
            Ag = e.alpha * p.cg + one_minus * Ag;
            Ab = e.alpha * p.cb + one_minus * Ab;
            T_after = T;
            S g[kParams];
            chain<S>(p, e, T * dot, dcr, dcg, dcb, g);
            add_grads<S>(g, s_id[j], gm, gc, gz, gcol);
            if (kCount) atomics += kParams;
        }
    }
    if (kCount) {
        count(kEvals, evals);
        count(kAtomics, atomics);
    }
}

// ---------------------------------------------------------------------------------------------
// Backward (B): per splat, warp per bucket, lane owns 8 pixels
// ---------------------------------------------------------------------------------------------
template <typename S, bool kCount>
__global__ void __launch_bounds__(32 * kBwdWarps) k_backward_splat(Tables t, const S* __restrict__ grad_image,
                                                                   const S* __restrict__ image,
                                                                   const S* __restrict__ means,
                                                                   const S* __restrict__ chol,
                                                                   const S* __restrict__ zlogit,
                                                                   const S* __restrict__ colors,
                                                                   const S* __restrict__ ckpt, S* gm, S* gc, S* gz,
                                                                   S* gcol) {
    __shared__ P<S> s_p[kBwdWarps][kBucket];
    __shared__ int s_id[kBwdWarps][kBucket];
    __shared__ S s_g[kBwdWarps][kBlock][3];
    const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
    const int b = blockIdx.x * kBwdWarps + warp;
    if (b >= t.B) return;
    const int tile = t.bucket_tile[b];
    if (tile < 0 || tile >= t.T) return;
    const int2 rg = tile_range(t, tile);
    const int start = rg.x + (b - t.bucket_off[tile]) * kBucket;
    if (start < rg.x) return;
    const int bsize = min(kBucket, rg.y - start);
    if (lane < bsize) {
        const int id = safe_id(t, start + lane);
        s_id[warp][lane] = id;
        s_p[warp][lane] = load_params<S>(id, means, chol, zlogit, colors);
    }
    const int x = (tile % t.tiles_x) * kTile + lane % kTile;
    const int y0 = (tile / t.tiles_x) * kTile + lane / kTile;
    const S px = S(x) + S(0.5);
    unsigned live = 0u;
    S T[kPxPerLane], rho[kPxPerLane];
#pragma unroll
    for (int r = 0; r < kPxPerLane; ++r) {
        const int y = y0 + 2 * r;
        const S* c = ckpt + (static_cast<size_t>(b) * kBlock + r * 32 + lane) * 4;
        T[r] = c[3];
        S Gr = S(0), Gg = S(0), Gb = S(0);
        rho[r] = S(0);
        if (x < t.W && y < t.H) {
            live |= 1u << r;
            const int pix = y * t.W + x;
            Gr = grad_image[3 * pix];
            Gg = grad_image[3 * pix + 1];
            Gb = grad_image[3 * pix + 2];
            rho[r] = Gr * (image[3 * pix] - c[0]) + Gg * (image[3 * pix + 1] - c[1]) + Gb * (image[3 * pix + 2] - c[2]);
        }
        s_g[warp][r * 32 + lane][0] = Gr;
        s_g[warp][r * 32 + lane][1] = Gg;
        s_g[warp][r * 32 + lane][2] = Gb;
    }
    __syncwarp();
    unsigned long long evals = 0, atomics = 0;
    for (int j = 0; j < bsize; ++j) {
        const P<S> p = s_p[warp][j];
        S acc[kParams];
#pragma unroll
        for (int k = 0; k < kParams; ++k) acc[k] = S(0);
        bool used = false;
#pragma unroll
        for (int r = 0; r < kPxPerLane; ++r) {
            if (((live >> r) & 1u) == 0u || T[r] < S(1e-4)) continue;
            const Eval<S> e = eval<S>(p, px, S(y0 + 2 * r) + S(0.5));
            if (kCount) ++evals;
            if (e.alpha < S(1.0 / 255.0)) continue;
            used = true;
            // splat2d_common.h:210-222
            const S Gr = s_g[warp][r * 32 + lane][0], Gg = s_g[warp][r * 32 + lane][1],
                    Gb = s_g[warp][r * 32 + lane][2];
            const S Tj = T[r];
            const S w = e.alpha * Tj;
            const S dot_c = Gr * p.cr + Gg * p.cg + Gb * p.cb;
            rho[r] -= dot_c * w;
            T[r] = T[r] * (S(1) - e.alpha);
            const S dL_dalpha = Tj * dot_c - rho[r] / (S(1) - e.alpha);
            S g[kParams];
            chain<S>(p, e, dL_dalpha, Gr * w, Gg * w, Gb * w, g);
#pragma unroll
            for (int k = 0; k < kParams; ++k) acc[k] += g[k];
        }
        if (__ballot_sync(kFullMask, used) == 0u) continue;
#pragma unroll
        for (int k = 0; k < kParams; ++k) {
#pragma unroll
            for (int o = 16; o > 0; o >>= 1) acc[k] += __shfl_down_sync(kFullMask, acc[k], o);
        }
        if (lane == 0) {
            add_grads<S>(acc, s_id[warp][j], gm, gc, gz, gcol);
            if (kCount) atomics += kParams;
        }
    }
    if (kCount) {
        count(kEvals, evals);
        count(kAtomics, atomics);
    }
}

// ---------------------------------------------------------------------------------------------
// Binning (phase0/splat2d/ops.py:206-255), float64 like the reference
// ---------------------------------------------------------------------------------------------
template <typename S>
__global__ void k_bin_rect(const S* __restrict__ means, const S* __restrict__ chol, const S* __restrict__ zlogit,
                           int n, int H, int W, int4* __restrict__ trect, uint32_t* __restrict__ counts) {
    const int i = blockIdx.x * blockDim.x + threadIdx.x;
    if (i >= n) return;
    const double mx = static_cast<double>(means[2 * i]), my = static_cast<double>(means[2 * i + 1]);
    const double l0 = static_cast<double>(chol[3 * i]), l1 = static_cast<double>(chol[3 * i + 1]),
                 l2 = static_cast<double>(chol[3 * i + 2]);
    const double o = 1.0 / (1.0 + exp(-static_cast<double>(zlogit[i])));
    const double r2 = 2.0 * log(255.0 * o);
    const double r = sqrt(fmax(r2, 0.0));
    const double q = l1 / (l0 * l2);
    const double ex = r * sqrt(1.0 / (l0 * l0) + q * q);
    const double ey = r / fabs(l2);
    const double x0 = floor(mx - ex - 0.5) - 1.0, x1 = ceil(mx + ex - 0.5) + 1.0;
    const double y0 = floor(my - ey - 0.5) - 1.0, y1 = ceil(my + ey - 0.5) + 1.0;
    const bool valid = r2 > 0.0 && x1 >= 0.0 && x0 <= W - 1 && y1 >= 0.0 && y0 <= H - 1;
    const int tx0 = static_cast<int>(floor(fmin(fmax(x0, 0.0), double(W - 1)) / 16.0));
    const int tx1 = static_cast<int>(floor(fmin(fmax(x1, 0.0), double(W - 1)) / 16.0));
    const int ty0 = static_cast<int>(floor(fmin(fmax(y0, 0.0), double(H - 1)) / 16.0));
    const int ty1 = static_cast<int>(floor(fmin(fmax(y1, 0.0), double(H - 1)) / 16.0));
    trect[i] = make_int4(tx0, ty0, tx1, ty1);
    counts[i] = valid ? static_cast<uint32_t>((tx1 - tx0 + 1) * (ty1 - ty0 + 1)) : 0u;
}

__global__ void k_bin_duplicate(const int4* __restrict__ trect, const uint32_t* __restrict__ counts,
                                const uint32_t* __restrict__ offsets, int n, int tiles_x, int id_bits,
                                unsigned long long* __restrict__ keys, uint32_t* __restrict__ vals) {
    const int i = blockIdx.x * blockDim.x + threadIdx.x;
    if (i >= n) return;
    const uint32_t c = counts[i];
    if (c == 0) return;
    const int4 r = trect[i];
    const int w = r.z - r.x + 1;
    const uint32_t off = offsets[i];
    for (uint32_t k = 0; k < c; ++k) {
        const unsigned long long tile =
            static_cast<unsigned long long>(r.y + static_cast<int>(k) / w) * tiles_x + (r.x + static_cast<int>(k) % w);
        keys[off + k] = (tile << id_bits) | static_cast<unsigned long long>(i);
        vals[off + k] = static_cast<uint32_t>(i);
    }
}

__global__ void k_bin_runs(const unsigned long long* __restrict__ keys, const uint32_t* __restrict__ vals, int m,
                           int id_bits, uint32_t* __restrict__ first, uint32_t* __restrict__ last,
                           int32_t* __restrict__ tile_ids) {
    const int i = blockIdx.x * blockDim.x + threadIdx.x;
    if (i >= m) return;
    const unsigned long long tile = keys[i] >> id_bits;
    if (i == 0 || (keys[i - 1] >> id_bits) != tile) first[tile] = i;
    if (i == m - 1 || (keys[i + 1] >> id_bits) != tile) last[tile] = i + 1;
    tile_ids[i] = static_cast<int32_t>(vals[i]);
}

__global__ void k_bin_counts(const uint32_t* __restrict__ first, const uint32_t* __restrict__ last, int T,
                             uint32_t* __restrict__ cnt, uint32_t* __restrict__ nb) {
    const int t = blockIdx.x * blockDim.x + threadIdx.x;
    if (t > T) return;
    const uint32_t c = t < T ? last[t] - first[t] : 0u;
    cnt[t] = c;
    nb[t] = (c + kBucket - 1) / kBucket;
}

__global__ void k_bin_tables(const uint32_t* __restrict__ cstart, const uint32_t* __restrict__ nb,
                             const uint32_t* __restrict__ bstart, int T, int32_t* __restrict__ tile_off,
                             int32_t* __restrict__ bucket_off, int32_t* __restrict__ bucket_tile) {
    const int t = blockIdx.x * blockDim.x + threadIdx.x;
    if (t > T) return;
    tile_off[t] = static_cast<int32_t>(cstart[t]);
    bucket_off[t] = static_cast<int32_t>(bstart[t]);
    if (t < T && bucket_tile)
        for (uint32_t k = 0; k < nb[t]; ++k) bucket_tile[bstart[t] + k] = t;
}

struct CountWs {
    int4* trect;
    uint32_t* counts;
    uint32_t* offsets;
    void* scan_ws;
    size_t scan_bytes;
};

static CountWs carve_count(Carver& c, int n) {
    CountWs w;
    w.trect = c.take<int4>(n + 1);
    w.counts = c.take<uint32_t>(n + 1);
    w.offsets = c.take<uint32_t>(n + 1);
    w.scan_bytes = scan_workspace_bytes(n);
    w.scan_ws = c.take<unsigned char>(w.scan_bytes);
    return w;
}

struct FillWs {
    unsigned long long *keys, *keys_sorted;
    uint32_t *vals, *vals_sorted, *first, *last, *cnt, *nb, *cstart, *bstart;
    void* sort_ws;
    size_t sort_bytes;
    void* scan_ws;
    size_t scan_bytes;
};

static FillWs carve_fill(Carver& c, long long m, int T) {
    FillWs w;
    w.keys = c.take<unsigned long long>(m + 1);
    w.keys_sorted = c.take<unsigned long long>(m + 1);
    w.vals = c.take<uint32_t>(m + 1);
    w.vals_sorted = c.take<uint32_t>(m + 1);
    w.first = c.take<uint32_t>(T + 1);
    w.last = c.take<uint32_t>(T + 1);
    w.cnt = c.take<uint32_t>(T + 2);
    w.nb = c.take<uint32_t>(T + 2);
    w.cstart = c.take<uint32_t>(T + 2);
    w.bstart = c.take<uint32_t>(T + 2);
    w.sort_bytes = sort_workspace_bytes<unsigned long long>(m);
    w.sort_ws = c.take<unsigned char>(w.sort_bytes);
    w.scan_bytes = scan_workspace_bytes(T + 1);
    w.scan_ws = c.take<unsigned char>(w.scan_bytes);
    return w;
}

bool g_counting = false;
long long g_ckpt_bytes = 0;

template <typename S>
Tables make_tables(const int32_t* tile_off, const int32_t* tile_ids, const int32_t* bucket_off,
                   const int32_t* bucket_tile, int N, long long M, int B, int H, int W) {
    Tables t;
    t.tile_off = tile_off;
    t.tile_ids = tile_ids;
    t.bucket_off = bucket_off;
    t.bucket_tile = bucket_tile;
    t.N = N;
    t.M = static_cast<int>(M);
    t.B = B;
    t.H = H;
    t.W = W;
    t.tiles_x = (W + kTile - 1) / kTile;
    t.T = t.tiles_x * ((H + kTile - 1) / kTile);
    return t;
}

template <typename S>
int forward_impl(const void* means, const void* chol, const void* zl, const void* colors, const int32_t* tile_off,
                 const int32_t* tile_ids, const int32_t* bucket_off, const int32_t* bucket_tile, int N, long long M,
                 int B, int H, int W, void* image, void* t_final, int32_t* n_contrib, int32_t* last_contrib,
                 void* ckpt, cudaStream_t st) {
    Tables t = make_tables<S>(tile_off, tile_ids, bucket_off, bucket_tile, N, M, B, H, W);
    if (g_counting) g_ckpt_bytes += static_cast<long long>(B) * kBlock * 4 * sizeof(S);
    auto kern = g_counting ? k_forward<S, true> : k_forward<S, false>;
    kern<<<t.T, kFwdThreads, 0, st>>>(t, static_cast<const S*>(means), static_cast<const S*>(chol),
                                 static_cast<const S*>(zl), static_cast<const S*>(colors), static_cast<S*>(image),
                                 static_cast<S*>(t_final), n_contrib, last_contrib, static_cast<S*>(ckpt));
    note_launch();
    return check_launch("splat2d_forward");
}

template <typename S>
int backward_impl(int splat_mode, const void* grad_image, const void* means, const void* chol, const void* zl,
                  const void* colors, const int32_t* tile_off, const int32_t* tile_ids, const int32_t* bucket_off,
                  const int32_t* bucket_tile, int N, long long M, int B, int H, int W, const void* t_final,
                  const int32_t* last_contrib, const void* image, const void* ckpt, void* g_means, void* g_chol,
                  void* g_z, void* g_colors, cudaStream_t st) {
    Tables t = make_tables<S>(tile_off, tile_ids, bucket_off, bucket_tile, N, M, B, H, W);
    SPLAT_CUDA(cudaMemsetAsync(g_means, 0, sizeof(S) * 2 * N, st));
    SPLAT_CUDA(cudaMemsetAsync(g_chol, 0, sizeof(S) * 3 * N, st));
    SPLAT_CUDA(cudaMemsetAsync(g_z, 0, sizeof(S) * N, st));
    SPLAT_CUDA(cudaMemsetAsync(g_colors, 0, sizeof(S) * 3 * N, st));
    if (M == 0) return SPLAT_OK;
    const S* gi = static_cast<const S*>(grad_image);
    S *gm = static_cast<S*>(g_means), *gc = static_cast<S*>(g_chol), *gz = static_cast<S*>(g_z),
      *gcol = static_cast<S*>(g_colors);
    if (splat_mode) {
        if (B == 0) return SPLAT_OK;
        auto kern = g_counting ? k_backward_splat<S, true> : k_backward_splat<S, false>;
        kern<<<div_up(B, kBwdWarps), 32 * kBwdWarps, 0, st>>>(
            t, gi, static_cast<const S*>(image), static_cast<const S*>(means), static_cast<const S*>(chol),
            static_cast<const S*>(zl), static_cast<const S*>(colors), static_cast<const S*>(ckpt), gm, gc, gz, gcol);
        note_launch();
    } else {
        auto kern = g_counting ? k_backward_pixel<S, true> : k_backward_pixel<S, false>;
        kern<<<t.T, kBlock, 0, st>>>(t, gi, static_cast<const S*>(means), static_cast<const S*>(chol),
                                     static_cast<const S*>(zl), static_cast<const S*>(colors),
                                     static_cast<const S*>(t_final), last_contrib, gm, gc, gz, gcol);
        note_launch();
    }
    return check_launch(splat_mode ? "splat2d_backward_splat" : "splat2d_backward_pixel");
}

}  // namespace s2
}  // namespace splat

using namespace splat;
using namespace splat::s2;

extern "C" {

size_t splat2d_bin_count_workspace_size(int n) {
    Carver c(nullptr, 0);
    s2::carve_count(c, n < 1 ? 1 : n);
    return c.used + 256;
}

size_t splat2d_bin_fill_workspace_size(long long m, int H, int W) {
    const int T = ((W + kTile - 1) / kTile) * ((H + kTile - 1) / kTile);
    Carver c(nullptr, 0);
    s2::carve_fill(c, m < 1 ? 1 : m, T);
    return c.used + 256;
}

int splat2d_bin_count(int is_f64, const void* means, const void* chol, const void* opacity_logit, int n, int H, int W,
                      uint32_t* num_instances, void* count_ws, size_t count_ws_bytes, void* stream) {
    SPLAT_REQUIRE(n >= 0 && H > 0 && W > 0, "splat2d_bin_count: bad sizes");
    SPLAT_REQUIRE(count_ws_bytes >= splat2d_bin_count_workspace_size(n), "splat2d_bin_count: workspace too small");
    cudaStream_t st = as_stream(stream);
    if (n == 0) {
        SPLAT_CUDA(cudaMemsetAsync(num_instances, 0, sizeof(uint32_t), st));
        return SPLAT_OK;
    }
    Carver c(count_ws, count_ws_bytes);
    CountWs w = s2::carve_count(c, n);
    if (is_f64)
        s2::k_bin_rect<double><<<div_up(n, 256), 256, 0, st>>>(static_cast<const double*>(means),
                                                               static_cast<const double*>(chol),
                                                               static_cast<const double*>(opacity_logit), n, H, W,
                                                               w.trect, w.counts);
    else
        s2::k_bin_rect<float><<<div_up(n, 256), 256, 0, st>>>(static_cast<const float*>(means),
                                                             static_cast<const float*>(chol),
                                                             static_cast<const float*>(opacity_logit), n, H, W,
                                                             w.trect, w.counts);
   
        note_launch();
    SPLAT_TRY(check_launch("splat2d_bin_rect"));
    return scan_exclusive_u32(w.counts, w.offsets, n, num_instances, w.scan_ws, w.scan_bytes, st);
}

int splat2d_bin_fill(int n, int H, int W, long long m, void* count_ws, size_t count_ws_bytes, void* fill_ws,
                     size_t fill_ws_bytes, int32_t* tile_offsets, int32_t* tile_ids, int32_t* bucket_offsets,
                     int32_t* bucket_tile, uint32_t* num_buckets, void* stream) {
    SPLAT_REQUIRE(n >= 0 && m >= 0 && m < (1ll << 31) && H > 0 && W > 0, "splat2d_bin_fill: bad sizes");
    SPLAT_REQUIRE(fill_ws_bytes >= splat2d_bin_fill_workspace_size(m, H, W), "splat2d_bin_fill: workspace too small");
    const int tiles_x = (W + kTile - 1) / kTile;
    const int T = tiles_x * ((H + kTile - 1) / kTile);
    cudaStream_t st = as_stream(stream);
    Carver cc(count_ws, count_ws_bytes);
    CountWs cw = s2::carve_count(cc, n < 1 ? 1 : n);
    Carver cf(fill_ws, fill_ws_bytes);
    FillWs f = s2::carve_fill(cf, m < 1 ? 1 : m, T);
    SPLAT_CUDA(cudaMemsetAsync(f.first, 0, sizeof(uint32_t) * T, st));
    SPLAT_CUDA(cudaMemsetAsync(f.last, 0, sizeof(uint32_t) * T, st));
    const int id_bits = bit_width(static_cast<unsigned long long>(n > 1 ? n - 1 : 1));
    const int tile_bits = bit_width(static_cast<unsigned long long>(T > 1 ? T - 1 : 1));
    if (m > 0) {
        s2::k_bin_duplicate<<<div_up(n, 256), 256, 0, st>>>(cw.trect, cw.counts, cw.offsets, n, tiles_x, id_bits,
                                                            f.keys, f.vals);
        note_launch();
        SPLAT_TRY(check_launch("splat2d_bin_duplicate"));
        SPLAT_TRY(radix_sort_pairs<unsigned long long>(f.keys, f.vals, f.keys_sorted, f.vals_sorted, m, 0,
                                                       id_bits + tile_bits, f.sort_ws, f.sort_bytes, st));
        s2::k_bin_runs<<<div_up(m, 256), 256, 0, st>>>(f.keys_sorted, f.vals_sorted, static_cast<int>(m), id_bits,
                                                       f.first, f.last, tile_ids);
        note_launch();
        SPLAT_TRY(check_launch("splat2d_bin_runs"));
    }
    s2::k_bin_counts<<<div_up(T + 1, 256), 256, 0, st>>>(f.first, f.last, T, f.cnt, f.nb);
    note_launch();
    SPLAT_TRY(check_launch("splat2d_bin_counts"));
    SPLAT_TRY(scan_exclusive_u32(f.cnt, f.cstart, T + 1, nullptr, f.scan_ws, f.scan_bytes, st));
    SPLAT_TRY(scan_exclusive_u32(f.nb, f.bstart, T + 1, num_buckets, f.scan_ws, f.scan_bytes, st));
    s2::k_bin_tables<<<div_up(T + 1, 256), 256, 0, st>>>(f.cstart, f.nb, f.bstart, T, tile_offsets, bucket_offsets,
                                                         bucket_tile);
    note_launch();
    return check_launch("splat2d_bin_tables");
}

int splat2d_forward(int is_f64, const void* means, const void* chol, const void* opacity_logit, const void* colors,
                    const int32_t* tile_offsets, const int32_t* tile_ids, const int32_t* bucket_offsets,
                    const int32_t* bucket_tile, int N, long long num_instances, int num_buckets, int H, int W,
                    void* image, void* t_final, int32_t* n_contrib, int32_t* last_contrib, void* ckpt, void* stream) {
    SPLAT_REQUIRE(H > 0 && W > 0 && N >= 0 && num_buckets >= 0 && num_instances >= 0 && num_instances < (1ll << 31),
                  "splat2d_forward: bad sizes");
    SPLAT_REQUIRE(N > 0 || num_instances == 0, "splat2d_forward: instances without splats");
    if (is_f64)
        return s2::forward_impl<double>(means, chol, opacity_logit, colors, tile_offsets, tile_ids, bucket_offsets,
                                        bucket_tile, N, num_instances, num_buckets, H, W, image, t_final, n_contrib,
                                        last_contrib, ckpt, as_stream(stream));
    return s2::forward_impl<float>(means, chol, opacity_logit, colors, tile_offsets, tile_ids, bucket_offsets,
                                   bucket_tile, N, num_instances, num_buckets, H, W, image, t_final, n_contrib,
                                   last_contrib, ckpt, as_stream(stream));
}

int splat2d_backward(int is_f64, int splat_mode, const void* grad_image, const void* means, const void* chol,
                     const void* opacity_logit, const void* colors, const int32_t* tile_offsets,
                     const int32_t* tile_ids, const int32_t* bucket_offsets, const int32_t* bucket_tile, int N,
                     long long num_instances, int num_buckets, int H, int W, const void* t_final,
                     const int32_t* last_contrib, const void* image, const void* ckpt, void* grad_means,
                     void* grad_chol, void* grad_opacity_logit, void* grad_colors, void* stream) {
    SPLAT_REQUIRE(H > 0 && W > 0 && N >= 0 && num_buckets >= 0 && num_instances >= 0 && num_instances < (1ll << 31),
                  "splat2d_backward: bad sizes");
    SPLAT_REQUIRE(N > 0 || num_instances == 0, "splat2d_backward: instances without splats");
    if (is_f64)
        return s2::backward_impl<double>(splat_mode, grad_image, means, chol, opacity_logit, colors, tile_offsets,
                                         tile_ids, bucket_offsets, bucket_tile, N, num_instances, num_buckets, H, W,
                                         t_final, last_contrib, image, ckpt, grad_means, grad_chol, grad_opacity_logit,
                                         grad_colors, as_stream(stream));
    return s2::backward_impl<float>(splat_mode, grad_image, means, chol, opacity_logit, colors, tile_offsets, tile_ids,
                                    bucket_offsets, bucket_tile, N, num_instances, num_buckets, H, W, t_final,
                                    last_contrib, image, ckpt, grad_means, grad_chol, grad_opacity_logit, grad_colors,
                                    as_stream(stream));
}

int splat2d_set_counting(int on) {
    s2::g_counting = on != 0;
    return SPLAT_OK;
}

int splat2d_reset_counters(void) {
    const unsigned long long zero[s2::kNumCounters] = {0, 0};
    SPLAT_CUDA(cudaMemcpyToSymbol(s2::g_counters, zero, sizeof(zero)));
    s2::g_ckpt_bytes = 0;
    return SPLAT_OK;
}

int splat2d_get_counters(long long* out3) {
    unsigned long long v[s2::kNumCounters];
    SPLAT_CUDA(cudaMemcpyFromSymbol(v, s2::g_counters, sizeof(v)));
    out3[0] = static_cast<long long>(v[s2::kAtomics]);
    out3[1] = s2::g_ckpt_bytes;
    out3[2] = static_cast<long long>(v[s2::kEvals]);
    return SPLAT_OK;
}

}  // extern "C"
