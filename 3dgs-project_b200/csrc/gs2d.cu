// gs2d.cu - the toy2d "gs2d" 2D Gaussian tile rasterizer: binning, forward, two backwards.
//
// Semantics follow toy2d/csrc/rasterize.cu and toy2d/gs2d/{binning,reference}.py exactly:
//   * a Gaussian reaches only pixels of tiles inside its 3-sigma tile rect (binning.py:44-58)
//   * integer pixel coordinates; power = -0.5 (A dx^2 + C dy^2) - B dx dy; skip if power > 0
//   * alpha = min(0.99, o exp(power)); skip if alpha < 1/255; the clamp has zero gradient
//   * front to back; a pixel stops before the splat that would push T below 1e-4
//   * out = sum c_i alpha_i T_i + T_final bg; n_contrib = list position of the last contributor + 1
//   * bucket_state[b][p] = (T, C) of pixel p at the start of the tile's 32-splat bucket b, written
//     for every bucket of every 256-splat round the tile block executes (rasterize.cu:131-147)
//
// Mechanism (this library's own; results are the reference's):
//   * binning runs on the GPU: radix sort of depth keys, duplication, radix sort of (tile, rank) keys
//   * bg is read on the device (the reference copies it to the host, one sync per call)
//   * forward and per-pixel backward: 128 threads per 16x16 tile, two pixels per thread; warp w owns the
//     8x8 subtile (w & 1, w >> 1). Each staged splat carries the box of pixels its alpha can lift to 1/255,
//     and a warp evaluates only the splats whose box meets its subtile (one ballot per 32 splats). The
//     per-pixel backward sums a splat's terms over the warp's 64 pixels before its atomics
//   * backward_splat uses the warp-per-bucket layout in which a lane owns 8 pixels of the tile and
//     replays (T, rho = G . (out - C)) from the bucket checkpoint; per splat the warp sums the lanes'
//     terms with shuffles and lane 0 issues one atomic set per (splat, bucket). It computes the same
//     dL/dalpha as rasterize.cu:333-338 (rho folds the colour behind the splat, background included).
#include "common.cuh"
#include "sort.cuh"

namespace splat {
namespace gs2d {

constexpr int kTile = 16;
constexpr int kBlock = kTile * kTile;
constexpr int kBucket = 32;
constexpr int kPxPerLane = kBlock / 32;  // 8
constexpr int kBwdWarps = 4;
constexpr float kAlphaMin = 1.0f / 255.0f;
constexpr float kAlphaMax = 0.99f;
constexpr float kTMin = 1e-4f;

constexpr int kThreads = kBlock / 2;  // forward and per-pixel backward: two pixels per thread
constexpr int kRound = 256;           // splats staged per round (the reference's round, which the checkpoints follow)

// toy2d's per-(pixel, splat) exponent, d = mean - pixel at integer pixel coordinates, written as the single
// expression of rasterize.cu:40-48 so that it rounds the same way: the alpha >= 1/255 and T >= 1e-4 decisions,
// and with them the contributor counts, are bit-exact only with that rounding.
__device__ __forceinline__ float toy_power(float A, float B, float C, float dx, float dy) {
    return -0.5f * (A * dx * dx + C * dy * dy) - B * dx * dy;
}

// Box (x0, x1, y0, y1) of the integer pixels where alpha = min(0.99, o e^power) can reach 1/255: those lie in
// the ellipse q = -2 power <= R = 2 ln(255 o), whose half-extents are sqrt(R C / det) and sqrt(R A / det),
// det = AC - B^2. R is widened by 0.1% and the box by one pixel, so the rounding of the per-pixel evaluation
// never reaches outside it. An opacity below 1/255 reaches nothing; a conic that is not positive definite, or
// values that are not finite (which the per-pixel rules turn into alpha = 0.99), give the unbounded box.
__device__ __forceinline__ float4 reach_box(float mx, float my, float A, float B, float C, float o) {
    const float inf = __int_as_float(0x7f800000);
    const float4 all = make_float4(-inf, inf, -inf, inf);
    if (o != o || !isfinite(mx) || !isfinite(my)) return all;
    if (!(o * 255.f >= 1.f)) return make_float4(inf, -inf, inf, -inf);
    const float det = A * C - B * B;
    if (!(det > 0.f && A > 0.f && C > 0.f)) return all;
    const float R = 2.002f * logf(255.f * o) + 1e-3f;
    const float ex = sqrtf(R * C / det) + 1.f, ey = sqrtf(R * A / det) + 1.f;
    if (!(ex == ex && ey == ey)) return all;
    return make_float4(mx - ex, mx + ex, my - ey, my + ey);
}

// The splats of one round in shared memory, structure of arrays: (mx, my, A, B), (C, opacity, r, g), b, box.
struct Stage {
    float4 geo[kRound];
    float4 cor[kRound];
    float blue[kRound];
    float4 box[kRound];
    int id[kRound];
};

__device__ __forceinline__ void stage_splat(Stage& st, int slot, int g, const float* __restrict__ means,
                                            const float* __restrict__ conic, const float* __restrict__ color,
                                            const float* __restrict__ opacity) {
    const float2 m = reinterpret_cast<const float2*>(means)[g];
    const float A = conic[3 * g], B = conic[3 * g + 1], C = conic[3 * g + 2], o = opacity[g];
    st.geo[slot] = make_float4(m.x, m.y, A, B);
    st.cor[slot] = make_float4(C, o, color[3 * g], color[3 * g + 1]);
    st.blue[slot] = color[3 * g + 2];
    st.box[slot] = reach_box(m.x, m.y, A, B, C, o);
    st.id[slot] = g;
}

// Value k (0..8) of warp_fold9 lands in lane kFold9Lane[k]; this is the inverse map (-1: no value).
__device__ __forceinline__ int fold9_value(int lane) {
    switch (lane) {
        case 0: return 0;
        case 2: return 1;
        case 4: return 2;
        case 8: return 3;
        case 10: return 4;
        case 16: return 5;
        case 18: return 6;
        case 20: return 7;
        case 24: return 8;
        default: return -1;
    }
}

// Tables handed in by the caller are clamped so that an inconsistent list can give wrong pixels but
// never an access outside the buffers: ranges into [0, M], Gaussian ids into [0, N).
__device__ __forceinline__ int2 clamp_range(int2 r, int M) {
    r.y = min(max(r.y, 0), M);
    r.x = min(max(r.x, 0), r.y);
    return r;
}
__device__ __forceinline__ int clamp_id(int id, int N) { return min(max(id, 0), N - 1); }

// ---------------------------------------------------------------------------------------------
// Binning
// ---------------------------------------------------------------------------------------------

// Order-preserving map from a float to an unsigned key; -0 is folded onto +0 and every NaN onto one
// positive NaN, so equal values (as torch.argsort compares them) get equal keys and NaN sorts last.
__device__ __forceinline__ uint32_t float_key(float v) {
    if (v == 0.0f) v = 0.0f;
    uint32_t b = __float_as_uint(v);
    if (v != v) b = 0x7fc00000u;
    return (b & 0x80000000u) ? ~b : (b | 0x80000000u);
}
__device__ __forceinline__ unsigned long long double_key(double v) {
    if (v == 0.0) v = 0.0;
    unsigned long long b = static_cast<unsigned long long>(__double_as_longlong(v));
    if (v != v) b = 0x7ff8000000000000ull;
    return (b & 0x8000000000000000ull) ? ~b : (b | 0x8000000000000000ull);
}

// binning.py:44-58, float32 operation for operation (m - r, ((m + r) + 16) - 1, / 16, trunc, clamp).
__global__ void k_bin_rect(const float* __restrict__ means, const int32_t* __restrict__ radii,
                           const void* __restrict__ depth, int depth_is_f64, int n, int tiles_x, int tiles_y,
                           int4* __restrict__ rect, uint32_t* __restrict__ counts,
                           unsigned long long* __restrict__ depth_key64, uint32_t* __restrict__ depth_key32,
                           uint32_t* __restrict__ ids) {
    const int i = blockIdx.x * blockDim.x + threadIdx.x;
    if (i >= n) return;
    const float mx = means[2 * i], my = means[2 * i + 1];
    const int rad = radii[i];
    const float r = static_cast<float>(rad);
    const float fx = static_cast<float>(tiles_x), fy = static_cast<float>(tiles_y);
    const float xmin_f = fminf(fmaxf(truncf(__fdiv_rn(__fsub_rn(mx, r), 16.0f)), 0.0f), fx);
    const float ymin_f = fminf(fmaxf(truncf(__fdiv_rn(__fsub_rn(my, r), 16.0f)), 0.0f), fy);
    const float xmax_f =
        fminf(fmaxf(truncf(__fdiv_rn(__fsub_rn(__fadd_rn(__fadd_rn(mx, r), 16.0f), 1.0f), 16.0f)), 0.0f), fx);
    const float ymax_f =
        fminf(fmaxf(truncf(__fdiv_rn(__fsub_rn(__fadd_rn(__fadd_rn(my, r), 16.0f), 1.0f), 16.0f)), 0.0f), fy);
    int xmin = static_cast<int>(xmin_f), ymin = static_cast<int>(ymin_f);
    int xmax = static_cast<int>(xmax_f), ymax = static_cast<int>(ymax_f);
    const bool valid = rad > 0;
    const int w = valid ? xmax - xmin : 0;
    const int h = valid ? ymax - ymin : 0;
    int cnt = w * h;
    if (cnt < 0) cnt = 0;
    if (cnt == 0) {
        xmax = xmin;
        ymax = ymin;
    }
    rect[i] = make_int4(xmin, ymin, xmax, ymax);
    counts[i] = static_cast<uint32_t>(cnt);
    if (depth_is_f64)
        depth_key64[i] = double_key(static_cast<const double*>(depth)[i]);
    else
        depth_key32[i] = float_key(static_cast<const float*>(depth)[i]);
    ids[i] = static_cast<uint32_t>(i);
}

__global__ void k_bin_rank(const uint32_t* __restrict__ sorted_ids, int n, int64_t* __restrict__ order,
                           uint32_t* __restrict__ rank) {
    const int i = blockIdx.x * blockDim.x + threadIdx.x;
    if (i >= n) return;
    const uint32_t g = sorted_ids[i];
    order[i] = static_cast<int64_t>(g);
    rank[g] = static_cast<uint32_t>(i);
}

// key = tile << rank_bits | depth rank: the same order as binning.py's tile * n + rank.
__global__ void k_bin_duplicate(const int4* __restrict__ rect, const uint32_t* __restrict__ counts,
                                const uint32_t* __restrict__ offsets, const uint32_t* __restrict__ rank, int n,
                                int tiles_x, int rank_bits, unsigned long long* __restrict__ keys,
                                uint32_t* __restrict__ vals, const uint32_t* __restrict__ m_eff) {
    const int i = blockIdx.x * blockDim.x + threadIdx.x;
    if (i >= n) return;
    if (m_eff && *m_eff == 0u) return;  // bounded fill past its capacity: no list (flagged by k_bin_clamp)
    const uint32_t c = counts[i];
    if (c == 0) return;
    const int4 rc = rect[i];
    const int w = rc.z - rc.x;
    const uint32_t off = offsets[i];
    const unsigned long long rk = rank[i];
    for (uint32_t k = 0; k < c; ++k) {
        const int tx = rc.x + static_cast<int>(k) % w;
        const int ty = rc.y + static_cast<int>(k) / w;
        const unsigned long long tile = static_cast<unsigned long long>(ty) * tiles_x + tx;
        keys[off + k] = (tile << rank_bits) | rk;
        vals[off + k] = static_cast<uint32_t>(i);
    }
}

// Run boundaries of the sorted keys give each tile's [first, last) (zero for empty tiles).
__global__ void k_bin_runs(const unsigned long long* __restrict__ keys, const uint32_t* __restrict__ vals, int m,
                           int rank_bits, uint32_t* __restrict__ first, uint32_t* __restrict__ last,
                           int32_t* __restrict__ point_list, const uint32_t* __restrict__ m_dev) {
    const int i = blockIdx.x * blockDim.x + threadIdx.x;
    if (m_dev) m = min(m, static_cast<int>(*m_dev));
    if (i >= m) return;
    const unsigned long long t = keys[i] >> rank_bits;
    if (i == 0 || (keys[i - 1] >> rank_bits) != t) first[t] = static_cast<uint32_t>(i);
    if (i == m - 1 || (keys[i + 1] >> rank_bits) != t) last[t] = static_cast<uint32_t>(i + 1);
    point_list[i] = static_cast<int32_t>(vals[i]);
}

__global__ void k_bin_tile_counts(const uint32_t* __restrict__ first, const uint32_t* __restrict__ last, int T,
                                  uint32_t* __restrict__ count, uint32_t* __restrict__ nb) {
    const int t = blockIdx.x * blockDim.x + threadIdx.x;
    if (t >= T) return;
    const uint32_t c = last[t] - first[t];
    count[t] = c;
    nb[t] = (c + kBucket - 1) / kBucket;
}

// ranges = (start, start + count) with start the exclusive prefix of the counts (binning.py:81-82),
// bucket_offsets = exclusive prefix of ceil(count / 32).
__global__ void k_bin_ranges(const uint32_t* __restrict__ count, const uint32_t* __restrict__ start,
                             const uint32_t* __restrict__ bstart, int T, int32_t* __restrict__ ranges,
                             int32_t* __restrict__ bucket_offsets) {
    const int t = blockIdx.x * blockDim.x + threadIdx.x;
    if (t >= T) return;
    ranges[2 * t] = static_cast<int32_t>(start[t]);
    ranges[2 * t + 1] = static_cast<int32_t>(start[t] + count[t]);
    bucket_offsets[t] = static_cast<int32_t>(bstart[t]);
}

// The bounded fill's instance count: M from the count, or 0 with *overflow set when M exceeds the capacity (the list
// is then empty rather than written past its buffers).
__global__ void k_bin_clamp(const uint32_t* __restrict__ m, long long capacity, uint32_t* __restrict__ m_eff,
                            uint32_t* __restrict__ overflow) {
    const uint32_t v = *m;
    const bool over = static_cast<long long>(v) > capacity;
    *m_eff = over ? 0u : v;
    if (over) *overflow = 1u;
}
// Buckets past the count up to the capacity name no tile (-1), so that a launch over the capacity skips them.
__global__ void k_bin_bucket_tail(const uint32_t* __restrict__ total, long long capacity,
                                  int32_t* __restrict__ bucket_to_tile) {
    const long long b = static_cast<long long>(blockIdx.x) * blockDim.x + threadIdx.x;
    if (b < capacity && b >= static_cast<long long>(*total)) bucket_to_tile[b] = -1;
}
__global__ void k_bin_bucket_tiles(const uint32_t* __restrict__ nb, const uint32_t* __restrict__ bstart, int T,
                                   int32_t* __restrict__ bucket_to_tile) {
    const int t = blockIdx.x * blockDim.x + threadIdx.x;
    if (t >= T) return;
    const uint32_t s = bstart[t];
    for (uint32_t k = 0; k < nb[t]; ++k) bucket_to_tile[s + k] = t;
}

struct BinScratch {
    int4* rect_tmp;
    uint32_t* counts;
    uint32_t* offsets;
    uint32_t* rank;
    unsigned long long* dkey64;
    uint32_t* dkey32;
    unsigned long long* dkey64_sorted;
    uint32_t* dkey32_sorted;
    uint32_t* ids;
    uint32_t* ids_sorted;
    void* sort_ws;
    size_t sort_ws_bytes;
    void* scan_ws;
    size_t scan_ws_bytes;
};

static BinScratch carve_count(Carver& c, int n) {
    BinScratch s;
    s.counts = c.take<uint32_t>(n + 1);
    s.offsets = c.take<uint32_t>(n + 1);
    s.rank = c.take<uint32_t>(n + 1);
    s.dkey64 = c.take<unsigned long long>(n + 1);
    s.dkey32 = c.take<uint32_t>(n + 1);
    s.dkey64_sorted = c.take<unsigned long long>(n + 1);
    s.dkey32_sorted = c.take<uint32_t>(n + 1);
    s.ids = c.take<uint32_t>(n + 1);
    s.ids_sorted = c.take<uint32_t>(n + 1);
    s.sort_ws_bytes = sort_workspace_bytes<unsigned long long>(n);
    s.sort_ws = c.take<unsigned char>(s.sort_ws_bytes);
    s.scan_ws_bytes = scan_workspace_bytes(n);
    s.scan_ws = c.take<unsigned char>(s.scan_ws_bytes);
    s.rect_tmp = nullptr;
    return s;
}

struct FillScratch {
    unsigned long long* keys;
    uint32_t* vals;
    unsigned long long* keys_sorted;
    uint32_t* vals_sorted;
    uint32_t* first;
    uint32_t* last;
    uint32_t* count;
    uint32_t* start;
    uint32_t* nb;
    uint32_t* bstart;
    uint32_t* m_eff;  // bounded fill: the instance count used (M, or 0 when M exceeds the capacity)
    void* sort_ws;
    size_t sort_ws_bytes;
    void* scan_ws;
    size_t scan_ws_bytes;
};

static FillScratch carve_fill(Carver& c, long long m, int T) {
    FillScratch s;
    s.keys = c.take<unsigned long long>(m + 1);
    s.vals = c.take<uint32_t>(m + 1);
    s.keys_sorted = c.take<unsigned long long>(m + 1);
    s.vals_sorted = c.take<uint32_t>(m + 1);
    s.first = c.take<uint32_t>(T + 1);
    s.last = c.take<uint32_t>(T + 1);
    s.count = c.take<uint32_t>(T + 1);
    s.start = c.take<uint32_t>(T + 1);
    s.nb = c.take<uint32_t>(T + 1);
    s.bstart = c.take<uint32_t>(T + 1);
    s.m_eff = c.take<uint32_t>(1);
    s.sort_ws_bytes = sort_workspace_bytes<unsigned long long>(m);
    s.sort_ws = c.take<unsigned char>(s.sort_ws_bytes);
    s.scan_ws_bytes = scan_workspace_bytes(T > m ? T : m);
    s.scan_ws = c.take<unsigned char>(s.scan_ws_bytes);
    return s;
}

// ---------------------------------------------------------------------------------------------
// Forward: 128 threads per 16x16 tile, two pixels per thread (lane: column lane & 7, rows lane >> 3 and
// (lane >> 3) + 4 of its warp's 8x8 subtile). A round stages 256 splats of the tile's list; each warp walks them
// 32 at a time and evaluates, in list order, only those whose reach box meets its subtile.
// kSave: the (T, C) state of both pixels is written at the start of each 32-splat bucket of every round the
// block executes (bucket_state non-null).
// ---------------------------------------------------------------------------------------------
template <bool kSave>
__global__ void __launch_bounds__(kThreads) k_render(const int2* __restrict__ ranges,
                                                     const int32_t* __restrict__ point_list,
                                                     const float* __restrict__ means, const float* __restrict__ conic,
                                                     const float* __restrict__ color,
                                                     const float* __restrict__ opacity, const float* __restrict__ bg,
                                                     int N, int M, int num_buckets, int W, int H, int tiles_x,
                                                     float* __restrict__ out, float* __restrict__ final_T,
                                                     int32_t* __restrict__ n_contrib,
                                                     const int32_t* __restrict__ bucket_offsets,
                                                     float4* __restrict__ bucket_state) {
    __shared__ Stage st;
    const int tile = blockIdx.y * tiles_x + blockIdx.x;
    const int tid = threadIdx.x, lane = tid & 31, warp = tid >> 5;
    const int tx0 = blockIdx.x * kTile, ty0 = blockIdx.y * kTile;
    const int sx0 = tx0 + (warp & 1) * 8, sy0 = ty0 + (warp >> 1) * 8;
    const int x = sx0 + (lane & 7), ya = sy0 + (lane >> 3), yb = ya + 4;
    const int la = (ya - ty0) * kTile + (x - tx0), lb = la + 4 * kTile;  // tile-local pixel indices
    const bool in_a = x < W && ya < H, in_b = x < W && yb < H;
    bool done_a = !in_a, done_b = !in_b;
    const float fx = static_cast<float>(x), fya = static_cast<float>(ya), fyb = static_cast<float>(yb);

    const int2 rg = clamp_range(ranges[tile], M);
    const int count = rg.y - rg.x;
    const int bbase = kSave ? bucket_offsets[tile] : 0;
    float Ta = 1.f, Ra = 0.f, Ga = 0.f, Ba = 0.f, Tb = 1.f, Rb = 0.f, Gb = 0.f, Bb = 0.f;
    int last_a = 0, last_b = 0;
    for (int base = 0; base < count; base += kRound) {
        if (__syncthreads_count(!(done_a && done_b)) == 0) break;
#pragma unroll
        for (int h = 0; h < kRound / kThreads; ++h) {
            const int slot = tid + h * kThreads;
            if (base + slot < count)
                stage_splat(st, slot, clamp_id(point_list[rg.x + base + slot], N), means, conic, color, opacity);
        }
        __syncthreads();
        const int n = min(kRound, count - base);
        for (int j0 = 0; j0 < n; j0 += kBucket) {
            if (kSave) {
                const int bkt = bbase + (base + j0) / kBucket;
                if (bkt >= 0 && bkt < num_buckets) {
                    float4* ck = bucket_state + static_cast<size_t>(bkt) * kBlock;
                    ck[la] = make_float4(Ta, Ra, Ga, Ba);
                    ck[lb] = make_float4(Tb, Rb, Gb, Bb);
                }
            }
            if (__all_sync(kFullMask, done_a && done_b)) continue;
            bool hit = false;
            if (lane < n - j0) {
                const float4 bx = st.box[j0 + lane];
                hit = bx.x <= sx0 + 7 && bx.y >= sx0 && bx.z <= sy0 + 7 && bx.w >= sy0;
            }
            unsigned pending = __ballot_sync(kFullMask, hit);
            while (pending != 0u && !(done_a && done_b)) {
                const int j = j0 + __ffs(pending) - 1;
                pending &= pending - 1u;
                const float4 ge = st.geo[j], co = st.cor[j];
                const float dx = ge.x - fx;
                if (!done_a) {
                    const float pw = toy_power(ge.z, ge.w, co.x, dx, ge.y - fya);
                    if (!(pw > 0.f)) {
                        const float al = fminf(kAlphaMax, co.y * expf(pw));
                        if (al >= kAlphaMin) {
                            const float t = Ta * (1.f - al);
                            if (t < kTMin) {
                                done_a = true;
                            } else {
                                const float w = al * Ta;
                                Ra += co.z * w;
                                Ga += co.w * w;
                                Ba += st.blue[j] * w;
                                Ta = t;
                                last_a = base + j + 1;
                            }
                        }
                    }
                }
                if (!done_b) {
                    const float pw = toy_power(ge.z, ge.w, co.x, dx, ge.y - fyb);
                    if (!(pw > 0.f)) {
                        const float al = fminf(kAlphaMax, co.y * expf(pw));
                        if (al >= kAlphaMin) {
                            const float t = Tb * (1.f - al);
                            if (t < kTMin) {
                                done_b = true;
                            } else {
                                const float w = al * Tb;
                                Rb += co.z * w;
                                Gb += co.w * w;
                                Bb += st.blue[j] * w;
                                Tb = t;
                                last_b = base + j + 1;
                            }
                        }
                    }
                }
            }
        }
        __syncthreads();
    }
    const size_t HW = static_cast<size_t>(H) * W;
    if (in_a) {
        const size_t pix = static_cast<size_t>(ya) * W + x;
        out[pix] = Ra + Ta * bg[0];
        out[HW + pix] = Ga + Ta * bg[1];
        out[2 * HW + pix] = Ba + Ta * bg[2];
        final_T[pix] = Ta;
        n_contrib[pix] = last_a;
    }
    if (in_b) {
        const size_t pix = static_cast<size_t>(yb) * W + x;
        out[pix] = Rb + Tb * bg[0];
        out[HW + pix] = Gb + Tb * bg[1];
        out[2 * HW + pix] = Bb + Tb * bg[2];
        final_T[pix] = Tb;
        n_contrib[pix] = last_b;
    }
}

// ---------------------------------------------------------------------------------------------
// Backward, per pixel (the reference's backward_pixel mode): the forward's thread layout walking the tile's list
// back to front from the block's largest contributor count, 256 splats per round. Each pixel recovers T in front
// of a splat by division and keeps B = G . (colour behind the splat, background included), so that
// dL/dalpha = T (G . c) - B / (1 - alpha). Per splat, the warp sums its 64 pixels' nine terms with halving
// exchanges and nine lanes issue the nine atomics at once.
// ---------------------------------------------------------------------------------------------
__global__ void __launch_bounds__(kThreads) k_backward_pixel(
    const int2* __restrict__ ranges, const int32_t* __restrict__ point_list, const float* __restrict__ means,
    const float* __restrict__ conic, const float* __restrict__ color, const float* __restrict__ opacity,
    const float* __restrict__ bg, int N, int M, int W, int H, int tiles_x, const float* __restrict__ final_T,
    const int32_t* __restrict__ n_contrib, const float* __restrict__ dL_dout, float* __restrict__ dmeans,
    float* __restrict__ dconic, float* __restrict__ dcolor, float* __restrict__ dopacity) {
    __shared__ Stage st;
    __shared__ int s_last[kThreads / 32];
    const int tile = blockIdx.y * tiles_x + blockIdx.x;
    const int tid = threadIdx.x, lane = tid & 31, warp = tid >> 5;
    const int sx0 = blockIdx.x * kTile + (warp & 1) * 8, sy0 = blockIdx.y * kTile + (warp >> 1) * 8;
    const int x = sx0 + (lane & 7), ya = sy0 + (lane >> 3), yb = ya + 4;
    const bool in_a = x < W && ya < H, in_b = x < W && yb < H;
    const float fx = static_cast<float>(x), fya = static_cast<float>(ya), fyb = static_cast<float>(yb);
    const size_t HW = static_cast<size_t>(H) * W;
    const size_t pa = in_a ? static_cast<size_t>(ya) * W + x : 0, pb = in_b ? static_cast<size_t>(yb) * W + x : 0;

    const float3 ga = in_a ? make_float3(dL_dout[pa], dL_dout[HW + pa], dL_dout[2 * HW + pa]) : make_float3(0.f, 0.f, 0.f);
    const float3 gb = in_b ? make_float3(dL_dout[pb], dL_dout[HW + pb], dL_dout[2 * HW + pb]) : make_float3(0.f, 0.f, 0.f);
    const float bg0 = bg[0], bg1 = bg[1], bg2 = bg[2];
    float Ta = in_a ? final_T[pa] : 0.f, Tb = in_b ? final_T[pb] : 0.f;
    float Ba = Ta * (ga.x * bg0 + ga.y * bg1 + ga.z * bg2), Bb = Tb * (gb.x * bg0 + gb.y * bg1 + gb.z * bg2);
    const int last_a = in_a ? n_contrib[pa] : 0, last_b = in_b ? n_contrib[pb] : 0;

    const int2 rg = clamp_range(ranges[tile], M);
    const int wlast = __reduce_max_sync(kFullMask, max(last_a, last_b));
    if (lane == 0) s_last[warp] = wlast;
    __syncthreads();
    int top = 0;
#pragma unroll
    for (int w = 0; w < kThreads / 32; ++w) top = max(top, s_last[w]);
    top = min(top, rg.y - rg.x);  // list positions >= top are used by no pixel of the tile
    const int value = fold9_value(lane);

    for (int hi = top; hi > 0; hi -= kRound) {
        const int lo = max(hi - kRound, 0);
        __syncthreads();
#pragma unroll
        for (int h = 0; h < kRound / kThreads; ++h) {
            const int slot = tid + h * kThreads;
            if (lo + slot < hi)
                stage_splat(st, slot, clamp_id(point_list[rg.x + lo + slot], N), means, conic, color, opacity);
        }
        __syncthreads();
        for (int j0 = ((hi - lo - 1) / kBucket) * kBucket; j0 >= 0; j0 -= kBucket) {
            if (lo + j0 >= wlast) continue;  // warp-uniform: none of this warp's pixels reached the bucket
            bool hit = false;
            if (lane < hi - lo - j0) {
                const float4 bx = st.box[j0 + lane];
                hit = bx.x <= sx0 + 7 && bx.y >= sx0 && bx.z <= sy0 + 7 && bx.w >= sy0;
            }
            unsigned pending = __ballot_sync(kFullMask, hit);
            while (pending != 0u) {  // back to front: highest list position first
                const int b = 31 - __clz(pending);
                pending &= ~(1u << b);
                const int j = j0 + b, pos = lo + j;
                const float4 ge = st.geo[j], co = st.cor[j];
                const float blue = st.blue[j];
                const float dx = ge.x - fx;
                float v[9] = {0.f, 0.f, 0.f, 0.f, 0.f, 0.f, 0.f, 0.f, 0.f};  // mx, my, A, B, C, r, g, b, opacity
                bool used = false;
#pragma unroll
                for (int q = 0; q < 2; ++q) {
                    if (pos >= (q ? last_b : last_a)) continue;
                    const float dy = ge.y - (q ? fyb : fya);
                    const float pw = toy_power(ge.z, ge.w, co.x, dx, dy);
                    if (pw > 0.f) continue;
                    const float G = expf(pw), a0 = co.y * G, al = fminf(kAlphaMax, a0);
                    if (!(al >= kAlphaMin)) continue;
                    used = true;
                    const float3 g = q ? gb : ga;
                    float& T = q ? Tb : Ta;
                    float& B = q ? Bb : Ba;
                    const float om = 1.f - al;
                    T = T / om;  // transmittance in front of this splat
                    const float gc = g.x * co.z + g.y * co.w + g.z * blue;
                    const float w = al * T;
                    v[5] += w * g.x;
                    v[6] += w * g.y;
                    v[7] += w * g.z;
                    const float dL_dalpha = T * gc - B / om;
                    B += w * gc;
                    if (!(a0 > kAlphaMax)) {  // the 0.99 clamp passes no gradient
                        const float dpw = a0 * dL_dalpha;
                        v[0] += (-ge.z * dx - ge.w * dy) * dpw;
                        v[1] += (-co.x * dy - ge.w * dx) * dpw;
                        v[2] += -0.5f * dx * dx * dpw;
                        v[3] += -dx * dy * dpw;
                        v[4] += -0.5f * dy * dy * dpw;
                        v[8] += G * dL_dalpha;
                    }
                }
                if (__ballot_sync(kFullMask, used) == 0u) continue;
                const float t = warp_fold9(v, lane);
                if (value >= 0) {
                    const int g = st.id[j];
                    float* dst = value < 2 ? dmeans + 2 * g + value
                               : value < 5 ? dconic + 3 * g + (value - 2)
                               : value < 8 ? dcolor + 3 * g + (value - 5)
                                           : dopacity + g;
                    atomicAdd(dst, t);
                }
            }
        }
    }
}

// ---------------------------------------------------------------------------------------------
// Backward, per splat: one warp per (tile, 32-splat bucket), lane owns 8 pixels
// ---------------------------------------------------------------------------------------------
__global__ void __launch_bounds__(32 * kBwdWarps) k_backward_splat(
    int num_buckets, const int32_t* __restrict__ bucket_to_tile, const int32_t* __restrict__ bucket_offsets,
    const int2* __restrict__ ranges, const int32_t* __restrict__ point_list, const float* __restrict__ means,
    const float* __restrict__ conic, const float* __restrict__ color, const float* __restrict__ opacity, int N,
    int M, int W, int H, int tiles_x, const float* __restrict__ out, const int32_t* __restrict__ n_contrib,
    const float* __restrict__ dL_dout, const float4* __restrict__ bucket_state, float* __restrict__ dmeans,
    float* __restrict__ dconic, float* __restrict__ dcolor, float* __restrict__ dopacity) {
    __shared__ float4 s_geo[kBwdWarps][kBucket];  // (mx, my, A, B)
    __shared__ float4 s_cor[kBwdWarps][kBucket];  // (C, opacity, r, g)
    __shared__ float4 s_box[kBwdWarps][kBucket];
    __shared__ float s_blue[kBwdWarps][kBucket];
    __shared__ int s_id[kBwdWarps][kBucket];
    __shared__ float3 s_grad[kBwdWarps][kBlock];

    const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
    const int b = blockIdx.x * kBwdWarps + warp;
    if (b >= num_buckets) return;  // whole warp; warps never synchronise with each other
    const int tile = bucket_to_tile[b];
    if (tile < 0 || tile >= tiles_x * ((H + kTile - 1) / kTile)) return;
    const int2 range = clamp_range(ranges[tile], M);
    const int bucket_start = (b - bucket_offsets[tile]) * kBucket;
    if (bucket_start < 0) return;
    const int bsize = min(kBucket, range.y - range.x - bucket_start);
    const int tile_x0 = (tile % tiles_x) * kTile;
    const int tile_y0 = (tile / tiles_x) * kTile;
    const size_t HW = static_cast<size_t>(H) * W;

    const int x = tile_x0 + (lane % kTile);
    const int y0 = tile_y0 + (lane / kTile);
    float T[kPxPerLane], rho[kPxPerLane];
    int lim[kPxPerLane];
    int lim_max = 0;
    const float4* ckpt = bucket_state + static_cast<size_t>(b) * kBlock;
#pragma unroll
    for (int r = 0; r < kPxPerLane; ++r) {
        const int y = y0 + 2 * r;
        float3 G = make_float3(0.0f, 0.0f, 0.0f);
        T[r] = 0.0f;
        rho[r] = 0.0f;
        lim[r] = 0;
        if (x < W && y < H) {
            const size_t pix = static_cast<size_t>(y) * W + x;
            lim[r] = n_contrib[pix] - bucket_start;
            if (lim[r] > 0) {
                G = make_float3(dL_dout[pix], dL_dout[HW + pix], dL_dout[2 * HW + pix]);
                const float4 st = ckpt[r * 32 + lane];
                T[r] = st.x;
                rho[r] = G.x * (out[pix] - st.y) + G.y * (out[HW + pix] - st.z) + G.z * (out[2 * HW + pix] - st.w);
                lim_max = max(lim_max, lim[r]);
            }
        }
        s_grad[warp][r * 32 + lane] = G;
    }
    lim_max = __reduce_max_sync(kFullMask, lim_max);
    if (lim_max <= 0) return;  // no pixel of the tile reaches this bucket
    const int n_splats = min(bsize, lim_max);
    if (lane < n_splats) {
        const int g = clamp_id(point_list[range.x + bucket_start + lane], N);
        const float2 m = reinterpret_cast<const float2*>(means)[g];
        const float A = conic[3 * g], B = conic[3 * g + 1], C = conic[3 * g + 2], o = opacity[g];
        s_id[warp][lane] = g;
        s_geo[warp][lane] = make_float4(m.x, m.y, A, B);
        s_cor[warp][lane] = make_float4(C, o, color[3 * g], color[3 * g + 1]);
        s_blue[warp][lane] = color[3 * g + 2];
        s_box[warp][lane] = reach_box(m.x, m.y, A, B, C, o);
    }
    __syncwarp();
    const float fx = static_cast<float>(x);
    const int value = fold9_value(lane);

    for (int j = 0; j < n_splats; ++j) {
        const float4 ge = s_geo[warp][j], co = s_cor[warp][j], bx = s_box[warp][j];
        const float blue = s_blue[warp][j];
        const bool col_hit = fx >= bx.x && fx <= bx.y;
        const float dx = ge.x - fx;
        float v[9] = {0.f, 0.f, 0.f, 0.f, 0.f, 0.f, 0.f, 0.f, 0.f};  // mx, my, A, B, C, r, g, b, opacity
        bool used = false;
#pragma unroll
        for (int r = 0; r < kPxPerLane; ++r) {
            const float yr = static_cast<float>(tile_y0 + 2 * r);  // this lane row pair: yr, yr + 1
            if (bx.z > yr + 1.f || bx.w < yr) continue;           // warp-uniform
            if (!col_hit || j >= lim[r]) continue;
            const float dy = ge.y - static_cast<float>(y0 + 2 * r);
            const float pw = toy_power(ge.z, ge.w, co.x, dx, dy);
            if (pw > 0.f) continue;
            const float G = expf(pw), a0 = co.y * G, al = fminf(kAlphaMax, a0);
            if (!(al >= kAlphaMin)) continue;
            used = true;
            const float3 gp = s_grad[warp][r * 32 + lane];
            const float w = al * T[r];
            const float dot_c = gp.x * co.z + gp.y * co.w + gp.z * blue;
            v[5] += w * gp.x;
            v[6] += w * gp.y;
            v[7] += w * gp.z;
            rho[r] -= w * dot_c;
            const float dL_dalpha = T[r] * dot_c - rho[r] / (1.0f - al);
            if (!(a0 > kAlphaMax)) {  // the 0.99 clamp passes no gradient
                v[8] += G * dL_dalpha;
                const float dpw = a0 * dL_dalpha;
                v[0] += (-ge.z * dx - ge.w * dy) * dpw;
                v[1] += (-co.x * dy - ge.w * dx) * dpw;
                v[2] += -0.5f * dx * dx * dpw;
                v[3] += -dx * dy * dpw;
                v[4] += -0.5f * dy * dy * dpw;
            }
            T[r] = T[r] * (1.0f - al);
        }
        if (__ballot_sync(kFullMask, used) == 0u) continue;
        const float t = warp_fold9(v, lane);
        if (value >= 0) {
            const int g = s_id[warp][j];
            float* dst = value < 2 ? dmeans + 2 * g + value
                       : value < 5 ? dconic + 3 * g + (value - 2)
                       : value < 8 ? dcolor + 3 * g + (value - 5)
                                   : dopacity + g;
            atomicAdd(dst, t);
        }
    }
}

}  // namespace gs2d
}  // namespace splat

// ---------------------------------------------------------------------------------------------
// C-ABI
// ---------------------------------------------------------------------------------------------
using namespace splat;
using namespace splat::gs2d;

extern "C" {

size_t gs2d_bin_count_workspace_size(int n) {
    Carver c(nullptr, 0);
    carve_count(c, n < 1 ? 1 : n);
    return c.used + 256;
}

size_t gs2d_bin_fill_workspace_size(long long m, int H, int W) {
    const int T = ((W + kTile - 1) / kTile) * ((H + kTile - 1) / kTile);
    Carver c(nullptr, 0);
    carve_fill(c, m < 1 ? 1 : m, T);
    return c.used + 256;
}

int gs2d_bin_count(const float* means, const int32_t* radii, const void* depth, int depth_is_f64, int n, int H,
                   int W, int32_t* rect, int64_t* order, uint32_t* num_instances, void* count_ws, size_t count_ws_bytes,
                   void* stream) {
    SPLAT_REQUIRE(n >= 0 && H > 0 && W > 0, "gs2d_bin_count: bad sizes n=%d H=%d W=%d", n, H, W);
    SPLAT_REQUIRE(count_ws_bytes >= gs2d_bin_count_workspace_size(n), "gs2d_bin_count: workspace too small");
    cudaStream_t st = as_stream(stream);
    if (n == 0) {
        SPLAT_CUDA(cudaMemsetAsync(num_instances, 0, sizeof(uint32_t), st));
        return SPLAT_OK;
    }
    const int tiles_x = (W + kTile - 1) / kTile, tiles_y = (H + kTile - 1) / kTile;
    Carver c(count_ws, count_ws_bytes);
    BinScratch s = carve_count(c, n);
    const unsigned int blocks = div_up(n, 256);
    k_bin_rect<<<blocks, 256, 0, st>>>(means, radii, depth, depth_is_f64, n, tiles_x, tiles_y,
                                       reinterpret_cast<int4*>(rect), s.counts, s.dkey64, s.dkey32, s.ids);
    note_launch();
    SPLAT_TRY(check_launch("gs2d_bin_rect"));
    if (depth_is_f64)
        SPLAT_TRY(radix_sort_pairs<unsigned long long>(s.dkey64, s.ids, s.dkey64_sorted, s.ids_sorted, n, 0, 64,
                                                       s.sort_ws, s.sort_ws_bytes, st));
    else
        SPLAT_TRY(radix_sort_pairs<uint32_t>(s.dkey32, s.ids, s.dkey32_sorted, s.ids_sorted, n, 0, 32, s.sort_ws,
                                             s.sort_ws_bytes, st));
    k_bin_rank<<<blocks, 256, 0, st>>>(s.ids_sorted, n, order, s.rank);
    note_launch();
    SPLAT_TRY(check_launch("gs2d_bin_rank"));
    SPLAT_TRY(scan_exclusive_u32(s.counts, s.offsets, n, num_instances, s.scan_ws, s.scan_ws_bytes, st));
    return SPLAT_OK;
}

}  // extern "C"

namespace {
// The fill shared by the exact and the bounded entry points. m: the instance count (exact), or the capacity with
// m_dev the count on the device (bounded); bucket_capacity > 0: fill the buckets past the count with -1.
int bin_fill(const int32_t* rect, int n, int H, int W, long long m, const uint32_t* m_dev, void* count_ws,
             size_t count_ws_bytes, void* fill_ws, size_t fill_ws_bytes, int32_t* point_list, int32_t* ranges,
             int32_t* bucket_offsets, int32_t* bucket_to_tile, uint32_t* num_buckets, long long bucket_capacity,
             uint32_t* overflow, cudaStream_t st) {
    const int tiles_x = (W + kTile - 1) / kTile, tiles_y = (H + kTile - 1) / kTile;
    const int T = tiles_x * tiles_y;
    Carver cc(count_ws, count_ws_bytes);
    BinScratch s = carve_count(cc, n < 1 ? 1 : n);
    Carver cf(fill_ws, fill_ws_bytes);
    FillScratch f = carve_fill(cf, m < 1 ? 1 : m, T);
    SPLAT_CUDA(cudaMemsetAsync(f.first, 0, sizeof(uint32_t) * T, st));
    SPLAT_CUDA(cudaMemsetAsync(f.last, 0, sizeof(uint32_t) * T, st));
    const uint32_t* m_eff = nullptr;
    if (m_dev) {
        k_bin_clamp<<<1, 1, 0, st>>>(m_dev, m, f.m_eff, overflow);
        note_launch();
        SPLAT_TRY(check_launch("gs2d_bin_clamp"));
        m_eff = f.m_eff;
    }
    const int rank_bits = bit_width(static_cast<unsigned long long>(n > 1 ? n - 1 : 1));
    const int tile_bits = bit_width(static_cast<unsigned long long>(T > 1 ? T - 1 : 1));
    if (m > 0) {
        k_bin_duplicate<<<div_up(n, 256), 256, 0, st>>>(reinterpret_cast<const int4*>(rect), s.counts, s.offsets,
                                                        s.rank, n, tiles_x, rank_bits, f.keys, f.vals, m_eff);
        note_launch();
        SPLAT_TRY(check_launch("gs2d_bin_duplicate"));
        SPLAT_TRY(radix_sort_pairs<unsigned long long>(f.keys, f.vals, f.keys_sorted, f.vals_sorted, m, 0,
                                                       rank_bits + tile_bits, f.sort_ws, f.sort_ws_bytes, st,
                                                       nullptr, nullptr, m_eff));
        k_bin_runs<<<div_up(m, 256), 256, 0, st>>>(f.keys_sorted, f.vals_sorted, static_cast<int>(m), rank_bits,
                                                   f.first, f.last, point_list, m_eff);
        note_launch();
        SPLAT_TRY(check_launch("gs2d_bin_runs"));
    }
    k_bin_tile_counts<<<div_up(T, 256), 256, 0, st>>>(f.first, f.last, T, f.count, f.nb);
    note_launch();
    SPLAT_TRY(check_launch("gs2d_bin_tile_counts"));
    SPLAT_TRY(scan_exclusive_u32(f.count, f.start, T, nullptr, f.scan_ws, f.scan_ws_bytes, st));
    SPLAT_TRY(scan_exclusive_u32(f.nb, f.bstart, T, num_buckets, f.scan_ws, f.scan_ws_bytes, st));
    k_bin_ranges<<<div_up(T, 256), 256, 0, st>>>(f.count, f.start, f.bstart, T, ranges, bucket_offsets);
    note_launch();
    SPLAT_TRY(check_launch("gs2d_bin_ranges"));
    if (bucket_to_tile) {
        if (bucket_capacity > 0) {
            k_bin_bucket_tail<<<static_cast<unsigned>(div_up(bucket_capacity, 256ll)), 256, 0, st>>>(
                num_buckets, bucket_capacity, bucket_to_tile);
            note_launch();
            SPLAT_TRY(check_launch("gs2d_bin_bucket_tail"));
        }
        k_bin_bucket_tiles<<<div_up(T, 256), 256, 0, st>>>(f.nb, f.bstart, T, bucket_to_tile);
        note_launch();
        SPLAT_TRY(check_launch("gs2d_bin_bucket_tiles"));
    }
    return SPLAT_OK;
}
}  // namespace

extern "C" {

int gs2d_bin_fill(const int32_t* rect, int n, int H, int W, long long m, void* count_ws, size_t count_ws_bytes,
                  void* fill_ws, size_t fill_ws_bytes, int32_t* point_list, int32_t* ranges, int32_t* bucket_offsets,
                  int32_t* bucket_to_tile, uint32_t* num_buckets, void* stream) {
    SPLAT_REQUIRE(n >= 0 && m >= 0 && H > 0 && W > 0, "gs2d_bin_fill: bad sizes");
    SPLAT_REQUIRE(m < (1ll << 31), "gs2d_bin_fill: %lld instances exceed int32 indexing", m);
    SPLAT_REQUIRE(fill_ws_bytes >= gs2d_bin_fill_workspace_size(m, H, W), "gs2d_bin_fill: workspace too small");
    return bin_fill(rect, n, H, W, m, nullptr, count_ws, count_ws_bytes, fill_ws, fill_ws_bytes, point_list, ranges,
                    bucket_offsets, bucket_to_tile, num_buckets, 0, nullptr, as_stream(stream));
}

int gs2d_bin_fill_bounded(const int32_t* rect, int n, int H, int W, long long instance_capacity,
                          const uint32_t* num_instances, void* count_ws, size_t count_ws_bytes, void* fill_ws,
                          size_t fill_ws_bytes, int32_t* point_list, int32_t* ranges, int32_t* bucket_offsets,
                          int32_t* bucket_to_tile, long long bucket_capacity, uint32_t* num_buckets,
                          uint32_t* overflow, void* stream) {
    const long long T = static_cast<long long>((W + kTile - 1) / kTile) * ((H + kTile - 1) / kTile);
    SPLAT_REQUIRE(n >= 0 && instance_capacity >= 0 && H > 0 && W > 0, "gs2d_bin_fill_bounded: bad sizes");
    SPLAT_REQUIRE(instance_capacity < (1ll << 31), "gs2d_bin_fill_bounded: capacity %lld exceeds int32 indexing",
                  instance_capacity);
    SPLAT_REQUIRE(num_instances && num_buckets && overflow && bucket_to_tile,
                  "gs2d_bin_fill_bounded: null count, bucket table or overflow word");
    SPLAT_REQUIRE(bucket_capacity >= instance_capacity / kBucket + T,
                  "gs2d_bin_fill_bounded: bucket capacity %lld below the bound %lld", bucket_capacity,
                  instance_capacity / kBucket + T);
    SPLAT_REQUIRE(fill_ws_bytes >= gs2d_bin_fill_workspace_size(instance_capacity, H, W),
                  "gs2d_bin_fill_bounded: workspace too small");
    return bin_fill(rect, n, H, W, instance_capacity, num_instances, count_ws, count_ws_bytes, fill_ws,
                    fill_ws_bytes, point_list, ranges, bucket_offsets, bucket_to_tile, num_buckets, bucket_capacity,
                    overflow, as_stream(stream));
}

int gs2d_forward(const float* means, const float* conic, const float* color, const float* opacity, const float* bg,
                 const int32_t* ranges, const int32_t* point_list, const int32_t* bucket_offsets, int N,
                 long long num_instances, int num_buckets, int H, int W, int save_buckets, float* out,
                 float* final_T, int32_t* n_contrib, float* bucket_state, void* stream) {
    SPLAT_REQUIRE(H > 0 && W > 0, "gs2d_forward: image must be non-empty (H=%d W=%d)", H, W);
    SPLAT_REQUIRE(N >= 0 && num_instances >= 0 && num_instances < (1ll << 31) && num_buckets >= 0,
                  "gs2d_forward: bad sizes N=%d M=%lld B=%d", N, num_instances, num_buckets);
    SPLAT_REQUIRE(N > 0 || num_instances == 0, "gs2d_forward: instances without Gaussians");
    SPLAT_REQUIRE(!save_buckets || num_buckets == 0 || bucket_state, "gs2d_forward: bucket_state missing");
    const int tiles_x = (W + kTile - 1) / kTile, tiles_y = (H + kTile - 1) / kTile;
    const dim3 grid(tiles_x, tiles_y), block(kThreads);
    const bool save = save_buckets && num_buckets > 0;
    auto kernel = save ? k_render<true> : k_render<false>;
    SPLAT_TIMED_LAUNCH("gs2d_k_render", as_stream(stream),
                       (kernel<<<grid, block, 0, as_stream(stream)>>>(
                           reinterpret_cast<const int2*>(ranges), point_list, means, conic, color, opacity, bg, N,
                           static_cast<int>(num_instances), num_buckets, W, H, tiles_x, out, final_T, n_contrib,
                           bucket_offsets, save ? reinterpret_cast<float4*>(bucket_state) : nullptr)));
    note_launch();
    return check_launch("gs2d_forward");
}

int gs2d_backward_pixel(const float* means, const float* conic, const float* color, const float* opacity,
                        const float* bg, const int32_t* ranges, const int32_t* point_list, int N,
                        long long num_instances, int H, int W, const float* final_T, const int32_t* n_contrib,
                        const float* dL_dout, float* dmeans, float* dconic, float* dcolor, float* dopacity,
                        void* stream) {
    SPLAT_REQUIRE(H > 0 && W > 0 && N >= 0 && num_instances >= 0 && num_instances < (1ll << 31),
                  "gs2d_backward_pixel: bad sizes");
    SPLAT_REQUIRE(N > 0 || num_instances == 0, "gs2d_backward_pixel: instances without Gaussians");
    cudaStream_t st = as_stream(stream);
    SPLAT_CUDA(cudaMemsetAsync(dmeans, 0, sizeof(float) * 2 * N, st));
    SPLAT_CUDA(cudaMemsetAsync(dconic, 0, sizeof(float) * 3 * N, st));
    SPLAT_CUDA(cudaMemsetAsync(dcolor, 0, sizeof(float) * 3 * N, st));
    SPLAT_CUDA(cudaMemsetAsync(dopacity, 0, sizeof(float) * N, st));
    const int tiles_x = (W + kTile - 1) / kTile, tiles_y = (H + kTile - 1) / kTile;
    k_backward_pixel<<<dim3(tiles_x, tiles_y), kThreads, 0, st>>>(
        reinterpret_cast<const int2*>(ranges), point_list, means, conic, color, opacity, bg, N,
        static_cast<int>(num_instances), W, H, tiles_x, final_T, n_contrib, dL_dout, dmeans, dconic, dcolor, dopacity);
    note_launch();
    return check_launch("gs2d_backward_pixel");
}

int gs2d_backward_splat(const float* means, const float* conic, const float* color, const float* opacity,
                        const int32_t* ranges, const int32_t* point_list, const int32_t* bucket_offsets,
                        const int32_t* bucket_to_tile, int num_buckets, int N, long long num_instances, int H,
                        int W, const float* out, const int32_t* n_contrib, const float* bucket_state,
                        const float* dL_dout, float* dmeans, float* dconic, float* dcolor, float* dopacity,
                        void* stream) {
    SPLAT_REQUIRE(H > 0 && W > 0 && N >= 0 && num_buckets >= 0 && num_instances >= 0 &&
                      num_instances < (1ll << 31), "gs2d_backward_splat: bad sizes");
    SPLAT_REQUIRE(N > 0 || num_instances == 0, "gs2d_backward_splat: instances without Gaussians");
    cudaStream_t st = as_stream(stream);
    SPLAT_CUDA(cudaMemsetAsync(dmeans, 0, sizeof(float) * 2 * N, st));
    SPLAT_CUDA(cudaMemsetAsync(dconic, 0, sizeof(float) * 3 * N, st));
    SPLAT_CUDA(cudaMemsetAsync(dcolor, 0, sizeof(float) * 3 * N, st));
    SPLAT_CUDA(cudaMemsetAsync(dopacity, 0, sizeof(float) * N, st));
    if (num_buckets == 0 || num_instances == 0) return SPLAT_OK;  // zero gradients (rasterize.cu:434)
    const int tiles_x = (W + kTile - 1) / kTile;
    SPLAT_TIMED_LAUNCH("gs2d_k_backward_splat", st,
                       (k_backward_splat<<<div_up(num_buckets, kBwdWarps), 32 * kBwdWarps, 0, st>>>(
                           num_buckets, bucket_to_tile, bucket_offsets, reinterpret_cast<const int2*>(ranges),
                           point_list, means, conic, color, opacity, N, static_cast<int>(num_instances), W, H,
                           tiles_x, out, n_contrib, dL_dout, reinterpret_cast<const float4*>(bucket_state), dmeans,
                           dconic, dcolor, dopacity)));
    note_launch();
    return check_launch("gs2d_backward_splat");
}

}  // extern "C"
