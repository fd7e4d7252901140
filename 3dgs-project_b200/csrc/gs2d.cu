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
// Differences in mechanism (not in results):
//   * binning runs on the GPU: radix sort of depth keys, duplication, radix sort of (tile, rank) keys
//   * bg is read on the device (the reference copies it to the host, one sync per call)
//   * colours are staged in shared memory with the geometry
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

struct Splat {
    float mx, my;
    float A, B, C;
    float o;
    float r, g, b;
};

__device__ __forceinline__ Splat load_splat(int id, const float* __restrict__ means, const float* __restrict__ conic,
                                            const float* __restrict__ color, const float* __restrict__ opacity) {
    Splat s;
    s.mx = means[2 * id];
    s.my = means[2 * id + 1];
    s.A = conic[3 * id];
    s.B = conic[3 * id + 1];
    s.C = conic[3 * id + 2];
    s.o = opacity[id];
    s.r = color[3 * id];
    s.g = color[3 * id + 1];
    s.b = color[3 * id + 2];
    return s;
}

// Same expression order as rasterize.cu:40-48.
__device__ __forceinline__ bool eval_splat(const Splat& s, float px, float py, float& dx, float& dy, float& G,
                                           float& alpha, bool& clamped) {
    dx = s.mx - px;
    dy = s.my - py;
    const float power = -0.5f * (s.A * dx * dx + s.C * dy * dy) - s.B * dx * dy;
    if (power > 0.0f) return false;
    G = expf(power);
    const float a = s.o * G;
    clamped = a > kAlphaMax;
    alpha = fminf(kAlphaMax, a);
    return alpha >= kAlphaMin;
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
                                uint32_t* __restrict__ vals) {
    const int i = blockIdx.x * blockDim.x + threadIdx.x;
    if (i >= n) return;
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
                           int32_t* __restrict__ point_list) {
    const int i = blockIdx.x * blockDim.x + threadIdx.x;
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
    s.sort_ws_bytes = sort_workspace_bytes<unsigned long long>(m);
    s.sort_ws = c.take<unsigned char>(s.sort_ws_bytes);
    s.scan_ws_bytes = scan_workspace_bytes(T > m ? T : m);
    s.scan_ws = c.take<unsigned char>(s.scan_ws_bytes);
    return s;
}

// ---------------------------------------------------------------------------------------------
// Forward: one 256-thread block per 16x16 tile, one pixel per thread (rasterize.cu:106-177)
// ---------------------------------------------------------------------------------------------
// kSave: the (T, C) state of every pixel is written at the start of each 32-splat bucket (bucket_state non-null).
// The splats of a staged batch are walked bucket by bucket, so the save is decided once per bucket.
template <bool kSave>
__global__ void __launch_bounds__(kBlock) k_forward(const int2* __restrict__ ranges,
                                                    const int32_t* __restrict__ point_list,
                                                    const float* __restrict__ means, const float* __restrict__ conic,
                                                    const float* __restrict__ color,
                                                    const float* __restrict__ opacity, const float* __restrict__ bg,
                                                    int N, int M, int num_buckets, int W, int H, int tiles_x,
                                                    float* __restrict__ out,
                                                    float* __restrict__ final_T, int32_t* __restrict__ n_contrib,
                                                    const int32_t* __restrict__ bucket_offsets,
                                                    float4* __restrict__ bucket_state) {
    __shared__ Splat s_splat[kBlock];
    const int tile = blockIdx.y * tiles_x + blockIdx.x;
    const int tid = threadIdx.x;
    const int px = blockIdx.x * kTile + (tid % kTile);
    const int py = blockIdx.y * kTile + (tid / kTile);
    const bool inside = px < W && py < H;
    bool done = !inside;

    const int2 range = clamp_range(ranges[tile], M);
    const int todo = range.y - range.x;
    const int rounds = (todo + kBlock - 1) / kBlock;
    const int bbase = bucket_state ? bucket_offsets[tile] : 0;
    const float fpx = static_cast<float>(px), fpy = static_cast<float>(py);

    float T = 1.0f;
    float Cr = 0.0f, Cg = 0.0f, Cb = 0.0f;
    int last = 0;
    for (int r = 0; r < rounds; ++r) {
        if (__syncthreads_count(done) == kBlock) break;
        const int k = range.x + r * kBlock + tid;
        if (k < range.y) s_splat[tid] = load_splat(clamp_id(point_list[k], N), means, conic, color, opacity);
        __syncthreads();
        const int n = min(kBlock, todo - r * kBlock);
        for (int j0 = 0; j0 < n; j0 += kBucket) {  // kBlock is a whole number of buckets
            if (kSave) {
                const int bkt = bbase + (r * kBlock + j0) / kBucket;
                if (bkt >= 0 && bkt < num_buckets)
                    bucket_state[static_cast<size_t>(bkt) * kBlock + tid] = make_float4(T, Cr, Cg, Cb);
            }
            if (done) continue;
            const int j1 = min(j0 + kBucket, n);
            for (int j = j0; j < j1; ++j) {
                const Splat& s = s_splat[j];
                float dx, dy, G, alpha;
                bool clamped;
                if (!eval_splat(s, fpx, fpy, dx, dy, G, alpha, clamped)) continue;
                const float test_T = T * (1.0f - alpha);
                if (test_T < kTMin) {
                    done = true;
                    break;
                }
                const float w = alpha * T;
                Cr += s.r * w;
                Cg += s.g * w;
                Cb += s.b * w;
                T = test_T;
                last = r * kBlock + j + 1;
            }
        }
    }
    if (inside) {
        const int pix = py * W + px;
        const int HW = H * W;
        out[pix] = Cr + T * bg[0];
        out[HW + pix] = Cg + T * bg[1];
        out[2 * HW + pix] = Cb + T * bg[2];
        final_T[pix] = T;
        n_contrib[pix] = last;
    }
}

// ---------------------------------------------------------------------------------------------
// Backward, per pixel (rasterize.cu:182-258): kept as the parity mode
// ---------------------------------------------------------------------------------------------
__global__ void __launch_bounds__(kBlock) k_backward_pixel(
    const int2* __restrict__ ranges, const int32_t* __restrict__ point_list, const float* __restrict__ means,
    const float* __restrict__ conic, const float* __restrict__ color, const float* __restrict__ opacity,
    const float* __restrict__ bg, int N, int M, int W, int H, int tiles_x, const float* __restrict__ final_T,
    const int32_t* __restrict__ n_contrib, const float* __restrict__ dL_dout, float* __restrict__ dmeans,
    float* __restrict__ dconic, float* __restrict__ dcolor, float* __restrict__ dopacity) {
    __shared__ Splat s_splat[kBlock];
    __shared__ int s_id[kBlock];
    const int tile = blockIdx.y * tiles_x + blockIdx.x;
    const int tid = threadIdx.x;
    const int px = blockIdx.x * kTile + (tid % kTile);
    const int py = blockIdx.y * kTile + (tid / kTile);
    const bool inside = px < W && py < H;
    const int pix = py * W + px;
    const int HW = H * W;
    const int2 range = clamp_range(ranges[tile], M);
    const int todo = range.y - range.x;
    const int rounds = (todo + kBlock - 1) / kBlock;

    const float T_final = inside ? final_T[pix] : 0.0f;
    const int last = inside ? n_contrib[pix] : 0;
    const float gr = inside ? dL_dout[pix] : 0.0f;
    const float gg = inside ? dL_dout[HW + pix] : 0.0f;
    const float gb = inside ? dL_dout[2 * HW + pix] : 0.0f;
    const float bg_dot = bg[0] * gr + bg[1] * gg + bg[2] * gb;
    const float fpx = static_cast<float>(px), fpy = static_cast<float>(py);

    float T = T_final;
    float ar = 0.0f, ag = 0.0f, ab = 0.0f;
    float last_alpha = 0.0f, lr = 0.0f, lg = 0.0f, lb = 0.0f;
    int contributor = todo;
    for (int r = 0; r < rounds; ++r) {
        __syncthreads();
        const int k = range.y - 1 - (r * kBlock + tid);
        if (k >= range.x) {
            const int id = clamp_id(point_list[k], N);
            s_id[tid] = id;
            s_splat[tid] = load_splat(id, means, conic, color, opacity);
        }
        __syncthreads();
        const int n = min(kBlock, todo - r * kBlock);
        for (int j = 0; j < n; ++j) {
            --contributor;
            if (!inside || contributor >= last) continue;
            const Splat& s = s_splat[j];
            float dx, dy, G, alpha;
            bool clamped;
            if (!eval_splat(s, fpx, fpy, dx, dy, G, alpha, clamped)) continue;
            const float one_minus = 1.0f - alpha;
            T = T / one_minus;
            ar = last_alpha * lr + (1.0f - last_alpha) * ar;
            ag = last_alpha * lg + (1.0f - last_alpha) * ag;
            ab = last_alpha * lb + (1.0f - last_alpha) * ab;
            last_alpha = alpha;
            lr = s.r;
            lg = s.g;
            lb = s.b;
            float dL_dalpha = ((s.r - ar) * gr + (s.g - ag) * gg + (s.b - ab) * gb) * T;
            dL_dalpha += (-T_final / one_minus) * bg_dot;
            const float w = alpha * T;
            const int id = s_id[j];
            atomicAdd(&dcolor[3 * id + 0], w * gr);
            atomicAdd(&dcolor[3 * id + 1], w * gg);
            atomicAdd(&dcolor[3 * id + 2], w * gb);
            if (!clamped) {
                const float dpow = s.o * G * dL_dalpha;
                atomicAdd(reinterpret_cast<float2*>(dmeans) + id,
                          make_float2((-s.A * dx - s.B * dy) * dpow, (-s.C * dy - s.B * dx) * dpow));
                atomicAdd(&dconic[3 * id + 0], -0.5f * dx * dx * dpow);
                atomicAdd(&dconic[3 * id + 1], -dx * dy * dpow);
                atomicAdd(&dconic[3 * id + 2], -0.5f * dy * dy * dpow);
                atomicAdd(&dopacity[id], G * dL_dalpha);
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
    __shared__ Splat s_splat[kBwdWarps][kBucket];
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
    const int HW = H * W;

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
            const int pix = y * W + x;
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
        const int id = clamp_id(point_list[range.x + bucket_start + lane], N);
        s_id[warp][lane] = id;
        s_splat[warp][lane] = load_splat(id, means, conic, color, opacity);
    }
    __syncwarp();
    const float fx = static_cast<float>(x);

    for (int j = 0; j < n_splats; ++j) {
        const Splat s = s_splat[warp][j];
        float g_mx = 0.f, g_my = 0.f, g_A = 0.f, g_B = 0.f, g_C = 0.f, g_r = 0.f, g_g = 0.f, g_b = 0.f, g_o = 0.f;
        bool used = false;
#pragma unroll
        for (int r = 0; r < kPxPerLane; ++r) {
            if (j >= lim[r]) continue;
            float dx, dy, G, alpha;
            bool clamped;
            if (!eval_splat(s, fx, static_cast<float>(y0 + 2 * r), dx, dy, G, alpha, clamped)) continue;
            used = true;
            const float3 gp = s_grad[warp][r * 32 + lane];
            const float w = alpha * T[r];
            const float dot_c = gp.x * s.r + gp.y * s.g + gp.z * s.b;
            g_r += w * gp.x;
            g_g += w * gp.y;
            g_b += w * gp.z;
            rho[r] -= w * dot_c;
            const float dL_dalpha = T[r] * dot_c - rho[r] / (1.0f - alpha);
            if (!clamped) {
                g_o += G * dL_dalpha;
                const float dpow = s.o * G * dL_dalpha;
                g_mx += (-s.A * dx - s.B * dy) * dpow;
                g_my += (-s.C * dy - s.B * dx) * dpow;
                g_A += -0.5f * dx * dx * dpow;
                g_B += -dx * dy * dpow;
                g_C += -0.5f * dy * dy * dpow;
            }
            T[r] = T[r] * (1.0f - alpha);
        }
        if (__ballot_sync(kFullMask, used) == 0u) continue;
#pragma unroll
        for (int o = 16; o > 0; o >>= 1) {
            g_mx += __shfl_down_sync(kFullMask, g_mx, o);
            g_my += __shfl_down_sync(kFullMask, g_my, o);
            g_A += __shfl_down_sync(kFullMask, g_A, o);
            g_B += __shfl_down_sync(kFullMask, g_B, o);
            g_C += __shfl_down_sync(kFullMask, g_C, o);
            g_r += __shfl_down_sync(kFullMask, g_r, o);
            g_g += __shfl_down_sync(kFullMask, g_g, o);
            g_b += __shfl_down_sync(kFullMask, g_b, o);
            g_o += __shfl_down_sync(kFullMask, g_o, o);
        }
        if (lane == 0) {
            const int id = s_id[warp][j];
            atomicAdd(reinterpret_cast<float2*>(dmeans) + id, make_float2(g_mx, g_my));
            atomicAdd(&dconic[3 * id + 0], g_A);
            atomicAdd(&dconic[3 * id + 1], g_B);
            atomicAdd(&dconic[3 * id + 2], g_C);
            atomicAdd(&dcolor[3 * id + 0], g_r);
            atomicAdd(&dcolor[3 * id + 1], g_g);
            atomicAdd(&dcolor[3 * id + 2], g_b);
            atomicAdd(&dopacity[id], g_o);
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

int gs2d_bin_fill(const int32_t* rect, int n, int H, int W, long long m, void* count_ws, size_t count_ws_bytes,
                  void* fill_ws, size_t fill_ws_bytes, int32_t* point_list, int32_t* ranges, int32_t* bucket_offsets,
                  int32_t* bucket_to_tile, uint32_t* num_buckets, void* stream) {
    SPLAT_REQUIRE(n >= 0 && m >= 0 && H > 0 && W > 0, "gs2d_bin_fill: bad sizes");
    SPLAT_REQUIRE(m < (1ll << 31), "gs2d_bin_fill: %lld instances exceed int32 indexing", m);
    const int tiles_x = (W + kTile - 1) / kTile, tiles_y = (H + kTile - 1) / kTile;
    const int T = tiles_x * tiles_y;
    SPLAT_REQUIRE(fill_ws_bytes >= gs2d_bin_fill_workspace_size(m, H, W), "gs2d_bin_fill: workspace too small");
    cudaStream_t st = as_stream(stream);
    Carver cc(count_ws, count_ws_bytes);
    BinScratch s = carve_count(cc, n < 1 ? 1 : n);
    Carver cf(fill_ws, fill_ws_bytes);
    FillScratch f = carve_fill(cf, m < 1 ? 1 : m, T);
    SPLAT_CUDA(cudaMemsetAsync(f.first, 0, sizeof(uint32_t) * T, st));
    SPLAT_CUDA(cudaMemsetAsync(f.last, 0, sizeof(uint32_t) * T, st));
    const int rank_bits = bit_width(static_cast<unsigned long long>(n > 1 ? n - 1 : 1));
    const int tile_bits = bit_width(static_cast<unsigned long long>(T > 1 ? T - 1 : 1));
    if (m > 0) {
        k_bin_duplicate<<<div_up(n, 256), 256, 0, st>>>(reinterpret_cast<const int4*>(rect), s.counts, s.offsets,
                                                        s.rank, n, tiles_x, rank_bits, f.keys, f.vals);
        note_launch();
        SPLAT_TRY(check_launch("gs2d_bin_duplicate"));
        SPLAT_TRY(radix_sort_pairs<unsigned long long>(f.keys, f.vals, f.keys_sorted, f.vals_sorted, m, 0,
                                                       rank_bits + tile_bits, f.sort_ws, f.sort_ws_bytes, st));
        k_bin_runs<<<div_up(m, 256), 256, 0, st>>>(f.keys_sorted, f.vals_sorted, static_cast<int>(m), rank_bits,
                                                   f.first, f.last, point_list);
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
        k_bin_bucket_tiles<<<div_up(T, 256), 256, 0, st>>>(f.nb, f.bstart, T, bucket_to_tile);
        note_launch();
        SPLAT_TRY(check_launch("gs2d_bin_bucket_tiles"));
    }
    return SPLAT_OK;
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
    const dim3 grid(tiles_x, tiles_y), block(kBlock);
    const bool save = save_buckets && num_buckets > 0;
    auto kernel = save ? k_forward<true> : k_forward<false>;
    kernel<<<grid, block, 0, as_stream(stream)>>>(
        reinterpret_cast<const int2*>(ranges), point_list, means, conic, color, opacity, bg, N,
        static_cast<int>(num_instances), num_buckets, W, H, tiles_x, out, final_T, n_contrib, bucket_offsets,
        save ? reinterpret_cast<float4*>(bucket_state) : nullptr);
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
    k_backward_pixel<<<dim3(tiles_x, tiles_y), kBlock, 0, st>>>(
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
    k_backward_splat<<<div_up(num_buckets, kBwdWarps), 32 * kBwdWarps, 0, st>>>(
        num_buckets, bucket_to_tile, bucket_offsets, reinterpret_cast<const int2*>(ranges), point_list, means, conic,
        color, opacity, N, static_cast<int>(num_instances), W, H, tiles_x, out, n_contrib, dL_dout,
        reinterpret_cast<const float4*>(bucket_state), dmeans,
        dconic, dcolor, dopacity);
    note_launch();
    return check_launch("gs2d_backward_splat");
}

}  // extern "C"
