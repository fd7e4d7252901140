// gs3d_forward.cu - 3DGS forward: preprocess, key duplication, 64-bit key sort, tile ranges and
// buckets, front-to-back blend (rules in gs3d_common.cuh).
//
// Launch sequence of one forward (all on the caller's stream):
//   gs3d_preprocess   k_preprocess (1 thread per Gaussian; SH rows loaded per warp with 16-byte
//                     loads through shared memory; listed tiles counted row by row in closed form),
//                     k_count_instances (M), then (gs3d_preprocess_order) radix sort of the
//                     Gaussians by depth bits (the four depth-digit passes of the 64-bit
//                     (tile << 32 | depth) key sort, done on N Gaussians instead of M instances; its
//                     last pass gathers the tile counts into that order), the counts scanned
//   (host reads M once to size the instance buffer, while the depth sort runs; the bucket buffer
//   is sized by a bound)
//   gs3d_render       k_duplicate in depth order, stable radix sort on the tile digits (completing
//                     the LSD sort of the 64-bit keys: same order, ties by Gaussian id),
//                     k_tile_bounds (32-ary search of each tile's first list position), k_tile_tables
//                     (ranges, buckets per tile and their scan, bucket -> tile), k_blend
// k_blend: one 128-thread block per 16x16 tile, two pixels per thread; each warp owns an 8x8 subtile
// and walks the tile list in 32-splat buckets staged in shared memory, skipping (by ballot) the splats
// whose culling rectangle misses its subtile - a rectangle that holds every pixel with alpha >= 1/255,
// so the skip changes no result. The (C, T) state of every pixel is saved at each bucket start for
// the backward; a block stops once every pixel has stopped.
#include "gs3d_common.cuh"

namespace splat {
namespace gs3d {

#ifndef SPLAT_PRE_THREADS
#define SPLAT_PRE_THREADS 128
#endif
constexpr int kPreThreads = SPLAT_PRE_THREADS;
constexpr int kPreWarps = kPreThreads / 32;
constexpr int kMaxRestBases = 15;

struct Params {
    const float* means;      // [N, 3]
    const float* scales;     // [N, 3] log scales
    const float* rotations;  // [N, 4] (w, x, y, z), not normalised
    const float* opacities;  // [N] logits
    const float* sh0;        // [N, 3]
    const float* sh_rest;    // [N, rest_bases, 3]
    const float* w2c;        // [4, 4] row-major
    const float* cam_pos;    // [3]
    int n;
};

__global__ void __launch_bounds__(kPreThreads) k_preprocess(Params P, Cam cam, PrimBuffers pb) {
    extern __shared__ __align__(16) float s_sh[];  // [kPreWarps][32 * rest_bases * 3]
    const int i = blockIdx.x * kPreThreads + threadIdx.x;
    const int lane = threadIdx.x & 31, warp = threadIdx.x >> 5;
    const bool valid = i < P.n;
    const int rest3 = cam.rest_bases * 3;

    float w2c[12];
#pragma unroll
    for (int k = 0; k < 12; ++k) w2c[k] = __ldg(P.w2c + k);

    float px = 0.f, py = 0.f, pz = 0.f;
    if (valid) {
        px = P.means[3 * i];
        py = P.means[3 * i + 1];
        pz = P.means[3 * i + 2];
    }
    const float xc = w2c[0] * px + w2c[1] * py + w2c[2] * pz + w2c[3];
    const float yc = w2c[4] * px + w2c[5] * py + w2c[6] * pz + w2c[7];
    const float zc = w2c[8] * px + w2c[9] * py + w2c[10] * pz + w2c[11];
    bool vis = valid && zc >= cam.near_plane && zc <= cam.far_plane;

    // The warp's SH rows (one contiguous block: its first Gaussian is a multiple of 32) start streaming into
    // shared memory now, while the geometry below is computed; the per-Gaussian inputs are loaded up front too.
    const unsigned any_near = __ballot_sync(kFullMask, vis);
    float* sh = s_sh + warp * 32 * rest3;
    const int first = i - lane;
    const bool stage = any_near && cam.active_sh_bases > 1 && rest3 > 0;
    const int nfl = stage ? min(32, P.n - first) * rest3 : 0;
    const float* src = P.sh_rest + static_cast<size_t>(first) * rest3;
    const int staged = stage ? stage_sh_begin(sh, src, nfl, lane) : 0;
    float4 q = make_float4(1.f, 0.f, 0.f, 0.f);
    float ls0 = 0.f, ls1 = 0.f, ls2 = 0.f, op_logit = 0.f;
    if (vis) {
        q = make_float4(P.rotations[4 * i], P.rotations[4 * i + 1], P.rotations[4 * i + 2], P.rotations[4 * i + 3]);
        ls0 = P.scales[3 * i];
        ls1 = P.scales[3 * i + 1];
        ls2 = P.scales[3 * i + 2];
        op_logit = P.opacities[i];
    }

    float mx = 0.f, my = 0.f, A = 0.f, B = 0.f, C = 0.f, o = 0.f, thr = 0.f;
    int rx0 = 0, ry0 = 0, rx1 = -1, ry1 = -1;
    uint32_t touched = 0;
    if (vis) {
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
        // camera-space covariance Sc = Wr S3 Wr^T
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
        const float tx = fminf(fmaxf(xc * inv_z, -1.3f * cam.cx / cam.fx), 1.3f * (cam.width - cam.cx) / cam.fx);
        const float ty = fminf(fmaxf(yc * inv_z, -1.3f * cam.cy / cam.fy), 1.3f * (cam.height - cam.cy) / cam.fy);
        const float j00 = cam.fx * inv_z, j02 = -cam.fx * tx * inv_z;
        const float j11 = cam.fy * inv_z, j12 = -cam.fy * ty * inv_z;
        // Sigma2 = J Sc J^T with J = [[j00, 0, j02], [0, j11, j12]]
        const float a = j00 * (j00 * Sc[0][0] + j02 * Sc[0][2]) + j02 * (j00 * Sc[2][0] + j02 * Sc[2][2]);
        const float b = j00 * (j11 * Sc[0][1] + j12 * Sc[0][2]) + j02 * (j11 * Sc[2][1] + j12 * Sc[2][2]);
        const float c = j11 * (j11 * Sc[1][1] + j12 * Sc[1][2]) + j12 * (j11 * Sc[2][1] + j12 * Sc[2][2]);
        const float ad = a + kDilation, cd = c + kDilation;
        const float det = ad * cd - b * b;
        o = 1.f / (1.f + expf(-op_logit));
        if (cam.proper_aa) o *= sqrtf(fmaxf((a * c - b * b) / det, 0.f));
        mx = cam.fx * xc * inv_z + cam.cx;
        my = cam.fy * yc * inv_z + cam.cy;
        vis = det > 0.f && o * 255.f >= 1.f && isfinite(mx) && isfinite(my);
        if (vis) {
            const float inv_det = 1.f / det;
            A = cd * inv_det;
            B = -b * inv_det;
            C = ad * inv_det;
            thr = logf(255.f * o);
            const float r2 = 2.f * (thr + kCullMargin);
            const float ex = sqrtf(r2 * ad), ey = sqrtf(r2 * cd);
            const float fx0 = ceilf(mx - ex - 0.5f) - 1.f, fx1 = floorf(mx + ex - 0.5f) + 1.f;
            const float fy0 = ceilf(my - ey - 0.5f) - 1.f, fy1 = floorf(my + ey - 0.5f) + 1.f;
            vis = fx1 >= 0.f && fy1 >= 0.f && fx0 <= cam.width - 1 && fy0 <= cam.height - 1;
            if (vis) {
                rx0 = static_cast<int>(fmaxf(fx0, 0.f));
                ry0 = static_cast<int>(fmaxf(fy0, 0.f));
                rx1 = static_cast<int>(fminf(fx1, static_cast<float>(cam.width - 1)));
                ry1 = static_cast<int>(fminf(fy1, static_cast<float>(cam.height - 1)));
                const Ellipse e = make_ellipse(mx, my, A, B, C, thr);
                const int2 rows = ellipse_rows(e, cam.height, cam.tiles_y);
                for (int tyi = rows.x; tyi <= rows.y; ++tyi) {
                    const int2 t = ellipse_row_tiles(e, tyi, cam.width, cam.height, cam.tiles_x);
                    touched += static_cast<uint32_t>(max(t.y - t.x + 1, 0));
                }
                vis = touched > 0;
            }
        }
    }

    // colour from the staged SH rows
    float3 col = make_float3(0.f, 0.f, 0.f);
    if (any_near) {
        if (stage) stage_sh_end(sh, src, nfl, staged, lane);
        if (vis) {
            float dx = px - __ldg(P.cam_pos), dy = py - __ldg(P.cam_pos + 1), dz = pz - __ldg(P.cam_pos + 2);
            const float inv_len = rsqrtf(dx * dx + dy * dy + dz * dz);
            dx *= inv_len;
            dy *= inv_len;
            dz *= inv_len;
            float bas[16];
            sh_basis(dx, dy, dz, cam.active_sh_bases, bas);
            col.x = bas[0] * P.sh0[3 * i] + 0.5f;
            col.y = bas[0] * P.sh0[3 * i + 1] + 0.5f;
            col.z = bas[0] * P.sh0[3 * i + 2] + 0.5f;
            const float* mine = sh + lane * rest3;
#pragma unroll
            for (int k = 1; k < 16; ++k) {  // unrolled, so bas stays in registers
                if (k < cam.active_sh_bases && k <= cam.rest_bases) {
                    col.x += bas[k] * mine[3 * (k - 1)];
                    col.y += bas[k] * mine[3 * (k - 1) + 1];
                    col.z += bas[k] * mine[3 * (k - 1) + 2];
                }
            }
        }
    }
    if (!valid) return;
    pb.n_touched[i] = touched;
    pb.ids[i] = static_cast<uint32_t>(i);
    // order-preserving bits of the depth (z > 0 in practice, negative z handled too); not visible = last
    const uint32_t zb = __float_as_uint(zc);
    pb.depth_key[i] = vis ? ((zb & 0x80000000u) ? ~zb : (zb | 0x80000000u)) : 0xffffffffu;
    if (!vis) return;
    pb.mean2d[i] = make_float2(mx, my);
    pb.conic_o[i] = make_float4(A, B, C, o);
    pb.color_z[i] = make_float4(col.x, col.y, col.z, zc);
    pb.rect[i] = make_ushort4(static_cast<unsigned short>(rx0), static_cast<unsigned short>(ry0),
                              static_cast<unsigned short>(rx1), static_cast<unsigned short>(ry1));
    pb.thr[i] = thr;
}

// M = the sum of the listed-tile counts, one atomic per block (its own counter word, counters[3]).
constexpr int kCountThreads = 256;
constexpr int kCountItems = 16;
__global__ void __launch_bounds__(kCountThreads) k_count_instances(const uint32_t* __restrict__ n_touched, int n,
                                                                   uint32_t* __restrict__ total) {
    __shared__ uint32_t s_warp[kCountThreads / 32];
    const long long base = static_cast<long long>(blockIdx.x) * kCountThreads * kCountItems;
    uint32_t sum = 0u;
#pragma unroll
    for (int k = 0; k < kCountItems; ++k) {
        const long long i = base + k * kCountThreads + threadIdx.x;
        if (i < n) sum += n_touched[i];
    }
    sum = __reduce_add_sync(kFullMask, sum);
    if ((threadIdx.x & 31) == 0) s_warp[threadIdx.x >> 5] = sum;
    __syncthreads();
    if (threadIdx.x == 0) {
        uint32_t t = 0u;
#pragma unroll
        for (int w = 0; w < kCountThreads / 32; ++w) t += s_warp[w];
        if (t) atomicAdd(total, t);
    }
}

#ifndef SPLAT_DUP_THREADS
#define SPLAT_DUP_THREADS 256
#endif
constexpr int kDupThreads = SPLAT_DUP_THREADS;
#ifndef SPLAT_DUP_STAGE
#define SPLAT_DUP_STAGE 2048
#endif
constexpr int kDupStage = SPLAT_DUP_STAGE;  // instances of a block staged in shared memory (8 B each)
#ifndef SPLAT_DUP_WARP_MIN
#define SPLAT_DUP_WARP_MIN 24
#endif
constexpr int kDupWarpMin = SPLAT_DUP_WARP_MIN;  // Gaussians listed in more tiles are enumerated by their warp

// Instance `slot` of the block (counted from the block's first output slot `base`): staged in shared memory
// when it fits, else written straight to global memory.
// cap: the instance buffer's capacity; slots at or past it are not written (a bounded render whose count exceeded
// its capacity, which k_check_capacity flags).
__device__ __forceinline__ void put_instance(uint32_t* s_key, uint32_t* s_val, const InstBuffers& ib,
                                             uint32_t base, uint32_t slot, uint32_t key, uint32_t id, uint32_t cap) {
    if (slot < kDupStage) {
        s_key[slot] = key;
        s_val[slot] = id;
    } else if (base + slot < cap) {
        ib.keys[base + slot] = key;
        ib.vals[base + slot] = id;
    }
}

// One (tile, id) per listed tile, Gaussians taken in (depth, id) order so that the stable tile sort that
// follows completes the LSD sort of the 64-bit (tile << 32 | depth) keys. Never more than the counted
// n_touched per Gaussian (a shortfall, which the shared row test rules out, is padded past the last tile).
// The 256 Gaussians of a block (consecutive in depth order) own one contiguous range of instance slots,
// so their instances are assembled in shared memory and stored with coalesced writes. A Gaussian listed in
// at most kDupWarpMin tiles is enumerated by its own thread; a larger one by its whole warp, lane per tile
// row, then lane per instance - the same rows and tiles in the same order.
__global__ void __launch_bounds__(kDupThreads) k_duplicate(int n, Cam cam, PrimBuffers pb, InstBuffers ib,
                                                            uint32_t cap) {
    __shared__ uint32_t s_key[kDupStage > 0 ? kDupStage : 1];
    __shared__ uint32_t s_val[kDupStage > 0 ? kDupStage : 1];
    const int lane = threadIdx.x & 31;
    const int r0 = blockIdx.x * kDupThreads;  // < n: the grid covers n
    const int r = r0 + threadIdx.x;
    const uint32_t pad_key = static_cast<uint32_t>(cam.tiles_x * cam.tiles_y);
    const uint32_t base = pb.offsets[r0];
    const uint32_t end = r0 + kDupThreads < n ? pb.offsets[r0 + kDupThreads] : pb.counters[0];

    uint32_t id = 0u, cnt = 0u, slot = 0u;
    Ellipse e{};
    if (r < n) {
        // the tile count is the step of the scanned offsets (no gather of n_touched), and the listing threshold
        // is recomputed from the opacity exactly as k_preprocess computed it, so the only gathers by id are the
        // two that the ellipse needs
        id = min(pb.order[r], static_cast<uint32_t>(n - 1));
        const uint32_t off = pb.offsets[r];
        cnt = (r + 1 < n ? pb.offsets[r + 1] : pb.counters[0]) - off;
        slot = off - base;
        if (cnt > 0u) {
            const float2 m = pb.mean2d[id];
            const float4 co = pb.conic_o[id];
            e = make_ellipse(m.x, m.y, co.x, co.y, co.z, logf(255.f * co.w));
        }
    }
    if (cnt > 0u && cnt <= static_cast<uint32_t>(kDupWarpMin)) {
        uint32_t k = 0u;
        const int2 rows = ellipse_rows(e, cam.height, cam.tiles_y);
        for (int ty = rows.x; ty <= rows.y && k < cnt; ++ty) {
            const int2 t = ellipse_row_tiles(e, ty, cam.width, cam.height, cam.tiles_x);
            for (int tx = t.x; tx <= t.y && k < cnt; ++tx, ++k)
                put_instance(s_key, s_val, ib, base, slot + k, static_cast<uint32_t>(ty * cam.tiles_x + tx), id, cap);
        }
        for (; k < cnt; ++k) put_instance(s_key, s_val, ib, base, slot + k, pad_key, id, cap);
    }
    unsigned big = __ballot_sync(kFullMask, cnt > static_cast<uint32_t>(kDupWarpMin));
    while (big) {
        const int src = __ffs(big) - 1;
        big &= big - 1u;
        Ellipse g;
        g.mx = __shfl_sync(kFullMask, e.mx, src);
        g.my = __shfl_sync(kFullMask, e.my, src);
        g.A = __shfl_sync(kFullMask, e.A, src);
        g.B = __shfl_sync(kFullMask, e.B, src);
        g.R = __shfl_sync(kFullMask, e.R, src);
        g.D = __shfl_sync(kFullMask, e.D, src);
        g.ey = __shfl_sync(kFullMask, e.ey, src);
        g.s = __shfl_sync(kFullMask, e.s, src);
        g.inv_a = __shfl_sync(kFullMask, e.inv_a, src);
        const uint32_t gid = __shfl_sync(kFullMask, id, src);
        const uint32_t gcnt = __shfl_sync(kFullMask, cnt, src);
        const uint32_t gslot = __shfl_sync(kFullMask, slot, src);
        const int2 rows = ellipse_rows(g, cam.height, cam.tiles_y);
        uint32_t k = 0u;  // instances written so far (warp-uniform)
        for (int ty0 = rows.x; ty0 <= rows.y && k < gcnt; ty0 += 32) {
            const int ty = ty0 + lane;
            int2 t = make_int2(1, 0);
            if (ty <= rows.y) t = ellipse_row_tiles(g, ty, cam.width, cam.height, cam.tiles_x);
            const uint32_t c = t.y >= t.x ? static_cast<uint32_t>(t.y - t.x + 1) : 0u;
            uint32_t incl = c;  // inclusive prefix of the row counts over the lanes
#pragma unroll
            for (int o = 1; o < 32; o <<= 1) {
                const uint32_t v = __shfl_up_sync(kFullMask, incl, o);
                if (lane >= o) incl += v;
            }
            const uint32_t chunk = __shfl_sync(kFullMask, incl, 31);
            for (uint32_t j0 = 0u; j0 < chunk; j0 += 32u) {
                const uint32_t j = j0 + lane;
                int owner = 0;  // first lane whose inclusive count exceeds j
#pragma unroll
                for (int step = 16; step > 0; step >>= 1) {
                    const uint32_t v = __shfl_sync(kFullMask, incl, owner + step - 1);
                    if (v <= j) owner += step;
                }
                const uint32_t before = __shfl_sync(kFullMask, incl, owner > 0 ? owner - 1 : 0);
                const int tx0 = __shfl_sync(kFullMask, t.x, owner);
                if (j < chunk && k + j < gcnt) {
                    const uint32_t row_start = owner > 0 ? before : 0u;
                    const uint32_t key = static_cast<uint32_t>((ty0 + owner) * cam.tiles_x + tx0) + (j - row_start);
                    put_instance(s_key, s_val, ib, base, gslot + k + j, key, gid, cap);
                }
            }
            k += min(chunk, gcnt - k);
        }
        for (uint32_t p = k + lane; p < gcnt; p += 32u) put_instance(s_key, s_val, ib, base, gslot + p, pad_key, gid, cap);
    }
    __syncthreads();
    const uint32_t staged = min(end - base, static_cast<uint32_t>(kDupStage));
    for (uint32_t j = threadIdx.x; j < staged && base + j < cap; j += kDupThreads) {
        ib.keys[base + j] = s_key[j];
        ib.vals[base + j] = s_val[j];
    }
}

// Tile ranges from the sorted tile keys without reading every key: warp t finds lb[t], the first list position
// whose key is >= t (t in [0, T]; keys lie in [0, T], T being the pad key), by a 32-ary search. Each round its
// lanes probe 32 cut points of the interval that holds the answer; the keys are sorted, so the probes below t
// form a prefix of the lanes and one ballot leaves the stretch between the last of them and the first probe at
// or above t (six rounds at 12M instances).
constexpr int kBoundsThreads = 256;

__global__ void __launch_bounds__(kBoundsThreads) k_tile_bounds(const uint32_t* __restrict__ keys, int m, int T,
                                                                uint32_t* __restrict__ lb,
                                                                const uint32_t* __restrict__ m_dev) {
    const int t = (blockIdx.x * kBoundsThreads + threadIdx.x) >> 5;
    const int lane = threadIdx.x & 31;
    if (t > T) return;  // whole warps
    if (m_dev) m = static_cast<int>(min(static_cast<long long>(m), static_cast<long long>(*m_dev)));
    int lo = 0, hi = m;  // lb[t] lies in [lo, hi]
    while (hi > lo) {
        const long long len = hi - lo;
        const int p = lo + static_cast<int>(len * (lane + 1) / 33);  // in [lo, hi), non-decreasing in lane
        const unsigned below = __ballot_sync(kFullMask, keys[p] < static_cast<uint32_t>(t));
        const int c = __popc(below);
        const int p_last = __shfl_sync(kFullMask, p, c > 0 ? c - 1 : 0);
        const int p_next = __shfl_sync(kFullMask, p, c < 32 ? c : 31);
        if (c > 0) lo = p_last + 1;
        if (c < 32) hi = p_next;
    }
    if (lane == 0) lb[t] = static_cast<uint32_t>(lo);
}

constexpr int kTableThreads = 1024;
constexpr int kTableItems = 8;                             // tiles per thread in one scan chunk
constexpr int kTableChunk = kTableThreads * kTableItems;  // tiles per scan chunk
constexpr int kTableTiles = 256;                           // tiles whose tables one block writes

__device__ __forceinline__ uint32_t table_block_scan(uint32_t v, uint32_t* s_warp, uint32_t& total) {
    const int lane = threadIdx.x & 31, warp = threadIdx.x >> 5;
    uint32_t inc = v;
#pragma unroll
    for (int o = 1; o < 32; o <<= 1) {
        const uint32_t u = __shfl_up_sync(kFullMask, inc, o);
        if (lane >= o) inc += u;
    }
    if (lane == 31) s_warp[warp] = inc;
    __syncthreads();
    if (warp == 0) {
        const uint32_t w = s_warp[lane];  // kTableThreads / 32 == 32 warps
        uint32_t wi = w;
#pragma unroll
        for (int o = 1; o < 32; o <<= 1) {
            const uint32_t u = __shfl_up_sync(kFullMask, wi, o);
            if (lane >= o) wi += u;
        }
        s_warp[lane] = wi - w;
        if (lane == 31) s_warp[32] = wi;
    }
    __syncthreads();
    const uint32_t res = inc - v + s_warp[warp];
    total = s_warp[32];
    __syncthreads();
    return res;
}

// Per-tile tables from lb: ranges (empty tiles get (0, 0)), buckets per tile, first bucket of each tile (the
// exclusive prefix, whose total goes to *total_buckets), and the bucket -> tile table. Block b writes the tables
// of tiles [256 b, 256 b + 256): it scans the bucket counts of every tile before the end of its share (8192 tiles
// per chunk, one chunk for a 1080p view), then its warps write the bucket -> tile entries of its tiles, one tile
// per warp with the lanes on consecutive buckets. The bucket outputs may be null (render-only path).
__global__ void __launch_bounds__(kTableThreads) k_tile_tables(const uint32_t* __restrict__ lb, int T, long long bcap,
                                                               uint2* __restrict__ ranges, uint32_t* __restrict__ nb,
                                                               uint32_t* __restrict__ bstart,
                                                               uint32_t* __restrict__ bucket_tile,
                                                               uint32_t* __restrict__ total_buckets) {
    static_assert(kTableThreads == 32 * 32, "table_block_scan takes 32 warps");
    __shared__ uint32_t s_warp[33];
    __shared__ uint32_t s_first[kTableTiles];
    __shared__ uint32_t s_count[kTableTiles];
    const int t0 = blockIdx.x * kTableTiles;
    const int t1 = min(t0 + kTableTiles, T);
    uint32_t carry = 0u;
    for (int c0 = 0; c0 < t1; c0 += kTableChunk) {
        const int tb = c0 + threadIdx.x * kTableItems;
        uint32_t b[kTableItems + 1];
#pragma unroll
        for (int k = 0; k <= kTableItems; ++k) b[k] = tb + k <= T ? lb[tb + k] : 0u;
        uint32_t nbk[kTableItems];
        uint32_t sum = 0u;
#pragma unroll
        for (int k = 0; k < kTableItems; ++k) {
            const uint32_t cnt = tb + k < T ? b[k + 1] - b[k] : 0u;
            nbk[k] = (cnt + kBucket - 1) / kBucket;
            sum += nbk[k];
        }
        uint32_t total;
        uint32_t run = table_block_scan(sum, s_warp, total) + carry;
#pragma unroll
        for (int k = 0; k < kTableItems; ++k) {
            const int t = tb + k;
            if (t >= t0 && t < t1) {
                ranges[t] = b[k + 1] > b[k] ? make_uint2(b[k], b[k + 1]) : make_uint2(0u, 0u);
                if (nb) {
                    nb[t] = nbk[k];
                    bstart[t] = run;
                }
                s_first[t - t0] = run;
                s_count[t - t0] = nbk[k];
            }
            run += nbk[k];
        }
        carry += total;
    }
    if (t1 == T && threadIdx.x == 0) {  // the last block has scanned every tile
        if (nb) {
            nb[T] = 0u;
            bstart[T] = carry;
        }
        if (total_buckets) *total_buckets = carry;
    }
    if (!bucket_tile) return;  // block-uniform
    __syncthreads();
    const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
    for (int j = warp; j < t1 - t0; j += kTableThreads / 32) {
        const uint32_t first = s_first[j], count = s_count[j];
        for (uint32_t k = lane; k < count; k += 32u)
            if (first + k < bcap) bucket_tile[first + k] = static_cast<uint32_t>(t0 + j);
    }
}

// One 128-thread block per 16x16 tile, two pixels per thread: each warp owns an 8x8 subtile, lane (column
// lane % 8, rows lane / 8 and lane / 8 + 4); a splat's parameters are read from shared memory once for both pixels,
// whose evaluations are independent. kTrain = false is the render-only variant: no checkpoints, per-pixel counts,
// final T, tile maxima or replay list are written (and bstart / ckpt / counters / reached may be null).
template <bool kTrain>
__global__ void __launch_bounds__(kTilePixels / 2) k_blend(Cam cam, const uint2* __restrict__ ranges,
                                                          const uint32_t* __restrict__ bstart,
                                                          const uint32_t* __restrict__ point_list,
                                                          const float2* __restrict__ mean2d,
                                                          const float4* __restrict__ conic_o,
                                                          const float4* __restrict__ color_z,
                                                          const ushort4* __restrict__ rect,
                                                          const float* __restrict__ bg, float* __restrict__ image,
                                                          float* __restrict__ final_T, uint32_t* __restrict__ n_contrib,
                                                          uint32_t* __restrict__ max_contrib,
                                                          float4* __restrict__ ckpt, uint32_t* __restrict__ counters,
                                                          uint32_t* __restrict__ reached, int n, int m, long long bcap) {
    constexpr int kThreads = kTilePixels / 2;
    __shared__ float2 s_mean[kTilePixels];
    __shared__ float4 s_con[kTilePixels];
    __shared__ float4 s_col[kTilePixels];
    __shared__ ushort4 s_rect[kTilePixels];
    __shared__ uint32_t s_max[kThreads / 32];
    __shared__ uint32_t s_reach[2];

    const int tile = blockIdx.x;
    const int tid = threadIdx.x, lane = tid & 31, warp = tid >> 5;
    const int tx0 = (tile % cam.tiles_x) * kTile, ty0 = (tile / cam.tiles_x) * kTile;
    const int sx0 = tx0 + (warp & 1) * 8, sy0 = ty0 + (warp >> 1) * 8;  // this warp's 8x8 subtile
    const int x = sx0 + (lane & 7), ya = sy0 + (lane >> 3), yb = ya + 4;
    const int local_a = (ya - ty0) * kTile + (x - tx0), local_b = local_a + 4 * kTile;
    const bool in_a = x < cam.width && ya < cam.height, in_b = x < cam.width && yb < cam.height;
    const float pxf = static_cast<float>(x) + 0.5f, pya = static_cast<float>(ya) + 0.5f, pyb = pya + 4.f;

    uint2 rg = ranges[tile];
    rg.y = min(rg.y, static_cast<uint32_t>(m));
    rg.x = min(rg.x, rg.y);
    const int count = static_cast<int>(rg.y - rg.x);
    const long long b0 = kTrain ? bstart[tile] : 0;

    float Ra = 0.f, Ga = 0.f, Ba = 0.f, Ta = 1.f, Rb = 0.f, Gb = 0.f, Bb = 0.f, Tb = 1.f;
    uint32_t last_a = 0, last_b = 0;
    bool done_a = !in_a, done_b = !in_b;
    for (int base = 0; base < count; base += kTilePixels) {
        if (__syncthreads_count(!(done_a && done_b)) == 0) break;
#pragma unroll
        for (int h = 0; h < 2; ++h) {
            const int slot = tid + h * kThreads;
            const int k = static_cast<int>(rg.x) + base + slot;
            if (k < static_cast<int>(rg.y)) {
                const int g = min(static_cast<int>(point_list[k]), n - 1);
                s_mean[slot] = mean2d[g];
                const float4 co = conic_o[g];
                s_con[slot] = make_float4(-0.5f * kLog2e * co.x, -kLog2e * co.y, -0.5f * kLog2e * co.z, co.w);
                const float4 cz = color_z[g];
                s_col[slot] = make_float4(fmaxf(cz.x, 0.f), fmaxf(cz.y, 0.f), fmaxf(cz.z, 0.f), 0.f);
                s_rect[slot] = rect[g];
            }
        }
        __syncthreads();
        const int in_batch = min(kTilePixels, count - base);
        for (int j0 = 0; j0 < in_batch; j0 += kBucket) {
            const long long bucket = b0 + ((base + j0) >> 5);
            if (kTrain && bucket < bcap) {
                ckpt[bucket * kTilePixels + local_a] = make_float4(Ra, Ga, Ba, Ta);
                ckpt[bucket * kTilePixels + local_b] = make_float4(Rb, Gb, Bb, Tb);
            }
            if (__all_sync(kFullMask, done_a && done_b)) continue;
            const int cnt = min(kBucket, in_batch - j0);
            bool hit = false;
            if (lane < cnt) {
                const ushort4 r = s_rect[j0 + lane];
                hit = r.x <= sx0 + 7 && r.z >= sx0 && r.y <= sy0 + 7 && r.w >= sy0;
            }
            unsigned pending = __ballot_sync(kFullMask, hit);
            while (pending && !(done_a && done_b)) {
                const int j = j0 + __ffs(pending) - 1;
                pending &= pending - 1;
                const float2 mm = s_mean[j];
                const float4 co = s_con[j];
                const float dx = mm.x - pxf;
                const float aa = co.w * hw_exp2(fminf(blend_q2(co.x, co.y, co.z, dx, mm.y - pya), 0.f));
                const float ab = co.w * hw_exp2(fminf(blend_q2(co.x, co.y, co.z, dx, mm.y - pyb), 0.f));
                const bool ua = !done_a && aa >= kAlphaMin, ub = !done_b && ab >= kAlphaMin;
                if (ua || ub) {
                    const float4 c = s_col[j];
                    if (ua) {
                        const float w = aa * Ta;
                        Ra += w * c.x;
                        Ga += w * c.y;
                        Ba += w * c.z;
                        Ta *= 1.f - aa;
                        last_a = static_cast<uint32_t>(base + j + 1);
                        done_a = Ta < kTMin;
                    }
                    if (ub) {
                        const float w = ab * Tb;
                        Rb += w * c.x;
                        Gb += w * c.y;
                        Bb += w * c.z;
                        Tb *= 1.f - ab;
                        last_b = static_cast<uint32_t>(base + j + 1);
                        done_b = Tb < kTMin;
                    }
                }
            }
        }
        __syncthreads();
    }
    if (kTrain) {
        const uint32_t wmax = __reduce_max_sync(kFullMask, max(last_a, last_b));
        if (lane == 0) s_max[warp] = wmax;
        __syncthreads();
        if (tid == 0) {
            uint32_t mxv = 0;
#pragma unroll
            for (int w = 0; w < kThreads / 32; ++w) mxv = max(mxv, s_max[w]);
            max_contrib[tile] = mxv;
            const uint32_t nreach = (mxv + kBucket - 1) / kBucket;
            s_reach[0] = nreach ? atomicAdd(counters + 2, nreach) : 0u;
            s_reach[1] = nreach;
        }
        __syncthreads();
        for (uint32_t i = tid; i < s_reach[1]; i += kThreads) {
            const long long slot = static_cast<long long>(s_reach[0]) + i, b = b0 + i;
            if (slot < bcap && b < bcap) reached[slot] = static_cast<uint32_t>(b);
        }
    }
    const size_t HW = static_cast<size_t>(cam.width) * cam.height;
    if (in_a) {
        const int pix = ya * cam.width + x;
        image[pix] = Ra + Ta * __ldg(bg);
        image[HW + pix] = Ga + Ta * __ldg(bg + 1);
        image[2 * HW + pix] = Ba + Ta * __ldg(bg + 2);
        if (kTrain) {
            final_T[pix] = Ta;
            n_contrib[pix] = last_a;
        }
    }
    if (in_b) {
        const int pix = yb * cam.width + x;
        image[pix] = Rb + Tb * __ldg(bg);
        image[HW + pix] = Gb + Tb * __ldg(bg + 1);
        image[2 * HW + pix] = Bb + Tb * __ldg(bg + 2);
        if (kTrain) {
            final_T[pix] = Tb;
            n_contrib[pix] = last_b;
        }
    }
}

int fill_cam(const gs3d_settings* s, Cam& cam) {
    SPLAT_REQUIRE(s != nullptr, "gs3d: settings missing");
    SPLAT_REQUIRE(s->width > 0 && s->height > 0 && s->width <= 65535 && s->height <= 65535,
                  "gs3d: image size %dx%d out of range", s->width, s->height);
    SPLAT_REQUIRE(s->active_sh_bases >= 1 && s->active_sh_bases <= 16, "gs3d: active_sh_bases %d not in [1, 16]",
                  s->active_sh_bases);
    SPLAT_REQUIRE(s->rest_bases >= 0 && s->rest_bases <= kMaxRestBases, "gs3d: rest_bases %d not in [0, 15]",
                  s->rest_bases);
    SPLAT_REQUIRE(s->fx > 0.f && s->fy > 0.f, "gs3d: focal lengths must be positive");
    SPLAT_REQUIRE(s->w2c && s->cam_position && s->bg, "gs3d: w2c, cam_position and bg are required");
    cam.fx = s->fx;
    cam.fy = s->fy;
    cam.cx = s->cx;
    cam.cy = s->cy;
    cam.near_plane = s->near_plane;
    cam.far_plane = s->far_plane;
    cam.width = s->width;
    cam.height = s->height;
    cam.tiles_x = (s->width + kTile - 1) / kTile;
    cam.tiles_y = (s->height + kTile - 1) / kTile;
    cam.active_sh_bases = s->active_sh_bases;
    cam.rest_bases = s->rest_bases;
    cam.proper_aa = s->proper_antialiasing;
    return SPLAT_OK;
}

// Duplication, the tile-digit sort passes and the per-tile tables (shared by the training and the render-only
// path; the render-only path passes no bucket outputs).
// A bounded render's count against its capacity: *overflow = 1 when the count exceeds it (the list then holds
// only the instances of the first slots).
__global__ void k_check_capacity(const uint32_t* __restrict__ count, long long capacity, uint32_t* __restrict__ overflow) {
    if (static_cast<long long>(*count) > capacity) *overflow = 1u;
}

// bounded: m is the instance buffer's capacity and the count is read on the device (pb.counters[0], the offsets
// scan's total), by the duplication, the tile sort and the tile bounds alike.
int bin_instances(int n, long long m, const Cam& cam, const PrimBuffers& pb, const TileBuffers& tb,
                  const InstBuffers& ib, long long bcap, uint32_t* bucket_tile, uint32_t* total_buckets,
                  cudaStream_t st, bool bounded = false) {
    const int T = cam.tiles_x * cam.tiles_y;
    const uint32_t* m_dev = bounded ? pb.counters : nullptr;
    if (m > 0) {
        SPLAT_TIMED_LAUNCH("k_duplicate", st, (k_duplicate<<<div_up(n, kDupThreads), kDupThreads, 0, st>>>(
                                                  n, cam, pb, ib, static_cast<uint32_t>(m))));
        note_launch();
        SPLAT_TRY(check_launch("gs3d_duplicate"));
        // the tile-digit passes (the pad key T needs bit_width(T) bits)
        const int tile_bits = bit_width(static_cast<unsigned long long>(T));
        SPLAT_TRY(radix_sort_pairs<uint32_t>(ib.keys, ib.vals, ib.keys_sorted, ib.point_list, m, 0, tile_bits,
                                             ib.sort_ws, ib.sort_bytes, st, nullptr, nullptr, m_dev));
    }
    k_tile_bounds<<<div_up(32ll * (T + 1), kBoundsThreads), kBoundsThreads, 0, st>>>(
        ib.keys_sorted, static_cast<int>(m), T, tb.lb, m_dev);
    note_launch();
    SPLAT_TRY(check_launch("gs3d_tile_bounds"));
    k_tile_tables<<<div_up(T, kTableTiles), kTableThreads, 0, st>>>(tb.lb, T, bcap, tb.ranges,
                                                                     bucket_tile ? tb.nb : nullptr,
                                                                     bucket_tile ? tb.bstart : nullptr, bucket_tile,
                                                                     total_buckets);
    note_launch();
    return check_launch("gs3d_tile_tables");
}

}  // namespace gs3d
}  // namespace splat

using namespace splat;
using namespace splat::gs3d;

extern "C" {

size_t gs3d_primitive_buffer_size(int n) { return prim_bytes(n); }
size_t gs3d_tile_buffer_size(int width, int height) { return tile_bytes(width, height); }
size_t gs3d_instance_buffer_size(long long num_instances) { return inst_bytes(num_instances); }
long long gs3d_bucket_bound(long long num_instances, int width, int height) {
    const int T = ((width + kTile - 1) / kTile) * ((height + kTile - 1) / kTile);
    return bucket_bound(num_instances, T);
}
size_t gs3d_bucket_buffer_size(long long bucket_capacity) { return bucket_bytes(bucket_capacity); }

int gs3d_preprocess_count(const float* means, const float* scales, const float* rotations, const float* opacities,
                          const float* sh0, const float* sh_rest, int n, const gs3d_settings* settings, void* prim_buf,
                          size_t prim_bytes_, uint32_t* num_instances, void* stream) {
    Cam cam;
    SPLAT_TRY(fill_cam(settings, cam));
    SPLAT_REQUIRE(n >= 0 && n < (1 << 30), "gs3d_preprocess: n=%d out of range", n);
    SPLAT_REQUIRE(prim_bytes_ >= prim_bytes(n), "gs3d_preprocess: primitive buffer too small");
    cudaStream_t st = as_stream(stream);
    Carver c(prim_buf, prim_bytes_);
    PrimBuffers pb = carve_prim(c, n);
    SPLAT_CUDA(cudaMemsetAsync(pb.counters, 0, kCounters * sizeof(uint32_t), st));
    if (n > 0) {
        Params P{means, scales, rotations, opacities, sh0, sh_rest, settings->w2c, settings->cam_position, n};
        const size_t smem = static_cast<size_t>(kPreWarps) * 32 * cam.rest_bases * 3 * sizeof(float);
        static bool configured = false;
        if (!configured) {
            SPLAT_CUDA(cudaFuncSetAttribute(k_preprocess, cudaFuncAttributeMaxDynamicSharedMemorySize,
                                            kPreWarps * 32 * kMaxRestBases * 3 * static_cast<int>(sizeof(float))));
            configured = true;
        }
        SPLAT_TIMED_LAUNCH("k_preprocess", st, (k_preprocess<<<div_up(n, kPreThreads), kPreThreads, smem, st>>>(P, cam, pb)));
        note_launch();
        SPLAT_TRY(check_launch("gs3d_preprocess"));
        k_count_instances<<<div_up(n, kCountThreads * kCountItems), kCountThreads, 0, st>>>(pb.n_touched, n,
                                                                                           pb.counters + 3);
        note_launch();
        SPLAT_TRY(check_launch("gs3d_count_instances"));
    }
    if (num_instances)
        SPLAT_CUDA(cudaMemcpyAsync(num_instances, pb.counters + 3, sizeof(uint32_t), cudaMemcpyDeviceToDevice, st));
    return SPLAT_OK;
}

int gs3d_preprocess_order(int n, void* prim_buf, size_t prim_bytes_, void* stream) {
    SPLAT_REQUIRE(n >= 0 && n < (1 << 30), "gs3d_preprocess_order: n=%d out of range", n);
    SPLAT_REQUIRE(prim_bytes_ >= prim_bytes(n), "gs3d_preprocess_order: primitive buffer too small");
    if (n == 0) return SPLAT_OK;
    cudaStream_t st = as_stream(stream);
    Carver c(prim_buf, prim_bytes_);
    PrimBuffers pb = carve_prim(c, n);
    // the depth-digit passes of the (tile << 32 | depth) key sort, on the Gaussians before duplication; the last
    // pass also gathers each Gaussian's tile count into depth order (the input of the offsets scan)
    SPLAT_TRY(radix_sort_pairs<uint32_t>(pb.depth_key, pb.ids, pb.depth_key_sorted, pb.order, n, 0, 32, pb.sort_ws,
                                         pb.sort_bytes, st, pb.n_touched, pb.offsets));
    return scan_exclusive_u32(pb.offsets, pb.offsets, n, pb.counters, pb.scan_ws, pb.scan_bytes, st);
}

int gs3d_preprocess(const float* means, const float* scales, const float* rotations, const float* opacities,
                    const float* sh0, const float* sh_rest, int n, const gs3d_settings* settings, void* prim_buf,
                    size_t prim_bytes_, uint32_t* num_instances, void* stream) {
    SPLAT_TRY(gs3d_preprocess_count(means, scales, rotations, opacities, sh0, sh_rest, n, settings, prim_buf,
                                    prim_bytes_, num_instances, stream));
    return gs3d_preprocess_order(n, prim_buf, prim_bytes_, stream);
}

int gs3d_render(int n, long long num_instances, const gs3d_settings* settings, void* prim_buf, size_t prim_bytes_,
                void* tile_buf, size_t tile_bytes_, void* inst_buf, size_t inst_bytes_, void* bucket_buf,
                size_t bucket_bytes_, long long bucket_capacity, float* image, void* stream) {
    Cam cam;
    SPLAT_TRY(fill_cam(settings, cam));
    const long long m = num_instances;
    const int T = cam.tiles_x * cam.tiles_y;
    SPLAT_REQUIRE(n >= 0 && m >= 0, "gs3d_render: bad sizes n=%d M=%lld", n, m);
    SPLAT_BOUND(m < (1ll << 31), "gs3d_render: %lld instances exceed the 2^31 the 32-bit lists index", m);
    SPLAT_BOUND(bucket_capacity >= bucket_bound(m, T),
                "gs3d_render: bucket capacity %lld is below the bound %lld for %lld instances in %d tiles",
                bucket_capacity, bucket_bound(m, T), m, T);
    SPLAT_REQUIRE(n > 0 || m == 0, "gs3d_render: instances without Gaussians");
    SPLAT_REQUIRE(prim_bytes_ >= prim_bytes(n) && tile_bytes_ >= tile_bytes(cam.width, cam.height) &&
                      inst_bytes_ >= inst_bytes(m) && bucket_bytes_ >= bucket_bytes(bucket_capacity),
                  "gs3d_render: a buffer is smaller than its size query");
    cudaStream_t st = as_stream(stream);
    Carver cp(prim_buf, prim_bytes_), ct(tile_buf, tile_bytes_), ci(inst_buf, inst_bytes_),
        cb(bucket_buf, bucket_bytes_);
    PrimBuffers pb = carve_prim(cp, n);
    TileBuffers tb = carve_tile(ct, cam.width, cam.height);
    InstBuffers ib = carve_inst(ci, m);
    BucketBuffers bb = carve_bucket(cb, bucket_capacity);
    SPLAT_CUDA(cudaMemsetAsync(pb.counters + 2, 0, sizeof(uint32_t), st));  // k_blend counts the replayed buckets
    SPLAT_TRY(bin_instances(n, m, cam, pb, tb, ib, bucket_capacity, bb.tile, pb.counters + 1, st));
    SPLAT_TIMED_LAUNCH("k_blend", st,
                       (k_blend<true><<<T, kTilePixels / 2, 0, st>>>(
                           cam, tb.ranges, tb.bstart, ib.point_list, pb.mean2d, pb.conic_o, pb.color_z, pb.rect,
                           settings->bg, image, tb.final_T, tb.n_contrib, tb.max_contrib, bb.ckpt, pb.counters,
                           bb.reached, n < 1 ? 1 : n, static_cast<int>(m), bucket_capacity)));
    note_launch();
    return check_launch("gs3d_blend");
}

int gs3d_render_bounded(int n, long long instance_capacity, const gs3d_settings* settings, void* prim_buf,
                        size_t prim_bytes_, void* tile_buf, size_t tile_bytes_, void* inst_buf, size_t inst_bytes_,
                        void* bucket_buf, size_t bucket_bytes_, long long bucket_capacity, float* image,
                        uint32_t* overflow, void* stream) {
    Cam cam;
    SPLAT_TRY(fill_cam(settings, cam));
    const long long m = instance_capacity;
    const int T = cam.tiles_x * cam.tiles_y;
    SPLAT_REQUIRE(n >= 0 && m >= 0, "gs3d_render_bounded: bad sizes n=%d capacity=%lld", n, m);
    SPLAT_REQUIRE(overflow != nullptr, "gs3d_render_bounded: overflow word is null");
    SPLAT_BOUND(m < (1ll << 31), "gs3d_render_bounded: capacity %lld exceeds the 2^31 the 32-bit lists index", m);
    SPLAT_BOUND(bucket_capacity >= bucket_bound(m, T),
                "gs3d_render_bounded: bucket capacity %lld is below the bound %lld for %lld instances in %d tiles",
                bucket_capacity, bucket_bound(m, T), m, T);
    SPLAT_REQUIRE(prim_bytes_ >= prim_bytes(n) && tile_bytes_ >= tile_bytes(cam.width, cam.height) &&
                      inst_bytes_ >= inst_bytes(m) && bucket_bytes_ >= bucket_bytes(bucket_capacity),
                  "gs3d_render_bounded: a buffer is smaller than its size query");
    if (n == 0)  // no Gaussians (the order step wrote no count): the exact form with no instances, the background
        return gs3d_render(0, 0, settings, prim_buf, prim_bytes_, tile_buf, tile_bytes_, inst_buf, inst_bytes_,
                           bucket_buf, bucket_bytes_, bucket_capacity, image, stream);
    cudaStream_t st = as_stream(stream);
    Carver cp(prim_buf, prim_bytes_), ct(tile_buf, tile_bytes_), ci(inst_buf, inst_bytes_),
        cb(bucket_buf, bucket_bytes_);
    PrimBuffers pb = carve_prim(cp, n);
    TileBuffers tb = carve_tile(ct, cam.width, cam.height);
    InstBuffers ib = carve_inst(ci, m);
    BucketBuffers bb = carve_bucket(cb, bucket_capacity);
    k_check_capacity<<<1, 1, 0, st>>>(pb.counters, m, overflow);
    note_launch();
    SPLAT_CUDA(cudaMemsetAsync(pb.counters + 2, 0, sizeof(uint32_t), st));  // k_blend counts the replayed buckets
    SPLAT_TRY(bin_instances(n, m, cam, pb, tb, ib, bucket_capacity, bb.tile, pb.counters + 1, st, true));
    SPLAT_TIMED_LAUNCH("k_blend", st,
                       (k_blend<true><<<T, kTilePixels / 2, 0, st>>>(
                           cam, tb.ranges, tb.bstart, ib.point_list, pb.mean2d, pb.conic_o, pb.color_z, pb.rect,
                           settings->bg, image, tb.final_T, tb.n_contrib, tb.max_contrib, bb.ckpt, pb.counters,
                           bb.reached, n, static_cast<int>(m), bucket_capacity)));
    note_launch();
    return check_launch("gs3d_blend");
}

int gs3d_render_inference(int n, long long num_instances, const gs3d_settings* settings, void* prim_buf,
                          size_t prim_bytes_, void* tile_buf, size_t tile_bytes_, void* inst_buf, size_t inst_bytes_,
                          float* image, void* stream) {
    Cam cam;
    SPLAT_TRY(fill_cam(settings, cam));
    const long long m = num_instances;
    const int T = cam.tiles_x * cam.tiles_y;
    SPLAT_REQUIRE(n >= 0 && m >= 0, "gs3d_render_inference: bad sizes n=%d M=%lld", n, m);
    SPLAT_BOUND(m < (1ll << 31), "gs3d_render_inference: %lld instances exceed the 2^31 the 32-bit lists index", m);
    SPLAT_REQUIRE(n > 0 || m == 0, "gs3d_render_inference: instances without Gaussians");
    SPLAT_REQUIRE(prim_bytes_ >= prim_bytes(n) && tile_bytes_ >= tile_bytes(cam.width, cam.height) &&
                      inst_bytes_ >= inst_bytes(m),
                  "gs3d_render_inference: a buffer is smaller than its size query");
    cudaStream_t st = as_stream(stream);
    Carver cp(prim_buf, prim_bytes_), ct(tile_buf, tile_bytes_), ci(inst_buf, inst_bytes_);
    PrimBuffers pb = carve_prim(cp, n);
    TileBuffers tb = carve_tile(ct, cam.width, cam.height);
    InstBuffers ib = carve_inst(ci, m);
    SPLAT_TRY(bin_instances(n, m, cam, pb, tb, ib, 0, nullptr, nullptr, st));
    SPLAT_TIMED_LAUNCH("k_blend", st,
                       (k_blend<false><<<T, kTilePixels / 2, 0, st>>>(
                           cam, tb.ranges, nullptr, ib.point_list, pb.mean2d, pb.conic_o, pb.color_z, pb.rect,
                           settings->bg, image, nullptr, nullptr, nullptr, nullptr, nullptr, nullptr,
                           n < 1 ? 1 : n, static_cast<int>(m), 0)));
    note_launch();
    return check_launch("gs3d_blend_inference");
}

}  // extern "C"
