// fastergs_macro_ref.cu - C entry point around the reference's own Faster-GS blend backward
// (blend_backward_macro_cu, phase1/fastergs_macro.patch:40-314), built for sm_100a by oracle/build.py into
// oracle/_ref/fastergs_macro/. TEST INFRASTRUCTURE: a GPU comparator for the parity test of this library's
// blend backward and for timing the two side by side; the product never loads it.
//
// The kernel source is not in this repository: the build extracts the patch's added lines into
// oracle/_ref/fastergs_macro/blend_backward_macro.inc, which is included below inside the namespace the patch
// adds it to. The mode bits are the patch's (backward.cu: 2 = subtile skip, 4 = transposing warp reduction,
// 8 = 8 warps per block, else 4); the launch is one warp per bucket, as there.
#include "fastergs_ref_config.cuh"

namespace faster_gs::rasterization::kernels::backward {
#include "blend_backward_macro.inc"
}

namespace {

using faster_gs::rasterization::kernels::backward::blend_backward_macro_cu;

struct Args {
    const uint2* ranges;
    const uint* bucket_offsets;
    const uint* point_list;
    const ushort4* bounds;
    const float2* mean2d;
    const float4* conic_opacity;
    const float3* color;
    const float* grad_image;
    const float* image;
    const uint* tile_max_n_processed;
    const uint* n_processed;
    const uint* bucket_tile;
    const float4* ckpt;
    float2* grad_mean2d;
    float* grad_conic;
    float* grad_opacity;
    float3* grad_color;
    float2* grad_mean2d_abs;
    uint n_buckets, n_primitives, width, height, grid_width;
    bool proper_antialiasing;
};

template <bool kAbs, int kWarps, bool kSkip, bool kTranspose>
void launch(const Args& a, cudaStream_t st) {
    const unsigned blocks = (a.n_buckets + kWarps - 1) / kWarps;
    blend_backward_macro_cu<kAbs, kWarps, kSkip, kTranspose><<<blocks, 32 * kWarps, 0, st>>>(
        a.ranges, a.bucket_offsets, a.point_list, a.bounds, a.mean2d, a.conic_opacity, a.color, a.grad_image, a.image,
        a.tile_max_n_processed, a.n_processed, a.bucket_tile, a.ckpt, a.grad_mean2d, a.grad_conic, a.grad_opacity,
        a.grad_color, a.grad_mean2d_abs, a.n_buckets, a.n_primitives, a.width, a.height, a.grid_width,
        a.proper_antialiasing);
}

template <bool kAbs, int kWarps, bool kSkip>
void by_reduce(int mode, const Args& a, cudaStream_t st) {
    if (mode & 4)
        launch<kAbs, kWarps, kSkip, true>(a, st);
    else
        launch<kAbs, kWarps, kSkip, false>(a, st);
}

template <bool kAbs, int kWarps>
void by_skip(int mode, const Args& a, cudaStream_t st) {
    if (mode & 2)
        by_reduce<kAbs, kWarps, true>(mode, a, st);
    else
        by_reduce<kAbs, kWarps, false>(mode, a, st);
}

template <bool kAbs>
void by_warps(int mode, const Args& a, cudaStream_t st) {
    if (mode & 8)
        by_skip<kAbs, 8>(mode, a, st);
    else
        by_skip<kAbs, 4>(mode, a, st);
}

}  // namespace

extern "C" {

// The arguments of blend_backward_macro_cu in its order; bucket_offsets is the inclusive scan of buckets per
// tile (the first bucket of tile t is bucket_offsets[t - 1]). Returns the launch's cudaError_t.
int fgs_ref_blend_backward_macro(int mode, int abs_grad, const void* ranges, const void* bucket_offsets,
                                 const void* point_list, const void* bounds, const void* mean2d,
                                 const void* conic_opacity, const void* color, const float* grad_image,
                                 const float* image, const void* tile_max_n_processed, const void* n_processed,
                                 const void* bucket_tile, const void* ckpt, void* grad_mean2d, float* grad_conic,
                                 float* grad_opacity, void* grad_color, void* grad_mean2d_abs, int n_buckets,
                                 int n_primitives, int width, int height, int grid_width, int proper_antialiasing,
                                 void* stream) {
    if (n_buckets <= 0) return 0;
    Args a{static_cast<const uint2*>(ranges), static_cast<const uint*>(bucket_offsets),
           static_cast<const uint*>(point_list), static_cast<const ushort4*>(bounds),
           static_cast<const float2*>(mean2d), static_cast<const float4*>(conic_opacity),
           static_cast<const float3*>(color), grad_image, image, static_cast<const uint*>(tile_max_n_processed),
           static_cast<const uint*>(n_processed), static_cast<const uint*>(bucket_tile),
           static_cast<const float4*>(ckpt), static_cast<float2*>(grad_mean2d), grad_conic, grad_opacity,
           static_cast<float3*>(grad_color), static_cast<float2*>(grad_mean2d_abs), static_cast<uint>(n_buckets),
           static_cast<uint>(n_primitives), static_cast<uint>(width), static_cast<uint>(height),
           static_cast<uint>(grid_width), proper_antialiasing != 0};
    cudaStream_t st = static_cast<cudaStream_t>(stream);
    if (abs_grad)
        by_warps<true>(mode, a, st);
    else
        by_warps<false>(mode, a, st);
    return static_cast<int>(cudaGetLastError());
}

}  // extern "C"
