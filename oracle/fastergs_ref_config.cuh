// fastergs_ref_config.cuh - the names under which the reference's own Faster-GS blend backward
// (blend_backward_macro_cu, the lines phase1/fastergs_macro.patch:40-314 add to kernels_backward.cuh) compiles
// as a GPU comparator. TEST INFRASTRUCTURE: only tests/ load the library built from it; the product never does.
//
// Faster-GS's rasterization_config.h and the helper_math.h it includes are not part of the reference (Faster-GS
// is not vendored), so this file supplies what the kernel names:
//   * the tile shape of the benchmark spec, 16x16 pixels, with Faster-GS's 8x4 subtiles: the kernel's static
//     checks hold for it (a lane keeps one column, 8 pixels per lane, a 2-row band inside one subtile row),
//     and it then reads this library's own forward buffers as they are
//   * this library's blend thresholds: alpha = opacity G is compared with 1/255 (the "original opacity
//     interpretation"), (1 - alpha) floored at 1e-6 in the backward
//   * the float3/float4 helpers the kernel uses (dot, difference, component-wise max with a scalar, broadcast
//     and truncating constructors)
#pragma once

#include <cuda_runtime.h>

typedef unsigned int uint;

namespace faster_gs::rasterization::config {
constexpr int tile_width = 16;
constexpr int tile_height = 16;
constexpr int block_size_blend = tile_width * tile_height;
constexpr int subtile_width = 8;
constexpr int subtile_height = 4;
constexpr int subgrid_width = tile_width / subtile_width;
constexpr int macro_pixels_per_lane = block_size_blend / 32;
constexpr float min_alpha_threshold = 1.0f / 255.0f;
constexpr float one_minus_alpha_eps = 1e-6f;
constexpr bool original_opacity_interpretation = true;
}  // namespace faster_gs::rasterization::config

namespace config = faster_gs::rasterization::config;

__device__ __forceinline__ float3 make_float3(float s) { return make_float3(s, s, s); }
__device__ __forceinline__ float3 make_float3(float4 v) { return make_float3(v.x, v.y, v.z); }
__device__ __forceinline__ float3 operator-(float3 a, float3 b) { return make_float3(a.x - b.x, a.y - b.y, a.z - b.z); }
__device__ __forceinline__ float dot(float3 a, float3 b) { return a.x * b.x + a.y * b.y + a.z * b.z; }
__device__ __forceinline__ float3 fmaxf(float3 a, float b) { return make_float3(fmaxf(a.x, b), fmaxf(a.y, b), fmaxf(a.z, b)); }
