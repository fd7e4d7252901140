// splat2d_ref_capi.cpp - plain C entry points over the REFERENCE's own splat2d CPU code
// (phase0/csrc/macrotile/splat2d_cpu.cpp, compiled from the reference tree by oracle/build.py).
// TEST INFRASTRUCTURE: the tests and bench.py's CPU baseline call it; the product never does.
//
// Mirrors the tensor plumbing of phase0/csrc/macrotile/bindings.cpp:484-618 (SceneView / FwdOut /
// Grads filled from raw pointers), with float (is_f64 = 0) and double (is_f64 = 1) variants.
#include <stdint.h>
#include <string.h>

#include "splat2d_common.h"

namespace {

template <typename S>
splat2d::SceneView<S> view(const void* means, const void* chol, const void* opacity_logit, const void* colors,
                           const int32_t* tile_off, const int32_t* tile_ids, const int32_t* bucket_off,
                           const int32_t* bucket_tile, int num_buckets, int H, int W) {
    splat2d::SceneView<S> v;
    v.means = static_cast<const S*>(means);
    v.chol = static_cast<const S*>(chol);
    v.opacity_logit = static_cast<const S*>(opacity_logit);
    v.colors = static_cast<const S*>(colors);
    v.tile_off = tile_off;
    v.tile_ids = tile_ids;
    v.bucket_off = bucket_off;
    v.bucket_tile = bucket_tile;
    v.height = H;
    v.width = W;
    v.tiles_x = (W + splat2d::kTile - 1) / splat2d::kTile;
    v.num_tiles = v.tiles_x * ((H + splat2d::kTile - 1) / splat2d::kTile);
    v.num_buckets = num_buckets;
    return v;
}

}  // namespace

extern "C" {

void splat2d_ref_forward(int is_f64, const void* means, const void* chol, const void* opacity_logit,
                         const void* colors, const int32_t* tile_off, const int32_t* tile_ids,
                         const int32_t* bucket_off, const int32_t* bucket_tile, int num_buckets, int H, int W,
                         void* image, void* t_final, int32_t* n_contrib, int32_t* last_contrib, void* ckpt) {
    if (is_f64) {
        auto v = view<double>(means, chol, opacity_logit, colors, tile_off, tile_ids, bucket_off, bucket_tile,
                              num_buckets, H, W);
        splat2d::FwdOut<double> o{static_cast<double*>(image), static_cast<double*>(t_final), n_contrib,
                                  last_contrib, static_cast<double*>(ckpt)};
        splat2d::forward_cpu<double>(v, o);
    } else {
        auto v = view<float>(means, chol, opacity_logit, colors, tile_off, tile_ids, bucket_off, bucket_tile,
                             num_buckets, H, W);
        splat2d::FwdOut<float> o{static_cast<float*>(image), static_cast<float*>(t_final), n_contrib, last_contrib,
                                 static_cast<float*>(ckpt)};
        splat2d::forward_cpu<float>(v, o);
    }
}

void splat2d_ref_backward(int is_f64, int splat_mode, const void* grad_image, const void* means, const void* chol,
                          const void* opacity_logit, const void* colors, const int32_t* tile_off,
                          const int32_t* tile_ids, const int32_t* bucket_off, const int32_t* bucket_tile,
                          int num_buckets, int H, int W, const void* t_final, const int32_t* last_contrib,
                          const void* image, const void* ckpt, void* g_means, void* g_chol, void* g_opacity,
                          void* g_colors) {
    if (is_f64) {
        auto v = view<double>(means, chol, opacity_logit, colors, tile_off, tile_ids, bucket_off, bucket_tile,
                              num_buckets, H, W);
        splat2d::Grads<double> g{static_cast<double*>(g_means), static_cast<double*>(g_chol),
                                 static_cast<double*>(g_opacity), static_cast<double*>(g_colors)};
        if (splat_mode)
            splat2d::backward_splat_cpu<double>(v, static_cast<const double*>(grad_image),
                                                static_cast<const double*>(image), static_cast<const double*>(ckpt), g);
        else
            splat2d::backward_pixel_cpu<double>(v, static_cast<const double*>(grad_image),
                                                static_cast<const double*>(t_final), last_contrib, g);
    } else {
        auto v = view<float>(means, chol, opacity_logit, colors, tile_off, tile_ids, bucket_off, bucket_tile,
                             num_buckets, H, W);
        splat2d::Grads<float> g{static_cast<float*>(g_means), static_cast<float*>(g_chol),
                                static_cast<float*>(g_opacity), static_cast<float*>(g_colors)};
        if (splat_mode)
            splat2d::backward_splat_cpu<float>(v, static_cast<const float*>(grad_image),
                                               static_cast<const float*>(image), static_cast<const float*>(ckpt), g);
        else
            splat2d::backward_pixel_cpu<float>(v, static_cast<const float*>(grad_image),
                                               static_cast<const float*>(t_final), last_contrib, g);
    }
}

void splat2d_ref_counters(int64_t* out3) {
    const splat2d::Counters& c = splat2d::counters();
    out3[0] = c.atomic_adds;
    out3[1] = c.checkpoint_bytes;
    out3[2] = c.splat_pixel_evals;
}

void splat2d_ref_reset_counters(void) { splat2d::counters() = splat2d::Counters(); }

}  // extern "C"
