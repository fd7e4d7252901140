/* splat_b200.h - C ABI of libsplat_b200.so, the B200 (sm_100a) Gaussian-splatting rasterizer.
 *
 * Conventions shared by every entry point:
 *   - all array arguments are DEVICE pointers (cudaMalloc'd or torch-owned), contiguous, in the
 *     dtype the name says; sizes are plain ints; no torch or CUDA types appear in the signatures
 *   - `stream` is a cudaStream_t passed as void* (NULL = legacy default stream); every launch goes
 *     on that stream and no entry point synchronises with the host
 *   - the return value is a status: SPLAT_OK (0) or one of the SPLAT_ERR_* codes; a failing call
 *     leaves a one-line message that splat_last_error() returns (thread-local)
 *   - entry points never launch a grid of zero blocks; empty inputs return SPLAT_OK with outputs
 *     zero-filled where the reference returns zeros
 *   - outputs are written, not accumulated: gradient buffers are cleared by the call itself
 *   - `workspace` buffers are caller-owned scratch of at least the queried size
 *
 * Each declaration names the reference interface it replaces (asadrizvi64/3dgs-project, path:line).
 */
#ifndef SPLAT_B200_H
#define SPLAT_B200_H

#include <stddef.h>
#include <stdint.h>

#ifdef __cplusplus
extern "C" {
#endif

#define SPLAT_ABI_VERSION 2

#define SPLAT_OK 0
#define SPLAT_ERR_ARG 1      /* bad shape, size or pointer */
#define SPLAT_ERR_CUDA 2     /* a CUDA call or launch failed */
#define SPLAT_ERR_OVERFLOW 3 /* a size bound was exceeded */
#define SPLAT_ERR_TIMEOUT 4  /* a bounded device-side wait gave up */

/* Message of the last failing call on this thread ("" if none). */
const char* splat_last_error(void);
/* SPLAT_ABI_VERSION of the loaded library. */
int splat_abi_version(void);
/* Kernels this library has launched in this process so far (all threads and devices). No counterpart in
 * the reference; benchmarks read it before and after a timed region. */
long long splat_launch_count(void);
/* Kernel timing for benchmarks (no counterpart in the reference): until called again for the same kernel, the
 * library records begin_event just before and end_event just after every launch of `kernel`, on the stream it
 * launches on (cudaEvent_t handles created by the caller, passed as void*; NULL events stop the timing). Kernels:
 * "k_preprocess", "k_duplicate", "k_blend" (training and render-only forward), "k_blend_backward",
 * "k_preprocess_backward", "k_adam", "gs2d_k_render" (gs2d forward), "gs2d_k_backward_splat". At most four
 * kernels at once. The events are re-recorded by every launch: read them before the kernel runs again. */
int splat_time_kernel(const char* kernel, void* begin_event, void* end_event);

/* ---------------------------------------------------------------------------------------------
 * Device-wide primitives (replace the CUB DeviceScan / DeviceRadixSort calls inside Faster-GS's
 * forward, whose call sites phase2/fastergs_readback.patch:46-89 shows)
 * ------------------------------------------------------------------------------------------- */
size_t splat_scan_workspace_size(long long n);
/* out[i] = sum(in[0..i)); *total (device, may be NULL) = sum of all n. in and out may alias. */
int splat_scan_exclusive_u32(const uint32_t* in, uint32_t* out, long long n, uint32_t* total, void* workspace,
                             size_t workspace_bytes, void* stream);
/* Exclusive scan that allocates nothing (no counterpart in the reference, whose entry points all take their
 * scratch from PyTorch's caching allocator). Same results as splat_scan_exclusive_u32, without the workspace:
 * its block sums live in one fixed device array of this library, SPLAT_SCAN_NOALLOC_MAX_N / 4096 uint32
 * (256 KiB) per device. For callers that cannot allocate device memory: a host that holds only the input and
 * output pointers and no device allocator (a C, cgo or JNI host driving buffers another framework owns), a
 * process whose device memory is already fully reserved, and callers on a latency-critical stream, where
 * cudaMalloc / cudaFree would synchronise the device.
 *  - n > SPLAT_SCAN_NOALLOC_MAX_N returns SPLAT_ERR_OVERFLOW before any launch.
 *  - The first call on each device looks up the array's address (cudaGetSymbolAddress on the current
 *    device, which must be the device of in, out and stream); make that first call before any stream capture.
 *    Every call checks that in, out and total are device memory of the current device (or managed memory)
 *    and returns SPLAT_ERR_ARG before any launch otherwise.
 *  - Every call on a device uses the same array. Nothing in it has to start at zero (each call writes every
 *    block sum it reads), but calls whose executions overlap in time (other streams, other host threads)
 *    race on it and give wrong results: serialise them. */
#define SPLAT_SCAN_NOALLOC_MAX_N (1LL << 28)
int splat_scan_exclusive_u32_noalloc(const uint32_t* in, uint32_t* out, long long n, uint32_t* total, void* stream);
size_t splat_sort_workspace_size(long long n, int key_bytes);
/* Stable LSD radix sort of (key, uint32 value) pairs by key bits [begin_bit, end_bit); key_bytes 4 or 8,
 * n < 2^30. Inputs are left untouched; outputs must not alias them. Its per-digit passes wait (bounded) on
 * counts published by earlier blocks of the same launch; see splat_check_device_waits. */
int splat_radix_sort_pairs(const void* keys_in, const uint32_t* vals_in, void* keys_out, uint32_t* vals_out,
                           long long n, int key_bytes, int begin_bit, int end_bit, void* workspace,
                           size_t workspace_bytes, void* stream);
/* SPLAT_ERR_TIMEOUT if a bounded device-side wait on the current device gave up since the last call
 * (about a second of polling without progress: the device stalled; the sorts themselves stay exact, their
 * tiles having recounted their offsets from the keys), else SPLAT_OK. Synchronises the device; clears the count.
 * No counterpart in the reference (CUB's single-sweep sort waits without a bound). */
int splat_check_device_waits(void);
/* Failure-detection hook (no counterpart in the reference): sets the number of empty polls after which a
 * radix-sort look-back wait gives up (default 2^20, about a second of back-off) and returns the previous value,
 * or -1 for polls < 1. A tiny limit makes waits give up on purpose, so that tests see SPLAT_ERR_TIMEOUT from
 * splat_check_device_waits; a tile whose wait gave up counts the earlier tiles' digits from the keys instead
 * (slow but exact), so the sort's result stays right. */
int splat_set_lookback_poll_limit(int polls);
/* The same count without a synchronisation: enqueues on `stream` a copy of it into dst (device uint32) and
 * clears it, so a caller that reads dst at a point where it waits anyway learns of a wait that gave up in
 * the work enqueued before. No counterpart in the reference. */
int splat_take_device_waits_async(uint32_t* dst, void* stream);

/* ---------------------------------------------------------------------------------------------
 * gs2d: toy2d 2D Gaussian rasterizer (replaces toy2d/csrc/rasterize.cu:366-454 and the device
 * binning of toy2d/gs2d/binning.py:35-88). means f32[N,2], conic f32[N,3] (A,B,C), color f32[N,3],
 * opacity f32[N], bg f32[3] (device: no host copy, unlike rasterize.cu:360-364). num_instances = M is
 * the length of point_list; ranges and ids are clamped to [0, M] and [0, N) on the device, so an
 * inconsistent table gives wrong pixels but never an out-of-bounds access.
 * ------------------------------------------------------------------------------------------- */
size_t gs2d_bin_count_workspace_size(int n);
size_t gs2d_bin_fill_workspace_size(long long num_instances, int H, int W);
/* Binning phase 1 (binning.py:44-67): rect i32[N,4] (xmin, ymin, xmax, ymax in tiles, max exclusive),
 * order i64[N] (stable depth argsort; depth is f32[N] or f64[N] when depth_is_f64), and the number of
 * (tile, Gaussian) instances M written to *num_instances (device u32). radii i32[N]. */
int gs2d_bin_count(const float* means, const int32_t* radii, const void* depth, int depth_is_f64, int n, int H,
                   int W, int32_t* rect, int64_t* order, uint32_t* num_instances, void* count_workspace,
                   size_t count_workspace_bytes, void* stream);
/* Binning phase 2 (binning.py:69-88), given M read back by the host and the phase-1 workspace:
 * point_list i32[M], ranges i32[T,2], bucket_offsets i32[T], bucket_to_tile i32[capacity >= M/32 + T]
 * (first num_buckets entries valid) and *num_buckets (device u32). */
int gs2d_bin_fill(const int32_t* rect, int n, int H, int W, long long num_instances, void* count_workspace,
                  size_t count_workspace_bytes, void* fill_workspace, size_t fill_workspace_bytes,
                  int32_t* point_list, int32_t* ranges, int32_t* bucket_offsets, int32_t* bucket_to_tile,
                  uint32_t* num_buckets, void* stream);
/* Binning phase 2 without a host read of M (no counterpart in the reference, which reads M and the bucket count
 * back to size its tensors): buffers sized from instance_capacity (point_list i32[instance_capacity], the fill
 * workspace from gs2d_bin_fill_workspace_size(instance_capacity, H, W)); M is read on the device from
 * *num_instances (gs2d_bin_count's output). bucket_to_tile holds bucket_capacity >= instance_capacity / 32 + T
 * entries: the first *num_buckets name their tiles, the rest -1 (so gs2d_forward / gs2d_backward_splat may be
 * given instance_capacity and bucket_capacity as the instance and bucket counts). The lists are those of
 * gs2d_bin_fill. If M > instance_capacity the lists are left empty and *overflow (device u32) is set to 1; the
 * library never clears it. */
int gs2d_bin_fill_bounded(const int32_t* rect, int n, int H, int W, long long instance_capacity,
                          const uint32_t* num_instances, void* count_workspace, size_t count_workspace_bytes,
                          void* fill_workspace, size_t fill_workspace_bytes, int32_t* point_list, int32_t* ranges,
                          int32_t* bucket_offsets, int32_t* bucket_to_tile, long long bucket_capacity,
                          uint32_t* num_buckets, uint32_t* overflow, void* stream);
/* rasterize.cu:366-394 `forward`: out f32[3,H,W], final_T f32[H,W], n_contrib i32[H,W],
 * bucket_state f32[num_buckets,256,4] = (T, C) when save_buckets (untouched entries keep the caller's
 * zero fill, as in the reference). */
int gs2d_forward(const float* means, const float* conic, const float* color, const float* opacity, const float* bg,
                 const int32_t* ranges, const int32_t* point_list, const int32_t* bucket_offsets, int N,
                 long long num_instances, int num_buckets, int H, int W, int save_buckets, float* out,
                 float* final_T, int32_t* n_contrib, float* bucket_state, void* stream);
/* rasterize.cu:396-417 `backward_pixel`: dmeans f32[N,2], dconic f32[N,3], dcolor f32[N,3], dopacity f32[N]. */
int gs2d_backward_pixel(const float* means, const float* conic, const float* color, const float* opacity,
                        const float* bg, const int32_t* ranges, const int32_t* point_list, int N,
                        long long num_instances, int H, int W, const float* final_T, const int32_t* n_contrib,
                        const float* dL_dout, float* dmeans, float* dconic, float* dcolor, float* dopacity,
                        void* stream);
/* rasterize.cu:419-448 `backward_splat` (warp per 32-splat bucket; zero gradients when num_buckets == 0). */
int gs2d_backward_splat(const float* means, const float* conic, const float* color, const float* opacity,
                        const int32_t* ranges, const int32_t* point_list, const int32_t* bucket_offsets,
                        const int32_t* bucket_to_tile, int num_buckets, int N, long long num_instances, int H,
                        int W, const float* out, const int32_t* n_contrib, const float* bucket_state,
                        const float* dL_dout, float* dmeans, float* dconic, float* dcolor, float* dopacity,
                        void* stream);

/* ---------------------------------------------------------------------------------------------
 * splat2d: phase0 2D op, float (is_f64 = 0) or double (is_f64 = 1). Replaces the extension of
 * phase0/csrc/macrotile/bindings.cpp:50-84,156-239 and the CPU binning of phase0/splat2d/ops.py:206-255.
 * means S[N,2], chol S[N,3] (l0,l1,l2), opacity_logit S[N], colors S[N,3]; CSR tile tables:
 * tile_offsets i32[T+1], tile_ids i32[M], bucket_offsets i32[T+1], bucket_tile i32[B].
 * ------------------------------------------------------------------------------------------- */
size_t splat2d_bin_count_workspace_size(int n);
size_t splat2d_bin_fill_workspace_size(long long num_instances, int H, int W);
/* ops.py:215-235: per-splat tile rect of the alpha >= 1/255 ellipse (+1 px slack), float64 math;
 * writes the instance count M to *num_instances (device u32). */
int splat2d_bin_count(int is_f64, const void* means, const void* chol, const void* opacity_logit, int n, int H,
                      int W, uint32_t* num_instances, void* count_workspace, size_t count_workspace_bytes,
                      void* stream);
/* ops.py:236-255: CSR lists (splat ids ascending within a tile), bucket tables; bucket_tile capacity
 * >= M/32 + T; *num_buckets (device u32). */
int splat2d_bin_fill(int n, int H, int W, long long num_instances, void* count_workspace,
                     size_t count_workspace_bytes, void* fill_workspace, size_t fill_workspace_bytes,
                     int32_t* tile_offsets, int32_t* tile_ids, int32_t* bucket_offsets, int32_t* bucket_tile,
                     uint32_t* num_buckets, void* stream);
/* bindings.cpp:156-178 `forward`: image S[H,W,3], t_final S[H,W], n_contrib i32[H,W] (count),
 * last_contrib i32[H,W] (position + 1), ckpt S[B,256,4] = (C, T); every checkpoint slot is written. */
int splat2d_forward(int is_f64, const void* means, const void* chol, const void* opacity_logit, const void* colors,
                    const int32_t* tile_offsets, const int32_t* tile_ids, const int32_t* bucket_offsets,
                    const int32_t* bucket_tile, int N, long long num_instances, int num_buckets, int H, int W,
                    void* image, void* t_final, int32_t* n_contrib, int32_t* last_contrib, void* ckpt,
                    void* stream);
/* bindings.cpp:180-220 `backward_pixel` (splat_mode = 0: uses t_final, last_contrib) and
 * `backward_splat` (splat_mode = 1: uses image, ckpt). grad_image S[H,W,3]; gradients S, same shapes
 * as the parameters. */
int splat2d_backward(int is_f64, int splat_mode, const void* grad_image, const void* means, const void* chol,
                     const void* opacity_logit, const void* colors, const int32_t* tile_offsets,
                     const int32_t* tile_ids, const int32_t* bucket_offsets, const int32_t* bucket_tile, int N,
                     long long num_instances, int num_buckets, int H, int W, const void* t_final,
                     const int32_t* last_contrib, const void* image, const void* ckpt, void* grad_means,
                     void* grad_chol, void* grad_opacity_logit, void* grad_colors, void* stream);
/* Op counters (bindings.cpp:222-230), counted on the device while enabled: out3 = {atomic_adds,
 * checkpoint_bytes, splat_pixel_evals}. get synchronises the device. */
int splat2d_set_counting(int on);
int splat2d_reset_counters(void);
int splat2d_get_counters(long long* out3);

/* ---------------------------------------------------------------------------------------------
 * gs3d: 3DGS rasterization, the Faster-GS `_C.forward` / `_C.backward` pair
 * (phase1/tests/test_parity.py:82-98 shows the calls; phase1/fastergs_macro.patch:403-452 and
 * upstream/upstream_main_kernels.patch:228-252 the backward's outputs). Parameters: means f32[N,3],
 * scales f32[N,3] (log), rotations f32[N,4] (w,x,y,z), opacities f32[N] (logits), sh0 f32[N,3],
 * sh_rest f32[N,rest_bases,3]. The four opaque buffers mirror Faster-GS's primitive / tile / instance /
 * bucket byte blobs; each is caller-allocated from its size query.
 * ------------------------------------------------------------------------------------------- */
typedef struct gs3d_settings {
    const float* w2c;          /* device f32[4,4], row-major world-to-camera */
    const float* cam_position; /* device f32[3] */
    const float* bg;           /* device f32[3] background colour */
    int active_sh_bases;       /* 1, 4, 9 or 16 */
    int rest_bases;            /* sh_rest.shape[1] (15 for degree 3) */
    int width;
    int height;
    float fx;
    float fy;
    float cx;
    float cy;
    float near_plane;
    float far_plane;
    int proper_antialiasing;
} gs3d_settings;

size_t gs3d_primitive_buffer_size(int n);
size_t gs3d_tile_buffer_size(int width, int height);
size_t gs3d_instance_buffer_size(long long num_instances);
/* Upper bound on the bucket count, floor((M + 31 T) / 32) + 1 (the bound of
 * phase2/tests/test_readback_equiv.py:100, for 16x16 tiles): sizes the bucket buffer without a host read. */
long long gs3d_bucket_bound(long long num_instances, int width, int height);
size_t gs3d_bucket_buffer_size(long long bucket_capacity);
size_t gs3d_backward_workspace_size(int n);
/* Forward, phase 1: projection, SH colour, conic, culling rectangle, exact listed-tile count and depth
 * per Gaussian, and the instance count M (device u32 *num_instances, may be NULL). It is
 * gs3d_preprocess_count followed by gs3d_preprocess_order. */
int gs3d_preprocess(const float* means, const float* scales, const float* rotations, const float* opacities,
                    const float* sh0, const float* sh_rest, int n, const gs3d_settings* settings, void* prim_buf,
                    size_t prim_bytes, uint32_t* num_instances, void* stream);
/* The two halves of gs3d_preprocess, so that the host can read M (written by the first) while the device
 * runs the second: the per-Gaussian preprocess and M; then the depth order of the Gaussians and the
 * instance offsets in that order (the reference's preprocess_cu + its depth sort, read back in one
 * round trip in phase2/fastergs_readback.patch:48-56). */
int gs3d_preprocess_count(const float* means, const float* scales, const float* rotations, const float* opacities,
                          const float* sh0, const float* sh_rest, int n, const gs3d_settings* settings, void* prim_buf,
                          size_t prim_bytes, uint32_t* num_instances, void* stream);
int gs3d_preprocess_order(int n, void* prim_buf, size_t prim_bytes, void* stream);
/* Forward, phase 2 (M read back by the host): duplication, 64-bit (tile | depth) key sort, tile ranges,
 * buckets, blend. image f32[3,H,W]; per-pixel final T and contributor counts stay in tile_buf. */
int gs3d_render(int n, long long num_instances, const gs3d_settings* settings, void* prim_buf, size_t prim_bytes,
                void* tile_buf, size_t tile_bytes, void* inst_buf, size_t inst_bytes, void* bucket_buf,
                size_t bucket_bytes, long long bucket_capacity, float* image, void* stream);
/* gs3d_render without the host read of M (no counterpart in the reference, whose forward reads M back to size its
 * buffers): the instance buffer is sized for instance_capacity (gs3d_instance_buffer_size(instance_capacity)) and
 * the bucket buffer for gs3d_bucket_bound(instance_capacity, ...); M is read on the device from the primitive
 * buffer (the total of gs3d_preprocess_order's offsets scan). The results are gs3d_render's when M <= capacity;
 * otherwise only the instances in the first instance_capacity slots are listed and *overflow (device u32) is set
 * to 1 (never cleared by the library). The backward takes instance_capacity and bucket_capacity as the instance and
 * bucket counts. */
int gs3d_render_bounded(int n, long long instance_capacity, const gs3d_settings* settings, void* prim_buf,
                        size_t prim_bytes, void* tile_buf, size_t tile_bytes, void* inst_buf, size_t inst_bytes,
                        void* bucket_buf, size_t bucket_bytes, long long bucket_capacity, float* image,
                        uint32_t* overflow, void* stream);
/* Render only (replaces Faster-GS's `_C.inference`, whose blend loop upstream/upstream_main_kernels.patch:131-165
 * shows): gs3d_preprocess, then this in place of gs3d_render. The same image as gs3d_render, without the
 * checkpoints, per-pixel counts and bucket tables a backward needs (no bucket buffer). */
int gs3d_render_inference(int n, long long num_instances, const gs3d_settings* settings, void* prim_buf,
                          size_t prim_bytes, void* tile_buf, size_t tile_bytes, void* inst_buf, size_t inst_bytes,
                          float* image, void* stream);
/* Backward: grad_image f32[3,H,W] -> grad_means f32[N,3], grad_scales f32[N,3], grad_rotations f32[N,4],
 * grad_opacities f32[N], grad_sh0 f32[N,3], grad_sh_rest f32[N,rest_bases,3] (zeros for Gaussians that
 * were not visible). The bucket count is read on the device, so no host sync happens.
 * densification_info f32[rows, N] (rows 0, 2 or 3; NULL when 0) is accumulated in place, as the reference's
 * backward does with its first argument: row 0 += 1 for every visible Gaussian, row 1 += |dL/dmean2d| with the
 * pixel gradient scaled by (W/2, H/2) to normalised device units, row 2 (three rows) += the same norm of the
 * per-pixel absolute mean2d gradients summed over the view. */
int gs3d_backward(const float* grad_image, const float* image, const float* means, const float* scales,
                  const float* rotations, const float* opacities, const float* sh_rest, int n, long long num_instances,
                  const gs3d_settings* settings, void* prim_buf, size_t prim_bytes, void* tile_buf,
                  size_t tile_bytes, void* inst_buf, size_t inst_bytes, void* bucket_buf, size_t bucket_bytes,
                  long long bucket_capacity, void* workspace, size_t workspace_bytes, float* grad_means,
                  float* grad_scales, float* grad_rotations, float* grad_opacities, float* grad_sh0,
                  float* grad_sh_rest, float* densification_info, int densification_rows, void* stream);
/* gs3d_backward in its two launches (the reference's _C.backward runs both back to back): the blend
 * backward accumulates the per-Gaussian 2D gradients (mean2d, conic, opacity, colour, and with three
 * densification rows the absolute mean2d gradients) into workspace, which it clears first; the preprocess
 * backward turns them into the parameter gradients and the densification rows. Called in this order on one
 * stream, with the same densification_rows, they give exactly gs3d_backward's results. */
int gs3d_backward_blend(const float* grad_image, const float* image, int n, long long num_instances,
                        const gs3d_settings* settings, void* prim_buf, size_t prim_bytes, void* tile_buf,
                        size_t tile_bytes, void* inst_buf, size_t inst_bytes, void* bucket_buf, size_t bucket_bytes,
                        long long bucket_capacity, void* workspace, size_t workspace_bytes, int densification_rows,
                        void* stream);
int gs3d_backward_preprocess(const float* means, const float* scales, const float* rotations,
                             const float* opacities, const float* sh_rest, int n, const gs3d_settings* settings,
                             void* prim_buf, size_t prim_bytes, void* workspace, size_t workspace_bytes,
                             float* grad_means, float* grad_scales, float* grad_rotations, float* grad_opacities,
                             float* grad_sh0, float* grad_sh_rest, float* densification_info,
                             int densification_rows, void* stream);
/* gs3d_backward_preprocess adding its gradients into the six outputs instead of storing them (no counterpart in
 * the reference, whose multi-view batches sum the views' gradients in autograd): the gradients of a batch's
 * views accumulate in one buffer, one view after the other on one stream. Gaussians a view does not see add
 * nothing (their zeros are not written). */
int gs3d_backward_preprocess_accumulate(const float* means, const float* scales, const float* rotations,
                                        const float* opacities, const float* sh_rest, int n,
                                        const gs3d_settings* settings, void* prim_buf, size_t prim_bytes,
                                        void* workspace, size_t workspace_bytes, float* grad_means,
                                        float* grad_scales, float* grad_rotations, float* grad_opacities,
                                        float* grad_sh0, float* grad_sh_rest, float* densification_info,
                                        int densification_rows, void* stream);
/* gs3d_backward_preprocess for the compact exchange (adam_step_dp_compact): the four non-SH gradients as
 * gs3d_backward_preprocess (accumulate = 0) or gs3d_backward_preprocess_accumulate (accumulate = 1) writes them,
 * and in place of the SH gradients six floats per Gaussian in sh_records (device f32[6n]): dL/dcolour where the
 * colour clamp passes it (0 elsewhere), then the unit view direction; zeros for a Gaussian this view does not see.
 * The records are always stored (each view of a batch has its own). */
int gs3d_backward_preprocess_records(const float* means, const float* scales, const float* rotations,
                                     const float* opacities, const float* sh_rest, int n,
                                     const gs3d_settings* settings, void* prim_buf, size_t prim_bytes,
                                     void* workspace, size_t workspace_bytes, float* grad_means, float* grad_scales,
                                     float* grad_rotations, float* grad_opacities, float* sh_records,
                                     int accumulate, float* densification_info, int densification_rows,
                                     void* stream);
/* The densification rows of gs3d_backward_preprocess alone, from the blend backward's workspace (the same
 * arithmetic, so the rows equal those gs3d_backward_preprocess accumulates). For callers that defer the
 * preprocess backward to gs3d_backward_preprocess_adam but read the statistics before the optimizer step. */
int gs3d_backward_densification(int n, const gs3d_settings* settings, void* prim_buf, size_t prim_bytes,
                                void* workspace, size_t workspace_bytes, float* densification_info,
                                int densification_rows, void* stream);
/* The preprocess backward fused with the Adam step of the six parameter tensors (no counterpart in the
 * reference, which runs `_C.backward`'s preprocess backward and then FusedAdam's `_C.adam_step` per group,
 * cluster/patches/fastergs_lean_adam.patch:251-307): each parameter gradient element is added to grad_in[g]
 * when given (the gradient other loss terms left, autograd's existing + new) and applied in place to the
 * parameter and its moments with FusedAdam's arithmetic; the gradient is never written to memory. Groups in
 * the order means, scales, rotations, opacities, sh0, sh_rest (sh_rest may be NULL when rest_bases is 0).
 * Bit-identical to gs3d_backward_preprocess followed by adam_step_multi over the six groups. No densification
 * rows (see gs3d_backward_densification). */
typedef struct gs3d_adam_state {
    float* exp_avg[6];
    float* exp_avg_sq[6];
    const float* grad_in[6]; /* may be NULL */
    double lr[6];
    int step[6]; /* t >= 1 of this update, per group */
    double beta1, beta2, eps;
} gs3d_adam_state;
int gs3d_backward_preprocess_adam(float* means, float* scales, float* rotations, float* opacities, float* sh0,
                                  float* sh_rest, int n, const gs3d_settings* settings, void* prim_buf,
                                  size_t prim_bytes, void* workspace, size_t workspace_bytes,
                                  const gs3d_adam_state* adam, void* stream);

/* ---------------------------------------------------------------------------------------------
 * Fused Adam (replaces the per-group `_C.adam_step` launches of Faster-GS's FusedAdam,
 * cluster/patches/fastergs_lean_adam.patch:251-307, with one launch over every group).
 * ------------------------------------------------------------------------------------------- */
#define SPLAT_ADAM_MAX_GROUPS 8
typedef struct adam_group {
    float* param;          /* device f32[n], updated in place */
    const float* grad;     /* device f32[n] */
    float* exp_avg;        /* device f32[n] first moment */
    float* exp_avg_sq;     /* device f32[n] second moment */
    long long n;
    double lr;
} adam_group;
/* One Adam step (step = t >= 1) over `count` groups (host array, at most SPLAT_ADAM_MAX_GROUPS). As in the
 * reference's wrapper, lr and the betas arrive in double precision for the bias corrections (step size
 * lr / (1 - beta1^t), 1 / sqrt(1 - beta2^t), computed in double and rounded once); the kernel uses their
 * float32 values. */
int adam_step_multi(int count, const adam_group* groups, int step, double beta1, double beta2, double eps,
                    void* stream);

/* Lean Adam (replaces `_C.adam_step_sparse`, cluster/patches/fastergs_lean_adam.patch:84-182, again with one
 * launch over every group). The per-element update of adam_step_multi, with two options:
 *  - visibility (device int32[n_primitives], may be NULL = every primitive): element i of a group belongs to
 *    primitive i / features; elements of primitives whose visibility is 0 keep their parameter and moments;
 *  - lowp_moments (per group): exp_avg / exp_avg_sq are bfloat16, read exactly and written with stochastic
 *    rounding - uniform noise in the 16 dropped bits, from the lowbias32 hash of ((uint32) i ^ seed) with
 *    seed = 0x9E3779B9 * step + 0x85EBCA6B for the first moment and the hash of that for the second - then
 *    truncated.
 * With visibility NULL and fp32 moments it computes exactly what adam_step_multi computes. */
typedef struct adam_lean_group {
    float* param;          /* device f32[n], updated in place */
    const float* grad;     /* device f32[n] */
    void* exp_avg;         /* device f32[n], or bf16[n] when lowp_moments */
    void* exp_avg_sq;      /* device f32[n], or bf16[n] when lowp_moments */
    long long n;
    double lr;
    int features;          /* elements per primitive, n = features * n_primitives when visibility is given */
    int lowp_moments;
} adam_lean_group;
int adam_step_multi_lean(int count, const adam_lean_group* groups, int step, double beta1, double beta2,
                         double eps, const int32_t* visibility, long long n_primitives, void* stream);

/* ---------------------------------------------------------------------------------------------
 * Data-parallel Adam over peer memory (multi-view training on one node; the reference has no multi-GPU
 * path, so none of these has a counterpart in it). Buffers that other GPUs address directly: allocated
 * with splat_peer_alloc (zeroed; ipc_handle receives 64 bytes to send to the other ranks), mapped on
 * another rank with splat_peer_open, unmapped with splat_peer_close, freed by the owner with splat_peer_free.
 * ------------------------------------------------------------------------------------------- */
int splat_peer_alloc(size_t bytes, void** ptr, unsigned char* ipc_handle);
int splat_peer_open(const unsigned char* ipc_handle, void** ptr);
int splat_peer_close(void* ptr);
int splat_peer_free(void* ptr);

#define SPLAT_DP_MAX_RANKS 8
#define SPLAT_DP_MAX_SEGMENTS 8
typedef struct dp_adam_segment {
    long long begin, end; /* element range of one parameter group in the flat vector */
    double lr;
} dp_adam_segment;
/* Rank `rank` of `world` (<= SPLAT_DP_MAX_RANKS) owns elements [lo, hi) (lo a multiple of 4 unless empty) of the flat
 * parameter vector. grads[k] / params[k] are rank k's flat gradient / parameter vectors as this GPU addresses
 * them (its own and peer mappings; 16-byte aligned). The kernel sums the slice's gradients over the ranks in
 * rank order, applies Adam (exp_avg / exp_avg_sq hold the slice's hi - lo moments; each element takes the lr
 * of its segment; bias corrections as in adam_step_multi) and stores the updated slice into every rank's
 * params. It waits on nothing: enqueue it after a device-side barrier that follows every rank's backward, and
 * enqueue a second barrier after it before any rank reads its parameters or writes its gradients again. */
int adam_step_dp_fused(int world, int rank, const float* const* grads, float* const* params, long long lo,
                       long long hi, float* exp_avg, float* exp_avg_sq, int segment_count,
                       const dp_adam_segment* segments, int step, double beta1, double beta2, double eps,
                       void* stream);

/* The same step over NVLink multicast memory (NVLS): grads_mc / params_mc are multicast addresses of the
 * flat gradient / parameter vectors (bound to every rank's buffer), params_local this rank's copy. The switch
 * sums the slice's gradients (multimem.ld_reduce) and one multicast store writes the updated slice to every
 * rank (multimem.st); lo and hi multiples of 4. Same ordering requirements as adam_step_dp_fused. */
int adam_step_dp_nvls(long long lo, long long hi, const float* grads_mc, float* params_mc, const float* params_local,
                      float* exp_avg, float* exp_avg_sq, int segment_count, const dp_adam_segment* segments, int step,
                      double beta1, double beta2, double eps, void* stream);

/* The step with compact SH gradients (no counterpart in the reference, which has no multi-GPU path): per view
 * and Gaussian a rank sends the six floats that gs3d_backward_preprocess_records stores (the colour gradient
 * and the view direction) instead of its 3 (rest_bases + 1) SH gradients, and the owner forms the products
 * basis_k(direction) * colour gradient itself, with the preprocess backward's rounding, summing a rank's views in
 * view order and the ranks in rank order: the same gradients, so the same update, as gs3d_backward_preprocess(_
 * accumulate) followed by adam_step_dp_fused, apart from the sign of zero sums (which Adam does not see).
 * Rank `rank` owns the Gaussians [lo, hi) of n (lo a multiple of 4 unless empty) and updates all their
 * parameters. Per rank k (as this GPU addresses it):
 *   params[k]: means 3n | scales 3n | rotations 4n | opacities n | sh0 3n | sh_rest 3 rest_bases n floats
 *   grads[k]:  means 3n | scales 3n | rotations 4n | opacities n | views x (6n floats of records)
 * exp_avg / exp_avg_sq: the owned Gaussians' moments in the parameter layout, with c = hi - lo rounded up to a
 * multiple of 4 in place of n. lr: six learning rates (means, scales, rotations, opacities, sh0, sh_rest); bias
 * corrections as in adam_step_multi. Same ordering requirements as adam_step_dp_fused. */
int adam_step_dp_compact(int world, int rank, const float* const* grads, float* const* params, long long n,
                         long long lo, long long hi, int views, int active_sh_bases, int rest_bases, float* exp_avg,
                         float* exp_avg_sq, const double* lr, int step, double beta1, double beta2, double eps,
                         void* stream);

/* ---------------------------------------------------------------------------------------------
 * Fused L1 + SSIM loss (the training loss around the rasterizer; replaces the external fused-ssim call of the
 * reference's trainer, whose share of the step results/phase1/README.md:46-47 reports, and the L1 term beside it).
 * img, gt: device f32[B, C, H, W]. loss = (1 - lambda) mean|img - gt| + lambda (1 - mean SSIM), SSIM with the
 * 11x11 Gaussian window (sigma 1.5), C1 = 0.01^2, C2 = 0.03^2, zero padding; padding_valid = 1 averages the
 * SSIM map only where the window lies inside the image. The forward writes loss and mean SSIM (device f32[1]
 * each, either may be NULL) and keeps in the workspace what the backward needs; the backward writes
 * grad_img = dloss/dimg times *grad_loss (device f32[1], NULL = 1). Deterministic (fixed-order sums).
 * ------------------------------------------------------------------------------------------- */
size_t splat_l1_ssim_workspace_size(int B, int C, int H, int W);
int splat_l1_ssim_forward(const float* img, const float* gt, int B, int C, int H, int W, float lambda,
                          int padding_valid, float* loss, float* ssim_mean, void* workspace, size_t workspace_bytes,
                          void* stream);
int splat_l1_ssim_backward(const float* img, const float* gt, int B, int C, int H, int W, float lambda,
                           int padding_valid, const float* grad_loss, float* grad_img, const void* workspace,
                           size_t workspace_bytes, void* stream);

#ifdef __cplusplus
}  /* extern "C" */
#endif

#endif /* SPLAT_B200_H */
