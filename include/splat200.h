/* splat200.h -- C ABI of libsplat200, the sm_100a gs3d rasteriser.
 *
 * Every function takes device pointers (float32 / int32, row-major, C
 * contiguous unless a stride argument says otherwise), plain sizes and a
 * cudaStream_t passed as void*, enqueues its kernels on that stream and
 * returns 0 on success or a negative status:
 *   -1 invalid argument, -2 CUDA error, -3 a bounded device wait gave up,
 *   -4 problem too large, -5 workspace too small.
 * splat_last_error() describes the calling thread's latest failure.  No
 * entry point allocates device memory; binning takes caller workspaces sized
 * by the *_workspace_bytes queries.
 *
 * Each entry point names the dsl_splat function whose Warp launch it
 * replaces (paths inside the dsl_splat project).
 */
#ifndef SPLAT200_H
#define SPLAT200_H

#include <stddef.h>

#ifdef __cplusplus
extern "C" {
#endif

int splat_abi_version(void);
const char* splat_last_error(void);

/* Number of CUDA kernels this library has launched in the process so far. */
unsigned long long splat_launch_count(void);

/* Reads and clears the device error word set by bounded waits (synchronises
 * the stream).  *code is 0 when no wait expired. */
int splat_device_error(int* code, void* stream);

/* No counterpart in the reference (Warp reports no device-side errors).
 * Queues, on stream, a copy of the device error word into device_dst (one
 * device int32) followed by its reset to zero; no host synchronisation, so a
 * caller can fold the word into a read it already makes.  Codes: -3 a bounded
 * wait expired, -4 a count total above INT32_MAX, -6 a guard met an
 * out-of-range index. */
int splat_device_error_read(int* device_dst, void* stream);

/* No counterpart in the reference; test support.  One thread runs the
 * decoupled look-back of tile 1 over status[0..1] (device uint32, zeroed by
 * the caller: never published) with spin_limit polls (at most 2^20): the
 * wait expires, the device error word receives -3 and the kernel returns,
 * writing the partial prefix to *out.  Shows on a GPU that an expired wait
 * ends and is reported. */
/* No counterpart in the reference (its native snippets call the C
 * library's atan2f and tanf); test support.  atan2_out[i] =
 * splat_atan2f(y[i], x[i]) and tan_out[i] = splat_tanf(x[i]), the AAA
 * preprocessing's own functions, for comparison with the CPU oracle's. */
int splat_test_trig(int n, const float* y, const float* x, float* atan2_out, float* tan_out,
                    void* stream);

int splat_test_lookback_expiry(const unsigned* status, unsigned spin_limit, unsigned* out,
                               void* stream);

/* splatting/cameras.py:29-85 _PrepareCameras.forward -> camera_kernels.py:11-66.
 * views (C,4,4), Ks (C,3,3) -> full (C,4,4), inverse/centers when
 * with_centers (C,4,4)/(C,3), errors (C) with the reference's codes
 * 1 (skewed K), 2 (non-finite or non-positive focal), 3 (singular view). */
int splat_cameras_prepare(int count, const float* views, const float* Ks, int width, int height,
                          int with_centers, float* full, float* inverse, float* centers,
                          int* errors, void* stream);

/* splatting/cameras.py:86-115 _PrepareCameras.backward -> camera_kernels.py:69-106.
 * grad_full (C,4,4) or NULL, grad_centers (C,3) or NULL -> grad_views (C,4,4). */
int splat_cameras_backward(int count, const float* Ks, const float* grad_full, int width,
                           int height, const float* inverse, const float* grad_centers,
                           float* grad_views, void* stream);

/* gs3d/projection.py:309-354 prepare -> project kernel :89-164.
 * Outputs centers (n,2), conics (n,4), radii (n), tiles (n), depths (n);
 * rows with radii == 0 leave centers/conics/depths unwritten, as the
 * reference does.  tile_mode: 0 radius, 1 snugbox, 2 accutile
 * (splatting/intersections.py:21-218); modes 1 and 2 replace tiles[i] with
 * the mode's tile count (:150-162) and keep the radius even when it is 0. */
int splat_project_forward(int n, const float* means, const float* quats, const float* scales,
                          const float* opacities, const float* view, const float* proj,
                          const float* K, int width, int height, float near_plane,
                          float far_plane, float radius_clip, float* centers, float* conics,
                          int* radii, int* tiles, float* depths, int tile_mode, void* stream);

/* gs3d/api.py:145-189 per-view preparation in one launch: the projection above,
 * the masked SH evaluation of primitives/spherical_harmonics.py:18-59
 * (sh.py:44-79; directions means - campos, campos NULL for SH0) writing
 * colors[i*color_stride + 0..2] and active (n,3), and the dense metadata of
 * splatting/metadata.py:34-70 (means2d (n,2), opacities (n), conics (n,3)).
 * sh == NULL skips SH; meta_means2d == NULL skips metadata.  normalize_quats != 0:
 * quats are raw and are normalised in-kernel with the bits of Torch's CUDA
 * F.normalize(quats, dim=-1) (inputs.py:252). */
int splat_project_forward_fused(int n, const float* means, const float* quats,
                                int normalize_quats, const float* scales,
                                const float* opacities, const float* view,
                                const float* proj, const float* K, int width, int height,
                                float near_plane, float far_plane, float radius_clip,
                                float* centers, float* conics, int* radii, int* tiles,
                                float* depths, int sh_degree, int sh_k, const float* sh,
                                const float* campos, float* colors, int color_stride,
                                unsigned char* active, float* meta_means2d,
                                float* meta_opacities, float* meta_conics, int tile_mode,
                                void* stream);

/* gs3d/api.py:132-189 (the per-camera projection loop) as one launch: the
 * Gaussian set projected for `views` cameras, each Gaussian's inputs and SH
 * row read once.  viewmats/projs (views,4,4), Ks (views,3,3), campos
 * (views,3) or NULL are stacked; outputs come through host arrays of
 * `views` device pointers (a NULL table: that output is absent), each entry
 * laid out as splat_project_forward_fused's.  Bit-identical to `views` calls
 * of splat_project_forward_fused. */
int splat_project_forward_views(int views, int n, const float* means, const float* quats,
                                int normalize_quats, const float* scales,
                                const float* opacities, const float* viewmats,
                                const float* projs, const float* Ks, int width, int height,
                                float near_plane, float far_plane, float radius_clip,
                                float* const* centers, float* const* conics, int* const* radii,
                                int* const* tiles, float* const* depths, int sh_degree,
                                int sh_k, const float* sh, const float* campos,
                                float* const* colors, int color_stride,
                                unsigned char* const* active, float* const* meta_means2d,
                                float* const* meta_opacities, float* const* meta_conics,
                                int tile_mode, void* stream);

/* splatting/metadata.py:34-70 prepare_metadata -> _prepare :12-31. */
int splat_metadata(int n, const int* radii, const float* centers, const float* conics,
                   float* means2d, float* opacities, float* conics3, void* stream);

/* gs3d/projection.py:357-428 backward -> project_backward :213-285.
 * Writes dense grads (culled rows zero; any output may be NULL).
 * camera_grads: NULL or float[32] (view 4x4 then projection 4x4) that the
 * call ADDS into (zero it first). */
int splat_project_backward(int n, const float* means, const float* quats, const float* scales,
                           const float* view, const float* proj, const float* K, int width,
                           int height, const int* radii, const float* grad_centers,
                           const float* grad_conics, float* grad_means, float* grad_quats,
                           float* grad_scales, float* grad_opacities, float* camera_grads,
                           void* stream);

/* The projection backward above fused with the SH backward of
 * primitives/spherical_harmonics.py:61-101 (sh.py:82-138): grad_colors rows
 * (stride color_stride) give dL/dcolors, the direction gradient is added to
 * grad_means and, negated, to camera_grads[32..34] (d campos).  accumulate
 * != 0 adds into all per-Gaussian outputs (multi-view sums); camera_grads is
 * NULL or float[35] (view 16, proj 16, campos 3), always added into.
 * quats_raw: NULL, or the unnormalised quaternions whose F.normalize gave
 * quats (inputs.py:252); grad_quats then receives the gradient w.r.t.
 * quats_raw (the normalisation's VJP is applied in the kernel), and quats
 * may be NULL (recomputed from quats_raw as splat_project_forward_fused
 * normalises them). */
int splat_project_backward_fused(int n, const float* means, const float* quats,
                                 const float* quats_raw, const float* scales,
                                 const float* view, const float* proj,
                                 const float* K, int width, int height, const int* radii,
                                 const float* grad_centers, const float* grad_conics,
                                 float* grad_means, float* grad_quats, float* grad_scales,
                                 float* grad_opacities, int accumulate, float* camera_grads,
                                 int sh_degree, int sh_k, const float* sh, const float* campos,
                                 const unsigned char* active, const float* grad_colors,
                                 int color_stride, float* grad_sh, void* stream);

/* The backward of splat_project_forward_views (the per-view backward calls
 * of gs3d/projection.py:357-428 + the SH VJP, summed over the views as
 * autograd sums them): Gaussian inputs and SH rows read once, each
 * gradient written once (accumulate: added).  Per-view inputs -- radii,
 * grad_centers, grad_conics, active, grad_colors -- come through host
 * arrays of `views` device pointers.  No camera gradients: use
 * splat_project_backward_fused per view for those. */
int splat_project_backward_views(int views, int n, const float* means, const float* quats,
                                 const float* quats_raw, const float* scales,
                                 const float* viewmats, const float* projs, const float* Ks,
                                 int width, int height, const int* const* radii,
                                 const float* const* grad_centers,
                                 const float* const* grad_conics, float* grad_means,
                                 float* grad_quats, float* grad_scales, float* grad_opacities,
                                 int accumulate, int sh_degree, int sh_k, const float* sh,
                                 const float* campos, const unsigned char* const* active,
                                 const float* const* grad_colors, int color_stride,
                                 float* grad_sh, void* stream);

/* primitives/spherical_harmonics.py:18-59 _SphericalHarmonics.forward -> sh.py:44-79.
 * sh (n,sh_k,3), dirs (n,3), radii (n) or NULL -> colors (n,3), active (n,3) or NULL. */
int splat_sh_forward(int n, int degree, int sh_k, const float* sh, const float* dirs,
                     const int* radii, float* colors, unsigned char* active, void* stream);

/* primitives/spherical_harmonics.py:61-101 backward -> sh.py:82-138.
 * grad_sh (n,sh_k,3) fully written; grad_dirs (n,3) or NULL. */
int splat_sh_backward(int n, int degree, int sh_k, const float* sh, const float* dirs,
                      const int* radii, const unsigned char* active, const float* upstream,
                      float* grad_sh, float* grad_dirs, void* stream);

/* primitives/tiling.py:57-64 scan_counts: inclusive int32 offsets of counts
 * (n); *total (device int64, may be NULL) receives the sum, formed in 64 bits
 * so that it never wraps.  A sum above INT32_MAX does not fit the int32
 * offsets: the device error word (splat_device_error) then reads -4 and the
 * offsets of that call are not valid. */
size_t splat_scan_workspace_bytes(int n);
int splat_scan_counts(int n, const int* counts, int* offsets, long long* total, void* workspace,
                      size_t workspace_bytes, void* stream);

/* No counterpart in the reference.  splat_scan_counts without any caller
 * scratch, for callers that cannot hand the library device memory at call
 * time (all device memory owned by the host's own pool, a render loop that
 * cannot afford cudaMalloc's implicit synchronisation, a plugin whose
 * framework forbids new allocations).  The scan's block sums live in a
 * file-scope __device__ array of 64 KiB that every GPU loading the library
 * holds until the process exits, so n is limited to 67108864 (16384 blocks
 * of 4096 counts); larger n returns -4 without launching.  Allocates
 * nothing: no cudaMalloc, no cudaFree.  The first call on a device looks up
 * the array's device address (cudaGetSymbolAddress) with that device
 * current; make that first call before any stream capture.  All calls share
 * the array, so calls that overlap on the GPU (different streams, or
 * different host threads without ordering) race; serialise them on one
 * stream.  Each call rewrites the scratch it reads, so nothing needs
 * clearing between calls.  Results are identical to splat_scan_counts,
 * including the 64-bit total and the -4 device error above INT32_MAX.  The
 * cached address belongs to the device's current context: after a
 * cudaDeviceReset in the same process, do not call this entry again. */
int splat_scan_counts_static(int n, const int* counts, int* offsets, long long* total,
                             void* stream);

/* splatting/binning.py:72-117 bin_and_sort, split in two calls around the
 * one host read of the pair count that the reference also makes
 * (primitives/tiling.py:64).  tile_mode as for the projection (conics are
 * required for modes 1 and 2; tiles must be the projection's counts for the
 * same mode):
 *   splat_bin_prepare: depth-key sort, pair offsets, per-tile ranges (T,2)
 *     (zeros for empty tiles, as identify_ranges leaves them; 8-byte
 *     aligned) and the pair count M into *pairs (device int64).
 *   splat_bin_emit: generates and sorts the M (tile, Gaussian) pairs into
 *     ids (M) -- the reference's point_list: per tile, Gaussians ordered by
 *     (float bits of depth, index), identical to the stable 64-bit key sort
 *     of primitives/tiling.py:80-86.
 * The workspace passed to prepare must be passed unchanged to emit. */
size_t splat_bin_workspace_bytes(int n, int width, int height, int tile_mode);
size_t splat_bin_pairs_workspace_bytes(long long pairs, int width, int height, int tile_mode);
int splat_bin_prepare(int n, const float* centers, const float* conics, const int* radii,
                      const int* tiles, const float* depths, int width, int height, int tile_mode,
                      void* workspace, size_t workspace_bytes, int* ranges, long long* pairs,
                      void* stream);
/* pairs: the length of ids.  Where splat_bin_pairs_workspace_bytes is 0
 * (the chunked scatter), pairs may be a capacity instead of the count
 * splat_bin_prepare returned: ids past the true count are left unwritten,
 * and pairs past a too-small capacity are dropped (emit again with the true
 * count).  Elsewhere it must be the true count. */
int splat_bin_emit(int n, long long pairs, int width, int height, int tile_mode,
                   const float* centers, const float* conics, const int* radii, void* workspace,
                   size_t workspace_bytes, void* pairs_workspace, size_t pairs_workspace_bytes,
                   int* ids, void* stream);

/* Scheduling order for the blend kernels: the T tiles by descending pair
 * count (ranges[t][1] - ranges[t][0]), written to order (T).  ranges needs
 * 8-byte alignment.  No reference counterpart (the reference launches tiles
 * in index order). */
int splat_tile_order(const int* ranges, int tiles, int* order, void* stream);

/* gs3d/render.py:359-406 render -> evaluate :41-125.  Blended channels are
 * feat_a's ch_a columns (row stride stride_a), then feat_b's ch_b columns,
 * then (append_one) a constant 1 -- the reference's cat([features, extras,
 * ones]) of gs3d/autograd.py:42-46 without materialising it.
 * background (channels).  image[pixel*pix_stride + c*ch_stride]; planar
 * (C,H,W) is pix_stride=1, ch_stride=H*W; interleaved (H,W,C) is
 * pix_stride=C, ch_stride=1.  alpha_image (H,W), when not NULL (append_one
 * only), receives the constant channel -- the alpha output -- instead of
 * image, so colour and alpha are separate dense buffers.  ids holds num_ids
 * entries (tile ranges are clamped to it) of Gaussian indices in [0, n).  At
 * most 32 channels.  tile_order: NULL, or the (T) permutation from
 * splat_tile_order -- block b then blends tile tile_order[b], so the heaviest
 * tiles start first (same outputs, shorter tail; also for the two calls
 * below). */
int splat_render_forward(int width, int height, const int* ranges, const int* ids,
                         long long num_ids, int n, const float* centers, const float* conics,
                         const float* feat_a, int ch_a, int stride_a, const float* feat_b,
                         int ch_b, int stride_b, int append_one, const float* background,
                         float* image, int pix_stride, int ch_stride, float* alpha_image,
                         float* final_t, int* contributors, const int* tile_order,
                         void* stream);

/* gs3d/render.py:129-169 render with contribution statistics (statistics.py:
 * 47-73, 393-418): as splat_render_forward, plus stat_count requests whose
 * (stat_count, H*W) pixel maps are stat_pixels; request r is a weighted sum
 * when bit r of stat_sum_mask is set, else a masked count.  Each accepted
 * sample of Gaussian g with weight w = alpha*T at a pixel whose map value v
 * is nonzero adds 1 to stat_counts[row*n + g] or v*w to stat_sums[row*n + g]
 * (row = index among requests of its kind). */
int splat_render_forward_statistics(
    int width, int height, const int* ranges, const int* ids, long long num_ids, int n,
    const float* centers, const float* conics, const float* feat_a, int ch_a, int stride_a,
    const float* feat_b, int ch_b, int stride_b, int append_one, const float* background,
    float* image, int pix_stride, int ch_stride, float* alpha_image, float* final_t,
    int* contributors, int stat_count, int stat_sum_mask, const float* stat_pixels,
    int* stat_counts, float* stat_sums, const int* tile_order, void* stream);

/* gs3d/render.py:409-463 backward -> :221-354.  Gradients are ADDED into
 * grad_centers (n,2), grad_conics (n,4), grad_a (n,ch_a), grad_b (n,ch_b)
 * and abs_centers (n,2) (NULL to skip a, b or abs); the last constant_tail
 * channels receive no feature gradient.  The upstream gradient of channel c
 * is upstream[pixel*up_pix_stride + c*up_ch_stride] (upstream NULL: zero),
 * except the appended constant channel when upstream_alpha is not NULL:
 * upstream_alpha[pixel*alpha_pix_stride]. */
int splat_render_backward(int width, int height, const int* ranges, const int* ids,
                          long long num_ids, int n, const float* centers, const float* conics,
                          const float* feat_a,
                          int ch_a, int stride_a, const float* feat_b, int ch_b, int stride_b,
                          int append_one, const float* background, const float* final_t,
                          const int* contributors, const float* upstream, int up_pix_stride,
                          int up_ch_stride, const float* upstream_alpha, int alpha_pix_stride,
                          float* grad_centers, float* grad_conics,
                          float* grad_a, float* grad_b, float* abs_centers, int constant_tail,
                          const int* tile_order, void* stream);

/* ---- RaDe-GS ----------------------------------------------------------------
 * Replaces the Warp launches of rade/projection.py:422-551 (prepare,
 * backward) and rade/render.py:550-670 (render, backward). */

/* rade/projection.py:194-260 project: as splat_project_forward, with the
 * covariance dilated by kernel_size (>= 0) and the opacity scaled by
 * rade/projection.py:50-54's coefficient; depths (n) is the radial distance
 * of the camera-space centre; planes / normals (n,3) receive the ray plane
 * and camera-space normal of every visible row.  normalize_quats: quats are
 * raw and normalised in-kernel with the bits of Torch's CUDA F.normalize
 * (inputs.py:252).  Optional, as in splat_project_forward_fused: the SH
 * colours (sh != NULL: (n,sh_k,3) coefficients of degree sh_degree on
 * directions means - campos (campos NULL: means), rade/api.py:153-165)
 * into colors (n,3) with the clamp mask into active (n,3) (may be NULL), and
 * the dense metadata (meta_means2d (n,2), meta_opacities (n), meta_conics
 * (n,3); NULL to skip, zero on culled rows). */
int splat_rade_project_forward(int n, const float* means, const float* quats,
                               int normalize_quats, const float* scales, const float* opacities,
                               const float* view, const float* proj, const float* K, int width,
                               int height, float near_plane, float far_plane, float radius_clip,
                               float kernel_size, float* centers, float* conics, int* radii,
                               int* tiles, float* depths, float* planes, float* normals,
                               int sh_degree, int sh_k, const float* sh, const float* campos,
                               float* colors, unsigned char* active, float* meta_means2d,
                               float* meta_opacities, float* meta_conics, void* stream);

/* rade/projection.py:320-398 project_backward: the VJP of projection_loss
 * (:294-317) for seeds on centers (n,2), conics (n,4), ray planes and
 * normals (n,3) (NULL: zero).  Per-Gaussian gradients (NULL to skip) are
 * WRITTEN, with zeros on culled rows; grad_quats is w.r.t. the raw
 * quaternions when normalize_quats.  grad_view / grad_proj (4,4) are
 * ACCUMULATED (NULL to skip).  With sh != NULL also the SH VJP
 * (primitives/sh.py:82-138) of the colour upstream seed_colors (n,3)
 * through the forward's clamp mask active: grad_sh (n,sh_k,3) WRITTEN,
 * the direction gradient added to grad_means and, negated, ACCUMULATED
 * into grad_campos (3) (NULL to skip). */
int splat_rade_project_backward(int n, const float* means, const float* quats,
                                int normalize_quats, const float* scales,
                                const float* opacities, const float* view, const float* proj,
                                const float* K, int width, int height, float kernel_size,
                                const int* radii, const float* seed_centers,
                                const float* seed_conics, const float* seed_planes,
                                const float* seed_normals, float* grad_means, float* grad_quats,
                                float* grad_scales, float* grad_opacities, float* grad_view,
                                float* grad_proj, int sh_degree, int sh_k, const float* sh,
                                const float* campos, const unsigned char* active,
                                const float* seed_colors, float* grad_sh, float* grad_campos,
                                void* stream);

/* rade/render.py:99-322 render / render_statistics.  Channels: colors' ch_a
 * columns (row stride stride_a) then extras' ch_b columns; background covers
 * them all.  Writes the five images of rade/render.py:38-47 RenderedPixels.
 * images(), each value of channel c at pixel p at base[p*pix + c*ch]: the C
 * features (feat_pix, feat_ch), alpha = 1 - T, expected depth, median depth
 * (one channel each) and the unit normal (normal_pix, normal_ch); the
 * reference's planar (C+6,H,W) image is pix = 1, ch = H*W at offsets 0, C,
 * C+1, C+2, C+3; channel-last images are pix = channels, ch = 1.  Also
 * auxiliary (2,H,W) = depth * ray scale, normal length; contributors (2,H,W)
 * = last and median contributor (-1 when none).  K: the (3,3) intrinsics on
 * the device.  Statistics and tile_order as splat_render_forward_statistics.
 * At most 64 channels. */
int splat_rade_render_forward(int width, int height, const int* ranges, const int* ids,
                              long long num_ids, int n, const float* centers, const float* conics,
                              const float* planes, const float* normals, const float* colors,
                              int ch_a, int stride_a, const float* extras, int ch_b, int stride_b,
                              const float* background, const float* K, float* features,
                              int feat_pix, int feat_ch, float* alpha, int alpha_pix,
                              float* depth, int depth_pix, float* median, int median_pix,
                              float* normal_image, int normal_pix, int normal_ch,
                              float* auxiliary, int* contributors, int stat_count,
                              int stat_sum_mask, const float* stat_pixels, int* stat_counts,
                              float* stat_sums, const int* tile_order, void* stream);

/* rade/render.py:325-547 backward, from the forward's alpha and normal
 * images (strides as in splat_rade_render_forward), auxiliary and
 * contributors.  Upstream images: the value of channel c at pixel p is
 * up[p*pix + c*ch] (NULL: zero) for the colour channels (ch_a, up_colors),
 * the extra channels (ch_b, up_extras; channel c of the blend is c - ch_a
 * there), alpha, expected depth, median depth and normals (3 channels); one
 * (H,W,C) image serves both with up_extras = up_colors + ch_a.
 * Gradients are ADDED into grad_centers (n,2), grad_conics (n,4),
 * grad_colors (n,ch_a), grad_extras (n,ch_b), abs_centers (n,2) (NULL to
 * skip the last three), grad_planes and grad_normals (n,3). */
int splat_rade_render_backward(
    int width, int height, const int* ranges, const int* ids, long long num_ids, int n,
    const float* centers, const float* conics, const float* planes, const float* normals,
    const float* colors, int ch_a, int stride_a, const float* extras, int ch_b, int stride_b,
    const float* background, const float* K, const float* alpha, int alpha_pix,
    const float* normal_image, int normal_pix, int normal_ch, const float* auxiliary,
    const int* contributors, const float* up_colors, int up_colors_pix, int up_colors_ch,
    const float* up_extras, int up_extras_pix, int up_extras_ch, const float* up_alpha,
    int up_alpha_pix, const float* up_depth, int up_depth_pix,
    const float* up_median, int up_median_pix, const float* up_normals, int up_normals_pix,
    int up_normals_ch, float* grad_centers, float* grad_conics, float* grad_colors,
    float* grad_extras, float* abs_centers, float* grad_planes, float* grad_normals,
    const int* tile_order, void* stream);

/* ---- AAA-Gaussians (dsl_splat/aaa) ------------------------------------------
 * One view of aaa.rasterize: adaptive 3D filter, 3D ray evaluation,
 * StopThePop HIER 64/8/4 hierarchical sorting.  The camera arrays are the
 * reference's lowered, transposed 4x4 storage (aaa/cameras.py:77-121:
 * viewmatrix = V^T, projmatrix = (P V)^T, device float32). */
typedef struct SplatAaaFrame {
  int n, width, height;
  const float* means;      /* (n,3) */
  const float* scales;     /* (n,3) activated */
  const float* quats;      /* (n,4) wxyz, 16-byte aligned: normalised, or raw when
                              normalize_quats */
  const float* opacities;  /* (n) activated */
  const float* sh;         /* (n,sh_k,3) SH inputs of preprocess_3d, or NULL */
  int sh_k, sh_degree;
  const float* filters;    /* (n) stored 3D filter, or NULL */
  const float* campos;     /* (3) */
  const float* view;       /* (4,4) viewmatrix storage */
  const float* proj;       /* (4,4) projmatrix storage */
  float tanfov_x, tanfov_y, principal_x, principal_y, scale_modifier;
  float focal_x;           /* width / (2 tanfov_x), computed in double (backward_preprocess.py:332) */
  float focal_max;         /* max of both focal lengths (backward_camera.py:267-270) */
  int sort_order;          /* 0-3 (aaa/settings.py GlobalSortOrder; 3 = PTD_MAX) */
  int ewa, new_aabb, near_clipping, tile_culling;
  int complete;            /* eval_3D and not cooperative (aaa/preprocess.py:321-322) */
  int cooperative;         /* load_balancing and tile_based_culling */
  int normalize_quats;     /* 1: quats are raw; the kernels normalise them with the bits of
                              Torch's F.normalize (inputs.py:252) and the preprocessing
                              adjoint returns the raw quaternions' gradient */
} SplatAaaFrame;

/* aaa/preprocess.py:165-451 -> aaa/preprocess3d.py:17-245 preprocess_3d
 * (adaptive 3D filter, EWA opacity compensation, Gaussian-to-screen
 * transform, frustum culling, axis bounds, first-32-tile culling).  Outputs
 * (n): centers/rects (n,2) float2, depths, transforms (n,4,4), opacity
 * (effective), radii, tiles, valid (u8), rgb/clamped (n,3) when sh; rows of
 * rejected Gaussians keep radii = tiles = valid = 0 and are otherwise left
 * unwritten.  cooperative: rectangles of more than 32 tiles are appended to
 * queued (n), *queue_size (device int, zeroed here) counts them.  atan2,
 * tan, exp and log are this library's own functions (the CPU oracle's). */
int splat_aaa_preprocess(const SplatAaaFrame* frame, float* centers, float* rects, float* depths,
                         float* transforms, float* opacity, int* radii, int* tiles, float* rgb,
                         unsigned char* valid, unsigned char* clamped, int* queued,
                         int* queue_size, void* stream);

/* aaa/preprocess.py:452-476 -> aaa/cooperative_culling.py:152-192
 * cull_remainder_3d: the queued Gaussians' tiles past the first 32 are
 * added to tiles; a Gaussian left without a tile gets radius 0, not valid. */
int splat_aaa_cull_remainder(int n, const int* queued, const int* queue_size,
                             const float* centers, const float* rects, const float* transforms,
                             const float* opacity, int width, int height, int* radii, int* tiles,
                             unsigned char* valid, void* stream);

/* aaa/metadata.py:55-91 _geometry for one view (after the remainder cull):
 * per Gaussian with radii > 0 the half extents rounded up (out_radii (n,2)
 * int32), the pixel projection of the mean (out_means2d (n,2): fx x/z + cx,
 * fy y/z + cy with (x, y, z) = view (row-major 4x4 world-to-camera) * mean
 * and z clamped to 1e-12) and the effective opacity (out_opacity (n));
 * zeros for the other rows.  rects/out_* 8-byte aligned. */
int splat_aaa_metadata(int n, const float* view, float fx, float fy, float cx, float cy,
                       const float* means, const float* rects, const int* radii,
                       const float* opacity, int* out_radii, float* out_means2d,
                       float* out_opacity, void* stream);

/* aaa/binning.py:278-342 bin_and_sort after the count scan (splat_scan_counts
 * of tiles, its total read by the host as the reference does at
 * primitives/tiling.py:64): aaa/binning_native.py:7-135's key emission
 * (tile, screen depth + 8 of the tile's closest point, Gaussian id; padding
 * pairs where the recount finds fewer tiles), the stable sort of the keys
 * (primitives/tiling.py:67-100) and identify_ranges (:39-54).  point_list
 * (pairs) ends with the padding ids (-1); ranges (T,2), zero for empty
 * tiles.  Images up to 65535 tiles, up to 2^30 pairs. */
size_t splat_aaa_bin_workspace_bytes(long long pairs);
int splat_aaa_bin(int n, long long pairs, const int* offsets, const float* centers,
                  const float* rects, const int* radii, const float* transforms,
                  const float* opacity, int width, int height, void* workspace,
                  size_t workspace_bytes, int* point_list, int* ranges, void* stream);

/* The emission alone (aaa/binning_native.py:85-135), unsorted, pairs in
 * Gaussian order: tiles_out (tile id; padding 2^b - 1 with b the bit length
 * of the tile count), depth_keys (float bits of depth + 8 minus those of
 * 7.0), ids (-1 for padding). */
int splat_aaa_emit(int n, long long pairs, const int* offsets, const float* centers,
                   const float* rects, const int* radii, const float* transforms,
                   const float* opacity, int width, int height, unsigned* tiles_out,
                   unsigned* depth_keys, int* ids, void* stream);

/* aaa/render.py:11-28 -> aaa/render_hierarchical_warp.py:694-801 render
 * (HIER 64/8/4 blend, 4x4 culling when cull): image (C,H,W) planar
 * = blended features + T * bg, final_t and contributors (H,W).  n Gaussians
 * (ids outside [0, n) are never read); colors (n,C) row-major, C = 1..64;
 * tile_order (T) a block schedule (splat_tile_order) or NULL.  Contribution
 * statistics (render_hierarchical_warp.py:608-653 render_statistics with the
 * observer of statistics.py:47-73): stat_count requests (0 disables, at most
 * 30) over the (stat_count, H*W) maps stat_pixels; every blended sample, of
 * weight alpha*T, whose pixel value v is nonzero adds 1 to its Gaussian's row
 * of stat_counts (a masked count) or v*alpha*T to its row of stat_sums (a
 * weighted sum: bit r of stat_sum_mask), rows of n in request order per
 * kind. */
int splat_aaa_render(int n, int width, int height, int channels, int cull, const int* ranges,
                     const int* points, const float* transforms, const float* opacity,
                     const float* colors, const float* bg, const int* tile_order, float* image,
                     float* final_t, int* contributors, int record_capacity, float* records,
                     int* record_counts, int* tile_overflow, int stat_count, int stat_sum_mask,
                     const float* stat_pixels, int* stat_counts, float* stat_sums,
                     void* stream);

/* Bytes of the optional blend records of splat_aaa_render for a capacity
 * (records: T*256*capacity entries of two floats, 8-byte aligned;
 * record_counts: T*256; tile_overflow: T).  With records (non-NULL,
 * capacity 1..256) the blend also stores, per pixel, every sample it blends
 * in blend order, up to record_capacity: entry j of tile-local pixel l of
 * tile t, at index ((t * capacity + j) * 256 + l), holds the sample's
 * position in the tile's slice of points (int bits) and its Gaussian value;
 * plus the per-pixel count (-1 past the capacity) and a per-tile overflow
 * flag.  The backward then reads them instead of replaying the queues (the
 * reference keeps no history: aaa/backward_render.py:1-5). */
size_t splat_aaa_record_bytes(int width, int height, int capacity);

/* aaa/backward_render.py:140-248 backward_render: replay of the forward's
 * queues; gradients ADDED into grad_transforms (n,16, the reference's
 * transposed layout, 16-byte aligned), grad_opacity (n), grad_colors (n,C),
 * grad_screen (n,2) and grad_screen_abs (n,2) (NULL to skip; abs requires
 * screen).  image/final_t: the forward's outputs; pixel_grad (C,H,W).
 * With the forward's blend records (records non-NULL, the same capacity)
 * each recorded pixel's samples are taken from them with the replay's
 * arithmetic and summed per Gaussian and tile, and only the tiles flagged in
 * tile_overflow are replayed.  The records are consumed: the backward
 * overwrites their entries, so a second backward must replay (records NULL). */
int splat_aaa_render_backward(int n, int width, int height, int channels, int cull,
                              const int* ranges, const int* points, const float* transforms, const float* opacity,
                              const float* colors, const float* bg, const int* tile_order,
                              const float* image, const float* final_t, const float* pixel_grad,
                              float* grad_transforms, float* grad_opacity, float* grad_colors,
                              float* grad_screen, float* grad_screen_abs, int record_capacity,
                              float* records, const int* record_counts, const int* tile_overflow,
                              void* stream);

/* aaa/backward_preprocess.py:270-346 -> preprocess_adjoint (:130-268):
 * gradients of the input opacities (n), means (n,3), scales (n,3) and
 * normalised quaternions (n,4, 16-byte aligned) from the replay's
 * transform (n,16) and effective-opacity (n) gradients (fully written).
 * Uses frame->focal_x. */
int splat_aaa_preprocess_backward(const SplatAaaFrame* frame, const int* radii,
                                  const float* up_transforms, const float* up_opacity,
                                  float* grad_opacity, float* grad_means, float* grad_scales,
                                  float* grad_quats, void* stream);

/* aaa/backward_camera.py:225-294 backward_camera -> camera_adjoint
 * (:61-224) without SH, rows summed on the device: camera_sums (23) =
 * projmatrix gradient (16, storage order), viewmatrix column-2 gradient (4),
 * campos gradient (3).  Uses frame->focal_max. */
int splat_aaa_camera_backward(const SplatAaaFrame* frame, const int* radii,
                              const float* effective_opacity, const float* up_transforms,
                              const float* up_opacity, float* camera_sums, void* stream);

/* Diagnostic: ours[i] = the blend's exp, cuda_exp[i] = CUDA expf, for x (n). */
int splat_debug_expf(int n, const float* x, float* ours, float* cuda_exp, void* stream);

#ifdef __cplusplus
}
#endif

#endif /* SPLAT200_H */
