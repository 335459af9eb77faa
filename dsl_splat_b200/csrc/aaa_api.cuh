// C-ABI entry points of the AAA-Gaussians path (declared in
// include/splat200.h).  Included at the end of splat200.cu, so they share its
// status reporting, launch counter and stream conventions: all work on the
// given stream, outputs and workspaces allocated by the caller, a negative
// status on bad arguments or a failed launch.
#pragma once
#include "../../include/splat200.h"
#include "aaa.cuh"
#include "aaa_render.cuh"

namespace {

using splat::aaa::AdjointParams;
using splat::aaa::HierParams;
using splat::aaa::PreprocessParams;

int aaa_check_frame(const SplatAaaFrame* f) {
  if (!f) return fail(kInvalidArgument, "null frame");
  if (f->n < 0 || f->width <= 0 || f->height <= 0)
    return fail(kInvalidArgument, "bad AAA frame sizes");
  if (f->n > 0 && (!f->means || !f->scales || !f->quats || !f->opacities || !f->campos ||
                   !f->view || !f->proj))
    return fail(kInvalidArgument, "null AAA frame input");
  if (!aligned(f->quats, 16)) return fail(kInvalidArgument, "quats need 16-byte alignment");
  if (f->sh && (f->sh_k < (f->sh_degree + 1) * (f->sh_degree + 1) || f->sh_degree < 0 ||
                f->sh_degree > 3))
    return fail(kInvalidArgument, "bad SH layout");
  if (!(f->tanfov_x > 0.0f) || !(f->tanfov_y > 0.0f) || !(f->scale_modifier > 0.0f))
    return fail(kInvalidArgument, "field of view tangents and scale modifier must be positive");
  const long long tiles = static_cast<long long>((f->width + 15) / 16) * ((f->height + 15) / 16);
  if (tiles >= 65536) return fail(kTooLarge, "AAA images are limited to 65535 tiles");
  return kOk;
}

// bytes of the AAA binning workspace for `pairs` pairs (layout below)
struct AaaBinLayout {
  size_t tiles_in, depth_in, ids_in, keys_a, vals_a, keys_b, vals_b, hist, status, counters,
      bytes;
  unsigned sort_tiles;
};

size_t round256(size_t v) { return (v + 255) & ~static_cast<size_t>(255); }

// the pair sort's onesweep shape (threads per block, keys per thread): at
// config 3's 10.4M pairs 8 keys per thread measured 696 us for the five
// passes against 795 us with 16 (512 threads: 714 / 963 us with 8 / 16).
// A per-tile shared-memory sort by depth key after two tile passes measured
// slower (730 us: the tiles' random gathers and ranking rounds).
constexpr int kAaaSortThreads = 256, kAaaSortItems = 8;
constexpr int kAaaSortTile = kAaaSortThreads * kAaaSortItems;

AaaBinLayout aaa_bin_layout(long long pairs) {
  AaaBinLayout L{};
  const size_t m = static_cast<size_t>(pairs > 0 ? pairs : 1);
  L.sort_tiles = blocks_for(static_cast<long long>(m), kAaaSortTile);
  size_t at = 0;
  auto take = [&](size_t bytes) {
    const size_t here = at;
    at += round256(bytes);
    return here;
  };
  L.tiles_in = take(4 * m);
  L.depth_in = take(4 * m);
  L.ids_in = take(4 * m);
  L.keys_a = take(4 * m);
  L.vals_a = take(4 * m);
  L.keys_b = take(4 * m);
  L.vals_b = take(4 * m);
  L.hist = take(4 * 5 * kRadix);
  L.status = take(4ull * 5 * L.sort_tiles * kRadix);
  L.counters = take(4 * 8);
  L.bytes = at;
  return L;
}

int bit_length(int v) {
  int b = 0;
  while (v) {
    ++b;
    v >>= 1;
  }
  return b;
}

template <int CHP>
int launch_hier(const HierParams& p, int tiles, bool backward, bool screen, bool absgrad,
                cudaStream_t s) {
  using namespace splat::aaa;
  int r = kOk;
  const unsigned blocks = static_cast<unsigned>(tiles) * kHierBlocksPerTile;
  const bool records = backward && p.records;
  if (records) {  // the recorded tiles from their records, then the replay of the overflowed ones
    r = record_backward_dispatch(p, tiles, screen, absgrad, s);
    if (r != kOk) return r;
  }
  HierParams q = p;
  if (records) {
    q.only_flagged = p.tile_overflow;
    q.records = nullptr;
  }
  if (!backward) {
    if (q.stat_count)
      aaa_hier_kernel<CHP, false, false, false, true><<<blocks, kHierThreads, 0, counted(s)>>>(q);
    else
      aaa_hier_kernel<CHP, false, false, false><<<blocks, kHierThreads, 0, counted(s)>>>(q);
  } else if (!screen)
    aaa_hier_kernel<CHP, true, false, false><<<blocks, kHierThreads, 0, counted(s)>>>(q);
  else if (!absgrad)
    aaa_hier_kernel<CHP, true, true, false><<<blocks, kHierThreads, 0, counted(s)>>>(q);
  else
    aaa_hier_kernel<CHP, true, true, true><<<blocks, kHierThreads, 0, counted(s)>>>(q);
  return check_launch("aaa_hier");
}

int dispatch_hier(const HierParams& p, bool backward, bool screen, bool absgrad, cudaStream_t s) {
  const int tiles = ((p.width + 15) / 16) * ((p.height + 15) / 16);
  if (p.channels <= 4) return launch_hier<4>(p, tiles, backward, screen, absgrad, s);
  if (p.channels <= 8) return launch_hier<8>(p, tiles, backward, screen, absgrad, s);
  if (p.channels <= 16) return launch_hier<16>(p, tiles, backward, screen, absgrad, s);
  if (p.channels <= 32) return launch_hier<32>(p, tiles, backward, screen, absgrad, s);
  return launch_hier<64>(p, tiles, backward, screen, absgrad, s);
}

int check_hier_inputs(int width, int height, int channels, const int* ranges, const int* points,
                      const float* transforms, const float* opacity, const float* colors,
                      const float* bg) {
  if (width <= 0 || height <= 0) return fail(kInvalidArgument, "bad image size");
  if (channels < 1 || channels > 64) return fail(kInvalidArgument, "AAA blend takes 1-64 channels");
  const long long tiles = static_cast<long long>((width + 15) / 16) * ((height + 15) / 16);
  if (tiles >= (1LL << 31)) return fail(kTooLarge, "too many tiles");
  if (!ranges || !transforms || !opacity || !colors || !bg)
    return fail(kInvalidArgument, "null AAA blend input");
  if (!aligned(transforms, 16)) return fail(kInvalidArgument, "transforms need 16-byte alignment");
  (void)points;
  return kOk;
}

}  // namespace

extern "C" {

int splat_test_trig(int n, const float* y, const float* x, float* atan2_out, float* tan_out,
                    void* stream) {
  if (n < 0) return fail(kInvalidArgument, "n < 0");
  if (n == 0) return kOk;
  if (!y || !x || !atan2_out || !tan_out) return fail(kInvalidArgument, "null trig buffer");
  splat::aaa::trig_probe_kernel<<<blocks_for(n, 256), 256, 0, counted(as_stream(stream))>>>(
      n, y, x, atan2_out, tan_out);
  return check_launch("test_trig");
}

int splat_aaa_preprocess(const SplatAaaFrame* f, float* centers, float* rects, float* depths,
                         float* transforms, float* opacity, int* radii, int* tiles, float* rgb,
                         unsigned char* valid, unsigned char* clamped, int* queued, int* queue_size,
                         void* stream) {
  int r = aaa_check_frame(f);
  if (r != kOk) return r;
  cudaStream_t s = as_stream(stream);
  if (f->cooperative && !queue_size) return fail(kInvalidArgument, "cooperative needs the queue");
  if (queue_size && cudaMemsetAsync(queue_size, 0, sizeof(int), s) != cudaSuccess)
    return check_launch("aaa_preprocess queue");
  if (f->n == 0) return kOk;
  if (!centers || !rects || !depths || !transforms || !opacity || !radii || !tiles || !valid ||
      (f->cooperative && !queued) || (f->sh && (!rgb || !clamped)))
    return fail(kInvalidArgument, "null AAA preprocess output");
  if (!aligned(centers, 8) || !aligned(rects, 8) || !aligned(transforms, 16))
    return fail(kInvalidArgument, "AAA preprocess outputs misaligned");
  PreprocessParams p{};
  p.n = f->n;
  p.means = f->means;
  p.scales = f->scales;
  p.quats = f->quats;
  p.normalize_quats = f->normalize_quats;
  p.opacities = f->opacities;
  p.sh = f->sh;
  p.sh_k = f->sh_k;
  p.degree = f->sh_degree;
  p.sort_order = f->sort_order;
  p.filters = f->filters;
  p.campos = f->campos;
  p.view = f->view;
  p.proj = f->proj;
  p.width = f->width;
  p.height = f->height;
  p.tanx = f->tanfov_x;
  p.tany = f->tanfov_y;
  p.principal_x = f->principal_x;
  p.principal_y = f->principal_y;
  p.modifier = f->scale_modifier;
  p.ewa = f->ewa;
  p.new_aabb = f->new_aabb;
  p.near_clipping = f->near_clipping;
  p.tile_culling = f->tile_culling;
  p.complete = f->complete;
  p.cooperative = f->cooperative;
  p.centers = centers;
  p.rects = rects;
  p.depths = depths;
  p.transforms = transforms;
  p.opacity_out = opacity;
  p.radii = radii;
  p.tiles = tiles;
  p.rgb = rgb;
  p.valid = valid;
  p.clamped = clamped;
  p.queued = queued;
  p.queue_size = queue_size;
  splat::aaa::aaa_preprocess_kernel<<<blocks_for(f->n, 128), 128, 0, counted(s)>>>(p);
  return check_launch("aaa_preprocess");
}

int splat_aaa_cull_remainder(int n, const int* queued, const int* queue_size, const float* centers,
                             const float* rects, const float* transforms, const float* opacity,
                             int width, int height, int* radii, int* tiles, unsigned char* valid,
                             void* stream) {
  if (n < 0 || width <= 0 || height <= 0) return fail(kInvalidArgument, "bad sizes");
  if (n == 0) return kOk;
  if (!queued || !queue_size || !centers || !rects || !transforms || !opacity || !radii || !tiles ||
      !valid)
    return fail(kInvalidArgument, "null AAA cull argument");
  if (!aligned(transforms, 16) || !aligned(centers, 8) || !aligned(rects, 8))
    return fail(kInvalidArgument, "AAA cull inputs misaligned");
  // the queue holds at most n entries: enough warps for a few per SM, each
  // taking queued Gaussians in a grid stride
  const int warps = std::min(n, sm_count() * 64);
  splat::aaa::aaa_cull_remainder_kernel<<<blocks_for(warps, 8), 256, 0, counted(as_stream(stream))>>>(
      queued, queue_size, centers, rects, transforms, opacity, width, height, radii, tiles, valid);
  return check_launch("aaa_cull_remainder");
}

int splat_aaa_metadata(int n, const float* view, float fx, float fy, float cx, float cy,
                       const float* means, const float* rects, const int* radii,
                       const float* opacity, int* out_radii, float* out_means2d,
                       float* out_opacity, void* stream) {
  if (n < 0) return fail(kInvalidArgument, "n < 0");
  if (n == 0) return kOk;
  if (!view || !means || !rects || !radii || !opacity || !out_radii || !out_means2d ||
      !out_opacity)
    return fail(kInvalidArgument, "null AAA metadata argument");
  if (!aligned(rects, 8) || !aligned(out_radii, 8) || !aligned(out_means2d, 8))
    return fail(kInvalidArgument, "AAA metadata rows misaligned");
  splat::aaa::aaa_metadata_kernel<<<blocks_for(n, 256), 256, 0, counted(as_stream(stream))>>>(
      n, view, fx, fy, cx, cy, means, rects, radii, opacity, out_radii, out_means2d, out_opacity);
  return check_launch("aaa_metadata");
}

size_t splat_aaa_bin_workspace_bytes(long long pairs) { return aaa_bin_layout(pairs).bytes; }

int splat_aaa_emit(int n, long long pairs, const int* offsets, const float* centers,
                   const float* rects, const int* radii, const float* transforms,
                   const float* opacity, int width, int height, unsigned* tiles_out,
                   unsigned* depth_keys, int* ids, void* stream) {
  if (n < 0 || pairs < 0 || width <= 0 || height <= 0) return fail(kInvalidArgument, "bad sizes");
  if (pairs >= (1LL << 30)) return fail(kTooLarge, "AAA binning holds at most 2^30 pairs");
  if (n == 0 || pairs == 0) return kOk;
  if (!offsets || !centers || !rects || !radii || !transforms || !opacity || !tiles_out ||
      !depth_keys || !ids)
    return fail(kInvalidArgument, "null AAA emit argument");
  if (!aligned(transforms, 16) || !aligned(centers, 8) || !aligned(rects, 8))
    return fail(kInvalidArgument, "AAA emit inputs misaligned");
  const int T = ((width + 15) / 16) * ((height + 15) / 16);
  const unsigned pad_tile = (1u << bit_length(T)) - 1u;
  const long long threads = (static_cast<long long>(n) + 31) / 32 * 32;
  splat::aaa::aaa_emit_kernel<<<blocks_for(threads, 128), 128, 0, counted(as_stream(stream))>>>(
      n, centers, rects, radii, transforms, opacity, offsets, width, height, pad_tile, pairs,
      tiles_out, depth_keys, ids);
  return check_launch("aaa_emit");
}

int splat_aaa_bin(int n, long long pairs, const int* offsets, const float* centers,
                  const float* rects, const int* radii, const float* transforms,
                  const float* opacity, int width, int height, void* workspace,
                  size_t workspace_bytes, int* point_list, int* ranges, void* stream) {
  if (n < 0 || pairs < 0 || width <= 0 || height <= 0) return fail(kInvalidArgument, "bad sizes");
  if (pairs >= (1LL << 30)) return fail(kTooLarge, "AAA binning holds at most 2^30 pairs");
  const int T = ((width + 15) / 16) * ((height + 15) / 16);
  if (T >= 65536) return fail(kTooLarge, "AAA images are limited to 65535 tiles");
  if (!ranges) return fail(kInvalidArgument, "null ranges");
  cudaStream_t s = as_stream(stream);
  if (cudaMemsetAsync(ranges, 0, sizeof(int) * 2 * static_cast<size_t>(T), s) != cudaSuccess)
    return check_launch("aaa_bin ranges");
  if (n == 0 || pairs == 0) return kOk;
  const AaaBinLayout L = aaa_bin_layout(pairs);
  if (!workspace || workspace_bytes < L.bytes)
    return fail(kWorkspaceTooSmall, "AAA bin workspace too small");
  if (!aligned(workspace, 256) || !point_list)
    return fail(kInvalidArgument, "workspace needs 256-byte alignment; point_list required");
  char* ws = static_cast<char*>(workspace);
  auto u32 = [&](size_t off) { return reinterpret_cast<uint32_t*>(ws + off); };
  uint32_t* tiles_in = u32(L.tiles_in);
  uint32_t* depth_in = u32(L.depth_in);
  int* ids_in = reinterpret_cast<int*>(ws + L.ids_in);
  int r = splat_aaa_emit(n, pairs, offsets, centers, rects, radii, transforms, opacity, width,
                         height, tiles_in, depth_in, ids_in, stream);
  if (r != kOk) return r;
  const int tile_bits = bit_length(T);
  const int tile_passes = tile_bits > 8 ? 2 : 1;
  if (cudaMemsetAsync(ws + L.hist, 0, 4 * 5 * kRadix, s) != cudaSuccess ||
      cudaMemsetAsync(ws + L.status, 0, L.counters + 4 * 8 - L.status, s) != cudaSuccess)
    return check_launch("aaa_bin memset");
  const unsigned m = static_cast<unsigned>(pairs);
  const int hist_blocks = static_cast<int>(std::min<long long>(blocks_for(pairs, 256), sm_count() * 4));
  splat::aaa::aaa_key_histograms_kernel<<<hist_blocks, 256, 0, counted(s)>>>(
      pairs, tiles_in, depth_in, tile_passes, u32(L.hist));
  // hist rows: depth bytes 0-2, tile bytes 0-1 (the pass order)
  const unsigned blocks = L.sort_tiles;
  auto status = [&](int pass) { return u32(L.status) + static_cast<size_t>(pass) * blocks * kRadix; };
  auto counter = [&](int pass) { return u32(L.counters) + pass; };
  // each pass's blocks form the exclusive prefix of its histogram row
  auto offs = [&](int pass) { return u32(L.hist) + pass * kRadix; };
  uint32_t *keys_a = u32(L.keys_a), *vals_a = u32(L.vals_a), *keys_b = u32(L.keys_b),
           *vals_b = u32(L.vals_b);
  onesweep_kernel<splat::aaa::DepthKeyLoader, true, kAaaSortThreads, kAaaSortItems, true>
      <<<blocks, kAaaSortThreads, 0, counted(s)>>>(
      splat::aaa::DepthKeyLoader{depth_in}, m, 0, offs(0), status(0), counter(0), keys_a, vals_a);
  onesweep_kernel<KeyValueLoader, true, kAaaSortThreads, kAaaSortItems, true>
      <<<blocks, kAaaSortThreads, 0, counted(s)>>>(
      KeyValueLoader{keys_a, vals_a}, m, 8, offs(1), status(1), counter(1), keys_b, vals_b);
  onesweep_kernel<KeyValueLoader, false, kAaaSortThreads, kAaaSortItems, true>
      <<<blocks, kAaaSortThreads, 0, counted(s)>>>(
      KeyValueLoader{keys_b, vals_b}, m, 16, offs(2), status(2), counter(2), keys_a, vals_a);
  onesweep_kernel<splat::aaa::TileGatherLoader, true, kAaaSortThreads, kAaaSortItems, true>
      <<<blocks, kAaaSortThreads, 0, counted(s)>>>(
      splat::aaa::TileGatherLoader{tiles_in, vals_a}, m, 0, offs(3), status(3), counter(3), keys_b,
      vals_b);
  const uint32_t* sorted_tiles = keys_b;
  const uint32_t* sorted_pairs = vals_b;
  if (tile_passes > 1) {
    onesweep_kernel<KeyValueLoader, true, kAaaSortThreads, kAaaSortItems, true>
      <<<blocks, kAaaSortThreads, 0, counted(s)>>>(
        KeyValueLoader{keys_b, vals_b}, m, 8, offs(4), status(4), counter(4), keys_a, vals_a);
    sorted_tiles = keys_a;
    sorted_pairs = vals_a;
  }
  const unsigned pad_tile = (1u << tile_bits) - 1u;
  const int range_blocks = static_cast<int>(std::min<long long>(blocks_for(pairs, 256), sm_count() * 8));
  splat::aaa::aaa_ranges_kernel<<<range_blocks, 256, 0, counted(s)>>>(
      pairs, sorted_tiles, sorted_pairs, ids_in, pad_tile, ranges, point_list);
  return check_launch("aaa_bin");
}

size_t splat_aaa_record_bytes(int width, int height, int capacity) {
  const size_t tiles = static_cast<size_t>((width + 15) / 16) * ((height + 15) / 16);
  return tiles * 256 * (8 * static_cast<size_t>(capacity > 0 ? capacity : 0) + 4) + 4 * tiles;
}

int splat_aaa_render(int n, int width, int height, int channels, int cull, const int* ranges,
                     const int* points, const float* transforms, const float* opacity,
                     const float* colors, const float* bg, const int* tile_order, float* image,
                     float* final_t, int* contributors, int record_capacity, float* records,
                     int* record_counts, int* tile_overflow, int stat_count, int stat_sum_mask,
                     const float* stat_pixels, int* stat_counts, float* stat_sums,
                     void* stream) {
  int r = check_hier_inputs(width, height, channels, ranges, points, transforms, opacity, colors, bg);
  if (r != kOk) return r;
  if (!image || !final_t || !contributors) return fail(kInvalidArgument, "null AAA blend output");
  const bool has_records = records != nullptr;
  if (has_records && (record_capacity <= 0 || record_capacity > 256 || !record_counts ||
                      !tile_overflow || !aligned(records, 8)))
    return fail(kInvalidArgument,
                "blend records need a capacity in [1, 256], counts, flags and 8-byte entries");
  const long long tiles = static_cast<long long>((width + 15) / 16) * ((height + 15) / 16);
  if (has_records &&
      cudaMemsetAsync(tile_overflow, 0, sizeof(int) * tiles, as_stream(stream)) != cudaSuccess)
    return check_launch("aaa_render records");
  if (n < 0) return fail(kInvalidArgument, "n < 0");
  if (stat_count < 0 || stat_count > 30 ||
      (stat_count && (!stat_pixels || (!stat_counts && stat_sum_mask != (1 << stat_count) - 1) ||
                      (!stat_sums && stat_sum_mask != 0))))
    return fail(kInvalidArgument, "bad AAA statistics arguments");
  HierParams p{};
  p.n = n;
  p.width = width;
  p.height = height;
  p.channels = channels;
  p.cull = cull;
  p.ranges = ranges;
  p.points = points;
  p.transforms = transforms;
  p.opacity = opacity;
  p.colors = colors;
  p.bg = bg;
  p.tile_order = tile_order;
  p.stat_count = stat_count;
  p.stat_sum_mask = stat_sum_mask;
  p.stat_pixels = stat_pixels;
  p.stat_counts = stat_counts;
  p.stat_sums = stat_sums;
  p.image = image;
  p.final_t = final_t;
  p.contributors = contributors;
  if (has_records) {
    p.record_capacity = record_capacity;
    p.records = reinterpret_cast<float2*>(records);
    p.record_counts = record_counts;
    p.tile_overflow = tile_overflow;
  }
  return dispatch_hier(p, false, false, false, as_stream(stream));
}

int splat_aaa_render_backward(int n, int width, int height, int channels, int cull,
                              const int* ranges,
                              const int* points, const float* transforms, const float* opacity,
                              const float* colors, const float* bg, const int* tile_order,
                              const float* image, const float* final_t, const float* pixel_grad,
                              float* grad_transforms, float* grad_opacity, float* grad_colors,
                              float* grad_screen, float* grad_screen_abs, int record_capacity,
                              float* records, const int* record_counts, const int* tile_overflow,
                              void* stream) {
  int r = check_hier_inputs(width, height, channels, ranges, points, transforms, opacity, colors, bg);
  if (r != kOk) return r;
  if (!image || !final_t || !pixel_grad || !grad_transforms || !grad_opacity || !grad_colors)
    return fail(kInvalidArgument, "null AAA replay argument");
  if (grad_screen_abs && !grad_screen)
    return fail(kInvalidArgument, "absolute screen gradients require the screen gradients");
  if (!aligned(grad_transforms, 16) || !aligned(grad_screen, 8) || !aligned(grad_screen_abs, 8))
    return fail(kInvalidArgument, "AAA gradient buffers misaligned");
  if (n < 0) return fail(kInvalidArgument, "n < 0");
  HierParams p{};
  p.n = n;
  p.width = width;
  p.height = height;
  p.channels = channels;
  p.cull = cull;
  p.ranges = ranges;
  p.points = points;
  p.transforms = transforms;
  p.opacity = opacity;
  p.colors = colors;
  p.bg = bg;
  p.tile_order = tile_order;
  p.image_in = image;
  p.final_t_in = final_t;
  p.pixel_grad = pixel_grad;
  p.grad_transforms = grad_transforms;
  p.grad_opacity = grad_opacity;
  p.grad_colors = grad_colors;
  p.grad_screen = grad_screen;
  p.grad_screen_abs = grad_screen_abs;
  if (records) {
    if (record_capacity <= 0 || record_capacity > 256 || !record_counts || !tile_overflow ||
        !aligned(records, 8))
      return fail(kInvalidArgument,
                  "blend records need a capacity in [1, 256], counts, flags and 8-byte entries");
    p.record_capacity = record_capacity;
    p.records = reinterpret_cast<float2*>(records);
    p.record_counts = const_cast<int*>(record_counts);
    p.tile_overflow = const_cast<int*>(tile_overflow);
  }
  return dispatch_hier(p, true, grad_screen != nullptr, grad_screen_abs != nullptr,
                       as_stream(stream));
}

int splat_aaa_preprocess_backward(const SplatAaaFrame* f, const int* radii,
                                  const float* up_transforms, const float* up_opacity,
                                  float* grad_opacity, float* grad_means, float* grad_scales,
                                  float* grad_quats, void* stream) {
  int r = aaa_check_frame(f);
  if (r != kOk) return r;
  if (f->n == 0) return kOk;
  if (!radii || !up_transforms || !up_opacity || !grad_opacity || !grad_means || !grad_scales ||
      !grad_quats)
    return fail(kInvalidArgument, "null AAA preprocess adjoint argument");
  if (!aligned(up_transforms, 16) || !aligned(grad_quats, 16))
    return fail(kInvalidArgument, "AAA adjoint buffers misaligned");
  AdjointParams p{};
  p.n = f->n;
  p.means = f->means;
  p.scales = f->scales;
  p.quats = f->quats;
  p.normalize_quats = f->normalize_quats;
  p.opacities = f->opacities;
  p.radii = radii;
  p.view = f->view;
  p.proj = f->proj;
  p.campos = f->campos;
  p.width = f->width;
  p.height = f->height;
  p.focal = f->focal_x;
  p.ewa = f->ewa;
  p.up_transforms = up_transforms;
  p.up_opacity = up_opacity;
  p.grad_opacity = grad_opacity;
  p.grad_means = grad_means;
  p.grad_scales = grad_scales;
  p.grad_quats = grad_quats;
  splat::aaa::aaa_preprocess_adjoint_kernel<<<blocks_for(f->n, 128), 128, 0,
                                              counted(as_stream(stream))>>>(p);
  return check_launch("aaa_preprocess_backward");
}

int splat_aaa_camera_backward(const SplatAaaFrame* f, const int* radii,
                              const float* effective_opacity, const float* up_transforms,
                              const float* up_opacity, float* camera_sums, void* stream) {
  int r = aaa_check_frame(f);
  if (r != kOk) return r;
  if (!camera_sums) return fail(kInvalidArgument, "null camera sums");
  cudaStream_t s = as_stream(stream);
  if (cudaMemsetAsync(camera_sums, 0, 23 * sizeof(float), s) != cudaSuccess)
    return check_launch("aaa_camera_backward memset");
  if (f->n == 0) return kOk;
  if (!radii || !effective_opacity || !up_transforms || !up_opacity)
    return fail(kInvalidArgument, "null AAA camera adjoint argument");
  if (!aligned(up_transforms, 16)) return fail(kInvalidArgument, "AAA adjoint buffers misaligned");
  AdjointParams p{};
  p.n = f->n;
  p.means = f->means;
  p.scales = f->scales;
  p.quats = f->quats;
  p.normalize_quats = f->normalize_quats;
  p.opacities = effective_opacity;
  p.radii = radii;
  p.filters = f->filters;
  p.view = f->view;
  p.proj = f->proj;
  p.campos = f->campos;
  p.width = f->width;
  p.height = f->height;
  p.focal = f->focal_max;
  p.modifier = f->scale_modifier;
  p.ewa = f->ewa;
  p.up_transforms = up_transforms;
  p.up_opacity = up_opacity;
  p.camera_sums = camera_sums;
  splat::aaa::aaa_camera_adjoint_kernel<<<blocks_for(f->n, 128), 128, 0, counted(s)>>>(p);
  return check_launch("aaa_camera_backward");
}

}  // extern "C"
