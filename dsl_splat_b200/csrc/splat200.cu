// C-ABI entry points of libsplat200 (declared in include/splat200.h).
//
// Plain device pointers, sizes and a cudaStream_t (as void*) in; a status
// code out (0 = success, negative = error; splat_last_error() describes the
// latest failure of the calling thread).  All work is enqueued on the given
// stream; nothing here allocates device memory: callers pass outputs and,
// for binning, a workspace sized by the *_workspace_bytes queries.
#include <algorithm>
#include <cstdio>
#include <cstring>
#include <mutex>
#include <string>

#include "binning.cuh"
#include "cameras.cuh"
#include "host_runtime.h"
#include "project.cuh"
#include "rade.cuh"
#include "render.cuh"
#include "splat_common.cuh"

using namespace splat;
using namespace splat::host;

namespace {

thread_local std::string g_last_error;

// Every kernel launch passes its stream through counted(), so
// splat_launch_count() reports how many kernels this library has launched.
unsigned long long g_launches = 0;

}  // namespace

namespace splat {
namespace host {

int fail(int status, const char* what) {
  g_last_error = what;
  return status;
}

int check_launch(const char* what) {
  const cudaError_t e = cudaGetLastError();
  if (e != cudaSuccess) {
    g_last_error = std::string(what) + ": " + cudaGetErrorString(e);
    return kCudaError;
  }
  return kOk;
}

cudaStream_t counted(cudaStream_t s) {
  __atomic_fetch_add(&g_launches, 1ULL, __ATOMIC_RELAXED);
  return s;
}

int sm_count() {
  int sms = 148, dev = 0;
  if (cudaGetDevice(&dev) == cudaSuccess)
    cudaDeviceGetAttribute(&sms, cudaDevAttrMultiProcessorCount, dev);
  return sms;
}

}  // namespace host
}  // namespace splat

namespace {

inline cudaStream_t as_stream(void* s) { return reinterpret_cast<cudaStream_t>(s); }

inline size_t align256(size_t x) { return (x + 255) & ~static_cast<size_t>(255); }

int tile_passes(int tiles) { return tiles <= 256 ? 1 : (tiles <= 65536 ? 2 : 3); }

// ---- binning workspace layout -------------------------------------------
// The chunked scatter (binning.cuh) keeps one uint32 per tile in shared
// memory per CTA; images whose tile grid does not fit use the onesweep path.
constexpr size_t kChunkSmemLimit = 200 * 1024;
constexpr size_t kChunkMatrixLimit = size_t(256) << 20;  // chunk-by-tile counts

struct ChunkPlan {
  bool use = false;
  uint32_t chunk = 0;      // Gaussians per chunk
  unsigned chunks = 0;     // K
  size_t smem_counts = 0;  // chunk_counts_kernel dynamic shared memory
  size_t smem_scatter = 0;
};

ChunkPlan chunk_plan(long long n, int gx, int gy, int tile_mode) {
  ChunkPlan c;
  // accutile tile sets are strips, not rectangles: the onesweep path emits them
  if (tile_mode == kTileAccutile) return c;
  const size_t T = static_cast<size_t>(gx) * gy;
  c.smem_counts = 4 * static_cast<size_t>(gx + 1) * (gy + 1);
  c.smem_scatter = 4 * T;
  if (c.smem_counts > kChunkSmemLimit || c.smem_scatter > kChunkSmemLimit) return c;
  // the uint32 work prefix (tiles + kChunkGaussianCost per Gaussian) must not wrap
  if (n > (1LL << 27)) return c;
  c.use = true;
  // Chunks are cut by work, not by count: about 1536 Gaussians each, and
  // large jobs get a whole number of rounds of kScatterSlots resident CTAs
  // (148 SMs x 6 by shared memory at 1080p; a fixed count keeps the plan
  // independent of the device queried).  Fewer chunks when the
  // chunk-by-tile matrix would grow large.
  constexpr size_t kScatterSlots = 148 * 6;
  const size_t nn = static_cast<size_t>(n > 0 ? n : 1);
  size_t chunks = (nn + 1535) / 1536;
  if (chunks > kScatterSlots / 2) chunks = (chunks + kScatterSlots - 1) / kScatterSlots * kScatterSlots;
  const size_t max_chunks = std::max<size_t>(1, kChunkMatrixLimit / (4 * T));
  c.chunks = static_cast<unsigned>(std::min(chunks, max_chunks));
  c.chunk = static_cast<uint32_t>((nn + c.chunks - 1) / c.chunks);
  return c;
}

struct BinLayout {
  size_t keys_a, vals_a, keys_b, vals_b, rects, offsets, block_sums;
  size_t zero_begin;  // everything from here to zero_end is cleared per call
  size_t depth_hist, diff, depth_status, counters, totals, work_status;
  size_t zero_end;
  size_t tile_digits;
  size_t chunk_counts, tile_totals, tile_starts, chunk_bounds, sorted_rects;  // chunked path
  size_t bytes;
};

// Depth passes: 256-thread onesweep blocks of kDepthItems keys per thread.
constexpr int kDepthThreads = 256;
constexpr int kDepthItems = 8;
size_t depth_tiles(long long n) {
  return static_cast<size_t>(blocks_for(n > 0 ? n : 1, kDepthThreads * kDepthItems));
}

BinLayout bin_layout(long long n, int width, int height, int tile_mode) {
  const int gx = (width + 15) / 16, gy = (height + 15) / 16;
  const size_t sort_tiles = static_cast<size_t>(blocks_for(n > 0 ? n : 1, kSortTile));
  const ChunkPlan plan = chunk_plan(n, gx, gy, tile_mode);
  const size_t T = static_cast<size_t>(gx) * gy;
  BinLayout L{};
  size_t o = 0;
  auto take = [&](size_t bytes) {
    const size_t at = o;
    o = align256(o + bytes);
    return at;
  };
  L.keys_a = take(4 * n);
  L.vals_a = take(4 * n);
  L.keys_b = take(4 * n);
  L.vals_b = take(4 * n);
  L.rects = take(8 * n);
  L.offsets = take(4 * (n + 1));  // pair offsets, or the work prefix of the chunked path
  L.block_sums = take(4 * (sort_tiles + 1));
  L.zero_begin = o;
  L.depth_hist = take(4 * 4 * kRadix);
  L.diff = take(plan.use ? 0 : 4 * static_cast<size_t>(gx + 1) * (gy + 1));
  L.depth_status = take(4 * 4 * depth_tiles(n) * kRadix);
  L.counters = take(4 * 8);  // onesweep tickets: depth passes 0-3, work scan 4
  L.totals = take(8 * 4);
  L.work_status = take(plan.use ? 8 * sort_tiles : 0);  // work scan look-back
  L.zero_end = o;
  L.tile_digits = take(plan.use ? 0 : 4 * 3 * kRadix);
  L.chunk_counts = take(plan.use ? 4 * static_cast<size_t>(plan.chunks) * T : 0);
  L.tile_totals = take(plan.use ? 4 * T : 0);
  L.tile_starts = take(plan.use ? 4 * T : 0);
  L.chunk_bounds = take(plan.use ? 4 * (static_cast<size_t>(plan.chunks) + 1) : 0);
  L.sorted_rects = take(plan.use ? 8 * n : 0);
  L.bytes = o;
  return L;
}

struct PairLayout {
  size_t keys0, vals0, keys1, vals1, status, counters, bytes;
};

PairLayout pair_layout(long long pairs, int width, int height, int tile_mode) {
  const int gx = (width + 15) / 16, gy = (height + 15) / 16;
  const int tiles = gx * gy;
  const int passes = tile_passes(tiles);
  const size_t sort_tiles = static_cast<size_t>(blocks_for(pairs > 0 ? pairs : 1, kSortTile));
  PairLayout L{};
  if (chunk_plan(1, gx, gy, tile_mode).use) return L;  // the chunked scatter needs no pair workspace
  // accutile materialises its pairs (keys0/vals0) before the first pass
  const bool emitted = tile_mode == kTileAccutile;
  size_t o = 0;
  auto take = [&](size_t bytes) {
    const size_t at = o;
    o = align256(o + bytes);
    return at;
  };
  L.keys0 = take(4 * pairs);
  L.vals0 = take(4 * pairs);
  L.keys1 = take(passes > 2 || (emitted && passes > 1) ? 4 * pairs : 0);
  L.vals1 = take(passes > 2 || (emitted && passes > 1) ? 4 * pairs : 0);
  L.status = take(4 * passes * sort_tiles * kRadix);
  L.counters = take(4 * 4);
  L.bytes = o;
  return L;
}

template <typename T>
T* at(void* base, size_t off) {
  return reinterpret_cast<T*>(static_cast<char*>(base) + off);
}

template <int DEG>
void launch_project_forward(const ProjectParams& p, cudaStream_t s) {
  project_forward_kernel<DEG><<<blocks_for(p.n, kProjectBlock), kProjectBlock, 0, counted(s)>>>(p);
}

int project_forward_dispatch(const ProjectParams& p, cudaStream_t s) {
  if (p.n == 0) return kOk;
  if (p.sh == nullptr) {
    launch_project_forward<-1>(p, s);
  } else {
    switch (p.sh_degree) {
      case 0: launch_project_forward<0>(p, s); break;
      case 1: launch_project_forward<1>(p, s); break;
      case 2: launch_project_forward<2>(p, s); break;
      case 3: launch_project_forward<3>(p, s); break;
      default: return fail(kInvalidArgument, "sh_degree must be in [0,3]");
    }
  }
  return check_launch("project_forward");
}

template <int DEG>
void launch_project_forward_views(const ProjectViewsParams& p, cudaStream_t s) {
  project_forward_views_kernel<DEG>
      <<<blocks_for(p.shared.n, kProjectBlock), kProjectBlock, 0, counted(s)>>>(p);
}

int project_forward_views_dispatch(const ProjectViewsParams& p, cudaStream_t s) {
  if (p.shared.n == 0 || p.views == 0) return kOk;
  if (p.shared.sh == nullptr) {
    launch_project_forward_views<-1>(p, s);
  } else {
    switch (p.shared.sh_degree) {
      case 0: launch_project_forward_views<0>(p, s); break;
      case 1: launch_project_forward_views<1>(p, s); break;
      case 2: launch_project_forward_views<2>(p, s); break;
      case 3: launch_project_forward_views<3>(p, s); break;
      default: return fail(kInvalidArgument, "sh_degree must be in [0,3]");
    }
  }
  return check_launch("project_forward_views");
}

template <int CHP>
void launch_render(const RenderParams& p, bool backward, cudaStream_t s) {
  const unsigned tiles = static_cast<unsigned>(p.gx * ((p.height + 15) / 16));
  // The staged batch lives in dynamic shared memory; the 32-channel variant
  // needs more than the default 48 KB (opt-in, per device, cheap to repeat).
  const size_t smem = sizeof(RenderShared<CHP>);
  if (backward) {
    if constexpr (CHP == 4) {
      // four channels: two pixels per lane as f32x2 pairs (128 threads per tile)
      render_backward2_kernel<<<tiles, kBlock / 2, smem, counted(s)>>>(p);
    } else {
      if (smem > 32 * 1024)
        cudaFuncSetAttribute(render_backward_kernel<CHP, 1>,
                             cudaFuncAttributeMaxDynamicSharedMemorySize, static_cast<int>(smem));
      render_backward_kernel<CHP, 1><<<tiles, kBlock, smem, counted(s)>>>(p);
    }
  } else if (CHP <= 8) {
    // up to eight channels: two pixels per lane with paired arithmetic
    if (smem > 32 * 1024)
      cudaFuncSetAttribute(p.stat_count ? render_forward2_kernel<CHP, true>
                                        : render_forward2_kernel<CHP, false>,
                           cudaFuncAttributeMaxDynamicSharedMemorySize, static_cast<int>(smem));
    // statistics requests get their own instantiation (no per-sample test)
    if (p.stat_count)
      render_forward2_kernel<CHP, true><<<tiles, kBlock / 2, smem, counted(s)>>>(p);
    else
      render_forward2_kernel<CHP, false><<<tiles, kBlock / 2, smem, counted(s)>>>(p);
  } else {
    if (smem > 32 * 1024)
      cudaFuncSetAttribute(render_forward_kernel<CHP>,
                           cudaFuncAttributeMaxDynamicSharedMemorySize, static_cast<int>(smem));
    render_forward_kernel<CHP><<<tiles, kBlock, smem, counted(s)>>>(p);
  }
}

int render_dispatch(const RenderParams& p, bool backward, cudaStream_t s) {
  if (p.channels <= 4)
    launch_render<4>(p, backward, s);
  else if (p.channels <= 8)
    launch_render<8>(p, backward, s);
  else if (p.channels <= 16)
    launch_render<16>(p, backward, s);
  else if (p.channels <= 32)
    launch_render<32>(p, backward, s);
  else
    return fail(kInvalidArgument, "at most 32 blended channels are supported");
  return check_launch(backward ? "render_backward" : "render_forward");
}

template <int CHP>
void launch_rade(const RadeRenderParams& p, bool backward, cudaStream_t s) {
  const unsigned tiles = static_cast<unsigned>(p.base.gx * ((p.base.height + 15) / 16));
  const size_t smem = sizeof(RenderShared<CHP>) + sizeof(RadeShared);
  if (backward) {
    // one pixel per lane (see rade_backward_kernel on the measured variants)
    if (smem > 32 * 1024)
      cudaFuncSetAttribute(rade_backward_kernel<CHP, 1>,
                           cudaFuncAttributeMaxDynamicSharedMemorySize, static_cast<int>(smem));
    rade_backward_kernel<CHP, 1><<<tiles, kBlock, smem, counted(s)>>>(p);
  } else {
    // two pixels per lane with paired arithmetic (kBlock / 2 threads per tile)
    if (smem > 32 * 1024)
      cudaFuncSetAttribute(rade_forward2_kernel<CHP>, cudaFuncAttributeMaxDynamicSharedMemorySize,
                           static_cast<int>(smem));
    rade_forward2_kernel<CHP><<<tiles, kBlock / 2, smem, counted(s)>>>(p);
  }
}

int rade_render_dispatch(const RadeRenderParams& p, bool backward, cudaStream_t s) {
  const int c = p.base.channels;
  if (c <= 4)
    launch_rade<4>(p, backward, s);
  else if (c <= 8)
    launch_rade<8>(p, backward, s);
  else if (c <= 16)
    launch_rade<16>(p, backward, s);
  else if (c <= 32)
    launch_rade<32>(p, backward, s);
  else if (c <= 36)
    launch_rade<36>(p, backward, s);
  else if (c <= 48)
    launch_rade<48>(p, backward, s);
  else if (c <= 64)
    launch_rade<64>(p, backward, s);
  else
    return fail(kInvalidArgument, "at most 64 blended channels are supported");
  return check_launch(backward ? "rade_render_backward" : "rade_render_forward");
}

// Shared argument checks and RenderParams fields of the two rade blend entries.
int rade_render_params(int width, int height, const int* ranges, const int* tile_order,
                       const int* ids, long long num_ids, int n, const float* centers,
                       const float* conics, const float* planes, const float* normals,
                       const float* colors, int ch_a, int stride_a, const float* extras, int ch_b,
                       int stride_b, const float* background, const float* K,
                       RadeRenderParams& p) {
  if (width <= 0 || height <= 0 || ch_a < 0 || ch_b < 0 || ch_a + ch_b <= 0 || n < 0 ||
      num_ids < 0 || num_ids >= (1LL << 31) || (ch_a > 0 && stride_a < ch_a) ||
      (ch_b > 0 && stride_b < ch_b))
    return fail(kInvalidArgument, "bad rade render sizes");
  // per-Gaussian rows are only read when there are Gaussians (an empty
  // tensor may have a null address)
  if (n > 0 && ((ch_a > 0 && !colors) || (ch_b > 0 && !extras) || !centers || !conics ||
                !planes || !normals))
    return fail(kInvalidArgument, "null rade render input");
  if (!ranges || (num_ids > 0 && !ids) || !background || !K)
    return fail(kInvalidArgument, "null rade render input");
  if (!aligned(centers, 8) || !aligned(conics, 16))
    return fail(kInvalidArgument, "center rows need 8-byte and conic rows 16-byte alignment");
  p = RadeRenderParams{};
  RenderParams& b = p.base;
  b.width = width;
  b.height = height;
  b.gx = (width + 15) / 16;
  b.ranges = ranges;
  b.tile_order = tile_order;
  b.ids = ids;
  b.num_ids = static_cast<int>(num_ids);
  b.n_gaussians = n;
  b.centers = centers;
  b.conics = conics;
  b.feat_a = colors;
  b.ch_a = ch_a;
  b.stride_a = stride_a;
  b.feat_b = extras;
  b.ch_b = ch_b;
  b.stride_b = stride_b;
  b.append_one = 0;
  b.channels = ch_a + ch_b;
  b.background = background;
  p.planes = planes;
  p.normals = normals;
  p.K = K;
  return kOk;
}

}  // namespace

extern "C" {

int splat_abi_version(void) { return 1; }

unsigned long long splat_launch_count(void) { return __atomic_load_n(&g_launches, __ATOMIC_RELAXED); }

const char* splat_last_error(void) { return g_last_error.c_str(); }

int splat_device_error(int* code, void* stream) {
  if (!code) return fail(kInvalidArgument, "code must not be null");
  cudaStream_t s = as_stream(stream);
  int value = 0;
  if (cudaMemcpyFromSymbolAsync(&value, g_splat_device_error, sizeof(int), 0,
                                cudaMemcpyDeviceToHost, s) != cudaSuccess ||
      cudaStreamSynchronize(s) != cudaSuccess)
    return check_launch("splat_device_error");
  const int zero = 0;
  if (cudaMemcpyToSymbolAsync(g_splat_device_error, &zero, sizeof(int), 0,
                              cudaMemcpyHostToDevice, s) != cudaSuccess ||
      cudaStreamSynchronize(s) != cudaSuccess)
    return check_launch("splat_device_error reset");
  *code = value;
  return kOk;
}

int splat_device_error_read(int* device_dst, void* stream) {
  if (!device_dst) return fail(kInvalidArgument, "device_dst must not be null");
  cudaStream_t s = as_stream(stream);
  void* word = nullptr;
  if (cudaGetSymbolAddress(&word, g_splat_device_error) != cudaSuccess)
    return check_launch("splat_device_error_read: symbol");
  if (cudaMemcpyAsync(device_dst, word, sizeof(int), cudaMemcpyDeviceToDevice, s) != cudaSuccess ||
      cudaMemsetAsync(word, 0, sizeof(int), s) != cudaSuccess)
    return check_launch("splat_device_error_read");
  return kOk;
}

int splat_test_lookback_expiry(const unsigned* status, unsigned spin_limit, unsigned* out,
                               void* stream) {
  if (!status || !out) return fail(kInvalidArgument, "null status/out");
  if (spin_limit > (1u << 20)) return fail(kInvalidArgument, "spin_limit above 2^20");
  lookback_expiry_kernel<<<1, 32, 0, counted(as_stream(stream))>>>(status, spin_limit, out);
  return check_launch("test_lookback_expiry");
}

// ---- cameras -------------------------------------------------------------

int splat_cameras_prepare(int count, const float* views, const float* Ks, int width, int height,
                          int with_centers, float* full, float* inverse, float* centers,
                          int* errors, void* stream) {
  if (count < 0 || width <= 0 || height <= 0) return fail(kInvalidArgument, "bad camera sizes");
  if (count == 0) return kOk;
  if (!views || !Ks || !full || !errors || (with_centers && (!inverse || !centers)))
    return fail(kInvalidArgument, "null camera buffer");
  cameras_prepare_kernel<<<blocks_for(count, 64), 64, 0, counted(as_stream(stream))>>>(
      count, views, Ks, width, height, with_centers, full, inverse, centers, errors);
  return check_launch("cameras_prepare");
}

int splat_cameras_backward(int count, const float* Ks, const float* grad_full, int width,
                           int height, const float* inverse, const float* grad_centers,
                           float* grad_views, void* stream) {
  if (count < 0 || width <= 0 || height <= 0) return fail(kInvalidArgument, "bad camera sizes");
  if (count == 0) return kOk;
  if (!Ks || !grad_views || (grad_centers && !inverse))
    return fail(kInvalidArgument, "null camera buffer");
  cameras_backward_kernel<<<blocks_for(count, 64), 64, 0, counted(as_stream(stream))>>>(
      count, Ks, grad_full, width, height, inverse, grad_centers, grad_views);
  return check_launch("cameras_backward");
}

// ---- projection ----------------------------------------------------------

int splat_project_forward(int n, const float* means, const float* quats, const float* scales,
                          const float* opacities, const float* view, const float* proj,
                          const float* K, int width, int height, float near_plane,
                          float far_plane, float radius_clip, float* centers, float* conics,
                          int* radii, int* tiles, float* depths, int tile_mode, void* stream) {
  if (n < 0 || width <= 0 || height <= 0) return fail(kInvalidArgument, "bad projection sizes");
  if (tile_mode < kTileRadius || tile_mode > kTileAccutile)
    return fail(kInvalidArgument, "tile_mode must be 0 (radius), 1 (snugbox) or 2 (accutile)");
  if (!aligned(quats, 16) || !aligned(conics, 16) || !aligned(centers, 8))
    return fail(kInvalidArgument, "quats/conics need 16-byte and centers 8-byte alignment");
  ProjectParams p{};
  p.n = n;
  p.tile_mode = tile_mode;
  p.means = means;
  p.quats = quats;
  p.scales = scales;
  p.opacities = opacities;
  p.view = view;
  p.proj = proj;
  p.K = K;
  p.width = width;
  p.height = height;
  p.near_plane = near_plane;
  p.far_plane = far_plane;
  p.radius_clip = radius_clip;
  p.centers = centers;
  p.conics = conics;
  p.radii = radii;
  p.tiles = tiles;
  p.depths = depths;
  return project_forward_dispatch(p, as_stream(stream));
}

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
                                void* stream) {
  if (n < 0 || width <= 0 || height <= 0) return fail(kInvalidArgument, "bad projection sizes");
  if (tile_mode < kTileRadius || tile_mode > kTileAccutile)
    return fail(kInvalidArgument, "tile_mode must be 0 (radius), 1 (snugbox) or 2 (accutile)");
  if (sh && (sh_degree < 0 || sh_degree > 3 || sh_k < (sh_degree + 1) * (sh_degree + 1) ||
             !colors || color_stride < 3))
    return fail(kInvalidArgument, "bad SH arguments");
  if (meta_means2d && (!meta_opacities || !meta_conics))
    return fail(kInvalidArgument, "metadata outputs come together");
  if (!aligned(meta_means2d, 8)) return fail(kInvalidArgument, "means2d needs 8-byte alignment");
  if (!aligned(quats, 16)) return fail(kInvalidArgument, "quats need 16-byte alignment");
  ProjectParams p{};
  p.n = n;
  p.means = means;
  p.quats = quats;
  p.normalize_quats = normalize_quats ? 1 : 0;
  p.tile_mode = tile_mode;
  p.scales = scales;
  p.opacities = opacities;
  p.view = view;
  p.proj = proj;
  p.K = K;
  p.width = width;
  p.height = height;
  p.near_plane = near_plane;
  p.far_plane = far_plane;
  p.radius_clip = radius_clip;
  p.centers = centers;
  p.conics = conics;
  p.radii = radii;
  p.tiles = tiles;
  p.depths = depths;
  p.sh_degree = sh_degree;
  p.sh_k = sh_k;
  p.sh = sh;
  p.campos = campos;
  p.colors = colors;
  p.color_stride = color_stride;
  p.active = active;
  p.meta_means2d = meta_means2d;
  p.meta_opacities = meta_opacities;
  p.meta_conics = meta_conics;
  return project_forward_dispatch(p, as_stream(stream));
}

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
                                int tile_mode, void* stream) {
  if (views < 0 || n < 0 || width <= 0 || height <= 0)
    return fail(kInvalidArgument, "bad projection sizes");
  if (tile_mode < kTileRadius || tile_mode > kTileAccutile)
    return fail(kInvalidArgument, "tile_mode must be 0 (radius), 1 (snugbox) or 2 (accutile)");
  if (sh && (sh_degree < 0 || sh_degree > 3 || sh_k < (sh_degree + 1) * (sh_degree + 1) ||
             !colors || color_stride < 3))
    return fail(kInvalidArgument, "bad SH arguments");
  if (!centers || !conics || !radii || !tiles || !depths)
    return fail(kInvalidArgument, "the per-view output tables are required");
  if (meta_means2d && (!meta_opacities || !meta_conics))
    return fail(kInvalidArgument, "metadata outputs come together");
  if (!aligned(quats, 16)) return fail(kInvalidArgument, "quats need 16-byte alignment");
  for (int v = 0; v < views; ++v)
    if (!aligned(centers[v], 8) || !aligned(conics[v], 16) ||
        (meta_means2d && !aligned(meta_means2d[v], 8)))
      return fail(kInvalidArgument, "centre rows need 8-byte, conic rows 16-byte alignment");
  ProjectViewsParams vp{};
  ProjectParams& p = vp.shared;
  p.n = n;
  p.means = means;
  p.quats = quats;
  p.normalize_quats = normalize_quats ? 1 : 0;
  p.tile_mode = tile_mode;
  p.scales = scales;
  p.opacities = opacities;
  p.width = width;
  p.height = height;
  p.near_plane = near_plane;
  p.far_plane = far_plane;
  p.radius_clip = radius_clip;
  p.sh_degree = sh_degree;
  p.sh_k = sh_k;
  p.sh = sh;
  p.color_stride = color_stride;
  // at most kMaxViews cameras per launch
  for (int v0 = 0; v0 < views; v0 += kMaxViews) {
    vp.views = std::min(kMaxViews, views - v0);
    vp.viewmats = viewmats + 16 * v0;
    vp.projs = projs + 16 * v0;
    vp.Ks = Ks + 9 * v0;
    vp.campos = campos ? campos + 3 * v0 : nullptr;
    for (int v = 0; v < vp.views; ++v) {
      vp.centers[v] = centers[v0 + v];
      vp.conics[v] = conics[v0 + v];
      vp.radii[v] = radii[v0 + v];
      vp.tiles[v] = tiles[v0 + v];
      vp.depths[v] = depths[v0 + v];
      vp.colors[v] = colors ? colors[v0 + v] : nullptr;
      vp.active[v] = active ? active[v0 + v] : nullptr;
      vp.meta_means2d[v] = meta_means2d ? meta_means2d[v0 + v] : nullptr;
      vp.meta_opacities[v] = meta_opacities ? meta_opacities[v0 + v] : nullptr;
      vp.meta_conics[v] = meta_conics ? meta_conics[v0 + v] : nullptr;
    }
    const int r = project_forward_views_dispatch(vp, as_stream(stream));
    if (r != kOk) return r;
  }
  return kOk;
}

int splat_metadata(int n, const int* radii, const float* centers, const float* conics,
                   float* means2d, float* opacities, float* conics3, void* stream) {
  if (n < 0) return fail(kInvalidArgument, "n < 0");
  if (n == 0) return kOk;
  if (!aligned(centers, 8) || !aligned(conics, 16) || !aligned(means2d, 8))
    return fail(kInvalidArgument, "centers/means2d need 8-byte and conics 16-byte alignment");
  metadata_kernel<<<blocks_for(n, 256), 256, 0, counted(as_stream(stream))>>>(n, radii, centers, conics,
                                                                     means2d, opacities, conics3);
  return check_launch("metadata");
}

int splat_project_backward(int n, const float* means, const float* quats, const float* scales,
                           const float* view, const float* proj, const float* K, int width,
                           int height, const int* radii, const float* grad_centers,
                           const float* grad_conics, float* grad_means, float* grad_quats,
                           float* grad_scales, float* grad_opacities, float* camera_grads,
                           void* stream) {
  if (n < 0 || width <= 0 || height <= 0) return fail(kInvalidArgument, "bad projection sizes");
  if (!aligned(quats, 16) || !aligned(grad_quats, 16) || !aligned(grad_conics, 16) ||
      !aligned(grad_centers, 8))
    return fail(kInvalidArgument, "quat/conic rows need 16-byte, center rows 8-byte alignment");
  ProjectBackwardParams p{};
  p.n = n;
  p.means = means;
  p.quats = quats;
  p.scales = scales;
  p.view = view;
  p.proj = proj;
  p.K = K;
  p.width = width;
  p.height = height;
  p.radii = radii;
  p.seed_centers = grad_centers;
  p.seed_conics = grad_conics;
  p.grad_means = grad_means;
  p.grad_quats = grad_quats;
  p.grad_scales = grad_scales;
  p.grad_opacities = grad_opacities;
  p.cam_grads = camera_grads;
  return project_backward_dispatch(p, as_stream(stream));
}

int splat_project_backward_fused(int n, const float* means, const float* quats,
                                 const float* quats_raw, const float* scales,
                                 const float* view, const float* proj,
                                 const float* K, int width, int height, const int* radii,
                                 const float* grad_centers, const float* grad_conics,
                                 float* grad_means, float* grad_quats, float* grad_scales,
                                 float* grad_opacities, int accumulate, float* camera_grads,
                                 int sh_degree, int sh_k, const float* sh, const float* campos,
                                 const unsigned char* active, const float* grad_colors,
                                 int color_stride, float* grad_sh, void* stream) {
  if (n < 0 || width <= 0 || height <= 0) return fail(kInvalidArgument, "bad projection sizes");
  if (grad_sh && (!sh || !active || !grad_colors || sh_degree < 0 || sh_degree > 3 ||
                  sh_k < (sh_degree + 1) * (sh_degree + 1)))
    return fail(kInvalidArgument, "bad SH backward arguments");
  if (!quats && !quats_raw) return fail(kInvalidArgument, "quats or quats_raw is required");
  if (!aligned(quats, 16) || !aligned(quats_raw, 16) || !aligned(grad_quats, 16) ||
      !aligned(grad_conics, 16) ||
      !aligned(grad_centers, 8))
    return fail(kInvalidArgument, "quat/conic rows need 16-byte, center rows 8-byte alignment");
  ProjectBackwardParams p{};
  p.n = n;
  p.means = means;
  p.quats = quats;
  p.scales = scales;
  p.view = view;
  p.proj = proj;
  p.K = K;
  p.width = width;
  p.height = height;
  p.radii = radii;
  p.seed_centers = grad_centers;
  p.seed_conics = grad_conics;
  p.grad_means = grad_means;
  p.grad_quats = grad_quats;
  p.grad_scales = grad_scales;
  p.grad_opacities = grad_opacities;
  p.accumulate = accumulate;
  p.cam_grads = camera_grads;
  p.sh_degree = sh_degree;
  p.sh_k = sh_k;
  p.sh = sh;
  p.campos = campos;
  p.active = active;
  p.seed_colors = grad_colors;
  p.color_stride = color_stride;
  p.grad_sh = grad_sh;
  p.quats_raw = quats_raw;
  return project_backward_dispatch(p, as_stream(stream));
}

// ---- spherical harmonics ---------------------------------------------------

int splat_sh_forward(int n, int degree, int sh_k, const float* sh, const float* dirs,
                     const int* radii, float* colors, unsigned char* active, void* stream) {
  if (n < 0 || degree < 0 || degree > 3 || sh_k < (degree + 1) * (degree + 1))
    return fail(kInvalidArgument, "bad SH arguments");
  if (n == 0) return kOk;
  cudaStream_t s = as_stream(stream);
  const unsigned g = blocks_for(n, kProjectBlock);
  switch (degree) {
    case 0: sh_forward_kernel<0><<<g, kProjectBlock, 0, counted(s)>>>(n, sh_k, sh, dirs, radii, colors, active); break;
    case 1: sh_forward_kernel<1><<<g, kProjectBlock, 0, counted(s)>>>(n, sh_k, sh, dirs, radii, colors, active); break;
    case 2: sh_forward_kernel<2><<<g, kProjectBlock, 0, counted(s)>>>(n, sh_k, sh, dirs, radii, colors, active); break;
    default: sh_forward_kernel<3><<<g, kProjectBlock, 0, counted(s)>>>(n, sh_k, sh, dirs, radii, colors, active); break;
  }
  return check_launch("sh_forward");
}

int splat_sh_backward(int n, int degree, int sh_k, const float* sh, const float* dirs,
                      const int* radii, const unsigned char* active, const float* upstream,
                      float* grad_sh, float* grad_dirs, void* stream) {
  if (n < 0 || degree < 0 || degree > 3 || sh_k < (degree + 1) * (degree + 1))
    return fail(kInvalidArgument, "bad SH arguments");
  if (n == 0) return kOk;
  cudaStream_t s = as_stream(stream);
  const unsigned g = blocks_for(n, kProjectBlock);
  switch (degree) {
    case 0: sh_backward_kernel<0><<<g, kProjectBlock, 0, counted(s)>>>(n, sh_k, sh, dirs, radii, active, upstream, grad_sh, grad_dirs); break;
    case 1: sh_backward_kernel<1><<<g, kProjectBlock, 0, counted(s)>>>(n, sh_k, sh, dirs, radii, active, upstream, grad_sh, grad_dirs); break;
    case 2: sh_backward_kernel<2><<<g, kProjectBlock, 0, counted(s)>>>(n, sh_k, sh, dirs, radii, active, upstream, grad_sh, grad_dirs); break;
    default: sh_backward_kernel<3><<<g, kProjectBlock, 0, counted(s)>>>(n, sh_k, sh, dirs, radii, active, upstream, grad_sh, grad_dirs); break;
  }
  return check_launch("sh_backward");
}

// ---- scan -------------------------------------------------------------------

size_t splat_scan_workspace_bytes(int n) {
  return 4 * (static_cast<size_t>(blocks_for(n > 0 ? n : 1, kSortTile)) + 2) + 256;
}

int splat_scan_counts(int n, const int* counts, int* offsets, long long* total, void* workspace,
                      size_t workspace_bytes, void* stream) {
  if (n < 0) return fail(kInvalidArgument, "n < 0");
  if (workspace_bytes < splat_scan_workspace_bytes(n))
    return fail(kWorkspaceTooSmall, "scan workspace too small");
  cudaStream_t s = as_stream(stream);
  uint32_t* block_sums = static_cast<uint32_t*>(workspace);
  const unsigned nb = blocks_for(n > 0 ? n : 1, kSortTile);
  if (n == 0) {
    if (total && cudaMemsetAsync(total, 0, sizeof(long long), s) != cudaSuccess)
      return check_launch("scan_counts");
    return kOk;
  }
  // the total is summed in 64 bits (never wraps); above INT32_MAX the device
  // error word receives kTooLarge, since the int32 offsets cannot hold it
  scan_count_block_sums_kernel<<<nb, kSortBlock, 0, counted(s)>>>(counts, n, block_sums);
  scan_count_prefix_kernel<<<1, 1024, 0, counted(s)>>>(block_sums, nb, total);
  scan_apply_kernel<<<nb, kSortBlock, 0, counted(s)>>>(counts, nullptr, n, block_sums, 1,
                                             reinterpret_cast<uint32_t*>(offsets));
  return check_launch("scan_counts");
}

}  // extern "C"

// ---- scan without caller scratch ------------------------------------------------
// Some callers cannot hand this library any device memory at call time: a
// host whose device memory is all owned by its own pool, a render loop that
// cannot afford cudaMalloc's implicit synchronisation, or a plugin running
// where its framework forbids new allocations.  splat_scan_counts_static
// serves them: the scan's block sums live in this file-scope array instead of
// a caller workspace.  Every GPU that loads the library holds the array
// (64 KiB) until the process exits.  It bounds n to kStaticScanBlocks blocks
// of kSortTile counts.
namespace {
constexpr unsigned kStaticScanBlocks = 16384;
constexpr long long kStaticScanMaxCount =
    static_cast<long long>(kStaticScanBlocks) * kSortTile;  // 67,108,864
static __device__ __align__(256) uint32_t g_static_scan_scratch[kStaticScanBlocks + 2];

// Device address of g_static_scan_scratch per device ordinal.  The host-side
// symbol is only a stand-in; the address comes from cudaGetSymbolAddress,
// called once per device with that device current.  The cached address
// belongs to that device's context: a process that resets the device
// (cudaDeviceReset) and keeps using this library must not call the static
// scan again afterwards (the address would be stale).
std::mutex g_static_scan_mutex;
void* g_static_scan_address[256] = {};

int static_scan_scratch(uint32_t** out) {
  int device = 0;
  if (cudaGetDevice(&device) != cudaSuccess || device < 0 || device >= 256)
    return check_launch("static scan: cudaGetDevice");
  std::lock_guard<std::mutex> lock(g_static_scan_mutex);
  if (g_static_scan_address[device] == nullptr) {
    void* address = nullptr;
    const cudaError_t e = cudaGetSymbolAddress(&address, g_static_scan_scratch);
    if (e != cudaSuccess || address == nullptr) {
      g_last_error = std::string("static scan: cudaGetSymbolAddress: ") + cudaGetErrorString(e);
      cudaGetLastError();
      return kCudaError;
    }
    g_static_scan_address[device] = address;
  }
  *out = static_cast<uint32_t*>(g_static_scan_address[device]);
  return kOk;
}
}  // namespace

extern "C" {

int splat_scan_counts_static(int n, const int* counts, int* offsets, long long* total,
                             void* stream) {
  if (n < 0) return fail(kInvalidArgument, "n < 0");
  if (n > kStaticScanMaxCount)
    return fail(kTooLarge, "splat_scan_counts_static handles at most 67108864 counts "
                           "(16384 blocks of 4096); use splat_scan_counts with a workspace");
  uint32_t* block_sums = nullptr;
  const int r = static_scan_scratch(&block_sums);
  if (r != kOk) return r;
  cudaStream_t s = as_stream(stream);
  if (n == 0) {
    if (total && cudaMemsetAsync(total, 0, sizeof(long long), s) != cudaSuccess)
      return check_launch("scan_counts_static");
    return kOk;
  }
  // Each call overwrites every block sum and the total it reads, so nothing
  // left by an earlier call needs clearing.
  const unsigned nb = blocks_for(n, kSortTile);
  scan_count_block_sums_kernel<<<nb, kSortBlock, 0, counted(s)>>>(counts, n, block_sums);
  scan_count_prefix_kernel<<<1, 1024, 0, counted(s)>>>(block_sums, nb, total);
  scan_apply_kernel<<<nb, kSortBlock, 0, counted(s)>>>(counts, nullptr, n, block_sums, 1,
                                                       reinterpret_cast<uint32_t*>(offsets));
  return check_launch("scan_counts_static");
}

// ---- binning ------------------------------------------------------------------

size_t splat_bin_workspace_bytes(int n, int width, int height, int tile_mode) {
  return bin_layout(n, width, height, tile_mode).bytes;
}

size_t splat_bin_pairs_workspace_bytes(long long pairs, int width, int height, int tile_mode) {
  return pair_layout(pairs, width, height, tile_mode).bytes;
}

int splat_bin_prepare(int n, const float* centers, const float* conics, const int* radii,
                      const int* tiles, const float* depths, int width, int height, int tile_mode,
                      void* workspace, size_t workspace_bytes, int* ranges, long long* pairs,
                      void* stream) {
  if (n < 0 || width <= 0 || height <= 0) return fail(kInvalidArgument, "bad binning sizes");
  if (tile_mode < kTileRadius || tile_mode > kTileAccutile)
    return fail(kInvalidArgument, "tile_mode must be 0 (radius), 1 (snugbox) or 2 (accutile)");
  if (tile_mode != kTileRadius && !conics)
    return fail(kInvalidArgument, "SnugBox/AccuTile require projected conics");
  if (!aligned(conics, 16)) return fail(kInvalidArgument, "conics need 16-byte alignment");
  const int gx = (width + 15) / 16, gy = (height + 15) / 16;
  if (gx > 65535 || gy > 65535 || static_cast<long long>(gx) * gy >= (1LL << 24))
    return fail(kTooLarge, "image has too many tiles");
  if (n >= (1 << 30)) return fail(kTooLarge, "too many Gaussians");
  const BinLayout L = bin_layout(n, width, height, tile_mode);
  if (!workspace || workspace_bytes < L.bytes) return fail(kWorkspaceTooSmall, "bin workspace too small");
  if (!ranges || !pairs) return fail(kInvalidArgument, "null ranges/pairs");
  if (!aligned(centers, 8) || !aligned(ranges, 8) || !aligned(workspace, 256))
    return fail(kInvalidArgument, "centers and ranges need 8-byte, workspace 256-byte alignment");
  cudaStream_t s = as_stream(stream);
  char* ws = static_cast<char*>(workspace);
  if (cudaMemsetAsync(ws + L.zero_begin, 0, L.zero_end - L.zero_begin, s) != cudaSuccess)
    return check_launch("bin_prepare memset");
  const int T = gx * gy;
  if (n == 0) {
    if (cudaMemsetAsync(ranges, 0, sizeof(int) * 2 * T, s) != cudaSuccess ||
        cudaMemsetAsync(pairs, 0, sizeof(long long), s) != cudaSuccess)
      return check_launch("bin_prepare empty");
    return kOk;
  }
  uint32_t* keys_a = at<uint32_t>(ws, L.keys_a);
  uint32_t* vals_a = at<uint32_t>(ws, L.vals_a);
  uint32_t* keys_b = at<uint32_t>(ws, L.keys_b);
  uint32_t* vals_b = at<uint32_t>(ws, L.vals_b);
  uint2* rects = at<uint2>(ws, L.rects);
  uint32_t* offsets = at<uint32_t>(ws, L.offsets);
  uint32_t* block_sums = at<uint32_t>(ws, L.block_sums);
  uint32_t* hist = at<uint32_t>(ws, L.depth_hist);
  int* diff = at<int>(ws, L.diff);
  uint32_t* status = at<uint32_t>(ws, L.depth_status);
  uint32_t* counters = at<uint32_t>(ws, L.counters);
  uint32_t* totals = at<uint32_t>(ws, L.totals);
  uint32_t* tile_digits = at<uint32_t>(ws, L.tile_digits);
  const unsigned sort_tiles = blocks_for(n, kSortTile);
  // depth passes: 256-thread onesweep blocks of kDepthItems keys per thread
  // (1024-thread blocks of 16 measured 36 us per pass at 1M keys, 256 x 16
  // 28 us: at this size more blocks in flight beat a shorter look-back chain)
  const unsigned dtiles = static_cast<unsigned>(depth_tiles(n));
  const ChunkPlan plan = chunk_plan(n, gx, gy, tile_mode);
  if (plan.use) diff = nullptr;
  const int sms = sm_count();
  const unsigned prep_grid = std::min<unsigned>(blocks_for(n, 256), static_cast<unsigned>(sms * 8));
  unsigned long long* total64 = at<unsigned long long>(ws, L.totals + 8);
  bin_prepare_kernel<<<prep_grid, 256, 0, counted(s)>>>(n, centers, conics, radii, tiles, depths,
                                                        gx, gy, tile_mode, keys_a, vals_a, rects,
                                                        diff, hist, total64);
  // four stable passes over the 32-bit depth keys: a -> b -> a -> b -> a
  for (int pass = 0; pass < 4; ++pass) {
    const bool even = (pass % 2) == 0;
    KeyValueLoader ld{even ? keys_a : keys_b, even ? vals_a : vals_b};
    onesweep_kernel<KeyValueLoader, true, kDepthThreads, kDepthItems, true>
        <<<dtiles, kDepthThreads, 0, counted(s)>>>(
            ld, static_cast<uint32_t>(n), 8 * pass, hist + pass * kRadix,
            status + static_cast<size_t>(pass) * dtiles * kRadix, counters + pass,
            even ? keys_b : keys_a, even ? vals_b : vals_a);
  }
  if (plan.use) {
    // per-(chunk, tile) pair counts of the depth-ordered Gaussians, their
    // prefix over chunks, and the tile ranges
    uint32_t* cnt = at<uint32_t>(ws, L.chunk_counts);
    uint32_t* tile_totals = at<uint32_t>(ws, L.tile_totals);
    uint32_t* bounds = at<uint32_t>(ws, L.chunk_bounds);
    // work prefix in depth order (tiles + a per-Gaussian cost) and the chunk
    // bounds, one pass (the total is bin_prepare's pair count + cost * n)
    work_scan_kernel<<<sort_tiles, kSortBlock, 0, counted(s)>>>(
        tiles, vals_a, static_cast<uint32_t>(n), kChunkGaussianCost, total64, plan.chunks,
        at<unsigned long long>(ws, L.work_status), counters + 4, offsets, bounds);
    if (plan.smem_counts > 48 * 1024)
      cudaFuncSetAttribute(chunk_counts_kernel, cudaFuncAttributeMaxDynamicSharedMemorySize,
                           static_cast<int>(plan.smem_counts));
    chunk_counts_kernel<<<plan.chunks, 256, plan.smem_counts, counted(s)>>>(
        vals_a, bounds, rects, gx, gy, at<uint2>(ws, L.sorted_rects), cnt);
    chunk_prefix_kernel<<<blocks_for(T, 32), 1024, 0, counted(s)>>>(cnt, plan.chunks, T,
                                                                      tile_totals);
    tile_ranges_kernel<<<1, 1024, 0, counted(s)>>>(tile_totals, T, ranges,
                                                   at<uint32_t>(ws, L.tile_starts), totals + 1);
  } else {
    // pair offsets in depth order: offsets[j] = sum of tiles[order[i]], i < j
    scan_block_sums_kernel<<<sort_tiles, kSortBlock, 0, counted(s)>>>(tiles, vals_a, n, block_sums);
    scan_block_prefix_kernel<<<1, 1024, 0, counted(s)>>>(block_sums, sort_tiles, totals + 0);
    scan_apply_kernel<<<sort_tiles, kSortBlock, 0, counted(s)>>>(tiles, vals_a, n, block_sums, 0,
                                                                 offsets);
    tile_counts_kernel<<<1, 1024, 0, counted(s)>>>(diff, gx, gy, tile_passes(T), ranges,
                                                   tile_digits, totals + 1);
  }
  // The 64-bit total cannot wrap; splat_bin_emit refuses totals >= 2^30.
  if (cudaMemcpyAsync(pairs, total64, sizeof(long long), cudaMemcpyDeviceToDevice, s) != cudaSuccess)
    return check_launch("bin_prepare pairs");
  return check_launch("bin_prepare");
}

int splat_bin_emit(int n, long long pairs, int width, int height, int tile_mode,
                   const float* centers, const float* conics, const int* radii, void* workspace,
                   size_t workspace_bytes, void* pairs_workspace, size_t pairs_workspace_bytes,
                   int* ids, void* stream) {
  if (n < 0 || pairs < 0 || width <= 0 || height <= 0) return fail(kInvalidArgument, "bad sizes");
  if (pairs >= (1LL << 30)) return fail(kTooLarge, "more than 2^30 Gaussian-tile pairs");
  if (tile_mode < kTileRadius || tile_mode > kTileAccutile)
    return fail(kInvalidArgument, "tile_mode must be 0 (radius), 1 (snugbox) or 2 (accutile)");
  if (tile_mode == kTileAccutile && (!centers || !conics || !radii))
    return fail(kInvalidArgument, "AccuTile emission needs centers, conics and radii");
  if (!aligned(centers, 8) || !aligned(conics, 16))
    return fail(kInvalidArgument, "centers need 8-byte and conics 16-byte alignment");
  if (pairs == 0) return kOk;
  const BinLayout L = bin_layout(n, width, height, tile_mode);
  const PairLayout P = pair_layout(pairs, width, height, tile_mode);
  if (!workspace || workspace_bytes < L.bytes) return fail(kWorkspaceTooSmall, "bin workspace too small");
  if (P.bytes > 0 && (!pairs_workspace || pairs_workspace_bytes < P.bytes))
    return fail(kWorkspaceTooSmall, "pair workspace too small");
  if (!ids) return fail(kInvalidArgument, "null ids");
  if (!aligned(workspace, 256) || !aligned(pairs_workspace, 256))
    return fail(kInvalidArgument, "workspaces need 256-byte alignment");
  const int gx = (width + 15) / 16, gy = (height + 15) / 16;
  const int passes = tile_passes(gx * gy);
  cudaStream_t s = as_stream(stream);
  char* ws = static_cast<char*>(workspace);
  const ChunkPlan plan = chunk_plan(n, gx, gy, tile_mode);
  if (plan.use) {
    if (plan.smem_scatter > 48 * 1024)
      cudaFuncSetAttribute(tile_scatter_kernel, cudaFuncAttributeMaxDynamicSharedMemorySize,
                           static_cast<int>(plan.smem_scatter));
    tile_scatter_kernel<<<plan.chunks, 32 * kScatterWarps, plan.smem_scatter, counted(s)>>>(
        at<uint32_t>(ws, L.vals_a), at<uint32_t>(ws, L.chunk_bounds),
        at<uint2>(ws, L.sorted_rects), gx, gy, at<uint32_t>(ws, L.chunk_counts),
        at<uint32_t>(ws, L.tile_starts), static_cast<uint32_t>(pairs),
        at<uint32_t>(ws, L.totals) + 1, reinterpret_cast<uint32_t*>(ids));
    return check_launch("bin_emit");
  }
  char* pw = static_cast<char*>(pairs_workspace);
  if (cudaMemsetAsync(pw + P.status, 0, P.bytes - P.status, s) != cudaSuccess)
    return check_launch("bin_emit memset");
  const uint32_t m = static_cast<uint32_t>(pairs);
  const unsigned sort_tiles = blocks_for(pairs, kSortTile);
  uint32_t* status = at<uint32_t>(pw, P.status);
  uint32_t* counters = at<uint32_t>(pw, P.counters);
  const uint32_t* tile_digits = at<uint32_t>(ws, L.tile_digits);
  EmitLoader emit{at<uint32_t>(ws, L.offsets), at<uint32_t>(ws, L.vals_a), at<uint2>(ws, L.rects),
                  static_cast<uint32_t>(n), gx};
  uint32_t* k0 = at<uint32_t>(pw, P.keys0);
  uint32_t* v0 = at<uint32_t>(pw, P.vals0);
  uint32_t* k1 = at<uint32_t>(pw, P.keys1);
  uint32_t* v1 = at<uint32_t>(pw, P.vals1);
  uint32_t* out = reinterpret_cast<uint32_t*>(ids);
  if (tile_mode == kTileAccutile) {
    // pairs of the depth-ordered Gaussians at their depth-order offsets, then
    // stable passes over the tile id
    emit_strips_kernel<<<blocks_for(n, 256), 256, 0, counted(s)>>>(
        static_cast<uint32_t>(n), at<uint32_t>(ws, L.vals_a), at<uint32_t>(ws, L.offsets),
        centers, conics, radii, gx, gy, m, k0, v0);
    uint32_t* src_k = k0;
    uint32_t* src_v = v0;
    for (int pass = 0; pass < passes; ++pass) {
      const bool last = pass == passes - 1;
      KeyValueLoader ld{src_k, src_v};
      uint32_t* dst_k = (src_k == k0) ? k1 : k0;
      uint32_t* dst_v = last ? out : ((src_v == v0) ? v1 : v0);
      uint32_t* st = status + static_cast<size_t>(pass) * sort_tiles * kRadix;
      if (last)
        onesweep_kernel<KeyValueLoader, false><<<sort_tiles, kSortBlock, 0, counted(s)>>>(
            ld, m, 8 * pass, tile_digits + pass * kRadix, st, counters + pass, nullptr, dst_v);
      else
        onesweep_kernel<KeyValueLoader, true><<<sort_tiles, kSortBlock, 0, counted(s)>>>(
            ld, m, 8 * pass, tile_digits + pass * kRadix, st, counters + pass, dst_k, dst_v);
      src_k = dst_k;
      src_v = dst_v;
    }
    return check_launch("bin_emit");
  }
  if (passes == 1) {
    onesweep_kernel<EmitLoader, false><<<sort_tiles, kSortBlock, 0, counted(s)>>>(
        emit, m, 0, tile_digits, status, counters, nullptr, out);
  } else {
    onesweep_kernel<EmitLoader, true><<<sort_tiles, kSortBlock, 0, counted(s)>>>(
        emit, m, 0, tile_digits, status, counters, k0, v0);
    uint32_t* src_k = k0;
    uint32_t* src_v = v0;
    for (int pass = 1; pass < passes; ++pass) {
      const bool last = pass == passes - 1;
      KeyValueLoader ld{src_k, src_v};
      uint32_t* dst_k = (src_k == k0) ? k1 : k0;
      uint32_t* dst_v = last ? out : ((src_v == v0) ? v1 : v0);
      uint32_t* st = status + static_cast<size_t>(pass) * sort_tiles * kRadix;
      if (last)
        onesweep_kernel<KeyValueLoader, false><<<sort_tiles, kSortBlock, 0, counted(s)>>>(
            ld, m, 8 * pass, tile_digits + pass * kRadix, st, counters + pass, nullptr, dst_v);
      else
        onesweep_kernel<KeyValueLoader, true><<<sort_tiles, kSortBlock, 0, counted(s)>>>(
            ld, m, 8 * pass, tile_digits + pass * kRadix, st, counters + pass, dst_k, dst_v);
      src_k = dst_k;
      src_v = dst_v;
    }
  }
  return check_launch("bin_emit");
}

// ---- blending -----------------------------------------------------------------

int splat_tile_order(const int* ranges, int tiles, int* order, void* stream) {
  if (tiles < 0) return fail(kInvalidArgument, "bad tile count");
  if (tiles == 0) return kOk;
  if (!ranges || !order) return fail(kInvalidArgument, "null ranges or order");
  if (!aligned(ranges, 8)) return fail(kInvalidArgument, "ranges need 8-byte alignment");
  tile_order_kernel<<<1, 1024, 0, counted(as_stream(stream))>>>(ranges, tiles, order);
  return check_launch("tile_order");
}

int splat_render_forward_statistics(
    int width, int height, const int* ranges, const int* ids, long long num_ids, int n,
    const float* centers, const float* conics, const float* feat_a, int ch_a, int stride_a,
    const float* feat_b, int ch_b, int stride_b, int append_one, const float* background,
    float* image, int pix_stride, int ch_stride, float* alpha_image, float* final_t,
    int* contributors, int stat_count, int stat_sum_mask, const float* stat_pixels,
    int* stat_counts, float* stat_sums, const int* tile_order, void* stream) {
  if (width <= 0 || height <= 0 || ch_a < 0 || ch_b < 0 || (ch_b > 0 && !feat_b) || n < 0 ||
      num_ids < 0 || num_ids >= (1LL << 31))
    return fail(kInvalidArgument, "bad render sizes");
  if (stat_count < 0 || stat_count > 30 || (stat_count > 0 && !stat_pixels))
    return fail(kInvalidArgument, "bad statistics arguments");
  if (!aligned(centers, 8) || !aligned(conics, 16))
    return fail(kInvalidArgument, "centers need 8-byte and conics 16-byte alignment");
  RenderParams p{};
  p.width = width;
  p.height = height;
  p.gx = (width + 15) / 16;
  p.ranges = ranges;
  p.tile_order = tile_order;
  p.ids = ids;
  p.num_ids = static_cast<int>(num_ids);
  p.centers = centers;
  p.conics = conics;
  p.feat_a = feat_a;
  p.ch_a = ch_a;
  p.stride_a = stride_a;
  p.feat_b = feat_b;
  p.ch_b = ch_b;
  p.stride_b = stride_b;
  p.append_one = append_one ? 1 : 0;
  p.channels = ch_a + ch_b + p.append_one;
  p.background = background;
  if (alpha_image && !append_one)
    return fail(kInvalidArgument, "alpha_image holds the appended constant channel");
  p.image = image;
  p.pix_stride = pix_stride;
  p.ch_stride = ch_stride;
  p.alpha_image = alpha_image;
  p.final_t = final_t;
  p.contributors = contributors;
  p.stat_count = stat_count;
  p.stat_sum_mask = stat_sum_mask;
  p.n_gaussians = n;
  p.stat_pixels = stat_pixels;
  p.stat_counts = stat_counts;
  p.stat_sums = stat_sums;
  if (p.channels <= 0) return fail(kInvalidArgument, "no channels");
  return render_dispatch(p, false, as_stream(stream));
}

int splat_render_forward(int width, int height, const int* ranges, const int* ids,
                         long long num_ids, int n, const float* centers, const float* conics,
                         const float* feat_a, int ch_a, int stride_a, const float* feat_b,
                         int ch_b, int stride_b, int append_one, const float* background,
                         float* image, int pix_stride, int ch_stride, float* alpha_image,
                         float* final_t, int* contributors, const int* tile_order,
                         void* stream) {
  return splat_render_forward_statistics(width, height, ranges, ids, num_ids, n, centers, conics,
                                         feat_a, ch_a, stride_a, feat_b, ch_b, stride_b,
                                         append_one, background, image, pix_stride, ch_stride,
                                         alpha_image, final_t, contributors, 0, 0, nullptr,
                                         nullptr, nullptr, tile_order, stream);
}

int splat_render_backward(int width, int height, const int* ranges, const int* ids,
                          long long num_ids, int n, const float* centers, const float* conics,
                          const float* feat_a,
                          int ch_a, int stride_a, const float* feat_b, int ch_b, int stride_b,
                          int append_one, const float* background, const float* final_t,
                          const int* contributors, const float* upstream, int up_pix_stride,
                          int up_ch_stride, const float* upstream_alpha, int alpha_pix_stride,
                          float* grad_centers, float* grad_conics,
                          float* grad_a, float* grad_b, float* abs_centers, int constant_tail,
                          const int* tile_order, void* stream) {
  if (width <= 0 || height <= 0 || ch_a < 0 || ch_b < 0 || (ch_b > 0 && !feat_b) || n < 0 ||
      num_ids < 0 || num_ids >= (1LL << 31))
    return fail(kInvalidArgument, "bad render sizes");
  RenderParams p{};
  p.width = width;
  p.height = height;
  p.gx = (width + 15) / 16;
  p.ranges = ranges;
  p.tile_order = tile_order;
  p.ids = ids;
  p.num_ids = static_cast<int>(num_ids);
  p.n_gaussians = n;
  p.centers = centers;
  p.conics = conics;
  p.feat_a = feat_a;
  p.ch_a = ch_a;
  p.stride_a = stride_a;
  p.feat_b = feat_b;
  p.ch_b = ch_b;
  p.stride_b = stride_b;
  p.append_one = append_one ? 1 : 0;
  p.channels = ch_a + ch_b + p.append_one;
  p.background = background;
  p.final_t = const_cast<float*>(final_t);
  p.contributors = const_cast<int*>(contributors);
  if (upstream_alpha && !append_one)
    return fail(kInvalidArgument, "upstream_alpha belongs to the appended constant channel");
  p.upstream = upstream;
  p.up_pix_stride = up_pix_stride;
  p.up_ch_stride = up_ch_stride;
  p.upstream_alpha = upstream_alpha;
  p.alpha_pix_stride = alpha_pix_stride;
  p.grad_centers = grad_centers;
  p.grad_conics = grad_conics;
  p.grad_a = grad_a;
  p.grad_b = grad_b;
  p.abs_centers = abs_centers;
  p.constant_tail = constant_tail;
  if (p.channels <= 0 || constant_tail < 0 || constant_tail > p.channels)
    return fail(kInvalidArgument, "bad channel counts");
  if (!grad_centers || !grad_conics) return fail(kInvalidArgument, "null gradient buffers");
  if (!aligned(centers, 8) || !aligned(conics, 16) || !aligned(grad_centers, 8) ||
      !aligned(grad_conics, 16) || !aligned(abs_centers, 8))
    return fail(kInvalidArgument, "center rows need 8-byte and conic rows 16-byte alignment");
  return render_dispatch(p, true, as_stream(stream));
}

// ---- RaDe-GS ----------------------------------------------------------------

int splat_rade_project_forward(int n, const float* means, const float* quats,
                               int normalize_quats, const float* scales, const float* opacities,
                               const float* view, const float* proj, const float* K, int width,
                               int height, float near_plane, float far_plane, float radius_clip,
                               float kernel_size, float* centers, float* conics, int* radii,
                               int* tiles, float* depths, float* planes, float* normals,
                               int sh_degree, int sh_k, const float* sh, const float* campos,
                               float* colors, unsigned char* active, float* meta_means2d,
                               float* meta_opacities, float* meta_conics, void* stream) {
  if (n < 0 || width <= 0 || height <= 0) return fail(kInvalidArgument, "bad projection sizes");
  if (!(kernel_size >= 0.0f)) return fail(kInvalidArgument, "kernel_size must be nonnegative");
  if (sh && (sh_degree < 0 || sh_degree > 3 || sh_k < (sh_degree + 1) * (sh_degree + 1) ||
             !colors))
    return fail(kInvalidArgument, "bad SH arguments");
  if (meta_means2d && (!meta_opacities || !meta_conics))
    return fail(kInvalidArgument, "metadata outputs come together");
  if (n == 0) return kOk;
  if (!means || !quats || !scales || !opacities || !view || !proj || !K || !centers || !conics ||
      !radii || !tiles || !depths || !planes || !normals)
    return fail(kInvalidArgument, "null rade projection buffer");
  RadeProjectParams p{};
  p.n = n;
  p.means = means;
  p.quats = quats;
  p.normalize_quats = normalize_quats ? 1 : 0;
  p.scales = scales;
  p.opacities = opacities;
  p.view = view;
  p.proj = proj;
  p.K = K;
  p.width = width;
  p.height = height;
  p.near_plane = near_plane;
  p.far_plane = far_plane;
  p.radius_clip = radius_clip;
  p.kernel_size = kernel_size;
  p.centers = centers;
  p.conics = conics;
  p.radii = radii;
  p.tiles = tiles;
  p.depths = depths;
  p.planes = planes;
  p.normals = normals;
  p.sh_degree = sh_degree;
  p.sh_k = sh_k;
  p.sh = sh;
  p.campos = campos;
  p.colors = colors;
  p.active = active;
  p.meta_means2d = meta_means2d;
  p.meta_opacities = meta_opacities;
  p.meta_conics = meta_conics;
  cudaStream_t s = as_stream(stream);
  const unsigned blocks = blocks_for(n, 256);
  if (!sh) {
    rade_project_kernel<-1><<<blocks, 256, 0, counted(s)>>>(p);
  } else {
    switch (sh_degree) {
      case 0: rade_project_kernel<0><<<blocks, 256, 0, counted(s)>>>(p); break;
      case 1: rade_project_kernel<1><<<blocks, 256, 0, counted(s)>>>(p); break;
      case 2: rade_project_kernel<2><<<blocks, 256, 0, counted(s)>>>(p); break;
      default: rade_project_kernel<3><<<blocks, 256, 0, counted(s)>>>(p); break;
    }
  }
  return check_launch("rade_project_forward");
}

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
                                void* stream) {
  if (n < 0 || width <= 0 || height <= 0) return fail(kInvalidArgument, "bad projection sizes");
  if (sh && (sh_degree < 0 || sh_degree > 3 || sh_k < (sh_degree + 1) * (sh_degree + 1) ||
             !active || !grad_sh))
    return fail(kInvalidArgument, "bad SH backward arguments");
  if (n == 0) return kOk;
  if (!means || !quats || !scales || !opacities || !view || !proj || !K || !radii)
    return fail(kInvalidArgument, "null rade projection buffer");
  RadeProjectParams p{};
  p.n = n;
  p.means = means;
  p.quats = quats;
  p.normalize_quats = normalize_quats ? 1 : 0;
  p.scales = scales;
  p.opacities = opacities;
  p.view = view;
  p.proj = proj;
  p.K = K;
  p.width = width;
  p.height = height;
  p.kernel_size = kernel_size;
  p.radii = const_cast<int*>(radii);
  p.seed_centers = seed_centers;
  p.seed_conics = seed_conics;
  p.seed_planes = seed_planes;
  p.seed_normals = seed_normals;
  p.grad_means = grad_means;
  p.grad_quats = grad_quats;
  p.grad_scales = grad_scales;
  p.grad_opacities = grad_opacities;
  p.grad_view = grad_view;
  p.grad_proj = grad_proj;
  p.sh_degree = sh_degree;
  p.sh_k = sh_k;
  p.sh = sh;
  p.campos = campos;
  p.active = const_cast<unsigned char*>(active);
  p.seed_colors = seed_colors;
  p.grad_sh = grad_sh;
  p.grad_campos = grad_campos;
  return rade_project_backward_dispatch(p, as_stream(stream));
}

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
                              float* stat_sums, const int* tile_order, void* stream) {
  RadeRenderParams p;
  const int rc = rade_render_params(width, height, ranges, tile_order, ids, num_ids, n, centers,
                                    conics, planes, normals, colors, ch_a, stride_a, extras, ch_b,
                                    stride_b, background, K, p);
  if (rc != kOk) return rc;
  if (!features || !alpha || !depth || !median || !normal_image || !auxiliary || !contributors)
    return fail(kInvalidArgument, "null rade output");
  if (stat_count < 0 || stat_count > 30 || (stat_count > 0 && !stat_pixels))
    return fail(kInvalidArgument, "bad statistics arguments");
  p.features = features;
  p.feat_pix = feat_pix;
  p.feat_ch = feat_ch;
  p.alpha = alpha;
  p.alpha_pix = alpha_pix;
  p.depth = depth;
  p.depth_pix = depth_pix;
  p.median = median;
  p.median_pix = median_pix;
  p.normal_image = normal_image;
  p.normal_pix = normal_pix;
  p.normal_ch = normal_ch;
  p.auxiliary = auxiliary;
  p.contributors = contributors;
  p.base.stat_count = stat_count;
  p.base.stat_sum_mask = stat_sum_mask;
  p.base.stat_pixels = stat_pixels;
  p.base.stat_counts = stat_counts;
  p.base.stat_sums = stat_sums;
  return rade_render_dispatch(p, false, as_stream(stream));
}

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
    const int* tile_order, void* stream) {
  RadeRenderParams p;
  const int rc = rade_render_params(width, height, ranges, tile_order, ids, num_ids, n, centers,
                                    conics, planes, normals, colors, ch_a, stride_a, extras, ch_b,
                                    stride_b, background, K, p);
  if (rc != kOk) return rc;
  if (!alpha || !normal_image || !auxiliary || !contributors)
    return fail(kInvalidArgument, "null rade forward output");
  if (n > 0 && (!grad_centers || !grad_conics || !grad_planes || !grad_normals))
    return fail(kInvalidArgument, "null gradient buffers");
  if (!aligned(grad_centers, 8) || !aligned(grad_conics, 16) || !aligned(abs_centers, 8))
    return fail(kInvalidArgument, "center rows need 8-byte and conic rows 16-byte alignment");
  p.alpha = const_cast<float*>(alpha);
  p.alpha_pix = alpha_pix;
  p.normal_image = const_cast<float*>(normal_image);
  p.normal_pix = normal_pix;
  p.normal_ch = normal_ch;
  p.auxiliary = const_cast<float*>(auxiliary);
  p.contributors = const_cast<int*>(contributors);
  p.up_colors = up_colors;
  p.up_colors_pix = up_colors_pix;
  p.up_colors_ch = up_colors_ch;
  p.up_extras = up_extras;
  p.up_extras_pix = up_extras_pix;
  p.up_extras_ch = up_extras_ch;
  p.up_alpha = up_alpha;
  p.up_alpha_pix = up_alpha_pix;
  p.up_depth = up_depth;
  p.up_depth_pix = up_depth_pix;
  p.up_median = up_median;
  p.up_median_pix = up_median_pix;
  p.up_normals = up_normals;
  p.up_normals_pix = up_normals_pix;
  p.up_normals_ch = up_normals_ch;
  p.base.grad_centers = grad_centers;
  p.base.grad_conics = grad_conics;
  p.base.grad_a = grad_colors;
  p.base.grad_b = grad_extras;
  p.base.abs_centers = abs_centers;
  p.grad_planes = grad_planes;
  p.grad_normals = grad_normals;
  return rade_render_dispatch(p, true, as_stream(stream));
}

// ---- diagnostics --------------------------------------------------------------

}  // extern "C"

namespace {
__global__ void expf_probe_kernel(int n, const float* __restrict__ x, float* __restrict__ ours,
                                  float* __restrict__ cuda_exp) {
  const int i = blockIdx.x * blockDim.x + threadIdx.x;
  if (i >= n) return;
  ours[i] = splat_expf(x[i]);
  cuda_exp[i] = expf(x[i]);
}
}  // namespace

extern "C" int splat_debug_expf(int n, const float* x, float* ours, float* cuda_exp, void* stream) {
  if (n <= 0) return kOk;
  expf_probe_kernel<<<blocks_for(n, 256), 256, 0, counted(as_stream(stream))>>>(n, x, ours, cuda_exp);
  return check_launch("debug_expf");
}

// ---- AAA-Gaussians --------------------------------------------------------------
#include "aaa_api.cuh"
