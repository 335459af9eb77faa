// Tile-cooperative front-to-back alpha blending and its reverse replay.
// Restates gs3d/render.py:41-125 (evaluate) and gs3d/render.py:221-354
// (backward).  One 256-thread CTA per 16x16 tile; each warp owns an 8x4
// block of pixels.  Batches of 256 Gaussians (id, centre, conic, opacity,
// cutoff and all feature channels) are staged in shared memory.  The
// per-pixel sample uses the same float32 operations as the CPU oracle, so
// acceptance decisions, final transmittance and contributor counts agree bit
// for bit; the colour sum uses one fma per channel with weight alpha*T.
//
// Two exact shortcuts keep the blend off samples that cannot contribute:
//  * power below a per-Gaussian cutoff (alpha < 0.951/255 there) skips exp;
//  * a warp skips a staged Gaussian whose cutoff ellipse misses the warp's
//    8x4 pixel centres (padded box test, then the exact ellipse-rectangle
//    test of footprint.cuh) -- one test per (warp, Gaussian), evaluated 32
//    Gaussians at a time, instead of 32 sample evaluations.
// Neither changes any decision: a skipped sample's alpha is below 1/255.
//
// Backward replays each pixel from its last contributor.  Per-sample
// gradients of a warp are summed with a butterfly (transpose) reduction --
// 16 values in 16 shuffles -- after which 16 lanes each hold one total and
// issue one red.global.add.f32 together.
#pragma once
#include "footprint.cuh"
#include "splat_common.cuh"

namespace splat {

struct RenderParams {
  int width, height, gx;
  const int* ranges;      // (T,2) [start, end) into ids
  const int* tile_order;  // (T) tile of block b (heaviest first), or null: block b = tile b
  const int* ids;         // sorted Gaussian ids
  int num_ids;            // length of ids (ranges are clamped to it)
  const float* centers;   // (n,2)
  const float* conics;    // (n,4) inv_a, inv_b, inv_c, opacity
  const float* feat_a;    // (n, stride_a), channels [0, ch_a)
  int ch_a, stride_a;
  const float* feat_b;    // (n, stride_b), channels [ch_a, ch_a + ch_b)
  int ch_b, stride_b;
  int append_one;         // implicit constant-1 channel after a and b
  int channels;           // ch_a + ch_b + append_one
  const float* background;  // (channels)
  // forward outputs
  float* image;           // image[pixel * pix_stride + c * ch_stride]
  int pix_stride, ch_stride;
  float* final_t;         // (H,W)
  int* contributors;      // (H,W)
  float* alpha_image;     // (H,W) or null: receives the appended constant channel
  // backward
  const float* upstream;  // upstream[pixel * up_pix_stride + c * up_ch_stride], or null (0)
  int up_pix_stride, up_ch_stride;
  const float* upstream_alpha;  // appended channel's upstream (pixel stride), or null: in upstream
  int alpha_pix_stride;
  float* grad_centers;    // (n,2) accumulated
  float* grad_conics;     // (n,4) accumulated
  float* grad_a;          // (n, ch_a) accumulated, or null
  float* grad_b;          // (n, ch_b) accumulated, or null
  float* abs_centers;     // (n,2) accumulated, or null
  int constant_tail;      // last channels without feature gradients
  // contribution statistics (statistics.py:47-73), forward only
  int stat_count;         // requests R (0 disables)
  int stat_sum_mask;      // bit r set: request r is a weighted sum, else a masked count
  int n_gaussians;        // number of Gaussians; row stride of stat_counts / stat_sums
  const float* stat_pixels;  // (R, H*W)
  int* stat_counts;       // (Rc, n)
  float* stat_sums;       // (Rs, n)
};

// statistics.py:57-73 observe: an accepted sample about to be blended with
// weight w = alpha*T adds 1 (masked count) or map*w (weighted sum) to its
// Gaussian wherever the pixel's map value is nonzero.
SPLAT_DEV void observe(const RenderParams& p, int g, int pixel, float w) {
  const size_t P = static_cast<size_t>(p.width) * p.height;
  int count_row = 0, sum_row = 0;
  for (int r = 0; r < p.stat_count; ++r) {
    const float v = p.stat_pixels[r * P + pixel];
    if ((p.stat_sum_mask >> r) & 1) {
      if (v != 0.0f) atomicAdd(p.stat_sums + static_cast<size_t>(sum_row) * p.n_gaussians + g, v * w);
      ++sum_row;
    } else {
      if (v != 0.0f) atomicAdd(p.stat_counts + static_cast<size_t>(count_row) * p.n_gaussians + g, 1);
      ++count_row;
    }
  }
}

template <int CHP>
struct RenderShared {
  int id[kBlock];
  float4 geom[kBlock];     // centre x, centre y, padded half extents of the cutoff ellipse
  float4 conic[kBlock];    // inv_a, inv_b, inv_c, opacity
  float cut[kBlock];       // power below which alpha < 1/255 for certain
  float4 bound[kBlock];    // EllipseBound ra, rc, level (w unused)
  float4 feat[kBlock][CHP / 4];  // channels of one slot, read with vector loads
};

// The tile this block blends: blocks run heaviest tile first when the
// caller passes tile_order (the order only changes which block finishes
// when; every block writes its own tile).
SPLAT_DEV int block_tile(const RenderParams& p) {
  return p.tile_order ? __ldg(p.tile_order + blockIdx.x) : static_cast<int>(blockIdx.x);
}

// Tiles by descending pair count (ranges), for RenderParams::tile_order: a
// counting sort of the counts scaled into 256 buckets (order inside a bucket
// is arbitrary).  One block of 1024 threads; each thread reads its tiles'
// counts once (kPer per round, all loads in flight together) and keeps them
// for the histogram and the placement.
__global__ void __launch_bounds__(1024)
    tile_order_kernel(const int* __restrict__ ranges, int T, int* __restrict__ order) {
  constexpr int kPer = 8;
  __shared__ int s_bucket[256];
  __shared__ int s_max;
  if (threadIdx.x == 0) s_max = 0;
  for (int b = threadIdx.x; b < 256; b += blockDim.x) s_bucket[b] = 0;
  __syncthreads();
  const int2* span = reinterpret_cast<const int2*>(ranges);
  int local = 0;
  for (int base = 0; base < T; base += kPer * 1024) {
    int count[kPer];
#pragma unroll
    for (int r = 0; r < kPer; ++r) {
      const int t = base + r * 1024 + threadIdx.x;
      const int2 v = t < T ? span[t] : make_int2(0, 0);
      count[r] = v.y - v.x;
    }
#pragma unroll
    for (int r = 0; r < kPer; ++r) local = max(local, count[r]);
  }
  local = __reduce_max_sync(0xffffffffu, local);
  if ((threadIdx.x & 31) == 0) atomicMax(&s_max, local);
  __syncthreads();
  const int shift = max(0, 32 - __clz(s_max) - 8);  // the largest count maps below 256
  for (int base = 0; base < T; base += kPer * 1024) {
    int count[kPer];
#pragma unroll
    for (int r = 0; r < kPer; ++r) {
      const int t = base + r * 1024 + threadIdx.x;
      const int2 v = t < T ? span[t] : make_int2(0, 0);
      count[r] = v.y - v.x;
    }
#pragma unroll
    for (int r = 0; r < kPer; ++r)
      if (base + r * 1024 + static_cast<int>(threadIdx.x) < T)
        atomicAdd(&s_bucket[255 - (count[r] >> shift)], 1);
  }
  __syncthreads();
  if (threadIdx.x < 32) {  // exclusive scan of the 256 buckets by one warp
    int v[8], sum = 0;
#pragma unroll
    for (int k = 0; k < 8; ++k) {
      v[k] = s_bucket[threadIdx.x * 8 + k];
      sum += v[k];
    }
    int incl = sum;
#pragma unroll
    for (int o = 1; o < 32; o <<= 1) {
      const int y = __shfl_up_sync(0xffffffffu, incl, o);
      if (threadIdx.x >= o) incl += y;
    }
    int run = incl - sum;
#pragma unroll
    for (int k = 0; k < 8; ++k) {
      s_bucket[threadIdx.x * 8 + k] = run;
      run += v[k];
    }
  }
  __syncthreads();
  for (int base = 0; base < T; base += kPer * 1024) {
    int count[kPer];
#pragma unroll
    for (int r = 0; r < kPer; ++r) {
      const int t = base + r * 1024 + threadIdx.x;
      const int2 v = t < T ? span[t] : make_int2(0, 0);
      count[r] = v.y - v.x;
    }
#pragma unroll
    for (int r = 0; r < kPer; ++r) {
      const int t = base + r * 1024 + threadIdx.x;
      if (t < T) order[atomicAdd(&s_bucket[255 - (count[r] >> shift)], 1)] = t;
    }
  }
}

// All CHP channels of staged slot j (padding channels are zero).
template <int CHP>
SPLAT_DEV void load_features(const RenderShared<CHP>& s, int j, float (&f)[CHP]) {
#pragma unroll
  for (int c4 = 0; c4 < CHP / 4; ++c4) {
    const float4 v = s.feat[j][c4];
    f[4 * c4] = v.x;
    f[4 * c4 + 1] = v.y;
    f[4 * c4 + 2] = v.z;
    f[4 * c4 + 3] = v.w;
  }
}

// Skipping samples with power < cut never changes a decision: alpha would
// be below 0.951/255 there (exp error < 1 ulp, log error < 1 ulp), and at
// power <= -80 splat_expf is 0 (alpha 0 or NaN, rejected either way).  So
// every evaluated sample has power in [cut, 0] with cut > -80, where
// splat_expf_core gives the same bits as splat_expf.
SPLAT_DEV float power_cutoff(float opacity) {
  if (!(opacity > 0.0f)) return 1.0f;  // alpha == 0: skip every sample
  return fmaxf(__logf(1.0f / (255.0f * opacity)) - 0.05f, -79.99999f);
}

// Half extents of {power >= cut} = {a dx^2 + 2 b dx dy + c dy^2 <= -2 cut},
// padded by one pixel (which absorbs the rounding of this estimate and of the
// per-sample power).  Negative: the Gaussian contributes nowhere.  Infinite:
// no bound (conic not positive definite), never skipped.
SPLAT_DEV float2 cutoff_extent(float4 q, float cut) {
  if (!(cut < 0.0f)) return make_float2(-1e30f, -1e30f);
  const float det = q.x * q.z - q.y * q.y;
  if (!(det > 0.0f) || !(q.x > 0.0f) || !(q.z > 0.0f)) return make_float2(INFINITY, INFINITY);
  const float level = -2.0f * cut;
  const float ex = sqrtf(level * q.z / det) + 1.0f;
  const float ey = sqrtf(level * q.x / det) + 1.0f;
  if (!(ex < INFINITY) || !(ey < INFINITY)) return make_float2(INFINITY, INFINITY);
  return make_float2(ex, ey);
}

template <int CHP>
SPLAT_DEV void stage_gaussian(const RenderParams& p, RenderShared<CHP>& s, int slot, int g) {
  if (static_cast<unsigned>(g) >= static_cast<unsigned>(p.n_gaussians)) {
    // an id outside [0, n) can only come from inconsistent inputs: stage an
    // invisible splat (skipped everywhere) instead of reading it
    s.id[slot] = 0;
    s.geom[slot] = make_float4(0.0f, 0.0f, -1e30f, -1e30f);
    s.conic[slot] = make_float4(0.0f, 0.0f, 0.0f, 0.0f);
    s.cut[slot] = 1.0f;
    s.bound[slot] = make_float4(0.0f, 0.0f, -1.0f, 0.0f);
#pragma unroll
    for (int c4 = 0; c4 < CHP / 4; ++c4) s.feat[slot][c4] = make_float4(0.0f, 0.0f, 0.0f, 0.0f);
    return;
  }
  s.id[slot] = g;
  const float2 xy = reinterpret_cast<const float2*>(p.centers)[g];
  const float4 q = reinterpret_cast<const float4*>(p.conics)[g];
  const float cut = power_cutoff(q.w);
  const float2 ext = cutoff_extent(q, cut);
  s.geom[slot] = make_float4(xy.x, xy.y, ext.x, ext.y);
  s.conic[slot] = q;
  s.cut[slot] = cut;
  const EllipseBound e = ellipse_bound(q.x, q.y, q.z, cut);
  s.bound[slot] = make_float4(e.ra, e.rc, e.level, 0.0f);
  const float* a = p.feat_a + static_cast<size_t>(g) * p.stride_a;
  float v[CHP];
#pragma unroll
  for (int c = 0; c < CHP; ++c) {
    v[c] = 0.0f;
    if (c < p.ch_a)
      v[c] = a[c];
    else if (c < p.ch_a + p.ch_b)
      v[c] = p.feat_b[static_cast<size_t>(g) * p.stride_b + (c - p.ch_a)];
    else if (c < p.channels)
      v[c] = 1.0f;
  }
#pragma unroll
  for (int c4 = 0; c4 < CHP / 4; ++c4)
    s.feat[slot][c4] = make_float4(v[4 * c4], v[4 * c4 + 1], v[4 * c4 + 2], v[4 * c4 + 3]);
}

// The reference's sample exponent, operation for operation (no contraction):
// power = -0.5*(a*dx*dx + c*dy*dy) - b*dx*dy  (gs3d/render.py:87-94).
SPLAT_DEV float sample_power(float4 q, float dx, float dy) {
  return (-0.5f * (q.x * dx * dx + q.z * dy * dy)) - q.y * dx * dy;
}

// Pixels of a lane: warp w owns the 8 x 4*PX block at ((w % 2) * 8,
// (w / 2) * 4 * PX) of the 16x16 tile, and lane l the PX pixels
// (l % 8, l / 8 + 4 i), i < PX.  The forward uses PX = 1 (eight warps per
// tile); the 4-channel backward PX = 2 (four warps, two pixels per lane).
template <int PX>
struct PixelSlot {
  int x, y;        // first pixel of the lane (the others are y + 4 i)
  float wcx, wcy;  // centre of the warp's block
  float wx0, wy0;  // its first pixel centre
};

template <int PX>
SPLAT_DEV PixelSlot<PX> pixel_slot(int tile, int gx) {
  const int t = threadIdx.x, warp = t >> 5, wl = t & 31;
  const int wx0 = (tile % gx) * kTile + (warp & 1) * 8;
  const int wy0 = (tile / gx) * kTile + (warp >> 1) * 4 * PX;
  PixelSlot<PX> s;
  s.x = wx0 + (wl & 7);
  s.y = wy0 + (wl >> 3);
  s.wcx = static_cast<float>(wx0) + 3.5f;
  s.wcy = static_cast<float>(wy0) + 0.5f * (4 * PX - 1);
  s.wx0 = static_cast<float>(wx0);
  s.wy0 = static_cast<float>(wy0);
  return s;
}

// True when staged slot j cannot reach any pixel of this warp: its padded
// cutoff box misses the warp's block, or (exact test) the minimum of its
// quadratic form over the block's pixel centres exceeds the cutoff level.
template <int CHP, int PX>
SPLAT_DEV bool misses_warp(const RenderShared<CHP>& s, int j, const PixelSlot<PX>& ps) {
  constexpr float kHalfH = 0.5f * (4 * PX - 1);
  const float4 geom = s.geom[j];
  if (fabsf(geom.x - ps.wcx) > geom.z + 3.5f || fabsf(geom.y - ps.wcy) > geom.w + kHalfH)
    return true;
  const float4 q = s.conic[j];
  const float4 b = s.bound[j];
  const EllipseBound e{b.x, b.y, b.z};
  const float u0 = ps.wx0 - geom.x, v0 = ps.wy0 - geom.y;
  return rectangle_min_form(q.x, q.y, q.z, e, u0, u0 + 7.0f, v0, v0 + 2.0f * kHalfH) > e.level;
}

// Ordered list of the staged slots in [j0, count) that can reach this warp's
// pixels, built with ballots (8 candidates per lane for a full batch).
// Returns its length; the list lives in `list` (per warp).
template <int CHP, int PX>
SPLAT_DEV int warp_candidates(const RenderShared<CHP>& s, const PixelSlot<PX>& ps, int j0,
                              int count, uint8_t* list) {
  const int wl = threadIdx.x & 31;
  const uint32_t lt = lanemask_lt();
  int n = 0;
  for (int base = j0; base < count; base += 32) {
    const int j = base + wl;
    const bool keep = j < count && !misses_warp(s, j, ps);
    const uint32_t b = __ballot_sync(0xffffffffu, keep);
    if (keep) list[n + __popc(b & lt)] = static_cast<uint8_t>(j);
    n += __popc(b);
  }
  __syncwarp();
  return n;
}

template <int CHP>
__global__ void __launch_bounds__(kBlock) render_forward_kernel(RenderParams p) {
  extern __shared__ float4 s_dynamic[];  // the staged batch (sizeof(RenderShared<CHP>) bytes)
  RenderShared<CHP>& s = *reinterpret_cast<RenderShared<CHP>*>(s_dynamic);
  __shared__ uint8_t s_list[kBlock / 32][kBlock];
  uint8_t* list = s_list[threadIdx.x >> 5];
  const int tile = block_tile(p);
  const PixelSlot<1> ps = pixel_slot<1>(tile, p.gx);
  const int x = ps.x, y = ps.y;
  const bool inside = x < p.width && y < p.height;
  const float fx = static_cast<float>(x), fy = static_cast<float>(y);
  const int first = max(p.ranges[2 * tile], 0);
  const int last = min(p.ranges[2 * tile + 1], p.num_ids);
  const float threshold = 1.0f / 255.0f;
  bool done = !inside;
  float T = 1.0f;
  float color[CHP];
#pragma unroll
  for (int c = 0; c < CHP; ++c) color[c] = 0.0f;
  int last_contributor = 0;
  for (int begin = first; begin < last; begin += kBlock) {
    if (__syncthreads_count(done) == kBlock) break;
    const int idx = begin + threadIdx.x;
    if (idx < last) stage_gaussian<CHP>(p, s, threadIdx.x, p.ids[idx]);
    __syncthreads();
    const int count = min(kBlock, last - begin);
    const int candidates = warp_candidates(s, ps, 0, count, list);
    for (int k = 0; k < candidates && !done; ++k) {
      const int j = list[k];
      const float4 q = s.conic[j];
      const float4 gm = s.geom[j];
      const float dx = gm.x - fx, dy = gm.y - fy;
      const float power = sample_power(q, dx, dy);
      if (power > 0.0f || power < s.cut[j]) continue;
      const float alpha = wmin(W32(0.99), q.w * splat_expf_core(power));
      if (!(alpha >= threshold)) continue;
      const float next_t = T * (1.0f - alpha);
      if (next_t < W32(0.0001)) {  // ends the pixel without being blended
        done = true;
        break;
      }
      const float w = alpha * T;
      float f[CHP];
      load_features(s, j, f);
      // padding channels are staged as zero: accumulating them is harmless
#pragma unroll
      for (int c = 0; c < CHP; ++c) color[c] = __fmaf_rn(f[c], w, color[c]);
      if (p.stat_count) observe(p, s.id[j], y * p.width + x, w);
      T = next_t;
      last_contributor = begin - first + j + 1;
    }
  }
  if (inside) {
    const int pixel = y * p.width + x;
    float* out = p.image + static_cast<size_t>(pixel) * p.pix_stride;
#pragma unroll
    for (int c = 0; c < CHP; ++c)
      if (c < p.channels) {
        const float v = color[c] + T * p.background[c];
        if (p.alpha_image && c == p.channels - 1)
          p.alpha_image[pixel] = v;
        else
          out[c * p.ch_stride] = v;
      }
    p.final_t[pixel] = T;
    p.contributors[pixel] = last_contributor;
  }
}

// The sample exponent of two pixels in one column (same dx), with
// sample_power's operation order: (-0.5*((a*dx)*dx + (c*dy)*dy)) - (b*dx)*dy.
// Scalar on purpose: ptxas contracts a packed multiply feeding a packed add
// into one fused multiply-add even under --fmad=false and .rn (measured on
// sm_100a), which would change these bits; the packed exp below has no
// multiply feeding an add outside its explicit fmas.
SPLAT_DEV f32x2 sample_power2(float4 q, float dx, float dy0, float dy1) {
  const float adx2 = (q.x * dx) * dx;
  const float bdx = q.y * dx;
  const float p0 = (-0.5f * (adx2 + (q.z * dy0) * dy0)) - bdx * dy0;
  const float p1 = (-0.5f * (adx2 + (q.z * dy1) * dy1)) - bdx * dy1;
  return pack2(p0, p1);
}

// Forward blend with two pixels per lane (kBlock / 2 threads per tile; warp
// w owns the 8x8 block, lane l the pixels (l % 8, l / 8) and (l % 8,
// l / 8 + 4)).  Per candidate the exponent, exp, alpha and transmittance of
// both pixels are computed as f32x2 pairs -- the same bits as the scalar
// kernel -- and each pixel then blends, ends or skips on its own.
template <int CHP, bool STATS>
__global__ void __launch_bounds__(kBlock / 2) render_forward2_kernel(RenderParams p) {
  extern __shared__ float4 s_dynamic[];  // the staged batch (sizeof(RenderShared<CHP>) bytes)
  RenderShared<CHP>& s = *reinterpret_cast<RenderShared<CHP>*>(s_dynamic);
  __shared__ uint8_t s_list[kBlock / 64][kBlock];
  uint8_t* list = s_list[threadIdx.x >> 5];
  const int tile = block_tile(p);
  const PixelSlot<2> ps = pixel_slot<2>(tile, p.gx);
  const int x = ps.x, y0 = ps.y, y1 = ps.y + 4;
  const bool inside0 = x < p.width && y0 < p.height;
  const bool inside1 = x < p.width && y1 < p.height;
  const float fx = static_cast<float>(x);
  const float fy0 = static_cast<float>(y0), fy1 = static_cast<float>(y1);
  const int first = max(p.ranges[2 * tile], 0);
  const int last = min(p.ranges[2 * tile + 1], p.num_ids);
  const float threshold = 1.0f / 255.0f;
  bool done0 = !inside0, done1 = !inside1;
  float T0 = 1.0f, T1 = 1.0f;
  // colour of both pixels as f32x2 pairs: a pixel that does not blend the
  // sample adds f * 0, which leaves its (never negative-zero) sum unchanged
  f32x2 color2[CHP];
#pragma unroll
  for (int c = 0; c < CHP; ++c) color2[c] = splat2(0.0f);
  int last0 = 0, last1 = 0;
  for (int begin = first; begin < last; begin += kBlock) {
    if (__syncthreads_count(done0 && done1) == static_cast<int>(blockDim.x)) break;
    for (int slot = threadIdx.x; slot < kBlock; slot += blockDim.x) {
      const int idx = begin + slot;
      if (idx < last) stage_gaussian<CHP>(p, s, slot, p.ids[idx]);
    }
    __syncthreads();
    const int count = min(kBlock, last - begin);
    const int candidates = warp_candidates(s, ps, 0, count, list);
    for (int k = 0; k < candidates && !(done0 && done1); ++k) {
      const int j = list[k];
      const float4 q = s.conic[j];
      const float4 gm = s.geom[j];
      const float cut = s.cut[j];
      const float dx = gm.x - fx;
      const f32x2 power = sample_power2(q, dx, gm.y - fy0, gm.y - fy1);
      float pw0, pw1;
      unpack2(power, pw0, pw1);
      const bool range0 = !done0 && pw0 <= 0.0f && pw0 >= cut;
      const bool range1 = !done1 && pw1 <= 0.0f && pw1 >= cut;
      if (!(range0 || range1)) continue;
      // a pixel out of range may hold any exponent here; its result is unused
      float a0, a1;
      unpack2(mul2(splat2(q.w), splat_expf_core2(power)), a0, a1);
      a0 = wmin(W32(0.99), a0);
      a1 = wmin(W32(0.99), a1);
      const bool accept0 = range0 && a0 >= threshold;
      const bool accept1 = range1 && a1 >= threshold;
      if (!(accept0 || accept1)) continue;
      const f32x2 alpha = pack2(a0, a1), t = pack2(T0, T1);
      float n0, n1, w0, w1;
      unpack2(mul2(t, sub2(splat2(1.0f), alpha)), n0, n1);  // T * (1 - alpha)
      unpack2(mul2(alpha, t), w0, w1);                      // alpha * T
      float f[CHP];
      load_features(s, j, f);
      const int position = begin - first + j + 1;
      // gs3d/render.py: a sample that would take T below 1e-4 ends the pixel
      // without being blended
      const bool blend0 = accept0 && n0 >= W32(0.0001);
      const bool blend1 = accept1 && n1 >= W32(0.0001);
      done0 = done0 || (accept0 && !blend0);
      done1 = done1 || (accept1 && !blend1);
      const f32x2 w2 = pack2(blend0 ? w0 : 0.0f, blend1 ? w1 : 0.0f);
#pragma unroll
      for (int c = 0; c < CHP; ++c) color2[c] = fma2(splat2(f[c]), w2, color2[c]);
      if (blend0) {
        if (STATS) observe(p, s.id[j], y0 * p.width + x, w0);
        T0 = n0;
        last0 = position;
      }
      if (blend1) {
        if (STATS) observe(p, s.id[j], y1 * p.width + x, w1);
        T1 = n1;
        last1 = position;
      }
    }
  }
  float color0[CHP], color1[CHP];
#pragma unroll
  for (int c = 0; c < CHP; ++c) unpack2(color2[c], color0[c], color1[c]);
#pragma unroll
  for (int i = 0; i < 2; ++i) {
    const bool inside = i ? inside1 : inside0;
    if (!inside) continue;
    const int pixel = (i ? y1 : y0) * p.width + x;
    const float T = i ? T1 : T0;
    float* out = p.image + static_cast<size_t>(pixel) * p.pix_stride;
#pragma unroll
    for (int c = 0; c < CHP; ++c)
      if (c < p.channels) {
        const float v = (i ? color1[c] : color0[c]) + T * p.background[c];
        if (p.alpha_image && c == p.channels - 1)
          p.alpha_image[pixel] = v;
        else
          out[c * p.ch_stride] = v;
      }
    p.final_t[pixel] = T;
    p.contributors[pixel] = i ? last1 : last0;
  }
}

// Butterfly (transpose) reduction of 16 values over the 32 lanes of a warp:
// 8 + 4 + 2 + 1 + 1 shuffles.  Returns, in every lane, the warp total of
// value butterfly_index(lane).
SPLAT_DEV float butterfly16(float (&v)[16], int lane) {
#pragma unroll
  for (int i = 0; i < 8; ++i) {
    const bool up = lane & 16;
    const float send = up ? v[i] : v[i + 8];
    const float keep = up ? v[i + 8] : v[i];
    v[i] = keep + __shfl_xor_sync(0xffffffffu, send, 16);
  }
#pragma unroll
  for (int i = 0; i < 4; ++i) {
    const bool up = lane & 8;
    const float send = up ? v[i] : v[i + 4];
    const float keep = up ? v[i + 4] : v[i];
    v[i] = keep + __shfl_xor_sync(0xffffffffu, send, 8);
  }
#pragma unroll
  for (int i = 0; i < 2; ++i) {
    const bool up = lane & 4;
    const float send = up ? v[i] : v[i + 2];
    const float keep = up ? v[i + 2] : v[i];
    v[i] = keep + __shfl_xor_sync(0xffffffffu, send, 4);
  }
  {
    const bool up = lane & 2;
    const float send = up ? v[0] : v[1];
    const float keep = up ? v[1] : v[0];
    v[0] = keep + __shfl_xor_sync(0xffffffffu, send, 2);
  }
  return v[0] + __shfl_xor_sync(0xffffffffu, v[0], 1);
}

SPLAT_DEV int butterfly_index(int lane) {
  return ((lane >> 4) & 1) * 8 + ((lane >> 3) & 1) * 4 + ((lane >> 2) & 1) * 2 + ((lane >> 1) & 1);
}

// The same reduction for 12 values (6 + 3 + 2 + 1 + 1 shuffles): pairs
// (i, i+6), then (i, i+3), then (i, i+2) with a zero fourth value, then
// (0, 1).  Returns in every lane the warp total of value
// butterfly12_index(lane); lanes whose index is 12 hold the padding.
SPLAT_DEV float butterfly12(float (&v)[12], int lane) {
#pragma unroll
  for (int i = 0; i < 6; ++i) {
    const bool up = lane & 16;
    const float send = up ? v[i] : v[i + 6];
    const float keep = up ? v[i + 6] : v[i];
    v[i] = keep + __shfl_xor_sync(0xffffffffu, send, 16);
  }
#pragma unroll
  for (int i = 0; i < 3; ++i) {
    const bool up = lane & 8;
    const float send = up ? v[i] : v[i + 3];
    const float keep = up ? v[i + 3] : v[i];
    v[i] = keep + __shfl_xor_sync(0xffffffffu, send, 8);
  }
  {
    const bool up = lane & 4;
    const float send0 = up ? v[0] : v[2];
    const float keep0 = up ? v[2] : v[0];
    const float send1 = up ? v[1] : 0.0f;
    const float keep1 = up ? 0.0f : v[1];
    v[0] = keep0 + __shfl_xor_sync(0xffffffffu, send0, 4);
    v[1] = keep1 + __shfl_xor_sync(0xffffffffu, send1, 4);
  }
  {
    const bool up = lane & 2;
    const float send = up ? v[0] : v[1];
    const float keep = up ? v[1] : v[0];
    v[0] = keep + __shfl_xor_sync(0xffffffffu, send, 2);
  }
  return v[0] + __shfl_xor_sync(0xffffffffu, v[0], 1);
}

SPLAT_DEV int butterfly12_index(int lane) {
  const int sub = ((lane >> 2) & 1) * 2 + ((lane >> 1) & 1);
  return sub == 3 ? 12 : ((lane >> 4) & 1) * 6 + ((lane >> 3) & 1) * 3 + sub;
}

// Destination row of gradient value k: 0-1 centre, 2-5 conic (incl.
// opacity), 6-7 |centre| sums, 8+c feature channel c.  The value of Gaussian
// g goes to base + g * stride; base is null where value k has no output.
struct GradientSlot {
  float* base;
  int stride;
};

SPLAT_DEV GradientSlot gradient_slot(const RenderParams& p, int k, int grad_channels) {
  if (k < 2) return {p.grad_centers + k, 2};
  if (k < 6) return {p.grad_conics + (k - 2), 4};
  if (k < 8) return {p.abs_centers ? p.abs_centers + (k - 6) : nullptr, 2};
  const int c = k - 8;
  if (c >= grad_channels) return {nullptr, 0};
  if (c < p.ch_a) return {p.grad_a ? p.grad_a + c : nullptr, p.ch_a};
  if (c < p.ch_a + p.ch_b) return {p.grad_b ? p.grad_b + (c - p.ch_a) : nullptr, p.ch_b};
  return {nullptr, 0};
}

// Reciprocal for the transmittance replay (relative error below 2^-22; the
// backward is compared by relative L2, not bit for bit).
SPLAT_DEV float rcp_approx(float x) {
  float r;
  asm("rcp.approx.ftz.f32 %0, %1;" : "=f"(r) : "f"(x));
  return r;
}

// Gradient contributions of one accepted sample of one pixel, added to
// val (0-1 centre, 2-5 conic incl. opacity, 6-7 |centre|, 8+c features).
// T is the transmittance behind the sample on entry and in front of it on
// return; acc the blended colour behind it, which takes the sample in.
template <int CHP, int NV>
SPLAT_DEV void accumulate_sample(float (&val)[NV], float4 q, const float (&f)[CHP], float G,
                                 float alpha, float dx, float dy, float& T, float bg_term,
                                 const float (&grad)[CHP], float (&acc)[CHP]) {
  const float inv_one_minus = rcp_approx(1.0f - alpha);
  T = T * inv_one_minus;
  // dL/dalpha = T * sum_c (colour_c - acc_c) dL/dC_c + bg_term / (1 - alpha),
  // then acc += alpha * (colour - acc)
  float grad_alpha = 0.0f;
#pragma unroll
  for (int c = 0; c < CHP; ++c) {
    const float d = f[c] - acc[c];
    grad_alpha = __fmaf_rn(d, grad[c], grad_alpha);
    acc[c] = __fmaf_rn(alpha, d, acc[c]);
  }
  const float w_feat = alpha * T;
#pragma unroll
  for (int c = 0; c < CHP && 8 + c < NV; ++c) val[8 + c] = __fmaf_rn(w_feat, grad[c], val[8 + c]);
  grad_alpha = __fmaf_rn(grad_alpha, T, bg_term * inv_one_minus);
  const float gv = q.w * grad_alpha;
  const float gdx = G * dx, gdy = G * dy;
  const float half_gv = -0.5f * gv;
  const float g0 = -gv * __fmaf_rn(gdy, q.y, gdx * q.x);
  const float g1 = -gv * __fmaf_rn(gdx, q.y, gdy * q.z);
  val[0] += g0;
  val[1] += g1;
  val[2] = __fmaf_rn(gdx * dx, half_gv, val[2]);
  val[3] = __fmaf_rn(-gdx * dy, gv, val[3]);
  val[4] = __fmaf_rn(gdy * dy, half_gv, val[4]);
  val[5] = __fmaf_rn(G, grad_alpha, val[5]);
  val[6] += fabsf(g0);
  val[7] += fabsf(g1);
}

// Reverse replay with PX pixels per lane (kBlock / PX threads per tile),
// launched with PX = 1 for views of more than four channels, which reduce
// groups of 16 values with butterfly16 (four-channel views use
// render_backward2_kernel).
template <int CHP, int PX>
__global__ void __launch_bounds__(kBlock / PX) render_backward_kernel(RenderParams p) {
  constexpr int kThreads = kBlock / PX;
  constexpr bool kTwelve = CHP == 4;
  constexpr int kGroups = kTwelve ? 1 : (8 + CHP + 15) / 16;
  constexpr int kSlots = kTwelve ? 12 : 16 * kGroups;
  extern __shared__ float4 s_dynamic[];  // the staged batch (sizeof(RenderShared<CHP>) bytes)
  RenderShared<CHP>& s = *reinterpret_cast<RenderShared<CHP>*>(s_dynamic);
  __shared__ uint8_t s_list[kThreads / 32][kBlock];
  __shared__ int s_max_last;
  // destination of the value that lane l holds after the reduction of group
  // grp (the same for every warp); null for odd lanes and unused values
  __shared__ GradientSlot s_dst[kGroups][32];
  uint8_t* list = s_list[threadIdx.x >> 5];
  const int tile = block_tile(p);
  const int wl = threadIdx.x & 31;
  const PixelSlot<PX> ps = pixel_slot<PX>(tile, p.gx);
  const int first = max(p.ranges[2 * tile], 0);
  const int last = min(p.ranges[2 * tile + 1], p.num_ids);
  const float threshold = 1.0f / 255.0f;
  const float fx = static_cast<float>(ps.x);
  // Per-pixel replay state: T is the transmittance in front of the current
  // sample, acc the blended colour of the accepted samples behind it, and
  // bg_term = -T_final * sum_c background_c * dL/dC_c.
  float fy[PX], T[PX], bg_term[PX];
  bool inside[PX];
  int last_contributor[PX];
  float grad[PX][CHP], acc[PX][CHP];
  int lane_last = 0;
#pragma unroll
  for (int i = 0; i < PX; ++i) {
    const int y = ps.y + 4 * i;
    fy[i] = static_cast<float>(y);
    inside[i] = ps.x < p.width && y < p.height;
    T[i] = 0.0f;
    bg_term[i] = 0.0f;
    last_contributor[i] = 0;
#pragma unroll
    for (int c = 0; c < CHP; ++c) {
      grad[i][c] = 0.0f;
      acc[i][c] = 0.0f;
    }
    if (inside[i]) {
      const int pixel = y * p.width + ps.x;
      const float final_T = p.final_t[pixel];
      T[i] = final_T;
      last_contributor[i] = p.contributors[pixel];
      const float* up = p.upstream ? p.upstream + static_cast<size_t>(pixel) * p.up_pix_stride
                                   : nullptr;
      float bg_grad = 0.0f;
#pragma unroll
      for (int c = 0; c < CHP; ++c)
        if (c < p.channels) {
          // the appended channel's upstream may live in its own buffer
          const float* src = (p.upstream_alpha && c == p.channels - 1)
                                 ? p.upstream_alpha + static_cast<size_t>(pixel) * p.alpha_pix_stride
                                 : (up ? up + c * p.up_ch_stride : nullptr);
          const float g = src ? __ldg(src) : 0.0f;
          grad[i][c] = g;
          bg_grad += p.background[c] * g;
        }
      bg_term[i] = -final_T * bg_grad;
    }
    lane_last = max(lane_last, last_contributor[i]);
  }
  if (threadIdx.x == 0) s_max_last = 0;
  if (threadIdx.x < 32 * kGroups) {
    // even lane l holds the warp total of value grp * 16 + butterfly_index(l)
    // (butterfly12_index(l) for 12 values); odd lanes write nothing
    const int grp = threadIdx.x >> 5;
    const int k = kTwelve ? butterfly12_index(wl) : grp * 16 + butterfly_index(wl);
    GradientSlot d = k < 8 + CHP ? gradient_slot(p, k, p.channels - p.constant_tail)
                                 : GradientSlot{nullptr, 0};
    if (wl & 1) d.base = nullptr;
    s_dst[grp][wl] = d;
  }
  __syncthreads();
  const int warp_last = __reduce_max_sync(0xffffffffu, lane_last);
  if (wl == 0 && warp_last > 0) atomicMax(&s_max_last, warp_last);
  __syncthreads();
  const int stop = min(first + s_max_last, last);  // later positions contribute nowhere
  for (int end = stop; end > first; end -= kBlock) {
    __syncthreads();
    for (int slot = threadIdx.x; slot < kBlock; slot += kThreads) {
      const int idx = end - 1 - slot;
      if (idx >= first) stage_gaussian<CHP>(p, s, slot, p.ids[idx]);
    }
    __syncthreads();
    const int count = min(kBlock, end - first);
    // only positions below warp_last (position = end - 1 - j - first) can
    // contribute to this warp's pixels
    const int candidates =
        warp_candidates(s, ps, max(0, end - first - warp_last), count, list);
    for (int k = 0; k < candidates; ++k) {
      const int j = list[k];
      const float4 gm = s.geom[j];
      const int position = end - 1 - j - first;  // contributor index - 1
      const float4 q = s.conic[j];
      const float cut = s.cut[j];
      const float dx = gm.x - fx;
      // evaluated by every lane; only in-range lanes use the result
      float dy[PX], G[PX], alpha[PX];
      bool accept[PX];
      bool any = false;
      {
#pragma unroll
        for (int i = 0; i < PX; ++i) {
          dy[i] = gm.y - fy[i];
          const float power = sample_power(q, dx, dy[i]);
          const bool in_range =
              inside[i] && position < last_contributor[i] && power <= 0.0f && power >= cut;
          G[i] = splat_expf_core(power);
          alpha[i] = wmin(W32(0.99), q.w * G[i]);
          accept[i] = in_range && alpha[i] >= threshold;
          any = any || accept[i];
        }
      }
      if (!__any_sync(0xffffffffu, any)) continue;
      float f[CHP];
      load_features(s, j, f);
      float val[kSlots];
#pragma unroll
      for (int v = 0; v < kSlots; ++v) val[v] = 0.0f;
#pragma unroll
      for (int i = 0; i < PX; ++i)
        if (accept[i])
          accumulate_sample(val, q, f, G[i], alpha[i], dx, dy[i], T[i], bg_term[i], grad[i],
                            acc[i]);
      const size_t g = static_cast<size_t>(s.id[j]);
      if constexpr (kTwelve) {
        const float total = butterfly12(val, wl);
        const GradientSlot d = s_dst[0][wl];
        if (d.base) red_add(d.base + g * d.stride, total);
      } else {
#pragma unroll
        for (int grp = 0; grp < kGroups; ++grp) {
          float v16[16];
#pragma unroll
          for (int v = 0; v < 16; ++v) v16[v] = val[grp * 16 + v];
          const float total = butterfly16(v16, wl);
          const GradientSlot d = s_dst[grp][wl];
          if (d.base) red_add(d.base + g * d.stride, total);
        }
      }
    }
  }
}

// Gradient contributions of one staged Gaussian to both pixels of a lane,
// as f32x2 pairs (low half: the lane's first pixel, high half: its second),
// summed over the two pixels into the 12 reduction values.  Per pixel the
// replay carries S = sum_c acc_c dL/dC_c instead of the blended colour acc
// behind the sample: dL/dalpha needs only sum_c (colour_c - acc_c) dL/dC_c
// = F - S with F = sum_c colour_c dL/dC_c, and acc += alpha (colour - acc)
// becomes S += alpha (F - S).  A pixel that does not take the sample enters
// with alpha = G = 0: rcp(1 - 0) = 1 and alpha (F - S) = 0 leave its T and
// S unchanged, and every contribution is an exact zero (all operands are
// finite).  feature_grads: channels whose gradient is written (the rest
// stay zero).
SPLAT_DEV void accumulate_pair(float (&val)[12], float4 q, const float (&f)[4], f32x2 G2,
                               f32x2 alpha2, float dx, f32x2 dy2, f32x2& T2, f32x2 bg2,
                               const f32x2 (&grad2)[4], f32x2& S2, int feature_grads) {
  float a0, a1;
  unpack2(alpha2, a0, a1);
  const f32x2 inv2 = pack2(rcp_approx(1.0f - a0), rcp_approx(1.0f - a1));
  T2 = mul2(T2, inv2);
  f32x2 F2 = mul2(splat2(f[0]), grad2[0]);
#pragma unroll
  for (int c = 1; c < 4; ++c) F2 = fma2(splat2(f[c]), grad2[c], F2);
  const f32x2 d2 = sub2(F2, S2);
  S2 = fma2(alpha2, d2, S2);
  const f32x2 w2 = mul2(alpha2, T2);
  float lo, hi;
#pragma unroll
  for (int c = 0; c < 4; ++c) {
    if (c < 3 || feature_grads > 3) {
      unpack2(mul2(w2, grad2[c]), lo, hi);
      val[8 + c] = lo + hi;
    } else {
      val[8 + c] = 0.0f;
    }
  }
  const f32x2 ga2 = fma2(d2, T2, mul2(bg2, inv2));    // dL/dalpha
  const f32x2 ngv2 = mul2(splat2(-q.w), ga2);         // -dL/dpower
  const f32x2 hgv2 = mul2(splat2(-0.5f * q.w), ga2);  // -0.5 dL/dpower
  const f32x2 gdx2 = mul2(G2, splat2(dx)), gdy2 = mul2(G2, dy2);
  const f32x2 g0 = mul2(ngv2, fma2(gdy2, splat2(q.y), mul2(gdx2, splat2(q.x))));
  const f32x2 g1 = mul2(ngv2, fma2(gdx2, splat2(q.y), mul2(gdy2, splat2(q.z))));
  float g0a, g0b, g1a, g1b;
  unpack2(g0, g0a, g0b);
  unpack2(g1, g1a, g1b);
  val[0] = g0a + g0b;
  val[1] = g1a + g1b;
  val[6] = fabsf(g0a) + fabsf(g0b);
  val[7] = fabsf(g1a) + fabsf(g1b);
  unpack2(mul2(mul2(gdx2, splat2(dx)), hgv2), lo, hi);
  val[2] = lo + hi;
  unpack2(mul2(mul2(gdx2, dy2), ngv2), lo, hi);
  val[3] = lo + hi;
  unpack2(mul2(mul2(gdy2, dy2), hgv2), lo, hi);
  val[4] = lo + hi;
  unpack2(mul2(G2, ga2), lo, hi);
  val[5] = lo + hi;
}

// Reverse replay for four channels with two pixels per lane, the per-pixel
// state and the gradient arithmetic held as f32x2 pairs (accumulate_pair).
// Acceptance decisions use the forward's exact sample exponent, so the
// replay visits the same samples the forward blended.
__global__ void __launch_bounds__(kBlock / 2) render_backward2_kernel(RenderParams p) {
  constexpr int CHP = 4;
  constexpr int kThreads = kBlock / 2;
  extern __shared__ float4 s_dynamic[];  // the staged batch (sizeof(RenderShared<4>) bytes)
  RenderShared<CHP>& s = *reinterpret_cast<RenderShared<CHP>*>(s_dynamic);
  __shared__ uint8_t s_list[kThreads / 32][kBlock];
  __shared__ int s_max_last;
  // destination of the value that lane l holds after butterfly12 (the same
  // for every warp); null for odd lanes and unused values
  __shared__ GradientSlot s_dst[32];
  uint8_t* list = s_list[threadIdx.x >> 5];
  const int tile = block_tile(p);
  const int wl = threadIdx.x & 31;
  const PixelSlot<2> ps = pixel_slot<2>(tile, p.gx);
  const int first = max(p.ranges[2 * tile], 0);
  const int last = min(p.ranges[2 * tile + 1], p.num_ids);
  const float threshold = 1.0f / 255.0f;
  const float fx = static_cast<float>(ps.x);
  // per pixel: T in front of the current sample, S = sum_c acc_c dL/dC_c
  // over the blended colour acc of the accepted samples behind it, and
  // bg = -T_final * sum_c background_c dL/dC_c
  float fy[2], T[2], bg[2], grad[2][CHP];
  int last_contributor[2];
#pragma unroll
  for (int i = 0; i < 2; ++i) {
    const int y = ps.y + 4 * i;
    fy[i] = static_cast<float>(y);
    T[i] = 0.0f;
    bg[i] = 0.0f;
    last_contributor[i] = 0;  // 0 outside the image: no position passes
#pragma unroll
    for (int c = 0; c < CHP; ++c) grad[i][c] = 0.0f;
    if (ps.x < p.width && y < p.height) {
      const int pixel = y * p.width + ps.x;
      const float final_T = p.final_t[pixel];
      T[i] = final_T;
      last_contributor[i] = p.contributors[pixel];
      const float* up = p.upstream ? p.upstream + static_cast<size_t>(pixel) * p.up_pix_stride
                                   : nullptr;
      float bg_grad = 0.0f;
#pragma unroll
      for (int c = 0; c < CHP; ++c)
        if (c < p.channels) {
          // the appended channel's upstream may live in its own buffer
          const float* src = (p.upstream_alpha && c == p.channels - 1)
                                 ? p.upstream_alpha + static_cast<size_t>(pixel) * p.alpha_pix_stride
                                 : (up ? up + c * p.up_ch_stride : nullptr);
          const float g = src ? __ldg(src) : 0.0f;
          grad[i][c] = g;
          bg_grad += p.background[c] * g;
        }
      bg[i] = -final_T * bg_grad;
    }
  }
  f32x2 T2 = pack2(T[0], T[1]), bg2 = pack2(bg[0], bg[1]), S2 = splat2(0.0f);
  f32x2 grad2[CHP];
#pragma unroll
  for (int c = 0; c < CHP; ++c) grad2[c] = pack2(grad[0][c], grad[1][c]);
  const int feature_grads = p.channels - p.constant_tail;
  const int lane_last = max(last_contributor[0], last_contributor[1]);
  if (threadIdx.x == 0) s_max_last = 0;
  if (threadIdx.x < 32) {
    GradientSlot d = gradient_slot(p, butterfly12_index(wl), p.channels - p.constant_tail);
    if ((wl & 1) || butterfly12_index(wl) >= 8 + CHP) d.base = nullptr;
    s_dst[wl] = d;
  }
  __syncthreads();
  const int warp_last = __reduce_max_sync(0xffffffffu, lane_last);
  if (wl == 0 && warp_last > 0) atomicMax(&s_max_last, warp_last);
  __syncthreads();
  const int stop = min(first + s_max_last, last);  // later positions contribute nowhere
  for (int end = stop; end > first; end -= kBlock) {
    __syncthreads();
    for (int slot = threadIdx.x; slot < kBlock; slot += kThreads) {
      const int idx = end - 1 - slot;
      if (idx >= first) stage_gaussian<CHP>(p, s, slot, p.ids[idx]);
    }
    __syncthreads();
    const int count = min(kBlock, end - first);
    // only positions below warp_last (position = end - 1 - j - first) can
    // contribute to this warp's pixels
    const int candidates =
        warp_candidates(s, ps, max(0, end - first - warp_last), count, list);
    for (int k = 0; k < candidates; ++k) {
      const int j = list[k];
      const float4 gm = s.geom[j];
      const int position = end - 1 - j - first;  // contributor index - 1
      const float4 q = s.conic[j];
      const float cut = s.cut[j];
      const float dx = gm.x - fx;
      const float dy0 = gm.y - fy[0], dy1 = gm.y - fy[1];
      const float pw0 = sample_power(q, dx, dy0), pw1 = sample_power(q, dx, dy1);
      const f32x2 e2 = splat_expf_core2(pack2(pw0, pw1));
      float g0, g1, a0, a1;
      unpack2(e2, g0, g1);
      unpack2(mul2(splat2(q.w), e2), a0, a1);
      a0 = wmin(W32(0.99), a0);
      a1 = wmin(W32(0.99), a1);
      const bool acc0 = position < last_contributor[0] && pw0 <= 0.0f && pw0 >= cut &&
                        a0 >= threshold;
      const bool acc1 = position < last_contributor[1] && pw1 <= 0.0f && pw1 >= cut &&
                        a1 >= threshold;
      if (!__any_sync(0xffffffffu, acc0 || acc1)) continue;
      float f[CHP];
      load_features(s, j, f);
      float val[12];
      accumulate_pair(val, q, f, pack2(acc0 ? g0 : 0.0f, acc1 ? g1 : 0.0f),
                      pack2(acc0 ? a0 : 0.0f, acc1 ? a1 : 0.0f), dx, pack2(dy0, dy1), T2, bg2,
                      grad2, S2, feature_grads);
      const float total = butterfly12(val, wl);
      const GradientSlot d = s_dst[wl];
      if (d.base) red_add(d.base + static_cast<size_t>(s.id[j]) * d.stride, total);
    }
  }
}

}  // namespace splat
