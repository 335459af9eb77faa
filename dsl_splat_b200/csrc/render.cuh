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
//  * a warp skips a staged Gaussian whose cutoff ellipse, padded by one
//    pixel, misses the warp's 8x4 pixels -- one uniform test per warp
//    instead of 32 sample evaluations.
// Neither changes any decision: a skipped sample's alpha is below 1/255.
//
// Backward replays each pixel from its last contributor.  Per-sample
// gradients of a warp are summed with a butterfly (transpose) reduction --
// 16 values in 16 shuffles -- after which 16 lanes each hold one total and
// issue one red.global.add.f32 together.
#pragma once
#include "splat_common.cuh"

namespace splat {

struct RenderParams {
  int width, height, gx;
  const int* ranges;      // (T,2) [start, end) into ids
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
  // backward
  const float* upstream;  // upstream[pixel * up_pix_stride + c * up_ch_stride]
  int up_pix_stride, up_ch_stride;
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
  float feat[CHP][kBlock];
};

// Skipping samples with power < cut never changes a decision: alpha would
// be below 0.951/255 there (exp error < 1 ulp, log error < 1 ulp).
SPLAT_DEV float power_cutoff(float opacity) {
  if (!(opacity > 0.0f)) return 1.0f;  // alpha == 0: skip every sample
  return __logf(1.0f / (255.0f * opacity)) - 0.05f;
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
#pragma unroll
    for (int c = 0; c < CHP; ++c) s.feat[c][slot] = 0.0f;
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
  const float* a = p.feat_a + static_cast<size_t>(g) * p.stride_a;
#pragma unroll
  for (int c = 0; c < CHP; ++c) {
    float v = 0.0f;
    if (c < p.ch_a)
      v = a[c];
    else if (c < p.ch_a + p.ch_b)
      v = p.feat_b[static_cast<size_t>(g) * p.stride_b + (c - p.ch_a)];
    else if (c < p.channels)
      v = 1.0f;
    s.feat[c][slot] = v;
  }
}

// The reference's sample exponent, operation for operation (no contraction):
// power = -0.5*(a*dx*dx + c*dy*dy) - b*dx*dy  (gs3d/render.py:87-94).
SPLAT_DEV float sample_power(float4 q, float dx, float dy) {
  return (-0.5f * (q.x * dx * dx + q.z * dy * dy)) - q.y * dx * dy;
}

// Pixel of thread t in tile `tile`: warp w covers the 8x4 block at
// ((w % 2) * 8, (w / 2) * 4) of the 16x16 tile.
struct PixelSlot {
  int x, y;
  float wcx, wcy;  // centre of the warp's 8x4 block
};

SPLAT_DEV PixelSlot pixel_slot(int tile, int gx) {
  const int t = threadIdx.x, warp = t >> 5, wl = t & 31;
  const int wx0 = (tile % gx) * kTile + (warp & 1) * 8;
  const int wy0 = (tile / gx) * kTile + (warp >> 1) * 4;
  PixelSlot s;
  s.x = wx0 + (wl & 7);
  s.y = wy0 + (wl >> 3);
  s.wcx = static_cast<float>(wx0) + 3.5f;
  s.wcy = static_cast<float>(wy0) + 1.5f;
  return s;
}

// True when the staged Gaussian cannot reach any pixel of this warp.
SPLAT_DEV bool misses_warp(float4 geom, const PixelSlot& ps) {
  return fabsf(geom.x - ps.wcx) > geom.z + 3.5f || fabsf(geom.y - ps.wcy) > geom.w + 1.5f;
}

// Ordered list of the staged slots in [j0, count) that can reach this warp's
// pixels, built with ballots (8 candidates per lane for a full batch).
// Returns its length; the list lives in `list` (per warp).
template <int CHP>
SPLAT_DEV int warp_candidates(const RenderShared<CHP>& s, const PixelSlot& ps, int j0, int count,
                              uint8_t* list) {
  const int wl = threadIdx.x & 31;
  const uint32_t lt = lanemask_lt();
  int n = 0;
  for (int base = j0; base < count; base += 32) {
    const int j = base + wl;
    const bool keep = j < count && !misses_warp(s.geom[j], ps);
    const uint32_t b = __ballot_sync(0xffffffffu, keep);
    if (keep) list[n + __popc(b & lt)] = static_cast<uint8_t>(j);
    n += __popc(b);
  }
  __syncwarp();
  return n;
}

template <int CHP>
__global__ void __launch_bounds__(kBlock) render_forward_kernel(RenderParams p) {
  __shared__ RenderShared<CHP> s;
  __shared__ uint8_t s_list[kBlock / 32][kBlock];
  uint8_t* list = s_list[threadIdx.x >> 5];
  const int tile = blockIdx.x;
  const PixelSlot ps = pixel_slot(tile, p.gx);
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
      const float alpha = wmin(W32(0.99), q.w * splat_expf(power));
      if (!(alpha >= threshold)) continue;
      const float next_t = T * (1.0f - alpha);
      if (next_t < W32(0.0001)) {
        done = true;
        break;
      }
      const float w = alpha * T;
#pragma unroll
      for (int c = 0; c < CHP; ++c)
        if (c < p.channels) color[c] = __fmaf_rn(s.feat[c][j], w, color[c]);
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
      if (c < p.channels) out[c * p.ch_stride] = color[c] + T * p.background[c];
    p.final_t[pixel] = T;
    p.contributors[pixel] = last_contributor;
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

// Destination of gradient value k of Gaussian g: 0-1 centre, 2-5 conic
// (incl. opacity), 6-7 |centre| sums, 8+c feature channel c.
SPLAT_DEV float* gradient_slot(const RenderParams& p, int g, int k, int grad_channels) {
  if (k < 2) return p.grad_centers + 2 * static_cast<size_t>(g) + k;
  if (k < 6) return p.grad_conics + 4 * static_cast<size_t>(g) + (k - 2);
  if (k < 8) return p.abs_centers ? p.abs_centers + 2 * static_cast<size_t>(g) + (k - 6) : nullptr;
  const int c = k - 8;
  if (c >= grad_channels) return nullptr;
  if (c < p.ch_a) return p.grad_a ? p.grad_a + static_cast<size_t>(g) * p.ch_a + c : nullptr;
  if (c < p.ch_a + p.ch_b)
    return p.grad_b ? p.grad_b + static_cast<size_t>(g) * p.ch_b + (c - p.ch_a) : nullptr;
  return nullptr;
}

template <int CHP>
__global__ void __launch_bounds__(kBlock) render_backward_kernel(RenderParams p) {
  constexpr int kValues = 8 + CHP;
  constexpr int kGroups = (kValues + 15) / 16;
  __shared__ RenderShared<CHP> s;
  __shared__ uint8_t s_list[kBlock / 32][kBlock];
  __shared__ int s_max_last;
  uint8_t* list = s_list[threadIdx.x >> 5];
  const int tile = blockIdx.x;
  const int wl = threadIdx.x & 31;
  const PixelSlot ps = pixel_slot(tile, p.gx);
  const int x = ps.x, y = ps.y;
  const bool inside = x < p.width && y < p.height;
  const float fx = static_cast<float>(x), fy = static_cast<float>(y);
  const int first = max(p.ranges[2 * tile], 0);
  const int last = min(p.ranges[2 * tile + 1], p.num_ids);
  const float threshold = 1.0f / 255.0f;
  const int pixel = y * p.width + x;
  float T = 0.0f, final_T = 0.0f, bg_grad = 0.0f, last_alpha = 0.0f;
  int last_contributor = 0;
  float grad[CHP], acc[CHP], last_color[CHP];
#pragma unroll
  for (int c = 0; c < CHP; ++c) {
    grad[c] = 0.0f;
    acc[c] = 0.0f;
    last_color[c] = 0.0f;
  }
  if (inside) {
    final_T = p.final_t[pixel];
    T = final_T;
    last_contributor = p.contributors[pixel];
    const float* up = p.upstream + static_cast<size_t>(pixel) * p.up_pix_stride;
#pragma unroll
    for (int c = 0; c < CHP; ++c)
      if (c < p.channels) {
        grad[c] = up[c * p.up_ch_stride];
        bg_grad += p.background[c] * grad[c];
      }
  }
  if (threadIdx.x == 0) s_max_last = 0;
  __syncthreads();
  const int warp_last = __reduce_max_sync(0xffffffffu, last_contributor);
  if (wl == 0 && warp_last > 0) atomicMax(&s_max_last, warp_last);
  __syncthreads();
  const int stop = min(first + s_max_last, last);  // later positions contribute nowhere
  const int grad_channels = p.channels - p.constant_tail;
  for (int end = stop; end > first; end -= kBlock) {
    __syncthreads();
    const int idx = end - 1 - static_cast<int>(threadIdx.x);
    if (idx >= first) stage_gaussian<CHP>(p, s, threadIdx.x, p.ids[idx]);
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
      const float dx = gm.x - fx, dy = gm.y - fy;
      bool accept = false;
      float G = 0.0f, alpha = 0.0f;
      if (inside && position < last_contributor) {
        const float power = sample_power(q, dx, dy);
        if (power <= 0.0f && power >= s.cut[j]) {
          G = splat_expf(power);
          alpha = wmin(W32(0.99), q.w * G);
          accept = alpha >= threshold;
        }
      }
      if (!__any_sync(0xffffffffu, accept)) continue;
      float val[kGroups * 16];
#pragma unroll
      for (int v = 0; v < kGroups * 16; ++v) val[v] = 0.0f;
      if (accept) {
        const float inv_one_minus = __frcp_rn(1.0f - alpha);
        T = T * inv_one_minus;
        float grad_alpha = 0.0f;
#pragma unroll
        for (int c = 0; c < CHP; ++c)
          if (c < p.channels) {
            const float col = s.feat[c][j];
            acc[c] = last_alpha * last_color[c] + (1.0f - last_alpha) * acc[c];
            last_color[c] = col;
            grad_alpha += (col - acc[c]) * grad[c];
          }
        const float w_feat = alpha * T;
#pragma unroll
        for (int c = 0; c < CHP; ++c) val[8 + c] = c < grad_channels ? w_feat * grad[c] : 0.0f;
        grad_alpha = grad_alpha * T + (-final_T * inv_one_minus) * bg_grad;
        last_alpha = alpha;
        const float gv = q.w * grad_alpha;
        const float gdx = G * dx, gdy = G * dy;
        val[0] = gv * (-gdx * q.x - gdy * q.y);
        val[1] = gv * (-gdy * q.z - gdx * q.y);
        val[2] = -0.5f * gdx * dx * gv;
        val[3] = -gdx * dy * gv;
        val[4] = -0.5f * gdy * dy * gv;
        val[5] = G * grad_alpha;
        val[6] = fabsf(val[0]);
        val[7] = fabsf(val[1]);
      }
      const int g = s.id[j];
      const int k_lane = butterfly_index(wl);
#pragma unroll
      for (int grp = 0; grp < kGroups; ++grp) {
        float v16[16];
#pragma unroll
        for (int k = 0; k < 16; ++k) v16[k] = val[grp * 16 + k];
        const float total = butterfly16(v16, wl);
        if ((wl & 1) == 0) {
          float* dst = gradient_slot(p, g, grp * 16 + k_lane, grad_channels);
          if (dst) red_add(dst, total);
        }
      }
    }
  }
}

}  // namespace splat
