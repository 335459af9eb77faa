// Tile-cooperative front-to-back alpha blending and its reverse replay.
// Restates gs3d/render.py:41-125 (evaluate) and gs3d/render.py:221-354
// (backward).  One 256-thread CTA per 16x16 tile; batches of 256 Gaussians
// (id, centre, conic, opacity and all feature channels) are staged in shared
// memory; the per-pixel sample uses the same float32 operations as the CPU
// oracle, so acceptance decisions, final transmittance and contributor
// counts agree bit for bit.  The colour sum uses one fma per channel with
// the premultiplied weight alpha*T.
//
// Backward replays each pixel from its last contributor; per-sample
// gradients are summed across the warp with shuffles and one lane issues
// vector reductions (red.global.add.v2/v4.f32) into the per-Gaussian
// gradient rows.
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
  int n_gaussians;        // row stride of stat_counts / stat_sums
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
  float2 xy[kBlock];
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

template <int CHP>
SPLAT_DEV void stage_gaussian(const RenderParams& p, RenderShared<CHP>& s, int slot, int g) {
  if (static_cast<unsigned>(g) >= static_cast<unsigned>(p.n_gaussians)) {
    // an id outside [0, n) can only come from inconsistent inputs: stage an
    // invisible splat (cut = +1 skips every sample) instead of reading it
    s.id[slot] = 0;
    s.xy[slot] = make_float2(0.0f, 0.0f);
    s.conic[slot] = make_float4(0.0f, 0.0f, 0.0f, 0.0f);
    s.cut[slot] = 1.0f;
#pragma unroll
    for (int c = 0; c < CHP; ++c) s.feat[c][slot] = 0.0f;
    return;
  }
  s.id[slot] = g;
  s.xy[slot] = reinterpret_cast<const float2*>(p.centers)[g];
  const float4 q = reinterpret_cast<const float4*>(p.conics)[g];
  s.conic[slot] = q;
  s.cut[slot] = power_cutoff(q.w);
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

template <int CHP>
__global__ void __launch_bounds__(kBlock) render_forward_kernel(RenderParams p) {
  __shared__ RenderShared<CHP> s;
  const int tile = blockIdx.x;
  const int lane = threadIdx.x;
  const int x = tile % p.gx * kTile + lane % kTile;
  const int y = tile / p.gx * kTile + lane / kTile;
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
    const int idx = begin + lane;
    if (idx < last) stage_gaussian<CHP>(p, s, lane, p.ids[idx]);
    __syncthreads();
    const int count = min(kBlock, last - begin);
    for (int j = 0; j < count && !done; ++j) {
      const float4 q = s.conic[j];
      const float2 c2 = s.xy[j];
      const float dx = c2.x - fx, dy = c2.y - fy;
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

template <int CHP>
__global__ void __launch_bounds__(kBlock) render_backward_kernel(RenderParams p) {
  __shared__ RenderShared<CHP> s;
  __shared__ int s_max_last;
  const int tile = blockIdx.x;
  const int lane = threadIdx.x;
  const int wl = lane & 31;
  const int x = tile % p.gx * kTile + lane % kTile;
  const int y = tile / p.gx * kTile + lane / kTile;
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
  if (lane == 0) s_max_last = 0;
  __syncthreads();
  if (last_contributor > 0) atomicMax(&s_max_last, last_contributor);
  __syncthreads();
  const int stop = min(first + s_max_last, last);  // later positions contribute nowhere
  const int grad_channels = p.channels - p.constant_tail;
  for (int end = stop; end > first; end -= kBlock) {
    __syncthreads();
    const int idx = end - 1 - lane;
    if (idx >= first) stage_gaussian<CHP>(p, s, lane, p.ids[idx]);
    __syncthreads();
    const int count = min(kBlock, end - first);
    for (int j = 0; j < count; ++j) {
      const int position = end - 1 - j - first;  // contributor index - 1
      bool accept = false;
      float gx_c = 0.0f, gy_c = 0.0f, q0 = 0.0f, q1 = 0.0f, q2 = 0.0f, q3 = 0.0f;
      float ax = 0.0f, ay = 0.0f, w_feat = 0.0f;
      if (inside && position < last_contributor) {
        const float4 q = s.conic[j];
        const float2 c2 = s.xy[j];
        const float dx = c2.x - fx, dy = c2.y - fy;
        const float power = sample_power(q, dx, dy);
        if (power <= 0.0f && power >= s.cut[j]) {
          const float G = splat_expf(power);
          const float alpha = wmin(W32(0.99), q.w * G);
          if (alpha >= threshold) {
            accept = true;
            T = T / (1.0f - alpha);
            float grad_alpha = 0.0f;
#pragma unroll
            for (int c = 0; c < CHP; ++c)
              if (c < p.channels) {
                const float col = s.feat[c][j];
                acc[c] = last_alpha * last_color[c] + (1.0f - last_alpha) * acc[c];
                last_color[c] = col;
                grad_alpha += (col - acc[c]) * grad[c];
              }
            w_feat = alpha * T;
            grad_alpha = grad_alpha * T + (-final_T / (1.0f - alpha)) * bg_grad;
            last_alpha = alpha;
            const float gv = q.w * grad_alpha;
            const float gdx = G * dx, gdy = G * dy;
            gx_c = gv * (-gdx * q.x - gdy * q.y);
            gy_c = gv * (-gdy * q.z - gdx * q.y);
            q0 = -0.5f * gdx * dx * gv;
            q1 = -gdx * dy * gv;
            q2 = -0.5f * gdy * dy * gv;
            q3 = G * grad_alpha;
            ax = fabsf(gx_c);
            ay = fabsf(gy_c);
          }
        }
      }
      if (!__any_sync(0xffffffffu, accept)) continue;
      const int g = s.id[j];
      gx_c = warp_sum(gx_c);
      gy_c = warp_sum(gy_c);
      q0 = warp_sum(q0);
      q1 = warp_sum(q1);
      q2 = warp_sum(q2);
      q3 = warp_sum(q3);
      if (p.abs_centers) {
        ax = warp_sum(ax);
        ay = warp_sum(ay);
      }
      if (wl == 0) {
        red_add_v2(p.grad_centers + 2 * static_cast<size_t>(g), gx_c, gy_c);
        red_add_v4(p.grad_conics + 4 * static_cast<size_t>(g), q0, q1, q2, q3);
        if (p.abs_centers) red_add_v2(p.abs_centers + 2 * static_cast<size_t>(g), ax, ay);
      }
#pragma unroll
      for (int c = 0; c < CHP; ++c) {
        if (c < grad_channels) {
          const float v = warp_sum(w_feat * grad[c]);
          if (wl == 0) {
            if (c < p.ch_a) {
              if (p.grad_a) red_add(p.grad_a + static_cast<size_t>(g) * p.ch_a + c, v);
            } else if (c < p.ch_a + p.ch_b) {
              if (p.grad_b) red_add(p.grad_b + static_cast<size_t>(g) * p.ch_b + (c - p.ch_a), v);
            }
          }
        }
      }
    }
  }
}

}  // namespace splat
