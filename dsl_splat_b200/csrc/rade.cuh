// RaDe-GS tile-cooperative geometry blend (rade/render.py).
//
// Forward restates rade/render.py:106-227 (evaluate) in IEEE float32 (the
// -fmad=false translation unit): acceptance, early termination and the last
// and median contributor agree bit for bit with the CPU oracle; exp is the
// shared Cody-Waite splat_expf.  The backward (rade/render.py:336-545)
// replays each pixel from its last contributor like the gs3d backward,
// carrying one scalar S for every blended quantity (features, depth, normal)
// instead of per-channel colour sums, and reduces each sample's gradient
// values over the warp with butterfly16.
#pragma once
#include "rade_project.cuh"
#include "render.cuh"

namespace splat {

// ---- blend ------------------------------------------------------------------

struct RadeRenderParams {
  RenderParams base;      // bins, centres, conics, features (a = colours, b = extras),
                          // background, statistics; base.channels = C (no appended channel)
  const float* planes;    // (n,3)
  const float* normals;   // (n,3)
  const float* K;         // (3,3) intrinsics (device)
  // forward outputs, value of channel c at pixel p at base[p * pix + c * ch]:
  // features (C channels), alpha, expected depth, median depth, normals (3);
  // planar auxiliary (2,H,W) and contributors (2,H,W).  The backward reads
  // alpha, normals, auxiliary and contributors back.
  float* features;
  int feat_pix, feat_ch;
  float* alpha;
  int alpha_pix;
  float* depth;
  int depth_pix;
  float* median;
  int median_pix;
  float* normal_image;
  int normal_pix, normal_ch;
  float* auxiliary;
  int* contributors;
  // backward inputs: the forward's outputs and the upstream images
  // (channel-last (H,W,k) with the given pixel / channel strides; null = 0);
  // the colour channels [0, ch_a) and the extra channels [ch_a, C) each
  // from their own image
  const float* up_colors;
  int up_colors_pix, up_colors_ch;
  const float* up_extras;
  int up_extras_pix, up_extras_ch;
  const float* up_alpha;
  int up_alpha_pix;
  const float* up_depth;
  int up_depth_pix;
  const float* up_median;
  int up_median_pix;
  const float* up_normals;
  int up_normals_pix, up_normals_ch;
  // backward outputs (accumulated; grad_a / grad_b / abs may be null)
  float* grad_planes;     // (n,3)
  float* grad_normals;    // (n,3)
};

struct RadeShared {
  float4 plane[kBlock];
  float4 normal[kBlock];
};

SPLAT_DEV void stage_rade(const RadeRenderParams& p, RadeShared& r, int slot, int g) {
  if (static_cast<unsigned>(g) >= static_cast<unsigned>(p.base.n_gaussians)) {
    r.plane[slot] = make_float4(0.0f, 0.0f, 0.0f, 0.0f);
    r.normal[slot] = make_float4(0.0f, 0.0f, 0.0f, 0.0f);
    return;
  }
  const float* pl = p.planes + 3 * static_cast<size_t>(g);
  const float* nm = p.normals + 3 * static_cast<size_t>(g);
  r.plane[slot] = make_float4(pl[0], pl[1], pl[2], 0.0f);
  r.normal[slot] = make_float4(nm[0], nm[1], nm[2], 0.0f);
}

template <int CHP>
SPLAT_DEV RadeShared& rade_shared(float4* dynamic) {
  return *reinterpret_cast<RadeShared*>(reinterpret_cast<char*>(dynamic) + sizeof(RenderShared<CHP>));
}

// rade/render.py:209-211: 1 / |(u, v, 1)| of the pixel centre's ray.
SPLAT_DEV float ray_scale(const RadeRenderParams& p, int x, int y) {
  const float u = (static_cast<float>(x) + 0.5f - __ldg(p.K + 2)) / __ldg(p.K);
  const float v = (static_cast<float>(y) + 0.5f - __ldg(p.K + 5)) / __ldg(p.K + 4);
  return 1.0f / sqrtf(u * u + v * v + 1.0f);
}

// rade/render.py:106-227 evaluate: one thread per pixel (kBlock per tile).
template <int CHP>
__global__ void __launch_bounds__(kBlock) rade_forward_kernel(RadeRenderParams p) {
  extern __shared__ float4 s_dynamic[];
  RenderShared<CHP>& s = *reinterpret_cast<RenderShared<CHP>*>(s_dynamic);
  RadeShared& r = rade_shared<CHP>(s_dynamic);
  __shared__ uint8_t s_list[kBlock / 32][kBlock];
  uint8_t* list = s_list[threadIdx.x >> 5];
  const RenderParams& b = p.base;
  const int tile = block_tile(b);
  const PixelSlot<1> ps = pixel_slot<1>(tile, b.gx);
  const int x = ps.x, y = ps.y;
  const bool inside = x < b.width && y < b.height;
  const float fx = static_cast<float>(x), fy = static_cast<float>(y);
  const int first = max(b.ranges[2 * tile], 0);
  const int last = min(b.ranges[2 * tile + 1], b.num_ids);
  const float threshold = 1.0f / 255.0f;
  bool done = !inside;
  float T = 1.0f, depth = 0.0f, median = 0.0f;
  float3 normal = make_float3(0.0f, 0.0f, 0.0f);
  int median_contributor = -1, last_contributor = 0;
  float color[CHP];
#pragma unroll
  for (int c = 0; c < CHP; ++c) color[c] = 0.0f;
  for (int begin = first; begin < last; begin += kBlock) {
    if (__syncthreads_count(done) == kBlock) break;
    const int idx = begin + threadIdx.x;
    if (idx < last) {
      const int g = b.ids[idx];
      stage_gaussian<CHP>(b, s, threadIdx.x, g);
      stage_rade(p, r, threadIdx.x, g);
    }
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
      if (next_t < W32(0.0001)) {
        done = true;
        break;
      }
      const float w = alpha * T;
      float f[CHP];
      load_features(s, j, f);
#pragma unroll
      for (int c = 0; c < CHP; ++c) color[c] = __fmaf_rn(f[c], w, color[c]);
      const float4 pl = r.plane[j];
      const float distance = pl.x * dx + pl.y * dy + pl.z;
      depth += distance * w;
      const float4 nm = r.normal[j];
      normal.x += nm.x * w;
      normal.y += nm.y * w;
      normal.z += nm.z * w;
      const int position = begin - first + j + 1;
      if (b.stat_count) observe(b, s.id[j], y * b.width + x, w);
      if (T > 0.5f) {
        median = distance;
        median_contributor = position;
      }
      T = next_t;
      last_contributor = position;
    }
  }
  if (!inside) return;
  const size_t P = static_cast<size_t>(b.width) * b.height;
  const int pixel = y * b.width + x;
  float* feat = p.features + static_cast<size_t>(pixel) * p.feat_pix;
#pragma unroll
  for (int c = 0; c < CHP; ++c)
    if (c < b.channels) feat[c * p.feat_ch] = color[c] + T * b.background[c];
  const float rln = ray_scale(p, x, y);
  const float alpha = 1.0f - T;
  const float length = sqrtf(normal.x * normal.x + normal.y * normal.y + normal.z * normal.z);
  const float unit_scale = wmax(length, W32(1.0e-12));
  p.alpha[static_cast<size_t>(pixel) * p.alpha_pix] = alpha;
  p.depth[static_cast<size_t>(pixel) * p.depth_pix] =
      last_contributor > 0 ? depth * rln / alpha : 0.0f;
  p.median[static_cast<size_t>(pixel) * p.median_pix] = median * rln;
  float* nrm = p.normal_image + static_cast<size_t>(pixel) * p.normal_pix;
  nrm[0] = normal.x / unit_scale;
  nrm[p.normal_ch] = normal.y / unit_scale;
  nrm[2 * p.normal_ch] = normal.z / unit_scale;
  p.auxiliary[pixel] = depth * rln;
  p.auxiliary[P + pixel] = length;
  p.contributors[pixel] = last_contributor;
  p.contributors[P + pixel] = median_contributor;
}

// rade/render.py:106-227 evaluate with two pixels per lane (kBlock / 2
// threads per tile; warp w owns the 8x8 block, lane l the pixels (l % 8,
// l / 8) and (l % 8, l / 8 + 4)): the exponent, exp, alpha and
// transmittance of both pixels as f32x2 pairs (the bits of the scalar
// kernel), the colour channels as one packed fma per channel with the
// weight of a pixel that does not blend the sample set to zero, and the
// plane distance, depth, normal and median per pixel.
template <int CHP>
__global__ void __launch_bounds__(kBlock / 2) rade_forward2_kernel(RadeRenderParams p) {
  extern __shared__ float4 s_dynamic[];
  RenderShared<CHP>& s = *reinterpret_cast<RenderShared<CHP>*>(s_dynamic);
  RadeShared& r = rade_shared<CHP>(s_dynamic);
  __shared__ uint8_t s_list[kBlock / 64][kBlock];
  uint8_t* list = s_list[threadIdx.x >> 5];
  const RenderParams& b = p.base;
  const int tile = block_tile(b);
  const PixelSlot<2> ps = pixel_slot<2>(tile, b.gx);
  const int x = ps.x, y0 = ps.y, y1 = ps.y + 4;
  const bool inside0 = x < b.width && y0 < b.height;
  const bool inside1 = x < b.width && y1 < b.height;
  const float fx = static_cast<float>(x);
  const float fy0 = static_cast<float>(y0), fy1 = static_cast<float>(y1);
  const int first = max(b.ranges[2 * tile], 0);
  const int last = min(b.ranges[2 * tile + 1], b.num_ids);
  const float threshold = 1.0f / 255.0f;
  bool done0 = !inside0, done1 = !inside1;
  float T0 = 1.0f, T1 = 1.0f;
  f32x2 color2[CHP];
#pragma unroll
  for (int c = 0; c < CHP; ++c) color2[c] = splat2(0.0f);
  float depth0 = 0.0f, depth1 = 0.0f, median0 = 0.0f, median1 = 0.0f;
  float3 n0 = make_float3(0.0f, 0.0f, 0.0f), n1 = make_float3(0.0f, 0.0f, 0.0f);
  int last0 = 0, last1 = 0, mc0 = -1, mc1 = -1;
  for (int begin = first; begin < last; begin += kBlock) {
    if (__syncthreads_count(done0 && done1) == static_cast<int>(blockDim.x)) break;
    for (int slot = threadIdx.x; slot < kBlock; slot += blockDim.x) {
      const int idx = begin + slot;
      if (idx < last) {
        const int g = b.ids[idx];
        stage_gaussian<CHP>(b, s, slot, g);
        stage_rade(p, r, slot, g);
      }
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
      const float dy0 = gm.y - fy0, dy1 = gm.y - fy1;
      const f32x2 power = sample_power2(q, dx, dy0, dy1);
      float pw0, pw1;
      unpack2(power, pw0, pw1);
      const bool range0 = !done0 && pw0 <= 0.0f && pw0 >= cut;
      const bool range1 = !done1 && pw1 <= 0.0f && pw1 >= cut;
      if (!(range0 || range1)) continue;
      float a0, a1;
      unpack2(mul2(splat2(q.w), splat_expf_core2(power)), a0, a1);
      a0 = wmin(W32(0.99), a0);
      a1 = wmin(W32(0.99), a1);
      const bool accept0 = range0 && a0 >= threshold;
      const bool accept1 = range1 && a1 >= threshold;
      if (!(accept0 || accept1)) continue;
      const f32x2 alpha = pack2(a0, a1), t = pack2(T0, T1);
      float nt0, nt1, w0, w1;
      unpack2(mul2(t, sub2(splat2(1.0f), alpha)), nt0, nt1);  // T * (1 - alpha)
      unpack2(mul2(alpha, t), w0, w1);                        // alpha * T
      const bool blend0 = accept0 && nt0 >= W32(0.0001);
      const bool blend1 = accept1 && nt1 >= W32(0.0001);
      done0 = done0 || (accept0 && !blend0);
      done1 = done1 || (accept1 && !blend1);
      if (!(blend0 || blend1)) continue;
      float f[CHP];
      load_features(s, j, f);
      const f32x2 w2 = pack2(blend0 ? w0 : 0.0f, blend1 ? w1 : 0.0f);
#pragma unroll
      for (int c = 0; c < CHP; ++c) color2[c] = fma2(splat2(f[c]), w2, color2[c]);
      const float4 pl = r.plane[j];
      const float4 nm = r.normal[j];
      const int position = begin - first + j + 1;
      if (blend0) {
        const float distance = pl.x * dx + pl.y * dy0 + pl.z;
        depth0 += distance * w0;
        n0.x += nm.x * w0;
        n0.y += nm.y * w0;
        n0.z += nm.z * w0;
        if (b.stat_count) observe(b, s.id[j], y0 * b.width + x, w0);
        if (T0 > 0.5f) {
          median0 = distance;
          mc0 = position;
        }
        T0 = nt0;
        last0 = position;
      }
      if (blend1) {
        const float distance = pl.x * dx + pl.y * dy1 + pl.z;
        depth1 += distance * w1;
        n1.x += nm.x * w1;
        n1.y += nm.y * w1;
        n1.z += nm.z * w1;
        if (b.stat_count) observe(b, s.id[j], y1 * b.width + x, w1);
        if (T1 > 0.5f) {
          median1 = distance;
          mc1 = position;
        }
        T1 = nt1;
        last1 = position;
      }
    }
  }
  const size_t P = static_cast<size_t>(b.width) * b.height;
#pragma unroll
  for (int i = 0; i < 2; ++i) {
    if (!(i ? inside1 : inside0)) continue;
    const int y = i ? y1 : y0;
    const int pixel = y * b.width + x;
    const float T = i ? T1 : T0;
    float* feat = p.features + static_cast<size_t>(pixel) * p.feat_pix;
#pragma unroll
    for (int c = 0; c < CHP; ++c) {
      float c0, c1;
      unpack2(color2[c], c0, c1);
      if (c < b.channels) feat[c * p.feat_ch] = (i ? c1 : c0) + T * b.background[c];
    }
    const float3 normal = i ? n1 : n0;
    const float depth = i ? depth1 : depth0;
    const int last_contributor = i ? last1 : last0;
    const float rln = ray_scale(p, x, y);
    const float alpha = 1.0f - T;
    const float length = sqrtf(normal.x * normal.x + normal.y * normal.y + normal.z * normal.z);
    const float unit_scale = wmax(length, W32(1.0e-12));
    p.alpha[static_cast<size_t>(pixel) * p.alpha_pix] = alpha;
    p.depth[static_cast<size_t>(pixel) * p.depth_pix] =
        last_contributor > 0 ? depth * rln / alpha : 0.0f;
    p.median[static_cast<size_t>(pixel) * p.median_pix] = (i ? median1 : median0) * rln;
    float* nrm = p.normal_image + static_cast<size_t>(pixel) * p.normal_pix;
    nrm[0] = normal.x / unit_scale;
    nrm[p.normal_ch] = normal.y / unit_scale;
    nrm[2 * p.normal_ch] = normal.z / unit_scale;
    p.auxiliary[pixel] = depth * rln;
    p.auxiliary[P + pixel] = length;
    p.contributors[pixel] = last_contributor;
    p.contributors[P + pixel] = i ? mc1 : mc0;
  }
}

// Destination of reduction value k of the rade backward: 0-1 centre, 2-5
// conic (incl. opacity), 6-7 |centre|, 8-10 plane, 11-13 normal, 14+c
// feature channel c.
SPLAT_DEV GradientSlot rade_gradient_slot(const RadeRenderParams& p, int k) {
  if (k < 8) return gradient_slot(p.base, k, 0);
  if (k < 11) return {p.grad_planes + (k - 8), 3};
  if (k < 14) return {p.grad_normals + (k - 11), 3};
  const int c = k - 14;
  if (c >= p.base.channels) return {nullptr, 0};
  return gradient_slot(p.base, 8 + c, p.base.channels);
}

// rade/render.py:336-545 backward with PX pixels per lane (kBlock / PX
// threads per tile; warp w owns an 8 x 4*PX block, lane l the pixels
// (l % 8, l / 8 + 4 i)).  Per pixel the replay carries S = sum over the
// blended quantities of (their blend behind the sample) x (their upstream
// gradient): dL/dalpha of a sample is T (F - S) - T_final/(1-alpha)
// dL/dT_final with F the sample's own sum_c f_c g_c + d g_depth +
// n . g_normal, and S += alpha (F - S) after it.  A lane sums its pixels'
// gradient values before the warp reduction (with PX = 2 one butterfly
// covers 64 pixels), and 16 lanes then add the warp totals with one red
// each.  Measured at config 4 (36 channels), one pixel per lane is fastest:
// PX = 2 needs 187 registers (8 warps per SM); direct atomics from lanes of
// sparsely covered samples, or a shared-memory accumulator flushed once per
// batch, were both slower than the reduction they replace, and summing the
// two values past the third group with warp sums (instead of a fourth,
// mostly padded butterfly) did not change the time.  What does limit it is
// latency at 16 warps per SM: bounding registers for three blocks per SM (80
// registers, about 300 bytes of spills per thread, 24 warps) took config 4's
// backward from 4.47 to 4.18 ms.
template <int PX>
struct RadePixel {
  float fy, T, bg_term, depth_gradient, median_gradient, S, last_alpha, last_F;
  float3 normal_gradient;
  int last_contributor, median_contributor;
  bool inside;
};

template <int CHP, int PX>
__global__ void __launch_bounds__(kBlock / PX, 3) rade_backward_kernel(RadeRenderParams p) {
  constexpr int kThreads = kBlock / PX;
  constexpr int kValues = 14 + CHP;
  constexpr int kGroups = (kValues + 15) / 16;
  extern __shared__ float4 s_dynamic[];
  RenderShared<CHP>& s = *reinterpret_cast<RenderShared<CHP>*>(s_dynamic);
  RadeShared& r = rade_shared<CHP>(s_dynamic);
  __shared__ uint8_t s_list[kThreads / 32][kBlock];
  __shared__ int s_max_last;
  // destination of the value that lane l holds after the reduction of group
  // grp (the same for every warp); null for odd lanes and unused values
  __shared__ GradientSlot s_dst[kGroups][32];
  uint8_t* list = s_list[threadIdx.x >> 5];
  const RenderParams& b = p.base;
  const int tile = block_tile(b);
  const int wl = threadIdx.x & 31;
  const PixelSlot<PX> ps = pixel_slot<PX>(tile, b.gx);
  const int first = max(b.ranges[2 * tile], 0);
  const int last = min(b.ranges[2 * tile + 1], b.num_ids);
  const float threshold = 1.0f / 255.0f;
  const float fx = static_cast<float>(ps.x);
  const size_t P = static_cast<size_t>(b.width) * b.height;
  const int C = b.channels;
  float grad[PX][CHP];
  RadePixel<PX> px[PX];
  int lane_last = 0;
#pragma unroll
  for (int i = 0; i < PX; ++i) {
    RadePixel<PX>& q = px[i];
    const int y = ps.y + 4 * i;
    q.fy = static_cast<float>(y);
    q.inside = ps.x < b.width && y < b.height;
    q.T = q.bg_term = q.depth_gradient = q.median_gradient = 0.0f;
    q.S = q.last_alpha = q.last_F = 0.0f;
    q.normal_gradient = make_float3(0.0f, 0.0f, 0.0f);
    q.last_contributor = 0;
    q.median_contributor = -1;
#pragma unroll
    for (int c = 0; c < CHP; ++c) grad[i][c] = 0.0f;
    if (q.inside) {
      const int pixel = y * b.width + ps.x;
      const float pixel_alpha = p.alpha[static_cast<size_t>(pixel) * p.alpha_pix];
      const float final_T = 1.0f - pixel_alpha;
      q.T = final_T;
      q.last_contributor = p.contributors[pixel];
      q.median_contributor = p.contributors[P + pixel];
      float bg_grad = 0.0f;
      const float* uc = p.up_colors ? p.up_colors + static_cast<size_t>(pixel) * p.up_colors_pix
                                    : nullptr;
      const float* ue = p.up_extras ? p.up_extras + static_cast<size_t>(pixel) * p.up_extras_pix
                                    : nullptr;
#pragma unroll
      for (int c = 0; c < CHP; ++c)
        if (c < C) {
          float gval = 0.0f;
          if (c < b.ch_a) {
            if (uc) gval = __ldg(uc + c * p.up_colors_ch);
          } else if (ue) {
            gval = __ldg(ue + (c - b.ch_a) * p.up_extras_ch);
          }
          grad[i][c] = gval;
          bg_grad += b.background[c] * gval;
        }
      bg_grad -=
          p.up_alpha ? __ldg(p.up_alpha + static_cast<size_t>(pixel) * p.up_alpha_pix) : 0.0f;
      if (pixel_alpha > 0.0f) {
        const float rln = ray_scale(p, ps.x, y);
        const float gd =
            p.up_depth ? __ldg(p.up_depth + static_cast<size_t>(pixel) * p.up_depth_pix) : 0.0f;
        bg_grad += gd * (p.auxiliary[pixel] / pixel_alpha) / pixel_alpha;
        q.depth_gradient = gd / pixel_alpha * rln;
        q.median_gradient =
            (p.up_median ? __ldg(p.up_median + static_cast<size_t>(pixel) * p.up_median_pix)
                         : 0.0f) * rln;
        float3 ng = make_float3(0.0f, 0.0f, 0.0f);
        if (p.up_normals) {
          const float* un = p.up_normals + static_cast<size_t>(pixel) * p.up_normals_pix;
          ng = make_float3(__ldg(un), __ldg(un + p.up_normals_ch), __ldg(un + 2 * p.up_normals_ch));
        }
        const float* nrm = p.normal_image + static_cast<size_t>(pixel) * p.normal_pix;
        const float3 unit = make_float3(nrm[0], nrm[p.normal_ch], nrm[2 * p.normal_ch]);
        const float length = p.auxiliary[P + pixel];
        if (length >= W32(1.0e-12)) {
          const float d = dot3(unit, ng);
          ng.x -= unit.x * d;
          ng.y -= unit.y * d;
          ng.z -= unit.z * d;
        }
        const float sc = wmax(length, W32(1.0e-12));
        q.normal_gradient = make_float3(ng.x / sc, ng.y / sc, ng.z / sc);
      }
      q.bg_term = -final_T * bg_grad;
    }
    lane_last = max(lane_last, q.last_contributor);
  }
  if (threadIdx.x == 0) s_max_last = 0;
  for (int t = threadIdx.x; t < 32 * kGroups; t += kThreads) {
    const int grp = t >> 5, lane = t & 31;
    const int k = grp * 16 + butterfly_index(lane);
    GradientSlot d = k < kValues ? rade_gradient_slot(p, k) : GradientSlot{nullptr, 0};
    if (lane & 1) d.base = nullptr;
    s_dst[grp][lane] = d;
  }
  __syncthreads();
  const int warp_last = __reduce_max_sync(0xffffffffu, lane_last);
  if (wl == 0 && warp_last > 0) atomicMax(&s_max_last, warp_last);
  __syncthreads();
  const int stop = min(first + s_max_last, last);
  for (int end = stop; end > first; end -= kBlock) {
    __syncthreads();
    for (int slot = threadIdx.x; slot < kBlock; slot += kThreads) {
      const int idx = end - 1 - slot;
      if (idx >= first) {
        const int g = b.ids[idx];
        stage_gaussian<CHP>(b, s, slot, g);
        stage_rade(p, r, slot, g);
      }
    }
    __syncthreads();
    const int count = min(kBlock, end - first);
    const int candidates = warp_candidates(s, ps, max(0, end - first - warp_last), count, list);
    for (int k = 0; k < candidates; ++k) {
      const int j = list[k];
      const float4 gm = s.geom[j];
      const int position = end - 1 - j - first;  // contributor index - 1
      const float4 q = s.conic[j];
      const float dx = gm.x - fx;
      float dy[PX], G[PX], alpha[PX];
      bool accept[PX];
      bool any = false;
#pragma unroll
      for (int i = 0; i < PX; ++i) {
        dy[i] = gm.y - px[i].fy;
        const float power = sample_power(q, dx, dy[i]);
        const bool in_range = px[i].inside && position < px[i].last_contributor &&
                              power <= 0.0f && power >= s.cut[j];
        G[i] = splat_expf_core(power);
        alpha[i] = wmin(W32(0.99), q.w * G[i]);
        accept[i] = in_range && alpha[i] >= threshold;
        any = any || accept[i];
      }
      if (!__any_sync(0xffffffffu, any)) continue;
      float common[14];
#pragma unroll
      for (int v = 0; v < 14; ++v) common[v] = 0.0f;
      float weight[PX];
#pragma unroll
      for (int i = 0; i < PX; ++i) weight[i] = 0.0f;
      if (any) {
        float f[CHP];
        load_features(s, j, f);
        const float4 pl = r.plane[j];
        const float4 nm = r.normal[j];
#pragma unroll
        for (int i = 0; i < PX; ++i) {
          if (!accept[i]) continue;
          RadePixel<PX>& st = px[i];
          const float inv_one_minus = rcp_approx(1.0f - alpha[i]);
          st.T = st.T * inv_one_minus;
          const float distance = pl.x * dx + pl.y * dy[i] + pl.z;
          float F = distance * st.depth_gradient + nm.x * st.normal_gradient.x +
                    nm.y * st.normal_gradient.y + nm.z * st.normal_gradient.z;
#pragma unroll
          for (int c = 0; c < CHP; ++c) F = __fmaf_rn(f[c], grad[i][c], F);
          st.S = __fmaf_rn(st.last_alpha, st.last_F - st.S, st.S);
          st.last_F = F;
          st.last_alpha = alpha[i];
          const float w = alpha[i] * st.T;
          weight[i] = w;
          float g_distance = w * st.depth_gradient;
          if (position == st.median_contributor - 1) g_distance += st.median_gradient;
          const float grad_alpha = __fmaf_rn(F - st.S, st.T, st.bg_term * inv_one_minus);
          const float gv = q.w * grad_alpha;
          const float gdx = G[i] * dx, gdy = G[i] * dy[i];
          const float ddx = __fmaf_rn(g_distance, pl.x, -gv * __fmaf_rn(gdy, q.y, gdx * q.x));
          const float ddy = __fmaf_rn(g_distance, pl.y, -gv * __fmaf_rn(gdx, q.y, gdy * q.z));
          common[0] += ddx;
          common[1] += ddy;
          common[2] += -0.5f * gdx * dx * gv;
          common[3] += -gdx * dy[i] * gv;
          common[4] += -0.5f * gdy * dy[i] * gv;
          common[5] += G[i] * grad_alpha;
          common[6] += fabsf(ddx);
          common[7] += fabsf(ddy);
          common[8] += g_distance * dx;
          common[9] += g_distance * dy[i];
          common[10] += g_distance;
          common[11] += st.normal_gradient.x * w;
          common[12] += st.normal_gradient.y * w;
          common[13] += st.normal_gradient.z * w;
        }
      }
      const size_t g = static_cast<size_t>(s.id[j]);
#pragma unroll
      for (int grp = 0; grp < kGroups; ++grp) {
        float v16[16];
#pragma unroll
        for (int v = 0; v < 16; ++v) {
          const int idx = grp * 16 + v;
          if (idx < 14) {
            v16[v] = common[idx < 14 ? idx : 0];
          } else if (idx < kValues) {
            const int c = idx - 14 < CHP ? idx - 14 : 0;
            float acc = weight[0] * grad[0][c];
#pragma unroll
            for (int i = 1; i < PX; ++i) acc = __fmaf_rn(weight[i], grad[i][c], acc);
            v16[v] = acc;
          } else {
            v16[v] = 0.0f;
          }
        }
        const float total = butterfly16(v16, wl);
        const GradientSlot d = s_dst[grp][wl];
        if (d.base) red_add(d.base + g * d.stride, total);
      }
    }
  }
}

}  // namespace splat
