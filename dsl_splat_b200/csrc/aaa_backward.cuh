// The record backward of the AAA blend (K27 from the forward's blend
// records): aaa/backward_render.py:140-248 with aaa/render_adjoint.py:279-352,
// for every tile whose pixels all kept their records.
//
// Compiled in its own translation unit (aaa_backward.cu) with multiply-add
// contraction and the approximate divide: its outputs are gradients,
// compared within a relative tolerance.
#pragma once
#include "aaa_blend_params.cuh"

namespace splat {
namespace aaa {

// ---- backward from the forward's blend records ---------------------------------
// One block per tile, one thread per pixel, three passes over the tile's
// records:
//  1. a histogram of the recorded tile-slice positions;
//  2. per pixel, its samples in blend order with the replay's arithmetic
//     (alpha = min(0.99, opacity * gaussian) as at insertion; T and the
//     accumulated colour by the same products), which leaves per sample
//     s = gaussian * dL/dalpha and the blend weight alpha * T -- written over
//     the record -- and files the sample under its position;
//  3. per position (one Gaussian), a warp sums the gradient terms of the
//     position's samples over the tile's pixels and adds each sum to global
//     memory once.  A Gaussian that blends in a tile does so in ~100 of its
//     256 pixels at 1080p, so this issues ~1/100 of the global reductions of
//     one reduction per sample.
// Tiles with a pixel past the record capacity are left to the replay kernel;
// a tile whose positions or sample count exceed the shared-memory lists
// takes the per-sample path (direct reductions), as does every sample it
// holds.
// accumulator row: transform rows 0-2 (d0, d1, d3) and the translation row
// (t0, t1, t3), opacity, screen x / y, |screen| x / y, four colours
constexpr int kAccTransform = 0, kAccOpacity = 12, kAccScreen = 13, kAccAbs = 15,
              kAccColor = 17, kAccStride = 21;
constexpr int kTilePositions = 1024;  // positions filed per tile
constexpr int kTileSamples = 24576;   // samples filed per tile (16-bit entries: j << 8 | pixel)
constexpr int kTileCache = 512;       // positions whose id, opacity and colours are staged

struct TileShared {
  float4 rgb[kTileCache];           // colours (four-channel features)
  float4 pixel_grad[256];           // dL/dcolour per pixel (four-channel features)
  float opacity[kTileCache];
  int ids[kTileCache];
  int offsets[kTilePositions + 1];  // exclusive prefix sums of the histogram
  int cursor[kTilePositions];       // the histogram, then the filing cursors
  int warp_sums[8];
  int max_pos, fallback;
  unsigned short list[kTileSamples];  // filed samples, grouped by position
};

// the transform rows a sample's gradient needs (row 2, the screen depth,
// does not enter it), the opacity and up to four colours
struct SampleData {
  float4 r0, r1, r3, rgb;
  float opacity;
};

SPLAT_DEV SampleData load_sample(const HierParams& p, int id) {
  SampleData d;
  const float4* rows = reinterpret_cast<const float4*>(p.transforms) + 4ll * id;
  d.r0 = rows[0];
  d.r1 = rows[1];
  d.r3 = rows[3];
  d.opacity = p.opacity[id];
  d.rgb = p.channels == 4 ? reinterpret_cast<const float4*>(p.colors)[id]
                          : make_float4(0.0f, 0.0f, 0.0f, 0.0f);
  return d;
}

// render_adjoint.py:285-351 for one sample: the transform and screen terms of
// an accumulator row; factor = opacity * dL/dalpha * gaussian
template <bool SCREEN, bool ABS>
SPLAT_DEV void ray_terms(float4 r0, float4 r1, float4 r3, float x, float y, float factor,
                         float out[kAccStride]) {
  const float g0[4] = {r0.x, r0.y, r0.z, r0.w};
  const float g1[4] = {r1.x, r1.y, r1.z, r1.w};
  const float g3[4] = {r3.x, r3.y, r3.z, r3.w};
  float a[4], b[4];
#pragma unroll
  for (int k = 0; k < 4; ++k) {
    a[k] = g0[k] - g3[k] * x;
    b[k] = g1[k] - g3[k] * y;
  }
  const float nx[3] = {a[0], a[1], a[2]}, ny[3] = {b[0], b[1], b[2]};
  const float dx = a[3], dy = b[3];
  float moment[3], direction[3];
#pragma unroll
  for (int k = 0; k < 3; ++k) moment[k] = dx * ny[k] - dy * nx[k];
  direction[0] = nx[1] * ny[2] - nx[2] * ny[1];
  direction[1] = nx[2] * ny[0] - nx[0] * ny[2];
  direction[2] = nx[0] * ny[1] - nx[1] * ny[0];
  const float dd = rdot3(direction, direction), mm = rdot3(moment, moment);
  const float xx = rdot3(nx, nx), yy = rdot3(ny, ny), xy = rdot3(nx, ny);
  const float ym = rdot3(ny, moment), xm = rdot3(nx, moment);
  const float xyy = x * yy, yxx = y * xx, ndy = -dy, cross = dy * x - dx * y;
  const float inverse_dd = 1.0f / dd;
  const float ratio = mm * inverse_dd * inverse_dd;
  float screen_x = 0.0f, screen_y = 0.0f;
#pragma unroll
  for (int axis = 0; axis < 3; ++axis) {
    const float dd0 = yy * nx[axis] - xy * ny[axis];
    const float dd1 = xx * ny[axis] - xy * nx[axis];
    const float dd3 = (xy * (y * nx[axis] + x * ny[axis]) - xyy * nx[axis]) - yxx * ny[axis];
    const float d0 = factor * (ratio * dd0 - (ndy * moment[axis]) * inverse_dd);
    const float d1 = factor * (ratio * dd1 - (dx * moment[axis]) * inverse_dd);
    const float d3 = factor * (ratio * dd3 - (cross * moment[axis]) * inverse_dd);
    screen_x += d0 * g3[axis];
    screen_y += d1 * g3[axis];
    out[kAccTransform + 3 * axis] = d0;
    out[kAccTransform + 3 * axis + 1] = d1;
    out[kAccTransform + 3 * axis + 2] = d3;
  }
  const float tr0 = factor * -ym * inverse_dd;
  const float tr1 = factor * xm * inverse_dd;
  out[kAccTransform + 9] = tr0;
  out[kAccTransform + 10] = tr1;
  out[kAccTransform + 11] = factor * -(y * xm - x * ym) * inverse_dd;
  screen_x += tr0 * g3[3];
  screen_y += tr1 * g3[3];
  out[kAccScreen] = screen_x;
  out[kAccScreen + 1] = screen_y;
  out[kAccAbs] = fabsf(screen_x);
  out[kAccAbs + 1] = fabsf(screen_y);
}

// one sample's terms into the global gradients (the per-sample path)
template <bool SCREEN, bool ABS, bool COLORS4>
SPLAT_DEV void flush_row(const HierParams& p, int id, const float* v) {
  float* t = p.grad_transforms + 16ll * id;
#pragma unroll
  for (int axis = 0; axis < 4; ++axis)
    red_add_v4(t + 4 * axis, v[kAccTransform + 3 * axis], v[kAccTransform + 3 * axis + 1], 0.0f,
               v[kAccTransform + 3 * axis + 2]);
  red_add(p.grad_opacity + id, v[kAccOpacity]);
  if (SCREEN) red_add_v2(p.grad_screen + 2ll * id, v[kAccScreen], v[kAccScreen + 1]);
  if (ABS) red_add_v2(p.grad_screen_abs + 2ll * id, v[kAccAbs], v[kAccAbs + 1]);
  if (COLORS4)
    red_add_v4(p.grad_colors + 4ll * id, v[kAccColor], v[kAccColor + 1], v[kAccColor + 2],
               v[kAccColor + 3]);
}

// The warp's sum of 32 per-lane rows, transposed: lane c returns the sum of
// component c (halving exchanges: 16 + 8 + 4 + 2 + 1 shuffles).
SPLAT_DEV float warp_row_sum(float (&v)[32], int lane) {
#pragma unroll
  for (int width = 16; width >= 1; width >>= 1) {
    const bool upper = lane & width;
#pragma unroll
    for (int k = 0; k < width; ++k) {
      const float send = upper ? v[k] : v[k + width];
      const float keep = upper ? v[k + width] : v[k];
      v[k] = keep + __shfl_xor_sync(kFull, send, width);
    }
  }
  return v[0];
}

// global address of accumulator component c of Gaussian id, or null when the
// component is not produced
template <bool SCREEN, bool ABS, bool COLORS4>
SPLAT_DEV float* component_address(const HierParams& p, int id, int c) {
  if (c < kAccOpacity) {
    const int axis = c / 3, k = c - 3 * axis;
    return p.grad_transforms + 16ll * id + 4 * axis + (k == 2 ? 3 : k);
  }
  if (c == kAccOpacity) return p.grad_opacity + id;
  if (c < kAccAbs) return SCREEN ? p.grad_screen + 2ll * id + (c - kAccScreen) : nullptr;
  if (c < kAccColor) return ABS ? p.grad_screen_abs + 2ll * id + (c - kAccAbs) : nullptr;
  if (c < kAccStride) return COLORS4 ? p.grad_colors + 4ll * id + (c - kAccColor) : nullptr;
  return nullptr;
}

// pixel of tile-local thread l: 4x4 regions in row-major order, each as
// 2x2 quads of 2x2 pixels (the blend's layout)
SPLAT_DEV int2 local_pixel(int l) {
  return make_int2(4 * ((l >> 4) & 3) + 2 * ((l >> 2) & 1) + (l & 1),
                   4 * (l >> 6) + 2 * ((l >> 3) & 1) + ((l >> 1) & 1));
}

template <int CHP, bool SCREEN, bool ABS>
__global__ void __launch_bounds__(256, 3) aaa_record_backward_kernel(HierParams p) {
  extern __shared__ float4 tile_shared_raw[];
  TileShared& s = *reinterpret_cast<TileShared*>(tile_shared_raw);
  const int tile = blockIdx.x;
  if (p.tile_overflow[tile]) return;  // the replay kernel's tile
  const int local = threadIdx.x, lane = local & 31, warp = local >> 5;
  const int gx = (p.width + 15) / 16;
  const int tile_x = tile % gx * 16, tile_y = tile / gx * 16;
  int2 xy = local_pixel(local);
  xy.x += tile_x;
  xy.y += tile_y;
  const bool inside = xy.x < p.width && xy.y < p.height;
  const int count = inside ? max(p.record_counts[(static_cast<long long>(tile) << 8) + local], 0) : 0;
  const int first = p.ranges[2 * tile], range_size = p.ranges[2 * tile + 1] - first;
  auto gaussian_of = [&](int pos) {
    if (pos < 0 || pos >= range_size) return -1;
    const int g = p.points[first + pos];
    return g >= 0 && g < p.n ? g : -1;
  };
  float2* rec = p.records + ((static_cast<long long>(tile) * p.record_capacity) << 8);
  const int C = p.channels;
  const bool colors4 = CHP == 4 && C == 4 && (reinterpret_cast<uintptr_t>(p.grad_colors) & 15) == 0;

  // 1. histogram of the positions
  for (int k = local; k < kTilePositions; k += 256) s.cursor[k] = 0;
  if (local == 0) {
    s.max_pos = -1;
    s.fallback = 0;
  }
  __syncthreads();
  int my_max = -1;
#pragma unroll 4
  for (int j = 0; j < count; ++j) {
    const int pos = __float_as_int(rec[(static_cast<long long>(j) << 8) + local].x);
    if (pos >= 0 && pos < kTilePositions) {
      atomicAdd(&s.cursor[pos], 1);
      my_max = max(my_max, pos);
    } else {
      s.fallback = 1;
    }
  }
  my_max = __reduce_max_sync(kFull, my_max);
  if (lane == 0) atomicMax(&s.max_pos, my_max);
  __syncthreads();
  // exclusive scan of the histogram: four bins per thread
  {
    int bins[4], sum = 0;
#pragma unroll
    for (int k = 0; k < 4; ++k) {
      bins[k] = s.cursor[4 * local + k];
      sum += bins[k];
    }
    int inclusive = sum;
#pragma unroll
    for (int d = 1; d < 32; d <<= 1) {
      const int v = __shfl_up_sync(kFull, inclusive, d);
      if (lane >= d) inclusive += v;
    }
    if (lane == 31) s.warp_sums[warp] = inclusive;
    __syncthreads();
    int before = inclusive - sum;
    for (int w = 0; w < warp; ++w) before += s.warp_sums[w];
#pragma unroll
    for (int k = 0; k < 4; ++k) {
      s.offsets[4 * local + k] = before;
      s.cursor[4 * local + k] = before;
      before += bins[k];
    }
    if (local == 255) {
      s.offsets[kTilePositions] = before;
      if (before > kTileSamples) s.fallback = 1;
    }
  }
  // the staged Gaussians and pixel gradients
  const int staged = min(min(s.max_pos + 1, range_size), kTileCache);
  for (int k = local; k < staged; k += 256) {
    const int id = gaussian_of(k);
    s.ids[k] = id;
    s.opacity[k] = id >= 0 ? p.opacity[id] : 0.0f;
    if (colors4)
      s.rgb[k] = id >= 0 ? reinterpret_cast<const float4*>(p.colors)[id] : make_float4(0, 0, 0, 0);
  }
  const long long idx = static_cast<long long>(xy.y) * p.width + xy.x;
  const long long plane = static_cast<long long>(p.width) * p.height;
  float gradient[CHP], final_color[CHP], color[CHP];
  float bg_grad = 0.0f;
  const float final_T = count > 0 ? p.final_t_in[idx] : 0.0f;
#pragma unroll
  for (int c = 0; c < CHP; ++c) {
    gradient[c] = final_color[c] = color[c] = 0.0f;
    if (c < C && count > 0) {
      gradient[c] = p.pixel_grad[c * plane + idx];
      final_color[c] = p.image_in[c * plane + idx] - final_T * p.bg[c];
      bg_grad += p.bg[c] * gradient[c];
    }
  }
  if (colors4) s.pixel_grad[local] = make_float4(gradient[0], gradient[1 % CHP], gradient[2 % CHP],
                                                gradient[3 % CHP]);
  __syncthreads();
  const bool direct = s.fallback != 0;

  // 2. the pixel's samples in blend order
  const float x = static_cast<float>(xy.x), y = static_cast<float>(xy.y);
  float T = 1.0f;
  float2 entry = count > 0 ? rec[local] : make_float2(0.0f, 0.0f);
  for (int j = 0; j < count; ++j) {
    const float2 next = j + 1 < count ? rec[(static_cast<long long>(j + 1) << 8) + local] : entry;
    const int pos = __float_as_int(entry.x);
    const float gaussian = entry.y;
    int id;
    float opacity;
    float4 rgb4 = make_float4(0.0f, 0.0f, 0.0f, 0.0f);
    if (pos >= 0 && pos < staged) {
      id = s.ids[pos];
      opacity = s.opacity[pos];
      if (colors4) rgb4 = s.rgb[pos];
    } else {
      id = gaussian_of(pos);
      opacity = id >= 0 ? p.opacity[id] : 0.0f;
      if (colors4 && id >= 0) rgb4 = reinterpret_cast<const float4*>(p.colors)[id];
    }
    float2* slot_entry = rec + (static_cast<long long>(j) << 8) + local;
    if (id < 0) {  // never blended; filed with zero terms
      if (!direct) {
        s.list[atomicAdd(&s.cursor[pos], 1)] = static_cast<unsigned short>((j << 8) | local);
        *slot_entry = make_float2(0.0f, 0.0f);
      }
      entry = next;
      continue;
    }
    const float alpha = wp_min(0.99f, opacity * gaussian);
    const float next_t = T * (1.0f - alpha);
    const float rgb4a[4] = {rgb4.x, rgb4.y, rgb4.z, rgb4.w};
    const float* rgb = p.colors + static_cast<long long>(id) * C;
    float alpha_gradient = 0.0f;
    const float weight = alpha * T;
    float terms[kAccStride];
#pragma unroll
    for (int c = 0; c < CHP; ++c) {
      if (c < C) {
        const float v = colors4 ? rgb4a[c & 3] : rgb[c];
        color[c] = color[c] + v * alpha * T;
        const float behind = (final_color[c] - color[c]) / next_t;
        alpha_gradient += (v - behind) * gradient[c];
        if (colors4) terms[kAccColor + (c & 3)] = weight * gradient[c];
        else red_add(p.grad_colors + static_cast<long long>(id) * C + c, weight * gradient[c]);
      }
    }
    alpha_gradient *= T;
    alpha_gradient += (-final_T / (1.0f - alpha)) * bg_grad;
    if (direct) {
      const SampleData d = load_sample(p, id);
      ray_terms<SCREEN, ABS>(d.r0, d.r1, d.r3, x, y, opacity * alpha_gradient * gaussian, terms);
      terms[kAccOpacity] = gaussian * alpha_gradient;
      if (colors4) flush_row<SCREEN, ABS, true>(p, id, terms);
      else flush_row<SCREEN, ABS, false>(p, id, terms);
    } else {
      s.list[atomicAdd(&s.cursor[pos], 1)] = static_cast<unsigned short>((j << 8) | local);
      *slot_entry = make_float2(weight, gaussian * alpha_gradient);
    }
    T = next_t;
    entry = next;
  }
  __syncthreads();
  if (direct) return;

  // 3. per position, the sum of its samples' terms over the tile
  const int npos = s.max_pos + 1;
  for (int pp = warp; pp < npos; pp += 8) {
    const int b = s.offsets[pp], e = s.offsets[pp + 1];
    if (b == e) continue;
    const int id = pp < staged ? s.ids[pp] : gaussian_of(pp);
    if (id < 0) continue;
    const float opacity = pp < staged ? s.opacity[pp] : p.opacity[id];
    const float4* rows = reinterpret_cast<const float4*>(p.transforms) + 4ll * id;
    const float4 r0 = rows[0], r1 = rows[1], r3 = rows[3];
    float acc[32];
#pragma unroll
    for (int c = 0; c < 32; ++c) acc[c] = 0.0f;
    // the entry code (j << 8) | pixel is also the record's index in the
    // tile; the next chunk's entry is requested before this one is computed
    int k = b + lane;
    unsigned code = k < e ? s.list[k] : 0u;
    float2 v = k < e ? rec[code] : make_float2(0.0f, 0.0f);
    for (; k - lane < e; k += 32) {
      const int kn = k + 32;
      const unsigned code_next = kn < e ? s.list[kn] : 0u;
      const float2 v_next = kn < e ? rec[code_next] : make_float2(0.0f, 0.0f);
      if (k >= e) break;
      const int l = static_cast<int>(code & 255u);
      const int2 pxy = local_pixel(l);
      float terms[kAccStride];
      ray_terms<SCREEN, ABS>(r0, r1, r3, static_cast<float>(tile_x + pxy.x),
                             static_cast<float>(tile_y + pxy.y), opacity * v.y, terms);
      terms[kAccOpacity] = v.y;
      if (colors4) {
        const float4 g = s.pixel_grad[l];
        terms[kAccColor] = v.x * g.x;
        terms[kAccColor + 1] = v.x * g.y;
        terms[kAccColor + 2] = v.x * g.z;
        terms[kAccColor + 3] = v.x * g.w;
      } else {
#pragma unroll
        for (int c = kAccColor; c < kAccStride; ++c) terms[c] = 0.0f;
      }
#pragma unroll
      for (int c = 0; c < kAccStride; ++c) acc[c] += terms[c];
      code = code_next;
      v = v_next;
    }
    const float total = warp_row_sum(acc, lane);
    float* dst = colors4 ? component_address<SCREEN, ABS, true>(p, id, lane)
                         : component_address<SCREEN, ABS, false>(p, id, lane);
    if (dst) red_add(dst, total);
  }
}

}  // namespace aaa
}  // namespace splat
