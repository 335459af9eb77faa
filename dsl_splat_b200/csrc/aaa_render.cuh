// AAA-Gaussians hierarchical (StopThePop HIER 64/8/4) blend and its replay
// backward: the B200 kernels for aaa/render_hierarchical_warp.py:105-691
// (K24) and aaa/backward_render.py:23-137 with aaa/render_adjoint.py:279-352
// (K27).
//
// One 256-thread CTA per 16x16 tile.  Each warp owns two 4x4 pixel regions
// (one per half warp) and their 64-entry tail queues, and eight 2x2 quads
// with 8-entry mid queues; every pixel keeps a 4-entry head in registers.
// The tile's depth-sorted Gaussians arrive in batches of 32 (one per lane):
// each is culled against and sampled at both regions' centres, the batch is
// sorted with Batcher's network and merged into the tails; a tail past 32
// entries drains 16 at a time through its quads' mid queues (sampled at the
// quad centre) into the pixel heads (sampled at the pixel), and the head's
// front sample is blended whenever a head is full.  The blend order is the
// approximate depth order these queues produce, so every comparison, tie
// rule and barrier of the reference is kept: the queue contents, and with
// them the images and counts, are bit-identical to the reference's (with
// the library's exp).  All synchronisation is warp-local (__syncwarp with
// the warp, half-warp or quad mask), as in the reference.
//
// The replay backward runs the same traversal from the start and, per
// blended sample, derives the colour weight and the alpha gradient from the
// saved final image and transmittance (front to back: the colour behind a
// sample is (final - accumulated) / T_next); it adds 13 gradient terms per
// sample (colour channels, 9 + 3 transform entries, opacity) plus the
// optional screen-translation statistics with red.global.add.
//
// Memory guards the reference does not have: an entry id of -1 never
// indexes the Gaussian arrays (the reference reads before the array start on
// degenerate depths, e.g. an infinite one; such entries get depth FLT_MAX,
// amplitude 0 and colour 0 here).  Scenes with finite depths never reach
// them.
#pragma once
#include "aaa.cuh"
#include "aaa_blend_params.cuh"

namespace splat {
namespace aaa {

constexpr float kInf = FLT_MAX;  // the renderer's INF (3.4028234663852886e38)

// ---- aaa/render_warp_geometry.py ------------------------------------------------

SPLAT_DEV float rdot4(const float a[4], const float b[4]) {
  return (a[0] * b[0] + a[1] * b[1]) + (a[2] * b[2] + a[3] * b[3]);
}

// g[r] - g[3] * s, component by component
SPLAT_DEV void plane_of(const M4& g, int r, float s, float out[4]) {
#pragma unroll
  for (int k = 0; k < 4; ++k) out[k] = g.m[r][k] - g.m[3][k] * s;
}

// :41-57 closest_ray: the point of the line where planes a and b meet that
// lies closest to the Gaussian's centre, and its squared distance
SPLAT_DEV float closest_ray(const float a[4], const float b[4], float pos[4]) {
  const float d[3] = {a[1] * b[2] - a[2] * b[1], a[2] * b[0] - a[0] * b[2], a[0] * b[1] - a[1] * b[0]};
  const float m[3] = {a[3] * b[0] - a[0] * b[3], a[3] * b[1] - a[1] * b[3], a[3] * b[2] - a[2] * b[3]};
  const float dd = rdot3(d, d);
  const float s[3] = {m[0] / dd, m[1] / dd, m[2] / dd};
  pos[0] = d[1] * s[2] - s[1] * d[2];
  pos[1] = d[2] * s[0] - s[2] * d[0];
  pos[2] = d[0] * s[1] - s[0] * d[1];
  pos[3] = 1.0f;
  return rdot3(m, s);
}

// :60-64 sample: -distance^2 / 2 and the screen depth of the ray of (x, y).
// Kept out of line (as region_frustum), with the transform passed by value
// in registers: the blend calls it from seven places, and one copy keeps
// the kernel's instruction footprint small.
__device__ __noinline__ float2 ray_sample_rows(float4 r0, float4 r1, float4 r2, float4 r3, float x,
                                               float y) {
  const float a[4] = {r0.x - r3.x * x, r0.y - r3.y * x, r0.z - r3.z * x, r0.w - r3.w * x};
  const float b[4] = {r1.x - r3.x * y, r1.y - r3.y * y, r1.z - r3.z * y, r1.w - r3.w * y};
  float pos[4];
  const float sq = closest_ray(a, b, pos);
  const float g2[4] = {r2.x, r2.y, r2.z, r2.w};
  const float g3[4] = {r3.x, r3.y, r3.z, r3.w};
  return make_float2(-0.5f * sq, rdot4(g2, pos) * __frcp_rn(rdot4(g3, pos)));
}

SPLAT_DEV float4 row4(const M4& g, int r) {
  return make_float4(g.m[r][0], g.m[r][1], g.m[r][2], g.m[r][3]);
}

SPLAT_DEV void ray_sample(const M4& g, float x, float y, float& power, float& depth) {
  const float2 v = ray_sample_rows(row4(g, 0), row4(g, 1), row4(g, 2), row4(g, 3), x, y);
  power = v.x;
  depth = v.y;
}

SPLAT_DEV void rtransform(const M4& g, const float p[4], float out[4]) {
#pragma unroll
  for (int r = 0; r < 4; ++r) {
    const float row[4] = {g.m[r][0], g.m[r][1], g.m[r][2], g.m[r][3]};
    out[r] = rdot4(row, p);
  }
}

// :67-120 frustum: half the smallest squared Gaussian-space distance from
// the centre to the frustum of the w x h pixel rectangle at (x, y)
__device__ __noinline__ float region_frustum_rows(float4 r0, float4 r1, float4 r2, float4 r3,
                                                  float x, float y, float w, float h) {
  M4 g;
  const float4 rows[4] = {r0, r1, r2, r3};
#pragma unroll
  for (int r = 0; r < 4; ++r) {
    g.m[r][0] = rows[r].x;
    g.m[r][1] = rows[r].y;
    g.m[r][2] = rows[r].z;
    g.m[r][3] = rows[r].w;
  }
  const float start[3] = {x, y, -1.0f}, extent[3] = {w, h, 2.0f};
  auto inside = [&](const float p[4], int axis) {
    const float delta = p[axis] - start[axis] * p[3];
    return delta > 0.0f && delta < extent[axis] * p[3];
  };
  const float mean[4] = {g.m[0][3], g.m[1][3], g.m[2][3], g.m[3][3]};
  float best = FLT_MAX;
  if (inside(mean, 0) && inside(mean, 1) && inside(mean, 2)) {
    best = 0.0f;
  } else {
    const float dx = copysignf(w * 0.5f, (mean[0] - x * mean[3]) - w * 0.5f * mean[3]);
    const float dy = copysignf(h * 0.5f, (mean[1] - y * mean[3]) - h * 0.5f * mean[3]);
    float ax[4], ay[4], other[4], pos[4], screen[4];
    plane_of(g, 0, x + w * 0.5f + dx, ax);
    plane_of(g, 1, y + h * 0.5f + dy, ay);
    auto test_plane = [&](const float a[4], int other_axis) {
      const float norm = a[3] / ((a[0] * a[0] + a[1] * a[1]) + a[2] * a[2]);
      const float p[4] = {-a[0] * norm, -a[1] * norm, -a[2] * norm, 1.0f};
      rtransform(g, p, screen);
      const float value = a[3] * norm;
      if (value < best && inside(screen, other_axis) && inside(screen, 2)) best = value;
    };
    auto test_edge = [&](const float a[4], const float b[4]) {
      const float sq = closest_ray(a, b, pos);
      rtransform(g, pos, screen);
      if (sq < best && inside(screen, 2)) best = sq;
    };
    test_plane(ax, 1);
    test_plane(ay, 0);
    test_edge(ax, ay);
    plane_of(g, 1, y + h * 0.5f - dy, other);
    test_edge(ax, other);
    plane_of(g, 0, x + w * 0.5f - dx, other);
    test_edge(other, ay);
  }
  return 0.5f * best;
}

SPLAT_DEV float region_frustum(const M4& g, float x, float y, float w, float h) {
  return region_frustum_rows(row4(g, 0), row4(g, 1), row4(g, 2), row4(g, 3), x, y, w, h);
}

// ---- kernel state -------------------------------------------------------------------



struct WarpQueues {  // per warp: two 4x4 tails, eight 2x2 mids
  float tail_d[2][64];
  int tail_id[2][64];
  float mid_d[8][8];
  int mid_id[8][8];
};

template <int CHP, bool BWD>
struct HierPixel {
  bool active;
  float T;
  int contributors, tail_count, mid_count, head_count;
  float hd[4], ha[4], hg[4];
  int hid[4];
  float color[CHP];
  float gradient[BWD ? CHP : 1], final_color[BWD ? CHP : 1];
  float final_T, bg_grad;
  int records;
};

// render_adjoint.py:285-351 accumulate: one accepted sample's gradients
template <bool SCREEN, bool ABS>
SPLAT_DEV void accumulate_ray_gradient(const HierParams& p, int id, float x, float y, float gaussian,
                                       float alpha_gradient) {
  const M4 g = load_m4(p.transforms, id);
  float a[4], b[4];
  plane_of(g, 0, x, a);
  plane_of(g, 1, y, b);
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
  const float factor = p.opacity[id] * alpha_gradient * gaussian;
  const float inverse_dd = __frcp_rn(dd);
  const float ratio = mm / dd * inverse_dd;
  float screen_x = 0.0f, screen_y = 0.0f;
  float* t = p.grad_transforms + 16ll * id;
#pragma unroll
  for (int axis = 0; axis < 3; ++axis) {
    const float dd0 = yy * nx[axis] - xy * ny[axis];
    const float dd1 = xx * ny[axis] - xy * nx[axis];
    const float dd3 = (xy * (y * nx[axis] + x * ny[axis]) - xyy * nx[axis]) - yxx * ny[axis];
    const float d0 = factor * (ratio * dd0 - (ndy * moment[axis]) * inverse_dd);
    const float d1 = factor * (ratio * dd1 - (dx * moment[axis]) * inverse_dd);
    const float d3 = factor * (ratio * dd3 - (cross * moment[axis]) * inverse_dd);
    if (SCREEN) {
      screen_x += d0 * g.m[3][axis];
      screen_y += d1 * g.m[3][axis];
    }
    // one vector reduction per row; the screen-depth entry (column 2 of the
    // reference's float4 blocks) receives +0 and stays zero
    red_add_v4(t + axis * 4, d0, d1, 0.0f, d3);
  }
  const float tr0 = factor * -ym * inverse_dd;
  const float tr1 = factor * xm * inverse_dd;
  const float tr3 = factor * -(y * xm - x * ym) * inverse_dd;
  red_add_v4(t + 12, tr0, tr1, 0.0f, tr3);
  red_add(p.grad_opacity + id, gaussian * alpha_gradient);
  if (SCREEN) {
    screen_x += tr0 * g.m[3][3];
    screen_y += tr1 * g.m[3][3];
    red_add_v2(p.grad_screen + 2ll * id, screen_x, screen_y);
    if (ABS) red_add_v2(p.grad_screen_abs + 2ll * id, fabsf(screen_x), fabsf(screen_y));
  }
}

// statistics.py:57-73 observe: a blended sample with weight w = alpha * T
// adds 1 (masked count) or map * w (weighted sum) to its Gaussian wherever
// the pixel's map value is nonzero (render_hierarchical_warp.py:160-163)
SPLAT_DEV void observe(const HierParams& p, int id, int pixel, float w) {
  const long long P = static_cast<long long>(p.width) * p.height;
  int count_row = 0, sum_row = 0;
  for (int r = 0; r < p.stat_count; ++r) {
    const float v = p.stat_pixels[r * P + pixel];
    if ((p.stat_sum_mask >> r) & 1) {
      if (v != 0.0f) atomicAdd(p.stat_sums + static_cast<long long>(sum_row) * p.n + id, v * w);
      ++sum_row;
    } else {
      if (v != 0.0f) atomicAdd(p.stat_counts + static_cast<long long>(count_row) * p.n + id, 1);
      ++count_row;
    }
  }
}

template <int CHP, bool BWD, bool SCREEN, bool ABS, bool STATS = false>
struct HierWarp {
  const HierParams& p;
  WarpQueues& q;
  int lane, half, hl, quad, mr, tile, local;
  int x0, y0, tile_x;
  int first, range_size;  // the tile's slice of point_list

  // The queues and heads carry an entry's position in the tile's slice of
  // point_list (an equivalent payload to the reference's Gaussian id: the
  // algorithm only moves it and tests it against -1); the Gaussian id of a
  // position, or -1.
  SPLAT_DEV int gaussian_of(int pos) const {
    if (pos < 0 || pos >= range_size) return -1;
    const int g = p.points[first + pos];
    return g >= 0 && g < p.n ? g : -1;
  }
  unsigned half_mask, quad_mask;
  HierPixel<CHP, BWD> px;
  int x, y;

  SPLAT_DEV HierWarp(const HierParams& params, WarpQueues& queues) : p(params), q(queues) {}

  // blend_step (render_hierarchical_warp.py:146-171) / blend_backward
  // (backward_render.py:32-70): the head's front sample
  SPLAT_DEV void blend() {
    px.head_count -= 1;
    if (!px.active) return;
    const float alpha = px.ha[0];
    const float next_t = px.T * (1.0f - alpha);
    if (next_t < 0.0001f) {
      px.active = false;  // the sample that would terminate is not blended
      return;
    }
    const int id = gaussian_of(px.hid[0]);
    const int C = p.channels;
    const float* rgb = p.colors + static_cast<long long>(id) * C;
    if (!BWD) {
#pragma unroll
      for (int c = 0; c < CHP; ++c)
        if (c < C) px.color[c] = px.color[c] + (id >= 0 ? rgb[c] : 0.0f) * alpha * px.T;
      if (STATS && id >= 0) observe(p, id, y * p.width + x, alpha * px.T);
      if (p.records) {
        if (px.records < p.record_capacity) {
          const long long at = ((static_cast<long long>(tile) * p.record_capacity + px.records) << 8) + local;
          p.records[at] = make_float2(__int_as_float(px.hid[0]), px.hg[0]);
        }
        ++px.records;
      }
    } else {
      float alpha_gradient = 0.0f;
      const float weight = alpha * px.T;
#pragma unroll
      for (int c = 0; c < CHP; ++c) {
        if (c < C) {
          const float v = id >= 0 ? rgb[c] : 0.0f;
          px.color[c] = px.color[c] + v * alpha * px.T;
          const float behind = (px.final_color[c] - px.color[c]) / next_t;
          alpha_gradient += (v - behind) * px.gradient[c];
          if (id >= 0 && !(CHP == 4 && C == 4 && (reinterpret_cast<uintptr_t>(p.grad_colors) & 15) == 0))
            red_add(p.grad_colors + static_cast<long long>(id) * C + c, weight * px.gradient[c]);
        }
      }
      if (id >= 0 && CHP == 4 && C == 4 && (reinterpret_cast<uintptr_t>(p.grad_colors) & 15) == 0) {
        // RGB + the constant channel: the four colour gradients in one reduction
        red_add_v4(p.grad_colors + 4ll * id, weight * px.gradient[0], weight * px.gradient[1],
                   weight * px.gradient[2], weight * px.gradient[3]);
      }
      alpha_gradient *= px.T;
      alpha_gradient += (-px.final_T / (1.0f - alpha)) * px.bg_grad;
      if (id >= 0)
        accumulate_ray_gradient<SCREEN, ABS>(p, id, static_cast<float>(x), static_cast<float>(y),
                                             px.hg[0], alpha_gradient);
    }
    px.T = next_t;
#pragma unroll
    for (int j = 1; j < 4; ++j) {
      px.hd[j - 1] = px.hd[j];
      px.ha[j - 1] = px.ha[j];
      px.hid[j - 1] = px.hid[j];
      px.hg[j - 1] = px.hg[j];
    }
    px.hd[3] = kInf;
  }

  // :221-238 insert_head: strict comparison keeps equal-depth entries first
  SPLAT_DEV void insert_head(float depth, float alpha, int id, float gaussian) {
#pragma unroll
    for (int s = 0; s < 4; ++s) {
      if (depth < px.hd[s]) {
        const float od = px.hd[s], oa = px.ha[s], og = px.hg[s];
        const int oi = px.hid[s];
        px.hd[s] = depth;
        px.ha[s] = alpha;
        px.hid[s] = id;
        px.hg[s] = gaussian;
        depth = od;
        alpha = oa;
        id = oi;
        gaussian = og;
      }
    }
    px.head_count += 1;
  }

  // :176-214 merge: the sorted N-entry run at qd[old..old+N) and the incoming
  // sorted run (lane `rank` of the group holds entry rank) into qd[0..2N)
  template <int N>
  SPLAT_DEV void merge(float* qd, int* qi, unsigned mask, int rank, int old, float depth, int id) {
    int new_pos = 0;
#pragma unroll
    for (int stride = N / 2; stride > 0; stride /= 2)
      if (qd[old + new_pos + stride] <= depth) new_pos += stride;
    new_pos += 1;
    if (qd[old] > depth) new_pos = 0;
    new_pos += rank;
    const float old_depth = qd[old + rank];
    __syncwarp(mask);
    qd[old + rank] = depth;
    __syncwarp(mask);
    int old_pos = 0;
#pragma unroll
    for (int stride = N / 2; stride > 0; stride /= 2)
      if (qd[old + old_pos + stride] < old_depth) old_pos += stride;
    old_pos += 1;
    if (qd[old] >= old_depth) old_pos = 0;
    old_pos += rank;
    const int old_id = qi[old + rank];
    __syncwarp(mask);
    qd[new_pos] = depth;
    qi[new_pos] = id;
    qd[old_pos] = old_depth;
    qi[old_pos] = old_id;
    __syncwarp(mask);
  }

  // :360-390 sort_batch: Batcher's network over the half's incoming run
  // [32, 64) of its tail, sixteen lanes, one compare-exchange each per step
  SPLAT_DEV void sort_batch() {
    float* qd = q.tail_d[half];
    int* qi = q.tail_id[half];
    auto exchange = [&](int a, int b) {
      const float da = qd[a], db = qd[b];
      if (da > db) {
        const int ia = qi[a], ib = qi[b];
        qd[a] = db;
        qi[a] = ib;
        qd[b] = da;
        qi[b] = ia;
      }
    };
#pragma unroll
    for (int size = 2; size <= 32; size *= 2) {
      int stride = size / 2;
      const int offset = hl & (stride - 1);
      __syncwarp(half_mask);
      int pos = 2 * hl - (hl & (stride - 1));
      exchange(32 + pos, 32 + pos + stride);
#pragma unroll
      for (stride /= 2; stride > 0; stride /= 2) {
        __syncwarp(half_mask);
        pos = 2 * hl - (hl & (stride - 1));
        if (offset >= stride) exchange(32 + pos - stride, 32 + pos);
      }
    }
  }

  // :262-306 front_mid: the quad consumes the front four entries of its mid
  // queue, sampling each at its own pixel
  SPLAT_DEV void front_mid(bool check_valid) {
    const int* mi = q.mid_id[quad];
    if (__any_sync(quad_mask, px.active)) {
      const int load_pos = mi[mr];
      const int load_gid = gaussian_of(load_pos);
      float amplitude = 0.0f;
      if ((!check_valid || load_pos != -1) && load_gid >= 0) amplitude = p.opacity[load_gid];
      for (int inner = 0; inner < 4; ++inner) {
        if (px.head_count >= 4) blend();
        const int id = mi[inner];
        if (check_valid && id == -1) continue;
        const int gid = __shfl_sync(quad_mask, load_gid, inner, 4);
        const float weight = __shfl_sync(quad_mask, amplitude, inner, 4);
        if (!px.active) continue;
        px.contributors += 1;
        if (gid < 0) continue;  // guard (see the header)
        float power, depth;
        ray_sample(load_m4(p.transforms, gid), static_cast<float>(x), static_cast<float>(y), power,
                   depth);
        if (depth < -1.0f || depth > 1.0f) continue;
        const float gaussian = splat_expf(power);
        const float alpha = wp_min(0.99f, weight * gaussian);
        if (alpha < 1.0f / 255.0f) continue;
        insert_head(depth, alpha, id, gaussian);
      }
    }
    px.mid_count -= 4;
    __syncwarp(half_mask);
  }

  // :308-355 push_mid: sixteen tail entries through the half's four quads
  SPLAT_DEV void push_mid(bool check_valid) {
    const int* ti = q.tail_id[half];
    float* md = q.mid_d[quad];
    int* mi = q.mid_id[quad];
    const int load_pos = ti[hl];
    const int mg = hl >> 2;
    for (int batch = 0; batch < 4; ++batch) {
      if (check_valid && px.tail_count == 0) break;
      const int source = 4 * batch + mr;
      const int id = ti[source];
      const int gpos = __shfl_sync(half_mask, load_pos, source, 16);
      const int gid = gaussian_of(gpos);
      float depth = kInf;
      if ((!check_valid || gpos != -1) && gid >= 0) {
        float power;
        ray_sample(load_m4(p.transforms, gid), static_cast<float>(x0 + 1 + 2 * (mg & 1)),
                   static_cast<float>(y0 + 1 + 2 * (mg >> 1)), power, depth);
      }
      if (check_valid && id == -1) depth = kInf;
      // :243-252 rank_mid
      int rank = 0;
#pragma unroll
      for (int j = 1; j < 4; ++j) {
        const int other_rank = (mr + j) & 3;
        const float other = __shfl_sync(quad_mask, depth, other_rank, 4);
        if (other < depth || (other == depth && other_rank < mr)) ++rank;
      }
      md[rank] = depth;
      mi[rank] = id;
      __syncwarp(quad_mask);
      const float d = md[mr];
      const int i = mi[mr];
      px.mid_count += 4;
      if (batch != 0 || px.mid_count > 4) {
        merge<4>(md, mi, quad_mask, mr, 4, d, i);
        front_mid(false);
      } else {
        md[4 + mr] = d;
        mi[4 + mr] = i;
      }
      __syncwarp(quad_mask);
      if (check_valid) px.tail_count -= min(4, px.tail_count);
    }
    if (!check_valid) px.tail_count -= 16;
  }

  // local: the thread's index among the tile's 256 (the block may hold a
  // part of the tile's warps)
  SPLAT_DEV void run(int tile_id, int local_index) {
    tile = tile_id;
    local = local_index;
    const int gx = (p.width + 15) / 16;
    tile_x = tile % gx * 16;
    const int tile_y = tile / gx * 16;
    lane = local & 31;
    half = lane >> 4;
    hl = lane & 15;
    quad = lane >> 2;
    mr = lane & 3;
    const int tail = local >> 4;
    x0 = tile_x + 4 * (tail & 3);
    y0 = tile_y + 4 * (tail >> 2);
    const int mg = hl >> 2;
    x = x0 + 2 * (mg & 1) + (mr & 1);
    y = y0 + 2 * (mg >> 1) + (mr >> 1);
    half_mask = 0xFFFFu << (lane & 16);
    quad_mask = 0xFu << (lane & 28);
    const int C = p.channels;
    px.active = x < p.width && y < p.height;
    px.T = 1.0f;
    px.contributors = px.tail_count = px.mid_count = px.head_count = 0;
#pragma unroll
    for (int k = 0; k < 4; ++k) {
      px.hd[k] = kInf;
      px.ha[k] = 0.0f;
      px.hg[k] = 0.0f;
      px.hid[k] = -1;
    }
#pragma unroll
    for (int c = 0; c < CHP; ++c) px.color[c] = 0.0f;
    px.final_T = 0.0f;
    px.bg_grad = 0.0f;
    px.records = 0;
    if (BWD) {
#pragma unroll
      for (int c = 0; c < CHP; ++c) px.gradient[c] = px.final_color[c] = 0.0f;
      if (px.active) {
        const long long idx = static_cast<long long>(y) * p.width + x;
        const long long plane = static_cast<long long>(p.width) * p.height;
        px.final_T = p.final_t_in[idx];
#pragma unroll
        for (int c = 0; c < CHP; ++c) {
          if (c < C) {
            px.gradient[c] = p.pixel_grad[c * plane + idx];
            px.final_color[c] = p.image_in[c * plane + idx] - px.final_T * p.bg[c];
            px.bg_grad += p.bg[c] * px.gradient[c];
          }
        }
      }
    }
    first = p.ranges[2 * tile];
    const int last = p.ranges[2 * tile + 1];
    range_size = last - first;
    const int tail0 = (tail & ~1);
    for (int progress = first; progress < last; progress += 32) {
      if (!__any_sync(kFull, px.active)) break;
      const int pos = progress + lane < last ? progress + lane - first : -1;
      const int gid = gaussian_of(pos);
      M4 g = {};
      float amplitude = 0.0f;
      if (gid >= 0) {
        g = load_m4(p.transforms, gid);
        if (p.cull) amplitude = p.opacity[gid];
      }
      int culled = 0;
#pragma unroll
      for (int h = 0; h < 2; ++h) {
        const int og = tail0 + h;
        if (p.cull && gid != -1) {
          const float power = region_frustum(g, static_cast<float>(tile_x + 4 * (og & 3)),
                                             static_cast<float>(y0), 3.0f, 3.0f);
          if (wp_min(0.99f, amplitude * splat_expf(-power)) < 1.0f / 255.0f) culled |= 1 << h;
        }
      }
#pragma unroll
      for (int h = 0; h < 2; ++h) {
        const int og = tail0 + h;
        float depth = kInf;
        if (gid != -1 && (!p.cull || !(culled & (1 << h)))) {
          float power;
          ray_sample(g, static_cast<float>(tile_x + 4 * (og & 3) + 2), static_cast<float>(y0 + 2),
                     power, depth);
        }
        q.tail_d[h][32 + lane] = depth;
        q.tail_id[h][32 + lane] = depth == kInf ? -1 : pos;
      }
      __syncwarp(kFull);
      sort_batch();
      __syncwarp(kFull);
#pragma unroll
      for (int h = 0; h < 2; ++h) {
        float* qd = q.tail_d[h];
        int* qi = q.tail_id[h];
        const int old_count = __shfl_sync(kFull, px.tail_count, h * 16);
        const float key = qd[32 + lane];
        const int id = qi[32 + lane];
        const int added = __popc(__ballot_sync(kFull, id != -1));
        if (h == half) px.tail_count += added;
        if (old_count != 0) {
          merge<32>(qd, qi, kFull, lane, 0, key, id);
        } else {
          qd[lane] = key;
          qi[lane] = id;
        }
      }
      __syncwarp(kFull);
      // not unrolled: each unrolled copy would inline push_mid (and its
      // front_mid and blend) once more; the smaller kernel measured 9 %
      // faster (instruction-cache misses were its top stall)
#pragma unroll 1
      for (int it = 0; it < 2; ++it) {
        if (px.tail_count > 32) {
          push_mid(false);
          __syncwarp(half_mask);
          float* qd = q.tail_d[half];
          int* qi = q.tail_id[half];
          for (int index = 0; index < 3 - it; ++index) {
            const int dest = hl + index * 16;
            qd[dest] = qd[dest + 16];
            qi[dest] = qi[dest + 16];
          }
          __syncwarp(half_mask);
        }
      }
      __syncwarp(kFull);
    }
    if (__any_sync(kFull, px.active)) {
      if (px.tail_count != 0) {
#pragma unroll 1
        for (int it = 0; it < 2; ++it) {
          push_mid(true);
          if (it == 0 && px.tail_count == 0) break;
          if (it == 0) {
            q.tail_d[half][hl] = q.tail_d[half][hl + 16];
            q.tail_id[half][hl] = q.tail_id[half][hl + 16];
            __syncwarp(half_mask);
          }
        }
      }
      if (__any_sync(kFull, px.active)) {
        if (px.mid_count != 0) {
          q.mid_d[quad][mr] = q.mid_d[quad][4 + mr];
          q.mid_id[quad][mr] = q.mid_id[quad][4 + mr];
          __syncwarp(quad_mask);
          front_mid(true);
        }
        while (px.active && px.head_count != 0) blend();
      }
    }
    if (!BWD && x < p.width && y < p.height) {
      const long long idx = static_cast<long long>(y) * p.width + x;
      const long long plane = static_cast<long long>(p.width) * p.height;
#pragma unroll
      for (int c = 0; c < CHP; ++c)
        if (c < C) p.image[c * plane + idx] = px.color[c] + px.T * p.bg[c];
      p.final_t[idx] = px.T;
      p.contributors[idx] = px.contributors;
    }
    if (!BWD && p.records) {
      const bool overflow = px.records > p.record_capacity;
      p.record_counts[(static_cast<long long>(tile) << 8) + local] = overflow ? -1 : px.records;
      if (overflow) p.tile_overflow[tile] = 1;
    }
  }
};

// The warps of a tile never interact, so a block holds two of them (a
// quarter of the tile): smaller blocks let more warps reside per SM at the
// kernels' register counts.  blockIdx.x = 4 * (tile slot) + quarter.
constexpr int kHierWarps = 2;
constexpr int kHierThreads = 32 * kHierWarps;
constexpr int kHierBlocksPerTile = 256 / kHierThreads;

// Register budget: the forward at 16 blocks (32 warps, 64 registers) per SM
// -- measured 5% faster than 12 blocks at 80 registers despite its spills --
// the replay (run for overflowed tiles only) at 8.
template <int CHP, bool BWD, bool SCREEN, bool ABS, bool STATS = false>
__global__ void __launch_bounds__(kHierThreads, BWD ? 8 : 16) aaa_hier_kernel(HierParams p) {
  __shared__ WarpQueues queues[kHierWarps];
  const int slot = blockIdx.x / kHierBlocksPerTile;
  const int tile = p.tile_order ? p.tile_order[slot] : slot;
  if (p.only_flagged && !p.only_flagged[tile]) return;
  const int local = (blockIdx.x % kHierBlocksPerTile) * kHierThreads + threadIdx.x;
  // every queue entry starts as an empty one (FLT_MAX, -1); the algorithm
  // writes each entry before reading it, so this only keeps unwritten shared
  // memory from ever being read as an id
  {
    WarpQueues& q = queues[threadIdx.x >> 5];
    const int lane = threadIdx.x & 31;
    float* d = &q.tail_d[0][0];
    int* i = &q.tail_id[0][0];
    for (int k = lane; k < 128; k += 32) {
      d[k] = kInf;
      i[k] = -1;
    }
    d = &q.mid_d[0][0];
    i = &q.mid_id[0][0];
    for (int k = lane; k < 64; k += 32) {
      d[k] = kInf;
      i[k] = -1;
    }
    __syncwarp();
  }
  HierWarp<CHP, BWD, SCREEN, ABS, STATS> w(p, queues[threadIdx.x >> 5]);
  w.run(tile, local);
}

}  // namespace aaa
}  // namespace splat
