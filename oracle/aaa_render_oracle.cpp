// CPU oracle for dsl_splat's AAA-Gaussians hierarchical blend (test
// infrastructure only: the tests use it as the checker; the product never
// links it).
//
// Restates aaa/render_hierarchical_warp.py:105-596 (the StopThePop HIER
// 64/8/4 renderer: per 4x4 pixel region a 64-entry tail queue, per 2x2 quad
// an 8-entry mid queue, per pixel a 4-entry head; 3D ray evaluation of
// aaa/render_warp_geometry.py) and its replay backward
// aaa/backward_render.py:23-137 with aaa/render_adjoint.py:279-352.
//
// Every synchronisation of that renderer is warp-local (__syncwarp with a
// full, half or quad mask, shuffles, ballots), so the eight warps of a tile
// never interact: each (tile, warp) is emulated on its own, lane by lane,
// with the warp's two tail queues and eight mid queues as plain arrays.
// Collective steps run every lane of their group before any lane goes on,
// which is the order the __syncwarp barriers impose.  The discrete
// decisions (queue order, culling, acceptance, termination) depend on the
// last bit of the depths, so the float32 operation order of the reference
// is kept (built with -ffp-contract=off; exp is oracle_expf, the same
// substitution the golden generator makes for wp.exp).
//
// Memory guards the reference does not have: an entry id of -1 never
// indexes the Gaussian arrays here (the reference would read before the
// array start on degenerate depths; such entries get depth FLT_MAX /
// amplitude 0 / colour 0 instead).  Scenes with finite depths never reach
// them.

#include <cfloat>
#include <cmath>
#include <cstring>
#include <utility>
#include <algorithm>

extern "C" float oracle_expf(float);

namespace {

constexpr float kInf = FLT_MAX;  // the renderer's INF constant (3.4028234663852886e38)
constexpr int kMaxChannels = 64;

struct Mat {
  float m[4][4];
};

// wp.min on floats: the first operand when it is smaller, else the second
float min_of(float a, float b) { return a < b ? a : b; }

struct F4 {
  float v[4];
};

Mat load_transform(const float* t, int id) {
  Mat g;
  std::memcpy(g.m, t + 16ll * id, sizeof(g.m));
  return g;
}

// aaa/render_warp_geometry.py:31-33 dot4: pairs summed, then the pairs
float dot4(const F4& a, const F4& b) {
  return (a.v[0] * b.v[0] + a.v[1] * b.v[1]) + (a.v[2] * b.v[2] + a.v[3] * b.v[3]);
}

// :26-28 dot3, left to right
float dot3(const float* a, const float* b) { return a[0] * b[0] + a[1] * b[1] + a[2] * b[2]; }

F4 row(const Mat& g, int r) { return F4{{g.m[r][0], g.m[r][1], g.m[r][2], g.m[r][3]}}; }

// g[r] - g[3] * s, component by component (product rounded, then the difference)
F4 plane(const Mat& g, int r, float s) {
  F4 out;
  for (int k = 0; k < 4; ++k) out.v[k] = g.m[r][k] - g.m[3][k] * s;
  return out;
}

F4 transform(const Mat& g, const F4& p) {
  return F4{{dot4(row(g, 0), p), dot4(row(g, 1), p), dot4(row(g, 2), p), dot4(row(g, 3), p)}};
}

struct Ray {
  F4 position;
  float squared_distance;
};

// :41-57 closest_ray: the point of the line where the planes a and b meet
// that is closest to the Gaussian's centre (Pluecker direction and moment)
Ray closest_ray(const F4& a, const F4& b) {
  const float d[3] = {a.v[1] * b.v[2] - a.v[2] * b.v[1], a.v[2] * b.v[0] - a.v[0] * b.v[2],
                      a.v[0] * b.v[1] - a.v[1] * b.v[0]};
  const float m[3] = {a.v[3] * b.v[0] - a.v[0] * b.v[3], a.v[3] * b.v[1] - a.v[1] * b.v[3],
                      a.v[3] * b.v[2] - a.v[2] * b.v[3]};
  const float dd = dot3(d, d);
  const float s[3] = {m[0] / dd, m[1] / dd, m[2] / dd};
  Ray r;
  r.position = F4{{d[1] * s[2] - s[1] * d[2], d[2] * s[0] - s[2] * d[0], d[0] * s[1] - s[0] * d[1],
                   1.0f}};
  r.squared_distance = dot3(m, s);
  return r;
}

// :60-64 sample: (-distance^2 / 2, screen depth) of the pixel ray (x, y)
void sample(const Mat& g, float x, float y, float* power, float* depth) {
  const Ray r = closest_ray(plane(g, 0, x), plane(g, 1, y));
  *depth = dot4(row(g, 2), r.position) * (1.0f / dot4(row(g, 3), r.position));
  *power = -0.5f * r.squared_distance;
}

bool inside(const F4& p, const float* start, const float* extent, int axis) {
  const float delta = p.v[axis] - start[axis] * p.v[3];
  return delta > 0.0f && delta < extent[axis] * p.v[3];
}

// :94-120 frustum: half the smallest squared Gaussian-space distance from
// the centre to the pixel rectangle's frustum (x..x+w, y..y+h, depth -1..1)
float frustum(const Mat& g, float x, float y, float w, float h) {
  const float start[3] = {x, y, -1.0f}, extent[3] = {w, h, 2.0f};
  const F4 mean{{g.m[0][3], g.m[1][3], g.m[2][3], g.m[3][3]}};
  float best = FLT_MAX;
  if (inside(mean, start, extent, 0) && inside(mean, start, extent, 1) &&
      inside(mean, start, extent, 2)) {
    best = 0.0f;
  } else {
    const float dx = std::copysign(w * 0.5f, (mean.v[0] - x * mean.v[3]) - w * 0.5f * mean.v[3]);
    const float dy = std::copysign(h * 0.5f, (mean.v[1] - y * mean.v[3]) - h * 0.5f * mean.v[3]);
    const F4 ax = plane(g, 0, x + w * 0.5f + dx);
    const F4 ay = plane(g, 1, y + h * 0.5f + dy);
    auto test_plane = [&](const F4& a, int other) {
      const float norm = a.v[3] / (a.v[0] * a.v[0] + a.v[1] * a.v[1] + a.v[2] * a.v[2]);
      const F4 screen = transform(g, F4{{-a.v[0] * norm, -a.v[1] * norm, -a.v[2] * norm, 1.0f}});
      const float value = a.v[3] * norm;
      if (value < best && inside(screen, start, extent, other) && inside(screen, start, extent, 2))
        best = value;
    };
    auto test_edge = [&](const F4& a, const F4& b) {
      const Ray r = closest_ray(a, b);
      if (r.squared_distance < best && inside(transform(g, r.position), start, extent, 2))
        best = r.squared_distance;
    };
    test_plane(ax, 1);
    test_plane(ay, 0);
    test_edge(ax, ay);
    test_edge(ax, plane(g, 1, y + h * 0.5f - dy));
    test_edge(plane(g, 0, x + w * 0.5f - dx), ay);
  }
  return 0.5f * best;
}

struct Entry {
  float depth;
  int id;
};

// render_adjoint.py:279-352 accumulate: gradients of one accepted sample
struct Grads {
  double* transforms;  // (n, 16), the reference's transposed layout
  double* opacity;     // (n)
  double* colors;      // (n, C)
  double* screen;      // (n, 2) or null
  double* screen_abs;  // (n, 2) or null
};

void atomic_add(double* p, float v) {
#pragma omp atomic
  *p += static_cast<double>(v);
}

void accumulate_ray_gradient(const Mat& g, float opacity, int id, float x, float y,
                             float gaussian, float alpha_gradient, const Grads& out) {
  const F4 a = plane(g, 0, x), b = plane(g, 1, y);
  const float nx[3] = {a.v[0], a.v[1], a.v[2]}, ny[3] = {b.v[0], b.v[1], b.v[2]};
  const float dx = a.v[3], dy = b.v[3];
  float moment[3], direction[3];
  for (int k = 0; k < 3; ++k) moment[k] = dx * ny[k] - dy * nx[k];
  direction[0] = nx[1] * ny[2] - nx[2] * ny[1];
  direction[1] = nx[2] * ny[0] - nx[0] * ny[2];
  direction[2] = nx[0] * ny[1] - nx[1] * ny[0];
  const float dd = dot3(direction, direction), mm = dot3(moment, moment);
  const float xx = dot3(nx, nx), yy = dot3(ny, ny), xy = dot3(nx, ny);
  const float ym = dot3(ny, moment), xm = dot3(nx, moment);
  float dd0[3], dd1[3], dd3[3], dm0[3], dm1[3], dm3[3];
  const float xyy = x * yy, yxx = y * xx, ndy = -dy, cross = dy * x - dx * y;
  for (int k = 0; k < 3; ++k) {
    dd0[k] = yy * nx[k] - xy * ny[k];
    dd1[k] = xx * ny[k] - xy * nx[k];
    dd3[k] = (xy * (y * nx[k] + x * ny[k]) - xyy * nx[k]) - yxx * ny[k];
    dm0[k] = ndy * moment[k];
    dm1[k] = dx * moment[k];
    dm3[k] = cross * moment[k];
  }
  const float factor = opacity * alpha_gradient * gaussian;
  const float inverse_dd = 1.0f / dd;
  const float ratio = mm / dd * inverse_dd;
  float screen_x = 0.0f, screen_y = 0.0f;
  double* t = out.transforms + 16ll * id;
  for (int axis = 0; axis < 3; ++axis) {
    const float d0 = factor * (ratio * dd0[axis] - dm0[axis] * inverse_dd);
    const float d1 = factor * (ratio * dd1[axis] - dm1[axis] * inverse_dd);
    const float d3 = factor * (ratio * dd3[axis] - dm3[axis] * inverse_dd);
    screen_x += d0 * g.m[3][axis];
    screen_y += d1 * g.m[3][axis];
    atomic_add(t + axis * 4, d0);
    atomic_add(t + axis * 4 + 1, d1);
    atomic_add(t + axis * 4 + 3, d3);
  }
  const float tr0 = factor * -ym * inverse_dd;
  const float tr1 = factor * -(-xm) * inverse_dd;
  const float tr3 = factor * -(y * xm - x * ym) * inverse_dd;
  atomic_add(t + 12, tr0);
  atomic_add(t + 13, tr1);
  atomic_add(t + 15, tr3);
  atomic_add(out.opacity + id, gaussian * alpha_gradient);
  if (out.screen) {
    screen_x += tr0 * g.m[3][3];
    screen_y += tr1 * g.m[3][3];
    atomic_add(out.screen + 2ll * id, screen_x);
    atomic_add(out.screen + 2ll * id + 1, screen_y);
    if (out.screen_abs) {
      atomic_add(out.screen_abs + 2ll * id, std::fabs(screen_x));
      atomic_add(out.screen_abs + 2ll * id + 1, std::fabs(screen_y));
    }
  }
}

struct Scene {
  int width, height, channels;
  const int* ranges;
  const int* points;
  const float* transforms;
  const float* opacity;
  const float* colors;
  const float* bg;
  bool cull;
  // replay backward only
  const float* image;       // (C, H, W) forward output
  const float* final_t;     // (H, W)
  const float* pixel_grad;  // (C, H, W)
  Grads grads;
  // forward contribution statistics (statistics.py:47-73), or stat_count 0
  int stat_count, stat_sum_mask;
  const float* stat_pixels;  // (stat_count, H*W)
  int* stat_counts;          // (masked counts, n)
  double* stat_sums;         // (weighted sums, n)
  int n;
};

// statistics.py:57-73 observe: a blended sample with weight w = alpha * T
// adds 1 (masked count) or map * w (weighted sum) to its Gaussian wherever
// the pixel's map value is nonzero
void observe(const Scene& s, int id, int pixel, float w) {
  const long long P = static_cast<long long>(s.width) * s.height;
  int count_row = 0, sum_row = 0;
  for (int r = 0; r < s.stat_count; ++r) {
    const float v = s.stat_pixels[r * P + pixel];
    if ((s.stat_sum_mask >> r) & 1) {
      if (v != 0.0f) atomic_add(s.stat_sums + static_cast<long long>(sum_row) * s.n + id, v * w);
      ++sum_row;
    } else {
      if (v != 0.0f) {
#pragma omp atomic
        s.stat_counts[static_cast<long long>(count_row) * s.n + id] += 1;
      }
      ++count_row;
    }
  }
}

struct Pixel {
  bool active;
  float transmittance;
  float color[kMaxChannels];
  int contributors;
  int tail_count, mid_count, head_count;
  float head_depth[4], head_alpha[4], head_gauss[4];
  int head_id[4];
  int x, y;
  // backward
  float gradient[kMaxChannels], final_color[kMaxChannels];
  float final_transmittance, background_gradient;
};

// One warp of one tile: lanes 0-15 own the 4x4 region `tail0`, lanes 16-31
// the region tail0 + 1; lane l's quad is its 4-lane group (mid queue).
class WarpReplay {
 public:
  WarpReplay(const Scene& s, int tile, int warp, bool backward)
      : s_(s), backward_(backward), warp_(warp) {
    const int gx = (s.width + 15) / 16;
    tile_x_ = tile % gx * 16;
    tile_y_ = tile / gx * 16;
    first_ = s.ranges[2 * tile];
    last_ = s.ranges[2 * tile + 1];
    for (int l = 0; l < 32; ++l) {
      Pixel& p = px_[l];
      std::memset(&p, 0, sizeof(p));
      const int local = warp * 32 + l, tail = local / 16, hl = l % 16, mg = hl / 4, mr = l % 4;
      x0_[l] = tile_x_ + 4 * (tail % 4);
      y0_[l] = tile_y_ + 4 * (tail / 4);
      p.x = x0_[l] + 2 * (mg & 1) + (mr & 1);
      p.y = y0_[l] + 2 * (mg / 2) + (mr / 2);
      p.active = p.x < s.width && p.y < s.height;
      p.transmittance = 1.0f;
      for (int k = 0; k < 4; ++k) {
        p.head_depth[k] = kInf;
        p.head_id[k] = -1;
      }
      if (backward_ && p.active) {
        const long long idx = static_cast<long long>(p.y) * s.width + p.x;
        const long long plane_size = static_cast<long long>(s.width) * s.height;
        p.final_transmittance = s.final_t[idx];
        for (int c = 0; c < s.channels; ++c) {
          p.gradient[c] = s.pixel_grad[c * plane_size + idx];
          p.final_color[c] = s.image[c * plane_size + idx] - p.final_transmittance * s.bg[c];
          p.background_gradient += s.bg[c] * p.gradient[c];
        }
      }
    }
    for (auto& q : tail_)
      for (auto& e : q) e = Entry{0.0f, 0};
    for (auto& q : mid_)
      for (auto& e : q) e = Entry{0.0f, 0};
  }

  void run();
  void write_forward(float* image, float* final_t, int* contributors) const;

 private:
  bool any_active(int lo, int hi) const {
    for (int l = lo; l < hi; ++l)
      if (px_[l].active) return true;
    return false;
  }
  Mat transform_of(int id) const { return load_transform(s_.transforms, id); }
  float opacity_of(int id) const { return id >= 0 ? s_.opacity[id] : 0.0f; }

  void blend(int l);
  void insert_head(int l, float depth, float alpha, int id, float gaussian);
  void merge(Entry* q, int n, int old_offset, const Entry* incoming);
  void sort_batch(Entry* q);
  void front_mid(int half, bool check_valid);
  void push_mid(int half, bool check_valid);

  const Scene& s_;
  bool backward_;
  int warp_;
  int tile_x_, tile_y_, first_, last_;
  int x0_[32], y0_[32];
  Pixel px_[32];
  Entry tail_[2][64];
  Entry mid_[8][8];
};

// render_hierarchical_warp.py:146-171 blend_step (forward) and
// backward_render.py:32-70 blend_backward (replay): the head's front sample.
void WarpReplay::blend(int l) {
  Pixel& p = px_[l];
  p.head_count -= 1;
  if (!p.active) return;
  const float alpha = p.head_alpha[0];
  const float next_t = p.transmittance * (1.0f - alpha);
  if (next_t < 0.0001f) {
    p.active = false;  // the sample that would terminate is not blended
    return;
  }
  const int id = p.head_id[0];
  const int C = s_.channels;
  const float* rgb = id >= 0 ? s_.colors + static_cast<long long>(id) * C : nullptr;
  if (!backward_) {
    for (int c = 0; c < C; ++c) p.color[c] = p.color[c] + (rgb ? rgb[c] : 0.0f) * alpha * p.transmittance;
    if (s_.stat_count && id >= 0) observe(s_, id, p.y * s_.width + p.x, alpha * p.transmittance);
  } else {
    float alpha_gradient = 0.0f;
    const float weight = alpha * p.transmittance;
    for (int c = 0; c < C; ++c) {
      const float v = rgb ? rgb[c] : 0.0f;
      p.color[c] = p.color[c] + v * alpha * p.transmittance;
      const float behind = (p.final_color[c] - p.color[c]) / next_t;
      alpha_gradient += (v - behind) * p.gradient[c];
      if (id >= 0) atomic_add(s_.grads.colors + static_cast<long long>(id) * C + c, weight * p.gradient[c]);
    }
    alpha_gradient *= p.transmittance;
    alpha_gradient += (-p.final_transmittance / (1.0f - alpha)) * p.background_gradient;
    if (id >= 0)
      accumulate_ray_gradient(transform_of(id), s_.opacity[id], id, static_cast<float>(p.x),
                              static_cast<float>(p.y), p.head_gauss[0], alpha_gradient, s_.grads);
  }
  p.transmittance = next_t;
  for (int j = 1; j < 4; ++j) {
    p.head_depth[j - 1] = p.head_depth[j];
    p.head_alpha[j - 1] = p.head_alpha[j];
    p.head_id[j - 1] = p.head_id[j];
    if (backward_) p.head_gauss[j - 1] = p.head_gauss[j];
  }
  p.head_depth[3] = kInf;
}

// :221-238 insert_head: strict comparison keeps equal-depth entries first
void WarpReplay::insert_head(int l, float depth, float alpha, int id, float gaussian) {
  Pixel& p = px_[l];
  for (int k = 0; k < 4; ++k) {
    if (depth < p.head_depth[k]) {
      std::swap(depth, p.head_depth[k]);
      std::swap(alpha, p.head_alpha[k]);
      std::swap(id, p.head_id[k]);
      std::swap(gaussian, p.head_gauss[k]);
    }
  }
  p.head_count += 1;
}

// :176-214 merge: the sorted n-entry run at q[old_offset..] and the sorted
// incoming run (lane r holds incoming[r]) into q[0..2n); equal old entries
// precede new ones.  Each lane's two binary searches, the temporary
// overwrite of the old run's depths by the incoming ones and the final
// scatter happen in the reference's barrier-separated phases.
void WarpReplay::merge(Entry* q, int n, int old_offset, const Entry* incoming) {
  int new_pos[32], old_pos[32];
  Entry old_entry[32];
  for (int r = 0; r < n; ++r) {
    const float depth = incoming[r].depth;
    int pos = 0;
    for (int stride = n / 2; stride > 0; stride /= 2)
      if (q[old_offset + pos + stride].depth <= depth) pos += stride;
    pos += 1;
    if (q[old_offset].depth > depth) pos = 0;
    new_pos[r] = pos + r;
    old_entry[r].depth = q[old_offset + r].depth;
  }
  for (int r = 0; r < n; ++r) q[old_offset + r].depth = incoming[r].depth;
  for (int r = 0; r < n; ++r) {
    const float depth = old_entry[r].depth;
    int pos = 0;
    for (int stride = n / 2; stride > 0; stride /= 2)
      if (q[old_offset + pos + stride].depth < depth) pos += stride;
    pos += 1;
    if (q[old_offset].depth >= depth) pos = 0;
    old_pos[r] = pos + r;
    old_entry[r].id = q[old_offset + r].id;
  }
  for (int r = 0; r < n; ++r) {
    q[new_pos[r]] = incoming[r];
    q[old_pos[r]] = old_entry[r];
  }
}

// :360-390 sort_batch: Batcher's network over the incoming run q[32..64),
// sixteen lanes, one compare-exchange each per step (the pairs of a step
// are disjoint)
void WarpReplay::sort_batch(Entry* q) {
  auto exchange = [&](int a, int b) {
    if (q[a].depth > q[b].depth) std::swap(q[a], q[b]);
  };
  for (int size = 2; size <= 32; size *= 2) {
    int stride = size / 2;
    for (int hl = 0; hl < 16; ++hl) {
      const int pos = 2 * hl - (hl & (stride - 1));
      exchange(32 + pos, 32 + pos + stride);
    }
    for (stride /= 2; stride > 0; stride /= 2) {
      for (int hl = 0; hl < 16; ++hl) {
        const int offset = hl & (size / 2 - 1);
        const int pos = 2 * hl - (hl & (stride - 1));
        if (offset >= stride) exchange(32 + pos - stride, 32 + pos);
      }
    }
  }
}

// :262-306 front_mid: each quad of half `half` consumes the front four
// entries of its mid queue, sampling them at each of its pixels
void WarpReplay::front_mid(int half, bool check_valid) {
  for (int quad = 4 * half; quad < 4 * half + 4; ++quad) {
    const int l0 = 4 * (quad % 8);
    if (!any_active(l0, l0 + 4)) continue;
    Entry* mq = mid_[quad];
    int load_id[4];
    float amplitude[4];
    for (int r = 0; r < 4; ++r) {
      load_id[r] = mq[r].id;
      amplitude[r] = 0.0f;
      if (!check_valid || load_id[r] != -1) amplitude[r] = opacity_of(load_id[r]);
    }
    for (int inner = 0; inner < 4; ++inner) {
      for (int l = l0; l < l0 + 4; ++l)
        if (px_[l].head_count >= 4) blend(l);
      const int id = mq[inner].id;
      if (check_valid && id == -1) continue;
      const int gid = load_id[inner];
      const float weight = amplitude[inner];
      for (int l = l0; l < l0 + 4; ++l) {
        Pixel& p = px_[l];
        if (!p.active) continue;
        p.contributors += 1;
        if (gid < 0) continue;  // guard (see the header)
        float power, depth;
        sample(transform_of(gid), static_cast<float>(p.x), static_cast<float>(p.y), &power,
               &depth);
        if (depth < -1.0f || depth > 1.0f) continue;
        const float gaussian = oracle_expf(power);
        const float alpha = min_of(0.99f, weight * gaussian);
        if (alpha < 1.0f / 255.0f) continue;
        insert_head(l, depth, alpha, id, gaussian);
      }
    }
  }
  for (int l = 16 * half; l < 16 * half + 16; ++l) px_[l].mid_count -= 4;
}

// :308-355 push_mid: sixteen tail entries of half `half`, four per batch,
// through the half's four quads (sampled at each quad's centre, ranked
// within the quad, merged with the quad's mid queue, front consumed)
void WarpReplay::push_mid(int half, bool check_valid) {
  Entry* tq = tail_[half];
  const int lane0 = 16 * half;
  for (int batch = 0; batch < 4; ++batch) {
    if (check_valid && px_[lane0].tail_count == 0) break;
    float depth[16];
    int id[16];
    for (int hl = 0; hl < 16; ++hl) {
      const int l = lane0 + hl, mr = l % 4, mg = hl / 4;
      const int source = 4 * batch + mr;
      id[hl] = tq[source].id;
      const int gid = id[hl];
      depth[hl] = kInf;
      if ((!check_valid || gid != -1) && gid >= 0) {
        float power;
        sample(transform_of(gid), static_cast<float>(x0_[l] + 1 + 2 * (mg & 1)),
               static_cast<float>(y0_[l] + 1 + 2 * (mg / 2)), &power, &depth[hl]);
      }
      if (check_valid && id[hl] == -1) depth[hl] = kInf;
    }
    for (int qd = 0; qd < 4; ++qd) {
      const int quad = 4 * half + qd;
      Entry* mq = mid_[quad];
      int rank[4];
      for (int r = 0; r < 4; ++r) {  // :243-252 rank_mid
        const float d = depth[4 * qd + r];
        int k = 0;
        for (int j = 1; j < 4; ++j) {
          const int other_rank = (r + j) % 4;
          const float other = depth[4 * qd + other_rank];
          if (other < d || (other == d && other_rank < r)) ++k;
        }
        rank[r] = k;
      }
      for (int r = 0; r < 4; ++r) mq[rank[r]] = Entry{depth[4 * qd + r], id[4 * qd + r]};
    }
    Entry incoming[8][4];
    for (int qd = 0; qd < 4; ++qd)
      for (int r = 0; r < 4; ++r) incoming[qd][r] = mid_[4 * half + qd][r];
    for (int l = lane0; l < lane0 + 16; ++l) px_[l].mid_count += 4;
    if (batch != 0 || px_[lane0].mid_count > 4) {
      for (int qd = 0; qd < 4; ++qd) merge(mid_[4 * half + qd], 4, 4, incoming[qd]);
      front_mid(half, false);
    } else {
      for (int qd = 0; qd < 4; ++qd)
        for (int r = 0; r < 4; ++r) mid_[4 * half + qd][4 + r] = incoming[qd][r];
    }
    if (check_valid)
      for (int l = lane0; l < lane0 + 16; ++l)
        px_[l].tail_count -= std::min(4, px_[l].tail_count);
  }
  if (!check_valid)
    for (int l = lane0; l < lane0 + 16; ++l) px_[l].tail_count -= 16;
}

// :410-594 render: the tile's sorted range in batches of 32, each culled
// and sampled at both 4x4 regions' centres, sorted, merged into the tails;
// tails beyond 32 entries drain sixteen at a time through the mids into the
// pixel heads; at the end everything drains.
void WarpReplay::run() {
  const int tail0 = 2 * warp_;
  for (int progress = first_; progress < last_; progress += 32) {
    if (!any_active(0, 32)) break;
    for (int l = 0; l < 32; ++l) {
      const int gid = progress + l < last_ ? s_.points[progress + l] : -1;
      Mat g{};
      float amplitude = 0.0f;
      if (gid >= 0) {
        g = transform_of(gid);
        if (s_.cull) amplitude = s_.opacity[gid];
      }
      int culled = 0;
      for (int half = 0; half < 2; ++half) {
        const int og = tail0 + half;
        if (s_.cull && gid != -1) {
          const float power = frustum(g, static_cast<float>(tile_x_ + 4 * (og & 3)),
                                      static_cast<float>(y0_[l]), 3.0f, 3.0f);
          if (min_of(0.99f, amplitude * oracle_expf(-power)) < 1.0f / 255.0f)
            culled |= 1 << half;
        }
      }
      for (int half = 0; half < 2; ++half) {
        const int og = tail0 + half;
        float depth = kInf;
        if (gid != -1 && (!s_.cull || !(culled & (1 << half)))) {
          float power;
          sample(g, static_cast<float>(tile_x_ + 4 * (og & 3) + 2),
                 static_cast<float>(y0_[l] + 2), &power, &depth);
        }
        tail_[half][32 + l] = Entry{depth, depth == kInf ? -1 : gid};
      }
    }
    for (int half = 0; half < 2; ++half) sort_batch(tail_[half]);
    for (int half = 0; half < 2; ++half) {
      Entry* q = tail_[half];
      const int old_count = px_[16 * half].tail_count;
      Entry incoming[32];
      int added = 0;
      for (int l = 0; l < 32; ++l) {
        incoming[l] = q[32 + l];
        if (incoming[l].id != -1) ++added;
      }
      for (int l = 16 * half; l < 16 * half + 16; ++l) px_[l].tail_count += added;
      if (old_count != 0) {
        merge(q, 32, 0, incoming);
      } else {
        for (int l = 0; l < 32; ++l) q[l] = incoming[l];
      }
    }
    for (int it = 0; it < 2; ++it) {
      for (int half = 0; half < 2; ++half) {
        if (px_[16 * half].tail_count <= 32) continue;
        push_mid(half, false);
        Entry* q = tail_[half];
        for (int hl = 0; hl < 16; ++hl)
          for (int index = 0; index < 3 - it; ++index) q[hl + index * 16] = q[hl + index * 16 + 16];
      }
    }
  }
  if (any_active(0, 32)) {
    for (int half = 0; half < 2; ++half) {
      if (px_[16 * half].tail_count == 0) continue;
      for (int it = 0; it < 2; ++it) {
        push_mid(half, true);
        if (it == 0 && px_[16 * half].tail_count == 0) break;
        if (it == 0) {
          Entry* q = tail_[half];
          for (int hl = 0; hl < 16; ++hl) q[hl] = q[hl + 16];
        }
      }
    }
    if (any_active(0, 32)) {
      for (int half = 0; half < 2; ++half) {
        if (px_[16 * half].mid_count == 0) continue;
        for (int qd = 0; qd < 4; ++qd) {
          Entry* mq = mid_[4 * half + qd];
          for (int r = 0; r < 4; ++r) mq[r] = mq[4 + r];
        }
        front_mid(half, true);
      }
      for (int l = 0; l < 32; ++l)
        while (px_[l].active && px_[l].head_count != 0) blend(l);
    }
  }
}

void WarpReplay::write_forward(float* image, float* final_t, int* contributors) const {
  const long long plane_size = static_cast<long long>(s_.width) * s_.height;
  for (int l = 0; l < 32; ++l) {
    const Pixel& p = px_[l];
    if (p.x >= s_.width || p.y >= s_.height) continue;
    const long long idx = static_cast<long long>(p.y) * s_.width + p.x;
    for (int c = 0; c < s_.channels; ++c)
      image[c * plane_size + idx] = p.color[c] + p.transmittance * s_.bg[c];
    final_t[idx] = p.transmittance;
    contributors[idx] = p.contributors;
  }
}

}  // namespace

extern "C" {

// aaa/render_hierarchical_warp.py:599-691 render (and render_statistics,
// :608-653) for one view: image (C, H, W) planar, final transmittance and
// evaluated-sample counts (H, W).  transforms (n, 4, 4) mathematical rows;
// colors (n, C); bg (C); ranges (T, 2); points the sorted ids.  With
// stat_count > 0 every blended sample is observed: request r (a
// (stat_count, H*W) map) is a weighted sum into stat_sums when bit r of
// stat_sum_mask is set, else a masked count into stat_counts (rows of n).
// Returns 0, or -1 if C is unsupported.
int oracle_aaa_render(int width, int height, int channels, const int* ranges, const int* points,
                      const float* transforms, const float* opacity, const float* colors,
                      const float* bg, int cull, float* image, float* final_t,
                      int* contributors, int n, int stat_count, int stat_sum_mask,
                      const float* stat_pixels, int* stat_counts, double* stat_sums) {
  if (channels < 1 || channels > kMaxChannels) return -1;
  Scene s{};
  s.n = n;
  s.stat_count = stat_count;
  s.stat_sum_mask = stat_sum_mask;
  s.stat_pixels = stat_pixels;
  s.stat_counts = stat_counts;
  s.stat_sums = stat_sums;
  s.width = width;
  s.height = height;
  s.channels = channels;
  s.ranges = ranges;
  s.points = points;
  s.transforms = transforms;
  s.opacity = opacity;
  s.colors = colors;
  s.bg = bg;
  s.cull = cull != 0;
  const int tiles = ((width + 15) / 16) * ((height + 15) / 16);
#pragma omp parallel for schedule(dynamic, 1)
  for (int unit = 0; unit < tiles * 8; ++unit) {
    WarpReplay w(s, unit / 8, unit % 8, false);
    w.run();
    w.write_forward(image, final_t, contributors);
  }
  return 0;
}

// aaa/backward_render.py:75-248 replay: gradients (float64 sums of the
// float32 per-sample terms) of the transforms (n, 16, the reference's
// transposed layout), opacities (n), colours (n, C) and, when non-null, the
// screen-translation statistics (n, 2) and their absolute sums (n, 2).
int oracle_aaa_render_backward(int width, int height, int channels, const int* ranges,
                               const int* points, const float* transforms,
                               const float* opacity, const float* colors, const float* bg,
                               int cull, const float* image, const float* final_t,
                               const float* pixel_grad, double* grad_transforms,
                               double* grad_opacity, double* grad_colors, double* grad_screen,
                               double* grad_screen_abs) {
  if (channels < 1 || channels > kMaxChannels) return -1;
  Scene s{};
  s.width = width;
  s.height = height;
  s.channels = channels;
  s.ranges = ranges;
  s.points = points;
  s.transforms = transforms;
  s.opacity = opacity;
  s.colors = colors;
  s.bg = bg;
  s.cull = cull != 0;
  s.image = image;
  s.final_t = final_t;
  s.pixel_grad = pixel_grad;
  s.grads = Grads{grad_transforms, grad_opacity, grad_colors, grad_screen, grad_screen_abs};
  const int tiles = ((width + 15) / 16) * ((height + 15) / 16);
#pragma omp parallel for schedule(dynamic, 1)
  for (int unit = 0; unit < tiles * 8; ++unit) {
    WarpReplay w(s, unit / 8, unit % 8, true);
    w.run();
  }
  return 0;
}

}  // extern "C"
