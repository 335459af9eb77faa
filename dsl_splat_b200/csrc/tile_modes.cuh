// tile_mode footprints: splatting/intersections.py:21-218.
//   0 radius   -- the tile_bounds square of the projection radius;
//   1 snugbox  -- that square clipped to the bounding box of the opacity-aware
//                 ellipse {power >= log(1/(255 o))}, widened for rounding;
//   2 accutile -- per-strip spans of that ellipse, strips along the shorter
//                 side of the box.
// Every step is the reference's float32 (and float64 for the determinant)
// operation sequence, with splat_logf for wp.log, so tile counts and the
// emitted tile sets agree bit for bit with the CPU oracle.
#pragma once
#include "splat_common.cuh"

namespace splat {

constexpr int kTileRadius = 0, kTileSnugbox = 1, kTileAccutile = 2;

struct TileFootprint {
  float cx, cy, a, b, c;
  int4 bounds;  // x0, y0, x1, y1
  bool precise;
  float level, det, ex, ey;
};

// intersections.py:45-108 footprint
SPLAT_DEV TileFootprint tile_footprint(float cx, float cy, float4 conic, int radius, int gx,
                                       int gy) {
  TileFootprint e;
  e.cx = cx;
  e.cy = cy;
  e.a = conic.x;
  e.b = conic.y;
  e.c = conic.z;
  e.precise = false;
  e.level = e.det = e.ex = e.ey = 0.0f;
  e.bounds = tile_bounds(cx, cy, radius, gx, gy);
  const float a = conic.x, b = conic.y, c = conic.z;
  const float det = __double2float_rn(__dsub_rn(__dmul_rn(static_cast<double>(a), c),
                                                __dmul_rn(static_cast<double>(b), b)));
  if (conic.w < __fdiv_rn(1.0f, 255.0f)) {
    e.bounds = make_int4(0, 0, 0, 0);
    return e;
  }
  if (!(a > 0.0f && c > 0.0f && det > 0.0f)) return e;  // keep the conservative square
  const float level = __fmul_rn(2.0f, splat_logf(__fmul_rn(conic.w, 255.0f)));
  const float reach = __fadd_rn(static_cast<float>(radius), 32.0f);
  float t = __fadd_rn(__fadd_rn(a, __fmul_rn(2.0f, fabsf(b))), c);
  t = __fmul_rn(__fmul_rn(t, reach), reach);
  t = __fadd_rn(__fadd_rn(t, fabsf(level)), 1.0f);
  const float roundoff = __fmul_rn(__fmul_rn(8.0f, 1.1920928955078125e-7f), t);
  e.level = __fadd_rn(wmax(0.0f, level), roundoff);
  e.det = det;
  e.ex = __fsqrt_rn(__fdiv_rn(__fmul_rn(e.level, c), det));
  e.ey = __fsqrt_rn(__fdiv_rn(__fmul_rn(e.level, a), det));
  if (!(isfinite(e.ex) && isfinite(e.ey))) return e;
  const float fgx = static_cast<float>(gx), fgy = static_cast<float>(gy);
  const int lo_x = f2i(wclamp(floorf(__fdiv_rn(__fsub_rn(cx, e.ex), 16.0f)), 0.0f, fgx));
  const int lo_y = f2i(wclamp(floorf(__fdiv_rn(__fsub_rn(cy, e.ey), 16.0f)), 0.0f, fgy));
  const int hi_x =
      f2i(wclamp(__fadd_rn(floorf(__fdiv_rn(__fadd_rn(cx, e.ex), 16.0f)), 1.0f), 0.0f, fgx));
  const int hi_y =
      f2i(wclamp(__fadd_rn(floorf(__fdiv_rn(__fadd_rn(cy, e.ey), 16.0f)), 1.0f), 0.0f, fgy));
  e.bounds = make_int4(max(e.bounds.x, lo_x), max(e.bounds.y, lo_y), min(e.bounds.z, hi_x),
                       min(e.bounds.w, hi_y));
  e.precise = true;
  return e;
}

// intersections.py:117-128: the ellipse's v-range on the grid line u = line*16
// (u = y for row strips, x for column strips).
SPLAT_DEV float2 line_intersection(const TileFootprint& e, int line, bool is_y) {
  const float u = is_y ? e.cy : e.cx, v = is_y ? e.cx : e.cy;
  const float c = is_y ? e.a : e.c, extent_u = is_y ? e.ey : e.ex;
  const float h = wclamp(__fsub_rn(static_cast<float>(line * 16), u), -extent_u, extent_u);
  const float root =
      __fsqrt_rn(wmax(0.0f, __fsub_rn(__fmul_rn(e.level, c), __fmul_rn(__fmul_rn(e.det, h), h))));
  const float bh = __fmul_rn(-e.b, h);
  return make_float2(__fadd_rn(v, __fdiv_rn(__fsub_rn(bh, root), c)),
                     __fadd_rn(v, __fdiv_rn(__fadd_rn(bh, root), c)));
}

// intersections.py:131-152: tile span of strip `row` from the ranges on its
// boundary lines and the ellipse's extrema inside the strip.
SPLAT_DEV int2 strip_span(const TileFootprint& e, int row, bool is_y, float2 low, float2 high) {
  const float u = is_y ? e.cy : e.cx, v = is_y ? e.cx : e.cy;
  const float a = is_y ? e.c : e.a, extent = is_y ? e.ex : e.ey;
  const int lower = is_y ? e.bounds.x : e.bounds.y, upper = is_y ? e.bounds.z : e.bounds.w;
  float lo = wmin(low.x, high.x), hi = wmax(low.y, high.y);
  const float arg_min = __fdiv_rn(__fmul_rn(e.b, extent), a);
  const float arg_max = __fdiv_rn(__fmul_rn(-e.b, extent), a);
  const float h0 = __fsub_rn(static_cast<float>(row * 16), u);
  const float h1 = __fsub_rn(static_cast<float>((row + 1) * 16), u);
  if (h0 <= arg_min && arg_min <= h1) lo = __fsub_rn(v, extent);
  if (h0 <= arg_max && arg_max <= h1) hi = __fadd_rn(v, extent);
  const float fl = static_cast<float>(lower), fu = static_cast<float>(upper);
  return make_int2(f2i(wclamp(floorf(__fdiv_rn(lo, 16.0f)), fl, fu)),
                   f2i(wclamp(__fadd_rn(floorf(__fdiv_rn(hi, 16.0f)), 1.0f), fl, fu)));
}

// The tile set of one Gaussian for a tile mode: its bounding rectangle and,
// for accutile, the strip walk (intersections.py:155-218 visit).
struct TileVisit {
  TileFootprint e;
  bool is_y, strips;
  int start, end;  // strip range (rows when is_y, else columns)
};

SPLAT_DEV TileVisit tile_visit(int mode, float cx, float cy, float4 conic, int radius, int gx,
                               int gy) {
  TileVisit v;
  if (mode != kTileRadius) {
    v.e = tile_footprint(cx, cy, conic, radius, gx, gy);
  } else {
    v.e.bounds = tile_bounds(cx, cy, radius, gx, gy);
    v.e.precise = false;
  }
  const int4 b = v.e.bounds;
  const int nx = max(0, b.z - b.x), ny = max(0, b.w - b.y);
  v.is_y = mode == kTileAccutile ? ny < nx : true;
  v.strips = mode == kTileAccutile && v.e.precise;
  v.start = v.is_y ? b.y : b.x;
  v.end = (nx == 0 || ny == 0) ? v.start : (v.is_y ? b.w : b.z);
  return v;
}

// Walks the strips, calling strip(row, span) for each (span in tiles along
// the strip); returns the number of tiles.
template <class Strip>
SPLAT_DEV int walk_strips(const TileVisit& v, Strip&& strip) {
  const int4 b = v.e.bounds;
  float2 low = make_float2(0.0f, 0.0f);
  if (v.strips && v.start < v.end) low = line_intersection(v.e, v.start, v.is_y);
  int count = 0;
  for (int row = v.start; row < v.end; ++row) {
    int2 span = v.is_y ? make_int2(b.x, b.z) : make_int2(b.y, b.w);
    if (v.strips) {
      const float2 high = line_intersection(v.e, row + 1, v.is_y);
      span = strip_span(v.e, row, v.is_y, low, high);
      low = high;
    }
    if (span.y > span.x) {
      strip(row, span);
      count += span.y - span.x;
    }
  }
  return count;
}

// Tile count of one Gaussian (the projection's tiles[i] for modes 1 and 2).
SPLAT_DEV int tile_count(const TileVisit& v) {
  if (!v.strips) {
    const int4 b = v.e.bounds;
    return max(0, b.z - b.x) * max(0, b.w - b.y);
  }
  return walk_strips(v, [](int, int2) {});
}

}  // namespace splat
