// splat_oracle.cpp -- TEST INFRASTRUCTURE ONLY.
//
// A CPU restatement of dsl_splat's original-3DGS (gs3d) rasteriser and of its
// RaDe-GS projection and render (rade/projection.py, rade/render.py), used as
// the parity checker for the CUDA path and as the timed CPU baseline.  Only
// tests/, __graft_entry__.smoke() and bench.py's CPU legs may load it; the
// product path (dsl_splat_b200) never does.
//
// Each function cites the reference file:line it restates (paths inside the
// dsl_splat project).  Arithmetic follows the reference expression by
// expression, in float32 with FP contraction disabled (this file is compiled
// with -ffp-contract=off); explicit fmaf() appears exactly where the
// reference calls fmaf / fused_multiply_add.  exp() in the blend is the
// shared Cody-Waite + Taylor exp described at splat_expf below, so that the
// CPU and GPU make the same alpha-threshold decisions.
//
// Parity status: pinned against golden vectors produced by running the
// reference's own gs3d kernel source (projection, SH, duplicate, ranges,
// render forward/backward) on the CPU through a Warp-API stand-in
// (tests/golden/make_golden.py).  Warp itself is not installable here, so
// the pin covers the reference's kernel logic evaluated in IEEE float32
// without FP contraction, not Warp's CUDA code generation.

#include <algorithm>
#include <cmath>
#include <cstdint>
#include <cstring>
#include <vector>
#ifdef _OPENMP
#include <omp.h>
#endif

namespace {

// A Python float literal inside a Warp kernel becomes float32 by rounding the
// double value; W32 reproduces that conversion.
#define W32(x) static_cast<float>(x)

// ---- scalar helpers with Warp / CUDA semantics --------------------------

inline float wmax(float a, float b) { return a > b ? a : b; }
inline float wmin(float a, float b) { return a < b ? a : b; }
inline float wclamp(float x, float a, float b) { return wmin(wmax(a, x), b); }
inline int iclamp(int x, int a, int b) { return std::min(std::max(a, x), b); }

// float -> int32 truncation with CUDA cvt.rzi.s32.f32 saturation (NaN -> 0).
inline int f2i(float x) {
  if (x != x) return 0;
  if (x >= 2147483648.0f) return INT32_MAX;
  if (x <= -2147483648.0f) return INT32_MIN;
  return static_cast<int>(x);
}

inline uint32_t float_bits(float v) {
  uint32_t u;
  std::memcpy(&u, &v, 4);
  return u;
}

inline float bits_float(uint32_t u) {
  float v;
  std::memcpy(&v, &u, 4);
  return v;
}

// exp(x) by Cody-Waite argument reduction (x = n ln2 + r, ln2 split into a
// 9-bit high part and a correction) followed by the degree-7 Taylor series of
// exp(r) in Horner form with fused multiply-adds, then scaling by 2^n
// through the exponent field.  Every step is an IEEE float32 operation, so
// the CUDA kernels (dsl_splat_b200/csrc/splat_common.cuh) produce identical
// bits.  Inputs below -80 return 0 (their alpha is far below 1/255).
float splat_expf(float x) {
  if (!(x > -80.0f)) return 0.0f;
  if (x > 88.0f) x = 88.0f;
  const float n = std::rint(x * 1.44269504088896341f);
  float r = std::fmaf(n, -0.693359375f, x);
  r = std::fmaf(n, 2.12194440054690583e-4f, r);
  float p = 1.98412698e-4f;               // 1/5040
  p = std::fmaf(p, r, 1.38888889e-3f);    // 1/720
  p = std::fmaf(p, r, 8.33333377e-3f);    // 1/120
  p = std::fmaf(p, r, 4.16666679e-2f);    // 1/24
  p = std::fmaf(p, r, 1.66666672e-1f);    // 1/6
  p = std::fmaf(p, r, 0.5f);
  p = std::fmaf(p, r, 1.0f);
  p = std::fmaf(p, r, 1.0f);
  const float scale = bits_float(static_cast<uint32_t>(static_cast<int>(n) + 127) << 23);
  return p * scale;
}

// log(x) for the tile-mode footprints (splatting/intersections.py:60, whose
// wp.log is the device logf): x = 2^k m with m in [sqrt(1/2), sqrt(2)),
// s = (m-1)/(m+1) computed as f/(2+f), log m = 2 atanh(s) summed as
// 2s (1 + s^2/3 + s^4/5 + s^6/7 + s^8/9) (|s| <= 0.1716, truncation below
// 2^-27 relative), k ln2 added with ln2 split into 0.693359375 and a
// correction.  Every step is one IEEE float32 operation, so the CUDA kernels
// (splat_common.cuh) produce identical bits.  +inf -> +inf, x <= 0 or NaN ->
// NaN / -inf as logf.
float splat_logf(float x) {
  if (!(x > 0.0f)) return x == 0.0f ? -INFINITY : NAN;
  if (x == INFINITY) return x;
  uint32_t u = float_bits(x);
  int k = 0;
  if (u < 0x00800000u) {  // subnormal: scale into the normal range
    x = x * 8388608.0f;   // 2^23, exact
    u = float_bits(x);
    k = -23;
  }
  k += static_cast<int>(u >> 23) - 127;
  float m = bits_float((u & 0x007FFFFFu) | 0x3F800000u);  // [1, 2)
  if (m > 1.41421356f) {
    m = m * 0.5f;  // exact
    k += 1;
  }
  const float f = m - 1.0f;  // exact (Sterbenz)
  const float s = f / (2.0f + f);
  const float z = s * s;
  float p = static_cast<float>(1.0 / 9.0);
  p = std::fmaf(p, z, static_cast<float>(1.0 / 7.0));
  p = std::fmaf(p, z, static_cast<float>(1.0 / 5.0));
  p = std::fmaf(p, z, static_cast<float>(1.0 / 3.0));
  p = std::fmaf(p, z, 1.0f);
  const float log_m = (2.0f * s) * p;
  const float kf = static_cast<float>(k);
  return kf * 0.693359375f + std::fmaf(kf, -2.12194440054690583e-4f, log_m);
}

// ---- GLM-order geometry (splatting/math.py, primitives/math.py) --------

// splatting/math.py:31-42 reference_matmul
void ref_matmul(const float a[3][3], const float b[3][3], float out[3][3]) {
  float r[3][3];
  for (int row = 0; row < 3; ++row)
    for (int col = 0; col < 3; ++col)
      r[row][col] = std::fmaf(a[row][2], b[2][col],
                              std::fmaf(a[row][0], b[0][col], a[row][1] * b[1][col]));
  std::memcpy(out, r, sizeof(r));
}

void transpose3(const float a[3][3], float out[3][3]) {
  float r[3][3];
  for (int i = 0; i < 3; ++i)
    for (int j = 0; j < 3; ++j) r[i][j] = a[j][i];
  std::memcpy(out, r, sizeof(r));
}

// splatting/math.py:44-47 point_row
inline float point_row(const float* m, int row, const float p[3]) {
  const float xy = std::fmaf(m[row * 4 + 0], p[0], m[row * 4 + 1] * p[1]);
  return std::fmaf(m[row * 4 + 2], p[2], xy) + m[row * 4 + 3];
}

// primitives/math.py:33-45 glm_rotation
void glm_rotation(const float q[4], float R[3][3]) {
  const float r = q[0], x = q[1], y = q[2], z = q[3];
  const float yy = y * y, zz = z * z;
  const float rz = r * z, xz = x * z, rx = r * x;
  const float d0 = yy + zz, d1 = std::fmaf(x, x, zz), d2 = std::fmaf(x, x, yy);
  R[0][0] = 1.0f - (d0 + d0);
  R[0][1] = 2.0f * std::fmaf(x, y, rz);
  R[0][2] = 2.0f * std::fmaf(-r, y, xz);
  R[1][0] = 2.0f * std::fmaf(x, y, -rz);
  R[1][1] = 1.0f - (d1 + d1);
  R[1][2] = 2.0f * std::fmaf(y, z, rx);
  R[2][0] = 2.0f * std::fmaf(r, y, xz);
  R[2][1] = 2.0f * std::fmaf(y, z, -rx);
  R[2][2] = 1.0f - (d2 + d2);
}

// gs3d/projection.py:37-86 screen_covariance (clamp_point from
// splatting/geometry.py:33-39).  Returns (a, b, c) of the dilated 2D
// covariance; b is GLM's cov[0][1] = projected[1][0].
void screen_covariance(const float pos[3], const float q[4], const float s[3],
                       const float* view, int width, int height, float fx, float fy,
                       float out[3]) {
  const float limx = W32(1.3) * static_cast<float>(width) / (2.0f * fx);
  const float limy = W32(1.3) * static_cast<float>(height) / (2.0f * fy);
  const float tx = wclamp(pos[0] / pos[2], -limx, limx) * pos[2];
  const float ty = wclamp(pos[1] / pos[2], -limy, limy) * pos[2];
  const float tz = pos[2];
  float R[3][3];
  glm_rotation(q, R);
  const float S[3][3] = {{s[0], 0.0f, 0.0f}, {0.0f, s[1], 0.0f}, {0.0f, 0.0f, s[2]}};
  float M[3][3], Mt[3][3], cov[3][3];
  ref_matmul(S, R, M);
  transpose3(M, Mt);
  ref_matmul(Mt, M, cov);
  const float J[3][3] = {{fx / tz, 0.0f, 0.0f},
                         {0.0f, fy / tz, 0.0f},
                         {-(fx * tx) / (tz * tz), -(fy * ty) / (tz * tz), 0.0f}};
  const float cam[3][3] = {{view[0], view[4], view[8]},
                           {view[1], view[5], view[9]},
                           {view[2], view[6], view[10]}};
  float T[3][3], Tt[3][3], covt[3][3], tmp[3][3], P[3][3];
  ref_matmul(cam, J, T);
  transpose3(T, Tt);
  transpose3(cov, covt);
  ref_matmul(Tt, covt, tmp);
  ref_matmul(tmp, T, P);
  out[0] = P[0][0] + W32(0.3);
  out[1] = P[1][0];
  out[2] = P[1][1] + W32(0.3);
}

// splatting/geometry.py:106-123 pixel_center
void pixel_center(const float mean[3], const float* proj, int width, int height,
                  float out[2]) {
  const float c0 = point_row(proj, 0, mean);
  const float c1 = point_row(proj, 1, mean);
  const float c3 = point_row(proj, 3, mean);
  const float inverse_w = 1.0f / (c3 + W32(1e-7));
  const double ndc_x = static_cast<double>(c0 * inverse_w);
  const double ndc_y = static_cast<double>(c1 * inverse_w);
  out[0] = static_cast<float>(((ndc_x + 1.0) * static_cast<double>(width) - 1.0) * 0.5);
  out[1] = static_cast<float>(((ndc_y + 1.0) * static_cast<double>(height) - 1.0) * 0.5);
}

// splatting/geometry.py:22-30 tile_bounds (x0, y0, x1, y1)
void tile_bounds(const float center[2], int radius, int gx, int gy, int b[4]) {
  const float r = static_cast<float>(radius);
  b[0] = iclamp(f2i((center[0] - r) / 16.0f), 0, gx);
  b[1] = iclamp(f2i((center[1] - r) / 16.0f), 0, gy);
  b[2] = iclamp(f2i(((center[0] + r) + 16.0f - 1.0f) / 16.0f), 0, gx);
  b[3] = iclamp(f2i(((center[1] + r) + 16.0f - 1.0f) / 16.0f), 0, gy);
}

// ---- tile modes (splatting/intersections.py:21-218) ---------------------
// 0 radius (the tile_bounds square), 1 snugbox (square clipped to the
// opacity-aware ellipse box), 2 accutile (per-strip ellipse spans).

struct Footprint {
  float cx, cy, a, b, c;
  int bounds[4];
  bool precise;
  float level, det, ex, ey;
};

// intersections.py:45-108 footprint
Footprint footprint(const float center[2], const float conic[4], int radius, int gx, int gy) {
  Footprint e{};
  e.cx = center[0];
  e.cy = center[1];
  e.a = conic[0];
  e.b = conic[1];
  e.c = conic[2];
  e.precise = false;
  tile_bounds(center, radius, gx, gy, e.bounds);
  const float a = conic[0], b = conic[1], c = conic[2];
  const float det = static_cast<float>(static_cast<double>(a) * static_cast<double>(c) -
                                       static_cast<double>(b) * static_cast<double>(b));
  if (conic[3] < 1.0f / 255.0f) {
    e.bounds[0] = e.bounds[1] = e.bounds[2] = e.bounds[3] = 0;
    return e;
  }
  if (!(a > 0.0f && c > 0.0f && det > 0.0f)) return e;  // keep the conservative square
  const float level = 2.0f * splat_logf(conic[3] * 255.0f);
  const float reach = static_cast<float>(radius) + 32.0f;
  const float roundoff = (8.0f * 1.1920928955078125e-7f) *
                         ((((a + 2.0f * std::fabs(b)) + c) * reach * reach + std::fabs(level)) +
                          1.0f);
  e.level = wmax(0.0f, level) + roundoff;
  e.det = det;
  e.ex = std::sqrt(e.level * c / det);
  e.ey = std::sqrt(e.level * a / det);
  if (!(std::isfinite(e.ex) && std::isfinite(e.ey))) return e;
  const float fgx = static_cast<float>(gx), fgy = static_cast<float>(gy);
  const int lo_x = f2i(wclamp(std::floor((e.cx - e.ex) / 16.0f), 0.0f, fgx));
  const int lo_y = f2i(wclamp(std::floor((e.cy - e.ey) / 16.0f), 0.0f, fgy));
  const int hi_x = f2i(wclamp(std::floor((e.cx + e.ex) / 16.0f) + 1.0f, 0.0f, fgx));
  const int hi_y = f2i(wclamp(std::floor((e.cy + e.ey) / 16.0f) + 1.0f, 0.0f, fgy));
  e.bounds[0] = std::max(e.bounds[0], lo_x);
  e.bounds[1] = std::max(e.bounds[1], lo_y);
  e.bounds[2] = std::min(e.bounds[2], hi_x);
  e.bounds[3] = std::min(e.bounds[3], hi_y);
  e.precise = true;
  return e;
}

// intersections.py:117-128 line_intersection: the ellipse's v-range on the
// grid line u = line*16 (u = x for column strips, y for row strips).
void line_intersection(const Footprint& e, int line, bool is_y, float out[2]) {
  float u = e.cx, v = e.cy, c = e.c, extent_u = e.ex;
  const float b = e.b;
  if (is_y) {
    u = e.cy;
    v = e.cx;
    c = e.a;
    extent_u = e.ey;
  }
  const float h = wclamp(static_cast<float>(line * 16) - u, -extent_u, extent_u);
  const float root = std::sqrt(wmax(0.0f, e.level * c - e.det * h * h));
  out[0] = v + (-b * h - root) / c;
  out[1] = v + (-b * h + root) / c;
}

// intersections.py:131-152 strip_span: tile span of strip `row` from the
// ranges on its two boundary lines and the interior extrema.
void strip_span(const Footprint& e, int row, bool is_y, const float low[2], const float high[2],
                int out[2]) {
  float u = e.cx, v = e.cy, a = e.a, extent = e.ey;
  const float b = e.b;
  int lower = e.bounds[1], upper = e.bounds[3];
  if (is_y) {
    u = e.cy;
    v = e.cx;
    a = e.c;
    extent = e.ex;
    lower = e.bounds[0];
    upper = e.bounds[2];
  }
  float lo = wmin(low[0], high[0]), hi = wmax(low[1], high[1]);
  const float arg_min = b * extent / a, arg_max = -b * extent / a;
  const float h0 = static_cast<float>(row * 16) - u, h1 = static_cast<float>((row + 1) * 16) - u;
  if (h0 <= arg_min && arg_min <= h1) lo = v - extent;
  if (h0 <= arg_max && arg_max <= h1) hi = v + extent;
  out[0] = f2i(wclamp(std::floor(lo / 16.0f), static_cast<float>(lower), static_cast<float>(upper)));
  out[1] = f2i(wclamp(std::floor(hi / 16.0f) + 1.0f, static_cast<float>(lower),
                      static_cast<float>(upper)));
}

// intersections.py:155-218 visit: the tiles of one Gaussian in emission
// order (emit(tile)), returning their count.
template <class Emit>
int visit_tiles(int mode, const float center[2], const float conic[4], int radius, int gx, int gy,
                Emit&& emit) {
  Footprint e{};
  tile_bounds(center, radius, gx, gy, e.bounds);
  e.precise = false;
  if (mode != 0) e = footprint(center, conic, radius, gx, gy);
  const int* bd = e.bounds;
  const int nx = std::max(0, bd[2] - bd[0]), ny = std::max(0, bd[3] - bd[1]);
  if (nx == 0 || ny == 0) return 0;
  const bool is_y = mode == 2 ? ny < nx : true;
  const int start = is_y ? bd[1] : bd[0], end = is_y ? bd[3] : bd[2];
  const bool strips = mode == 2 && e.precise;
  float low[2] = {0.0f, 0.0f};
  if (strips) line_intersection(e, start, is_y, low);
  int count = 0;
  for (int row = start; row < end; ++row) {
    int span[2] = {is_y ? bd[0] : bd[1], is_y ? bd[2] : bd[3]};
    if (strips) {
      float high[2];
      line_intersection(e, row + 1, is_y, high);
      strip_span(e, row, is_y, low, high, span);
      low[0] = high[0];
      low[1] = high[1];
    }
    for (int col = span[0]; col < span[1]; ++col) emit(is_y ? row * gx + col : col * gx + row);
    count += std::max(0, span[1] - span[0]);
  }
  return count;
}

// ---- 4x4 inverse (Laplace expansion by 2x2 minors, Eberly 2008) --------
// Used for camera centres; the CUDA camera kernel performs the same steps.
bool inverse44(const float* m, float* inv, float* det_out) {
  const float a00 = m[0], a01 = m[1], a02 = m[2], a03 = m[3];
  const float a10 = m[4], a11 = m[5], a12 = m[6], a13 = m[7];
  const float a20 = m[8], a21 = m[9], a22 = m[10], a23 = m[11];
  const float a30 = m[12], a31 = m[13], a32 = m[14], a33 = m[15];
  const float s0 = a00 * a11 - a10 * a01;
  const float s1 = a00 * a12 - a10 * a02;
  const float s2 = a00 * a13 - a10 * a03;
  const float s3 = a01 * a12 - a11 * a02;
  const float s4 = a01 * a13 - a11 * a03;
  const float s5 = a02 * a13 - a12 * a03;
  const float c5 = a22 * a33 - a32 * a23;
  const float c4 = a21 * a33 - a31 * a23;
  const float c3 = a21 * a32 - a31 * a22;
  const float c2 = a20 * a33 - a30 * a23;
  const float c1 = a20 * a32 - a30 * a22;
  const float c0 = a20 * a31 - a30 * a21;
  const float det = s0 * c5 - s1 * c4 + s2 * c3 + s3 * c2 - s4 * c1 + s5 * c0;
  *det_out = det;
  if (det == 0.0f) return false;
  const float d = 1.0f / det;
  inv[0] = (a11 * c5 - a12 * c4 + a13 * c3) * d;
  inv[1] = (-a01 * c5 + a02 * c4 - a03 * c3) * d;
  inv[2] = (a31 * s5 - a32 * s4 + a33 * s3) * d;
  inv[3] = (-a21 * s5 + a22 * s4 - a23 * s3) * d;
  inv[4] = (-a10 * c5 + a12 * c2 - a13 * c1) * d;
  inv[5] = (a00 * c5 - a02 * c2 + a03 * c1) * d;
  inv[6] = (-a30 * s5 + a32 * s2 - a33 * s1) * d;
  inv[7] = (a20 * s5 - a22 * s2 + a23 * s1) * d;
  inv[8] = (a10 * c4 - a11 * c2 + a13 * c0) * d;
  inv[9] = (-a00 * c4 + a01 * c2 - a03 * c0) * d;
  inv[10] = (a30 * s4 - a31 * s2 + a33 * s0) * d;
  inv[11] = (-a20 * s4 + a21 * s2 - a23 * s0) * d;
  inv[12] = (-a10 * c3 + a11 * c1 - a12 * c0) * d;
  inv[13] = (a00 * c3 - a01 * c1 + a02 * c0) * d;
  inv[14] = (-a30 * s3 + a31 * s1 - a32 * s0) * d;
  inv[15] = (a20 * s3 - a21 * s1 + a22 * s0) * d;
  return true;
}

// ---- SH basis (primitives/sh.py:7-41) ----------------------------------

float sh_basis(const float d[3], int k) {
  const float x = d[0], y = d[1], z = d[2];
  switch (k) {
    case 0: return W32(0.28209479177387814);
    case 1: return -W32(0.4886025119029199) * y;
    case 2: return W32(0.4886025119029199) * z;
    case 3: return -W32(0.4886025119029199) * x;
    case 4: return W32(1.0925484305920792) * x * y;
    case 5: return -W32(1.0925484305920792) * y * z;
    case 6: return W32(0.31539156525252005) * (2.0f * z * z - x * x - y * y);
    case 7: return -W32(1.0925484305920792) * x * z;
    case 8: return W32(0.5462742152960396) * (x * x - y * y);
    case 9: return -W32(0.5900435899266435) * y * (3.0f * x * x - y * y);
    case 10: return W32(2.890611442640554) * x * y * z;
    case 11: return -W32(0.4570457994644658) * y * (4.0f * z * z - x * x - y * y);
    case 12: return W32(0.3731763325901154) * z * (2.0f * z * z - 3.0f * x * x - 3.0f * y * y);
    case 13: return -W32(0.4570457994644658) * x * (4.0f * z * z - x * x - y * y);
    case 14: return W32(1.445305721320277) * z * (x * x - y * y);
    default: return -W32(0.5900435899266435) * x * (x * x - 3.0f * y * y);
  }
}

// d basis_k / d unit, hand-differentiated from sh.py:7-41 (what Warp's
// wp.grad(basis) evaluates at sh.py:127).
void sh_basis_grad(const float d[3], int k, float g[3]) {
  const float x = d[0], y = d[1], z = d[2];
  const float c1 = W32(0.4886025119029199), c4 = W32(1.0925484305920792);
  const float c6 = W32(0.31539156525252005), c8 = W32(0.5462742152960396);
  const float c9 = -W32(0.5900435899266435), c10 = W32(2.890611442640554);
  const float c11 = -W32(0.4570457994644658), c12 = W32(0.3731763325901154);
  const float c14 = W32(1.445305721320277);
  g[0] = g[1] = g[2] = 0.0f;
  switch (k) {
    case 0: break;
    case 1: g[1] = -c1; break;
    case 2: g[2] = c1; break;
    case 3: g[0] = -c1; break;
    case 4: g[0] = c4 * y; g[1] = c4 * x; break;
    case 5: g[1] = -c4 * z; g[2] = -c4 * y; break;
    case 6: g[0] = -2.0f * c6 * x; g[1] = -2.0f * c6 * y; g[2] = 4.0f * c6 * z; break;
    case 7: g[0] = -c4 * z; g[2] = -c4 * x; break;
    case 8: g[0] = 2.0f * c8 * x; g[1] = -2.0f * c8 * y; break;
    case 9: g[0] = c9 * 6.0f * x * y; g[1] = c9 * (3.0f * x * x - 3.0f * y * y); break;
    case 10: g[0] = c10 * y * z; g[1] = c10 * x * z; g[2] = c10 * x * y; break;
    case 11:
      g[0] = c11 * (-2.0f * x * y);
      g[1] = c11 * (4.0f * z * z - x * x - 3.0f * y * y);
      g[2] = c11 * (8.0f * y * z);
      break;
    case 12:
      g[0] = c12 * (-6.0f * x * z);
      g[1] = c12 * (-6.0f * y * z);
      g[2] = c12 * (6.0f * z * z - 3.0f * x * x - 3.0f * y * y);
      break;
    case 13:
      g[0] = c11 * (4.0f * z * z - 3.0f * x * x - y * y);
      g[1] = c11 * (-2.0f * x * y);
      g[2] = c11 * (8.0f * x * z);
      break;
    case 14: g[0] = c14 * 2.0f * x * z; g[1] = -c14 * 2.0f * y * z; g[2] = c14 * (x * x - y * y); break;
    default:
      g[0] = c9 * (3.0f * x * x - 3.0f * y * y);
      g[1] = c9 * (-6.0f * x * y);
      break;
  }
}


// ---- RaDe-GS geometry (rade/projection.py) ------------------------------

// Row-wise matrix-vector product, each row summed left to right (Warp mat*vec).
void matvec3(const float m[3][3], const float v[3], float out[3]) {
  float r[3];
  for (int i = 0; i < 3; ++i) r[i] = m[i][0] * v[0] + m[i][1] * v[1] + m[i][2] * v[2];
  std::memcpy(out, r, sizeof(r));
}

// Warp's normalize: v / |v| per component, the zero vector when |v| == 0.
void normalize3(const float v[3], float out[3]) {
  const float l = std::sqrt(v[0] * v[0] + v[1] * v[1] + v[2] * v[2]);
  if (l > 0.0f) {
    out[0] = v[0] / l;
    out[1] = v[1] / l;
    out[2] = v[2] / l;
  } else {
    out[0] = out[1] = out[2] = 0.0f;
  }
}

struct RayGeometry {
  float cov[3];     // (a, b, c) of the undilated screen covariance
  float plane[3];   // ray plane (d/du, d/dv per pixel, distance at the centre)
  float normal[3];  // unit camera-space normal
};

// rade/projection.py:102-190 geometry, for the camera-space position t.
void rade_geometry(const float pos[3], const float q[4], const float s[3], const float* view,
                   int width, int height, float fx, float fy, RayGeometry& out) {
  // rade/projection.py:39-47 clamp_point
  const float limx = W32(1.3) * static_cast<float>(width) / (2.0f * fx);
  const float limy = W32(1.3) * static_cast<float>(height) / (2.0f * fy);
  const float t0 = wclamp(pos[0] / pos[2], -limx, limx) * pos[2];
  const float t1 = wclamp(pos[1] / pos[2], -limy, limy) * pos[2];
  const float z = pos[2];
  const float u = t0 / z, v = t1 / z;
  float R[3][3];
  glm_rotation(q, R);
  const float cam[3][3] = {{view[0], view[4], view[8]},
                           {view[1], view[5], view[9]},
                           {view[2], view[6], view[10]}};
  const float J[3][3] = {{fx / z, 0.0f, 0.0f},
                         {0.0f, fy / z, 0.0f},
                         {-fx * t0 / (z * z), -fy * t1 / (z * z), 0.0f}};
  float Tm[3][3];
  ref_matmul(cam, J, Tm);
  // rade/projection.py:87-92 raster_covariance
  const float S[3][3] = {{s[0], 0.0f, 0.0f}, {0.0f, s[1], 0.0f}, {0.0f, 0.0f, s[2]}};
  float SR[3][3], M[3][3], Mt[3][3], C[3][3];
  ref_matmul(S, R, SR);
  ref_matmul(SR, Tm, M);
  transpose3(M, Mt);
  ref_matmul(Mt, M, C);
  out.cov[0] = C[0][0];
  out.cov[1] = C[1][0];
  out.cov[2] = C[1][1];
  // smallest axis with find_min_from_triple's tie order
  const int bigger = s[0] < s[1] ? 1 : 0;
  const int i0 = (bigger + 1) % 3, i1 = (bigger + 2) % 3;
  const int minimum = s[i0] > s[i1] ? i1 : i0;
  float inv_cov[3][3];
  if (s[minimum] > W32(1.0e-7)) {
    const float Si[3][3] = {{1.0f / s[0], 0.0f, 0.0f},
                            {0.0f, 1.0f / s[1], 0.0f},
                            {0.0f, 0.0f, 1.0f / s[2]}};
    float SiR[3][3], Mi[3][3], Mit[3][3];
    ref_matmul(Si, R, SiR);
    ref_matmul(SiR, cam, Mi);
    transpose3(Mi, Mit);
    ref_matmul(Mit, Mi, inv_cov);
  } else {
    const float axis[3] = {R[minimum][0], R[minimum][1], R[minimum][2]};
    float camt[3][3], ac[3];
    transpose3(cam, camt);
    matvec3(camt, axis, ac);
    for (int i = 0; i < 3; ++i)
      for (int j = 0; j < 3; ++j) inv_cov[i][j] = ac[i] * ac[j];
  }
  const float uvh[3] = {u, v, 1.0f};
  float d[3], direction[3];
  matvec3(inv_cov, uvh, d);
  normalize3(d, direction);
  const float len_sq = direction[0] * direction[0] + direction[1] * direction[1] +
                       direction[2] * direction[2];
  if (len_sq == 0.0f || !std::isfinite(direction[0])) {
    out.plane[0] = out.plane[1] = out.plane[2] = 0.0f;
    out.normal[0] = out.normal[1] = 0.0f;
    out.normal[2] = -1.0f;
    return;
  }
  const float length = std::sqrt(t0 * t0 + t1 * t1 + z * z);
  const float factor = length / (u * u + v * v + 1.0f);
  const float nj_inv[3][3] = {{v * v + 1.0f, -u * v, -u}, {-u * v, u * u + 1.0f, -v},
                              {0.0f, 0.0f, 0.0f}};
  const float denom = wmax(direction[0] * u + direction[1] * v + direction[2] * 1.0f,
                           W32(1.0e-7));
  const float dd[3] = {direction[0] / denom, direction[1] / denom, direction[2] / denom};
  float plane[3];
  matvec3(nj_inv, dd, plane);
  out.plane[0] = plane[0] * factor / fx;
  out.plane[1] = plane[1] * factor / fy;
  out.plane[2] = std::sqrt(pos[0] * pos[0] + pos[1] * pos[1] + pos[2] * pos[2]);
  const float ray_normal[3] = {-plane[0] * factor, -plane[1] * factor, -1.0f};
  const float nj[3][3] = {{1.0f / z, 0.0f, t0 / length},
                          {0.0f, 1.0f / z, t1 / length},
                          {-t0 / (z * z), -t1 / (z * z), z / length}};
  float n[3];
  matvec3(nj, ray_normal, n);
  normalize3(n, out.normal);
}

// rade/projection.py:50-54 opacity_coefficient
float opacity_coefficient(const float cov[3], float kernel) {
  const float det0 = wmax(W32(1.0e-6), cov[0] * cov[2] - cov[1] * cov[1]);
  const float det1 =
      wmax(W32(1.0e-6), (cov[0] + kernel) * (cov[2] + kernel) - cov[1] * cov[1]);
  return std::sqrt(det0 / det1);
}

}  // namespace

extern "C" {

float oracle_expf(float x) { return splat_expf(x); }
float oracle_logf(float x) { return splat_logf(x); }

// splatting/camera_kernels.py:11-66 prepare_kernel.  Returns nonzero when any
// camera reports an error (codes in errors[]).
int oracle_cameras_prepare(int count, const float* views, const float* Ks, int width,
                           int height, int with_centers, float* full, float* inverse,
                           float* centers, int* errors) {
  int any = 0;
  for (int i = 0; i < count; ++i) {
    const float* K = Ks + 9 * i;
    const float* V = views + 16 * i;
    bool finite = true;
    for (int j = 0; j < 9; ++j) finite = finite && std::isfinite(K[j]);
    int error = 0;
    if (!finite || K[0] <= 0.0f || K[4] <= 0.0f)
      error = 2;
    else if (K[1] != 0.0f || K[3] != 0.0f || K[6] != 0.0f || K[7] != 0.0f || K[8] != 1.0f)
      error = 1;
    errors[i] = error;
    if (error) {
      any = 1;
      continue;
    }
    const float px = 2.0f * K[0] / static_cast<float>(width);
    const float py = 2.0f * K[4] / static_cast<float>(height);
    const float cx = 2.0f * K[2] / static_cast<float>(width) - 1.0f;
    const float cy = 2.0f * K[5] / static_cast<float>(height) - 1.0f;
    float* F = full + 16 * i;
    for (int col = 0; col < 4; ++col) {
      F[0 * 4 + col] = px * V[0 * 4 + col] + cx * V[2 * 4 + col];
      F[1 * 4 + col] = py * V[1 * 4 + col] + cy * V[2 * 4 + col];
      F[2 * 4 + col] = V[2 * 4 + col];
      F[3 * 4 + col] = V[2 * 4 + col];
    }
    if (with_centers) {
      float inv[16], det;
      if (!inverse44(V, inv, &det)) {
        errors[i] = 3;
        any = 1;
        continue;
      }
      std::memcpy(inverse + 16 * i, inv, sizeof(inv));
      for (int r = 0; r < 3; ++r) centers[3 * i + r] = inv[r * 4 + 3];
    }
  }
  return any;
}

// splatting/camera_kernels.py:69-106 backward_kernel
void oracle_cameras_backward(int count, const float* Ks, const float* grad_full, int width,
                             int height, const float* inverse, const float* grad_centers,
                             float* grad_views) {
  for (int i = 0; i < count; ++i) {
    const float* K = Ks + 9 * i;
    const float px = 2.0f * K[0] / static_cast<float>(width);
    const float py = 2.0f * K[4] / static_cast<float>(height);
    const float cx = 2.0f * K[2] / static_cast<float>(width) - 1.0f;
    const float cy = 2.0f * K[5] / static_cast<float>(height) - 1.0f;
    const float* g = grad_full ? grad_full + 16 * i : nullptr;
    const float* inv = inverse ? inverse + 16 * i : nullptr;
    const float* gc = grad_centers ? grad_centers + 3 * i : nullptr;
    for (int row = 0; row < 4; ++row)
      for (int col = 0; col < 4; ++col) {
        float value = 0.0f;
        if (g) {
          if (row == 0) value = px * g[0 * 4 + col];
          else if (row == 1) value = py * g[1 * 4 + col];
          else if (row == 2)
            value = (cx * g[0 * 4 + col] + cy * g[1 * 4 + col]) + g[2 * 4 + col] + g[3 * 4 + col];
        }
        if (gc) {
          float vjp = 0.0f;
          for (int k = 0; k < 3; ++k) vjp += inv[k * 4 + row] * gc[k];
          value -= vjp * inv[col * 4 + 3];
        }
        grad_views[16 * i + row * 4 + col] = value;
      }
  }
}

// gs3d/projection.py:89-164 project.  Culled rows keep radii = tiles = 0 and
// leave centers/conics/depths untouched.  tile_mode != 0 replaces the tile
// count with the mode's (:150-162); such a Gaussian keeps its radius even
// when the count is 0.
void oracle_project_forward(int n, const float* means, const float* quats, const float* scales,
                            const float* opacities, const float* view, const float* proj,
                            const float* K, int width, int height, float near_plane,
                            float far_plane, float radius_clip, float* centers, float* conics,
                            int* radii, int* tiles, float* depths, int tile_mode) {
  const int gx = (width + 15) / 16, gy = (height + 15) / 16;
  const float fx = K[0], fy = K[4];
#pragma omp parallel for schedule(static)
  for (int i = 0; i < n; ++i) {
    radii[i] = 0;
    tiles[i] = 0;
    const float* m = means + 3 * i;
    const float t[3] = {point_row(view, 0, m), point_row(view, 1, m), point_row(view, 2, m)};
    if (t[2] <= near_plane || t[2] >= far_plane) continue;
    float cov[3];
    screen_covariance(t, quats + 4 * i, scales + 3 * i, view, width, height, fx, fy, cov);
    const float a = cov[0], b = cov[1], c = cov[2];
    const float det = a * c - b * b;
    if (det == 0.0f) continue;
    const float mid = 0.5f * (a + c);
    const int radius = f2i(std::ceil(3.0f * std::sqrt(mid + std::sqrt(wmax(W32(0.1), mid * mid - det)))));
    if (static_cast<float>(radius) <= radius_clip) continue;
    float center[2];
    pixel_center(m, proj, width, height, center);
    int bnd[4];
    tile_bounds(center, radius, gx, gy, bnd);
    const int count = (bnd[2] - bnd[0]) * (bnd[3] - bnd[1]);
    if (count == 0) continue;
    const float inverse = 1.0f / (a * c - b * b);
    centers[2 * i] = center[0];
    centers[2 * i + 1] = center[1];
    conics[4 * i + 0] = c * inverse;
    conics[4 * i + 1] = -b * inverse;
    conics[4 * i + 2] = a * inverse;
    conics[4 * i + 3] = opacities[i];
    radii[i] = radius;
    tiles[i] = count;
    if (tile_mode != 0)
      tiles[i] = visit_tiles(tile_mode, center, conics + 4 * i, radius, gx, gy, [](int) {});
    depths[i] = t[2];
  }
}

// primitives/sh.py:44-79 forward kernel (masked when radii != null).
// coeffs: (n, K, 3) with K >= (degree+1)^2; dirs: (n, 3) = means - camera.
void oracle_sh_forward(int n, int degree, int K, const float* coeffs, const float* dirs,
                       const int* radii, float* colors, unsigned char* active) {
  const int count = (degree + 1) * (degree + 1);
#pragma omp parallel for schedule(static)
  for (int i = 0; i < n; ++i) {
    const bool visible = radii ? radii[i] > 0 : true;
    float value[3] = {0.0f, 0.0f, 0.0f};
    if (visible) {
      float unit[3] = {0.0f, 0.0f, 0.0f};
      if (degree > 0) {
        const float* d = dirs + 3 * i;
        const float len = std::sqrt(d[0] * d[0] + d[1] * d[1] + d[2] * d[2]);
        const float den = wmax(len, W32(1e-12));
        for (int j = 0; j < 3; ++j) unit[j] = d[j] / den;
      }
      for (int k = 0; k < count; ++k) {
        const float b = sh_basis(unit, k);
        for (int ch = 0; ch < 3; ++ch) value[ch] = value[ch] + b * coeffs[(i * K + k) * 3 + ch];
      }
      for (int ch = 0; ch < 3; ++ch) value[ch] = value[ch] + 0.5f;
    }
    for (int ch = 0; ch < 3; ++ch) {
      colors[3 * i + ch] = wmax(value[ch], 0.0f);
      if (active) active[3 * i + ch] = (visible && value[ch] >= 0.0f) ? 1 : 0;
    }
  }
}

// primitives/sh.py:82-138 backward kernel.  grad_coeffs (n,K,3) is fully
// written (zeros for culled rows and unused coefficients); grad_dirs may be
// null when directions need no gradient.
void oracle_sh_backward(int n, int degree, int K, const float* coeffs, const float* dirs,
                        const int* radii, const unsigned char* active, const float* upstream,
                        float* grad_coeffs, float* grad_dirs) {
  const int count = (degree + 1) * (degree + 1);
#pragma omp parallel for schedule(static)
  for (int i = 0; i < n; ++i) {
    for (int k = 0; k < K * 3; ++k) grad_coeffs[i * K * 3 + k] = 0.0f;
    const bool visible = radii ? radii[i] > 0 : true;
    float dg[3] = {0.0f, 0.0f, 0.0f};
    if (visible) {
      float unit[3] = {0.0f, 0.0f, 0.0f}, cg[3] = {0.0f, 0.0f, 0.0f};
      float length = 1.0f;
      for (int ch = 0; ch < 3; ++ch)
        if (active[3 * i + ch]) cg[ch] = upstream[3 * i + ch];
      if (degree > 0) {
        const float* d = dirs + 3 * i;
        length = std::sqrt(d[0] * d[0] + d[1] * d[1] + d[2] * d[2]);
        const float den = wmax(length, W32(1e-12));
        for (int j = 0; j < 3; ++j) unit[j] = d[j] / den;
      }
      float ug[3] = {0.0f, 0.0f, 0.0f};
      for (int k = 0; k < count; ++k) {
        const float b = sh_basis(unit, k);
        for (int ch = 0; ch < 3; ++ch) grad_coeffs[(i * K + k) * 3 + ch] = b * cg[ch];
        float bg[3];
        sh_basis_grad(unit, k, bg);
        const float* c = coeffs + (i * K + k) * 3;
        const float w = c[0] * cg[0] + c[1] * cg[1] + c[2] * cg[2];
        for (int j = 0; j < 3; ++j) ug[j] += w * bg[j];
      }
      const float den = wmax(length, W32(1e-12));
      for (int j = 0; j < 3; ++j) dg[j] = ug[j] / den;
      if (length >= W32(1e-12)) {
        const float dot = (unit[0] * ug[0] + unit[1] * ug[1] + unit[2] * ug[2]) / length;
        for (int j = 0; j < 3; ++j) dg[j] -= unit[j] * dot;
      }
    }
    if (grad_dirs)
      for (int j = 0; j < 3; ++j) grad_dirs[3 * i + j] = dg[j];
  }
}

// primitives/tiling.py:57-64 scan_counts: inclusive int32 scan; returns M.
long long oracle_scan_counts(int n, const int* counts, int* offsets) {
  long long total = 0;
  for (int i = 0; i < n; ++i) {
    total += counts[i];
    offsets[i] = static_cast<int>(total);
  }
  return total;
}

// splatting/binning.py:16-37 duplicate, primitives/tiling.py:67-100
// sort_tile_pairs (stable radix sort of (tile<<32 | depth bits, id) pairs)
// and primitives/tiling.py:39-54 identify_ranges.  ranges: (T, 2), written
// in full (zeros for empty tiles); keys_out/ids_out hold M entries.
void oracle_bin_and_sort(int n, const float* centers, const int* radii, const float* depths,
                         const int* offsets, int width, int height, uint64_t* keys_out,
                         int* ids_out, int* ranges, const float* conics, int tile_mode) {
  const int gx = (width + 15) / 16, gy = (height + 15) / 16;
  const long long M = n ? offsets[n - 1] : 0;
  std::vector<uint64_t> keys(M);
  std::vector<int> ids(M);
#pragma omp parallel for schedule(dynamic, 256)
  for (int i = 0; i < n; ++i) {
    if (radii[i] <= 0) continue;
    long long off = i > 0 ? offsets[i - 1] : 0;
    const uint32_t depth = float_bits(depths[i]);
    // splatting/binning.py:40-67 duplicate_precise emits through the same visit
    visit_tiles(tile_mode, centers + 2 * i, conics ? conics + 4 * i : nullptr, radii[i], gx, gy,
                [&](int tile) {
                  keys[off] = (static_cast<uint64_t>(static_cast<uint32_t>(tile)) << 32) | depth;
                  ids[off] = i;
                  ++off;
                });
  }
  std::vector<long long> order(M);
  for (long long p = 0; p < M; ++p) order[p] = p;
  std::stable_sort(order.begin(), order.end(),
                   [&](long long a, long long b) { return keys[a] < keys[b]; });
  const int T = gx * gy;
  for (int t = 0; t < 2 * T; ++t) ranges[t] = 0;
  for (long long p = 0; p < M; ++p) {
    keys_out[p] = keys[order[p]];
    ids_out[p] = ids[order[p]];
  }
  for (long long p = 0; p < M; ++p) {
    const uint32_t cur = static_cast<uint32_t>(keys_out[p] >> 32);
    if (p == 0) {
      ranges[2 * cur] = 0;
    } else {
      const uint32_t prev = static_cast<uint32_t>(keys_out[p - 1] >> 32);
      if (cur != prev) {
        ranges[2 * prev + 1] = static_cast<int>(p);
        ranges[2 * cur] = static_cast<int>(p);
      }
    }
    if (p == M - 1) ranges[2 * cur + 1] = static_cast<int>(M);
  }
}

// gs3d/render.py:41-125 evaluate (forward blend).  image is planar (C,H,W).
void oracle_render_forward(int width, int height, int channels, const int* ranges,
                           const int* ids, const float* centers, const float* conics,
                           const float* features, const float* background, float* image,
                           float* final_t, int* contributors) {
  const int gx = (width + 15) / 16, gy = (height + 15) / 16;
  const int T = gx * gy;
  const float threshold = 1.0f / 255.0f;
#pragma omp parallel for schedule(dynamic, 1)
  for (int tile = 0; tile < T; ++tile) {
    std::vector<float> color(channels);
    const int first = ranges[2 * tile], last = ranges[2 * tile + 1];
    for (int lane = 0; lane < 256; ++lane) {
      const int x = tile % gx * 16 + lane % 16, y = tile / gx * 16 + lane / 16;
      if (!(x < width && y < height)) continue;
      const int pixel = y * width + x;
      float transmittance = 1.0f;
      std::fill(color.begin(), color.end(), 0.0f);
      int contributor = 0, last_contributor = 0;
      for (int idx = first; idx < last; ++idx) {
        contributor += 1;
        const int g = ids[idx];
        const float dx = centers[2 * g] - static_cast<float>(x);
        const float dy = centers[2 * g + 1] - static_cast<float>(y);
        const float* q = conics + 4 * g;
        const float power = -0.5f * (q[0] * dx * dx + q[2] * dy * dy) - q[1] * dx * dy;
        if (power <= 0.0f) {
          const float alpha = wmin(W32(0.99), q[3] * splat_expf(power));
          if (alpha >= threshold) {
            const float next_t = transmittance * (1.0f - alpha);
            if (next_t < W32(0.0001)) break;
            const float* v = features + static_cast<size_t>(g) * channels;
            for (int ch = 0; ch < channels; ++ch)
              color[ch] = color[ch] + v[ch] * alpha * transmittance;
            transmittance = next_t;
            last_contributor = contributor;
          }
        }
      }
      const size_t P = static_cast<size_t>(width) * height;
      for (int ch = 0; ch < channels; ++ch)
        image[ch * P + pixel] = color[ch] + transmittance * background[ch];
      final_t[pixel] = transmittance;
      contributors[pixel] = last_contributor;
    }
  }
}

// gs3d/render.py:221-354 backward (reverse replay).  upstream is planar
// (C,H,W).  Gradient outputs are accumulated in double (grad_* buffers are
// double) and must be zeroed by the caller.  abs_centers may be null.
void oracle_render_backward(int width, int height, int channels, int constant_tail,
                            const int* ranges, const int* ids, const float* centers,
                            const float* conics, const float* features,
                            const float* background, const float* final_t,
                            const int* contributors, const float* upstream,
                            double* grad_centers, double* grad_conics, double* grad_features,
                            double* abs_centers) {
  const int gx = (width + 15) / 16, gy = (height + 15) / 16;
  const int T = gx * gy;
  const float threshold = 1.0f / 255.0f;
  const size_t P = static_cast<size_t>(width) * height;
#pragma omp parallel for schedule(dynamic, 1)
  for (int tile = 0; tile < T; ++tile) {
    std::vector<float> gradient(channels), accumulated(channels), last_color(channels);
    const int first = ranges[2 * tile], last = ranges[2 * tile + 1];
    for (int lane = 0; lane < 256; ++lane) {
      const int x = tile % gx * 16 + lane % 16, y = tile / gx * 16 + lane / 16;
      if (!(x < width && y < height)) continue;
      const int pixel = y * width + x;
      const float final_transmittance = final_t[pixel];
      float transmittance = final_transmittance;
      const int last_contributor = contributors[pixel];
      float background_gradient = 0.0f;
      for (int ch = 0; ch < channels; ++ch) {
        gradient[ch] = upstream[ch * P + pixel];
        background_gradient += background[ch] * gradient[ch];
        accumulated[ch] = 0.0f;
        last_color[ch] = 0.0f;
      }
      float last_alpha = 0.0f;
      int contributor = last - first;
      for (int idx = last - 1; idx >= first; --idx) {
        contributor -= 1;
        if (contributor >= last_contributor) continue;
        const int g = ids[idx];
        const float dx = centers[2 * g] - static_cast<float>(x);
        const float dy = centers[2 * g + 1] - static_cast<float>(y);
        const float* q = conics + 4 * g;
        const float power = -0.5f * (q[0] * dx * dx + q[2] * dy * dy) - q[1] * dx * dy;
        if (!(power <= 0.0f)) continue;
        const float gaussian_value = splat_expf(power);
        const float alpha = wmin(W32(0.99), q[3] * gaussian_value);
        if (!(alpha >= threshold)) continue;
        transmittance = transmittance / (1.0f - alpha);
        const float* color = features + static_cast<size_t>(g) * channels;
        float grad_alpha = 0.0f;
        for (int ch = 0; ch < channels; ++ch) {
          accumulated[ch] = last_alpha * last_color[ch] + (1.0f - last_alpha) * accumulated[ch];
          last_color[ch] = color[ch];
          grad_alpha += (color[ch] - accumulated[ch]) * gradient[ch];
          if (ch < channels - constant_tail) {
#pragma omp atomic
            grad_features[static_cast<size_t>(g) * channels + ch] +=
                static_cast<double>(alpha * transmittance * gradient[ch]);
          }
        }
        grad_alpha = grad_alpha * transmittance +
                     (-final_transmittance / (1.0f - alpha)) * background_gradient;
        last_alpha = alpha;
        const float grad_value = q[3] * grad_alpha;
        const float gdx = gaussian_value * dx, gdy = gaussian_value * dy;
        const float ddx = grad_value * (-gdx * q[0] - gdy * q[1]);
        const float ddy = grad_value * (-gdy * q[2] - gdx * q[1]);
#pragma omp atomic
        grad_centers[2 * g] += ddx;
#pragma omp atomic
        grad_centers[2 * g + 1] += ddy;
        if (abs_centers) {
#pragma omp atomic
          abs_centers[2 * g] += std::fabs(ddx);
#pragma omp atomic
          abs_centers[2 * g + 1] += std::fabs(ddy);
        }
#pragma omp atomic
        grad_conics[4 * g + 0] += -0.5f * gdx * dx * grad_value;
#pragma omp atomic
        grad_conics[4 * g + 1] += -gdx * dy * grad_value;
#pragma omp atomic
        grad_conics[4 * g + 2] += -0.5f * gdy * dy * grad_value;
#pragma omp atomic
        grad_conics[4 * g + 3] += gaussian_value * grad_alpha;
      }
    }
  }
}

// gs3d/projection.py:198-285 project_backward: the VJP of projection_loss
// with the reference's custom adjoints adj_clamp_point
// (splatting/geometry.py:42-51), adj_invert_covariance
// (splatting/geometry.py:61-71) and adj_reference_rotation
// (splatting/math.py:13-28), derived by hand.  Culled rows get zeros.
// grad_view / grad_proj (4x4, double) are accumulated over Gaussians and
// must be zeroed by the caller; either may be null.
void oracle_project_backward(int n, const float* means, const float* quats,
                             const float* scales, const float* opacities, const float* view,
                             const float* proj, const float* K, int width, int height,
                             const int* radii, const float* seed_centers,
                             const float* seed_conics, float* grad_means, float* grad_quats,
                             float* grad_scales, float* grad_opacities, double* grad_view,
                             double* grad_proj) {
  const float fx = K[0], fy = K[4];
  (void)opacities;
  std::vector<double> gv(16, 0.0), gp(16, 0.0);
#pragma omp parallel
  {
    double lv[16] = {0}, lp[16] = {0};
#pragma omp for schedule(static)
    for (int i = 0; i < n; ++i) {
      float gm[3] = {0, 0, 0}, gq4[4] = {0, 0, 0, 0}, gs[3] = {0, 0, 0}, go = 0.0f;
      if (radii[i] > 0) {
        const float* m = means + 3 * i;
        const float* q = quats + 4 * i;
        const float* s = scales + 3 * i;
        const float* sc = seed_centers + 2 * i;
        const float* sq = seed_conics + 4 * i;
        // forward recompute
        const float t[3] = {point_row(view, 0, m), point_row(view, 1, m), point_row(view, 2, m)};
        const float limx = W32(1.3) * static_cast<float>(width) / (2.0f * fx);
        const float limy = W32(1.3) * static_cast<float>(height) / (2.0f * fy);
        const float xr = t[0] / t[2], yr = t[1] / t[2];
        const float tcx = wclamp(xr, -limx, limx) * t[2];
        const float tcy = wclamp(yr, -limy, limy) * t[2];
        const float tz = t[2];
        float R[3][3];
        glm_rotation(q, R);
        float M[3][3], Sig[3][3];
        for (int r = 0; r < 3; ++r)
          for (int c = 0; c < 3; ++c) M[r][c] = s[r] * R[r][c];
        for (int r = 0; r < 3; ++r)
          for (int c = 0; c < 3; ++c)
            Sig[r][c] = M[0][r] * M[0][c] + M[1][r] * M[1][c] + M[2][r] * M[2][c];
        const float J[3][3] = {{fx / tz, 0.0f, 0.0f},
                               {0.0f, fy / tz, 0.0f},
                               {-(fx * tcx) / (tz * tz), -(fy * tcy) / (tz * tz), 0.0f}};
        const float Wc[3][3] = {{view[0], view[4], view[8]},
                                {view[1], view[5], view[9]},
                                {view[2], view[6], view[10]}};
        float Tm[3][3], A[3][3], P[3][3];
        for (int r = 0; r < 3; ++r)
          for (int c = 0; c < 3; ++c)
            Tm[r][c] = Wc[r][0] * J[0][c] + Wc[r][1] * J[1][c] + Wc[r][2] * J[2][c];
        // A = Tm^T Sig^T
        for (int r = 0; r < 3; ++r)
          for (int c = 0; c < 3; ++c)
            A[r][c] = Tm[0][r] * Sig[c][0] + Tm[1][r] * Sig[c][1] + Tm[2][r] * Sig[c][2];
        for (int r = 0; r < 3; ++r)
          for (int c = 0; c < 3; ++c)
            P[r][c] = A[r][0] * Tm[0][c] + A[r][1] * Tm[1][c] + A[r][2] * Tm[2][c];
        const float a = P[0][0] + W32(0.3), b = P[1][0], c = P[1][1] + W32(0.3);
        // adj_invert_covariance
        const float det = a * c - b * b;
        const float factor = 1.0f / (det * det + W32(0.0000001));
        const float X = sq[0], Y = sq[1], Z = sq[2];
        const float da = factor * (-c * c * X + b * c * Y + (det - a * c) * Z);
        const float db = factor * (2.0f * b * c * X - (det + 2.0f * b * b) * Y + 2.0f * a * b * Z);
        const float dc = factor * (-a * a * Z + a * b * Y + (det - a * c) * X);
        go = sq[3];
        float dP[3][3] = {{da, 0, 0}, {db, dc, 0}, {0, 0, 0}};
        // P = A Tm
        float dA[3][3], dTm[3][3];
        for (int r = 0; r < 3; ++r)
          for (int cc = 0; cc < 3; ++cc) {
            dA[r][cc] = dP[r][0] * Tm[cc][0] + dP[r][1] * Tm[cc][1] + dP[r][2] * Tm[cc][2];
            dTm[r][cc] = A[0][r] * dP[0][cc] + A[1][r] * dP[1][cc] + A[2][r] * dP[2][cc];
          }
        // A = Tm^T Sig^T: dTm += Sig^T dA^T ; dSig = dA^T Tm^T
        float dSig[3][3];
        for (int r = 0; r < 3; ++r)
          for (int cc = 0; cc < 3; ++cc) {
            dTm[r][cc] += Sig[0][r] * dA[cc][0] + Sig[1][r] * dA[cc][1] + Sig[2][r] * dA[cc][2];
            dSig[r][cc] = dA[0][r] * Tm[cc][0] + dA[1][r] * Tm[cc][1] + dA[2][r] * Tm[cc][2];
          }
        // Tm = Wc J
        float dWc[3][3], dJ[3][3];
        for (int r = 0; r < 3; ++r)
          for (int cc = 0; cc < 3; ++cc) {
            dWc[r][cc] = dTm[r][0] * J[cc][0] + dTm[r][1] * J[cc][1] + dTm[r][2] * J[cc][2];
            dJ[r][cc] = Wc[0][r] * dTm[0][cc] + Wc[1][r] * dTm[1][cc] + Wc[2][r] * dTm[2][cc];
          }
        // Sig = M^T M: dM = M (dSig + dSig^T)
        float dM[3][3];
        for (int r = 0; r < 3; ++r)
          for (int cc = 0; cc < 3; ++cc) {
            float acc = 0.0f;
            for (int k = 0; k < 3; ++k) acc += M[r][k] * (dSig[k][cc] + dSig[cc][k]);
            dM[r][cc] = acc;
          }
        // M = S R
        float dR[3][3];
        for (int r = 0; r < 3; ++r) {
          gs[r] = dM[r][0] * R[r][0] + dM[r][1] * R[r][1] + dM[r][2] * R[r][2];
          for (int cc = 0; cc < 3; ++cc) dR[r][cc] = s[r] * dM[r][cc];
        }
        // adj_reference_rotation
        {
          const float qr = q[0], qx = q[1], qy = q[2], qz = q[3];
          const float(*g)[3] = dR;
          gq4[0] = 2.0f * (qz * (g[0][1] - g[1][0]) + qy * (g[2][0] - g[0][2]) +
                           qx * (g[1][2] - g[2][1]));
          gq4[1] = 2.0f * (qy * (g[0][1] + g[1][0]) + qz * (g[0][2] + g[2][0]) +
                           qr * (g[1][2] - g[2][1])) -
                   4.0f * qx * (g[1][1] + g[2][2]);
          gq4[2] = 2.0f * (qx * (g[0][1] + g[1][0]) + qr * (g[2][0] - g[0][2]) +
                           qz * (g[1][2] + g[2][1])) -
                   4.0f * qy * (g[0][0] + g[2][2]);
          gq4[3] = 2.0f * (qr * (g[0][1] - g[1][0]) + qx * (g[0][2] + g[2][0]) +
                           qy * (g[1][2] + g[2][1])) -
                   4.0f * qz * (g[0][0] + g[1][1]);
        }
        // J(tc)
        const float tz2 = tz * tz, tz3 = tz2 * tz;
        const float dtcx = dJ[2][0] * (-fx / tz2);
        const float dtcy = dJ[2][1] * (-fy / tz2);
        const float dtcz = dJ[0][0] * (-fx / tz2) + dJ[1][1] * (-fy / tz2) +
                           dJ[2][0] * (2.0f * fx * tcx / tz3) + dJ[2][1] * (2.0f * fy * tcy / tz3);
        // adj_clamp_point
        const float dt[3] = {(xr >= -limx && xr <= limx) ? dtcx : 0.0f,
                             (yr >= -limy && yr <= limy) ? dtcy : 0.0f, dtcz};
        for (int j = 0; j < 3; ++j) gm[j] += view[0 * 4 + j] * dt[0] + view[1 * 4 + j] * dt[1] + view[2 * 4 + j] * dt[2];
        for (int r = 0; r < 3; ++r) {
          for (int j = 0; j < 3; ++j) lv[r * 4 + j] += static_cast<double>(dt[r]) * m[j];
          lv[r * 4 + 3] += dt[r];
        }
        for (int r = 0; r < 3; ++r)
          for (int cc = 0; cc < 3; ++cc) lv[cc * 4 + r] += dWc[r][cc];
        // pixel_center
        const float c0 = point_row(proj, 0, m), c1 = point_row(proj, 1, m), c3 = point_row(proj, 3, m);
        const float iw = 1.0f / (c3 + W32(1e-7));
        const float dnx = sc[0] * static_cast<float>(width) * 0.5f;
        const float dny = sc[1] * static_cast<float>(height) * 0.5f;
        const float dclip0 = dnx * iw, dclip1 = dny * iw;
        const float diw = dnx * c0 + dny * c1;
        const float dclip3 = -diw * iw * iw;
        const float dclip[4] = {dclip0, dclip1, 0.0f, dclip3};
        for (int j = 0; j < 3; ++j) gm[j] += proj[0 * 4 + j] * dclip0 + proj[1 * 4 + j] * dclip1 + proj[3 * 4 + j] * dclip3;
        for (int r = 0; r < 4; ++r) {
          if (r == 2) continue;
          for (int j = 0; j < 3; ++j) lp[r * 4 + j] += static_cast<double>(dclip[r]) * m[j];
          lp[r * 4 + 3] += dclip[r];
        }
      }
      if (grad_means)
        for (int j = 0; j < 3; ++j) grad_means[3 * i + j] = gm[j];
      if (grad_quats)
        for (int j = 0; j < 4; ++j) grad_quats[4 * i + j] = gq4[j];
      if (grad_scales)
        for (int j = 0; j < 3; ++j) grad_scales[3 * i + j] = gs[j];
      if (grad_opacities) grad_opacities[i] = go;
    }
#pragma omp critical
    for (int j = 0; j < 16; ++j) {
      gv[j] += lv[j];
      gp[j] += lp[j];
    }
  }
  if (grad_view)
    for (int j = 0; j < 16; ++j) grad_view[j] += gv[j];
  if (grad_proj)
    for (int j = 0; j < 16; ++j) grad_proj[j] += gp[j];
}

// ---- RaDe-GS ---------------------------------------------------------------

// rade/projection.py:194-260 project.  Culled rows keep radii = tiles = 0 and
// leave the other outputs untouched.  depths is the radial distance
// sqrtf(x*x + y*y + z*z) of the camera-space centre (norm3df's value).
void oracle_rade_project(int n, const float* means, const float* quats, const float* scales,
                         const float* opacities, const float* view, const float* proj,
                         const float* K, int width, int height, float near_plane,
                         float far_plane, float radius_clip, float kernel_size, float* centers,
                         float* conics, int* radii, int* tiles, float* depths, float* planes,
                         float* normals) {
  const int gx = (width + 15) / 16, gy = (height + 15) / 16;
  const float fx = K[0], fy = K[4];
#pragma omp parallel for schedule(static)
  for (int i = 0; i < n; ++i) {
    radii[i] = 0;
    tiles[i] = 0;
    const float* m = means + 3 * i;
    const float t[3] = {point_row(view, 0, m), point_row(view, 1, m), point_row(view, 2, m)};
    if (t[2] <= near_plane || t[2] >= far_plane) continue;
    RayGeometry rays;
    rade_geometry(t, quats + 4 * i, scales + 3 * i, view, width, height, fx, fy, rays);
    const float a = rays.cov[0] + kernel_size, b = rays.cov[1], c = rays.cov[2] + kernel_size;
    const float det = a * c - b * b;
    if (det == 0.0f) continue;
    const float mid = 0.5f * (a + c);
    const int radius =
        f2i(std::ceil(3.0f * std::sqrt(mid + std::sqrt(wmax(W32(0.1), mid * mid - det)))));
    if (static_cast<float>(radius) <= radius_clip) continue;
    float center[2];
    pixel_center(m, proj, width, height, center);
    int bnd[4];
    tile_bounds(center, radius, gx, gy, bnd);
    const int count = (bnd[2] - bnd[0]) * (bnd[3] - bnd[1]);
    if (count == 0) continue;
    const float inverse = 1.0f / (a * c - b * b);
    centers[2 * i] = center[0];
    centers[2 * i + 1] = center[1];
    conics[4 * i + 0] = c * inverse;
    conics[4 * i + 1] = -b * inverse;
    conics[4 * i + 2] = a * inverse;
    conics[4 * i + 3] = opacities[i] * opacity_coefficient(rays.cov, kernel_size);
    radii[i] = radius;
    tiles[i] = count;
    depths[i] = std::sqrt(t[0] * t[0] + t[1] * t[1] + t[2] * t[2]);
    for (int k = 0; k < 3; ++k) {
      planes[3 * i + k] = rays.plane[k];
      normals[3 * i + k] = rays.normal[k];
    }
  }
}

// rade/render.py:106-227 evaluate.  image is planar (C+6, H, W): C features,
// alpha, expected depth, median depth, unit normal; auxiliary (2, H, W):
// depth * rln and the normal sum's length; contributors (2, H, W): last and
// median contributor (-1: none).
void oracle_rade_render(int width, int height, int channels, const int* ranges, const int* ids,
                        const float* centers, const float* conics, const float* features,
                        const float* background, const float* planes, const float* normals,
                        const float* K, float* image, float* auxiliary, int* contributors) {
  const int gx = (width + 15) / 16, gy = (height + 15) / 16;
  const int T = gx * gy;
  const float threshold = 1.0f / 255.0f;
  const size_t P = static_cast<size_t>(width) * height;
#pragma omp parallel for schedule(dynamic, 1)
  for (int tile = 0; tile < T; ++tile) {
    std::vector<float> color(channels);
    const int first = ranges[2 * tile], last = ranges[2 * tile + 1];
    for (int lane = 0; lane < 256; ++lane) {
      const int x = tile % gx * 16 + lane % 16, y = tile / gx * 16 + lane / 16;
      if (!(x < width && y < height)) continue;
      const int pixel = y * width + x;
      float transmittance = 1.0f, depth = 0.0f, median = 0.0f;
      float normal[3] = {0.0f, 0.0f, 0.0f};
      int median_contributor = -1, contributor = 0, last_contributor = 0;
      std::fill(color.begin(), color.end(), 0.0f);
      for (int idx = first; idx < last; ++idx) {
        contributor += 1;
        const int g = ids[idx];
        const float dx = centers[2 * g] - static_cast<float>(x);
        const float dy = centers[2 * g + 1] - static_cast<float>(y);
        const float* q = conics + 4 * g;
        const float power = -0.5f * (q[0] * dx * dx + q[2] * dy * dy) - q[1] * dx * dy;
        if (!(power <= 0.0f)) continue;
        const float alpha = wmin(W32(0.99), q[3] * splat_expf(power));
        if (!(alpha >= threshold)) continue;
        const float next_t = transmittance * (1.0f - alpha);
        if (next_t < W32(0.0001)) break;
        const float* v = features + static_cast<size_t>(g) * channels;
        for (int ch = 0; ch < channels; ++ch)
          color[ch] = color[ch] + v[ch] * alpha * transmittance;
        const float* pl = planes + 3 * g;
        const float distance = pl[0] * dx + pl[1] * dy + pl[2];
        const float weight = alpha * transmittance;
        depth += distance * weight;
        for (int k = 0; k < 3; ++k) normal[k] += normals[3 * g + k] * weight;
        if (transmittance > 0.5f) {
          median = distance;
          median_contributor = contributor;
        }
        transmittance = next_t;
        last_contributor = contributor;
      }
      for (int ch = 0; ch < channels; ++ch)
        image[ch * P + pixel] = color[ch] + transmittance * background[ch];
      const float u = (static_cast<float>(x) + 0.5f - K[2]) / K[0];
      const float v = (static_cast<float>(y) + 0.5f - K[5]) / K[4];
      const float rln = 1.0f / std::sqrt(u * u + v * v + 1.0f);
      const float alpha = 1.0f - transmittance;
      const float expected = last_contributor > 0 ? depth * rln / alpha : 0.0f;
      const float length =
          std::sqrt(normal[0] * normal[0] + normal[1] * normal[1] + normal[2] * normal[2]);
      const float scale = wmax(length, W32(1.0e-12));
      image[(channels + 0) * P + pixel] = alpha;
      image[(channels + 1) * P + pixel] = expected;
      image[(channels + 2) * P + pixel] = median * rln;
      for (int k = 0; k < 3; ++k) image[(channels + 3 + k) * P + pixel] = normal[k] / scale;
      auxiliary[pixel] = depth * rln;
      auxiliary[P + pixel] = length;
      contributors[pixel] = last_contributor;
      contributors[P + pixel] = median_contributor;
    }
  }
}

// rade/render.py:336-545 backward.  Upstream images are channel-last
// (H, W, k) and may be null (zero).  Gradients accumulate in double into
// zeroed buffers; abs_centers may be null.
void oracle_rade_render_backward(
    int width, int height, int channels, const int* ranges, const int* ids,
    const float* centers, const float* conics, const float* features, const float* background,
    const float* planes, const float* normals, const float* K, const float* image,
    const float* auxiliary, const int* contributors, const float* up_features,
    const float* up_alpha, const float* up_depth, const float* up_median,
    const float* up_normals, double* grad_centers, double* grad_conics, double* grad_features,
    double* abs_centers, double* grad_planes, double* grad_normals) {
  const int gx = (width + 15) / 16, gy = (height + 15) / 16;
  const int T = gx * gy;
  const float threshold = 1.0f / 255.0f;
  const size_t P = static_cast<size_t>(width) * height;
#pragma omp parallel for schedule(dynamic, 1)
  for (int tile = 0; tile < T; ++tile) {
    std::vector<float> gradient(channels), accumulated(channels), last_color(channels);
    const int first = ranges[2 * tile], last = ranges[2 * tile + 1];
    for (int lane = 0; lane < 256; ++lane) {
      const int x = tile % gx * 16 + lane % 16, y = tile / gx * 16 + lane / 16;
      if (!(x < width && y < height)) continue;
      const int pixel = y * width + x;
      const float final_transmittance = 1.0f - image[channels * P + pixel];
      float transmittance = final_transmittance;
      const int last_contributor = contributors[pixel];
      float background_gradient = 0.0f;
      for (int ch = 0; ch < channels; ++ch) {
        gradient[ch] = up_features ? up_features[static_cast<size_t>(pixel) * channels + ch] : 0.0f;
        background_gradient += background[ch] * gradient[ch];
        accumulated[ch] = 0.0f;
        last_color[ch] = 0.0f;
      }
      background_gradient -= up_alpha ? up_alpha[pixel] : 0.0f;
      const int median_contributor = contributors[P + pixel];
      float depth_gradient = 0.0f, median_gradient = 0.0f;
      float normal_gradient[3] = {0.0f, 0.0f, 0.0f};
      const float pixel_alpha = image[channels * P + pixel];
      if (pixel_alpha > 0.0f) {
        const float u = (static_cast<float>(x) + 0.5f - K[2]) / K[0];
        const float v = (static_cast<float>(y) + 0.5f - K[5]) / K[4];
        const float rln = 1.0f / std::sqrt(u * u + v * v + 1.0f);
        const float gd = up_depth ? up_depth[pixel] : 0.0f;
        background_gradient += gd * (auxiliary[pixel] / pixel_alpha) / pixel_alpha;
        depth_gradient = gd / pixel_alpha * rln;
        median_gradient = (up_median ? up_median[pixel] : 0.0f) * rln;
        for (int k = 0; k < 3; ++k) normal_gradient[k] = up_normals ? up_normals[3 * pixel + k] : 0.0f;
        const float unit[3] = {image[(channels + 3) * P + pixel], image[(channels + 4) * P + pixel],
                               image[(channels + 5) * P + pixel]};
        const float length = auxiliary[P + pixel];
        if (length >= W32(1.0e-12)) {
          const float d = unit[0] * normal_gradient[0] + unit[1] * normal_gradient[1] +
                          unit[2] * normal_gradient[2];
          for (int k = 0; k < 3; ++k) normal_gradient[k] = normal_gradient[k] - unit[k] * d;
        }
        const float scale = wmax(length, W32(1.0e-12));
        for (int k = 0; k < 3; ++k) normal_gradient[k] = normal_gradient[k] / scale;
      }
      float last_alpha = 0.0f, accumulated_depth = 0.0f, last_depth = 0.0f;
      float accumulated_normal[3] = {0.0f, 0.0f, 0.0f}, last_normal[3] = {0.0f, 0.0f, 0.0f};
      int contributor = last - first;
      for (int idx = last - 1; idx >= first; --idx) {
        contributor -= 1;
        if (contributor >= last_contributor) continue;
        const int g = ids[idx];
        const float dx = centers[2 * g] - static_cast<float>(x);
        const float dy = centers[2 * g + 1] - static_cast<float>(y);
        const float* q = conics + 4 * g;
        const float power = -0.5f * (q[0] * dx * dx + q[2] * dy * dy) - q[1] * dx * dy;
        const float gaussian_value = splat_expf(power);
        const float alpha = wmin(W32(0.99), q[3] * gaussian_value);
        if (!(power <= 0.0f) || !(alpha >= threshold)) continue;
        transmittance = transmittance / (1.0f - alpha);
        const float* color = features + static_cast<size_t>(g) * channels;
        float grad_alpha = 0.0f;
        for (int ch = 0; ch < channels; ++ch) {
          accumulated[ch] = last_alpha * last_color[ch] + (1.0f - last_alpha) * accumulated[ch];
          last_color[ch] = color[ch];
          grad_alpha += (color[ch] - accumulated[ch]) * gradient[ch];
#pragma omp atomic
          grad_features[static_cast<size_t>(g) * channels + ch] +=
              static_cast<double>(alpha * transmittance * gradient[ch]);
        }
        const float* pl = planes + 3 * g;
        const float distance = pl[0] * dx + pl[1] * dy + pl[2];
        const float* nm = normals + 3 * g;
        accumulated_depth = last_alpha * last_depth + (1.0f - last_alpha) * accumulated_depth;
        for (int k = 0; k < 3; ++k)
          accumulated_normal[k] =
              last_alpha * last_normal[k] + (1.0f - last_alpha) * accumulated_normal[k];
        grad_alpha += (distance - accumulated_depth) * depth_gradient +
                      ((nm[0] - accumulated_normal[0]) * normal_gradient[0] +
                       (nm[1] - accumulated_normal[1]) * normal_gradient[1] +
                       (nm[2] - accumulated_normal[2]) * normal_gradient[2]);
        last_depth = distance;
        for (int k = 0; k < 3; ++k) last_normal[k] = nm[k];
        const float weight = alpha * transmittance;
        float g_distance = weight * depth_gradient;
        if (contributor == median_contributor - 1) g_distance += median_gradient;
#pragma omp atomic
        grad_planes[3 * g + 0] += g_distance * dx;
#pragma omp atomic
        grad_planes[3 * g + 1] += g_distance * dy;
#pragma omp atomic
        grad_planes[3 * g + 2] += g_distance;
        for (int k = 0; k < 3; ++k) {
#pragma omp atomic
          grad_normals[3 * g + k] += normal_gradient[k] * weight;
        }
        grad_alpha = grad_alpha * transmittance +
                     (-final_transmittance / (1.0f - alpha)) * background_gradient;
        last_alpha = alpha;
        const float grad_value = q[3] * grad_alpha;
        const float gdx = gaussian_value * dx, gdy = gaussian_value * dy;
        float ddx = grad_value * (-gdx * q[0] - gdy * q[1]);
        float ddy = grad_value * (-gdy * q[2] - gdx * q[1]);
        ddx += g_distance * pl[0];
        ddy += g_distance * pl[1];
#pragma omp atomic
        grad_centers[2 * g] += ddx;
#pragma omp atomic
        grad_centers[2 * g + 1] += ddy;
        if (abs_centers) {
#pragma omp atomic
          abs_centers[2 * g] += std::fabs(ddx);
#pragma omp atomic
          abs_centers[2 * g + 1] += std::fabs(ddy);
        }
#pragma omp atomic
        grad_conics[4 * g + 0] += -0.5f * gdx * dx * grad_value;
#pragma omp atomic
        grad_conics[4 * g + 1] += -gdx * dy * grad_value;
#pragma omp atomic
        grad_conics[4 * g + 2] += -0.5f * gdy * dy * grad_value;
#pragma omp atomic
        grad_conics[4 * g + 3] += gaussian_value * grad_alpha;
      }
    }
  }
}

int oracle_num_threads(void) {
#ifdef _OPENMP
  return omp_get_max_threads();
#else
  return 1;
#endif
}

void oracle_set_num_threads(int n) {
#ifdef _OPENMP
  if (n > 0) omp_set_num_threads(n);
#else
  (void)n;
#endif
}

}  // extern "C"
