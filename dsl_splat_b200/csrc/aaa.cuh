// AAA-Gaussians (adaptive 3D antialiasing, 3D ray evaluation, StopThePop
// hierarchical sorting): the B200 kernels replacing dsl_splat/aaa's Warp
// launches for one view of aaa.rasterize's default settings
// (aaa/config.py:41-54: eval_3D, load balancing, tile-based and 4x4
// culling, HIER 64/8/4, sort order PTD_MAX).
//
//   aaa_preprocess_kernel      aaa/preprocess3d.py:17-245 (K19)
//   aaa_cull_remainder_kernel  aaa/cooperative_culling.py:152-192 (K20)
//   aaa_emit_kernel            aaa/binning_native.py:7-135 (K22)
//   sort passes + ranges       primitives/tiling.py:39-100 on the AAA keys
//
// Compiled in the -fmad=false unit: the tile counts, the culling decisions
// and the sort keys depend on the last bit of these expressions, so every
// multiply-add is two roundings unless the reference's GLM / native code
// fuses it (__fmaf_rn here).  atan2 and tan are this library's own
// (splat_atan2f / splat_tanf below), as are exp and log: the CPU oracle
// evaluates the same functions, so integer outputs agree bit for bit.
#pragma once
#include <cfloat>

#include "binning.cuh"
#include "splat_common.cuh"

namespace splat {
namespace aaa {

// ---- atan2 and tan -----------------------------------------------------------
// Evaluated in double precision (no library call) and rounded once to float:
// the float result is the correctly rounded one except in near-halfway
// cases, and the CPU oracle runs the same steps.  The constants are the
// nearest doubles to their exact values (trig_constants.py prints them).
// atan(i / 8)
__constant__ double kAtanTable[9] = {
    0.0, 0.12435499454676144, 0.24497866312686414, 0.35877067027057225, 0.4636476090008061,
    0.5585993153435624, 0.6435011087932844, 0.7188299996216245, 0.7853981633974483};
// 1 / (2k + 1)
__constant__ double kAtanSeries[8] = {
    1.0, 0.3333333333333333, 0.2, 0.14285714285714285, 0.1111111111111111, 0.09090909090909091,
    0.07692307692307693, 0.06666666666666667};
// 1 / (2j + 1)!
__constant__ double kSinSeries[11] = {
    1.0, 0.16666666666666666, 0.008333333333333333, 0.0001984126984126984,
    2.7557319223985893e-06, 2.505210838544172e-08, 1.6059043836821613e-10,
    7.647163731819816e-13, 2.8114572543455206e-15, 8.22063524662433e-18, 1.9572941063391263e-20};
// 1 / (2j)!
__constant__ double kCosSeries[12] = {
    1.0, 0.5, 0.041666666666666664, 0.001388888888888889, 2.48015873015873e-05,
    2.755731922398589e-07, 2.08767569878681e-09, 1.1470745597729725e-11, 4.779477332387385e-14,
    1.5619206968586225e-16, 4.110317623312165e-19, 8.896791392450574e-22};
constexpr double kTwoOverPi = 0.6366197723675814;

// atan(t), 0 <= t <= 1: with c the nearest multiple of 1/8, atan(t) =
// atan(c) + atan(u), u = (t - c) / (1 + t c), |u| <= 1/16, and atan(u) from
// its alternating series to u^15 / 15 (Horner in u^2; the next term is below
// 2^-69 relative).
SPLAT_DEV double atan_unit(double t) {
  const int i = static_cast<int>(__dadd_rn(__dmul_rn(t, 8.0), 0.5));
  const double c = __dmul_rn(static_cast<double>(i), 0.125);
  const double u = __ddiv_rn(__dsub_rn(t, c), __dadd_rn(1.0, __dmul_rn(t, c)));
  const double u2 = __dmul_rn(u, u);
  double p = kAtanSeries[7];
#pragma unroll
  for (int k = 6; k >= 0; --k) p = __dsub_rn(kAtanSeries[k], __dmul_rn(u2, p));
  return __dadd_rn(kAtanTable[i], __dmul_rn(u, p));
}

SPLAT_DEV float splat_atan2f(float yf, float xf) {
  const double kPi = 3.141592653589793, kHalfPi = 1.5707963267948966;
  if (isnan(yf) || isnan(xf)) return yf + xf;
  const double y = yf, x = xf;
  if (y == 0.0) return static_cast<float>(signbit(x) ? copysign(kPi, y) : y);
  if (x == 0.0) return static_cast<float>(copysign(kHalfPi, y));
  if (isinf(y) || isinf(x)) {
    double r;
    if (isinf(y) && isinf(x)) r = x > 0 ? kPi / 4 : 3 * kPi / 4;
    else if (isinf(y)) r = kHalfPi;
    else r = x > 0 ? 0.0 : kPi;
    return static_cast<float>(copysign(r, y));
  }
  const double ax = fabs(x), ay = fabs(y);
  double r = ay <= ax ? atan_unit(__ddiv_rn(ay, ax)) : __dsub_rn(kHalfPi, atan_unit(__ddiv_rn(ax, ay)));
  if (x < 0.0) r = __dsub_rn(kPi, r);
  return static_cast<float>(copysign(r, y));
}

// tan(x): reduction by the nearest multiple k of pi/2 (pi/2 in three parts
// of 33, 33 and 53 significant bits, derived from Machin's formula, so that
// k * part is exact for |x| < 2^20); sin and cos of the remainder |r| <~
// pi/4 from their Taylor series (to r^21 / 21! and r^22 / 22!, Horner in
// r^2), tan = sin / cos (-cos / sin for odd k).
SPLAT_DEV float splat_tanf(float xf) {
  if (isnan(xf) || isinf(xf)) return xf - xf;
  const double x = xf;
  const double k = nearbyint(__dmul_rn(x, kTwoOverPi));
  const double r = __dsub_rn(__dsub_rn(__dsub_rn(x, __dmul_rn(k, 1.5707963267341256)),
                                       __dmul_rn(k, 6.077100506303966e-11)),
                             __dmul_rn(k, 2.0222662487959506e-21));
  const double r2 = __dmul_rn(r, r);
  double s = kSinSeries[10], c = kCosSeries[11];
#pragma unroll
  for (int j = 9; j >= 0; --j) s = __dsub_rn(kSinSeries[j], __dmul_rn(r2, s));
#pragma unroll
  for (int j = 10; j >= 0; --j) c = __dsub_rn(kCosSeries[j], __dmul_rn(r2, c));
  s = __dmul_rn(r, s);
  const bool odd = fmod(fabs(k), 2.0) == 1.0;
  return static_cast<float>(odd ? __ddiv_rn(-c, s) : __ddiv_rn(s, c));
}

// test support: splat_atan2f(y, x) and splat_tanf(x) element-wise
__global__ void trig_probe_kernel(int n, const float* y, const float* x, float* atan2_out,
                                  float* tan_out) {
  const int i = blockIdx.x * blockDim.x + threadIdx.x;
  if (i >= n) return;
  atan2_out[i] = splat_atan2f(y[i], x[i]);
  tan_out[i] = splat_tanf(x[i]);
}

// ---- matrices -------------------------------------------------------------------

struct M4 {
  float m[4][4];
};

// primitives/math.py:60-68 glm_matmul44: fma(a3,b3, fma(a2,b2, fma(a0,b0, a1*b1)))
SPLAT_DEV M4 glm_matmul(const M4& a, const M4& b) {
  M4 out;
#pragma unroll
  for (int i = 0; i < 4; ++i)
#pragma unroll
    for (int j = 0; j < 4; ++j)
      out.m[i][j] = __fmaf_rn(a.m[i][3], b.m[3][j],
                              __fmaf_rn(a.m[i][2], b.m[2][j],
                                        __fmaf_rn(a.m[i][0], b.m[0][j], a.m[i][1] * b.m[1][j])));
  return out;
}

// aaa/geometry.py:18-37 load_camera: the stored array is the transpose
SPLAT_DEV M4 load_transposed(const float* a) {
  M4 out;
#pragma unroll
  for (int r = 0; r < 4; ++r)
#pragma unroll
    for (int c = 0; c < 4; ++c) out.m[r][c] = a[c * 4 + r];
  return out;
}

SPLAT_DEV void mat3_mul(const float a[3][3], const float b[3][3], float out[3][3]) {
#pragma unroll
  for (int r = 0; r < 3; ++r)
#pragma unroll
    for (int c = 0; c < 3; ++c) out[r][c] = (a[r][0] * b[0][c] + a[r][1] * b[1][c]) + a[r][2] * b[2][c];
}

SPLAT_DEV void mat3_vec(const float a[3][3], const float v[3], float out[3]) {
#pragma unroll
  for (int r = 0; r < 3; ++r) out[r] = (a[r][0] * v[0] + a[r][1] * v[1]) + a[r][2] * v[2];
}

SPLAT_DEV float dot3p(const float a[3], const float b[3]) {
  return (a[0] * b[0] + a[1] * b[1]) + a[2] * b[2];
}

// primitives/math.py:44-57 glm_rotation (quaternion r, x, y, z)
SPLAT_DEV void glm_rotation(float r, float x, float y, float z, float R[3][3]) {
  const float yy = y * y, zz = z * z;
  const float rz = r * z, xz = x * z, rx = r * x;
  const float d0 = yy + zz, d1 = __fmaf_rn(x, x, zz), d2 = __fmaf_rn(x, x, yy);
  R[0][0] = 1.0f - (d0 + d0);
  R[0][1] = 2.0f * __fmaf_rn(x, y, rz);
  R[0][2] = 2.0f * __fmaf_rn(-r, y, xz);
  R[1][0] = 2.0f * __fmaf_rn(x, y, -rz);
  R[1][1] = 1.0f - (d1 + d1);
  R[1][2] = 2.0f * __fmaf_rn(y, z, rx);
  R[2][0] = 2.0f * __fmaf_rn(r, y, xz);
  R[2][1] = 2.0f * __fmaf_rn(y, z, -rx);
  R[2][2] = 1.0f - (d2 + d2);
}

// ---- aaa/native_geometry.py ---------------------------------------------------------

struct V4 {
  float v[4];
};

SPLAT_DEV V4 row_of(const M4& g, int r) { return V4{{g.m[r][0], g.m[r][1], g.m[r][2], g.m[r][3]}}; }

SPLAT_DEV float fdot3(float a0, float a1, float a2, float b0, float b1, float b2) {
  return __fmaf_rn(a2, b2, __fmaf_rn(a0, b0, a1 * b1));
}

SPLAT_DEV float fdot4(const V4& a, const V4& b) {
  return __fmaf_rn(a.v[0], b.v[0], a.v[1] * b.v[1]) + __fmaf_rn(a.v[2], b.v[2], a.v[3] * b.v[3]);
}

SPLAT_DEV V4 ftransform(const M4& g, const V4& p) {
  return V4{{fdot4(row_of(g, 0), p), fdot4(row_of(g, 1), p), fdot4(row_of(g, 2), p),
             fdot4(row_of(g, 3), p)}};
}

struct FrustumDepth {
  float half_distance, depth;
};

// :87-171 frustum_depth_native: half the smallest squared Gaussian-space
// distance from the centre to the frustum [x, x+w] x [y, y+h] x (-1, 1) and
// the screen depth where it is reached; `sequential` keeps the nearer y
// plane's products rounded separately (the serial first-32-tile loop).
SPLAT_DEV FrustumDepth frustum_depth(const M4& g, float x, float y, float w, float h,
                                     bool sequential) {
  const float start[3] = {x, y, -1.0f}, extent[3] = {w, h, 2.0f};
  auto inside = [&](const V4& p, int dim) {
    const float delta = p.v[dim] - start[dim] * p.v[3];
    return delta > 0.0f && delta < extent[dim] * p.v[3];
  };
  auto plane_at = [&](int axis, float coordinate, bool far) {
    V4 out;
#pragma unroll
    for (int j = 0; j < 4; ++j)
      out.v[j] = (sequential && axis == 1 && !far) ? g.m[axis][j] - g.m[3][j] * coordinate
                                                    : __fmaf_rn(-g.m[3][j], coordinate, g.m[axis][j]);
    return out;
  };
  const V4 mean{{g.m[0][3], g.m[1][3], g.m[2][3], g.m[3][3]}};
  V4 best_pos{{1.0f, 1.0f, 1.0f, 1.0f}};
  float best = FLT_MAX;
  if (inside(mean, 0) && inside(mean, 1) && inside(mean, 2)) {
    best = 0.0f;
    best_pos = mean;
  } else {
    const float dx = copysignf(w * 0.5f, (mean.v[0] - x * mean.v[3]) - w * 0.5f * mean.v[3]);
    const float dy = copysignf(h * 0.5f, (mean.v[1] - y * mean.v[3]) - h * 0.5f * mean.v[3]);
    const V4 ax = plane_at(0, x + w * 0.5f + dx, false);
    const V4 ay = plane_at(1, y + h * 0.5f + dy, false);
    auto plane = [&](const V4& a, int other) {
      const float norm = a.v[3] / fdot3(a.v[0], a.v[1], a.v[2], a.v[0], a.v[1], a.v[2]);
      const V4 p{{-a.v[0] * norm, -a.v[1] * norm, -a.v[2] * norm, 1.0f}};
      const V4 screen = ftransform(g, p);
      const float value = a.v[3] * norm;
      if (value < best && inside(screen, other) && inside(screen, 2)) {
        best = value;
        best_pos = screen;
      }
    };
    plane(ax, 1);
    plane(ay, 0);
    auto edge = [&](const V4& a, const V4& b) {
      const float d[3] = {a.v[1] * b.v[2] - a.v[2] * b.v[1], a.v[2] * b.v[0] - a.v[0] * b.v[2],
                          a.v[0] * b.v[1] - a.v[1] * b.v[0]};
      const float m[3] = {a.v[3] * b.v[0] - a.v[0] * b.v[3], a.v[3] * b.v[1] - a.v[1] * b.v[3],
                          a.v[3] * b.v[2] - a.v[2] * b.v[3]};
      const float dd = fdot3(d[0], d[1], d[2], d[0], d[1], d[2]);
      const float md[3] = {m[0] / dd, m[1] / dd, m[2] / dd};
      const V4 p{{d[1] * md[2] - md[1] * d[2], d[2] * md[0] - md[2] * d[0],
                  d[0] * md[1] - md[0] * d[1], 1.0f}};
      const float squared = fdot3(m[0], m[1], m[2], md[0], md[1], md[2]);
      const V4 screen = ftransform(g, p);
      if (squared < best && inside(screen, 2)) {
        best = squared;
        best_pos = screen;
      }
    };
    edge(ax, ay);
    edge(ax, plane_at(1, y + h * 0.5f - dy, true));
    edge(plane_at(0, x + w * 0.5f - dx, false), ay);
  }
  return FrustumDepth{0.5f * best, best_pos.v[2] / best_pos.v[3]};
}

SPLAT_DEV float pdot4(const V4& a, const V4& b) {
  return (a.v[0] * b.v[0] + a.v[1] * b.v[1]) + (a.v[2] * b.v[2] + a.v[3] * b.v[3]);
}

SPLAT_DEV V4 cwmul(const V4& a, const V4& b) {
  return V4{{a.v[0] * b.v[0], a.v[1] * b.v[1], a.v[2] * b.v[2], a.v[3] * b.v[3]}};
}

// :174-222 bound_axis_native: tangents of the two view-space angles (in the
// axis-z plane) that bound the cutoff ellipsoid, clipped to +-(pi/2 - 1e-5)
// and unwrapped around the mean's own angle.
SPLAT_DEV void bound_axis(const M4& g2v, const float mean[3], float cutoff, int axis, float out[2]) {
  const float pi = 3.14159265358979323846f;
  const float length_squared = (mean[0] * mean[0] + mean[1] * mean[1]) + mean[2] * mean[2];
  const float norm = 1.0f / sqrtf(length_squared);
  const float direction[3] = {mean[0] * norm, mean[1] * norm, mean[2] * norm};
  const float theta_mu = splat_atan2f(direction[axis], direction[2]);
  const V4 t{{cutoff, cutoff, cutoff, -1.0f}};
  const V4 a = row_of(g2v, axis), z = row_of(g2v, 2);
  const float aa = pdot4(t, cwmul(a, a)), zz = pdot4(t, cwmul(z, z)), az = pdot4(t, cwmul(a, z));
  const float discriminant = az * az - zz * aa;
  float lower = -(1.57079632679489661923f - 1e-5f), upper = -lower;
  if (discriminant > 0.0f) {
    const float root = sqrtf(discriminant);
    float lo = splat_atan2f(-(az + root), -zz), hi = splat_atan2f(-(az - root), -zz);
    for (int k = 0; k < 8 && lo > theta_mu; ++k) lo -= pi;
    for (int k = 0; k < 8 && lo < theta_mu - pi; ++k) lo += pi;
    for (int k = 0; k < 8 && hi < theta_mu; ++k) hi += pi;
    for (int k = 0; k < 8 && hi > theta_mu + pi; ++k) hi -= pi;
    auto wrap = [&](float theta) {
      theta = fmodf(theta, 2.0f * pi);
      if (theta > pi) theta -= 2.0f * pi;
      if (theta <= -pi) theta += 2.0f * pi;
      return theta;
    };
    const float nl = wrap(lo), nh = wrap(hi);
    if (theta_mu < 0.0f && fabsf(nl) < fabsf(nh)) {
      lo += 2.0f * pi;
      hi += 2.0f * pi;
    } else if (theta_mu > 0.0f && fabsf(nh) < fabsf(nl)) {
      lo -= 2.0f * pi;
      hi -= 2.0f * pi;
    }
    lower = fmaxf(lower, lo);
    upper = fminf(upper, hi);
  }
  out[0] = splat_tanf(lower);
  out[1] = splat_tanf(upper);
}

// :224-247 screen_bounds_native: centre and half extent of the cutoff
// quadric's screen projection; false when it is unbounded in front of the
// camera or leaves the depth range.
SPLAT_DEV bool screen_bounds(const M4& g2s, float cutoff, float center[2], float extent[2]) {
  const V4 t{{cutoff, cutoff, cutoff, -1.0f}};
  const V4 x = row_of(g2s, 0), y = row_of(g2s, 1), z = row_of(g2s, 2), w = row_of(g2s, 3);
  const float s = pdot4(t, cwmul(w, w));
  if (s >= 0.0f) return false;
  const float inv = 1.0f / s;
  const V4 f{{inv * t.v[0], inv * t.v[1], inv * t.v[2], inv * t.v[3]}};
  const float px = pdot4(f, cwmul(x, w)), py = pdot4(f, cwmul(y, w)), pz = pdot4(f, cwmul(z, w));
  const float hz = pz * pz - pdot4(f, cwmul(z, z));
  const float ez = sqrtf(fmaxf(hz, 0.0f));
  if (pz - ez < -1.0f || pz + ez > 1.0f) return false;
  const float hx = px * px - pdot4(f, cwmul(x, x)), hy = py * py - pdot4(f, cwmul(y, y));
  center[0] = px;
  center[1] = py;
  extent[0] = sqrtf(fmaxf(hx, 0.0f));
  extent[1] = sqrtf(fmaxf(hy, 0.0f));
  return extent[0] >= 0.0f;
}

// primitives/sh.py:141-180 evaluate_sh in its own term order
SPLAT_DEV void evaluate_sh(const float* coeffs, int degree, const float mean[3],
                           const float* camera, float out[3]) {
  const float diff[3] = {mean[0] - camera[0], mean[1] - camera[1], mean[2] - camera[2]};
  const float len = sqrtf(dot3p(diff, diff));
  const float x = diff[0] / len, y = diff[1] / len, z = diff[2] / len;
  const float C0 = 0.28209479177387814f, C1 = 0.4886025119029199f;
  const float C2[5] = {1.0925484305920792f, 1.0925484305920792f, 0.31539156525252005f,
                       1.0925484305920792f, 0.5462742152960396f};
  const float C3[7] = {0.5900435899266435f, 2.890611442640554f, 0.4570457994644658f,
                       0.3731763325901154f, 0.4570457994644658f, 1.445305721320277f,
                       0.5900435899266435f};
  for (int ch = 0; ch < 3; ++ch) {
    auto c = [&](int k) { return coeffs[k * 3 + ch]; };
    float r = C0 * c(0);
    if (degree > 0) {
      r = r - (C1 * y) * c(1);
      r = r + (C1 * z) * c(2);
      r = r - (C1 * x) * c(3);
      if (degree > 1) {
        const float xx = x * x, yy = y * y, zz = z * z, xy = x * y, yz = y * z, xz = x * z;
        r = r + (C2[0] * xy) * c(4);
        r = r - (C2[1] * yz) * c(5);
        r = r + (C2[2] * ((2.0f * zz - xx) - yy)) * c(6);
        r = r - (C2[3] * xz) * c(7);
        r = r + (C2[4] * (xx - yy)) * c(8);
        if (degree > 2) {
          r = r - ((C3[0] * y) * (3.0f * xx - yy)) * c(9);
          r = r + ((C3[1] * xy) * z) * c(10);
          r = r - ((C3[2] * y) * ((4.0f * zz - xx) - yy)) * c(11);
          r = r + ((C3[3] * z) * ((2.0f * zz - 3.0f * xx) - 3.0f * yy)) * c(12);
          r = r - ((C3[4] * x) * ((4.0f * zz - xx) - yy)) * c(13);
          r = r + ((C3[5] * z) * (xx - yy)) * c(14);
          r = r - ((C3[6] * x) * (xx - 3.0f * yy)) * c(15);
        }
      }
    }
    out[ch] = r + 0.5f;
  }
}

// the tile rectangle of a Gaussian's bounds (cooperative_culling.py:39-48)
SPLAT_DEV int4 bounds_rect(float cx, float cy, float ex, float ey, int gx, int gy) {
  return make_int4(iclamp(f2i(floorf((cx - ex) / 16.0f)), 0, gx),
                   iclamp(f2i(floorf((cy - ey) / 16.0f)), 0, gy),
                   iclamp(f2i(ceilf((cx + ex) / 16.0f)), 0, gx),
                   iclamp(f2i(ceilf((cy + ey) / 16.0f)), 0, gy));
}

SPLAT_DEV M4 load_m4(const float* t, long long i) {
  const float4* rows = reinterpret_cast<const float4*>(t) + 4 * i;
  M4 g;
#pragma unroll
  for (int r = 0; r < 4; ++r) {
    const float4 v = rows[r];
    g.m[r][0] = v.x;
    g.m[r][1] = v.y;
    g.m[r][2] = v.z;
    g.m[r][3] = v.w;
  }
  return g;
}

// ---- the first 32 tiles of each rectangle, flattened over the warp ----------------
// Each lane brings up to 32 tiles of its Gaussian's rectangle (row-major from
// (bx, by), rw tiles wide) and the warp walks the concatenation of all lanes'
// tiles 32 at a time, so the walk takes ceil(sum / 32) steps instead of the
// largest lane's count (4x fewer at 1080p: most rectangles are small, a few
// reach 32).  Every lane calls visit(owner, pass, rank, x, y, depth) once per
// step (it may shuffle): owner is the lane whose tile this lane tested, pass
// whether the tile is within the owner's threshold, rank the number of the
// owner's passing tiles before this one.  Returns the lane's own passing
// tiles.  All 32 lanes must call it.
template <bool SEQUENTIAL, typename Visit>
SPLAT_DEV int warp_first_tiles(int tiles, int bx, int by, int rw, const M4& g, float threshold,
                               Visit&& visit) {
  const unsigned full = 0xffffffffu;
  const int lane = threadIdx.x & 31;
  int inclusive = tiles;
#pragma unroll
  for (int d = 1; d < 32; d <<= 1) {
    const int v = __shfl_up_sync(full, inclusive, d);
    if (lane >= d) inclusive += v;
  }
  const int start = inclusive - tiles;
  const int total = __shfl_sync(full, inclusive, 31);
  int own_hits = 0;
  for (int base = 0; base < total; base += 32) {
    const int f = base + lane;
    int owner = 0;  // the last lane whose tiles start at or before f (it has tiles)
#pragma unroll
    for (int step = 16; step >= 1; step >>= 1) {
      const int candidate = owner + step;
      if (__shfl_sync(full, start, candidate) <= f) owner = candidate;
    }
    const int owner_start = __shfl_sync(full, start, owner);
    const int obx = __shfl_sync(full, bx, owner), oby = __shfl_sync(full, by, owner);
    const int orw = __shfl_sync(full, rw, owner);
    const float limit = __shfl_sync(full, threshold, owner);
    M4 og;
#pragma unroll
    for (int r = 0; r < 4; ++r)
#pragma unroll
      for (int c = 0; c < 4; ++c) og.m[r][c] = __shfl_sync(full, g.m[r][c], owner);
    bool pass = false;
    int x = 0, y = 0;
    float depth = 0.0f;
    if (f < total) {
      const int t = f - owner_start;
      x = obx + t % orw;
      y = oby + t / orw;
      const FrustumDepth fd = frustum_depth(og, static_cast<float>(x * 16),
                                            static_cast<float>(y * 16), 15.0f, 15.0f, SEQUENTIAL);
      pass = fd.half_distance <= limit;
      depth = fd.depth;
    }
    const unsigned hits = __ballot_sync(full, pass);
    const int first_lane = owner_start > base ? owner_start - base : 0;  // owner's first item here
    const unsigned earlier = hits & lanemask_lt() & ~((1u << first_lane) - 1u);
    const int rank = __shfl_sync(full, own_hits, owner) + __popc(earlier);
    visit(owner, pass, rank, x, y, depth);
    const int lo = min(max(start - base, 0), 32), hi = min(max(start + tiles - base, 0), 32);
    const unsigned upto_hi = hi >= 32 ? full : (1u << hi) - 1u;
    const unsigned upto_lo = lo >= 32 ? full : (1u << lo) - 1u;
    own_hits += __popc(hits & upto_hi & ~upto_lo);
  }
  return own_hits;
}

// ---- K19: preprocessing ------------------------------------------------------------

struct PreprocessParams {
  int n;
  const float* means;       // (n,3)
  const float* scales;      // (n,3)
  const float* quats;       // (n,4) normalised, or raw when normalize_quats
  int normalize_quats;      // normalise in-kernel with the bits of Torch's F.normalize
  const float* opacities;   // (n)
  const float* sh;          // (n,K,3) or null
  int sh_k, degree, sort_order;
  const float* filters;     // (n) or null
  const float* campos;      // (3)
  const float* view;        // (4,4) transposed storage
  const float* proj;        // (4,4) transposed storage
  int width, height;
  float tanx, tany, principal_x, principal_y, modifier;
  int ewa, new_aabb, near_clipping, tile_culling, complete, cooperative;
  // outputs
  float* centers;           // (n,2)
  float* rects;             // (n,2)
  float* depths;            // (n)
  float* transforms;        // (n,4,4)
  float* opacity_out;       // (n)
  int* radii;               // (n)
  int* tiles;               // (n)
  float* rgb;               // (n,3) or null
  unsigned char* valid;     // (n)
  unsigned char* clamped;   // (n,3) or null
  int* queued;              // (n) when cooperative
  int* queue_size;          // (1), zeroed by the caller
};

__global__ void __launch_bounds__(128) aaa_preprocess_kernel(PreprocessParams p) {
  const int i = blockIdx.x * blockDim.x + threadIdx.x;
  if (i < p.n) {
    p.radii[i] = 0;
    p.tiles[i] = 0;
    p.valid[i] = 0;
  }
  // the per-Gaussian part up to the rectangle; false: rejected (lanes stay
  // for the warp's tile walk)
  float pm[3], t[3], cam[3], opacity = 0.0f, threshold = 0.0f, center[2], extent[2];
  M4 g2s = {};
  int4 b = make_int4(0, 0, 0, 0);
  int count = 0, radius = 0;
  auto front = [&]() -> bool {
    const M4 V = load_transposed(p.view), P = load_transposed(p.proj);
    const float fx = static_cast<float>(p.width) / (2.0f * p.tanx);
    const float fy = static_cast<float>(p.height) / (2.0f * p.tany);
    const float W = static_cast<float>(p.width), H = static_cast<float>(p.height);
    M4 viewport = {};
    viewport.m[0][0] = W / 2.0f;
    viewport.m[0][3] = W / 2.0f - 0.5f;
    viewport.m[1][1] = H / 2.0f;
    viewport.m[1][3] = H / 2.0f - 0.5f;
    viewport.m[2][2] = 1.0f;
    viewport.m[3][3] = 1.0f;
    const M4 clip = glm_matmul(viewport, P);
    const int gx = (p.width + 15) / 16, gy = (p.height + 15) / 16;
    pm[0] = p.means[3 * i];
    pm[1] = p.means[3 * i + 1];
    pm[2] = p.means[3 * i + 2];
    // primitives/math.py:89-94 glm_view_position; the load-balanced
    // specialisation rounds the z product before the sum
#pragma unroll
    for (int r = 0; r < 3; ++r) {
      const float xy = __fmaf_rn(V.m[r][0], pm[0], V.m[r][1] * pm[1]);
      const float total = (!p.complete && r == 2) ? xy + V.m[r][2] * pm[2]
                                                  : __fmaf_rn(V.m[r][2], pm[2], xy);
      t[r] = total + V.m[r][3];
    }
    if (p.near_clipping && t[2] < 0.2f) return false;
    float R[3][3];
    {
      float4 q = reinterpret_cast<const float4*>(p.quats)[i];
      if (p.normalize_quats) q = torch_normalize4(q);
      glm_rotation(q.x, q.y, q.z, q.w, R);
    }
    cam[0] = p.campos[0];
    cam[1] = p.campos[1];
    cam[2] = p.campos[2];
    const float rel[3] = {pm[0] - cam[0], pm[1] - cam[1], pm[2] - cam[2]};
    const float inv_len = 1.0f / sqrtf((rel[0] * rel[0] + rel[1] * rel[1]) + rel[2] * rel[2]);
    const float dir[3] = {rel[0] * inv_len, rel[1] * inv_len, rel[2] * inv_len};
    float ray[3];
    mat3_vec(R, dir, ray);
    const float s[3] = {p.scales[3 * i], p.scales[3 * i + 1], p.scales[3 * i + 2]};
    const float var[3] = {s[0] * s[0], s[1] * s[1], s[2] * s[2]};
    // primitives/math.py:71-86 glm_filter_view_depth
    const float depth =
        __fmaf_rn(V.m[2][0], pm[0], V.m[2][1] * pm[1]) + (V.m[2][2] * pm[2] + V.m[2][3]);
    const float focal = fmaxf(fx, fy);
    float filter_variance = (depth / focal) * (depth / focal) * 0.3f;
    if (p.filters) filter_variance = fmaxf(p.filters[i] * p.filters[i], filter_variance);
    float dilated[3];
#pragma unroll
    for (int k = 0; k < 3; ++k) dilated[k] = sqrtf(s[k] * s[k] + filter_variance);
    const float ray2[3] = {ray[0] * ray[0], ray[1] * ray[1], ray[2] * ray[2]};
    const float before_terms[3] = {var[1] * var[2], var[0] * var[2], var[0] * var[1]};
    const float area_before = dot3p(ray2, before_terms);
    const float sd[3] = {dilated[0] * dilated[0], dilated[1] * dilated[1], dilated[2] * dilated[2]};
    const float after_terms[3] = {sd[1] * sd[2], sd[0] * sd[2], sd[0] * sd[1]};
    const float area_after = dot3p(ray2, after_terms);
    opacity = p.opacities[i];
    if (p.ewa) opacity *= sqrtf(area_before / area_after);
    const float min_alpha = 1.0f / 255.0f;
    if (opacity < min_alpha) return false;
    threshold = splat_logf(opacity / min_alpha);
    const float cutoff = fminf(11.11f, 2.0f * threshold);
    const float root_mod = sqrtf(p.modifier);
    const float scale[3] = {dilated[0] * root_mod, dilated[1] * root_mod, dilated[2] * root_mod};
    const float invscale[3] = {(1.0f / dilated[0]) / root_mod, (1.0f / dilated[1]) / root_mod,
                               (1.0f / dilated[2]) / root_mod};
    // camera inside the cutoff ellipsoid: rejected
    {
      const float D[3][3] = {
          {invscale[0], 0.0f, 0.0f}, {0.0f, invscale[1], 0.0f}, {0.0f, 0.0f, invscale[2]}};
      float world2gauss[3][3];
      mat3_mul(D, R, world2gauss);
      const float to_camera[3] = {cam[0] - pm[0], cam[1] - pm[1], cam[2] - pm[2]};
      float cam_gauss[3];
      mat3_vec(world2gauss, to_camera, cam_gauss);
      if (dot3p(cam_gauss, cam_gauss) < cutoff) return false;
    }
    const float S[3][3] = {{scale[0], 0.0f, 0.0f}, {0.0f, scale[1], 0.0f}, {0.0f, 0.0f, scale[2]}};
    float SR[3][3];
    mat3_mul(S, R, SR);
    M4 world = {};
#pragma unroll
    for (int r = 0; r < 3; ++r) {
#pragma unroll
      for (int c = 0; c < 3; ++c) world.m[r][c] = SR[c][r];
      world.m[r][3] = pm[r];
    }
    world.m[3][3] = 1.0f;
    g2s = glm_matmul(clip, world);
    if (frustum_depth(g2s, 0.0f, 0.0f, W - 1.0f, H - 1.0f, false).half_distance > threshold)
      return false;
    if (p.new_aabb) {
      M4 g2v = glm_matmul(V, world);
#pragma unroll
      for (int r = 0; r < 3; ++r) g2v.m[r][3] = t[r];
      float bx[2], by[2];
      bound_axis(g2v, t, cutoff, 0, bx);
      bound_axis(g2v, t, cutoff, 1, by);
#pragma unroll
      for (int k = 0; k < 2; ++k) {
        bx[k] = p.principal_x + fx * bx[k];
        by[k] = p.principal_y + fy * by[k];
      }
      center[0] = (bx[1] + bx[0]) / 2.0f;
      center[1] = (by[1] + by[0]) / 2.0f;
      extent[0] = (bx[1] - bx[0]) / 2.0f;
      extent[1] = (by[1] - by[0]) / 2.0f;
    } else if (!screen_bounds(g2s, cutoff, center, extent)) {
      return false;
    }
    b = bounds_rect(center[0], center[1], extent[0], extent[1], gx, gy);
    count = (b.z - b.x) * (b.w - b.y);
    if (count == 0) return false;
    if (p.complete && p.tile_culling) {
      count = 0;
      for (int y = b.y; y < b.w; ++y)
        for (int x = b.x; x < b.z; ++x)
          if (frustum_depth(g2s, static_cast<float>(x * 16), static_cast<float>(y * 16), 15.0f,
                            15.0f, true).half_distance <= threshold)
            ++count;
      if (count == 0) return false;
    }
    radius = f2i(ceilf(fmaxf(extent[0], extent[1])));
    if (p.complete && radius <= 0) return false;
    return true;
  };
  const bool alive = i < p.n && front() && (!p.cooperative || radius != 0);
  if (p.cooperative) {  // the first 32 tiles; longer rectangles queue for the remainder
    const int rect_count = alive ? count : 0;
    count = warp_first_tiles<false>(min(rect_count, 32), b.x, b.y, b.z - b.x, g2s, threshold,
                                    [](int, bool, int, int, int, float) {});
    if (!alive) return;
    if (rect_count > 32) {
      p.queued[atomicAdd(p.queue_size, 1)] = i;
    } else if (count == 0) {
      return;
    }
  } else if (!alive) {
    return;
  }
  reinterpret_cast<float2*>(p.centers)[i] = make_float2(center[0], center[1]);
  reinterpret_cast<float2*>(p.rects)[i] = make_float2(extent[0], extent[1]);
  p.depths[i] = t[2];
  float4* out = reinterpret_cast<float4*>(p.transforms) + 4ll * i;
#pragma unroll
  for (int r = 0; r < 4; ++r) out[r] = make_float4(g2s.m[r][0], g2s.m[r][1], g2s.m[r][2], g2s.m[r][3]);
  p.opacity_out[i] = opacity;
  p.radii[i] = radius;
  p.tiles[i] = count;
  if ((p.complete || p.cooperative) && radius != 0) {
    if (p.sort_order != 0) {
      const float to_camera[3] = {cam[0] - pm[0], cam[1] - pm[1], cam[2] - pm[2]};
      p.depths[i] = sqrtf(dot3p(to_camera, to_camera));
    }
    if (p.sh) {
      float color[3];
      evaluate_sh(p.sh + static_cast<long long>(i) * p.sh_k * 3, p.degree, pm, cam, color);
#pragma unroll
      for (int ch = 0; ch < 3; ++ch) {
        p.clamped[3 * i + ch] = color[ch] < 0.0f ? 1 : 0;
        p.rgb[3 * i + ch] = fmaxf(color[ch], 0.0f);
      }
    }
    p.valid[i] = 1;
  }
}

// ---- K20: the queued rectangles' tiles past the first 32 --------------------------
// One warp per queued Gaussian (grid-stride over the queue); its lanes test
// the tiles in strides of 32 and the warp sums the hits.
__global__ void __launch_bounds__(256)
    aaa_cull_remainder_kernel(const int* __restrict__ queued, const int* __restrict__ queue_size,
                              const float* __restrict__ centers, const float* __restrict__ rects,
                              const float* __restrict__ transforms,
                              const float* __restrict__ opacity, int width, int height,
                              int* __restrict__ radii, int* __restrict__ tiles,
                              unsigned char* __restrict__ valid) {
  const int lane = threadIdx.x & 31;
  const int warps = gridDim.x * (blockDim.x / 32);
  const int size = *queue_size;
  const int gx = (width + 15) / 16, gy = (height + 15) / 16;
  for (int slot = blockIdx.x * (blockDim.x / 32) + (threadIdx.x >> 5); slot < size; slot += warps) {
    const int i = queued[slot];
    const float2 c = reinterpret_cast<const float2*>(centers)[i];
    const float2 e = reinterpret_cast<const float2*>(rects)[i];
    const int4 b = bounds_rect(c.x, c.y, e.x, e.y, gx, gy);
    const int rect_width = b.z - b.x, rect_count = rect_width * (b.w - b.y);
    const M4 g = load_m4(transforms, i);
    const float threshold = splat_logf(opacity[i] / (1.0f / 255.0f));
    int count = 0;
    for (int t = 32 + lane; t < rect_count; t += 32) {
      const int x = b.x + t % rect_width, y = b.y + t / rect_width;
      if (frustum_depth(g, static_cast<float>(x * 16), static_cast<float>(y * 16), 15.0f, 15.0f,
                        false).half_distance <= threshold)
        ++count;
    }
#pragma unroll
    for (int o = 16; o > 0; o >>= 1) count += __shfl_xor_sync(0xffffffffu, count, o);
    if (lane == 0) {
      const int total = tiles[i] + count;
      tiles[i] = total;
      if (total == 0) {
        radii[i] = 0;
        valid[i] = 0;
      }
    }
  }
}

// ---- metadata: aaa/metadata.py:55-91 _geometry for one view ---------------------
// Per Gaussian with radii > 0 (after the remainder cull): the half extents
// rounded up (int2), the pixel projection of the mean (fx x/z + cx, fy y/z +
// cy, z clamped to 1e-12; densification statistics only) and the effective
// opacity; zeros elsewhere.  One launch instead of the reference's Torch
// matmul and masks.
__global__ void __launch_bounds__(256)
    aaa_metadata_kernel(int n, const float* __restrict__ view, float fx, float fy, float cx,
                        float cy, const float* __restrict__ means,
                        const float* __restrict__ rects, const int* __restrict__ radii,
                        const float* __restrict__ opacity, int* __restrict__ out_radii,
                        float* __restrict__ out_means2d, float* __restrict__ out_opacity) {
  const int i = blockIdx.x * blockDim.x + threadIdx.x;
  if (i >= n) return;
  int2 r = make_int2(0, 0);
  float2 m2 = make_float2(0.0f, 0.0f);
  float o = 0.0f;
  if (radii[i] > 0) {
    const float2 e = reinterpret_cast<const float2*>(rects)[i];
    r = make_int2(f2i(ceilf(e.x)), f2i(ceilf(e.y)));
    const float m[3] = {means[3 * i], means[3 * i + 1], means[3 * i + 2]};
    float v[3];
#pragma unroll
    for (int k = 0; k < 3; ++k)
      v[k] = ((view[4 * k] * m[0] + view[4 * k + 1] * m[1]) + view[4 * k + 2] * m[2]) +
             view[4 * k + 3];
    const float z = fmaxf(v[2], 1e-12f);
    m2 = make_float2(fx * v[0] / z + cx, fy * v[1] / z + cy);
    o = opacity[i];
  }
  reinterpret_cast<int2*>(out_radii)[i] = r;
  reinterpret_cast<float2*>(out_means2d)[i] = m2;
  out_opacity[i] = o;
}

// ---- K22: keys of every visible Gaussian's tiles ------------------------------------
// Per Gaussian i: its rectangle's tiles in row-major order -- the first 32
// tested with the sequential plane products (walked by the whole warp:
// warp_first_tiles), the rest with the fused ones --
// one pair per tile within the threshold, written from offsets[i-1] on and
// never at or past offsets[i]; the rest of that range is padding.  A pair is
// stored as three words: the tile (padding: pad_tile = 2^b - 1, b the bit
// length of the tile count, which sorts after every real tile as the
// reference's 0xffffffff does under its end_bit), the depth key and the
// Gaussian id (padding: -1).  Depth key: the float bits of screen depth + 8
// (in [7, 9] for every emitted pair: the depth lies in the frustum's
// [-1, 1]) minus the bits of 7.0, a 22-bit order-preserving key.
constexpr uint32_t kDepthKeyBase = 0x40E00000u;  // bits of 7.0f
constexpr uint32_t kDepthKeyMax = 0x41100000u - kDepthKeyBase;  // 9.0f

SPLAT_DEV uint32_t depth_key(float depth) {
  uint32_t bits = __float_as_uint(depth + 8.0f);
  bits = bits < kDepthKeyBase ? kDepthKeyBase : (bits > 0x41100000u ? 0x41100000u : bits);
  return bits - kDepthKeyBase;
}

__global__ void __launch_bounds__(128)
    aaa_emit_kernel(int n, const float* __restrict__ centers, const float* __restrict__ rects,
                    const int* __restrict__ radii, const float* __restrict__ transforms,
                    const float* __restrict__ opacity, const int* __restrict__ offsets, int width,
                    int height, uint32_t pad_tile, long long num_pairs,
                    uint32_t* __restrict__ tile_out, uint32_t* __restrict__ depth_out,
                    int* __restrict__ id_out) {
  const unsigned full = 0xffffffffu;
  const int lane = threadIdx.x & 31;
  const int i = blockIdx.x * blockDim.x + threadIdx.x;  // rounded up to whole warps
  const int gx = (width + 15) / 16, gy = (height + 15) / 16;
  const bool active = i < n && radii[i] > 0;
  int4 b = make_int4(0, 0, 0, 0);
  int rw = 0, count = 0;
  long long off = 0, stop = 0;
  float threshold = 0.0f;
  M4 g = {};
  if (active) {
    const float2 c = reinterpret_cast<const float2*>(centers)[i];
    const float2 e = reinterpret_cast<const float2*>(rects)[i];
    b = bounds_rect(c.x, c.y, e.x, e.y, gx, gy);
    rw = b.z - b.x;
    count = rw * (b.w - b.y);
    off = i ? offsets[i - 1] : 0;
    stop = offsets[i];
    threshold = splat_logf(opacity[i] / (1.0f / 255.0f));
    g = load_m4(transforms, i);
  }
  {  // the first 32 tiles of every rectangle, walked by the whole warp
    const long long first_off = off;
    const int hits = warp_first_tiles<true>(
        active ? min(count, 32) : 0, b.x, b.y, rw, g, threshold,
        [&](int owner, bool pass, int rank, int x, int y, float depth) {
          const long long target = __shfl_sync(full, first_off, owner) + rank;
          const long long end = __shfl_sync(full, stop, owner);
          const int id = __shfl_sync(full, i, owner);
          if (pass && target < end && target < num_pairs) {
            tile_out[target] = static_cast<uint32_t>(y * gx + x);
            depth_out[target] = depth_key(depth);
            id_out[target] = id;
          }
        });
    off = first_off + hits;
  }
  // long rectangles: the warp takes them one owner at a time, 32 tiles per
  // step, and ranks each step's hits by ballot (row-major order kept)
  unsigned remaining = __ballot_sync(full, active && count > 32);
  while (remaining) {
    const int owner = __ffs(remaining) - 1;
    const int id = __shfl_sync(full, i, owner);
    const int x0 = __shfl_sync(full, b.x, owner), y0 = __shfl_sync(full, b.y, owner);
    const int row_width = __shfl_sync(full, rw, owner), total = __shfl_sync(full, count, owner);
    long long pos = __shfl_sync(full, off, owner);
    const long long end = __shfl_sync(full, stop, owner);
    const float limit = __shfl_sync(full, threshold, owner);
    M4 shared;
#pragma unroll
    for (int r = 0; r < 4; ++r)
#pragma unroll
      for (int c = 0; c < 4; ++c) shared.m[r][c] = __shfl_sync(full, g.m[r][c], owner);
    for (int base = 32; base < total; base += 32) {
      const int t = base + lane;
      const int x = x0 + t % row_width, y = y0 + t / row_width;
      FrustumDepth f{0.0f, 0.0f};
      bool contributes = false;
      if (t < total) {
        f = frustum_depth(shared, static_cast<float>(x * 16), static_cast<float>(y * 16), 15.0f,
                          15.0f, false);
        contributes = f.half_distance <= limit;
      }
      const unsigned hits = __ballot_sync(full, contributes);
      const long long target = pos + __popc(hits & ((1u << lane) - 1u));
      if (contributes && target < end && target < num_pairs) {
        tile_out[target] = static_cast<uint32_t>(y * gx + x);
        depth_out[target] = depth_key(f.depth);
        id_out[target] = id;
      }
      pos += __popc(hits);
    }
    if (lane == owner) off = pos;
    remaining &= remaining - 1;
  }
  if (active) {
    for (long long j = off; j < stop && j < num_pairs; ++j) {
      tile_out[j] = pad_tile;
      depth_out[j] = kDepthKeyMax;
      id_out[j] = -1;
    }
  }
}

// ---- sort of the pairs by (tile, depth key), stable ---------------------------------
// Least-significant-digit onesweep passes (binning.cuh's onesweep_kernel):
// three 8-bit passes over the 22-bit depth key carrying the pair index,
// then one or two over the tile (gathered through the index on the first),
// so equal keys keep emission order, as the reference's stable 64-bit sort.

struct DepthKeyLoader {  // first pass: key = depth key of pair idx, value = idx
  const uint32_t* keys;
  struct Shared {};
  SPLAT_DEV void prepare(uint32_t, uint32_t, Shared&) {}
  SPLAT_DEV void load(uint32_t idx, const Shared&, uint32_t& key, uint32_t& val) const {
    key = keys[idx];
    val = idx;
  }
};

struct TileGatherLoader {  // first tile pass: key = tile of the carried pair index
  const uint32_t* tiles;
  const uint32_t* vals;
  struct Shared {};
  SPLAT_DEV void prepare(uint32_t, uint32_t, Shared&) {}
  SPLAT_DEV void load(uint32_t idx, const Shared&, uint32_t& key, uint32_t& val) const {
    val = vals[idx];
    key = tiles[val];
  }
};

// 256-bin histograms of the depth key bytes 0-2 and the tile bytes 0-1
// (hist[5][256]), per block in shared memory, then added to global.
__global__ void __launch_bounds__(256)
    aaa_key_histograms_kernel(long long m, const uint32_t* __restrict__ tiles,
                              const uint32_t* __restrict__ dkeys, int tile_passes,
                              uint32_t* __restrict__ hist) {
  __shared__ uint32_t s_hist[5 * kRadix];
  for (int k = threadIdx.x; k < 5 * kRadix; k += blockDim.x) s_hist[k] = 0u;
  __syncthreads();
  for (long long p = blockIdx.x * static_cast<long long>(blockDim.x) + threadIdx.x; p < m;
       p += static_cast<long long>(gridDim.x) * blockDim.x) {
    const uint32_t d = dkeys[p], t = tiles[p];
    atomicAdd(&s_hist[0 * kRadix + (d & 255u)], 1u);
    atomicAdd(&s_hist[1 * kRadix + ((d >> 8) & 255u)], 1u);
    atomicAdd(&s_hist[2 * kRadix + ((d >> 16) & 255u)], 1u);
    atomicAdd(&s_hist[3 * kRadix + (t & 255u)], 1u);
    if (tile_passes > 1) atomicAdd(&s_hist[4 * kRadix + ((t >> 8) & 255u)], 1u);
  }
  __syncthreads();
  for (int k = threadIdx.x; k < 5 * kRadix; k += blockDim.x)
    if (s_hist[k]) atomicAdd(&hist[k], s_hist[k]);
}

// identify_ranges (primitives/tiling.py:39-54) over the sorted tiles, which
// skips the padding tile; ranges were zeroed.  ids[j] = the Gaussian of the
// sorted pair j.
__global__ void __launch_bounds__(256)
    aaa_ranges_kernel(long long m, const uint32_t* __restrict__ sorted_tiles,
                      const uint32_t* __restrict__ sorted_pairs, const int* __restrict__ pair_ids,
                      uint32_t pad_tile, int* __restrict__ ranges, int* __restrict__ ids) {
  for (long long j = blockIdx.x * static_cast<long long>(blockDim.x) + threadIdx.x; j < m;
       j += static_cast<long long>(gridDim.x) * blockDim.x) {
    ids[j] = pair_ids[sorted_pairs[j]];
    const uint32_t current = sorted_tiles[j];
    if (j == 0) {
      if (current != pad_tile) ranges[2 * current] = 0;
    } else {
      const uint32_t previous = sorted_tiles[j - 1];
      if (current != previous) {
        if (previous != pad_tile) ranges[2 * previous + 1] = static_cast<int>(j);
        if (current != pad_tile) ranges[2 * current] = static_cast<int>(j);
      }
    }
    if (j == m - 1 && current != pad_tile) ranges[2 * current + 1] = static_cast<int>(m);
  }
}

// ---- K28: preprocessing adjoint ----------------------------------------------------
// aaa/backward_preprocess.py:130-268 preprocess_adjoint: the reference's
// analytic gradients of the opacities, means, scales and (normalised)
// quaternions from the gradients of the Gaussian-to-screen transforms
// (the replay's transposed (n,16) layout) and of the effective opacities.
// Not exact AD: the filter variance is recomputed from |view depth| /
// focal_x and held fixed, as in the reference.  Rows with radius 0 get zero
// geometry gradients and pass the opacity gradient through.

// Warp's 4x4 product, sums left to right
SPLAT_DEV void mul4(const float a[4][4], const float b[4][4], float out[4][4]) {
#pragma unroll
  for (int r = 0; r < 4; ++r)
#pragma unroll
    for (int c = 0; c < 4; ++c) {
      float acc = a[r][0] * b[0][c];
#pragma unroll
      for (int k = 1; k < 4; ++k) acc = acc + a[r][k] * b[k][c];
      out[r][c] = acc;
    }
}

// rotation with rows = GLM columns, in the adjoints' plain expression order
SPLAT_DEV void plain_rotation(float qr, float qx, float qy, float qz, float R[3][3]) {
  R[0][0] = 1.0f - 2.0f * (qy * qy + qz * qz);
  R[0][1] = 2.0f * (qx * qy + qr * qz);
  R[0][2] = 2.0f * (qx * qz - qr * qy);
  R[1][0] = 2.0f * (qx * qy - qr * qz);
  R[1][1] = 1.0f - 2.0f * (qx * qx + qz * qz);
  R[1][2] = 2.0f * (qy * qz + qr * qx);
  R[2][0] = 2.0f * (qx * qz + qr * qy);
  R[2][1] = 2.0f * (qy * qz - qr * qx);
  R[2][2] = 1.0f - 2.0f * (qx * qx + qy * qy);
}

struct AdjointParams {
  int n;
  const float* means;
  const float* scales;
  const float* quats;          // normalised, or raw when normalize_quats
  int normalize_quats;         // K28 then returns the gradient of the raw quaternions
  const float* opacities;      // raw input opacities (K28) / effective (K29)
  const int* radii;
  const float* filters;        // K29: (n) or null
  const float* view;           // transposed storage
  const float* proj;           // transposed storage
  const float* campos;
  int width, height;
  float focal;                 // K28: width / (2 tanfovx); K29: max of both focals
  float modifier;              // K29
  int ewa;
  const float* up_transforms;  // (n,16) transposed layout
  const float* up_opacity;     // (n)
  // K28 outputs
  float* grad_opacity;
  float* grad_means;
  float* grad_scales;
  float* grad_quats;
  // K29 output: 23 sums (projection 16, view column 2 (4), camera position 3)
  float* camera_sums;
};

__global__ void __launch_bounds__(128) aaa_preprocess_adjoint_kernel(AdjointParams p) {
  const int i = blockIdx.x * blockDim.x + threadIdx.x;
  if (i >= p.n) return;
  const M4 V = load_transposed(p.view), P = load_transposed(p.proj);
  const float W = static_cast<float>(p.width), H = static_cast<float>(p.height);
  const float viewport[4][4] = {{W / 2.0f, 0.0f, 0.0f, W / 2.0f - 0.5f},
                                {0.0f, H / 2.0f, 0.0f, H / 2.0f - 0.5f},
                                {0.0f, 0.0f, 1.0f, 0.0f},
                                {0.0f, 0.0f, 0.0f, 1.0f}};
  float world_to_screen[4][4], screen_t[4][4];
  mul4(viewport, P.m, world_to_screen);
#pragma unroll
  for (int r = 0; r < 4; ++r)
#pragma unroll
    for (int c = 0; c < 4; ++c) screen_t[r][c] = world_to_screen[c][r];
  const float up_o = p.up_opacity[i];
  p.grad_opacity[i] = up_o;
  float* gm = p.grad_means + 3ll * i;
  float* gs = p.grad_scales + 3ll * i;
  float* gq = p.grad_quats + 4ll * i;
  if (p.radii[i] <= 0) {
#pragma unroll
    for (int k = 0; k < 3; ++k) gm[k] = gs[k] = 0.0f;
    reinterpret_cast<float4*>(gq)[0] = make_float4(0.0f, 0.0f, 0.0f, 0.0f);
    return;
  }
  const float mean[3] = {p.means[3 * i], p.means[3 * i + 1], p.means[3 * i + 2]};
  const float view_z = ((V.m[2][0] * mean[0] + V.m[2][1] * mean[1]) + V.m[2][2] * mean[2]) + V.m[2][3];
  const float filter_scale = fabsf(view_z) / p.focal * sqrtf(0.3f);
  const float variance = filter_scale * filter_scale;
  const float scale[3] = {p.scales[3 * i], p.scales[3 * i + 1], p.scales[3 * i + 2]};
  float squared[3], dil_sq[3], dilated[3];
#pragma unroll
  for (int k = 0; k < 3; ++k) {
    squared[k] = scale[k] * scale[k];
    dil_sq[k] = squared[k] + variance;
    dilated[k] = sqrtf(dil_sq[k]);
  }
  const float4 raw_q = reinterpret_cast<const float4*>(p.quats)[i];
  const float4 q4 = p.normalize_quats ? torch_normalize4(raw_q) : raw_q;
  const float qr = q4.x, qx = q4.y, qy = q4.z, qz = q4.w;
  float R[3][3];
  plain_rotation(qr, qx, qy, qz, R);
  float up_t[4][4], world_grad[4][4];
  const float4* up = reinterpret_cast<const float4*>(p.up_transforms) + 4ll * i;
#pragma unroll
  for (int c = 0; c < 4; ++c) {
    const float4 v = up[c];  // up[16 i + 4 c + r] -> up_t[r][c]
    up_t[0][c] = v.x;
    up_t[1][c] = v.y;
    up_t[2][c] = v.z;
    up_t[3][c] = v.w;
  }
  mul4(screen_t, up_t, world_grad);
  float columns[3][3];
#pragma unroll
  for (int r = 0; r < 3; ++r)
#pragma unroll
    for (int c = 0; c < 3; ++c) columns[r][c] = world_grad[c][r];
  float mean_grad[3] = {world_grad[0][3], world_grad[1][3], world_grad[2][3]};
  float comp_scale[3] = {0.0f, 0.0f, 0.0f}, comp_dir[3] = {0.0f, 0.0f, 0.0f};
  float direction[3] = {0.0f, 0.0f, 0.0f};
  if (p.ewa) {
    const float* cam = p.campos;
    const float ray[3] = {mean[0] - cam[0], mean[1] - cam[1], mean[2] - cam[2]};
    const float len = sqrtf(dot3p(ray, ray));
#pragma unroll
    for (int k = 0; k < 3; ++k) direction[k] = ray[k] / len;
    float rotated[3];
    mat3_vec(R, direction, rotated);
    const float rs[3] = {rotated[0] * rotated[0], rotated[1] * rotated[1], rotated[2] * rotated[2]};
    const float before[3] = {squared[1] * squared[2], squared[0] * squared[2], squared[0] * squared[1]};
    const float after[3] = {dil_sq[1] * dil_sq[2], dil_sq[0] * dil_sq[2], dil_sq[0] * dil_sq[1]};
    const float a = dot3p(rs, before), b = dot3p(rs, after);
    const float compensation = sqrtf(a / b);
    const float factor = up_o * p.opacities[i] * compensation / (a * b);
    p.grad_opacity[i] = up_o * compensation;
    const float da[3] = {scale[0] * (rs[1] * squared[2] + rs[2] * squared[1]),
                         scale[1] * (rs[0] * squared[2] + rs[2] * squared[0]),
                         scale[2] * (rs[0] * squared[1] + rs[1] * squared[0])};
    const float db[3] = {scale[0] * (rs[1] * dil_sq[2] + rs[2] * dil_sq[1]),
                         scale[1] * (rs[0] * dil_sq[2] + rs[2] * dil_sq[0]),
                         scale[2] * (rs[0] * dil_sq[1] + rs[1] * dil_sq[0])};
#pragma unroll
    for (int k = 0; k < 3; ++k) {
      comp_scale[k] = factor * (b * da[k] - a * db[k]);
      comp_dir[k] = factor * (b * (rotated[k] * before[k]) - a * (rotated[k] * after[k]));
    }
    float Rt[3][3];
#pragma unroll
    for (int r = 0; r < 3; ++r)
#pragma unroll
      for (int c = 0; c < 3; ++c) Rt[r][c] = R[c][r];
    float d_dir[3];
    mat3_vec(Rt, comp_dir, d_dir);
    const float along = dot3p(direction, d_dir);
#pragma unroll
    for (int k = 0; k < 3; ++k) mean_grad[k] = mean_grad[k] + (d_dir[k] - direction[k] * along) / len;
  }
#pragma unroll
  for (int axis = 0; axis < 3; ++axis) {
    gs[axis] = scale[axis] * dot3p(R[axis], columns[axis]) / dilated[axis] + comp_scale[axis];
#pragma unroll
    for (int k = 0; k < 3; ++k)
      columns[axis][k] = columns[axis][k] * dilated[axis] + direction[k] * comp_dir[axis];
  }
#pragma unroll
  for (int k = 0; k < 3; ++k) gm[k] = mean_grad[k];
  const float (*d)[3] = columns;
  const float g0 = (2.0f * qz * (d[0][1] - d[1][0]) + 2.0f * qy * (d[2][0] - d[0][2])) +
                   2.0f * qx * (d[1][2] - d[2][1]);
  const float g1 = ((2.0f * qy * (d[1][0] + d[0][1]) + 2.0f * qz * (d[2][0] + d[0][2])) +
                    2.0f * qr * (d[1][2] - d[2][1])) - 4.0f * qx * (d[2][2] + d[1][1]);
  const float g2 = ((2.0f * qx * (d[1][0] + d[0][1]) + 2.0f * qr * (d[2][0] - d[0][2])) +
                    2.0f * qz * (d[1][2] + d[2][1])) - 4.0f * qy * (d[2][2] + d[0][0]);
  const float g3 = ((2.0f * qr * (d[0][1] - d[1][0]) + 2.0f * qx * (d[2][0] + d[0][2])) +
                    2.0f * qy * (d[1][2] + d[2][1])) - 4.0f * qz * (d[1][1] + d[0][0]);
  float4 g = make_float4(g0, g1, g2, g3);
  if (p.normalize_quats) {
    // VJP of F.normalize(x) = x / max(|x|, 1e-12) (inputs.py:252):
    // (g - n (n . g)) / |x|, or g / 1e-12 where the norm is clamped
    const float norm = sqrtf((raw_q.x * raw_q.x + raw_q.z * raw_q.z) +
                             (raw_q.y * raw_q.y + raw_q.w * raw_q.w));
    if (norm > 1e-12f) {
      const float d = ((q4.x * g.x + q4.y * g.y) + q4.z * g.z) + q4.w * g.w;
      g = make_float4((g.x - q4.x * d) / norm, (g.y - q4.y * d) / norm, (g.z - q4.z * d) / norm,
                      (g.w - q4.w * d) / norm);
    } else {
      g = make_float4(g.x / 1e-12f, g.y / 1e-12f, g.z / 1e-12f, g.w / 1e-12f);
    }
  }
  reinterpret_cast<float4*>(gq)[0] = g;
}

// ---- K29: camera adjoint -------------------------------------------------------------
// aaa/backward_camera.py:61-224 camera_adjoint (without SH: aaa.rasterize
// evaluates colours before this stage): per visible Gaussian the 23 camera
// terms -- dL/d(projection matrix) in the transposed storage (16), the
// adaptive filter's depth term times (mean, 1) (4), dL/d(camera position)
// through the EWA compensation (3) -- summed per warp with shuffles and
// added with one atomic per term and warp (the reference writes (n,23) rows
// and sums them on the host).
__global__ void __launch_bounds__(128) aaa_camera_adjoint_kernel(AdjointParams p) {
  const int i = blockIdx.x * blockDim.x + threadIdx.x;
  float row[23];
#pragma unroll
  for (int k = 0; k < 23; ++k) row[k] = 0.0f;
  if (i < p.n && p.radii[i] > 0) {
    const M4 V = load_transposed(p.view), P = load_transposed(p.proj);
    const float W = static_cast<float>(p.width), H = static_cast<float>(p.height);
    const float viewport[4][4] = {{W / 2.0f, 0.0f, 0.0f, W / 2.0f - 0.5f},
                                  {0.0f, H / 2.0f, 0.0f, H / 2.0f - 0.5f},
                                  {0.0f, 0.0f, 1.0f, 0.0f},
                                  {0.0f, 0.0f, 0.0f, 1.0f}};
    float viewport_t[4][4], clip[4][4], clip_t[4][4];
#pragma unroll
    for (int r = 0; r < 4; ++r)
#pragma unroll
      for (int c = 0; c < 4; ++c) viewport_t[r][c] = viewport[c][r];
    mul4(viewport, P.m, clip);
#pragma unroll
    for (int r = 0; r < 4; ++r)
#pragma unroll
      for (int c = 0; c < 4; ++c) clip_t[r][c] = clip[c][r];
    const float root_modifier = sqrtf(p.modifier);
    const float mean[3] = {p.means[3 * i], p.means[3 * i + 1], p.means[3 * i + 2]};
    const float depth = ((V.m[2][0] * mean[0] + V.m[2][1] * mean[1]) + V.m[2][2] * mean[2]) + V.m[2][3] * 1.0f;
    const float adaptive = 0.3f * (depth / p.focal) * (depth / p.focal);
    float variance = adaptive;
    bool filter_active = true;
    if (p.filters) {
      const float fixed = p.filters[i] * p.filters[i];
      variance = fmaxf(variance, fixed);
      filter_active = adaptive > fixed;
    }
    const float scale[3] = {p.scales[3 * i], p.scales[3 * i + 1], p.scales[3 * i + 2]};
    float squared[3], dil_sq[3], dilated[3];
#pragma unroll
    for (int k = 0; k < 3; ++k) {
      squared[k] = scale[k] * scale[k];
      dil_sq[k] = squared[k] + variance;
      dilated[k] = sqrtf(dil_sq[k]);
    }
    float4 q4 = reinterpret_cast<const float4*>(p.quats)[i];
    if (p.normalize_quats) q4 = torch_normalize4(q4);
    float R[3][3];
    plain_rotation(q4.x, q4.y, q4.z, q4.w, R);
    const float D[3][3] = {{dilated[0], 0.0f, 0.0f}, {0.0f, dilated[1], 0.0f}, {0.0f, 0.0f, dilated[2]}};
    float DR[3][3];
    mat3_mul(D, R, DR);
    float world[4][4] = {};
#pragma unroll
    for (int r = 0; r < 3; ++r) {
#pragma unroll
      for (int c = 0; c < 3; ++c) world[r][c] = DR[c][r] * root_modifier;
      world[r][3] = mean[r];
    }
    world[3][3] = 1.0f;
    float screen_gradient[4][4], world_t[4][4], tmp[4][4], projection_gradient[4][4],
        world_gradient[4][4];
    const float4* up = reinterpret_cast<const float4*>(p.up_transforms) + 4ll * i;
#pragma unroll
    for (int c = 0; c < 4; ++c) {
      const float4 v = up[c];
      screen_gradient[0][c] = v.x;
      screen_gradient[1][c] = v.y;
      screen_gradient[2][c] = v.z;
      screen_gradient[3][c] = v.w;
    }
#pragma unroll
    for (int r = 0; r < 4; ++r)
#pragma unroll
      for (int c = 0; c < 4; ++c) world_t[r][c] = world[c][r];
    mul4(viewport_t, screen_gradient, tmp);
    mul4(tmp, world_t, projection_gradient);
    mul4(clip_t, screen_gradient, world_gradient);
    float variance_gradient = 0.0f;
#pragma unroll
    for (int axis = 0; axis < 3; ++axis) {
      const float column[3] = {world_gradient[0][axis], world_gradient[1][axis], world_gradient[2][axis]};
      variance_gradient = variance_gradient + dot3p(column, R[axis]) * root_modifier / (2.0f * dilated[axis]);
    }
    float camera_gradient[3] = {0.0f, 0.0f, 0.0f};
    const float* cam = p.campos;
    const float ray[3] = {mean[0] - cam[0], mean[1] - cam[1], mean[2] - cam[2]};
    const float distance = sqrtf(dot3p(ray, ray));
    const float direction[3] = {ray[0] / distance, ray[1] / distance, ray[2] / distance};
    if (p.ewa) {
      float rotated[3];
      mat3_vec(R, direction, rotated);
      const float rs[3] = {rotated[0] * rotated[0], rotated[1] * rotated[1], rotated[2] * rotated[2]};
      const float before[3] = {squared[1] * squared[2], squared[0] * squared[2], squared[0] * squared[1]};
      const float after[3] = {dil_sq[1] * dil_sq[2], dil_sq[0] * dil_sq[2], dil_sq[0] * dil_sq[1]};
      const float a = dot3p(rs, before), b = dot3p(rs, after);
      const float factor = p.up_opacity[i] * p.opacities[i];
      float rotated_gradient[3], direction_gradient[3], Rt[3][3];
#pragma unroll
      for (int k = 0; k < 3; ++k)
        rotated_gradient[k] = factor * ((rotated[k] * before[k]) / a - (rotated[k] * after[k]) / b);
#pragma unroll
      for (int r = 0; r < 3; ++r)
#pragma unroll
        for (int c = 0; c < 3; ++c) Rt[r][c] = R[c][r];
      mat3_vec(Rt, rotated_gradient, direction_gradient);
      const float along = dot3p(direction, direction_gradient);
#pragma unroll
      for (int k = 0; k < 3; ++k)
        camera_gradient[k] = camera_gradient[k] - (direction_gradient[k] - direction[k] * along) / distance;
      const float area[3] = {dil_sq[1] + dil_sq[2], dil_sq[0] + dil_sq[2], dil_sq[0] + dil_sq[1]};
      variance_gradient = variance_gradient - 0.5f * factor * dot3p(rs, area) / b;
    }
    const float depth_gradient =
        filter_active ? variance_gradient * 0.6f * depth / (p.focal * p.focal) : 0.0f;
#pragma unroll
    for (int r = 0; r < 4; ++r) {
#pragma unroll
      for (int c = 0; c < 4; ++c) row[r * 4 + c] = projection_gradient[c][r];
      row[16 + r] = depth_gradient * (r < 3 ? mean[r] : 1.0f);
    }
#pragma unroll
    for (int k = 0; k < 3; ++k) row[20 + k] = camera_gradient[k];
  }
  const int lane = threadIdx.x & 31;
#pragma unroll
  for (int k = 0; k < 23; ++k) {
    float v = row[k];
#pragma unroll
    for (int o = 16; o > 0; o >>= 1) v += __shfl_xor_sync(0xffffffffu, v, o);
    if (lane == 0 && v != 0.0f) red_add(p.camera_sums + k, v);
  }
}

}  // namespace aaa
}  // namespace splat
