// CPU oracle for dsl_splat's AAA-Gaussians preprocessing (test
// infrastructure only: the tests use it as the checker; the product never
// links it).
//
// Restates aaa/preprocess3d.py:17-245 (preprocess_3d): the adaptive 3D
// filter, the EWA opacity compensation, the Gaussian-to-screen transform,
// the frustum-distance cull, the perspective-correct axis bounds (or the
// screen-space quadric bounds), per-tile culling, and the long-rectangle
// queue of the load-balanced path.  The arithmetic keeps the reference's
// rounding choices (its GLM matrix products and the fmaf / separate-rounding
// split of aaa/native_geometry.py and primitives/math.py), because tile
// counts and culling flip on the last bit of those predicates.  Built with
// -ffp-contract=off, so every a*b+c below is two roundings unless fmaf says
// otherwise.  Matrices are float[4][4] with mathematical rows; the camera
// arrays arrive in the reference's transposed storage (aaa/geometry.py:18-37).

#include <cfloat>
#include <climits>
#include <cmath>
#include <cstring>

// the oracle's own natural logarithm (splat_oracle.cpp), shared with the
// golden generator so that both round the opacity threshold alike
extern "C" float oracle_logf(float);

// ---- atan2 and tan: the arithmetic both sides of the comparison use ----------
// aaa/native_geometry.py's bound_axis calls atan2f and tanf; CUDA's and the
// host libm's results may differ in the last bit, and the axis bounds feed
// integer tile counts.  The oracle and the CUDA kernels therefore both
// evaluate these two functions as written here: in double precision from
// their power series (no library call), rounded once to float.  The double
// result is within a few 1e-16 relative of the true value, so the float is
// the correctly rounded one except in (rare) near-halfway cases -- it then
// agrees with any correctly rounded libm as well.

// The constants of atan2 and tan, the nearest doubles to their exact values
// (dsl_splat_b200/csrc/trig_constants.py prints them).
// atan(i / 8)
static const double kAtanTable[9] = {
    0.0, 0.12435499454676144, 0.24497866312686414, 0.35877067027057225, 0.4636476090008061,
    0.5585993153435624, 0.6435011087932844, 0.7188299996216245, 0.7853981633974483};
// 1 / (2k + 1)
static const double kAtanSeries[8] = {
    1.0, 0.3333333333333333, 0.2, 0.14285714285714285, 0.1111111111111111, 0.09090909090909091,
    0.07692307692307693, 0.06666666666666667};
// 1 / (2j + 1)!
static const double kSinSeries[11] = {
    1.0, 0.16666666666666666, 0.008333333333333333, 0.0001984126984126984,
    2.7557319223985893e-06, 2.505210838544172e-08, 1.6059043836821613e-10,
    7.647163731819816e-13, 2.8114572543455206e-15, 8.22063524662433e-18, 1.9572941063391263e-20};
// 1 / (2j)!
static const double kCosSeries[12] = {
    1.0, 0.5, 0.041666666666666664, 0.001388888888888889, 2.48015873015873e-05,
    2.755731922398589e-07, 2.08767569878681e-09, 1.1470745597729725e-11, 4.779477332387385e-14,
    1.5619206968586225e-16, 4.110317623312165e-19, 8.896791392450574e-22};
static const double kTwoOverPi = 0.6366197723675814;

// atan(t) for 0 <= t <= 1: with c the nearest multiple of 1/8, atan(t) =
// atan(c) + atan(u), u = (t - c) / (1 + t c), |u| <= 1/16, and atan(u) from
// its alternating series to u^15 / 15 (Horner in u^2).
static double atan_unit(double t) {
  const int i = static_cast<int>(t * 8.0 + 0.5);
  const double c = i * 0.125;
  const double u = (t - c) / (1.0 + t * c);
  const double u2 = u * u;
  double p = kAtanSeries[7];
  for (int k = 6; k >= 0; --k) p = kAtanSeries[k] - u2 * p;
  return kAtanTable[i] + u * p;
}

extern "C" float oracle_atan2f(float yf, float xf) {
  const double kPi = 3.141592653589793, kHalfPi = 1.5707963267948966;
  if (std::isnan(yf) || std::isnan(xf)) return yf + xf;
  const double y = yf, x = xf;
  if (y == 0.0) return static_cast<float>(std::signbit(x) ? std::copysign(kPi, y) : y);
  if (x == 0.0) return static_cast<float>(std::copysign(kHalfPi, y));
  if (std::isinf(y) || std::isinf(x)) {
    double r;
    if (std::isinf(y) && std::isinf(x)) r = x > 0 ? kPi / 4 : 3 * kPi / 4;
    else if (std::isinf(y)) r = kHalfPi;
    else r = x > 0 ? 0.0 : kPi;
    return static_cast<float>(std::copysign(r, y));
  }
  const double ax = std::fabs(x), ay = std::fabs(y);
  double r = ay <= ax ? atan_unit(ay / ax) : kHalfPi - atan_unit(ax / ay);
  if (x < 0.0) r = kPi - r;
  return static_cast<float>(std::copysign(r, y));
}

// tan(x): x reduced by the nearest multiple k of pi/2 (pi/2 split into three
// parts of 33, 33 and 53 significant bits, so k * part is exact for the
// arguments that occur, |x| < 2^20); sin and cos of the remainder |r| <~
// pi/4 from their Taylor series (to r^21 / 21! and r^22 / 22!, Horner in
// r^2), tan = sin / cos, or -cos / sin for odd k.
extern "C" float oracle_tanf(float xf) {
  if (std::isnan(xf) || std::isinf(xf)) return xf - xf;
  const double x = xf;
  const double k = std::nearbyint(x * kTwoOverPi);
  const double r = ((x - k * 1.5707963267341256) - k * 6.077100506303966e-11) -
                   k * 2.0222662487959506e-21;
  const double r2 = r * r;
  double s = kSinSeries[10], c = kCosSeries[11];
  for (int j = 9; j >= 0; --j) s = kSinSeries[j] - r2 * s;
  for (int j = 10; j >= 0; --j) c = kCosSeries[j] - r2 * c;
  s *= r;
  const bool odd = std::fmod(std::fabs(k), 2.0) == 1.0;
  return static_cast<float>(odd ? -c / s : s / c);
}

namespace {

struct V4 {
  float v[4];
  float& operator[](int i) { return v[i]; }
  float operator[](int i) const { return v[i]; }
};

struct M4 {
  float m[4][4];
  V4 row(int r) const { return V4{{m[r][0], m[r][1], m[r][2], m[r][3]}}; }
};

// primitives/math.py:48-60 glm_matmul44: each entry
// fma(a3,b3, fma(a2,b2, fma(a0,b0, a1*b1))).
M4 glm_matmul(const M4& a, const M4& b) {
  M4 out;
  for (int i = 0; i < 4; ++i)
    for (int j = 0; j < 4; ++j)
      out.m[i][j] = std::fmaf(a.m[i][3], b.m[3][j],
                              std::fmaf(a.m[i][2], b.m[2][j],
                                        std::fmaf(a.m[i][0], b.m[0][j], a.m[i][1] * b.m[1][j])));
  return out;
}

// aaa/geometry.py:18-37 load_camera: the stored array is the transpose.
M4 load_transposed(const float* a) {
  M4 out;
  for (int r = 0; r < 4; ++r)
    for (int c = 0; c < 4; ++c) out.m[r][c] = a[c * 4 + r];
  return out;
}

// Warp matrix products as the kernel source writes them (3x3, sums left to
// right with one rounding per product and per sum).
void mat3_mul(const float a[3][3], const float b[3][3], float out[3][3]) {
  for (int r = 0; r < 3; ++r)
    for (int c = 0; c < 3; ++c) {
      float acc = a[r][0] * b[0][c];
      acc = acc + a[r][1] * b[1][c];
      acc = acc + a[r][2] * b[2][c];
      out[r][c] = acc;
    }
}

void mat3_vec(const float a[3][3], const float v[3], float out[3]) {
  for (int r = 0; r < 3; ++r) {
    float acc = a[r][0] * v[0];
    acc = acc + a[r][1] * v[1];
    acc = acc + a[r][2] * v[2];
    out[r] = acc;
  }
}

float dot3_plain(const float a[3], const float b[3]) {
  float acc = a[0] * b[0];
  acc = acc + a[1] * b[1];
  return acc + a[2] * b[2];
}

// primitives/math.py:33-45 glm_rotation (quaternion r, x, y, z).
void glm_rotation(const float* q, float R[3][3]) {
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

// aaa/native_geometry.py:87-171 frustum_depth_native: half the smallest
// squared Gaussian-space distance from the mean to the pixel rectangle's
// frustum [x, x+w] x [y, y+h] x (-1, 1), and the screen depth where it is
// reached.  The dot products fuse as the snippet writes them; `sequential`
// keeps the closer y plane's products rounded (the serial tile loop).
struct FrustumDepth {
  float half_distance, depth;
};

float fdot3(float a0, float a1, float a2, float b0, float b1, float b2) {
  return std::fmaf(a2, b2, std::fmaf(a0, b0, a1 * b1));
}

float fdot4(const V4& a, const V4& b) {
  return std::fmaf(a[0], b[0], a[1] * b[1]) + std::fmaf(a[2], b[2], a[3] * b[3]);
}

V4 ftransform(const M4& g, const V4& p) {
  return V4{{fdot4(g.row(0), p), fdot4(g.row(1), p), fdot4(g.row(2), p), fdot4(g.row(3), p)}};
}

FrustumDepth frustum_depth(const M4& g, float x, float y, float w, float h, bool sequential) {
  const float start[3] = {x, y, -1.0f}, extent[3] = {w, h, 2.0f};
  auto inside = [&](const V4& p, int dim) {
    const float delta = p[dim] - start[dim] * p[3];
    return delta > 0.0f && delta < extent[dim] * p[3];
  };
  auto plane_at = [&](int axis, float coordinate, bool far) {
    V4 out;
    for (int j = 0; j < 4; ++j)
      out[j] = (sequential && axis == 1 && !far)
                   ? g.m[axis][j] - g.m[3][j] * coordinate
                   : std::fmaf(-g.m[3][j], coordinate, g.m[axis][j]);
    return out;
  };
  const V4 mean{{g.m[0][3], g.m[1][3], g.m[2][3], g.m[3][3]}};
  V4 best_pos{{1.0f, 1.0f, 1.0f, 1.0f}};
  float best = FLT_MAX;
  if (inside(mean, 0) && inside(mean, 1) && inside(mean, 2)) {
    best = 0.0f;
    best_pos = mean;
  } else {
    const float dx = std::copysign(w * 0.5f, (mean[0] - x * mean[3]) - w * 0.5f * mean[3]);
    const float dy = std::copysign(h * 0.5f, (mean[1] - y * mean[3]) - h * 0.5f * mean[3]);
    const V4 ax = plane_at(0, x + w * 0.5f + dx, false);
    const V4 ay = plane_at(1, y + h * 0.5f + dy, false);
    // closest point of one side plane, kept if it lies on the frustum face
    auto plane = [&](const V4& a, int other) {
      const float norm = a[3] / fdot3(a[0], a[1], a[2], a[0], a[1], a[2]);
      const V4 p{{-a[0] * norm, -a[1] * norm, -a[2] * norm, 1.0f}};
      const V4 screen = ftransform(g, p);
      const float value = a[3] * norm;
      if (value < best && inside(screen, other) && inside(screen, 2)) {
        best = value;
        best_pos = screen;
      }
    };
    plane(ax, 1);
    plane(ay, 0);
    // closest point of the line where two side planes meet (Pluecker form)
    auto edge = [&](const V4& a, const V4& b) {
      const float d[3] = {a[1] * b[2] - a[2] * b[1], a[2] * b[0] - a[0] * b[2],
                          a[0] * b[1] - a[1] * b[0]};
      const float m[3] = {a[3] * b[0] - a[0] * b[3], a[3] * b[1] - a[1] * b[3],
                          a[3] * b[2] - a[2] * b[3]};
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
  return FrustumDepth{0.5f * best, best_pos[2] / best_pos[3]};
}

float pdot4(const V4& a, const V4& b) { return (a[0] * b[0] + a[1] * b[1]) + (a[2] * b[2] + a[3] * b[3]); }

V4 cw(const V4& a, const V4& b) { return V4{{a[0] * b[0], a[1] * b[1], a[2] * b[2], a[3] * b[3]}}; }

// aaa/native_geometry.py:174-213 bound_axis_native: the tangents of the two
// view-space angles (about the camera, in the axis-z plane) that bound the
// Gaussian's cutoff ellipsoid, clipped to +-(pi/2 - 1e-5) and unwrapped
// around the mean's own angle.
void bound_axis(const M4& g2v, const float mean[3], float cutoff, int axis, float out[2]) {
  const float pi = 3.14159265358979323846f;
  const float length_squared = (mean[0] * mean[0] + mean[1] * mean[1]) + mean[2] * mean[2];
  const float norm = 1.0f / std::sqrt(length_squared);
  const float direction[3] = {mean[0] * norm, mean[1] * norm, mean[2] * norm};
  const float theta_mu = oracle_atan2f(direction[axis], direction[2]);
  const V4 t{{cutoff, cutoff, cutoff, -1.0f}};
  const V4 a = g2v.row(axis), z = g2v.row(2);
  const float aa = pdot4(t, cw(a, a)), zz = pdot4(t, cw(z, z)), az = pdot4(t, cw(a, z));
  const float discriminant = az * az - zz * aa;
  float lower = -(1.57079632679489661923f - 1e-5f), upper = -lower;
  if (discriminant > 0.0f) {
    const float root = std::sqrt(discriminant);
    float lo = oracle_atan2f(-(az + root), -zz), hi = oracle_atan2f(-(az - root), -zz);
    // both angles and theta_mu lie in [-pi, pi]: a few steps at most
    for (int k = 0; k < 8 && lo > theta_mu; ++k) lo -= pi;
    for (int k = 0; k < 8 && lo < theta_mu - pi; ++k) lo += pi;
    for (int k = 0; k < 8 && hi < theta_mu; ++k) hi += pi;
    for (int k = 0; k < 8 && hi > theta_mu + pi; ++k) hi -= pi;
    auto wrap = [&](float theta) {
      theta = std::fmod(theta, 2.0f * pi);
      if (theta > pi) theta -= 2.0f * pi;
      if (theta <= -pi) theta += 2.0f * pi;
      return theta;
    };
    const float nl = wrap(lo), nh = wrap(hi);
    if (theta_mu < 0.0f && std::fabs(nl) < std::fabs(nh)) {
      lo += 2.0f * pi;
      hi += 2.0f * pi;
    } else if (theta_mu > 0.0f && std::fabs(nh) < std::fabs(nl)) {
      lo -= 2.0f * pi;
      hi -= 2.0f * pi;
    }
    lower = std::fmax(lower, lo);
    upper = std::fmin(upper, hi);
  }
  out[0] = oracle_tanf(lower);
  out[1] = oracle_tanf(upper);
}

// aaa/native_geometry.py:224-247 screen_bounds_native: centre and half
// extent of the cutoff quadric's screen projection; false when the quadric
// is not bounded in front of the camera or leaves the depth range.
bool screen_bounds(const M4& g2s, float cutoff, float center[2], float extent[2]) {
  const V4 t{{cutoff, cutoff, cutoff, -1.0f}};
  const V4 x = g2s.row(0), y = g2s.row(1), z = g2s.row(2), w = g2s.row(3);
  const float s = pdot4(t, cw(w, w));
  if (s >= 0.0f) return false;
  const float inv = 1.0f / s;
  const V4 f{{inv * t[0], inv * t[1], inv * t[2], inv * t[3]}};
  const float px = pdot4(f, cw(x, w)), py = pdot4(f, cw(y, w)), pz = pdot4(f, cw(z, w));
  const float hz = pz * pz - pdot4(f, cw(z, z));
  const float ez = std::sqrt(std::fmax(hz, 0.0f));
  if (pz - ez < -1.0f || pz + ez > 1.0f) return false;
  const float hx = px * px - pdot4(f, cw(x, x)), hy = py * py - pdot4(f, cw(y, y));
  center[0] = px;
  center[1] = py;
  extent[0] = std::sqrt(std::fmax(hx, 0.0f));
  extent[1] = std::sqrt(std::fmax(hy, 0.0f));
  return extent[0] >= 0.0f;
}

// float -> int as the kernels convert: truncation, NaN -> 0, saturating.
int to_int(float v) {
  if (std::isnan(v)) return 0;
  if (v >= 2147483648.0f) return INT_MAX;
  if (v <= -2147483648.0f) return INT_MIN;
  return static_cast<int>(v);
}

int clampi(int v, int lo, int hi) { return v < lo ? lo : (v > hi ? hi : v); }

// primitives/sh.py:141-180 evaluate_sh, in its own term order: constants
// times direction products first, then times the coefficient, each term
// added or subtracted in turn, plus 0.5.
void evaluate_sh(const float* coeffs, int degree, const float mean[3], const float camera[3],
                 float out[3]) {
  const float diff[3] = {mean[0] - camera[0], mean[1] - camera[1], mean[2] - camera[2]};
  const float len = std::sqrt(dot3_plain(diff, diff));
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

}  // namespace

extern "C" {

// aaa/preprocess3d.py:17-245 preprocess_3d for one view.  Rejected rows keep
// radii = tiles = 0 and valid = 0 and leave the geometry rows untouched.
// With `cooperative`, rectangles of more than 32 tiles are appended to
// `queued` (slot order is unspecified) and keep the count of their first 32
// tiles; the follow-up collective cull decides them.
//   sh: (n, K, 3) when use_sh; filters: (n,) or null; view/proj: the 4x4
//   arrays in the reference's transposed storage; transforms: (n, 4, 4).
void oracle_aaa_preprocess(int n, const float* means, const float* scales, const float* quats,
                           const float* opacities, const float* sh, int K, int use_sh,
                           int degree, int sort_order, const float* filters,
                           const float* campos, const float* view, const float* proj,
                           int width, int height, float tanx, float tany, float principal_x,
                           float principal_y, float modifier, int ewa, int new_aabb,
                           int near_clipping, int tile_culling, int complete, int cooperative,
                           float* centers, float* rects, float* depths, float* transforms,
                           float* opacity_out, int* radii, int* tiles, float* rgb,
                           unsigned char* valid, unsigned char* clamped, int* queued,
                           int* queue_size) {
  const M4 V = load_transposed(view), P = load_transposed(proj);
  const float fx = static_cast<float>(width) / (2.0f * tanx);
  const float fy = static_cast<float>(height) / (2.0f * tany);
  const float W = static_cast<float>(width), H = static_cast<float>(height);
  M4 viewport = {};
  viewport.m[0][0] = W / 2.0f;
  viewport.m[0][3] = W / 2.0f - 0.5f;
  viewport.m[1][1] = H / 2.0f;
  viewport.m[1][3] = H / 2.0f - 0.5f;
  viewport.m[2][2] = 1.0f;
  viewport.m[3][3] = 1.0f;
  const M4 clip = glm_matmul(viewport, P);
  const int gx = (width + 15) / 16, gy = (height + 15) / 16;
  *queue_size = 0;
#pragma omp parallel for schedule(dynamic, 64)
  for (int i = 0; i < n; ++i) {
    radii[i] = 0;
    tiles[i] = 0;
    valid[i] = 0;
    const float* p = means + 3 * i;
    // primitives/math.py:74-88 glm_view_position; the load-balanced
    // specialisation rounds the z product before the sum
    float t[3];
    for (int r = 0; r < 3; ++r) {
      const float xy = std::fmaf(V.m[r][0], p[0], V.m[r][1] * p[1]);
      const float total = (!complete && r == 2) ? xy + V.m[r][2] * p[2]
                                                : std::fmaf(V.m[r][2], p[2], xy);
      t[r] = total + V.m[r][3];
    }
    if (near_clipping && t[2] < 0.2f) continue;
    float R[3][3];
    glm_rotation(quats + 4 * i, R);
    // primitives/math.py:91-97 glm_normalize3 (reciprocal length, then scale)
    const float rel[3] = {p[0] - campos[0], p[1] - campos[1], p[2] - campos[2]};
    const float inv_len = 1.0f / std::sqrt(rel[0] * rel[0] + rel[1] * rel[1] + rel[2] * rel[2]);
    const float dir[3] = {rel[0] * inv_len, rel[1] * inv_len, rel[2] * inv_len};
    float ray[3];
    mat3_vec(R, dir, ray);
    const float* s = scales + 3 * i;
    const float var[3] = {s[0] * s[0], s[1] * s[1], s[2] * s[2]};
    // primitives/math.py:63-71 glm_filter_view_depth: 3D filter from the
    // pixel footprint at this depth (0.3 px^2), or the stored filter if larger
    const float depth = std::fmaf(V.m[2][0], p[0], V.m[2][1] * p[1]) + (V.m[2][2] * p[2] + V.m[2][3]);
    const float focal = std::fmax(fx, fy);
    float filter_variance = (depth / focal) * (depth / focal) * 0.3f;
    if (filters) filter_variance = std::fmax(filters[i] * filters[i], filter_variance);
    // primitives/math.py:22-30 glm_dilated_scale
    float dilated[3];
    for (int k = 0; k < 3; ++k) dilated[k] = std::sqrt(s[k] * s[k] + filter_variance);
    const float ray2[3] = {ray[0] * ray[0], ray[1] * ray[1], ray[2] * ray[2]};
    const float before_terms[3] = {var[1] * var[2], var[0] * var[2], var[0] * var[1]};
    const float area_before = dot3_plain(ray2, before_terms);
    const float sd[3] = {dilated[0] * dilated[0], dilated[1] * dilated[1], dilated[2] * dilated[2]};
    const float after_terms[3] = {sd[1] * sd[2], sd[0] * sd[2], sd[0] * sd[1]};
    const float area_after = dot3_plain(ray2, after_terms);
    float opacity = opacities[i];
    if (ewa) opacity *= std::sqrt(area_before / area_after);
    const float min_alpha = 1.0f / 255.0f;
    if (opacity < min_alpha) continue;
    const float threshold = oracle_logf(opacity / min_alpha);
    const float cutoff = std::fmin(11.11f, 2.0f * threshold);
    const float root_mod = std::sqrt(modifier);
    const float scale[3] = {dilated[0] * root_mod, dilated[1] * root_mod, dilated[2] * root_mod};
    const float invscale[3] = {(1.0f / dilated[0]) / root_mod, (1.0f / dilated[1]) / root_mod,
                               (1.0f / dilated[2]) / root_mod};
    // camera inside the cutoff ellipsoid: rejected
    float D[3][3] = {{invscale[0], 0.0f, 0.0f}, {0.0f, invscale[1], 0.0f}, {0.0f, 0.0f, invscale[2]}};
    float world2gauss[3][3];
    mat3_mul(D, R, world2gauss);
    const float to_camera[3] = {campos[0] - p[0], campos[1] - p[1], campos[2] - p[2]};
    float cam_gauss[3];
    mat3_vec(world2gauss, to_camera, cam_gauss);
    if (dot3_plain(cam_gauss, cam_gauss) < cutoff) continue;
    // Gaussian space (unit sphere) -> world: transpose(S R) and the mean
    float S[3][3] = {{scale[0], 0.0f, 0.0f}, {0.0f, scale[1], 0.0f}, {0.0f, 0.0f, scale[2]}};
    float SR[3][3];
    mat3_mul(S, R, SR);
    M4 world = {};
    for (int r = 0; r < 3; ++r) {
      for (int c = 0; c < 3; ++c) world.m[r][c] = SR[c][r];
      world.m[r][3] = p[r];
    }
    world.m[3][3] = 1.0f;
    const M4 g2s = glm_matmul(clip, world);
    if (frustum_depth(g2s, 0.0f, 0.0f, W - 1.0f, H - 1.0f, false).half_distance > threshold) continue;
    float center[2], extent[2];
    if (new_aabb) {
      M4 g2v = glm_matmul(V, world);
      for (int r = 0; r < 3; ++r) g2v.m[r][3] = t[r];
      float bx[2], by[2];
      bound_axis(g2v, t, cutoff, 0, bx);
      bound_axis(g2v, t, cutoff, 1, by);
      for (int k = 0; k < 2; ++k) {
        bx[k] = principal_x + fx * bx[k];
        by[k] = principal_y + fy * by[k];
      }
      center[0] = (bx[1] + bx[0]) / 2.0f;
      center[1] = (by[1] + by[0]) / 2.0f;
      extent[0] = (bx[1] - bx[0]) / 2.0f;
      extent[1] = (by[1] - by[0]) / 2.0f;
    } else if (!screen_bounds(g2s, cutoff, center, extent)) {
      continue;
    }
    const int xmin = clampi(to_int(std::floor((center[0] - extent[0]) / 16.0f)), 0, gx);
    const int ymin = clampi(to_int(std::floor((center[1] - extent[1]) / 16.0f)), 0, gy);
    const int xmax = clampi(to_int(std::ceil((center[0] + extent[0]) / 16.0f)), 0, gx);
    const int ymax = clampi(to_int(std::ceil((center[1] + extent[1]) / 16.0f)), 0, gy);
    int count = (xmax - xmin) * (ymax - ymin);
    if (count == 0) continue;
    if (complete && tile_culling) {
      count = 0;
      for (int y = ymin; y < ymax; ++y)
        for (int x = xmin; x < xmax; ++x)
          if (frustum_depth(g2s, static_cast<float>(x * 16), static_cast<float>(y * 16), 15.0f,
                            15.0f, true).half_distance <= threshold)
            ++count;
      if (count == 0) continue;
    }
    const int radius = to_int(std::ceil(std::fmax(extent[0], extent[1])));
    if (complete && radius <= 0) continue;
    if (cooperative) {
      if (radius == 0) continue;
      const int rect_count = count, rect_width = xmax - xmin;
      count = 0;
      const int first = rect_count < 32 ? rect_count : 32;
      for (int k = 0; k < first; ++k) {
        const int x = xmin + k % rect_width, y = ymin + k / rect_width;
        if (frustum_depth(g2s, static_cast<float>(x * 16), static_cast<float>(y * 16), 15.0f,
                          15.0f, false).half_distance <= threshold)
          ++count;
      }
      if (rect_count > 32) {
        int slot;
#pragma omp atomic capture
        slot = (*queue_size)++;
        queued[slot] = i;
      } else if (count == 0) {
        continue;
      }
    }
    centers[2 * i] = center[0];
    centers[2 * i + 1] = center[1];
    rects[2 * i] = extent[0];
    rects[2 * i + 1] = extent[1];
    depths[i] = t[2];
    for (int r = 0; r < 4; ++r)
      for (int c = 0; c < 4; ++c) transforms[16 * i + 4 * r + c] = g2s.m[r][c];
    opacity_out[i] = opacity;
    radii[i] = radius;
    tiles[i] = count;
    if ((complete || cooperative) && radius != 0) {
      if (sort_order != 0) depths[i] = std::sqrt(dot3_plain(to_camera, to_camera));
      if (use_sh) {
        float color[3];
        evaluate_sh(sh + static_cast<long long>(i) * K * 3, degree, p, campos, color);
        for (int ch = 0; ch < 3; ++ch) {
          clamped[3 * i + ch] = color[ch] < 0.0f ? 1 : 0;
          rgb[3 * i + ch] = std::fmax(color[ch], 0.0f);
        }
      }
      valid[i] = 1;
    }
  }
}

// aaa/cooperative_culling.py:152-192 cull_remainder_3d: each queued
// Gaussian's tiles past the first 32 (the rectangle is recomputed from the
// stored centre and extent, :39-48) are added to its count; a Gaussian left
// with no tile is rejected (radius 0, not valid).
void oracle_aaa_cull_remainder(const int* queued, int queue_size, const float* centers,
                               const float* rects, const float* transforms,
                               const float* opacity, int width, int height, int* radii,
                               int* tiles, unsigned char* valid) {
  const int gx = (width + 15) / 16, gy = (height + 15) / 16;
#pragma omp parallel for schedule(dynamic, 1)
  for (int slot = 0; slot < queue_size; ++slot) {
    const int i = queued[slot];
    const float* c = centers + 2 * i;
    const float* e = rects + 2 * i;
    const int xmin = clampi(to_int(std::floor((c[0] - e[0]) / 16.0f)), 0, gx);
    const int ymin = clampi(to_int(std::floor((c[1] - e[1]) / 16.0f)), 0, gy);
    const int xmax = clampi(to_int(std::ceil((c[0] + e[0]) / 16.0f)), 0, gx);
    const int ymax = clampi(to_int(std::ceil((c[1] + e[1]) / 16.0f)), 0, gy);
    const int rect_width = xmax - xmin, rect_count = rect_width * (ymax - ymin);
    M4 g;
    for (int r = 0; r < 4; ++r)
      for (int k = 0; k < 4; ++k) g.m[r][k] = transforms[16 * i + 4 * r + k];
    const float threshold = oracle_logf(opacity[i] / (1.0f / 255.0f));
    int count = 0;
    for (int t = 32; t < rect_count; ++t) {
      const int x = xmin + t % rect_width, y = ymin + t / rect_width;
      const float lo[2] = {static_cast<float>(x * 16), static_cast<float>(y * 16)};
      const float hi[2] = {static_cast<float>(x * 16 + 15), static_cast<float>(y * 16 + 15)};
      if (frustum_depth(g, lo[0], lo[1], hi[0] - lo[0], hi[1] - lo[1], false).half_distance <= threshold)
        ++count;
    }
    tiles[i] += count;
    if (tiles[i] == 0) {
      radii[i] = 0;
      valid[i] = 0;
    }
  }
}

// aaa/binning_native.py:7-135 duplicate_aaa_default, restated serially.
// The reference's warp visits its long rectangles one owner at a time and
// ranks each 32-tile batch by ballot, so per Gaussian the output is: its
// rectangle's tiles in row-major order -- the first 32 tested with the
// sequential plane products, the rest with the fused ones -- a key for each
// tile within the threshold, written from offsets[i-1] on and never past
// offsets[i]; the rest of its range is padding (tile 0xffffffff, depth
// FLT_MAX, id -1).  Key = tile id << 32 | bits(screen depth + 8).
// offsets: inclusive scan of the visible Gaussians' tile counts.
void oracle_aaa_duplicate(int n, const float* centers, const float* rects, const int* radii,
                          const float* transforms, const float* opacity, const int* offsets,
                          int width, int height, unsigned long long* keys, int* values,
                          int num_keys) {
  const int gx = (width + 15) / 16, gy = (height + 15) / 16;
  auto key_of = [](unsigned tile, float depth) {
    unsigned bits;
    std::memcpy(&bits, &depth, 4);
    return (static_cast<unsigned long long>(tile) << 32) | bits;
  };
#pragma omp parallel for schedule(dynamic, 16)
  for (int i = 0; i < n; ++i) {
    if (radii[i] <= 0) continue;
    const float* c = centers + 2 * i;
    const float* e = rects + 2 * i;
    const int xmin = clampi(to_int(std::floor((c[0] - e[0]) / 16.0f)), 0, gx);
    const int ymin = clampi(to_int(std::floor((c[1] - e[1]) / 16.0f)), 0, gy);
    const int xmax = clampi(to_int(std::ceil((c[0] + e[0]) / 16.0f)), 0, gx);
    const int ymax = clampi(to_int(std::ceil((c[1] + e[1]) / 16.0f)), 0, gy);
    const int rect_width = xmax - xmin, count = rect_width * (ymax - ymin);
    int pos = i ? offsets[i - 1] : 0;
    const int stop = offsets[i];
    M4 g;
    for (int r = 0; r < 4; ++r)
      for (int k = 0; k < 4; ++k) g.m[r][k] = transforms[16 * i + 4 * r + k];
    const float threshold = oracle_logf(opacity[i] / (1.0f / 255.0f));
    for (int t = 0; t < count; ++t) {
      const int x = xmin + t % rect_width, y = ymin + t / rect_width;
      const FrustumDepth f = frustum_depth(g, static_cast<float>(x * 16), static_cast<float>(y * 16),
                                           15.0f, 15.0f, t < 32);
      if (f.half_distance > threshold) continue;
      if (pos < stop && pos < num_keys) {
        keys[pos] = key_of(static_cast<unsigned>(y * gx + x), f.depth + 8.0f);
        values[pos] = i;
      }
      ++pos;
    }
    for (int j = pos; j < stop && j < num_keys; ++j) {
      keys[j] = key_of(0xffffffffu, FLT_MAX);
      values[j] = -1;
    }
  }
}

// aaa/backward_preprocess.py:130-268 preprocess_adjoint: the reference's
// analytic adjoint of the preprocessing (not exact AD: the filter variance is
// recomputed from |view depth| / focal_x and held fixed, the 3D filter and
// scale modifier get no gradient, and the mean gradient is the transform's
// translation column plus the EWA compensation's direction term).
//   up_transforms: (n, 4, 4) dL/d(Gaussian-to-screen), the layout the
//   forward writes; up_opacity: dL/d(effective opacity).  Rows with radius 0
//   get zero geometry gradients and pass the opacity gradient through.
void oracle_aaa_preprocess_backward(int n, const float* means, const float* scales,
                                    const float* quats, const float* opacities, const int* radii,
                                    const float* view, const float* proj, const float* campos,
                                    int width, int height, float focal_x, int ewa,
                                    const float* up_transforms, const float* up_opacity,
                                    float* grad_opacity, float* grad_means, float* grad_scales,
                                    float* grad_quats) {
  const M4 V = load_transposed(view), P = load_transposed(proj);
  const float W = static_cast<float>(width), H = static_cast<float>(height);
  float viewport[4][4] = {{W / 2.0f, 0.0f, 0.0f, W / 2.0f - 0.5f},
                          {0.0f, H / 2.0f, 0.0f, H / 2.0f - 0.5f},
                          {0.0f, 0.0f, 1.0f, 0.0f},
                          {0.0f, 0.0f, 0.0f, 1.0f}};
  // Warp's 4x4 product, sums left to right
  auto mul4 = [](const float a[4][4], const float b[4][4], float out[4][4]) {
    for (int r = 0; r < 4; ++r)
      for (int c = 0; c < 4; ++c) {
        float acc = a[r][0] * b[0][c];
        for (int k = 1; k < 4; ++k) acc = acc + a[r][k] * b[k][c];
        out[r][c] = acc;
      }
  };
  float world_to_screen[4][4];
  mul4(viewport, P.m, world_to_screen);
  float screen_t[4][4];
  for (int r = 0; r < 4; ++r)
    for (int c = 0; c < 4; ++c) screen_t[r][c] = world_to_screen[c][r];
  const float root_03 = std::sqrt(0.3f);
#pragma omp parallel for schedule(static)
  for (int i = 0; i < n; ++i) {
    grad_opacity[i] = up_opacity[i];
    float* gm = grad_means + 3 * i;
    float* gs = grad_scales + 3 * i;
    float* gq = grad_quats + 4 * i;
    if (radii[i] <= 0) {
      for (int k = 0; k < 3; ++k) gm[k] = gs[k] = 0.0f;
      for (int k = 0; k < 4; ++k) gq[k] = 0.0f;
      continue;
    }
    const float* mean = means + 3 * i;
    const float view_z = ((V.m[2][0] * mean[0] + V.m[2][1] * mean[1]) + V.m[2][2] * mean[2]) + V.m[2][3];
    const float filter_scale = std::fabs(view_z) / focal_x * root_03;
    const float variance = filter_scale * filter_scale;
    const float* scale = scales + 3 * i;
    float squared[3], dil_sq[3], dilated[3];
    for (int k = 0; k < 3; ++k) {
      squared[k] = scale[k] * scale[k];
      dil_sq[k] = squared[k] + variance;
      dilated[k] = std::sqrt(dil_sq[k]);
    }
    // quaternion rotation with rows = GLM columns, the plain expression order
    const float* q = quats + 4 * i;
    const float qr = q[0], qx = q[1], qy = q[2], qz = q[3];
    const float R[3][3] = {
        {1.0f - 2.0f * (qy * qy + qz * qz), 2.0f * (qx * qy + qr * qz), 2.0f * (qx * qz - qr * qy)},
        {2.0f * (qx * qy - qr * qz), 1.0f - 2.0f * (qx * qx + qz * qz), 2.0f * (qy * qz + qr * qx)},
        {2.0f * (qx * qz + qr * qy), 2.0f * (qy * qz - qr * qx), 1.0f - 2.0f * (qx * qx + qy * qy)}};
    // world_grad = transpose(world_to_screen) * transpose(dL/dg2s)
    float up_t[4][4], world_grad[4][4];
    for (int r = 0; r < 4; ++r)
      for (int c = 0; c < 4; ++c) up_t[r][c] = up_transforms[16 * i + 4 * c + r];
    mul4(screen_t, up_t, world_grad);
    float columns[3][3];
    for (int r = 0; r < 3; ++r)
      for (int c = 0; c < 3; ++c) columns[r][c] = world_grad[c][r];
    float mean_grad[3] = {world_grad[0][3], world_grad[1][3], world_grad[2][3]};
    float comp_scale[3] = {0.0f, 0.0f, 0.0f}, comp_dir[3] = {0.0f, 0.0f, 0.0f};
    float direction[3] = {0.0f, 0.0f, 0.0f};
    if (ewa) {
      const float ray[3] = {mean[0] - campos[0], mean[1] - campos[1], mean[2] - campos[2]};
      const float len = std::sqrt(dot3_plain(ray, ray));
      for (int k = 0; k < 3; ++k) direction[k] = ray[k] / len;
      float rotated[3];
      mat3_vec(R, direction, rotated);
      const float rs[3] = {rotated[0] * rotated[0], rotated[1] * rotated[1], rotated[2] * rotated[2]};
      const float before[3] = {squared[1] * squared[2], squared[0] * squared[2], squared[0] * squared[1]};
      const float after[3] = {dil_sq[1] * dil_sq[2], dil_sq[0] * dil_sq[2], dil_sq[0] * dil_sq[1]};
      const float a = dot3_plain(rs, before), b = dot3_plain(rs, after);
      const float compensation = std::sqrt(a / b);
      const float factor = up_opacity[i] * opacities[i] * compensation / (a * b);
      grad_opacity[i] = up_opacity[i] * compensation;
      const float da[3] = {scale[0] * (rs[1] * squared[2] + rs[2] * squared[1]),
                           scale[1] * (rs[0] * squared[2] + rs[2] * squared[0]),
                           scale[2] * (rs[0] * squared[1] + rs[1] * squared[0])};
      const float db[3] = {scale[0] * (rs[1] * dil_sq[2] + rs[2] * dil_sq[1]),
                           scale[1] * (rs[0] * dil_sq[2] + rs[2] * dil_sq[0]),
                           scale[2] * (rs[0] * dil_sq[1] + rs[1] * dil_sq[0])};
      for (int k = 0; k < 3; ++k) {
        comp_scale[k] = factor * (b * da[k] - a * db[k]);
        comp_dir[k] = factor * (b * (rotated[k] * before[k]) - a * (rotated[k] * after[k]));
      }
      float Rt[3][3];
      for (int r = 0; r < 3; ++r)
        for (int c = 0; c < 3; ++c) Rt[r][c] = R[c][r];
      float d_dir[3];
      mat3_vec(Rt, comp_dir, d_dir);
      const float along = dot3_plain(direction, d_dir);
      for (int k = 0; k < 3; ++k) mean_grad[k] = mean_grad[k] + (d_dir[k] - direction[k] * along) / len;
    }
    for (int axis = 0; axis < 3; ++axis) {
      gs[axis] = scale[axis] * dot3_plain(R[axis], columns[axis]) / dilated[axis] + comp_scale[axis];
      for (int k = 0; k < 3; ++k)
        columns[axis][k] = columns[axis][k] * dilated[axis] + direction[k] * comp_dir[axis];
    }
    for (int k = 0; k < 3; ++k) gm[k] = mean_grad[k];
    // quaternion gradient of the rotation's columns
    const float (*d)[3] = columns;
    gq[0] = (2.0f * qz * (d[0][1] - d[1][0]) + 2.0f * qy * (d[2][0] - d[0][2])) +
            2.0f * qx * (d[1][2] - d[2][1]);
    gq[1] = ((2.0f * qy * (d[1][0] + d[0][1]) + 2.0f * qz * (d[2][0] + d[0][2])) +
             2.0f * qr * (d[1][2] - d[2][1])) - 4.0f * qx * (d[2][2] + d[1][1]);
    gq[2] = ((2.0f * qx * (d[1][0] + d[0][1]) + 2.0f * qr * (d[2][0] - d[0][2])) +
             2.0f * qz * (d[1][2] + d[2][1])) - 4.0f * qy * (d[2][2] + d[0][0]);
    gq[3] = ((2.0f * qr * (d[0][1] - d[1][0]) + 2.0f * qx * (d[2][0] + d[0][2])) +
             2.0f * qy * (d[1][2] + d[2][1])) - 4.0f * qz * (d[1][1] + d[0][0]);
  }
}

// aaa/backward_camera.py:14-53 sh_basis_gradient: d(basis k)/d(direction).
static void sh_basis_gradient(const float d[3], int k, float g[3]) {
  const float x = d[0], y = d[1], z = d[2];
  auto set = [&](float c, float a, float b, float e) { g[0] = c * a; g[1] = c * b; g[2] = c * e; };
  switch (k) {
    case 0: g[0] = g[1] = g[2] = 0.0f; return;
    case 1: g[0] = 0.0f; g[1] = -0.4886025119029199f; g[2] = 0.0f; return;
    case 2: g[0] = 0.0f; g[1] = 0.0f; g[2] = 0.4886025119029199f; return;
    case 3: g[0] = -0.4886025119029199f; g[1] = 0.0f; g[2] = 0.0f; return;
    case 4: set(1.0925484305920792f, y, x, 0.0f); return;
    case 5: set(-1.0925484305920792f, 0.0f, z, y); return;
    case 6: set(0.31539156525252005f, -2.0f * x, -2.0f * y, 4.0f * z); return;
    case 7: set(-1.0925484305920792f, z, 0.0f, x); return;
    case 8: set(0.5462742152960396f, 2.0f * x, -2.0f * y, 0.0f); return;
    case 9: set(-0.5900435899266435f, 6.0f * x * y, 3.0f * (x * x - y * y), 0.0f); return;
    case 10: set(2.890611442640554f, y * z, x * z, x * y); return;
    case 11: set(0.4570457994644658f, 2.0f * x * y, x * x + 3.0f * y * y - 4.0f * z * z, -8.0f * y * z); return;
    case 12: set(0.3731763325901154f, -6.0f * x * z, -6.0f * y * z, 6.0f * z * z - 3.0f * (x * x + y * y)); return;
    case 13: set(0.4570457994644658f, 3.0f * x * x + y * y - 4.0f * z * z, 2.0f * x * y, -8.0f * x * z); return;
    case 14: set(1.445305721320277f, 2.0f * x * z, -2.0f * y * z, x * x - y * y); return;
    default: set(-0.5900435899266435f, 3.0f * (x * x - y * y), -6.0f * x * y, 0.0f); return;
  }
}

// aaa/backward_camera.py:61-224 camera_adjoint: each visible Gaussian's
// contribution to the camera gradients, 23 floats -- dL/d(projection
// matrix) in the reference's transposed storage (16), the adaptive filter's
// depth term times (mean, 1) (4), dL/d(camera position) through the EWA
// compensation and the SH view direction (3).  The host sums the rows.
//   up_colors: (n*3) dL/d(SH colour), masked where the forward clamped.
void oracle_aaa_camera_backward(int n, const float* means, const float* scales, const float* quats,
                                const float* filters, const int* radii,
                                const float* effective_opacity, const float* view,
                                const float* proj, const float* campos, int width, int height,
                                float focal, float modifier, int ewa, const float* up_transforms,
                                const float* up_opacity, const float* sh, int K, int degree,
                                const unsigned char* clamped, const float* up_colors,
                                float* rows) {
  const M4 V = load_transposed(view), P = load_transposed(proj);
  const float W = static_cast<float>(width), H = static_cast<float>(height);
  const float viewport[4][4] = {{W / 2.0f, 0.0f, 0.0f, W / 2.0f - 0.5f},
                                {0.0f, H / 2.0f, 0.0f, H / 2.0f - 0.5f},
                                {0.0f, 0.0f, 1.0f, 0.0f},
                                {0.0f, 0.0f, 0.0f, 1.0f}};
  auto mul4 = [](const float a[4][4], const float b[4][4], float out[4][4]) {
    for (int r = 0; r < 4; ++r)
      for (int c = 0; c < 4; ++c) {
        float acc = a[r][0] * b[0][c];
        for (int k = 1; k < 4; ++k) acc = acc + a[r][k] * b[k][c];
        out[r][c] = acc;
      }
  };
  auto transpose4 = [](const float a[4][4], float out[4][4]) {
    for (int r = 0; r < 4; ++r)
      for (int c = 0; c < 4; ++c) out[r][c] = a[c][r];
  };
  float viewport_t[4][4], clip[4][4], clip_t[4][4];
  transpose4(viewport, viewport_t);
  mul4(viewport, P.m, clip);
  transpose4(clip, clip_t);
  const float root_modifier = std::sqrt(modifier);
#pragma omp parallel for schedule(static)
  for (int i = 0; i < n; ++i) {
    float* row = rows + 23 * i;
    if (radii[i] <= 0) {
      for (int k = 0; k < 23; ++k) row[k] = 0.0f;
      continue;
    }
    const float* mean = means + 3 * i;
    const float depth = ((V.m[2][0] * mean[0] + V.m[2][1] * mean[1]) + V.m[2][2] * mean[2]) + V.m[2][3] * 1.0f;
    const float adaptive = 0.3f * (depth / focal) * (depth / focal);
    float variance = adaptive;
    bool filter_active = true;
    if (filters) {
      const float fixed = filters[i] * filters[i];
      variance = std::fmax(variance, fixed);
      filter_active = adaptive > fixed;
    }
    const float* scale = scales + 3 * i;
    float squared[3], dil_sq[3], dilated[3];
    for (int k = 0; k < 3; ++k) {
      squared[k] = scale[k] * scale[k];
      dil_sq[k] = squared[k] + variance;
      dilated[k] = std::sqrt(dil_sq[k]);
    }
    const float* q = quats + 4 * i;
    const float qr = q[0], qx = q[1], qy = q[2], qz = q[3];
    const float R[3][3] = {
        {1.0f - 2.0f * (qy * qy + qz * qz), 2.0f * (qx * qy + qr * qz), 2.0f * (qx * qz - qr * qy)},
        {2.0f * (qx * qy - qr * qz), 1.0f - 2.0f * (qx * qx + qz * qz), 2.0f * (qy * qz + qr * qx)},
        {2.0f * (qx * qz + qr * qy), 2.0f * (qy * qz - qr * qx), 1.0f - 2.0f * (qx * qx + qy * qy)}};
    float D[3][3] = {{dilated[0], 0.0f, 0.0f}, {0.0f, dilated[1], 0.0f}, {0.0f, 0.0f, dilated[2]}};
    float DR[3][3];
    mat3_mul(D, R, DR);
    float world[4][4] = {};
    for (int r = 0; r < 3; ++r) {
      for (int c = 0; c < 3; ++c) world[r][c] = DR[c][r] * root_modifier;
      world[r][3] = mean[r];
    }
    world[3][3] = 1.0f;
    float screen_gradient[4][4], world_t[4][4], tmp[4][4], projection_gradient[4][4], world_gradient[4][4];
    for (int r = 0; r < 4; ++r)
      for (int c = 0; c < 4; ++c) screen_gradient[r][c] = up_transforms[16 * i + 4 * c + r];
    transpose4(world, world_t);
    mul4(viewport_t, screen_gradient, tmp);
    mul4(tmp, world_t, projection_gradient);
    mul4(clip_t, screen_gradient, world_gradient);
    float variance_gradient = 0.0f;
    for (int axis = 0; axis < 3; ++axis) {
      const float column[3] = {world_gradient[0][axis], world_gradient[1][axis], world_gradient[2][axis]};
      variance_gradient = variance_gradient + dot3_plain(column, R[axis]) * root_modifier / (2.0f * dilated[axis]);
    }
    float camera_gradient[3] = {0.0f, 0.0f, 0.0f};
    const float ray[3] = {mean[0] - campos[0], mean[1] - campos[1], mean[2] - campos[2]};
    const float distance = std::sqrt(dot3_plain(ray, ray));
    const float direction[3] = {ray[0] / distance, ray[1] / distance, ray[2] / distance};
    float Rt[3][3];
    for (int r = 0; r < 3; ++r)
      for (int c = 0; c < 3; ++c) Rt[r][c] = R[c][r];
    auto tangent_step = [&](const float g[3]) {  // camera -= (g - d (d.g)) / distance
      const float along = dot3_plain(direction, g);
      for (int k = 0; k < 3; ++k)
        camera_gradient[k] = camera_gradient[k] - (g[k] - direction[k] * along) / distance;
    };
    if (ewa) {
      float rotated[3];
      mat3_vec(R, direction, rotated);
      const float rs[3] = {rotated[0] * rotated[0], rotated[1] * rotated[1], rotated[2] * rotated[2]};
      const float before[3] = {squared[1] * squared[2], squared[0] * squared[2], squared[0] * squared[1]};
      const float after[3] = {dil_sq[1] * dil_sq[2], dil_sq[0] * dil_sq[2], dil_sq[0] * dil_sq[1]};
      const float a = dot3_plain(rs, before), b = dot3_plain(rs, after);
      const float factor = up_opacity[i] * effective_opacity[i];
      float rotated_gradient[3], direction_gradient[3];
      for (int k = 0; k < 3; ++k)
        rotated_gradient[k] = factor * ((rotated[k] * before[k]) / a - (rotated[k] * after[k]) / b);
      mat3_vec(Rt, rotated_gradient, direction_gradient);
      tangent_step(direction_gradient);
      const float area[3] = {dil_sq[1] + dil_sq[2], dil_sq[0] + dil_sq[2], dil_sq[0] + dil_sq[1]};
      variance_gradient = variance_gradient - 0.5f * factor * dot3_plain(rs, area) / b;
    }
    if (sh) {
      float color_grad[3];
      for (int c = 0; c < 3; ++c) color_grad[c] = clamped[3 * i + c] ? 0.0f : up_colors[3 * i + c];
      float direction_grad[3] = {0.0f, 0.0f, 0.0f};
      const int count = (degree + 1) * (degree + 1);
      for (int k = 0; k < count; ++k) {
        const float* coeff = sh + (static_cast<long long>(i) * K + k) * 3;
        const float weight = dot3_plain(coeff, color_grad);
        float basis[3];
        sh_basis_gradient(direction, k, basis);
        for (int c = 0; c < 3; ++c) direction_grad[c] = direction_grad[c] + weight * basis[c];
      }
      tangent_step(direction_grad);
    }
    const float depth_gradient = filter_active ? variance_gradient * 0.6f * depth / (focal * focal) : 0.0f;
    for (int r = 0; r < 4; ++r) {
      for (int c = 0; c < 4; ++c) row[r * 4 + c] = projection_gradient[c][r];
      row[16 + r] = depth_gradient * (r < 3 ? mean[r] : 1.0f);
    }
    for (int k = 0; k < 3; ++k) row[20 + k] = camera_gradient[k];
  }
}

}  // extern "C"
