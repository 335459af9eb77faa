// Exact test of a Gaussian's cutoff ellipse against a rectangle of pixel
// centres, used by the blend kernels to drop (warp, Gaussian) visits in which
// no pixel can accept the sample.
//
// A sample is evaluated only where power = -F/2 >= cut, with the quadratic
// form F(u, v) = a u^2 + 2 b u v + c v^2 of the conic (a, b, c) at the offset
// (u, v) of the pixel centre from the Gaussian centre.  For a positive
// definite conic, min F over a rectangle is attained on a face of the
// rectangle that faces the centre (a segment from any point of the rectangle
// to the centre, along which F decreases, leaves the rectangle through such a
// face), and on a face the minimiser is the clamped stationary point.  The
// two candidate faces are the lines u = clamp(0, u0, u1) and
// v = clamp(0, v0, v1); evaluating both and taking the smaller value gives
// the minimum (a point on a non-facing line is still inside the rectangle,
// so it never undercuts the minimum).
//
// Rounding: the kernels compute the per-sample power with a relative error of
// a few ulp of S = a u^2 + c v^2, and S <= F / (1 - |rho|) with
// rho = b / sqrt(a c).  The level is therefore widened by 4e-6 / (1 - |rho|)
// (about 67 ulp per unit of that ratio) plus 1e-5 absolute, and conics with
// 1 - |rho| <= 1e-4 or that are not positive definite are never rejected.
#pragma once

#if defined(__CUDACC__)
#define SPLAT_HD __host__ __device__ __forceinline__
#else
#include <math.h>
#define SPLAT_HD inline
#endif

namespace splat {

struct EllipseBound {
  float ra;     // -b / a: minimiser of F over u for fixed v is ra * v
  float rc;     // -b / c: minimiser of F over v for fixed u is rc * u
  float level;  // reject a rectangle whose min F exceeds this
};

SPLAT_HD EllipseBound ellipse_bound(float a, float b, float c, float cut) {
  EllipseBound e{0.0f, 0.0f, INFINITY};
  if (!(cut < 0.0f)) {  // no sample of this Gaussian can pass alpha >= 1/255
    e.level = -1.0f;
    return e;
  }
  if (!(a > 0.0f) || !(c > 0.0f) || !(a * c - b * b > 0.0f)) return e;
  const float slack = 1.0f - fabsf(b) / sqrtf(a * c);
  if (!(slack > 1e-4f)) return e;
  e.ra = -b / a;
  e.rc = -b / c;
  e.level = -2.0f * cut * (1.0f + 4e-6f / slack) + 1e-5f;
  if (!(e.level < INFINITY)) e.level = INFINITY;
  return e;
}

// min F over u in [u0, u1], v in [v0, v1] (offsets of pixel centres from the
// Gaussian centre; the sign convention does not matter since F(-d) = F(d)).
SPLAT_HD float rectangle_min_form(float a, float b, float c, const EllipseBound& e, float u0,
                                  float u1, float v0, float v1) {
  const float ue = fminf(fmaxf(0.0f, u0), u1);
  const float ve = fminf(fmaxf(0.0f, v0), v1);
  const float vs = fminf(fmaxf(e.rc * ue, v0), v1);
  const float us = fminf(fmaxf(e.ra * ve, u0), u1);
  const float f1 = a * ue * ue + 2.0f * b * ue * vs + c * vs * vs;
  const float f2 = a * us * us + 2.0f * b * us * ve + c * ve * ve;
  return fminf(f1, f2);
}

}  // namespace splat
