// gs3d projection + SH backward (one launch per view).
//
// The hand-derived VJP of projection_loss (gs3d/projection.py:198-285) with
// the reference's custom adjoints for the Jacobian clamp
// (splatting/geometry.py:42-51), the regularised inverse covariance
// (splatting/geometry.py:61-71) and the quaternion rotation
// (splatting/math.py:13-28), fused with the SH VJP (primitives/sh.py:82-138)
// and the VJP of the quaternion normalisation (inputs.py:252).
//
// This translation unit is compiled with multiply-add contraction
// (-fmad=true), unlike the forward kernels: its outputs are gradients,
// compared within a relative tolerance, and contraction removes a large part
// of the VJP's floating-point instructions.
//
// Pipeline.  A warp owns a chunk of 32 consecutive Gaussians at a time and
// walks its chunks with a grid stride.  The inputs of a chunk (SH rows, radii,
// means, quaternions, scales and the upstream gradients: about 300 bytes per
// Gaussian at degree 3) are copied into one of two per-warp shared-memory
// stages with 16-byte cp.async while the warp computes the chunk before it,
// so loads stay in flight during the arithmetic.  The SH gradient rows are
// written over the staged SH rows and leave with coalesced 16-byte stores.
#include <algorithm>

#include "host_runtime.h"
#include "project.cuh"
#include "rade_project.cuh"
#include "splat_common.cuh"

namespace splat {

// The inputs of one Gaussian's projection VJP.
struct VjpInput {
  float m0, m1, m2;  // mean
  float4 q;          // normalised quaternion (w, x, y, z)
  float s[3];        // scales
  float2 sc;         // dL/dcenter
  float4 sq;         // dL/dconic (a, b, c) and dL/dopacity
};

// Hand-derived VJP of gs3d/projection.py:198-210 projection_loss for one
// visible Gaussian.  Returns grads through the out-parameters; camera
// partials are added into cv (view, 16) and cp (proj, 16).
SPLAT_DEV void projection_vjp(const ProjectBackwardParams& p, const VjpInput& in, float gm[3],
                              float gq[4], float gs[3], float cv[16], float cp[16]) {
  const float fx = p.K[0], fy = p.K[4];
  const float* view = p.view;
  const float* proj = p.proj;
  const float4 q = in.q;
  const float* s = in.s;
  const float2 sc = in.sc;
  const float4 sq = in.sq;
  const float m0 = in.m0, m1 = in.m1, m2 = in.m2;
  const float m[3] = {m0, m1, m2};
  const float t0 = point_row(view, 0, m0, m1, m2);
  const float t1 = point_row(view, 1, m0, m1, m2);
  const float tz = point_row(view, 2, m0, m1, m2);
  const float limx = W32(1.3) * static_cast<float>(p.width) / (2.0f * fx);
  const float limy = W32(1.3) * static_cast<float>(p.height) / (2.0f * fy);
  const float xr = t0 / tz, yr = t1 / tz;
  const float tcx = wclamp(xr, -limx, limx) * tz;
  const float tcy = wclamp(yr, -limy, limy) * tz;
  const Mat3 R = glm_rotation(q.x, q.y, q.z, q.w);
  float M[3][3], Sig[3][3];
#pragma unroll
  for (int r = 0; r < 3; ++r)
#pragma unroll
    for (int c = 0; c < 3; ++c) M[r][c] = s[r] * R.m[r][c];
#pragma unroll
  for (int r = 0; r < 3; ++r)
#pragma unroll
    for (int c = 0; c < 3; ++c) Sig[r][c] = M[0][r] * M[0][c] + M[1][r] * M[1][c] + M[2][r] * M[2][c];
  const float J[3][3] = {{fx / tz, 0.0f, 0.0f},
                         {0.0f, fy / tz, 0.0f},
                         {-(fx * tcx) / (tz * tz), -(fy * tcy) / (tz * tz), 0.0f}};
  const float Wc[3][3] = {{view[0], view[4], view[8]}, {view[1], view[5], view[9]},
                          {view[2], view[6], view[10]}};
  float Tm[3][3], A[3][3], P[3][3];
#pragma unroll
  for (int r = 0; r < 3; ++r)
#pragma unroll
    for (int c = 0; c < 3; ++c) Tm[r][c] = Wc[r][0] * J[0][c] + Wc[r][1] * J[1][c] + Wc[r][2] * J[2][c];
#pragma unroll
  for (int r = 0; r < 3; ++r)
#pragma unroll
    for (int c = 0; c < 3; ++c)
      A[r][c] = Tm[0][r] * Sig[c][0] + Tm[1][r] * Sig[c][1] + Tm[2][r] * Sig[c][2];
#pragma unroll
  for (int r = 0; r < 3; ++r)
#pragma unroll
    for (int c = 0; c < 3; ++c) P[r][c] = A[r][0] * Tm[0][c] + A[r][1] * Tm[1][c] + A[r][2] * Tm[2][c];
  const float a = P[0][0] + W32(0.3), b = P[1][0], c = P[1][1] + W32(0.3);
  // adj_invert_covariance (splatting/geometry.py:61-71)
  const float det = a * c - b * b;
  const float factor = 1.0f / (det * det + W32(0.0000001));
  const float X = sq.x, Y = sq.y, Z = sq.z;
  const float da = factor * (-c * c * X + b * c * Y + (det - a * c) * Z);
  const float db = factor * (2.0f * b * c * X - (det + 2.0f * b * b) * Y + 2.0f * a * b * Z);
  const float dc = factor * (-a * a * Z + a * b * Y + (det - a * c) * X);
  const float dP[3][3] = {{da, 0.0f, 0.0f}, {db, dc, 0.0f}, {0.0f, 0.0f, 0.0f}};
  float dA[3][3], dTm[3][3], dSig[3][3];
#pragma unroll
  for (int r = 0; r < 3; ++r)
#pragma unroll
    for (int k = 0; k < 3; ++k) {
      dA[r][k] = dP[r][0] * Tm[k][0] + dP[r][1] * Tm[k][1] + dP[r][2] * Tm[k][2];
      dTm[r][k] = A[0][r] * dP[0][k] + A[1][r] * dP[1][k] + A[2][r] * dP[2][k];
    }
#pragma unroll
  for (int r = 0; r < 3; ++r)
#pragma unroll
    for (int k = 0; k < 3; ++k) {
      dTm[r][k] += Sig[0][r] * dA[k][0] + Sig[1][r] * dA[k][1] + Sig[2][r] * dA[k][2];
      dSig[r][k] = dA[0][r] * Tm[k][0] + dA[1][r] * Tm[k][1] + dA[2][r] * Tm[k][2];
    }
  float dWc[3][3], dJ[3][3];
#pragma unroll
  for (int r = 0; r < 3; ++r)
#pragma unroll
    for (int k = 0; k < 3; ++k) {
      dWc[r][k] = dTm[r][0] * J[k][0] + dTm[r][1] * J[k][1] + dTm[r][2] * J[k][2];
      dJ[r][k] = Wc[0][r] * dTm[0][k] + Wc[1][r] * dTm[1][k] + Wc[2][r] * dTm[2][k];
    }
  float dR[3][3];
#pragma unroll
  for (int r = 0; r < 3; ++r) {
    float dM[3];
#pragma unroll
    for (int k = 0; k < 3; ++k)
      dM[k] = M[r][0] * (dSig[0][k] + dSig[k][0]) + M[r][1] * (dSig[1][k] + dSig[k][1]) +
              M[r][2] * (dSig[2][k] + dSig[k][2]);
    gs[r] = dM[0] * R.m[r][0] + dM[1] * R.m[r][1] + dM[2] * R.m[r][2];
#pragma unroll
    for (int k = 0; k < 3; ++k) dR[r][k] = s[r] * dM[k];
  }
  // adj_reference_rotation (splatting/math.py:13-28)
  {
    const float qr = q.x, qx = q.y, qy = q.z, qz = q.w;
    gq[0] = 2.0f * (qz * (dR[0][1] - dR[1][0]) + qy * (dR[2][0] - dR[0][2]) + qx * (dR[1][2] - dR[2][1]));
    gq[1] = 2.0f * (qy * (dR[0][1] + dR[1][0]) + qz * (dR[0][2] + dR[2][0]) + qr * (dR[1][2] - dR[2][1])) -
            4.0f * qx * (dR[1][1] + dR[2][2]);
    gq[2] = 2.0f * (qx * (dR[0][1] + dR[1][0]) + qr * (dR[2][0] - dR[0][2]) + qz * (dR[1][2] + dR[2][1])) -
            4.0f * qy * (dR[0][0] + dR[2][2]);
    gq[3] = 2.0f * (qr * (dR[0][1] - dR[1][0]) + qx * (dR[0][2] + dR[2][0]) + qy * (dR[1][2] + dR[2][1])) -
            4.0f * qz * (dR[0][0] + dR[1][1]);
  }
  const float tz2 = tz * tz, tz3 = tz2 * tz;
  const float dtcx = dJ[2][0] * (-fx / tz2);
  const float dtcy = dJ[2][1] * (-fy / tz2);
  const float dtcz = dJ[0][0] * (-fx / tz2) + dJ[1][1] * (-fy / tz2) +
                     dJ[2][0] * (2.0f * fx * tcx / tz3) + dJ[2][1] * (2.0f * fy * tcy / tz3);
  // adj_clamp_point (splatting/geometry.py:42-51)
  const float dt[3] = {(xr >= -limx && xr <= limx) ? dtcx : 0.0f,
                       (yr >= -limy && yr <= limy) ? dtcy : 0.0f, dtcz};
#pragma unroll
  for (int j = 0; j < 3; ++j) gm[j] = view[j] * dt[0] + view[4 + j] * dt[1] + view[8 + j] * dt[2];
#pragma unroll
  for (int r = 0; r < 3; ++r) {
#pragma unroll
    for (int j = 0; j < 3; ++j) cv[r * 4 + j] += dt[r] * m[j];
    cv[r * 4 + 3] += dt[r];
  }
#pragma unroll
  for (int r = 0; r < 3; ++r)
#pragma unroll
    for (int k = 0; k < 3; ++k) cv[k * 4 + r] += dWc[r][k];
  // pixel_center (splatting/geometry.py:106-123)
  const float c0 = point_row(proj, 0, m0, m1, m2);
  const float c1 = point_row(proj, 1, m0, m1, m2);
  const float c3 = point_row(proj, 3, m0, m1, m2);
  const float iw = 1.0f / (c3 + W32(1e-7));
  const float dnx = sc.x * static_cast<float>(p.width) * 0.5f;
  const float dny = sc.y * static_cast<float>(p.height) * 0.5f;
  const float dc0 = dnx * iw, dc1 = dny * iw;
  const float diw = dnx * c0 + dny * c1;
  const float dc3 = -diw * iw * iw;
#pragma unroll
  for (int j = 0; j < 3; ++j) {
    gm[j] += proj[j] * dc0 + proj[4 + j] * dc1 + proj[12 + j] * dc3;
    cp[0 + j] += dc0 * m[j];
    cp[4 + j] += dc1 * m[j];
    cp[12 + j] += dc3 * m[j];
  }
  cp[3] += dc0;
  cp[7] += dc1;
  cp[15] += dc3;
}


constexpr int kBackwardBlock = 128;
constexpr int kBackwardWarps = kBackwardBlock / 32;

// Per-warp stage of one chunk (offsets in 32-bit words).  SH rows keep an
// odd number of 16-byte quads per row, so the eight lanes of each 16-byte
// shared-memory wavefront read their own rows on distinct banks.
template <int DEG>
struct BackwardStage {
  static constexpr bool kSh = DEG >= 0;
  static constexpr int kCols = kSh ? 3 * (DEG + 1) * (DEG + 1) : 0;  // floats of a row in use
  static constexpr int kRowQuads = kSh ? (((kCols + 3) / 4) | 1) : 0;
  static constexpr int kRow = 4 * kRowQuads;                          // row stride, floats
  static constexpr int kSh0 = 0;
  static constexpr int kRadii = kSh0 + 32 * kRow;
  static constexpr int kMeans = kRadii + 32;
  static constexpr int kQuats = kMeans + 96;
  static constexpr int kScales = kQuats + 128;
  static constexpr int kCenters = kScales + 96;
  static constexpr int kConics = kCenters + 64;
  static constexpr int kColors = kConics + 128;             // (32,3) dL/dcolors
  static constexpr int kActive = kColors + (kSh ? 96 : 0);  // (32,3) bytes
  static constexpr int kWords = kActive + (kSh ? 24 : 0);
  static_assert(kRadii % 4 == 0 && kActive % 4 == 0 && kWords % 4 == 0, "16-byte slices");
};

// Which inputs move with 16-byte cp.async (set by the host: the pointer is
// 16-byte aligned; SH rows also need whole quads, colours a row stride of 3).
// Partial chunks always use plain copies.
enum : unsigned {
  kAsyncRadii = 1u << 0,
  kAsyncMeans = 1u << 1,
  kAsyncQuats = 1u << 2,
  kAsyncScales = 1u << 3,
  kAsyncCenters = 1u << 4,
  kAsyncConics = 1u << 5,
  kAsyncColors = 1u << 6,
  kAsyncActive = 1u << 7,
  kAsyncSh = 1u << 8,
  kVectorGradSh = 1u << 9,  // grad_sh rows leave as 16-byte stores
};

SPLAT_DEV void cp_async16(void* dst, const void* src) {
  const unsigned s = static_cast<unsigned>(__cvta_generic_to_shared(dst));
  asm volatile("cp.async.cg.shared.global [%0], [%1], 16;\n" ::"r"(s), "l"(src) : "memory");
}
SPLAT_DEV void cp_async_commit() { asm volatile("cp.async.commit_group;\n" ::: "memory"); }
template <int N>
SPLAT_DEV void cp_async_wait() {
  asm volatile("cp.async.wait_group %0;\n" ::"n"(N) : "memory");
}

// words [0, count) of one chunk's slice of an input: 16-byte async copies
// (count a multiple of 4) or plain word copies.
SPLAT_DEV void stage_slice(uint32_t* dst, const void* src, int count, bool async, int lane) {
  const uint32_t* s = static_cast<const uint32_t*>(src);
  if (async) {
    for (int t = lane; t < count / 4; t += 32) cp_async16(dst + 4 * t, s + 4 * t);
  } else {
    for (int t = lane; t < count; t += 32) dst[t] = __ldg(s + t);
  }
}

template <int DEG>
SPLAT_DEV void stage_chunk(const ProjectBackwardParams& p, unsigned mask, int base, uint32_t* st,
                           int lane) {
  using L = BackwardStage<DEG>;
  const int rows = min(32, p.n - base);
  const bool full = rows == 32;
  const size_t b = static_cast<size_t>(base);
  const float* quats = p.quats_raw ? p.quats_raw : p.quats;
  stage_slice(st + L::kRadii, p.radii + b, rows, full && (mask & kAsyncRadii), lane);
  stage_slice(st + L::kMeans, p.means + 3 * b, 3 * rows, full && (mask & kAsyncMeans), lane);
  stage_slice(st + L::kQuats, quats + 4 * b, 4 * rows, full && (mask & kAsyncQuats), lane);
  stage_slice(st + L::kScales, p.scales + 3 * b, 3 * rows, full && (mask & kAsyncScales), lane);
  stage_slice(st + L::kCenters, p.seed_centers + 2 * b, 2 * rows, full && (mask & kAsyncCenters),
              lane);
  stage_slice(st + L::kConics, p.seed_conics + 4 * b, 4 * rows, full && (mask & kAsyncConics),
              lane);
  if constexpr (L::kSh) {
    if (full && (mask & kAsyncColors)) {
      stage_slice(st + L::kColors, p.seed_colors + 3 * b, 96, true, lane);
    } else {
      float* dst = reinterpret_cast<float*>(st + L::kColors);
      for (int t = lane; t < 3 * rows; t += 32) {
        const int r = t / 3;
        dst[t] = __ldg(p.seed_colors + (b + r) * p.color_stride + (t - 3 * r));
      }
    }
    uint8_t* act = reinterpret_cast<uint8_t*>(st + L::kActive);
    if (full && (mask & kAsyncActive)) {
      if (lane < 6) cp_async16(act + 16 * lane, p.active + 3 * b + 16 * lane);
    } else {
      for (int t = lane; t < 3 * rows; t += 32) act[t] = p.active[3 * b + t];
    }
    float* sh = reinterpret_cast<float*>(st + L::kSh0);
    const size_t rs = static_cast<size_t>(p.sh_k) * 3;
    if constexpr (L::kCols % 4 == 0) {
      if (full && (mask & kAsyncSh)) {
        constexpr int Q = L::kCols / 4;
#pragma unroll
        for (int j = 0; j < Q; ++j) {
          const int t = lane + 32 * j;
          const int r = t / Q, q = t - r * Q;
          cp_async16(sh + r * L::kRow + 4 * q, p.sh + (b + r) * rs + 4 * q);
        }
        return;
      }
    }
    for (int t = lane; t < rows * L::kCols; t += 32) {
      const int r = t / L::kCols, c = t - r * L::kCols;
      sh[r * L::kRow + c] = __ldg(p.sh + (b + r) * rs + c);
    }
  }
}

// The SH VJP (primitives/sh.py:82-138) of one staged row, read and
// overwritten with its coefficient gradient as 16-byte quads, four basis
// functions (twelve floats) at a time where the degree allows.
template <int DEG>
SPLAT_DEV float3 sh_vjp_quads(float* row, float d0, float d1, float d2, float3 cg) {
  constexpr int B = (DEG + 1) * (DEG + 1);
  constexpr int kGroup = B % 4 == 0 ? 4 : B;  // basis functions per group
  constexpr int kGroupQuads = (3 * kGroup + 3) / 4;
  float ux = 0.0f, uy = 0.0f, uz = 0.0f, length = 1.0f;
  if (DEG > 0) {
    length = sqrtf(d0 * d0 + d1 * d1 + d2 * d2);
    const float den = wmax(length, W32(1e-12));
    ux = d0 / den;
    uy = d1 / den;
    uz = d2 / den;
  }
  float4* r4 = reinterpret_cast<float4*>(row);
  float g0 = 0.0f, g1 = 0.0f, g2 = 0.0f;
#pragma unroll
  for (int g = 0; g < B / kGroup; ++g) {
    float c[4 * kGroupQuads];
#pragma unroll
    for (int q = 0; q < kGroupQuads; ++q) {
      const float4 v = r4[g * kGroupQuads + q];
      c[4 * q] = v.x;
      c[4 * q + 1] = v.y;
      c[4 * q + 2] = v.z;
      c[4 * q + 3] = v.w;
    }
#pragma unroll
    for (int kk = 0; kk < kGroup; ++kk) {
      const int k = g * kGroup + kk;
      const float b = sh_basis(ux, uy, uz, k);
      if (DEG > 0) {
        const float w = c[3 * kk] * cg.x + c[3 * kk + 1] * cg.y + c[3 * kk + 2] * cg.z;
        const float3 bg = sh_basis_grad(ux, uy, uz, k);
        g0 += w * bg.x;
        g1 += w * bg.y;
        g2 += w * bg.z;
      }
      c[3 * kk] = b * cg.x;
      c[3 * kk + 1] = b * cg.y;
      c[3 * kk + 2] = b * cg.z;
    }
#pragma unroll
    for (int q = 0; q < kGroupQuads; ++q)
      r4[g * kGroupQuads + q] = make_float4(c[4 * q], c[4 * q + 1], c[4 * q + 2], c[4 * q + 3]);
  }
  if (DEG == 0) return make_float3(0.0f, 0.0f, 0.0f);
  const float den = wmax(length, W32(1e-12));
  float3 dg = make_float3(g0 / den, g1 / den, g2 / den);
  if (length >= W32(1e-12)) {
    const float dot = (ux * g0 + uy * g1 + uz * g2) / length;
    dg.x -= ux * dot;
    dg.y -= uy * dot;
    dg.z -= uz * dot;
  }
  return dg;
}

SPLAT_DEV void put(float* dst, float v, bool accumulate) {
  if (accumulate)
    *dst += v;
  else
    *dst = v;
}

// The warp's SH gradient rows (staged in place of the SH rows) to grad_sh:
// kCols columns from the stage and zeros for the rest of each row.
template <int DEG>
SPLAT_DEV void store_sh_rows(const ProjectBackwardParams& p, unsigned mask, int base,
                             const uint32_t* st, int lane) {
  using L = BackwardStage<DEG>;
  const int rows = min(32, p.n - base);
  const float* sh = reinterpret_cast<const float*>(st + L::kSh0);
  const int rs = p.sh_k * 3;
  float* dst = p.grad_sh + static_cast<size_t>(base) * rs;
  const bool acc = p.accumulate != 0;
  if constexpr (L::kCols % 4 == 0) {
    if (rows == 32 && (mask & kVectorGradSh)) {
      constexpr int Q = L::kCols / 4;
      const float4* s4 = reinterpret_cast<const float4*>(sh);
      float4* d4 = reinterpret_cast<float4*>(dst);
      const int rq = rs / 4;
      if (rq == Q) {
#pragma unroll
        for (int j = 0; j < Q; ++j) {
          const int t = lane + 32 * j;
          const int r = t / Q, q = t - r * Q;
          float4 v = s4[r * L::kRowQuads + q];
          if (acc) {
            const float4 o = d4[t];
            v = make_float4(o.x + v.x, o.y + v.y, o.z + v.z, o.w + v.w);
          }
          d4[t] = v;
        }
      } else {
        for (int t = lane; t < 32 * rq; t += 32) {
          const int r = t / rq, q = t - r * rq;
          float4 v = q < Q ? s4[r * L::kRowQuads + q] : make_float4(0.0f, 0.0f, 0.0f, 0.0f);
          if (acc) {
            const float4 o = d4[t];
            v = make_float4(o.x + v.x, o.y + v.y, o.z + v.z, o.w + v.w);
          }
          d4[t] = v;
        }
      }
      return;
    }
  }
  for (int t = lane; t < rows * rs; t += 32) {
    const int r = t / rs, c = t - r * rs;
    put(dst + t, c < L::kCols ? sh[r * L::kRow + c] : 0.0f, acc);
  }
}

template <int DEG, bool CAMERA>
SPLAT_DEV void backward_chunk(const ProjectBackwardParams& p, unsigned mask, int base,
                              uint32_t* st, int lane, float* cam) {
  using L = BackwardStage<DEG>;
  const int rows = min(32, p.n - base);
  const float* sf = reinterpret_cast<const float*>(st);
  if (lane < rows) {
    const int i = base + lane;
    float gm[3] = {0.0f, 0.0f, 0.0f}, gq[4] = {0.0f, 0.0f, 0.0f, 0.0f}, gs[3] = {0.0f, 0.0f, 0.0f};
    float go = 0.0f;
    const bool visible = static_cast<int>(st[L::kRadii + lane]) > 0;
    const float m0 = sf[L::kMeans + 3 * lane], m1 = sf[L::kMeans + 3 * lane + 1],
                m2 = sf[L::kMeans + 3 * lane + 2];
    if (visible) {
      const float4 qs = reinterpret_cast<const float4*>(sf + L::kQuats)[lane];
      VjpInput in;
      in.m0 = m0;
      in.m1 = m1;
      in.m2 = m2;
      in.q = p.quats_raw ? torch_normalize4(qs) : qs;
#pragma unroll
      for (int k = 0; k < 3; ++k) in.s[k] = sf[L::kScales + 3 * lane + k];
      in.sc = reinterpret_cast<const float2*>(sf + L::kCenters)[lane];
      in.sq = reinterpret_cast<const float4*>(sf + L::kConics)[lane];
      if (CAMERA) {
        projection_vjp(p, in, gm, gq, gs, cam, cam + 16);
      } else {
        float cv_local[16], cp_local[16];
        projection_vjp(p, in, gm, gq, gs, cv_local, cp_local);
      }
      go = in.sq.w;
      if (p.quats_raw) {
        // VJP of F.normalize(x) = x / max(|x|, 1e-12) (inputs.py:252):
        // (g - n (n . g)) / |x|, or g / 1e-12 where the norm is clamped.
        const float norm = sqrtf((qs.x * qs.x + qs.z * qs.z) + (qs.y * qs.y + qs.w * qs.w));
        if (norm > W32(1e-12)) {
          const float4 n = in.q;
          const float d = n.x * gq[0] + n.y * gq[1] + n.z * gq[2] + n.w * gq[3];
          gq[0] = (gq[0] - n.x * d) / norm;
          gq[1] = (gq[1] - n.y * d) / norm;
          gq[2] = (gq[2] - n.z * d) / norm;
          gq[3] = (gq[3] - n.w * d) / norm;
        } else {
#pragma unroll
          for (int k = 0; k < 4; ++k) gq[k] = gq[k] / W32(1e-12);
        }
      }
    }
    if constexpr (L::kSh) {
      float* row = reinterpret_cast<float*>(st + L::kSh0) + lane * L::kRow;
      if (visible) {
        const float* col = sf + L::kColors + 3 * lane;
        const uint8_t* act = reinterpret_cast<const uint8_t*>(st + L::kActive) + 3 * lane;
        const float3 cg = make_float3(act[0] ? col[0] : 0.0f, act[1] ? col[1] : 0.0f,
                                      act[2] ? col[2] : 0.0f);
        float d0 = m0, d1 = m1, d2 = m2;
        if (p.campos) {
          d0 = m0 - p.campos[0];
          d1 = m1 - p.campos[1];
          d2 = m2 - p.campos[2];
        }
        const float3 dd = sh_vjp_quads<DEG>(row, d0, d1, d2, cg);
        if (DEG > 0) {
          gm[0] += dd.x;
          gm[1] += dd.y;
          gm[2] += dd.z;
          if (CAMERA && p.campos) {
            cam[32] -= dd.x;
            cam[33] -= dd.y;
            cam[34] -= dd.z;
          }
        }
      } else {
        float4* r4 = reinterpret_cast<float4*>(row);
#pragma unroll
        for (int q = 0; q < L::kRowQuads; ++q) r4[q] = make_float4(0.0f, 0.0f, 0.0f, 0.0f);
      }
    }
    const bool acc = p.accumulate != 0;
    if (p.grad_means) {
#pragma unroll
      for (int k = 0; k < 3; ++k) put(p.grad_means + 3 * static_cast<size_t>(i) + k, gm[k], acc);
    }
    if (p.grad_quats) {
      float4* o = reinterpret_cast<float4*>(p.grad_quats) + i;
      float4 v = make_float4(gq[0], gq[1], gq[2], gq[3]);
      if (acc) {
        const float4 old = *o;
        v = make_float4(old.x + v.x, old.y + v.y, old.z + v.z, old.w + v.w);
      }
      *o = v;
    }
    if (p.grad_scales) {
#pragma unroll
      for (int k = 0; k < 3; ++k) put(p.grad_scales + 3 * static_cast<size_t>(i) + k, gs[k], acc);
    }
    if (p.grad_opacities) put(p.grad_opacities + i, go, acc);
  }
  if constexpr (L::kSh) {
    __syncwarp();
    store_sh_rows<DEG>(p, mask, base, st, lane);
  }
}

template <int DEG, bool CAMERA>
__global__ void __launch_bounds__(kBackwardBlock)
    project_backward_kernel(ProjectBackwardParams p, unsigned mask) {
  using L = BackwardStage<DEG>;
  constexpr int kCam = 35;
  extern __shared__ __align__(16) uint32_t s_stage[];
  const int lane = threadIdx.x & 31, warp = threadIdx.x >> 5;
  uint32_t* stages = s_stage + static_cast<size_t>(warp) * 2 * L::kWords;
  float cam[CAMERA ? kCam : 1];
  if (CAMERA) {
#pragma unroll
    for (int j = 0; j < kCam; ++j) cam[j] = 0.0f;
  }
  const int stride = gridDim.x * kBackwardWarps * 32;
  int base = (blockIdx.x * kBackwardWarps + warp) * 32;
  if (base < p.n) stage_chunk<DEG>(p, mask, base, stages, lane);
  cp_async_commit();
  for (int k = 0; base < p.n; base += stride, ++k) {
    uint32_t* cur = stages + (k & 1) * L::kWords;
    uint32_t* next = stages + ((k + 1) & 1) * L::kWords;
    // `next` held the chunk before this one; the __syncwarp closing that
    // iteration ordered every lane's reads of it before these copies.
    if (p.n - base > stride) stage_chunk<DEG>(p, mask, base + stride, next, lane);
    cp_async_commit();
    cp_async_wait<1>();  // this chunk's copies have landed
    __syncwarp();
    backward_chunk<DEG, CAMERA>(p, mask, base, cur, lane, cam);
    __syncwarp();
  }
  cp_async_wait<0>();
  if (CAMERA) {
    // Warp shuffles, then warp leaders through shared memory, then one
    // atomic per entry per block (gs3d/projection.py:269-283).
    __shared__ float s_cam[kBackwardWarps][kCam];
#pragma unroll
    for (int j = 0; j < kCam; ++j) {
      const float v = warp_sum(cam[j]);
      if (lane == 0) s_cam[warp][j] = v;
    }
    __syncthreads();
    if (threadIdx.x < kCam) {
      float v = 0.0f;
      for (int w = 0; w < kBackwardWarps; ++w) v += s_cam[w][threadIdx.x];
      atomicAdd(p.cam_grads + threadIdx.x, v);
    }
  }
}

// ---- several views in one launch ------------------------------------------
//
// The backward of project_forward_views_kernel: per chunk of 32 Gaussians a
// warp stages the SH rows, means, quaternions and scales once, then walks
// the views, adding each view's projection VJP into registers and its SH
// coefficient gradient into a second shared-memory row; the (linear)
// normalisation VJP is applied once to the summed quaternion gradient and
// every gradient is written once.  Camera gradients are not formed here (the
// host runs the per-view kernel when they are requested).
struct ProjectBackwardViewsParams {
  ProjectBackwardParams shared;  // Gaussian inputs/outputs and settings; per-view fields unused
  int views;
  const float* viewmats;  // (views,4,4)
  const float* projs;     // (views,4,4)
  const float* Ks;        // (views,3,3)
  const float* campos;    // (views,3) or null
  const int* radii[kMaxViews];
  const float* seed_centers[kMaxViews];
  const float* seed_conics[kMaxViews];
  const float* seed_colors[kMaxViews];  // (n, color_stride); null without SH gradients
  const uint8_t* active[kMaxViews];
};

template <int DEG>
struct ViewsStage {
  using B = BackwardStage<DEG>;
  static constexpr int kSh0 = 0;                        // coefficient rows
  static constexpr int kGrad0 = kSh0 + 32 * B::kRow;    // gradient rows
  static constexpr int kMeans = kGrad0 + 32 * B::kRow;
  static constexpr int kQuats = kMeans + 96;
  static constexpr int kScales = kQuats + 128;
  static constexpr int kWords = kScales + 96;
  static_assert(kMeans % 4 == 0 && kWords % 4 == 0, "16-byte slices");
};

// sh_vjp_quads reading the coefficient row and adding the coefficient
// gradient into a separate row (primitives/sh.py:116-120 summed over views).
template <int DEG>
SPLAT_DEV float3 sh_vjp_accumulate(const float* coef, float* grad, float d0, float d1, float d2,
                                   float3 cg) {
  constexpr int B = (DEG + 1) * (DEG + 1);
  constexpr int kGroup = B % 4 == 0 ? 4 : B;
  constexpr int kGroupQuads = (3 * kGroup + 3) / 4;
  float ux = 0.0f, uy = 0.0f, uz = 0.0f, length = 1.0f;
  if (DEG > 0) {
    length = sqrtf(d0 * d0 + d1 * d1 + d2 * d2);
    const float den = wmax(length, W32(1e-12));
    ux = d0 / den;
    uy = d1 / den;
    uz = d2 / den;
  }
  const float4* c4 = reinterpret_cast<const float4*>(coef);
  float4* g4 = reinterpret_cast<float4*>(grad);
  float g0 = 0.0f, g1 = 0.0f, g2 = 0.0f;
#pragma unroll
  for (int g = 0; g < B / kGroup; ++g) {
    float c[4 * kGroupQuads], o[4 * kGroupQuads];
#pragma unroll
    for (int q = 0; q < kGroupQuads; ++q) {
      const float4 v = c4[g * kGroupQuads + q], w = g4[g * kGroupQuads + q];
      c[4 * q] = v.x;
      c[4 * q + 1] = v.y;
      c[4 * q + 2] = v.z;
      c[4 * q + 3] = v.w;
      o[4 * q] = w.x;
      o[4 * q + 1] = w.y;
      o[4 * q + 2] = w.z;
      o[4 * q + 3] = w.w;
    }
#pragma unroll
    for (int kk = 0; kk < kGroup; ++kk) {
      const int k = g * kGroup + kk;
      const float b = sh_basis(ux, uy, uz, k);
      if (DEG > 0) {
        const float w = c[3 * kk] * cg.x + c[3 * kk + 1] * cg.y + c[3 * kk + 2] * cg.z;
        const float3 bg = sh_basis_grad(ux, uy, uz, k);
        g0 += w * bg.x;
        g1 += w * bg.y;
        g2 += w * bg.z;
      }
      o[3 * kk] += b * cg.x;
      o[3 * kk + 1] += b * cg.y;
      o[3 * kk + 2] += b * cg.z;
    }
#pragma unroll
    for (int q = 0; q < kGroupQuads; ++q)
      g4[g * kGroupQuads + q] = make_float4(o[4 * q], o[4 * q + 1], o[4 * q + 2], o[4 * q + 3]);
  }
  if (DEG == 0) return make_float3(0.0f, 0.0f, 0.0f);
  const float den = wmax(length, W32(1e-12));
  float3 dg = make_float3(g0 / den, g1 / den, g2 / den);
  if (length >= W32(1e-12)) {
    const float dot = (ux * g0 + uy * g1 + uz * g2) / length;
    dg.x -= ux * dot;
    dg.y -= uy * dot;
    dg.z -= uz * dot;
  }
  return dg;
}

template <int DEG>
__global__ void __launch_bounds__(kBackwardBlock)
    project_backward_views_kernel(ProjectBackwardViewsParams vp, unsigned mask) {
  using L = ViewsStage<DEG>;
  using B = BackwardStage<DEG>;
  const ProjectBackwardParams& p = vp.shared;
  extern __shared__ __align__(16) uint32_t s_stage[];
  const int lane = threadIdx.x & 31, warp = threadIdx.x >> 5;
  uint32_t* st = s_stage + static_cast<size_t>(warp) * L::kWords;
  float* sf = reinterpret_cast<float*>(st);
  const bool sh_grads = B::kSh && p.grad_sh != nullptr;
  const int stride = gridDim.x * kBackwardWarps * 32;
  for (int base = (blockIdx.x * kBackwardWarps + warp) * 32; base < p.n; base += stride) {
    const int rows = min(32, p.n - base);
    const bool full = rows == 32;
    const size_t b = static_cast<size_t>(base);
    const float* quats = p.quats_raw ? p.quats_raw : p.quats;
    stage_slice(st + L::kMeans, p.means + 3 * b, 3 * rows, full && (mask & kAsyncMeans), lane);
    stage_slice(st + L::kQuats, quats + 4 * b, 4 * rows, full && (mask & kAsyncQuats), lane);
    stage_slice(st + L::kScales, p.scales + 3 * b, 3 * rows, full && (mask & kAsyncScales), lane);
    if constexpr (B::kSh) {
      if (sh_grads) {
        float* sh = sf + L::kSh0;
        const size_t rs = static_cast<size_t>(p.sh_k) * 3;
        bool staged = false;
        if constexpr (B::kCols % 4 == 0) {
          if (full && (mask & kAsyncSh)) {
            constexpr int Q = B::kCols / 4;
#pragma unroll
            for (int j = 0; j < Q; ++j) {
              const int t = lane + 32 * j;
              const int r = t / Q, q = t - r * Q;
              cp_async16(sh + r * B::kRow + 4 * q, p.sh + (b + r) * rs + 4 * q);
            }
            staged = true;
          }
        }
        if (!staged)
          for (int t = lane; t < rows * B::kCols; t += 32) {
            const int r = t / B::kCols, c = t - r * B::kCols;
            sh[r * B::kRow + c] = __ldg(p.sh + (b + r) * rs + c);
          }
        float4* g4 = reinterpret_cast<float4*>(sf + L::kGrad0);
        for (int t = lane; t < 32 * B::kRowQuads; t += 32) g4[t] = make_float4(0.f, 0.f, 0.f, 0.f);
      }
    }
    cp_async_commit();
    cp_async_wait<0>();
    __syncwarp();
    if (lane < rows) {
      const int i = base + lane;
      const float m0 = sf[L::kMeans + 3 * lane], m1 = sf[L::kMeans + 3 * lane + 1],
                  m2 = sf[L::kMeans + 3 * lane + 2];
      const float4 qs = reinterpret_cast<const float4*>(sf + L::kQuats)[lane];
      VjpInput in;
      in.m0 = m0;
      in.m1 = m1;
      in.m2 = m2;
      in.q = p.quats_raw ? torch_normalize4(qs) : qs;
#pragma unroll
      for (int k = 0; k < 3; ++k) in.s[k] = sf[L::kScales + 3 * lane + k];
      float gm[3] = {0.0f, 0.0f, 0.0f}, gq[4] = {0.0f, 0.0f, 0.0f, 0.0f}, gs[3] = {0.0f, 0.0f, 0.0f};
      float go = 0.0f;
      for (int v = 0; v < vp.views; ++v) {
        if (vp.radii[v][i] <= 0) continue;
        ProjectBackwardParams pv = p;
        pv.view = vp.viewmats + 16 * v;
        pv.proj = vp.projs + 16 * v;
        pv.K = vp.Ks + 9 * v;
        in.sc = reinterpret_cast<const float2*>(vp.seed_centers[v])[i];
        in.sq = reinterpret_cast<const float4*>(vp.seed_conics[v])[i];
        float vm[3], vq[4], vs[3], cv_local[16], cp_local[16];
#pragma unroll
        for (int k = 0; k < 3; ++k) vm[k] = vs[k] = 0.0f;
#pragma unroll
        for (int k = 0; k < 4; ++k) vq[k] = 0.0f;
        projection_vjp(pv, in, vm, vq, vs, cv_local, cp_local);
#pragma unroll
        for (int k = 0; k < 3; ++k) {
          gm[k] += vm[k];
          gs[k] += vs[k];
        }
#pragma unroll
        for (int k = 0; k < 4; ++k) gq[k] += vq[k];
        go += in.sq.w;
        if constexpr (B::kSh) {
          if (sh_grads) {
            const float* col = vp.seed_colors[v] + static_cast<size_t>(i) * p.color_stride;
            const uint8_t* act = vp.active[v] + 3 * static_cast<size_t>(i);
            const float3 cg = make_float3(act[0] ? col[0] : 0.0f, act[1] ? col[1] : 0.0f,
                                          act[2] ? col[2] : 0.0f);
            float d0 = m0, d1 = m1, d2 = m2;
            if (vp.campos) {
              d0 = m0 - vp.campos[3 * v];
              d1 = m1 - vp.campos[3 * v + 1];
              d2 = m2 - vp.campos[3 * v + 2];
            }
            const float3 dd = sh_vjp_accumulate<DEG>(sf + L::kSh0 + lane * B::kRow,
                                                     sf + L::kGrad0 + lane * B::kRow, d0, d1,
                                                     d2, cg);
            if (DEG > 0) {
              gm[0] += dd.x;
              gm[1] += dd.y;
              gm[2] += dd.z;
            }
          }
        }
      }
      if (p.quats_raw) {
        // the normalisation VJP is linear in the upstream gradient: applied
        // once to the sum over views
        const float norm = sqrtf((qs.x * qs.x + qs.z * qs.z) + (qs.y * qs.y + qs.w * qs.w));
        if (norm > W32(1e-12)) {
          const float4 n = in.q;
          const float d = n.x * gq[0] + n.y * gq[1] + n.z * gq[2] + n.w * gq[3];
          gq[0] = (gq[0] - n.x * d) / norm;
          gq[1] = (gq[1] - n.y * d) / norm;
          gq[2] = (gq[2] - n.z * d) / norm;
          gq[3] = (gq[3] - n.w * d) / norm;
        } else {
#pragma unroll
          for (int k = 0; k < 4; ++k) gq[k] = gq[k] / W32(1e-12);
        }
      }
      const bool acc = p.accumulate != 0;
      if (p.grad_means) {
#pragma unroll
        for (int k = 0; k < 3; ++k) put(p.grad_means + 3 * static_cast<size_t>(i) + k, gm[k], acc);
      }
      if (p.grad_quats) {
        float4* o = reinterpret_cast<float4*>(p.grad_quats) + i;
        float4 val = make_float4(gq[0], gq[1], gq[2], gq[3]);
        if (acc) {
          const float4 old = *o;
          val = make_float4(old.x + val.x, old.y + val.y, old.z + val.z, old.w + val.w);
        }
        *o = val;
      }
      if (p.grad_scales) {
#pragma unroll
        for (int k = 0; k < 3; ++k) put(p.grad_scales + 3 * static_cast<size_t>(i) + k, gs[k], acc);
      }
      if (p.grad_opacities) put(p.grad_opacities + i, go, acc);
    }
    if constexpr (B::kSh) {
      if (sh_grads) {
        __syncwarp();
        // store_sh_rows reads the gradient rows at the stage's SH offset
        store_sh_rows<DEG>(p, mask, base, st + L::kGrad0, lane);
      }
    }
    __syncwarp();
  }
}

namespace {

using host::aligned;

unsigned async_mask(const ProjectBackwardParams& p) {
  unsigned m = 0;
  if (aligned(p.radii, 16)) m |= kAsyncRadii;
  if (aligned(p.means, 16)) m |= kAsyncMeans;
  if (aligned(p.quats_raw ? p.quats_raw : p.quats, 16)) m |= kAsyncQuats;
  if (aligned(p.scales, 16)) m |= kAsyncScales;
  if (aligned(p.seed_centers, 16)) m |= kAsyncCenters;
  if (aligned(p.seed_conics, 16)) m |= kAsyncConics;
  if (p.grad_sh) {
    const int cols = 3 * (p.sh_degree + 1) * (p.sh_degree + 1);
    const bool quads = cols % 4 == 0 && (3 * p.sh_k) % 4 == 0;
    if (p.color_stride == 3 && aligned(p.seed_colors, 16)) m |= kAsyncColors;
    if (aligned(p.active, 16)) m |= kAsyncActive;
    if (quads && aligned(p.sh, 16)) m |= kAsyncSh;
    if (quads && aligned(p.grad_sh, 16)) m |= kVectorGradSh;
  }
  return m;
}

template <int DEG, bool CAMERA>
int launch(const ProjectBackwardParams& p, cudaStream_t s) {
  using L = BackwardStage<DEG>;
  const size_t smem = static_cast<size_t>(kBackwardWarps) * 2 * L::kWords * sizeof(uint32_t);
  auto kernel = project_backward_kernel<DEG, CAMERA>;
  if (cudaFuncSetAttribute(kernel, cudaFuncAttributeMaxDynamicSharedMemorySize,
                           static_cast<int>(smem)) != cudaSuccess)
    return host::check_launch("project_backward smem");
  static int resident = 0;  // blocks per SM (the same on every device of a process)
  if (resident == 0) {
    int r = 0;
    if (cudaOccupancyMaxActiveBlocksPerMultiprocessor(&r, kernel, kBackwardBlock, smem) !=
            cudaSuccess || r < 1)
      r = 1;
    resident = r;
  }
  const unsigned grid = std::min(host::blocks_for(p.n, kBackwardBlock),
                                 static_cast<unsigned>(host::sm_count() * resident));
  kernel<<<grid, kBackwardBlock, smem, host::counted(s)>>>(p, async_mask(p));
  return kOk;
}

template <bool CAMERA>
int launch_degree(const ProjectBackwardParams& p, cudaStream_t s) {
  if (p.grad_sh == nullptr) return launch<-1, CAMERA>(p, s);
  switch (p.sh_degree) {
    case 0: return launch<0, CAMERA>(p, s);
    case 1: return launch<1, CAMERA>(p, s);
    case 2: return launch<2, CAMERA>(p, s);
    case 3: return launch<3, CAMERA>(p, s);
    default: return host::fail(kInvalidArgument, "sh_degree must be in [0,3]");
  }
}

}  // namespace

template <int DEG>
int launch_views(const ProjectBackwardViewsParams& vp, cudaStream_t s) {
  using L = ViewsStage<DEG>;
  const size_t smem = static_cast<size_t>(kBackwardWarps) * L::kWords * sizeof(uint32_t);
  auto kernel = project_backward_views_kernel<DEG>;
  if (cudaFuncSetAttribute(kernel, cudaFuncAttributeMaxDynamicSharedMemorySize,
                           static_cast<int>(smem)) != cudaSuccess)
    return host::check_launch("project_backward_views smem");
  static int resident = 0;  // blocks per SM (the same on every device of a process)
  if (resident == 0) {
    int r = 0;
    if (cudaOccupancyMaxActiveBlocksPerMultiprocessor(&r, kernel, kBackwardBlock, smem) !=
            cudaSuccess || r < 1)
      r = 1;
    resident = r;
  }
  const unsigned grid = std::min(host::blocks_for(vp.shared.n, kBackwardBlock),
                                 static_cast<unsigned>(host::sm_count() * resident));
  kernel<<<grid, kBackwardBlock, smem, host::counted(s)>>>(vp, async_mask(vp.shared));
  return kOk;
}

int project_backward_views_dispatch(const ProjectBackwardViewsParams& vp, cudaStream_t s) {
  if (vp.shared.n == 0 || vp.views == 0) return kOk;
  int r;
  if (vp.shared.grad_sh == nullptr) {
    r = launch_views<-1>(vp, s);
  } else {
    switch (vp.shared.sh_degree) {
      case 0: r = launch_views<0>(vp, s); break;
      case 1: r = launch_views<1>(vp, s); break;
      case 2: r = launch_views<2>(vp, s); break;
      case 3: r = launch_views<3>(vp, s); break;
      default: return host::fail(kInvalidArgument, "sh_degree must be in [0,3]");
    }
  }
  if (r != kOk) return r;
  return host::check_launch("project_backward_views");
}

int project_backward_dispatch(const ProjectBackwardParams& p, cudaStream_t s) {
  if (p.n == 0) return kOk;
  const int r = p.cam_grads ? launch_degree<true>(p, s) : launch_degree<false>(p, s);
  if (r != kOk) return r;
  return host::check_launch("project_backward");
}

namespace {
template <int DEG>
void launch_rade_backward(const RadeProjectParams& p, cudaStream_t s) {
  // grid-stride, 128 threads (about 150 registers each: three blocks per
  // SM); a few blocks per SM keep the camera atomics per block few
  const unsigned blocks =
      std::min(host::blocks_for(p.n, 128), static_cast<unsigned>(6 * host::sm_count()));
  rade_project_backward_kernel<DEG><<<blocks, 128, 0, host::counted(s)>>>(p);
}
}  // namespace

int rade_project_backward_dispatch(const RadeProjectParams& p, cudaStream_t s) {
  if (p.n == 0) return kOk;
  if (p.sh == nullptr) {
    launch_rade_backward<-1>(p, s);
  } else {
    switch (p.sh_degree) {
      case 0: launch_rade_backward<0>(p, s); break;
      case 1: launch_rade_backward<1>(p, s); break;
      case 2: launch_rade_backward<2>(p, s); break;
      case 3: launch_rade_backward<3>(p, s); break;
      default: return host::fail(kInvalidArgument, "sh_degree must be in [0,3]");
    }
  }
  return host::check_launch("rade_project_backward");
}

}  // namespace splat

using namespace splat;

extern "C" int splat_project_backward_views(
    int views, int n, const float* means, const float* quats, const float* quats_raw,
    const float* scales, const float* viewmats, const float* projs, const float* Ks, int width,
    int height, const int* const* radii, const float* const* grad_centers,
    const float* const* grad_conics, float* grad_means, float* grad_quats, float* grad_scales,
    float* grad_opacities, int accumulate, int sh_degree, int sh_k, const float* sh,
    const float* campos, const unsigned char* const* active, const float* const* grad_colors,
    int color_stride, float* grad_sh, void* stream) {
  using host::aligned;
  using host::fail;
  if (views < 0 || n < 0 || width <= 0 || height <= 0)
    return fail(kInvalidArgument, "bad projection sizes");
  if (grad_sh && (!sh || !active || !grad_colors || sh_degree < 0 || sh_degree > 3 ||
                  sh_k < (sh_degree + 1) * (sh_degree + 1) || color_stride < 3))
    return fail(kInvalidArgument, "bad SH backward arguments");
  if (!quats && !quats_raw) return fail(kInvalidArgument, "quats or quats_raw is required");
  if (!radii || !grad_centers || !grad_conics)
    return fail(kInvalidArgument, "the per-view input tables are required");
  if (!aligned(quats, 16) || !aligned(quats_raw, 16) || !aligned(grad_quats, 16))
    return fail(kInvalidArgument, "quat rows need 16-byte alignment");
  for (int v = 0; v < views; ++v)
    if (!aligned(grad_conics[v], 16) || !aligned(grad_centers[v], 8))
      return fail(kInvalidArgument, "conic rows need 16-byte, centre rows 8-byte alignment");
  ProjectBackwardViewsParams vp{};
  ProjectBackwardParams& p = vp.shared;
  p.n = n;
  p.means = means;
  p.quats = quats;
  p.quats_raw = quats_raw;
  p.scales = scales;
  p.width = width;
  p.height = height;
  p.grad_means = grad_means;
  p.grad_quats = grad_quats;
  p.grad_scales = grad_scales;
  p.grad_opacities = grad_opacities;
  p.sh_degree = sh_degree;
  p.sh_k = sh_k;
  p.sh = sh;
  p.color_stride = color_stride;
  p.grad_sh = grad_sh;
  // at most kMaxViews cameras per launch; later launches accumulate
  for (int v0 = 0; v0 < views; v0 += kMaxViews) {
    p.accumulate = (accumulate || v0 > 0) ? 1 : 0;
    vp.views = std::min(kMaxViews, views - v0);
    vp.viewmats = viewmats + 16 * v0;
    vp.projs = projs + 16 * v0;
    vp.Ks = Ks + 9 * v0;
    vp.campos = campos ? campos + 3 * v0 : nullptr;
    for (int v = 0; v < vp.views; ++v) {
      vp.radii[v] = radii[v0 + v];
      vp.seed_centers[v] = grad_centers[v0 + v];
      vp.seed_conics[v] = grad_conics[v0 + v];
      vp.seed_colors[v] = grad_colors ? grad_colors[v0 + v] : nullptr;
      vp.active[v] = active ? active[v0 + v] : nullptr;
    }
    const int r = project_backward_views_dispatch(vp, reinterpret_cast<cudaStream_t>(stream));
    if (r != kOk) return r;
  }
  return kOk;
}
