// RaDe-GS projection (rade/projection.py) fused with the SH colours and the
// training metadata, and its backward.
//
// Forward restates rade/projection.py:39-260 (clamp_point, opacity
// coefficient, raster_covariance, geometry, project) operation by operation
// in IEEE float32; it is compiled into the -fmad=false translation unit, so
// radii, tile counts, sort distances, centres, conics, planes and normals
// agree bit for bit with the CPU oracle.  The reference builds its kernels
// with --use_fast_math; the approximate divide/sqrt are not reproduced, and
// the sort distance is sqrtf(x*x+y*y+z*z) (norm3df's value).  Raw
// quaternions are normalised in-kernel with Torch's CUDA F.normalize bits
// (inputs.py:252), and the SH colours are primitives/sh.py:44-79 on
// directions means - camera centre, as rade/api.py:153-165 computes them.
//
// Backward (compiled into the -fmad=true unit): the VJP of
// rade/projection.py:294-317 projection_loss (Warp autodiff in the
// reference) derived by hand, with adj_opacity_coefficient :57-70,
// adj_reference_normalize :78-84, adj_invert_covariance and
// adj_reference_rotation, then the SH VJP (primitives/sh.py:82-138) and the
// normalisation's VJP.
#pragma once
#include "project.cuh"

namespace splat {

struct RadeProjectParams {
  int n;
  const float* means;      // (n,3)
  const float* quats;      // (n,4) wxyz, normalised unless normalize_quats
  int normalize_quats;     // normalise in-kernel as Torch's F.normalize does on CUDA
  const float* scales;     // (n,3)
  const float* opacities;  // (n)
  const float* view;       // 4x4 row-major world->camera
  const float* proj;       // 4x4 full projection
  const float* K;          // 3x3 intrinsics
  int width, height;
  float near_plane, far_plane, radius_clip, kernel_size;
  // forward outputs (visible rows only, except radii / tiles)
  float* centers;  // (n,2)
  float* conics;   // (n,4)
  int* radii;      // (n)
  int* tiles;      // (n)
  float* depths;   // (n) radial distance of the camera-space centre
  float* planes;   // (n,3)
  float* normals;  // (n,3)
  // optional fused SH colours (sh == nullptr disables): primitives/sh.py
  int sh_degree;
  int sh_k;              // coefficients stored per Gaussian (>= (deg+1)^2)
  const float* sh;       // (n,K,3)
  const float* campos;   // (3) camera centre; null => directions = means
  float* colors;         // (n,3), zero on culled rows
  uint8_t* active;       // (n,3) clamp mask (forward output, backward input), or null
  // optional dense metadata (splatting/metadata.py:12-31), null disables
  float* meta_means2d;   // (n,2)
  float* meta_opacities; // (n)
  float* meta_conics;    // (n,3)
  // backward: seeds (null = zero) and gradients (null = not needed)
  const float* seed_centers;  // (n,2)
  const float* seed_conics;   // (n,4)
  const float* seed_planes;   // (n,3)
  const float* seed_normals;  // (n,3)
  float* grad_means;          // (n,3)
  float* grad_quats;          // (n,4)
  float* grad_scales;         // (n,3)
  float* grad_opacities;      // (n)
  float* grad_view;           // (4,4) accumulated
  float* grad_proj;           // (4,4) accumulated
  const float* seed_colors;   // (n,3) upstream of the SH colours, or null
  float* grad_sh;             // (n,K,3) written (zeros on culled rows), or null
  float* grad_campos;         // (3) accumulated, or null
};

// Backward entry of the -fmad=true translation unit.
int rade_project_backward_dispatch(const RadeProjectParams& p, cudaStream_t s);

SPLAT_DEV float4 load_quat(const RadeProjectParams& p, int i) {
  const float4 q = make_float4(p.quats[4 * i], p.quats[4 * i + 1], p.quats[4 * i + 2],
                               p.quats[4 * i + 3]);
  return p.normalize_quats ? torch_normalize4(q) : q;
}

// Row k of R without dynamic register indexing.
SPLAT_DEV float3 mat_row(const Mat3& R, int k) {
  return k == 0 ? make_float3(R.m[0][0], R.m[0][1], R.m[0][2])
                : (k == 1 ? make_float3(R.m[1][0], R.m[1][1], R.m[1][2])
                          : make_float3(R.m[2][0], R.m[2][1], R.m[2][2]));
}

SPLAT_DEV float3 mat_vec(const Mat3& m, float3 v) {
  return make_float3(m.m[0][0] * v.x + m.m[0][1] * v.y + m.m[0][2] * v.z,
                     m.m[1][0] * v.x + m.m[1][1] * v.y + m.m[1][2] * v.z,
                     m.m[2][0] * v.x + m.m[2][1] * v.y + m.m[2][2] * v.z);
}

SPLAT_DEV float dot3(float3 a, float3 b) { return a.x * b.x + a.y * b.y + a.z * b.z; }

// Warp's normalize: v / |v| per component, the zero vector when |v| == 0.
SPLAT_DEV float3 normalize3(float3 v) {
  const float l = sqrtf(v.x * v.x + v.y * v.y + v.z * v.z);
  if (l > 0.0f) return make_float3(v.x / l, v.y / l, v.z / l);
  return make_float3(0.0f, 0.0f, 0.0f);
}

SPLAT_DEV Mat3 view_rotation(const float* V) {
  // camera = transpose of the view's rotation block (rade/projection.py:119-129)
  return Mat3{{{V[0], V[4], V[8]}, {V[1], V[5], V[9]}, {V[2], V[6], V[10]}}};
}

// rade/projection.py:174-180 min-axis choice (find_min_from_triple's ties).
SPLAT_DEV int min_axis(float3 s) {
  const float sv[3] = {s.x, s.y, s.z};
  const int bigger = s.x < s.y ? 1 : 0;
  const int i0 = (bigger + 1) % 3, i1 = (bigger + 2) % 3;
  return sv[i0] > sv[i1] ? i1 : i0;
}

SPLAT_DEV float axis_value(float3 s, int k) { return k == 0 ? s.x : (k == 1 ? s.y : s.z); }

struct RadeRay {
  float3 cov;     // (a, b, c) of the undilated screen covariance
  float3 plane;   // ray plane
  float3 normal;  // unit camera-space normal
};

// rade/projection.py:102-190 geometry at camera-space position pos.
SPLAT_DEV RadeRay rade_geometry(float3 pos, float4 q, float3 s, const float* V, int width,
                                int height, float fx, float fy) {
  const float limx = W32(1.3) * static_cast<float>(width) / (2.0f * fx);
  const float limy = W32(1.3) * static_cast<float>(height) / (2.0f * fy);
  const float t0 = wclamp(pos.x / pos.z, -limx, limx) * pos.z;
  const float t1 = wclamp(pos.y / pos.z, -limy, limy) * pos.z;
  const float z = pos.z;
  const float u = t0 / z, v = t1 / z;
  const Mat3 R = glm_rotation(q.x, q.y, q.z, q.w);
  const Mat3 C = view_rotation(V);
  const Mat3 J = {{{fx / z, 0.0f, 0.0f},
                   {0.0f, fy / z, 0.0f},
                   {-fx * t0 / (z * z), -fy * t1 / (z * z), 0.0f}}};
  const Mat3 Tm = ref_matmul(C, J);
  const Mat3 S = {{{s.x, 0.0f, 0.0f}, {0.0f, s.y, 0.0f}, {0.0f, 0.0f, s.z}}};
  const Mat3 M = ref_matmul(ref_matmul(S, R), Tm);
  const Mat3 cov = ref_matmul(transpose(M), M);
  RadeRay out;
  out.cov = make_float3(cov.m[0][0], cov.m[1][0], cov.m[1][1]);
  const int mn = min_axis(s);
  Mat3 ic;
  if (axis_value(s, mn) > W32(1.0e-7)) {
    const Mat3 Si = {{{1.0f / s.x, 0.0f, 0.0f}, {0.0f, 1.0f / s.y, 0.0f}, {0.0f, 0.0f, 1.0f / s.z}}};
    const Mat3 Mi = ref_matmul(ref_matmul(Si, R), C);
    ic = ref_matmul(transpose(Mi), Mi);
  } else {
    const float3 ac = mat_vec(transpose(C), mat_row(R, mn));
    const float a3[3] = {ac.x, ac.y, ac.z};
#pragma unroll
    for (int i = 0; i < 3; ++i)
#pragma unroll
      for (int j = 0; j < 3; ++j) ic.m[i][j] = a3[i] * a3[j];
  }
  const float3 uvh = make_float3(u, v, 1.0f);
  const float3 dir = normalize3(mat_vec(ic, uvh));
  if (dot3(dir, dir) == 0.0f || !isfinite(dir.x)) {
    out.plane = make_float3(0.0f, 0.0f, 0.0f);
    out.normal = make_float3(0.0f, 0.0f, -1.0f);
    return out;
  }
  const float length = sqrtf(t0 * t0 + t1 * t1 + z * z);
  const float factor = length / (u * u + v * v + 1.0f);
  const float denom = wmax(dot3(dir, uvh), W32(1.0e-7));
  const float3 dd = make_float3(dir.x / denom, dir.y / denom, dir.z / denom);
  const float pl0 = (v * v + 1.0f) * dd.x + (-u * v) * dd.y + (-u) * dd.z;
  const float pl1 = (-u * v) * dd.x + (u * u + 1.0f) * dd.y + (-v) * dd.z;
  out.plane = make_float3(pl0 * factor / fx, pl1 * factor / fy,
                          sqrtf(pos.x * pos.x + pos.y * pos.y + pos.z * pos.z));
  const float3 rn = make_float3(-pl0 * factor, -pl1 * factor, -1.0f);
  const Mat3 NJ = {{{1.0f / z, 0.0f, t0 / length},
                    {0.0f, 1.0f / z, t1 / length},
                    {-t0 / (z * z), -t1 / (z * z), z / length}}};
  out.normal = normalize3(mat_vec(NJ, rn));
  return out;
}

// rade/projection.py:50-54 opacity_coefficient
SPLAT_DEV float opacity_coefficient(float3 cov, float k) {
  const float det0 = wmax(W32(1.0e-6), cov.x * cov.z - cov.y * cov.y);
  const float det1 = wmax(W32(1.0e-6), (cov.x + k) * (cov.z + k) - cov.y * cov.y);
  return sqrtf(det0 / det1);
}

// rade/projection.py:194-260 project for one Gaussian; returns whether it
// is visible (radii > 0) and writes its rows.
SPLAT_DEV bool rade_project_one(const RadeProjectParams& p, int i, float m0, float m1, float m2,
                                float4& conic_out, float2& center_out) {
  p.radii[i] = 0;
  p.tiles[i] = 0;
  const float3 pos = make_float3(point_row(p.view, 0, m0, m1, m2), point_row(p.view, 1, m0, m1, m2),
                                 point_row(p.view, 2, m0, m1, m2));
  if (pos.z <= p.near_plane || pos.z >= p.far_plane) return false;
  const float4 q = load_quat(p, i);
  const float3 s = make_float3(p.scales[3 * i], p.scales[3 * i + 1], p.scales[3 * i + 2]);
  const RadeRay rays = rade_geometry(pos, q, s, p.view, p.width, p.height, p.K[0], p.K[4]);
  const float a = rays.cov.x + p.kernel_size, b = rays.cov.y, c = rays.cov.z + p.kernel_size;
  const float det = a * c - b * b;
  if (det == 0.0f) return false;
  const float mid = 0.5f * (a + c);
  const int radius = f2i(ceilf(3.0f * sqrtf(mid + sqrtf(wmax(W32(0.1), mid * mid - det)))));
  if (static_cast<float>(radius) <= p.radius_clip) return false;
  const float2 center = pixel_center(m0, m1, m2, p.proj, p.width, p.height);
  const int gx = (p.width + kTile - 1) / kTile, gy = (p.height + kTile - 1) / kTile;
  const int4 bnd = tile_bounds(center.x, center.y, radius, gx, gy);
  const int count = (bnd.z - bnd.x) * (bnd.w - bnd.y);
  if (count == 0) return false;
  const float inverse = 1.0f / (a * c - b * b);
  const float4 conic = make_float4(c * inverse, -b * inverse, a * inverse,
                                   p.opacities[i] * opacity_coefficient(rays.cov, p.kernel_size));
  p.centers[2 * i] = center.x;
  p.centers[2 * i + 1] = center.y;
  p.conics[4 * i + 0] = conic.x;
  p.conics[4 * i + 1] = conic.y;
  p.conics[4 * i + 2] = conic.z;
  p.conics[4 * i + 3] = conic.w;
  p.radii[i] = radius;
  p.tiles[i] = count;
  p.depths[i] = sqrtf(pos.x * pos.x + pos.y * pos.y + pos.z * pos.z);
  p.planes[3 * i] = rays.plane.x;
  p.planes[3 * i + 1] = rays.plane.y;
  p.planes[3 * i + 2] = rays.plane.z;
  p.normals[3 * i] = rays.normal.x;
  p.normals[3 * i + 1] = rays.normal.y;
  p.normals[3 * i + 2] = rays.normal.z;
  conic_out = conic;
  center_out = center;
  return true;
}

// rade/projection.py:194-260 project, then (DEG >= 0) the SH colours and
// (meta_means2d != null) splatting/metadata.py:12-31's dense metadata.
template <int DEG>
__global__ void __launch_bounds__(256) rade_project_kernel(RadeProjectParams p) {
  const int i = blockIdx.x * blockDim.x + threadIdx.x;
  if (i >= p.n) return;
  const float m0 = p.means[3 * i], m1 = p.means[3 * i + 1], m2 = p.means[3 * i + 2];
  float4 conic = make_float4(0.0f, 0.0f, 0.0f, 0.0f);
  float2 center = make_float2(0.0f, 0.0f);
  const bool visible = rade_project_one(p, i, m0, m1, m2, conic, center);
  if constexpr (DEG >= 0) {
    float3 v = make_float3(0.0f, 0.0f, 0.0f);
    if (visible) {
      float d0 = m0, d1 = m1, d2 = m2;
      if (p.campos != nullptr) {
        d0 = m0 - p.campos[0];
        d1 = m1 - p.campos[1];
        d2 = m2 - p.campos[2];
      }
      v = sh_eval<DEG>(p.sh + static_cast<size_t>(i) * p.sh_k * 3, d0, d1, d2);
    }
    p.colors[3 * i + 0] = wmax(v.x, 0.0f);
    p.colors[3 * i + 1] = wmax(v.y, 0.0f);
    p.colors[3 * i + 2] = wmax(v.z, 0.0f);
    if (p.active != nullptr) {
      p.active[3 * i + 0] = visible && v.x >= 0.0f;
      p.active[3 * i + 1] = visible && v.y >= 0.0f;
      p.active[3 * i + 2] = visible && v.z >= 0.0f;
    }
  }
  if (p.meta_means2d != nullptr) {
    p.meta_means2d[2 * i] = visible ? center.x : 0.0f;
    p.meta_means2d[2 * i + 1] = visible ? center.y : 0.0f;
    p.meta_opacities[i] = visible ? conic.w : 0.0f;
    p.meta_conics[3 * i + 0] = visible ? conic.x : 0.0f;
    p.meta_conics[3 * i + 1] = visible ? conic.y : 0.0f;
    p.meta_conics[3 * i + 2] = visible ? conic.z : 0.0f;
  }
}

// ---- projection VJP ----------------------------------------------------------

SPLAT_DEV float seed(const float* base, int i, int stride, int k) {
  return base ? base[static_cast<size_t>(i) * stride + k] : 0.0f;
}

SPLAT_DEV Mat3 mat_mul(const Mat3& a, const Mat3& b) {
  Mat3 r;
#pragma unroll
  for (int i = 0; i < 3; ++i)
#pragma unroll
    for (int j = 0; j < 3; ++j)
      r.m[i][j] = a.m[i][0] * b.m[0][j] + a.m[i][1] * b.m[1][j] + a.m[i][2] * b.m[2][j];
  return r;
}

// a * b^T
SPLAT_DEV Mat3 mat_mul_bt(const Mat3& a, const Mat3& b) { return mat_mul(a, transpose(b)); }
// a^T * b
SPLAT_DEV Mat3 mat_mul_at(const Mat3& a, const Mat3& b) { return mat_mul(transpose(a), b); }

// d/dv of normalize(v) applied to g: (g - n (n.g)) / |v|.
SPLAT_DEV float3 normalize_vjp(float3 v, float3 g) {
  const float l = sqrtf(v.x * v.x + v.y * v.y + v.z * v.z);
  if (!(l > 0.0f)) return make_float3(0.0f, 0.0f, 0.0f);
  const float3 n = make_float3(v.x / l, v.y / l, v.z / l);
  const float d = dot3(n, g);
  return make_float3((g.x - n.x * d) / l, (g.y - n.y * d) / l, (g.z - n.z * d) / l);
}

// Gradients of one visible Gaussian: writes the per-Gaussian rows and adds
// the camera contributions (view rows 0-2, projection rows 0, 1, 3) to gv /
// gp.
template <int DEG>
SPLAT_DEV void rade_project_vjp(const RadeProjectParams& p, int i, float (&gv)[12],
                                float (&gp)[12], float (&gc)[3]) {
  const float* V = p.view;
  const float fx = p.K[0], fy = p.K[4];
  const float m[3] = {p.means[3 * i], p.means[3 * i + 1], p.means[3 * i + 2]};
  const float3 pos = make_float3(point_row(V, 0, m[0], m[1], m[2]), point_row(V, 1, m[0], m[1], m[2]),
                                 point_row(V, 2, m[0], m[1], m[2]));
  const float4 q_raw = make_float4(p.quats[4 * i], p.quats[4 * i + 1], p.quats[4 * i + 2],
                                   p.quats[4 * i + 3]);
  const float4 q = p.normalize_quats ? torch_normalize4(q_raw) : q_raw;
  const float3 s = make_float3(p.scales[3 * i], p.scales[3 * i + 1], p.scales[3 * i + 2]);
  const float opacity = p.opacities[i];
  const float ks = p.kernel_size;
  // -- forward recomputation (rade_geometry's intermediates) --
  const float limx = W32(1.3) * static_cast<float>(p.width) / (2.0f * fx);
  const float limy = W32(1.3) * static_cast<float>(p.height) / (2.0f * fy);
  const float xr = pos.x / pos.z, yr = pos.y / pos.z;
  const bool in_x = xr >= -limx && xr <= limx, in_y = yr >= -limy && yr <= limy;
  const float cx = wclamp(xr, -limx, limx), cy = wclamp(yr, -limy, limy);
  const float t0 = cx * pos.z, t1 = cy * pos.z, z = pos.z;
  const float u = t0 / z, v = t1 / z;
  const float z2 = z * z, z3 = z2 * z;
  const Mat3 R = glm_rotation(q.x, q.y, q.z, q.w);
  const Mat3 C = view_rotation(V);
  const Mat3 J = {{{fx / z, 0.0f, 0.0f}, {0.0f, fy / z, 0.0f}, {-fx * t0 / z2, -fy * t1 / z2, 0.0f}}};
  const Mat3 Tm = mat_mul(C, J);
  Mat3 SR;
  const float sv[3] = {s.x, s.y, s.z};
#pragma unroll
  for (int k = 0; k < 3; ++k)
#pragma unroll
    for (int j = 0; j < 3; ++j) SR.m[k][j] = sv[k] * R.m[k][j];
  const Mat3 M = mat_mul(SR, Tm);
  const float3 cov = make_float3(M.m[0][0] * M.m[0][0] + M.m[1][0] * M.m[1][0] + M.m[2][0] * M.m[2][0],
                                 M.m[0][1] * M.m[0][0] + M.m[1][1] * M.m[1][0] + M.m[2][1] * M.m[2][0],
                                 M.m[0][1] * M.m[0][1] + M.m[1][1] * M.m[1][1] + M.m[2][1] * M.m[2][1]);
  // gradient accumulators
  float3 g_pos = make_float3(0.0f, 0.0f, 0.0f);  // camera-space position
  float g_t0 = 0.0f, g_t1 = 0.0f, g_z = 0.0f, g_u = 0.0f, g_v = 0.0f;
  Mat3 g_R = {}, g_C = {};
  float g_s[3] = {0.0f, 0.0f, 0.0f};
  float3 g_cov = make_float3(0.0f, 0.0f, 0.0f);
  // -- conic: adj_invert_covariance at the dilated covariance and
  //    adj_opacity_coefficient (rade/projection.py:57-70) --
  {
    const float a = cov.x + ks, b = cov.y, c = cov.z + ks;
    const float gx = seed(p.seed_conics, i, 4, 0), gy = seed(p.seed_conics, i, 4, 1);
    const float gz = seed(p.seed_conics, i, 4, 2), go = seed(p.seed_conics, i, 4, 3);
    const float det = a * c - b * b;
    const float f = 1.0f / (det * det + W32(1e-7));
    g_cov.x += f * (-c * c * gx + b * c * gy + (det - a * c) * gz);
    g_cov.y += f * (2.0f * b * c * gx - (det + 2.0f * b * b) * gy + 2.0f * a * b * gz);
    g_cov.z += f * (-a * a * gz + a * b * gy + (det - a * c) * gx);
    const float det0 = wmax(W32(1.0e-6), cov.x * cov.z - cov.y * cov.y);
    const float det1 = wmax(W32(1.0e-6), (cov.x + ks) * (cov.z + ks) - cov.y * cov.y);
    const float coef = sqrtf(det0 / det1);
    if (p.grad_opacities) p.grad_opacities[i] = go * coef;
    const float gcoef = go * opacity;
    const float d0 = gcoef * 0.5f / (coef + W32(1.0e-6)) / det1;
    const float d1 = -d0 * coef;
    g_cov.x += d0 * cov.z + d1 * (cov.z + ks);
    g_cov.y += -2.0f * cov.y * (d0 + d1);
    g_cov.z += d0 * cov.x + d1 * (cov.x + ks);
  }
  // -- ray plane and normal (rade/projection.py:149-189) --
  const int mn = min_axis(s);
  const bool full_rank = axis_value(s, mn) > W32(1.0e-7);
  Mat3 IC, A;  // inverse covariance and, full rank, A = diag(1/s) R
  float3 ac = make_float3(0.0f, 0.0f, 0.0f);
  Mat3 Mi = {};
  if (full_rank) {
    const float si[3] = {1.0f / s.x, 1.0f / s.y, 1.0f / s.z};
#pragma unroll
    for (int k = 0; k < 3; ++k)
#pragma unroll
      for (int j = 0; j < 3; ++j) A.m[k][j] = si[k] * R.m[k][j];
    Mi = mat_mul(A, C);
    IC = mat_mul_at(Mi, Mi);
  } else {
    ac = mat_vec(transpose(C), mat_row(R, mn));
    const float a3[3] = {ac.x, ac.y, ac.z};
#pragma unroll
    for (int k = 0; k < 3; ++k)
#pragma unroll
      for (int j = 0; j < 3; ++j) IC.m[k][j] = a3[k] * a3[j];
  }
  const float3 uvh = make_float3(u, v, 1.0f);
  const float3 dvec = mat_vec(IC, uvh);
  const float3 dir = normalize3(dvec);
  const bool has_plane = !(dot3(dir, dir) == 0.0f || !isfinite(dir.x));
  if (has_plane) {
    const float3 gpl = make_float3(seed(p.seed_planes, i, 3, 0), seed(p.seed_planes, i, 3, 1),
                                   seed(p.seed_planes, i, 3, 2));
    const float3 gn = make_float3(seed(p.seed_normals, i, 3, 0), seed(p.seed_normals, i, 3, 1),
                                  seed(p.seed_normals, i, 3, 2));
    const float L = sqrtf(t0 * t0 + t1 * t1 + z * z);
    const float Q = u * u + v * v + 1.0f;
    const float factor = L / Q;
    const float dot_du = dot3(dir, uvh);
    const float den = wmax(dot_du, W32(1.0e-7));
    const float3 dd = make_float3(dir.x / den, dir.y / den, dir.z / den);
    const float pl0 = (v * v + 1.0f) * dd.x - u * v * dd.y - u * dd.z;
    const float pl1 = -u * v * dd.x + (u * u + 1.0f) * dd.y - v * dd.z;
    const float3 rn = make_float3(-pl0 * factor, -pl1 * factor, -1.0f);
    const Mat3 NJ = {{{1.0f / z, 0.0f, t0 / L}, {0.0f, 1.0f / z, t1 / L}, {-t0 / z2, -t1 / z2, z / L}}};
    const float3 nv = mat_vec(NJ, rn);
    // adj_reference_normalize: (g - n (n.g)) / |n| with n = normalize(nv)
    float3 g_nv;
    {
      const float3 n = normalize3(nv);
      const float d = dot3(n, gn);
      const float ln = sqrtf(dot3(n, n));
      g_nv = make_float3((gn.x - n.x * d) / ln, (gn.y - n.y * d) / ln, (gn.z - n.z * d) / ln);
    }
    // nv = NJ rn
    const float3 g_rn = mat_vec(transpose(NJ), g_nv);
    float g_L = 0.0f;
    g_z += g_nv.x * rn.x * (-1.0f / z2) + g_nv.y * rn.y * (-1.0f / z2) +
           g_nv.z * (rn.x * (2.0f * t0 / z3) + rn.y * (2.0f * t1 / z3) + rn.z / L);
    g_t0 += g_nv.x * rn.z / L - g_nv.z * rn.x / z2;
    g_t1 += g_nv.y * rn.z / L - g_nv.z * rn.y / z2;
    g_L -= (g_nv.x * rn.z * t0 + g_nv.y * rn.z * t1 + g_nv.z * rn.z * z) / (L * L);
    // rn = (-pl0 f, -pl1 f, -1) and plane = (pl0 f / fx, pl1 f / fy, |pos|)
    float g_pl0 = -g_rn.x * factor + gpl.x * factor / fx;
    float g_pl1 = -g_rn.y * factor + gpl.y * factor / fy;
    float g_f = -(g_rn.x * pl0 + g_rn.y * pl1) + gpl.x * pl0 / fx + gpl.y * pl1 / fy;
    {
      const float lp = sqrtf(dot3(pos, pos));
      g_pos.x += gpl.z * pos.x / lp;
      g_pos.y += gpl.z * pos.y / lp;
      g_pos.z += gpl.z * pos.z / lp;
    }
    // pl = NJinv dd (rows 0 and 1)
    const float3 g_dd = make_float3(g_pl0 * (v * v + 1.0f) - g_pl1 * u * v,
                                    -g_pl0 * u * v + g_pl1 * (u * u + 1.0f), -u * g_pl0 - v * g_pl1);
    g_u += g_pl0 * (-v * dd.y - dd.z) + g_pl1 * (-v * dd.x + 2.0f * u * dd.y);
    g_v += g_pl0 * (2.0f * v * dd.x - u * dd.y) + g_pl1 * (-u * dd.x - dd.z);
    // dd = dir / max(dir.uvh, 1e-7)
    float3 g_dir = make_float3(g_dd.x / den, g_dd.y / den, g_dd.z / den);
    if (dot_du > W32(1.0e-7)) {
      const float g_dot = -dot3(g_dd, dd) / den;
      g_dir.x += g_dot * u;
      g_dir.y += g_dot * v;
      g_dir.z += g_dot;
      g_u += g_dot * dir.x;
      g_v += g_dot * dir.y;
    }
    // factor = L / Q
    g_L += g_f / Q;
    const float g_Q = -g_f * factor / Q;
    g_u += g_Q * 2.0f * u;
    g_v += g_Q * 2.0f * v;
    // L = |(t0, t1, z)|
    g_t0 += g_L * t0 / L;
    g_t1 += g_L * t1 / L;
    g_z += g_L * z / L;
    // dir = normalize(dvec), dvec = IC uvh
    const float3 g_dvec = normalize_vjp(dvec, g_dir);
    const float3 g_uvh = mat_vec(transpose(IC), g_dvec);
    g_u += g_uvh.x;
    g_v += g_uvh.y;
    const float gd[3] = {g_dvec.x, g_dvec.y, g_dvec.z};
    const float uv3[3] = {u, v, 1.0f};
    Mat3 g_IC;
#pragma unroll
    for (int k = 0; k < 3; ++k)
#pragma unroll
      for (int j = 0; j < 3; ++j) g_IC.m[k][j] = gd[k] * uv3[j];
    Mat3 sym;  // g_IC + g_IC^T
#pragma unroll
    for (int k = 0; k < 3; ++k)
#pragma unroll
      for (int j = 0; j < 3; ++j) sym.m[k][j] = g_IC.m[k][j] + g_IC.m[j][k];
    if (full_rank) {
      // IC = Mi^T Mi, Mi = A C, A = diag(1/s) R
      const Mat3 g_Mi = mat_mul(Mi, sym);
      const Mat3 g_A = mat_mul_bt(g_Mi, C);
      const Mat3 gC = mat_mul_at(A, g_Mi);
      const float si[3] = {1.0f / s.x, 1.0f / s.y, 1.0f / s.z};
#pragma unroll
      for (int k = 0; k < 3; ++k) {
        float acc = 0.0f;
#pragma unroll
        for (int j = 0; j < 3; ++j) {
          g_C.m[k][j] += gC.m[k][j];
          g_R.m[k][j] += si[k] * g_A.m[k][j];
          acc += g_A.m[k][j] * R.m[k][j];
        }
        g_s[k] -= acc * si[k] * si[k];
      }
    } else {
      // IC = ac ac^T, ac = C^T axis, axis = R[mn]
      const float3 g_ac = mat_vec(sym, ac);
      const float3 ax = mat_row(R, mn);
      const float axis[3] = {ax.x, ax.y, ax.z};
      const float ga[3] = {g_ac.x, g_ac.y, g_ac.z};
#pragma unroll
      for (int k = 0; k < 3; ++k)
#pragma unroll
        for (int j = 0; j < 3; ++j) g_C.m[k][j] += axis[k] * ga[j];
      const float3 g_axis = mat_vec(C, g_ac);
      const float ga3[3] = {g_axis.x, g_axis.y, g_axis.z};
#pragma unroll
      for (int k = 0; k < 3; ++k)
#pragma unroll
        for (int j = 0; j < 3; ++j) g_R.m[k][j] += k == mn ? ga3[j] : 0.0f;
    }
  }
  // -- covariance (rade/projection.py:87-92, 141-142) --
  {
    Mat3 g_M = {};
#pragma unroll
    for (int k = 0; k < 3; ++k) {
      g_M.m[k][0] = 2.0f * g_cov.x * M.m[k][0] + g_cov.y * M.m[k][1];
      g_M.m[k][1] = 2.0f * g_cov.z * M.m[k][1] + g_cov.y * M.m[k][0];
    }
    const Mat3 g_SR = mat_mul_bt(g_M, Tm);
    const Mat3 g_Tm = mat_mul_at(SR, g_M);
#pragma unroll
    for (int k = 0; k < 3; ++k) {
      float acc = 0.0f;
#pragma unroll
      for (int j = 0; j < 3; ++j) {
        acc += g_SR.m[k][j] * R.m[k][j];
        g_R.m[k][j] += sv[k] * g_SR.m[k][j];
      }
      g_s[k] += acc;
    }
    const Mat3 gC = mat_mul_bt(g_Tm, J);
    const Mat3 g_J = mat_mul_at(C, g_Tm);
#pragma unroll
    for (int k = 0; k < 3; ++k)
#pragma unroll
      for (int j = 0; j < 3; ++j) g_C.m[k][j] += gC.m[k][j];
    g_z += -g_J.m[0][0] * fx / z2 - g_J.m[1][1] * fy / z2 + g_J.m[2][0] * 2.0f * fx * t0 / z3 +
           g_J.m[2][1] * 2.0f * fy * t1 / z3;
    g_t0 -= g_J.m[2][0] * fx / z2;
    g_t1 -= g_J.m[2][1] * fy / z2;
  }
  // -- u = t0 / z, v = t1 / z, then clamp_point (rade/projection.py:39-47) --
  g_t0 += g_u / z;
  g_t1 += g_v / z;
  g_z -= (g_u * t0 + g_v * t1) / z2;
  if (in_x) g_pos.x += g_t0; else g_pos.z += g_t0 * cx;
  if (in_y) g_pos.y += g_t1; else g_pos.z += g_t1 * cy;
  g_pos.z += g_z;
  // -- position = view * mean, camera = view rotation^T --
  const float gpv[3] = {g_pos.x, g_pos.y, g_pos.z};
  float g_mean[3];
#pragma unroll
  for (int j = 0; j < 3; ++j) g_mean[j] = V[j] * gpv[0] + V[4 + j] * gpv[1] + V[8 + j] * gpv[2];
#pragma unroll
  for (int r = 0; r < 3; ++r) {
#pragma unroll
    for (int j = 0; j < 3; ++j) gv[4 * r + j] += gpv[r] * m[j] + g_C.m[j][r];
    gv[4 * r + 3] += gpv[r];
  }
  // -- centre (splatting/geometry.py:106-123) --
  {
    const float gcx = seed(p.seed_centers, i, 2, 0), gcy = seed(p.seed_centers, i, 2, 1);
    const float* P = p.proj;
    const float c0 = point_row(P, 0, m[0], m[1], m[2]);
    const float c1 = point_row(P, 1, m[0], m[1], m[2]);
    const float c3 = point_row(P, 3, m[0], m[1], m[2]);
    const float iw = 1.0f / (c3 + W32(1e-7));
    const float hw = 0.5f * static_cast<float>(p.width), hh = 0.5f * static_cast<float>(p.height);
    const float g0 = gcx * hw * iw, g1 = gcy * hh * iw;
    const float g3 = -(gcx * hw * c0 + gcy * hh * c1) * iw * iw;
    const float grow[3] = {g0, g1, g3};
    const int rows[3] = {0, 1, 3};
#pragma unroll
    for (int r = 0; r < 3; ++r) {
#pragma unroll
      for (int j = 0; j < 3; ++j) {
        g_mean[j] += grow[r] * P[4 * rows[r] + j];
        gp[4 * r + j] += grow[r] * m[j];
      }
      gp[4 * r + 3] += grow[r];
    }
  }
  // SH colours (primitives/sh.py:82-138) on directions means - campos
  if constexpr (DEG >= 0) {
    if (p.sh != nullptr) {
      float d0 = m[0], d1 = m[1], d2 = m[2];
      if (p.campos != nullptr) {
        d0 = m[0] - p.campos[0];
        d1 = m[1] - p.campos[1];
        d2 = m[2] - p.campos[2];
      }
      const float3 cg = make_float3(
          p.seed_colors && p.active[3 * i] ? p.seed_colors[3 * i] : 0.0f,
          p.seed_colors && p.active[3 * i + 1] ? p.seed_colors[3 * i + 1] : 0.0f,
          p.seed_colors && p.active[3 * i + 2] ? p.seed_colors[3 * i + 2] : 0.0f);
      const float3 dg = sh_vjp_global<DEG>(p.sh + static_cast<size_t>(i) * p.sh_k * 3, p.sh_k, d0,
                                           d1, d2, cg,
                                           p.grad_sh + static_cast<size_t>(i) * p.sh_k * 3, false);
      g_mean[0] += dg.x;
      g_mean[1] += dg.y;
      g_mean[2] += dg.z;
      gc[0] -= dg.x;
      gc[1] -= dg.y;
      gc[2] -= dg.z;
    }
  }
  if (p.grad_means) {
    p.grad_means[3 * i] = g_mean[0];
    p.grad_means[3 * i + 1] = g_mean[1];
    p.grad_means[3 * i + 2] = g_mean[2];
  }
  if (p.grad_scales) {
    p.grad_scales[3 * i] = g_s[0];
    p.grad_scales[3 * i + 1] = g_s[1];
    p.grad_scales[3 * i + 2] = g_s[2];
  }
  if (p.grad_quats) {
    // splatting/math.py:13-28 adj_reference_rotation
    const float r = q.x, x = q.y, y = q.z, zq = q.w;
    const Mat3& G = g_R;
    p.grad_quats[4 * i] = 2.0f * (zq * (G.m[0][1] - G.m[1][0]) + y * (G.m[2][0] - G.m[0][2]) +
                                  x * (G.m[1][2] - G.m[2][1]));
    p.grad_quats[4 * i + 1] = 2.0f * (y * (G.m[0][1] + G.m[1][0]) + zq * (G.m[0][2] + G.m[2][0]) +
                                      r * (G.m[1][2] - G.m[2][1])) -
                              4.0f * x * (G.m[1][1] + G.m[2][2]);
    p.grad_quats[4 * i + 2] = 2.0f * (x * (G.m[0][1] + G.m[1][0]) + r * (G.m[2][0] - G.m[0][2]) +
                                      zq * (G.m[1][2] + G.m[2][1])) -
                              4.0f * y * (G.m[0][0] + G.m[2][2]);
    p.grad_quats[4 * i + 3] = 2.0f * (r * (G.m[0][1] - G.m[1][0]) + x * (G.m[0][2] + G.m[2][0]) +
                                      y * (G.m[1][2] + G.m[2][1])) -
                              4.0f * zq * (G.m[0][0] + G.m[1][1]);
    if (p.normalize_quats) {
      // VJP of F.normalize(x) = x / max(|x|, 1e-12) (inputs.py:252):
      // (g - n (n . g)) / |x|, or g / 1e-12 where the norm is clamped
      float* gq = p.grad_quats + 4 * i;
      const float norm = sqrtf((q_raw.x * q_raw.x + q_raw.z * q_raw.z) +
                               (q_raw.y * q_raw.y + q_raw.w * q_raw.w));
      if (norm > W32(1e-12)) {
        const float d = q.x * gq[0] + q.y * gq[1] + q.z * gq[2] + q.w * gq[3];
        gq[0] = (gq[0] - q.x * d) / norm;
        gq[1] = (gq[1] - q.y * d) / norm;
        gq[2] = (gq[2] - q.z * d) / norm;
        gq[3] = (gq[3] - q.w * d) / norm;
      } else {
#pragma unroll
        for (int k = 0; k < 4; ++k) gq[k] = gq[k] / W32(1e-12);
      }
    }
  }
}

// rade/projection.py:324-396 project_backward: per-Gaussian rows (culled
// rows get explicit zeros) and the camera gradients (view rows 0-2,
// projection rows 0, 1, 3, camera centre), summed per thread over a
// grid-stride range, then per warp, then per block before one atomic per
// entry and block.
template <int DEG>
__global__ void __launch_bounds__(128) rade_project_backward_kernel(RadeProjectParams p) {
  __shared__ float s_cam[27];
  if (threadIdx.x < 27) s_cam[threadIdx.x] = 0.0f;
  __syncthreads();
  float gv[12], gp[12], gc[3];
#pragma unroll
  for (int k = 0; k < 12; ++k) gv[k] = gp[k] = 0.0f;
  gc[0] = gc[1] = gc[2] = 0.0f;
  for (int i = blockIdx.x * blockDim.x + threadIdx.x; i < p.n; i += gridDim.x * blockDim.x) {
    if (p.radii[i] > 0) {
      rade_project_vjp<DEG>(p, i, gv, gp, gc);
    } else {
      if (p.grad_means) p.grad_means[3 * i] = p.grad_means[3 * i + 1] = p.grad_means[3 * i + 2] = 0.0f;
      if (p.grad_scales)
        p.grad_scales[3 * i] = p.grad_scales[3 * i + 1] = p.grad_scales[3 * i + 2] = 0.0f;
      if (p.grad_quats)
        p.grad_quats[4 * i] = p.grad_quats[4 * i + 1] = p.grad_quats[4 * i + 2] =
            p.grad_quats[4 * i + 3] = 0.0f;
      if (p.grad_opacities) p.grad_opacities[i] = 0.0f;
      if (DEG >= 0 && p.grad_sh) {
        float* row = p.grad_sh + static_cast<size_t>(i) * p.sh_k * 3;
        for (int k = 0; k < 3 * p.sh_k; ++k) row[k] = 0.0f;
      }
    }
  }
  if (!p.grad_view && !p.grad_proj && !p.grad_campos) return;
#pragma unroll
  for (int k = 0; k < 12; ++k) {
    const float a = warp_sum(gv[k]);
    const float b = warp_sum(gp[k]);
    if ((threadIdx.x & 31) == 0) {
      atomicAdd(&s_cam[k], a);
      atomicAdd(&s_cam[12 + k], b);
    }
  }
#pragma unroll
  for (int k = 0; k < 3; ++k) {
    const float c = warp_sum(gc[k]);
    if ((threadIdx.x & 31) == 0) atomicAdd(&s_cam[24 + k], c);
  }
  __syncthreads();
  if (threadIdx.x < 12) {
    // view rows 0-2; projection rows 0, 1, 3
    if (p.grad_view) atomicAdd(p.grad_view + threadIdx.x, s_cam[threadIdx.x]);
    const int row = threadIdx.x / 4 == 2 ? 3 : threadIdx.x / 4;
    if (p.grad_proj) atomicAdd(p.grad_proj + 4 * row + threadIdx.x % 4, s_cam[12 + threadIdx.x]);
  } else if (threadIdx.x < 15 && p.grad_campos) {
    atomicAdd(p.grad_campos + (threadIdx.x - 12), s_cam[24 + threadIdx.x - 12]);
  }
}

}  // namespace splat
