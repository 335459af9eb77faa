// RaDe-GS projection and tile-cooperative geometry blend.
//
// Forward restates rade/projection.py:39-260 (clamp_point, opacity
// coefficient, raster_covariance, geometry, project) and rade/render.py:
// 106-227 (evaluate) operation by operation in IEEE float32 (this header is
// compiled into the -fmad=false translation unit), so radii, tile counts,
// sort distances and the blend's discrete decisions (acceptance, early
// termination, last and median contributor) agree bit for bit with the CPU
// oracle.  The reference builds these kernels with --use_fast_math; its
// approximate divide/sqrt/exp are not reproduced (exp is the shared
// Cody-Waite splat_expf, the sort distance sqrtf(x*x+y*y+z*z)).
//
// Backward: the projection VJP (rade/projection.py:294-398, Warp autodiff of
// projection_loss with adj_opacity_coefficient :57-70,
// adj_reference_normalize :78-84, adj_invert_covariance and
// adj_reference_rotation) is derived by hand below; the blend backward
// (rade/render.py:336-545) replays each pixel from its last contributor
// like the gs3d backward, carrying one scalar S for every blended quantity
// (features, depth, normal) instead of per-channel colour sums, and reduces
// each sample's gradient values over the warp with butterfly16.
#pragma once
#include "project.cuh"
#include "render.cuh"

namespace splat {

struct RadeProjectParams {
  int n;
  const float* means;      // (n,3)
  const float* quats;      // (n,4) normalised wxyz
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
};

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
    const float3 ac = mat_vec(transpose(C), make_float3(R.m[mn][0], R.m[mn][1], R.m[mn][2]));
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

// rade/projection.py:194-260 project
__global__ void __launch_bounds__(256) rade_project_kernel(RadeProjectParams p) {
  const int i = blockIdx.x * blockDim.x + threadIdx.x;
  if (i >= p.n) return;
  p.radii[i] = 0;
  p.tiles[i] = 0;
  const float m0 = p.means[3 * i], m1 = p.means[3 * i + 1], m2 = p.means[3 * i + 2];
  const float3 pos = make_float3(point_row(p.view, 0, m0, m1, m2), point_row(p.view, 1, m0, m1, m2),
                                 point_row(p.view, 2, m0, m1, m2));
  if (pos.z <= p.near_plane || pos.z >= p.far_plane) return;
  const float4 q = make_float4(p.quats[4 * i], p.quats[4 * i + 1], p.quats[4 * i + 2],
                               p.quats[4 * i + 3]);
  const float3 s = make_float3(p.scales[3 * i], p.scales[3 * i + 1], p.scales[3 * i + 2]);
  const RadeRay rays = rade_geometry(pos, q, s, p.view, p.width, p.height, p.K[0], p.K[4]);
  const float a = rays.cov.x + p.kernel_size, b = rays.cov.y, c = rays.cov.z + p.kernel_size;
  const float det = a * c - b * b;
  if (det == 0.0f) return;
  const float mid = 0.5f * (a + c);
  const int radius = f2i(ceilf(3.0f * sqrtf(mid + sqrtf(wmax(W32(0.1), mid * mid - det)))));
  if (static_cast<float>(radius) <= p.radius_clip) return;
  const float2 center = pixel_center(m0, m1, m2, p.proj, p.width, p.height);
  const int gx = (p.width + kTile - 1) / kTile, gy = (p.height + kTile - 1) / kTile;
  const int4 bnd = tile_bounds(center.x, center.y, radius, gx, gy);
  const int count = (bnd.z - bnd.x) * (bnd.w - bnd.y);
  if (count == 0) return;
  const float inverse = 1.0f / (a * c - b * b);
  p.centers[2 * i] = center.x;
  p.centers[2 * i + 1] = center.y;
  p.conics[4 * i + 0] = c * inverse;
  p.conics[4 * i + 1] = -b * inverse;
  p.conics[4 * i + 2] = a * inverse;
  p.conics[4 * i + 3] = p.opacities[i] * opacity_coefficient(rays.cov, p.kernel_size);
  p.radii[i] = radius;
  p.tiles[i] = count;
  p.depths[i] = sqrtf(pos.x * pos.x + pos.y * pos.y + pos.z * pos.z);
  p.planes[3 * i] = rays.plane.x;
  p.planes[3 * i + 1] = rays.plane.y;
  p.planes[3 * i + 2] = rays.plane.z;
  p.normals[3 * i] = rays.normal.x;
  p.normals[3 * i + 1] = rays.normal.y;
  p.normals[3 * i + 2] = rays.normal.z;
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
SPLAT_DEV void rade_project_vjp(const RadeProjectParams& p, int i, float (&gv)[12],
                                float (&gp)[12]) {
  const float* V = p.view;
  const float fx = p.K[0], fy = p.K[4];
  const float m[3] = {p.means[3 * i], p.means[3 * i + 1], p.means[3 * i + 2]};
  const float3 pos = make_float3(point_row(V, 0, m[0], m[1], m[2]), point_row(V, 1, m[0], m[1], m[2]),
                                 point_row(V, 2, m[0], m[1], m[2]));
  const float4 q = make_float4(p.quats[4 * i], p.quats[4 * i + 1], p.quats[4 * i + 2],
                               p.quats[4 * i + 3]);
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
    ac = mat_vec(transpose(C), make_float3(R.m[mn][0], R.m[mn][1], R.m[mn][2]));
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
      const float axis[3] = {R.m[mn][0], R.m[mn][1], R.m[mn][2]};
      const float ga[3] = {g_ac.x, g_ac.y, g_ac.z};
#pragma unroll
      for (int k = 0; k < 3; ++k)
#pragma unroll
        for (int j = 0; j < 3; ++j) g_C.m[k][j] += axis[k] * ga[j];
      const float3 g_axis = mat_vec(C, g_ac);
      g_R.m[mn][0] += g_axis.x;
      g_R.m[mn][1] += g_axis.y;
      g_R.m[mn][2] += g_axis.z;
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
  }
}

// rade/projection.py:324-396 project_backward: per-Gaussian rows (culled
// rows get explicit zeros) and the camera matrices' gradients, summed per
// thread over a grid-stride range, then per warp, then per block before one
// atomic per matrix entry and block.
__global__ void __launch_bounds__(256) rade_project_backward_kernel(RadeProjectParams p) {
  __shared__ float s_cam[24];
  if (threadIdx.x < 24) s_cam[threadIdx.x] = 0.0f;
  __syncthreads();
  float gv[12], gp[12];
#pragma unroll
  for (int k = 0; k < 12; ++k) gv[k] = gp[k] = 0.0f;
  for (int i = blockIdx.x * blockDim.x + threadIdx.x; i < p.n; i += gridDim.x * blockDim.x) {
    if (p.radii[i] > 0) {
      rade_project_vjp(p, i, gv, gp);
    } else {
      if (p.grad_means) p.grad_means[3 * i] = p.grad_means[3 * i + 1] = p.grad_means[3 * i + 2] = 0.0f;
      if (p.grad_scales)
        p.grad_scales[3 * i] = p.grad_scales[3 * i + 1] = p.grad_scales[3 * i + 2] = 0.0f;
      if (p.grad_quats)
        p.grad_quats[4 * i] = p.grad_quats[4 * i + 1] = p.grad_quats[4 * i + 2] =
            p.grad_quats[4 * i + 3] = 0.0f;
      if (p.grad_opacities) p.grad_opacities[i] = 0.0f;
    }
  }
  if (!p.grad_view && !p.grad_proj) return;
#pragma unroll
  for (int k = 0; k < 12; ++k) {
    const float a = warp_sum(gv[k]);
    const float b = warp_sum(gp[k]);
    if ((threadIdx.x & 31) == 0) {
      atomicAdd(&s_cam[k], a);
      atomicAdd(&s_cam[12 + k], b);
    }
  }
  __syncthreads();
  if (threadIdx.x < 12) {
    // view rows 0-2; projection rows 0, 1, 3
    if (p.grad_view) atomicAdd(p.grad_view + threadIdx.x, s_cam[threadIdx.x]);
    const int row = threadIdx.x / 4 == 2 ? 3 : threadIdx.x / 4;
    if (p.grad_proj) atomicAdd(p.grad_proj + 4 * row + threadIdx.x % 4, s_cam[12 + threadIdx.x]);
  }
}

// ---- blend ------------------------------------------------------------------

struct RadeRenderParams {
  RenderParams base;      // bins, centres, conics, features (a = colours, b = extras),
                          // background, statistics; base.channels = C (no appended channel)
  const float* planes;    // (n,3)
  const float* normals;   // (n,3)
  const float* K;         // (3,3) intrinsics (device)
  // forward outputs, value of channel c at pixel p at base[p * pix + c * ch]:
  // features (C channels), alpha, expected depth, median depth, normals (3);
  // planar auxiliary (2,H,W) and contributors (2,H,W).  The backward reads
  // alpha, normals, auxiliary and contributors back.
  float* features;
  int feat_pix, feat_ch;
  float* alpha;
  int alpha_pix;
  float* depth;
  int depth_pix;
  float* median;
  int median_pix;
  float* normal_image;
  int normal_pix, normal_ch;
  float* auxiliary;
  int* contributors;
  // backward inputs: the forward's outputs and the upstream images
  // (channel-last (H,W,k) with the given pixel / channel strides; null = 0)
  const float* up_features;
  int up_feat_pix, up_feat_ch;
  const float* up_alpha;
  int up_alpha_pix;
  const float* up_depth;
  int up_depth_pix;
  const float* up_median;
  int up_median_pix;
  const float* up_normals;
  int up_normals_pix, up_normals_ch;
  // backward outputs (accumulated; grad_a / grad_b / abs may be null)
  float* grad_planes;     // (n,3)
  float* grad_normals;    // (n,3)
};

struct RadeShared {
  float4 plane[kBlock];
  float4 normal[kBlock];
};

SPLAT_DEV void stage_rade(const RadeRenderParams& p, RadeShared& r, int slot, int g) {
  if (static_cast<unsigned>(g) >= static_cast<unsigned>(p.base.n_gaussians)) {
    r.plane[slot] = make_float4(0.0f, 0.0f, 0.0f, 0.0f);
    r.normal[slot] = make_float4(0.0f, 0.0f, 0.0f, 0.0f);
    return;
  }
  const float* pl = p.planes + 3 * static_cast<size_t>(g);
  const float* nm = p.normals + 3 * static_cast<size_t>(g);
  r.plane[slot] = make_float4(pl[0], pl[1], pl[2], 0.0f);
  r.normal[slot] = make_float4(nm[0], nm[1], nm[2], 0.0f);
}

template <int CHP>
SPLAT_DEV RadeShared& rade_shared(float4* dynamic) {
  return *reinterpret_cast<RadeShared*>(reinterpret_cast<char*>(dynamic) + sizeof(RenderShared<CHP>));
}

// rade/render.py:209-211: 1 / |(u, v, 1)| of the pixel centre's ray.
SPLAT_DEV float ray_scale(const RadeRenderParams& p, int x, int y) {
  const float u = (static_cast<float>(x) + 0.5f - __ldg(p.K + 2)) / __ldg(p.K);
  const float v = (static_cast<float>(y) + 0.5f - __ldg(p.K + 5)) / __ldg(p.K + 4);
  return 1.0f / sqrtf(u * u + v * v + 1.0f);
}

// rade/render.py:106-227 evaluate: one thread per pixel (kBlock per tile).
template <int CHP>
__global__ void __launch_bounds__(kBlock) rade_forward_kernel(RadeRenderParams p) {
  extern __shared__ float4 s_dynamic[];
  RenderShared<CHP>& s = *reinterpret_cast<RenderShared<CHP>*>(s_dynamic);
  RadeShared& r = rade_shared<CHP>(s_dynamic);
  __shared__ uint8_t s_list[kBlock / 32][kBlock];
  uint8_t* list = s_list[threadIdx.x >> 5];
  const RenderParams& b = p.base;
  const int tile = block_tile(b);
  const PixelSlot<1> ps = pixel_slot<1>(tile, b.gx);
  const int x = ps.x, y = ps.y;
  const bool inside = x < b.width && y < b.height;
  const float fx = static_cast<float>(x), fy = static_cast<float>(y);
  const int first = max(b.ranges[2 * tile], 0);
  const int last = min(b.ranges[2 * tile + 1], b.num_ids);
  const float threshold = 1.0f / 255.0f;
  bool done = !inside;
  float T = 1.0f, depth = 0.0f, median = 0.0f;
  float3 normal = make_float3(0.0f, 0.0f, 0.0f);
  int median_contributor = -1, last_contributor = 0;
  float color[CHP];
#pragma unroll
  for (int c = 0; c < CHP; ++c) color[c] = 0.0f;
  for (int begin = first; begin < last; begin += kBlock) {
    if (__syncthreads_count(done) == kBlock) break;
    const int idx = begin + threadIdx.x;
    if (idx < last) {
      const int g = b.ids[idx];
      stage_gaussian<CHP>(b, s, threadIdx.x, g);
      stage_rade(p, r, threadIdx.x, g);
    }
    __syncthreads();
    const int count = min(kBlock, last - begin);
    const int candidates = warp_candidates(s, ps, 0, count, list);
    for (int k = 0; k < candidates && !done; ++k) {
      const int j = list[k];
      const float4 q = s.conic[j];
      const float4 gm = s.geom[j];
      const float dx = gm.x - fx, dy = gm.y - fy;
      const float power = sample_power(q, dx, dy);
      if (power > 0.0f || power < s.cut[j]) continue;
      const float alpha = wmin(W32(0.99), q.w * splat_expf_core(power));
      if (!(alpha >= threshold)) continue;
      const float next_t = T * (1.0f - alpha);
      if (next_t < W32(0.0001)) {
        done = true;
        break;
      }
      const float w = alpha * T;
      float f[CHP];
      load_features(s, j, f);
#pragma unroll
      for (int c = 0; c < CHP; ++c) color[c] = __fmaf_rn(f[c], w, color[c]);
      const float4 pl = r.plane[j];
      const float distance = pl.x * dx + pl.y * dy + pl.z;
      depth += distance * w;
      const float4 nm = r.normal[j];
      normal.x += nm.x * w;
      normal.y += nm.y * w;
      normal.z += nm.z * w;
      const int position = begin - first + j + 1;
      if (b.stat_count) observe(b, s.id[j], y * b.width + x, w);
      if (T > 0.5f) {
        median = distance;
        median_contributor = position;
      }
      T = next_t;
      last_contributor = position;
    }
  }
  if (!inside) return;
  const size_t P = static_cast<size_t>(b.width) * b.height;
  const int pixel = y * b.width + x;
  float* feat = p.features + static_cast<size_t>(pixel) * p.feat_pix;
#pragma unroll
  for (int c = 0; c < CHP; ++c)
    if (c < b.channels) feat[c * p.feat_ch] = color[c] + T * b.background[c];
  const float rln = ray_scale(p, x, y);
  const float alpha = 1.0f - T;
  const float length = sqrtf(normal.x * normal.x + normal.y * normal.y + normal.z * normal.z);
  const float unit_scale = wmax(length, W32(1.0e-12));
  p.alpha[static_cast<size_t>(pixel) * p.alpha_pix] = alpha;
  p.depth[static_cast<size_t>(pixel) * p.depth_pix] =
      last_contributor > 0 ? depth * rln / alpha : 0.0f;
  p.median[static_cast<size_t>(pixel) * p.median_pix] = median * rln;
  float* nrm = p.normal_image + static_cast<size_t>(pixel) * p.normal_pix;
  nrm[0] = normal.x / unit_scale;
  nrm[p.normal_ch] = normal.y / unit_scale;
  nrm[2 * p.normal_ch] = normal.z / unit_scale;
  p.auxiliary[pixel] = depth * rln;
  p.auxiliary[P + pixel] = length;
  p.contributors[pixel] = last_contributor;
  p.contributors[P + pixel] = median_contributor;
}

// rade/render.py:106-227 evaluate with two pixels per lane (kBlock / 2
// threads per tile; warp w owns the 8x8 block, lane l the pixels (l % 8,
// l / 8) and (l % 8, l / 8 + 4)): the exponent, exp, alpha and
// transmittance of both pixels as f32x2 pairs (the bits of the scalar
// kernel), the colour channels as one packed fma per channel with the
// weight of a pixel that does not blend the sample set to zero, and the
// plane distance, depth, normal and median per pixel.
template <int CHP>
__global__ void __launch_bounds__(kBlock / 2) rade_forward2_kernel(RadeRenderParams p) {
  extern __shared__ float4 s_dynamic[];
  RenderShared<CHP>& s = *reinterpret_cast<RenderShared<CHP>*>(s_dynamic);
  RadeShared& r = rade_shared<CHP>(s_dynamic);
  __shared__ uint8_t s_list[kBlock / 64][kBlock];
  uint8_t* list = s_list[threadIdx.x >> 5];
  const RenderParams& b = p.base;
  const int tile = block_tile(b);
  const PixelSlot<2> ps = pixel_slot<2>(tile, b.gx);
  const int x = ps.x, y0 = ps.y, y1 = ps.y + 4;
  const bool inside0 = x < b.width && y0 < b.height;
  const bool inside1 = x < b.width && y1 < b.height;
  const float fx = static_cast<float>(x);
  const float fy0 = static_cast<float>(y0), fy1 = static_cast<float>(y1);
  const int first = max(b.ranges[2 * tile], 0);
  const int last = min(b.ranges[2 * tile + 1], b.num_ids);
  const float threshold = 1.0f / 255.0f;
  bool done0 = !inside0, done1 = !inside1;
  float T0 = 1.0f, T1 = 1.0f;
  f32x2 color2[CHP];
#pragma unroll
  for (int c = 0; c < CHP; ++c) color2[c] = splat2(0.0f);
  float depth0 = 0.0f, depth1 = 0.0f, median0 = 0.0f, median1 = 0.0f;
  float3 n0 = make_float3(0.0f, 0.0f, 0.0f), n1 = make_float3(0.0f, 0.0f, 0.0f);
  int last0 = 0, last1 = 0, mc0 = -1, mc1 = -1;
  for (int begin = first; begin < last; begin += kBlock) {
    if (__syncthreads_count(done0 && done1) == static_cast<int>(blockDim.x)) break;
    for (int slot = threadIdx.x; slot < kBlock; slot += blockDim.x) {
      const int idx = begin + slot;
      if (idx < last) {
        const int g = b.ids[idx];
        stage_gaussian<CHP>(b, s, slot, g);
        stage_rade(p, r, slot, g);
      }
    }
    __syncthreads();
    const int count = min(kBlock, last - begin);
    const int candidates = warp_candidates(s, ps, 0, count, list);
    for (int k = 0; k < candidates && !(done0 && done1); ++k) {
      const int j = list[k];
      const float4 q = s.conic[j];
      const float4 gm = s.geom[j];
      const float cut = s.cut[j];
      const float dx = gm.x - fx;
      const float dy0 = gm.y - fy0, dy1 = gm.y - fy1;
      const f32x2 power = sample_power2(q, dx, dy0, dy1);
      float pw0, pw1;
      unpack2(power, pw0, pw1);
      const bool range0 = !done0 && pw0 <= 0.0f && pw0 >= cut;
      const bool range1 = !done1 && pw1 <= 0.0f && pw1 >= cut;
      if (!(range0 || range1)) continue;
      float a0, a1;
      unpack2(mul2(splat2(q.w), splat_expf_core2(power)), a0, a1);
      a0 = wmin(W32(0.99), a0);
      a1 = wmin(W32(0.99), a1);
      const bool accept0 = range0 && a0 >= threshold;
      const bool accept1 = range1 && a1 >= threshold;
      if (!(accept0 || accept1)) continue;
      const f32x2 alpha = pack2(a0, a1), t = pack2(T0, T1);
      float nt0, nt1, w0, w1;
      unpack2(mul2(t, sub2(splat2(1.0f), alpha)), nt0, nt1);  // T * (1 - alpha)
      unpack2(mul2(alpha, t), w0, w1);                        // alpha * T
      const bool blend0 = accept0 && nt0 >= W32(0.0001);
      const bool blend1 = accept1 && nt1 >= W32(0.0001);
      done0 = done0 || (accept0 && !blend0);
      done1 = done1 || (accept1 && !blend1);
      if (!(blend0 || blend1)) continue;
      float f[CHP];
      load_features(s, j, f);
      const f32x2 w2 = pack2(blend0 ? w0 : 0.0f, blend1 ? w1 : 0.0f);
#pragma unroll
      for (int c = 0; c < CHP; ++c) color2[c] = fma2(splat2(f[c]), w2, color2[c]);
      const float4 pl = r.plane[j];
      const float4 nm = r.normal[j];
      const int position = begin - first + j + 1;
      if (blend0) {
        const float distance = pl.x * dx + pl.y * dy0 + pl.z;
        depth0 += distance * w0;
        n0.x += nm.x * w0;
        n0.y += nm.y * w0;
        n0.z += nm.z * w0;
        if (b.stat_count) observe(b, s.id[j], y0 * b.width + x, w0);
        if (T0 > 0.5f) {
          median0 = distance;
          mc0 = position;
        }
        T0 = nt0;
        last0 = position;
      }
      if (blend1) {
        const float distance = pl.x * dx + pl.y * dy1 + pl.z;
        depth1 += distance * w1;
        n1.x += nm.x * w1;
        n1.y += nm.y * w1;
        n1.z += nm.z * w1;
        if (b.stat_count) observe(b, s.id[j], y1 * b.width + x, w1);
        if (T1 > 0.5f) {
          median1 = distance;
          mc1 = position;
        }
        T1 = nt1;
        last1 = position;
      }
    }
  }
  const size_t P = static_cast<size_t>(b.width) * b.height;
#pragma unroll
  for (int i = 0; i < 2; ++i) {
    if (!(i ? inside1 : inside0)) continue;
    const int y = i ? y1 : y0;
    const int pixel = y * b.width + x;
    const float T = i ? T1 : T0;
    float* feat = p.features + static_cast<size_t>(pixel) * p.feat_pix;
#pragma unroll
    for (int c = 0; c < CHP; ++c) {
      float c0, c1;
      unpack2(color2[c], c0, c1);
      if (c < b.channels) feat[c * p.feat_ch] = (i ? c1 : c0) + T * b.background[c];
    }
    const float3 normal = i ? n1 : n0;
    const float depth = i ? depth1 : depth0;
    const int last_contributor = i ? last1 : last0;
    const float rln = ray_scale(p, x, y);
    const float alpha = 1.0f - T;
    const float length = sqrtf(normal.x * normal.x + normal.y * normal.y + normal.z * normal.z);
    const float unit_scale = wmax(length, W32(1.0e-12));
    p.alpha[static_cast<size_t>(pixel) * p.alpha_pix] = alpha;
    p.depth[static_cast<size_t>(pixel) * p.depth_pix] =
        last_contributor > 0 ? depth * rln / alpha : 0.0f;
    p.median[static_cast<size_t>(pixel) * p.median_pix] = (i ? median1 : median0) * rln;
    float* nrm = p.normal_image + static_cast<size_t>(pixel) * p.normal_pix;
    nrm[0] = normal.x / unit_scale;
    nrm[p.normal_ch] = normal.y / unit_scale;
    nrm[2 * p.normal_ch] = normal.z / unit_scale;
    p.auxiliary[pixel] = depth * rln;
    p.auxiliary[P + pixel] = length;
    p.contributors[pixel] = last_contributor;
    p.contributors[P + pixel] = i ? mc1 : mc0;
  }
}

// Destination of reduction value k of the rade backward: 0-1 centre, 2-5
// conic (incl. opacity), 6-7 |centre|, 8-10 plane, 11-13 normal, 14+c
// feature channel c.
SPLAT_DEV GradientSlot rade_gradient_slot(const RadeRenderParams& p, int k) {
  if (k < 8) return gradient_slot(p.base, k, 0);
  if (k < 11) return {p.grad_planes + (k - 8), 3};
  if (k < 14) return {p.grad_normals + (k - 11), 3};
  const int c = k - 14;
  if (c >= p.base.channels) return {nullptr, 0};
  return gradient_slot(p.base, 8 + c, p.base.channels);
}

// rade/render.py:336-545 backward with PX pixels per lane (kBlock / PX
// threads per tile; warp w owns an 8 x 4*PX block, lane l the pixels
// (l % 8, l / 8 + 4 i)).  Per pixel the replay carries S = sum over the
// blended quantities of (their blend behind the sample) x (their upstream
// gradient): dL/dalpha of a sample is T (F - S) - T_final/(1-alpha)
// dL/dT_final with F the sample's own sum_c f_c g_c + d g_depth +
// n . g_normal, and S += alpha (F - S) after it.  A lane sums its pixels'
// gradient values before the warp reduction (with PX = 2 one butterfly
// covers 64 pixels), and 16 lanes then add the warp totals with one red
// each.  Measured at config 4 (36 channels), one pixel per lane is fastest:
// PX = 2 needs 187 registers (8 warps per SM); direct atomics from lanes of
// sparsely covered samples, or a shared-memory accumulator flushed once per
// batch, were both slower than the reduction they replace.
template <int PX>
struct RadePixel {
  float fy, T, bg_term, depth_gradient, median_gradient, S, last_alpha, last_F;
  float3 normal_gradient;
  int last_contributor, median_contributor;
  bool inside;
};

template <int CHP, int PX>
__global__ void __launch_bounds__(kBlock / PX) rade_backward_kernel(RadeRenderParams p) {
  constexpr int kThreads = kBlock / PX;
  constexpr int kValues = 14 + CHP;
  constexpr int kGroups = (kValues + 15) / 16;
  extern __shared__ float4 s_dynamic[];
  RenderShared<CHP>& s = *reinterpret_cast<RenderShared<CHP>*>(s_dynamic);
  RadeShared& r = rade_shared<CHP>(s_dynamic);
  __shared__ uint8_t s_list[kThreads / 32][kBlock];
  __shared__ int s_max_last;
  // destination of the value that lane l holds after the reduction of group
  // grp (the same for every warp); null for odd lanes and unused values
  __shared__ GradientSlot s_dst[kGroups][32];
  uint8_t* list = s_list[threadIdx.x >> 5];
  const RenderParams& b = p.base;
  const int tile = block_tile(b);
  const int wl = threadIdx.x & 31;
  const PixelSlot<PX> ps = pixel_slot<PX>(tile, b.gx);
  const int first = max(b.ranges[2 * tile], 0);
  const int last = min(b.ranges[2 * tile + 1], b.num_ids);
  const float threshold = 1.0f / 255.0f;
  const float fx = static_cast<float>(ps.x);
  const size_t P = static_cast<size_t>(b.width) * b.height;
  const int C = b.channels;
  float grad[PX][CHP];
  RadePixel<PX> px[PX];
  int lane_last = 0;
#pragma unroll
  for (int i = 0; i < PX; ++i) {
    RadePixel<PX>& q = px[i];
    const int y = ps.y + 4 * i;
    q.fy = static_cast<float>(y);
    q.inside = ps.x < b.width && y < b.height;
    q.T = q.bg_term = q.depth_gradient = q.median_gradient = 0.0f;
    q.S = q.last_alpha = q.last_F = 0.0f;
    q.normal_gradient = make_float3(0.0f, 0.0f, 0.0f);
    q.last_contributor = 0;
    q.median_contributor = -1;
#pragma unroll
    for (int c = 0; c < CHP; ++c) grad[i][c] = 0.0f;
    if (q.inside) {
      const int pixel = y * b.width + ps.x;
      const float pixel_alpha = p.alpha[static_cast<size_t>(pixel) * p.alpha_pix];
      const float final_T = 1.0f - pixel_alpha;
      q.T = final_T;
      q.last_contributor = p.contributors[pixel];
      q.median_contributor = p.contributors[P + pixel];
      float bg_grad = 0.0f;
      const float* up = p.up_features ? p.up_features + static_cast<size_t>(pixel) * p.up_feat_pix
                                      : nullptr;
#pragma unroll
      for (int c = 0; c < CHP; ++c)
        if (c < C) {
          grad[i][c] = up ? __ldg(up + c * p.up_feat_ch) : 0.0f;
          bg_grad += b.background[c] * grad[i][c];
        }
      bg_grad -=
          p.up_alpha ? __ldg(p.up_alpha + static_cast<size_t>(pixel) * p.up_alpha_pix) : 0.0f;
      if (pixel_alpha > 0.0f) {
        const float rln = ray_scale(p, ps.x, y);
        const float gd =
            p.up_depth ? __ldg(p.up_depth + static_cast<size_t>(pixel) * p.up_depth_pix) : 0.0f;
        bg_grad += gd * (p.auxiliary[pixel] / pixel_alpha) / pixel_alpha;
        q.depth_gradient = gd / pixel_alpha * rln;
        q.median_gradient =
            (p.up_median ? __ldg(p.up_median + static_cast<size_t>(pixel) * p.up_median_pix)
                         : 0.0f) * rln;
        float3 ng = make_float3(0.0f, 0.0f, 0.0f);
        if (p.up_normals) {
          const float* un = p.up_normals + static_cast<size_t>(pixel) * p.up_normals_pix;
          ng = make_float3(__ldg(un), __ldg(un + p.up_normals_ch), __ldg(un + 2 * p.up_normals_ch));
        }
        const float* nrm = p.normal_image + static_cast<size_t>(pixel) * p.normal_pix;
        const float3 unit = make_float3(nrm[0], nrm[p.normal_ch], nrm[2 * p.normal_ch]);
        const float length = p.auxiliary[P + pixel];
        if (length >= W32(1.0e-12)) {
          const float d = dot3(unit, ng);
          ng.x -= unit.x * d;
          ng.y -= unit.y * d;
          ng.z -= unit.z * d;
        }
        const float sc = wmax(length, W32(1.0e-12));
        q.normal_gradient = make_float3(ng.x / sc, ng.y / sc, ng.z / sc);
      }
      q.bg_term = -final_T * bg_grad;
    }
    lane_last = max(lane_last, q.last_contributor);
  }
  if (threadIdx.x == 0) s_max_last = 0;
  for (int t = threadIdx.x; t < 32 * kGroups; t += kThreads) {
    const int grp = t >> 5, lane = t & 31;
    const int k = grp * 16 + butterfly_index(lane);
    GradientSlot d = k < kValues ? rade_gradient_slot(p, k) : GradientSlot{nullptr, 0};
    if (lane & 1) d.base = nullptr;
    s_dst[grp][lane] = d;
  }
  __syncthreads();
  const int warp_last = __reduce_max_sync(0xffffffffu, lane_last);
  if (wl == 0 && warp_last > 0) atomicMax(&s_max_last, warp_last);
  __syncthreads();
  const int stop = min(first + s_max_last, last);
  for (int end = stop; end > first; end -= kBlock) {
    __syncthreads();
    for (int slot = threadIdx.x; slot < kBlock; slot += kThreads) {
      const int idx = end - 1 - slot;
      if (idx >= first) {
        const int g = b.ids[idx];
        stage_gaussian<CHP>(b, s, slot, g);
        stage_rade(p, r, slot, g);
      }
    }
    __syncthreads();
    const int count = min(kBlock, end - first);
    const int candidates = warp_candidates(s, ps, max(0, end - first - warp_last), count, list);
    for (int k = 0; k < candidates; ++k) {
      const int j = list[k];
      const float4 gm = s.geom[j];
      const int position = end - 1 - j - first;  // contributor index - 1
      const float4 q = s.conic[j];
      const float dx = gm.x - fx;
      float dy[PX], G[PX], alpha[PX];
      bool accept[PX];
      bool any = false;
#pragma unroll
      for (int i = 0; i < PX; ++i) {
        dy[i] = gm.y - px[i].fy;
        const float power = sample_power(q, dx, dy[i]);
        const bool in_range = px[i].inside && position < px[i].last_contributor &&
                              power <= 0.0f && power >= s.cut[j];
        G[i] = splat_expf_core(power);
        alpha[i] = wmin(W32(0.99), q.w * G[i]);
        accept[i] = in_range && alpha[i] >= threshold;
        any = any || accept[i];
      }
      if (!__any_sync(0xffffffffu, any)) continue;
      float common[14];
#pragma unroll
      for (int v = 0; v < 14; ++v) common[v] = 0.0f;
      float weight[PX];
#pragma unroll
      for (int i = 0; i < PX; ++i) weight[i] = 0.0f;
      if (any) {
        float f[CHP];
        load_features(s, j, f);
        const float4 pl = r.plane[j];
        const float4 nm = r.normal[j];
#pragma unroll
        for (int i = 0; i < PX; ++i) {
          if (!accept[i]) continue;
          RadePixel<PX>& st = px[i];
          const float inv_one_minus = rcp_approx(1.0f - alpha[i]);
          st.T = st.T * inv_one_minus;
          const float distance = pl.x * dx + pl.y * dy[i] + pl.z;
          float F = distance * st.depth_gradient + nm.x * st.normal_gradient.x +
                    nm.y * st.normal_gradient.y + nm.z * st.normal_gradient.z;
#pragma unroll
          for (int c = 0; c < CHP; ++c) F = __fmaf_rn(f[c], grad[i][c], F);
          st.S = __fmaf_rn(st.last_alpha, st.last_F - st.S, st.S);
          st.last_F = F;
          st.last_alpha = alpha[i];
          const float w = alpha[i] * st.T;
          weight[i] = w;
          float g_distance = w * st.depth_gradient;
          if (position == st.median_contributor - 1) g_distance += st.median_gradient;
          const float grad_alpha = __fmaf_rn(F - st.S, st.T, st.bg_term * inv_one_minus);
          const float gv = q.w * grad_alpha;
          const float gdx = G[i] * dx, gdy = G[i] * dy[i];
          const float ddx = __fmaf_rn(g_distance, pl.x, -gv * __fmaf_rn(gdy, q.y, gdx * q.x));
          const float ddy = __fmaf_rn(g_distance, pl.y, -gv * __fmaf_rn(gdx, q.y, gdy * q.z));
          common[0] += ddx;
          common[1] += ddy;
          common[2] += -0.5f * gdx * dx * gv;
          common[3] += -gdx * dy[i] * gv;
          common[4] += -0.5f * gdy * dy[i] * gv;
          common[5] += G[i] * grad_alpha;
          common[6] += fabsf(ddx);
          common[7] += fabsf(ddy);
          common[8] += g_distance * dx;
          common[9] += g_distance * dy[i];
          common[10] += g_distance;
          common[11] += st.normal_gradient.x * w;
          common[12] += st.normal_gradient.y * w;
          common[13] += st.normal_gradient.z * w;
        }
      }
      const size_t g = static_cast<size_t>(s.id[j]);
#pragma unroll
      for (int grp = 0; grp < kGroups; ++grp) {
        float v16[16];
#pragma unroll
        for (int v = 0; v < 16; ++v) {
          const int idx = grp * 16 + v;
          if (idx < 14) {
            v16[v] = common[idx < 14 ? idx : 0];
          } else if (idx < kValues) {
            const int c = idx - 14 < CHP ? idx - 14 : 0;
            float acc = weight[0] * grad[0][c];
#pragma unroll
            for (int i = 1; i < PX; ++i) acc = __fmaf_rn(weight[i], grad[i][c], acc);
            v16[v] = acc;
          } else {
            v16[v] = 0.0f;
          }
        }
        const float total = butterfly16(v16, wl);
        const GradientSlot d = s_dst[grp][wl];
        if (d.base) red_add(d.base + g * d.stride, total);
      }
    }
  }
}

}  // namespace splat
