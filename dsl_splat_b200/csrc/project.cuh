// gs3d projection forward, fused with SH0-3 and metadata, and the shared
// math of the backward.
//
// Forward restates gs3d/projection.py:37-164 (screen_covariance, project),
// splatting/geometry.py:22-123 and primitives/sh.py:7-79 operation by
// operation (compiled with -fmad=false; __fmaf_rn where the reference calls
// fmaf).  The projection backward kernel lives in project_backward.cu; the
// standalone SH VJP (primitives/sh.py:82-138) is here.
#pragma once
#include "splat_common.cuh"
#include "tile_modes.cuh"

namespace splat {

struct ProjectParams {
  int n;
  const float* means;      // (n,3)
  const float* quats;      // (n,4) normalised wxyz, or raw when normalize_quats
  int normalize_quats;     // normalise in-kernel exactly as Torch's F.normalize does on CUDA
  int tile_mode;           // kTileRadius / kTileSnugbox / kTileAccutile (tile count only)
  const float* scales;     // (n,3)
  const float* opacities;  // (n)
  const float* view;       // 4x4 row-major world->camera
  const float* proj;       // 4x4 full projection (camera_kernels.py:42-52)
  const float* K;          // 3x3 intrinsics
  int width, height;
  float near_plane, far_plane, radius_clip;
  float* centers;  // (n,2)  written for visible rows only
  float* conics;   // (n,4)  (inv_a, inv_b, inv_c, opacity), visible rows only
  int* radii;      // (n)
  int* tiles;      // (n)
  float* depths;   // (n)    visible rows only
  // optional fused SH (sh == nullptr disables)
  int sh_degree;
  int sh_k;                // coefficients stored per Gaussian (K >= (deg+1)^2)
  const float* sh;         // (n,K,3)
  const float* campos;     // (3) camera centre; null => directions = means
  float* colors;           // (n, color_stride) first 3 columns written
  int color_stride;
  uint8_t* active;         // (n,3) or null
  // optional dense metadata (splatting/metadata.py:12-31), null disables
  float* meta_means2d;     // (n,2)
  float* meta_opacities;   // (n)
  float* meta_conics;      // (n,3)
};

struct Mat3 {
  float m[3][3];
};

// splatting/math.py:31-42 reference_matmul
SPLAT_DEV Mat3 ref_matmul(const Mat3& a, const Mat3& b) {
  Mat3 r;
#pragma unroll
  for (int row = 0; row < 3; ++row)
#pragma unroll
    for (int col = 0; col < 3; ++col)
      r.m[row][col] = __fmaf_rn(a.m[row][2], b.m[2][col],
                                __fmaf_rn(a.m[row][0], b.m[0][col], a.m[row][1] * b.m[1][col]));
  return r;
}

SPLAT_DEV Mat3 transpose(const Mat3& a) {
  Mat3 r;
#pragma unroll
  for (int i = 0; i < 3; ++i)
#pragma unroll
    for (int j = 0; j < 3; ++j) r.m[i][j] = a.m[j][i];
  return r;
}

// splatting/math.py:44-47 point_row
SPLAT_DEV float point_row(const float* m, int row, float p0, float p1, float p2) {
  const float xy = __fmaf_rn(m[row * 4 + 0], p0, m[row * 4 + 1] * p1);
  return __fmaf_rn(m[row * 4 + 2], p2, xy) + m[row * 4 + 3];
}

// primitives/math.py:33-45 glm_rotation
SPLAT_DEV Mat3 glm_rotation(float r, float x, float y, float z) {
  const float yy = y * y, zz = z * z;
  const float rz = r * z, xz = x * z, rx = r * x;
  const float d0 = yy + zz, d1 = __fmaf_rn(x, x, zz), d2 = __fmaf_rn(x, x, yy);
  Mat3 R;
  R.m[0][0] = 1.0f - (d0 + d0);
  R.m[0][1] = 2.0f * __fmaf_rn(x, y, rz);
  R.m[0][2] = 2.0f * __fmaf_rn(-r, y, xz);
  R.m[1][0] = 2.0f * __fmaf_rn(x, y, -rz);
  R.m[1][1] = 1.0f - (d1 + d1);
  R.m[1][2] = 2.0f * __fmaf_rn(y, z, rx);
  R.m[2][0] = 2.0f * __fmaf_rn(r, y, xz);
  R.m[2][1] = 2.0f * __fmaf_rn(y, z, -rx);
  R.m[2][2] = 1.0f - (d2 + d2);
  return R;
}

// gs3d/projection.py:37-86 screen_covariance
SPLAT_DEV float3 screen_covariance(float px, float py, float pz, float4 q, float3 s,
                                   const float* view, int width, int height, float fx,
                                   float fy) {
  const float limx = W32(1.3) * static_cast<float>(width) / (2.0f * fx);
  const float limy = W32(1.3) * static_cast<float>(height) / (2.0f * fy);
  const float tx = wclamp(px / pz, -limx, limx) * pz;
  const float ty = wclamp(py / pz, -limy, limy) * pz;
  const float tz = pz;
  const Mat3 R = glm_rotation(q.x, q.y, q.z, q.w);
  const Mat3 S = {{{s.x, 0.0f, 0.0f}, {0.0f, s.y, 0.0f}, {0.0f, 0.0f, s.z}}};
  const Mat3 M = ref_matmul(S, R);
  const Mat3 cov = ref_matmul(transpose(M), M);
  const Mat3 J = {{{fx / tz, 0.0f, 0.0f},
                   {0.0f, fy / tz, 0.0f},
                   {-(fx * tx) / (tz * tz), -(fy * ty) / (tz * tz), 0.0f}}};
  const Mat3 cam = {{{view[0], view[4], view[8]}, {view[1], view[5], view[9]},
                     {view[2], view[6], view[10]}}};
  const Mat3 T = ref_matmul(cam, J);
  const Mat3 P = ref_matmul(ref_matmul(transpose(T), transpose(cov)), T);
  return make_float3(P.m[0][0] + W32(0.3), P.m[1][0], P.m[1][1] + W32(0.3));
}

// splatting/geometry.py:106-123 pixel_center
SPLAT_DEV float2 pixel_center(float m0, float m1, float m2, const float* proj, int width,
                              int height) {
  const float c0 = point_row(proj, 0, m0, m1, m2);
  const float c1 = point_row(proj, 1, m0, m1, m2);
  const float c3 = point_row(proj, 3, m0, m1, m2);
  const float inverse_w = 1.0f / (c3 + W32(1e-7));
  const double ndc_x = static_cast<double>(c0 * inverse_w);
  const double ndc_y = static_cast<double>(c1 * inverse_w);
  return make_float2(
      static_cast<float>(((ndc_x + 1.0) * static_cast<double>(width) - 1.0) * 0.5),
      static_cast<float>(((ndc_y + 1.0) * static_cast<double>(height) - 1.0) * 0.5));
}

// primitives/sh.py:7-41 basis (Warp literals are float32-rounded doubles).
SPLAT_DEV float sh_basis(float x, float y, float z, int k) {
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

// d basis_k / d unit (what wp.grad(basis) evaluates at primitives/sh.py:127).
SPLAT_DEV float3 sh_basis_grad(float x, float y, float z, int k) {
  const float c1 = W32(0.4886025119029199), c4 = W32(1.0925484305920792);
  const float c6 = W32(0.31539156525252005), c8 = W32(0.5462742152960396);
  const float c9 = -W32(0.5900435899266435), c10 = W32(2.890611442640554);
  const float c11 = -W32(0.4570457994644658), c12 = W32(0.3731763325901154);
  const float c14 = W32(1.445305721320277);
  switch (k) {
    case 0: return make_float3(0.0f, 0.0f, 0.0f);
    case 1: return make_float3(0.0f, -c1, 0.0f);
    case 2: return make_float3(0.0f, 0.0f, c1);
    case 3: return make_float3(-c1, 0.0f, 0.0f);
    case 4: return make_float3(c4 * y, c4 * x, 0.0f);
    case 5: return make_float3(0.0f, -c4 * z, -c4 * y);
    case 6: return make_float3(-2.0f * c6 * x, -2.0f * c6 * y, 4.0f * c6 * z);
    case 7: return make_float3(-c4 * z, 0.0f, -c4 * x);
    case 8: return make_float3(2.0f * c8 * x, -2.0f * c8 * y, 0.0f);
    case 9: return make_float3(c9 * 6.0f * x * y, c9 * (3.0f * x * x - 3.0f * y * y), 0.0f);
    case 10: return make_float3(c10 * y * z, c10 * x * z, c10 * x * y);
    case 11:
      return make_float3(c11 * (-2.0f * x * y), c11 * (4.0f * z * z - x * x - 3.0f * y * y),
                         c11 * (8.0f * y * z));
    case 12:
      return make_float3(c12 * (-6.0f * x * z), c12 * (-6.0f * y * z),
                         c12 * (6.0f * z * z - 3.0f * x * x - 3.0f * y * y));
    case 13:
      return make_float3(c11 * (4.0f * z * z - 3.0f * x * x - y * y), c11 * (-2.0f * x * y),
                         c11 * (8.0f * x * z));
    case 14:
      return make_float3(c14 * 2.0f * x * z, -c14 * 2.0f * y * z, c14 * (x * x - y * y));
    default:
      return make_float3(c9 * (3.0f * x * x - 3.0f * y * y), c9 * (-6.0f * x * y), 0.0f);
  }
}

// primitives/sh.py:44-79 forward for one Gaussian (visible rows only).
template <int DEG>
SPLAT_DEV float3 sh_eval(const float* __restrict__ coef, float d0, float d1, float d2) {
  float ux = 0.0f, uy = 0.0f, uz = 0.0f;
  if (DEG > 0) {
    const float len = sqrtf(d0 * d0 + d1 * d1 + d2 * d2);
    const float den = wmax(len, W32(1e-12));
    ux = d0 / den;
    uy = d1 / den;
    uz = d2 / den;
  }
  float v0 = 0.0f, v1 = 0.0f, v2 = 0.0f;
#pragma unroll
  for (int k = 0; k < (DEG + 1) * (DEG + 1); ++k) {
    const float b = sh_basis(ux, uy, uz, k);
    v0 = v0 + b * coef[3 * k + 0];
    v1 = v1 + b * coef[3 * k + 1];
    v2 = v2 + b * coef[3 * k + 2];
  }
  return make_float3(v0 + 0.5f, v1 + 0.5f, v2 + 0.5f);
}

// SH rows are staged per warp through shared memory: each of the warp's 32
// Gaussians owns a row of kShCols floats there (stride kShCols + 1, so lanes
// reading their own rows hit distinct banks), and global rows move with
// consecutive lanes on consecutive addresses.
constexpr int kProjectBlock = 128;
constexpr int kProjectWarps = kProjectBlock / 32;

template <int DEG>
struct ShTile {
  static constexpr int kCols = DEG >= 0 ? 3 * (DEG + 1) * (DEG + 1) : 1;
  static constexpr int kStride = kCols + 1;
};

// rows [base, base+32) of a (n, row_stride) array, first kCols columns.
template <int DEG>
SPLAT_DEV void warp_load_sh(const float* __restrict__ src, int row_stride, int base, int n,
                            float* tile) {
  constexpr int C = ShTile<DEG>::kCols, S = ShTile<DEG>::kStride;
  const int lane = threadIdx.x & 31;
  const int rows = min(32, n - base);
  if (row_stride == C && rows == 32) {
    // The warp's rows are one contiguous block of 32*C floats: lane-strided
    // independent loads, unrolled so many are in flight at once.
    const float* g = src + static_cast<size_t>(base) * C;
#pragma unroll 12
    for (int k = 0; k < C; ++k) {
      const int e = k * 32 + lane;
      const int r = e / C;
      tile[r * S + (e - r * C)] = g[e];
    }
  } else {
    for (int r = 0; r < rows; ++r) {
      const float* row = src + static_cast<size_t>(base + r) * row_stride;
      for (int t = lane; t < C; t += 32) tile[r * S + t] = row[t];
    }
  }
  __syncwarp();
}

// One camera's view of the inputs and the outputs it writes (ProjectParams
// fields; the multi-view kernel takes them from per-view tables).
struct ProjectCamera {
  const float* view;    // 4x4 row-major world->camera
  const float* proj;    // 4x4 full projection
  const float* K;       // 3x3 intrinsics
  const float* campos;  // (3) or null
};

struct ProjectOutputs {
  float* centers;
  float* conics;
  int* radii;
  int* tiles;
  float* depths;
  float* colors;
  uint8_t* active;
  float* meta_means2d;
  float* meta_opacities;
  float* meta_conics;
};

// The per-Gaussian inputs, read once per Gaussian whatever the number of views.
struct GaussianInput {
  float m0, m1, m2;
  float4 q;  // normalised quaternion (w, x, y, z)
  float3 s;
  float opacity;
};

SPLAT_DEV GaussianInput load_gaussian(const float* means, const float* quats, int normalize,
                                      const float* scales, const float* opacities, int i) {
  GaussianInput g;
  g.m0 = means[3 * i];
  g.m1 = means[3 * i + 1];
  g.m2 = means[3 * i + 2];
  g.q = reinterpret_cast<const float4*>(quats)[i];
  if (normalize) g.q = torch_normalize4(g.q);
  g.s = make_float3(scales[3 * i], scales[3 * i + 1], scales[3 * i + 2]);
  g.opacity = opacities[i];
  return g;
}

// gs3d/projection.py:89-164 (+ primitives/sh.py:44-79, splatting/metadata.py:12-31)
// for Gaussian i seen by one camera; `row` is its staged SH row (null: no SH).
// p supplies the settings shared by all views (image size, planes, clip,
// tile mode, SH degree and colour stride).
template <int DEG>
SPLAT_DEV void project_gaussian(const ProjectParams& p, const ProjectCamera& cam,
                                const ProjectOutputs& out, int i, const GaussianInput& g,
                                const float* row) {
  const int gx = (p.width + 15) / 16, gy = (p.height + 15) / 16;
  int radius_out = 0, count_out = 0;
  float2 center = make_float2(0.0f, 0.0f);
  float4 conic = make_float4(0.0f, 0.0f, 0.0f, 0.0f);
  const float m0 = g.m0, m1 = g.m1, m2 = g.m2;
  do {
    const float t0 = point_row(cam.view, 0, m0, m1, m2);
    const float t1 = point_row(cam.view, 1, m0, m1, m2);
    const float t2 = point_row(cam.view, 2, m0, m1, m2);
    if (t2 <= p.near_plane || t2 >= p.far_plane) break;
    const float3 cov = screen_covariance(t0, t1, t2, g.q, g.s, cam.view, p.width, p.height,
                                         cam.K[0], cam.K[4]);
    const float a = cov.x, b = cov.y, c = cov.z;
    const float det = a * c - b * b;
    if (det == 0.0f) break;
    const float mid = 0.5f * (a + c);
    const int radius = f2i(ceilf(3.0f * sqrtf(mid + sqrtf(wmax(W32(0.1), mid * mid - det)))));
    if (static_cast<float>(radius) <= p.radius_clip) break;
    center = pixel_center(m0, m1, m2, cam.proj, p.width, p.height);
    const int4 bnd = tile_bounds(center.x, center.y, radius, gx, gy);
    const int count = (bnd.z - bnd.x) * (bnd.w - bnd.y);
    if (count == 0) break;
    const float inverse = 1.0f / (a * c - b * b);
    conic = make_float4(c * inverse, -b * inverse, a * inverse, g.opacity);
    reinterpret_cast<float2*>(out.centers)[i] = center;
    reinterpret_cast<float4*>(out.conics)[i] = conic;
    out.depths[i] = t2;
    radius_out = radius;
    count_out = count;
    // gs3d/projection.py:150-162: the mode's tile count replaces the square's
    // (the Gaussian keeps its radius even when that count is 0)
    if (p.tile_mode != kTileRadius)
      count_out = tile_count(tile_visit(p.tile_mode, center.x, center.y, conic, radius, gx, gy));
  } while (false);
  out.radii[i] = radius_out;
  out.tiles[i] = count_out;
  const bool visible = radius_out > 0;
  if (DEG >= 0 && row != nullptr) {
    float3 v = make_float3(0.0f, 0.0f, 0.0f);
    if (visible) {
      float d0 = m0, d1 = m1, d2 = m2;
      if (cam.campos != nullptr) {
        d0 = m0 - cam.campos[0];
        d1 = m1 - cam.campos[1];
        d2 = m2 - cam.campos[2];
      }
      v = sh_eval<(DEG < 0 ? 0 : DEG)>(row, d0, d1, d2);
    }
    float* col = out.colors + static_cast<size_t>(i) * p.color_stride;
    col[0] = wmax(v.x, 0.0f);
    col[1] = wmax(v.y, 0.0f);
    col[2] = wmax(v.z, 0.0f);
    if (out.active != nullptr) {
      out.active[3 * i + 0] = visible && v.x >= 0.0f;
      out.active[3 * i + 1] = visible && v.y >= 0.0f;
      out.active[3 * i + 2] = visible && v.z >= 0.0f;
    }
  }
  if (out.meta_means2d != nullptr) {
    // culled rows (including those culled after the centre was computed)
    // are zero, as splatting/metadata.py:28-32 writes them
    reinterpret_cast<float2*>(out.meta_means2d)[i] = visible ? center : make_float2(0.0f, 0.0f);
    out.meta_opacities[i] = visible ? conic.w : 0.0f;
    out.meta_conics[3 * i + 0] = visible ? conic.x : 0.0f;
    out.meta_conics[3 * i + 1] = visible ? conic.y : 0.0f;
    out.meta_conics[3 * i + 2] = visible ? conic.z : 0.0f;
  }
}

template <int DEG>
__global__ void __launch_bounds__(kProjectBlock) project_forward_kernel(ProjectParams p) {
  __shared__ float s_sh[kProjectWarps][32 * ShTile<DEG>::kStride];
  const int lane = threadIdx.x & 31, warp = threadIdx.x >> 5;
  const int base = (blockIdx.x * kProjectWarps + warp) * 32;
  if (base >= p.n) return;  // uniform per warp
  float* tile = s_sh[warp];
  const bool sh = DEG >= 0 && p.sh != nullptr;
  if (sh) warp_load_sh<DEG>(p.sh, p.sh_k * 3, base, p.n, tile);
  const int i = base + lane;
  if (i >= p.n) return;
  const GaussianInput g =
      load_gaussian(p.means, p.quats, p.normalize_quats, p.scales, p.opacities, i);
  project_gaussian<DEG>(p, ProjectCamera{p.view, p.proj, p.K, p.campos},
                        ProjectOutputs{p.centers, p.conics, p.radii, p.tiles, p.depths, p.colors,
                                       p.active, p.meta_means2d, p.meta_opacities,
                                       p.meta_conics},
                        i, g, sh ? tile + lane * ShTile<DEG>::kStride : nullptr);
}

// Up to kMaxViews cameras of one Gaussian set in one launch: each warp stages
// its 32 SH rows and each thread loads its Gaussian once, then projects it
// for every camera (the same arithmetic as project_forward_kernel).  Camera
// v's matrices are rows v of the stacked arrays; its outputs come from the
// per-view pointer tables.
constexpr int kMaxViews = 16;

struct ProjectViewsParams {
  ProjectParams shared;  // inputs, settings; its camera/output fields are unused
  int views;
  const float* viewmats;  // (views,4,4)
  const float* projs;     // (views,4,4)
  const float* Ks;        // (views,3,3)
  const float* campos;    // (views,3) or null
  float* centers[kMaxViews];
  float* conics[kMaxViews];
  int* radii[kMaxViews];
  int* tiles[kMaxViews];
  float* depths[kMaxViews];
  float* colors[kMaxViews];
  uint8_t* active[kMaxViews];
  float* meta_means2d[kMaxViews];
  float* meta_opacities[kMaxViews];
  float* meta_conics[kMaxViews];
};

template <int DEG>
__global__ void __launch_bounds__(kProjectBlock) project_forward_views_kernel(ProjectViewsParams vp) {
  const ProjectParams& p = vp.shared;
  __shared__ float s_sh[kProjectWarps][32 * ShTile<DEG>::kStride];
  const int lane = threadIdx.x & 31, warp = threadIdx.x >> 5;
  const int base = (blockIdx.x * kProjectWarps + warp) * 32;
  if (base >= p.n) return;  // uniform per warp
  float* tile = s_sh[warp];
  const bool sh = DEG >= 0 && p.sh != nullptr;
  if (sh) warp_load_sh<DEG>(p.sh, p.sh_k * 3, base, p.n, tile);
  const int i = base + lane;
  if (i >= p.n) return;
  const GaussianInput g =
      load_gaussian(p.means, p.quats, p.normalize_quats, p.scales, p.opacities, i);
  const float* row = sh ? tile + lane * ShTile<DEG>::kStride : nullptr;
  for (int v = 0; v < vp.views; ++v) {
    const ProjectCamera cam{vp.viewmats + 16 * v, vp.projs + 16 * v, vp.Ks + 9 * v,
                            vp.campos ? vp.campos + 3 * v : nullptr};
    const ProjectOutputs out{vp.centers[v], vp.conics[v], vp.radii[v], vp.tiles[v],
                             vp.depths[v], vp.colors[v], vp.active[v], vp.meta_means2d[v],
                             vp.meta_opacities[v], vp.meta_conics[v]};
    project_gaussian<DEG>(p, cam, out, i, g, row);
  }
}

// splatting/metadata.py:12-31 _prepare (standalone stage).
static __global__ void metadata_kernel(int n, const int* __restrict__ radii,
                                const float* __restrict__ centers,
                                const float* __restrict__ conics, float* __restrict__ means2d,
                                float* __restrict__ opacities, float* __restrict__ conics3) {
  const int i = blockIdx.x * blockDim.x + threadIdx.x;
  if (i >= n) return;
  float2 c = make_float2(0.0f, 0.0f);
  float4 q = make_float4(0.0f, 0.0f, 0.0f, 0.0f);
  if (radii[i] > 0) {
    c = reinterpret_cast<const float2*>(centers)[i];
    q = reinterpret_cast<const float4*>(conics)[i];
  }
  reinterpret_cast<float2*>(means2d)[i] = c;
  opacities[i] = q.w;
  conics3[3 * i + 0] = q.x;
  conics3[3 * i + 1] = q.y;
  conics3[3 * i + 2] = q.z;
}

// rows [base, base+32) of a (n, row_stride) array from the warp's tile: the
// first kCols columns from the tile, any further ones as zeros; consecutive
// lanes store consecutive addresses.
template <int DEG>
SPLAT_DEV void warp_store_sh(float* __restrict__ dst, int row_stride, int base, int n,
                             const float* tile) {
  constexpr int C = ShTile<DEG>::kCols, S = ShTile<DEG>::kStride;
  const int lane = threadIdx.x & 31;
  const int rows = min(32, n - base);
  __syncwarp();
  if (row_stride == C && rows == 32) {
    float* g = dst + static_cast<size_t>(base) * C;
#pragma unroll 12
    for (int k = 0; k < C; ++k) {
      const int e = k * 32 + lane;
      const int r = e / C;
      g[e] = tile[r * S + (e - r * C)];
    }
  } else {
    for (int r = 0; r < rows; ++r) {
      float* row = dst + static_cast<size_t>(base + r) * row_stride;
      for (int t = lane; t < row_stride; t += 32) row[t] = t < C ? tile[r * S + t] : 0.0f;
    }
  }
}

// The standalone SH kernels stage each warp's 32 coefficient rows through
// shared memory (warp_load_sh / warp_store_sh): a lane reading its own
// Gaussian's 48 floats straight from global memory touches 32 cache lines
// per warp-wide load.  128 threads per block.

// primitives/sh.py:44-79 standalone SH forward (masked when radii != null).
template <int DEG>
__global__ void __launch_bounds__(kProjectBlock)
sh_forward_kernel(int n, int sh_k, const float* __restrict__ sh, const float* __restrict__ dirs,
                  const int* __restrict__ radii, float* __restrict__ colors,
                  uint8_t* __restrict__ active) {
  constexpr int S = ShTile<DEG>::kStride;
  __shared__ float tiles[kProjectWarps][32 * S];
  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
  const int base = (blockIdx.x * kProjectWarps + warp) * 32;
  if (base >= n) return;
  float* tile = tiles[warp];
  warp_load_sh<DEG>(sh, 3 * sh_k, base, n, tile);
  const int i = base + lane;
  if (i >= n) return;
  const bool visible = radii ? radii[i] > 0 : true;
  float3 v = make_float3(0.0f, 0.0f, 0.0f);
  if (visible) v = sh_eval<DEG>(tile + lane * S, dirs[3 * i], dirs[3 * i + 1], dirs[3 * i + 2]);
  colors[3 * i + 0] = wmax(v.x, 0.0f);
  colors[3 * i + 1] = wmax(v.y, 0.0f);
  colors[3 * i + 2] = wmax(v.z, 0.0f);
  if (active) {
    active[3 * i + 0] = visible && v.x >= 0.0f;
    active[3 * i + 1] = visible && v.y >= 0.0f;
    active[3 * i + 2] = visible && v.z >= 0.0f;
  }
}

// primitives/sh.py:82-138 VJP for one Gaussian, in place: row holds the
// first (DEG+1)^2 coefficient triples and receives their gradient; returns
// the direction gradient.
template <int DEG>
SPLAT_DEV float3 sh_vjp(float* row, float d0, float d1, float d2, float3 cg) {
  float ux = 0.0f, uy = 0.0f, uz = 0.0f, length = 1.0f;
  if (DEG > 0) {
    length = sqrtf(d0 * d0 + d1 * d1 + d2 * d2);
    const float den = wmax(length, W32(1e-12));
    ux = d0 / den;
    uy = d1 / den;
    uz = d2 / den;
  }
  float g0 = 0.0f, g1 = 0.0f, g2 = 0.0f;
#pragma unroll
  for (int k = 0; k < (DEG + 1) * (DEG + 1); ++k) {
    const float b = sh_basis(ux, uy, uz, k);
    float* o = row + 3 * k;
    if (DEG > 0) {  // the coefficients' weight, read before the row is overwritten
      const float w = o[0] * cg.x + o[1] * cg.y + o[2] * cg.z;
      const float3 bg = sh_basis_grad(ux, uy, uz, k);
      g0 += w * bg.x;
      g1 += w * bg.y;
      g2 += w * bg.z;
    }
    o[0] = b * cg.x;
    o[1] = b * cg.y;
    o[2] = b * cg.z;
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

// primitives/sh.py:82-138 VJP for one Gaussian from global rows: writes (or
// adds into) the (K,3) coefficient gradient (zeros past (DEG+1)^2 when
// writing) and returns the direction gradient.
template <int DEG>
SPLAT_DEV float3 sh_vjp_global(const float* __restrict__ coef, int sh_k, float d0, float d1,
                               float d2, float3 cg, float* __restrict__ gcoef, bool accumulate) {
  float ux = 0.0f, uy = 0.0f, uz = 0.0f, length = 1.0f;
  if (DEG > 0) {
    length = sqrtf(d0 * d0 + d1 * d1 + d2 * d2);
    const float den = wmax(length, W32(1e-12));
    ux = d0 / den;
    uy = d1 / den;
    uz = d2 / den;
  }
  float g0 = 0.0f, g1 = 0.0f, g2 = 0.0f;
#pragma unroll
  for (int k = 0; k < (DEG + 1) * (DEG + 1); ++k) {
    const float b = sh_basis(ux, uy, uz, k);
    float* o = gcoef + 3 * k;
    if (accumulate) {
      o[0] += b * cg.x;
      o[1] += b * cg.y;
      o[2] += b * cg.z;
    } else {
      o[0] = b * cg.x;
      o[1] = b * cg.y;
      o[2] = b * cg.z;
    }
    if (DEG > 0) {
      const float w = coef[3 * k] * cg.x + coef[3 * k + 1] * cg.y + coef[3 * k + 2] * cg.z;
      const float3 bg = sh_basis_grad(ux, uy, uz, k);
      g0 += w * bg.x;
      g1 += w * bg.y;
      g2 += w * bg.z;
    }
  }
  if (!accumulate)
    for (int k = (DEG + 1) * (DEG + 1); k < sh_k; ++k) {
      gcoef[3 * k] = 0.0f;
      gcoef[3 * k + 1] = 0.0f;
      gcoef[3 * k + 2] = 0.0f;
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
__global__ void __launch_bounds__(kProjectBlock)
sh_backward_kernel(int n, int sh_k, const float* __restrict__ sh, const float* __restrict__ dirs,
                   const int* __restrict__ radii, const uint8_t* __restrict__ active,
                   const float* __restrict__ upstream, float* __restrict__ grad_sh,
                   float* __restrict__ grad_dirs) {
  constexpr int C = ShTile<DEG>::kCols, S = ShTile<DEG>::kStride;
  __shared__ float tiles[kProjectWarps][32 * S];
  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
  const int base = (blockIdx.x * kProjectWarps + warp) * 32;
  if (base >= n) return;
  float* tile = tiles[warp];
  warp_load_sh<DEG>(sh, 3 * sh_k, base, n, tile);
  const int i = base + lane;
  if (i < n) {
    const bool visible = radii ? radii[i] > 0 : true;
    float* row = tile + lane * S;
    float3 dg = make_float3(0.0f, 0.0f, 0.0f);
    if (visible) {
      const float3 cg = make_float3(active[3 * i] ? upstream[3 * i] : 0.0f,
                                    active[3 * i + 1] ? upstream[3 * i + 1] : 0.0f,
                                    active[3 * i + 2] ? upstream[3 * i + 2] : 0.0f);
      dg = sh_vjp<DEG>(row, dirs[3 * i], dirs[3 * i + 1], dirs[3 * i + 2], cg);
    } else {
      for (int k = 0; k < C; ++k) row[k] = 0.0f;
    }
    if (grad_dirs) {
      grad_dirs[3 * i + 0] = dg.x;
      grad_dirs[3 * i + 1] = dg.y;
      grad_dirs[3 * i + 2] = dg.z;
    }
  }
  warp_store_sh<DEG>(grad_sh, 3 * sh_k, base, n, tile);
}

struct ProjectBackwardParams {
  int n;
  const float* means;
  const float* quats;
  const float* scales;
  const float* view;
  const float* proj;
  const float* K;
  int width, height;
  const int* radii;
  const float* seed_centers;  // (n,2) dL/dcenters
  const float* seed_conics;   // (n,4) dL/dconics (incl. opacity)
  float* grad_means;          // (n,3) or null
  float* grad_quats;          // (n,4) or null
  // When set, grad_quats receives the gradient w.r.t. quats_raw (the
  // normalisation's VJP applied in-kernel); quats may then be null, and the
  // normalised quaternions are recomputed from quats_raw.
  const float* quats_raw;     // (n,4) or null
  float* grad_scales;         // (n,3) or null
  float* grad_opacities;      // (n)   or null
  int accumulate;             // add into grad_* instead of overwriting
  // camera reductions (float[35]: view 16, proj 16, campos 3), null disables
  float* cam_grads;
  // optional fused SH backward
  int sh_degree;
  int sh_k;
  const float* sh;
  const float* campos;
  const uint8_t* active;
  const float* seed_colors;   // (n, color_stride)
  int color_stride;
  float* grad_sh;             // (n,K,3)
};

// Projection (+ SH) backward launch (project_backward.cu, compiled with
// multiply-add contraction: gradients are compared within tolerance, not
// bit for bit).  Returns a status code.
int project_backward_dispatch(const ProjectBackwardParams& p, cudaStream_t s);

}  // namespace splat
