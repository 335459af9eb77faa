// Per-camera preparation (full = P*V, camera centres) and its pose VJP.
// Restates splatting/camera_kernels.py:11-106 with the same separate float32
// products and sums (that module compiles with fuse_fp=False; this library
// compiles with -fmad=false).
#pragma once
#include "splat_common.cuh"

namespace splat {

// 4x4 inverse by 2x2 minors (Laplace expansion; Eberly, "The Laplace
// Expansion Theorem: Computing the Determinants and Inverses of Matrices").
// Returns the determinant; inv is written only when it is nonzero.
SPLAT_DEV float inverse44(const float* m, float* inv) {
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
  if (det == 0.0f) return det;
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
  return det;
}

// splatting/camera_kernels.py:11-66 prepare_kernel.
__global__ void cameras_prepare_kernel(int count, const float* __restrict__ views,
                                       const float* __restrict__ Ks, int width, int height,
                                       int with_centers, float* __restrict__ full,
                                       float* __restrict__ inverse, float* __restrict__ centers,
                                       int* __restrict__ errors) {
  const int i = blockIdx.x * blockDim.x + threadIdx.x;
  if (i >= count) return;
  const float* K = Ks + 9 * i;
  const float* V = views + 16 * i;
  bool finite = true;
  for (int j = 0; j < 9; ++j) finite = finite && isfinite(K[j]);
  int error = 0;
  if (!finite || K[0] <= 0.0f || K[4] <= 0.0f)
    error = 2;
  else if (K[1] != 0.0f || K[3] != 0.0f || K[6] != 0.0f || K[7] != 0.0f || K[8] != 1.0f)
    error = 1;
  errors[i] = error;
  if (error != 0) return;
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
    float m[16], inv[16];
    for (int j = 0; j < 16; ++j) m[j] = V[j];
    if (inverse44(m, inv) == 0.0f) {
      errors[i] = 3;
      return;
    }
    for (int j = 0; j < 16; ++j) inverse[16 * i + j] = inv[j];
    for (int r = 0; r < 3; ++r) centers[3 * i + r] = inv[r * 4 + 3];
  }
}

// splatting/camera_kernels.py:69-106 backward_kernel.
__global__ void cameras_backward_kernel(int count, const float* __restrict__ Ks,
                                        const float* __restrict__ grad_full, int width,
                                        int height, const float* __restrict__ inverse,
                                        const float* __restrict__ grad_centers,
                                        float* __restrict__ grad_views) {
  const int i = blockIdx.x * blockDim.x + threadIdx.x;
  if (i >= count) return;
  const float* K = Ks + 9 * i;
  const float px = 2.0f * K[0] / static_cast<float>(width);
  const float py = 2.0f * K[4] / static_cast<float>(height);
  const float cx = 2.0f * K[2] / static_cast<float>(width) - 1.0f;
  const float cy = 2.0f * K[5] / static_cast<float>(height) - 1.0f;
  const float* g = grad_full ? grad_full + 16 * i : nullptr;
  const float* inv = inverse + 16 * i;
  const float* gc = grad_centers ? grad_centers + 3 * i : nullptr;
  for (int row = 0; row < 4; ++row)
    for (int col = 0; col < 4; ++col) {
      float value = 0.0f;
      if (g) {
        if (row == 0)
          value = px * g[0 * 4 + col];
        else if (row == 1)
          value = py * g[1 * 4 + col];
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

}  // namespace splat
