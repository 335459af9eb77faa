// The blend's kernel parameters and the few helpers that the forward
// (aaa_render.cuh, built without multiply-add contraction for bit-exact
// images) and the record backward (aaa_backward.cuh, its own translation
// unit, built with contraction) share.
#pragma once
#include <cuda_runtime.h>

#include "splat_common.cuh"

namespace splat {
namespace aaa {

constexpr unsigned kFull = 0xffffffffu;

SPLAT_DEV float wp_min(float a, float b) { return a < b ? a : b; }  // wp.min on floats

SPLAT_DEV float rdot3(const float a[3], const float b[3]) { return (a[0] * b[0] + a[1] * b[1]) + a[2] * b[2]; }

struct HierParams {
  int width, height, channels, cull;
  int n;                    // Gaussians (ids outside [0, n) are never read)
  const int* ranges;        // (T,2)
  const int* points;        // sorted Gaussian ids
  const float* transforms;  // (n,4,4), 16-byte aligned
  const float* opacity;     // (n)
  const float* colors;      // (n,C)
  const float* bg;          // (C)
  const int* tile_order;    // block -> tile schedule, or null
  // forward outputs: planar (C,H,W), (H,W), (H,W)
  float* image;
  float* final_t;
  int* contributors;
  // replay inputs (the forward's outputs) and gradients
  const float* image_in;
  const float* final_t_in;
  const float* pixel_grad;  // (C,H,W)
  float* grad_transforms;   // (n,16), the reference's transposed layout
  float* grad_opacity;      // (n)
  float* grad_colors;       // (n,C)
  float* grad_screen;       // (n,2) or null
  float* grad_screen_abs;   // (n,2) or null
  // blend records (forward, optional): per tile-local pixel its blended
  // samples in blend order, at most record_capacity (<= 256), entry
  // ((tile * capacity + j) << 8) + local = (tile-slice position as int bits,
  // Gaussian value); the record backward overwrites each filed entry with
  // (blend weight, gaussian * dL/dalpha)
  int record_capacity;
  float2* records;
  int* record_counts;       // (T*256): count, or -1 when the capacity overflowed
  int* tile_overflow;       // (T): 1 when a pixel of the tile overflowed
  const int* only_flagged;  // replay: run only the tiles whose flag is set
  // forward contribution statistics (statistics.py:47-73), or stat_count 0:
  // request r is a weighted sum when bit r of stat_sum_mask is set, else a
  // masked count; rows of n
  int stat_count, stat_sum_mask;
  const float* stat_pixels;  // (stat_count, H*W)
  int* stat_counts;
  float* stat_sums;
};

// The record backward of a recorded blend (aaa_backward.cu): every tile not
// flagged in p.tile_overflow, from its blend records.
int record_backward_dispatch(const HierParams& p, int tiles, bool screen, bool absgrad,
                             cudaStream_t s);

}  // namespace aaa
}  // namespace splat
