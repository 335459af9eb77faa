// Shared device helpers for the sm_100a gs3d rasteriser.
//
// The library is compiled with -fmad=false: every a*b+c below is two IEEE
// roundings unless the code calls __fmaf_rn, which mirrors the reference's
// explicit fmaf / fused_multiply_add calls (dsl_splat primitives/math.py,
// splatting/math.py) and makes integer outputs (radii, tile counts, keys)
// reproducible by the CPU oracle bit for bit.
#pragma once

#include <cuda_runtime.h>
#include <stdint.h>

#define SPLAT_DEV __device__ __forceinline__

namespace splat {

constexpr int kTile = 16;              // 16x16-pixel tiles (gs3d/render.py:57-61)
constexpr int kBlock = 256;            // one CTA per tile, one thread per pixel
constexpr uint32_t kCulledKey = 0xFFFFFFFFu;

// Status codes returned by every C entry point (0 = success).
enum Status : int {
  kOk = 0,
  kInvalidArgument = -1,
  kCudaError = -2,
  kDeviceTimeout = -3,
  kTooLarge = -4,
  kWorkspaceTooSmall = -5,
  kInconsistentInput = -6,  // device-side guard skipped an out-of-range index
};

// A Python float literal in a Warp kernel is the double value rounded to
// float32; W32 makes the same conversion.
#define W32(x) static_cast<float>(x)

SPLAT_DEV float wmax(float a, float b) { return a > b ? a : b; }
SPLAT_DEV float wmin(float a, float b) { return a < b ? a : b; }
SPLAT_DEV float wclamp(float x, float a, float b) { return wmin(wmax(a, x), b); }
SPLAT_DEV int iclamp(int x, int a, int b) { return min(max(a, x), b); }

// float -> int32, truncating, saturating, NaN -> 0 (Warp int() on CUDA).
SPLAT_DEV int f2i(float x) { return __float2int_rz(x); }

// exp(x): Cody-Waite argument reduction (x = n ln2 + r with ln2 split into
// a 9-bit head 0.693359375 and a correction), the degree-7 Taylor series of
// exp(r) evaluated by Horner's rule with fused multiply-adds, and scaling by
// 2^n through the exponent field.  Each step is one IEEE float32 operation,
// so the CPU oracle computes the same bits and both sides take the same
// alpha-threshold decisions.  Maximum error below 1 ulp on [-80, 0].
SPLAT_DEV float splat_expf_core(float x);

SPLAT_DEV float splat_expf(float x) {
  if (!(x > -80.0f)) return 0.0f;
  if (x > 88.0f) x = 88.0f;
  return splat_expf_core(x);
}

// splat_expf for arguments already known to lie in (-80, 88]: the same bits
// without the range guards.
SPLAT_DEV float splat_expf_core(float x) {
  const float n = rintf(__fmul_rn(x, 1.44269504088896341f));
  float r = __fmaf_rn(n, -0.693359375f, x);
  r = __fmaf_rn(n, 2.12194440054690583e-4f, r);
  float p = 1.98412698e-4f;
  p = __fmaf_rn(p, r, 1.38888889e-3f);
  p = __fmaf_rn(p, r, 8.33333377e-3f);
  p = __fmaf_rn(p, r, 4.16666679e-2f);
  p = __fmaf_rn(p, r, 1.66666672e-1f);
  p = __fmaf_rn(p, r, 0.5f);
  p = __fmaf_rn(p, r, 1.0f);
  p = __fmaf_rn(p, r, 1.0f);
  const float scale = __int_as_float((static_cast<int>(n) + 127) << 23);
  return __fmul_rn(p, scale);
}

// F.normalize(x, dim=-1) for one wxyz quaternion with the bits Torch's CUDA
// kernels produce (inputs.py:252): x / clamp_min(|x|, 1e-12), where |x|^2 is
// summed as (x0^2 + x2^2) + (x1^2 + x3^2) and every operation is a single
// IEEE float32 operation (NaN norms propagate like clamp_min).
SPLAT_DEV float4 torch_normalize4(float4 x) {
  const float sq = __fadd_rn(__fadd_rn(__fmul_rn(x.x, x.x), __fmul_rn(x.z, x.z)),
                             __fadd_rn(__fmul_rn(x.y, x.y), __fmul_rn(x.w, x.w)));
  float norm = __fsqrt_rn(sq);
  if (norm < W32(1e-12)) norm = W32(1e-12);
  return make_float4(__fdiv_rn(x.x, norm), __fdiv_rn(x.y, norm), __fdiv_rn(x.z, norm),
                     __fdiv_rn(x.w, norm));
}

// Packed float32 pairs (sm_100 f32x2 arithmetic): each half is an
// independent IEEE round-to-nearest float32 operation, so a pair computes
// the same bits as two scalar operations in one issue slot.  Caution: ptxas
// fuses a packed multiply whose only use is a packed add/sub into a fused
// multiply-add, ignoring .rn and --fmad=false; bit-exact code must not chain
// mul2 into add2/sub2.
typedef unsigned long long f32x2;

SPLAT_DEV f32x2 pack2(float lo, float hi) {
  f32x2 r;
  asm("mov.b64 %0, {%1, %2};" : "=l"(r) : "f"(lo), "f"(hi));
  return r;
}
SPLAT_DEV void unpack2(f32x2 v, float& lo, float& hi) {
  asm("mov.b64 {%0, %1}, %2;" : "=f"(lo), "=f"(hi) : "l"(v));
}
SPLAT_DEV f32x2 add2(f32x2 a, f32x2 b) {
  f32x2 r;
  asm("add.rn.f32x2 %0, %1, %2;" : "=l"(r) : "l"(a), "l"(b));
  return r;
}
SPLAT_DEV f32x2 sub2(f32x2 a, f32x2 b) {
  f32x2 r;
  asm("sub.rn.f32x2 %0, %1, %2;" : "=l"(r) : "l"(a), "l"(b));
  return r;
}
SPLAT_DEV f32x2 mul2(f32x2 a, f32x2 b) {
  f32x2 r;
  asm("mul.rn.f32x2 %0, %1, %2;" : "=l"(r) : "l"(a), "l"(b));
  return r;
}
SPLAT_DEV f32x2 fma2(f32x2 a, f32x2 b, f32x2 c) {
  f32x2 r;
  asm("fma.rn.f32x2 %0, %1, %2, %3;" : "=l"(r) : "l"(a), "l"(b), "l"(c));
  return r;
}
SPLAT_DEV f32x2 splat2(float v) { return pack2(v, v); }

// splat_expf_core on both halves: the same operations, paired.
SPLAT_DEV f32x2 splat_expf_core2(f32x2 x) {
  float t0, t1;
  unpack2(mul2(x, splat2(1.44269504088896341f)), t0, t1);
  const float n0 = rintf(t0), n1 = rintf(t1);
  const f32x2 n = pack2(n0, n1);
  f32x2 r = fma2(n, splat2(-0.693359375f), x);
  r = fma2(n, splat2(2.12194440054690583e-4f), r);
  f32x2 p = fma2(splat2(1.98412698e-4f), r, splat2(1.38888889e-3f));
  p = fma2(p, r, splat2(8.33333377e-3f));
  p = fma2(p, r, splat2(4.16666679e-2f));
  p = fma2(p, r, splat2(1.66666672e-1f));
  p = fma2(p, r, splat2(0.5f));
  p = fma2(p, r, splat2(1.0f));
  p = fma2(p, r, splat2(1.0f));
  const float s0 = __int_as_float((static_cast<int>(n0) + 127) << 23);
  const float s1 = __int_as_float((static_cast<int>(n1) + 127) << 23);
  return mul2(p, pack2(s0, s1));
}

// log(x) for the tile-mode footprints (splatting/intersections.py:60):
// x = 2^k m with m in [sqrt(1/2), sqrt(2)), s = (m-1)/(m+1) as f/(2+f),
// log m = 2 atanh(s) = 2s (1 + s^2/3 + s^4/5 + s^6/7 + s^8/9), plus k ln2
// with ln2 split into 0.693359375 and a correction.  The same IEEE float32
// steps as the CPU oracle, so tile bounds agree bit for bit (within 2.4 ulp
// of log).  +inf -> +inf, 0 -> -inf, negative or NaN -> NaN.
SPLAT_DEV float splat_logf(float x) {
  if (!(x > 0.0f)) return x == 0.0f ? -INFINITY : __int_as_float(0x7fc00000);
  if (x == INFINITY) return x;
  uint32_t u = __float_as_uint(x);
  int k = 0;
  if (u < 0x00800000u) {  // subnormal: scale into the normal range
    x = __fmul_rn(x, 8388608.0f);
    u = __float_as_uint(x);
    k = -23;
  }
  k += static_cast<int>(u >> 23) - 127;
  float m = __uint_as_float((u & 0x007FFFFFu) | 0x3F800000u);
  if (m > 1.41421356f) {
    m = __fmul_rn(m, 0.5f);
    k += 1;
  }
  const float f = __fsub_rn(m, 1.0f);
  const float s = __fdiv_rn(f, __fadd_rn(2.0f, f));
  const float z = __fmul_rn(s, s);
  float p = W32(1.0 / 9.0);
  p = __fmaf_rn(p, z, W32(1.0 / 7.0));
  p = __fmaf_rn(p, z, W32(1.0 / 5.0));
  p = __fmaf_rn(p, z, W32(1.0 / 3.0));
  p = __fmaf_rn(p, z, 1.0f);
  const float log_m = __fmul_rn(__fmul_rn(2.0f, s), p);
  const float kf = static_cast<float>(k);
  return __fadd_rn(__fmul_rn(kf, 0.693359375f), __fmaf_rn(kf, -2.12194440054690583e-4f, log_m));
}

// splatting/geometry.py:22-30 tile_bounds: CUDA getRect truncation.
SPLAT_DEV int4 tile_bounds(float cx, float cy, int radius, int gx, int gy) {
  const float r = static_cast<float>(radius);
  int4 b;
  b.x = iclamp(f2i(__fdiv_rn(__fsub_rn(cx, r), 16.0f)), 0, gx);
  b.y = iclamp(f2i(__fdiv_rn(__fsub_rn(cy, r), 16.0f)), 0, gy);
  b.z = iclamp(f2i(__fdiv_rn(__fsub_rn(__fadd_rn(__fadd_rn(cx, r), 16.0f), 1.0f), 16.0f)), 0, gx);
  b.w = iclamp(f2i(__fdiv_rn(__fsub_rn(__fadd_rn(__fadd_rn(cy, r), 16.0f), 1.0f), 16.0f)), 0, gy);
  return b;
}

// Relaxed device-scope loads/stores for look-back status words.
SPLAT_DEV uint32_t ld_relaxed(const uint32_t* p) {
  uint32_t v;
  asm volatile("ld.relaxed.gpu.global.u32 %0, [%1];" : "=r"(v) : "l"(p) : "memory");
  return v;
}
SPLAT_DEV void st_relaxed(uint32_t* p, uint32_t v) {
  asm volatile("st.relaxed.gpu.global.u32 [%0], %1;" ::"l"(p), "r"(v) : "memory");
}
SPLAT_DEV unsigned long long ld_relaxed64(const unsigned long long* p) {
  unsigned long long v;
  asm volatile("ld.relaxed.gpu.global.u64 %0, [%1];" : "=l"(v) : "l"(p) : "memory");
  return v;
}
SPLAT_DEV void st_relaxed64(unsigned long long* p, unsigned long long v) {
  asm volatile("st.relaxed.gpu.global.u64 [%0], %1;" ::"l"(p), "l"(v) : "memory");
}

// Vector reductions into global memory (sm_90+).
SPLAT_DEV void red_add_v2(float* p, float a, float b) {
  asm volatile("red.relaxed.gpu.global.add.v2.f32 [%0], {%1, %2};" ::"l"(p), "f"(a), "f"(b)
               : "memory");
}
SPLAT_DEV void red_add_v4(float* p, float a, float b, float c, float d) {
  asm volatile("red.relaxed.gpu.global.add.v4.f32 [%0], {%1, %2, %3, %4};" ::"l"(p), "f"(a),
               "f"(b), "f"(c), "f"(d)
               : "memory");
}
SPLAT_DEV void red_add(float* p, float a) {
  asm volatile("red.relaxed.gpu.global.add.f32 [%0], %1;" ::"l"(p), "f"(a) : "memory");
}

SPLAT_DEV float warp_sum(float v) {
#pragma unroll
  for (int o = 16; o > 0; o >>= 1) v += __shfl_xor_sync(0xffffffffu, v, o);
  return v;
}

SPLAT_DEV uint32_t lanemask_lt() {
  uint32_t m;
  asm("mov.u32 %0, %%lanemask_lt;" : "=r"(m));
  return m;
}

}  // namespace splat
