// The AAA record backward (aaa_backward.cuh) and its launch.
//
// This translation unit is compiled with multiply-add contraction
// (-fmad=true) and the approximate divide and square root, unlike the
// blend it differentiates: its outputs are gradients, compared within a
// relative tolerance, and contraction removes a large part of the
// per-sample arithmetic.
#include "aaa_backward.cuh"
#include "host_runtime.h"

namespace splat {
namespace aaa {
namespace {

using host::check_launch;
using host::counted;

template <int CHP, bool SCREEN, bool ABS>
int launch_record(const HierParams& p, int tiles, cudaStream_t s) {
  const size_t smem = sizeof(TileShared);
  static bool configured = false;  // the shared-memory opt-in, once per instantiation
  if (!configured) {
    if (cudaFuncSetAttribute(aaa_record_backward_kernel<CHP, SCREEN, ABS>,
                             cudaFuncAttributeMaxDynamicSharedMemorySize,
                             static_cast<int>(smem)) != cudaSuccess)
      return check_launch("aaa_record_backward shared memory");
    configured = true;
  }
  aaa_record_backward_kernel<CHP, SCREEN, ABS><<<tiles, 256, smem, counted(s)>>>(p);
  return check_launch("aaa_record_backward");
}

template <int CHP>
int launch_record_flags(const HierParams& p, int tiles, bool screen, bool absgrad,
                        cudaStream_t s) {
  if (!screen) return launch_record<CHP, false, false>(p, tiles, s);
  if (!absgrad) return launch_record<CHP, true, false>(p, tiles, s);
  return launch_record<CHP, true, true>(p, tiles, s);
}

}  // namespace

int record_backward_dispatch(const HierParams& p, int tiles, bool screen, bool absgrad,
                             cudaStream_t s) {
  if (p.channels <= 4) return launch_record_flags<4>(p, tiles, screen, absgrad, s);
  if (p.channels <= 8) return launch_record_flags<8>(p, tiles, screen, absgrad, s);
  if (p.channels <= 16) return launch_record_flags<16>(p, tiles, screen, absgrad, s);
  if (p.channels <= 32) return launch_record_flags<32>(p, tiles, screen, absgrad, s);
  return launch_record_flags<64>(p, tiles, screen, absgrad, s);
}

}  // namespace aaa
}  // namespace splat
