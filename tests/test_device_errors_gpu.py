"""Device-side errors reach the host without faulting or hanging the GPU.

* The count scan forms its total in 64 bits: 2^20 counts of 4096 sum to
  2^32, which the total reports exactly (no wrap) while the device error word
  reads -4, because the int32 offsets cannot hold it.  Both scan entry
  points (caller workspace and fixed in-library scratch) are checked.
* A bounded look-back wait on a status word that nothing publishes expires
  after its spin limit, records -3 and returns; the binning's host read then
  raises instead of training on wrong ranges.
"""

import pytest
import torch

from dsl_splat_b200 import _native as nv
from dsl_splat_b200 import gs3d
from dsl_splat_b200._native import lib
from dsl_splat_b200.scenes import make_scene

pytestmark = pytest.mark.gpu


def _stream(d):
    return torch.cuda.current_stream(d).cuda_stream


def test_scan_total_is_64_bit_and_reports_overflow():
    d = torch.device("cuda", 0)
    assert nv.device_error(d) == 0
    n = 1 << 20
    counts = torch.full((n,), 4096, dtype=torch.int32, device=d)
    offsets = torch.empty(n, dtype=torch.int32, device=d)
    total = torch.zeros(1, dtype=torch.int64, device=d)
    ws = torch.empty(lib.splat_scan_workspace_bytes(n), dtype=torch.uint8, device=d)
    assert lib.splat_scan_counts(n, counts.data_ptr(), offsets.data_ptr(), total.data_ptr(),
                                 ws.data_ptr(), ws.numel(), _stream(d)) == 0
    assert int(total) == 1 << 32
    assert nv.device_error(d) == -4
    total.fill_(0)
    assert lib.splat_scan_counts_static(n, counts.data_ptr(), offsets.data_ptr(),
                                        total.data_ptr(), _stream(d)) == 0
    assert int(total) == 1 << 32
    assert nv.device_error(d) == -4
    # one count less than the limit is exact and clean
    small = torch.full((1 << 19,), 4096, dtype=torch.int32, device=d)
    small[0] = 4095
    assert lib.splat_scan_counts(len(small), small.data_ptr(), offsets.data_ptr(),
                                 total.data_ptr(), ws.data_ptr(), ws.numel(), _stream(d)) == 0
    assert int(total) == (1 << 31) - 1
    assert nv.device_error(d) == 0
    assert int(offsets[len(small) - 1]) == (1 << 31) - 1


def test_expired_lookback_wait_is_reported_and_raised():
    d = torch.device("cuda", 0)
    assert nv.device_error(d) == 0
    status = torch.zeros(2, dtype=torch.int32, device=d)  # never published
    out = torch.zeros(1, dtype=torch.int32, device=d)
    assert lib.splat_test_lookback_expiry(status.data_ptr(), 4096, out.data_ptr(),
                                          _stream(d)) == 0
    torch.cuda.synchronize(d)  # the kernel ended: its wait was bounded
    assert int(out) == 0
    assert nv.device_error(d) == -3
    # an error recorded before a rasterize call surfaces in its binning read
    assert lib.splat_test_lookback_expiry(status.data_ptr(), 64, out.data_ptr(),
                                          _stream(d)) == 0
    s = make_scene(0, n=500)
    with pytest.raises(nv.SplatError, match="device error -3"):
        gs3d.rasterize(s.means.to(d), s.quats.to(d), s.scales.to(d), s.opacities.to(d),
                       s.viewmats.to(d), s.Ks.to(d), s.width, s.height,
                       sh_coeffs=s.sh_coeffs.to(d))
    assert nv.device_error(d) == 0  # the read reset it
    gs3d.rasterize(s.means.to(d), s.quats.to(d), s.scales.to(d), s.opacities.to(d),
                   s.viewmats.to(d), s.Ks.to(d), s.width, s.height, sh_coeffs=s.sh_coeffs.to(d))
