"""splat_scan_counts_static: the count scan without caller scratch.

Callers that cannot allocate device memory at call time (a host whose device
memory is all owned by its own pool, a render loop that cannot afford
cudaMalloc's implicit synchronisation, a plugin whose framework forbids new
allocations) use this entry point; its scratch is a fixed 64 KiB device array
inside the library.  These checks call it through the C ABI twice in a row and
compare with splat_scan_counts (which takes a caller workspace): integer
results, so they must be identical.  The file sorts last so that a run which
stops at the first failure has already run every other test; it also passes
alone in a fresh process (the first call performs the per-device set-up).
"""

import pytest
import torch

from dsl_splat_b200._native import lib

pytestmark = pytest.mark.gpu

MAX_COUNT = 16384 * 4096


def _with_workspace(counts: torch.Tensor):
    n = len(counts)
    offsets = torch.empty(n, dtype=torch.int32, device=counts.device)
    total = torch.zeros(1, dtype=torch.int64, device=counts.device)
    ws = torch.empty(lib.splat_scan_workspace_bytes(n), dtype=torch.uint8, device=counts.device)
    stream = torch.cuda.current_stream(counts.device).cuda_stream
    assert lib.splat_scan_counts(n, counts.data_ptr(), offsets.data_ptr(), total.data_ptr(),
                                 ws.data_ptr(), ws.numel(), stream) == 0
    return offsets, total


def _static(counts: torch.Tensor):
    n = len(counts)
    offsets = torch.full((n,), -7, dtype=torch.int32, device=counts.device)
    total = torch.full((1,), -7, dtype=torch.int64, device=counts.device)
    stream = torch.cuda.current_stream(counts.device).cuda_stream
    status = lib.splat_scan_counts_static(n, counts.data_ptr(), offsets.data_ptr(),
                                          total.data_ptr(), stream)
    assert status == 0, lib.splat_last_error()
    return offsets, total


def test_static_scan_matches_workspace_scan_twice():
    dev = torch.device("cuda", 0)
    g = torch.Generator(device="cpu").manual_seed(5)
    first = torch.randint(0, 40, (3_000_001,), generator=g, dtype=torch.int32).to(dev)
    second = torch.randint(0, 9000, (70_000,), generator=g, dtype=torch.int32).to(dev)
    for counts in (first, second):  # two calls in a row reuse the shared scratch
        want_off, want_total = _with_workspace(counts)
        got_off, got_total = _static(counts)
        torch.cuda.synchronize(dev)
        assert torch.equal(got_off, want_off)
        assert int(got_total) == int(want_total) == int(counts.sum())


def test_static_scan_rejects_counts_beyond_its_scratch():
    stream = torch.cuda.current_stream(0).cuda_stream
    status = lib.splat_scan_counts_static(MAX_COUNT + 1, None, None, None, stream)
    assert status == -4
    assert b"at most 67108864" in lib.splat_last_error()
