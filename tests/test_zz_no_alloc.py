"""splat_scan_exclusive_u32_noalloc through the C ABI: the scan whose block sums live in the library's fixed
device array instead of a caller workspace. Two calls in a row (different sizes, then the maximum size) must give
exactly what splat_scan_exclusive_u32 gives on the same inputs; a size above the maximum is rejected before any
launch. Collected last so that it also runs after every other GPU test in the same process."""
from __future__ import annotations

import pytest
import torch

from gs_b200 import _lib as L

pytestmark = pytest.mark.gpu

MAX_N = 1 << 28  # SPLAT_SCAN_NOALLOC_MAX_N
SPLAT_ERR_ARG = 1
SPLAT_ERR_OVERFLOW = 3


def _scan_with_workspace(x: torch.Tensor):
    n = x.numel()
    out = torch.empty_like(x)
    tot = torch.zeros(1, dtype=torch.int32, device=x.device)
    ws = L.workspace(L.query("splat_scan_workspace_size", n), x.device)
    L.call("splat_scan_exclusive_u32", L.ptr(x), L.ptr(out), n, L.ptr(tot), L.ptr(ws), ws.numel(), L.stream_of(x))
    return out, tot


def _scan_noalloc(x: torch.Tensor):
    out = torch.empty_like(x)
    tot = torch.zeros(1, dtype=torch.int32, device=x.device)
    L.call("splat_scan_exclusive_u32_noalloc", L.ptr(x), L.ptr(out), x.numel(), L.ptr(tot), L.stream_of(x))
    return out, tot


def test_noalloc_scan_matches_workspace_scan_twice_in_a_row(cuda):
    g = torch.Generator(device=cuda).manual_seed(11)
    for n, hi in ((1_000_003, 50), (MAX_N, 4)):  # the second call reuses the array the first one wrote
        x = torch.randint(0, hi, (n,), dtype=torch.int32, device=cuda, generator=g)
        got, got_total = _scan_noalloc(x)
        ref, ref_total = _scan_with_workspace(x)
        torch.cuda.synchronize()
        assert torch.equal(got, ref), f"n={n}"
        assert int(got_total.item()) == int(ref_total.item()) == int(x.sum(dtype=torch.int64).item())


def test_noalloc_scan_small_and_empty(cuda):
    for n in (0, 1, 4095, 4096, 4097):
        x = torch.arange(n, dtype=torch.int32, device=cuda) % 7
        got, got_total = _scan_noalloc(x)
        ref, ref_total = _scan_with_workspace(x)
        assert torch.equal(got, ref)
        assert int(got_total.item()) == int(ref_total.item())


def test_noalloc_scan_rejects_sizes_above_the_maximum(cuda):
    lib = L.load()
    status = lib.splat_scan_exclusive_u32_noalloc(None, None, MAX_N + 1, None, None)
    assert status == SPLAT_ERR_OVERFLOW
    assert b"exceeds its maximum" in lib.splat_last_error()


def test_noalloc_scan_rejects_buffers_that_are_not_on_the_current_device(cuda):
    """The fixed array is the current device's, so host memory is refused before any launch."""
    import ctypes

    import numpy as np

    lib = L.load()
    host = np.zeros(64, dtype=np.uint32)
    dev_out = torch.empty(64, dtype=torch.int32, device=cuda)
    status = lib.splat_scan_exclusive_u32_noalloc(host.ctypes.data_as(ctypes.c_void_p), L.ptr(dev_out), 64, None,
                                                  None)
    assert status == SPLAT_ERR_ARG
    assert b"in " in lib.splat_last_error() or b"in must" in lib.splat_last_error()
