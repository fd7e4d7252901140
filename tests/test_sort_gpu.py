"""Device scan and stable radix sort through the C ABI vs numpy (bit-exact)."""
from __future__ import annotations

import numpy as np
import pytest
import torch

from gs_b200 import _lib as L

pytestmark = pytest.mark.gpu


def _sort(keys: torch.Tensor, vals: torch.Tensor, begin: int, end: int):
    n = keys.numel()
    kb = keys.element_size()
    ko, vo = torch.empty_like(keys), torch.empty_like(vals)
    ws = L.workspace(L.query("splat_sort_workspace_size", n, kb), keys.device)
    L.call("splat_radix_sort_pairs", L.ptr(keys), L.ptr(vals), L.ptr(ko), L.ptr(vo), n, kb, begin, end, L.ptr(ws),
           ws.numel(), L.stream_of(keys))
    return ko, vo


@pytest.mark.parametrize("n", [0, 1, 31, 4095, 4096, 4097, 100_003, 2_000_000])
@pytest.mark.parametrize("key_bytes,bits", [(4, (0, 32)), (8, (0, 64)), (8, (0, 45)), (4, (3, 17))])
def test_radix_sort_matches_stable_argsort(n, key_bytes, bits, cuda):
    rng = np.random.default_rng(n + key_bytes + bits[1])
    begin, end = bits
    if key_bytes == 4:
        k = rng.integers(0, 2**32, n, dtype=np.uint64).astype(np.uint32)
        kt = torch.tensor(k.view(np.int32), device=cuda)
        mask = np.uint64(((1 << end) - 1) ^ ((1 << begin) - 1))
        sort_key = k.astype(np.uint64) & mask
    else:
        k = rng.integers(0, 2**63, n, dtype=np.uint64) * np.uint64(2) + rng.integers(0, 2, n, dtype=np.uint64)
        k[: n // 3] = k[: n // 3] & np.uint64(0xFFF)  # many duplicates
        kt = torch.tensor(k.view(np.int64), device=cuda)
        mask = np.uint64((1 << 64) - 1 if end == 64 else ((1 << end) - 1) ^ ((1 << begin) - 1))
        sort_key = k & mask
    vals = torch.arange(n, dtype=torch.int32, device=cuda)
    ko, vo = _sort(kt, vals, begin, end)
    perm = np.argsort(sort_key, kind="stable")
    assert np.array_equal(vo.cpu().numpy(), perm.astype(np.int32))
    got = ko.cpu().numpy().view(np.uint32 if key_bytes == 4 else np.uint64)
    assert np.array_equal(got, k[perm])


@pytest.mark.parametrize("n", [0, 1, 4096, 4097, 1_000_001, 20_000_000])
def test_scan_matches_cumsum(n, cuda):
    rng = np.random.default_rng(n)
    x = rng.integers(0, 50, n).astype(np.int32)
    xt = torch.tensor(x, device=cuda)
    out = torch.empty_like(xt)
    tot = torch.zeros(1, dtype=torch.int32, device=cuda)
    ws = L.workspace(L.query("splat_scan_workspace_size", n), cuda)
    L.call("splat_scan_exclusive_u32", L.ptr(xt), L.ptr(out), n, L.ptr(tot), L.ptr(ws), ws.numel(), L.stream_of(xt))
    ref = np.cumsum(x, dtype=np.int64) - x
    assert np.array_equal(out.cpu().numpy().astype(np.int64), ref)
    assert int(tot.item()) == int(x.sum())
