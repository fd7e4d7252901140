"""Failure detection without a GPU fault (the reference's failure modes: a zero-block launch on an empty view,
phase2/fastergs_readback.patch:32-34; an unbounded CUB look-back wait; a count past 32-bit indexing).

On the host (no device work): bounds a caller exceeds come back as SPLAT_ERR_OVERFLOW before any launch, and the
look-back poll limit is validated. On the GPU: a radix sort whose look-back waits are made to give up (a poll limit
of one) returns normally with an exact result (the tiles recount their offsets), reports SPLAT_ERR_TIMEOUT from
splat_check_device_waits, and the forward that follows raises; Gaussians with NaN or infinite parameters are culled, leaving the image
and the other Gaussians' gradients as if they were absent.
"""
from __future__ import annotations

import ctypes

import pytest
import torch

from gs_b200 import _lib as L
from gs_b200 import gs3d, scenes

SPLAT_ERR_ARG, SPLAT_ERR_OVERFLOW, SPLAT_ERR_TIMEOUT = 1, 3, 4


def _settings(width=64, height=48):
    fake = 0x1000  # never dereferenced: the calls below return before any device work
    return gs3d._Settings(fake, fake, fake, 16, 15, width, height, 50.0, 50.0, width / 2, height / 2, 0.2, 1000.0, 0)


def test_instance_count_past_32_bit_lists_is_an_overflow():
    lib = L.load()
    s = _settings()
    big = 1 << 31
    status = lib.gs3d_render(1, big, ctypes.byref(s), None, 0, None, 0, None, 0, None, 0, 1 << 40, None, None)
    assert status == SPLAT_ERR_OVERFLOW
    assert b"instances exceed" in lib.splat_last_error()
    status = lib.gs3d_render_inference(1, big, ctypes.byref(s), None, 0, None, 0, None, 0, None, None)
    assert status == SPLAT_ERR_OVERFLOW


def test_bucket_capacity_below_its_bound_is_an_overflow():
    lib = L.load()
    s = _settings()
    m = 10_000
    bound = int(lib.gs3d_bucket_bound(m, 64, 48))
    status = lib.gs3d_render(1, m, ctypes.byref(s), None, 0, None, 0, None, 0, None, 0, bound - 1, None, None)
    assert status == SPLAT_ERR_OVERFLOW
    assert b"below the bound" in lib.splat_last_error()


def test_lookback_poll_limit_is_validated():
    lib = L.load()
    assert lib.splat_set_lookback_poll_limit(0) == -1
    prev = lib.splat_set_lookback_poll_limit(1 << 20)
    assert prev == 1 << 20  # the default
    assert lib.splat_set_lookback_poll_limit(prev) == 1 << 20


@pytest.mark.gpu
def test_a_lookback_wait_that_gives_up_is_reported(cuda):
    """One empty poll and the wait gives up: 16k tiles of a 64M-key sort, far more than are resident at once, so
    tiles find predecessors that have not published; the sort completes and the count reports it."""
    lib = L.load()
    L.check_device_waits(cuda)  # start from a clear count
    n = 1 << 26
    g = torch.Generator(device=cuda).manual_seed(5)
    keys = torch.randint(0, 2**31 - 1, (n,), dtype=torch.int32, device=cuda, generator=g)
    vals = torch.arange(n, dtype=torch.int32, device=cuda)
    ko, vo = torch.empty_like(keys), torch.empty_like(vals)
    ws = L.workspace(L.query("splat_sort_workspace_size", n, 4), cuda)
    prev = lib.splat_set_lookback_poll_limit(1)
    try:
        L.call("splat_radix_sort_pairs", L.ptr(keys), L.ptr(vals), L.ptr(ko), L.ptr(vo), n, 4, 0, 32, L.ptr(ws),
               ws.numel(), L.stream_of(keys))
        torch.cuda.synchronize()
        assert lib.splat_check_device_waits() == SPLAT_ERR_TIMEOUT
        assert b"gave up" in lib.splat_last_error()
    finally:
        lib.splat_set_lookback_poll_limit(prev)
    # the tiles whose waits gave up recounted their offsets from the keys: the sort is still exact
    ref_keys, ref_idx = torch.sort(keys.long(), stable=True)
    assert torch.equal(ko.long(), ref_keys) and torch.equal(vo.long(), ref_idx)
    # the default limit again: the same sort reports nothing
    ko.zero_()
    L.call("splat_radix_sort_pairs", L.ptr(keys), L.ptr(vals), L.ptr(ko), L.ptr(vo), n, 4, 0, 32, L.ptr(ws),
           ws.numel(), L.stream_of(keys))
    assert lib.splat_check_device_waits() == 0
    assert torch.equal(ko.long(), ref_keys) and torch.equal(vo.long(), ref_idx)


@pytest.mark.gpu
def test_the_forward_after_a_failed_wait_raises(cuda):
    """The forward reads the count of failed waits with its instance count: after a forward whose sorts gave up,
    the next forward raises instead of returning an image built on a wrong order."""
    lib = L.load()
    sc = scenes.gs3d_config("c3", seed=0)
    params = [sc[k].to(cuda).contiguous() for k in ("means", "scales", "rotations", "opacities", "sh0", "sh_rest")]
    settings = scenes.settings_tuple(sc["cameras"][0], sc["active_sh_bases"], cuda)
    L.check_device_waits(cuda)
    want = gs3d.forward(*params, *settings)[0]
    prev = lib.splat_set_lookback_poll_limit(1)
    try:
        got = gs3d.forward(*params, *settings)[0]
        with pytest.raises(RuntimeError, match="gave up"):
            gs3d.forward(*params, *settings)
    finally:
        lib.splat_set_lookback_poll_limit(prev)
    lib.splat_check_device_waits()  # clear the count the limited forwards left
    assert torch.equal(got, want)  # the sorts stayed exact
    gs3d.forward(*params, *settings)  # the default limit: no failed wait to report


@pytest.mark.gpu
@pytest.mark.parametrize("field,value", [("means", float("nan")), ("means", float("inf")), ("scales", float("nan")),
                                         ("scales", float("inf")), ("rotations", float("nan")),
                                         ("opacities", float("nan")), ("opacities", float("-inf"))])
def test_non_finite_gaussians_are_culled(field, value, cuda):
    """Gaussians with a NaN or infinite mean, scale, rotation or opacity are not visible: the image and the other
    Gaussians' gradients equal those of the scene without them, and their own gradients are zero."""
    names = ("means", "scales", "rotations", "opacities", "sh0", "sh_rest")
    sc = scenes.gs3d_test_scene("tiny", seed=13)
    bad = torch.tensor([3, 77, 400, 901])
    keep = torch.ones(sc["means"].shape[0], dtype=torch.bool)
    keep[bad] = False
    poisoned = {k: sc[k].clone() for k in names}
    poisoned[field][bad] = value
    settings = scenes.settings_tuple(sc["cameras"][0], sc["active_sh_bases"], cuda)

    def run(p):
        leaves = [p[k].to(cuda).contiguous().requires_grad_(True) for k in names]
        img = gs3d.diff_rasterize(*leaves, torch.empty(0), gs3d.RasterizerSettings(*settings))
        dout = torch.randn(img.shape, generator=torch.Generator().manual_seed(2)).to(cuda)
        return img.detach(), torch.autograd.grad(img, leaves, dout)

    img_bad, g_bad = run(poisoned)
    img_ref, g_ref = run({k: sc[k][keep] for k in names})
    assert bool(torch.isfinite(img_bad).all())
    assert torch.equal(img_bad, img_ref)
    for a, b in zip(g_bad, g_ref):
        assert bool(torch.isfinite(a).all())
        assert float(a[bad.to(cuda)].abs().sum()) == 0.0
        d = (a[keep.to(cuda)] - b).double().norm() / b.double().norm().clamp_min(1e-30)
        assert float(d) < 1e-6
