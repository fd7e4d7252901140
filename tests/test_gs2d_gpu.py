"""gs2d on the GPU through the C ABI vs the reference's own outputs and the pinned oracle.

Tolerances are the reference's (toy2d/tests/test_cuda.py:10, G0): fp32 results within 1e-5 norm-based
relative error of the float64 reference, except the 4096-Gaussian C1 fit whose gradients get the
1e-4 atomic-order tolerance. Integer outputs (bins, contributor counts) must be bit-exact; counts are
compared on every pixel whose decisions the float64 oracle does not flag as within 1e-5 of a threshold.
"""
from __future__ import annotations

import numpy as np
import pytest
import torch

from conftest import golden
from gs_b200 import gs2d
from oracle import gs2d_oracle as O

pytestmark = pytest.mark.gpu

SMALL = ["tiny", "sparse_odd", "dense", "opaque"]
ALL = SMALL + ["c1"]
NAMES = ("dmeans", "dconic", "dcolor", "dopacity")


def _inputs(g, dev):
    x = [torch.tensor(g[k], dtype=torch.float32, device=dev).requires_grad_(True)
         for k in ("means", "conic", "color", "opacity")]
    bg = torch.tensor(g["bg"], dtype=torch.float32, device=dev)
    return x, bg


def _bins(g, dev):
    return gs2d.bin_gaussians(torch.tensor(g["means"], dtype=torch.float32, device=dev),
                              torch.tensor(g["radii"], device=dev), torch.tensor(g["depth"], device=dev),
                              int(g["H"]), int(g["W"]))


@pytest.mark.parametrize("scene", ALL)
def test_binning_bit_exact(scene, cuda):
    g = golden(f"gs2d_{scene}")
    b = _bins(g, cuda)
    for key in ("rect", "order", "point_list", "ranges", "bucket_offsets", "bucket_to_tile"):
        assert np.array_equal(getattr(b, key).cpu().numpy(), g[key]), key
    assert b.num_buckets == int(g["num_buckets"])


def test_binning_float32_depth_and_ties(cuda):
    """Tied float32 depths keep index order (stable argsort), like torch.argsort(stable=True)."""
    gen = torch.Generator().manual_seed(5)
    n, H, W = 700, 70, 90
    means = torch.rand(n, 2, generator=gen) * torch.tensor([W, H])
    radii = torch.randint(0, 12, (n,), generator=gen, dtype=torch.int32)
    depth = torch.randint(0, 9, (n,), generator=gen).float()  # many ties
    b = gs2d.bin_gaussians(means.to(cuda), radii.to(cuda), depth.to(cuda), H, W)
    o = O.bin_gaussians(means.numpy(), radii.numpy(), depth.numpy(), H, W)
    for key in ("rect", "order", "point_list", "ranges", "bucket_offsets", "bucket_to_tile"):
        assert np.array_equal(getattr(b, key).cpu().numpy(), getattr(o, key)), key


@pytest.mark.parametrize("scene", ALL)
def test_forward(scene, cuda):
    g = golden(f"gs2d_{scene}")
    x, bg = _inputs(g, cuda)
    b = _bins(g, cuda)
    out, final_T, n_contrib, bstate = gs2d.ext().forward(*[t.detach() for t in x], bg, b.ranges, b.point_list,
                                                         b.bucket_offsets, b.num_buckets, b.H, b.W, True)
    ob = O.bin_gaussians(g["means"].astype(np.float32), g["radii"], g["depth"], int(g["H"]), int(g["W"]))
    ref = O.forward(g["means"], g["conic"], g["color"], g["opacity"], g["bg"], ob)
    safe = ~ref.near
    assert safe.mean() > 0.9
    # images within 1e-5 absolute on every pixel whose decisions are not within float32 rounding of a threshold
    err = np.abs(out.cpu().numpy() - g["image"]).max(axis=0)
    assert err[safe].max() < 1e-5
    assert O.rel_err(out.cpu().numpy(), g["image"]) < (1e-5 if scene != "c1" else 3e-5)
    assert np.array_equal(n_contrib.cpu().numpy()[safe], ref.n_contrib[safe])
    assert np.allclose(final_T.cpu().numpy()[safe], ref.final_T[safe], rtol=1e-4, atol=1e-6)
    assert O.rel_err(bstate.cpu().numpy(), ref.bucket_state) < 1e-5


@pytest.mark.parametrize("scene", ALL)
@pytest.mark.parametrize("backend", ["pixel", "splat"])
def test_backward(scene, backend, cuda):
    g = golden(f"gs2d_{scene}")
    x, bg = _inputs(g, cuda)
    b = _bins(g, cuda)
    out = gs2d.rasterize(*x, b, bg, backend=backend)
    assert O.rel_err(out.detach().cpu().numpy(), g["image"]) < (1e-5 if scene != "c1" else 3e-5)
    grads = torch.autograd.grad(out, x, torch.tensor(g["dout"], dtype=torch.float32, device=cuda))
    tol = 1e-4 if scene == "c1" else 1e-5
    for name, got in zip(NAMES, grads):
        e = O.rel_err(got.cpu().numpy(), g[name])
        assert e < tol, f"{backend}/{scene}/{name}: {e:.2e}"


@pytest.mark.parametrize("scene", ["dense", "c1"])
def test_backward_modes_agree(scene, cuda):
    g = golden(f"gs2d_{scene}")
    b = _bins(g, cuda)
    res = {}
    for backend in ("pixel", "splat"):
        x, bg = _inputs(g, cuda)
        out = gs2d.rasterize(*x, b, bg, backend=backend)
        res[backend] = torch.autograd.grad(out, x, torch.tensor(g["dout"], dtype=torch.float32, device=cuda))
    for name, a, c in zip(NAMES, res["pixel"], res["splat"]):
        assert O.rel_err(c.cpu().numpy(), a.cpu().numpy()) < 1e-5, name


def test_empty_view_gives_zero_gradients(cuda):
    """Every Gaussian off-screen: no instances, no buckets, zero gradients, no launch error."""
    n, H, W = 20, 33, 47
    means = torch.full((n, 2), -500.0, device=cuda)
    radii = torch.full((n,), 3, dtype=torch.int32, device=cuda)
    b = gs2d.bin_gaussians(means, radii, torch.rand(n, device=cuda), H, W)
    assert b.point_list.numel() == 0 and b.num_buckets == 0
    x = [means.clone().requires_grad_(True), torch.tensor([[0.1, 0.0, 0.1]], device=cuda).repeat(n, 1).requires_grad_(True),
         torch.rand(n, 3, device=cuda).requires_grad_(True), torch.rand(n, device=cuda).requires_grad_(True)]
    bg = torch.tensor([0.2, 0.5, 0.8], device=cuda)
    for backend in ("pixel", "splat"):
        out = gs2d.rasterize(*x, b, bg, backend=backend)
        assert torch.allclose(out, bg[:, None, None].expand(3, H, W))
        grads = torch.autograd.grad(out, x, torch.ones_like(out))
        torch.cuda.synchronize()
        assert all(float(t.abs().sum()) == 0.0 for t in grads)


def test_cpu_tensors_are_rejected():
    with pytest.raises(RuntimeError, match="CUDA"):
        gs2d.ext().forward(torch.zeros(1, 2), torch.zeros(1, 3), torch.zeros(1, 3), torch.zeros(1),
                           torch.zeros(3), torch.zeros(1, 2, dtype=torch.int32), torch.zeros(0, dtype=torch.int32),
                           torch.zeros(1, dtype=torch.int32), 0, 16, 16, False)


def _bins_bounded(g, dev, capacity):
    return gs2d.bin_gaussians(torch.tensor(g["means"], dtype=torch.float32, device=dev),
                              torch.tensor(g["radii"], device=dev), torch.tensor(g["depth"], device=dev),
                              int(g["H"]), int(g["W"]), capacity=capacity)


@pytest.mark.parametrize("scene", ALL)
def test_bounded_binning_same_lists(scene, cuda):
    """Bounded binning (no host read) gives the reference's lists: the first M entries of point_list, the same
    ranges and bucket offsets, the reference's buckets followed by -1 up to the bound, and no overflow."""
    g = golden(f"gs2d_{scene}")
    M, B = len(g["point_list"]), int(g["num_buckets"])
    b = _bins_bounded(g, cuda, capacity=M + 37)
    for key in ("rect", "order", "ranges", "bucket_offsets"):
        assert np.array_equal(getattr(b, key).cpu().numpy(), g[key]), key
    assert np.array_equal(b.point_list.cpu().numpy()[:M], g["point_list"])
    btt = b.bucket_to_tile.cpu().numpy()
    assert b.num_buckets == btt.size >= B
    assert np.array_equal(btt[:B], g["bucket_to_tile"]) and (btt[B:] == -1).all()
    b.check()


@pytest.mark.parametrize("scene", ["dense", "c1"])
def test_bounded_binning_same_render_and_gradients(scene, cuda):
    """The image and the gradients of a bounded binning equal the exact binning's (same lists; the extra buckets
    name no tile); the splat backward's atomics allow 1e-6."""
    g = golden(f"gs2d_{scene}")
    res = []
    for b in (_bins(g, cuda), _bins_bounded(g, cuda, capacity=2 * len(g["point_list"]))):
        x, bg = _inputs(g, cuda)
        out = gs2d.rasterize(*x, b, bg, backend="splat")
        grads = torch.autograd.grad(out, x, torch.tensor(g["dout"], dtype=torch.float32, device=cuda))
        res.append((out.detach(), grads))
    assert torch.equal(res[0][0], res[1][0])
    for name, a, c in zip(NAMES, res[0][1], res[1][1]):
        assert O.rel_err(c.cpu().numpy(), a.cpu().numpy()) < 1e-6, name


def test_bounded_binning_overflow_is_flagged(cuda):
    """More instances than the capacity: the lists are left empty (background image, zero gradients), nothing is
    written past the buffers, and Bins.check() raises."""
    g = golden("gs2d_dense")
    b = _bins_bounded(g, cuda, capacity=len(g["point_list"]) // 2)
    assert b.ranges.cpu().numpy().tolist() == [[0, 0]] * b.ranges.shape[0]
    x, bg = _inputs(g, cuda)
    out = gs2d.rasterize(*x, b, bg, backend="splat")
    assert torch.allclose(out, bg[:, None, None].expand_as(out))
    with pytest.raises(RuntimeError, match="capacity"):
        b.check()
