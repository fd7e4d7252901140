"""3DGS on the GPU through the C ABI.

  * integer outputs (listed tiles per Gaussian, 64-bit keys, their sort, tile ranges, buckets) bit-exact
    against the float32 numpy oracle fed the device's own preprocess outputs
  * preprocess floats against the float64 PyTorch reference (1e-5 relative)
  * image within 1e-5 absolute of the float64 reference on the pixels whose decisions are not within
    float32 rounding of a threshold (at most 0.1% of pixels may sit there), gradients within 1e-4
    norm-based relative error (the atomic-order tolerance of the benchmark spec)
  * empty view: no instances, zero gradients, no launch error; inputs rejected off the GPU
Scenes follow the reference's GPU test generator (phase1/tests/test_parity.py:43-84).
"""
from __future__ import annotations

import numpy as np
import pytest
import torch

from gs_b200 import gs3d, scenes
from oracle import gs3d_oracle as O
from oracle import gs3d_torch as R

pytestmark = pytest.mark.gpu

GRAD_NAMES = ("means", "scales", "rotations", "opacities", "sh0", "sh_rest")


def rel(a, b) -> float:
    a, b = a.double().flatten().cpu(), b.double().flatten().cpu()
    nb = float(b.norm())
    return float((a - b).norm()) / nb if nb > 0 else float((a - b).norm())


def _setup(name, seed=0, aa=False, dev="cuda"):
    sc = scenes.gs3d_test_scene(name, seed, proper_antialiasing=aa)
    cam = sc["cameras"][0]
    params = [sc[k].to(dev).contiguous() for k in ("means", "scales", "rotations", "opacities", "sh0", "sh_rest")]
    settings = scenes.settings_tuple(cam, sc["active_sh_bases"], dev)
    return sc, cam, params, settings


@pytest.mark.parametrize("name", ["micro", "tiny", "partial_tiles", "garden_res", "heavy_overlap", "small_splats"])
def test_binning_bit_exact(name, cuda):
    sc, cam, params, settings = _setup(name)
    W, H = cam["width"], cam["height"]
    image, prim, tile, inst, bucket, m, nb, _ = gs3d.forward(*params, *settings)
    torch.cuda.synchronize()
    n = params[0].shape[0]
    pv = gs3d.primitive_views(prim, n)
    vis = (pv["n_touched"] > 0).cpu().numpy()
    ref = O.bin_instances(pv["mean2d"].cpu().numpy(), pv["conic_o"].cpu().numpy(), pv["thr"].cpu().numpy(),
                          pv["color_z"][:, 3].cpu().numpy(), vis, W, H)
    n_touched, keys, ids, keys_sorted, point_list, ranges, buckets = ref
    assert np.array_equal(pv["n_touched"].cpu().numpy(), n_touched)
    assert m == keys.size
    iv = gs3d.instance_views(inst, m, prim, n)
    assert np.array_equal(iv["keys_sorted"].cpu().numpy().view(np.uint64), keys_sorted)
    assert np.array_equal(iv["point_list"].cpu().numpy(), point_list)
    # the depth passes: Gaussians ordered by (depth, id), the ones not visible last
    order = pv["order"].cpu().numpy()
    zk = O.depth_order_key(pv["color_z"][:, 3].cpu().numpy())
    zk = np.where(vis, zk.astype(np.uint64), np.uint64(0xFFFFFFFF))
    assert np.array_equal(order, np.argsort(zk, kind="stable"))
    tv = gs3d.tile_views(tile, W, H)
    assert np.array_equal(tv["ranges"].cpu().numpy(), ranges)
    assert np.array_equal(tv["nb"].cpu().numpy()[:-1], buckets)
    # the bucket bound of phase2/tests/test_readback_equiv.py:100 (16x16 tiles here)
    T = ranges.shape[0]
    assert int(buckets.sum()) <= (m + 31 * T) // 32 + 1 <= nb


@pytest.mark.parametrize("name", ["micro", "tiny"])
@pytest.mark.parametrize("aa", [False, True])
def test_forward_and_gradients_vs_float64_reference(name, aa, cuda):
    sc, cam, params, settings = _setup(name, seed=1, aa=aa)
    leaves = [p.clone().requires_grad_(True) for p in params]
    img = gs3d.diff_rasterize(*leaves, torch.empty(0), gs3d.RasterizerSettings(*settings))
    g = torch.Generator().manual_seed(7)
    dout = torch.randn(img.shape, generator=g).to(cuda)
    grads = torch.autograd.grad(img, leaves, dout)
    # reference on the GPU's own tile lists
    _, prim, tile, inst, _, m, _, _ = gs3d.forward(*params, *settings)
    tv = gs3d.tile_views(tile, cam["width"], cam["height"])
    lists = R.tile_lists_from(tv["ranges"], gs3d.instance_views(inst, m)["point_list"])
    ref_leaves = [p.detach().cpu().double().requires_grad_(True) for p in params]
    cpu_settings = tuple(s.cpu().double() if torch.is_tensor(s) else s for s in settings)
    ref = R.render(*ref_leaves, cpu_settings, lists)
    err = (img.detach().cpu().double() - ref.detach()).abs().amax(0)
    assert float((err > 1e-5).double().mean()) <= 1e-3, f"{int((err > 1e-5).sum())} pixels off, max {float(err.max()):.2e}"
    assert rel(img.detach(), ref.detach()) < 1e-5
    ref_grads = torch.autograd.grad(ref, ref_leaves, dout.cpu().double())
    for nm, a, b in zip(GRAD_NAMES, grads, ref_grads):
        e = rel(a, b)
        assert e < 1e-4, f"{name} aa={aa} {nm}: {e:.3e}"


def test_preprocess_matches_float64_reference(cuda):
    sc, cam, params, settings = _setup("partial_tiles", seed=3)
    n = params[0].shape[0]
    _, prim, *_ = gs3d.forward(*params, *settings)
    pv = gs3d.primitive_views(prim, n)
    vis = pv["n_touched"] > 0
    d = [p.cpu().double() for p in params]
    s = tuple(x.cpu().double() if torch.is_tensor(x) else x for x in settings)
    mean2d, conic, o, color, z, _ = R.preprocess(*d, s[0], s[1], s[3], s[4], s[5], s[6], s[7], s[8], s[9], s[12])
    v = vis.cpu()
    assert int(v.sum()) > 0.5 * n
    assert rel(pv["mean2d"].cpu()[v], mean2d[v]) < 1e-6
    assert rel(pv["conic_o"][:, :3].cpu()[v], conic[v]) < 1e-5
    assert rel(pv["conic_o"][:, 3].cpu()[v], o[v]) < 1e-6
    assert rel(pv["color_z"][:, :3].cpu()[v], color[v]) < 1e-5
    assert rel(pv["color_z"][:, 3].cpu()[v], z[v]) < 1e-6


def test_deterministic_up_to_atomics(cuda):
    """Two backward runs agree to the atomic-order noise (phase1/tests/test_parity.py:131-140)."""
    sc, cam, params, settings = _setup("partial_tiles", seed=2)
    outs = []
    for _ in range(2):
        leaves = [p.clone().requires_grad_(True) for p in params]
        img = gs3d.diff_rasterize(*leaves, torch.empty(0), gs3d.RasterizerSettings(*settings))
        outs.append((img.detach(), torch.autograd.grad(img, leaves, torch.ones_like(img))))
    assert torch.equal(outs[0][0], outs[1][0])
    assert max(rel(a, b) for a, b in zip(outs[0][1], outs[1][1])) < 1e-6


def test_single_call_backward_matches_split(cuda):
    """gs3d_backward (one C call) gives the results of gs3d_backward_blend + gs3d_backward_preprocess, which the
    Python mirror uses, up to the atomic-order noise."""
    import ctypes

    from gs_b200 import _lib as L

    sc, cam, params, settings = _setup("partial_tiles", seed=5)
    image, prim, tile, inst, bucket, m, nb, sel = gs3d.forward(*params, *settings)
    dout = torch.randn_like(image)
    n = params[0].shape[0]
    d_split = torch.zeros(3, n, device=cuda)
    split = gs3d.backward(d_split, dout, image, params[0], params[1], params[2], params[3], params[5], prim, tile, inst,
                          bucket, *settings, m, nb, sel)
    rest = params[5].shape[1]
    keep: list = []
    s = gs3d._settings(params[0].device, *settings, rest, keep)
    ws = torch.empty(L.query("gs3d_backward_workspace_size", n), dtype=torch.uint8, device=cuda)
    single = tuple(torch.empty_like(g) for g in split)
    d_single = torch.zeros(3, n, device=cuda)
    L.call("gs3d_backward", L.ptr(dout), L.ptr(image), *map(L.ptr, params[:4]), L.ptr(params[5]), n, m,
           ctypes.byref(s), L.ptr(prim), prim.numel(), L.ptr(tile), tile.numel(), L.ptr(inst), inst.numel(),
           L.ptr(bucket), bucket.numel(), nb, L.ptr(ws), ws.numel(), *map(L.ptr, single), L.ptr(d_single), 3,
           L.stream_of(image))
    assert max(rel(a, b) for a, b in zip(single, split)) < 1e-5  # float atomics: summation order differs
    assert rel(d_single, d_split) < 1e-5


@pytest.mark.parametrize("rows", [2, 3])
def test_densification_rows_vs_float64_reference(rows, cuda):
    """densification_info accumulated in place over two backward calls: row 0 counts the views a Gaussian was
    visible in, row 1 sums |dL/dmean2d| scaled by (W/2, H/2), row 2 the same norm of the summed per-pixel absolute
    mean2d gradients (per-pixel copies of mean2d in the reference give those)."""
    sc, cam, params, settings = _setup("tiny", seed=8)
    W, H = cam["width"], cam["height"]
    n = params[0].shape[0]
    image, prim, tile, inst, bucket, m, nb, sel = gs3d.forward(*params, *settings)
    g = torch.Generator().manual_seed(9)
    dout = torch.randn(image.shape, generator=g).to(cuda)
    dinfo = torch.zeros(rows, n, device=cuda)
    for _ in range(2):
        gs3d.backward(dinfo, dout, image, params[0], params[1], params[2], params[3], params[5], prim, tile, inst,
                      bucket, *settings, m, nb, sel)
    vis = gs3d.primitive_views(prim, n)["n_touched"].cpu() > 0
    tv = gs3d.tile_views(tile, W, H)
    lists = R.tile_lists_from(tv["ranges"], gs3d.instance_views(inst, m)["point_list"])
    ref_leaves = [p.detach().cpu().double() for p in params]
    cpu_settings = tuple(s.cpu().double() if torch.is_tensor(s) else s for s in settings)
    taps: list = []
    ref = R.render(*ref_leaves, cpu_settings, lists, mean2d_taps=taps)
    ref.backward(dout.cpu().double())
    scale = torch.tensor([0.5 * W, 0.5 * H], dtype=torch.float64)
    gm = taps[0].grad  # dL/dmean2d [N, 2]
    want1 = 2 * (gm * scale).norm(dim=1)
    got = dinfo.cpu().double()
    assert torch.equal(got[0], 2 * vis.double())
    assert rel(got[1], want1) < 1e-4
    if rows == 3:
        absg = torch.zeros(n, 2, dtype=torch.float64)
        for gid, tx, ty in taps[1:]:
            absg[gid, 0] += tx.grad.abs().sum()
            absg[gid, 1] += ty.grad.abs().sum()
        assert rel(got[2], 2 * (absg * scale).norm(dim=1)) < 1e-4


@pytest.mark.parametrize("name", ["micro", "tiny", "garden_res", "heavy_overlap", "empty"])
def test_render_only_path_matches_training_forward(name, cuda):
    """gs3d.inference (Faster-GS `_C.inference`) gives the training forward's image bit for bit."""
    sc, cam, params, settings = _setup(name, seed=11)
    img = gs3d.forward(*params, *settings)[0]
    inf = gs3d.inference(*params, *settings)
    assert torch.equal(img, inf)


def test_render_only_c5_scale(cuda):
    """Config C5 (6M Gaussians, 3840x2160): the render-only image equals the training forward's, one frame."""
    sc = scenes.gs3d_config("c5", seed=0)
    params = [sc[k].to(cuda).contiguous() for k in ("means", "scales", "rotations", "opacities", "sh0", "sh_rest")]
    cam = sc["cameras"][0]
    settings = scenes.settings_tuple(cam, sc["active_sh_bases"], cuda)
    inf = gs3d.inference(*params, *settings)
    img = gs3d.forward(*params, *settings)[0]
    assert torch.equal(img, inf)
    assert bool(torch.isfinite(inf).all()) and float(inf.std()) > 0


def test_empty_scene(cuda):
    """All Gaussians behind the camera: no instances, zero gradients, no launch error (test_parity.py:143-153)."""
    sc, cam, params, settings = _setup("empty", seed=3)
    image, prim, tile, inst, bucket, m, nb, sel = gs3d.forward(*params, *settings)
    assert m == 0
    leaves = [p.clone().requires_grad_(True) for p in params]
    img = gs3d.diff_rasterize(*leaves, torch.empty(0), gs3d.RasterizerSettings(*settings))
    grads = torch.autograd.grad(img, leaves, torch.ones_like(img))
    torch.cuda.synchronize()
    assert all(float(gr.abs().sum()) == 0.0 for gr in grads)
    bg = settings[2].view(3, 1, 1).expand_as(img)
    assert torch.allclose(img, bg)


def test_back_to_back_calls_without_sync(cuda):
    """30 forward/backward calls on changing inputs keep agreeing with single calls
    (phase2/tests/test_readback_equiv.py:118-130)."""
    outs = []
    for k in range(30):
        sc, cam, params, settings = _setup("tiny", seed=100 + k)
        leaves = [p.clone().requires_grad_(True) for p in params]
        img = gs3d.diff_rasterize(*leaves, torch.empty(0), gs3d.RasterizerSettings(*settings))
        outs.append(img.detach())
    torch.cuda.synchronize()
    for k in (0, 13, 29):
        sc, cam, params, settings = _setup("tiny", seed=100 + k)
        img = gs3d.forward(*params, *settings)[0]
        assert torch.equal(img, outs[k])


def _graphdeco_proj(view: torch.Tensor, tanfovx: float, tanfovy: float, znear=0.01, zfar=100.0) -> torch.Tensor:
    """graphdeco's full projection: viewmatrix @ P^T with its pinhole P (getProjectionMatrix, centred)."""
    P = torch.zeros(4, 4, dtype=view.dtype, device=view.device)
    P[0, 0], P[1, 1] = 1.0 / tanfovx, 1.0 / tanfovy
    P[3, 2] = 1.0
    P[2, 2], P[2, 3] = zfar / (zfar - znear), -(zfar * znear) / (zfar - znear)
    return view @ P.T


def test_rasterize_gaussians_graphdeco_entry(cuda):
    sc, cam, params, settings = _setup("tiny", seed=4)
    means, scales, rot, op, sh0, shr = params
    shs = torch.cat([sh0, shr], 1)
    view = settings[0].T.contiguous()
    W, H = cam["width"], cam["height"]
    tx, ty = W / (2 * cam["focal_x"]), H / (2 * cam["focal_y"])
    img, radii = gs3d.rasterize_gaussians(means, torch.exp(scales), rot, torch.sigmoid(op), shs, view,
                                          _graphdeco_proj(view, tx, ty), settings[2], tx, ty, H, W, 3, settings[1])
    # same camera with a centred principal point through the Faster-GS entry
    s2 = list(settings)
    s2[8], s2[9] = W / 2.0, H / 2.0
    ref, prim = gs3d.forward(*params, *s2)[:2]
    # log(exp(s)) and logit(sigmoid(o)) round differently, so a pixel may flip a threshold decision
    err = (img.detach() - ref).abs().amax(0)
    assert float((err > 1e-4).double().mean()) < 1e-3 and float(err.mean()) < 1e-5
    # graphdeco's radius: ceil(3 sqrt(lambda_max)) of the dilated 2D covariance, 0 where not listed
    n = means.shape[0]
    pv = gs3d.primitive_views(prim, n)
    vis = pv["n_touched"] > 0
    co = pv["conic_o"][vis].double()  # the other Gaussians' entries are not written by the forward
    cov = torch.linalg.inv(torch.stack([torch.stack([co[:, 0], co[:, 1]], -1), torch.stack([co[:, 1], co[:, 2]], -1)],
                                       -2))
    # graphdeco's larger eigenvalue: mid + sqrt(max(mid^2 - det, 0.1)) of the 2D covariance
    a, b, c = cov[:, 0, 0], cov[:, 0, 1], cov[:, 1, 1]
    mid = 0.5 * (a + c)
    lam = mid + torch.sqrt(torch.clamp(mid * mid - (a * c - b * b), min=0.1))
    want = torch.zeros_like(radii)
    want[vis] = torch.ceil(3 * torch.sqrt(lam)).int()
    assert radii.shape == (n,) and radii.dtype == torch.int32 and int((radii > 0).sum()) > 0
    # rasterize_gaussians renders log(exp(s)) and logit(sigmoid(o)): a ceil may flip, by one pixel at most
    assert int((radii - want).abs().max()) <= 1 and float((radii != want).double().mean()) < 1e-2
    # a projection that is not the centred pinhole of viewmatrix is refused
    bad = _graphdeco_proj(view, tx, ty).clone()
    bad[0, 0] *= 1.1
    with pytest.raises(ValueError, match="projmatrix"):
        gs3d.rasterize_gaussians(means, torch.exp(scales), rot, torch.sigmoid(op), shs, view, bad, settings[2], tx,
                                 ty, H, W, 3, settings[1])


def test_inputs_must_be_cuda():
    sc = scenes.gs3d_test_scene("micro")
    cam = sc["cameras"][0]
    params = [sc[k] for k in ("means", "scales", "rotations", "opacities", "sh0", "sh_rest")]
    with pytest.raises(RuntimeError, match="CUDA"):
        gs3d.forward(*params, *scenes.settings_tuple(cam, 16, "cpu"))


def test_backward_accumulates_the_views_of_a_batch(cuda):
    """backward(..., out=grads, accumulate=True) adds a view's gradients into ``out``
    (gs3d_backward_preprocess_accumulate): two views summed in one buffer equal the two views' separate gradients
    added, up to the atomic-order noise of the blend backward."""
    sc = scenes.gs3d_config("c2", seed=3)
    params = [sc[k].to(cuda).contiguous() for k in GRAD_NAMES]
    cams = [sc["cameras"][0], scenes.camera(1297, 840, (3.0, -1.0, -7.0))]
    n = params[0].shape[0]
    outs, douts, fwd = [], [], []
    for k, cam in enumerate(cams):
        s = scenes.settings_tuple(cam, sc["active_sh_bases"], cuda)
        f = gs3d.forward(*params, *s)
        d = torch.randn(f[0].shape, generator=torch.Generator().manual_seed(40 + k)).to(cuda)
        fwd.append((s, f))
        douts.append(d)
        outs.append(gs3d.backward(None, d, f[0], params[0], params[1], params[2], params[3], params[5], *f[1:5], *s,
                                  *f[5:]))
    acc = tuple(torch.full_like(g, float("nan")) for g in outs[0])
    for k, ((s, f), d) in enumerate(zip(fwd, douts)):
        gs3d.backward(None, d, f[0], params[0], params[1], params[2], params[3], params[5], *f[1:5], *s, *f[5:],
                      out=acc, accumulate=k > 0)
    for name, a, g0, g1 in zip(GRAD_NAMES, acc, outs[0], outs[1]):
        assert bool(torch.isfinite(a).all()), name
        assert rel(a, g0 + g1) < 1e-5, f"{name}: {rel(a, g0 + g1):.2e}"
    assert n > 0


@pytest.mark.parametrize("name", ["micro", "tiny", "garden_res", "heavy_overlap", "empty"])
def test_bounded_forward_matches_exact_forward(name, cuda):
    """The bounded forward (no host read of M; buffers for a capacity) gives the exact forward's image, sorted list,
    tile ranges, contributor counts and final T bit for bit, and the backward from either gives the same gradients
    (the blend backward's atomic order allows 1e-5); the overflow word stays 0."""
    sc, cam, params, settings = _setup(name, seed=5)
    W, H = cam["width"], cam["height"]
    ex = gs3d.forward(*params, *settings)
    m = ex[5]
    overflow = torch.zeros(1, dtype=torch.int32, device=cuda)
    bd = gs3d.forward(*params, *settings, capacity=m + 1000, overflow=overflow)
    assert bd[5] == m + 1000
    assert torch.equal(ex[0], bd[0])
    if m:  # the bounded buffer's slots past M are never written: compare the first M (and gather nothing by them)
        ie, ib = gs3d.instance_views(ex[3], m), gs3d.instance_views(bd[3], m + 1000)
        for key in ("tiles_sorted", "point_list"):
            assert torch.equal(ie[key], ib[key][:m]), key
    te, tb = gs3d.tile_views(ex[2], W, H), gs3d.tile_views(bd[2], W, H)
    for key in ("ranges", "n_contrib", "final_T", "max_contrib"):
        assert torch.equal(te[key], tb[key]), key
    dout = torch.randn(3, H, W, device=cuda, generator=torch.Generator(device=cuda).manual_seed(2)) * 1e-2
    grads = []
    for r in (ex, bd):
        image, prim, tile, inst, bucket, mm, nb, sel = r
        grads.append(gs3d.backward(None, dout, image, params[0], params[1], params[2], params[3], params[5], prim,
                                   tile, inst, bucket, *settings, mm, nb, sel))
    for a, b in zip(*grads):  # atomic-order noise (heavy overlap stacks many atomics on each Gaussian)
        assert rel(b, a) < 1e-5
    assert int(overflow.item()) == 0


def test_bounded_forward_overflow_is_flagged(cuda):
    """A capacity below M: the overflow word is set, nothing is written past the buffers, and the call returns."""
    sc, cam, params, settings = _setup("garden_res", seed=5)
    m = gs3d.forward(*params, *settings)[5]
    assert m > 1000
    overflow = torch.zeros(1, dtype=torch.int32, device=cuda)
    out = gs3d.forward(*params, *settings, capacity=m // 2, overflow=overflow)
    torch.cuda.synchronize()
    assert int(overflow.item()) == 1
    assert bool(torch.isfinite(out[0]).all())
