"""CPU checks of the 3DGS oracles themselves (no GPU).

The listing rule (closed-form x-extent of the alpha >= 1/255 ellipse per tile row) against brute force in
float64: every tile holding a pixel centre inside the ellipse is listed (complete), and every listed tile's
continuous pixel-centre rectangle meets the ellipse up to float32 rounding (tight). The float64 PyTorch
reference is checked against finite differences on a tiny scene.
"""
from __future__ import annotations

import numpy as np
import torch

from gs_b200 import scenes
from oracle import gs3d_oracle as O
from oracle import gs3d_torch as R


def _random_ellipses(n, W, H, seed):
    rng = np.random.default_rng(seed)
    mx = rng.uniform(-20, W + 20, n).astype(np.float32)
    my = rng.uniform(-20, H + 20, n).astype(np.float32)
    sx = rng.uniform(0.5, 40, n)
    sy = rng.uniform(0.5, 40, n)
    th = rng.uniform(0, np.pi, n)
    c, s = np.cos(th), np.sin(th)
    cxx = c * c * sx ** 2 + s * s * sy ** 2
    cxy = c * s * (sx ** 2 - sy ** 2)
    cyy = s * s * sx ** 2 + c * c * sy ** 2
    det = cxx * cyy - cxy * cxy
    A, B, C = (cyy / det).astype(np.float32), (-cxy / det).astype(np.float32), (cxx / det).astype(np.float32)
    thr = np.log(255 * rng.uniform(0.01, 1.0, n)).astype(np.float32)
    return mx, my, A, B, C, thr


def test_listing_is_complete_and_tight():
    W, H = 150, 100
    tiles_x, tiles_y = (W + 15) // 16, (H + 15) // 16
    mx, my, A, B, C, thr = _random_ellipses(400, W, H, 0)
    g, tx, ty = O.listed_tiles(mx, my, A, B, C, thr, W, H)
    listed = set(zip(g.tolist(), tx.tolist(), ty.tolist()))
    assert len(listed) == g.size  # no tile twice
    ys, xs = np.mgrid[0:H, 0:W]
    cx, cy = xs + 0.5, ys + 0.5
    for i in range(mx.size):
        dx, dy = cx - float(mx[i]), cy - float(my[i])
        q = float(A[i]) * dx * dx + 2 * float(B[i]) * dx * dy + float(C[i]) * dy * dy
        inside = q <= 2 * float(thr[i]) * (1 - 1e-5)
        need = set(zip((xs[inside] // 16).tolist(), (ys[inside] // 16).tolist()))
        have = {(a, b) for gi, a, b in listed if gi == i}
        assert need <= have, f"ellipse {i}: tiles {sorted(need - have)} missing"
        for a, b in have:  # tight: the tile rectangle reaches the ellipse (float64, small slack)
            x0, x1 = a * 16 + 0.5, min(a * 16 + 16, W) - 0.5
            y0, y1 = b * 16 + 0.5, min(b * 16 + 16, H) - 0.5
            gx, gy = np.meshgrid(np.linspace(x0, x1, 64), np.linspace(y0, y1, 64))
            ddx, ddy = gx - float(mx[i]), gy - float(my[i])
            qq = float(A[i]) * ddx * ddx + 2 * float(B[i]) * ddx * ddy + float(C[i]) * ddy * ddy
            assert qq.min() <= 2 * float(thr[i]) * 1.02 + 0.05, f"ellipse {i}: tile {(a, b)} is not reached"


def test_bin_instances_orders_by_tile_then_depth_then_id():
    W, H = 96, 64
    n = 200
    mx, my, A, B, C, thr = _random_ellipses(n, W, H, 1)
    rng = np.random.default_rng(2)
    depth = rng.integers(1, 6, n).astype(np.float32)  # ties on purpose
    res = O.bin_instances(np.stack([mx, my], 1), np.stack([A, B, C, np.ones(n, np.float32)], 1), thr, depth,
                          np.ones(n, bool), W, H)
    n_touched, keys, ids, keys_sorted, point_list, ranges, buckets = res
    tile = (keys_sorted >> np.uint64(32)).astype(np.int64)
    assert np.all(np.diff(tile) >= 0)
    for t in range(ranges.shape[0]):
        s, e = ranges[t]
        seg = point_list[s:e]
        zs = depth[seg]
        assert np.all((np.diff(zs) > 0) | ((np.diff(zs) == 0) & (np.diff(seg) > 0)))
    assert int(n_touched.sum()) == keys.size == int((ranges[:, 1] - ranges[:, 0]).sum())


def test_torch_reference_gradcheck():
    """The float64 reference is differentiable where it should be (finite differences on a tiny scene)."""
    sc = scenes.gs3d_test_scene("micro", seed=5)
    cam = sc["cameras"][0]
    keep = torch.arange(0, 200, 10)
    p = [sc[k][keep].double() for k in ("means", "scales", "rotations", "opacities", "sh0", "sh_rest")]
    s = tuple(x.double() if torch.is_tensor(x) else x for x in scenes.settings_tuple(cam, 16, "cpu"))
    T = ((cam["width"] + 15) // 16) * ((cam["height"] + 15) // 16)
    lists = [torch.arange(keep.numel()) for _ in range(T)]  # every Gaussian listed everywhere, in index order
    leaves = [t.clone().requires_grad_(True) for t in p]

    def f(*x):
        return R.render(*x, s, lists)[:, ::7, ::7]

    assert torch.autograd.gradcheck(f, tuple(leaves[:4]) + (leaves[4].detach(), leaves[5].detach()), eps=1e-6,
                                    atol=1e-5, rtol=1e-3, nondet_tol=0.0, check_undefined_grad=False)
