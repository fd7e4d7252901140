"""3DGS parity at the benchmark's own configurations, through the C ABI, against the C++ restatement
(oracle/liboracle.so) on the same seeded inputs:

    C2  100k Gaussians, one 1297x840 view: everything on the whole view
    C3  3M Gaussians in 64 clusters, 1920x1080: preprocess, sort and tile tables on the whole view; image,
        counts and gradients on three bands of tile rows (top, middle, bottom)
    C4  1M Gaussians, all eight 1280x720 ring views: everything on every whole view
    C5  6M Gaussians in 256 clusters, 3840x2160, render-only: preprocess, sort and tile tables on the whole
        frame; the render-only image (gs3d.inference) and the training forward's counts on three bands

Criteria (the benchmark spec's, phase1/tests/test_parity.py:114-128 and phase2/tests/test_readback_equiv.py:90-130
for the pattern):
  * listed-tile counts agree with the oracle's own preprocess on all but 1e-4 of the Gaussians, and the
    preprocess floats within 1e-5 (norm-relative) on the Gaussians both list
  * on the device's own primitives: the sorted 64-bit (tile | depth) keys, the point list, the tile ranges and
    the bucket tables bit-exact
  * per-pixel contributor counts bit-exact and image / final T within 1e-5 absolute, on the pixels none of whose
    alpha >= 1/255 or T < 1e-4 decisions lies within the rounding bound of two exp2 implementations (the oracle
    flags those; at most 0.2% of the compared pixels may be flagged)
  * the six parameter gradients within 1e-4 norm-relative (upstream gradient N(0, 1e-3), zero outside the
    compared bands)
"""
from __future__ import annotations

import numpy as np
import pytest
import torch

from gs_b200 import gs3d, scenes
from oracle import gs3d_cpu

pytestmark = pytest.mark.gpu

NAMES = ("means", "scales", "rotations", "opacities", "sh0", "sh_rest")


def _rel(a: np.ndarray, b: np.ndarray) -> float:
    a, b = np.asarray(a, np.float64).ravel(), np.asarray(b, np.float64).ravel()
    nb = float(np.linalg.norm(b))
    return float(np.linalg.norm(a - b)) / (nb if nb > 0 else 1.0)


def _np_cam(cam: dict) -> dict:
    return {k: (v.numpy() if torch.is_tensor(v) else v) for k, v in cam.items()}


def _bands(tiles_y: int, rows: int | None) -> list[tuple[int, int]]:
    if rows is None:
        return [(0, tiles_y)]
    mid = tiles_y // 2 - rows // 2
    return [(0, rows), (mid, mid + rows), (tiles_y - rows, tiles_y)]


def check_view(sc: dict, cam: dict, band_rows: int | None, grads: bool, render_only: bool = False,
               seed: int = 0) -> dict:
    """Runs one view on the device and on the oracle and asserts the criteria above. Returns the figures."""
    dev = torch.device("cuda:0")
    params = [sc[k].to(dev).contiguous() for k in NAMES]
    settings = scenes.settings_tuple(cam, sc["active_sh_bases"], dev)
    n, W, H = params[0].shape[0], cam["width"], cam["height"]
    tiles_y = (H + 15) // 16
    bands = _bands(tiles_y, band_rows)

    image, prim, tile, inst, bucket, m, nb, sel = gs3d.forward(*params, *settings)
    pv = {k: v.cpu().numpy() for k, v in gs3d.primitive_views(prim, n).items()}
    iv = gs3d.instance_views(inst, m, prim, n)
    tv = {k: v.cpu().numpy() for k, v in gs3d.tile_views(tile, W, H).items()}
    keys_dev = iv["keys_sorted"].cpu().numpy().view(np.uint64)
    plist_dev = iv["point_list"].cpu().numpy()
    if render_only:
        image = gs3d.inference(*params, *settings)
    img_dev = image.cpu().numpy()

    o = gs3d_cpu.Oracle([sc[k].numpy() for k in NAMES], _np_cam(cam), sc["active_sh_bases"])
    # preprocess against the oracle's own float path
    o.preprocess()
    op = o.primitives()
    vis_o, vis_d = op["n_touched"] > 0, pv["n_touched"] > 0
    listed_diff = float(np.mean(op["n_touched"] != pv["n_touched"].astype(np.int32)))
    assert listed_diff <= 1e-4, f"listed-tile counts differ on {listed_diff:.2e} of the Gaussians"
    both = vis_o & vis_d
    assert both.sum() > 0.05 * n or n < 1000
    for key, cols in (("mean2d", slice(None)), ("conic_o", slice(0, 3)), ("conic_o", slice(3, 4)),
                      ("color_z", slice(0, 3)), ("color_z", slice(3, 4))):
        e = _rel(pv[key][both][:, cols], op[key][both][:, cols])
        assert e < 1e-5, f"preprocess {key}[{cols}] rel err {e:.2e}"

    # binning, tile tables and blend on the device's own primitives
    o.set_primitives(pv["mean2d"], pv["conic_o"], pv["color_z"], pv["thr"], pv["n_touched"].astype(np.int32))
    assert o.bin() == m
    ob = o.binning()
    assert np.array_equal(keys_dev, ob["keys_sorted"]), "sorted 64-bit keys differ"
    assert np.array_equal(plist_dev.astype(np.int64), ob["point_list"]), "point lists differ"
    assert np.array_equal(tv["ranges"].astype(np.int64), ob["ranges"]), "tile ranges differ"
    counts = ob["ranges"][:, 1] - ob["ranges"][:, 0]
    per_tile = (counts + 31) // 32
    assert np.array_equal(tv["nb"][:-1].astype(np.int64), per_tile), "buckets per tile differ"
    assert np.array_equal(tv["bstart"][:-1].astype(np.int64), np.cumsum(per_tile) - per_tile), "bucket starts differ"
    assert int(per_tile.sum()) <= nb

    for r0, r1 in bands:
        o.blend(r0, r1)
    fr = o.frame()
    rows = np.zeros(H, bool)
    for r0, r1 in bands:
        rows[r0 * 16:min(r1 * 16, H)] = True
    cmp = np.broadcast_to(rows[:, None], (H, W)) & ~fr["near"]
    near_frac = float(fr["near"][rows].mean())
    assert near_frac <= 2e-3, f"{near_frac:.2%} of the compared pixels sit at a threshold"
    nc_dev = tv["n_contrib"]
    assert np.array_equal(nc_dev[cmp], fr["n_contrib"][cmp].astype(nc_dev.dtype)), (
        f"{int((nc_dev[cmp] != fr['n_contrib'][cmp]).sum())} contributor counts differ")
    img_err = float(np.abs(img_dev[:, cmp] - fr["image"][:, cmp]).max())
    assert img_err <= 1e-5, f"image max abs err {img_err:.2e}"
    t_err = float(np.abs(tv["final_T"][cmp] - fr["final_T"][cmp]).max())
    assert t_err <= 1e-5, f"final T max abs err {t_err:.2e}"
    out = {"m": m, "near_frac": near_frac, "img_err": img_err, "listed_diff": listed_diff}

    if grads:
        rng = np.random.default_rng(seed + 17)
        dout = (1e-3 * rng.standard_normal((3, H, W))).astype(np.float32)
        dout[:, ~rows] = 0.0
        g_dev = gs3d.backward(None, torch.from_numpy(dout).to(dev), image, params[0], params[1], params[2],
                              params[3], params[5], prim, tile, inst, bucket, *settings, m, nb, sel)
        g_dev = [g.cpu().numpy() for g in g_dev]
        g_ref = o.backward(dout, bands=bands)
        for name, a, b in zip(NAMES, g_dev, g_ref):
            e = _rel(a, b)
            assert e < 1e-4, f"gradient of {name}: rel err {e:.2e}"
            out[f"grad_{name}"] = e
    return out


def test_c2_single_view(cuda):
    sc = scenes.gs3d_config("c2", seed=0)
    check_view(sc, sc["cameras"][0], band_rows=None, grads=True)


def test_c3_scene_view_bands(cuda):
    sc = scenes.gs3d_config("c3", seed=0)
    check_view(sc, sc["cameras"][0], band_rows=3, grads=True)


@pytest.mark.parametrize("view", range(8))
def test_c4_training_views(view, cuda, c4_scene):
    check_view(c4_scene, c4_scene["cameras"][view], band_rows=None, grads=True, seed=view)


def test_c5_render_only_bands(cuda):
    sc = scenes.gs3d_config("c5", seed=0)
    check_view(sc, sc["cameras"][0], band_rows=3, grads=False, render_only=True)


@pytest.fixture(scope="module")
def c4_scene():
    return scenes.gs3d_config("c4", seed=0)
