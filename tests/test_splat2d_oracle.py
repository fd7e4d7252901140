"""The splat2d oracle against the reference's own outputs, on the CPU.

Pins oracle/splat2d_oracle.py: binning bit-exact vs ops.bin_tiles; forward vs ref_render (1e-12) and
vs the reference's compiled extension core (t_final, n_contrib, last_contrib, checkpoints); gradients
vs autograd of ref_render (1e-10, test_gradcheck.py:73-81) and vs both extension backwards.
"""
from __future__ import annotations

import numpy as np
import pytest

from conftest import golden
from oracle import splat2d_oracle as O
from oracle import splat2d_ref

SCENES = [f"seed{s}_n{n}" for s in (0, 1, 2) for n in (8, 32)] + ["dense", "sparse", "random_n1500"]
GROUPS = ("g_means", "g_chol", "g_opacity_logit", "g_colors")


def _scene(name):
    g = golden(f"splat2d_{name}")
    return g, int(g["H"]), int(g["W"])


@pytest.mark.parametrize("name", SCENES)
def test_binning_bit_exact(name):
    g, H, W = _scene(name)
    b = O.bin_tiles(g["means"], g["chol"], g["opacity_logit"], H, W)
    for k in ("tile_offsets", "tile_ids", "bucket_offsets", "bucket_tile"):
        assert np.array_equal(getattr(b, k), g[k]), k


@pytest.mark.parametrize("name", SCENES)
def test_forward_and_backward(name):
    g, H, W = _scene(name)
    b = O.bin_tiles(g["means"], g["chol"], g["opacity_logit"], H, W)
    f = O.forward(g["means"], g["chol"], g["opacity_logit"], g["colors"], b, H, W)
    assert O.rel_err(f.image, g["image"]) < 1e-12
    assert np.array_equal(f.n_contrib, g["ext_n_contrib"])
    assert np.array_equal(f.last_contrib, g["ext_last_contrib"])
    assert np.allclose(f.t_final, g["ext_t_final"], rtol=1e-12, atol=0)
    if "ext_ckpt" in g:
        assert np.allclose(f.ckpt, g["ext_ckpt"], rtol=1e-12, atol=1e-15)
    if name != "sparse":  # the guarded scenes: every (pixel, splat) pair contributes
        assert np.array_equal(f.n_contrib, g["contrib_count"])
    grads = O.backward(g["grad_image"], g["means"], g["chol"], g["opacity_logit"], g["colors"], b, H, W, f)
    for k, got in zip(GROUPS, grads):
        assert O.rel_err(got, g[k]) < 1e-10, k
        for mode in ("pixel", "splat"):
            assert O.rel_err(got, g[f"ext_{mode}_{k}"]) < 1e-10, (k, mode)


@pytest.mark.skipif(not splat2d_ref.available(), reason="reference tree absent at build time")
@pytest.mark.parametrize("name", ["seed0_n32", "dense", "sparse"])
def test_reference_build_reproduces_golden(name):
    """oracle/_ref (the reference's own C++ compiled here) gives the stored outputs again."""
    g, H, W = _scene(name)
    b = O.bin_tiles(g["means"], g["chol"], g["opacity_logit"], H, W)
    rs = splat2d_ref.RefScene(g["means"], g["chol"], g["opacity_logit"], g["colors"], b, H, W)
    fwd = rs.forward()
    assert np.array_equal(fwd[2], g["ext_n_contrib"])
    splat2d_ref.reset_counters()
    grads = rs.backward(True, g["grad_image"], fwd)
    assert splat2d_ref.counters()["atomic_adds"] == int(g["expected_splat_atomics"])
    for k, got in zip(GROUPS, grads):
        assert O.rel_err(got, g[f"ext_splat_{k}"]) < 1e-14


def test_atomic_formulas_hold_in_the_reference():
    """test_opcount.py:404-411 on the stored counts: the formulas the GPU counters are checked with."""
    for name in ("seed0_n32", "dense", "sparse"):
        g, _, _ = _scene(name)
        assert int(g["ext_pixel_atomics"]) == int(g["expected_pixel_atomics"])
        assert int(g["ext_splat_atomics"]) == int(g["expected_splat_atomics"])
