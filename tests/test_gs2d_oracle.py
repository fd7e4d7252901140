"""The gs2d oracle against the reference's own outputs (tests/golden/gs2d_*.npz), on the CPU.

Pins oracle/gs2d_oracle.py before any GPU result is compared with it:
  binning       bit-exact vs gs2d.bin_gaussians        (toy2d/gs2d/binning.py:35-88)
  forward       1e-12 vs gs2d.render_reference (fp64)   (toy2d/tests/test_cpu.py:43-48)
  final_T, n_contrib   equal to tests/kernel_emulator.forward
  backward      1e-9 vs autograd of render_reference   (toy2d/tests/test_cpu.py:51-66)
"""
from __future__ import annotations

import numpy as np
import pytest

from conftest import golden
from oracle import gs2d_oracle as O

SMALL = ["tiny", "sparse_odd", "dense", "opaque"]
ALL = SMALL + ["c1"]


def _bins(g):
    return O.bin_gaussians(g["means"].astype(np.float32), g["radii"], g["depth"], int(g["H"]), int(g["W"]))


@pytest.mark.parametrize("scene", ALL)
def test_binning_bit_exact(scene):
    g = golden(f"gs2d_{scene}")
    b = _bins(g)
    for key in ("rect", "order", "point_list", "ranges", "bucket_offsets", "bucket_to_tile"):
        assert np.array_equal(getattr(b, key), g[key]), key
    assert b.num_buckets == int(g["num_buckets"])


@pytest.mark.parametrize("scene", SMALL)
def test_forward_matches_reference(scene):
    g = golden(f"gs2d_{scene}")
    f = O.forward(g["means"], g["conic"], g["color"], g["opacity"], g["bg"], _bins(g))
    assert O.rel_err(f.out, g["image"]) < 1e-12
    assert np.array_equal(f.n_contrib, g["n_contrib"])
    assert np.allclose(f.final_T, g["final_T"], rtol=0, atol=1e-13)


@pytest.mark.parametrize("scene", SMALL)
def test_backward_matches_autograd(scene):
    g = golden(f"gs2d_{scene}")
    b = _bins(g)
    f = O.forward(g["means"], g["conic"], g["color"], g["opacity"], g["bg"], b)
    grads = O.backward(g["means"], g["conic"], g["color"], g["opacity"], g["bg"], b, f, g["dout"])
    for name, got in zip(("dmeans", "dconic", "dcolor", "dopacity"), grads):
        assert O.rel_err(got, g[name]) < 1e-9, name


def test_c1_forward_and_backward():
    g = golden("gs2d_c1")
    b = _bins(g)
    f = O.forward(g["means"], g["conic"], g["color"], g["opacity"], g["bg"], b)
    assert O.rel_err(f.out, g["image"]) < 1e-12
    grads = O.backward(g["means"], g["conic"], g["color"], g["opacity"], g["bg"], b, f, g["dout"])
    for name, got in zip(("dmeans", "dconic", "dcolor", "dopacity"), grads):
        assert O.rel_err(got, g[name]) < 1e-9, name


def test_oracle_detects_a_planted_mistake():
    """A changed rule (alpha cut-off moved) must show up in the comparison, or the test is vacuous."""
    g = golden("gs2d_dense")
    b = _bins(g)
    saved = O.ALPHA_MIN
    try:
        O.ALPHA_MIN = 1.0 / 64.0
        f = O.forward(g["means"], g["conic"], g["color"], g["opacity"], g["bg"], b)
    finally:
        O.ALPHA_MIN = saved
    assert O.rel_err(f.out, g["image"]) > 1e-6
