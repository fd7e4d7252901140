"""gs2d's parameter layer against the reference's own (tests/golden/gs2d_params.npz, written by importing
toy2d/gs2d/params.py): Gaussians2D's seeded initialisation, activate() and its gradients, radii_from_cov() on the
seeded scenes and on hand-made covariances (eigenvalue floor, degenerate and negative determinants). CPU only."""
from __future__ import annotations

import numpy as np
import pytest
import torch
from conftest import golden

from gs_b200 import gs2d

G = golden("gs2d_params")
CASES = sorted({k.split("/")[0] for k in G if not k.startswith("edge")})
RAW = ("xy", "log_scale", "theta", "rgb_logit", "opacity_logit")


@pytest.mark.parametrize("key", CASES)
def test_seeded_init_activation_radii_and_gradients_match_the_reference(key):
    tag, n, hw, seed = key.split("_")
    H, W = (int(v) for v in hw.split("x"))
    dtype = torch.float32 if tag == "f32" else torch.float64
    g = gs2d.Gaussians2D(int(n), H, W, seed=int(seed[1:]), dtype=dtype)
    raw = {"xy": g.xy, "log_scale": g.log_scale, "theta": g.theta, "rgb_logit": g.rgb_logit,
           "opacity_logit": g.opacity_logit}
    for name, t in raw.items():
        assert np.array_equal(t.detach().numpy(), G[f"{key}/{name}"]), name  # same draws, bit for bit
    assert np.array_equal(g.depth.numpy(), G[f"{key}/depth"])
    out = gs2d.activate(*raw.values())
    for name, t in zip(("means", "conic", "color", "opacity", "cov"), out):
        assert np.array_equal(t.detach().numpy(), G[f"{key}/{name}"]), name  # the same operations in order
    assert np.array_equal(gs2d.radii_from_cov(out[4].detach()).numpy(), G[f"{key}/radii"])
    w = torch.Generator().manual_seed(int(seed[1:]) + 99)
    loss = sum((torch.randn(t.shape, generator=w, dtype=dtype) * t).sum() for t in out[:4])
    grads = torch.autograd.grad(loss, list(raw.values()))
    for name, t in zip(RAW, grads):
        np.testing.assert_allclose(t.numpy(), G[f"{key}/d_{name}"], rtol=1e-6 if tag == "f32" else 1e-12,
                                   atol=1e-7 if tag == "f32" else 1e-14, err_msg=name)


def test_radii_edge_covariances_match_the_reference():
    cov = torch.from_numpy(G["edge/cov"])
    assert np.array_equal(gs2d.radii_from_cov(cov).numpy(), G["edge/radii"])
