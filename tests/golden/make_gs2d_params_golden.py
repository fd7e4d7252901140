"""Writes tests/golden/gs2d_params.npz from the REFERENCE's own toy2d parameter layer (toy2d/gs2d/params.py).

    python tests/golden/make_gs2d_params_golden.py /path/to/reference

Runs only where the reference tree exists (imported from <reference>/toy2d, never copied). Stores, for the seeded
Gaussians2D scenes the reference's tests and bench build (sizes, image shapes and seeds below), float32 and
float64: the raw parameters (xy, log_scale, theta, rgb_logit, opacity_logit, depth), the outputs of activate()
(means, conic, color, opacity, cov), radii_from_cov(cov), and the gradients of a fixed weighted sum of activate()'s
outputs with respect to the raw parameters; plus radii_from_cov on hand-made covariances (the eigenvalue floor,
degenerate and negative determinants).
"""
from __future__ import annotations

import sys
from pathlib import Path

import numpy as np
import torch

HERE = Path(__file__).resolve().parent
CASES = [(64, 32, 48, 0, ("f32", "f64")), (1000, 128, 96, 1, ("f32", "f64")), (4096, 256, 256, 7, ("f32",))]


def main(ref_root: str) -> None:
    sys.path.insert(0, str(Path(ref_root) / "toy2d"))
    from gs2d.params import Gaussians2D, activate, radii_from_cov  # reference code

    rec = {}
    for n, H, W, seed, tags in CASES:
        for tag in tags:
            dtype = torch.float32 if tag == "f32" else torch.float64
            g = Gaussians2D(n, H, W, seed=seed, dtype=dtype)
            key = f"{tag}_{n}_{H}x{W}_s{seed}"
            raw = {"xy": g.xy, "log_scale": g.log_scale, "theta": g.theta, "rgb_logit": g.rgb_logit,
                   "opacity_logit": g.opacity_logit}
            for name, t in raw.items():
                rec[f"{key}/{name}"] = t.detach().numpy()
            rec[f"{key}/depth"] = g.depth.numpy()
            out = activate(*raw.values())
            for name, t in zip(("means", "conic", "color", "opacity", "cov"), out):
                rec[f"{key}/{name}"] = t.detach().numpy()
            rec[f"{key}/radii"] = radii_from_cov(out[4].detach()).numpy()
            w = torch.Generator().manual_seed(seed + 99)
            loss = sum((torch.randn(t.shape, generator=w, dtype=dtype) * t).sum() for t in out[:4])
            grads = torch.autograd.grad(loss, list(raw.values()))
            for name, t in zip(raw, grads):
                rec[f"{key}/d_{name}"] = t.numpy()
    cov = torch.tensor([[1.0, 0.0, 1.0], [0.01, 0.0, 0.01], [4.0, 1.99, 1.0], [4.0, 3.0, 1.0], [0.0, 0.0, 0.0],
                        [100.0, -40.0, 25.0], [1e-4, 0.0, 1e-4], [2.25, 0.5, 9.0]], dtype=torch.float64)
    rec["edge/cov"] = cov.numpy()
    rec["edge/radii"] = radii_from_cov(cov).numpy()
    np.savez_compressed(HERE / "gs2d_params.npz", **rec)
    print(f"gs2d_params: {len(rec)} arrays")


if __name__ == "__main__":
    main(sys.argv[1])
