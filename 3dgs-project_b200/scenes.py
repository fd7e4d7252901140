"""Seeded synthetic inputs with the shapes and distributions of the five benchmark configs.

None of the configs comes from a public dataset; these generators stand in for them (the reference's
real-scene numbers use Mip-NeRF360 captures, which are not available here).

    gs2d_c1   C1: 4096 anisotropic 2D Gaussians, 256x256, sinusoid target (toy2d fit)
    gs3d_scene(kind)  C2 single view (100k), C3 scene view (3M, 64 clusters), C4 batched training
              (1M, 8-camera ring), C5 render-only (6M, 256 clusters) plus small test scenes
"""
from __future__ import annotations

import math

import torch


def sinusoid_target(H: int, W: int, seed: int, n_waves: int = 32, dtype=torch.float64) -> torch.Tensor:
    """(3, H, W) smooth random image: per channel 0.5 + sum of n_waves sinusoids, scaled into [0, 1]."""
    g = torch.Generator().manual_seed(seed)
    ys, xs = torch.meshgrid(torch.arange(H, dtype=dtype), torch.arange(W, dtype=dtype), indexing="ij")
    out = torch.empty(3, H, W, dtype=dtype)
    for c in range(3):
        amp = torch.rand(n_waves, generator=g, dtype=dtype)
        fx = (torch.rand(n_waves, generator=g, dtype=dtype) * 2 - 1) * (8 * math.pi / W)
        fy = (torch.rand(n_waves, generator=g, dtype=dtype) * 2 - 1) * (8 * math.pi / H)
        ph = torch.rand(n_waves, generator=g, dtype=dtype) * (2 * math.pi)
        acc = torch.zeros(H, W, dtype=dtype)
        for k in range(n_waves):
            acc += amp[k] * torch.sin(fx[k] * xs + fy[k] * ys + ph[k])
        out[c] = 0.5 + 0.5 * acc / amp.sum()
    return out


def gs2d_c1(seed: int = 0) -> dict:
    """Config C1 (float64 on the CPU; cast as needed): means U[0,256)^2, log-scales N(ln 3, 0.3),
    rotation U[0, pi), opacity logits N(0, 1), RGB U[0, 1] used directly as colour, depth U[0, 1)."""
    n, H, W = 4096, 256, 256
    g = torch.Generator().manual_seed(seed)
    f64 = torch.float64
    xy = torch.rand(n, 2, generator=g, dtype=f64) * 256.0
    log_scale = math.log(3.0) + 0.3 * torch.randn(n, 2, generator=g, dtype=f64)
    theta = torch.rand(n, generator=g, dtype=f64) * math.pi
    opacity_logit = torch.randn(n, generator=g, dtype=f64)
    rgb = torch.rand(n, 3, generator=g, dtype=f64)
    depth = torch.rand(n, generator=g, dtype=f64)
    return dict(n=n, H=H, W=W, xy=xy, log_scale=log_scale, theta=theta, opacity_logit=opacity_logit, rgb=rgb,
                depth=depth, target=sinusoid_target(H, W, seed + 1))
