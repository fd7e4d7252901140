"""Float64 PyTorch restatement of the L1 + SSIM training loss (TEST INFRASTRUCTURE only).

SSIM as published (Wang et al. 2004) and as the fused-ssim package used by the reference's trainer computes it
(that package is not vendored): 11x11 Gaussian window with sigma 1.5, normalised; C1 = 0.01^2, C2 = 0.03^2;
per-channel convolution with zero padding; "valid" keeps only the outputs whose window lies inside the image.
"""
from __future__ import annotations

import math

import torch
import torch.nn.functional as F


def window(dtype=torch.float64) -> torch.Tensor:
    d = torch.arange(11, dtype=dtype) - 5
    g = torch.exp(-d * d / (2 * 1.5 ** 2))
    g = g / g.sum()
    return g[:, None] * g[None, :]


def ssim_map(x: torch.Tensor, y: torch.Tensor, padding: str = "same") -> torch.Tensor:
    if x.dim() == 3:
        x, y = x[None], y[None]
    C = x.shape[1]
    w = window(x.dtype).to(x.device)[None, None].expand(C, 1, 11, 11).contiguous()
    pad = 5 if padding == "same" else 0

    def conv(t):
        return F.conv2d(t, w, padding=pad, groups=C)

    m1, m2 = conv(x), conv(y)
    s1 = conv(x * x) - m1 * m1
    s2 = conv(y * y) - m2 * m2
    s12 = conv(x * y) - m1 * m2
    c1, c2 = 0.01 ** 2, 0.03 ** 2
    return ((2 * m1 * m2 + c1) * (2 * s12 + c2)) / ((m1 * m1 + m2 * m2 + c1) * (s1 + s2 + c2))


def l1_ssim_loss(x, y, lam: float = 0.2, padding: str = "same"):
    return (1 - lam) * (x - y).abs().mean() + lam * (1 - ssim_map(x, y, padding).mean())


assert math.isclose(float(window().sum()), 1.0)
