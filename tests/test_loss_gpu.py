"""Fused L1 + SSIM loss (csrc/ssim.cu) against the float64 PyTorch restatement (oracle/ssim_torch.py): loss and
mean SSIM within 1e-5, gradients within 1e-4 norm-relative, on ragged sizes, batches, both paddings; deterministic."""
from __future__ import annotations

import pytest
import torch

from gs_b200 import loss as LS
from oracle import ssim_torch as R

pytestmark = pytest.mark.gpu


def rel(a, b):
    a, b = a.double().flatten().cpu(), b.double().flatten().cpu()
    return float((a - b).norm() / b.norm())


@pytest.mark.parametrize("shape", [(3, 64, 80), (2, 3, 37, 45), (1, 1, 11, 11), (3, 135, 240)])
@pytest.mark.parametrize("padding", ["same", "valid"])
@pytest.mark.parametrize("lam", [0.2, 1.0])
def test_l1_ssim_matches_float64_reference(shape, padding, lam, cuda):
    if padding == "valid" and min(shape[-2:]) <= 10:
        pytest.skip("valid needs images larger than the window")
    g = torch.Generator().manual_seed(sum(shape))
    gt = torch.rand(*shape, generator=g)
    img = (gt + 0.1 * torch.randn(*shape, generator=g)).clamp(0, 1)
    x = img.to(cuda).requires_grad_(True)
    loss = LS.l1_ssim_loss(x, gt.to(cuda), lam, padding)
    loss.backward()
    xr = img.double().requires_grad_(True)
    ref = R.l1_ssim_loss(xr, gt.double(), lam, padding)
    ref.backward()
    assert abs(float(loss.detach()) - float(ref.detach())) < 1e-5
    assert rel(x.grad, xr.grad) < 1e-4


def test_fused_ssim_call_shape(cuda):
    g = torch.Generator().manual_seed(3)
    a, b = torch.rand(2, 3, 50, 70, generator=g), torch.rand(2, 3, 50, 70, generator=g)
    x = a.to(cuda).requires_grad_(True)
    s = LS.fused_ssim(x, b.to(cuda))
    s.backward()
    xr = a.double().requires_grad_(True)
    sr = R.ssim_map(xr, b.double()).mean()
    sr.backward()
    assert abs(float(s.detach()) - float(sr.detach())) < 1e-5
    assert rel(x.grad, xr.grad) < 1e-4


def test_deterministic_and_rejects_bad_input(cuda):
    g = torch.Generator().manual_seed(4)
    a = torch.rand(3, 200, 300, generator=g).to(cuda)
    b = torch.rand(3, 200, 300, generator=g).to(cuda)
    vals = []
    for _ in range(2):
        x = a.clone().requires_grad_(True)
        l = LS.l1_ssim_loss(x, b)
        l.backward()
        vals.append((l.detach().clone(), x.grad.clone()))
    assert torch.equal(vals[0][0], vals[1][0]) and torch.equal(vals[0][1], vals[1][1])
    with pytest.raises(RuntimeError):
        LS.l1_ssim_loss(a, b[:, :, :10])
    with pytest.raises(RuntimeError):
        LS.l1_ssim_loss(a.cpu(), b.cpu())
