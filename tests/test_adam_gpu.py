"""Fused Adam (one launch over all groups) vs torch.optim.Adam and vs the update formula of
cluster/patches/fastergs_lean_adam.patch:112-117 (cluster/tests/test_lean_adam.py:30-35)."""
from __future__ import annotations

import math

import pytest
import torch

from gs_b200 import adam as gs_adam

pytestmark = pytest.mark.gpu


def adam_ref(p, g, m, v, step, lr, b1=0.9, b2=0.999, eps=1e-15):
    m.mul_(b1).add_(g, alpha=1 - b1)
    v.mul_(b2).addcmul_(g, g, value=1 - b2)
    denom = v.sqrt() / math.sqrt(1 - b2 ** step) + eps
    p.addcdiv_(m, denom, value=-lr / (1 - b1 ** step))


def test_matches_formula_over_many_groups(cuda):
    torch.manual_seed(0)
    sizes = [(100_003, 3), (100_003, 4), (100_003, 1), (100_003, 15, 3), (7,), (4097, 2)]
    lrs = [1.6e-4, 1e-3, 5e-2, 2.5e-3, 0.1, 3e-3]
    ps = [torch.randn(*s, device=cuda) for s in sizes]
    ref = [p.clone().double() for p in ps]
    ms = [torch.zeros_like(p) for p in ps]
    vs = [torch.zeros_like(p) for p in ps]
    rm = [torch.zeros_like(p) for p in ref]
    rv = [torch.zeros_like(p) for p in ref]
    for step in range(1, 31):
        gs = [torch.randn_like(p) * 1e-3 for p in ps]
        gs_adam.adam_step([(p, g, m, v, lr) for p, g, m, v, lr in zip(ps, gs, ms, vs, lrs)], step)
        for p, g, m, v, lr in zip(ref, gs, rm, rv, lrs):
            adam_ref(p, g.double(), m, v, step, lr)
    for p, r in zip(ps, ref):
        assert torch.allclose(p.double(), r, rtol=0, atol=1e-5 * float(r.abs().max()))


def test_fused_adam_optimizer_matches_torch_adam(cuda):
    torch.manual_seed(1)
    a = [torch.randn(1000, 3, device=cuda, requires_grad=True), torch.randn(1000, 15, 3, device=cuda,
                                                                              requires_grad=True)]
    b = [t.detach().clone().requires_grad_(True) for t in a]
    opt_a = gs_adam.FusedAdam([{"params": [a[0]], "lr": 1e-3}, {"params": [a[1]], "lr": 2e-3}], lr=0.0, eps=1e-15)
    opt_b = torch.optim.Adam([{"params": [b[0]], "lr": 1e-3}, {"params": [b[1]], "lr": 2e-3}], lr=0.0, eps=1e-15)
    for _ in range(20):
        for x in (a, b):
            loss = sum((t ** 2).sum() for t in x)
            loss.backward()
        opt_a.step()
        opt_b.step()
        opt_a.zero_grad()
        opt_b.zero_grad()
    for x, y in zip(a, b):
        assert torch.allclose(x, y, rtol=1e-5, atol=1e-6)
    # state_dict layout matches torch.optim.Adam
    sa, sb = opt_a.state_dict()["state"], opt_b.state_dict()["state"]
    assert sa.keys() == sb.keys()
    for k in sa:
        assert set(sa[k]) == set(sb[k])
        # the reference's fmaf(beta2, v - g^2, g^2) weighs g^2 by 1 - float(0.999), torch by float(1 - 0.999):
        # 1.3e-5 apart
        assert torch.allclose(sa[k]["exp_avg_sq"], sb[k]["exp_avg_sq"], rtol=5e-5, atol=1e-12)
