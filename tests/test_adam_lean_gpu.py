"""Lean Adam (adam_step_multi_lean) on the GPU, following the checks of the reference's
cluster/tests/test_lean_adam.py:
  1 no mask, fp32 moments: bit-identical to adam_step_multi over 50 steps (N = 100,003 x 45)
  2 with a mask: visible rows identical to the dense update, invisible rows untouched, for the group shapes
    [N,15,3], [N,3], [N,1], [N,4], [N,1,3]
  3 bf16 moments with stochastic rounding track fp32 over 3000 steps; a beta2 = 0.999 EMA does not stall
  4 the visibility export of a real forward marks every primitive that receives a gradient
plus: the stochastic rounding bits equal the CPU restatement's (oracle/adam_oracle.py) bit for bit, and FusedAdam's
sparse / bfloat16 options run end to end through diff_rasterize."""
from __future__ import annotations

import math

import numpy as np
import pytest
import torch

from gs_b200 import adam as A
from gs_b200 import gs3d
from oracle import adam_oracle as O

pytestmark = pytest.mark.gpu

N = 100_003


def test_dense_lean_equals_original(cuda):
    torch.manual_seed(0)
    p0 = torch.randn(N, 15, 3, device=cuda)
    pa, pb = p0.clone(), p0.clone()
    ma, va, mb, vb = (torch.zeros_like(p0) for _ in range(4))
    for step in range(1, 51):
        g = torch.randn_like(p0) * 1e-3
        A.adam_step([(pa, g, ma, va, 1e-3)], step)
        A.adam_step_lean([(pb, g, mb, vb, 1e-3)], step)
    assert torch.equal(pa, pb) and torch.equal(ma, mb) and torch.equal(va, vb)


def test_masked_update(cuda):
    torch.manual_seed(1)
    p0 = torch.randn(N, 15, 3, device=cuda)
    vis = (torch.rand(N, device=cuda) < 0.4).int() * torch.randint(1, 50, (N,), device=cuda, dtype=torch.int32)
    pa, pb = p0.clone(), p0.clone()
    ma, va = torch.randn_like(p0).abs(), torch.rand_like(p0)
    mb, vb = ma.clone(), va.clone()
    m_before, v_before = ma.clone(), va.clone()
    g = torch.randn_like(p0) * 1e-3
    A.adam_step([(pa, g, ma, va, 1e-3)], 7)
    A.adam_step_lean([(pb, g, mb, vb, 1e-3)], 7, visibility=vis)
    sel = vis > 0
    assert torch.equal(pa[sel], pb[sel]) and torch.equal(ma[sel], mb[sel]) and torch.equal(va[sel], vb[sel])
    assert torch.equal(pb[~sel], p0[~sel]) and torch.equal(mb[~sel], m_before[~sel])
    assert torch.equal(vb[~sel], v_before[~sel])
    for shape in [(N, 3), (N, 1), (N, 4), (N, 1, 3)]:  # features per primitive 3, 1, 4, 3
        q = torch.randn(*shape, device=cuda)
        q0 = q.clone()
        mq, vq = torch.zeros_like(q), torch.zeros_like(q)
        A.adam_step_lean([(q, torch.randn_like(q), mq, vq, 1e-2)], 1, visibility=vis)
        assert torch.equal(q[~sel], q0[~sel]) and bool((q[sel] != q0[sel]).all()), shape


def test_groups_of_several_shapes_in_one_launch(cuda):
    """Six groups with the Gaussian widths in one launch == each group alone (mask applied per primitive)."""
    torch.manual_seed(2)
    n = 20_011
    vis = (torch.rand(n, device=cuda) < 0.5).int()
    shapes = [(n, 3), (n, 3), (n, 4), (n, 1), (n, 1, 3), (n, 15, 3)]
    ps = [torch.randn(*s, device=cuda) for s in shapes]
    gs = [torch.randn_like(p) for p in ps]
    lowp = [False, False, False, False, True, True]
    ms = [torch.zeros_like(p, dtype=torch.bfloat16 if lp else torch.float32) for p, lp in zip(ps, lowp)]
    vs = [torch.zeros_like(m) for m in ms]
    one = [(p.clone(), g, m.clone(), v.clone(), 1e-2 * (k + 1)) for k, (p, g, m, v) in enumerate(zip(ps, gs, ms, vs))]
    A.adam_step_lean(one, 3, visibility=vis)
    for k, (p, g, m, v) in enumerate(zip(ps, gs, ms, vs)):
        A.adam_step_lean([(p, g, m, v, 1e-2 * (k + 1))], 3, visibility=vis)
        assert torch.equal(p, one[k][0]) and torch.equal(m, one[k][2]) and torch.equal(v, one[k][3])


def test_stochastic_rounding_bits_match_oracle(cuda):
    """beta1 = beta2 = 0 makes the stored moments SR(g) and SR(g*g) exactly, so the stored bf16 bits test the hash,
    the seed and the rounding against the CPU restatement bit for bit."""
    torch.manual_seed(3)
    n, step = 50_021, 17
    g = torch.randn(n, device=cuda) * 1e-2
    p = torch.zeros(n, device=cuda)
    m = torch.zeros(n, device=cuda, dtype=torch.bfloat16)
    v = torch.zeros_like(m)
    A.adam_step_lean([(p, g, m, v, 1e-3)], step, betas=(0.0, 0.0))
    gn = g.cpu().numpy()
    r1, r2 = O.sr_randoms(n, step)
    want_m = O.float_to_bf16_bits_sr(gn, r1)
    want_v = O.float_to_bf16_bits_sr((gn * gn).astype(np.float32), r2)
    assert np.array_equal(m.view(torch.int16).cpu().numpy().view(np.uint16), want_m)
    assert np.array_equal(v.view(torch.int16).cpu().numpy().view(np.uint16), want_v)


def test_lean_update_matches_oracle(cuda):
    torch.manual_seed(4)
    n = 30_007
    vis = (torch.rand(n // 3, device=cuda) < 0.6).int()
    p = torch.randn(n // 3, 3, device=cuda)
    g = torch.randn_like(p) * 1e-3
    m = (torch.randn_like(p) * 1e-3).to(torch.bfloat16)
    v = (torch.rand_like(p) * 1e-6).to(torch.bfloat16)
    ref = O.adam_lean(p.cpu().numpy().ravel(), g.cpu().numpy().ravel(), m.view(torch.int16).cpu().numpy().view(np.uint16).ravel(),
                      v.view(torch.int16).cpu().numpy().view(np.uint16).ravel(), 9, 2e-3, visibility=vis.cpu().numpy(),
                      features=3, lowp=True)
    A.adam_step_lean([(p, g, m, v, 2e-3)], 9, visibility=vis)
    got_p = p.cpu().numpy().ravel()
    assert np.allclose(got_p, ref[0], rtol=1e-6, atol=1e-9)
    # moments: identical bits except where a float64-emulated fma rounded the pre-rounding value differently
    gm = m.view(torch.int16).cpu().numpy().view(np.uint16).ravel()
    gv = v.view(torch.int16).cpu().numpy().view(np.uint16).ravel()
    assert (gm != ref[1]).mean() < 1e-3 and (gv != ref[2]).mean() < 1e-3


def test_bf16_moments_track_fp32(cuda):
    torch.manual_seed(5)
    pr = torch.randn(N, 15, 3, device=cuda)
    pinit = pr.clone()
    pl = pr.clone()
    mr, vr = torch.zeros_like(pr), torch.zeros_like(pr)
    ml, vl = torch.zeros_like(pr, dtype=torch.bfloat16), torch.zeros_like(pr, dtype=torch.bfloat16)
    scale = torch.rand(N, 1, 1, device=cuda) * 1e-3 + 1e-6
    bias = torch.randn_like(pr) * scale
    lr = 1.25e-4
    for step in range(1, 3001):
        g = bias + torch.randn_like(pr) * scale
        A.adam_step([(pr, g, mr, vr, lr)], step)
        A.adam_step_lean([(pl, g, ml, vl, lr)], step)
    rel_v = float(((vl.float() - vr).abs() / (vr.abs() + 1e-30)).median())
    rel_m = float((ml.float() - mr).norm() / mr.norm())
    rel_upd = float(((pr - pinit) - (pl - pinit)).norm() / (pr - pinit).norm())
    assert rel_v < 0.05 and rel_m < 0.05 and rel_upd < 0.02, (rel_v, rel_m, rel_upd)
    # stall control: constant gradient after a warm start; the EMA must keep approaching g^2
    g_const = torch.full((1 << 20,), 1.0, device=cuda)
    v_sr = torch.full_like(g_const, 0.5).to(torch.bfloat16)
    m_sr = torch.zeros_like(v_sr)
    q = torch.zeros_like(g_const)
    for step in range(1, 3001):
        A.adam_step_lean([(q, g_const, m_sr, v_sr, 0.0)], 10_000 + step)
    expected = 1.0 - 0.5 * 0.999 ** 3000
    assert abs(float(v_sr.float().mean()) - expected) < 0.005


def _visibility_scene(dev, n=20_000):
    g = torch.Generator(device=dev).manual_seed(6)
    sign = torch.where(torch.rand(n, 1, device=dev, generator=g) < 0.5, -1.0, 1.0)
    means = (torch.randn(n, 3, device=dev, generator=g) * torch.tensor([2.0, 2.0, 1.0], device=dev)
             + sign * torch.tensor([0, 0, 5.0], device=dev))
    params = [means, torch.full((n, 3), math.log(0.03), device=dev),
              torch.cat([torch.ones(n, 1, device=dev), torch.zeros(n, 3, device=dev)], 1),
              torch.zeros(n, 1, device=dev), torch.rand(n, 1, 3, device=dev, generator=g), torch.zeros(n, 15, 3, device=dev)]
    settings = gs3d.RasterizerSettings(w2c=torch.eye(4, device=dev), cam_position=torch.zeros(3, device=dev),
                                       bg_color=torch.zeros(3, device=dev), active_sh_bases=1, width=320, height=240,
                                       focal_x=300.0, focal_y=300.0, center_x=160.0, center_y=120.0, near_plane=0.2,
                                       far_plane=1000.0, proper_antialiasing=False)
    return params, settings


def test_visibility_export_covers_gradients(cuda):
    params, settings = _visibility_scene(cuda)
    leaves = [p.clone().requires_grad_(True) for p in params]
    gs3d._Rasterize.track_visibility = True
    try:
        img = gs3d.diff_rasterize(*leaves, torch.empty(0), settings)
        img.sum().backward()
        vmask = gs3d._Rasterize.last_visibility
    finally:
        gs3d._Rasterize.track_visibility = False
    n = params[0].shape[0]
    gnz = leaves[0].grad.abs().sum(1) > 0
    assert vmask is not None and vmask.shape == (n,) and vmask.dtype == torch.int32
    assert bool((vmask[gnz] > 0).all())
    assert int((vmask > 0).sum()) > 0 and int((vmask == 0).sum()) > 0


def test_fused_adam_sparse_and_bf16_options(cuda):
    params, settings = _visibility_scene(cuda)
    names = ("means", "scales", "rotations", "opacities", "sh0", "sh_rest")
    leaves = [p.clone().requires_grad_(True) for p in params]
    opt = A.FusedAdam([{"params": [p], "lr": 1e-3, "name": nm} for p, nm in zip(leaves, names)], lr=0.0, eps=1e-15,
                      sparse=True, lowp_moment_groups=("sh_rest",))
    try:
        before = [p.detach().clone() for p in leaves]
        img = gs3d.diff_rasterize(*leaves, torch.empty(0), settings)
        (img * torch.randn_like(img)).sum().backward()
        opt.step()
        vis = gs3d._Rasterize.last_visibility > 0
        assert opt.state[leaves[5]]["exp_avg"].dtype == torch.bfloat16
        assert opt.state[leaves[0]]["exp_avg"].dtype == torch.float32
        for p, b in zip(leaves, before):
            assert torch.equal(p.detach()[~vis], b[~vis])
        assert not torch.equal(leaves[0].detach()[vis], before[0][vis])
        assert opt.n_dense_fallbacks == 0
    finally:
        gs3d._Rasterize.track_visibility = False
