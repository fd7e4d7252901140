"""Parameter files: the reference trainer's training-state checkpoint layout and the 3DGS PLY layout (CPU)."""
from __future__ import annotations

import torch

from gs_b200 import scenes, state


def _params(n=257, seed=0):
    sc = scenes.gaussians_3d(n, seed)
    return [sc[k] for k in ("means", "scales", "rotations", "opacities", "sh0", "sh_rest")]


def test_ply_round_trip(tmp_path):
    means, scales, rot, op, sh0, rest = _params()
    p = tmp_path / "scene.ply"
    state.save_ply(p, means, scales, rot, op, sh0, rest)
    head = p.read_bytes()[:2000].decode("ascii", errors="ignore")
    assert "element vertex 257" in head and "property float f_rest_44" in head and "property float rot_3" in head
    back = state.load_ply(p)
    for name, t in zip(("means", "scales", "rotations", "opacities", "sh0", "sh_rest"),
                       (means, scales, rot, op, sh0, rest)):
        assert torch.equal(back[name].reshape(t.shape), t.float()), name


def test_ply_rest_is_channel_major(tmp_path):
    means, scales, rot, op, sh0, rest = _params(3)
    rest = torch.arange(3 * 15 * 3, dtype=torch.float32).reshape(3, 15, 3)
    p = tmp_path / "s.ply"
    state.save_ply(p, means, scales, rot, op, sh0, rest)
    raw = p.read_bytes()
    end = raw.index(b"end_header\n") + len(b"end_header\n")
    import numpy as np
    row = np.frombuffer(raw, dtype="<f4", offset=end)[:62]
    # f_rest_0..14 are channel 0 (red) of coefficients 1..15, then green, then blue
    assert list(row[9:12]) == [0.0, 3.0, 6.0] and row[9 + 15] == 1.0


def test_training_state_layout(tmp_path):
    means, scales, rot, op, sh0, rest = _params()
    leaves = [t.clone().requires_grad_(True) for t in (means, sh0, rest, op, scales, rot)]
    opt = torch.optim.Adam([{"params": [t]} for t in leaves], lr=1e-3)
    sum(t.sum() for t in leaves).backward()
    opt.step()
    p = tmp_path / "state_0000100.pt"
    state.save_state(p, *leaves, optimizer=opt, iteration=100, extent=3.5, active_sh_degree=3)
    st = state.load_state(p)
    assert st["iteration"] == 100 and st["extent"] == 3.5 and st["active_sh_degree"] == 3
    assert set(st["params"]) == set(state.PARAM_KEYS)
    assert torch.equal(st["params"]["_means"], leaves[0].detach())
    assert len(st["optimizer"]["state"]) == 6
