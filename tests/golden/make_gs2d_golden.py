"""Writes tests/golden/gs2d_<scene>.npz from the REFERENCE's own toy2d code.

    python tests/golden/make_gs2d_golden.py /path/to/reference

Runs only where the reference tree exists (it is imported from <reference>/toy2d, never copied). For
each of the reference's test scenes (toy2d/tests/scenes.py:8-17) and for config C1 it stores:
  inputs   means, conic, color, opacity (float64), bg, depth, radii
  bins     rect, order, point_list, ranges, bucket_offsets, bucket_to_tile   (gs2d.bin_gaussians)
  forward  image (gs2d.render_reference, float64)
  backward dmeans, dconic, dcolor, dopacity for dout (autograd of render_reference, float64)
  emulator final_T, n_contrib (tests/kernel_emulator.forward) for the small scenes
"""
from __future__ import annotations

import sys
import time
from pathlib import Path

import numpy as np
import torch

HERE = Path(__file__).resolve().parent
ROOT = HERE.parent.parent


def main(ref_root: str) -> None:
    toy = Path(ref_root) / "toy2d"
    sys.path.insert(0, str(toy))
    sys.path.append(str(ROOT))
    from gs2d import Gaussians2D, bin_gaussians, render_reference  # reference code
    from gs2d.params import activate, radii_from_cov  # reference code
    from tests import kernel_emulator as emu  # reference code
    from tests.scenes import SCENES, upstream_grad  # reference code

    from __graft_entry__ import load_package

    load_package()
    from gs_b200 import scenes as synth

    def save(name, means, conic, color, opacity, bg, depth, radii, bins, dout, with_emu):
        leaves = [t.detach().double().clone().requires_grad_(True) for t in (means, conic, color, opacity)]
        t0 = time.time()
        img = render_reference(*leaves, bins, bg.double())
        grads = torch.autograd.grad(img, leaves, dout.double())
        rec = dict(
            means=leaves[0].detach().numpy(), conic=leaves[1].detach().numpy(), color=leaves[2].detach().numpy(),
            opacity=leaves[3].detach().numpy(), bg=bg.double().numpy(), depth=depth.numpy(),
            radii=radii.numpy(), H=bins.H, W=bins.W,
            rect=bins.rect.numpy(), order=bins.order.numpy(), point_list=bins.point_list.numpy(),
            ranges=bins.ranges.numpy(), bucket_offsets=bins.bucket_offsets.numpy(),
            bucket_to_tile=bins.bucket_to_tile.numpy(), num_buckets=bins.num_buckets,
            image=img.detach().numpy(), dout=dout.float().numpy() if name == "c1" else dout.double().numpy(),
            dmeans=grads[0].numpy(), dconic=grads[1].numpy(), dcolor=grads[2].numpy(), dopacity=grads[3].numpy())
        if with_emu:
            _, final_T, n_contrib, _ = emu.forward(*[t.detach() for t in leaves], bg.double(), bins)
            rec["final_T"] = np.array(final_T)
            rec["n_contrib"] = np.array(n_contrib, dtype=np.int32)
        np.savez_compressed(HERE / f"gs2d_{name}.npz", **rec)
        print(f"gs2d_{name}: N={means.shape[0]} {bins.H}x{bins.W} M={bins.point_list.numel()} "
              f"B={bins.num_buckets} ({time.time() - t0:.1f}s)")

    # the reference's own test scenes, built as toy2d/tests/scenes.py:21-31 builds them
    for name, (n, H, W, scale_mult, op_shift, seed) in SCENES.items():
        g = Gaussians2D(n, H, W, seed=seed, dtype=torch.float64)
        with torch.no_grad():
            g.log_scale += torch.log(torch.tensor(scale_mult, dtype=torch.float64))
            g.opacity_logit += op_shift
        means, conic, color, opacity, cov = (t.detach() for t in g.activated())
        radii = radii_from_cov(cov)
        bins = bin_gaussians(means, radii, g.depth, H, W)
        bg = torch.tensor((0.2, 0.5, 0.8), dtype=torch.float64)
        save(name, means, conic, color, opacity, bg, g.depth.detach(), radii, bins, upstream_grad(H, W), True)

    # config C1: 4096 Gaussians, 256x256, black background, L2 loss against the sinusoid target
    c1 = synth.gs2d_c1(seed=0)
    means, conic, color, opacity, cov = activate(c1["xy"], c1["log_scale"], c1["theta"],
                                                 torch.logit(c1["rgb"]), c1["opacity_logit"])
    color = c1["rgb"]
    radii = radii_from_cov(cov)
    bins = bin_gaussians(means, radii, c1["depth"], c1["H"], c1["W"])
    with torch.no_grad():
        img = render_reference(means, conic, color, opacity, bins, torch.zeros(3, dtype=torch.float64))
    # the upstream gradient is rounded to float32 (and stored as such) so the fixture stays small
    dout = (2.0 * (img - c1["target"]) / img.numel()).float().double()
    save("c1", means, conic, color, opacity, torch.zeros(3, dtype=torch.float64), c1["depth"], radii, bins, dout,
         False)


if __name__ == "__main__":
    if len(sys.argv) != 2:
        sys.exit("usage: make_gs2d_golden.py <reference root>")
    main(sys.argv[1])
