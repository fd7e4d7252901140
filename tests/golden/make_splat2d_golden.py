"""Writes tests/golden/splat2d_<scene>.npz from the REFERENCE's own phase0 code.

    python tests/golden/make_splat2d_golden.py <reference root>

Imports <reference>/phase0 (splat2d.ops and tests/gradcheck/conftest.py) - never copied - and the
reference's compiled CPU extension core (oracle/_ref/libsplat2d_ref.so, built by oracle/build.py from
phase0/csrc/macrotile/splat2d_cpu.cpp). For each of the reference's scenes (guarded seeds 0-2 x N 8/32,
dense_n96, sparse_n150; phase0/tests/gradcheck/conftest.py:124-163) plus one larger random scene:
  inputs     means, chol, opacity_logit, colors (float64), grad_image (the scene's seeded dL/dimage)
  bins       tile_offsets, tile_ids, bucket_offsets, bucket_tile            (ops.bin_tiles)
  reference  image, grads (ref_render + autograd, float64); contributes count (ref_state)
  extension  t_final, n_contrib, last_contrib, ckpt and both backwards' gradients, float64, plus the
             op counters of each backward, and the atomic-count formulas of test_opcount.py:372-395
"""
from __future__ import annotations

import importlib.util
import sys
from pathlib import Path

import numpy as np
import torch

HERE = Path(__file__).resolve().parent
ROOT = HERE.parent.parent


def main(ref_root: str) -> None:
    phase0 = Path(ref_root) / "phase0"
    sys.path.insert(0, str(phase0))
    sys.path.append(str(ROOT))
    from splat2d import ops  # reference code

    spec = importlib.util.spec_from_file_location("ref_gradcheck_conftest",
                                                  phase0 / "tests" / "gradcheck" / "conftest.py")
    conf = importlib.util.module_from_spec(spec)
    sys.modules[spec.name] = conf
    spec.loader.exec_module(conf)  # reference code

    from oracle import build as oracle_build
    from oracle import splat2d_ref

    oracle_build.build(ref_root)
    assert splat2d_ref.available()

    scenes = {f"seed{s}_n{n}": conf.guarded_scene(s, n) for s in conf.SEEDS for n in conf.GRADCHECK_N}
    scenes["dense"] = conf.dense_scene_cached()
    scenes["sparse"] = conf.sparse_scene_cached()
    big = conf.make_scene("random_n1500", 21, 1500, 96, 136, sigma=(2.0, 9.0), opacity=(0.1, 0.95),
                          mean_box=(-0.05, 1.05))
    scenes["random_n1500"] = big

    for name, sc in scenes.items():
        H, W = sc.height, sc.width
        params = sc.params(torch.float64)
        bins = ops.bin_tiles(*params[:3], H, W)
        image = ops.ref_render(*params, H, W)
        g_img = sc.grad_image(torch.float64)
        grads = torch.autograd.grad(image, params, g_img)
        st = ops.ref_state(*[p.detach() for p in params], H, W)
        rs = splat2d_ref.RefScene(*[p.detach().numpy() for p in params], bins, H, W)
        fwd = rs.forward()
        rec = dict(
            means=params[0].detach().numpy(), chol=params[1].detach().numpy(),
            opacity_logit=params[2].detach().numpy(), colors=params[3].detach().numpy(), H=H, W=W,
            grad_image=g_img.numpy(), tile_offsets=bins.tile_offsets.numpy(), tile_ids=bins.tile_ids.numpy(),
            bucket_offsets=bins.bucket_offsets.numpy(), bucket_tile=bins.bucket_tile.numpy(),
            image=image.detach().numpy(), g_means=grads[0].numpy(), g_chol=grads[1].numpy(),
            g_opacity_logit=grads[2].numpy(), g_colors=grads[3].numpy(),
            contrib_count=st.contributes.sum(-1).numpy().astype(np.int32),
            ext_image=fwd[0], ext_t_final=fwd[1], ext_n_contrib=fwd[2], ext_last_contrib=fwd[3])
        if bins.num_buckets <= 64:  # checkpoints of the small scenes only (they grow by 8 KB per bucket)
            rec["ext_ckpt"] = fwd[4]
        for mode in ("pixel", "splat"):
            splat2d_ref.reset_counters()
            g = rs.backward(mode == "splat", g_img.numpy(), fwd)
            cnt = splat2d_ref.counters()
            for k, v in zip(("g_means", "g_chol", "g_opacity_logit", "g_colors"), g):
                rec[f"ext_{mode}_{k}"] = v
            rec[f"ext_{mode}_atomics"] = cnt["atomic_adds"]
        # test_opcount.py:372-395: sum_p n_contrib * 9 and sum over (tile, bucket) of splats used * 9
        rec["expected_pixel_atomics"] = int(fwd[2].sum()) * 9
        total = 0
        offs = bins.tile_offsets.tolist()
        ids = bins.tile_ids.long()
        for t in range(bins.tiles_x * bins.tiles_y):
            x0, y0 = (t % bins.tiles_x) * 16, (t // bins.tiles_x) * 16
            region = st.contributes[y0:y0 + 16, x0:x0 + 16]
            for start in range(offs[t], offs[t + 1], 32):
                bucket = ids[start:min(start + 32, offs[t + 1])]
                total += int(region[:, :, bucket].flatten(0, 1).any(dim=0).sum())
        rec["expected_splat_atomics"] = total * 9
        np.savez_compressed(HERE / f"splat2d_{name}.npz", **rec)
        print(f"splat2d_{name}: N={sc.n} {H}x{W} M={bins.tile_ids.numel()} B={bins.num_buckets}")


if __name__ == "__main__":
    if len(sys.argv) != 2:
        sys.exit("usage: make_splat2d_golden.py <reference root>")
    main(sys.argv[1])
