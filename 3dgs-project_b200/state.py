"""Saving and loading the six parameter tensors.

* `save_state` / `load_state`: the training-state checkpoint the reference's trainer hook writes
  (cluster/patches/fastergs_save_state.py:27-35): a torch.save dict with 'iteration', 'params' (the six tensors
  under Faster-GS's attribute names), 'optimizer' (the optimizer's state_dict), 'extent' and 'active_sh_degree'.
* `save_ply` / `load_ply`: the binary little-endian PLY layout of 3D Gaussian Splatting scenes (x y z, nx ny nz,
  f_dc_0..2, f_rest_* with the coefficients of one colour channel after another, opacity, scale_0..2, rot_0..3),
  parameters stored raw (log scales, opacity logits, unnormalised quaternions w x y z), as written by the 3DGS
  reference implementation and read by its viewers.
"""
from __future__ import annotations

import numpy as np
import torch

PARAM_KEYS = ("_means", "_sh_coefficients_0", "_sh_coefficients_rest", "_opacities", "_scales", "_rotations")


def save_state(path, means, sh0, sh_rest, opacities, scales, rotations, optimizer=None, iteration: int = 0,
               extent: float | None = None, active_sh_degree: int | None = None) -> None:
    tensors = (means, sh0, sh_rest, opacities, scales, rotations)
    torch.save({"iteration": int(iteration),
                "params": {k: t.detach().clone() for k, t in zip(PARAM_KEYS, tensors)},
                "optimizer": None if optimizer is None else optimizer.state_dict(),
                "extent": extent, "active_sh_degree": active_sh_degree}, path)


def load_state(path, map_location="cpu") -> dict:
    state = torch.load(path, map_location=map_location, weights_only=False)
    missing = [k for k in PARAM_KEYS if k not in state.get("params", {})]
    if missing:
        raise RuntimeError(f"{path}: not a training state (missing {missing})")
    return state


def _columns(rest_bases: int) -> list[str]:
    cols = ["x", "y", "z", "nx", "ny", "nz", "f_dc_0", "f_dc_1", "f_dc_2"]
    cols += [f"f_rest_{k}" for k in range(3 * rest_bases)]
    cols += ["opacity", "scale_0", "scale_1", "scale_2", "rot_0", "rot_1", "rot_2", "rot_3"]
    return cols


def save_ply(path, means, scales, rotations, opacities, sh0, sh_rest) -> None:
    """means [N,3], scales [N,3] (log), rotations [N,4] (w,x,y,z), opacities [N] or [N,1] (logits),
    sh0 [N,1,3] or [N,3], sh_rest [N,K,3]."""
    n = means.shape[0]
    rest = sh_rest.reshape(n, -1, 3)
    k = rest.shape[1]
    cols = [means.reshape(n, 3), torch.zeros(n, 3, dtype=means.dtype, device=means.device), sh0.reshape(n, 3),
            rest.transpose(1, 2).reshape(n, 3 * k), opacities.reshape(n, 1), scales.reshape(n, 3),
            rotations.reshape(n, 4)]
    data = torch.cat([c.detach().to(torch.float32).cpu() for c in cols], 1).numpy()
    names = _columns(k)
    header = ["ply", "format binary_little_endian 1.0", f"element vertex {n}"]
    header += [f"property float {c}" for c in names] + ["end_header"]
    with open(path, "wb") as f:
        f.write(("\n".join(header) + "\n").encode("ascii"))
        f.write(np.ascontiguousarray(data, dtype="<f4").tobytes())


def load_ply(path) -> dict[str, torch.Tensor]:
    """The tensors of save_ply, in the rasterizer's layout: means, scales, rotations, opacities [N,1],
    sh0 [N,1,3], sh_rest [N,K,3]."""
    with open(path, "rb") as f:
        raw = f.read()
    end = raw.index(b"end_header\n") + len(b"end_header\n")
    lines = raw[:end].decode("ascii").splitlines()
    if lines[0] != "ply" or lines[1] != "format binary_little_endian 1.0":
        raise RuntimeError(f"{path}: not a binary little-endian PLY")
    n = int(next(l for l in lines if l.startswith("element vertex")).split()[-1])
    names = [l.split()[-1] for l in lines if l.startswith("property")]
    if any(not l.startswith("property float") for l in lines if l.startswith("property")):
        raise RuntimeError(f"{path}: only float properties are supported")
    data = np.frombuffer(raw, dtype="<f4", count=n * len(names), offset=end).reshape(n, len(names))
    col = {nm: k for k, nm in enumerate(names)}

    def take(keys):
        return torch.from_numpy(np.ascontiguousarray(data[:, [col[k] for k in keys]]))

    k = sum(1 for nm in names if nm.startswith("f_rest_")) // 3
    rest = take([f"f_rest_{j}" for j in range(3 * k)]).reshape(n, 3, k).transpose(1, 2).contiguous()
    return {"means": take(["x", "y", "z"]), "scales": take(["scale_0", "scale_1", "scale_2"]),
            "rotations": take(["rot_0", "rot_1", "rot_2", "rot_3"]), "opacities": take(["opacity"]),
            "sh0": take(["f_dc_0", "f_dc_1", "f_dc_2"]).reshape(n, 1, 3), "sh_rest": rest}
