"""Float64 PyTorch reference of the 3DGS forward, differentiable end to end (TEST INFRASTRUCTURE: the
gradient ground truth of the tests; the product never calls it).

It restates the rules of 3dgs-project_b200/csrc/gs3d_common.cuh (the library's own restatement of
Faster-GS @ c60ea26, whose blend rules phase1/fastergs_macro.patch:174-211 shows; Faster-GS itself is not
vendored in the reference, so this path's parity is UNPINNED: no reference output exists to check it against):
  preprocess   EWA projection with the clamped Jacobian, +0.3 dilation, optional antialiasing factor,
               conic, sigmoid opacity, real SH of degree <= 3 plus 0.5, pixel-unit mean
  blend        per pixel, front to back over the Gaussians LISTED for the pixel's tile (the tile lists are an
               input: the GPU's own, or the C oracle's), alpha = opacity G, skip below 1/255, stop after the
               splat that drops T below 1e-4, colour clamped at 0, image = C + T bg
Autograd of ``render`` gives dL/d(means, scales, rotations, opacity logits, sh0, sh_rest). Cost is
O(listed Gaussians x pixels): small scenes only.
"""
from __future__ import annotations

import math

import torch

SH0 = 0.28209479177387814
SH1 = 0.4886025119029199
SH2 = (1.0925484305920792, -1.0925484305920792, 0.31539156525252005, -1.0925484305920792, 0.5462742152960396)
SH3 = (-0.5900435899266435, 2.890611442640554, -0.4570457994644658, 0.3731763325901154, -0.4570457994644658,
       1.445305721320277, -0.5900435899266435)
TILE = 16
ALPHA_MIN = 1.0 / 255.0
T_MIN = 1e-4
DILATION = 0.3


def sh_basis(d: torch.Tensor, bases: int) -> torch.Tensor:
    x, y, z = d.unbind(-1)
    out = [torch.full_like(x, SH0)]
    if bases > 1:
        out += [-SH1 * y, SH1 * z, -SH1 * x]
    if bases > 4:
        xx, yy, zz = x * x, y * y, z * z
        out += [SH2[0] * x * y, SH2[1] * y * z, SH2[2] * (2 * zz - xx - yy), SH2[3] * x * z, SH2[4] * (xx - yy)]
        if bases > 9:
            out += [SH3[0] * y * (3 * xx - yy), SH3[1] * x * y * z, SH3[2] * y * (4 * zz - xx - yy),
                    SH3[3] * z * (2 * zz - 3 * xx - 3 * yy), SH3[4] * x * (4 * zz - xx - yy), SH3[5] * z * (xx - yy),
                    SH3[6] * x * (xx - 3 * yy)]
    return torch.stack(out, -1)


def quat_to_rot(q: torch.Tensor) -> torch.Tensor:
    q = q / q.norm(dim=-1, keepdim=True)
    w, x, y, z = q.unbind(-1)
    return torch.stack([
        torch.stack([1 - 2 * (y * y + z * z), 2 * (x * y - w * z), 2 * (x * z + w * y)], -1),
        torch.stack([2 * (x * y + w * z), 1 - 2 * (x * x + z * z), 2 * (y * z - w * x)], -1),
        torch.stack([2 * (x * z - w * y), 2 * (y * z + w * x), 1 - 2 * (x * x + y * y)], -1)], -2)


def preprocess(means, scales, rotations, opacities, sh0, sh_rest, w2c, cam_position, active_sh_bases, width, height,
               fx, fy, cx, cy, proper_antialiasing):
    """Differentiable per-Gaussian projection: mean2d [N,2], conic (A, B, C) [N,3], opacity [N], colour [N,3],
    depth z [N], and the Sigma2 + dilation diagonal (for the culling rectangle)."""
    Wr, t = w2c[:3, :3], w2c[:3, 3]
    pc = means @ Wr.T + t
    x, y, z = pc.unbind(-1)
    R = quat_to_rot(rotations)
    M = R * torch.exp(scales)[:, None, :]
    S3 = M @ M.transpose(1, 2)
    Sc = Wr @ S3 @ Wr.T
    tx = torch.clamp(x / z, -1.3 * cx / fx, 1.3 * (width - cx) / fx)
    ty = torch.clamp(y / z, -1.3 * cy / fy, 1.3 * (height - cy) / fy)
    zero = torch.zeros_like(z)
    J = torch.stack([torch.stack([fx / z, zero, -fx * tx / z], -1),
                     torch.stack([zero, fy / z, -fy * ty / z], -1)], -2)
    S2 = J @ Sc @ J.transpose(1, 2)
    a, b, c = S2[:, 0, 0], S2[:, 0, 1], S2[:, 1, 1]
    ad, cd = a + DILATION, c + DILATION
    det = ad * cd - b * b
    o = torch.sigmoid(opacities.reshape(-1))
    if proper_antialiasing:
        o = o * torch.sqrt(torch.clamp((a * c - b * b) / det, min=0.0))
    conic = torch.stack([cd / det, -b / det, ad / det], -1)
    mean2d = torch.stack([fx * x / z + cx, fy * y / z + cy], -1)
    d = means - cam_position
    d = d / d.norm(dim=-1, keepdim=True)
    basis = sh_basis(d, active_sh_bases)
    coeffs = torch.cat([sh0.reshape(-1, 1, 3), sh_rest[:, : active_sh_bases - 1]], 1)
    color = (basis[..., None] * coeffs).sum(1) + 0.5
    return mean2d, conic, o, color, z, det


def render(means, scales, rotations, opacities, sh0, sh_rest, settings: tuple, tile_lists: list[torch.Tensor],
           mean2d_taps: list | None = None):
    """Image [3, H, W]. ``tile_lists[t]`` holds tile t's Gaussian ids in blend order.
    ``mean2d_taps`` (a list) receives the 2D means as a leaf that keeps its gradient, then for every (Gaussian,
    tile) pair blended a (id, x copy, y copy) triple of per-pixel copies of that mean, whose gradients are the
    per-pixel terms of dL/dmean2d (the densification statistics test sums their absolute values)."""
    (w2c, cam_position, bg, bases, width, height, fx, fy, cx, cy, _near, _far, aa) = settings
    dt = means.dtype
    w2c, cam_position, bg = w2c.to(dt), cam_position.to(dt), bg.to(dt)
    mean2d, conic, o, color, z, _ = preprocess(means, scales, rotations, opacities, sh0, sh_rest, w2c, cam_position,
                                               bases, width, height, fx, fy, cx, cy, aa)
    if mean2d_taps is not None:
        mean2d = mean2d.detach().requires_grad_(True)
        mean2d_taps.append(mean2d)
    col = torch.clamp(color, min=0.0)
    tiles_x = (width + TILE - 1) // TILE
    out = torch.zeros(3, height, width, dtype=dt)
    for t, lst in enumerate(tile_lists):
        tx0, ty0 = (t % tiles_x) * TILE, (t // tiles_x) * TILE
        w, h = min(TILE, width - tx0), min(TILE, height - ty0)
        ys, xs = torch.meshgrid(torch.arange(h, dtype=dt) + ty0 + 0.5, torch.arange(w, dtype=dt) + tx0 + 0.5,
                                indexing="ij")
        T = torch.ones(h, w, dtype=dt)
        C = torch.zeros(3, h, w, dtype=dt)
        done = torch.zeros(h, w, dtype=torch.bool)
        for g in lst.tolist():
            if mean2d_taps is not None:
                mx = (mean2d[g, 0] + torch.zeros_like(xs)).detach().requires_grad_(True)
                my = (mean2d[g, 1] + torch.zeros_like(ys)).detach().requires_grad_(True)
                mean2d_taps.append((g, mx, my))
                # the copies carry the per-pixel terms; the leaf gets their sum through the straight-through link
                mx = mx + (mean2d[g, 0] - mean2d[g, 0].detach())
                my = my + (mean2d[g, 1] - mean2d[g, 1].detach())
            else:
                mx, my = mean2d[g, 0], mean2d[g, 1]
            dx = mx - xs
            dy = my - ys
            power = -0.5 * (conic[g, 0] * dx * dx + 2 * conic[g, 1] * dx * dy + conic[g, 2] * dy * dy)
            alpha = o[g] * torch.exp(torch.clamp(power, max=0.0))
            with torch.no_grad():
                ok = ~done & (alpha >= ALPHA_MIN)
            if not bool(ok.any()):
                continue
            a = torch.where(ok, alpha, torch.zeros_like(alpha))
            C = C + (a * T)[None] * col[g][:, None, None]
            T = T * (1 - a)
            with torch.no_grad():
                done = done | (ok & (T < T_MIN))
        out = _paste(out, C + T[None] * bg[:, None, None], ty0, tx0)
    return out


def _paste(out, p, ty0, tx0):
    """out with the tile block p written at (ty0, tx0), differentiably."""
    pad = torch.nn.functional.pad(p, (tx0, out.shape[2] - tx0 - p.shape[2], ty0, out.shape[1] - ty0 - p.shape[1]))
    mask = torch.zeros(out.shape[1:], dtype=torch.bool)
    mask[ty0:ty0 + p.shape[1], tx0:tx0 + p.shape[2]] = True
    return torch.where(mask[None], pad, out)


def tile_lists_from(ranges: torch.Tensor, point_list: torch.Tensor) -> list[torch.Tensor]:
    r = ranges.cpu().long()
    pl = point_list.cpu().long()
    return [pl[int(s):int(e)] for s, e in r.tolist()]


def sigmoid(x):
    return 1.0 / (1.0 + math.exp(-x))
