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


def splat2d_bench_scene(n: int, h: int, w: int, seed: int = 0, sigma=(2.0, 10.0), opacity=(0.05, 0.6)):
    """The scene generator of the reference's splat2d backward benchmark (bench/phase0/backward_bench.py:35-49):
    float64 means over the image +-2%, Cholesky factors of per-axis sigma in [2, 10] px with a bounded shear,
    opacity logits of U(0.05, 0.6), colours U(0, 1); index order is depth order."""
    g = torch.Generator().manual_seed(seed)

    def u(lo, hi, *shape):
        return lo + (hi - lo) * torch.rand(*shape, generator=g, dtype=torch.float64)

    means = torch.stack([u(-0.02 * w, 1.02 * w, n), u(-0.02 * h, 1.02 * h, n)], dim=-1)
    l0 = 1.0 / u(sigma[0], sigma[1], n)
    l2 = 1.0 / u(sigma[0], sigma[1], n)
    l1 = u(-0.5, 0.5, n) * torch.minimum(l0, l2)
    o = u(opacity[0], opacity[1], n)
    colors = u(0.0, 1.0, n, 3)
    return means, torch.stack([l0, l1, l2], dim=-1), torch.log(o / (1.0 - o)), colors


# ---------------------------------------------------------------------------------------------
# 3DGS scenes
# ---------------------------------------------------------------------------------------------
def look_at_w2c(eye, target=(0.0, 0.0, 0.0), up=(0.0, 1.0, 0.0), dtype=torch.float32) -> torch.Tensor:
    """World-to-camera [4, 4] (OpenCV axes: x right, y down, z forward) for a camera at ``eye``."""
    e = torch.tensor(eye, dtype=torch.float64)
    t = torch.tensor(target, dtype=torch.float64)
    u = torch.tensor(up, dtype=torch.float64)
    fwd = t - e
    fwd = fwd / fwd.norm()
    right = torch.linalg.cross(fwd, u)
    if right.norm() < 1e-9:
        right = torch.linalg.cross(fwd, torch.tensor([1.0, 0.0, 0.0], dtype=torch.float64))
    right = right / right.norm()
    down = torch.linalg.cross(fwd, right)
    R = torch.stack([right, down, fwd])  # rows: camera axes in world coordinates
    w2c = torch.eye(4, dtype=torch.float64)
    w2c[:3, :3] = R
    w2c[:3, 3] = -R @ e
    return w2c.to(dtype)


def gaussians_3d(n: int, seed: int, centers: torch.Tensor | None = None, sigma: float = 2.0,
                 sh_degree: int = 3) -> dict:
    """Gaussian parameters distributed as the benchmark configs describe: means N(0, sigma^2 I3) (or a mixture
    of isotropic clusters around ``centers``), log-scales N(-3, 0.5), quaternions from N(0,1)^4 (normalised),
    opacity logits N(0, 1.5), SH DC N(0, 0.5) and higher bands N(0, 0.05). float32, CPU."""
    g = torch.Generator().manual_seed(seed)
    if centers is None:
        means = sigma * torch.randn(n, 3, generator=g)
    else:
        k = torch.randint(0, centers.shape[0], (n,), generator=g)
        means = centers[k] + sigma * torch.randn(n, 3, generator=g)
    scales = -3.0 + 0.5 * torch.randn(n, 3, generator=g)
    rot = torch.randn(n, 4, generator=g)
    rot = rot / rot.norm(dim=1, keepdim=True)
    opacities = 1.5 * torch.randn(n, 1, generator=g)
    bases = (sh_degree + 1) ** 2
    sh0 = 0.5 * torch.randn(n, 1, 3, generator=g)
    sh_rest = 0.05 * torch.randn(n, 15, 3, generator=g)
    if bases < 16:
        sh_rest[:, bases - 1:] = 0.0
    return dict(means=means, scales=scales, rotations=rot, opacities=opacities, sh0=sh0, sh_rest=sh_rest,
                active_sh_bases=bases)


def camera(width: int, height: int, eye, fov_y_deg: float = 60.0, near: float = 0.2, far: float = 1000.0,
           bg=(0.0, 0.0, 0.0)) -> dict:
    fy = 0.5 * height / math.tan(math.radians(fov_y_deg) / 2.0)
    return dict(w2c=look_at_w2c(eye), cam_position=torch.tensor(eye, dtype=torch.float32),
                bg_color=torch.tensor(bg, dtype=torch.float32), width=width, height=height, focal_x=fy, focal_y=fy,
                center_x=width / 2.0, center_y=height / 2.0, near_plane=near, far_plane=far)


def gs3d_config(name: str, seed: int = 0) -> dict:
    """C2 single view (100k, 1297x840), C3 scene view (3M in 64 clusters, 1920x1080), C4 training batch
    (1M, 8 cameras on a ring, 1280x720) and C5 render-only (6M in 256 clusters, 3840x2160, 120-frame orbit)."""
    g = torch.Generator().manual_seed(seed + 1000)
    if name == "c2":
        scene = gaussians_3d(100_000, seed, sigma=2.0)
        cams = [camera(1297, 840, (0.0, 0.0, -8.0))]
    elif name == "c3":
        centers = torch.rand(64, 3, generator=g) * 20.0 - 10.0
        scene = gaussians_3d(3_000_000, seed, centers=centers, sigma=1.5)
        d = torch.randn(3, generator=g)
        d = d / d.norm() * 12.0
        cams = [camera(1920, 1080, tuple(d.tolist()))]
    elif name == "c4":
        scene = gaussians_3d(1_000_000, seed, sigma=2.0)
        cams = []
        for k in range(8):
            a = 2 * math.pi * k / 8
            el = math.radians(15.0)
            eye = (10 * math.cos(el) * math.cos(a), -10 * math.sin(el), 10 * math.cos(el) * math.sin(a))
            cams.append(camera(1280, 720, eye))
    elif name == "c5":
        centers = torch.rand(256, 3, generator=g) * 40.0 - 20.0
        scene = gaussians_3d(6_000_000, seed, centers=centers, sigma=2.0)
        cams = []
        for k in range(120):
            a = 2 * math.pi * k / 120
            cams.append(camera(3840, 2160, (15 * math.cos(a), 0.0, 15 * math.sin(a))))
    else:
        raise ValueError(name)
    scene["cameras"] = cams
    return scene


# The reference's own GPU test scenes (phase1/tests/test_parity.py:43-49, phase2/tests/test_readback_equiv.py:35-42):
# (n, width, height, scale range, opacity range, depth range)
TEST_SCENES = {
    "micro": (200, 64, 48, (0.01, 0.1), (0.05, 0.95), (2.0, 8.0)),
    "tiny": (1_000, 160, 120, (0.01, 0.1), (0.05, 0.95), (2.0, 8.0)),
    "partial_tiles": (20_000, 333, 250, (0.005, 0.08), (0.05, 0.95), (2.0, 8.0)),
    "garden_res": (200_000, 1297, 840, (0.002, 0.03), (0.02, 0.99), (2.0, 8.0)),
    "small_splats": (500_000, 1297, 840, (0.0005, 0.006), (0.02, 0.99), (2.0, 8.0)),
    "heavy_overlap": (50_000, 640, 480, (0.05, 0.4), (0.3, 0.99), (2.0, 8.0)),
    "empty": (100, 64, 48, (0.01, 0.1), (0.1, 0.9), (-5.0, -2.0)),
}


def gs3d_test_scene(name: str, seed: int = 0, proper_antialiasing: bool = False, distinct_depths: bool = True) -> dict:
    """A test scene generated the way the reference's GPU tests generate theirs: z ~ U(depth range) (a shuffled even
    grid when ``distinct_depths``, so the depth sort has no ties), x, y within +-0.6 of the frustum, log-uniform
    scales, quaternions N(0, 1), opacity U(range) as logits, sh0 0.8 N(0, 1), sh_rest 0.1 N(0, 1), identity camera
    with focal 0.9 W and the principal point off-centre by (+0.3, -0.2), near 0.2, far 1000, random background."""
    n, w, h, sc, op, dp = TEST_SCENES[name]
    g = torch.Generator().manual_seed(seed)

    def u(lo, hi, *shape):
        return lo + (hi - lo) * torch.rand(*shape, generator=g)

    focal = 0.9 * w
    if distinct_depths:
        z = dp[0] + (dp[1] - dp[0]) * (torch.randperm(n, generator=g).float() + 0.5) / n
    else:
        z = u(dp[0], dp[1], n)
    x = (u(-0.6, 0.6, n) * w / focal) * z
    y = (u(-0.6, 0.6, n) * h / focal) * z
    o = u(op[0], op[1], n, 1)
    scene = dict(means=torch.stack([x, y, z], -1), scales=torch.log(u(sc[0], sc[1], n, 3)),
                 rotations=torch.randn(n, 4, generator=g), opacities=torch.log(o / (1 - o)),
                 sh0=0.8 * torch.randn(n, 1, 3, generator=g), sh_rest=0.1 * torch.randn(n, 15, 3, generator=g),
                 active_sh_bases=16)
    scene["cameras"] = [dict(w2c=torch.eye(4), cam_position=torch.zeros(3), bg_color=torch.rand(3, generator=g),
                             width=w, height=h, focal_x=focal, focal_y=focal, center_x=w / 2 + 0.3,
                             center_y=h / 2 - 0.2, near_plane=0.2, far_plane=1000.0,
                             proper_antialiasing=proper_antialiasing)]
    return scene


def settings_tuple(cam: dict, active_sh_bases: int, device) -> tuple:
    """Camera dict -> the Faster-GS settings tuple (w2c, cam_position, bg, bases, W, H, fx, fy, cx, cy, near, far, aa)."""
    return (cam["w2c"].to(device), cam["cam_position"].to(device), cam["bg_color"].to(device), active_sh_bases,
            cam["width"], cam["height"], cam["focal_x"], cam["focal_y"], cam["center_x"], cam["center_y"],
            cam["near_plane"], cam["far_plane"], cam.get("proper_antialiasing", False))
