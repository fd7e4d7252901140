"""Drop-in for the toy2d ``gs2d`` package (toy2d/gs2d/__init__.py): same names, same arguments.

    from gs_b200.gs2d import Gaussians2D, bin_gaussians, rasterize
    means, conic, color, opacity, cov = model.activated()
    bins = bin_gaussians(means, radii_from_cov(cov), model.depth, H, W)
    img = rasterize(means, conic, color, opacity, bins, backend="splat")

Everything rasterizer-side runs in libsplat_b200.so on the GPU: binning (toy2d/gs2d/binning.py:35-88),
forward (toy2d/csrc/rasterize.cu:366-394), backward_pixel (:396-417) and backward_splat (:419-448).
The activation of the learnable parameters stays in PyTorch autograd, as in the reference
(toy2d/gs2d/params.py:35-59). backend="ref" (the reference's dense PyTorch renderer) is not offered:
this package has no CPU path.
"""
from __future__ import annotations

import math
from dataclasses import dataclass

import torch

from . import _lib as L

TILE = 16     # tile side in pixels
BUCKET = 32   # splats per bucket of the per-splat backward
BLOCK = TILE * TILE


@dataclass
class Bins:
    """Tile lists and bucket tables (toy2d/gs2d/binning.py:16-33)."""

    H: int
    W: int
    tiles_x: int
    tiles_y: int
    rect: torch.Tensor            # (N, 4) int32 xmin, ymin, xmax, ymax in tiles (max exclusive)
    order: torch.Tensor           # (N,) int64 Gaussian ids, front to back
    point_list: torch.Tensor      # (M,) int32 Gaussian id per (tile, Gaussian) pair, tile-major, depth-sorted
    ranges: torch.Tensor          # (T, 2) int32 [start, end) into point_list per tile
    bucket_offsets: torch.Tensor  # (T,) int32 first bucket of each tile
    bucket_to_tile: torch.Tensor  # (B,) int32 tile of each bucket
    num_buckets: int
    # bounded binning (bin_gaussians with a capacity): int32 [1] on the device, 1 if the instances exceeded the
    # capacity (the list is then empty); None for exact binning
    overflow: torch.Tensor | None = None

    def check(self) -> None:
        """Bounded binning: raise if the instances exceeded the capacity (one host read; exact binning: no-op)."""
        if self.overflow is not None and int(self.overflow.item()):
            raise RuntimeError("bin_gaussians: the (tile, Gaussian) instances exceeded the capacity; the tile lists "
                               "were left empty - bin again with a larger capacity")

    def to(self, device):
        kw = {k: (v.to(device) if torch.is_tensor(v) else v) for k, v in self.__dict__.items()}
        return Bins(**kw)


class Gaussians2D(torch.nn.Module):
    """Learnable 2D Gaussians (toy2d/gs2d/params.py:17-32): same parameters and seeded init."""

    def __init__(self, n: int, H: int, W: int, seed: int = 0, dtype=torch.float32):
        super().__init__()
        g = torch.Generator().manual_seed(seed)
        spacing = math.sqrt(H * W / n) * 0.5
        self.xy = torch.nn.Parameter(torch.rand(n, 2, generator=g, dtype=dtype) * torch.tensor([W, H], dtype=dtype))
        self.log_scale = torch.nn.Parameter(torch.log(spacing * (0.5 + torch.rand(n, 2, generator=g, dtype=dtype))))
        self.theta = torch.nn.Parameter(torch.rand(n, generator=g, dtype=dtype) * math.pi)
        self.rgb_logit = torch.nn.Parameter(0.5 * torch.randn(n, 3, generator=g, dtype=dtype))
        self.opacity_logit = torch.nn.Parameter(0.5 * torch.randn(n, generator=g, dtype=dtype))
        self.register_buffer("depth", torch.rand(n, generator=g, dtype=dtype))

    def activated(self):
        return activate(self.xy, self.log_scale, self.theta, self.rgb_logit, self.opacity_logit)


def activate(xy, log_scale, theta, rgb_logit, opacity_logit):
    """(means, conic, color, opacity, cov) from the learnable parameters (toy2d/gs2d/params.py:35-48).

    cov = R diag(s^2) R^T with R the rotation by theta; conic = cov^-1 as (A, B, C)."""
    var = torch.exp(2.0 * log_scale)
    cos, sin = torch.cos(theta), torch.sin(theta)
    vx, vy = var[:, 0], var[:, 1]
    cxx = cos * cos * vx + sin * sin * vy
    cxy = cos * sin * (vx - vy)
    cyy = sin * sin * vx + cos * cos * vy
    det = cxx * cyy - cxy * cxy
    conic = torch.stack([cyy / det, -cxy / det, cxx / det], dim=-1)
    return xy, conic, torch.sigmoid(rgb_logit), torch.sigmoid(opacity_logit), torch.stack([cxx, cxy, cyy], dim=-1)


@torch.no_grad()
def radii_from_cov(cov: torch.Tensor) -> torch.Tensor:
    """ceil(3 sqrt(lambda_max)) with the eigenvalue floor of 3DGS (toy2d/gs2d/params.py:52-59)."""
    cxx, cxy, cyy = cov.unbind(-1)
    det = cxx * cyy - cxy * cxy
    mid = 0.5 * (cxx + cyy)
    lam = mid + torch.sqrt(torch.clamp(mid * mid - det, min=0.1))
    r = torch.ceil(3.0 * torch.sqrt(lam))
    return torch.where(det > 0, r, torch.zeros_like(r)).to(torch.int32)


@torch.no_grad()
def bin_gaussians(means: torch.Tensor, radii: torch.Tensor, depth: torch.Tensor, H: int, W: int,
                  capacity: int | None = None) -> Bins:
    """Tile binning on the GPU; bit-identical to toy2d/gs2d/binning.py:35-88.

    Exact (capacity None): two host reads, as in the reference - the instance count (to size point_list) and the
    bucket count (to size the per-bucket state).
    Bounded (capacity = the most (tile, Gaussian) instances to hold): no host read. The buffers are sized from the
    capacity (point_list holds `capacity` entries, of which the tile ranges index the first M; bucket_to_tile and
    num_buckets the bound capacity // 32 + tiles + 1, the buckets past the count naming tile -1), the counts stay on
    the device, and the same tile lists and buckets result. If M exceeds the capacity the lists are left empty and
    Bins.overflow is set (Bins.check() raises). Nothing in this path waits on the device, so a training step that
    uses it can be captured in a CUDA graph."""
    L.check_cuda("means", means)
    dev = means.device
    n = int(means.shape[0])
    tiles_x, tiles_y = (W + TILE - 1) // TILE, (H + TILE - 1) // TILE
    T = tiles_x * tiles_y
    m = means.detach().float().contiguous()
    r = radii.to(device=dev, dtype=torch.int32).contiguous()
    d = depth.detach().to(dev)
    if d.dtype not in (torch.float32, torch.float64):
        d = d.double()
    d = d.contiguous()
    stream = L.stream_of(m)
    rect = torch.empty(n, 4, dtype=torch.int32, device=dev)
    order = torch.empty(n, dtype=torch.int64, device=dev)
    counts = torch.zeros(2, dtype=torch.int32, device=dev)
    cws = L.workspace(L.query("gs2d_bin_count_workspace_size", n), dev)
    L.call("gs2d_bin_count", L.ptr(m), L.ptr(r), L.ptr(d), int(d.dtype == torch.float64), n, H, W, L.ptr(rect),
           L.ptr(order), L.ptr(counts), L.ptr(cws), cws.numel(), stream)
    if capacity is not None:
        cap = int(capacity)
        if cap < 0 or cap >= 2 ** 31:
            raise ValueError(f"capacity {cap} out of range")
        cap_b = cap // BUCKET + T + 1
        fws = L.workspace(L.query("gs2d_bin_fill_workspace_size", cap, H, W), dev)
        point_list = torch.empty(max(cap, 1), dtype=torch.int32, device=dev)
        ranges = torch.empty(T, 2, dtype=torch.int32, device=dev)
        bucket_offsets = torch.empty(T, dtype=torch.int32, device=dev)
        bucket_to_tile = torch.empty(cap_b, dtype=torch.int32, device=dev)
        overflow = torch.zeros(1, dtype=torch.int32, device=dev)
        L.call("gs2d_bin_fill_bounded", L.ptr(rect), n, H, W, cap, L.ptr(counts), L.ptr(cws), cws.numel(), L.ptr(fws),
               fws.numel(), L.ptr(point_list), L.ptr(ranges), L.ptr(bucket_offsets), L.ptr(bucket_to_tile), cap_b,
               L.ptr(counts[1:]), L.ptr(overflow), stream)
        return Bins(H, W, tiles_x, tiles_y, rect, order, point_list[:cap] if cap else point_list[:0], ranges,
                    bucket_offsets, bucket_to_tile, cap_b, overflow)
    M = int(counts[0].item())
    fws = L.workspace(L.query("gs2d_bin_fill_workspace_size", M, H, W), dev)
    point_list = torch.empty(M, dtype=torch.int32, device=dev)
    ranges = torch.empty(T, 2, dtype=torch.int32, device=dev)
    bucket_offsets = torch.empty(T, dtype=torch.int32, device=dev)
    bucket_to_tile = torch.empty(M // BUCKET + T + 1, dtype=torch.int32, device=dev)
    L.call("gs2d_bin_fill", L.ptr(rect), n, H, W, M, L.ptr(cws), cws.numel(), L.ptr(fws), fws.numel(),
           L.ptr(point_list), L.ptr(ranges), L.ptr(bucket_offsets), L.ptr(bucket_to_tile), L.ptr(counts[1:]), stream)
    B = int(counts[1].item())
    L.check_device_waits(dev)
    return Bins(H, W, tiles_x, tiles_y, rect, order, point_list, ranges, bucket_offsets,
                bucket_to_tile[:B].clone(), B)


class _Ext:
    """The pybind module of toy2d/csrc/rasterize.cu:450-454, as a Python object over the C ABI."""

    @staticmethod
    def forward(means, conic, color, opacity, bg, ranges, point_list, bucket_offsets, num_buckets, H, W,
                save_buckets):
        for name, t in (("means", means), ("conic", conic), ("color", color), ("opacity", opacity)):
            L.check_cuda(name, t, torch.float32)
        for name, t in (("ranges", ranges), ("point_list", point_list), ("bucket_offsets", bucket_offsets)):
            L.check_cuda(name, t, torch.int32)
        dev = means.device
        H, W, num_buckets = int(H), int(W), int(num_buckets)
        bgd = bg.detach().to(device=dev, dtype=torch.float32).contiguous()
        out = torch.empty(3, H, W, dtype=torch.float32, device=dev)
        final_T = torch.empty(H, W, dtype=torch.float32, device=dev)
        n_contrib = torch.empty(H, W, dtype=torch.int32, device=dev)
        if save_buckets:
            bucket_state = torch.zeros(num_buckets, BLOCK, 4, dtype=torch.float32, device=dev)
        else:
            bucket_state = torch.empty(0, dtype=torch.float32, device=dev)
        L.call("gs2d_forward", L.ptr(means), L.ptr(conic), L.ptr(color), L.ptr(opacity), L.ptr(bgd), L.ptr(ranges),
               L.ptr(point_list), L.ptr(bucket_offsets), int(means.shape[0]), int(point_list.numel()), num_buckets, H, W,
               int(bool(save_buckets)), L.ptr(out),
               L.ptr(final_T), L.ptr(n_contrib), L.ptr(bucket_state) if save_buckets else None, L.stream_of(means))
        return [out, final_T, n_contrib, bucket_state]

    @staticmethod
    def backward_pixel(means, conic, color, opacity, bg, ranges, point_list, final_T, n_contrib, dL_dout):
        L.check_cuda("dL_dout", dL_dout, torch.float32)
        L.check_cuda("final_T", final_T, torch.float32)
        L.check_cuda("n_contrib", n_contrib, torch.int32)
        H, W = int(final_T.shape[0]), int(final_T.shape[1])
        n = int(means.shape[0])
        dev = means.device
        bgd = bg.detach().to(device=dev, dtype=torch.float32).contiguous()
        g = [torch.empty_like(means), torch.empty_like(conic), torch.empty_like(color), torch.empty_like(opacity)]
        L.call("gs2d_backward_pixel", L.ptr(means), L.ptr(conic), L.ptr(color), L.ptr(opacity), L.ptr(bgd),
               L.ptr(ranges), L.ptr(point_list), n, int(point_list.numel()), H, W, L.ptr(final_T), L.ptr(n_contrib),
               L.ptr(dL_dout),
               *map(L.ptr, g), L.stream_of(means))
        return g

    @staticmethod
    def backward_splat(means, conic, color, opacity, bg, ranges, point_list, bucket_offsets, bucket_to_tile, out,
                       final_T, n_contrib, bucket_state, dL_dout):
        L.check_cuda("dL_dout", dL_dout, torch.float32)
        L.check_cuda("out", out, torch.float32)
        L.check_cuda("bucket_state", bucket_state, torch.float32)
        L.check_cuda("bucket_to_tile", bucket_to_tile, torch.int32)
        H, W = int(final_T.shape[0]), int(final_T.shape[1])
        n = int(means.shape[0])
        nb = int(bucket_to_tile.shape[0])
        g = [torch.empty_like(means), torch.empty_like(conic), torch.empty_like(color), torch.empty_like(opacity)]
        L.call("gs2d_backward_splat", L.ptr(means), L.ptr(conic), L.ptr(color), L.ptr(opacity), L.ptr(ranges),
               L.ptr(point_list), L.ptr(bucket_offsets), L.ptr(bucket_to_tile), nb, n, int(point_list.numel()), H, W,
               L.ptr(out),
               L.ptr(n_contrib), L.ptr(bucket_state) if nb else None, L.ptr(dL_dout), *map(L.ptr, g),
               L.stream_of(means))
        return g


_EXT = _Ext()


def ext() -> _Ext:
    """Stands in for toy2d/gs2d/raster.py:17-26 `ext()` (no JIT build: the library is prebuilt)."""
    L.load()
    return _EXT


class _Rasterize(torch.autograd.Function):
    """toy2d/gs2d/raster.py:29-53, over the C ABI."""

    @staticmethod
    def forward(ctx, means, conic, color, opacity, bg, bins: Bins, mode: str):
        save = mode == "splat"
        out, final_T, n_contrib, bstate = ext().forward(
            means.contiguous(), conic.contiguous(), color.contiguous(), opacity.contiguous(), bg, bins.ranges,
            bins.point_list, bins.bucket_offsets, bins.num_buckets, bins.H, bins.W, save)
        ctx.bins, ctx.mode = bins, mode
        ctx.save_for_backward(means, conic, color, opacity, bg, out, final_T, n_contrib, bstate)
        return out

    @staticmethod
    def backward(ctx, dout):
        means, conic, color, opacity, bg, out, final_T, n_contrib, bstate = ctx.saved_tensors
        b = ctx.bins
        dout = dout.contiguous().float()
        args = (means.contiguous(), conic.contiguous(), color.contiguous(), opacity.contiguous(), bg)
        if ctx.mode == "pixel":
            g = ext().backward_pixel(*args, b.ranges, b.point_list, final_T, n_contrib, dout)
        else:
            g = ext().backward_splat(*args, b.ranges, b.point_list, b.bucket_offsets, b.bucket_to_tile, out, final_T,
                                     n_contrib, bstate, dout)
        dmeans, dconic, dcolor, dopacity = g
        return dmeans, dconic, dcolor, dopacity, None, None, None


def rasterize(means, conic, color, opacity, bins: Bins, bg=None, backend: str = "splat"):
    """Render a (3, H, W) image (toy2d/gs2d/raster.py:56-64); backend 'pixel' or 'splat'."""
    if bg is None:
        bg = torch.zeros(3, dtype=means.dtype, device=means.device)
    if backend == "ref":
        raise ValueError("backend 'ref' is the reference's dense PyTorch renderer; this package renders on the "
                         "GPU only (backend 'pixel' or 'splat')")
    if backend not in ("pixel", "splat"):
        raise ValueError(f"unknown backend {backend!r}")
    return _Rasterize.apply(means, conic, color, opacity, bg, bins, backend)
