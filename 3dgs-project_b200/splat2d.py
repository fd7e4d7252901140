"""Drop-in for phase0's ``splat2d.ops`` (phase0/splat2d/ops.py): same names, same arguments.

    from gs_b200.splat2d import render, bin_tiles, load_extension
    image = render(means, chol, opacity_logit, colors, H, W, mode="splat")   # [H, W, 3]

float32 and float64 parameters are both supported (bindings.cpp:170 dispatches on the dtype).
Binning (ops.py:206-255) runs on the GPU in float64 like the reference's CPU loop; forward,
backward_pixel and backward_splat run in libsplat_b200.so. There is no CPU build: CPU tensors raise.
The pure-PyTorch ground truth ``ref_render`` / ``ref_state`` (ops.py:358-398) is test infrastructure
and lives with the oracle, not here.
"""
from __future__ import annotations

import ctypes
from collections.abc import Callable
from dataclasses import dataclass
from typing import Any, Literal, Protocol, cast

import torch
from torch import Tensor

from . import _lib as L

Mode = Literal["pixel", "splat"]
MODES: tuple[Mode, ...] = ("pixel", "splat")

TILE = 16
TILE_PIXELS = TILE * TILE
BUCKET = 32
NUM_PARAMS = 9
CKPT_STRIDE = 4
ALPHA_MIN = 1.0 / 255.0
ALPHA_MAX = 0.99
T_STOP = 1e-4


class Extension(Protocol):
    """Typed view of the extension object (ops.py:48-101)."""

    def forward(self, means: Tensor, chol: Tensor, opacity_logit: Tensor, colors: Tensor, tile_offsets: Tensor,
                tile_ids: Tensor, bucket_offsets: Tensor, bucket_tile: Tensor, height: int,
                width: int) -> list[Tensor]: ...

    def backward_pixel(self, grad_image: Tensor, means: Tensor, chol: Tensor, opacity_logit: Tensor, colors: Tensor,
                       tile_offsets: Tensor, tile_ids: Tensor, bucket_offsets: Tensor, bucket_tile: Tensor,
                       t_final: Tensor, last_contrib: Tensor, height: int, width: int) -> list[Tensor]: ...

    def backward_splat(self, grad_image: Tensor, means: Tensor, chol: Tensor, opacity_logit: Tensor, colors: Tensor,
                       tile_offsets: Tensor, tile_ids: Tensor, bucket_offsets: Tensor, bucket_tile: Tensor,
                       image: Tensor, ckpt: Tensor, height: int, width: int) -> list[Tensor]: ...

    def get_counters(self) -> dict[str, int]: ...

    def reset_counters(self) -> None: ...


def _check_scene(means, chol, opacity_logit, colors, tables, height, width):
    """bindings.cpp:50-84 (make_scene): shapes, one floating dtype, int32 tables, one device, non-empty image."""
    if means.dim() != 2 or means.shape[1] != 2:
        raise RuntimeError("means must be [N, 2]")
    n = means.shape[0]
    if tuple(chol.shape) != (n, 3):
        raise RuntimeError("chol must be [N, 3]")
    if tuple(opacity_logit.shape) != (n,):
        raise RuntimeError("opacity_logit must be [N]")
    if tuple(colors.shape) != (n, 3):
        raise RuntimeError("colors must be [N, 3]")
    if not (chol.dtype == opacity_logit.dtype == colors.dtype == means.dtype):
        raise RuntimeError("all splat parameters must share one floating dtype")
    if means.dtype not in (torch.float32, torch.float64):
        raise RuntimeError("splat parameters must be float32 or float64")
    for t in tables:
        if t.dtype != torch.int32:
            raise RuntimeError("tile/bucket tables must be int32")
    if height <= 0 or width <= 0:
        raise RuntimeError("image must be non-empty")
    for t in (chol, opacity_logit, colors, *tables):
        if t.device != means.device:
            raise RuntimeError("all inputs must be on the same device as means")
    if not means.is_cuda:
        raise RuntimeError("splat2d on this package is GPU-only: means must be a CUDA tensor")
    T = ((width + TILE - 1) // TILE) * ((height + TILE - 1) // TILE)
    if tables[0].numel() != T + 1:
        raise RuntimeError("tile_offsets has the wrong length")
    if tables[2].numel() != T + 1:
        raise RuntimeError("bucket_offsets has the wrong length")
    return [t.contiguous() for t in (means, chol, opacity_logit, colors)], [t.contiguous() for t in tables]


class _CudaExtension:
    """The GPU extension object: forward, backward_pixel, backward_splat, get/reset_counters."""

    def forward(self, means, chol, opacity_logit, colors, tile_offsets, tile_ids, bucket_offsets, bucket_tile,
                height, width):
        (m, c, z, col), tabs = _check_scene(means, chol, opacity_logit, colors,
                                            (tile_offsets, tile_ids, bucket_offsets, bucket_tile), height, width)
        H, W = int(height), int(width)
        opts = dict(dtype=m.dtype, device=m.device)
        # the kernel writes every pixel of these four (one thread per pixel of every tile), so no fill is needed
        image = torch.empty(H, W, 3, **opts)
        t_final = torch.empty(H, W, **opts)
        n_contrib = torch.empty(H, W, dtype=torch.int32, device=m.device)
        last_contrib = torch.empty(H, W, dtype=torch.int32, device=m.device)
        B = int(tabs[3].numel())
        ckpt = torch.empty(B, TILE_PIXELS, CKPT_STRIDE, **opts)
        L.call("splat2d_forward", int(m.dtype == torch.float64), L.ptr(m), L.ptr(c), L.ptr(z), L.ptr(col),
               *map(L.ptr, tabs), int(m.shape[0]), int(tabs[1].numel()), B, H, W, L.ptr(image), L.ptr(t_final),
               L.ptr(n_contrib), L.ptr(last_contrib), L.ptr(ckpt), L.stream_of(m))
        return [image, t_final, n_contrib, last_contrib, ckpt]

    def _backward(self, splat_mode, grad_image, means, chol, opacity_logit, colors, tables, height, width,
                  t_final=None, last_contrib=None, image=None, ckpt=None):
        (m, c, z, col), tabs = _check_scene(means, chol, opacity_logit, colors, tables, height, width)
        H, W = int(height), int(width)
        g_img = grad_image.contiguous().to(m.dtype)
        if tuple(g_img.shape) != (H, W, 3):
            raise RuntimeError("grad_image must be [H, W, 3]")
        B = int(tabs[3].numel())
        if splat_mode:
            if ckpt.shape[0] != B:
                raise RuntimeError("ckpt must have one slot per bucket")
            image, ckpt = image.contiguous(), ckpt.contiguous()
        else:
            if last_contrib.dtype != torch.int32:
                raise RuntimeError("last_contrib must be int32")
            t_final, last_contrib = t_final.contiguous(), last_contrib.contiguous()
        grads = [torch.empty_like(m), torch.empty_like(c), torch.empty_like(z), torch.empty_like(col)]
        L.call("splat2d_backward", int(m.dtype == torch.float64), int(splat_mode), L.ptr(g_img), L.ptr(m), L.ptr(c),
               L.ptr(z), L.ptr(col), *map(L.ptr, tabs), int(m.shape[0]), int(tabs[1].numel()), B, H, W,
               L.ptr(t_final), L.ptr(last_contrib), L.ptr(image), L.ptr(ckpt) if B else None, *map(L.ptr, grads),
               L.stream_of(m))
        return grads

    def backward_pixel(self, grad_image, means, chol, opacity_logit, colors, tile_offsets, tile_ids, bucket_offsets,
                       bucket_tile, t_final, last_contrib, height, width):
        return self._backward(0, grad_image, means, chol, opacity_logit, colors,
                              (tile_offsets, tile_ids, bucket_offsets, bucket_tile), height, width,
                              t_final=t_final, last_contrib=last_contrib)

    def backward_splat(self, grad_image, means, chol, opacity_logit, colors, tile_offsets, tile_ids, bucket_offsets,
                       bucket_tile, image, ckpt, height, width):
        return self._backward(1, grad_image, means, chol, opacity_logit, colors,
                              (tile_offsets, tile_ids, bucket_offsets, bucket_tile), height, width, image=image,
                              ckpt=ckpt)

    def get_counters(self) -> dict[str, int]:
        out = (ctypes.c_longlong * 3)()
        L.call("splat2d_get_counters", ctypes.addressof(out))
        return {"atomic_adds": int(out[0]), "checkpoint_bytes": int(out[1]), "splat_pixel_evals": int(out[2])}

    def reset_counters(self) -> None:
        """Zero the counters and start counting (counting costs a few percent, so it starts off)."""
        L.call("splat2d_reset_counters")
        L.call("splat2d_set_counting", 1)

    def stop_counting(self) -> None:
        L.call("splat2d_set_counting", 0)


_EXT = _CudaExtension()


def load_extension(with_cuda: bool | None = None, verbose: bool = False) -> Extension:
    """ops.py:155-182. Only the CUDA build exists here; with_cuda=False raises."""
    if with_cuda is False:
        raise RuntimeError("this package has no CPU build of splat2d (GPU only)")
    L.load()
    return cast(Extension, _EXT)


def _ext_for(t: Tensor) -> Extension:
    if not t.is_cuda:
        raise RuntimeError("splat2d on this package is GPU-only: inputs must be CUDA tensors")
    return load_extension(with_cuda=True)


@dataclass(frozen=True)
class TileBins:
    """CSR tile lists (splat ids in list order) and the 32-splat bucket tables (ops.py:190-203)."""

    tile_offsets: Tensor  # int32 [num_tiles + 1]
    tile_ids: Tensor  # int32 [tile_offsets[-1]]
    bucket_offsets: Tensor  # int32 [num_tiles + 1]
    bucket_tile: Tensor  # int32 [num_buckets]
    tiles_x: int
    tiles_y: int

    @property
    def num_buckets(self) -> int:
        return int(self.bucket_tile.numel())


@torch.no_grad()
def bin_tiles(means: Tensor, chol: Tensor, opacity_logit: Tensor, height: int, width: int) -> TileBins:
    """Tiles hit by the exact bounding box of each splat's alpha >= 1/255 ellipse, one pixel of slack on
    each side (ops.py:206-255); float64 arithmetic on the GPU, lists in ascending splat id per tile."""
    L.check_cuda("means", means)
    dev = means.device
    dt = means.dtype if means.dtype in (torch.float32, torch.float64) else torch.float64
    m, c, z = (t.detach().to(dt).contiguous() for t in (means, chol, opacity_logit))
    n = int(m.shape[0])
    tiles_x, tiles_y = (width + TILE - 1) // TILE, (height + TILE - 1) // TILE
    T = tiles_x * tiles_y
    stream = L.stream_of(m)
    counts = torch.zeros(2, dtype=torch.int32, device=dev)
    cws = L.workspace(L.query("splat2d_bin_count_workspace_size", n), dev)
    L.call("splat2d_bin_count", int(dt == torch.float64), L.ptr(m), L.ptr(c), L.ptr(z), n, height, width,
           L.ptr(counts), L.ptr(cws), cws.numel(), stream)
    M = int(counts[0].item())
    fws = L.workspace(L.query("splat2d_bin_fill_workspace_size", M, height, width), dev)
    tile_offsets = torch.empty(T + 1, dtype=torch.int32, device=dev)
    tile_ids = torch.empty(M, dtype=torch.int32, device=dev)
    bucket_offsets = torch.empty(T + 1, dtype=torch.int32, device=dev)
    bucket_tile = torch.empty(M // BUCKET + T + 1, dtype=torch.int32, device=dev)
    L.call("splat2d_bin_fill", n, height, width, M, L.ptr(cws), cws.numel(), L.ptr(fws), fws.numel(),
           L.ptr(tile_offsets), L.ptr(tile_ids), L.ptr(bucket_offsets), L.ptr(bucket_tile), L.ptr(counts[1:]), stream)
    B = int(counts[1].item())
    L.check_device_waits(dev)
    return TileBins(tile_offsets, tile_ids, bucket_offsets, bucket_tile[:B].clone(), tiles_x, tiles_y)


class _Splat2dFunction(torch.autograd.Function):
    """ops.py:258-325 over the C ABI."""

    @staticmethod
    def forward(ctx: Any, means, chol, opacity_logit, colors, bins: TileBins, height: int, width: int, mode: Mode):
        ext = _ext_for(means)
        image, t_final, _n, last_contrib, ckpt = ext.forward(means, chol, opacity_logit, colors, bins.tile_offsets,
                                                             bins.tile_ids, bins.bucket_offsets, bins.bucket_tile,
                                                             height, width)
        ctx.save_for_backward(means, chol, opacity_logit, colors, image, t_final, last_contrib, ckpt)
        ctx.bins, ctx.height, ctx.width, ctx.mode = bins, height, width, mode
        return image

    @staticmethod
    def backward(ctx: Any, grad_image: Tensor):
        means, chol, opacity_logit, colors, image, t_final, last_contrib, ckpt = ctx.saved_tensors
        bins: TileBins = ctx.bins
        ext = _ext_for(means)
        tables = (bins.tile_offsets, bins.tile_ids, bins.bucket_offsets, bins.bucket_tile)
        if ctx.mode == "pixel":
            g = ext.backward_pixel(grad_image, means, chol, opacity_logit, colors, *tables, t_final, last_contrib,
                                   ctx.height, ctx.width)
        else:
            g = ext.backward_splat(grad_image, means, chol, opacity_logit, colors, *tables, image, ckpt, ctx.height,
                                   ctx.width)
        return g[0], g[1], g[2], g[3], None, None, None, None


def render(means: Tensor, chol: Tensor, opacity_logit: Tensor, colors: Tensor, height: int, width: int,
           mode: Mode = "splat", depths: Tensor | None = None) -> Tensor:
    """Render an [H, W, 3] image (ops.py:328-347). Splats are taken in index order unless ``depths``."""
    if mode not in MODES:
        raise ValueError(f"mode must be one of {MODES}, got {mode!r}")
    if depths is not None:
        order = torch.argsort(depths, stable=True)
        means, chol = means[order], chol[order]
        opacity_logit, colors = opacity_logit[order], colors[order]
    bins = bin_tiles(means, chol, opacity_logit, height, width)
    apply = cast(Callable[..., Tensor], _Splat2dFunction.apply)
    return apply(means, chol, opacity_logit, colors, bins, height, width, mode)
