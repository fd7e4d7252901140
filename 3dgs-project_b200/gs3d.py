"""3DGS rasterization over libsplat_b200.so, shaped like the reference's 3DGS boundary.

Faster-GS-compatible (the calls of phase1/tests/test_parity.py:82-98 and cluster/tests/test_lean_adam.py:109-123):
    image, prim_buf, tile_buf, inst_buf, bucket_buf, n_instances, n_buckets, selector = forward(
        means, scales, rotations, opacities, sh0, sh_rest, *settings.as_tuple())
    grads = backward(densification_info, grad_image, image, means, scales, rotations, opacities, sh_rest,
                     prim_buf, tile_buf, inst_buf, bucket_buf, *settings.as_tuple(), n_instances, n_buckets, selector)
    image = diff_rasterize(means, scales, rotations, opacities, sh0, sh_rest, densification_info, settings)
graphdeco-style (requested by the benchmark spec): rasterize_gaussians(means3D, scales, rotations, opacities, shs,
    viewmatrix, projmatrix, ...) with activated inputs, mapped onto the same kernels.

The rasterization rules are Faster-GS's (alpha = opacity * G with no 0.99 clamp, a pixel stops after the splat that
drops T below 1e-4, (1 - alpha) floored at 1e-6 in the backward); they are listed in csrc/gs3d_common.cuh.
One host read per forward (the instance count, to size the instance buffer), taken while the device sorts the Gaussians
by depth, so the device does not wait for it; the bucket buffer is sized by a bound and ``n_buckets`` returns that
bound, as phase2/tests/test_readback_equiv.py:100-104 allows.
"""
from __future__ import annotations

import ctypes
import math
import threading
from typing import Any, NamedTuple

import torch

from . import _lib as L

TILE = 16


class _Settings(ctypes.Structure):
    """Mirror of gs3d_settings in include/splat_b200.h."""

    _fields_ = [("w2c", ctypes.c_void_p), ("cam_position", ctypes.c_void_p), ("bg", ctypes.c_void_p),
                ("active_sh_bases", ctypes.c_int), ("rest_bases", ctypes.c_int), ("width", ctypes.c_int),
                ("height", ctypes.c_int), ("fx", ctypes.c_float), ("fy", ctypes.c_float), ("cx", ctypes.c_float),
                ("cy", ctypes.c_float), ("near_plane", ctypes.c_float), ("far_plane", ctypes.c_float),
                ("proper_antialiasing", ctypes.c_int)]


class _AdamState(ctypes.Structure):
    """Mirror of gs3d_adam_state in include/splat_b200.h."""

    _fields_ = [("exp_avg", ctypes.c_void_p * 6), ("exp_avg_sq", ctypes.c_void_p * 6),
                ("grad_in", ctypes.c_void_p * 6), ("lr", ctypes.c_double * 6), ("step", ctypes.c_int * 6),
                ("beta1", ctypes.c_double), ("beta2", ctypes.c_double), ("eps", ctypes.c_double)]


class RasterizerSettings(NamedTuple):
    """Faster-GS's RasterizerSettings (field names as used in cluster/tests/test_lean_adam.py:119-121)."""

    w2c: torch.Tensor
    cam_position: torch.Tensor
    bg_color: torch.Tensor
    active_sh_bases: int
    width: int
    height: int
    focal_x: float
    focal_y: float
    center_x: float
    center_y: float
    near_plane: float
    far_plane: float
    proper_antialiasing: bool

    def as_tuple(self) -> tuple:
        return tuple(self)


def _settings(dev, w2c, cam_position, bg, active_sh_bases, width, height, fx, fy, cx, cy, near, far, aa, rest_bases,
              keep: list):
    w2c = w2c.detach().to(device=dev, dtype=torch.float32).contiguous()
    cam = cam_position.detach().to(device=dev, dtype=torch.float32).contiguous()
    bgd = bg.detach().to(device=dev, dtype=torch.float32).contiguous()
    if w2c.numel() != 16 or cam.numel() != 3 or bgd.numel() != 3:
        raise RuntimeError("w2c must be [4, 4], cam_position and bg_color [3]")
    keep += [w2c, cam, bgd]
    return _Settings(w2c.data_ptr(), cam.data_ptr(), bgd.data_ptr(), int(active_sh_bases), int(rest_bases),
                     int(width), int(height), float(fx), float(fy), float(cx), float(cy), float(near), float(far),
                     int(bool(aa)))


def _check_params(means, scales, rotations, opacities, sh0, sh_rest):
    n = means.shape[0]
    shapes = {"means": (means, (n, 3)), "scales": (scales, (n, 3)), "rotations": (rotations, (n, 4))}
    for name, (t, shp) in shapes.items():
        L.check_cuda(name, t, torch.float32)
        if tuple(t.shape) != shp:
            raise RuntimeError(f"{name} must be {list(shp)}, got {list(t.shape)}")
    for name, t in (("opacities", opacities), ("sh0", sh0), ("sh_rest", sh_rest)):
        L.check_cuda(name, t, torch.float32)
    if opacities.numel() != n:
        raise RuntimeError("opacities must hold N values")
    if sh0.numel() != 3 * n:
        raise RuntimeError("sh0 must be [N, 1, 3]")
    if sh_rest.numel() % (3 * max(n, 1)) != 0 or (n and sh_rest.shape[0] != n):
        raise RuntimeError("sh_rest must be [N, rest_bases, 3]")
    return n, (sh_rest.numel() // (3 * n) if n else 0)


_readback = threading.local()


def _readback_slot(dev):
    """(pinned int32[2], stream, event, event) of this host thread and device for the forward's one read: the copy
    runs on its own stream, so the compute stream goes on with the depth order instead of waiting for the copy
    engine. A forward waits on its read before it returns, so one slot per thread and device is never in use twice
    at a time."""
    slots = getattr(_readback, "slots", None)
    if slots is None:
        slots = _readback.slots = {}
    key = dev.index if dev.index is not None else torch.cuda.current_device()
    if key not in slots:
        slots[key] = (torch.empty(2, dtype=torch.int32, pin_memory=True), torch.cuda.Stream(key), torch.cuda.Event(),
                      torch.cuda.Event())
    return slots[key]


def _preprocess(means, scales, rotations, opacities, sh0, sh_rest, settings_args, read_count: bool = True):
    """Preprocess and depth order of one view; returns M read back from the device, or None (read_count False: no
    host read, the bounded render reads M on the device)."""
    n, rest = _check_params(means, scales, rotations, opacities, sh0, sh_rest)
    dev = means.device
    keep: list = []
    s = _settings(dev, *settings_args, rest, keep)
    stream = L.stream_of(means)
    width, height = settings_args[4], settings_args[5]
    prim = torch.empty(L.query("gs3d_primitive_buffer_size", n), dtype=torch.uint8, device=dev)
    tile = torch.empty(L.query("gs3d_tile_buffer_size", width, height), dtype=torch.uint8, device=dev)
    count = torch.empty(2, dtype=torch.int32, device=dev)
    L.call("gs3d_preprocess_count", L.ptr(means), L.ptr(scales), L.ptr(rotations), L.ptr(opacities), L.ptr(sh0),
           L.ptr(sh_rest), n, ctypes.byref(s), L.ptr(prim), prim.numel(), L.ptr(count), stream)
    if not read_count:
        L.call("gs3d_preprocess_order", n, L.ptr(prim), prim.numel(), stream)
        return n, dev, s, keep, stream, prim, tile, None
    # the device's count of look-back waits that gave up (the sorts of the forwards before this one)
    L.call("splat_take_device_waits_async", L.ptr(count[1:]), stream)
    host, side, ready, counted = _readback_slot(dev)
    ready.record(torch.cuda.current_stream(dev))
    with torch.cuda.stream(side):
        side.wait_event(ready)
        host.copy_(count, non_blocking=True)
        counted.record(side)
    # the depth order runs on the device while the host waits for M (the one host read of a forward)
    L.call("gs3d_preprocess_order", n, L.ptr(prim), prim.numel(), stream)
    counted.synchronize()
    m, waits = host.tolist()
    if waits:
        raise RuntimeError(f"{waits} bounded device-side wait(s) in the radix sort gave up: the device stalled (the "
                           f"sorts recounted their offsets and stayed exact)")
    return n, dev, s, keep, stream, prim, tile, m


@torch.no_grad()
def inference(means, scales, rotations, opacities, sh0, sh_rest, w2c, cam_position, bg_color, active_sh_bases,
              width, height, focal_x, focal_y, center_x, center_y, near_plane, far_plane, proper_antialiasing):
    """Faster-GS `_C.inference`: the image [3, H, W] alone (render-only path: no buffers for a backward)."""
    n, dev, s, keep, stream, prim, tile, m = _preprocess(
        means, scales, rotations, opacities, sh0, sh_rest,
        (w2c, cam_position, bg_color, active_sh_bases, width, height, focal_x, focal_y, center_x, center_y,
         near_plane, far_plane, proper_antialiasing))
    inst = torch.empty(L.query("gs3d_instance_buffer_size", m), dtype=torch.uint8, device=dev)
    image = torch.empty(3, height, width, dtype=torch.float32, device=dev)
    L.call("gs3d_render_inference", n, m, ctypes.byref(s), L.ptr(prim), prim.numel(), L.ptr(tile), tile.numel(),
           L.ptr(inst), inst.numel(), L.ptr(image), stream)
    return image


@torch.no_grad()
def forward(means, scales, rotations, opacities, sh0, sh_rest, w2c, cam_position, bg_color, active_sh_bases, width,
            height, focal_x, focal_y, center_x, center_y, near_plane, far_plane, proper_antialiasing, *,
            capacity: int | None = None, overflow: torch.Tensor | None = None):
    """Faster-GS `_C.forward`: (image[3,H,W], prim_buf, tile_buf, inst_buf, bucket_buf, n_instances, n_buckets, 0).

    capacity (keyword, no counterpart in the reference): the bounded form, with no host read - buffers sized for
    `capacity` instances, M read on the device (gs3d_render_bounded), n_instances returned as the capacity (which
    the backward takes as it is). If M exceeds it, overflow (device int32 [1], required) is set to 1 and the image
    lists only the first `capacity` instances; check it where a host read is acceptable."""
    n, dev, s, keep, stream, prim, tile, m = _preprocess(
        means, scales, rotations, opacities, sh0, sh_rest,
        (w2c, cam_position, bg_color, active_sh_bases, width, height, focal_x, focal_y, center_x, center_y,
         near_plane, far_plane, proper_antialiasing), read_count=capacity is None)
    if capacity is not None:
        if overflow is None:
            raise RuntimeError("the bounded forward needs an overflow word (device int32 [1])")
        L.check_cuda("overflow", overflow, torch.int32)
        m = int(capacity)
        bcap = int(L.load().gs3d_bucket_bound(m, width, height))
        inst = torch.empty(L.query("gs3d_instance_buffer_size", m), dtype=torch.uint8, device=dev)
        bucket = torch.empty(L.query("gs3d_bucket_buffer_size", bcap), dtype=torch.uint8, device=dev)
        image = torch.empty(3, height, width, dtype=torch.float32, device=dev)
        L.call("gs3d_render_bounded", n, m, ctypes.byref(s), L.ptr(prim), prim.numel(), L.ptr(tile), tile.numel(),
               L.ptr(inst), inst.numel(), L.ptr(bucket), bucket.numel(), bcap, L.ptr(image), L.ptr(overflow), stream)
        return image, prim, tile, inst, bucket, m, bcap, 0
    bcap = int(L.load().gs3d_bucket_bound(m, width, height))
    inst = torch.empty(L.query("gs3d_instance_buffer_size", m), dtype=torch.uint8, device=dev)
    bucket = torch.empty(L.query("gs3d_bucket_buffer_size", bcap), dtype=torch.uint8, device=dev)
    image = torch.empty(3, height, width, dtype=torch.float32, device=dev)
    L.call("gs3d_render", n, m, ctypes.byref(s), L.ptr(prim), prim.numel(), L.ptr(tile), tile.numel(), L.ptr(inst),
           inst.numel(), L.ptr(bucket), bucket.numel(), bcap, L.ptr(image), stream)
    return image, prim, tile, inst, bucket, m, bcap, 0


@torch.no_grad()
def backward(densification_info, grad_image, image, means, scales, rotations, opacities, sh_rest, prim_buf,
             tile_buf, inst_buf, bucket_buf, w2c, cam_position, bg_color, active_sh_bases, width, height, focal_x,
             focal_y, center_x, center_y, near_plane, far_plane, proper_antialiasing, n_instances, n_buckets,
             selector, *mode, out: tuple | None = None, stage_event: torch.cuda.Event | None = None,
             accumulate: bool = False, records: torch.Tensor | None = None):
    """Faster-GS `_C.backward` (the trailing blend-backward mode of the phase1 patch is accepted and ignored:
    there is one blend backward here). Returns (means, scales, rotations, opacities[N,1], sh0[N,1,3], sh_rest) and
    accumulates densification_info ([0 | 2 | 3, N]) in place: visible count, |dL/dmean2d| in normalised device
    units, and with three rows the norm of the summed per-pixel absolute mean2d gradients.
    ``out`` may supply the six contiguous float32 result tensors (e.g. views of one flat gradient buffer);
    with ``accumulate`` the gradients are added into them (the views of one batch into one buffer).
    It runs as its two launches (gs3d_backward_blend, gs3d_backward_preprocess); ``stage_event``, if given, is
    recorded on the stream between them. ``records`` (with ``out`` holding the four non-SH gradient tensors): the
    compact exchange's form, PendingBackward.preprocess_records; returns None."""
    pending = backward_blend(densification_info, grad_image, image, means, scales, rotations, opacities, sh_rest,
                             prim_buf, tile_buf, inst_buf, bucket_buf, w2c, cam_position, bg_color, active_sh_bases,
                             width, height, focal_x, focal_y, center_x, center_y, near_plane, far_plane,
                             proper_antialiasing, n_instances, n_buckets, selector, defer_densification=True)
    if stage_event is not None:
        stage_event.record(torch.cuda.current_stream(means.device))
    if records is not None:
        if out is None:
            raise RuntimeError("records need the four non-SH gradient tensors in out")
        pending.preprocess_records(out, records, accumulate=accumulate)
        return None
    return pending.preprocess(out=out, accumulate=accumulate)


class PendingBackward:
    """One view's backward after its blend backward: the per-Gaussian 2D gradients sit in the workspace and the
    preprocess backward is still to run, either on its own (preprocess: the six parameter gradients) or fused with
    the Adam step of the six parameter tensors (preprocess_adam: the gradients are never stored)."""

    def __init__(self, ws, s, keep, prim_buf, tensors, n, rest, rows, dinfo, stream):
        self.ws, self.s, self.keep, self.prim = ws, s, keep, prim_buf
        self.means, self.scales, self.rotations, self.opacities, self.sh_rest = tensors
        self.n, self.rest, self.rows, self.dinfo, self.stream = n, rest, rows, dinfo, stream

    def preprocess(self, out: tuple | None = None, accumulate: bool = False) -> tuple:
        """The six parameter gradients (gs3d_backward_preprocess), with the densification rows when they were
        deferred to this call. accumulate (with ``out``): add them into ``out`` instead
        (gs3d_backward_preprocess_accumulate), as the views of one batch do."""
        if accumulate and out is None:
            raise RuntimeError("accumulate needs the out tensors to add into")
        n, rest, dev = self.n, self.rest, self.means.device
        if out is not None:
            grads = tuple(out)
            for t, numel in zip(grads, (3 * n, 3 * n, 4 * n, n, 3 * n, 3 * rest * n)):
                L.check_cuda("out", t, torch.float32)
                if t.numel() != numel:
                    raise RuntimeError("out tensors must match the parameter shapes")
        else:
            grads = (torch.empty(n, 3, device=dev), torch.empty(n, 3, device=dev), torch.empty(n, 4, device=dev),
                     torch.empty(n, 1, device=dev), torch.empty(n, 1, 3, device=dev),
                     torch.empty(n, rest, 3, device=dev))
        L.call("gs3d_backward_preprocess_accumulate" if accumulate else "gs3d_backward_preprocess",
               L.ptr(self.means), L.ptr(self.scales), L.ptr(self.rotations),
               L.ptr(self.opacities), L.ptr(self.sh_rest), n, ctypes.byref(self.s), L.ptr(self.prim),
               self.prim.numel(), L.ptr(self.ws), self.ws.numel(), *map(L.ptr, grads), L.ptr(self.dinfo), self.rows,
               self.stream)
        self.rows, self.dinfo = 0, None
        return grads

    def preprocess_records(self, out4, records: torch.Tensor, accumulate: bool = False) -> None:
        """The preprocess backward for the compact exchange (gs3d_backward_preprocess_records): the gradients of
        means, scales, rotations and opacities into ``out4`` (stored, or added with ``accumulate``), and in place of
        the SH gradients six floats per Gaussian into ``records`` (float32, 6n elements): the colour gradient where
        the colour clamp passes it, then the unit view direction; zeros for Gaussians this view does not see."""
        n = self.n
        out4 = tuple(out4)
        if len(out4) != 4:
            raise RuntimeError("four gradient tensors (means, scales, rotations, opacities) expected")
        for t, numel in zip(out4, (3 * n, 3 * n, 4 * n, n)):
            L.check_cuda("out", t, torch.float32)
            if t.numel() != numel:
                raise RuntimeError("out tensors must match the parameter shapes")
        L.check_cuda("records", records, torch.float32)
        if records.numel() != 6 * n:
            raise RuntimeError(f"records must hold 6 floats per Gaussian ({6 * n}), got {records.numel()}")
        L.call("gs3d_backward_preprocess_records", L.ptr(self.means), L.ptr(self.scales), L.ptr(self.rotations),
               L.ptr(self.opacities), L.ptr(self.sh_rest), n, ctypes.byref(self.s), L.ptr(self.prim),
               self.prim.numel(), L.ptr(self.ws), self.ws.numel(), *map(L.ptr, out4), L.ptr(records),
               int(bool(accumulate)), L.ptr(self.dinfo), self.rows, self.stream)
        self.rows, self.dinfo = 0, None

    def preprocess_adam(self, params, exp_avg, exp_avg_sq, lrs, steps, betas=(0.9, 0.999), eps: float = 1e-15,
                        grad_in=None) -> None:
        """The preprocess backward fused with one Adam step of the six parameter tensors (means, scales, rotations,
        opacities, sh0, sh_rest; updated in place with their moments): gs3d_backward_preprocess_adam. grad_in: per
        tensor, the gradient other loss terms already left (added first), or None. Bit-identical to preprocess()
        followed by FusedAdam's step over the same six tensors."""
        if self.rows:
            raise RuntimeError("densification rows were deferred to the preprocess backward; take them first")
        params = list(params)
        if len(params) != 6 or len(exp_avg) != 6 or len(exp_avg_sq) != 6 or len(lrs) != 6 or len(steps) != 6:
            raise RuntimeError("six parameter tensors (means, scales, rotations, opacities, sh0, sh_rest) expected")
        for got, want in zip((params[0], params[1], params[2], params[3], params[5]),
                             (self.means, self.scales, self.rotations, self.opacities, self.sh_rest)):
            if got.data_ptr() != want.data_ptr():
                raise RuntimeError("preprocess_adam updates the tensors the forward read; got another tensor")
        grad_in = list(grad_in) if grad_in is not None else [None] * 6
        st = _AdamState()
        keep = []
        for k in range(6):
            p, m, v, g = params[k], exp_avg[k], exp_avg_sq[k], grad_in[k]
            for name, t in (("param", p), ("exp_avg", m), ("exp_avg_sq", v)):
                L.check_cuda(name, t, torch.float32)
                if t.numel() != p.numel():
                    raise RuntimeError(f"{name} of group {k} does not match its parameter")
            if g is not None:
                g = g.detach().to(torch.float32).contiguous()
                if g.numel() != p.numel():
                    raise RuntimeError(f"grad_in of group {k} does not match its parameter")
                keep.append(g)
            st.exp_avg[k] = m.data_ptr()
            st.exp_avg_sq[k] = v.data_ptr()
            st.grad_in[k] = g.data_ptr() if g is not None else None
            st.lr[k] = float(lrs[k])
            st.step[k] = int(steps[k])
        st.beta1, st.beta2, st.eps = float(betas[0]), float(betas[1]), float(eps)
        L.call("gs3d_backward_preprocess_adam", *map(L.ptr, params), self.n, ctypes.byref(self.s), L.ptr(self.prim),
               self.prim.numel(), L.ptr(self.ws), self.ws.numel(), ctypes.byref(st), self.stream)


@torch.no_grad()
def backward_blend(densification_info, grad_image, image, means, scales, rotations, opacities, sh_rest, prim_buf,
                   tile_buf, inst_buf, bucket_buf, w2c, cam_position, bg_color, active_sh_bases, width, height,
                   focal_x, focal_y, center_x, center_y, near_plane, far_plane, proper_antialiasing, n_instances,
                   n_buckets, selector, *mode, defer_densification: bool = False) -> PendingBackward:
    """The blend backward of `_C.backward` alone (gs3d_backward_blend): returns the PendingBackward whose
    preprocess()/preprocess_adam() finishes it. The densification rows are accumulated now
    (gs3d_backward_densification) unless defer_densification leaves them to preprocess()."""
    n = means.shape[0]
    rest = sh_rest.shape[1] if sh_rest.dim() == 3 else 0
    dev = means.device
    keep: list = []
    s = _settings(dev, w2c, cam_position, bg_color, active_sh_bases, width, height, focal_x, focal_y, center_x,
                  center_y, near_plane, far_plane, proper_antialiasing, rest, keep)
    g_img = grad_image.detach().to(torch.float32).contiguous()
    ws = torch.empty(L.query("gs3d_backward_workspace_size", n), dtype=torch.uint8, device=dev)
    rows, dinfo = _densification(densification_info, n)
    stream = L.stream_of(means)
    L.call("gs3d_backward_blend", L.ptr(g_img), L.ptr(image), n, int(n_instances), ctypes.byref(s), L.ptr(prim_buf),
           prim_buf.numel(), L.ptr(tile_buf), tile_buf.numel(), L.ptr(inst_buf), inst_buf.numel(), L.ptr(bucket_buf),
           bucket_buf.numel(), int(n_buckets), L.ptr(ws), ws.numel(), rows, stream)
    if rows and not defer_densification:
        L.call("gs3d_backward_densification", n, ctypes.byref(s), L.ptr(prim_buf), prim_buf.numel(), L.ptr(ws),
               ws.numel(), L.ptr(dinfo), rows, stream)
        rows, dinfo = 0, None
    return PendingBackward(ws, s, keep, prim_buf, (means, scales, rotations, opacities, sh_rest), n, rest, rows,
                           dinfo, stream)


def _densification(densification_info, n: int):
    """(rows, tensor or None): the reference's densification_info argument, float32 [0 | 2 | 3, N] on the GPU,
    accumulated in place (an empty tensor or None means no statistics)."""
    if densification_info is None or densification_info.numel() == 0:
        return 0, None
    L.check_cuda("densification_info", densification_info, torch.float32)
    if densification_info.dim() != 2 or densification_info.shape[0] not in (2, 3) or densification_info.shape[1] != n:
        raise RuntimeError(f"densification_info must be [2 or 3, {n}], got {tuple(densification_info.shape)}")
    return int(densification_info.shape[0]), densification_info


class _Rasterize(torch.autograd.Function):
    """The autograd function behind diff_rasterize (phase1/fastergs_macro.patch:565-594 shows its backward).

    Visibility hand-off for the sparse optimizer (cluster/patches/fastergs_lean_adam.patch:213-220,328-345): while
    track_visibility is set, each forward stores the per-primitive n_touched_tiles (int32 [N], > 0 = visible in
    that view) in last_visibility."""

    track_visibility: bool = False
    last_visibility: torch.Tensor | None = None
    # A FusedAdam(fuse_backward=True) that owns the six parameter tensors takes the preprocess backward into its
    # step: backward then runs the blend backward (and the densification rows) only and returns no parameter
    # gradients; the optimizer's next step() applies the gradients inside the fused kernel.
    fused_optimizer: Any = None

    @staticmethod
    def forward(ctx: Any, means, scales, rotations, opacities, sh0, sh_rest, densification_info,
                settings: RasterizerSettings, want_radii: bool = False, capacity: int | None = None,
                overflow: torch.Tensor | None = None):
        params = [t.contiguous() for t in (means, scales, rotations, opacities, sh0, sh_rest)]
        image, prim, tile, inst, bucket, m, nb, sel = forward(*params, *settings.as_tuple(), capacity=capacity,
                                                              overflow=overflow)
        if _Rasterize.track_visibility:
            _Rasterize.last_visibility = n_touched_tiles(prim, params[0].shape[0])
        ctx.settings = settings
        ctx.buffer_state = (m, nb, sel)
        ctx.densification_info = densification_info
        ctx.shapes = (opacities.shape, sh0.shape, sh_rest.shape)
        ctx.save_for_backward(image, params[0], params[1], params[2], params[3], params[5], prim, tile, inst, bucket,
                              params[4])
        if want_radii:
            radii = screen_radii(prim, params[0].shape[0])
            ctx.mark_non_differentiable(radii)
            return image, radii
        return image

    @staticmethod
    def backward(ctx: Any, grad_image, *unused):
        image, means, scales, rotations, opacities, sh_rest, prim, tile, inst, bucket, sh0 = ctx.saved_tensors
        opt = _Rasterize.fused_optimizer
        six = (means, scales, rotations, opacities, sh0, sh_rest)
        if opt is not None and opt._owns(six):
            pending = backward_blend(ctx.densification_info, grad_image, image, means, scales, rotations, opacities,
                                     sh_rest, prim, tile, inst, bucket, *ctx.settings.as_tuple(), *ctx.buffer_state)
            opt._defer(pending, six)
            return (None,) * 11
        g = backward(ctx.densification_info, grad_image, image, means, scales, rotations, opacities, sh_rest, prim,
                     tile, inst, bucket, *ctx.settings.as_tuple(), *ctx.buffer_state)
        op_shape, sh0_shape, rest_shape = ctx.shapes
        return (g[0], g[1], g[2], g[3].reshape(op_shape), g[4].reshape(sh0_shape), g[5].reshape(rest_shape), None,
                None, None, None, None)


def diff_rasterize(means, scales, rotations, opacities, sh0, sh_rest, densification_info,
                   settings: RasterizerSettings, *, capacity: int | None = None,
                   overflow: torch.Tensor | None = None) -> torch.Tensor:
    """Differentiable render of one view: image [3, H, W]. capacity / overflow (keyword, no counterpart in the
    reference): the bounded forward (see forward), with no host read."""
    return _Rasterize.apply(means, scales, rotations, opacities, sh0, sh_rest, densification_info, settings, False,
                            capacity, overflow)


def rasterize_gaussians(means3D, scales, rotations, opacities, shs, viewmatrix, projmatrix, bg, tanfovx, tanfovy,
                        image_height, image_width, sh_degree, campos, scale_modifier=1.0, near_plane=0.2,
                        far_plane=1000.0):
    """graphdeco-style entry: activated inputs (scales > 0, opacities in (0, 1), any quaternions, shs [N, K, 3]);
    viewmatrix is the transposed world-to-view matrix as graphdeco passes it (p_view = p_h @ viewmatrix) and
    projmatrix its full projection (viewmatrix @ P^T). The rasterizer is the pinhole model with the principal point
    at the image centre and focal lengths W / (2 tanfovx), H / (2 tanfovy); projmatrix must be that projection of
    viewmatrix (its x, y and w columns are checked; the depth column carries graphdeco's znear / zfar, which the
    model does not use), else ValueError. Returns (image [3, H, W], radii int32 [N]): graphdeco's screen radius,
    ceil(3 sqrt(largest eigenvalue of the dilated 2D covariance)), taken from the forward's own primitive buffer,
    0 for Gaussians the view does not list."""
    W, H = int(image_width), int(image_height)
    fx = W / (2.0 * float(tanfovx))
    fy = H / (2.0 * float(tanfovy))
    check_projmatrix(viewmatrix, projmatrix, float(tanfovx), float(tanfovy))
    w2c = viewmatrix.transpose(0, 1).contiguous()
    bases = (int(sh_degree) + 1) ** 2
    settings = RasterizerSettings(w2c, campos, bg, bases, W, H, fx, fy, W / 2.0, H / 2.0, near_plane, far_plane,
                                  False)
    log_scales = torch.log(scales * scale_modifier)
    logits = torch.logit(opacities.reshape(-1, 1).clamp(1e-7, 1 - 1e-7))
    sh0, sh_rest = shs[:, :1].contiguous(), shs[:, 1:].contiguous()
    return _Rasterize.apply(means3D, log_scales, rotations, logits, sh0, sh_rest, torch.empty(0), settings, True, None,
                            None)


def check_projmatrix(viewmatrix: torch.Tensor, projmatrix: torch.Tensor, tanfovx: float, tanfovy: float,
                     rtol: float = 1e-4) -> None:
    """projmatrix = viewmatrix @ P^T for graphdeco's pinhole P: its columns 0, 1 and 3 are viewmatrix's columns 0 and
    1 divided by tanfovx and tanfovy and its column 2. Raises ValueError otherwise (an off-centre or other
    projection, which the pinhole settings cannot express)."""
    v = viewmatrix.detach().double().cpu().reshape(4, 4)
    p = projmatrix.detach().double().cpu().reshape(4, 4)
    want = torch.stack([v[:, 0] / tanfovx, v[:, 1] / tanfovy, v[:, 2]], 1)
    got = torch.stack([p[:, 0], p[:, 1], p[:, 3]], 1)
    err = float((got - want).abs().max()) / max(float(want.abs().max()), 1e-30)
    if not err <= rtol:
        raise ValueError(f"projmatrix is not the centred pinhole projection of viewmatrix with tanfovx={tanfovx} and "
                         f"tanfovy={tanfovy} (relative difference {err:.2e}); use the Faster-GS entry (forward / "
                         f"diff_rasterize) with explicit focal lengths and principal point")


@torch.no_grad()
def screen_radii(prim_buf: torch.Tensor, n: int) -> torch.Tensor:
    """graphdeco's per-Gaussian screen radius from a forward's primitive buffer: ceil(3 sqrt(lambda_max)) of the dilated
    2D covariance (the inverse of the stored conic), int32, 0 where the Gaussian is not listed in any tile."""
    v = primitive_views(prim_buf, n)
    A, B, C = (v["conic_o"][:, k].double() for k in range(3))
    det = A * C - B * B
    a, b, c = C / det, -B / det, A / det  # covariance = conic^-1
    mid = 0.5 * (a + c)
    lam = mid + torch.sqrt(torch.clamp(mid * mid - (a * c - b * b), min=0.1))
    radii = torch.ceil(3.0 * torch.sqrt(lam)).to(torch.int32)
    return torch.where(v["n_touched"] > 0, radii, torch.zeros_like(radii))


def _align(x: int) -> int:
    return (x + 255) & ~255


def primitive_views(prim_buf: torch.Tensor, n: int) -> dict[str, torch.Tensor]:
    """Typed views into a primitive buffer (the layout of carve_prim in csrc/gs3d_common.cuh):
    mean2d [N,2], conic_o [N,4] (A, B, C, opacity), color_z [N,4] (r, g, b, depth), rect [N,4] (int16 pixels),
    thr [N], n_touched [N] (int32), depth_key / ids / depth_key_sorted [N], order [N] (ids in depth order),
    offsets [N] (instance offsets in that order), counters [8] (int32: instance count M, bucket count B, replayed
    buckets, M again). Per-Gaussian values are valid where n_touched > 0."""
    nn = max(n, 1)
    off = 0
    out = {}
    for name, elem, width, dtype in (("mean2d", 8, 2, torch.float32), ("conic_o", 16, 4, torch.float32),
                                     ("color_z", 16, 4, torch.float32), ("rect", 8, 4, torch.int16),
                                     ("thr", 4, 1, torch.float32), ("n_touched", 4, 1, torch.int32),
                                     ("depth_key", 4, 1, torch.int32), ("ids", 4, 1, torch.int32),
                                     ("depth_key_sorted", 4, 1, torch.int32), ("order", 4, 1, torch.int32),
                                     ("offsets", 4, 1, torch.int32)):
        off = _align(off)
        t = prim_buf[off:off + elem * nn].view(dtype)
        out[name] = t.view(nn, width)[:n] if width > 1 else t[:n]
        off += elem * nn
    off = _align(off)
    out["counters"] = prim_buf[off:off + 32].view(torch.int32)
    out["rect"] = out["rect"].to(torch.int32) & 0xFFFF
    return out


def n_touched_tiles(prim_buf: torch.Tensor, n: int) -> torch.Tensor:
    """Faster-GS `_C.n_touched_tiles` (cluster/patches/fastergs_lean_adam.patch:316-323): int32 [N], > 0 = visible."""
    return primitive_views(prim_buf, n)["n_touched"].clone()


def tile_views(tile_buf: torch.Tensor, width: int, height: int) -> dict[str, torch.Tensor]:
    """ranges [T,2], buckets per tile [T+1], first bucket [T+1], max_contrib [T], final_T [H,W], n_contrib [H,W]."""
    T = ((width + TILE - 1) // TILE) * ((height + TILE - 1) // TILE)
    off = 0
    out = {}
    for name, count, dtype, shape in (("ranges", 2 * T, torch.int32, (T, 2)), ("nb", T + 1, torch.int32, (T + 1,)),
                                      ("bstart", T + 1, torch.int32, (T + 1,)),
                                      ("max_contrib", T, torch.int32, (T,)),
                                      ("final_T", width * height, torch.float32, (height, width)),
                                      ("n_contrib", width * height, torch.int32, (height, width))):
        off = _align(off)
        out[name] = tile_buf[off:off + 4 * count].view(dtype).view(shape)
        off += 4 * count
    return out


def instance_views(inst_buf: torch.Tensor, m: int, prim_buf: torch.Tensor | None = None,
                   n: int = 0) -> dict[str, torch.Tensor]:
    """tiles (generation order), vals, tiles_sorted, point_list [M] (int32). With the primitive buffer, also
    keys_sorted: the 64-bit (tile << 32 | order-preserving depth bits) keys in sorted order (as int64)."""
    mm = max(m, 1)
    off = 0
    out = {}
    for name in ("tiles", "vals", "tiles_sorted", "point_list"):
        off = _align(off)
        out[name] = inst_buf[off:off + 4 * mm].view(torch.int32)[:m]
        off += 4 * mm
    if prim_buf is not None:
        z = primitive_views(prim_buf, n)["color_z"][:, 3].contiguous()
        zb = z.view(torch.int32).to(torch.int64) & 0xFFFFFFFF
        zk = torch.where(zb >= 2 ** 31, zb ^ 0xFFFFFFFF, zb | 2 ** 31)
        out["keys_sorted"] = (out["tiles_sorted"].to(torch.int64) << 32) | zk[out["point_list"].long()]
    return out


def bucket_views(bucket_buf: torch.Tensor, bcap: int) -> dict[str, torch.Tensor]:
    """tile [B] (tile of each bucket), reached [B] (the buckets the forward reached, in no set order), ckpt [B, 256, 4]
    ((C.r, C.g, C.b, T) of each tile pixel, row-major, at the bucket's start): the layout of carve_bucket in
    csrc/gs3d_common.cuh. Only the first counters[1] buckets exist; the rest of the capacity is unused."""
    bb = max(bcap, 1)
    off = 0
    out = {}
    for name, count in (("tile", bb), ("reached", bb)):
        off = _align(off)
        out[name] = bucket_buf[off:off + 4 * count].view(torch.int32)
        off += 4 * count
    off = _align(off)
    out["ckpt"] = bucket_buf[off:off + 16 * TILE * TILE * bb].view(torch.float32).view(bb, TILE * TILE, 4)
    return out


def backward_workspace_views(ws: torch.Tensor, n: int) -> dict[str, torch.Tensor]:
    """The per-Gaussian sums the blend backward leaves in its workspace (carve_grad in csrc/gs3d_backward.cu):
    mean2d [N, 2] (dL/dmean2d, pixels), conic_o [N, 4] (dL/dA, dL/dB, dL/dC, dL/dopacity), color [N, 4]
    (dL/d max(colour, 0), w unused), mean2d_abs [N, 2] (sums of |per-pixel dL/dmean2d|, written with three
    densification rows only)."""
    nn = max(n, 1)
    off = _align(4)
    out = {}
    for name, width in (("mean2d", 2), ("conic_o", 4), ("color", 4), ("mean2d_abs", 2)):
        off = _align(off)
        out[name] = ws[off:off + 4 * width * nn].view(torch.float32).view(nn, width)[:n]
        off += 4 * width * nn
    return out


def focal_from_fov(fov_y_deg: float, height: int) -> float:
    return 0.5 * height / math.tan(math.radians(fov_y_deg) / 2.0)
