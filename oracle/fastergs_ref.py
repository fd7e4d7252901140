"""ctypes binding of the reference's own Faster-GS blend backward (blend_backward_macro_cu,
phase1/fastergs_macro.patch:40-314) built by oracle/build.py into oracle/_ref/fastergs_macro (TEST INFRASTRUCTURE:
the parity tests and bench.py's reference arm only; the product never loads it).

``RefInputs`` takes the reference kernel's arguments from one forward of this library (16x16 tiles, the tile shape
the kernel is built for here) and ``run`` launches it on the current stream into fresh zeroed outputs.
"""
from __future__ import annotations

import ctypes
from pathlib import Path

import torch

REF_LIB = Path(__file__).resolve().parent / "_ref" / "fastergs_macro" / "libfastergs_macro_ref.so"
_ref = None


def ref_lib():
    global _ref
    if _ref is None:
        if not REF_LIB.exists():
            raise RuntimeError("oracle/_ref/fastergs_macro/libfastergs_macro_ref.so is not built (python "
                               "oracle/build.py with the reference tree present)")
        lib = ctypes.CDLL(str(REF_LIB))
        lib.fgs_ref_blend_backward_macro.restype = ctypes.c_int
        lib.fgs_ref_blend_backward_macro.argtypes = ([ctypes.c_int] * 2 + [ctypes.c_void_p] * 18 + [ctypes.c_int] * 6
                                                      + [ctypes.c_void_p])
        _ref = lib
    return _ref


class RefInputs:
    """The reference kernel's arguments, taken from one forward of this library."""

    def __init__(self, params, settings, image, prim, tile, inst, bucket, m, nb, W, H):
        from gs_b200 import gs3d

        n = params[0].shape[0]
        self.n, self.W, self.H = n, W, H
        pv = gs3d.primitive_views(prim, n)
        self.tv = gs3d.tile_views(tile, W, H)
        self.iv = gs3d.instance_views(inst, m)
        self.bv = gs3d.bucket_views(bucket, nb)
        self.n_buckets = int(pv["counters"][1])
        self.mean2d, self.conic_o = pv["mean2d"], pv["conic_o"]
        self.color3 = pv["color_z"][:, :3].contiguous()
        self.color_mask = pv["color_z"][:, :3] >= 0
        self.visible = pv["n_touched"] > 0  # the primitive entries of the others are not written by the forward
        r = pv["rect"]  # (x0, y0, x1, y1) inclusive -> Faster-GS screen bounds (x0, x1 + 1, y0, y1 + 1)
        self.bounds = torch.stack([r[:, 0], r[:, 2] + 1, r[:, 1], r[:, 3] + 1], 1).to(torch.int16).contiguous()
        self.image = image
        self.prim = prim
        self.aa = bool(settings[12])

    def run(self, grad_image, mode: int, abs_grad: bool, stream=None):
        dev = self.image.device
        n = self.n
        out = {"mean2d": torch.zeros(n, 2, device=dev), "conic": torch.zeros(3, n, device=dev),
               "opacity": torch.zeros(n, device=dev), "color": torch.zeros(n, 3, device=dev),
               "mean2d_abs": torch.zeros(n, 2, device=dev)}
        tv, P = self.tv, lambda t: ctypes.c_void_p(t.data_ptr())
        st = torch.cuda.current_stream(dev).cuda_stream if stream is None else stream
        rc = ref_lib().fgs_ref_blend_backward_macro(
            mode, int(abs_grad), P(tv["ranges"]), P(tv["bstart"][1:]), P(self.iv["point_list"]), P(self.bounds),
            P(self.mean2d), P(self.conic_o), P(self.color3), P(grad_image), P(self.image), P(tv["max_contrib"]),
            P(tv["n_contrib"]), P(self.bv["tile"]), P(self.bv["ckpt"]), P(out["mean2d"]), P(out["conic"]),
            P(out["opacity"]), P(out["color"]), P(out["mean2d_abs"]), self.n_buckets, n, self.W, self.H,
            (self.W + 15) // 16, int(self.aa), ctypes.c_void_p(st))
        if rc != 0:
            raise RuntimeError(f"reference kernel launch failed: cudaError {rc}")
        return out
