"""ctypes wrapper of oracle/_ref/libsplat2d_ref.so: the REFERENCE's own splat2d CPU code
(phase0/csrc/macrotile/splat2d_cpu.cpp), built from the reference tree by oracle/build.py.

TEST INFRASTRUCTURE: tests and bench.py's CPU baseline only. ``available()`` is False where the
reference tree was absent at build time.
"""
from __future__ import annotations

import ctypes
from pathlib import Path

import numpy as np

LIB = Path(__file__).resolve().parent / "_ref" / "libsplat2d_ref.so"
_lib = None


def available() -> bool:
    return LIB.exists()


def _load():
    global _lib
    if _lib is None:
        _lib = ctypes.CDLL(str(LIB))
        P, I = ctypes.c_void_p, ctypes.c_int
        _lib.splat2d_ref_forward.argtypes = [I] + [P] * 8 + [I, I, I] + [P] * 5
        _lib.splat2d_ref_backward.argtypes = [I, I] + [P] * 9 + [I, I, I] + [P] * 8
        _lib.splat2d_ref_counters.argtypes = [P]
    return _lib


def _p(a: np.ndarray):
    return a.ctypes.data_as(ctypes.c_void_p)


class RefScene:
    """Contiguous arrays of one scene in the dtype the reference runs in."""

    def __init__(self, means, chol, opacity_logit, colors, bins, H, W, dtype=np.float64):
        self.dtype = dtype
        self.f64 = int(dtype == np.float64)
        self.means = np.ascontiguousarray(means, dtype)
        self.chol = np.ascontiguousarray(chol, dtype)
        self.z = np.ascontiguousarray(opacity_logit, dtype)
        self.colors = np.ascontiguousarray(colors, dtype)
        self.tables = [np.ascontiguousarray(t, np.int32) for t in
                       (bins.tile_offsets, bins.tile_ids, bins.bucket_offsets, bins.bucket_tile)]
        self.B = int(self.tables[3].size)
        self.H, self.W = H, W

    def _scene_ptrs(self):
        return [_p(self.means), _p(self.chol), _p(self.z), _p(self.colors), *map(_p, self.tables)]

    def forward(self):
        lib = _load()
        H, W = self.H, self.W
        image = np.zeros((H, W, 3), self.dtype)
        t_final = np.ones((H, W), self.dtype)
        n_contrib = np.zeros((H, W), np.int32)
        last = np.zeros((H, W), np.int32)
        ckpt = np.zeros((max(self.B, 1), 256, 4), self.dtype)
        lib.splat2d_ref_forward(self.f64, *self._scene_ptrs(), self.B, H, W, _p(image), _p(t_final), _p(n_contrib),
                                _p(last), _p(ckpt))
        return image, t_final, n_contrib, last, ckpt[: self.B]

    def backward(self, splat_mode: bool, grad_image, fwd):
        lib = _load()
        image, t_final, _, last, ckpt = fwd
        gi = np.ascontiguousarray(grad_image, self.dtype)
        grads = [np.zeros_like(self.means), np.zeros_like(self.chol), np.zeros_like(self.z),
                 np.zeros_like(self.colors)]
        ck = np.ascontiguousarray(ckpt if ckpt.size else np.zeros((1, 256, 4), self.dtype))
        lib.splat2d_ref_backward(self.f64, int(splat_mode), _p(gi), *self._scene_ptrs(), self.B, self.H, self.W,
                                 _p(np.ascontiguousarray(t_final)), _p(np.ascontiguousarray(last)),
                                 _p(np.ascontiguousarray(image)), _p(ck), *map(_p, grads))
        return grads


def counters() -> dict[str, int]:
    out = (ctypes.c_longlong * 3)()
    _load().splat2d_ref_counters(ctypes.addressof(out))
    return {"atomic_adds": out[0], "checkpoint_bytes": out[1], "splat_pixel_evals": out[2]}


def reset_counters() -> None:
    _load().splat2d_ref_reset_counters()
