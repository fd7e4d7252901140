"""ctypes wrapper of oracle/liboracle.so, the C++ restatement of the 3DGS training step
(TEST INFRASTRUCTURE: tests and bench.py's CPU baseline only).

``Oracle`` runs preprocess, binning, blend, blend backward and preprocess backward on the CPU with all host
threads; ``time_training_step`` times one training step of a config-sized view on a bounded sample of tile
rows and reports views/s.
"""
from __future__ import annotations

import ctypes
import os
import time
from pathlib import Path

import numpy as np

LIB = Path(__file__).resolve().parent / "liboracle.so"
_lib = None
_P = ctypes.c_void_p


class Settings(ctypes.Structure):
    _fields_ = [("w2c", ctypes.c_float * 16), ("cam_position", ctypes.c_float * 3), ("bg", ctypes.c_float * 3),
                ("active_sh_bases", ctypes.c_int), ("rest_bases", ctypes.c_int), ("width", ctypes.c_int),
                ("height", ctypes.c_int), ("fx", ctypes.c_float), ("fy", ctypes.c_float), ("cx", ctypes.c_float),
                ("cy", ctypes.c_float), ("near_plane", ctypes.c_float), ("far_plane", ctypes.c_float),
                ("proper_antialiasing", ctypes.c_int)]


def load():
    global _lib
    if _lib is None:
        if not LIB.exists():
            raise RuntimeError("oracle/liboracle.so is not built (python oracle/build.py)")
        lib = ctypes.CDLL(str(LIB))
        lib.gs3o_create.restype = _P
        lib.gs3o_destroy.argtypes = [_P]
        lib.gs3o_threads.restype = ctypes.c_int
        lib.gs3o_set_threads.argtypes = [ctypes.c_int]
        lib.gs3o_preprocess.argtypes = [_P] * 7 + [ctypes.c_int, _P]
        lib.gs3o_set_primitives.argtypes = [_P] * 6
        lib.gs3o_bin.argtypes = [_P]
        lib.gs3o_bin.restype = ctypes.c_longlong
        lib.gs3o_blend.argtypes = [_P, ctypes.c_int, ctypes.c_int]
        lib.gs3o_backward_reset.argtypes = [_P]
        lib.gs3o_blend_backward.argtypes = [_P, _P, ctypes.c_int, ctypes.c_int]
        lib.gs3o_blend_backward_fast.argtypes = [_P, _P, ctypes.c_int, ctypes.c_int]
        lib.gs3o_preprocess_backward.argtypes = [_P] * 12
        lib.gs3o_adam.argtypes = [_P] * 4 + [ctypes.c_longlong, ctypes.c_int] + [ctypes.c_double] * 4
        for name in ("mean2d", "conic_o", "color_z", "thr", "n_touched", "point_list", "keys_sorted", "ranges",
                     "image", "final_T", "n_contrib", "near", "g_mean2d", "g_conic_o", "g_color"):
            getattr(lib, f"gs3o_{name}").restype = _P
            getattr(lib, f"gs3o_{name}").argtypes = [_P]
        _lib = lib
    return _lib


def available() -> bool:
    return LIB.exists()


def _ptr(a: np.ndarray):
    return a.ctypes.data_as(ctypes.c_void_p)


def settings_from(cam: dict, active_sh_bases: int, rest_bases: int = 15) -> Settings:
    s = Settings()
    w = np.asarray(cam["w2c"], np.float32).reshape(16)
    for k in range(16):
        s.w2c[k] = float(w[k])
    for k in range(3):
        s.cam_position[k] = float(np.asarray(cam["cam_position"]).reshape(3)[k])
        s.bg[k] = float(np.asarray(cam["bg_color"]).reshape(3)[k])
    s.active_sh_bases, s.rest_bases = int(active_sh_bases), int(rest_bases)
    s.width, s.height = int(cam["width"]), int(cam["height"])
    s.fx, s.fy, s.cx, s.cy = (float(cam[k]) for k in ("focal_x", "focal_y", "center_x", "center_y"))
    s.near_plane, s.far_plane = float(cam["near_plane"]), float(cam["far_plane"])
    s.proper_antialiasing = int(bool(cam.get("proper_antialiasing", False)))
    return s


class Oracle:
    """One view of one scene on the CPU. Arrays are float32 numpy, in the layouts of the device path."""

    def __init__(self, params: list[np.ndarray], cam: dict, active_sh_bases: int):
        self.lib = load()
        self.ctx = self.lib.gs3o_create()
        self.params = [np.ascontiguousarray(p, np.float32) for p in params]
        self.n = self.params[0].shape[0]
        self.rest = self.params[5].size // (3 * max(self.n, 1))
        self.s = settings_from(cam, active_sh_bases, self.rest)
        self.W, self.H = self.s.width, self.s.height
        self.tiles_y = (self.H + 15) // 16
        self.m = 0

    def __del__(self):
        if getattr(self, "ctx", None):
            self.lib.gs3o_destroy(self.ctx)

    def _arr(self, name, dtype, count):
        p = getattr(self.lib, f"gs3o_{name}")(self.ctx)
        return np.ctypeslib.as_array(ctypes.cast(p, ctypes.POINTER(np.ctypeslib.as_ctypes_type(dtype))),
                                     shape=(count,)).copy()

    def preprocess(self):
        self.lib.gs3o_preprocess(self.ctx, *map(_ptr, self.params), self.n, ctypes.byref(self.s))

    def set_primitives(self, mean2d, conic_o, color_z, thr, n_touched):
        keep = [np.ascontiguousarray(a, t) for a, t in ((mean2d, np.float32), (conic_o, np.float32),
                                                         (color_z, np.float32), (thr, np.float32),
                                                         (n_touched, np.int32))]
        self.lib.gs3o_set_primitives(self.ctx, *map(_ptr, keep))

    def bin(self) -> int:
        self.m = int(self.lib.gs3o_bin(self.ctx))
        return self.m

    def blend(self, row0=0, row1=None):
        self.lib.gs3o_blend(self.ctx, row0, self.tiles_y if row1 is None else row1)

    def backward(self, grad_image: np.ndarray, row0=0, row1=None, bands=None):
        """The six parameter gradients of the blend backward over tile rows [row0, row1) (or over each
        (row0, row1) of ``bands``), chained through the preprocess backward."""
        g = np.ascontiguousarray(grad_image, np.float32)
        self.lib.gs3o_backward_reset(self.ctx)
        for r0, r1 in (bands or [(row0, self.tiles_y if row1 is None else row1)]):
            self.lib.gs3o_blend_backward(self.ctx, _ptr(g), r0, r1)
        n, rest = self.n, self.rest
        out = [np.zeros((n, 3), np.float32), np.zeros((n, 3), np.float32), np.zeros((n, 4), np.float32),
               np.zeros((n, 1), np.float32), np.zeros((n, 1, 3), np.float32), np.zeros((n, rest, 3), np.float32)]
        p = self.params
        self.lib.gs3o_preprocess_backward(self.ctx, _ptr(p[0]), _ptr(p[1]), _ptr(p[2]), _ptr(p[3]), _ptr(p[5]),
                                          *map(_ptr, out))
        return out

    def blend_backward_sums(self, grad_image: np.ndarray, bands=None) -> dict:
        """The blend backward alone, in float64: per-Gaussian dL/dmean2d [N, 2], (dL/dA, dL/dB, dL/dC, dL/dopacity)
        [N, 4] and dL/dcolour [N, 3] summed over tile rows [r0, r1) of ``bands`` (default: all rows)."""
        g = np.ascontiguousarray(grad_image, np.float32)
        self.lib.gs3o_backward_reset(self.ctx)
        for r0, r1 in (bands or [(0, self.tiles_y)]):
            self.lib.gs3o_blend_backward(self.ctx, _ptr(g), r0, r1)
        n = self.n
        return {"mean2d": self._arr("g_mean2d", np.float64, 2 * n).reshape(n, 2),
                "conic_o": self._arr("g_conic_o", np.float64, 4 * n).reshape(n, 4),
                "color": self._arr("g_color", np.float64, 3 * n).reshape(n, 3)}

    def primitives(self) -> dict:
        n = self.n
        return {"mean2d": self._arr("mean2d", np.float32, 2 * n).reshape(n, 2),
                "conic_o": self._arr("conic_o", np.float32, 4 * n).reshape(n, 4),
                "color_z": self._arr("color_z", np.float32, 4 * n).reshape(n, 4),
                "thr": self._arr("thr", np.float32, n), "n_touched": self._arr("n_touched", np.int32, n)}

    def binning(self) -> dict:
        T = ((self.W + 15) // 16) * self.tiles_y
        return {"point_list": self._arr("point_list", np.int64, self.m),
                "keys_sorted": self._arr("keys_sorted", np.uint64, self.m),
                "ranges": self._arr("ranges", np.int64, 2 * T).reshape(T, 2)}

    def frame(self) -> dict:
        P = self.W * self.H
        return {"image": self._arr("image", np.float32, 3 * P).reshape(3, self.H, self.W),
                "final_T": self._arr("final_T", np.float32, P).reshape(self.H, self.W),
                "n_contrib": self._arr("n_contrib", np.int32, P).reshape(self.H, self.W),
                "near": self._arr("near", np.uint8, P).reshape(self.H, self.W).astype(bool)}


def use_all_threads(threads: int | None = None) -> int:
    """Sets the oracle's OpenMP thread count (default: every host CPU; torch.distributed.run sets OMP_NUM_THREADS=1,
    which would otherwise leave it single-threaded) and returns the count now in effect."""
    lib = load()
    lib.gs3o_set_threads(int(threads or os.cpu_count() or 1))
    return int(lib.gs3o_threads())


class TrainingStepSample:
    """One training step of one view on the CPU, on a bounded sample: preprocess, binning, preprocess backward and
    Adam over every parameter in full; blend + blend backward on ``rows`` tile rows spread evenly over the image,
    extrapolated to the whole view. Gradient outputs and optimiser state are allocated and touched once,
    untimed, as a training loop holds them."""

    def __init__(self, sc: dict, cam: dict, threads: int | None = None):
        import torch

        self.threads = use_all_threads(threads)
        params = [sc[k].numpy() if torch.is_tensor(sc[k]) else sc[k]
                  for k in ("means", "scales", "rotations", "opacities", "sh0", "sh_rest")]
        self.o = Oracle(params, {k: (v.numpy() if torch.is_tensor(v) else v) for k, v in cam.items()},
                        sc["active_sh_bases"])
        o = self.o
        rng = np.random.default_rng(0)
        self.grad = (1e-3 * rng.standard_normal((3, o.H, o.W))).astype(np.float32)
        n, rest = o.n, o.rest
        self.out = [np.zeros((n, 3), np.float32), np.zeros((n, 3), np.float32), np.zeros((n, 4), np.float32),
                    np.zeros((n, 1), np.float32), np.zeros((n, 1, 3), np.float32), np.zeros((n, rest, 3), np.float32)]
        self.state = []
        for prm in o.params:
            q, m, v = prm.copy(), np.empty_like(prm), np.empty_like(prm)
            m.fill(0.0)
            v.fill(0.0)
            self.state.append((q, m, v))
        self.rows = 1
        self.t = 0

    def step(self) -> dict:
        o, p = self.o, self.o.params
        t0 = time.perf_counter()
        o.preprocess()
        t1 = time.perf_counter()
        o.bin()
        t2 = time.perf_counter()
        rows = self.sample_rows()
        for r in rows:
            o.blend(r, r + 1)
        o.lib.gs3o_backward_reset(o.ctx)
        for r in rows:
            o.lib.gs3o_blend_backward_fast(o.ctx, _ptr(self.grad), r, r + 1)
        t3 = time.perf_counter()
        o.lib.gs3o_preprocess_backward(o.ctx, _ptr(p[0]), _ptr(p[1]), _ptr(p[2]), _ptr(p[3]), _ptr(p[5]),
                                       *map(_ptr, self.out))
        t4 = time.perf_counter()
        self.t += 1
        for (q, m, v), g in zip(self.state, self.out):
            o.lib.gs3o_adam(_ptr(q), _ptr(g), _ptr(m), _ptr(v), q.size, self.t, 1e-3, 0.9, 0.999, 1e-15)
        t5 = time.perf_counter()
        blend_full = (t3 - t2) * o.tiles_y / len(rows)
        parts = {"preprocess": t1 - t0, "binning": t2 - t1, "blend_fwd_bwd_band": t3 - t2,
                 "blend_fwd_bwd_full_view_est": blend_full, "preprocess_backward": t4 - t3, "adam": t5 - t4}
        return {"seconds": (t1 - t0) + (t2 - t1) + blend_full + (t4 - t3) + (t5 - t4), "parts": parts,
                "rows": len(rows), "instances": o.m}

    def sample_rows(self) -> list[int]:
        """``rows`` tile rows spread evenly over the image (the middle of each of ``rows`` equal bands), so the
        sample's blend cost is an unbiased estimate of the view's."""
        ty = self.o.tiles_y
        k = min(max(self.rows, 1), ty)
        return sorted({min(int((i + 0.5) * ty / k), ty - 1) for i in range(k)})

    def calibrate(self, target_s: float) -> dict:
        """One step on one tile row, then the band widened so that a step takes about ``target_s``."""
        self.rows = 1
        s = self.step()
        fixed = s["seconds"] - s["parts"]["blend_fwd_bwd_full_view_est"]
        per_row = max(s["parts"]["blend_fwd_bwd_band"], 1e-6)
        self.rows = int(min(max((target_s - fixed) / per_row, 1), self.o.tiles_y))
        return s

    def describe(self) -> str:
        o = self.o
        return (f"one training step of one {o.W}x{o.H} view, {o.n} Gaussians: preprocess, binning ({o.m} instances), "
                f"preprocess backward and Adam in full; blend + blend backward on {len(self.sample_rows())} of "
                f"{o.tiles_y} tile rows spread evenly over the image, scaled to the whole view")


def time_training_step(sc: dict, cam: dict, budget_s: float = 20.0) -> dict:
    """One training step of one view on the CPU (TrainingStepSample), its band sized for about ``budget_s``."""
    smp = TrainingStepSample(sc, cam)
    smp.calibrate(budget_s * 0.6)
    res = smp.step()
    return {"value": round(1.0 / res["seconds"], 5), "unit": "views/s", "cores": smp.threads, "kind": "port",
            "sample": smp.describe(), "seconds": {k: round(v, 3) for k, v in res["parts"].items()},
            "threads": smp.threads}


def time_render_frame(sc: dict, cam: dict, budget_s: float = 20.0) -> dict:
    """One render-only frame on the CPU: preprocess, binning, and the blend over a band of tile rows (grown until
    about ``budget_s`` of work), extrapolated to the whole frame."""
    import torch

    params = [sc[k].numpy() if torch.is_tensor(sc[k]) else sc[k]
              for k in ("means", "scales", "rotations", "opacities", "sh0", "sh_rest")]
    threads = use_all_threads()
    o = Oracle(params, {k: (v.numpy() if torch.is_tensor(v) else v) for k, v in cam.items()}, sc["active_sh_bases"])
    t0 = time.perf_counter()
    o.preprocess()
    t1 = time.perf_counter()
    o.bin()
    t2 = time.perf_counter()
    mid = o.tiles_y // 2
    rows, blend_s, band = 0, 0.0, 1
    while True:
        r0 = max(mid - band // 2, 0)
        r1 = min(r0 + band, o.tiles_y)
        ta = time.perf_counter()
        o.blend(r0, r1)
        tb = time.perf_counter()
        rows, blend_s = r1 - r0, tb - ta
        if tb - t0 > budget_s * 0.6 or r1 - r0 >= o.tiles_y:
            break
        band = min(band * 2, o.tiles_y)
    full = blend_s * o.tiles_y / max(rows, 1)
    frame_s = (t1 - t0) + (t2 - t1) + full
    return {"value": round(1.0 / frame_s, 5), "unit": "frames/s", "cores": threads, "kind": "port",
            "sample": f"one {o.W}x{o.H} frame of {o.n} Gaussians: preprocess and binning ({o.m} instances) in full, "
                      f"blend on {rows} of {o.tiles_y} tile rows ({blend_s:.2f} s), scaled to the whole frame",
            "seconds": {"preprocess": round(t1 - t0, 3), "binning": round(t2 - t1, 3),
                        "blend_full_frame_est": round(full, 3)}}
