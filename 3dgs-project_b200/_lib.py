"""ctypes binding of libsplat_b200.so (the C ABI declared in include/splat_b200.h).

The library is loaded on first use and never replaced by anything else: if it is missing, or a
tensor handed to it is not a CUDA tensor, the call raises. There is no CPU path.
"""
from __future__ import annotations

import ctypes
import os
from pathlib import Path

import torch

# SPLAT_B200_LIB may name another build of the same library (e.g. a tuning variant); it is still this C ABI.
LIB_PATH = Path(os.environ.get("SPLAT_B200_LIB", Path(__file__).resolve().with_name("libsplat_b200.so")))
ABI_VERSION = 2

_P = ctypes.c_void_p
_I = ctypes.c_int
_LL = ctypes.c_longlong
_SZ = ctypes.c_size_t

# name -> (restype, argtypes)
_SIGNATURES: dict[str, tuple[object, list[object]]] = {
    "splat_last_error": (ctypes.c_char_p, []),
    "splat_abi_version": (_I, []),
    "splat_launch_count": (_LL, []),
    "splat_time_kernel": (_I, [ctypes.c_char_p, _P, _P]),
    "splat_scan_workspace_size": (_SZ, [_LL]),
    "splat_scan_exclusive_u32": (_I, [_P, _P, _LL, _P, _P, _SZ, _P]),
    "splat_scan_exclusive_u32_noalloc": (_I, [_P, _P, _LL, _P, _P]),
    "splat_sort_workspace_size": (_SZ, [_LL, _I]),
    "splat_radix_sort_pairs": (_I, [_P, _P, _P, _P, _LL, _I, _I, _I, _P, _SZ, _P]),
    "splat_check_device_waits": (_I, []),
    "splat_set_lookback_poll_limit": (_I, [_I]),
    "splat_l1_ssim_workspace_size": (_SZ, [_I, _I, _I, _I]),
    "splat_peer_alloc": (_I, [_SZ, _P, _P]),
    "splat_peer_open": (_I, [_P, _P]),
    "splat_peer_close": (_I, [_P]),
    "splat_peer_free": (_I, [_P]),
    "adam_step_dp_nvls": (_I, [_LL, _LL, _P, _P, _P, _P, _P, _I, _P, _I, ctypes.c_double, ctypes.c_double,
                               ctypes.c_double, _P]),
    "adam_step_dp_fused": (_I, [_I, _I, _P, _P, _LL, _LL, _P, _P, _I, _P, _I, ctypes.c_double, ctypes.c_double,
                                ctypes.c_double, _P]),
    "adam_step_dp_compact": (_I, [_I, _I, _P, _P, _LL, _LL, _LL, _I, _I, _I, _P, _P, _P, _I, ctypes.c_double,
                                  ctypes.c_double, ctypes.c_double, _P]),
    "splat_l1_ssim_forward": (_I, [_P, _P, _I, _I, _I, _I, ctypes.c_float, _I, _P, _P, _P, _SZ, _P]),
    "splat_l1_ssim_backward": (_I, [_P, _P, _I, _I, _I, _I, ctypes.c_float, _I, _P, _P, _P, _SZ, _P]),
    "splat_take_device_waits_async": (_I, [_P, _P]),
    "gs2d_bin_count_workspace_size": (_SZ, [_I]),
    "gs2d_bin_fill_workspace_size": (_SZ, [_LL, _I, _I]),
    "gs2d_bin_count": (_I, [_P, _P, _P, _I, _I, _I, _I, _P, _P, _P, _P, _SZ, _P]),
    "gs2d_bin_fill_bounded": (_I, [_P, _I, _I, _I, _LL, _P, _P, _SZ, _P, _SZ, _P, _P, _P, _P, _LL, _P, _P, _P]),
    "gs2d_bin_fill": (_I, [_P, _I, _I, _I, _LL, _P, _SZ, _P, _SZ, _P, _P, _P, _P, _P, _P]),
    "gs2d_forward": (_I, [_P] * 8 + [_I, _LL, _I, _I, _I, _I] + [_P] * 5),
    "gs2d_backward_pixel": (_I, [_P] * 7 + [_I, _LL, _I, _I] + [_P] * 8),
    "gs2d_backward_splat": (_I, [_P] * 8 + [_I, _I, _LL, _I, _I] + [_P] * 9),
    "splat2d_bin_count_workspace_size": (_SZ, [_I]),
    "splat2d_bin_fill_workspace_size": (_SZ, [_LL, _I, _I]),
    "splat2d_bin_count": (_I, [_I, _P, _P, _P, _I, _I, _I, _P, _P, _SZ, _P]),
    "splat2d_bin_fill": (_I, [_I, _I, _I, _LL, _P, _SZ, _P, _SZ, _P, _P, _P, _P, _P, _P]),
    "splat2d_forward": (_I, [_I] + [_P] * 8 + [_I, _LL, _I, _I, _I] + [_P] * 6),
    "splat2d_backward": (_I, [_I, _I] + [_P] * 9 + [_I, _LL, _I, _I, _I] + [_P] * 9),
    "splat2d_set_counting": (_I, [_I]),
    "splat2d_reset_counters": (_I, []),
    "splat2d_get_counters": (_I, [_P]),
    "gs3d_primitive_buffer_size": (_SZ, [_I]),
    "gs3d_tile_buffer_size": (_SZ, [_I, _I]),
    "gs3d_instance_buffer_size": (_SZ, [_LL]),
    "gs3d_bucket_bound": (_LL, [_LL, _I, _I]),
    "gs3d_bucket_buffer_size": (_SZ, [_LL]),
    "gs3d_backward_workspace_size": (_SZ, [_I]),
    "gs3d_preprocess": (_I, [_P] * 6 + [_I, _P, _P, _SZ, _P, _P]),
    "gs3d_preprocess_count": (_I, [_P] * 6 + [_I, _P, _P, _SZ, _P, _P]),
    "gs3d_preprocess_order": (_I, [_I, _P, _SZ, _P]),
    "gs3d_render": (_I, [_I, _LL, _P, _P, _SZ, _P, _SZ, _P, _SZ, _P, _SZ, _LL, _P, _P]),
    "gs3d_render_bounded": (_I, [_I, _LL, _P, _P, _SZ, _P, _SZ, _P, _SZ, _P, _SZ, _LL, _P, _P, _P]),
    "gs3d_render_inference": (_I, [_I, _LL, _P, _P, _SZ, _P, _SZ, _P, _SZ, _P, _P]),
    "gs3d_backward": (_I, [_P] * 7 + [_I, _LL, _P] + [_P, _SZ] * 4 + [_LL, _P, _SZ] + [_P] * 7 + [_I, _P]),
    "gs3d_backward_blend": (_I, [_P, _P, _I, _LL, _P] + [_P, _SZ] * 4 + [_LL, _P, _SZ, _I, _P]),
    "gs3d_backward_preprocess": (_I, [_P] * 5 + [_I, _P, _P, _SZ, _P, _SZ] + [_P] * 7 + [_I, _P]),
    "gs3d_backward_preprocess_accumulate": (_I, [_P] * 5 + [_I, _P, _P, _SZ, _P, _SZ] + [_P] * 7 + [_I, _P]),
    "gs3d_backward_preprocess_records": (_I, [_P] * 5 + [_I, _P, _P, _SZ, _P, _SZ] + [_P] * 5 + [_I, _P, _I, _P]),
    "gs3d_backward_densification": (_I, [_I, _P, _P, _SZ, _P, _SZ, _P, _I, _P]),
    "gs3d_backward_preprocess_adam": (_I, [_P] * 6 + [_I, _P, _P, _SZ, _P, _SZ, _P, _P]),
    "adam_step_multi": (_I, [_I, _P, _I, ctypes.c_double, ctypes.c_double, ctypes.c_double, _P]),
    "adam_step_multi_lean": (_I, [_I, _P, _I, ctypes.c_double, ctypes.c_double, ctypes.c_double, _P, _LL, _P]),
}

_lib: ctypes.CDLL | None = None


def load() -> ctypes.CDLL:
    """Load (once) and type the shared library; raise if it is missing or of another ABI."""
    global _lib
    if _lib is None:
        if not LIB_PATH.exists():
            raise RuntimeError(
                f"{LIB_PATH.name} is not built; run `python 3dgs-project_b200/build.py` "
                "(or __graft_entry__.build()) first")
        lib = ctypes.CDLL(str(LIB_PATH))
        for name, (res, args) in _SIGNATURES.items():
            fn = getattr(lib, name)
            fn.restype = res
            fn.argtypes = args
        if lib.splat_abi_version() != ABI_VERSION:
            raise RuntimeError(f"{LIB_PATH.name} has ABI {lib.splat_abi_version()}, expected {ABI_VERSION}")
        _lib = lib
    return _lib


def call(name: str, *args) -> None:
    """Call one status-returning entry point; a non-zero status becomes RuntimeError(message)."""
    lib = load()
    fn = getattr(lib, name)
    if len(args) != len(fn.argtypes):  # ctypes would pass surplus arguments unconverted
        raise TypeError(f"{name} takes {len(fn.argtypes)} arguments, got {len(args)}")
    status = fn(*args)
    if status != 0:
        msg = lib.splat_last_error().decode(errors="replace")
        raise RuntimeError(f"{name}: {msg} (status {status})")


def check_device_waits(device: torch.device) -> None:
    """Raise if a bounded device-side wait (radix sort look-back) gave up on ``device`` since the last check.
    Costs one small synchronous copy; call it where the host already waits for the device."""
    with torch.cuda.device(device):
        call("splat_check_device_waits")


class KernelTimer:
    """Live device times of named kernels (splat_time_kernel): before each step, arm() hands the library a fresh
    pair of CUDA events per kernel, which it records on the launching stream around that kernel's next launches;
    times() returns, per kernel, the milliseconds of each armed step (the last launch of the kernel in that step)."""

    def __init__(self, *kernels: str):
        self.kernels = kernels
        self.pairs: dict[str, list] = {k: [] for k in kernels}

    def arm(self) -> None:
        for k in self.kernels:
            a, b = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
            a.record()  # creates the CUDA events; the library records them again around the launch
            b.record()
            call("splat_time_kernel", k.encode(), ctypes.c_void_p(a.cuda_event), ctypes.c_void_p(b.cuda_event))
            self.pairs[k].append((a, b))

    def stop(self) -> None:
        for k in self.kernels:
            call("splat_time_kernel", k.encode(), None, None)

    def times(self) -> dict[str, list[float]]:
        torch.cuda.synchronize()
        return {k: [a.elapsed_time(b) for a, b in v] for k, v in self.pairs.items()}

    def __enter__(self):
        return self

    def __exit__(self, *exc):
        self.stop()
        return False


def query(name: str, *args) -> int:
    return int(getattr(load(), name)(*args))


def ptr(t: torch.Tensor | None) -> int | None:
    """Device address of a CUDA tensor (None passes NULL)."""
    if t is None:
        return None
    return t.data_ptr()


def stream_of(t: torch.Tensor) -> int:
    return torch.cuda.current_stream(t.device).cuda_stream


def check_cuda(name: str, t: torch.Tensor, dtype: torch.dtype | None = None) -> torch.Tensor:
    """The reference's CHECK_INPUT (toy2d/csrc/rasterize.cu:355-358): CUDA, contiguous, dtype."""
    if not isinstance(t, torch.Tensor):
        raise TypeError(f"{name} must be a tensor")
    if not t.is_cuda:
        raise RuntimeError(f"{name} must be a CUDA tensor")
    if dtype is not None and t.dtype != dtype:
        raise RuntimeError(f"{name} has the wrong dtype ({t.dtype}, expected {dtype})")
    if not t.is_contiguous():
        raise RuntimeError(f"{name} must be contiguous")
    return t


def workspace(nbytes: int, device: torch.device) -> torch.Tensor:
    return torch.empty(max(int(nbytes), 1), dtype=torch.uint8, device=device)


def exported_symbols() -> list[str]:
    return list(_SIGNATURES)
