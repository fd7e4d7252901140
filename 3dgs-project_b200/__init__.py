"""B200-native tile-based Gaussian-splatting rasterizer (sm_100a CUDA behind a C ABI).

Drop-in replacements for the rasterize ops of asadrizvi64/3dgs-project:
    gs2d     the toy2d 2D op      (toy2d/gs2d: rasterize, bin_gaussians, Gaussians2D, ...)
    splat2d  the phase0 2D op     (phase0/splat2d/ops.py: render, bin_tiles, load_extension, ...)
    gs3d     3DGS forward/backward (graphdeco-style rasterize_gaussians and the Faster-GS-shaped
             _C.forward / _C.backward pair), fused Adam and multi-view data parallelism

The directory name is not a Python identifier; tests, bench.py and __graft_entry__.py register it
under the module name ``gs_b200`` (see ``load_package`` in __graft_entry__.py).
"""
from . import _lib  # noqa: F401

__all__ = ["_lib"]
