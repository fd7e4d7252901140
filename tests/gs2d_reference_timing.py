"""Times this library's toy2d kernels against the reference's own (toy2d/csrc/rasterize.cu, rebuilt for sm_100a by
oracle/build.py into oracle/_ref/gs2d_cuda_ref) on one GPU, on the reference bench's sweep and scenes
(toy2d/bench.py:43-70: seeded Gaussians2D, bins from bin_gaussians, which is bit-exact against the reference's).
A measurement helper next to the parity test tests/test_gs2d_ref_gpu.py, not a test itself:

    python tests/gs2d_reference_timing.py

One JSON line per (size, n): CUDA-event medians in ms of forward, forward saving bucket states, backward_pixel and
backward_splat, for "ours" and "reference".
"""
from __future__ import annotations

import importlib.util
import json
import statistics
import sys
from pathlib import Path

import torch

ROOT = Path(__file__).resolve().parent.parent
sys.path.insert(0, str(ROOT))

from __graft_entry__ import load_package  # noqa: E402

load_package()
from gs_b200 import gs2d  # noqa: E402

REF_SO = ROOT / "oracle" / "_ref" / "gs2d_cuda_ref" / "gs2d_cuda_ref.so"


def timed(fn, warmup: int = 5, iters: int = 50) -> float:
    for _ in range(warmup):
        fn()
    ts = []
    for _ in range(iters):
        a, b = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
        a.record()
        fn()
        b.record()
        torch.cuda.synchronize()
        ts.append(a.elapsed_time(b))
    return round(statistics.median(ts), 4)


def main() -> int:
    if not REF_SO.exists():
        print(json.dumps({"unavailable": "the reference's toy2d CUDA extension is not built"}))
        return 0
    spec = importlib.util.spec_from_file_location("gs2d_cuda_ref", REF_SO)
    ref = importlib.util.module_from_spec(spec)
    spec.loader.exec_module(ref)
    dev = torch.device("cuda", 0)
    for size in (512, 1024):
        for n in (10_000, 50_000, 200_000):
            H = W = size
            g = gs2d.Gaussians2D(n, H, W, seed=0).to(dev)
            with torch.no_grad():
                means, conic, color, opacity, cov = (t.contiguous() for t in g.activated())
                bins = gs2d.bin_gaussians(means, gs2d.radii_from_cov(cov), g.depth, H, W)
            bg = torch.zeros(3, device=dev)
            dout = torch.randn(3, H, W, generator=torch.Generator(device=dev).manual_seed(1), device=dev)
            common = (means, conic, color, opacity, bg, bins.ranges, bins.point_list)
            row = {"size": size, "n": n, "pairs": int(bins.point_list.numel())}
            for name, e in (("ours", gs2d.ext()), ("reference", ref)):
                def fwd(save, e=e):
                    return e.forward(*common, bins.bucket_offsets, bins.num_buckets, H, W, save)

                out, final_T, n_contrib, _ = fwd(False)
                out_s, final_T_s, n_contrib_s, bstate = fwd(True)
                row[name] = {
                    "forward": timed(lambda: fwd(False)),
                    "forward_save_buckets": timed(lambda: fwd(True)),
                    "backward_pixel": timed(lambda: e.backward_pixel(*common, final_T, n_contrib, dout)),
                    "backward_splat": timed(lambda: e.backward_splat(*common, bins.bucket_offsets, bins.bucket_to_tile,
                                                                     out_s, final_T_s, n_contrib_s, bstate, dout)),
                }
            print(json.dumps(row), flush=True)
    return 0


if __name__ == "__main__":
    sys.exit(main())
