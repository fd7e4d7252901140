"""Times this library's splat2d kernels against the reference's own (phase0/csrc/macrotile, rebuilt for sm_100a by
oracle/build.py into oracle/_ref/splat2d_cuda_ref) on one GPU, on the scenes of the reference's
bench/phase0/backward_bench.py (defaults 1920x1080, 50k splats, sigma 2-10 px, opacity 0.05-0.6). A measurement helper
next to the parity test tests/test_splat2d_ref_gpu.py, not a test itself:

    python tests/splat2d_reference_timing.py

One JSON line per scene: CUDA-event medians in ms of forward, backward_pixel and backward_splat (each including its
output allocation, as the reference's bench times them), for "ours" and "reference".
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
sys.path.insert(0, str(ROOT / "tests"))

from __graft_entry__ import load_package  # noqa: E402

load_package()
from gs_b200 import splat2d  # noqa: E402
from test_splat2d_ref_gpu import scene  # noqa: E402

REF_SO = ROOT / "oracle" / "_ref" / "splat2d_cuda_ref" / "splat2d_cuda_ref.so"


def timed(fn, warmup: int = 5, iters: int = 30) -> float:
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
        print(json.dumps({"unavailable": "the reference's splat2d CUDA extension is not built"}))
        return 0
    spec = importlib.util.spec_from_file_location("splat2d_cuda_ref", REF_SO)
    ref = importlib.util.module_from_spec(spec)
    spec.loader.exec_module(ref)
    dev = torch.device("cuda", 0)
    for n, h, w in ((50_000, 1080, 1920), (200_000, 1080, 1920), (20_000, 540, 960)):
        p64 = [t.to(dev) for t in scene(n, h, w)]
        bins = splat2d.bin_tiles(*p64[:3], h, w)
        tb = (bins.tile_offsets, bins.tile_ids, bins.bucket_offsets, bins.bucket_tile)
        p32 = [t.float().contiguous() for t in p64]
        g_img = torch.randn(h, w, 3, generator=torch.Generator().manual_seed(1)).to(dev)
        row = {"n": n, "height": h, "width": w, "list_entries": int(bins.tile_ids.numel()),
               "buckets": bins.num_buckets}
        for name, e in (("ours", splat2d.load_extension(with_cuda=True)), ("reference", ref)):
            image, t_final, n_contrib, last_contrib, ckpt = e.forward(*p32, *tb, h, w)
            row[name] = {
                "forward": timed(lambda e=e: e.forward(*p32, *tb, h, w)),
                "backward_pixel": timed(lambda e=e: e.backward_pixel(g_img, *p32, *tb, t_final, last_contrib, h, w)),
                "backward_splat": timed(lambda e=e: e.backward_splat(g_img, *p32, *tb, image, ckpt, h, w)),
            }
        print(json.dumps(row), flush=True)
    return 0


if __name__ == "__main__":
    sys.exit(main())
