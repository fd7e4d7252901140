"""splat2d against the reference's own CUDA kernels on the same GPU and the same inputs.

The reference's extension with its CUDA kernels (phase0/csrc/macrotile, built as phase0/splat2d/ops.py:33-45 does
with -DWITH_CUDA) is compiled from the reference tree for sm_100a by oracle/build.py into
oracle/_ref/splat2d_cuda_ref and loaded here from that file. Both get the same scene (the generator of
bench/phase0/backward_bench.py:35-49, float32 on the GPU) and the same tile tables (this package's bin_tiles, which is
bit-exact against the reference's), then:
  * forward: n_contrib and last_contrib exact; image, t_final and checkpoints within 1e-5 absolute
  * backward_pixel and backward_splat: the four gradients within 1e-4 of the reference's, relative to their norm -
    the benchmark spec's atomic-order tolerance (the two per-splat backwards reduce in different orders; measured
    1.5e-5 at 20k splats)
"""
from __future__ import annotations

import importlib.util
from pathlib import Path

import pytest
import torch

from gs_b200 import scenes, splat2d

pytestmark = pytest.mark.gpu

REF_SO = Path(__file__).resolve().parent.parent / "oracle" / "_ref" / "splat2d_cuda_ref" / "splat2d_cuda_ref.so"


@pytest.fixture(scope="module")
def ref_ext():
    if not REF_SO.exists():
        pytest.skip("the reference's splat2d CUDA extension is not built (oracle/build.py builds it where the "
                    "reference tree exists)")
    spec = importlib.util.spec_from_file_location("splat2d_cuda_ref", REF_SO)
    mod = importlib.util.module_from_spec(spec)
    spec.loader.exec_module(mod)
    return mod


def scene(n, h, w, seed=0, sigma=(2.0, 10.0), opacity=(0.05, 0.6)):
    """The scene generator of bench/phase0/backward_bench.py:35-49 (float64, index order = depth order)."""
    return scenes.splat2d_bench_scene(n, h, w, seed, sigma, opacity)


def rel(a, b) -> float:
    a, b = a.double().flatten(), b.double().flatten()
    nb = float(b.norm())
    return float((a - b).norm()) / nb if nb > 0 else float((a - b).norm())


@pytest.mark.parametrize("n,h,w", [(2000, 256, 320), (20_000, 540, 960), (50_000, 1080, 1920)])
def test_splat2d_matches_reference_cuda(n, h, w, ref_ext, cuda):
    p64 = [t.to(cuda) for t in scene(n, h, w)]
    bins = splat2d.bin_tiles(*p64[:3], h, w)
    tb = (bins.tile_offsets, bins.tile_ids, bins.bucket_offsets, bins.bucket_tile)
    p32 = [t.float().contiguous() for t in p64]
    ours = splat2d.load_extension(with_cuda=True)
    o = ours.forward(*p32, *tb, h, w)
    r = ref_ext.forward(*p32, *tb, h, w)
    names = ("image", "t_final", "n_contrib", "last_contrib", "ckpt")
    for k, (a, b) in enumerate(zip(o, r)):
        if k in (2, 3):
            assert torch.equal(a, b), names[k]
        else:
            assert (a - b).abs().max().item() <= 1e-5, names[k]
    image, t_final, n_contrib, last_contrib, ckpt = r
    g_img = torch.randn(h, w, 3, generator=torch.Generator().manual_seed(1)).to(cuda)
    for a, b in zip(ours.backward_pixel(g_img, *p32, *tb, t_final, last_contrib, h, w),
                    ref_ext.backward_pixel(g_img, *p32, *tb, t_final, last_contrib, h, w)):
        assert rel(a, b) < 1e-4
    for a, b in zip(ours.backward_splat(g_img, *p32, *tb, image, ckpt, h, w),
                    ref_ext.backward_splat(g_img, *p32, *tb, image, ckpt, h, w)):
        assert rel(a, b) < 1e-4
    torch.cuda.synchronize()
