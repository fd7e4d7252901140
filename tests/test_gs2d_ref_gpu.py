"""gs2d against the reference's own toy2d CUDA rasterizer on the same GPU and the same inputs.

The reference's extension (toy2d/csrc/rasterize.cu, which toy2d/gs2d/raster.py:13-26 JIT-builds) is compiled from the
reference tree for sm_100a by oracle/build.py into oracle/_ref/gs2d_cuda_ref and loaded here from that file. Both
extensions get the same seeded Gaussians2D scenes (the reference bench's, toy2d/bench.py:43-70) and the same bins
(bin_gaussians is bit-exact against the reference's), then:
  * forward: n_contrib exact; image, final T and the saved bucket states within 1e-5 absolute
  * backward_pixel and backward_splat: the four gradients within 1e-5 of the reference's, relative to their norm
    (float atomics: summation order differs between the two implementations)
"""
from __future__ import annotations

import importlib.util
from pathlib import Path

import pytest
import torch

from gs_b200 import gs2d

pytestmark = pytest.mark.gpu

REF_SO = Path(__file__).resolve().parent.parent / "oracle" / "_ref" / "gs2d_cuda_ref" / "gs2d_cuda_ref.so"


@pytest.fixture(scope="module")
def ref_ext():
    if not REF_SO.exists():
        pytest.skip("the reference's toy2d CUDA extension is not built (oracle/build.py builds it where the "
                    "reference tree exists)")
    spec = importlib.util.spec_from_file_location("gs2d_cuda_ref", REF_SO)
    mod = importlib.util.module_from_spec(spec)
    spec.loader.exec_module(mod)
    return mod


def rel(a, b) -> float:
    a, b = a.double().flatten(), b.double().flatten()
    nb = float(b.norm())
    return float((a - b).norm()) / nb if nb > 0 else float((a - b).norm())


@pytest.mark.parametrize("size,n", [(256, 4096), (512, 10_000), (512, 50_000), (1024, 10_000)])
def test_gs2d_matches_reference_cuda(size, n, ref_ext, cuda):
    H = W = size
    g = gs2d.Gaussians2D(n, H, W, seed=0).to(cuda)
    with torch.no_grad():
        means, conic, color, opacity, cov = (t.contiguous() for t in g.activated())
        bins = gs2d.bin_gaussians(means, gs2d.radii_from_cov(cov), g.depth, H, W)
    bg = torch.tensor([0.1, 0.2, 0.3], device=cuda)
    dout = torch.randn(3, H, W, generator=torch.Generator(device=cuda).manual_seed(size + n), device=cuda)
    ours = gs2d.ext()
    common = (means, conic, color, opacity, bg, bins.ranges, bins.point_list)
    fwd_args = (bins.bucket_offsets, bins.num_buckets, H, W)

    for save in (False, True):
        o = ours.forward(*common, *fwd_args, save)
        r = ref_ext.forward(*common, *fwd_args, save)
        assert torch.equal(o[2], r[2]), "n_contrib"
        assert (o[0] - r[0]).abs().max().item() <= 1e-5, "image"
        assert (o[1] - r[1]).abs().max().item() <= 1e-5, "final T"
        if save:
            assert (o[3] - r[3]).abs().max().item() <= 1e-5, "bucket states"
    out, final_T, n_contrib, bstate = r
    gp_o = ours.backward_pixel(*common, final_T, n_contrib, dout)
    gp_r = ref_ext.backward_pixel(*common, final_T, n_contrib, dout)
    gs_o = ours.backward_splat(*common, bins.bucket_offsets, bins.bucket_to_tile, out, final_T, n_contrib, bstate,
                               dout)
    gs_r = ref_ext.backward_splat(*common, bins.bucket_offsets, bins.bucket_to_tile, out, final_T, n_contrib,
                                  bstate, dout)
    for a, b in zip(gp_o, gp_r):
        assert rel(a, b) < 1e-5
    for a, b in zip(gs_o, gs_r):
        assert rel(a, b) < 1e-5
    torch.cuda.synchronize()
