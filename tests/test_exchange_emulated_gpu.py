"""The exchange kernels' multi-rank arithmetic on one GPU: two ranks emulated by two sets of buffers on the same
device, each rank's kernel launched in turn with the device addresses of both sets (the kernels wait on nothing,
so running rank 0's and then rank 1's launch is the same computation as running them side by side on two GPUs).

Each "rank" renders two views of a small scene; each view's blend backward runs once and its preprocess backward
runs into both forms from the same sums (six gradient tensors, and the compact form's four tensors plus records).
The reference is the sum of the two ranks' gradients (rank order) followed by one adam_step_multi over the six
groups. adam_step_dp_fused (peer form) and adam_step_dp_compact must give the same parameters bit for bit, in every
rank's copy."""
from __future__ import annotations

import ctypes
import math

import pytest
import torch

from gs_b200 import _lib as L
from gs_b200 import adam as A
from gs_b200 import dist as D
from gs_b200 import gs3d, scenes

pytestmark = pytest.mark.gpu

NAMES = ("means", "scales", "rotations", "opacities", "sh0", "sh_rest")
LRS = [1.6e-4, 5e-3, 1e-3, 5e-2, 2.5e-3, 2.5e-3]


def _rank_gradients(tensors, cams, dev, seed):
    """Six accumulated gradient tensors, and the compact form's four non-SH tensors plus one record block per view,
    from the same blend backward of each view."""
    n = tensors[0].shape[0]
    full = [torch.zeros_like(t) for t in tensors]
    small = [torch.zeros_like(t) for t in tensors[:4]]
    records = []
    g = torch.Generator(device=dev).manual_seed(seed)
    for k, cam in enumerate(cams):
        s = scenes.settings_tuple(cam, 16, dev)
        p = tensors
        img, prim, tile, inst, bucket, m, nb, sel = gs3d.forward(*p, *s)
        dout = torch.randn(img.shape, device=dev, generator=g) * 1e-2
        pend = gs3d.backward_blend(None, dout, img, p[0], p[1], p[2], p[3], p[5], prim, tile, inst, bucket, *s, m, nb,
                                   sel, defer_densification=True)
        pend.preprocess(out=full, accumulate=k > 0)
        rec = torch.empty(6 * n, device=dev)
        pend.preprocess_records(small, rec, accumulate=k > 0)
        records.append(rec)
    return full, small, records


@pytest.mark.parametrize("n", [8_000, 8_003])
def test_two_rank_exchange_kernels_on_one_gpu(n, cuda):
    dev = cuda
    sc = scenes.gaussians_3d(n, 11, sigma=1.0)
    tensors = [sc[k].to(dev).contiguous() for k in NAMES]
    cams = [scenes.camera(192, 128, (6 * math.cos(2 * math.pi * k / 4), 0.4, 6 * math.sin(2 * math.pi * k / 4)))
            for k in range(4)]
    ranks = [_rank_gradients(tensors, [cams[r], cams[r + 2]], dev, 30 + r) for r in range(2)]
    sizes = [t.numel() for t in tensors]
    total = sum(sizes)

    # reference: gradients summed in rank order, one Adam step of the six groups
    ref = [t.clone() for t in tensors]
    summed = [a + b for a, b in zip(ranks[0][0], ranks[1][0])]
    A.adam_step([(p, g, torch.zeros_like(p), torch.zeros_like(p), lr) for p, g, lr in zip(ref, summed, LRS)], 1)
    ref_flat = torch.cat([t.flatten() for t in ref])

    # peer form: flat vectors per rank
    params = [torch.cat([t.flatten() for t in tensors]) for _ in range(2)]
    grads = [torch.cat([t.flatten() for t in ranks[r][0]]) for r in range(2)]
    segs, off = [], 0
    for sz, lr in zip(sizes, LRS):
        segs.append(D._Segment(off, off + sz, lr))
        off += sz
    seg_arr = (D._Segment * 6)(*segs)
    gptr = (ctypes.c_void_p * 8)(*[g.data_ptr() for g in grads])
    pptr = (ctypes.c_void_p * 8)(*[p.data_ptr() for p in params])
    stream = L.stream_of(params[0])
    for r in range(2):
        lo, hi = D.owned_slice(total, r, 2)
        m = torch.zeros(max(hi - lo, 1), device=dev)
        v = torch.zeros_like(m)
        L.call("adam_step_dp_fused", 2, r, ctypes.addressof(gptr), ctypes.addressof(pptr), lo, hi, L.ptr(m), L.ptr(v),
               6, ctypes.addressof(seg_arr), 1, 0.9, 0.999, 1e-15, stream)
    torch.cuda.synchronize()
    assert all(torch.equal(p, ref_flat) for p in params), "peer form differs from the all-reduce + Adam reference"

    # compact form: parameters in the same layout, gradients = four non-SH groups then one record block per view
    lay = D.compact_layout(n, 15, 2)
    cparams = [torch.cat([t.flatten() for t in tensors]) for _ in range(2)]
    cgrads = []
    for r in range(2):
        _, small, records = ranks[r]
        cgrads.append(torch.cat([t.flatten() for t in small] + records))
        assert cgrads[-1].numel() == lay["grad_total"]
    gptr = (ctypes.c_void_p * 8)(*[g.data_ptr() for g in cgrads])
    pptr = (ctypes.c_void_p * 8)(*[p.data_ptr() for p in cparams])
    lr = (ctypes.c_double * 6)(*LRS)
    for r in range(2):
        lo, hi = D.owned_gaussians(n, r, 2)
        cpad = (hi - lo + 3) // 4 * 4
        m = torch.zeros(max(59 * cpad, 1), device=dev)
        v = torch.zeros_like(m)
        L.call("adam_step_dp_compact", 2, r, ctypes.addressof(gptr), ctypes.addressof(pptr), n, lo, hi, 2, 16, 15,
               L.ptr(m), L.ptr(v), ctypes.addressof(lr), 1, 0.9, 0.999, 1e-15, stream)
    torch.cuda.synchronize()
    for p in cparams:
        for name, (a, b) in lay["params"].items():
            assert torch.equal(p[a:b], ref_flat[a:b]), f"compact form differs from the reference in {name}"
