"""The exchange + Adam forms on 2 GPUs - PeerAdam (csrc/dp_adam.cu) with peer loads / stores and with NVLink
multicast, and NcclAdam (NCCL reduce-scatter, Adam on the owned slice, all-gather) - against an NCCL all-reduce of
the gradients followed by adam_step_multi on every rank. With two ranks the gradient sum g0 + g1 is the same single
addition in all of them, so parameters and the owned moments must agree bit for bit. Skipped with fewer than two
GPUs. NVLS is left to NCCL's default here; the ranks exchange only on the host between steps."""
from __future__ import annotations

import datetime
import os

import pytest
import torch
import torch.distributed as dist
import torch.multiprocessing as mp

pytestmark = pytest.mark.gpu


def _worker(rank: int, world: int, port: int, q, form: str) -> None:
    try:
        os.environ["MASTER_ADDR"] = "127.0.0.1"
        os.environ["MASTER_PORT"] = str(port)
        torch.cuda.set_device(rank)
        dev = torch.device("cuda", rank)
        dist.init_process_group("nccl", rank=rank, world_size=world, timeout=datetime.timedelta(seconds=60),
                                device_id=dev)
        import sys
        sys.path.insert(0, os.getcwd())
        import __graft_entry__ as ge
        ge.load_package()
        from gs_b200 import adam as A
        from gs_b200 import dist as D

        n = 10_007
        g0 = torch.Generator(device=dev).manual_seed(0)
        init = [torch.randn(n, 3, device=dev, generator=g0), torch.randn(n, 4, device=dev, generator=g0),
                torch.randn(n, 1, device=dev, generator=g0), torch.randn(n, 15, 3, device=dev, generator=g0)]
        lrs = [1e-3, 2e-3, 5e-2, 2.5e-3]
        opt = D.NcclAdam(init, lrs) if form == "nccl" else D.PeerAdam(init, lrs, nvls=form == "nvls")
        ref = [t.clone() for t in init]
        m = [torch.zeros_like(t) for t in init]
        v = [torch.zeros_like(t) for t in init]
        gr = torch.Generator(device=dev).manual_seed(100 + rank)
        for step in range(1, 4):
            grads = [torch.randn(t.shape, device=dev, generator=gr) * 1e-2 for t in init]
            for gv, g in zip(opt.grads, grads):
                gv.copy_(g)
            opt.step()
            summed = [g.clone() for g in grads]
            for s in summed:
                dist.all_reduce(s)
            A.adam_step([(p, s, mm, vv, lr) for p, s, mm, vv, lr in zip(ref, summed, m, v, lrs)], step)
        torch.cuda.synchronize()
        ok_p = all(torch.equal(a, b) for a, b in zip(opt.params, ref))
        flat_m = torch.cat([x.flatten() for x in m])[opt.lo:opt.hi]  # the multicast path pads the vector to 4
        ok_m = torch.equal(opt.exp_avg[:flat_m.numel()], flat_m)
        # the copied-in path: step(grads=...) gives the same as writing into opt.grads
        used_nvls = getattr(opt, "nvls", False)
        opt.close()
        q.put((rank, ok_p, ok_m, None if used_nvls or form != "nvls" else "no NVLS"))
        dist.destroy_process_group()
    except Exception as exc:  # report instead of hanging the parent
        q.put((rank, False, False, repr(exc)))


@pytest.mark.parametrize("form", ["peer", "nvls", "nccl"])
def test_exchange_matches_allreduce_adam(form):
    if torch.cuda.device_count() < 2:
        pytest.skip("needs two GPUs")
    ctx = mp.get_context("spawn")
    q = ctx.Queue()
    port = 29600 + os.getpid() % 300 + {"peer": 0, "nvls": 7, "nccl": 13}[form]
    procs = [ctx.Process(target=_worker, args=(r, 2, port, q, form)) for r in range(2)]
    for p in procs:
        p.start()
    res = [q.get(timeout=300) for _ in procs]
    for p in procs:
        p.join(timeout=60)
        if p.is_alive():  # never leave a rank behind
            p.kill()
    for rank, ok_p, ok_m, err in res:
        if err == "no NVLS":
            pytest.skip("this node has no NVLink multicast")
        assert err is None, f"rank {rank}: {err}"
        assert ok_p and ok_m, f"rank {rank}: params equal {ok_p}, moments equal {ok_m}"


def _compact_worker(rank: int, world: int, port: int, q, n: int, views: int) -> None:
    """Each view's blend backward runs once; its preprocess backward runs twice from the same sums, into PeerAdam's
    six gradient tensors and into CompactPeerAdam's four non-SH tensors and records (the preprocess backward is
    deterministic; the blend backward's atomics are not, so two blend backwards would not give the same bits)."""
    try:
        os.environ["MASTER_ADDR"] = "127.0.0.1"
        os.environ["MASTER_PORT"] = str(port)
        torch.cuda.set_device(rank)
        dev = torch.device("cuda", rank)
        dist.init_process_group("nccl", rank=rank, world_size=world, timeout=datetime.timedelta(seconds=60),
                                device_id=dev)
        import math
        import sys
        sys.path.insert(0, os.getcwd())
        import __graft_entry__ as ge
        ge.load_package()
        from gs_b200 import dist as D
        from gs_b200 import gs3d, scenes

        sc = scenes.gaussians_3d(n, 7, sigma=1.0)
        names = ("means", "scales", "rotations", "opacities", "sh0", "sh_rest")
        cams = [scenes.camera(256, 192, (6 * math.cos(2 * math.pi * k / (world * views)), 0.5,
                                         6 * math.sin(2 * math.pi * k / (world * views))))
                for k in range(world * views)]
        mine = D.shard_views(cams, rank, world)
        tensors = [sc[k].to(dev).contiguous() for k in names]
        lrs = [1.6e-4, 5e-3, 1e-3, 5e-2, 2.5e-3, 2.5e-3]
        full = D.PeerAdam(tensors, lrs, nvls=False)
        compact = D.CompactPeerAdam(tensors, lrs, views=len(mine), active_sh_bases=16)
        g = torch.Generator(device=dev).manual_seed(50 + rank)
        same, seen_zero = [], 0
        for step in range(3):
            for k, cam in enumerate(mine):
                s = scenes.settings_tuple(cam, 16, dev)
                p = full.params
                img, prim, tile, inst, bucket, m, nb, sel = gs3d.forward(*p, *s)
                seen_zero += int((gs3d.n_touched_tiles(prim, n) == 0).sum())
                dout = torch.randn(img.shape, device=dev, generator=g) * 1e-2
                pend = gs3d.backward_blend(None, dout, img, p[0], p[1], p[2], p[3], p[5], prim, tile, inst, bucket,
                                           *s, m, nb, sel, defer_densification=True)
                pend.preprocess(out=full.grads, accumulate=k > 0)
                pend.preprocess_records(compact.grads, compact.records[k], accumulate=k > 0)
            full.step()
            compact.step()
            torch.cuda.synchronize()
            same.append(all(torch.equal(a, b) for a, b in zip(full.params, compact.params)))
        moved = not torch.equal(full.params[5], tensors[5])
        full.close()
        compact.close()
        q.put((rank, all(same), moved and seen_zero > 0, None))
        dist.destroy_process_group()
    except Exception as exc:  # report instead of hanging the parent
        q.put((rank, False, False, repr(exc)))


@pytest.mark.parametrize("n, views", [(20_000, 2), (20_003, 1)])
def test_compact_exchange_matches_peer(n, views):
    """CompactPeerAdam (SH gradients sent as colour-gradient / direction records) gives bit-identical parameters to
    PeerAdam over three steps: with two views per rank (the records of a rank summed in view order) and 16-byte
    accesses, and with one view per rank and an odd Gaussian count (element-wise accesses)."""
    if torch.cuda.device_count() < 2:
        pytest.skip("needs two GPUs")
    ctx = mp.get_context("spawn")
    q = ctx.Queue()
    port = 29600 + os.getpid() % 300 + 20 + views
    procs = [ctx.Process(target=_compact_worker, args=(r, 2, port, q, n, views)) for r in range(2)]
    for p in procs:
        p.start()
    res = [q.get(timeout=300) for _ in procs]
    for p in procs:
        p.join(timeout=60)
        if p.is_alive():
            p.kill()
    for rank, same, exercised, err in res:
        assert err is None, f"rank {rank}: {err}"
        assert exercised, f"rank {rank}: the SH parameters did not move or every Gaussian was seen"
        assert same, f"rank {rank}: compact and full exchanges differ"


def _hook_worker(port: int, q, form: str) -> None:
    """One rank (world size 1): the diff_rasterize backward writes into the exchange's gradient buffer (the autograd
    hook), so step(grads=[p.grad ...]) finds the leaves' .grad empty and copies nothing; the gradients in the buffer
    equal gs3d.backward's on the same view to the blend backward's atomic-order noise, and the step moved the
    parameters."""
    try:
        os.environ["MASTER_ADDR"] = "127.0.0.1"
        os.environ["MASTER_PORT"] = str(port)
        torch.cuda.set_device(0)
        dev = torch.device("cuda", 0)
        dist.init_process_group("nccl", rank=0, world_size=1, timeout=datetime.timedelta(seconds=60), device_id=dev)
        import sys
        sys.path.insert(0, os.getcwd())
        import __graft_entry__ as ge
        ge.load_package()
        from gs_b200 import dist as D
        from gs_b200 import gs3d, scenes

        sc = scenes.gs3d_test_scene("tiny", 4)
        names = ("means", "scales", "rotations", "opacities", "sh0", "sh_rest")
        tensors = [sc[k].to(dev).contiguous() for k in names]
        settings = scenes.settings_tuple(sc["cameras"][0], sc["active_sh_bases"], dev)
        lrs = [1.6e-4, 5e-3, 1e-3, 5e-2, 2.5e-3, 2.5e-3]
        opt = D.NcclAdam(tensors, lrs) if form == "nccl" else D.PeerAdam(tensors, lrs, nvls=False)
        leaves = [p.requires_grad_(True) for p in opt.params]
        img = gs3d.diff_rasterize(*leaves, torch.empty(0), gs3d.RasterizerSettings(*settings))
        dout = torch.randn(img.shape, device=dev, generator=torch.Generator(device=dev).manual_seed(9)) * 1e-2
        img.backward(dout)
        untouched = all(p.grad is None for p in leaves)
        opt.step(grads=[p.grad for p in leaves])
        r = gs3d.forward(*tensors, *settings)
        g = gs3d.backward(None, dout, r[0], tensors[0], tensors[1], tensors[2], tensors[3], tensors[5], *r[1:5],
                          *settings, *r[5:8])
        torch.cuda.synchronize()
        err = max(float((a.flatten() - b.flatten()).norm() / b.flatten().norm().clamp_min(1e-30))
                  for a, b in zip(opt.grads, g))
        moved = max(float((a.detach() - b).abs().max()) for a, b in zip(opt.params, tensors))
        opt.close()
        dist.destroy_process_group()
        q.put((untouched, err, moved, None))
    except Exception as exc:  # report instead of hanging the parent
        q.put((False, 1.0, 0.0, repr(exc)))


@pytest.mark.parametrize("form", ["peer", "nccl"])
def test_autograd_backward_writes_into_the_exchange(form):
    if torch.cuda.device_count() < 1:
        pytest.skip("needs a GPU")
    ctx = mp.get_context("spawn")
    q = ctx.Queue()
    port = 29600 + os.getpid() % 300 + 40 + (form == "nccl")
    p = ctx.Process(target=_hook_worker, args=(port, q, form))
    p.start()
    untouched, err, moved, exc = q.get(timeout=300)
    p.join(timeout=60)
    if p.is_alive():
        p.kill()
    assert exc is None, exc
    assert untouched, "the leaves got a .grad: the backward did not write into the exchange's buffer"
    assert err < 1e-5 and moved > 0, (err, moved)
