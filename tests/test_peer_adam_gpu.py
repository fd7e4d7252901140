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
