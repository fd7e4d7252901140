"""Multi-process host logic of the data-parallel step, on CPU with gloo (world size 2).

Checks the view sharding, that one all-reduce of the flat buffer sums every group's gradients, and that the
replicas stay identical after the same Adam step; a rank that raises is seen by the other as a failed
collective (short process-group timeout), not as a hang.
"""
from __future__ import annotations

import datetime
import os
import socket

import pytest
import torch
import torch.distributed as dist
import torch.multiprocessing as mp

from __graft_entry__ import load_package  # spawned ranks re-import this module: register the package first

load_package()
from gs_b200 import dist as gdist  # noqa: E402


def _free_port() -> int:
    with socket.socket() as s:
        s.bind(("127.0.0.1", 0))
        return s.getsockname()[1]


def _init(rank, world, port, timeout_s=60):
    os.environ["MASTER_ADDR"] = "127.0.0.1"
    os.environ["MASTER_PORT"] = str(port)
    dist.init_process_group("gloo", rank=rank, world_size=world, timeout=datetime.timedelta(seconds=timeout_s))


def _worker(rank, world, port, q):
    try:
        _init(rank, world, port)
        n = 37
        views = list(range(8))
        mine = gdist.shard_views(views, rank, world)
        g = gdist.FlatGradients(n, 15)
        torch.manual_seed(100 + rank)
        per_view = []
        for v in mine:
            torch.manual_seed(1000 + v)
            grads = [torch.randn(v.shape) for v in g.views]
            per_view.append(grads)
            g.add_(grads)
        g.all_reduce()
        # the expected sum over all 8 views, computed locally
        expect = [torch.zeros_like(v) for v in g.views]
        for v in views:
            torch.manual_seed(1000 + v)
            for e, t in zip(expect, [torch.randn(x.shape) for x in g.views]):
                e.add_(t)
        ok_sum = all(torch.allclose(a, b, atol=1e-5) for a, b in zip(g.views, expect))
        # same Adam-like update on both ranks keeps the replicas equal
        p = torch.ones(n, 3)
        p -= 0.1 * g.views[0].sign()
        gathered = [torch.zeros_like(p) for _ in range(world)]
        dist.all_gather(gathered, p)
        q.put((rank, mine, ok_sum, all(torch.equal(gathered[0], x) for x in gathered)))
        dist.destroy_process_group()
    except Exception as exc:  # report instead of hanging the parent
        q.put((rank, None, False, repr(exc)))


def test_two_ranks_shard_views_and_sum_gradients():
    ctx = mp.get_context("spawn")
    q = ctx.Queue()
    port = _free_port()
    procs = [ctx.Process(target=_worker, args=(r, 2, port, q)) for r in range(2)]
    for p in procs:
        p.start()
    res = sorted(q.get(timeout=120) for _ in procs)
    for p in procs:
        p.join(timeout=60)
    assert res[0][1] == [0, 2, 4, 6] and res[1][1] == [1, 3, 5, 7]
    assert all(r[2] for r in res), res
    assert all(r[3] is True for r in res), res


def _dying_worker(rank, world, port, q):
    _init(rank, world, port, timeout_s=5)
    if rank == 1:
        dist.destroy_process_group()
        raise SystemExit(3)  # leaves between steps, before the collective
    t = torch.ones(4)
    try:
        dist.all_reduce(t)
        q.put((rank, "completed"))
    except Exception as exc:
        q.put((rank, type(exc).__name__))


def test_a_rank_that_leaves_makes_the_collective_fail_not_hang():
    ctx = mp.get_context("spawn")
    q = ctx.Queue()
    port = _free_port()
    procs = [ctx.Process(target=_dying_worker, args=(r, 2, port, q)) for r in range(2)]
    for p in procs:
        p.start()
    rank, outcome = q.get(timeout=120)
    for p in procs:
        p.join(timeout=60)
        if p.is_alive():
            p.kill()
    assert rank == 0 and outcome != "completed"


def test_shard_views_rejects_bad_ranks():
    with pytest.raises(ValueError):
        gdist.shard_views([1, 2], 2, 2)
    assert gdist.shard_views(list(range(8)), 3, 8) == [3]


def test_owned_slices_tile_the_vector():
    for total in (0, 1, 5, 17, 4096, 177_000_001):
        for world in (1, 2, 3, 4, 7, 8):
            spans = [gdist.owned_slice(total, r, world) for r in range(world)]
            assert spans[0][0] == 0 and spans[-1][1] == total
            for (a, b), (c, d) in zip(spans, spans[1:]):
                assert b == c
            assert all(lo <= hi and (lo % 4 == 0 or lo == hi) for lo, hi in spans)
    with pytest.raises(ValueError):
        gdist.owned_slice(10, 2, 2)


def test_owned_gaussians_and_compact_layout():
    """The compact exchange's ownership is by whole Gaussians (starts at multiples of 4) and its buffers hold the
    parameter groups in the reference's order and one 6n-float record block per view after the non-SH gradients."""
    for n in (0, 1, 5, 17, 4096, 3_000_001):
        for world in (1, 2, 3, 8):
            spans = [gdist.owned_gaussians(n, r, world) for r in range(world)]
            assert spans[0][0] == 0 and spans[-1][1] == n
            assert all(b == c for (_, b), (c, _) in zip(spans, spans[1:]))
            assert all(lo <= hi and (lo % 4 == 0 or lo == hi) for lo, hi in spans)
    lay = gdist.compact_layout(10, 15, 3)
    assert lay["params"]["means"] == (0, 30) and lay["params"]["sh0"] == (110, 140)
    assert lay["params"]["sh_rest"] == (140, 590) and lay["param_total"] == 590
    assert lay["grads"] == {"means": (0, 30), "scales": (30, 60), "rotations": (60, 100), "opacities": (100, 110)}
    assert lay["records"] == [(110, 170), (170, 230), (230, 290)] and lay["grad_total"] == 290
    assert gdist.exchange_for(2, "compact") == "compact"


def test_auto_exchange_picks_compact_only_for_record_writers():
    """"auto" may pick the compact form (whose backward writes records instead of SH gradients) only for callers that
    say they write records; the others get a form that takes the six gradient tensors."""
    for world in (2, 3, 4, 5, 8):
        assert gdist.exchange_for(world) in ("peer", "nvls", "nccl")
        assert gdist.exchange_for(world, records=True) in ("peer", "nvls", "nccl", "compact")
    assert gdist.exchange_for(4, records=True) == gdist.AUTO_EXCHANGE[4]
    assert gdist.exchange_for(4) == gdist.AUTO_EXCHANGE_FULL[4]
    with pytest.raises(ValueError):
        gdist.exchange_for(2, "ring")


class _FakeMulticast:
    """Stands in for MulticastFlat on the host: allocation in the constructor, then a bind() that runs one
    collective per buffer (as the rendezvous does) and yields a multicast address, or none; a record of how it was
    closed."""

    closed: list = []

    def __init__(self, mc: int):
        self._mc = mc
        self.mc = 0

    def bind(self) -> None:
        t = torch.tensor([1.0])
        dist.all_reduce(t)  # the rendezvous is a collective: a rank missing here would leave the others waiting
        self.mc = self._mc

    def close(self, barrier: bool = True) -> None:
        _FakeMulticast.closed.append(barrier)


def _agree_worker(rank, world, port, q, case):
    try:
        _init(rank, world, port, timeout_s=30)
        made = [0]

        def make():
            made[0] += 1
            if case == "raises" and rank == 1 and made[0] == 2:  # the second allocation fails on one rank only
                raise RuntimeError("out of memory")
            return _FakeMulticast(0 if case == "no_mc" and rank == 0 else 0x1000 * made[0])

        got = gdist.agree_on_buffers(make, 2)
        # the ranks then take the same next collective step whichever way they went
        t = torch.tensor([1.0])
        dist.all_reduce(t)
        q.put((rank, None if got is None else len(got), list(_FakeMulticast.closed), float(t.item())))
        dist.destroy_process_group()
    except Exception as exc:  # report instead of hanging the parent
        q.put((rank, "error", repr(exc), 0.0))


@pytest.mark.parametrize("case", ["ok", "raises", "no_mc"])
def test_ranks_agree_on_the_multicast_buffers(case):
    """PeerAdam's choice of the multicast form: the same answer on every rank, also when an allocation fails or a
    buffer lacks a multicast address on one rank only; what was made is closed without a barrier. The failure is
    injected on the host, in the buffer factory, whose bind() runs a collective as the rendezvous does: a rank
    that skipped it while the other entered it would leave the test waiting for the process-group timeout."""
    ctx = mp.get_context("spawn")
    q = ctx.Queue()
    port = _free_port()
    procs = [ctx.Process(target=_agree_worker, args=(r, 2, port, q, case)) for r in range(2)]
    for p in procs:
        p.start()
    res = sorted(q.get(timeout=120) for _ in procs)
    for p in procs:
        p.join(timeout=60)
    for rank, got, closed, total in res:
        assert got != "error", closed
        assert total == 2.0
        if case == "ok":
            assert got == 2 and closed == []
        else:
            assert got is None
            assert closed and not any(closed)  # closed, and never with a barrier
    assert {r[0] for r in res} == {0, 1}
