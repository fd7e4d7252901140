"""Benchmark of the 3DGS training step on B200, one process per GPU.

    python bench.py [--gpus N] [--steps K] [--warmup W] [--impl ours|reference]
                    [--exchange auto|peer|nvls|compact|nccl]
                    [--workload c3|c2|c4|c1|c5|gs2d|splat2d|blend-bwd|ssim]
    python -m torch.distributed.run --nnodes=1 --nproc-per-node N --master-addr 127.0.0.1 --master-port P \
        bench.py --gpus N --steps K --warmup W

Workload (default c3): the scene of config C3 - 3M Gaussians from 64 isotropic clusters, SH degree 3, seeded
synthetic parameters (no dataset is available) - rendered at 1920x1080 / 60 deg. One step on each rank is the
training step of one view: forward, backward with dL/dimage ~ N(0, 1e-3) (one fixed seeded image whose sign
alternates step to step, so that Adam keeps the scene at its configured state), then Adam over the six parameter groups
(N = 1: one fused Adam launch; N > 1: the gradient exchange and Adam, in the form --exchange names: one peer-memory
kernel per rank, one NVLink-multicast kernel per rank, the peer kernel with compact SH gradients, or NCCL
reduce-scatter + Adam on the slice + all-gather; auto takes the fastest measured at that rank count). The forwards
are bounded (a view's instance count is read back once, in a warm-up step; no timed step waits on the host). Each
rank trains on the configured camera with its own upstream gradient, so the work per GPU is the single-GPU step's
as N grows (weak scaling) and
    value = N * K / (max over ranks of the device time of K steps)  [views/s],  ms_per_step = that time / K.
The Gaussian state (2.8 GB with moments) is far larger than the 126 MB L2, so no flush is needed between steps.
``e2e`` runs the same step through the public API (diff_rasterize + autograd + FusedAdam, the exchange's optimizer
for N > 1) with the upstream gradient copied from pinned host memory every step and the loss read back, starting from
the same configured parameters. After the timed steps the ranks compare a checksum of their parameters
(``params_checksum``). The c3 line also carries ``c4_strong_scaling``: config C4 (1M Gaussians, the fixed 8-view
1280x720 batch split over the N ranks, the views' gradients summed, one exchange + Adam per step) in the same run.

--workload c2 / c4 run the training step on those configs (c4: strong scaling of the 8-view batch). c1 measures the
toy2d fit step, c5 the render-only orbit, ssim the fused L1 + SSIM loss, each with its own metric line and a
roofline object from kernels timed live (splat_time_kernel). gs2d, splat2d and blend-bwd time single kernels on the
reference's own benchmark scenes: this library's, or with --impl reference the reference's own CUDA kernels (its
toy2d and phase0 extensions and Faster-GS's blend_backward_macro_cu, built from its sources for sm_100a into
oracle/_ref by oracle/build.py) on the same inputs and the same GPU.

--impl reference, for the training workloads, times the CPU restatement of the same step (oracle/liboracle.so,
OpenMP over every host core; the reference has no CPU 3DGS path) on rank 0 only: W warm-up and K timed steps, each a
bounded sample (preprocess, binning, preprocess backward and Adam in full, the blend and its backward on tile rows
spread over the image, scaled to the view) sized so that the run takes about --ref-budget seconds; the same metric,
unit and config as this library's arm.
"""
from __future__ import annotations

import argparse
import json
import os
import statistics
import subprocess
import sys
import time
from pathlib import Path

ROOT = Path(__file__).resolve().parent
sys.path.insert(0, str(ROOT))

import numpy as np  # noqa: E402
import torch  # noqa: E402

from __graft_entry__ import load_package  # noqa: E402

load_package()
from gs_b200 import _lib as L  # noqa: E402
from gs_b200 import adam as gs_adam  # noqa: E402
from gs_b200 import dist as gs_dist  # noqa: E402
from gs_b200 import gs3d, scenes  # noqa: E402

METRIC = "fwd+bwd ms/iter (3M Gaussians, 1080p, SH3); train views/s at 1/2/4/8 B200"
LRS = {"means": 1.6e-4, "scales": 5e-3, "rotations": 1e-3, "opacities": 5e-2, "sh0": 2.5e-3, "sh_rest": 2.5e-3}
NAMES = ("means", "scales", "rotations", "opacities", "sh0", "sh_rest")
WIDTHS = (3, 3, 4, 1, 3, 45)  # floats per Gaussian in each group: 59 in total
# dram__bytes_read.sum + dram__bytes_write.sum of one launch on the C3 workload, from one ncu capture each
# (profiles/); None where not captured.
BLEND_BWD_TRAFFIC = 240830464 + 5681408
ADAM_TRAFFIC = 2832050688 + 2067712256
FUSED_TRAFFIC = None  # not captured yet


class Clocks:
    """nvidia-smi sampled every 50 ms; only the samples stamped inside the timed region (mark_start / mark_end) are
    summarised."""

    Q = ("timestamp,index,clocks.sm,clocks.max.sm,power.draw,clocks_event_reasons.active,"
         "clocks_event_reasons.hw_slowdown,clocks_event_reasons.hw_thermal_slowdown,"
         "clocks_event_reasons.sw_thermal_slowdown,clocks_event_reasons.sw_power_cap")

    def __init__(self, gpu_index: int):
        self.gpu = gpu_index
        self.proc = None
        self.t0 = self.t1 = None

    def __enter__(self):
        try:
            self.proc = subprocess.Popen(["nvidia-smi", "-i", str(self.gpu), f"--query-gpu={self.Q}",
                                          "--format=csv,noheader,nounits", "-lms", "50"],
                                         stdout=subprocess.PIPE, stderr=subprocess.DEVNULL, text=True)
            time.sleep(0.5)  # nvidia-smi takes a moment to start sampling
        except OSError:
            self.proc = None
        return self

    def mark_start(self) -> None:
        import datetime

        self.t0 = datetime.datetime.now()

    def mark_end(self) -> None:
        import datetime

        self.t1 = datetime.datetime.now()

    def __exit__(self, *exc):
        self.rows = []
        if self.proc is None:
            return False
        time.sleep(0.1)
        self.proc.terminate()
        out, _ = self.proc.communicate(timeout=10)
        import datetime

        for line in out.splitlines():
            parts = [p.strip() for p in line.split(",")]
            if len(parts) < 10:
                continue
            try:
                ts = datetime.datetime.strptime(parts[0], "%Y/%m/%d %H:%M:%S.%f")
            except ValueError:
                continue
            self.rows.append((ts, parts[1:]))
        return False

    def summary(self) -> dict:
        rows = getattr(self, "rows", [])
        inside = [r for ts, r in rows if self.t0 is not None and self.t1 is not None and self.t0 <= ts <= self.t1]
        note = "samples inside the timed region"
        if not inside and rows and self.t0 is not None:  # a region shorter than the sampling period: the nearest
            inside = [min(rows, key=lambda tr: abs((tr[0] - self.t0).total_seconds()))[1]]
            note = "no sample fell inside the timed region; the nearest one"
        if not inside:
            return {"sm_mhz": None, "sm_max_mhz": None, "reasons": ["unsampled"]}
        sm = [float(r[1]) for r in inside if r[1].replace(".", "").isdigit()]
        mx = [float(r[2]) for r in inside if r[2].replace(".", "").isdigit()]
        pw = [float(r[3]) for r in inside if r[3].replace(".", "").isdigit()]
        reasons = set()
        for r in inside:
            for name, v in zip(("hw_slowdown", "hw_thermal_slowdown", "sw_thermal_slowdown", "sw_power_cap"), r[5:9]):
                if v.lower() == "active":
                    reasons.add(name)
        return {"sm_mhz": statistics.median(sm) if sm else None, "sm_max_mhz": max(mx) if mx else None,
                "reasons": sorted(reasons), "samples": len(inside), "power_w": statistics.median(pw) if pw else None,
                "note": note}


def setup_dist(n_gpus: int):
    world = int(os.environ.get("WORLD_SIZE", "1"))
    rank = int(os.environ.get("RANK", "0"))
    local = int(os.environ.get("LOCAL_RANK", "0"))
    if world > 1:
        import datetime

        torch.cuda.set_device(local)
        torch.distributed.init_process_group("nccl", timeout=datetime.timedelta(seconds=300),
                                             device_id=torch.device("cuda", local))
    else:
        torch.cuda.set_device(0)
    return world, rank, local


def scene_for(workload: str, rank: int, world: int):
    if workload == "c3":
        # Weak scaling: every rank trains on the configured view with its own upstream gradient (view_seed), so a
        # GPU's work per step is the N = 1 step's and the scaling measures what the exchange costs. (Distinct views
        # per rank, whose costs differ, are the C4 batch of the c4_strong_scaling object.)
        sc = scenes.gs3d_config("c3", seed=0)
        return sc, sc["cameras"][:1]
    if workload == "c4":
        sc = scenes.gs3d_config("c4", seed=0)
        cams = sc["cameras"]
        return sc, [cams[k] for k in range(rank, len(cams), world)]
    if workload == "c2":
        sc = scenes.gs3d_config("c2", seed=0)
        return sc, sc["cameras"]
    raise ValueError(workload)


class Trainer:
    """Replicated Gaussians, flat gradient buffer, Adam state; one training step (of one or several views) per call."""

    def __init__(self, sc: dict, dev, world: int, fuse: bool = False, lean: bool = False, exchange: str = "auto",
                 views: int = 1):
        self.dev = dev
        self.world = world
        self.fuse = fuse and world == 1  # preprocess backward + Adam in one kernel (N > 1: the exchange kernel)
        # the reference's lean Adam: visibility-sparse, bfloat16 moments for the SH-rest group (N = 1 only)
        self.lean = lean and world == 1 and not self.fuse
        self.bases = sc["active_sh_bases"]
        self.peer = None
        self.exchange = None
        if world > 1:  # the gradient exchange and Adam: peer-memory kernel, NVLink multicast kernel or NCCL
            self.exchange = gs_dist.exchange_for(world, exchange, records=True)  # its backward writes records
            self.peer = gs_dist.make_exchange([sc[k].to(dev).contiguous() for k in NAMES], [LRS[k] for k in NAMES],
                                              form=self.exchange, eps=1e-15, views=views,
                                              active_sh_bases=self.bases)
            self.params, self.grads = self.peer.params, self.peer.grads
        else:
            self.params = [sc[k].to(dev).contiguous() for k in NAMES]
            self.flat = torch.zeros(59 * self.params[0].shape[0], device=dev)
            self.grads, off = [], 0
            for p, w in zip(self.params, WIDTHS):
                self.grads.append(self.flat[off:off + w * p.shape[0]].view(p.shape))
                off += w * p.shape[0]
            lowp = [self.lean and nm == "sh_rest" for nm in NAMES]
            self.m = [torch.zeros_like(p, dtype=torch.bfloat16 if lo else p.dtype) for p, lo in zip(self.params, lowp)]
            self.v = [torch.zeros_like(p, dtype=torch.bfloat16 if lo else p.dtype) for p, lo in zip(self.params, lowp)]
        self.n = self.params[0].shape[0]
        self.t = 0
        self.settings = {}
        # Bounded forwards (no host read of the instance count): a view's first forward reads M back; later ones
        # size their instance buffers for 1.25 M + 64K and read M on the device. `overflow` is checked once after
        # the timed steps (check_capacity).
        self.capacity = {}
        self.overflow = torch.zeros(1, dtype=torch.int32, device=dev)
        self.ev = {k: [] for k in ("fwd", "bwd", "comm", "xkernel", "adam", "blend_bwd")}
        self.last = None

    def _settings(self, cam: dict):
        key = id(cam)  # the camera's settings are staged on the device once, as a training loop keeps them
        if key not in self.settings:
            self.settings[key] = scenes.settings_tuple(cam, self.bases, self.dev)
        return self.settings[key]

    def step(self, cam: dict, dout: torch.Tensor, timed: bool):
        """One view: forward, backward, then the optimizer (N > 1: the exchange and Adam)."""
        return self.step_batch([cam], [dout], timed)[0]

    def step_batch(self, cams: list, douts: list, timed: bool) -> list:
        """The views of one batch on this rank: forward and backward of each, their gradients summed into the flat
        buffer (the first view stores, the others accumulate), then one optimizer step. Returns the instance counts.
        Timed stages, per step: fwd and bwd summed over the batch's views, blend_bwd (the blend backward with the
        clear of its sums), comm (N > 1: the exchange with Adam), adam (N = 1)."""
        mk = lambda: torch.cuda.Event(enable_timing=True)  # noqa: E731
        views, insts = [], []
        self.t += 1
        for k, (cam, dout) in enumerate(zip(cams, douts)):
            s = self._settings(cam)
            fs, fe, bs, be = (mk(), mk(), mk(), mk()) if timed else (None, None, None, None)
            if timed:
                fs.record()
            cap = self.capacity.get(id(cam))
            image, prim, tile, inst, bucket, m, nb, sel = gs3d.forward(*self.params, *s, capacity=cap,
                                                                       overflow=self.overflow)
            if cap is None:
                self.capacity[id(cam)] = m + m // 4 + 65536
            if timed:
                fe.record()
            self.last = (prim, tile, m, cam)
            insts.append(m)
            if self.fuse:  # one view: the blend backward, then the preprocess backward fused with Adam ("adam")
                pend = gs3d.backward_blend(None, dout, image, self.params[0], self.params[1], self.params[2],
                                           self.params[3], self.params[5], prim, tile, inst, bucket, *s, m, nb, sel)
                if timed:
                    bs.record()
                pend.preprocess_adam(self.params, self.m, self.v, [LRS[nm] for nm in NAMES], [self.t] * 6,
                                     (0.9, 0.999), 1e-15)
                if timed:
                    be.record()
                    for key, pairs in (("fwd", [(fs, fe)]), ("bwd", [(fe, bs)]), ("blend_bwd", [(fe, bs)]),
                                       ("comm", []), ("adam", [(bs, be)])):
                        self.ev[key].append(pairs)
                return insts
            records = self.peer.records[k] if self.exchange == "compact" else None
            gs3d.backward(None, dout, image, self.params[0], self.params[1], self.params[2], self.params[3],
                          self.params[5], prim, tile, inst, bucket, *s, m, nb, sel, out=self.grads,
                          stage_event=bs, accumulate=k > 0, records=records)
            if timed:
                be.record()
            views.append((fs, fe, bs, be))
        cs, ce = (mk(), mk()) if timed else (None, None)
        if timed:
            cs.record()
        if self.peer is not None:  # the exchange and Adam
            self.peer.kernel_events = [] if timed else None  # the exchange kernel alone, without its barriers
            self.peer.step()
        else:
            groups = [(p, g, mm, vv, LRS[nm]) for p, g, mm, vv, nm in zip(self.params, self.grads, self.m, self.v,
                                                                          NAMES)]
            if self.lean:
                gs_adam.adam_step_lean(groups, self.t, visibility=gs3d.primitive_views(prim, self.n)["n_touched"],
                                       eps=1e-15)
            else:
                gs_adam.adam_step(groups, self.t, eps=1e-15)
        if timed:
            ce.record()
            self.ev["fwd"].append([(a, b) for a, b, _, _ in views])
            self.ev["bwd"].append([(b, d) for _, b, _, d in views])
            self.ev["blend_bwd"].append([(b, c) for _, b, c, _ in views])
            self.ev["comm"].append([(cs, ce)] if self.peer is not None else [])
            self.ev["xkernel"].append(list(self.peer.kernel_events) if self.peer is not None else [])
            self.ev["adam"].append([] if self.peer is not None else [(cs, ce)])
        return insts

    def instances_of(self, prim) -> int:
        """The instance count M of the view whose primitive buffer is `prim` (one host read): the bounded forward
        returns its capacity as n_instances."""
        return int(gs3d.primitive_views(prim, self.n)["counters"][0].item())

    def check_capacity(self) -> None:
        """One host read: raise if a bounded forward's instances exceeded its capacity."""
        if int(self.overflow.item()):
            raise RuntimeError("a bounded forward listed more instances than its capacity; the run is invalid")

    def stage_ms(self) -> dict:
        """Mean per-step milliseconds of each stage over the timed steps."""
        return {key: sum(sum(a.elapsed_time(b) for a, b in pairs) for pairs in v) / max(len(v), 1)
                for key, v in self.ev.items()}

    def reset_timing(self) -> None:
        self.ev = {k: [] for k in self.ev}

    def checksum(self) -> dict:
        """Every rank holds the same parameters after a step: per group the float64 sum and sum of squares,
        gathered from every rank and compared exactly (an exchange that lost or misplaced a slice fails here)."""
        local = torch.stack([torch.stack([p.double().sum(), p.double().square().sum()]) for p in self.params])
        if self.world == 1:
            return {"ranks": 1, "identical": True, "sum": float(local[:, 0].sum())}
        got = [torch.empty_like(local) for _ in range(self.world)]
        torch.distributed.all_gather(got, local)
        same = all(torch.equal(got[0], g) for g in got[1:])
        if not same:
            raise RuntimeError("the ranks' parameters differ after the timed steps: the exchange is broken")
        return {"ranks": self.world, "identical": True, "sum": float(local[:, 0].sum())}

    def close(self) -> None:
        if self.peer is not None:
            self.params = self.grads = []
            self.peer.close()
            self.peer = None


def run_config(args, world: int, sc: dict, cams: list) -> dict:
    """The line's config: the same object for this library's arm and the reference arm of one command line."""
    cam = cams[0]
    W, H, n = cam["width"], cam["height"], sc["means"].shape[0]
    what = {"c3": f"3DGS training step of one {W}x{H} view per GPU per step (every GPU the configured camera, with "
                  f"its own upstream gradient), {n} Gaussians, SH3; fwd + bwd + Adam",
            "c2": f"3DGS training step of the {W}x{H} view, {n} Gaussians, SH3; fwd + bwd + Adam",
            "c4": f"3DGS training step of the 8-view {W}x{H} batch sharded over the GPUs, {n} Gaussians, SH3; "
                  f"fwd + bwd of each view, gradients summed, one exchange + Adam"}[args.workload]
    cfg = {"workload": f"{args.workload}: {what}", "gaussians": n, "width": W, "height": H,
           "views_per_gpu_per_step": len(cams), "parallelism": f"dp{world} (views)",
           "l2": "state (59 floats x 4 moments per Gaussian) larger than L2; no flush",
           "adam": "lean: visibility-sparse update, bfloat16 SH-rest moments with stochastic rounding"
                   if args.lean and world == 1 else "dense float32 (every Gaussian, every step)",
           "fused_preprocess_backward_adam": bool(args.fuse and world == 1)}
    if world > 1:
        cfg["exchange"] = gs_dist.exchange_for(world, args.exchange, records=True)  # the trainer's choice
    return cfg


def time_steps(tr: Trainer, cams: list, douts_for, steps: int, warmup: int, world: int, local: int,
               with_clocks: bool = True) -> dict:
    """Warm-up steps, then `steps` timed steps between a barrier and a device synchronisation on each side; the
    device time of the timed region (CUDA events on this rank's stream), its maximum over ranks, the instance
    counts, the launch count, clocks."""
    for _ in range(warmup):
        tr.step_batch(cams, douts_for(tr.t), False)
    torch.cuda.synchronize()
    if world > 1:
        torch.distributed.barrier()
    tr.reset_timing()
    start, end = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
    clk = Clocks(local) if with_clocks else None
    if clk:
        clk.__enter__()
    t0 = time.perf_counter()
    launches0 = L.query("splat_launch_count")
    if clk:
        clk.mark_start()
    start.record()
    insts = []
    for _ in range(steps):
        insts += tr.step_batch(cams, douts_for(tr.t), True)
    end.record()
    torch.cuda.synchronize()
    if clk:
        clk.mark_end()
    launches = L.query("splat_launch_count") - launches0
    wall = time.perf_counter() - t0
    if clk:
        clk.__exit__(None, None, None)
    if world > 1:
        torch.distributed.barrier()
    ms = torch.tensor([start.elapsed_time(end)], device=tr.dev)
    if world > 1:
        torch.distributed.all_reduce(ms, op=torch.distributed.ReduceOp.MAX)
    return {"ms_max": float(ms.item()), "insts": insts, "launches": launches, "wall": wall,
            "clocks": clk.summary() if clk else None, "stage": tr.stage_ms()}


def run_ours(args) -> None:
    world, rank, local = setup_dist(args.gpus)
    dev = torch.device("cuda", local)
    sc, cams = scene_for(args.workload, rank, world)
    cam = cams[0]
    tr = Trainer(sc, dev, world, fuse=args.fuse, lean=args.lean, exchange=args.exchange, views=len(cams))
    # Each view's upstream gradient is the config's fixed random image with its sign alternating step to step: under
    # Adam a fixed gradient would move every parameter by about lr per step in one direction, and after a few hundred
    # steps the scene (visible Gaussians, instances, blend depth) would no longer be the configured one. Alternating
    # signs keep it there, so every timed step (and the end-to-end run, which restarts from the same parameters)
    # renders the configured scene; the work of a step does not depend on the sign.
    hosts = [upstream_gradient(view_seed(args.workload, rank, world, k), c["height"], c["width"])
             for k, c in enumerate(cams)]
    douts = ([h.to(dev) for h in hosts], [(-h).to(dev) for h in hosts])
    r = time_steps(tr, cams, lambda t: douts[t % 2], args.steps, args.warmup, world, local)
    L.check_device_waits(dev)  # a sort wait of the last forward that gave up is reported here, not after the run
    tr.check_capacity()
    stage = r["stage"]
    reach = blend_reach(tr, cam["width"], cam["height"])
    checksum = tr.checksum()

    # end to end through the public API: pinned host upstream gradients in, loss out, every step
    e2e = run_e2e(sc, cams, dev, world, args, tr)
    roof = roofline(tr, stage, reach, cam["width"] * cam["height"])
    exch = exchange_figures(tr, stage, world, dev) if tr.peer is not None else None
    tr.close()
    del tr
    torch.cuda.empty_cache()

    # the benchmark spec's batched-training config C4 beside the headline: the fixed 8-view batch sharded over the
    # ranks (strong scaling), in the same process
    c4 = c4_strong(args, world, rank, local, dev) if args.workload == "c3" and not args.no_c4 else None

    if rank == 0:
        views = world * len(cams) if args.workload != "c4" else 8
        value = views * args.steps / (r["ms_max"] / 1000.0)
        line = {
            "metric": METRIC, "value": round(value, 3), "unit": "views/s", "n_gpus": world, "steps": args.steps,
            "warmup": args.warmup, "ms_per_step": round(r["ms_max"] / args.steps, 4), "higher_is_better": True,
            "scaling": "strong" if args.workload == "c4" else "weak", "vs_baseline": None, "dtype": "f32",
            "data": "synthetic (seeded, config-shaped)", "config": run_config(args, world, sc, cams),
            "instances_per_view": reach["instances"],
            "stage_ms": {k: round(v, 4) for k, v in stage.items()},
            "fwd_bwd_ms": round(stage["fwd"] + stage["bwd"], 4),
            "wall_s": round(r["wall"], 3), "clocks": r["clocks"], "e2e": e2e, "gpu_launches": r["launches"],
            "params_checksum": checksum,
        }
        line.update(roof)
        if exch is not None:
            line["exchange"] = exch
        if c4 is not None:
            line["c4_strong_scaling"] = c4
        line["cpu_baseline"] = cpu_baseline(args, sc, cam) if not args.no_cpu_baseline else None
        print(json.dumps(line), flush=True)
    if world > 1:
        torch.distributed.destroy_process_group()


def view_seed(workload: str, rank: int, world: int, k: int) -> int:
    """Seed of the upstream gradient of this rank's k-th view: per rank for C3 (one view each), per view of the
    batch for C4 (view rank + k * world of the round-robin split)."""
    return rank + k * world if workload == "c4" else rank


def c4_strong(args, world: int, rank: int, local: int, dev) -> dict:
    """Config C4 at this rank count: 1M Gaussians, the 8-view 1280x720 ring batch split round-robin over the ranks
    (8 / N views per rank per step), each view's gradients summed into the flat buffer, one exchange + Adam per step.
    The batch is fixed as N grows (strong scaling): views/s = 8 x steps / (max over ranks of the device time)."""
    sc = scenes.gs3d_config("c4", seed=0)
    cams = gs_dist.shard_views(sc["cameras"], rank, world)
    tr = Trainer(sc, dev, world, exchange=args.exchange, views=len(cams))
    hosts = [upstream_gradient(rank + k * world, c["height"], c["width"]) for k, c in enumerate(cams)]
    douts = ([h.to(dev) for h in hosts], [(-h).to(dev) for h in hosts])
    steps = max(args.steps // 4, 10)
    r = time_steps(tr, cams, lambda t: douts[t % 2], steps, args.warmup, world, local, with_clocks=False)
    L.check_device_waits(dev)
    tr.check_capacity()
    checksum = tr.checksum()
    stage = {k: round(v, 4) for k, v in r["stage"].items()}
    exch = tr.exchange
    tr.close()
    del tr
    torch.cuda.empty_cache()
    return {"workload": "c4: 1M Gaussians, 8 views of 1280x720 per step sharded over the GPUs, one exchange + Adam",
            "value": round(8 * steps / (r["ms_max"] / 1000.0), 3), "unit": "views/s", "scaling": "strong",
            "steps": steps, "warmup": args.warmup, "ms_per_step": round(r["ms_max"] / steps, 4),
            "views_per_gpu_per_step": len(cams), "exchange": exch if world > 1 else None, "stage_ms": stage,
            "gpu_launches": r["launches"], "params_checksum": checksum}


def upstream_gradient(rank: int, H: int, W: int) -> torch.Tensor:
    """The config's upstream gradient dL/dimage ~ N(0, 1e-3), seeded per rank (host, float32 [3, H, W])."""
    return 1e-3 * torch.randn(3, H, W, generator=torch.Generator().manual_seed(77 + rank))


def run_e2e(sc, cams, dev, world, args, tr: Trainer) -> dict:
    """The training step through the public API (diff_rasterize + autograd + FusedAdam at N = 1, the exchange's
    optimizer over the ranks at N > 1), over this rank's views of the step (their losses summed, one backward, one
    optimizer step). Every step copies its views' upstream gradients from pinned host memory (on a copy stream,
    into one of two device buffers per view, issued one step ahead, after the step's first forward is enqueued, so
    that the copies overlap the step's kernels) and copies its loss back into pinned host memory; all of those copies
    sit inside the timed region. The forwards are bounded (no host read of the instance count), as in the
    device-timed run."""
    peer = None
    start = [sc[k].to(dev).contiguous() for k in NAMES]  # the configured scene, as the device-timed run started
    if world > 1:  # the leaves are views of the exchange's parameter buffer; step() takes their .grad
        peer = gs_dist.make_exchange(start, [LRS[nm] for nm in NAMES], form=tr.exchange, eps=1e-15, views=len(cams),
                                     active_sh_bases=sc["active_sh_bases"])
        leaves = [p.requires_grad_(True) for p in peer.params]
    else:  # with fuse_backward the rasterizer's preprocess backward runs inside the optimizer's fused step
        leaves = [p.requires_grad_(True) for p in start]
        lean = {"sparse": True, "lowp_moment_groups": ("sh_rest",)} if tr.lean else {}
        opt = gs_adam.FusedAdam([{"params": [p], "lr": LRS[nm], "name": nm} for p, nm in zip(leaves, NAMES)],
                                lr=0.0, eps=1e-15, fuse_backward=tr.fuse and len(cams) == 1, **lean)
    rank = torch.distributed.get_rank() if world > 1 else 0
    # as in the device-timed run, each view's gradient with its sign alternating step to step
    hosts = [upstream_gradient(view_seed(args.workload, rank, world, k), c["height"], c["width"]).pin_memory()
             for k, c in enumerate(cams)]
    settings = [gs3d.RasterizerSettings(*scenes.settings_tuple(c, tr.bases, dev)) for c in cams]
    # bounded forwards, as in the device-timed run: each view's instance count read once here, its forwards then
    # sized for 1.25 M + 64K instances with the count kept on the device (overflow checked after the timed steps)
    overflow = torch.zeros(1, dtype=torch.int32, device=dev)
    caps = []
    for st in settings:
        m = gs3d.forward(*[p.detach() for p in leaves], *st.as_tuple())[5]
        caps.append(m + m // 4 + 65536)
    compute = torch.cuda.current_stream(dev)
    copier = torch.cuda.Stream(dev)
    dbuf = [[torch.empty_like(h, device=dev) for h in hosts] for _ in range(2)]
    copied = [torch.cuda.Event() for _ in range(2)]
    used = [torch.cuda.Event() for _ in range(2)]
    done = [torch.cuda.Event() for _ in range(2)]
    total = args.warmup + args.steps
    losses = torch.empty(total, dtype=torch.float32).pin_memory()

    def issue_copy(k):
        b = k % 2
        with torch.cuda.stream(copier):
            copier.wait_event(used[b])  # the step that last read these buffers is done with them
            for d, h in zip(dbuf[b], hosts):
                d.copy_(h, non_blocking=True)
            copied[b].record(copier)

    def step(k):
        b = k % 2
        compute.wait_event(copied[b])
        loss = None
        for v, (st, dout) in enumerate(zip(settings, dbuf[b])):
            img = gs3d.diff_rasterize(*leaves, torch.empty(0), st, capacity=caps[v], overflow=overflow)
            # the next step's copies go out once this step's first forward is enqueued
            if v == 0 and k + 1 < total and k + 1 != args.warmup:  # the first timed copy is issued in the region
                issue_copy(k + 1)
            term = (img * dout).sum()
            loss = term if loss is None else loss + term
        if k % 2:
            loss = -loss
        for p in leaves:
            p.grad = None
        loss.backward()
        used[b].record(compute)
        if peer is not None:
            peer.step(grads=[p.grad for p in leaves])
        else:
            opt.step()
        # the loss goes back to the host on the copy stream, so the compute stream does not wait for the copy
        done[b].record(compute)
        with torch.cuda.stream(copier):
            copier.wait_event(done[b])
            losses[k:k + 1].copy_(loss.detach().view(1), non_blocking=True)
            loss.record_stream(copier)

    for e in used:
        e.record(compute)
    issue_copy(0)
    for k in range(args.warmup):
        step(k)
    torch.cuda.synchronize()
    if world > 1:
        torch.distributed.barrier()
    a, b = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
    with Clocks(dev.index) as clk:
        clk.mark_start()
        a.record(compute)
        copier.wait_stream(compute)  # the first timed copy starts after the timed region does
        issue_copy(args.warmup)
        for k in range(args.warmup, total):
            step(k)
        compute.wait_stream(copier)  # the last step's loss has reached the host when the region ends
        b.record(compute)
        torch.cuda.synchronize()
        clk.mark_end()
    assert bool(torch.isfinite(losses).all())
    if int(overflow.item()):
        raise RuntimeError("an end-to-end forward listed more instances than its capacity; the run is invalid")
    ms = torch.tensor([a.elapsed_time(b)], device=dev)
    if world > 1:
        torch.distributed.all_reduce(ms, op=torch.distributed.ReduceOp.MAX)
    if peer is not None:
        for p in leaves:
            p.grad = None
        del leaves
        peer.close()
    gs3d._Rasterize.fused_optimizer = None
    views = 8 if args.workload == "c4" else world * len(cams)
    return {"value": round(views * args.steps / (float(ms.item()) / 1000.0), 3), "unit": "views/s",
            "h2d_bytes_per_step": int(sum(h.numel() for h in hosts) * 4), "d2h_bytes_per_step": 4,
            "clocks": clk.summary(),
            "note": "from the configured scene, as the device-timed run; upstream gradients (sign alternating step to "
                    "step) copied from pinned host memory one step ahead on a copy stream; loss copied back to pinned "
                    "host memory every step, on the copy stream"}


def blend_reach(tr: Trainer, width: int, height: int) -> dict:
    """What the last step's blend backward had to touch: per tile the list positions up to its last contributor
    (min(max_contrib, range length)), the 32-splat buckets those make, and the bucket count of the whole view."""
    prim, tile, _, _ = tr.last
    m = tr.instances_of(prim)
    tv = gs3d.tile_views(tile, width, height)
    rg = tv["ranges"].long()
    reach = torch.minimum(tv["max_contrib"].long(), (rg[:, 1] - rg[:, 0]).clamp(min=0))
    return {"instances": m, "buckets": int(gs3d.primitive_views(prim, tr.n)["counters"][1].item()),
            "reached_positions": int(reach.sum().item()), "reached_buckets": int(((reach + 31) // 32).sum().item())}


def roofline(tr: Trainer, stage: dict, reach: dict, pixels: int) -> dict:
    """Roofline of the kernel with the largest share of the step, each timed live with CUDA events around its call
    in every timed step (k_blend_backward with the clear of its accumulators, or k_adam).
      k_blend_backward: 16 B of checkpoint per pixel of every reached bucket + 28 B per pixel (upstream gradient,
        image, contributor count) + 40 B per reached list position (id, mean2d, conic + opacity, colour) + 36 B per
        Gaussian (accumulator clear). Its limiter is instruction issue (FP32, ex2, shuffles), not HBM: the HBM
        fraction it reports is low by nature; profiles/ holds its issue and pipe utilisation.
      k_adam: 59 floats x 4 B x 7 accesses (param, grad, m, v read; param, m, v written) = 1652 B per Gaussian.
      k_adam_lean (--lean): per visible Gaussian 59 floats of parameter read and written and of gradient read
        (708 B), the 14 float32 moments of the first five groups read and written (224 B) and the 45 bfloat16
        SH-rest moments read and written (360 B): 1292 B, + 4 B of visibility per Gaussian; invisible Gaussians
        are not touched.
      k_preprocess_backward fused with Adam (--fuse): 59 floats x 4 B x 6 accesses (param, m, v read and written)
        + 4 B (n_touched) per Gaussian, + 56 B per visible Gaussian (the blend backward's mean2d, conic + opacity
        and colour sums, colour + depth): 1420 N + 56 V."""
    peaks_path = ROOT / "MEASURED_PEAKS.json"
    hbm, src = 6650.0, "fallback"
    if peaks_path.exists():
        v = json.loads(peaks_path.read_text()).get("hbm_gbs")
        if v:
            hbm, src = float(v), "measured"
    blend = {"kernel": "k_blend_backward (+ accumulator clear)", "ms": stage["blend_bwd"],
             "bytes": 16.0 * 256 * reach["reached_buckets"] + 28.0 * pixels + 40.0 * reach["reached_positions"]
             + 36.0 * tr.n, "traffic": BLEND_BWD_TRAFFIC, "limiter": "issue (FP32 / ex2 / shuffles)"}
    adam = {"kernel": "k_adam", "ms": stage["adam"], "bytes": 1652.0 * tr.n, "traffic": ADAM_TRAFFIC,
            "limiter": "HBM"}
    if tr.lean:
        visible = int((gs3d.primitive_views(tr.last[0], tr.n)["n_touched"] > 0).sum().item())
        adam = {"kernel": "k_adam_lean", "ms": stage["adam"], "bytes": 1292.0 * visible + 4.0 * tr.n,
                "traffic": None, "limiter": "HBM", "visible": visible}
    if tr.fuse:
        visible = int((gs3d.primitive_views(tr.last[0], tr.n)["n_touched"] > 0).sum().item())
        adam = {"kernel": "k_preprocess_backward (fused with Adam)", "ms": stage["adam"],
                "bytes": 1420.0 * tr.n + 56.0 * visible, "traffic": FUSED_TRAFFIC, "limiter": "HBM",
                "visible": visible}
    top, other = (blend, adam) if blend["ms"] >= adam["ms"] or tr.peer is not None else (adam, blend)

    def entry(k):
        ach = k["bytes"] / (k["ms"] / 1000.0) / 1e9 if k["ms"] > 0 else 0.0
        out = {"bound": "hbm", "achieved": round(ach, 1), "peak": hbm, "unit": "GB/s", "frac": round(ach / hbm, 4),
               "traffic": k["traffic"], "kernel": k["kernel"], "kernel_ms": round(k["ms"], 4),
               "algorithmic_bytes": int(k["bytes"]), "limiter": k["limiter"],
               "peak_source": f"{src} (MEASURED_PEAKS.json hbm_gbs)" if src == "measured" else src}
        if "visible" in k:
            out["visible_gaussians"] = k["visible"]
        return out

    out = entry(top)
    if tr.peer is None:  # with N > 1 Adam runs inside the fused exchange kernel instead (see "exchange")
        out["next_kernel"] = entry(other)
    out["blend_reach"] = reach
    return {"roofline": out}


def exchange_figures(tr: Trainer, stage: dict, world: int, dev) -> dict:
    """N > 1: the exchange + Adam of one step, against NVLink (measured 770 GB/s per direction).

    Peer form (adam_step_dp_fused between two barriers): each rank reads its slice's gradients from the other G - 1
    ranks while they read theirs from it, and writes its updated slice to them while they write theirs to it:
    2 (G - 1) slices cross its links in each direction.
    Multicast form (adam_step_dp_nvls between two barriers): the switch reduces, so a rank sends its whole gradient
    buffer (G slices) out and takes its reduced slice in; its multicast store sends one slice out and the switch
    delivers all G slices in: G + 1 slices in each direction.
    NCCL form (reduce-scatter, Adam on the slice, all-gather): a ring reduce-scatter and all-gather each move
    G - 1 slices in each direction: 2 (G - 1), as the peer form.
    Compact form (adam_step_dp_compact between two barriers): a rank owns whole Gaussians; per owned Gaussian it
    reads 11 + 6 V gradient floats (V views per rank) from each of the G - 1 other ranks and writes its 59 parameters
    to each of them."""
    g = tr.world
    form = tr.exchange
    if form == "compact":
        owned = tr.peer.hi - tr.peer.lo
        width = sum(gs_dist.widths(tr.peer.rest))
        cross = (g - 1) * 4.0 * owned * (11 + 6 * tr.peer.views + width)
        vector = 4.0 * tr.peer.n * width
    else:
        slice_bytes = 4.0 * (tr.peer.hi - tr.peer.lo)
        cross = (g + 1) * slice_bytes if form == "nvls" else 2 * (g - 1) * slice_bytes
        vector = 4.0 * tr.peer.total
    kernel = {"nvls": "adam_step_dp_nvls", "peer": "adam_step_dp_fused", "compact": "adam_step_dp_compact",
              "nccl": "ncclReduceScatter + adam_step_dp_fused on the slice + ncclAllGather"}[form]
    # the kernel alone (its barriers excluded) and the whole stage with the barriers, each the maximum over the
    # ranks; the stage also holds a rank's wait for slower ranks at the first barrier
    both = torch.tensor([stage["xkernel"], stage["comm"]], dtype=torch.float64, device=dev)
    if world > 1:
        torch.distributed.all_reduce(both, op=torch.distributed.ReduceOp.MAX)
    t, t_stage = float(both[0]), float(both[1])
    ach = cross / (t / 1000.0) / 1e9 if t > 0 else 0.0
    # the same exchange measured as an all-reduce: bus bandwidth 2 (G - 1) / G x vector bytes / time, against the
    # measured 8-rank NCCL all-reduce bus bandwidth of this pool (725 GB/s at 1 GiB), which also carries no Adam step
    bus = 2.0 * (g - 1) / g * vector / (t / 1000.0) / 1e9 if t > 0 else 0.0
    return {"form": form, "kernel": kernel, "ms": round(t, 4), "stage_ms_with_barriers": round(t_stage, 4),
            "bytes_each_direction": int(cross),
            "achieved": round(ach, 1), "peak": 770.0, "unit": "GB/s", "frac": round(ach / 770.0, 4),
            "peak_source": "measured peer copy, per direction",
            "allreduce_bus_gbs": round(bus, 1), "allreduce_bus_frac_of_nccl": round(bus / 725.0, 4)}


def cpu_baseline(args, sc, cam):
    try:
        from oracle import gs3d_cpu
    except Exception as exc:  # the C restatement is built by __graft_entry__.build()
        return {"value": None, "unit": "views/s", "cores": os.cpu_count(), "kind": "port",
                "sample": f"unavailable: {exc}"}
    return gs3d_cpu.time_training_step(sc, cam, budget_s=args.cpu_budget)


def run_reference(args) -> None:
    """The reference arm: the same metric, unit and config as this library's arm of the same command line, timed on
    the reference's side of the path. For the 3DGS training workloads (c3, c2, c4) that is the CPU restatement
    (oracle/liboracle.so, the reference has no CPU 3DGS path) on every host thread of rank 0 alone: W warm-up and K
    timed steps, each a bounded sample (TrainingStepSample) sized so the run takes about --ref-budget seconds.
    --workload gs2d / splat2d / blend-bwd time the reference's own CUDA kernels instead (built from its sources
    into oracle/_ref), c1 and c5 their CPU paths."""
    world = int(os.environ.get("WORLD_SIZE", "1"))
    rank = int(os.environ.get("RANK", "0"))
    if rank != 0:
        return
    if args.workload in ("gs2d", "splat2d", "blend-bwd"):
        if not torch.cuda.is_available():
            print(json.dumps({"impl": "reference", "unavailable": "the reference's CUDA kernels need a GPU and none "
                                                                  "is visible"}))
            return
        return {"gs2d": run_gs2d, "splat2d": run_splat2d, "blend-bwd": run_blend_bwd}[args.workload](args, ref=True)
    if args.workload == "ssim":
        print(json.dumps({"impl": "reference", "unavailable": "the reference's SSIM is the external fused-ssim "
                                                              "package, which the reference does not vendor"}))
        return
    if args.workload in ("c1", "c5"):
        return {"c1": run_c1, "c5": run_c5}[args.workload](args, ref=True)
    from oracle import gs3d_cpu

    sc, cams = scene_for(args.workload, 0, world)
    views_per_step = 8 if args.workload == "c4" else world * len(cams)
    smp = gs3d_cpu.TrainingStepSample(sc, cams[0])
    per_step = max(1.0, args.ref_budget / max(args.steps + args.warmup, 1))
    t0 = time.perf_counter()
    smp.calibrate(per_step)  # the first warm-up step
    for _ in range(args.warmup - 1):
        smp.step()
    runs = [smp.step() for _ in range(args.steps)]
    wall = time.perf_counter() - t0
    # one view's step; a step of the whole job renders views_per_step views, each with its own preprocess, binning,
    # blend and preprocess backward, and applies Adam once
    secs = [views_per_step * (r["seconds"] - r["parts"]["adam"]) + r["parts"]["adam"] for r in runs]
    step_s = float(statistics.median(secs))
    value = views_per_step / step_s
    res = {"value": round(value, 5), "unit": "views/s", "cores": smp.threads, "kind": "port",
           "sample": smp.describe() + (f"; x{views_per_step} views per step" if views_per_step > 1 else ""),
           "seconds_per_view": {k: round(float(statistics.median(r["parts"][k] for r in runs)), 3)
                                for k in runs[0]["parts"]}}
    line = {"metric": METRIC, "value": round(value, 5), "unit": "views/s", "n_gpus": world, "steps": args.steps,
            "warmup": args.warmup, "ms_per_step": round(1000.0 * step_s, 3), "higher_is_better": True,
            "scaling": "strong" if args.workload == "c4" else "weak", "vs_baseline": None, "dtype": "f32",
            "data": "synthetic (seeded, config-shaped)", "config": run_config(args, world, sc, cams),
            "instances_per_view": runs[0]["instances"], "impl": "reference", "cpu_baseline": res,
            "wall_s": round(wall, 3),
            "e2e": {"value": round(value, 5), "unit": "views/s", "h2d_bytes_per_step": 0, "d2h_bytes_per_step": 0}}
    print(json.dumps(line), flush=True)


# ---------------------------------------------------------------------------------------------
# Other configs of the benchmark spec, measured on request (--workload c1 | c5); the headline stays C3.
# ---------------------------------------------------------------------------------------------

def c1_inputs(dev):
    """Config C1: 4096 anisotropic 2D Gaussians (activated as the spec prescribes), 256x256, black background,
    a 32-sinusoid target; float32 on the device."""
    from gs_b200 import gs2d

    sc = scenes.gs2d_c1(0)
    var = torch.exp(2.0 * sc["log_scale"])
    cos, sin = torch.cos(sc["theta"]), torch.sin(sc["theta"])
    cxx = cos * cos * var[:, 0] + sin * sin * var[:, 1]
    cxy = cos * sin * (var[:, 0] - var[:, 1])
    cyy = sin * sin * var[:, 0] + cos * cos * var[:, 1]
    det = cxx * cyy - cxy * cxy
    conic = torch.stack([cyy / det, -cxy / det, cxx / det], -1)
    radii = gs2d.radii_from_cov(torch.stack([cxx, cxy, cyy], -1))
    f = lambda t: t.to(dev, torch.float32).contiguous()  # noqa: E731
    return (sc, f(sc["xy"]), f(conic), f(sc["rgb"]), f(torch.sigmoid(sc["opacity_logit"])), radii.to(dev),
            f(sc["depth"]), sc["target"].to(torch.float32))


def hbm_peak() -> tuple[float, str]:
    peaks_path = ROOT / "MEASURED_PEAKS.json"
    if peaks_path.exists():
        v = json.loads(peaks_path.read_text()).get("hbm_gbs")
        if v:
            return float(v), "measured (MEASURED_PEAKS.json hbm_gbs)"
    return 6650.0, "fallback"


def hbm_roofline(kernel: str, ms: float, nbytes: float, traffic, limiter: str, **extra) -> dict:
    peak, src = hbm_peak()
    ach = nbytes / (ms / 1000.0) / 1e9 if ms > 0 else 0.0
    out = {"bound": "hbm", "achieved": round(ach, 1), "peak": peak, "unit": "GB/s", "frac": round(ach / peak, 4),
           "traffic": traffic, "kernel": kernel, "kernel_ms": round(ms, 4), "algorithmic_bytes": int(nbytes),
           "limiter": limiter, "peak_source": src}
    out.update(extra)
    return out


def run_c1(args, ref: bool = False) -> None:
    """One toy2d fit step per step: binning, forward and splat backward of the C1 scene against its target (L2).
    With ref: the reference's CPU path, restated in numpy float64 (oracle/gs2d_oracle.py, pinned to the reference's
    own outputs): W warm-up and K timed full fit steps, one thread."""
    from gs_b200 import gs2d

    if ref:
        sc, means, conic, color, opacity, radii, depth, target = c1_inputs(torch.device("cpu"))
        for _ in range(args.warmup):
            c1_cpu(sc, means, conic, color, opacity, radii, depth, target)
        runs = [c1_cpu(sc, means, conic, color, opacity, radii, depth, target) for _ in range(args.steps)]
        v = float(statistics.median(r["value"] for r in runs))
        print(json.dumps({"metric": "toy2d fit step (4096 Gaussians, 256x256): fits/s", "value": round(v, 4),
                          "unit": "fits/s", "n_gpus": 1, "steps": args.steps, "warmup": args.warmup,
                          "ms_per_step": round(1000.0 / v, 3), "higher_is_better": True,
                          "scaling": "replicas only", "vs_baseline": None, "dtype": "f64",
                          "data": "synthetic (seeded, config-shaped)", "config": C1_CONFIG, "impl": "reference",
                          "cpu_baseline": runs[0],
                          "e2e": {"value": round(v, 4), "unit": "fits/s", "h2d_bytes_per_step": 0,
                                  "d2h_bytes_per_step": 0}}), flush=True)
        return
    torch.cuda.set_device(0)
    dev = torch.device("cuda", 0)
    sc, means, conic, color, opacity, radii, depth, target = c1_inputs(dev)
    H, W = sc["H"], sc["W"]
    leaves = [t.clone().requires_grad_(True) for t in (means, conic, color, opacity)]
    # One exact binning at setup sizes the step's bounded binning (no host read per step) and gives M and B for the
    # byte counts below. The parameters do not change between steps (the step has no optimizer), so M does not
    # either; the capacity leaves 50% headroom and any overflow is checked after the timed steps.
    exact = gs2d.bin_gaussians(means, radii, depth, H, W)
    M, B, P = int(exact.point_list.numel()), int(exact.num_buckets), H * W
    capacity = M + M // 2 + 1024
    static_tgt = target.reshape(3, H, W).to(dev).contiguous()
    last = {}

    def step():
        bins = gs2d.bin_gaussians(leaves[0].detach(), radii, depth, H, W, capacity=capacity)
        last["bins"] = bins
        img = gs2d.rasterize(*leaves, bins, backend="splat")
        loss = ((img - static_tgt) ** 2).mean()
        for p in leaves:
            p.grad = None
        loss.backward()
        return loss

    # warm-up on a side stream (as CUDA graph capture asks), then the step captured once as a CUDA graph: a step is
    # one replay, with no host work or host read inside it
    side = torch.cuda.Stream(dev)
    side.wait_stream(torch.cuda.current_stream(dev))
    with torch.cuda.stream(side):
        for _ in range(max(args.warmup, 3)):
            step()
    torch.cuda.current_stream(dev).wait_stream(side)
    torch.cuda.synchronize()
    graph = torch.cuda.CUDAGraph()
    launches0 = L.query("splat_launch_count")
    with torch.cuda.graph(graph):
        static_loss = step()
    per_step_launches = L.query("splat_launch_count") - launches0
    for _ in range(args.warmup):
        graph.replay()
    torch.cuda.synchronize()
    a, b = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
    a.record()
    for _ in range(args.steps):
        graph.replay()
    b.record()
    torch.cuda.synchronize()
    ms = a.elapsed_time(b) / args.steps
    launches = per_step_launches * args.steps
    last["bins"].check()  # no step's instances exceeded the capacity
    # the two kernels' device times, from eager steps (event pairs around each launch)
    timer = L.KernelTimer("gs2d_k_render", "gs2d_k_backward_splat")
    for _ in range(min(args.steps, 50)):
        timer.arm()
        step()
    torch.cuda.synchronize()
    timer.stop()
    kt = {k: float(statistics.median(v)) for k, v in timer.times().items()}
    # forward (saving bucket states): 40 B per list entry (id + 9 splat floats), 20 B per pixel (image, T, count),
    # 4 KB per bucket of (T, C) states; backward: the states, 28 B per pixel, 40 B per list entry
    fwd = hbm_roofline("gs2d k_render (forward, bucket states saved)", kt["gs2d_k_render"],
                       40.0 * M + 20.0 * P + 4096.0 * B, None,
                       "latency / issue: the whole working set fits in L2, so HBM is not the bound")
    bwd = hbm_roofline("gs2d k_backward_splat", kt["gs2d_k_backward_splat"], 4096.0 * B + 28.0 * P + 40.0 * M, None,
                       "latency / issue: the whole working set fits in L2, so HBM is not the bound")
    top, other = (fwd, bwd) if fwd["kernel_ms"] >= bwd["kernel_ms"] else (bwd, fwd)
    top["next_kernel"] = other
    top["step_share"] = round((fwd["kernel_ms"] + bwd["kernel_ms"]) / ms, 4)
    # end to end: each step copies its target from pinned host memory into the graph's input and reads its loss back
    host = target.reshape(3, H, W).contiguous().pin_memory()
    losses = torch.empty(args.steps, dtype=torch.float32).pin_memory()
    a2, b2 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
    a2.record()
    for k in range(args.steps):
        static_tgt.copy_(host, non_blocking=True)
        graph.replay()
        losses[k:k + 1].copy_(static_loss.detach().view(1), non_blocking=True)
    b2.record()
    torch.cuda.synchronize()
    ms_e2e = a2.elapsed_time(b2) / args.steps
    line = {"metric": "toy2d fit step (4096 Gaussians, 256x256): fits/s", "value": round(1000.0 / ms, 2),
            "unit": "fits/s", "n_gpus": 1, "steps": args.steps, "warmup": args.warmup, "ms_per_step": round(ms, 4),
            "higher_is_better": True, "scaling": "replicas only", "vs_baseline": None, "dtype": "f32",
            "data": "synthetic (seeded, config-shaped)", "config": C1_CONFIG,
            "e2e": {"value": round(1000.0 / ms_e2e, 2), "unit": "fits/s", "h2d_bytes_per_step": int(host.numel() * 4),
                    "d2h_bytes_per_step": 4},
            "gpu_launches": launches, "host_reads_per_step": 0,
            "binning": {"mode": "bounded (no host read)", "capacity": capacity, "instances": M, "buckets": B},
            "roofline": top}
    graph.reset()
    if not args.no_cpu_baseline:
        line["cpu_baseline"] = c1_cpu(sc, means, conic, color, opacity, radii, depth, target)
    print(json.dumps(line), flush=True)


C1_CONFIG = {"workload": "c1: binning + forward + splat backward of 4096 2D Gaussians, 256x256, L2 loss",
             "l2": "the whole working set fits in L2; steps run back to back",
             "step": "one CUDA graph replay: bounded binning (no host read), forward, loss, splat backward"}


def c1_cpu(sc, means, conic, color, opacity, radii, depth, target) -> dict:
    """The numpy restatement of the toy2d op (oracle/gs2d_oracle.py): binning, forward, backward, one step."""
    from oracle import gs2d_oracle as G

    H, W = sc["H"], sc["W"]
    c = lambda t: t.detach().cpu().double().numpy()  # noqa: E731
    t0 = time.perf_counter()
    b = G.bin_gaussians(c(means), radii.cpu().numpy(), c(depth), H, W)
    fwd = G.forward(c(means), c(conic), c(color), c(opacity), np.zeros(3), b)
    dout = 2.0 * (fwd.out - target.reshape(3, H, W).double().numpy()) / fwd.out.size
    G.backward(c(means), c(conic), c(color), c(opacity), np.zeros(3), b, fwd, dout)
    s = time.perf_counter() - t0
    return {"value": round(1.0 / s, 4), "unit": "fits/s", "cores": 1, "kind": "port",
            "sample": "one full fit step (binning, forward, backward) in numpy float64, one thread"}


C5_METRIC = "render-only frames/s (6M Gaussians, 3840x2160, 120-frame orbit)"
C5_CONFIG = {"workload": "c5: gs3d.inference per frame of the orbit, frames round-robin over ranks",
             "l2": "parameters (1.4 GB) larger than L2; no flush"}


def run_c5(args, ref: bool = False) -> None:
    """Render-only throughput of config C5: the 120-frame orbit, frames split round-robin over the ranks (replicas
    only: frames are independent). With ref: the C++ restatement's render of the orbit's frames on every host thread
    of rank 0 (preprocess and binning in full, the blend on a band of tile rows, scaled to the frame), W warm-up and
    K timed frames."""
    world, rank, local = setup_dist(args.gpus) if not ref else (int(os.environ.get("WORLD_SIZE", "1")),
                                                                int(os.environ.get("RANK", "0")), 0)
    sc = scenes.gs3d_config("c5", seed=0)
    if ref:
        from oracle import gs3d_cpu

        per = max(1.0, args.ref_budget / max(args.steps + args.warmup, 1))
        res = [gs3d_cpu.time_render_frame(sc, sc["cameras"][k % 120], budget_s=per)
               for k in range(args.warmup + args.steps)][args.warmup:]
        v = float(statistics.median(r["value"] for r in res))
        print(json.dumps({"metric": C5_METRIC, "value": round(v, 5), "unit": "frames/s", "n_gpus": world,
                          "steps": args.steps, "warmup": args.warmup, "ms_per_step": round(1000.0 / v, 3),
                          "higher_is_better": True, "scaling": "weak (replicas only)", "vs_baseline": None,
                          "dtype": "f32", "data": "synthetic (seeded, config-shaped)", "config": C5_CONFIG,
                          "impl": "reference", "cpu_baseline": res[0],
                          "e2e": {"value": round(v, 5), "unit": "frames/s", "h2d_bytes_per_step": 0,
                                  "d2h_bytes_per_step": 0}}), flush=True)
        return
    dev = torch.device("cuda", local)
    params = [sc[k].to(dev).contiguous() for k in NAMES]
    cams = gs_dist.shard_views(sc["cameras"], rank, world)
    sets = [scenes.settings_tuple(c, sc["active_sh_bases"], dev) for c in cams]
    for k in range(args.warmup):
        gs3d.inference(*params, *sets[k % len(sets)])
    torch.cuda.synchronize()
    if world > 1:
        torch.distributed.barrier()
    frames = min(args.steps, len(sets))
    timer = L.KernelTimer("k_preprocess", "k_duplicate", "k_blend")
    a, b = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
    with Clocks(local) as clk:
        launches0 = L.query("splat_launch_count")
        clk.mark_start()
        a.record()
        for k in range(frames):
            timer.arm()
            gs3d.inference(*params, *sets[k])
        b.record()
        torch.cuda.synchronize()
        clk.mark_end()
        launches = L.query("splat_launch_count") - launches0
    timer.stop()
    L.check_device_waits(dev)
    ms = torch.tensor([a.elapsed_time(b)], device=dev)
    if world > 1:
        torch.distributed.all_reduce(ms, op=torch.distributed.ReduceOp.MAX)
    kt = timer.times()
    # per frame (untimed): visible Gaussians V and instances M, for the kernels' algorithmic bytes
    n, P = params[0].shape[0], cams[0]["width"] * cams[0]["height"]
    vis, inst = [], []
    for k in range(frames):
        _, prim, _, _, _, m, _, _ = gs3d.forward(*params, *sets[k])
        vis.append(int((gs3d.primitive_views(prim, n)["n_touched"] > 0).sum().item()))
        inst.append(m)
        del prim
    V, M = float(np.mean(vis)), float(np.mean(inst))
    # preprocess: 44 B per Gaussian (geometry, opacity) + 192 B of SH per visible one read, 52 B per visible one
    # written; duplicate: 12 B per visible Gaussian read, 8 B per instance written (tile key, id); render-only blend:
    # 40 B per list entry (id, mean2d, conic + opacity, colour), 12 B per pixel written (image)
    kms = {k: float(np.mean(v)) for k, v in kt.items()}
    entries = [
        hbm_roofline("k_preprocess", kms["k_preprocess"], 44.0 * n + 244.0 * V, None, "HBM"),
        hbm_roofline("k_duplicate", kms["k_duplicate"], 12.0 * V + 8.0 * M, None, "HBM / latency"),
        hbm_roofline("k_blend (render-only)", kms["k_blend"], 40.0 * M + 12.0 * P, None,
                     "issue (FP32 / ex2): its HBM fraction is low by nature"),
    ]
    entries.sort(key=lambda e: -e["kernel_ms"])
    top = entries[0]
    top["other_kernels"] = entries[1:]
    top["frame_share"] = round(sum(e["kernel_ms"] for e in entries) / (float(ms.item()) / frames), 4)
    top["visible_gaussians"], top["instances"] = round(V), round(M)
    # end to end: every frame's image copied back to pinned host memory, on a copy stream into two alternating
    # pinned buffers, so that frame k's copy over PCIe overlaps the rendering of frame k + 1; the end event waits
    # for the last copy
    outs = [torch.empty(3, cams[0]["height"], cams[0]["width"]).pin_memory() for _ in range(2)]
    out = outs[0]
    copier = torch.cuda.Stream(dev)
    main = torch.cuda.current_stream(dev)
    a2, b2 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
    a2.record()
    for k in range(frames):
        img = gs3d.inference(*params, *sets[k])
        copier.wait_stream(main)
        with torch.cuda.stream(copier):
            outs[k % 2].copy_(img, non_blocking=True)
        img.record_stream(copier)
    main.wait_stream(copier)
    b2.record()
    torch.cuda.synchronize()
    ms2 = torch.tensor([a2.elapsed_time(b2)], device=dev)
    if world > 1:
        torch.distributed.all_reduce(ms2, op=torch.distributed.ReduceOp.MAX)
    if rank == 0:
        total = world * frames
        line = {"metric": C5_METRIC,
                "value": round(total / (float(ms.item()) / 1000.0), 3), "unit": "frames/s", "n_gpus": world,
                "steps": frames, "warmup": args.warmup, "ms_per_step": round(float(ms.item()) / frames, 4),
                "higher_is_better": True, "scaling": "weak (replicas only)", "vs_baseline": None, "dtype": "f32",
                "data": "synthetic (seeded, config-shaped)", "config": C5_CONFIG,
                "e2e": {"value": round(total / (float(ms2.item()) / 1000.0), 3), "unit": "frames/s",
                        "h2d_bytes_per_step": 0, "d2h_bytes_per_step": int(out.numel() * 4)},
                "gpu_launches": launches, "clocks": clk.summary(), "roofline": top}
        if not args.no_cpu_baseline:
            from oracle import gs3d_cpu

            line["cpu_baseline"] = gs3d_cpu.time_render_frame(sc, sc["cameras"][0], budget_s=args.cpu_budget)
        print(json.dumps(line), flush=True)
    if world > 1:
        torch.distributed.destroy_process_group()


def run_ssim(args) -> None:
    """The fused L1 + SSIM loss beside the rasterizer (the fused-ssim step of the reference's training loop, with
    lambda_dssim = 0.2): forward and backward of gs_b200.loss.l1_ssim_loss on one 3 x 1080 x 1920 image per step,
    through the autograd op as a training loop calls it. The two images (50 MB) fit in L2, so a 256 MB buffer is
    written before every timed step, and the step's own CUDA events bracket it alone (a short device-side sleep
    after the flush lets the host queue the step, so host overhead is not timed as device time). Algorithmic
    bytes per element of the image: forward 8 read (image, target) + 12 written (three derivative maps), backward
    20 read (maps, image, target) + 4 written (gradient): 44 B."""
    from gs_b200 import loss as gs_loss

    dev = torch.device("cuda", 0)
    torch.cuda.set_device(dev)
    H, W = 1080, 1920
    g = torch.Generator().manual_seed(11)
    gt_h = torch.rand(1, 3, H, W, generator=g)
    img_h = (gt_h + 0.05 * torch.randn(1, 3, H, W, generator=g)).clamp(0.0, 1.0)
    gt = gt_h.to(dev)
    img = img_h.to(dev).requires_grad_(True)

    def step(y):
        img.grad = None
        loss = gs_loss.l1_ssim_loss(img, y, 0.2)
        loss.backward()
        return loss

    for _ in range(args.warmup):
        step(gt)
    torch.cuda.synchronize()
    flush = torch.empty(64 * 1024 * 1024, dtype=torch.float32, device=dev)  # 256 MB, twice the L2
    pairs = [(torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)) for _ in range(args.steps)]
    with Clocks(0) as clk:
        launches0 = L.query("splat_launch_count")
        clk.mark_start()
        for a, b in pairs:
            flush.zero_()
            torch.cuda._sleep(200_000)
            a.record()
            step(gt)
            b.record()
        torch.cuda.synchronize()
        clk.mark_end()
        launches = L.query("splat_launch_count") - launches0
    ms = sum(a.elapsed_time(b) for a, b in pairs) / args.steps
    # end to end: the target copied from pinned host memory every step (as a training loop loads it), the loss
    # copied back into pinned host memory, steps back to back
    host = gt_h.contiguous().pin_memory()
    gt_d = torch.empty_like(gt)
    losses = torch.empty(args.steps, dtype=torch.float32).pin_memory()
    a2, b2 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
    a2.record()
    for k in range(args.steps):
        gt_d.copy_(host, non_blocking=True)
        losses[k:k + 1].copy_(step(gt_d).detach().view(1), non_blocking=True)
    b2.record()
    torch.cuda.synchronize()
    ms_e2e = a2.elapsed_time(b2) / args.steps
    elems = 3 * H * W
    peaks_path = ROOT / "MEASURED_PEAKS.json"
    hbm, src = 6650.0, "fallback"
    if peaks_path.exists():
        v = json.loads(peaks_path.read_text()).get("hbm_gbs")
        if v:
            hbm, src = float(v), "measured (MEASURED_PEAKS.json hbm_gbs)"
    achieved = 44.0 * elems / (ms / 1000.0) / 1e9
    line = {"metric": "fused L1 + SSIM loss, forward + backward, 3 x 1080 x 1920: evaluations/s",
            "value": round(1000.0 / ms, 2), "unit": "evaluations/s", "n_gpus": 1, "steps": args.steps,
            "warmup": args.warmup, "ms_per_step": round(ms, 4), "higher_is_better": True, "scaling": "replicas only",
            "vs_baseline": None, "dtype": "f32", "data": "synthetic (seeded target, image = target + noise)",
            "config": {"workload": "ssim: l1_ssim_loss(img, gt, 0.2) forward + backward per step, 11x11 window",
                       "l2": "256 MB written before every timed step (the images fit in L2)"},
            "roofline": {"bound": "hbm", "achieved": round(achieved, 1), "peak": hbm, "unit": "GB/s",
                         "frac": round(achieved / hbm, 4), "traffic": None,
                         "kernel": "k_ssim_forward + k_ssim_backward (one step)",
                         "algorithmic_bytes": int(44 * elems), "peak_source": src},
            "e2e": {"value": round(1000.0 / ms_e2e, 2), "unit": "evaluations/s",
                    "h2d_bytes_per_step": int(host.numel() * 4), "d2h_bytes_per_step": 4},
            "clocks": clk.summary(), "gpu_launches": launches}
    print(json.dumps(line), flush=True)


# The reference's toy2d kernel timings on an H100 (toy2d/results/bench-cfda5b4-4473561.json): (size, n) ->
# (forward, forward saving buckets, backward pixel, backward splat) in ms, CUDA-event medians.
GS2D_H100_MS = {
    (512, 10000): (0.0760, 0.0814, 0.3039, 0.1671), (512, 50000): (0.0895, 0.0956, 0.2410, 0.2572),
    (512, 200000): (0.1912, 0.2227, 0.2844, 0.4969), (1024, 10000): (0.0866, 0.1007, 1.1088, 0.3631),
    (1024, 50000): (0.1259, 0.1463, 0.8664, 0.4918), (1024, 200000): (0.2252, 0.2700, 0.7995, 0.8257),
}


def median_ms(fn, warmup: int, iters: int) -> float:
    """Median CUDA-event time of fn() on the current stream, after warm-up calls."""
    for _ in range(warmup):
        fn()
    times = []
    for _ in range(iters):
        a, b = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
        a.record()
        fn()
        b.record()
        torch.cuda.synchronize()
        times.append(a.elapsed_time(b))
    return float(statistics.median(times))


def load_reference_module(name: str):
    """The reference's own CUDA extension built by oracle/build.py into oracle/_ref/<name>/<name>.so (its toy2d and
    phase0 kernels), imported from the built file; None when it is not built."""
    import importlib.util

    so = ROOT / "oracle" / "_ref" / name / f"{name}.so"
    if not so.exists():
        return None
    spec = importlib.util.spec_from_file_location(name, so)
    mod = importlib.util.module_from_spec(spec)
    spec.loader.exec_module(mod)
    return mod


def run_gs2d(args, ref: bool = False) -> None:
    """The reference's toy2d kernel benchmark (toy2d/bench.py:43-70): the same seeded Gaussians2D scenes (bit-exact
    binning, so the same pairs and buckets), the same four kernels, CUDA-event medians. This library's ext(), or with
    ref the reference's own toy2d/csrc/rasterize.cu built for sm_100a (oracle/_ref/gs2d_cuda_ref); the reference's
    published H100 figures beside them where it published the configuration."""
    from gs_b200 import gs2d

    dev = torch.device("cuda", 0)
    torch.cuda.set_device(dev)
    e = load_reference_module("gs2d_cuda_ref") if ref else gs2d.ext()
    if e is None:
        print(json.dumps({"impl": "reference", "unavailable": "the reference's toy2d CUDA extension is not built "
                                                              "(oracle/build.py needs the reference tree)"}))
        return
    rows = []
    launches0 = L.query("splat_launch_count")
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

            def fwd(save):
                return e.forward(*common, bins.bucket_offsets, bins.num_buckets, H, W, save)

            out, final_T, n_contrib, _ = fwd(False)
            out_s, final_T_s, n_contrib_s, bstate = fwd(True)
            w, it = max(args.warmup, 5), max(args.steps, 20)
            r = {"size": size, "n": n, "pairs": int(bins.point_list.numel()), "buckets": int(bins.num_buckets),
                 "forward_ms": median_ms(lambda: fwd(False), w, it),
                 "forward_save_buckets_ms": median_ms(lambda: fwd(True), w, it),
                 "backward_pixel_ms": median_ms(lambda: e.backward_pixel(*common, final_T, n_contrib, dout), w, it),
                 "backward_splat_ms": median_ms(lambda: e.backward_splat(*common, bins.bucket_offsets,
                                                                         bins.bucket_to_tile, out_s, final_T_s,
                                                                         n_contrib_s, bstate, dout), w, it)}
            pub = GS2D_H100_MS.get((size, n))
            if pub:
                r["reference_h100_ms"] = dict(zip(("forward", "forward_save_buckets", "backward_pixel",
                                                   "backward_splat"), pub))
            rows.append({k: (round(v, 4) if isinstance(v, float) else v) for k, v in r.items()})
    line = {"metric": "toy2d kernel ms (the reference's toy2d/bench.py sweep)", "unit": "ms",
            "higher_is_better": False, "n_gpus": 1, "data": "synthetic (the reference's seeded scenes)",
            "dtype": "f32", "config": {"workload": "gs2d: the reference's toy2d kernel sweep, 512^2 and 1024^2 x "
                                                   "10k / 50k / 200k Gaussians"},
            "results": rows}
    if ref:
        line["impl"] = "reference"
        line["reference_kernels"] = "toy2d/csrc/rasterize.cu built for sm_100a (oracle/_ref/gs2d_cuda_ref)"
    else:
        line["gpu_launches"] = L.query("splat_launch_count") - launches0
    print(json.dumps(line), flush=True)


def run_splat2d(args, ref: bool = False) -> None:
    """The reference's splat2d backward benchmark scenes (bench/phase0/backward_bench.py: 1920x1080 with 50k and
    200k splats, sigma 2-10 px, opacity 0.05-0.6, and a 960x540 / 20k case), float32, the same tile tables for
    both (bin_tiles, bit-exact against the reference's): CUDA-event medians of forward, backward_pixel and
    backward_splat, each with its output allocation as the reference's bench times them. This library's
    extension, or with ref the reference's own phase0/csrc/macrotile kernels built for sm_100a
    (oracle/_ref/splat2d_cuda_ref)."""
    from gs_b200 import splat2d

    dev = torch.device("cuda", 0)
    torch.cuda.set_device(dev)
    e = load_reference_module("splat2d_cuda_ref") if ref else splat2d.load_extension(with_cuda=True)
    if e is None:
        print(json.dumps({"impl": "reference", "unavailable": "the reference's splat2d CUDA extension is not built "
                                                              "(oracle/build.py needs the reference tree)"}))
        return
    rows = []
    launches0 = L.query("splat_launch_count")
    w, it = max(args.warmup, 5), max(args.steps, 20)
    for n, h, wd in ((50_000, 1080, 1920), (200_000, 1080, 1920), (20_000, 540, 960)):
        p64 = [t.to(dev) for t in scenes.splat2d_bench_scene(n, h, wd)]
        bins = splat2d.bin_tiles(*p64[:3], h, wd)
        tb = (bins.tile_offsets, bins.tile_ids, bins.bucket_offsets, bins.bucket_tile)
        p32 = [t.float().contiguous() for t in p64]
        g_img = torch.randn(h, wd, 3, generator=torch.Generator().manual_seed(1)).to(dev)
        image, t_final, n_contrib, last_contrib, ckpt = e.forward(*p32, *tb, h, wd)
        rows.append({"n": n, "height": h, "width": wd, "list_entries": int(bins.tile_ids.numel()),
                     "buckets": bins.num_buckets,
                     "forward_ms": round(median_ms(lambda: e.forward(*p32, *tb, h, wd), w, it), 4),
                     "backward_pixel_ms": round(median_ms(lambda: e.backward_pixel(g_img, *p32, *tb, t_final,
                                                                                   last_contrib, h, wd), w, it), 4),
                     "backward_splat_ms": round(median_ms(lambda: e.backward_splat(g_img, *p32, *tb, image, ckpt,
                                                                                   h, wd), w, it), 4)})
    line = {"metric": "splat2d kernel ms (the reference's phase0 backward benchmark scenes)", "unit": "ms",
            "higher_is_better": False, "n_gpus": 1, "data": "synthetic (the reference's scene generator)",
            "dtype": "f32", "config": {"workload": "splat2d: 1920x1080 x 50k / 200k, 960x540 x 20k"}, "results": rows}
    if ref:
        line["impl"] = "reference"
        line["reference_kernels"] = "phase0/csrc/macrotile built for sm_100a (oracle/_ref/splat2d_cuda_ref)"
    else:
        line["gpu_launches"] = L.query("splat_launch_count") - launches0
    print(json.dumps(line), flush=True)


def run_blend_bwd(args, ref: bool = False) -> None:
    """The 3DGS blend backward alone on the C3 view (3M Gaussians, 1920x1080, upstream gradient N(0, 1e-3)) and on
    C2: this library's forward builds the buffers once, then K timed launches of the blend backward (each with the
    clear of its sums): this library's k_blend_backward (gs3d_backward_blend), or with ref the reference's own
    Faster-GS blend_backward_macro_cu in each of its launcher modes (oracle/_ref/fastergs_macro, 16x16 tiles)
    reading the same buffers. The buffers (2 GB at C3) exceed L2; no flush."""
    dev = torch.device("cuda", 0)
    torch.cuda.set_device(dev)
    if ref:
        from oracle import fastergs_ref

        try:
            fastergs_ref.ref_lib()
        except RuntimeError as exc:
            print(json.dumps({"impl": "reference", "unavailable": str(exc)}))
            return
    rows = []
    launches0 = L.query("splat_launch_count")
    w, it = max(args.warmup, 5), max(args.steps, 20)
    for cfg in ("c3", "c2"):
        sc = scenes.gs3d_config(cfg, seed=0)
        cam = sc["cameras"][0]
        params = [sc[k].to(dev).contiguous() for k in NAMES]
        settings = scenes.settings_tuple(cam, sc["active_sh_bases"], dev)
        W, H = cam["width"], cam["height"]
        image, prim, tile, inst, bucket, m, nb, sel = gs3d.forward(*params, *settings)
        dout = upstream_gradient(0, H, W).to(dev)
        row = {"config": cfg, "gaussians": params[0].shape[0], "width": W, "height": H, "instances": m}
        if ref:
            ri = fastergs_ref.RefInputs(params, settings, image, prim, tile, inst, bucket, m, nb, W, H)
            for mode in (1, 3, 7, 15):
                row[f"mode{mode}_ms"] = round(median_ms(lambda: ri.run(dout, mode, False), w, it), 4)
        else:
            row["k_blend_backward_ms"] = round(median_ms(
                lambda: gs3d.backward_blend(None, dout, image, params[0], params[1], params[2], params[3], params[5],
                                            prim, tile, inst, bucket, *settings, m, nb, sel), w, it), 4)
        rows.append(row)
        del image, prim, tile, inst, bucket, params
        torch.cuda.empty_cache()
    line = {"metric": "3DGS blend backward ms (one view)", "unit": "ms", "higher_is_better": False, "n_gpus": 1,
            "data": "synthetic (seeded, config-shaped)", "dtype": "f32",
            "config": {"workload": "blend-bwd: the blend backward over this library's forward buffers, C3 and C2"},
            "results": rows}
    if ref:
        line["impl"] = "reference"
        line["reference_kernels"] = ("blend_backward_macro_cu (phase1/fastergs_macro.patch:40-314) built for "
                                     "sm_100a at 16x16 tiles; modes: 2 subtile skip, 4 transposing reduction, 8 eight "
                                     "warps per block")
    else:
        line["gpu_launches"] = L.query("splat_launch_count") - launches0
    print(json.dumps(line), flush=True)


def main() -> None:
    ap = argparse.ArgumentParser()
    ap.add_argument("--gpus", type=int, default=1)
    ap.add_argument("--steps", type=int, default=200)
    ap.add_argument("--warmup", type=int, default=3)
    ap.add_argument("--impl", choices=["ours", "reference"], default="ours")
    ap.add_argument("--workload", choices=["c3", "c4", "c2", "c1", "c5", "gs2d", "splat2d", "blend-bwd", "ssim"],
                    default="c3")
    ap.add_argument("--exchange", choices=["auto", "peer", "nvls", "compact", "nccl"], default="auto",
                    help="N > 1: the gradient exchange + Adam form (auto: the fastest measured at that rank count)")
    ap.add_argument("--no-c4", action="store_true", help="skip the C4 strong-scaling object of the c3 line")
    ap.add_argument("--cpu-budget", type=float, default=20.0, help="seconds of CPU work for the baseline sample")
    ap.add_argument("--ref-budget", type=float, default=150.0,
                    help="--impl reference: seconds of CPU work for its warm-up and timed steps together")
    ap.add_argument("--no-cpu-baseline", action="store_true")
    ap.add_argument("--lean", action="store_true",
                    help="N = 1: the reference's lean Adam (visibility-sparse, bfloat16 SH-rest moments) instead of "
                         "the dense float32 update")
    ap.add_argument("--fuse", action="store_true",
                    help="N = 1: the preprocess backward fused with Adam (FusedAdam(fuse_backward=True)) instead of "
                         "separate launches; measured slower on C3 (1.01 ms against 0.24 + 0.74 ms)")
    args = ap.parse_args()
    if args.warmup < 3:
        args.warmup = 3
    if args.impl == "reference":
        run_reference(args)
    elif args.workload == "c1":
        run_c1(args)
    elif args.workload == "c5":
        run_c5(args)
    elif args.workload == "gs2d":
        run_gs2d(args)
    elif args.workload == "splat2d":
        run_splat2d(args)
    elif args.workload == "blend-bwd":
        run_blend_bwd(args)
    elif args.workload == "ssim":
        run_ssim(args)
    else:
        run_ours(args)


if __name__ == "__main__":
    main()
