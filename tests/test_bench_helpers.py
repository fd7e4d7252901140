"""Host-side figures of bench.py, on CPU: the exchange kernels' NVLink byte model and the summary of the clock
samples taken during a timed region (which decides whether a run is kept)."""
from __future__ import annotations

import datetime
import types

import pytest

import bench


def _trainer(world: int, lo: int, hi: int, total: int, form: str):
    peer = types.SimpleNamespace(lo=lo, hi=hi, total=total)
    return types.SimpleNamespace(world=world, peer=peer, exchange=form)


@pytest.mark.parametrize("world,form,slices", [(2, "peer", 2), (2, "nvls", 3), (2, "nccl", 2), (4, "peer", 6),
                                               (4, "nvls", 5), (4, "nccl", 6), (8, "peer", 14), (8, "nvls", 9),
                                               (8, "nccl", 14)])
def test_exchange_bytes_per_direction(world, form, slices):
    total = 8_000_000
    chunk = total // world
    tr = _trainer(world, 0, chunk, total, form)
    out = bench.exchange_figures(tr, {"xkernel": 1.0, "comm": 1.25}, 1, "cpu")
    assert out["form"] == form and out["ms"] == 1.0 and out["stage_ms_with_barriers"] == 1.25
    assert out["bytes_each_direction"] == slices * 4 * chunk
    assert out["achieved"] == pytest.approx(slices * 4 * chunk / 1e-3 / 1e9, rel=1e-6)
    assert out["frac"] == pytest.approx(out["achieved"] / 770.0, abs=1e-4)
    # as an all-reduce of the whole vector: 2 (G - 1) / G of it over the time
    assert out["allreduce_bus_gbs"] == pytest.approx(2.0 * (world - 1) / world * 4 * total / 1e-3 / 1e9, rel=1e-3)


@pytest.mark.parametrize("world,views", [(2, 1), (4, 2), (8, 1)])
def test_compact_exchange_bytes_per_direction(world, views):
    """Per owned Gaussian the compact form reads 11 + 6 V gradient floats from each other rank and writes its 59
    parameters to each of them."""
    n = 1_000_000
    owned = n // world
    peer = types.SimpleNamespace(lo=0, hi=owned, n=n, rest=15, views=views)
    tr = types.SimpleNamespace(world=world, peer=peer, exchange="compact")
    out = bench.exchange_figures(tr, {"xkernel": 1.0, "comm": 1.0}, 1, "cpu")
    assert out["bytes_each_direction"] == (world - 1) * 4 * owned * (11 + 6 * views + 59)
    assert out["allreduce_bus_gbs"] == pytest.approx(2.0 * (world - 1) / world * 4 * 59 * n / 1e-3 / 1e9, rel=1e-3)


def _clocks(rows, t0, t1):
    c = bench.Clocks(0)
    c.rows = rows
    c.t0, c.t1 = t0, t1
    return c


def _row(ts, sm, mx, watts, reasons=()):
    names = ("hw_slowdown", "hw_thermal_slowdown", "sw_thermal_slowdown", "sw_power_cap")
    flags = ["Active" if n in reasons else "Not Active" for n in names]
    return ts, ["0", str(sm), str(mx), str(watts), "0x0"] + flags


def test_clock_summary_uses_only_the_timed_region():
    t = datetime.datetime(2026, 1, 1, 12, 0, 0)
    s = datetime.timedelta(seconds=1)
    rows = [_row(t, 1200, 1965, 200, ("hw_slowdown",)),  # before the region: ignored
            _row(t + 2 * s, 1965, 1965, 600, ("sw_power_cap",)),
            _row(t + 3 * s, 1950, 1965, 610),
            _row(t + 4 * s, 1965, 1965, 620),
            _row(t + 9 * s, 800, 1965, 100, ("hw_thermal_slowdown",))]  # after it: ignored
    out = _clocks(rows, t + 1.5 * s, t + 5 * s).summary()
    assert out["samples"] == 3
    assert out["sm_mhz"] == 1965.0 and out["sm_max_mhz"] == 1965.0 and out["power_w"] == 610.0
    assert out["reasons"] == ["sw_power_cap"]


def test_clock_summary_of_a_short_region_takes_the_nearest_sample():
    t = datetime.datetime(2026, 1, 1, 12, 0, 0)
    ms = datetime.timedelta(milliseconds=1)
    rows = [_row(t, 1965, 1965, 300), _row(t + 50 * ms, 1900, 1965, 310)]
    out = _clocks(rows, t + 40 * ms, t + 45 * ms).summary()
    assert out["samples"] == 1 and out["sm_mhz"] == 1900.0 and "nearest" in out["note"]
    assert _clocks([], None, None).summary()["reasons"] == ["unsampled"]


def _reference_line(*extra: str) -> dict:
    import json
    import subprocess
    import sys
    from pathlib import Path

    root = Path(bench.__file__).resolve().parent
    out = subprocess.run([sys.executable, str(root / "bench.py"), "--impl", "reference", *extra],
                         capture_output=True, text=True, timeout=600, cwd=root)
    assert out.returncode == 0, out.stderr[-2000:]
    return json.loads(out.stdout.strip().splitlines()[-1])


@pytest.mark.parametrize("workload", ["ssim", "gs2d", "splat2d", "blend-bwd"])
def test_reference_arm_without_its_kernels_says_unavailable(workload):
    """The reference's SSIM is not vendored, and its CUDA kernels need a GPU: those reference arms print one JSON
    line saying why and exit 0 (here, without a GPU)."""
    line = _reference_line("--workload", workload)
    assert line["impl"] == "reference" and "unavailable" in line


def test_reference_arm_of_c1_times_the_cpu_path():
    """The c1 reference arm times the numpy restatement of the reference's CPU path for K steps."""
    line = _reference_line("--workload", "c1", "--steps", "1", "--warmup", "3")
    assert line["impl"] == "reference" and line["steps"] == 1 and line["value"] > 0
    assert line["config"] == bench.C1_CONFIG
