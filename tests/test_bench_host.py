"""Host-side logic of bench.py, on the CPU: the row split across ranks and
the clock record restricted to the timed region."""
import argparse
import os
import tempfile
from datetime import datetime

import bench


def test_shard_rows_cover_the_problem():
    for n in (10_000_000, 1_000_003, 7):
        for world in (1, 2, 3, 8):
            rows = [bench.shard_rows(n, world, r) for r in range(world)]
            assert sum(rows) == n and max(rows) - min(rows) <= 1


def test_workload_rows_weak_and_strong():
    args = argparse.Namespace(workload="config3", n=None)
    assert bench.workload_rows(args, 8, 0) == (1_250_000, 10_000_000)
    args = argparse.Namespace(workload="config4", n=None)
    assert bench.workload_rows(args, 2, 1) == (6_250_000, 12_500_000)     # an eighth per GPU


class _Done:
    def terminate(self):
        pass

    def wait(self, timeout=None):
        return 0


def _clocks_from(lines):
    c = bench.Clocks.__new__(bench.Clocks)
    c.f = tempfile.NamedTemporaryFile("w+", suffix=".csv", delete=False)
    c.f.write("\n".join(lines) + "\n")
    c.f.flush()
    c.p = _Done()
    return c


def _line(t, mhz, cap):
    stamp = datetime.fromtimestamp(t).strftime("%Y/%m/%d %H:%M:%S.%f")[:-3]
    return (f"0, {mhz}, 1965, 900.0, 0x0, Not Active, Not Active, Not Active, "
            f"{'Active' if cap else 'Not Active'}, {stamp}")


def test_clock_samples_outside_the_timed_region_are_dropped():
    t0 = 1_800_000_000.0
    idle = [_line(t0 + 0.05 * i, 1965, False) for i in range(6)]           # before the region
    busy = [_line(t0 + 0.5 + 0.05 * i, 1500, True) for i in range(4)]       # inside it
    c = _clocks_from(idle + busy)
    name = c.f.name
    rec = c.stop((t0 + 0.49, t0 + 0.70))
    assert not os.path.exists(name)
    assert rec["samples"] == 4 and rec["sm_mhz"] == 1500.0
    assert rec["reasons"] == ["sw_power_cap"] and rec["sm_max_mhz"] == 1965.0
    # no sample inside the window: every sample is kept rather than none
    rec = _clocks_from(idle).stop((t0 + 10.0, t0 + 11.0))
    assert rec["samples"] == 6 and rec["sm_mhz"] == 1965.0 and rec["reasons"] == []
