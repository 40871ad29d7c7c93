"""Host-side logic of bench.py, on the CPU: the row split across ranks and
the clock record restricted to the timed region."""
import os
import tempfile
import time
from datetime import datetime

import numpy as np
import torch

import bench


def test_shard_rows_cover_the_problem():
    for n in (10_000_000, 1_000_003, 7):
        for world in (1, 2, 3, 8):
            rows = [bench.shard_rows(n, world, r) for r in range(world)]
            assert sum(rows) == n and max(rows) - min(rows) <= 1


def test_workload_rows_weak_and_strong():
    assert bench.workload_rows("config3", None, 8, 0) == (0, 1_250_000, 10_000_000)
    assert bench.workload_rows("config3", None, 8, 3) == (3_750_000, 1_250_000, 10_000_000)
    assert bench.workload_rows("config3", 1_000_003, 8, 7) == (875_003, 125_000, 1_000_003)
    assert bench.workload_rows("config4", None, 2, 1) == (6_250_000, 6_250_000, 12_500_000)   # an eighth per GPU
    for n, world in ((10_000_000, 8), (1_000_003, 3), (7, 2)):
        rows = [bench.workload_rows("config3", n, world, r) for r in range(world)]
        assert [r0 for r0, _, _ in rows] == [sum(m for _, m, _ in rows[:i]) for i in range(world)]


def test_rows_do_not_depend_on_the_split():
    """A row's values are the same whichever rank generates it (block-seeded generator)."""
    for wl in ("config3", "config4", "config5"):
        whole = bench.gen_rows(wl, 0, 3 * bench.BLOCK // 2, "cpu")
        for a, b in ((0, 1000), (bench.BLOCK - 7, bench.BLOCK + 9), (70_000, 3 * bench.BLOCK // 2)):
            assert torch.equal(bench.gen_rows(wl, a, b, "cpu"), whole[a:b]), (wl, a, b)


def test_start_centroids_are_distinct_global_rows():
    idx = bench.start_rows(100_000_000, 16384)
    assert len(set(idx.tolist())) == 16384 and np.all(np.diff(idx) > 0) and idx[-1] < 100_000_000
    P = bench.gen_rows("config3", 0, 200_000, "cpu")
    C0 = bench.start_centroids(P[50_000:], 50_000, 200_000, 1024, 1, "cpu")
    idx = bench.start_rows(200_000, 1024)
    mine = idx >= 50_000
    assert torch.equal(C0[torch.from_numpy(np.nonzero(mine)[0])], P[torch.from_numpy(idx[mine])])
    assert int((C0[torch.from_numpy(np.nonzero(~mine)[0])] != 0).sum()) == 0


class _Done:
    def terminate(self):
        pass

    def wait(self, timeout=None):
        return 0


def _clocks_from(lines):
    c = bench.Clocks.__new__(bench.Clocks)
    c.f = tempfile.NamedTemporaryFile("w+", suffix=".csv", delete=False)
    c.f.write("\n".join(lines) + ("\n" if lines else ""))
    c.f.flush()
    c.p = _Done()
    return c


def _line(t, mhz, cap, thermal=False):
    stamp = datetime.fromtimestamp(t).strftime("%Y/%m/%d %H:%M:%S.%f")[:-3]
    return (f"0, {mhz}, 1965, 900.0, 0x0, Not Active, Not Active, "
            f"{'Active' if thermal else 'Not Active'}, {'Active' if cap else 'Not Active'}, {stamp}")


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
    # a throttle reason that rejects a run is reported by name
    rec = _clocks_from([_line(t0, 1800, False, thermal=True)]).stop((t0 - 0.01, t0 + 0.01))
    assert rec["reasons"] == ["sw_thermal_slowdown"] and rec["samples"] == 1


def test_clocks_wait_for_the_first_sample():
    """wait_ready returns once a whole sample line is in the file, and gives up after its
    limit when none comes (the timed region then proceeds without one)."""
    c = _clocks_from([])
    t = time.time()
    c.wait_ready(limit_s=0.3)
    assert 0.25 <= time.time() - t < 2.0
    with open(c.f.name, "a") as f:
        f.write(_line(time.time(), 1965, False) + "\n")
    t = time.time()
    c.wait_ready(limit_s=5.0)
    assert time.time() - t < 1.0
    assert c.stop()["samples"] == 1
