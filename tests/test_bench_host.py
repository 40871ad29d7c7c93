"""Host-side logic of bench.py, on the CPU: the row split across ranks and
the clock record restricted to the timed region."""
import os
import tempfile
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
