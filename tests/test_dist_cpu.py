"""The multi-rank host logic on CPU: two gloo ranks shard the rows the way
bench.py does, each forms its shard's fixed-point int64 sums and counts (the
oracle stands in for the device kernels), an int64 all-reduce combines them,
and every rank finalises.  Integer sums make the result identical to the
single-process update bit for bit -- the property the NCCL path relies on."""
import os
import socket

import numpy as np
import pytest
import torch
import torch.distributed as dist
import torch.multiprocessing as mp

import oracle as O


def _free_port():
    with socket.socket() as s:
        s.bind(("127.0.0.1", 0))
        return s.getsockname()[1]


def _shard_rows(n, world, rank):
    import bench
    return bench.shard_rows(n, world, rank)


def _worker(rank, world, port, out):
    os.environ.update(MASTER_ADDR="127.0.0.1", MASTER_PORT=str(port))
    dist.init_process_group("gloo", rank=rank, world_size=world)
    try:
        P = O.make_config1(20_000, 16, seed=6)
        C0 = O.kmeanspp(P, 24, seed=6)
        n, d = P.shape
        k = C0.shape[0]
        counts = [_shard_rows(n, world, r) for r in range(world)]
        r0 = sum(counts[:rank])
        shard = P[r0:r0 + counts[rank]]
        # global operand scale and fixed-point precision: max over ranks, total n
        pmax = torch.tensor([float(np.abs(shard).max())], dtype=torch.float64)
        dist.all_reduce(pmax, op=dist.ReduceOp.MAX)
        frac = O.fixed_frac(float(np.float32(pmax.item())), n)
        C = C0.copy()
        for _ in range(3):
            lab = O.assign_fp32(shard, C)
            _, _, cnt, S = O.update_fixed(shard, lab, C, frac)
            buf = torch.from_numpy(np.concatenate([S.reshape(-1), cnt]).astype(np.int64))
            dist.all_reduce(buf)
            S_all = buf[: k * d].numpy().reshape(k, d)
            cnt_all = buf[k * d:].numpy()
            # finalise exactly as the device does: (float)((S * 2^-frac) / count)
            Cn = C.copy()
            nz = cnt_all > 0
            Cn[nz] = ((S_all[nz].astype(np.float64) * 2.0 ** -frac) / cnt_all[nz, None]).astype(np.float32)
            C = Cn
        out[rank] = C
    finally:
        dist.destroy_process_group()


def test_two_gloo_ranks_match_single_process():
    world = 2
    port = _free_port()
    with mp.Manager() as m:
        out = m.dict()
        mp.start_processes(_worker, args=(world, port, out), nprocs=world, start_method="spawn", join=True)
        res = [out[r] for r in range(world)]
    P = O.make_config1(20_000, 16, seed=6)
    C0 = O.kmeanspp(P, 24, seed=6)
    frac = O.fixed_frac(float(np.abs(P).max()), len(P))
    _, C_single, _, _ = O.lloyd(P, C0, 3, update_mode=1, frac=frac)
    for C in res:
        assert np.array_equal(C.view(np.uint32), C_single.view(np.uint32))


def _start_worker(rank, world, port, out):
    import bench
    os.environ.update(MASTER_ADDR="127.0.0.1", MASTER_PORT=str(port))
    dist.init_process_group("gloo", rank=rank, world_size=world)
    try:
        n = 150_000
        r0, n_local, n_total = bench.workload_rows("config3", n, world, rank)
        P = bench.gen_rows("config3", r0, r0 + n_local, "cpu")
        out[rank] = bench.start_centroids(P, r0, n_total, 1024, world, "cpu").numpy()
    finally:
        dist.destroy_process_group()


def test_bench_start_centroids_are_the_same_for_any_rank_count():
    """bench.py's shards: each of two gloo ranks generates only its own rows, and the start
    centroids assembled across them equal the single-process ones bit for bit."""
    import bench
    world = 2
    port = _free_port()
    with mp.Manager() as m:
        out = m.dict()
        mp.start_processes(_start_worker, args=(world, port, out), nprocs=world, start_method="spawn", join=True)
        res = [out[r] for r in range(world)]
    P = bench.gen_rows("config3", 0, 150_000, "cpu")
    want = bench.start_centroids(P, 0, 150_000, 1024, 1, "cpu").numpy()
    for C in res:
        assert np.array_equal(C.view(np.uint32), want.view(np.uint32))
