"""The multi-GPU path's host logic on CPU with world_size-2 gloo ranks.

bench.py under torchrun splits the (batch x head) slices of a job into
contiguous per-rank ranges (fp4attn_b200.shard_range), generates each shard's
inputs on its own rank from per-slice seeds, and takes the max over ranks of
the device timings with an all_reduce.  The attention itself needs no
collective: slices are independent.  These tests run that logic on CPU ranks
(no GPU) and check that shards cover the job exactly once and that a shard's
inputs equal the same slices of the whole job.
"""
import os
import socket

import pytest
import torch
import torch.distributed as dist
import torch.multiprocessing as mp

import fp4attn_b200 as fa
import fp4attn_b200.workloads as wl


@pytest.mark.parametrize("n,world", [(64, 1), (64, 2), (512, 8), (7, 3), (3, 4), (0, 2)])
def test_shard_range_partitions(n, world):
    ranges = [fa.shard_range(n, world, r) for r in range(world)]
    assert ranges[0][0] == 0 and ranges[-1][1] == n
    for (a, b), (c, d) in zip(ranges, ranges[1:]):
        assert b == c and a <= b
    sizes = [b - a for a, b in ranges]
    assert max(sizes) - min(sizes) <= 1


def test_shard_range_rejects_bad_requests():
    for args in ((4, 0, 0), (4, 2, 2), (4, 2, -1), (-1, 2, 0)):
        with pytest.raises(ValueError):
            fa.shard_range(*args)


def _free_port():
    with socket.socket() as s:
        s.bind(("127.0.0.1", 0))
        return s.getsockname()[1]


def _worker(rank, world, port, q):
    os.environ.update(MASTER_ADDR="127.0.0.1", MASTER_PORT=str(port))
    dist.init_process_group("gloo", rank=rank, world_size=world)
    try:
        w = wl.Workload("shard_test", 2, 3, 16, 24, 32, outlier_frac=0.05, outlier_mult=8.0)
        lo, hi = fa.shard_range(w.slices, world, rank)
        Q, K, V = wl.make_inputs(w, 11, slices=(lo, hi), device="cpu")
        # gather every rank's range and inputs, as a validation pass would
        ranges = [None] * world
        dist.all_gather_object(ranges, (lo, hi))
        parts = [None] * world
        dist.all_gather_object(parts, (Q, K, V))
        # max-over-ranks of a per-rank timing, as bench.py reports it
        t = torch.tensor([float(rank + 1)], dtype=torch.float64)
        dist.all_reduce(t, op=dist.ReduceOp.MAX)
        if rank == 0:
            Qf, Kf, Vf = wl.make_inputs(w, 11, device="cpu")
            ok = all(torch.equal(parts[r][0], Qf[a:b]) and torch.equal(parts[r][1], Kf[a:b]) and
                     torch.equal(parts[r][2], Vf[a:b]) for r, (a, b) in enumerate(ranges))
            covered = sorted(i for a, b in ranges for i in range(a, b)) == list(range(w.slices))
            q.put((ok, covered, t.item()))
    finally:
        dist.destroy_process_group()


def test_two_rank_shards_match_the_whole_job():
    world = 2
    ctx = mp.get_context("spawn")
    q = ctx.Queue()
    port = _free_port()
    procs = [ctx.Process(target=_worker, args=(r, world, port, q)) for r in range(world)]
    for p in procs:
        p.start()
    for p in procs:
        p.join(timeout=120)
        assert p.exitcode == 0
    ok, covered, tmax = q.get(timeout=10)
    assert ok and covered and tmax == float(world)


def _failing_worker(rank, world, port, q, fail_rank):
    """A bench-like rank: joins the group, then meets the others at a barrier
    before its timed region.  `fail_rank` dies first (as a rank whose device
    set-up failed would), so the others' barrier must end in an error within
    the group's short timeout instead of waiting for good."""
    import datetime
    import time
    os.environ.update(MASTER_ADDR="127.0.0.1", MASTER_PORT=str(port))
    dist.init_process_group("gloo", rank=rank, world_size=world, timeout=datetime.timedelta(seconds=5))
    if rank == fail_rank:
        os._exit(3)  # no clean-up: the process just disappears
    t0 = time.monotonic()
    try:
        dist.barrier()
        q.put((rank, "barrier passed", time.monotonic() - t0))
    except Exception as e:  # gloo reports the lost peer or the timeout
        q.put((rank, type(e).__name__, time.monotonic() - t0))
    q.close()
    q.join_thread()  # the report reaches the pipe before the process goes
    os._exit(0)


def test_a_failed_rank_is_reported_not_waited_for():
    world, fail_rank = 2, 1
    ctx = mp.get_context("spawn")
    q = ctx.Queue()
    port = _free_port()
    procs = [ctx.Process(target=_failing_worker, args=(r, world, port, q, fail_rank)) for r in range(world)]
    for p in procs:
        p.start()
    for p in procs:
        p.join(timeout=120)
    alive = [p for p in procs if p.is_alive()]
    for p in alive:
        p.kill()
    assert not alive, "a rank was still waiting after 120 s"
    assert procs[fail_rank].exitcode == 3
    rank, outcome, waited = q.get(timeout=10)
    assert rank == 0 and outcome != "barrier passed"
    assert waited < 60
