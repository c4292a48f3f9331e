"""The benchmark's N > 1 host path on the CPU: two ranks as spawned processes over gloo (127.0.0.1), through the same
`bench.collectives` the GPU box uses with nccl. Replicas exchange no data: the only cross-rank steps are a barrier and
the max over ranks of the timed region, and whole-job throughput is every rank's units over the slowest rank's time.
A rank that leaves between steps ends the others' next collective with an error on the host (its closed connection,
or at the latest the process group's timeout), never a wait without end."""
import os
import socket
import sys
import time
from types import SimpleNamespace

import pytest
import torch.multiprocessing as mp

ROOT = os.path.dirname(os.path.dirname(os.path.abspath(__file__)))
sys.path.insert(0, ROOT)
import bench  # noqa: E402


def free_port():
    with socket.socket() as s:
        s.bind(("127.0.0.1", 0))
        return s.getsockname()[1]


def env(rank, world, port):
    os.environ.update(MASTER_ADDR="127.0.0.1", MASTER_PORT=str(port), RANK=str(rank), WORLD_SIZE=str(world),
                      LOCAL_RANK=str(rank))


def replicas(rank, world, port, out):
    import torch.distributed as dist
    env(rank, world, port)
    barrier, maxreduce = bench.collectives(world, backend="gloo", timeout_s=60)
    try:
        barrier()
        dev_s = 1.0 + 0.5 * rank           # rank 1 is the slow one
        wall_s = 2.0 - 0.25 * rank         # rank 0 is slow on the host clock
        dev_max, wall_max = maxreduce(dev_s), maxreduce(wall_s)
        value, e2e = bench.aggregate(64 * 20, world, dev_max, wall_max)
        barrier()
        out.put((rank, dev_max, wall_max, value, e2e))
    finally:
        dist.destroy_process_group()


def absent_peer(rank, world, port, out):
    import torch.distributed as dist
    env(rank, world, port)
    barrier, maxreduce = bench.collectives(world, backend="gloo", timeout_s=3)
    try:
        if rank == 1:
            out.put((rank, "left"))         # leaves between steps: never reaches the next collective
            return
        t0 = time.time()
        try:
            maxreduce(1.0)
            out.put((rank, "returned", time.time() - t0, ""))
        except Exception as e:              # the process group's timeout, as an error on the host
            out.put((rank, "error", time.time() - t0, type(e).__name__))
    finally:
        try:
            dist.destroy_process_group()
        except Exception:
            pass


def run(fn, world=2, timeout=120):
    ctx = mp.get_context("spawn")
    q = ctx.Queue()
    port = free_port()
    ps = [ctx.Process(target=fn, args=(r, world, port, q)) for r in range(world)]
    for p in ps:
        p.start()
    got = [q.get(timeout=timeout) for _ in range(world)]
    for p in ps:
        p.join(timeout=timeout)
        if p.is_alive():
            p.kill()
    return sorted(got, key=lambda x: x[0]), [p.exitcode for p in ps]


def test_world2_max_over_ranks_and_whole_job_throughput():
    got, codes = run(replicas)
    assert codes == [0, 0]
    for rank, dev_max, wall_max, value, e2e in got:
        assert dev_max == 1.5 and wall_max == 2.0          # every rank sees the slowest rank's times
        assert value == pytest.approx(2 * 64 * 20 / 1.5)  # both ranks' tokens over the slowest device time
        assert e2e == pytest.approx(2 * 64 * 20 / 2.0)


def test_a_rank_that_leaves_ends_the_others_wait_with_an_error():
    got, codes = run(absent_peer)
    assert got[1] == (1, "left")
    # the survivor's collective fails (the peer's connection closed, or the 3 s timeout) instead of waiting for good
    assert got[0][1] == "error" and got[0][2] < 60, got[0]


def test_single_rank_needs_no_process_group():
    barrier, maxreduce = bench.collectives(1)
    barrier()
    assert maxreduce(3.25) == 3.25
    assert bench.aggregate(1280, 1, 0.5, 0.64) == (2560.0, 2000.0)


def test_reference_arm_runs_on_rank0_only():
    # under torchrun every rank starts; the ranks other than 0 exit without work (no model, no oracle)
    args = SimpleNamespace(steps=2, warmup=1)
    t0 = time.time()
    assert bench.run_reference(args, rank=1, world=2) is None
    assert time.time() - t0 < 1.0
