"""bench.py's multi-rank plumbing on CPU: two gloo ranks (the GPU box runs the
same code with NCCL, one process per GPU).  Sessions shard as independent
replicas, so the only collectives are the barrier and the max-over-ranks of
the timings; the whole-job rate is steps * world / slowest time."""
import multiprocessing as mp
import os
import socket
import sys

import pytest

ROOT = os.path.dirname(os.path.dirname(os.path.abspath(__file__)))


def _free_port() -> int:
    with socket.socket() as s:
        s.bind(("127.0.0.1", 0))
        return s.getsockname()[1]


def _worker(rank, world, port, q):
    os.environ.update(RANK=str(rank), WORLD_SIZE=str(world), LOCAL_RANK=str(rank),
                      MASTER_ADDR="127.0.0.1", MASTER_PORT=str(port), CW_DIST_BACKEND="gloo")
    sys.path.insert(0, ROOT)
    import bench
    d = bench.Dist()
    try:
        d.barrier()
        slowest_ms = d.max(10.0 + 5.0 * rank)     # rank 1 is the slow one
        rate = bench.replica_rate(100, d.world, slowest_ms / 1000.0)
        d.barrier()
        q.put((rank, d.world, d.rank, slowest_ms, rate))
    finally:
        d.close()


@pytest.mark.timeout(120)
def test_two_rank_max_and_rate():
    ctx = mp.get_context("spawn")
    q = ctx.Queue()
    port = _free_port()
    procs = [ctx.Process(target=_worker, args=(r, 2, port, q)) for r in range(2)]
    for p in procs:
        p.start()
    out = sorted(q.get(timeout=90) for _ in procs)
    for p in procs:
        p.join(timeout=30)
        assert p.exitcode == 0
    assert [o[0] for o in out] == [0, 1]
    for rank, world, drank, slowest, rate in out:
        assert world == 2 and drank == rank
        assert slowest == 15.0          # the max over ranks, on every rank
        assert rate == pytest.approx(100 * 2 / 0.015)


def test_single_process_needs_no_group():
    sys.path.insert(0, ROOT)
    import bench
    d = bench.Dist()
    assert d.world == 1 and not d.pg
    assert d.max(3.5) == 3.5
    d.barrier()
    d.close()
    assert bench.replica_rate(256, 1, 0.25) == 1024


def test_reference_arm_runs_on_rank0_only(monkeypatch):
    """Under torchrun only rank 0 times the CPU reference; other ranks return
    at once without touching the model or opening a process group."""
    sys.path.insert(0, ROOT)
    import bench

    monkeypatch.setenv("RANK", "1")
    monkeypatch.setenv("WORLD_SIZE", "2")
    monkeypatch.setattr(bench, "np", None)  # any model work on rank 1 would fail
    monkeypatch.setattr(bench, "Dist", None)  # nor may it open a process group
    assert bench.run_reference(object()) is None
    monkeypatch.setattr(bench, "parse", lambda: type("A", (), {"impl": "reference"})())
    assert bench.main() is None


def test_reference_arm_uses_every_host_core(monkeypatch):
    """torchrun exports OMP_NUM_THREADS=1; the reference arm must not inherit it."""
    sys.path.insert(0, ROOT)
    import bench

    monkeypatch.setenv("OMP_NUM_THREADS", "1")
    assert bench.host_threads() == len(os.sched_getaffinity(0))
