"""Multi-process host logic of bench.py on CPU: world_size-2 gloo ranks.

The PCMM shards by query batch (independent ciphertexts), so the only
collectives are the barrier around the timed region and the max of the
per-rank device times; the whole-job rate counts every rank's ciphertexts
over the slowest rank's time.  The reference arm runs on rank 0 only.
"""
import os
import socket
import sys

import pytest
import torch.multiprocessing as mp

ROOT = os.path.dirname(os.path.dirname(os.path.abspath(__file__)))


def _free_port() -> int:
    with socket.socket() as s:
        s.bind(("127.0.0.1", 0))
        return s.getsockname()[1]


def _rank_main(rank, world, port, times, out):
    os.environ.update({"RANK": str(rank), "LOCAL_RANK": str(rank), "WORLD_SIZE": str(world),
                       "MASTER_ADDR": "127.0.0.1", "MASTER_PORT": str(port),
                       "HELRM_DIST_BACKEND": "gloo"})
    sys.path.insert(0, ROOT)
    import bench
    d = bench.Dist(timeout_s=60)
    try:
        assert d.backend == "gloo" and d.world == world and d.rank == rank
        d.barrier()
        t = d.max(times[rank])
        rate = bench.whole_job_rate(d.world, 64, 5, t)
        # reference arm: only rank 0 does work and prints; the others return
        class A:
            pass
        if rank != 0:
            bench.run_reference(A(), d)  # must return before touching the oracle
        out.put((rank, t, rate))
    finally:
        d.close()


@pytest.mark.parametrize("world", [2])
def test_max_over_ranks_and_whole_job_rate(world):
    ctx = mp.get_context("spawn")
    q = ctx.Queue()
    port = _free_port()
    times = [0.40, 0.55]
    procs = [ctx.Process(target=_rank_main, args=(r, world, port, times, q)) for r in range(world)]
    for p in procs:
        p.start()
    for p in procs:
        p.join(timeout=120)
    codes = [p.exitcode for p in procs]
    assert codes == [0] * world, codes
    res = sorted(q.get(timeout=10) for _ in range(world))
    for rank, t, rate in res:
        assert t == pytest.approx(max(times))
        assert rate == pytest.approx(world * 64 * 5 / max(times))


def test_single_process_dist_is_a_no_op():
    sys.path.insert(0, ROOT)
    import bench
    env = {k: os.environ.pop(k) for k in ("WORLD_SIZE", "RANK", "LOCAL_RANK") if k in os.environ}
    try:
        d = bench.Dist()
        assert d.world == 1 and d.pg is None
        d.barrier()
        assert d.max(1.25) == 1.25
        assert bench.whole_job_rate(1, 64, 5, 2.0) == 160.0
        d.close()
    finally:
        os.environ.update(env)
