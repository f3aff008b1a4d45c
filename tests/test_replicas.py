"""The multi-GPU path of bench.py is replicas only: each rank runs its own
stream, and the ranks meet only at the barrier around the timed region and
in the maximum of their times.  That host logic runs here on CPU, two gloo
ranks in child processes."""

import os
import socket
import sys

import torch.multiprocessing as mp

ROOT = os.path.dirname(os.path.dirname(os.path.abspath(__file__)))


def _free_port():
    with socket.socket() as s:
        s.bind(("127.0.0.1", 0))
        return s.getsockname()[1]


def _rank_main(rank, world, port, out):
    os.environ.update(RANK=str(rank), WORLD_SIZE=str(world), LOCAL_RANK=str(rank), MASTER_ADDR="127.0.0.1",
                      MASTER_PORT=str(port))
    sys.path.insert(0, ROOT)
    import bench
    ranks = bench.Ranks()  # gloo over host sockets: no NCCL communicator
    ranks.barrier()
    seconds = 1.0 + 0.5 * rank  # the slower rank sets the job's time
    slowest = ranks.max(seconds)
    value = bench.aggregate(256, slowest, ranks.world)
    out.put((rank, ranks.world, slowest, value))
    ranks.close()


def test_two_replicas_report_the_slowest_rank():
    ctx = mp.get_context("spawn")
    out = ctx.Queue()
    port = _free_port()
    procs = [ctx.Process(target=_rank_main, args=(r, 2, port, out)) for r in range(2)]
    for p in procs:
        p.start()
    results = sorted(out.get(timeout=120) for _ in procs)
    for p in procs:
        p.join(timeout=60)
        assert p.exitcode == 0
    for rank, world, slowest, value in results:
        assert world == 2
        assert slowest == 1.5
        assert value == 2 * 256 / 1.5


def test_one_process_needs_no_group(monkeypatch):
    monkeypatch.delenv("WORLD_SIZE", raising=False)
    sys.path.insert(0, ROOT)
    import bench
    ranks = bench.Ranks("gloo")
    assert ranks.world == 1 and ranks.dist is None
    assert ranks.max(3.25) == 3.25
    assert bench.aggregate(256, 0.5, 1) == 512
    ranks.close()
