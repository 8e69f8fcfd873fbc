"""bench.py's multi-rank host logic on CPU: two gloo ranks, as torchrun would
start them (one process per rank, rendezvous on 127.0.0.1). The decode path
has no collective; the only cross-rank steps are the barriers around the timed
region and the max over ranks of the timed milliseconds."""
import contextlib
import io
import os
import socket
import sys

import pytest

REPO = os.path.dirname(os.path.dirname(os.path.abspath(__file__)))

torch = pytest.importorskip("torch")
mp = torch.multiprocessing


def _free_port():
    with socket.socket() as s:
        s.bind(("127.0.0.1", 0))
        return s.getsockname()[1]


def _rank(rank, world, port, queue):
    os.environ.update(MASTER_ADDR="127.0.0.1", MASTER_PORT=str(port), WORLD_SIZE=str(world),
                      RANK=str(rank), LOCAL_RANK=str(rank))
    sys.path.insert(0, REPO)
    import bench
    import torch.distributed as dist

    w, r, local = bench.dist_setup(world, backend="gloo")
    bench.barrier(w)
    rank_ms = [10.0, 12.5][r]
    max_ms, value = bench.aggregate(w, rank_ms, 100)
    # The reference arm runs on rank 0 alone; the others return at once.
    out = io.StringIO()
    if r != 0:
        with contextlib.redirect_stdout(out):
            bench.run_reference(None, w, r)
    bench.barrier(w)
    dist.destroy_process_group()
    queue.put((r, w, local, max_ms, value, out.getvalue()))


def test_two_gloo_ranks_aggregate_max_over_ranks():
    ctx = mp.get_context("spawn")
    queue = ctx.Queue()
    port = _free_port()
    procs = [ctx.Process(target=_rank, args=(r, 2, port, queue)) for r in range(2)]
    for p in procs:
        p.start()
    results = sorted(queue.get(timeout=120) for _ in procs)
    for p in procs:
        p.join(timeout=60)
        assert p.exitcode == 0
    assert [r[:3] for r in results] == [(0, 2, 0), (1, 2, 1)]
    for _, _, _, max_ms, value, printed in results:
        assert max_ms == 12.5  # the slowest rank
        assert value == pytest.approx(2 * 100 / 0.0125)  # all ranks' tokens / that time
    assert results[1][5] == ""  # rank 1 printed no reference line


def test_single_process_needs_no_process_group(monkeypatch):
    sys.path.insert(0, REPO)
    import bench

    for var in ("WORLD_SIZE", "RANK", "LOCAL_RANK"):
        monkeypatch.delenv(var, raising=False)
    assert bench.dist_setup(1) == (1, 0, 0)
    assert bench.aggregate(1, 20.0, 50) == (20.0, 2500.0)
