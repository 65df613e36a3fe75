"""bench.py's reductions over ranks, on CPU: _max_min_over_ranks / _max_over_ranks (the element-wise
max and min that the per-phase split and the timed region of the multi-GPU line use), run as two
gloo ranks (the same collective calls as NCCL ranks). The placement-balance summary is checked in
test_pool_host.py."""
import os
import socket
from datetime import timedelta

import torch.distributed as dist
import torch.multiprocessing as mp

import bench


def _free_port() -> int:
    with socket.socket() as s:
        s.bind(("127.0.0.1", 0))
        return s.getsockname()[1]


def _reduce_worker(rank, world, port, q):
    os.environ.update(MASTER_ADDR="127.0.0.1", MASTER_PORT=str(port))
    dist.init_process_group("gloo", rank=rank, world_size=world, timeout=timedelta(seconds=30))
    try:
        hi, lo = bench._max_min_over_ranks([float(rank), -2.0 * rank, 5.0], "cpu")
        mx = bench._max_over_ranks(1.5 + rank, "cpu")
        q.put((rank, hi, lo, mx))
    finally:
        dist.destroy_process_group()


def _run_ranks(world):
    """Both ranks as spawned processes on a fresh port; their exit codes and the result queue. A rank
    still running after the join timeout is killed (it is this test's own child)."""
    ctx = mp.get_context("spawn")
    q = ctx.Queue()
    port = _free_port()
    procs = [ctx.Process(target=_reduce_worker, args=(r, world, port, q)) for r in range(world)]
    for p in procs:
        p.start()
    for p in procs:
        p.join(timeout=60)
    for p in procs:
        if p.is_alive():
            p.kill()
            p.join()
    return [p.exitcode for p in procs], q


def test_max_min_over_ranks_gloo():
    world = 2
    for _ in range(3):    # the free port can be taken by another process before the ranks bind it
        codes, q = _run_ranks(world)
        if codes == [0] * world:
            break
    assert codes == [0] * world, codes
    got = sorted(q.get(timeout=5) for _ in range(world))
    for rank, hi, lo, mx in got:
        assert hi == [1.0, 0.0, 5.0], (rank, hi)     # every rank receives the same result
        assert lo == [0.0, -2.0, 5.0], (rank, lo)
        assert mx == 2.5, (rank, mx)
