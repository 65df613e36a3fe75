"""Host-side pieces of bench.py's multi-GPU line, on CPU.

* _max_min_over_ranks / _max_over_ranks: the element-wise max and min over ranks that the per-phase
  split and the timed region use, run as two gloo ranks (the same collective calls as NCCL ranks).
* _placement_balance: routed slots and distinct experts per rank from gathered routes, checked
  against counts done by hand.
"""
import os
import socket
from datetime import timedelta

import pytest
import torch
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


def test_max_min_over_ranks_gloo():
    world = 2
    ctx = mp.get_context("spawn")
    q = ctx.Queue()
    port = _free_port()
    procs = [ctx.Process(target=_reduce_worker, args=(r, world, port, q)) for r in range(world)]
    for p in procs:
        p.start()
    for p in procs:
        p.join(timeout=60)
        assert p.exitcode == 0, p.exitcode
    got = sorted(q.get(timeout=5) for _ in range(world))
    for rank, hi, lo, mx in got:
        assert hi == [1.0, 0.0, 5.0], (rank, hi)     # every rank receives the same result
        assert lo == [0.0, -2.0, 5.0], (rank, lo)
        assert mx == 2.5, (rank, mx)


def test_placement_balance_counts():
    # 4 experts: 0, 1 on rank 0; 2, 3 on rank 1. Routes [steps, world, M, k].
    owner = torch.tensor([0, 0, 1, 1])
    allidx = torch.tensor([
        [[[0, 2], [0, 1]], [[3, 2], [0, 2]]],   # step 0: rank-0 slots 4, rank-1 slots 4; distinct {0,1,2,3}
        [[[1, 1], [1, 0]], [[0, 3], [1, 0]]],   # step 1: rank-0 slots 7, rank-1 slots 1; distinct {0,1,3}
    ])
    b = bench._placement_balance(allidx, owner, 2)
    assert b["slots_per_step_max_rank"] == pytest.approx(5.5)       # rank 0: (4 + 7) / 2
    assert b["slots_per_step_min_rank"] == pytest.approx(2.5)       # rank 1: (4 + 1) / 2
    assert b["slots_max_over_mean"] == pytest.approx(5.5 / 4.0)
    assert b["distinct_experts_per_step_max_rank"] == pytest.approx(2.0)   # rank 0: 2 and 2
    assert b["distinct_experts_per_step_min_rank"] == pytest.approx(1.5)   # rank 1: 2 and 1
