"""Device expert cache and bench helpers on the CPU (no GPU needed).

* eva_pool_plan / eva_pool_copy reject bad arguments before any device work: missing pool or
  layers, a record size that is not a multiple of 16 bytes, a split plan with only one of its two
  outputs, a prefetch asking for a split, missing routes in an exact plan.
* The bench's placement-balance summary counts each rank's routed slots and distinct experts.
"""
import ctypes

import numpy as np
import torch

from eva_b200 import _lib

FAKE = 256   # never dereferenced: every call below fails its checks first


def _pool(record_bytes=4096, n_slots=4):
    return _lib.EvaExpertPool(n_slots, 0, record_bytes, FAKE, FAKE, FAKE, FAKE)


def _plan(L, pool, layers=FAKE, sel=FAKE, rw=FAKE, rows=2, topk=4, prefetch=0, jobs=FAKE, hit=None, miss=None):
    return L.eva_pool_plan(ctypes.byref(pool) if pool is not None else None, layers, 0, sel, 0, rw, rows, topk,
                           prefetch, jobs, hit, miss, None)


def test_pool_entry_points_reject_bad_arguments_without_a_gpu():
    L = _lib.load()
    bad = _lib.EVA_ERR_INVALID
    assert _plan(L, None) == bad                                   # no pool
    assert _plan(L, _pool(), layers=None) == bad                   # no layer table
    assert _plan(L, _pool(record_bytes=4100)) == bad               # records not a multiple of 16 bytes
    assert _plan(L, _pool(n_slots=0)) == bad                       # empty pool
    assert _plan(L, _pool(), hit=FAKE) == bad                      # split with one output only
    assert _plan(L, _pool(), miss=FAKE) == bad
    assert _plan(L, _pool(), prefetch=1, hit=FAKE, miss=FAKE) == bad   # a prefetch has no routes to split
    assert _plan(L, _pool(), sel=None) == bad                      # exact plan without routes
    assert _plan(L, _pool(), rows=-1) == bad
    assert _plan(L, _pool(), jobs=None) == bad
    assert L.eva_pool_copy(None, FAKE, 0, FAKE, None) == bad
    assert L.eva_pool_copy(ctypes.byref(_pool()), FAKE, 0, None, None) == bad
    assert L.eva_host_mapped(None) == 0


def test_placement_balance_counts_slots_and_experts_per_rank():
    import bench
    owner = torch.tensor([0, 0, 1, 1, 1, 0])
    # two steps, two ranks' tokens, 2 tokens each, top-2
    allidx = torch.tensor([[[[0, 2], [3, 4]], [[1, 5], [2, 3]]],
                           [[[0, 1], [0, 5]], [[4, 2], [1, 0]]]])
    b = bench._placement_balance(allidx, owner, 2)
    own = owner[allidx]
    slots = [float((own == r).sum()) / 2 for r in range(2)]
    assert b["slots_per_step_max_rank"] == max(slots) and b["slots_per_step_min_rank"] == min(slots)
    assert np.isclose(b["slots_max_over_mean"], max(slots) / np.mean(slots))
    # step 0 touches experts {0,1,2,3,4,5}: rank 0 owns 0,1,5 and rank 1 owns 2,3,4; step 1 {0,1,2,4,5}
    assert b["distinct_experts_per_step_max_rank"] == 3 and b["distinct_experts_per_step_min_rank"] == 2.5
