"""Expert-parallel exchange on the CPU: placement, the dispatch plan, and EPMoE's all-to-all logic
over gloo ranks (world size 2 and 3) with the oracle doing each rank's device work, against the
single-process oracle layer."""
import os
import socket
import tempfile

import numpy as np
import pytest
import torch
import torch.multiprocessing as mp

from eva_b200 import config as C
from eva_b200.ep import ExpertPlacement
from oracle.ep_oracle import ep_plan

SMALL = C.MoEConfig("small", hidden=256, inter=128, n_experts=12, topk=4, router="sigmoid", n_group=4,
                    topk_group=2, route_scale=2.5, norm_topk=True, shared_inter=256, bits=3, shared_bits=4)


def test_placement_contiguous_and_balanced():
    p = ExpertPlacement.contiguous(12, 4)
    assert p.owner.tolist() == [0, 0, 0, 1, 1, 1, 2, 2, 2, 3, 3, 3]
    assert p.local_id.tolist() == [0, 1, 2] * 4
    assert p.experts_of(2) == (6, 7, 8)
    load = 1.0 / np.arange(1, 257) ** 1.1
    rng = np.random.default_rng(3)
    perm = rng.permutation(256)
    b = ExpertPlacement.balanced(load[perm], 8)
    per_rank = np.bincount(b.owner, minlength=8)
    assert (per_rank == 32).all()
    loads = np.array([load[perm][b.owner == r].sum() for r in range(8)])
    c = ExpertPlacement.contiguous(256, 8)
    cl = np.array([load[perm][c.owner == r].sum() for r in range(8)])
    assert loads.max() <= cl.max() and loads.max() - loads.min() < cl.max() - cl.min()
    # the hottest expert's rank takes only the coldest ones besides it
    assert loads.max() < load[0] + 31 * load[256 - 7 * 32 - 31:].mean() + 1e-9
    flat = ExpertPlacement.balanced(np.ones(256) + 1e-3 * rng.random(256), 8)
    fl = np.array([(flat.owner == r).sum() for r in range(8)])
    assert (fl == 32).all()
    for r in range(8):
        ids = b.experts_of(r)
        assert [int(b.local_id[e]) for e in ids] == list(range(32))
    with pytest.raises(ValueError):
        ExpertPlacement.from_owner([0, 1, 2], 2)


def test_plan_covers_every_active_slot_once():
    rng = np.random.default_rng(0)
    M, k, E, W = 37, 4, 12, 3
    idx = np.stack([rng.choice(E, k, replace=False) for _ in range(M)]).astype(np.int32)
    w = rng.random((M, k)).astype(np.float32)
    w[rng.random((M, k)) < 0.2] = 0
    pl = ExpertPlacement.contiguous(E, W)
    for seg in (0, M):
        cap = W * M
        counts, pos, ssel, srw, over = ep_plan(idx, w, pl.owner, pl.local_id, W, cap, seg)
        assert not over
        seen = np.zeros((M, k), int)
        for r in range(W):
            ms = np.flatnonzero(pos[r] >= 0)
            assert len(ms) == counts[r]
            assert (np.diff(pos[r, ms]) == 1).all()                 # contiguous, token order
            assert not len(ms) or pos[r, ms[0]] == (r * seg if seg else counts[:r].sum())
            for m in ms:
                on = (w[m] != 0) & (pl.owner[idx[m]] == r)
                assert on.any()
                assert (srw[pos[r, m]][on] == w[m][on]).all() and (srw[pos[r, m]][~on] == 0).all()
                assert (ssel[pos[r, m]][on] == pl.local_id[idx[m][on]]).all()
                seen[m] += on
        assert (seen == (w != 0)).all()
    # capacity: the fixed segment too small for rank 0's rows
    counts, pos, _, _, over = ep_plan(idx, w, pl.owner, pl.local_id, W, W * 4, 4)
    assert over and (pos < W * 4).all() and ((pos >= 0).sum(axis=1) <= 4).all()


def _free_port():
    with socket.socket() as s:
        s.bind(("127.0.0.1", 0))
        return s.getsockname()[1]


def _worker(rank, world, port, outdir, mode, M):
    os.environ["MASTER_ADDR"] = "127.0.0.1"
    os.environ["MASTER_PORT"] = str(port)
    import torch.distributed as dist
    from datetime import timedelta
    from eva_b200.ep import EPMoE
    from eva_b200.experts import make_layer
    from oracle.ep_oracle import OracleEpOps
    dist.init_process_group("gloo", rank=rank, world_size=world, timeout=timedelta(seconds=60))
    try:
        pl = ExpertPlacement.balanced(np.arange(SMALL.n_experts, 0, -1), world)
        layer = make_layer(SMALL, "cpu", seed=5, experts=pl.experts_of(rank))
        ep = EPMoE(layer, pl, max_tokens=M, mode=mode, ops=OracleEpOps(layer, pl))
        g = torch.Generator().manual_seed(100 + rank)
        x = torch.randn(M - rank, SMALL.hidden, generator=g).to(torch.bfloat16) if mode == "exact" else \
            torch.randn(M, SMALL.hidden, generator=g).to(torch.bfloat16)
        out32 = torch.empty(x.shape[0], SMALL.hidden)
        ep.forward(x, out_f32=out32)
        np.save(os.path.join(outdir, f"x{rank}.npy"), x.view(torch.int16).numpy())
        np.save(os.path.join(outdir, f"y{rank}.npy"), out32.numpy())
    finally:
        dist.destroy_process_group()


@pytest.mark.parametrize("world,mode,M", [(2, "fixed", 6), (2, "exact", 9), (3, "exact", 7)])
def test_ep_forward_matches_single_process_oracle(oracle, world, mode, M):
    from eva_b200.experts import make_layer
    full = make_layer(SMALL, "cpu", seed=5)
    with tempfile.TemporaryDirectory() as d:
        mp.start_processes(_worker, args=(world, _free_port(), d, mode, M), nprocs=world, start_method="spawn")
        for r in range(world):
            xb = np.load(os.path.join(d, f"x{r}.npy")).view(np.uint16)
            y = np.load(os.path.join(d, f"y{r}.npy"))
            ref, _, _, _ = oracle.layer_forward(xb, full)
            err = np.abs(y - ref).max() / np.abs(ref).max()
            assert err < 1e-5, (r, err)


def test_expert_subset_holds_the_same_records():
    from eva_b200.experts import make_layer
    full = make_layer(SMALL, "cpu", seed=9)
    part = make_layer(SMALL, "cpu", seed=9, experts=(7, 2, 11))
    rec = full.record_bytes
    for i, e in enumerate((7, 2, 11)):
        assert torch.equal(part.storage[i * rec:(i + 1) * rec], full.storage[e * rec:(e + 1) * rec])
    assert torch.equal(part.storage[3 * rec:], full.storage[SMALL.n_experts * rec:])
    assert part.packed.shape == (9, 3) and part.n_local == 3
    with pytest.raises(ValueError):
        make_layer(SMALL, "cpu", experts=(1, 1))


def _dropout_worker(rank, world, port, outdir):
    """Rank 1 joins the group but never enters the step; rank 0's step must end with an error
    within the process group's timeout instead of waiting for it."""
    os.environ["MASTER_ADDR"] = "127.0.0.1"
    os.environ["MASTER_PORT"] = str(port)
    import time
    import torch.distributed as dist
    from datetime import timedelta
    from eva_b200.ep import EPMoE
    from eva_b200.experts import make_layer
    from oracle.ep_oracle import OracleEpOps
    dist.init_process_group("gloo", rank=rank, world_size=world, timeout=timedelta(seconds=3))
    pl = ExpertPlacement.contiguous(SMALL.n_experts, world)
    layer = make_layer(SMALL, "cpu", seed=5, experts=pl.experts_of(rank))
    ep = EPMoE(layer, pl, max_tokens=4, mode="exact", ops=OracleEpOps(layer, pl))   # both ranks set up
    x = torch.randn(4, SMALL.hidden, generator=torch.Generator().manual_seed(1)).to(torch.bfloat16)
    ep.forward(x, out_f32=torch.empty(4, SMALL.hidden))   # one healthy step on both ranks
    if rank == 1:
        time.sleep(8)                  # leaves between steps: past rank 0's timeout, no collective
        return
    t0 = time.time()
    try:
        ep.forward(x, out_f32=torch.empty(4, SMALL.hidden))
        outcome = "completed"
    except Exception as e:             # the collective's timeout surfaces as an exception on the host
        outcome = f"raised {type(e).__name__}: {' '.join(str(e).split())[:300]}"
    with open(os.path.join(outdir, "rank0.txt"), "w") as f:
        f.write(f"{outcome}\n{time.time() - t0:.1f}\n")


def test_ep_step_fails_on_the_host_when_a_rank_never_joins():
    import time
    with tempfile.TemporaryDirectory() as d:
        ctx = mp.start_processes(_dropout_worker, args=(2, _free_port(), d), nprocs=2, start_method="spawn",
                                 join=False)
        t_end = time.time() + 120
        done = False
        while not done and time.time() < t_end:
            done = ctx.join(timeout=1)
        if not done:
            for p in ctx.processes:
                if p.is_alive():
                    p.kill()
            pytest.fail("workers did not finish")
        outcome, took = open(os.path.join(d, "rank0.txt")).read().splitlines()[:2]
        # the step that rank 1 never joined ends by the group's 3 s timeout: not at once (some other
        # error), not by waiting for the rank
        assert outcome.startswith("raised"), outcome
        assert "timed out" in outcome.lower() or "timeout" in outcome.lower(), outcome
        assert 2.5 <= float(took) < 30.0, took
