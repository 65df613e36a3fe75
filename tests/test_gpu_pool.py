"""Device-side expert cache (eva_pool_plan / eva_pool_copy) on a B200 (-m gpu).

* The planner's slot choice, stamps, CLOCK hand and pointer tables equal a Python model of the same
  policy after every plan of a random sequence of exact plans and prefetches over three layers that
  share one pool, and every resident slot holds its expert's record bytes.
* Split plans divide the routes into those of resident experts and those of experts being copied.
* When a prefetch leaves too few slots for another layer's exact plan, the status says so and the
  routes of the experts left without a slot get weight 0.
* An expert-parallel stack whose layers share a pool smaller than their experts gives the same
  outputs as whole resident layers (resident experts' launch overlapping the misses' copies, the
  copied experts' launch after them, prefetches on the copy stream), with no host synchronisation
  in the step.
"""
import numpy as np
import pytest
import torch

from eva_b200 import config as C
from eva_b200.experts import ROW, make_layer, record_layout
from eva_b200.residency import ExpertPool

pytestmark = pytest.mark.gpu
DEV = "cuda"
SMALL = C.MoEConfig("pool", hidden=512, inter=256, n_experts=16, topk=4, router="sigmoid", n_group=4,
                    topk_group=2, route_scale=2.5, norm_topk=True, shared_inter=384, bits=3, shared_bits=4)


class PoolModel:
    """The planner's policy restated: hits stamped first; misses in expert order take the next slot of
    the CLOCK hand that is free or stamped before `protect`; exact plans use stamp counter + 1 and
    protect it, prefetches (the layer's last exact needed set) use counter + 1 and protect counter."""

    def __init__(self, n_slots, n_layers, n_local):
        self.owner = [-1] * n_slots
        self.stamp = [0] * n_slots
        self.hand, self.counter = 0, 0
        self.slot_of = [[-1] * n_local for _ in range(n_layers)]
        self.last = [set() for _ in range(n_layers)]

    def plan(self, li, needed, prefetch):
        n = len(self.owner)
        if prefetch:
            needed = self.last[li]
        else:
            self.last[li] = set(needed)
        cur = self.counter
        stamp = cur + 1
        protect = cur if prefetch else stamp
        if not prefetch:
            self.counter = stamp
        for e in sorted(needed):
            if self.slot_of[li][e] >= 0:
                self.stamp[self.slot_of[li][e]] = stamp
        jobs = []
        for e in sorted(needed):
            if self.slot_of[li][e] >= 0:
                continue
            s = None
            for _ in range(2 * n):
                c = self.hand
                self.hand = (self.hand + 1) % n
                if self.owner[c] < 0 or self.stamp[c] < protect:
                    s = c
                    break
            if s is None:
                assert prefetch, "an exact plan always finds a slot"
                break
            if self.owner[s] >= 0:
                ol, oe = self.owner[s] >> 16, self.owner[s] & 0xffff
                self.slot_of[ol][oe] = -1
            self.owner[s] = (li << 16) | e
            self.stamp[s] = stamp
            self.slot_of[li][e] = s
            jobs.append((e, s))
        return jobs


@pytest.mark.parametrize("start", [0, 2**31 - 20], ids=["counter-0", "counter-past-int32"])
def test_planner_matches_policy_model_and_copies_records(start):
    """start: the plan counter the pool begins at. From 2^31 - 20 the run's plans take it past the
    int32 range (as hours of serving would), and stamp ordering must still hold."""
    L, n_slots = 3, 20
    hosts = [make_layer(SMALL, "cpu", seed=40 + i) for i in range(L)]
    rec = hosts[0].record_bytes
    pool = ExpertPool(DEV, n_slots, rec)
    pool.state[6:8].view(torch.int64).fill_(start)
    pls = [pool.add_layer(h) for h in hosts]
    model = PoolModel(n_slots, L, SMALL.n_experts)
    model.counter = start
    offs, _, _ = record_layout(SMALL.hidden, SMALL.inter, SMALL.bits)
    rng = np.random.default_rng(0)
    for step in range(12):
        for li in range(L):
            if step > 0 and rng.random() < 0.5:
                pls[li].prefetch()
                model.plan(li, None, True)
            M = int(rng.integers(1, 5))
            sel = np.stack([rng.choice(SMALL.n_experts, SMALL.topk, replace=False) for _ in range(M)]).astype(np.int32)
            rw = rng.random((M, SMALL.topk)).astype(np.float32)
            rw[rng.random(rw.shape) < 0.2] = 0
            needed = {int(e) for e, w in zip(sel.ravel(), rw.ravel()) if w != 0}
            split = step % 2 == 1
            r = pls[li].plan(torch.tensor(sel, device=DEV), torch.tensor(rw, device=DEV), split=split)
            jobs = model.plan(li, needed, False)
            torch.cuda.synchronize()
            if split:                                  # routes of copied experts -> rw_miss, others -> rw_hit
                copied = np.isin(sel, [e for e, _ in jobs])
                hit, miss, _ = r
                assert np.array_equal(hit.cpu().numpy(), np.where(copied, 0, rw))
                assert np.array_equal(miss.cpu().numpy(), np.where(copied, rw, 0))
            assert pool.status() == 0
            assert pool.owner.cpu().tolist() == model.owner
            assert pool.stamp.cpu().tolist() == model.stamp
            assert pool.state[0].item() == model.hand and pool.plan_counter() == model.counter
            assert [(int(a), int(b)) for a, b in zip(pls[li].jobs[1::2].cpu()[: len(jobs)],
                                                     pls[li].jobs[2::2].cpu()[: len(jobs)])] == jobs
            for lj in range(L):
                assert pls[lj].slot_of.cpu().tolist() == model.slot_of[lj]
                tab = pls[lj].packed.cpu().numpy()
                for e, s in enumerate(model.slot_of[lj]):
                    if s < 0:
                        assert not tab[:, e].any()
                    else:
                        base = pool.slots.data_ptr() + s * rec
                        assert all(tab[row, e] == base + offs[key][0] for key, row in ROW.items())
            for e in sorted(needed):                   # every needed expert's slot holds its record
                s = model.slot_of[li][e]
                got = pool.slots[s * rec:(s + 1) * rec].cpu()
                assert torch.equal(got, hosts[li].storage[e * rec:(e + 1) * rec])
    assert pool.bytes_copied() % rec == 0 and pool.bytes_copied() > 0


def test_capacity_drops_routes_of_experts_left_without_a_slot():
    """A prefetch protects its layer's slots against the next exact plan of another layer: with 20
    slots, 10 protected by layer 1's prefetch and 16 needed by layer 2, 6 of layer 2's experts get no
    slot; the status says so and their routes get weight 0 (in place, and in the split outputs)."""
    hosts = [make_layer(SMALL, "cpu", seed=80 + i) for i in range(3)]
    for split in (False, True):
        pool = ExpertPool(DEV, 20, hosts[0].record_bytes)
        pls = [pool.add_layer(h) for h in hosts]
        sel1 = torch.arange(10, dtype=torch.int32, device=DEV).view(5, 2)
        pls[1].plan(sel1, torch.ones(5, 2, device=DEV))
        pls[1].prefetch()
        sel2 = torch.arange(16, dtype=torch.int32, device=DEV).view(4, 4)
        rw2 = torch.full((4, 4), 0.5, device=DEV)
        r = pls[2].plan(sel2, rw2, split=split)
        torch.cuda.synchronize()
        assert pool.status() & 4
        bound = pls[2].slot_of.cpu().numpy() >= 0
        assert bound.sum() == 10
        kept = bound[sel2.cpu().numpy()]
        if split:
            hit, miss, _ = r
            assert np.array_equal(hit.cpu().numpy(), np.zeros((4, 4), np.float32))
            assert np.array_equal(miss.cpu().numpy(), np.where(kept, 0.5, 0).astype(np.float32))
        else:
            assert np.array_equal(rw2.cpu().numpy(), np.where(kept, 0.5, 0).astype(np.float32))
        assert not pls[2].packed.cpu().numpy()[:, ~bound].any()


@pytest.mark.parametrize("M,n_slots", [(8, 16), (24, 24)])
def test_pooled_stack_matches_resident_layers(M, n_slots):
    from eva_b200.ep import EPMoE, ExpertPlacement
    from eva_b200.runner import EvaMoE
    L = 3
    hosts = [make_layer(SMALL, "cpu", seed=60 + i) for i in range(L)]
    pool = ExpertPool(DEV, n_slots, hosts[0].record_bytes)
    pls = [pool.add_layer(h) for h in hosts]
    for a, b in zip(pls, pls[1:]):
        a.next = b
    pl = ExpertPlacement.contiguous(SMALL.n_experts, 1)
    eps = [EPMoE(h, pl, max_tokens=M, residency=r) for h, r in zip(hosts, pls)]
    full = [EvaMoE(h.to(DEV), max_rows=M) for h in hosts]
    g = torch.Generator(device=DEV).manual_seed(M)
    for step in range(4):
        x = torch.randn(M, SMALL.hidden, device=DEV, generator=g).to(torch.bfloat16)
        for li in range(L):
            a = torch.empty(M, SMALL.hidden, device=DEV)
            b = torch.empty(M, SMALL.hidden, device=DEV)
            eps[li].forward(x, out_f32=a)
            full[li].forward(x, out_f32=b)
            torch.cuda.synchronize()
            assert eps[li].status() == 0 and full[li].status() == 0 and pool.status() == 0
            err = (a - b).abs().max().item() / b.abs().max().item()
            assert err < 1e-4, (step, li, err)
            x = b.to(torch.bfloat16)
    assert pool.bytes_copied() > 0
    for ep in eps:
        ep.close()
