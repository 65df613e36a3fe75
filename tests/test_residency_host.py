"""Expert residency policy on the CPU: free slots first, least-recently-used eviction that never
evicts an expert the current step needs, and the budget error."""
import pytest

from eva_b200.residency import SlotLRU


def test_lru_assigns_free_slots_then_evicts_least_recent():
    p = SlotLRU(3)
    assert [p.assign(e, set())[0] for e in (10, 11, 12)] == [0, 1, 2]
    assert p.lookup(10) == 0              # touch 10: 11 is now least recent
    slot, ev = p.assign(13, {13})
    assert (slot, ev) == (1, 11) and p.lookup(11) is None
    slot, ev = p.assign(14, {14, 12})     # 12 protected: evict 10 (least recent unprotected)
    assert ev == 10 and slot == 0
    assert sorted(p.slot_of.items()) == [(12, 2), (13, 1), (14, 0)]


def test_lru_refuses_when_every_slot_is_needed():
    p = SlotLRU(2)
    p.assign(1, {1, 2, 3})
    p.assign(2, {1, 2, 3})
    with pytest.raises(RuntimeError):
        p.assign(3, {1, 2, 3})
    with pytest.raises(ValueError):
        p.assign(1, set())
    with pytest.raises(ValueError):
        SlotLRU(0)
