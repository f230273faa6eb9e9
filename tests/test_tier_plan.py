"""CPU checks of the pinned-host tier's slot bookkeeping (tier.plan_slots):
free slots first, then least-recently-used eviction that never evicts an
expert the same call needs, hits refresh their slot's clock."""
import numpy as np


def _state(E, slots):
    return np.full(E, -1, np.int64), np.full(slots, -1, np.int64), np.zeros(slots, np.int64)


def test_free_slots_then_lru(fm):
    plan = fm.tier.plan_slots
    slot_of, owner, used = _state(10, 3)
    assert plan(np.array([4, 7]), slot_of, owner, used, 1) == [(4, 0), (7, 1)]
    assert plan(np.array([7, 2]), slot_of, owner, used, 2) == [(2, 2)]   # 7 is a hit
    assert used.tolist() == [1, 2, 2]
    # all slots taken: the least recently used one (expert 4, clock 1) goes
    assert plan(np.array([9]), slot_of, owner, used, 3) == [(9, 0)]
    assert slot_of[4] == -1 and slot_of[9] == 0 and owner.tolist() == [9, 7, 2]
    # the needed experts keep their slots even when older than the others
    assert plan(np.array([7, 2, 5]), slot_of, owner, used, 4) == [(5, 0)]
    assert sorted(owner.tolist()) == [2, 5, 7]
    assert all(slot_of[owner[s]] == s for s in range(3))


def test_repeated_calls_are_hits(fm):
    plan = fm.tier.plan_slots
    slot_of, owner, used = _state(8, 4)
    plan(np.array([0, 1, 2, 3]), slot_of, owner, used, 1)
    for c in range(2, 6):
        assert plan(np.array([3, 1]), slot_of, owner, used, c) == []
    # 0 and 2 were last used at clock 1: evicted first, lower clock first then lower slot
    assert plan(np.array([5, 6]), slot_of, owner, used, 6) == [(5, 0), (6, 2)]
