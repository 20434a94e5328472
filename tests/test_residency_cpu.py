"""Slot bookkeeping of partial residency (vxmoe.residency.SlotAssigner, the
reference's ExpertPool.assign, models/flashnext/expert_pool.py:123-159):
hits move to the most recent end, misses take free slots and then the least
recently used entry not needed by the same request, a request larger than
the pool fails before anything changes, and a released layer's slots come
back."""
from __future__ import annotations

import pytest

from vxmoe.residency import SlotAssigner


def test_free_slots_then_lru_eviction():
    a = SlotAssigner(4)
    slots, misses, evicted = a.assign("L0", [5, 6, 5, 7])
    assert sorted(slots) == [5, 6, 7] and len(misses) == 3 and evicted == []
    assert len(set(slots.values())) == 3
    slots2, misses2, _ = a.assign("L1", [5])          # another layer: a different key
    assert misses2 == [(5, slots2[5])] and slots2[5] not in slots.values()
    # L0's 6 is now the least recently used after touching 5 and 7
    a.assign("L0", [5, 7])
    slots3, misses3, evicted3 = a.assign("L1", [9])
    assert evicted3 == [("L0", 6)] and slots3[9] == slots[6]
    assert a.slot("L0", 6) is None and a.slot("L1", 9) == slots[6]
    assert a.hits == 2 and a.misses == 5


def test_eviction_skips_experts_of_the_same_request():
    a = SlotAssigner(3)
    a.assign("L", [1, 2, 3])
    slots, misses, evicted = a.assign("L", [3, 1, 4])   # 2 is the only entry not requested
    assert evicted == [("L", 2)] and misses == [(4, slots[4])]
    assert a.slot("L", 1) is not None and a.slot("L", 3) is not None


def test_capacity_and_release():
    a = SlotAssigner(2)
    a.assign("A", [1, 2])
    with pytest.raises(ValueError):
        a.assign("B", [1, 2, 3])
    assert a.slot("A", 1) is not None and a.slot("A", 2) is not None   # unchanged
    assert sorted(a.release("A")) == [("A", 1), ("A", 2)]
    assert a.usable_slots == 2
    slots, misses, evicted = a.assign("B", [7, 8])
    assert len(misses) == 2 and evicted == []
    with pytest.raises(ValueError):
        SlotAssigner(0)
