"""The two-tier expert store's pool policy (CPU): least recently used
placement, no eviction among the experts of one call, pool-size errors."""
import pytest

from exq_b200.offload import SlotPool


def test_pool_places_reuses_and_evicts_least_recently_used():
    p = SlotPool(3)
    place, loads = p.assign([4, 9])
    assert set(place) == {4, 9} and sorted(e for e, _ in loads) == [4, 9]
    place, loads = p.assign([9, 2])               # 9 hits, 2 loads into the free entry
    assert loads == [(2, place[2])] and len(set(place.values())) == 2
    place, loads = p.assign([7])                  # full: evicts 4, the least recently used
    assert p.evicted == [4]
    assert not p.resident(4) and p.resident(9) and p.resident(2) and p.resident(7)
    assert p.hits == 1 and p.misses == 4
    assert sorted(p.where.values()) == [0, 1, 2]


def test_pool_never_evicts_an_expert_of_the_same_call():
    p = SlotPool(2)
    p.assign([1, 2])
    place, loads = p.assign([2, 3])               # 1 is evicted, not 2
    assert p.resident(2) and p.resident(3) and not p.resident(1)
    assert place[2] != place[3]


def test_pool_rejects_more_experts_than_entries():
    p = SlotPool(2)
    with pytest.raises(ValueError):
        p.assign([1, 2, 3])
    with pytest.raises(ValueError):
        SlotPool(0)


def test_pool_duplicates_count_once():
    p = SlotPool(2)
    place, loads = p.assign([5, 5, 5])
    assert len(loads) == 1 and p.misses == 1 and p.hits == 0
