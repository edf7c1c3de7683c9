"""LRU neuron-cache accounting of reference runtime/temporal.py:55-75 (test infrastructure only)."""
from __future__ import annotations

from collections import OrderedDict


def neuron_payload(hidden: int = 5120, bits: int = 16) -> int:
    """runtime/temporal.py:55."""
    return int(3 * hidden * bits / 8)


def lru_events(masks, capacity: int, hidden: int = 5120, bits: int = 16):
    """One contiguous token sequence through an LRU of `capacity` neurons.

    Per token: hits, misses, evicted and bytes (misses * payload), with the
    reference's eviction rule (least-recent neuron not in the current set).
    """
    cache: OrderedDict[int, None] = OrderedDict()
    events = []
    for row in masks:
        active = [int(v) for v in row]
        if capacity < len(active):
            raise ValueError("cache capacity must hold the complete active set")
        active_set = set(active)
        hits = sum(v in cache for v in active)
        misses = len(active) - hits
        for v in active:
            if v in cache:
                cache.move_to_end(v)
            else:
                cache[v] = None
        evicted = 0
        while len(cache) > capacity:
            victim = next(key for key in cache if key not in active_set)
            del cache[victim]
            evicted += 1
        events.append({"hits": hits, "misses": misses, "evicted": evicted,
                       "bytes_transferred": misses * neuron_payload(hidden, bits), "cache_size": len(cache)})
    return events


class SlotCache:
    """Slot-level restatement of the device cache policy (qcc_cache_resolve).

    n_hot always-resident records occupy resident slots [0, n_hot) in the
    order of `hot_ids`; `capacity` cache slots follow.  Per step (sorted,
    unique ids): hot records and cached records are resident; each miss takes
    the least recently used slot the step does not use -- empty slots first,
    ties by the held record's id, then slot -- which keeps exactly the entries
    the reference's OrderedDict LRU keeps (runtime/temporal.py:57-75).
    """

    def __init__(self, n_records: int, hot_ids, capacity: int):
        self.n_hot = len(hot_ids)
        self.capacity = capacity
        self.slot_of = [-1] * n_records
        for slot, n in enumerate(hot_ids):
            self.slot_of[int(n)] = slot
        self.owner = [-1] * capacity
        self.last_use = [-1] * capacity

    def step(self, ids, step: int) -> dict:
        resident, misses, active = [], [], set()
        hits = hot = 0
        for n in (int(v) for v in ids):
            s = self.slot_of[n]
            if s >= 0:
                resident.append(s)
                if s < self.n_hot:
                    hot += 1
                else:
                    hits += 1
                    active.add(s - self.n_hot)
            else:
                misses.append(n)
        for c in active:
            self.last_use[c] = step
        order = sorted((c for c in range(self.capacity) if c not in active),
                       key=lambda c: (self.last_use[c] + 1, self.owner[c] + 1, c))
        served = min(len(misses), len(order))
        miss_slots, evicted = [], 0
        for i in range(served):
            c = order[i]
            old = self.owner[c]
            if old >= 0:
                self.slot_of[old] = -1
                evicted += 1
            self.owner[c] = misses[i]
            self.last_use[c] = step
            self.slot_of[misses[i]] = self.n_hot + c
            miss_slots.append(self.n_hot + c)
        return {"resident": resident, "miss_ids": misses[:served], "miss_slots": miss_slots, "hits": hits,
                "hot_hits": hot, "misses": served, "evicted": evicted, "overflow": served < len(misses)}
