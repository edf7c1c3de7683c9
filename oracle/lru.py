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
