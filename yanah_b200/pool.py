"""Expert slot pool bookkeeping (host side) and its offline replay.

`SlotPool` keeps the reference's contract (moe_prefetch/pool.py:90-282) so
that the orchestrator, the speculative scheduler and recorded traces behave
identically on top of HBM slots (`backend.CudaExpertMemory`):

* CLOCK over the demand slots: a hit sets the slot's reference bit; the
  victim scan moves a hand around the pool, clears set bits and takes the
  first slot that is unpinned, not reserved for a speculative read, not in
  the speculative partition and has a clear bit. Free slots are used first,
  lowest index first.
* Speculative partition: `spec_slot_cap` slots (the first ones handed out)
  belong to speculation, invisible to the scan. A forecast read is reserved
  in the partition (never evicts); a forecast that is demanded is adopted in
  place (its slot joins the cache) and the partition takes one CLOCK victim
  to stay full; an unused forecast goes back to the partition.
* Pins protect the slots of the layer being computed.

The reference's offline cache simulator (moe_prefetch/cache_sim.py) is not
part of this package: the streaming decoder writes its routing trace in that
tool's format (yanah_b200/trace.py), so the reference's own simulator can
replay it.
"""
from __future__ import annotations

import threading
from dataclasses import dataclass, field
from typing import Callable, Dict, List, Optional, Sequence, Tuple

Key = Tuple[int, int]  # (layer, expert)


@dataclass
class PoolStats:
    hits: int = 0
    misses: int = 0
    evictions: int = 0
    adopted: int = 0
    spec_reserved: int = 0
    spec_discarded: int = 0
    spec_refused: int = 0
    adopt_evictions: int = 0
    admitted: int = 0

    @property
    def hit_rate(self) -> float:
        return self.hits / max(1, self.hits + self.misses)


class SlotPool:
    def __init__(self, geometry, slots: int, spec_slot_cap: int = 32, spec_headroom: Optional[int] = None,
                 memory=None):
        k = geometry.top_k
        if slots < 3 * k:
            raise ValueError(f"pool of {slots} slots: at least 3 x top_k = {3 * k} are needed "
                             f"(one layer's experts pinned, with room to evict)")
        if slots - spec_slot_cap < 3 * k:
            raise ValueError(f"pool of {slots} slots with a speculative partition of {spec_slot_cap}: "
                             f"{slots - spec_slot_cap} demand slots left, at least {3 * k} are needed")
        self.g, self.slots, self.memory = geometry, slots, memory
        self.slot_bytes = geometry.slot_nbytes
        self.spec_slot_cap = spec_slot_cap
        self.spec_headroom = spec_headroom if spec_headroom is not None else 2 * k + 8
        n = slots
        self.key_of: List[Optional[Key]] = [None] * n
        self.ref_bit = [False] * n
        self.pins = [0] * n
        self.in_flight = [False] * n
        self.spec_owned = [False] * n
        self.map: Dict[Key, int] = {}
        self._next_fresh = 0            # never-used slots are handed out in index order
        self._freed: List[int] = []     # slots given back by `abandon` (used before fresh ones)
        self.hand = 0
        self.pinned_count = 0
        self.in_flight_count = 0
        self.spec_free: List[int] = []
        for _ in range(spec_slot_cap):
            s = self._take_free()
            self.spec_owned[s] = True
            self.spec_free.append(s)
        self._spec_deficit = 0
        self._returned: List[int] = []
        self._lock = threading.Lock()
        self.stats = PoolStats()

    # ------------------------------------------------------------ internals
    def _has_free(self) -> bool:
        return bool(self._freed) or self._next_fresh < self.slots

    def _take_free(self) -> int:
        if self._freed:
            return self._freed.pop()
        s = self._next_fresh
        self._next_fresh += 1
        return s

    def _victim(self) -> int:
        if self._has_free():
            return self._take_free()
        for _ in range(3 * self.slots):
            s = self.hand
            self.hand = s + 1 if s + 1 < self.slots else 0
            if self.pins[s] or self.in_flight[s] or self.spec_owned[s]:
                continue
            if self.ref_bit[s]:
                self.ref_bit[s] = False
                continue
            old = self.key_of[s]
            if old is not None:
                del self.map[old]
                self.key_of[s] = None
                self.stats.evictions += 1
            return s
        raise MemoryError(f"no evictable slot among {self.slots}: every slot is pinned, reserved for a "
                          f"forecast read or in the speculative partition")

    # ----------------------------------------------------------------- memory
    def views(self, slot: int):
        return self.memory.views(slot)

    def lookup(self, key: Key) -> Optional[int]:
        return self.map.get(key)

    def is_resident(self, key: Key) -> bool:
        return key in self.map

    def resident_count(self) -> int:
        return len(self.map)

    # ------------------------------------------------------------------ demand
    def pin(self, slot: int) -> None:
        if not self.pins[slot]:
            self.pinned_count += 1
        self.pins[slot] += 1

    def unpin(self, slot: int) -> None:
        self.pins[slot] -= 1
        if not self.pins[slot]:
            self.pinned_count -= 1

    def hit(self, key: Key) -> Optional[int]:
        s = self.map.get(key)
        if s is None:
            return None
        self.ref_bit[s] = True
        self.pin(s)
        self.stats.hits += 1
        return s

    def claim_for_demand(self, key: Key) -> int:
        s = self._victim()
        self.pin(s)
        self.stats.misses += 1
        return s

    def publish(self, slot: int, key: Key) -> None:
        self.key_of[slot] = key
        self.map[key] = slot
        self.ref_bit[slot] = True

    def abandon(self, slot: int) -> None:
        self.unpin(slot)
        self._freed.append(slot)

    # ------------------------------------------------------------- speculation
    def reserve_speculative(self, key: Key) -> Optional[int]:
        self.drain_returned()
        if key in self.map:
            return None
        if not self.spec_free:
            self._refill_partition()
        if not self.spec_free:
            self.stats.spec_refused += 1
            return None
        s = self.spec_free.pop()
        self.in_flight[s] = True
        self.in_flight_count += 1
        self.stats.spec_reserved += 1
        return s

    def _refill_partition(self) -> None:
        while self._spec_deficit > 0:
            try:
                v = self._victim()
            except MemoryError:
                return
            self.spec_owned[v] = True
            self.ref_bit[v] = False
            self.spec_free.append(v)
            self._spec_deficit -= 1
            self.stats.adopt_evictions += 1

    def adopt(self, slot: int, key: Key) -> None:
        if not (self.in_flight[slot] and self.key_of[slot] is None and self.spec_owned[slot]):
            raise RuntimeError(f"slot {slot} is not a completed speculative read")
        self.in_flight[slot] = False
        self.in_flight_count -= 1
        self.spec_owned[slot] = False
        self.publish(slot, key)
        self.pin(slot)
        self.stats.adopted += 1
        self.stats.hits += 1
        self._spec_deficit += 1
        self._refill_partition()

    def return_speculative(self, slot: int) -> None:
        with self._lock:
            self._returned.append(slot)

    def drain_returned(self) -> None:
        with self._lock:
            back, self._returned = self._returned, []
        for s in back:
            if self.in_flight[s]:
                self.in_flight[s] = False
                self.in_flight_count -= 1
                self.stats.spec_discarded += 1
                self.spec_free.append(s)

    # ------------------------------------------------------------------ prefill
    def admit(self, layer: int, experts_by_frequency: Sequence[int], share: int,
              copy_into: Callable[[int, object], None]) -> int:
        written = 0
        for e in list(experts_by_frequency)[:share]:
            key = (layer, e)
            s = self.map.get(key)
            if s is not None:
                self.ref_bit[s] = True
                continue
            s = self._victim()
            copy_into(e, self.views(s) if self.memory is not None else None)
            self.publish(s, key)
            written += 1
        self.stats.admitted += written
        return written

    def close(self) -> None:
        if self.memory is not None:
            self.memory.close()
