"""Prompt passes through a prefill sweep over tagged host memory, for parity
of the sweep's bookkeeping with the reference (moe_prefetch/sweep.py:80-138).

Used twice with the same inputs: by tests/golden/make_golden.py on the
reference's PrefillSweep / SlotPool (to write the fixture) and by
tests/test_sweep_golden.py on yanah_b200.sweep / yanah_b200.pool (to compare).
Every slot holds an 8-byte tag (layer, expert); the reader writes tags, the
fake `moe` checks the tag of every staging row it is given, so the log also
proves which bytes reached which staging slot and which pool slot.
"""
from __future__ import annotations

import struct
from typing import List

import numpy as np

TAG = struct.Struct("<ii")


class TagMemory:
    def __init__(self, n: int):
        self.n = n
        self._buf = bytearray(TAG.size * max(1, n))
        self._view = memoryview(self._buf)

    def views(self, i: int) -> List[memoryview]:
        return [self._view[TAG.size * i:TAG.size * (i + 1)]]

    def tag(self, i: int):
        return TAG.unpack(bytes(self.views(i)[0]))

    def close(self) -> None:
        pass


class DoneFuture:
    def result(self, timeout=None):
        return None


class TagReader:
    """submit_runs of io_lanes.py:157-173 over tags: logs each call's experts."""

    def __init__(self):
        self.log = []

    def submit_runs(self, layer, experts, dst_for):
        experts = [int(e) for e in experts]
        self.log.append([layer, experts])
        for e in experts:
            dst_for(e)[0][:] = TAG.pack(layer, e)
        return [DoneFuture()]


def make_prompts(rng, n_passes: int, L: int, T: int, E: int, k: int, zipf: float = 1.1):
    """Routed ids (n_passes, L, T, k), k distinct experts per row, Zipf(zipf)
    popularity permuted per layer; routing weights (n_passes, L, T, k)."""
    pop = 1.0 / np.arange(1, E + 1) ** zipf
    pop /= pop.sum()
    ids = np.zeros((n_passes, L, T, k), np.int64)
    for l in range(L):
        perm = rng.permutation(E)
        p = pop[np.argsort(perm)]
        for s in range(n_passes):
            for t in range(T):
                ids[s, l, t] = rng.choice(E, size=k, replace=False, p=p)
    w = rng.random((n_passes, L, T, k))
    return ids, w / w.sum(axis=-1, keepdims=True)


def warm_pool(pool, keys) -> None:
    """Demand-load `keys` (layer, expert) in order: claim, tag, publish, unpin."""
    for key in keys:
        key = (int(key[0]), int(key[1]))
        if pool.hit(key) is None:
            s = pool.claim_for_demand(key)
            pool.views(s)[0][:] = TAG.pack(*key)
            pool.publish(s, key)
        else:
            s = pool.lookup(key)
        pool.unpin(s)


def drive_sweep(sweep_cls, pool, ids: np.ndarray, w: np.ndarray, group: int) -> dict:
    """Run every pass of `ids` through `sweep_cls(pool, reader, ...)`, the last
    pass admitting. Returns the event logs, outputs, pool maps and stats."""
    reader = TagReader()
    moe_log = []

    def moe(layer, x, ids_l, w_l, memory, rows):
        for e, r in rows.items():
            assert memory.tag(r) == (layer, e), (layer, e, r, memory.tag(r))
        present = np.isin(ids_l, np.fromiter(rows.keys(), dtype=np.int64))
        moe_log.append([layer, sorted([int(e), int(r)] for e, r in rows.items())])
        return (w_l * (ids_l + 1) * present).sum(axis=1)

    sweep = sweep_cls(pool, reader, min_tokens=16, group=group, make_memory=TagMemory)
    outs, maps = [], []
    n_passes, L = ids.shape[:2]
    for p in range(n_passes):
        for l in range(L):
            out = sweep.run_layer(l, None, ids[p, l], w[p, l], moe, p == n_passes - 1)
            outs.append(np.asarray(out, np.float64).tolist())
            maps.append(sorted([int(k[0]), int(k[1]), int(s)] for k, s in pool.map.items()))
        sweep.stats.passes += 1
    # every resident slot holds its key's bytes (admissions copied from staging)
    for k, s in pool.map.items():
        assert TAG.unpack(bytes(pool.views(s)[0])) == tuple(k), (k, s)
    st = sweep.stats
    ps = pool.stats
    return {
        "reader": reader.log, "moe": moe_log, "outs": outs, "maps": maps,
        "sweep_stats": [st.passes, st.layers, st.pool_copies, st.host_records, st.admitted],
        "pool_stats": [ps.hits, ps.misses, ps.evictions, ps.admitted],
        "fair_share": sweep.fair_share(),
    }
