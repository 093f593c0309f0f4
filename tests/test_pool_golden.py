"""Slot-pool bookkeeping and trace replay against the reference's own code.

Fixtures (tests/golden/pool_*.npz, written by tests/golden/make_golden.py):
the reference SlotPool (moe_prefetch/pool.py) driven by the orchestrator-like
sequence of tests/pool_driver.py on a seeded Zipf(1.1) / repeat-0.6 routing
trace. Every slot decision and the pool statistics are compared exactly.
(The fixtures also hold the reference cache_sim's replay of those traces; the
streaming path's trace is pinned against cache_sim in
tests/test_orchestrator_golden.py and tests/test_gpu_orchestrator.py.)
"""
from __future__ import annotations

from pathlib import Path

import numpy as np
import pytest

from tests.pool_driver import NullMemory, drive_slot_pool, fc_from_arrays, stats_tuple
from yanah_b200.formats import ModelGeometry
from yanah_b200.pool import SlotPool

GOLDEN = Path(__file__).resolve().parent / "golden"
CASES = ["pool_small.npz", "pool_wide.npz"]


def _load(name):
    z = np.load(GOLDEN / name)
    routed = z["routed"].astype(np.int64)
    S, L, k = routed.shape
    return z, routed, fc_from_arrays(z, S, L), S, L, k


@pytest.mark.parametrize("name", CASES)
def test_slot_pool_decisions_match_reference(name):
    z, routed, fc, S, L, k = _load(name)
    E = 128 if "small" in name else 512
    g = ModelGeometry(n_layers=L, n_mtp_layers=0, n_experts=E, top_k=k, hidden=64, moe_inter=32, bits=4,
                      group_size=32)
    pool = SlotPool(g, int(z["slots"]), spec_slot_cap=int(z["spec"]), memory=NullMemory())
    log = drive_slot_pool(pool, routed, fc)
    ref = z["pool_log"].tolist()
    assert len(log) == len(ref)
    first = next((i for i, (a, b) in enumerate(zip(log, ref)) if a != b), None)
    assert first is None, (first, log[first - 2:first + 3], ref[first - 2:first + 3])
    assert stats_tuple(pool.stats) == z["pool_stats"].tolist()
    # the workload exercises every path: hits, misses, adoptions, refills, discards, and (the small pool
    # fills up) CLOCK evictions
    st = pool.stats
    assert st.hits and st.misses and st.adopted and st.adopt_evictions and st.spec_discarded
    assert st.evictions or "wide" in name
