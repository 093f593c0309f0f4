"""Prefill sweep bookkeeping against the reference's own code.

Fixture (tests/golden/sweep.json, written by tests/golden/make_golden.py): the
reference PrefillSweep (moe_prefetch/sweep.py:80-138) over the reference
SlotPool, driven by tests/sweep_driver.py on seeded prompt passes. The same
driver runs yanah_b200.sweep.PrefillSweep over yanah_b200.pool.SlotPool here;
everything is compared exactly: which experts each host read fetched, the
staging rows given to every grouped `moe` call, the outputs, the pool map
after every layer (admissions and their CLOCK victims) and the statistics.
"""
from __future__ import annotations

import json
from pathlib import Path

import numpy as np
import pytest

from tests.sweep_driver import TagMemory, drive_sweep, warm_pool
from yanah_b200.formats import ModelGeometry
from yanah_b200.pool import SlotPool
from yanah_b200.sweep import GROUP, HostTierReader, PrefillSweep

GOLDEN = Path(__file__).resolve().parent / "golden" / "sweep.json"


def _cases():
    return json.loads(GOLDEN.read_text())["cases"]


@pytest.mark.parametrize("i", [0, 1])
def test_sweep_matches_reference(i):
    c = _cases()[i]
    g = ModelGeometry(n_layers=c["L"], n_mtp_layers=0, n_experts=c["E"], top_k=c["k"], hidden=64, moe_inter=32,
                      bits=4, group_size=32)
    pool = SlotPool(g, c["slots"], spec_slot_cap=c["spec"], memory=TagMemory(c["slots"]))
    warm_pool(pool, c["warm"])
    res = drive_sweep(PrefillSweep, pool, np.array(c["ids"]), np.array(c["w"]), c["group"])
    for key in ("reader", "moe", "maps", "sweep_stats", "pool_stats", "fair_share"):
        assert res[key] == c[key], key
    assert np.array_equal(np.array(res["outs"]), np.array(c["outs"]))
    # case 0 (warm pool) exercises resident copies, host reads and admissions with evictions; case 1 starts
    # cold (no resident copies) and admits into free slots, then evicts
    st = res["sweep_stats"]
    assert st[3] > 0 and st[4] > 0 and res["pool_stats"][2] > 0
    assert (st[2] > 0) == (i == 0)
    assert max(len(m[1]) for m in res["moe"]) <= c["group"]


def test_sweep_groups_depend_on_routing_only():
    # a cold and a warm pool give the same staging groups (sweep.py: group
    # composition never depends on residency)
    c = _cases()[0]
    ids, w = np.array(c["ids"]), np.array(c["w"])
    logs = []
    for warm in ([], c["warm"]):
        g = ModelGeometry(n_layers=c["L"], n_mtp_layers=0, n_experts=c["E"], top_k=c["k"], hidden=64, moe_inter=32,
                          bits=4, group_size=32)
        pool = SlotPool(g, c["slots"], spec_slot_cap=c["spec"], memory=TagMemory(c["slots"]))
        warm_pool(pool, warm)
        res = drive_sweep(PrefillSweep, pool, ids[:1], w[:1], c["group"])
        logs.append((res["moe"], res["outs"]))
    assert logs[0] == logs[1]


def test_host_tier_runs():
    assert HostTierReader.runs([]) == []
    assert HostTierReader.runs([3]) == [[3]]
    assert HostTierReader.runs([0, 1, 2, 4, 6, 7]) == [[0, 1, 2], [4], [6, 7]]
    assert GROUP == 32
