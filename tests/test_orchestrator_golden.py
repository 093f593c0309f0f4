"""The streaming path's host bookkeeping against the reference's own engine.

Fixture tests/golden/orchestrator.json.gz (tests/golden/make_golden.py,
tests/orch_driver.py): the reference's MoEOrchestrator, SlotPool,
RouterForecast and SpeculativeScheduler decoding 16 bs1 tokens through eight
Qwen3-Next-shaped layers over the C oracle, with a 200-slot pool (64 in the
speculative partition), lookahead 2, threshold 0.062, cap 32, top 24.

Checked exactly, on CPU: the per-layer bookkeeping of the CUDA streaming
decoder (`PoolPolicy` over `SlotPool`) fed the same routing and forecast
probabilities makes every slot decision the reference engine made (demand
reads with their slots, forecast reads with their slots, the `ready` rows of
moe_ready, the `rows` of moe_rest) and ends every layer with the same pool
statistics; and the trace writer produces the reference's cache_sim trace
arrays byte for byte.
"""
from __future__ import annotations

import gzip
import hashlib
import json
from pathlib import Path

import numpy as np
import pytest

from yanah_b200.formats import ModelGeometry
from yanah_b200.forecast import RouterForecast
from yanah_b200.pool import SlotPool
from yanah_b200.streaming import PoolPolicy
from yanah_b200.trace import trace_arrays

GOLDEN = Path(__file__).resolve().parent / "golden"


def load_fixture() -> dict:
    with gzip.open(GOLDEN / "orchestrator.json.gz", "rt") as f:
        return json.load(f)


def fixture_trace(fx):
    """Entries (generation, layer, ids, {target: [(expert, p)]}) with exact fp32 p."""
    out = []
    for gen, l, ids, fc in fx["trace"]:
        cands = {int(t): [(int(e), float(np.uint32(pb).view(np.float32))) for e, pb in c] for t, c in fc.items()}
        out.append((gen, l, ids, cands))
    return out


_TRAJ = {}


def oracle_probs(fx):
    """Lookahead probabilities of every (step, layer), from the oracle's own
    decode of the fixture's inputs (the reference run's numbers); the layer
    input digests must equal the reference run's."""
    if "p" not in _TRAJ:
        from tests import orch_driver as od
        cfg = od.orch_config()
        H, R = od.oracle_trajectory(cfg, od.token_inputs(cfg, fx["config"]["steps"]))
        assert [od.digest(h) for hs in H for h in hs] == fx["h_digest"]
        _TRAJ["p"] = [[r["fprobs"] for r in rs] for rs in R]
        _TRAJ["ids"] = [[r["ids"][0].tolist() for r in rs] for rs in R]
    return _TRAJ["p"], _TRAJ["ids"]


class _NoMemory:
    def views(self, i):
        return []

    def close(self):
        pass


def replay_policy(fx, trace):
    """Drive PoolPolicy layer by layer in the streaming decoder's order;
    returns the per-layer logs in the fixture's vocabulary."""
    c = fx["config"]
    L, E = c["n_layers"], c["n_experts"]
    g = ModelGeometry(n_layers=L, n_mtp_layers=0, n_experts=E, top_k=c["top_k"], hidden=c["hidden"],
                      moe_inter=c["moe_inter"], bits=4, group_size=64)
    pool = SlotPool(g, c["slots"], spec_slot_cap=c["spec"], memory=_NoMemory())
    pol = PoolPolicy(pool, RouterForecast(g), c["threshold"], c["issue_cap"], c["top"])
    fprobs, oracle_ids = oracle_probs(fx)
    per_layer, demand, spec, ready_rows, rest_rows = [], [], [], [], []
    for i, (gen, l, ids, cands) in enumerate(trace):
        s_ = i // L
        assert oracle_ids[s_][l] == ids
        if l == 0:
            pol.end_token()
        out, ready, misses, adopted = pol.classify(l, np.array([ids]))
        demand += [[l, e, out[e]] for e in misses]
        ready_rows.append([[e, s] for e, s in ready.items()])
        targets = [t for t in range(l + 1, l + 1 + c["lookahead"]) if t < L]
        probs = {t: fprobs[s_][l][j] for j, t in enumerate(targets)}
        reserved, got = pol.issue(targets, probs)
        assert {t: [(e, float(np.float32(p))) for e, p in v] for t, v in got.items()} == cands, (gen, l)
        spec += [[t, e, s] for t in targets for e, s in reserved.get(t, [])]
        pol.publish(l, misses, out)
        pol.expire(l)
        rest_rows.append([[e, s] for e, s in out.items()])
        pol.release(out)
        st = pool.stats
        per_layer.append([getattr(st, f) for f in fx["pool_fields"][:9]])
    return per_layer, demand, spec, ready_rows, rest_rows


def test_fixture_exercises_every_path():
    fx = load_fixture()
    final = dict(zip(fx["pool_fields"], fx["per_layer"][-1]))
    assert final["hits"] and final["misses"] and final["evictions"] and final["adopted"]
    assert final["spec_reserved"] and final["spec_discarded"] and final["adopt_evictions"]
    assert len(fx["per_layer"]) == fx["config"]["steps"] * fx["config"]["n_layers"]


def test_pool_policy_makes_the_reference_engines_decisions():
    fx = load_fixture()
    trace = fixture_trace(fx)
    per_layer, demand, spec, ready_rows, rest_rows = replay_policy(fx, trace)
    ev = fx["events"]
    ref_demand = [e[2:] for e in ev if e[0] == "read" and e[1] == "demand"]
    ref_spec = [e[2:] for e in ev if e[0] == "read" and e[1] == "spec"]
    ref_ready = [e[2] for e in ev if e[0] == "moe_ready"]
    ref_rest = [e[2] for e in ev if e[0] == "moe_rest"]
    assert demand == ref_demand
    assert spec == ref_spec
    assert ready_rows == ref_ready
    assert [sorted(r) for r in rest_rows] == [sorted(r) for r in ref_rest]
    ref_pl = [row[:9] for row in fx["per_layer"]]
    first = next((i for i, (a, b) in enumerate(zip(per_layer, ref_pl)) if a != b), None)
    assert first is None, (first, per_layer[first], ref_pl[first])


def test_trace_writer_matches_reference_format():
    fx = load_fixture()
    trace = fixture_trace(fx)
    meta = json.loads(fx["save_trace_meta"])
    arrays = trace_arrays(trace, {gen: 0 for gen, *_ in trace}, meta)
    got = {k: hashlib.sha1(np.ascontiguousarray(v).tobytes()).hexdigest() for k, v in arrays.items() if k != "meta"}
    assert got == fx["save_trace_sha"]
    assert str(arrays["meta"]) == fx["save_trace_meta"]


def test_cache_sim_replay_of_the_trace_is_recorded():
    """The reference cache_sim's replay of this trace: its counters are a
    function of the trace alone, so a CUDA run that reproduces the trace
    reproduces them. They differ from the engine's own counts (cache_sim's
    CLOCK ring excludes the partition and an adoption takes a CLOCK victim
    for the forecast's key), which is the reference's own model gap."""
    fx = load_fixture()
    cs = fx["cache_sim"]
    S, L = fx["config"]["steps"], fx["config"]["n_layers"]
    assert len(cs["snaps"]) == S * L
    final = cs["final"]
    assert final["uses"] == sum(len(set(ids)) for _, _, ids, _ in fx["trace"])
    assert final["hits"] + final["adopted"] + final["demand"] == final["uses"]
    assert sum(len(m) for _, m in cs["miss_log"]) == final["demand"]
