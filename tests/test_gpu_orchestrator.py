"""The CUDA backend and the streaming decoder under the reference's engine.

Fixture tests/golden/orchestrator.json.gz: the reference's MoEOrchestrator
(moe_prefetch/orchestrator.py:158-343) with its SlotPool, RouterForecast and
SpeculativeScheduler decoding 16 bs1 tokens through eight Qwen3-Next-shaped
layers over the C oracle, every backend hook call and record read recorded
(tests/orch_driver.py). The reference's Python cannot travel to a GPU
machine, so its calls are replayed here, on inputs the oracle rebuilds.

* Drop-in: the recorded hook sequence (fence, pre_moe, route_and_forecast /
  route, moe_ready with the orchestrator's `ready` rows, moe_rest with its
  `rows`, moe_finalize, launch) and the record reads into the slots the
  reference pool chose, replayed on CudaMoEBackend and CudaExpertMemory:
  routed ids and lookahead probabilities bit-exact with the oracle, every
  layer output within REL_L2_TOL of the oracle's.
* Cache trace: the CUDA streaming decoder (its own pool, forecasts, copies)
  on the same layer inputs makes every decision the reference engine made
  (per-layer pool statistics, demand reads and forecast reads with their
  slots), records the same routing trace with bit-identical forecast
  candidates, and writes it as the same cache_sim trace arrays, so the
  reference cache_sim's replay of it (counters, miss log) is the fixture's.
"""
from __future__ import annotations

import gzip
import hashlib
import json
from pathlib import Path

import numpy as np
import pytest

torch = pytest.importorskip("torch")

from tests import orch_driver as od
from tests.gpu_helpers import REL_L2_TOL, bf16_dev, bf16_np, rel_l2

pytestmark = pytest.mark.gpu
GOLDEN = Path(__file__).resolve().parent / "golden"


@pytest.fixture(scope="module")
def fx():
    with gzip.open(GOLDEN / "orchestrator.json.gz", "rt") as f:
        return json.load(f)


@pytest.fixture(scope="module")
def world(fx):
    """Config, oracle trajectory (layer inputs and results) and the pinned host tier."""
    from yanah_b200.streaming import HostTier
    cfg = od.orch_config()
    H, R = od.oracle_trajectory(cfg, od.token_inputs(cfg, fx["config"]["steps"]))
    assert [od.digest(h) for hs in H for h in hs] == fx["h_digest"]
    host = HostTier(cfg, "cuda")
    yield cfg, H, R, host
    del host


def test_reference_orchestrator_calls_replayed_on_cuda_backend(fx, world):
    from yanah_b200.backend import CudaMoEBackend
    cfg, Hin, R, host = world
    c = fx["config"]
    be = CudaMoEBackend(cfg, "cuda", lookahead=c["lookahead"])
    mem = be.make_expert_memory(c["slots"])
    L = cfg.n_layers
    s = -1
    st = {}
    checked = 0
    worst = 0.0
    for ev in fx["events"]:
        kind = ev[0]
        if kind == "embed":
            s = ev[1]
        elif kind == "fence":
            be.fence()
        elif kind == "read":
            _, _, l, e, slot = ev
            mem.load([slot], [host.buf[l][e * host.rec[l]:(e + 1) * host.rec[l]]], host.rec[l], stream=be.stream)
        elif kind == "pre_moe":
            l = ev[1]
            h = bf16_dev(Hin[s][l][None])
            st = {"l": l, "h": h}
            st["h_res"], st["x"], st["logits"] = be.pre_moe(l, h)
        elif kind in ("route_and_forecast", "route"):
            l = ev[1]
            r = R[s][l]
            if kind == "route":
                ids, w = be.route(st["logits"])
                probs = {}
            else:
                ids, w, probs = be.route_and_forecast(st["logits"], st["h_res"], ev[2])
            assert np.array_equal(ids, r["ids"].astype(np.int64)), (s, l)
            for j, t in enumerate(od.targets_of(l, L)):
                if kind == "route_and_forecast":
                    assert np.array_equal(probs[t].view(np.uint32), r["fprobs"][j].view(np.uint32)), (s, l, t)
            st["ids"], st["w"] = ids, w
        elif kind == "moe_ready":
            st["handle"] = be.moe_ready(ev[1], st["x"], st["ids"], mem, {e: sl for e, sl in ev[2]})
        elif kind == "moe_rest":
            l = ev[1]
            out = be.moe_rest(l, st["x"], st["ids"], st["w"], mem, {e: sl for e, sl in ev[2]}, st["handle"])
            with torch.cuda.stream(be.stream):
                st["res"] = st["h_res"] + be.moe_finalize(l, out)
        elif kind == "launch":
            be.launch(st["res"])
            be.stream.synchronize()
            err = rel_l2(bf16_np(st["res"]), R[s][ev[1]]["out"])
            worst = max(worst, err)
            assert err < REL_L2_TOL, (s, ev[1], err)
            checked += 1
        elif kind in ("moe", "layer_end"):
            assert kind == "layer_end", "the pool path with resident-first overlap calls moe_ready/moe_rest"
    assert checked == c["steps"] * L
    assert be.check_error() == 0
    print(f"replayed {len(fx['events'])} orchestrator events, {checked} layers, worst rel_l2 {worst:.2e}")


def test_streaming_decoder_matches_reference_engine(fx, world):
    from yanah_b200.streaming import StreamingDecoder
    from yanah_b200.trace import trace_arrays
    cfg, Hin, R, host = world
    c = fx["config"]
    dec = StreamingDecoder(cfg, spec_slot_cap=c["spec"], lookahead=c["lookahead"], threshold=c["threshold"],
                           issue_cap=c["issue_cap"], top=c["top"], device="cuda", host=host, slots=c["slots"])
    assert dec.pool.slots == c["slots"]
    reads = {"demand": [], "spec": []}
    copy = dec._copy

    def logged(stream, pairs, layer, after):
        reads["demand" if stream is dec.copy else "spec"].extend([layer, e, sl] for e, sl in pairs)
        return copy(stream, pairs, layer, after)
    dec._copy = logged
    dec.trace = []
    L = cfg.n_layers
    per_layer = []
    fields = fx["pool_fields"][:9]
    worst = 0.0
    for s in range(c["steps"]):
        dec.begin_token()
        for l in range(L):
            h = bf16_dev(Hin[s][l][None])
            h_next = dec.layer(l, h)
            per_layer.append([getattr(dec.pool.stats, f) for f in fields])
            torch.cuda.synchronize()
            err = rel_l2(bf16_np(h_next), R[s][l]["out"])
            worst = max(worst, err)
            assert err < REL_L2_TOL, (s, l, err)
    assert dec.be.check_error() == 0
    ref_pl = [row[:9] for row in fx["per_layer"]]
    first = next((i for i, (a, b) in enumerate(zip(per_layer, ref_pl)) if a != b), None)
    assert first is None, (first, per_layer[first], ref_pl[first])
    ev = fx["events"]
    assert reads["demand"] == [e[2:] for e in ev if e[0] == "read" and e[1] == "demand"]
    assert reads["spec"] == [e[2:] for e in ev if e[0] == "read" and e[1] == "spec"]
    # the routing trace, forecast candidates bit for bit, and its cache_sim arrays
    ref_trace = fx["trace"]
    assert len(dec.trace) == len(ref_trace)
    for (g, l, ids, fc), (rg, rl, rids, rfc) in zip(dec.trace, ref_trace):
        assert (g, l, ids) == (rg, rl, rids)
        got = {str(t): [[e, int(np.float32(p).view(np.uint32))] for e, p in cands] for t, cands in fc.items()}
        assert got == rfc, (g, l)
    meta = json.loads(fx["save_trace_meta"])
    arrays = trace_arrays(dec.trace, {g: 0 for g, *_ in dec.trace}, meta)
    sha = {k: hashlib.sha1(np.ascontiguousarray(v).tobytes()).hexdigest() for k, v in arrays.items() if k != "meta"}
    assert sha == fx["save_trace_sha"]
    cs = fx["cache_sim"]["final"]
    print(f"streaming: {len(per_layer)} layers equal to the reference engine; cache_sim on this trace: "
          f"hits {cs['hits']} adopted {cs['adopted']} demand {cs['demand']} prefetch {cs['prefetch']} "
          f"wasted {cs['wasted']}; worst rel_l2 {worst:.2e}")
