"""The reference's own decode engine driven over the C oracle (fixture side).

tests/golden/make_golden.py runs this with the reference importable: a
ModelBackend whose numbers come from the C oracle (oracle/cpu.py) is driven by
the reference's MoEOrchestrator (moe_prefetch/orchestrator.py:226-343) over the
reference's SlotPool (pool.py:90-282), RouterForecast in backend mode
(predictor.py:100-118) and SpeculativeScheduler (io_lanes.py:252-373). It
records

* every backend hook call with the arguments the orchestrator passed
  (pre_moe, route_and_forecast / route, moe_ready with its `ready` rows,
  moe_rest / moe with its `rows`, launch, fence);
* every record read with its slot, demand (ExpertReader.submit_batch) and
  speculative (SpeculativeScheduler._work);
* the pool statistics and the orchestrator counters after every layer;
* the orchestrator's routing trace (orchestrator.py:270) and its replay by
  the reference's cache_sim (cache_sim.py:88-200, in simulate's order
  :296-323): per-(step, layer) counters, the final dictionary, the miss log;
* a digest of every layer's input row, so a test can check that it rebuilt
  the same trajectory with the oracle.

Speculative reads complete before the next layer's classification (the
scheduler's workers run at the start of the next layer, when the orchestrator
fences: `prefetch arrives in time`, as cache_sim assumes); demand reads
complete at once. That makes the reference run deterministic.

Test infrastructure only: the GPU tests replay the recorded calls on the CUDA
backend (tests/test_gpu_orchestrator.py); nothing in the product imports this.
"""
from __future__ import annotations

import concurrent.futures as cf
import hashlib
from types import SimpleNamespace
from typing import Dict, List

import numpy as np

from oracle import cpu
from yanah_b200.synthetic import StackConfig, hidden_stream_id

STEPS = 16
SLOTS, SPEC = 200, 64
LOOKAHEAD, THRESHOLD, ISSUE_CAP, TOP = 2, 0.062, 32, 24
INPUT_STREAM = 77
POOL_FIELDS = ("hits", "misses", "evictions", "adopted", "spec_reserved", "spec_discarded", "spec_refused",
               "adopt_evictions", "admitted")
SIM_FIELDS = ("uses", "hits", "adopted", "demand", "prefetch", "wasted", "refused", "tokens")


def orch_config() -> StackConfig:
    """Eight Qwen3-Next-shaped layers (4-bit first and last, 2-bit between)."""
    return StackConfig("orch_parity", 8, (4, 2, 2, 2, 2, 2, 2, 4), seed=5)


def token_inputs(cfg: StackConfig, steps: int = STEPS) -> np.ndarray:
    return cpu.synth_bf16(steps * cfg.hidden, cfg.seed, hidden_stream_id(INPUT_STREAM), 1.0).reshape(steps, cfg.hidden)


def digest(bits: np.ndarray) -> str:
    return hashlib.sha1(np.ascontiguousarray(bits, np.uint16).tobytes()).hexdigest()[:16]


def targets_of(layer: int, n_layers: int) -> List[int]:
    return [t for t in range(layer + 1, layer + 1 + LOOKAHEAD) if t < n_layers]


def oracle_trajectory(cfg: StackConfig, inputs: np.ndarray):
    """Layer inputs h[s][l] (bf16 bits) of the oracle's own decode, and each
    layer's post-attention results (ids, weights, lookahead probabilities)."""
    o = cpu.OracleStack(cfg)
    H, L = [], []
    for s in range(inputs.shape[0]):
        h = inputs[s]
        hs, ls = [], []
        for l in range(cfg.n_layers):
            hs.append(h)
            r = o.layer(l, h[None], targets_of(l, cfg.n_layers))
            ls.append(r)
            h = r["out"][0]
        H.append(hs)
        L.append(ls)
        o._records.clear()
    return H, L


# -------------------------------------------------------------- reference run
class _Row:
    """A bf16 residual row. `h_res + moe_finalize(...)` gives the oracle's
    layer output (bf16(h + bf16(routed + shared)), the rounding of MLX bf16
    arrays), which the backend computed already."""

    def __init__(self, bits):
        self.bits = np.ascontiguousarray(bits, np.uint16)

    def __add__(self, other):
        assert isinstance(other, _Finalized) and np.array_equal(other.h_res, self.bits)
        return _Row(other.out)


class _Finalized:
    def __init__(self, h_res, out):
        self.h_res, self.out = h_res, out


class _Deferred:
    """Executor stand-in for the scheduler's workers: submitted reads run at
    the next flush (the orchestrator's fence at the start of a layer)."""

    def __init__(self):
        self.q = []

    def submit(self, fn, *a, **k):
        self.q.append((fn, a, k))
        return None

    def flush(self):
        q, self.q = self.q, []
        for fn, a, k in q:
            fn(*a, **k)

    def shutdown(self, wait=True):
        self.flush()


class _SlotIds:
    """Pool memory whose `views(i)` names the slot (no bytes: the oracle
    reads records by expert id; the log keeps the slot of every read)."""

    def views(self, i):
        return [int(i)]

    def close(self):
        pass


class _Reader:
    def __init__(self, log):
        self.log = log
        self.stats = SimpleNamespace(spec_records=0)
        self.kind = "spec"

    def read_record(self, key, views):
        self.log.append(["read", self.kind, int(key[0]), int(key[1]), int(views[0])])

    def submit_batch(self, jobs):
        futs = []
        self.kind = "demand"
        for key, views in jobs:
            self.read_record(key, views)
            f = cf.Future()
            f.set_result(None)
            futs.append(f)
        self.kind = "spec"
        return futs

    def wait(self, futs):
        pass


class OracleBackend:
    """ModelBackend over the C oracle, recording every hook call."""

    supports_lazy_moe = True

    def __init__(self, cfg: StackConfig, geometry, inputs: np.ndarray, log: list, deferred: _Deferred):
        self.cfg, self.geometry, self.inputs, self.log, self.deferred = cfg, geometry, inputs, log, deferred
        self.o = cpu.OracleStack(cfg)
        self.step = -1
        self.h_digest: List[str] = []
        self._res = None

    def embed(self, tokens):
        self.step = int(tokens[0])
        self.log.append(["embed", self.step])
        return _Row(self.inputs[self.step])

    def pre_moe(self, layer, h):
        self.log.append(["pre_moe", layer])
        self.h_digest.append(digest(h.bits))
        self._h_bits = h.bits
        self._res = self.o.layer(layer, h.bits[None], targets_of(layer, self.cfg.n_layers))
        self._layer = layer
        return h, "x", "logits"

    def route_and_forecast(self, logits, h_res, targets):
        r = self._res
        have = targets_of(self._layer, self.cfg.n_layers)
        self.log.append(["route_and_forecast", self._layer, [int(t) for t in targets]])
        return r["ids"].astype(np.int64), r["w"], {t: r["fprobs"][have.index(t)].copy() for t in targets if t in have}

    def route(self, logits):
        self.log.append(["route", self._layer])
        return self._res["ids"].astype(np.int64), self._res["w"]

    def moe_ready(self, layer, x, ids, memory, ready):
        self.log.append(["moe_ready", layer, [[int(e), int(s)] for e, s in ready.items()]])
        return list(ready)

    def moe_rest(self, layer, x, ids, w, memory, rows, handle):
        self.log.append(["moe_rest", layer, [[int(e), int(s)] for e, s in rows.items()]])
        return self._res["out"][0]

    def moe(self, layer, x, ids, w, memory, rows, sync=True):
        self.log.append(["moe", layer, [[int(e), int(s)] for e, s in rows.items()]])
        return self._res["out"][0]

    def moe_finalize(self, layer, routed):
        return _Finalized(self._h_bits, routed)

    def launch(self, h):
        self.log.append(["launch", self._layer])

    def fence(self):
        self.log.append(["fence"])
        self.deferred.flush()

    def lm_logits(self, h):
        return h


def run_reference(ref_modules, cfg: StackConfig, inputs: np.ndarray) -> dict:
    """Drive the reference's MoEOrchestrator over the oracle backend; returns
    the fixture dictionary (see the module docstring)."""
    orchestrator, pool_mod, io_lanes, predictor, layout, cache_sim = ref_modules
    g = layout.ModelGeometry(n_layers=cfg.n_layers, n_mtp_layers=0, n_experts=cfg.n_experts, top_k=cfg.top_k,
                             hidden=cfg.hidden, moe_inter=cfg.moe_inter, bits=4, group_size=cfg.group_size)
    log: list = []
    deferred = _Deferred()
    be = OracleBackend(cfg, g, inputs, log, deferred)
    pool = pool_mod.SlotPool(g, SLOTS, spec_slot_cap=SPEC, memory=_SlotIds())
    reader = _Reader(log)
    budget = io_lanes.IOLaneBudget(2)
    sched = io_lanes.SpeculativeScheduler(reader, pool, budget, top_per_layer=TOP, threshold=THRESHOLD,
                                          issue_cap=ISSUE_CAP)
    sched._workers.shutdown(wait=True)
    sched._workers = deferred
    fc = predictor.RouterForecast(g)
    orch = orchestrator.MoEOrchestrator(be, pool, reader, forecast=fc, scheduler=sched, lookahead=LOOKAHEAD)
    orch.trace = []
    per_layer = []
    orig_layer = orch._pool_layer

    def pool_layer(layer, h, pre):
        out = orig_layer(layer, h, pre)
        st = pool.stats
        os_ = orch.stats
        per_layer.append([int(getattr(st, f)) for f in POOL_FIELDS] +
                         [int(os_.resident_hits), int(os_.adopted_ready), int(os_.adopted_waited),
                          int(os_.demand_misses)])
        log.append(["layer_end", layer])
        return out
    orch._pool_layer = pool_layer
    outputs = []
    for s in range(inputs.shape[0]):
        _, h = orch.forward(np.array([s]))
        outputs.append(digest(h.bits))
    sched.drain()
    trace = [[int(gen), int(l), [int(e) for e in ids],
              {str(t): [[int(e), int(np.float32(p).view(np.uint32))] for e, p in c] for t, c in fcd.items()}]
             for gen, l, ids, fcd in orch.trace]
    # the reference's cache_sim on that trace: save_trace -> load_trace -> simulate's loop
    import os
    import tempfile
    with tempfile.TemporaryDirectory() as d:
        path = os.path.join(d, "trace.npz")
        cache_sim.save_trace(path, orch.trace, {gen: 0 for gen, *_ in orch.trace},
                             {"n_layers": cfg.n_layers, "model": cfg.name})
        z = np.load(path)
        arrays = {k: z[k] for k in z.files}
        tr = cache_sim.load_trace(path)
    sim = cache_sim.PoolSim(SLOTS, SPEC)
    miss_log: list = []
    sim.miss_log = miss_log
    pol = cache_sim.ForecastPolicy(tr, THRESHOLD, ISSUE_CAP)
    S, L, _ = tr.routed.shape
    snaps = []
    for s in range(S):
        sim.measure = True
        for l in range(L):
            sim.layer(l, tr.routed[s, l])
            pol.issue(sim, s, l)
            sim.expire(l)
            snaps.append([int(sim.c[n]) for n in SIM_FIELDS])
        sim.end_token()
    final = cache_sim.simulate(tr, np.ones(S, bool), SLOTS, SPEC, forecast=pol, miss_log=[])
    return {
        "config": {"name": cfg.name, "n_layers": cfg.n_layers, "bits": list(cfg.expert_bits), "seed": cfg.seed,
                   "hidden": cfg.hidden, "n_experts": cfg.n_experts, "top_k": cfg.top_k, "moe_inter": cfg.moe_inter,
                   "shared_inter": cfg.shared_inter, "steps": int(inputs.shape[0]), "slots": SLOTS, "spec": SPEC,
                   "lookahead": LOOKAHEAD, "threshold": THRESHOLD, "issue_cap": ISSUE_CAP, "top": TOP,
                   "input_stream": INPUT_STREAM},
        "events": log,
        "pool_fields": list(POOL_FIELDS) + ["resident_hits", "adopted_ready", "adopted_waited", "demand_misses"],
        "per_layer": per_layer,
        "trace": trace,
        "h_digest": be.h_digest,
        "out_digest": outputs,
        "save_trace_sha": {k: hashlib.sha1(np.ascontiguousarray(v).tobytes()).hexdigest() for k, v in arrays.items()
                           if k != "meta"},
        "save_trace_meta": str(arrays["meta"]),
        "cache_sim": {"fields": list(SIM_FIELDS), "snaps": snaps,
                      "final": {k: (float(v) if isinstance(v, float) else int(v)) for k, v in final.items()},
                      "miss_log": [[int(l), [int(e) for e in m]] for l, m in miss_log]},
    }
