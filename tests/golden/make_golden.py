"""Generate the golden fixtures in this directory from the reference's own code.

Run where a checkout of the reference is readable, giving its path (or
setting YANAH_REFERENCE); the fixtures it writes are committed, so nothing
that runs on a GPU machine needs the reference:

    python tests/golden/make_golden.py --reference <reference checkout>

What each fixture pins (the reference function that produced it):

* ``layout.json`` — ``moe_prefetch/layout.py:28-61`` ``ModelGeometry``
  record/slot sizes and ``quantize_2bit.py:90-103`` ``out_spec`` piece lists
  (order ``moe_prefetch/repack.py:27-29``) for the record formats the kernels
  read.
* ``route.npz`` — ``moe_prefetch/orchestrator.py:141-150`` fallback routing
  (softmax, top-k by argpartition, renormalise) on tie-free logits.
* ``rmsnorm.npz`` — ``moe_prefetch/predictor.py:31-34`` ``rms_norm`` (fp32,
  eps 1e-6) on bf16-valued rows.
* ``select.npz`` — ``moe_prefetch/predictor.py:100-111``
  ``RouterForecast.select`` (top candidates in descending probability) on
  tie-free probability vectors, plus ``observe`` recall counters.
* ``softmax.npz`` — the fp32 softmax of ``predictor.py:95-97`` (lookahead
  probabilities) on random logits.
* ``pool_small.npz``, ``pool_wide.npz`` — ``moe_prefetch/pool.py:90-282``
  ``SlotPool`` driven by ``tests/pool_driver.drive_slot_pool`` (slot
  decisions and stats), and ``moe_prefetch/cache_sim.py:88-200`` ``PoolSim``
  + ``ForecastPolicy`` replaying the same seeded routing trace in
  ``simulate``'s order (:296-323), with per-(step, layer) counters, the
  final dictionary and the demand-miss log.
* ``sweep.json`` — ``moe_prefetch/sweep.py:80-138`` ``PrefillSweep`` over the
  reference ``SlotPool``, driven by ``tests/sweep_driver.drive_sweep``: staging
  groups, resident copies and host reads per group, the rows given to each
  grouped ``moe`` call, the outputs, the pool after every layer (the final
  pass admits each layer's fair share) and the statistics.
* ``repack.json`` — ``moe_prefetch/repack.py:66-126`` ``repack`` on the tiny
  seeded checkpoints of ``tests/repack_driver.py``: the SHA-256 and size of
  each experts.bin, the text of each experts.json, and, for the mixed-bit
  checkpoint, the error it raises.
* ``orchestrator.json.gz`` — ``moe_prefetch/orchestrator.py:158-343``
  ``MoEOrchestrator`` (pool path, lazy, resident-first overlap) over the
  reference ``SlotPool``, ``RouterForecast`` and ``SpeculativeScheduler``,
  driven by ``tests/orch_driver.py`` over the C oracle on an eight-layer
  Qwen3-Next-shaped stack: every backend hook call with its arguments, every
  record read with its slot, the pool statistics after every layer, the
  routing trace, the reference ``cache_sim.save_trace`` arrays (digests) and
  the ``cache_sim`` replay of that trace (per-layer counters, final
  dictionary, miss log).
* ``speculation.json`` — ``moe_prefetch/speculative.py:39-77``
  ``AdaptiveSpeculationPolicy`` driven by ``tests/speculation_driver.py``
  through seeded decode sessions: every action, step time, emitted count,
  depth and stop flag.
* ``expert_mlp.npz`` — ``moe_prefetch/test_synthetic.py:46-51``
  ``expert_mlp`` (fp16 weights, fp32 SwiGLU MLP) on weights that are exactly
  representable as 4-bit affine codes, so the quantised CUDA/oracle path and
  the reference's float MLP compute with identical weights.
"""
from __future__ import annotations

import argparse
import json
import os
import sys
from pathlib import Path

import numpy as np

HERE = Path(__file__).resolve().parent
REPO = HERE.parent.parent


def _bf16_round(x: np.ndarray) -> np.ndarray:
    """Round fp32 to the nearest bf16 value (ties to even), returned as fp32."""
    u = np.ascontiguousarray(x, np.float32).view(np.uint32).astype(np.uint64)
    u = (u + 0x7FFF + ((u >> 16) & 1)) >> 16 << 16
    return u.astype(np.uint32).view(np.float32)


def _tie_free_logits(rng, T: int, E: int, k: int, gap: float = 0.05) -> np.ndarray:
    """bf16-valued logits whose k-th and (k+1)-th largest differ by > gap
    (ties elsewhere do not change the routed set)."""
    rows = []
    for _ in range(1000):
        lg = _bf16_round((rng.standard_normal(E) * 2.0).astype(np.float32))
        s = np.sort(lg)[::-1]
        if s[k - 1] - s[k] > gap:
            rows.append(lg)
        if len(rows) == T:
            return np.stack(rows)
    raise RuntimeError("no tie-free rows found")


def make_layout(ref) -> dict:
    from moe_prefetch.layout import ModelGeometry
    from moe_prefetch.repack import Piece, RecordSpec
    from quantize_2bit import out_spec

    geoms = []
    for kw in (dict(), dict(bits=2, group_size=32), dict(bits=2, group_size=64), dict(bits=8, group_size=64),
               dict(hidden=2048, moe_inter=1536, n_experts=64, top_k=4, n_layers=40, bits=4, group_size=64)):
        g = ModelGeometry(**kw)
        geoms.append({"kwargs": kw, "expert_nbytes": g.expert_nbytes, "slot_nbytes": g.slot_nbytes,
                      "total_moe_layers": g.total_moe_layers})
    # the MLX 4-bit g64 source record of a Qwen3-Next expert (H=2048, I=512)
    H, I = 2048, 512
    src = []
    for proj in ("gate_proj", "up_proj", "down_proj"):
        rows, cols = (H, I) if proj == "down_proj" else (I, H)
        src += [Piece(f"{proj}.weight", "U32", [rows, cols * 4 // 32], rows * cols // 2),
                Piece(f"{proj}.scales", "F16", [rows, cols // 64], rows * cols // 64 * 2),
                Piece(f"{proj}.biases", "F16", [rows, cols // 64], rows * cols // 64 * 2)]
    src_spec = RecordSpec(src, 64, 4, 48, 1, 512)
    specs = [{"bits": 4, "group_size": 64, "spec": src_spec.to_json()}]
    for bits, group in ((2, 32), (2, 64), (4, 128), (8, 64)):
        specs.append({"bits": bits, "group_size": group, "spec": out_spec(src_spec, 4, bits, group).to_json()})
    return {"geometries": geoms, "record_specs": specs}


def make_route(rng):
    from moe_prefetch.orchestrator import MoEOrchestrator

    class _G:
        pass

    out = {}
    for name, (T, E, k) in {"e512_k10": (6, 512, 10), "e64_k4": (5, 64, 4), "e100_k8": (4, 100, 8)}.items():
        lg = _tie_free_logits(rng, T, E, k)
        me = _G()
        me.b = object()          # a backend without its own `route`
        me.g = _G()
        me.g.top_k = k
        ids, w = MoEOrchestrator.route(me, lg)
        out[f"{name}_logits"] = lg
        out[f"{name}_ids"] = np.asarray(ids, np.int64)
        out[f"{name}_w"] = np.asarray(w, np.float32)
    return out


def make_rmsnorm(rng):
    from moe_prefetch.predictor import rms_norm
    h = _bf16_round(rng.standard_normal((3, 2048)).astype(np.float32) * 1.5)
    w = _bf16_round((1.0 + 0.1 * rng.standard_normal(2048)).astype(np.float32))
    return {"h": h, "w": w, "out": rms_norm(h, w, 1e-6).astype(np.float32)}


def make_select(rng):
    from moe_prefetch.layout import ModelGeometry
    from moe_prefetch.predictor import RouterForecast
    out = {}
    fc = RouterForecast(ModelGeometry())
    scores, picks, probs = [], [], []
    for i in range(6):
        for _ in range(100):
            lg = rng.standard_normal(512).astype(np.float32) * 2
            p = np.exp(lg - lg.max())
            p = (p / p.sum()).astype(np.float32)
            if len(np.unique(np.sort(p)[-25:])) == 25:   # the top 25 are distinct
                break
        sel = fc.select(3, p, 24)
        scores.append(p)
        picks.append([e for e, _ in sel])
        probs.append([q for _, q in sel])
        routed = np.argsort(-p)[: 10] if i % 2 == 0 else rng.choice(512, 10, replace=False)
        fc.observe(3, routed)
    out["scores"] = np.stack(scores)
    out["ids"] = np.asarray(picks, np.int64)
    out["probs"] = np.asarray(probs, np.float64)
    out["stats"] = np.asarray([fc.stats.forecasts, fc.stats.candidates, fc.stats.actual, fc.stats.covered])
    return out


def make_softmax(rng):
    lg = (rng.standard_normal((4, 512)) * 3).astype(np.float32)
    z = lg - lg.max(axis=-1, keepdims=True)
    p = np.exp(z)
    p /= p.sum(axis=-1, keepdims=True)
    return {"logits": lg, "probs": p.astype(np.float32)}


def make_expert_mlp(rng):
    """Codes q in [0,16), scale 2^-5, bias -8*2^-5 per group of 32: every
    weight (q-8)/32 is exact in fp16, bf16 and fp32."""
    import moe_prefetch.test_synthetic as ts
    H, I, gs = ts.G.hidden, ts.G.moe_inter, 32
    codes = {"gate_proj": rng.integers(0, 16, (I, H)), "up_proj": rng.integers(0, 16, (I, H)),
             "down_proj": rng.integers(0, 16, (H, I))}
    w = {k: ((v - 8) / 32.0).astype(np.float16) for k, v in codes.items()}
    blob = np.concatenate([w["gate_proj"].ravel(), w["up_proj"].ravel(), w["down_proj"].ravel()])
    x = (np.round(rng.standard_normal((3, H)) * 32) / 32).clip(-4, 4).astype(np.float32)
    y = np.stack([ts.expert_mlp(blob, x[t]) for t in range(3)]).astype(np.float32)
    return {"gate_codes": codes["gate_proj"].astype(np.uint8), "up_codes": codes["up_proj"].astype(np.uint8),
            "down_codes": codes["down_proj"].astype(np.uint8), "group_size": np.int64(gs),
            "scale": np.float32(1 / 32), "bias": np.float32(-8 / 32), "x": x, "y": y}


def make_pool(rng, S: int, L: int, E: int, k: int, n_cand: int, spec: int):
    """Reference SlotPool driven by tests/pool_driver.drive_slot_pool and the
    reference cache_sim replay (PoolSim + ForecastPolicy, the loop order of
    cache_sim.simulate) with per-(step, layer) counter snapshots."""
    sys.path.insert(0, str(REPO))
    from tests.pool_driver import NullMemory, drive_slot_pool, fc_to_arrays, make_trace, stats_tuple
    from moe_prefetch import cache_sim
    from moe_prefetch.layout import ModelGeometry
    from moe_prefetch.pool import SlotPool

    routed, fc = make_trace(rng, S, L, E, k, n_cand=n_cand)
    slots = int(0.2 * E * L)
    g = ModelGeometry(n_layers=L, n_mtp_layers=0, n_experts=E, top_k=k, hidden=64, moe_inter=32, bits=4,
                      group_size=32)
    pool = SlotPool(g, slots, spec_slot_cap=spec, memory=NullMemory())
    log = drive_slot_pool(pool, routed, fc)
    trace = cache_sim.Trace(routed, np.zeros(S, np.int64), fc, {"n_layers": L})
    test = (np.arange(S) >= S // 4).astype(np.int8)
    names = ["uses", "hits", "adopted", "demand", "prefetch", "wasted", "refused", "tokens"]
    sim = cache_sim.PoolSim(slots, spec)
    miss_log = []
    sim.miss_log = miss_log
    pol = cache_sim.ForecastPolicy(trace, 0.062, 32)
    snaps = []
    for s in range(S):
        sim.measure = bool(test[s])
        for l in range(L):
            sim.layer(l, trace.routed[s, l])
            pol.issue(sim, s, l)
            sim.expire(l)
            snaps.append([sim.c[n] for n in names])
        sim.end_token()
    final = cache_sim.simulate(trace, test, slots, spec, forecast=cache_sim.ForecastPolicy(trace, 0.062, 32))
    assert all(final[n] == sim.c[n] for n in names)
    ml_layer = np.array([l for l, m in miss_log for _ in m], np.int16)
    ml_expert = np.array([e for _, m in miss_log for e in m], np.int16)
    ml_len = np.array([len(m) for _, m in miss_log], np.int16)
    return {"routed": routed.astype(np.int16), "test": test, "slots": np.int64(slots), "spec": np.int64(spec),
            "pool_log": np.array(log, np.int64), "pool_stats": np.array(stats_tuple(pool.stats), np.int64),
            "snaps": np.array(snaps, np.int64).reshape(S, L, len(names)),
            "final_keys": np.array(sorted(final)), "final_vals": np.array([final[k2] for k2 in sorted(final)], np.float64),
            "miss_layer": ml_layer, "miss_expert": ml_expert, "miss_len": ml_len, **fc_to_arrays(fc)}


def make_sweep(seed: int = 20261202) -> dict:
    """Reference PrefillSweep + SlotPool on two seeded prompt sets: a warm pool
    with staging groups of 8 (several groups per layer, CLOCK evictions on
    admission) and a cold pool with the default group of 32."""
    sys.path.insert(0, str(REPO))
    from tests.sweep_driver import TagMemory, drive_sweep, make_prompts, warm_pool
    from moe_prefetch.layout import ModelGeometry
    from moe_prefetch.pool import SlotPool
    from moe_prefetch.sweep import PrefillSweep

    rng = np.random.default_rng(seed)
    cases = []
    for (L, E, k, T, passes, slots, spec, group, n_warm) in [(4, 64, 4, 48, 3, 40, 8, 8, 30),
                                                              (3, 128, 8, 40, 2, 48, 8, 32, 0)]:
        ids, w = make_prompts(rng, passes, L, T, E, k)
        warm = [(int(rng.integers(L)), int(rng.integers(E))) for _ in range(n_warm)]
        g = ModelGeometry(n_layers=L, n_mtp_layers=0, n_experts=E, top_k=k, hidden=64, moe_inter=32, bits=4,
                          group_size=32)
        pool = SlotPool(g, slots, spec_slot_cap=spec, memory=TagMemory(slots))
        warm_pool(pool, warm)
        res = drive_sweep(PrefillSweep, pool, ids, w, group)
        cases.append({"L": L, "E": E, "k": k, "slots": slots, "spec": spec, "group": group, "warm": warm,
                      "ids": ids.tolist(), "w": w.tolist(), **res})
    return {"cases": cases}


def make_repack() -> dict:
    """Reference repack on every checkpoint of tests/repack_driver.CASES."""
    import hashlib
    import tempfile
    sys.path.insert(0, str(REPO))
    from tests.repack_driver import CASES, write_checkpoint
    from moe_prefetch.repack import repack

    out = {}
    for case in CASES:
        with tempfile.TemporaryDirectory() as tmp:
            model, dst = os.path.join(tmp, "model"), os.path.join(tmp, "out")
            write_checkpoint(model, case)
            try:
                repack(model, dst)
            except ValueError as exc:
                out[case] = {"error": type(exc).__name__, "message": str(exc)}
                continue
            with open(os.path.join(dst, "experts.bin"), "rb") as fh:
                data = fh.read()
            with open(os.path.join(dst, "experts.json")) as fh:
                text = fh.read()
            out[case] = {"sha256": hashlib.sha256(data).hexdigest(), "bytes": len(data), "json": text}
    return out


SPEC_SESSIONS = [(1, 3, 0.8, 0.2), (2, 4, 0.3, 0.35), (3, 8, 0.6, 0.3), (4, 16, 0.9, 0.1), (5, 2, 0.1, 0.4),
                 (6, 4, 0.95, 0.05)]


def make_speculation() -> dict:
    """Reference AdaptiveSpeculationPolicy through the seeded sessions of SPEC_SESSIONS."""
    sys.path.insert(0, str(REPO))
    from tests.speculation_driver import drive_policy
    from moe_prefetch.speculative import AdaptiveSpeculationPolicy

    return {"sessions": [{"args": list(a), "log": drive_policy(AdaptiveSpeculationPolicy, *a)}
                         for a in SPEC_SESSIONS]}


def make_orchestrator() -> dict:
    """The reference's MoEOrchestrator, SlotPool, RouterForecast and
    SpeculativeScheduler driven over the C oracle on an eight-layer
    Qwen3-Next-shaped stack (tests/orch_driver.py): hook calls, record reads,
    pool statistics per layer, the routing trace and its cache_sim replay."""
    sys.path.insert(0, str(REPO))
    from moe_prefetch import cache_sim, io_lanes, layout, orchestrator, pool, predictor
    from tests import orch_driver as od
    cfg = od.orch_config()
    return od.run_reference((orchestrator, pool, io_lanes, predictor, layout, cache_sim), cfg, od.token_inputs(cfg))


def write_orchestrator() -> None:
    import gzip
    with gzip.open(HERE / "orchestrator.json.gz", "wt") as f:
        json.dump(make_orchestrator(), f, separators=(",", ":"))


def main():
    ap = argparse.ArgumentParser()
    ap.add_argument("--reference", default=os.environ.get("YANAH_REFERENCE"),
                    required="YANAH_REFERENCE" not in os.environ,
                    help="path of the reference checkout (default: $YANAH_REFERENCE)")
    ap.add_argument("--only", choices=["sweep", "repack", "speculation", "orchestrator"],
                    help="write only this fixture")
    args = ap.parse_args()
    ref = Path(args.reference)
    sys.path.insert(0, str(ref))
    if args.only == "sweep":
        (HERE / "sweep.json").write_text(json.dumps(make_sweep()) + "\n")
        return
    if args.only == "speculation":
        (HERE / "speculation.json").write_text(json.dumps(make_speculation()) + "\n")
        return
    if args.only == "orchestrator":
        write_orchestrator()
        return
    if args.only == "repack":
        (HERE / "repack.json").write_text(json.dumps(make_repack(), indent=1) + "\n")
        return
    rng = np.random.default_rng(20260101)
    (HERE / "layout.json").write_text(json.dumps(make_layout(ref), indent=1) + "\n")
    np.savez_compressed(HERE / "route.npz", **make_route(rng))
    np.savez_compressed(HERE / "rmsnorm.npz", **make_rmsnorm(rng))
    np.savez_compressed(HERE / "select.npz", **make_select(rng))
    np.savez_compressed(HERE / "softmax.npz", **make_softmax(rng))
    np.savez_compressed(HERE / "expert_mlp.npz", **make_expert_mlp(rng))
    np.savez_compressed(HERE / "pool_small.npz", **make_pool(rng, S=40, L=12, E=128, k=8, n_cand=16, spec=32))
    np.savez_compressed(HERE / "pool_wide.npz", **make_pool(rng, S=12, L=24, E=512, k=10, n_cand=12, spec=64))
    (HERE / "sweep.json").write_text(json.dumps(make_sweep()) + "\n")
    (HERE / "repack.json").write_text(json.dumps(make_repack(), indent=1) + "\n")
    (HERE / "speculation.json").write_text(json.dumps(make_speculation()) + "\n")
    write_orchestrator()
    print("wrote", sorted(p.name for p in HERE.iterdir() if p.suffix in (".json", ".npz")))


if __name__ == "__main__":
    main()
