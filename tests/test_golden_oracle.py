"""The CPU oracle against golden vectors produced by the reference's own code.

The fixtures in tests/golden/ were written by tests/golden/make_golden.py
from the reference's numpy host code (orchestrator fallback routing,
predictor.rms_norm, RouterForecast.select, the test_synthetic fp16 expert MLP,
layout/repack record geometry). The oracle defines bf16 rounding points that
the reference leaves to MLX, so float results are compared within the bf16
tolerances written in each test; ids, orders and sizes are compared exactly.
"""
from __future__ import annotations

import json
from pathlib import Path

import numpy as np
import pytest

from oracle import cpu
from yanah_b200.forecast import RouterForecast
from yanah_b200.formats import ModelGeometry, expert_record_spec, f32_to_bf16_bits, pack

GOLDEN = Path(__file__).resolve().parent / "golden"

# bf16 keeps 8 significant bits: one rounding is a relative error <= 2^-9;
# the oracle rounds up to three times on these paths (value, product, result).
BF16_RTOL = 2.0 ** -6


def _load(name):
    return np.load(GOLDEN / name)


def test_geometry_sizes_match_reference():
    d = json.loads((GOLDEN / "layout.json").read_text())
    for g in d["geometries"]:
        mine = ModelGeometry(**g["kwargs"])
        assert mine.expert_nbytes == g["expert_nbytes"], g["kwargs"]
        assert mine.slot_nbytes == g["slot_nbytes"], g["kwargs"]
        assert mine.total_moe_layers == g["total_moe_layers"]
    # the Qwen3-Next 4-bit g64 record of the reference's real-dims tests
    assert d["geometries"][0]["expert_nbytes"] == 1_769_472


def test_record_specs_match_reference():
    d = json.loads((GOLDEN / "layout.json").read_text())
    for s in d["record_specs"]:
        ref = s["spec"]
        mine = expert_record_spec(2048, 512, s["bits"], s["group_size"], n_layers=48, n_experts=512,
                                  n_mtp_layers=1).to_json()
        assert [p["name"] for p in mine["pieces"]] == [p["name"] for p in ref["pieces"]]
        for a, b in zip(mine["pieces"], ref["pieces"]):
            assert (a["dtype"], list(a["shape"]), a["nbytes"]) == (b["dtype"], list(b["shape"]), b["nbytes"]), a
        assert mine["record_bytes"] == ref["record_bytes"]
        assert mine["slot_bytes"] == ref["slot_bytes"]


@pytest.mark.parametrize("case", ["e512_k10", "e64_k4", "e100_k8"])
def test_route_matches_reference_fallback(case):
    g = _load("route.npz")
    lg, ref_ids, ref_w = g[f"{case}_logits"], g[f"{case}_ids"], g[f"{case}_w"]
    k = ref_ids.shape[1]
    ids, w = cpu.route(lg, k)
    for t in range(lg.shape[0]):
        assert set(ids[t].tolist()) == set(ref_ids[t].tolist()), t
        ref = dict(zip(ref_ids[t].tolist(), ref_w[t].tolist()))
        for e, v in zip(ids[t].tolist(), w[t].tolist()):
            assert abs(v - ref[e]) <= BF16_RTOL * ref[e] + 1e-6, (t, e, v, ref[e])
        # descending weight, and every weight a bf16 value
        assert np.all(np.diff(w[t]) <= 0)
        assert np.array_equal(f32_to_bf16_bits(w[t]).astype(np.uint32) << 16, w[t].view(np.uint32))


def test_route_tie_rule_lower_id_first():
    """Ties are where the reference (argpartition) is unspecified: the oracle's
    rule is lower id first, checked on a fully tied row."""
    lg = np.zeros((1, 64), np.float32)
    ids, w = cpu.route(lg, 8)
    assert ids[0].tolist() == list(range(8))
    assert np.allclose(w[0], 1.0 / 8)


def test_rmsnorm_matches_reference():
    g = _load("rmsnorm.npz")
    h = f32_to_bf16_bits(g["h"])
    w = f32_to_bf16_bits(g["w"])
    assert np.array_equal(h.astype(np.uint32) << 16, g["h"].view(np.uint32))  # inputs are bf16 values
    out = cpu.bf16_to_f32(cpu.rmsnorm(h, w, 1e-6))
    ref = g["out"]
    assert np.all(np.abs(out - ref) <= BF16_RTOL * np.abs(ref) + 1e-6)


def test_softmax_matches_numpy_fp32():
    g = _load("softmax.npz")
    for t in range(g["logits"].shape[0]):
        p = cpu.softmax_f32(g["logits"][t])
        np.testing.assert_allclose(p, g["probs"][t], rtol=2e-6, atol=1e-12)


def test_select_matches_reference():
    g = _load("select.npz")
    fc = RouterForecast()
    for i, p in enumerate(g["scores"]):
        sel = fc.select(3, p, 24)
        assert [e for e, _ in sel] == g["ids"][i].tolist(), i
        assert [q for _, q in sel] == g["probs"][i].tolist(), i
    assert (fc.stats.forecasts, fc.stats.candidates) == tuple(g["stats"][:2].tolist())


def test_select_observe_recall():
    fc = RouterForecast()
    p = np.linspace(1.0, 0.0, 64, endpoint=False)
    fc.select(5, p, 8)          # candidates 0..7
    fc.select(5, p[::-1], 8)    # a second forecast of the same layer joins the set: 56..63
    fc.observe(5, np.array([0, 1, 60, 30, 30]))
    assert (fc.stats.actual, fc.stats.covered, fc.stats.forecasts, fc.stats.candidates) == (4, 3, 2, 16)
    fc.observe(5, np.array([1]))  # nothing pending any more: no change
    assert fc.stats.actual == 4
    assert fc.stats.recall == 0.75


def _mlp_record(g):
    """The fixture's 4-bit codes as an oracle record (gate, up, down pieces)."""
    H, I = g["gate_codes"].shape[1], g["gate_codes"].shape[0]
    gs = int(g["group_size"])
    spec = expert_record_spec(H, I, 4, gs)
    parts = []
    for name in ("gate", "up", "down"):
        codes = g[f"{name}_codes"].astype(np.int64)
        rows, cols = codes.shape
        parts.append(pack(codes, 4).view(np.uint8).ravel())
        parts.append(np.full((rows, cols // gs), g["scale"], np.float16).view(np.uint8).ravel())
        parts.append(np.full((rows, cols // gs), g["bias"], np.float16).view(np.uint8).ravel())
    rec = np.concatenate(parts)
    assert rec.size == spec.record_bytes
    R = cpu.Record(4, gs)
    for i, o in enumerate(spec.offsets):
        R.off[i] = o
    return rec, R, H, I


def test_expert_mlp_matches_reference_fp16_mlp():
    import ctypes as C
    g = _load("expert_mlp.npz")
    rec, R, H, I = _mlp_record(g)
    dims = cpu.Dims(H, 64, 4, I, 0, 1, 1e-6)
    for t in range(g["x"].shape[0]):
        x = f32_to_bf16_bits(g["x"][t])
        act = np.empty(I, np.uint16)
        y = np.empty(H, np.uint16)
        cpu.lib().yo_expert(C.byref(dims), cpu._p(rec), C.byref(R), cpu._p(x), cpu._p(act), cpu._p(y))
        out = cpu.bf16_to_f32(y)
        ref = g["y"][t]
        rel = float(np.linalg.norm(out - ref) / np.linalg.norm(ref))
        assert rel < 1e-2, (t, rel)
