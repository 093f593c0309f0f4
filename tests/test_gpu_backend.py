"""The ModelBackend mirror (yanah_b200.backend) driven the way the reference's
orchestrator drives its backend on the pool path (orchestrator.py:226-300):
pre_moe -> route_and_forecast -> moe_ready (experts already resident) ->
moe_rest -> moe_finalize -> residual, with expert records copied from pinned
host memory into shuffled pool slots (the host tier -> HBM slot path).

Bit-exact against the oracle: routing ids and weights, lookahead
probabilities. Within REL_L2_TOL: layer outputs.
"""
from __future__ import annotations

import numpy as np
import pytest

torch = pytest.importorskip("torch")

from oracle import cpu
from tests.gpu_helpers import REL_L2_TOL, bf16_dev, bf16_np, hidden_rows, rel_l2, small_config
from yanah_b200.backend import CudaMoEBackend

pytestmark = pytest.mark.gpu


def _pool(cfg, backend, o, seed=0):
    """Every (layer, expert) record in its own shuffled slot, loaded from pinned host memory."""
    E, L = cfg.n_experts, cfg.n_layers
    mem = backend.make_expert_memory(E * L)
    perm = np.random.default_rng(seed).permutation(E * L)
    slot_of = {}
    for l in range(L):
        recs, slots = [], []
        for e in range(E):
            r = torch.from_numpy(o.record(l, e)).pin_memory()
            recs.append(r)
            slots.append(int(perm[l * E + e]))
            slot_of[(l, e)] = int(perm[l * E + e])
        mem.load(slots, recs, cfg.record_spec(l).record_bytes, backend.stream)
        backend.stream.synchronize()
    return mem, slot_of


@pytest.mark.parametrize("bits", [(4, 2, 2), (2, 4)])
def test_backend_pool_path_matches_oracle(bits):
    cfg = small_config(bits=bits, seed=17)
    be = CudaMoEBackend(cfg, "cuda", lookahead=2)
    o = cpu.OracleStack(cfg)
    mem, slot_of = _pool(cfg, be, o)
    h = bf16_dev(hidden_rows(cfg, 1, stream=3))
    for l in range(cfg.n_layers):
        h_res, x, logits = be.pre_moe(l, h)
        targets = [t for t in (l + 1, l + 2) if t < cfg.n_layers]
        ids, w, probs = be.route_and_forecast(logits, h_res, targets)
        ref = o.layer(l, bf16_np(h), targets=targets)
        assert np.array_equal(ids, ref["ids"]), l
        assert np.array_equal(w.cpu().numpy().view(np.uint32), ref["w"].view(np.uint32)), l
        for i, t in enumerate(targets):
            assert np.array_equal(probs[t].view(np.uint32), ref["fprobs"][i].view(np.uint32)), (l, t)
        experts = [int(e) for e in np.unique(ids)]
        rows = {e: slot_of[(l, e)] for e in experts}
        ready = {e: s for e, s in rows.items() if e % 2 == 0}       # the "hits"
        handle = be.moe_ready(l, x, ids, mem, ready)
        out = be.moe_rest(l, x, ids, w, mem, rows, handle)
        h = h_res + be.moe_finalize(l, out)
        be.fence()
        err = rel_l2(bf16_np(h), ref["out"])
        assert err < REL_L2_TOL, (l, err)
        h = bf16_dev(ref["out"])  # teacher forcing: the next layer starts from the oracle's row
    assert be.check_error() == 0


def test_backend_moe_equals_ready_rest_split():
    cfg = small_config(bits=(4,), seed=5)
    be = CudaMoEBackend(cfg, "cuda")
    o = cpu.OracleStack(cfg)
    mem, slot_of = _pool(cfg, be, o, seed=1)
    h = bf16_dev(hidden_rows(cfg, 1, stream=9))
    h_res, x, logits = be.pre_moe(0, h)
    ids, w = be.route(logits)
    rows = {int(e): slot_of[(0, int(e))] for e in np.unique(ids)}
    whole = be.moe(0, x, ids, w, mem, rows, sync=True).clone()
    handle = be.moe_ready(0, x, ids, mem, {e: s for e, s in rows.items() if e % 3 == 0})
    split = be.moe_rest(0, x, ids, w, mem, rows, handle)
    be.fence()
    assert np.array_equal(bf16_np(whole), bf16_np(split))
    # no expert of this row in `rows` (a staging group that holds none of them): no contribution
    none = be.moe(0, x, ids, w, mem, {}, sync=True)
    assert not none.float().abs().any()
    assert be.check_error() == 0
