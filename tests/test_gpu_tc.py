"""GPU parity of the tensor-core (tcgen05) grouped expert GEMM used for
prompt prefill, against the CPU oracle.

Bit-exact: normalised rows, routed ids and weights (the batch routing path).
Within REL_L2_TOL (1e-2 relative L2): every sampled pair's SwiGLU activations
and expert output, and the layer output.
"""
from __future__ import annotations

import numpy as np
import pytest

torch = pytest.importorskip("torch")

from oracle import cpu
from tests.gpu_helpers import REL_L2_TOL, bf16_dev, bf16_np, hidden_rows, rel_l2, small_config
from yanah_b200.prefill import PrefillStack, kperm_inverse
from yanah_b200.synthetic import lfm2_stack

pytestmark = pytest.mark.gpu


def _check(cfg, T, sample_pairs):
    st = PrefillStack(cfg, max_rows=T, layers=[0])
    h = hidden_rows(cfg, T, stream=31)
    hd = bf16_dev(h)
    out = torch.empty_like(hd)
    st.layer(0, hd, out)
    torch.cuda.synchronize()
    assert st.check_error() == 0
    orc = cpu.OracleStack(cfg, threads=8)
    pa = orc.post_attention(0, h)
    assert np.array_equal(bf16_np(st.x[:T]), pa["x"])
    assert np.array_equal(st.ids[:T].cpu().numpy(), pa["ids"])
    assert np.array_equal(st.w[:T].cpu().numpy().view(np.uint32), pa["w"].view(np.uint32))
    ids, pair_row, pair_of = st.plan(T)
    # the device plan: every (row, column) pair exactly once, pairs of an expert contiguous
    assert np.array_equal(np.sort(pair_of.reshape(-1)), np.arange(T * cfg.top_k))
    assert np.array_equal(pair_row[pair_of.reshape(-1)], np.repeat(np.arange(T), cfg.top_k))
    e_of_pair = ids.reshape(-1)[np.argsort(pair_of.reshape(-1))]
    assert np.all(np.diff(e_of_pair) >= 0)
    P = T * cfg.top_k
    act = kperm_inverse(bf16_np(st.act[:P]))
    y = bf16_np(st.y[:P])
    rng = np.random.default_rng(0)
    for p in sorted(set(rng.choice(P, size=min(sample_pairs, P), replace=False).tolist()) | {0, P - 1}):
        t = int(pair_row[p])
        j = int(np.nonzero(pair_of[t] == p)[0][0])
        a_ref, y_ref = orc.expert(0, int(ids[t, j]), pa["x"][t])
        assert rel_l2(act[p], a_ref) < REL_L2_TOL, (p, rel_l2(act[p], a_ref))
        assert rel_l2(y[p], y_ref) < REL_L2_TOL, (p, rel_l2(y[p], y_ref))
    rows = sorted(set(rng.choice(T, size=min(8, T), replace=False).tolist()))
    ref = orc.layer(0, h[rows])["out"]
    assert rel_l2(bf16_np(out)[rows], ref) < REL_L2_TOL


def test_tc_small_config():
    cfg = small_config(bits=(4,), gs=64, hidden=512, n_experts=16, top_k=2, inter=512, shared=0, seed=7)
    _check(cfg, T=40, sample_pairs=80)


def test_tc_lfm2_two_chained_layers():
    # the residual stream after one layer is large (|h| ~ 6e4): the second
    # layer's activations exceed the fp16 range, which the down GEMM's bf16
    # operands must hold
    cfg = lfm2_stack(n_layers=40)
    T = 96
    st = PrefillStack(cfg, max_rows=T, layers=[0, 1])
    h = bf16_dev(hidden_rows(cfg, T, stream=33))
    h1, h2 = torch.empty_like(h), torch.empty_like(h)
    st.layer(0, h, h1)
    st.layer(1, h1, h2)
    torch.cuda.synchronize()
    assert st.check_error() == 0
    h1n, out = bf16_np(h1), bf16_np(h2)
    assert np.abs(cpu.bf16_to_f32(h1n)).max() > 6.6e4 / 4  # the large-residual regime this test is about
    assert np.all(np.isfinite(cpu.bf16_to_f32(out)))
    orc = cpu.OracleStack(cfg, threads=8)
    rows = [0, 17, 95]
    ref = orc.layer(1, h1n[rows])["out"]  # the oracle's second layer on the same input rows
    assert rel_l2(out[rows], ref) < REL_L2_TOL


def test_tc_lfm2_layer():
    # a ragged prefill batch: 3 prompts of 37, 300 and 5 rows (342 rows, 1368 pairs)
    _check(lfm2_stack(n_layers=40), T=342, sample_pairs=48)


def test_tc_lfm2_verify_rows():
    # a speculative-verify batch (1 + 4 draft rows) on the same grouped GEMM:
    # few rows per expert, every pair checked
    _check(lfm2_stack(n_layers=40), T=5, sample_pairs=20)


@pytest.mark.parametrize("bits,gs", [(2, 64), (2, 32), (4, 64)])
def test_grouped_prompt_pass_qwen3_shape(bits, gs):
    """A Qwen3-Next-shaped prompt pass of 300 rows (512 experts, top-10, an
    8-bit shared expert behind its gate) through the backend hooks the
    orchestrator calls (pre_moe, route, moe, moe_finalize) on the grouped
    tensor-core path, for each routed record format: routed ids bit-exact,
    layer outputs within REL_L2_TOL of the oracle."""
    from yanah_b200.backend import CudaMoEBackend
    from yanah_b200.device import fill_synthetic_experts
    cfg = small_config(bits=(bits,), gs=gs, hidden=2048, n_experts=512, top_k=10, inter=512, shared=512, seed=12)
    be = CudaMoEBackend(cfg, "cuda", lookahead=0)
    mem = be.make_expert_memory(cfg.n_experts)
    fill_synthetic_experts(mem.arena, cfg, 0)
    T = 300
    h = hidden_rows(cfg, T, stream=41)
    hd = bf16_dev(h)
    h_res, x, logits = be.pre_moe(0, hd)
    ids, w = be.route(logits)
    rows = {int(e): int(e) for e in np.unique(ids)}
    routed = be.moe(0, x, ids, w, mem, rows)
    with torch.cuda.stream(be.stream):
        out = h_res + be.moe_finalize(0, routed)
    torch.cuda.synchronize()
    assert be.check_error() == 0
    orc = cpu.OracleStack(cfg, threads=8)
    pa = orc.post_attention(0, h)
    assert np.array_equal(ids, pa["ids"])
    sample = [0, 1, 57, 150, 298, 299]
    ref = orc.layer(0, h[sample])["out"]
    err = rel_l2(bf16_np(out)[sample], ref)
    assert err < REL_L2_TOL, err
