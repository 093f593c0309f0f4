"""GPU prompt passes through the prefill sweep (staging groups over an HBM
slot pool in front of the pinned host tier, grouped GEMMs on the tensor
cores), against the CPU oracle and the all-resident prefill.

* Bit-exact: the outputs of a cold-pool and a warm-pool pass (group
  composition depends on routing alone, sweep.py); every pool record after
  the admitting pass equals the host tier's bytes.
* Within REL_L2_TOL (1e-2 relative L2): each layer's output against the
  oracle's layer on the same input rows, and against the all-resident
  prefill path (`PrefillStack`), whose per-pair results are the same but
  which sums a row's columns in one pass instead of per staging group.
"""
from __future__ import annotations

import numpy as np
import pytest

torch = pytest.importorskip("torch")

from oracle import cpu
from tests.gpu_helpers import REL_L2_TOL, bf16_dev, bf16_np, hidden_rows, rel_l2, small_config
from yanah_b200.backend import CudaMoEBackend
from yanah_b200.pool import SlotPool
from yanah_b200.prefill import PrefillStack
from yanah_b200.streaming import HostTier
from yanah_b200.sweep import HostTierReader, PrefillSweep, SweepStreams, copy_record, prompt_pass
from yanah_b200.synthetic import lfm2_stack

pytestmark = pytest.mark.gpu


def _pool(be, tier, slots, spec, warm):
    pool = SlotPool(be.geometry, slots, spec_slot_cap=spec, memory=be.make_expert_memory(slots))
    for l, e in warm:
        s = pool.claim_for_demand((l, e))
        rb = tier.rec[l]
        copy_record(pool.views(s), [tier.buf[l][e * rb:(e + 1) * rb]])
        pool.publish(s, (l, e))
        pool.unpin(s)
    return pool


def _sweep(be, tier, pool, group):
    streams = SweepStreams()
    return PrefillSweep(pool, HostTierReader(tier, streams), group=group, make_memory=be.make_expert_memory,
                        streams=streams)


def _pass_by_layer(be, sw, h, layers, admit):
    """Layer outputs of one prompt pass (each layer's input is the previous output)."""
    outs = []
    for l in layers:
        h = prompt_pass(be, sw, h, admit=admit, layers=[l])
        outs.append(h)
    torch.cuda.synchronize()
    assert be.check_error() == 0
    return outs


def _routed(be, h, layer):
    _, _, logits = be.pre_moe(layer, h)
    ids, _ = be.route(logits)
    return ids


def test_sweep_small_stack_cold_warm_oracle():
    cfg = small_config(bits=(4, 4), gs=64, hidden=512, n_experts=16, top_k=2, inter=512, shared=0, seed=7)
    T, group = 40, 4
    be = CudaMoEBackend(cfg)
    tier = HostTier(cfg, be.device)
    h = hidden_rows(cfg, T, stream=41)
    hd = bf16_dev(h)

    cold = _sweep(be, tier, _pool(be, tier, 12, 2, []), group)
    out_cold = _pass_by_layer(be, cold, hd, [0, 1], admit=False)
    assert cold.pool.resident_count() == 0 and cold.stats.pool_copies == 0

    warm_keys = [(0, 1), (0, 5), (0, 9), (1, 2), (1, 3), (1, 14)]
    warm = _sweep(be, tier, _pool(be, tier, 12, 2, warm_keys), group)
    out_warm = _pass_by_layer(be, warm, hd, [0, 1], admit=True)
    for a, b in zip(out_cold, out_warm):
        assert torch.equal(a.view(torch.int16), b.view(torch.int16))
    st = warm.stats
    distinct = len(np.unique(_routed(be, hd, 0))) + len(np.unique(_routed(be, out_warm[0], 1)))
    assert st.pool_copies + st.host_records == distinct
    assert st.pool_copies > 0 and st.layers == 2 and st.passes == 2

    # admission wrote records from staging into the pool (CLOCK may evict an earlier admission): every
    # resident record equals the host tier's bytes
    torch.cuda.synchronize()
    assert warm.pool.stats.admitted > 0 and st.admitted == warm.pool.stats.admitted
    for (l, e), s in warm.pool.map.items():
        rb = tier.rec[l]
        got = warm.pool.memory.arena.slot_view(s)[:rb].cpu()
        assert torch.equal(got, tier.buf[l][e * rb:(e + 1) * rb]), (l, e)

    orc = cpu.OracleStack(cfg, threads=8)
    rows = [0, 7, 22, T - 1]
    ins = [h, bf16_np(out_warm[0])]
    for l in range(2):
        ref = orc.layer(l, ins[l][rows])["out"]
        assert rel_l2(bf16_np(out_warm[l])[rows], ref) < REL_L2_TOL, l

    ps = PrefillStack(cfg, max_rows=T, layers=[0, 1])
    y0 = torch.empty_like(hd)
    ps.layer(0, hd, y0)
    torch.cuda.synchronize()
    assert ps.check_error() == 0
    assert rel_l2(bf16_np(out_warm[0]), bf16_np(y0)) < REL_L2_TOL
    cold.close()
    warm.close()


def test_moe_partial_groups_sum_to_full_few_rows():
    # a pass of 6 rows (the single-row routing path): two staging groups' partial
    # contributions add up to the pool path's full routed output
    cfg = small_config(bits=(4,), gs=64, hidden=1024, n_experts=16, top_k=2, inter=512, shared=0, seed=5)
    be = CudaMoEBackend(cfg)
    tier = HostTier(cfg, be.device)
    mem = be.make_expert_memory(cfg.n_experts)
    rb = tier.rec[0]
    for e in range(cfg.n_experts):
        copy_record(mem.views(e), [tier.buf[0][e * rb:(e + 1) * rb]])
    hd = bf16_dev(hidden_rows(cfg, 6, stream=43))
    _, x, logits = be.pre_moe(0, hd)
    ids, w = be.route(logits)
    full = be.moe(0, x, ids, w, mem, {e: e for e in range(cfg.n_experts)})
    ex = np.unique(ids).tolist()
    a, b = ex[: len(ex) // 2], ex[len(ex) // 2:]
    pa = be.moe(0, x, ids, w, mem, {e: e for e in a})
    pb = be.moe(0, x, ids, w, mem, {e: e for e in b})
    torch.cuda.synchronize()
    assert be.check_error() == 0
    assert rel_l2(bf16_np(pa + pb), bf16_np(full)) < REL_L2_TOL
    # rows whose experts are all in one group get nothing from the other
    only_a = np.all(np.isin(ids, a), axis=1)
    if only_a.any():
        assert not bf16_np(pb)[only_a].any()


def test_sweep_lfm2_layer():
    # LFM2 shape (64 experts, top-4, I 1536): 300 prompt rows, staging groups of 32
    cfg = lfm2_stack(n_layers=40)
    T = 300
    be = CudaMoEBackend(cfg)
    tier = HostTier(cfg, be.device, layers=[0])
    sw = _sweep(be, tier, _pool(be, tier, 40, 4, [(0, e) for e in range(0, 64, 5)]), 32)
    h = hidden_rows(cfg, T, stream=45)
    hd = bf16_dev(h)
    out = _pass_by_layer(be, sw, hd, [0], admit=True)[0]
    assert sw.stats.pool_copies > 0 and sw.stats.host_records > 0
    orc = cpu.OracleStack(cfg, threads=8)
    rows = [0, 150, T - 1]
    assert rel_l2(bf16_np(out)[rows], orc.layer(0, h[rows])["out"]) < REL_L2_TOL
    ps = PrefillStack(cfg, max_rows=T, layers=[0])
    y0 = torch.empty_like(hd)
    ps.layer(0, hd, y0)
    torch.cuda.synchronize()
    assert ps.check_error() == 0
    assert rel_l2(bf16_np(out), bf16_np(y0)) < REL_L2_TOL
    sw.close()


def test_sweep_from_repacked_file_tier(tmp_path):
    # the host tier read from an experts.bin written by the record writer gives
    # the same prompt pass, bit for bit, as the tier generated in memory
    from tests.repack_driver import write_checkpoint_from_tier
    from yanah_b200.repack import FileHostTier, repack

    cfg = small_config(bits=(4, 4), gs=64, hidden=512, n_experts=16, top_k=2, inter=512, shared=0, seed=9)
    be = CudaMoEBackend(cfg)
    tier = HostTier(cfg, be.device)
    write_checkpoint_from_tier(str(tmp_path / "model"), cfg, tier, [0, 1])
    repack(str(tmp_path / "model"), str(tmp_path / "out"))
    ftier = FileHostTier(str(tmp_path / "out"))
    assert ftier.slot == cfg.record_spec(0).slot_bytes
    hd = bf16_dev(hidden_rows(cfg, 24, stream=47))
    outs = []
    for t in (tier, ftier):
        sw = _sweep(be, t, _pool(be, t, 12, 2, [(0, 3), (1, 7)]), 4)
        outs.append(_pass_by_layer(be, sw, hd, [0, 1], admit=True))
        sw.close()
    for a, b in zip(*outs):
        assert torch.equal(a.view(torch.int16), b.view(torch.int16))


def test_sweep_qwen3_shape_two_bit_and_shared_expert():
    """A Qwen3-Next-shaped prompt pass (512 experts, top-10, 2-bit g64 and
    g32 routed records, 8-bit shared expert) through the sweep over a pool
    holding part of the stack: cold and warm pools give bit-identical layer
    outputs, each within REL_L2_TOL of the oracle's layer on the same rows."""
    cfg = small_config(bits=(2, 2), gs=64, hidden=2048, n_experts=512, top_k=10, inter=512, shared=512, seed=13)
    for gs in (64, 32):
        cfg.group_size = gs
        T, group = 96, 32
        be = CudaMoEBackend(cfg)
        tier = HostTier(cfg, be.device)
        h = hidden_rows(cfg, T, stream=43)
        hd = bf16_dev(h)
        cold = _sweep(be, tier, _pool(be, tier, 300, 8, []), group)
        out_cold = _pass_by_layer(be, cold, hd, [0, 1], admit=False)
        warm_keys = [(l, int(e)) for l in (0, 1) for e in np.unique(_routed(be, hd, l))[:40]]
        warm = _sweep(be, tier, _pool(be, tier, 300, 8, warm_keys), group)
        out_warm = _pass_by_layer(be, warm, hd, [0, 1], admit=True)
        for a, b in zip(out_cold, out_warm):
            assert torch.equal(a.view(torch.int16), b.view(torch.int16))
        assert cold.stats.host_records > 0 and warm.stats.pool_copies > 0
        orc = cpu.OracleStack(cfg, threads=8)
        rows = [0, 31, 95]
        inp = [h, bf16_np(out_cold[0])]
        for l in (0, 1):
            ref = orc.layer(l, inp[l][rows])["out"]
            err = rel_l2(bf16_np(out_cold[l])[rows], ref)
            assert err < REL_L2_TOL, (gs, l, err)
        cold.close()
        warm.close()
