"""GPU parity of the union-of-experts batch path (``yn_ep_layer`` with one
rank) against the CPU oracle.

Bit-exact: normalised rows, routed ids and weights. Within REL_L2_TOL (1e-2
relative L2): every routed output row y(t, j), the gated shared-expert
output and the layer output. Steps replayed from a CUDA graph give the same
bits as eager launches (the per-step flag/counter targets advance).
"""
from __future__ import annotations

import numpy as np
import pytest

torch = pytest.importorskip("torch")

from oracle import cpu
from tests.gpu_helpers import REL_L2_TOL, bf16_dev, bf16_np, hidden_rows, rel_l2, small_config
from yanah_b200.ep import ExpertParallelStack
from yanah_b200.synthetic import qwen3_next_stack

pytestmark = pytest.mark.gpu


def _check_layer(cfg, layer, batch, oracle_rows=None):
    ep = ExpertParallelStack(cfg, batch=batch, layers=[layer])
    h = hidden_rows(cfg, batch, stream=layer + 11)
    out = bf16_np(ep.step(bf16_dev(h)))
    torch.cuda.synchronize()
    assert ep.check_error() == 0
    got = ep.home_outputs()
    orc = cpu.OracleStack(cfg, threads=8)
    pa = orc.post_attention(layer, h)
    assert np.array_equal(got["x"], pa["x"])
    assert np.array_equal(got["ids"], pa["ids"])
    assert np.array_equal(got["w"].view(np.uint32), pa["w"].view(np.uint32))
    rows = range(batch) if oracle_rows is None else oracle_rows
    for t in rows:
        for j in range(cfg.top_k):
            _, y = orc.expert(layer, int(pa["ids"][t, j]), pa["x"][t])
            assert rel_l2(got["y"][t, j], y) < REL_L2_TOL, (t, j, rel_l2(got["y"][t, j], y))
        if cfg.shared_inter:
            ysh = orc.shared_down(layer, pa["act_sh"][t], pa["sgate"][t])
            assert rel_l2(got["ysh"][t], ysh) < REL_L2_TOL, (t, rel_l2(got["ysh"][t], ysh))
    ref = orc.layer(layer, h[list(rows)])["out"]
    assert rel_l2(out[list(rows)], ref) < REL_L2_TOL
    ep.close()


@pytest.mark.parametrize("layer", [0, 4])  # 4-bit g64, 2-bit g64 experts
def test_batch_layer_matches_oracle(layer):
    _check_layer(qwen3_next_stack(n_layers=48), layer, batch=16)


def test_batch_4bit_group32_matches_oracle():
    cfg = small_config(bits=(4,), gs=32, hidden=2048, n_experts=64, top_k=8, inter=512, shared=512, seed=5)
    _check_layer(cfg, 0, batch=24)


def test_batch_of_64_rows():
    # the largest batch: every routed pair of 64 rows through one 2-bit layer;
    # the oracle checks a sample of rows (popular and rare experts alike)
    _check_layer(qwen3_next_stack(n_layers=48), 5, batch=64, oracle_rows=[0, 7, 31, 63])


def test_graph_replay_matches_eager_steps():
    cfg = qwen3_next_stack(n_layers=48)
    layers = [2, 3, 4, 5]
    h = bf16_dev(hidden_rows(cfg, 32, stream=3))
    eager = ExpertParallelStack(cfg, batch=32, layers=layers)
    a1 = bf16_np(eager.step(h))
    a2 = bf16_np(eager.step(bf16_dev(a1)))
    graph = ExpertParallelStack(cfg, batch=32, layers=layers)
    graph.capture()
    b1 = bf16_np(graph.step(h))
    b2 = bf16_np(graph.step(bf16_dev(b1)))
    torch.cuda.synchronize()
    assert eager.check_error() == 0 and graph.check_error() == 0
    assert np.array_equal(a1, b1) and np.array_equal(a2, b2)
    eager.close()
    graph.close()


def test_batch_lfm2_verify_rows():
    # a speculative-verify batch (1 + 4 rows) on the LFM2-shaped layer: 64 experts, top-4, I 1536, no shared expert
    from yanah_b200.synthetic import lfm2_stack
    _check_layer(lfm2_stack(n_layers=40), 3, batch=5)


def test_peer_wait_gives_up_with_an_error_and_the_gpu_stays_usable():
    """Rank 0 of a two-rank layer whose peer never raises its flags (the peer
    buffer is one of this process's own, which no kernel ever flags): the
    layer's waits give up after their limit (2 s), the rank's error word holds
    YN_ERR_PEER_TIMEOUT, the call returns, and a normal one-rank layer on the
    same GPU afterwards still matches the oracle."""
    import ctypes as C
    import time

    from yanah_b200 import _lib
    from yanah_b200.device import stream_ptr
    cfg = qwen3_next_stack(n_layers=48)
    B = 16
    one = ExpertParallelStack(cfg, batch=B, layers=[4])  # every expert local, slot = expert id
    lib, D = _lib.lib(), C.byref(one.dims)
    cfg2 = _lib.EpConfig(0, 2, B // 2, 0, cfg.n_experts // 2, 1)
    sym_b, loc_b = int(lib.yn_ep_sym_bytes(D, C.byref(cfg2))), int(lib.yn_ep_local_bytes(D, C.byref(cfg2)))
    sym = torch.zeros(sym_b, dtype=torch.uint8, device="cuda")
    silent_peer = torch.zeros(sym_b, dtype=torch.uint8, device="cuda")
    local = torch.zeros(loc_b, dtype=torch.uint8, device="cuda")
    _lib.check(lib.yn_ep_init(sym.data_ptr(), local.data_ptr(), D, C.byref(cfg2), stream_ptr()))
    peers = (C.c_void_p * 2)(sym.data_ptr(), silent_peer.data_ptr())
    h = bf16_dev(hidden_rows(cfg, B // 2, stream=5))
    out = torch.empty_like(h)
    torch.cuda.synchronize()
    t0 = time.time()
    _lib.check(lib.yn_ep_layer(D, C.byref(one.structs[0]), 0, C.byref(cfg2), h.data_ptr(), out.data_ptr(), peers,
                               local.data_ptr(), stream_ptr()))
    code = C.c_int32(0)
    _lib.check(lib.yn_ep_error(local.data_ptr(), D, C.byref(cfg2), stream_ptr(), C.byref(code)))
    waited = time.time() - t0
    assert code.value == 6, code.value          # YN_ERR_PEER_TIMEOUT
    assert 1.5 < waited < 30.0, waited
    # the context is intact: the one-rank layer is still right
    hb = hidden_rows(cfg, B, stream=6)
    got = bf16_np(one.step(bf16_dev(hb)))
    torch.cuda.synchronize()
    assert one.check_error() == 0
    ref = cpu.OracleStack(cfg, threads=8).layer(4, hb[[0, 9]])["out"]
    assert rel_l2(got[[0, 9]], ref) < REL_L2_TOL
    one.close()
