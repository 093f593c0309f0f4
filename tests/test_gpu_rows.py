"""Persistent multi-row decode (yn_rows_flow_decode): a batch of up to 8 rows
through every layer of the LFM2-24B-A2B-shaped stack in one launch (the MoE
forward of a speculative-verify pass), checked layer by layer against the
oracle on the kernel's own layer inputs."""
import numpy as np
import pytest
import torch

from oracle import cpu
from tests.gpu_helpers import REL_L2_TOL, bf16_dev, bf16_np, hidden_rows, rel_l2

pytestmark = pytest.mark.gpu


@pytest.mark.parametrize("T,n_layers", [(5, 40), (8, 3), (1, 3)])
def test_rows_flow_every_layer_vs_oracle(T, n_layers):
    """T rows (5: the 1 + 4 verify batch over the whole 40-layer stack; 8: the
    most the kernel takes; 1: a single row). At every layer, on the kernel's
    own input rows: routed ids and weights equal the oracle's bit for bit
    (speculative.py:121-193 compares the target model's choices, so routing
    must not drift), and the layer output is within REL_L2_TOL of the
    oracle's. A traced and an untraced launch give identical outputs."""
    from yanah_b200.stack import ResidentStack
    from yanah_b200.synthetic import lfm2_stack
    cfg = lfm2_stack(seed=0, n_layers=n_layers)
    L, K, H = cfg.n_layers, cfg.top_k, cfg.hidden
    st = ResidentStack(cfg, "cuda")
    x = bf16_dev(hidden_rows(cfg, T, stream=21))
    got = torch.empty_like(x)
    ids = torch.full((L, T, K), -1, dtype=torch.int32, device="cuda")
    wts = torch.zeros((L, T, K), dtype=torch.float32, device="cuda")
    hin = torch.zeros((L, T, H), dtype=torch.bfloat16, device="cuda")
    st.rows_decode(x, got, trace=ids, trace_hidden=hin, trace_weights=wts)
    plain = torch.empty_like(x)
    st.rows_decode(x, plain)
    torch.cuda.synchronize()
    assert st.rows_error() == 0
    assert torch.equal(got.view(torch.int16), plain.view(torch.int16))
    ids, wts, hin, got = ids.cpu().numpy(), wts.cpu().numpy(), bf16_np(hin), bf16_np(got)
    del st
    torch.cuda.empty_cache()
    assert np.array_equal(hin[0], bf16_np(x))
    o = cpu.OracleStack(cfg)
    worst = 0.0
    for l in range(L):
        r = o.layer(l, hin[l])
        assert np.array_equal(ids[l], r["ids"]), (l, ids[l], r["ids"])
        assert np.array_equal(wts[l].view(np.uint32), r["w"].view(np.uint32)), l
        nxt = hin[l + 1] if l + 1 < L else got
        for t in range(T):
            err = rel_l2(nxt[t][None], r["out"][t][None])
            worst = max(worst, err)
            assert err < REL_L2_TOL, (l, t, err)
        o._records.clear()
    print(f"T={T}: {L} layers, ids/weights bit-exact, worst row rel_l2 {worst:.2e}")


def test_rows_flow_rejects_other_shapes():
    """The kernel is compiled for one shape: another stack's dims are refused
    with YN_E_UNSUPPORTED before anything is launched."""
    from yanah_b200 import _lib
    from yanah_b200.stack import ResidentStack
    from yanah_b200.synthetic import qwen3_next_stack
    cfg = qwen3_next_stack(seed=0, n_layers=1)
    st = ResidentStack(cfg, "cuda")
    x = torch.zeros((2, cfg.hidden), dtype=torch.bfloat16, device="cuda")
    with pytest.raises(_lib.YanahError) as e:
        st.rows_decode(x, torch.empty_like(x))
    assert e.value.code == _lib.YN_E_UNSUPPORTED


def test_rows_flow_slot_table_and_identical_rows():
    """Two layouts and two batch shapes that the random-row test does not
    reach. (1) Experts behind an expert -> slot table in a permuted arena
    with spare slots: the same outputs, bit for bit, as the identity layout
    (only the record addresses change). (2) Five identical rows: every row
    routes to the same k experts, so each expert has all five rows and ~37
    CTAs; every output row equals the single-row decode of that row, bit for
    bit (the GEMV columns are independent and the work split is the same)."""
    from yanah_b200 import _lib
    from yanah_b200.device import DeviceLayer, ExpertArena
    from yanah_b200.stack import ResidentStack
    from yanah_b200.synthetic import dense_layer, lfm2_stack
    import ctypes as C
    cfg = lfm2_stack(seed=0, n_layers=2)
    st = ResidentStack(cfg, "cuda")
    row = hidden_rows(cfg, 1, stream=33)
    x = bf16_dev(np.repeat(row, 5, axis=0))
    base = torch.empty_like(x)
    st.rows_decode(x, base)
    one_in = x[:1].clone()
    one = torch.empty_like(one_in)
    st.rows_decode(one_in, one)
    torch.cuda.synchronize()
    assert st.rows_error() == 0
    b = bf16_np(base)
    for t in range(1, 5):
        assert np.array_equal(b[t], b[0]), t
    assert np.array_equal(b[0], bf16_np(one)[0])
    # the same stack behind slot tables: expert e in slot (5 e + 2) mod (E + 3) of a larger arena
    E = cfg.n_experts
    slot_of = np.array([(5 * e + 2) % (E + 3) for e in range(E)], np.int32)
    assert len(set(slot_of.tolist())) == E
    keep = []
    for i, l in enumerate(st.layer_ids):
        old = st.arenas[i]
        arena = ExpertArena(E + 3, old.slot_bytes, st.device)
        arena.buf.fill_(0xA5)
        for e in range(E):
            arena.slot_view(int(slot_of[e])).copy_(old.slot_view(e))
        smap = torch.from_numpy(slot_of).to(st.device)
        layer = DeviceLayer(cfg, l, dense_layer(cfg, l), arena, 0, smap, st.device)
        keep.append((arena, smap, layer))
    structs = [k[2].struct() for k in keep]
    arr = (_lib.Layer * len(structs))(*structs)
    tb = st.table.numel()
    _lib.check(_lib.lib().yn_stack_prepare(C.byref(st.dims), arr, len(structs), st.table.data_ptr(), tb))
    st.structs, st.layer_array = structs, arr
    moved = torch.empty_like(x)
    st.rows_decode(x, moved)
    torch.cuda.synchronize()
    assert st.rows_error() == 0
    assert np.array_equal(bf16_np(moved), b)
