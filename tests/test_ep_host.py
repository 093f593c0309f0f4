"""Host logic of expert parallelism, on CPU.

* expert ranges and home rows partition the experts and the batch;
* `plan_pairs` groups the local pairs by expert as the device plan does;
* two gloo ranks run the expert-parallel decomposition of one layer with the
  oracle as the arithmetic (home rows routed locally, rows gathered from every
  rank, the pairs of local experts computed by their owner, output rows sent to
  their home rank, combined there in column order) and get the same bits as
  the one-rank oracle layer; the IPC-handle exchange goes through the same
  process group.
"""
from __future__ import annotations

import os
import socket

import numpy as np
import pytest

torch = pytest.importorskip("torch")
import torch.distributed as dist
import torch.multiprocessing as mp

from yanah_b200.ep import _exchange_handles, expert_range, home_rows, plan_pairs


def test_expert_ranges_and_home_rows_partition():
    for E, G in [(512, 1), (512, 2), (512, 8), (100, 3), (64, 8)]:
        rs = [expert_range(E, r, G) for r in range(G)]
        assert rs[0][0] == 0 and rs[-1][1] == E
        assert all(a[1] == b[0] for a, b in zip(rs, rs[1:]))
    assert [home_rows(64, r, 4) for r in range(4)] == [(0, 16), (16, 32), (32, 48), (48, 64)]
    with pytest.raises(ValueError):
        home_rows(64, 0, 3)


def test_plan_pairs_groups_by_expert():
    rng = np.random.default_rng(1)
    ids = np.stack([rng.choice(64, 6, replace=False) for _ in range(20)])
    experts, off, pairs = plan_pairs(ids, 16, 40)
    flat = ids.reshape(-1)
    assert list(experts) == sorted(set(flat[(flat >= 16) & (flat < 40)]))
    for s, e in enumerate(experts):
        seg = pairs[off[s]:off[s + 1]]
        assert np.all(flat[seg] == e) and np.all(np.diff(seg) > 0)
    assert off[-1] == np.count_nonzero((flat >= 16) & (flat < 40))


def _free_port() -> int:
    with socket.socket() as s:
        s.bind(("127.0.0.1", 0))
        return s.getsockname()[1]


def _tiny_config():
    from yanah_b200.synthetic import StackConfig
    return StackConfig("tiny", 1, (4,), hidden=256, n_experts=16, top_k=4, moe_inter=64, shared_inter=64,
                       group_size=64, zipf_s=1.1, seed=9)


def _worker(rank: int, world: int, port: int, batch: int, out_q):
    from oracle import cpu
    from yanah_b200.synthetic import hidden_stream_id
    os.environ["MASTER_ADDR"] = "127.0.0.1"
    os.environ["MASTER_PORT"] = str(port)
    dist.init_process_group("gloo", rank=rank, world_size=world)
    try:
        cfg = _tiny_config()
        H, K, E = cfg.hidden, cfg.top_k, cfg.n_experts
        orc = cpu.OracleStack(cfg, threads=1)
        h = cpu.synth_bf16(batch * H, cfg.seed, hidden_stream_id(4), 1.0).reshape(batch, H)
        r0, r1 = home_rows(batch, rank, world)
        lo, hi = expert_range(E, rank, world)
        # home rows: post-attention and routing
        pa = orc.post_attention(0, h[r0:r1])
        # dispatch: every rank gets every row and its ids
        # (bf16 bits travel as int32: gloo has no 16-bit integer type)
        x_parts = [torch.empty((r1 - r0, H), dtype=torch.int32) for _ in range(world)]
        id_parts = [torch.empty((r1 - r0, K), dtype=torch.int32) for _ in range(world)]
        dist.all_gather(x_parts, torch.from_numpy(pa["x"].astype(np.int32)))
        dist.all_gather(id_parts, torch.from_numpy(pa["ids"]))
        x_all = torch.cat(x_parts).numpy().astype(np.uint16)
        ids_all = torch.cat(id_parts).numpy()
        # owner: pairs of local experts, one expert at a time
        experts, off, pairs = plan_pairs(ids_all, lo, hi)
        y_send = np.zeros((batch, K, H), np.uint16)
        mine = np.zeros((batch, K), np.int32)
        for s, e in enumerate(experts):
            for p in pairs[off[s]:off[s + 1]]:
                t, j = divmod(int(p), K)
                y_send[t, j] = orc.expert(0, int(e), x_all[t])[1]
                mine[t, j] = 1
        # combine: each output row reaches its home rank; each (t, j) comes from exactly one owner
        y_all = [torch.empty((batch, K, H), dtype=torch.int32) for _ in range(world)]
        m_all = [torch.empty((batch, K), dtype=torch.int32) for _ in range(world)]
        dist.all_gather(y_all, torch.from_numpy(y_send.astype(np.int32)))
        dist.all_gather(m_all, torch.from_numpy(mine))
        owners = torch.stack(m_all).numpy()
        assert np.all(owners.sum(0) == 1)
        y_home = np.zeros((r1 - r0, K, H), np.uint16)
        for r in range(world):
            sel = owners[r, r0:r1].astype(bool)
            y_home[sel] = y_all[r].numpy().astype(np.uint16)[r0:r1][sel]
        out = np.empty((r1 - r0, H), np.uint16)
        for t in range(r1 - r0):
            ysh = orc.shared_down(0, pa["act_sh"][t], pa["sgate"][t])
            out[t] = orc.combine(y_home[t], pa["w"][t], ysh, h[r0 + t], 2)
        ref = orc.layer(0, h[r0:r1])["out"]
        handles = _exchange_handles(bytes([rank]) * 64, world)
        out_q.put((rank, bool(np.array_equal(out, ref)), [hb[0] for hb in handles]))
    except Exception as e:  # report instead of leaving the parent waiting
        out_q.put((rank, repr(e), None))
        raise
    finally:
        dist.destroy_process_group()


@pytest.mark.parametrize("world", [2])
def test_gloo_expert_parallel_layer_matches_one_rank(world):
    ctx = mp.get_context("spawn")
    q = ctx.Queue()
    port = _free_port()
    procs = [ctx.Process(target=_worker, args=(r, world, port, 8, q)) for r in range(world)]
    for p in procs:
        p.start()
    results = [q.get(timeout=240) for _ in procs]
    for p in procs:
        p.join(timeout=60)
    assert all(p.exitcode == 0 for p in procs), results
    for rank, same, handles in results:
        assert same is True, f"rank {rank}: {same}"
        assert handles == list(range(world))
